"""The C restatement of the ANF hybrid linear (oracle_anf_hybrid_f32, following
src/kernel/cuda/fused_linear_hybrid.cu:7-153 and fused_linear_int2.cu:8-12)
against an independent numpy restatement, and the temporal hot-column rule of
src/python/cuda_bridge.c:1352-1404 (restated in oracle.AnfTccState).  The
reference has no CPU implementation of this path; on the GPU the restatement
is compared with the reference's own CUDA kernels (tests/test_gpu_hybrid.py)."""
import numpy as np
import pytest

import oracle as O


def numpy_hybrid(x, w2, s2, w4, s4, zp4, nb, hot, n, k):
    t = np.arange(k)
    q2 = (w2[:, t // 4] >> (2 * (t % 4))) & 3
    y = x.astype(np.float64) @ ((q2.astype(np.float64) - 1.5) * s2[:, None]).T
    if hot is None:
        return y
    bs = -(-k // nb) if nb > 1 else k
    b = np.minimum(t // bs, nb - 1) if nb > 1 else np.zeros(k, dtype=np.int64)
    for j in hot:
        if j >= n:
            continue
        byte = w4[j, t // 2]
        q = np.where(t % 2 == 1, byte >> 4, byte & 0xF).astype(np.float64)
        z = zp4[j, b] if zp4 is not None else 0.0
        y[:, j] = x.astype(np.float64) @ ((q - 8.0) * s4[j, b] + z)
    return y


@pytest.mark.parametrize("m,n,k,nb,zp", [(1, 64, 256, 1, True), (3, 50, 37, 5, True), (2, 33, 100, 3, False),
                                         (4, 20, 8, 8, True)])
def test_hybrid_restatement(m, n, k, nb, zp):
    rng = np.random.default_rng(m + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w2 = rng.integers(0, 256, size=(n, (k + 3) // 4), dtype=np.uint8)
    s2 = rng.uniform(0.01, 0.05, size=n).astype(np.float32)
    w4 = rng.integers(0, 256, size=(n, (k + 1) // 2), dtype=np.uint8)
    s4 = rng.uniform(0.005, 0.02, size=(n, nb)).astype(np.float32)
    zp4 = rng.uniform(-0.05, 0.05, size=(n, nb)).astype(np.float32) if zp else None
    hot = np.array([3, n + 1, 0, 3, n - 1], dtype=np.uint32)
    got = O.anf_hybrid(x, w2, s2, w4, s4, zp4, nb, hot, n, k)
    ref = numpy_hybrid(x, w2, s2, w4, s4, zp4, nb, hot, n, k)
    assert np.max(np.abs(got - ref)) <= 1e-4 * max(1.0, np.max(np.abs(ref)))
    draft = O.anf_hybrid(x, w2, s2, None, None, None, nb, None, n, k)
    cold = [j for j in range(n) if j not in (0, 3, n - 1)]
    assert np.array_equal(draft[:, cold], got[:, cold])


def test_tcc_rule():
    st = O.AnfTccState(warmup=2, max_changed_ratio=0.35, min_hot=4)
    a = list(range(10))
    assert st.select(a) == a and st.select(a) == a          # warm-up: full lists
    assert st.select(a) == []                               # nothing new: no refine at all
    b = a[:7] + [20, 21, 22]
    assert st.select(b) == [20, 21, 22]                     # 3/10 <= 0.35
    c = b[:6] + [30, 31, 32, 33]
    assert st.select(c) == c                                # 4/10 > 0.35: full list
    assert st.select([1, 2, 3]) == [1, 2, 3]                # below min_hot: full list
    assert st.select([]) == []


def _c_select(V, hot, have_int4=1):
    import ctypes
    hot = np.ascontiguousarray(hot, dtype=np.uint32)
    out = np.zeros(max(1, hot.size), dtype=np.uint32)
    cnt = ctypes.c_size_t(0)
    rc = V.lib.vspec_b200_debug_anf_tcc_select(hot.ctypes.data if hot.size else None, hot.size, have_int4,
                                               out.ctypes.data, ctypes.byref(cnt))
    assert rc == 0
    return [int(v) for v in out[:cnt.value]]


@pytest.mark.parametrize("env,warmup,ratio,min_hot", [
    ({}, 4, 0.35, 1),
    ({"VSPEC_ANF_TCC_WARMUP": "2", "VSPEC_ANF_TCC_MIN_HOT": "4"}, 2, 0.35, 4),
    ({"VSPEC_ANF_TCC_WARMUP": "0", "VSPEC_ANF_TCC_MAX_CHANGED_RATIO": "5"}, 4, 1.0, 1),      # 0 keeps 4; ratio clamps to 1
    ({"VSPEC_ANF_TCC_MAX_CHANGED_RATIO": "0", "VSPEC_ANF_TCC_WARMUP": "1"}, 1, 0.01, 1),     # clamps to 0.01
])
def test_bridge_tcc_rule_in_c_matches_restatement(monkeypatch, env, warmup, ratio, min_hot):
    """The C bridge's temporal rule (host code, no CUDA call) step by step
    against AnfTccState under the same environment, including the clamps of
    cuda_bridge.c:366-389."""
    import vspec_b200 as V
    monkeypatch.delenv("VSPEC_ENABLE_ANF", raising=False)
    _c_select(V, [1, 2, 3])                      # rule off: resets the thread's state
    for k_, v_ in env.items():
        monkeypatch.setenv(k_, v_)
    monkeypatch.setenv("VSPEC_ENABLE_ANF", "1")
    monkeypatch.setenv("VSPEC_ANF_TCC_ENABLE", "y")
    monkeypatch.setenv("VSPEC_ANF_MODE", "active")
    st = O.AnfTccState(warmup=warmup, max_changed_ratio=ratio, min_hot=min_hot)
    rng = np.random.default_rng(warmup * 10 + min_hot)
    hot = list(rng.choice(500, size=20, replace=False))
    for step in range(12):
        if step:
            change = [1, 3, 9, 0, 20, 2][step % 6]
            keep = list(rng.permutation(hot)[: len(hot) - change])
            fresh = [int(v) for v in rng.choice(np.setdiff1d(np.arange(500), hot), size=change, replace=False)]
            hot = keep + fresh
        assert _c_select(V, hot) == st.select(hot), step
    assert _c_select(V, hot, have_int4=0) == [int(v) for v in hot]   # no int4 weights: full list, no state change
    monkeypatch.setenv("VSPEC_ANF_MODE", "shadow")                     # not "active": the rule is off
    assert _c_select(V, hot[:5]) == [int(v) for v in hot[:5]]
