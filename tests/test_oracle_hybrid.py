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
