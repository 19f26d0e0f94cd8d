"""ANF hybrid linear on the GPU: the int2 draft of every column
plus the int4 recompute of the hot columns (src/kernel/cuda/fused_linear_hybrid.cu:7-153)
against the C oracle and against the reference's own CUDA kernels, compiled from
their sources into oracle/_ref/libvspec_ref_cuda.so and run on the same device
buffers; the host bridge (src/python/cuda_bridge.c:1160-1683) with its temporal
hot-column rule against the oracle's restatement of that rule."""
import ctypes
import os

import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import RTOL_F32, empty_dev, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu

REF_CUDA_PATH = os.path.join(os.path.dirname(O.__file__), "_ref", "libvspec_ref_cuda.so")


def _ref_cuda():
    if not os.path.exists(REF_CUDA_PATH):
        return None
    lib = ctypes.CDLL(REF_CUDA_PATH)
    fn = lib.vspec_cuda_fused_linear_hybrid_device
    fn.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_size_t] * 5
    fn.restype = None
    return fn


def make_case(rng, m, n, k, n_blocks, hot_count, zp=True):
    x = rng.standard_normal((m, k)).astype(np.float32)
    w2 = rng.integers(0, 256, size=(n, (k + 3) // 4), dtype=np.uint8)
    s2 = rng.uniform(0.01, 0.05, size=n).astype(np.float32)
    w4 = rng.integers(0, 256, size=(n, (k + 1) // 2), dtype=np.uint8)
    s4 = rng.uniform(0.005, 0.02, size=(n, n_blocks)).astype(np.float32)
    zp4 = rng.uniform(-0.05, 0.05, size=(n, n_blocks)).astype(np.float32) if zp else None
    hot = rng.choice(n, size=min(hot_count, n), replace=False).astype(np.uint32)
    return x, w2, s2, w4, s4, zp4, hot


CASES = [
    (1, 8192, 4096, 1, 96, True),     # the reference's ANF lane-B benchmark shape
    (3, 1000, 1000, 3, 50, True),     # k % 32 != 0 (byte loads), blocks of ceil(1000/3)
    (9, 300, 512, 4, 40, False),      # m > 8 (two row passes), no zero-points
    (2, 64, 37, 5, 9, True),          # odd k, blocks of ceil(37/5) = 8
    (4, 2048, 2048, 16, 300, True),
]


@pytest.mark.parametrize("m,n,k,nb,hc,zp", CASES)
def test_hybrid_device_matches_oracle_and_reference(m, n, k, nb, hc, zp):
    torch = torch_cuda()
    rng = np.random.default_rng(m * 7 + n + k)
    x, w2, s2, w4, s4, zp4, hot = make_case(rng, m, n, k, nb, hc, zp)
    hot = np.concatenate([hot, np.array([n + 5, hot[0]], dtype=np.uint32)])   # out of range (skipped), duplicate
    dx, dw2, ds2, dw4, ds4, dh = to_dev(x), to_dev(w2), to_dev(s2), to_dev(w4), to_dev(s4), to_dev(hot)
    dzp = to_dev(zp4) if zp4 is not None else None
    dy = empty_dev((m, n), torch.float32)
    V.lib.vspec_cuda_fused_linear_hybrid_device(dx.data_ptr(), dw2.data_ptr(), ds2.data_ptr(), dw4.data_ptr(),
                                                ds4.data_ptr(), dzp.data_ptr() if dzp is not None else None,
                                                dy.data_ptr(), dh.data_ptr(), hot.size, m, n, k, nb)
    torch.cuda.synchronize()
    got = dy.cpu().numpy()
    ref = O.anf_hybrid(x, w2, s2, w4, s4, zp4, nb, hot, n, k)
    err = rel_err(got, ref)
    print(f"hybrid m={m} n={n} k={k} nb={nb}: vs oracle {err:.2e}")
    assert err <= RTOL_F32
    fn = _ref_cuda()
    if fn is None:
        pytest.skip("oracle/_ref/libvspec_ref_cuda.so not built")
    dr = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    fn(dx.data_ptr(), dw2.data_ptr(), ds2.data_ptr(), dw4.data_ptr(), ds4.data_ptr(),
       dzp.data_ptr() if dzp is not None else None, dr.data_ptr(), dh.data_ptr(), hot.size, m, n, k, nb)
    torch.cuda.synchronize()
    refc = dr.cpu().numpy()
    err_r = rel_err(got, refc)
    print(f"  vs reference CUDA {err_r:.2e}; reference CUDA vs oracle {rel_err(refc, ref):.2e}")
    assert err_r <= RTOL_F32


def test_hybrid_draft_only_and_native_stream_call():
    torch = torch_cuda()
    rng = np.random.default_rng(5)
    m, n, k = 2, 512, 1024
    x, w2, s2, w4, s4, zp4, hot = make_case(rng, m, n, k, 2, 20)
    dx, dw2, ds2 = to_dev(x), to_dev(w2), to_dev(s2)
    dy = empty_dev((m, n), torch.float32)
    V.anf_hybrid_linear(dx.data_ptr(), dw2.data_ptr(), ds2.data_ptr(), None, None, None, dy.data_ptr(), None, 0,
                        m, n, k, 1)
    torch.cuda.synchronize()
    assert rel_err(dy.cpu().numpy(), O.anf_hybrid(x, w2, s2, None, None, None, 1, None, n, k)) <= RTOL_F32
    st = torch.cuda.Stream()
    dw4, ds4, dzp, dh = to_dev(w4), to_dev(s4), to_dev(zp4), to_dev(hot)
    with torch.cuda.stream(st):
        V.anf_hybrid_linear(dx.data_ptr(), dw2.data_ptr(), ds2.data_ptr(), dw4.data_ptr(), ds4.data_ptr(),
                            dzp.data_ptr(), dy.data_ptr(), dh.data_ptr(), hot.size, m, n, k, 2, stream=st.cuda_stream)
    st.synchronize()
    assert rel_err(dy.cpu().numpy(), O.anf_hybrid(x, w2, s2, w4, s4, zp4, 2, hot, n, k)) <= RTOL_F32


def _bridge(x, w2, s2, w4, s4, zp4, hot, n, nb, profile=None):
    m, k = x.shape
    out = np.empty((m, n), dtype=np.float32)
    ptr = lambda a: a.ctypes.data if a is not None else None
    hc = 0 if hot is None else hot.size
    if profile is None:
        ok = V.lib.vspec_cuda_fused_linear_hybrid_bridge(ptr(x), ptr(w2), ptr(s2), ptr(w4), ptr(s4), ptr(zp4), m, k, n,
                                                         ptr(hot) if hc else None, hc, nb, ptr(out))
    else:
        ok = V.lib.vspec_cuda_fused_linear_hybrid_profile_bridge(ptr(x), ptr(w2), ptr(s2), ptr(w4), ptr(s4),
                                                                 ptr(zp4), m, k, n, ptr(hot) if hc else None, hc, nb,
                                                                 ptr(out), *[ctypes.addressof(v) for v in profile])
    assert ok == 1
    return out


def test_hybrid_bridge_full_path(monkeypatch):
    torch_cuda()
    monkeypatch.delenv("VSPEC_ENABLE_ANF", raising=False)
    rng = np.random.default_rng(9)
    m, n, k, nb = 1, 4096, 2048, 2
    x, w2, s2, w4, s4, zp4, hot = make_case(rng, m, n, k, nb, 64)
    got = _bridge(x, w2, s2, w4, s4, zp4, hot, n, nb)
    assert rel_err(got, O.anf_hybrid(x, w2, s2, w4, s4, zp4, nb, hot, n, k)) <= RTOL_F32
    # NULL zero-points: zero-filled device copy; profile outputs filled
    prof = [ctypes.c_float(-1.0) for _ in range(4)]
    got = _bridge(x, w2, s2, w4, s4, None, hot, n, nb, profile=prof)
    assert rel_err(got, O.anf_hybrid(x, w2, s2, w4, s4, None, nb, hot, n, k)) <= RTOL_F32
    assert all(v.value >= 0.0 for v in prof) and prof[3].value >= prof[1].value
    # argument failures return 0 (hot list without int4 weights)
    out = np.empty((m, n), dtype=np.float32)
    assert V.lib.vspec_cuda_fused_linear_hybrid_bridge(x.ctypes.data, w2.ctypes.data, s2.ctypes.data, None, None,
                                                       None, m, k, n, hot.ctypes.data, hot.size, nb,
                                                       out.ctypes.data) == 0


def test_hybrid_bridge_temporal_rule(monkeypatch):
    """Under VSPEC_ENABLE_ANF=1 VSPEC_ANF_TCC_ENABLE=1 VSPEC_ANF_MODE=active,
    after the warm-up only the newly listed hot columns are refined when they
    are at most the changed ratio of the list; the others keep the draft,
    exactly as the reference bridge returns them.  Hot lists change by 8
    columns per call, one call by 60 (above the ratio: the full list)."""
    torch_cuda()
    monkeypatch.setenv("VSPEC_ENABLE_ANF", "1")
    monkeypatch.setenv("VSPEC_ANF_TCC_ENABLE", "1")
    monkeypatch.setenv("VSPEC_ANF_MODE", "active")
    monkeypatch.setenv("VSPEC_ANF_TCC_WARMUP", "3")
    rng = np.random.default_rng(13)
    m, n, k, hc = 2, 2048, 1024, 96
    x, w2, s2, w4, s4, zp4, _ = make_case(rng, m, n, k, 1, 1)
    state = O.AnfTccState(warmup=3, max_changed_ratio=0.35, min_hot=1)
    hot = rng.choice(n, size=hc, replace=False).astype(np.uint32)
    kinds = []
    for step in range(10):
        if step > 0:
            change = 60 if step == 7 else 8
            keep = rng.permutation(hc)[: hc - change]
            fresh = rng.choice(np.setdiff1d(np.arange(n), hot), size=change, replace=False)
            hot = np.concatenate([hot[keep], fresh]).astype(np.uint32)
        active = state.select(hot)
        kinds.append("subset" if len(active) < hc else "full")
        got = _bridge(x, w2, s2, w4, s4, zp4, hot, n, 1)
        ref = O.anf_hybrid(x, w2, s2, w4, s4, zp4, 1, np.array(active, dtype=np.uint32) if active else None, n, k)
        assert rel_err(got, ref) <= RTOL_F32, step
    assert kinds == ["full"] * 3 + ["subset"] * 4 + ["full"] + ["subset"] * 2, kinds
    monkeypatch.setenv("VSPEC_ANF_TCC_ENABLE", "0")   # off again: the full hot list, state reset
    hot = np.arange(hc, dtype=np.uint32)
    got = _bridge(x, w2, s2, w4, s4, zp4, hot, n, 1)
    assert rel_err(got, O.anf_hybrid(x, w2, s2, w4, s4, zp4, 1, hot, n, k)) <= RTOL_F32
