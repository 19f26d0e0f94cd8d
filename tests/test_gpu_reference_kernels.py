"""The comparison point: Vspec-Engine's own CUDA kernels, compiled unchanged for
sm_100a (oracle/_ref/libvspec_ref_cuda.so), on the same B200 and inputs as
this library.

* W4 GEMV at the literal 4096 x 4096 shape (fp32 group scales and an fp32
  zero-point array of 8, 32 groups of 128): the reference's
  vspec_cuda_fused_linear_int4_device (src/kernel/cuda/fused_linear_int4.cu:
  477-505, fused_int4_kernel_tiled) and this library's vspec_b200_lowbit_linear
  on the same device buffers.  Both are checked against the oracle, then timed
  back to back over rotating weight copies larger than L2 (CUDA events).
* Single-head attention through the same host-pointer entry point,
  vspec_cuda_attention_fused_single_f32 (attention_fused.cu:144-217): the
  reference's three kernels against this library's implementation, at the
  paged-attention workload's mean context, host-timed per call (both copy
  K and V to the device inside the call).

The measured times are printed (pytest -s) for the comparison record."""
import ctypes
import os
import time

import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import RTOL_F32, empty_dev, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu

REF_CUDA_PATH = os.path.join(os.path.dirname(O.__file__), "_ref", "libvspec_ref_cuda.so")


def _ref_cuda():
    if not os.path.exists(REF_CUDA_PATH):
        pytest.skip("oracle/_ref/libvspec_ref_cuda.so not built")
    lib = ctypes.CDLL(REF_CUDA_PATH)
    if not hasattr(lib, "vspec_cuda_fused_linear_int4_device"):
        pytest.skip("the prebuilt reference CUDA library lacks the int4 GEMV")
    lib.vspec_cuda_fused_linear_int4_device.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_size_t] * 4
    lib.vspec_cuda_fused_linear_int4_device.restype = None
    lib.vspec_cuda_attention_fused_single_f32.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_size_t] * 2 + \
        [ctypes.c_void_p]
    lib.vspec_cuda_attention_fused_single_f32.restype = None
    return lib


def test_reference_int4_gemv_kernel_vs_library_literal_shape():
    torch = torch_cuda()
    ref = _ref_cuda()
    n = k = 4096
    g, m = 32, 1
    rng = np.random.default_rng(0)
    copies = 64   # 64 x 9.5 MB > 4x L2
    ws = [rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8) for _ in range(copies)]
    s = rng.uniform(0.005, 0.02, size=(n, g)).astype(np.float32)
    zp = np.full((n, g), 8.0, dtype=np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    want = O.lowbit_matmul(x, ws[0], n, k, 4, s, zp, g)
    dws = [to_dev(w) for w in ws]
    ds, dzp, dx = to_dev(s), to_dev(zp), to_dev(x)
    dy_ref = empty_dev((m, n), torch.float32)
    dy = empty_dev((m, n), torch.float32)
    ref.vspec_cuda_fused_linear_int4_device(dx.data_ptr(), dws[0].data_ptr(), ds.data_ptr(), dzp.data_ptr(),
                                            dy_ref.data_ptr(), m, n, k, g)
    V.lowbit_linear(dx.data_ptr(), dws[0].data_ptr(), ds.data_ptr(), dzp.data_ptr(), dy.data_ptr(), m, n, k, g, 4)
    torch.cuda.synchronize()
    assert rel_err(dy_ref.cpu().numpy(), want) <= RTOL_F32
    assert rel_err(dy.cpu().numpy(), want) <= RTOL_F32

    def timed(fn, reps=5):
        for w in dws[:4]:
            fn(w)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            for w in dws:
                fn(w)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / (reps * len(dws))

    us_ref = timed(lambda w: ref.vspec_cuda_fused_linear_int4_device(dx.data_ptr(), w.data_ptr(), ds.data_ptr(),
                                                                     dzp.data_ptr(), dy_ref.data_ptr(), m, n, k, g))
    us = timed(lambda w: V.lowbit_linear(dx.data_ptr(), w.data_ptr(), ds.data_ptr(), dzp.data_ptr(), dy.data_ptr(), m,
                                         n, k, g, 4))
    nbytes = n * k // 2 + 2 * n * g * 4 + m * k * 4 + m * n * 4
    print(f"\nW4 GEMV 4096x4096 fp32 s+zp: reference fused_int4_kernel_tiled {us_ref:.2f} us "
          f"({nbytes / us_ref / 1e3:.0f} GB/s), this library {us:.2f} us ({nbytes / us / 1e3:.0f} GB/s), "
          f"{us_ref / us:.1f}x")
    assert us < us_ref


def test_reference_single_head_attention_vs_library_same_entry_point():
    torch_cuda()
    ref = _ref_cuda()
    t, d = 4352, 128   # the mean context of the paged-attention workload
    rng = np.random.default_rng(1)
    q = rng.standard_normal(d).astype(np.float32)
    kk = rng.standard_normal((t, d)).astype(np.float32)
    vv = rng.standard_normal((t, d)).astype(np.float32)
    want = O.paged_attention(q.reshape(1, 1, d), kk, vv, np.zeros((1, 1), np.int32), np.array([t], np.int32), 1, 1,
                             d, t, 1.0 / np.sqrt(d), f64=True).reshape(-1)
    outs = {}
    times = {}
    for name, fn in (("reference", ref.vspec_cuda_attention_fused_single_f32),
                     ("library", V.lib.vspec_cuda_attention_fused_single_f32)):
        out = np.zeros(d, dtype=np.float32)
        for _ in range(3):
            fn(q.ctypes.data, kk.ctypes.data, vv.ctypes.data, t, d, out.ctypes.data)
        calls = 40
        t0 = time.perf_counter()
        for _ in range(calls):
            fn(q.ctypes.data, kk.ctypes.data, vv.ctypes.data, t, d, out.ctypes.data)
        times[name] = (time.perf_counter() - t0) * 1e3 / calls
        outs[name] = out.copy()
        assert rel_err(out, want) <= RTOL_F32, name
    print(f"\nsingle-head attention t={t} d={d} (host buffers, copies inside): reference "
          f"{times['reference']:.3f} ms/call, this library {times['library']:.3f} ms/call")
