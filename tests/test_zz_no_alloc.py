"""vspec_b200_lowbit_linear_static: the GEMV whose scratch is a static device
array (the library allocates nothing inside the call).

Called through the C ABI and compared with vspec_b200_lowbit_linear (library
workspace) within the fp32 test tolerance, on two calls in a row, so the second
call also checks that the first left the static counters zero.  The file sorts
last so it also runs after every other test in one process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import vspec_b200 as V
from gpu_util import RTOL_F32, empty_dev, make_lowbit, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu

lib = V.lib
lib.vspec_b200_lowbit_linear_static.argtypes = [ctypes.POINTER(V.LinearArgs), ctypes.c_void_p]
lib.vspec_b200_lowbit_linear_static.restype = ctypes.c_int


def _args(dx, dw, ds, dzp, dy, m, n, k, g, bits, flags, zp_const=0.0, dres=None, dnw=None):
    return V.LinearArgs(dx.data_ptr(), dw.data_ptr(), ds.data_ptr() if ds is not None else None,
                        dzp.data_ptr() if dzp is not None else None, zp_const, dy.data_ptr(),
                        dres.data_ptr() if dres is not None else None, dnw.data_ptr() if dnw is not None else None,
                        1e-6, m, n, k, g, bits, flags, None, 0)


# (m, n, k, groups, bits, fp16 scales, zero-points, flags): the bench GEMV, a
# ragged-N int3 shape, an m=8 int2 shape, a SwiGLU int4 shape, an odd-k shape
# (generic kernel) and m > 8 (row-block chunking)
CASES = [
    (1, 12288, 4096, 32, 4, True, False, V.F_UNSIGNED),
    (3, 1000, 2048, 16, 3, False, True, 0),
    (8, 640, 1024, 8, 2, True, True, 0),
    (2, 1024, 1024, 8, 4, False, True, V.F_SWIGLU),
    (1, 300, 1000, 5, 4, False, True, 0),
    (11, 512, 1024, 8, 4, False, False, 0),
]


@pytest.mark.parametrize("m,n,k,g,bits,sz16,with_zp,flags", CASES)
def test_static_scratch_matches_library_workspace_twice(m, n, k, g, bits, sz16, with_zp, flags):
    torch = torch_cuda()
    rng = np.random.default_rng(1000 + m * 7 + n + bits)
    w, s, zp = make_lowbit(rng, n, k, bits, g, sz_f16=sz16, zp_mode="array" if with_zp else "none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    if sz16:
        flags |= V.F_SZ_F16
    out_cols = n // 2 if flags & V.F_SWIGLU else n
    dx, dw, ds = to_dev(x), to_dev(w), to_dev(s)
    dzp = to_dev(zp) if zp is not None else None
    zc = 0.0 if with_zp else 8.0
    y_ref = empty_dev((m, out_cols), torch.float32)
    V.check(lib.vspec_b200_lowbit_linear(ctypes.byref(_args(dx, dw, ds, dzp, y_ref, m, n, k, g, bits, flags, zc)),
                                         None), "vspec_b200_lowbit_linear")
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()
    for call in range(2):
        y = empty_dev((m, out_cols), torch.float32)
        y.fill_(float("nan"))
        rc = lib.vspec_b200_lowbit_linear_static(ctypes.byref(_args(dx, dw, ds, dzp, y, m, n, k, g, bits, flags, zc)),
                                                 None)
        V.check(rc, "vspec_b200_lowbit_linear_static")
        torch.cuda.synchronize()
        err = rel_err(y.cpu().numpy(), ref)
        assert err <= RTOL_F32, f"call {call}: {err:.3e}"


def test_static_scratch_rejects_oversized_shapes_and_workspaces():
    torch_cuda()
    # lm_head-sized output at m=8 needs more split-K scratch than the 16 MiB array
    m, n, k = 8, 1_048_576, 4096
    need = lib.vspec_b200_lowbit_linear_workspace_bytes(m, n, k, 0)
    assert need > 16 << 20
    fake = ctypes.c_void_p(256)   # never dereferenced: rejected before any launch
    a = V.LinearArgs(fake, fake, fake, None, 0.0, fake, None, None, 1e-6, m, n, k, k // 128, 4, 0, None, 0)
    assert lib.vspec_b200_lowbit_linear_static(ctypes.byref(a), None) == 1   # VSPEC_B200_ERR_ARG
    assert "static scratch" in V.last_error()
    a = V.LinearArgs(fake, fake, fake, None, 0.0, fake, None, None, 1e-6, 1, 128, 128, 1, 4, 0, fake, 1024)
    assert lib.vspec_b200_lowbit_linear_static(ctypes.byref(a), None) == 1
    assert "d_workspace must be NULL" in V.last_error()
