"""vspec_b200_lowbit_linear_static: the GEMV whose scratch is a static device
array, for callers that cannot allocate device memory inside a call (a runtime
whose arena/pool allocator owns the device, or a decode loop that must not
stall on the library workspace growing).

Every case is called through the C ABI twice in a row and compared with the
oracle and with vspec_b200_lowbit_linear (library workspace) within the fp32
tolerance.  The cases name the kernel the dispatcher picks, and all but one
reach a kernel that counts in the static array's split-K counters, so the
second call also shows that the first left nothing behind.  A subprocess runs
the same comparison with the ring kernel switched off, so the register-streamed
split kernel uses the array too.  The file sorts last so it also runs after
every other test in one process.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import RTOL_F32, empty_dev, make_lowbit, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu

lib = V.lib
lib.vspec_b200_lowbit_linear_static.argtypes = [ctypes.POINTER(V.LinearArgs), ctypes.c_void_p]
lib.vspec_b200_lowbit_linear_static.restype = ctypes.c_int


def _args(dx, dw, ds, dzp, dy, m, n, k, g, bits, flags, zp_const=0.0):
    return V.LinearArgs(dx.data_ptr(), dw.data_ptr(), ds.data_ptr() if ds is not None else None,
                        dzp.data_ptr() if dzp is not None else None, zp_const, dy.data_ptr(), None, None,
                        1e-6, m, n, k, g, bits, flags, None, 0)


def _oracle(x, w, s, zp, n, k, g, bits, swiglu, zp_const):
    if zp is None:
        zp = np.full(s.shape, zp_const, dtype=s.dtype)
    y = O.lowbit_matmul(x, w, n, k, bits, s, zp, g).astype(np.float64)
    if swiglu:
        gate, up = y[:, : n // 2], y[:, n // 2:]
        y = gate / (1.0 + np.exp(-gate)) * up
    return y


# (m, n, k, groups, bits, fp16 scales, zero-points, flags, kernel the dispatcher picks)
CASES = [
    (1, 4096, 4096, 32, 2, True, True, 0, "ring: int2 at m=1"),
    (4, 12288, 4096, 32, 4, True, False, 0, "ring: m=4, bench N"),
    (1, 4096, 8192, 64, 4, False, True, 0, "ring: k > 4096"),
    (3, 1000, 2048, 16, 3, False, True, 0, "ring: ragged n"),
    (8, 640, 1024, 8, 2, True, True, 0, "ring: m=8"),
    (2, 1024, 1024, 8, 4, False, True, V.F_SWIGLU, "ring: SwiGLU"),
    (64, 1024, 4096, 32, 4, True, True, 0, "tcgen05 GEMM with split-K"),
    (11, 512, 1024, 8, 4, False, False, 0, "tcgen05 GEMM, m=11"),
    (1, 300, 1000, 5, 4, False, True, 0, "generic kernel (no scratch)"),
]


def _run_case(m, n, k, g, bits, sz16, with_zp, flags):
    torch = torch_cuda()
    rng = np.random.default_rng(1000 + m * 7 + n + bits)
    w, s, zp = make_lowbit(rng, n, k, bits, g, sz_f16=sz16, zp_mode="array" if with_zp else "none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    if sz16:
        flags |= V.F_SZ_F16
    swiglu = bool(flags & V.F_SWIGLU)
    out_cols = n // 2 if swiglu else n
    dx, dw, ds = to_dev(x), to_dev(w), to_dev(s)
    dzp = to_dev(zp) if zp is not None else None
    zc = 0.0 if with_zp else 8.0
    oracle_y = _oracle(x, w, s, zp, n, k, g, bits, swiglu, zc)
    y_ref = empty_dev((m, out_cols), torch.float32)
    V.check(lib.vspec_b200_lowbit_linear(ctypes.byref(_args(dx, dw, ds, dzp, y_ref, m, n, k, g, bits, flags, zc)),
                                         None), "vspec_b200_lowbit_linear")
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()
    tol = RTOL_F32 if m <= 8 else 2e-2   # m > 8: tcgen05 GEMM, fp16 operands
    assert rel_err(ref, oracle_y) <= tol
    ys = [empty_dev((m, out_cols), torch.float32) for _ in range(2)]
    free = []
    for call, y in enumerate(ys):
        y.fill_(float("nan"))
        torch.cuda.synchronize()
        free.append(torch.cuda.mem_get_info()[0])
        rc = lib.vspec_b200_lowbit_linear_static(ctypes.byref(_args(dx, dw, ds, dzp, y, m, n, k, g, bits, flags, zc)),
                                                 None)
        V.check(rc, "vspec_b200_lowbit_linear_static")
        torch.cuda.synchronize()
        out = y.cpu().numpy()
        assert rel_err(out, ref) <= RTOL_F32, f"call {call}: {rel_err(out, ref):.3e} against the workspace path"
        assert rel_err(out, oracle_y) <= tol, f"call {call}: {rel_err(out, oracle_y):.3e} against the oracle"
    free.append(torch.cuda.mem_get_info()[0])
    # the second call (set-up done, kernels loaded) must not change the device's free memory
    assert free[2] == free[1], f"second call changed free device memory by {free[1] - free[2]} bytes"
    flag = ctypes.c_int(0)
    V.check(lib.vspec_b200_gemv_timeout_flag(ctypes.byref(flag)), "timeout flag")
    assert flag.value == 0


@pytest.mark.parametrize("m,n,k,g,bits,sz16,with_zp,flags,kernel", CASES, ids=[c[-1] for c in CASES])
def test_static_scratch_matches_oracle_and_workspace_twice(m, n, k, g, bits, sz16, with_zp, flags, kernel):
    _run_case(m, n, k, g, bits, sz16, with_zp, flags)


def test_static_scratch_split_kernel_in_fresh_process():
    """With the ring kernel switched off (VSPEC_B200_GEMV_RING=0, read once per
    process) the m <= 8 cases run the register-streamed split kernel, whose
    merge also counts in the static array."""
    torch_cuda()
    here = os.path.dirname(os.path.abspath(__file__))
    code = ("import sys; sys.argv=['x']; import test_zz_no_alloc as T; "
            "[T._run_case(*c[:8]) for c in T.CASES if c[0] <= 8]; print('split ok')")
    env = dict(os.environ, VSPEC_B200_GEMV_RING="0", VSPEC_B200_GEMV_ROWS="0")
    root = os.path.dirname(here)
    env["PYTHONPATH"] = os.pathsep.join([here, os.path.join(root, "vspec-engine_b200", "python"),
                                         os.path.join(root, "oracle"), env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", code], env=env, cwd=here, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "split ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


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


@pytest.mark.parametrize("byte", [0x01, 0xFF])
def test_static_scratch_recovers_from_counters_left_part_way(byte):
    """A launch whose bounded wait gave up can leave split-K counts part-way in
    the static array, which the caller cannot reach.  Every call clears the
    counter region before its launch, so the calls after such a state (made here
    by filling the region from the host, no kernel involved) still match the
    oracle and the workspace path."""
    torch_cuda()
    lib.vspec_b200_debug_poison_static_scratch.argtypes = [ctypes.c_int]
    lib.vspec_b200_debug_poison_static_scratch.restype = ctypes.c_int
    for c in CASES:
        if c[-1] in ("ring: m=4, bench N", "ring: m=8", "tcgen05 GEMM with split-K"):
            V.check(lib.vspec_b200_debug_poison_static_scratch(byte), "poison static scratch")
            _run_case(*c[:8])
