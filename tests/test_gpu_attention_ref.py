"""The CPU backend's attention semantics on the GPU (vspec_b200_attention_ref_f32,
the device side of vspec_attention_ref_single_query, src/attention/attention_ref.c:
7-88) against the oracle restatement, which is pinned bit for bit to the
reference's compiled backend in test_oracle_pins.py.

Tolerance: every score, clamp threshold, noise-reducer step and Kahan dot follows
the reference's operation order with IEEE operations, so the scores are the
oracle's; the probabilities go through CUDA's expf (within 2 ulp) where the
oracle calls the C library's, and the output sums are chunked in double.  An
output may therefore differ by a few float ulps of the probabilities times the
values: |gpu - oracle| <= TOL * max|v| per head, TOL = 2e-6."""
import ctypes
import time

import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import empty_dev, to_dev, torch_cuda
from test_oracle_pins import ATTENTION_DEMO_GOLDEN, _attention_demo_inputs, attention_ref_inputs

pytestmark = pytest.mark.gpu

TOL = 2e-6
MODULE_ENV = ("VSPEC_FUSED_BITS", "VSPEC_3BIT_RUNTIME_MODULE", "VSPEC_3BIT_BLOCK_SIZE")


def _run(q, k, v, module, block, stream=0):
    torch = torch_cuda()
    t, h, d = k.shape
    ws = V.lib.vspec_b200_attention_ref_workspace_bytes(t, h, d)
    assert ws > 0
    dq, dk, dv = to_dev(q), to_dev(k), to_dev(v)
    dout = empty_dev((h, d), torch.float32)
    dws = empty_dev((ws,), torch.uint8)
    V.attention_ref(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dout.data_ptr(), t, h, d, module, block,
                    dws.data_ptr(), ws, stream)
    torch.cuda.synchronize()
    return dout.cpu().numpy()


def _check(got, want, v):
    t, h, d = v.shape
    for hh in range(h):
        bound = TOL * max(float(np.max(np.abs(v[:, hh, :]))), 1e-30)
        err = float(np.max(np.abs(got[hh].astype(np.float64) - want[hh])))
        assert err <= bound, (hh, err, bound)


CASES = [(37, 3, 128, False), (37, 3, 128, True), (5, 2, 100, False), (1, 1, 4, False), (300, 2, 64, False),
         (33, 2, 1024, False), (2049, 2, 128, True)]


@pytest.mark.parametrize("module,block", [(0, 64), (1, 64), (1, 32)])
def test_attention_ref_gpu_vs_oracle(module, block):
    for seed, (t, h, d, extreme) in enumerate(CASES):
        q, k, v = attention_ref_inputs(100 + seed, t, h, d, extreme)
        want = O.attention_ref(q, k, v, module, block)
        got = _run(q, k, v, module, block)
        assert np.all(np.isfinite(got))
        _check(got, want, v)


def test_attention_ref_gpu_module_from_environment(monkeypatch):
    """three_bit_module = -1 reads the switch as the reference does, per call."""
    q, k, v = attention_ref_inputs(7, 37, 3, 128, True)
    for name in MODULE_ENV:
        monkeypatch.delenv(name, raising=False)
    _check(_run(q, k, v, -1, 0), O.attention_ref(q, k, v, 0), v)
    monkeypatch.setenv("VSPEC_3BIT_RUNTIME_MODULE", "1")
    _check(_run(q, k, v, -1, 0), O.attention_ref(q, k, v, 1, 64), v)
    monkeypatch.setenv("VSPEC_3BIT_BLOCK_SIZE", "32")
    _check(_run(q, k, v, -1, 0), O.attention_ref(q, k, v, 1, 32), v)
    monkeypatch.setenv("VSPEC_3BIT_RUNTIME_MODULE", "0")
    monkeypatch.setenv("VSPEC_FUSED_BITS", "3")
    _check(_run(q, k, v, -1, 0), O.attention_ref(q, k, v, 1, 32), v)


def test_attention_ref_gpu_full_size():
    """8 heads x 4096 tokens x 128, module off and on: parity with the oracle, and
    the device time of the four launches next to the oracle's CPU time."""
    torch = torch_cuda()
    t, h, d = 4096, 8, 128
    q, k, v = attention_ref_inputs(5, t, h, d)
    ws = V.lib.vspec_b200_attention_ref_workspace_bytes(t, h, d)
    dq, dk, dv = to_dev(q), to_dev(k), to_dev(v)
    dout = empty_dev((h, d), torch.float32)
    dws = empty_dev((ws,), torch.uint8)
    for module in (0, 1):
        t0 = time.perf_counter()
        want = O.attention_ref(q, k, v, module, 64)
        cpu_ms = (time.perf_counter() - t0) * 1e3
        call = lambda: V.attention_ref(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dout.data_ptr(), t, h, d, module,
                                       64, dws.data_ptr(), ws)
        call()
        torch.cuda.synchronize()
        _check(dout.cpu().numpy(), want, v)
        for _ in range(3):
            call()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        e0.record()
        for _ in range(reps):
            call()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        print(f"\nattention_ref {h}x{t}x{d} module={module}: GPU {us:.1f} us/call, oracle CPU {cpu_ms:.1f} ms")


def _cache(k, v):
    t, h, d = k.shape
    return V.KVCache(k.ctypes.data, v.ctypes.data, t, h, d, t, 0, None, None, None, None, 0, 0, 0, None, None, 0)


def test_attention_demo_golden_through_cpu_semantics_backend(monkeypatch):
    """examples/attention_demo.c:32-60 after runtime init (which turns the 3-bit
    module on): the printed output, through the backend's launch_attention."""
    for name in MODULE_ENV:
        monkeypatch.delenv(name, raising=False)
    monkeypatch.setenv("VSPEC_FUSED_BITS", "4")
    monkeypatch.setenv("VSPEC_3BIT_RUNTIME_MODULE", "1")
    torch_cuda()
    q, k, v = _attention_demo_inputs()
    cache = _cache(k, v)
    out = np.zeros((2, 4), dtype=np.float32)
    ctx = V.KernelContext(q.ctypes.data, ctypes.addressof(cache), out.ctypes.data)
    be = V.lib.vspec_b200_make_cpu_semantics_backend()
    assert be.name == b"cpu-semantics-b200"
    launch = ctypes.CFUNCTYPE(None, ctypes.POINTER(V.KernelContext))(be.launch_attention)
    launch(ctypes.byref(ctx))
    assert np.array_equal(np.round(out.astype(np.float64), 4), ATTENTION_DEMO_GOLDEN)
    _check(out, O.attention_ref(q, k, v, 1, 64), v)
    # without runtime init (module off) the host entry follows the clamp-only variant
    monkeypatch.delenv("VSPEC_3BIT_RUNTIME_MODULE")
    q2, k2, v2 = attention_ref_inputs(9, 41, 4, 64, True)
    cache2 = _cache(k2, v2)
    out2 = np.zeros((4, 64), dtype=np.float32)
    ctx2 = V.KernelContext(q2.ctypes.data, ctypes.addressof(cache2), out2.ctypes.data)
    V.lib.vspec_b200_launch_attention_ref(ctypes.byref(ctx2))
    _check(out2, O.attention_ref(q2, k2, v2, 0), v2)


def test_attention_ref_argument_errors():
    torch = torch_cuda()
    assert V.lib.vspec_b200_attention_ref_workspace_bytes(10, 2, 1025) == 0
    assert V.lib.vspec_b200_attention_ref_workspace_bytes(0, 2, 64) == 0
    t, h, d = 10, 2, 64
    ws = V.lib.vspec_b200_attention_ref_workspace_bytes(t, h, d)
    buf = empty_dev((t * h * d,), torch.float32)
    dws = empty_dev((ws + 256,), torch.uint8)
    p = buf.data_ptr()
    call = V.lib.vspec_b200_attention_ref_f32
    assert call(p, p, p, t, h, d, 0, 0, dws.data_ptr(), ws - 1, p, 0) == V.ERR_ARG        # workspace too small
    assert call(p, p, p, t, h, d, 0, 0, dws.data_ptr() + 16, ws, p, 0) == V.ERR_ARG      # misaligned workspace
    assert call(p, p, p, t, h, d, 0, 48, dws.data_ptr(), ws, p, 0) == V.ERR_ARG          # block not 32/64
    assert call(p, p, p, t, h, 1025, 0, 0, dws.data_ptr(), ws, p, 0) == V.ERR_ARG        # head_dim > 1024
    assert call(p, p, p, t, h, d, 0, 0, dws.data_ptr(), ws, p, 0) == V.OK
    torch.cuda.synchronize()
