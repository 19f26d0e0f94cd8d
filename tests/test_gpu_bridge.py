"""GPU tests of the reference-named host-pointer surface: the cuda_bridge.c
exports (registry semantics, stats, dispatch paths), the VspecKernelContext
launchers, the CUDA VspecBackend, and host-side failure paths."""
import ctypes
from ctypes import byref, c_int, c_size_t, c_uint64

import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import RTOL_F32, make_lowbit, rel_err, torch_cuda

pytestmark = pytest.mark.gpu


def stats():
    s = [c_uint64() for _ in range(6)]
    assert V.lib.vspec_cuda_int4_cached_stats_bridge(*[byref(x) for x in s]) == 1
    return [x.value for x in s]


def test_registry_register_cached_many_and_stats():
    torch_cuda()
    rng = np.random.default_rng(1)
    k = 512
    ws = []
    for n in (96, 32, 64):
        w, s, zp = make_lowbit(rng, n, k, 4, 4, zp_mode="int")
        ws.append((n, w, s, zp))
    x = rng.standard_normal((2, k)).astype(np.float32)
    before = stats()
    handles = []
    for n, w, s, zp in ws:
        h = V.lib.vspec_cuda_fused_linear_int4_register_weight_bridge(w.ctypes.data, s.ctypes.data, zp.ctypes.data,
                                                                       k, n, 4)
        assert h > 0
        handles.append(h)
    # same arrays again -> same handle, counted as reuse (cuda_bridge.c:433-436)
    n, w, s, zp = ws[0]
    assert V.lib.vspec_cuda_fused_linear_int4_register_weight_bridge(w.ctypes.data, s.ctypes.data, zp.ctypes.data, k,
                                                                      n, 4) == handles[0]
    for (n, w, s, zp), h in zip(ws, handles):
        out = np.zeros((2, n), dtype=np.float32)
        assert V.lib.vspec_cuda_fused_linear_int4_cached_bridge(x.ctypes.data, 2, k, h, n, out.ctypes.data) == 1
        assert rel_err(out, O.lowbit_matmul(x, w, n, k, 4, s, zp, 4)) <= RTOL_F32
    # wrong expected_n -> miss, 0
    out = np.zeros((2, 96), dtype=np.float32)
    assert V.lib.vspec_cuda_fused_linear_int4_cached_bridge(x.ctypes.data, 2, k, handles[1], 96, out.ctypes.data) == 0
    # many: outputs concatenated [m][n_i] blocks
    hs = (c_int * 3)(*handles)
    dims = (c_size_t * 3)(*[n for n, *_ in ws])
    total = sum(n for n, *_ in ws)
    out = np.zeros(2 * total, dtype=np.float32)
    assert V.lib.vspec_cuda_fused_linear_int4_cached_many_bridge(x.ctypes.data, 2, k, ctypes.cast(hs, ctypes.c_void_p),
                                                                 ctypes.cast(dims, ctypes.c_void_p), 3,
                                                                 out.ctypes.data) == 1
    off = 0
    for n, w, s, zp in ws:
        blk = out[off: off + 2 * n].reshape(2, n)
        assert rel_err(blk, O.lowbit_matmul(x, w, n, k, 4, s, zp, 4)) <= RTOL_F32
        off += 2 * n
    after = stats()
    assert after[3] - before[3] == 4      # register calls
    assert after[4] - before[4] == 1      # register reuse
    assert after[2] - before[2] == 1      # one miss
    assert after[1] - before[1] == 3 + 3  # hits: 3 cached + 3 inside many


def test_uncached_int4_bridge_and_dispatch_paths():
    torch_cuda()
    rng = np.random.default_rng(2)
    m, n, k, g = 3, 80, 256, 2
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    x = rng.standard_normal((m, k)).astype(np.float32)
    out = np.zeros((m, n), dtype=np.float32)
    assert V.lib.vspec_cuda_fused_linear_int4_bridge(x.ctypes.data, w.ctypes.data, s.ctypes.data, zp.ctypes.data, m, k,
                                                     n, g, out.ctypes.data) == 1
    ref = O.lowbit_matmul(x, w, n, k, 4, s, zp, g)
    assert rel_err(out, ref) <= RTOL_F32
    # dispatch: bits 4 registers on first use and reports path 1
    handle, path = c_int(0), c_int(0)
    out[:] = 0
    assert V.lib.vspec_cuda_gemm_dispatch_bridge(x.ctypes.data, None, w.ctypes.data, s.ctypes.data, zp.ctypes.data, m, k,
                                                 n, g, 4, byref(handle), out.ctypes.data, byref(path)) == 1
    assert handle.value > 0 and path.value == 1 and rel_err(out, ref) <= RTOL_F32
    # bits 3 -> path 3 (stochastic-rounding int3 bridge); no packed -> fp32 GEMM path 4
    w3, s3, _ = make_lowbit(rng, n, k, 3, 1, zp_mode="none")
    assert V.lib.vspec_cuda_gemm_dispatch_bridge(x.ctypes.data, None, w3.ctypes.data, s3.ctypes.data, None, m, k, n, 1,
                                                 3, None, out.ctypes.data, byref(path)) == 1
    assert path.value == 3
    wf = rng.standard_normal((n, k)).astype(np.float32)
    assert V.lib.vspec_cuda_gemm_dispatch_bridge(x.ctypes.data, wf.ctypes.data, None, None, None, m, k, n, 0, 0, None,
                                                 out.ctypes.data, byref(path)) == 1
    assert path.value == 4
    assert rel_err(out, x.astype(np.float64) @ wf.T.astype(np.float64)) <= RTOL_F32


def test_int3_bridge_reproduces_reference_stochastic_rounding():
    """cuda_bridge.c:1155 runs the int3 kernel with stochastic rounding; the
    per-element rounding decisions are reproduced, so the result matches the
    oracle restatement of fused_linear_int3.cu:82-147 to fp32 rounding."""
    torch_cuda()
    rng = np.random.default_rng(3)
    m, n, k = 2, 48, 300
    w3, s3, _ = make_lowbit(rng, n, k, 3, 1, zp_mode="none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    out = np.zeros((m, n), dtype=np.float32)
    assert V.lib.vspec_cuda_fused_linear_int3_bridge(x.ctypes.data, w3.ctypes.data, s3.ctypes.data, m, k, n,
                                                     out.ctypes.data) == 1
    ref = np.zeros((m, n), dtype=np.float32)
    O.ORACLE.oracle_int3_blocknorm_f32(x.ctypes.data, m, k, w3.ctypes.data, n, s3.ctypes.data, 1, ref.ctypes.data)
    assert rel_err(out, ref) <= RTOL_F32
    plain = O.lowbit_matmul(x, w3, n, k, 3, s3, None, 1)
    assert rel_err(ref, plain) > 1e-4     # stochastic rounding does change the result


def make_ctx(x, w, s, out, m, n, k, qtype):
    ctx = V.KernelContext()
    ctx.input = x.ctypes.data
    ctx.weight = w.ctypes.data
    ctx.output = out.ctypes.data
    ctx.qmeta.type = qtype
    ctx.qmeta.scales = s.ctypes.data
    ctx.qmeta.scale_count = n
    ctx.config.m, ctx.config.n, ctx.config.k = m, n, k
    return ctx


def test_backend_int4_demo_golden():
    """examples/int4_demo.c through vspec_make_cuda_backend(): the CPU backend's
    mean-code zero-point semantics give the demo's printed output."""
    torch_cuda()
    a = np.array([1, 2, 3, 4, 4, 3, 2, 1], dtype=np.float32)
    q = np.array([[1, 0, -1, 2], [2, -2, 1, 0], [-1, 1, 1, -2]], dtype=np.int8)
    packed = O.pack_rows(q, 4)
    s = np.array([0.5, 0.25, 0.75], dtype=np.float32)
    out = np.zeros(6, dtype=np.float32)
    be = V.lib.vspec_make_cuda_backend()
    assert be.name == b"cuda-b200"
    launch = ctypes.CFUNCTYPE(None, ctypes.POINTER(V.KernelContext))(be.launch_linear)
    ctx = make_ctx(a, packed, s, out, 2, 3, 4, V.QUANT_INT4)
    launch(byref(ctx))
    golden = np.array([0.500, -0.375, -1.125, -0.500, 0.375, 1.125], dtype=np.float32)
    assert np.allclose(out, golden, atol=5e-4)


def test_context_launchers():
    torch_cuda()
    rng = np.random.default_rng(4)
    m, n, k = 2, 64, 384
    x = rng.standard_normal((m, k)).astype(np.float32)
    # int4 context: per-row scales, zp = NULL (fused_linear_int4.cu:634)
    w, s, _ = make_lowbit(rng, n, k, 4, 1, zp_mode="none")
    out = np.zeros((m, n), dtype=np.float32)
    ctx = make_ctx(x, w, s, out, m, n, k, V.QUANT_INT4)
    V.lib.vspec_cuda_launch_fused_linear_int4(byref(ctx))
    assert rel_err(out, O.lowbit_matmul(x, w, n, k, 4, s, None, 1)) <= RTOL_F32
    # int3 storage context == plain per-row int3
    w3, s3, _ = make_lowbit(rng, n, k, 3, 1, zp_mode="none")
    out[:] = 0
    ctx = make_ctx(x, w3, s3, out, m, n, k, V.QUANT_INT3)
    V.lib.vspec_cuda_launch_fused_linear_int3_storage(byref(ctx))
    assert rel_err(out, O.lowbit_matmul(x, w3, n, k, 3, s3, None, 1)) <= RTOL_F32
    # int3 context: clamp 2.8 std, block-normalized, stochastic rounding
    out[:] = 0
    V.lib.vspec_cuda_launch_fused_linear_int3(byref(ctx))
    xc = np.zeros_like(x)
    O.ORACLE.oracle_clamp_rows_std(x.ctypes.data, m, k, 2.8, xc.ctypes.data)
    ref = np.zeros((m, n), dtype=np.float32)
    O.ORACLE.oracle_int3_blocknorm_f32(xc.ctypes.data, m, k, w3.ctypes.data, n, s3.ctypes.data, 1, ref.ctypes.data)
    assert rel_err(out, ref) <= RTOL_F32
    # int2 context: unsigned codes (q - 1.5) * s
    w2, s2, _ = make_lowbit(rng, n, k, 2, 1, zp_mode="none")
    out[:] = 0
    ctx = make_ctx(x, w2, s2, out, m, n, k, V.QUANT_INT2)
    V.lib.vspec_cuda_launch_fused_linear_int2(byref(ctx))
    ref2 = x.astype(np.float64) @ ((O.unpack_rows_np(w2, n, k, 2, unsigned=True).astype(np.float64) + 0.5)
                                   * s2.astype(np.float64)).T
    assert rel_err(out, ref2) <= RTOL_F32


def test_f32_helper_bridges():
    torch_cuda()
    rng = np.random.default_rng(6)
    rows, dim = 3, 256
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, dim).astype(np.float32)
    out = np.zeros_like(x)
    V.lib.vspec_cuda_rmsnorm_f32_bridge(x.ctypes.data, w.ctypes.data, 1e-6, rows, dim, out.ctypes.data)
    ref = x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * w
    assert rel_err(out, ref) <= 1e-5
    d = x.reshape(-1).copy()
    V.lib.vspec_cuda_silu_f32_bridge(d.ctypes.data, d.size)
    assert rel_err(d, x.reshape(-1) / (1 + np.exp(-x.reshape(-1).astype(np.float64)))) <= 1e-5
    b = rng.standard_normal(x.size).astype(np.float32)
    o = np.zeros(x.size, dtype=np.float32)
    V.lib.vspec_cuda_mul_f32_bridge(x.ctypes.data, b.ctypes.data, x.size, o.ctypes.data)
    assert np.array_equal(o, x.reshape(-1) * b)
    wl = rng.standard_normal((40, dim)).astype(np.float32)
    yl = np.zeros((rows, 40), dtype=np.float32)
    V.lib.vspec_cuda_linear_f32_bridge(x.ctypes.data, wl.ctypes.data, rows, dim, 40, yl.ctypes.data)
    assert rel_err(yl, x.astype(np.float64) @ wl.T) <= 1e-5
    free, total = c_size_t(), c_size_t()
    assert V.lib.vspec_cuda_mem_info_bridge(byref(free), byref(total)) == 1 and total.value > 100e9
    maj, mnr, sms = c_int(), c_int(), c_int()
    assert V.lib.vspec_cuda_device_capability_bridge(byref(maj), byref(mnr), byref(sms)) == 1
    assert maj.value == 10 and sms.value >= 100
    assert V.lib.vspec_cuda_int4_tensorcore_available_bridge() == 1


def test_allocation_failure_makes_bridges_fail_closed():
    """Host-side fault injection: a failed device allocation makes the bridge
    return 0 (the reference caller then falls back) and leaves the library usable."""
    torch_cuda()
    rng = np.random.default_rng(8)
    n, k = 32, 256
    w, s, zp = make_lowbit(rng, n, k, 4, 2)
    x = rng.standard_normal((1, k)).astype(np.float32)
    V.lib.vspec_b200_debug_fail_alloc_after(0)
    assert V.lib.vspec_cuda_fused_linear_int4_register_weight_bridge(w.ctypes.data, s.ctypes.data, zp.ctypes.data, k,
                                                                       n, 2) == 0
    h = V.lib.vspec_cuda_fused_linear_int4_register_weight_bridge(w.ctypes.data, s.ctypes.data, zp.ctypes.data, k, n, 2)
    assert h > 0
    out = np.zeros(n, dtype=np.float32)
    assert V.lib.vspec_cuda_fused_linear_int4_cached_bridge(x.ctypes.data, 1, k, h, n, out.ctypes.data) == 1
    assert rel_err(out, O.lowbit_matmul(x, w, n, k, 4, s, zp, 2)[0]) <= RTOL_F32


def test_cached_bridge_graph_replays_follow_inputs_and_m():
    """A registered weight's call runs directly first, then as one captured
    graph (upload, linear, download): consecutive calls with new activations,
    a change of activation count (recapture) and back all match the oracle,
    and the stats count every call as a hit."""
    torch_cuda()
    rng = np.random.default_rng(404)
    n, k, g = 2048, 4096, 32
    w = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, size=(n, g)).astype(np.float32)
    zp = rng.uniform(-2.0, 2.0, size=(n, g)).astype(np.float32)
    h = V.lib.vspec_cuda_fused_linear_int4_register_weight_bridge(w.ctypes.data, s.ctypes.data, zp.ctypes.data, k, n,
                                                                   g)
    assert h > 0
    before = [ctypes.c_uint64() for _ in range(6)]
    V.lib.vspec_cuda_int4_cached_stats_bridge(*[ctypes.byref(c) for c in before])
    for m in (1, 1, 1, 3, 3, 1, 1):
        x = rng.standard_normal((m, k)).astype(np.float32)
        out = np.full((m, n), np.nan, dtype=np.float32)
        assert V.lib.vspec_cuda_fused_linear_int4_cached_bridge(x.ctypes.data, m, k, h, n, out.ctypes.data) == 1
        assert rel_err(out, O.lowbit_matmul(x, w, n, k, 4, s, zp, g)) <= RTOL_F32, m
    after = [ctypes.c_uint64() for _ in range(6)]
    V.lib.vspec_cuda_int4_cached_stats_bridge(*[ctypes.byref(c) for c in after])
    assert after[1].value - before[1].value == 7   # hits
