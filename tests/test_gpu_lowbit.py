"""GPU parity of the low-bit dequant-matmul (fast tensor-core path and the
any-shape path) against the oracle, through the C ABI."""
import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import RTOL_BF16, RTOL_F32, dequant_np, empty_dev, make_lowbit, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu


def run_linear(x, w, s, zp, n, k, bits, n_groups, flags=0, zp_const=0.0, residual=None, norm_w=None, eps=1e-6,
               generic=False, out_cols=None, path=None):
    torch = torch_cuda()
    m = x.shape[0]
    dx, dw = to_dev(x), to_dev(w)
    ds = to_dev(s) if s is not None else None
    dzp = to_dev(zp) if zp is not None else None
    if s is not None and s.dtype == np.float16:
        flags |= V.F_SZ_F16
    dy = empty_dev((m, out_cols or n), torch.float32)
    dres = to_dev(residual) if residual is not None else None
    dnw = to_dev(norm_w) if norm_w is not None else None
    V.lowbit_linear(dx.data_ptr(), dw.data_ptr(), ds.data_ptr() if ds is not None else None,
                    dzp.data_ptr() if dzp is not None else None, dy.data_ptr(), m, n, k, n_groups, bits, flags=flags,
                    zp_const=zp_const, residual=dres.data_ptr() if dres is not None else None,
                    norm_weight=dnw.data_ptr() if dnw is not None else None, eps=eps, generic=generic, path=path)
    torch.cuda.synchronize()
    return dy.cpu().numpy()


# ---------------------------------------------------------------- decode
@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("fast", [True, False])
def test_unpack_codes_bit_exact(bits, fast):
    torch = torch_cuda()
    rng = np.random.default_rng(bits)
    n, k = 37, 512
    w = rng.integers(0, 256, size=(n, O.row_bytes(k, bits)), dtype=np.uint8)
    dw = to_dev(w)
    out = empty_dev((n, k), torch.int8)
    for unsigned in (False, True):
        V.unpack_codes(dw.data_ptr(), n, k, bits, out.data_ptr(), unsigned=unsigned, fast=fast)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        expect = O.unpack_rows(w, n, k, bits)
        if unsigned:
            expect = O.unpack_rows_np(w, n, k, bits, unsigned=True)
        assert np.array_equal(got, expect)


def test_numpy_dequant_matches_oracle():
    rng = np.random.default_rng(5)
    for bits in (2, 3, 4):
        n, k, g = 9, 384, 3
        w, s, zp = make_lowbit(rng, n, k, bits, g)
        x = rng.standard_normal((2, k)).astype(np.float32)
        y64 = x.astype(np.float64) @ dequant_np(w, n, k, bits, s, zp, g).T
        assert np.max(np.abs(O.lowbit_matmul_f64(x, w, n, k, bits, s, zp, g) - y64)) < 1e-9


# ------------------------------------------------------------- config 1
@pytest.mark.parametrize("reading", ["literal", "unsigned"])
def test_config1_w4_gemv(reading):
    """The literal 4096 x 4096 GEMV point: x ~N(0,1) [1x4096]; 4096x4096 uniform codes 0..15 in the int4
    layout; fp32 group-128 scales ~U(0.005,0.02); zero-point 8; seed 0."""
    rng = np.random.default_rng(0)
    n = k = 4096
    g = k // 128
    x = rng.standard_normal((1, k)).astype(np.float32)
    w = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, size=(n, g)).astype(np.float32)
    if reading == "literal":   # signed decode, zp tensor = 8 (what ..._with_zero_points computes)
        zp = np.full((n, g), 8.0, dtype=np.float32)
        y = run_linear(x, w, s, zp, n, k, 4, g)
        ref = O.lowbit_matmul(x, w, n, k, 4, s, zp, g)
    else:                      # unsigned codes u - 8  ==  signed decode of (bytes ^ 0x88), zp = 0
        y = run_linear(x, w, s, None, n, k, 4, g, flags=V.F_UNSIGNED)
        ref = O.lowbit_matmul(x, w ^ np.uint8(0x88), n, k, 4, s, None, g)
    err = rel_err(y, ref)
    print(f"config1 {reading}: rel err {err:.3e}")
    assert err <= RTOL_F32


# ------------------------------------------------------------- config 2 (sweep)
@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("n", [4096, 12288])
@pytest.mark.parametrize("m", [1, 8, 64])
def test_config2_sweep(bits, n, m):
    """K=4096, N in {4096,12288}, M in {1,8,64}; group 128 fp16 scales ~U(0.005,0.02);
    zero-point at mid-range (unsigned reading); fp32 activations ~N(0,1)."""
    rng = np.random.default_rng(1000 * bits + n + m)
    k, g = 4096, 32
    w = rng.integers(0, 256, size=(n, O.row_bytes(k, bits)), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, size=(n, g)).astype(np.float16)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = run_linear(x, w, s, None, n, k, bits, g, flags=V.F_UNSIGNED)
    ref = x.astype(np.float64) @ dequant_np(w, n, k, bits, s.astype(np.float32), None, g, unsigned=True).T
    err = rel_err(y, ref)
    print(f"sweep bits={bits} n={n} m={m}: rel err {err:.3e}")
    assert err <= RTOL_F32


# ------------------------------------------------------------- shapes / options
@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("m,n,k,g", [(1, 48, 256, 2), (3, 50, 384, 1), (8, 16, 1024, 8), (5, 33, 640, 5),
                                     (2, 40, 200, 1), (1, 7, 100, 4), (4, 24, 96, 3)])
def test_shapes_fp32_scales(bits, m, n, k, g):
    rng = np.random.default_rng(m * 7 + n * 11 + k + g + bits)
    w, s, zp = make_lowbit(rng, n, k, bits, g)
    x = rng.standard_normal((m, k)).astype(np.float32)
    ref = O.lowbit_matmul(x, w, n, k, bits, s, zp, g)
    for generic in (False, True):
        y = run_linear(x, w, s, zp, n, k, bits, g, generic=generic)
        assert rel_err(y, ref) <= RTOL_F32, (generic, rel_err(y, ref))


@pytest.mark.parametrize("bits", [3, 4])
def test_fp16_scales_and_null_zero_points(bits):
    rng = np.random.default_rng(bits + 40)
    m, n, k, g = 2, 64, 512, 4
    w, s, zp = make_lowbit(rng, n, k, bits, g, sz_f16=True)
    x = rng.standard_normal((m, k)).astype(np.float32)
    assert rel_err(run_linear(x, w, s, zp, n, k, bits, g), O.lowbit_matmul(x, w, n, k, bits, s, zp, g)) <= RTOL_F32
    assert rel_err(run_linear(x, w, s, None, n, k, bits, g), O.lowbit_matmul(x, w, n, k, bits, s, None, g)) <= RTOL_F32


def test_activation_scale_extremes():
    """Per-row power-of-two rescale keeps fp32 accuracy for huge and tiny rows."""
    rng = np.random.default_rng(9)
    n, k, g = 64, 1024, 8
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    x = rng.standard_normal((4, k)).astype(np.float32)
    x[0] *= 3e4
    x[1] *= 1e-6
    x[2, ::7] *= 1e3
    x[3] = 0.0
    y = run_linear(x, w, s, zp, n, k, 4, g)
    ref = O.lowbit_matmul_f64(x, w, n, k, 4, s, zp, g)
    for i in range(3):
        assert rel_err(y[i], ref[i]) <= RTOL_F32
    assert np.all(y[3] == 0.0)


def test_fused_epilogues_residual_rmsnorm_swiglu():
    rng = np.random.default_rng(21)
    m, k, g = 3, 1024, 8
    # residual
    n = 96
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    x = rng.standard_normal((m, k)).astype(np.float32)
    res = rng.standard_normal((m, n)).astype(np.float32)
    y = run_linear(x, w, s, zp, n, k, 4, g, flags=V.F_RESIDUAL, residual=res)
    assert rel_err(y, O.lowbit_matmul_f64(x, w, n, k, 4, s, zp, g) + res) <= RTOL_F32
    # RMSNorm input (src/kernel/cuda/cuda_rmsnorm_f32.cu:9-36 semantics)
    nw = rng.uniform(0.5, 1.5, k).astype(np.float32)
    eps = 1e-6
    xh = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + eps) * nw
    y = run_linear(x, w, s, zp, n, k, 4, g, flags=V.F_RMSNORM, norm_w=nw, eps=eps)
    assert rel_err(y, xh @ dequant_np(w, n, k, 4, s, zp, g).T) <= RTOL_F32
    # SwiGLU: rows [0,n/2) gate, [n/2,n) up
    n = 128
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    full = O.lowbit_matmul_f64(x, w, n, k, 4, s, zp, g)
    gate, up = full[:, : n // 2], full[:, n // 2:]
    ref = gate / (1.0 + np.exp(-gate)) * up
    y = run_linear(x, w, s, zp, n, k, 4, g, flags=V.F_SWIGLU, out_cols=n // 2)
    assert rel_err(y, ref) <= RTOL_F32


def test_reference_named_device_launchers():
    """vspec_cuda_fused_linear_int{4,3,2}_device (cuda_fused.h:34-75) and the dequant /
    expand kernels keep the reference semantics."""
    torch = torch_cuda()
    rng = np.random.default_rng(31)
    m, n, k = 2, 40, 256
    x = rng.standard_normal((m, k)).astype(np.float32)
    dx = to_dev(x)
    dy = empty_dev((m, n), torch.float32)
    keep = []   # device tensors must outlive the asynchronous launches

    def dev(a):
        keep.append(to_dev(a))
        return keep[-1].data_ptr()

    # int4, group-wise with zp
    g = 2
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    V.lib.vspec_cuda_fused_linear_int4_device(dx.data_ptr(), dev(w), dev(s), dev(zp), dy.data_ptr(), m, n, k, g)
    torch.cuda.synchronize()
    assert rel_err(dy.cpu().numpy(), O.lowbit_matmul(x, w, n, k, 4, s, zp, g)) <= RTOL_F32
    # int3 without stochastic rounding == per-row plain contraction
    w3, s3, _ = make_lowbit(rng, n, k, 3, 1, zp_mode="none")
    V.lib.vspec_cuda_fused_linear_int3_device(dx.data_ptr(), dev(w3), dev(s3), dy.data_ptr(), m, n, k, 0)
    torch.cuda.synchronize()
    assert rel_err(dy.cpu().numpy(), O.lowbit_matmul(x, w3, n, k, 3, s3, None, 1)) <= RTOL_F32
    # int2: unsigned codes, (q - 1.5) * s[row]
    w2, s2, _ = make_lowbit(rng, n, k, 2, 1, zp_mode="none")
    V.lib.vspec_cuda_fused_linear_int2_device(dx.data_ptr(), dev(w2), dev(s2), dy.data_ptr(), m, n, k)
    torch.cuda.synchronize()
    ref2 = x.astype(np.float64) @ (((O.unpack_rows_np(w2, n, k, 2, unsigned=True) + 2).astype(np.float64) - 1.5)
                                   * s2.astype(np.float64)).T
    assert rel_err(dy.cpu().numpy(), ref2) <= RTOL_F32
    # dequant int4 -> f32 (bit-exact: one fp32 multiply per element)
    dwf = empty_dev((n, k), torch.float32)
    V.lib.vspec_cuda_dequant_int4_to_f32_device(dev(w), dev(s), dev(zp), dwf.data_ptr(), n, k, g)
    torch.cuda.synchronize()
    expect = ((O.unpack_rows(w, n, k, 4).astype(np.float32) - np.repeat(zp, k // g, axis=1))
              * np.repeat(s, k // g, axis=1))
    assert np.array_equal(dwf.cpu().numpy(), expect)
    # int3 -> int4 storage expansion: decoded codes identical
    d4 = empty_dev((n, (k + 1) // 2), torch.uint8)
    V.lib.vspec_cuda_expand_int3_to_int4_device(dev(w3), d4.data_ptr(), n, k)
    torch.cuda.synchronize()
    assert np.array_equal(O.unpack_rows(d4.cpu().numpy(), n, k, 4), O.unpack_rows(w3, n, k, 3))


def test_split_merge_is_deterministic_and_self_cleaning():
    """The split-K merge sums partials in a fixed order and leaves its counters at
    zero: repeated launches give bit-identical outputs, with the library-managed
    workspace and with a caller workspace."""
    torch = torch_cuda()
    rng = np.random.default_rng(99)
    for bits, m, n, k, g in [(4, 1, 4096, 4096, 32), (3, 2, 1000, 2048, 16), (2, 8, 4096, 1024, 8)]:
        w, s, zp = make_lowbit(rng, n, k, bits, g)
        x = rng.standard_normal((m, k)).astype(np.float32)
        dx, dw, ds, dz = to_dev(x), to_dev(w), to_dev(s), to_dev(zp)
        outs = []
        ws_bytes = V.lib.vspec_b200_lowbit_linear_workspace_bytes(m, n, k, 0)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
        for use_ws in (False, True, False, True):
            dy = empty_dev((m, n), torch.float32)
            V.lowbit_linear(dx.data_ptr(), dw.data_ptr(), ds.data_ptr(), dz.data_ptr(), dy.data_ptr(), m, n, k, g,
                            bits, workspace=ws.data_ptr() if use_ws else None, workspace_bytes=ws_bytes)
            torch.cuda.synchronize()
            outs.append(dy.cpu().numpy())
        for o in outs[1:]:
            assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32))
        counters = ws[:65536].view(torch.int32)
        assert int(counters.abs().sum().item()) == 0
        assert rel_err(outs[0], O.lowbit_matmul(x, w, n, k, bits, s, zp, g)) <= RTOL_F32


def test_workspace_too_small_is_rejected():
    torch = torch_cuda()
    rng = np.random.default_rng(7)
    n, k, g = 256, 1024, 8
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    x = rng.standard_normal((1, k)).astype(np.float32)
    dx, dw, ds, dz = to_dev(x), to_dev(w), to_dev(s), to_dev(zp)
    dy = empty_dev((1, n), torch.float32)
    ws = torch.zeros(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(V.VspecB200Error, match="workspace too small"):
        V.lowbit_linear(dx.data_ptr(), dw.data_ptr(), ds.data_ptr(), dz.data_ptr(), dy.data_ptr(), 1, n, k, g, 4,
                        workspace=ws.data_ptr(), workspace_bytes=16)



FAST_PATHS = [V.PATH_WARPMMA, V.PATH_TCGEN05, V.PATH_RING, V.PATH_ROWS]


def test_tcgen05_path_smoke():
    """One small launch of the TMA/TMEM/tcgen05 kernel first, on its own."""
    rng = np.random.default_rng(1)
    m, n, k, g = 1, 256, 1024, 8
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = run_linear(x, w, s, zp, n, k, 4, g, path=V.PATH_TCGEN05)
    flag = __import__("ctypes").c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(__import__("ctypes").byref(flag)), "timeout flag")
    assert flag.value == 0
    assert rel_err(y, O.lowbit_matmul(x, w, n, k, 4, s, zp, g)) <= RTOL_F32


def test_ring_path_smoke():
    """One small launch of the TMA-ring kernel on its own."""
    rng = np.random.default_rng(2)
    m, n, k, g = 1, 256, 1024, 8
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = run_linear(x, w, s, zp, n, k, 4, g, path=V.PATH_RING)
    flag = __import__("ctypes").c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(__import__("ctypes").byref(flag)), "timeout flag")
    assert flag.value == 0
    assert rel_err(y, O.lowbit_matmul(x, w, n, k, 4, s, zp, g)) <= RTOL_F32


@pytest.mark.parametrize("path", FAST_PATHS)
@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("m,n,k,g", [(1, 4096, 4096, 32), (1, 1000, 2048, 16), (3, 384, 1024, 8), (4, 130, 512, 1),
                                     (2, 12288, 4096, 32), (1, 200, 12288, 96), (8, 640, 1024, 8),
                                     (6, 300, 2048, 16)])
def test_fast_paths_match_oracle(path, bits, m, n, k, g):
    if path == V.PATH_TCGEN05 and m > 4:
        pytest.skip("the tcgen05 GEMV takes m <= 4")
    if path == V.PATH_ROWS and k % (2048 if bits == 4 else 1024) != 0:
        pytest.skip("the row-sliced GEMV takes k % 1024 == 0 (int4: k % 2048 == 0)")
    rng = np.random.default_rng(path * 100 + bits * 10 + m + n + k)
    w, s, zp = make_lowbit(rng, n, k, bits, g, sz_f16=(n % 2 == 0))
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = run_linear(x, w, s, zp, n, k, bits, g, path=path)
    ref = x.astype(np.float64) @ dequant_np(w, n, k, bits, s.astype(np.float32), zp.astype(np.float32), g).T
    err = rel_err(y, ref)
    print(f"path={path} bits={bits} m={m} n={n} k={k}: {err:.2e}")
    assert err <= RTOL_F32


@pytest.mark.parametrize("path", FAST_PATHS)
def test_fast_paths_fused_epilogues(path):
    rng = np.random.default_rng(70 + path)
    m, k, g = (3, 2048, 16) if path == V.PATH_ROWS else (3, 1024, 8)   # row-sliced int4: k % 2048
    n = 512   # SwiGLU halves of 256 rows fill one tile of every fast path
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    x = rng.standard_normal((m, k)).astype(np.float32)
    res = rng.standard_normal((m, n)).astype(np.float32)
    full = O.lowbit_matmul_f64(x, w, n, k, 4, s, zp, g)
    y = run_linear(x, w, s, zp, n, k, 4, g, flags=V.F_RESIDUAL, residual=res, path=path)
    assert rel_err(y, full + res) <= RTOL_F32
    nw = rng.uniform(0.5, 1.5, k).astype(np.float32)
    xh = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * nw
    y = run_linear(x, w, s, zp, n, k, 4, g, flags=V.F_RMSNORM, norm_w=nw, eps=1e-6, path=path)
    assert rel_err(y, xh @ dequant_np(w, n, k, 4, s, zp, g).T) <= RTOL_F32
    gate, up = full[:, : n // 2], full[:, n // 2:]
    y = run_linear(x, w, s, zp, n, k, 4, g, flags=V.F_SWIGLU, out_cols=n // 2, path=path)
    assert rel_err(y, gate / (1.0 + np.exp(-gate)) * up) <= RTOL_F32


def test_rows_path_smoke():
    """One small launch of the row-sliced kernel on its own."""
    rng = np.random.default_rng(3)
    m, n, k, g = 1, 256, 2048, 16
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = run_linear(x, w, s, zp, n, k, 4, g, path=V.PATH_ROWS)
    flag = __import__("ctypes").c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(__import__("ctypes").byref(flag)), "timeout flag")
    assert flag.value == 0
    assert rel_err(y, O.lowbit_matmul(x, w, n, k, 4, s, zp, g)) <= RTOL_F32


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("m,n,k,g,flags", [
    (1, 24, 2048, 16, 0),                  # three CTAs of eight rows, one box each
    (1, 18000, 2048, 16, 0),               # 60-61 rows per CTA: one 64-row group
    (6, 9000, 2048, 8, 0),                 # m > 4 (two activation tiles), groups of 256 codes
    (2, 4104, 2048, 16, 0),                # rows per CTA not a multiple of 16
    (2, 36000, 2048, 16, 0x10),            # SwiGLU: a gate group and its up group per CTA
    (3, 10000, 4096, 32, 0x4),             # residual
    (1, 5000, 4096, 16, 0x8),              # RMSNorm input, groups of 256 codes
    (8, 4096, 4096, 32, 0),                # m = 8: large activation fragments in shared memory
])
def test_rows_path_shapes(bits, m, n, k, g, flags):
    """Row-sliced kernel at shapes that exercise its geometry: tiny CTAs, row
    groups, partial 16-row blocks, every epilogue; fp32 scales + zero-points
    (fp16 when g is a multiple of 8)."""
    rng = np.random.default_rng(bits * 1000 + m * 10 + (n % 997) + flags)
    w, s, zp = make_lowbit(rng, n, k, bits, g, sz_f16=(g % 8 == 0))
    x = rng.standard_normal((m, k)).astype(np.float32)
    sf, zf = s.astype(np.float32), zp.astype(np.float32)
    full = O.lowbit_matmul(x, w, n, k, bits, sf, zf, g).astype(np.float64)
    if flags & V.F_SWIGLU:
        gate, up = full[:, : n // 2], full[:, n // 2:]
        ref = gate / (1.0 + np.exp(-gate)) * up
        y = run_linear(x, w, s, zp, n, k, bits, g, flags=flags, out_cols=n // 2, path=V.PATH_ROWS)
    elif flags & V.F_RESIDUAL:
        res = rng.standard_normal((m, n)).astype(np.float32)
        ref = full + res
        y = run_linear(x, w, s, zp, n, k, bits, g, flags=flags, residual=res, path=V.PATH_ROWS)
    elif flags & V.F_RMSNORM:
        nw = rng.uniform(0.5, 1.5, k).astype(np.float32)
        xh = (x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6)
              * nw).astype(np.float32)
        ref = O.lowbit_matmul(xh, w, n, k, bits, sf, zf, g)
        y = run_linear(x, w, s, zp, n, k, bits, g, flags=flags, norm_w=nw, eps=1e-6, path=V.PATH_ROWS)
    else:
        ref = full
        y = run_linear(x, w, s, zp, n, k, bits, g, path=V.PATH_ROWS)
    flag = __import__("ctypes").c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(__import__("ctypes").byref(flag)), "timeout flag")
    assert flag.value == 0
    err = rel_err(y, ref)
    print(f"rows bits={bits} m={m} n={n} k={k} flags={flags}: {err:.2e}")
    assert err <= RTOL_F32


def test_rows_path_deterministic_and_unsupported_shapes():
    """Two launches give bit-identical output; shapes outside the kernel's
    contract are refused on the host when requested explicitly."""
    rng = np.random.default_rng(123)
    m, n, k, g = 2, 12288, 4096, 32
    w, s, _ = make_lowbit(rng, n, k, 4, g, sz_f16=True, zp_mode="none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    f = V.F_UNSIGNED | V.F_SZ_F16
    y1 = run_linear(x, w, s, None, n, k, 4, g, flags=f, path=V.PATH_ROWS)
    y2 = run_linear(x, w, s, None, n, k, 4, g, flags=f, path=V.PATH_ROWS)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    ref = x.astype(np.float64) @ dequant_np(w, n, k, 4, s.astype(np.float32), None, g, unsigned=True).T
    assert rel_err(y1, ref) <= RTOL_F32
    w5, s5, zp5 = make_lowbit(rng, 64, 640, 4, 5)
    x5 = rng.standard_normal((1, 640)).astype(np.float32)
    with pytest.raises(V.VspecB200Error, match="not supported"):
        run_linear(x5, w5, s5, zp5, 64, 640, 4, 5, path=V.PATH_ROWS)
    # more rows per CTA than one 64-row group: refused explicitly, the ring kernel in auto dispatch
    wl, sl, zl = make_lowbit(rng, 40000, 2048, 4, 16)
    xl = rng.standard_normal((1, 2048)).astype(np.float32)
    with pytest.raises(V.VspecB200Error, match="not supported"):
        run_linear(xl, wl, sl, zl, 40000, 2048, 4, 16, path=V.PATH_ROWS)
    assert rel_err(run_linear(xl, wl, sl, zl, 40000, 2048, 4, 16), O.lowbit_matmul(xl, wl, 40000, 2048, 4, sl, zl, 16)) \
        <= RTOL_F32


@pytest.mark.parametrize("m,n", [(1, 12288), (4, 9984), (7, 12288)])
def test_ring_cluster_merge_epilogues(m, n):
    """Shapes whose tiles split over 2..8 CTAs per tile take the cluster
    (distributed shared memory) split-K merge: residual and RMSNorm epilogues
    against the oracle, and the result bit-identical to a second launch."""
    rng = np.random.default_rng(90 + m)
    k, g, bits = 4096, 32, 4
    w, s, zp = make_lowbit(rng, n, k, bits, g, sz_f16=True, zp_mode="none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    res = rng.standard_normal((m, n)).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, k).astype(np.float32)
    xh = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * nw
    deq = dequant_np(w, n, k, bits, s, None, g, unsigned=True)
    y = run_linear(x, w, s, None, n, k, bits, g, flags=V.F_RESIDUAL | V.F_UNSIGNED | V.F_SZ_F16, residual=res,
                   path=V.PATH_RING)
    assert rel_err(y, x.astype(np.float64) @ deq.T + res) <= RTOL_F32
    f = V.F_RMSNORM | V.F_UNSIGNED | V.F_SZ_F16
    y1 = run_linear(x, w, s, None, n, k, bits, g, flags=f, norm_w=nw, eps=1e-6, path=V.PATH_RING)
    y2 = run_linear(x, w, s, None, n, k, bits, g, flags=f, norm_w=nw, eps=1e-6, path=V.PATH_RING)
    assert rel_err(y1, xh @ deq.T) <= RTOL_F32
    assert np.array_equal(y1, y2)


def test_large_n_beyond_tile_counters():
    """More output tiles than split-K counters (the fixed 16384-slot region):
    automatic dispatch stays correct (the any-shape kernel runs) and the
    explicit warp-MMA path refuses the shape instead of overrunning them."""
    rng = np.random.default_rng(77)
    m, n, k, g, bits = 5, 270000, 128, 1, 4
    w, s, zp = make_lowbit(rng, n, k, bits, g)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = run_linear(x, w, s, zp, n, k, bits, g)
    ref = x.astype(np.float64) @ dequant_np(w, n, k, bits, s, zp, g).T
    assert rel_err(y, ref) <= RTOL_F32
    with pytest.raises(V.VspecB200Error, match="not supported"):
        run_linear(x, w, s, zp, n, k, bits, g, path=V.PATH_WARPMMA)


@pytest.mark.parametrize("m,flags", [(8, 0), (8, V.F_RESIDUAL), (7, V.F_RMSNORM), (8, V.F_SWIGLU), (5, 0)])
def test_deep_k_many_rows_auto_dispatch(m, flags):
    """k = 12288 (the Qwen3-8B down projection) at 5-8 activation rows: the
    fast kernels cannot hold every k-block of all rows in shared memory, so
    automatic dispatch runs the rows in halves on them (the one-warp-per-row
    kernel took ~1.5 ms per call there).  Checked against the oracle with the
    timeout flag clear."""
    import ctypes
    rng = np.random.default_rng(900 + m + flags)
    n, k, g, bits = 1024, 12288, 96, 4
    w, s, zp = make_lowbit(rng, n, k, bits, g, sz_f16=True, zp_mode="none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    f = V.F_UNSIGNED | flags
    deq = dequant_np(w, n, k, bits, s.astype(np.float32), None, g, unsigned=True)
    if flags & V.F_RMSNORM:
        nw = rng.uniform(0.5, 1.5, k).astype(np.float32)
        xh = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * nw
        y = run_linear(x, w, s, None, n, k, bits, g, flags=f, norm_w=nw)
        ref = xh @ deq.T
    elif flags & V.F_RESIDUAL:
        res = rng.standard_normal((m, n)).astype(np.float32)
        y = run_linear(x, w, s, None, n, k, bits, g, flags=f, residual=res)
        ref = x.astype(np.float64) @ deq.T + res
    elif flags & V.F_SWIGLU:
        full = x.astype(np.float64) @ deq.T
        gate, up = full[:, : n // 2], full[:, n // 2:]
        y = run_linear(x, w, s, None, n, k, bits, g, flags=f, out_cols=n // 2)
        ref = gate / (1.0 + np.exp(-gate)) * up
    else:
        y = run_linear(x, w, s, None, n, k, bits, g, flags=f)
        ref = x.astype(np.float64) @ deq.T
    flag = ctypes.c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(ctypes.byref(flag)), "timeout flag")
    assert flag.value == 0
    assert rel_err(y, ref) <= RTOL_F32


@pytest.mark.parametrize("m,n,flags", [(8, 12288, 0), (5, 12288, V.F_RESIDUAL), (6, 12288, V.F_RMSNORM),
                                         (8, 24576, V.F_SWIGLU)])
def test_large_weights_many_rows_run_in_halves(m, n, flags):
    """More than four activation rows on weights of n * k >= 12288 * 4096: automatic dispatch runs the
    rows in two halves of one MMA column tile each (faster there than one two-tile call).  Every
    epilogue against the oracle, with the timeout flag clear."""
    import ctypes
    rng = np.random.default_rng(950 + m + flags)
    k, g, bits = 4096, 32, 4
    w, s, zp = make_lowbit(rng, n, k, bits, g, sz_f16=True, zp_mode="none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    f = V.F_UNSIGNED | flags
    deq = dequant_np(w, n, k, bits, s.astype(np.float32), None, g, unsigned=True)
    if flags & V.F_RMSNORM:
        nw = rng.uniform(0.5, 1.5, k).astype(np.float32)
        xh = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * nw
        y = run_linear(x, w, s, None, n, k, bits, g, flags=f, norm_w=nw)
        ref = xh @ deq.T
    elif flags & V.F_RESIDUAL:
        res = rng.standard_normal((m, n)).astype(np.float32)
        y = run_linear(x, w, s, None, n, k, bits, g, flags=f, residual=res)
        ref = x.astype(np.float64) @ deq.T + res
    elif flags & V.F_SWIGLU:
        full = x.astype(np.float64) @ deq.T
        gate, up = full[:, : n // 2], full[:, n // 2:]
        y = run_linear(x, w, s, None, n, k, bits, g, flags=f, out_cols=n // 2)
        ref = gate / (1.0 + np.exp(-gate)) * up
    else:
        y = run_linear(x, w, s, None, n, k, bits, g, flags=f)
        ref = x.astype(np.float64) @ deq.T
    flag = ctypes.c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(ctypes.byref(flag)), "timeout flag")
    assert flag.value == 0
    assert rel_err(y, ref) <= RTOL_F32


@pytest.mark.parametrize("k", [5120, 6144])
def test_ring_split_k_merge_back_to_back(k):
    """The Qwen3-32B-shape lm_head (n = 151936) at k = 5120 / 6144 runs the ring
    kernel's general split-K (CTA runs crossing tile boundaries, cross-CTA
    merges through the workspace).  32 launches back to back in a CUDA graph,
    every one against the oracle: a merge that reads a partial before it is
    visible shows up as a few stale rows in some launches."""
    torch = torch_cuda()
    import ctypes
    rng = np.random.default_rng(k)
    m, n, g, bits, reps = 1, 151936, k // 128, 4, 32
    w, s, _ = make_lowbit(rng, n, k, bits, g, sz_f16=True, zp_mode="none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    ref = O.lowbit_matmul(x, w, n, k, bits, s, None, g)
    dx, dw, ds = to_dev(x), to_dev(w), to_dev(s)
    ys = [empty_dev((m, n), torch.float32) for _ in range(reps)]
    st = torch.cuda.Stream()

    def step():
        for y in ys:
            V.lowbit_linear(dx.data_ptr(), dw.data_ptr(), ds.data_ptr(), None, y.data_ptr(), m, n, k, g, bits,
                            flags=V.F_SZ_F16, stream=st.cuda_stream, path=V.PATH_RING)
    with torch.cuda.stream(st):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        step()
    for _ in range(2):
        for y in ys:
            y.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        errs = [rel_err(y.cpu().numpy(), ref) for y in ys]
        assert max(errs) <= RTOL_F32, [f"{e:.1e}" for e in errs]
    del graph
    flag = ctypes.c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(ctypes.byref(flag)), "timeout flag")
    assert flag.value == 0


@pytest.mark.parametrize("m,n,k,bits,flags", [(1, 12288, 4096, 4, 0), (4, 24576, 4096, 4, 0x10), (2, 12288, 4096, 3, 0),
                                              (1, 6144, 4096, 2, 0)])
def test_rows_ring_wrap_back_to_back(m, n, k, bits, flags):
    """Row-sliced GEMV shapes whose shared-memory ring wraps (fewer stages than
    units), 32 launches back to back in a CUDA graph, replayed 3 times: every
    launch matches the oracle and no bounded wait gives up.  A ring whose stage
    count is not a multiple of the 8 consumer warps let a warp's parity wait
    pass one phase early when TMA copies landed out of order (a timeout in a
    few thousand launches)."""
    torch = torch_cuda()
    import ctypes
    rng = np.random.default_rng(n + m + bits)
    g, reps = k // 128, 32
    w, s, _ = make_lowbit(rng, n, k, bits, g, sz_f16=True, zp_mode="none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    full = O.lowbit_matmul(x, w, n, k, bits, s, None, g).astype(np.float64)
    swiglu = bool(flags & V.F_SWIGLU)
    ref = full[:, : n // 2] / (1.0 + np.exp(-full[:, : n // 2])) * full[:, n // 2:] if swiglu else full
    out_cols = n // 2 if swiglu else n
    dx, dw, ds = to_dev(x), to_dev(w), to_dev(s)
    ys = [empty_dev((m, out_cols), torch.float32) for _ in range(reps)]
    st = torch.cuda.Stream()

    def step():
        for y in ys:
            V.lowbit_linear(dx.data_ptr(), dw.data_ptr(), ds.data_ptr(), None, y.data_ptr(), m, n, k, g, bits,
                            flags=V.F_SZ_F16 | flags, stream=st.cuda_stream, path=V.PATH_ROWS)
    with torch.cuda.stream(st):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        step()
    for _ in range(3):
        for y in ys:
            y.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        errs = [rel_err(y.cpu().numpy(), ref) for y in ys]
        assert max(errs) <= RTOL_F32, [f"{e:.1e}" for e in errs]
    del graph
    flag = ctypes.c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(ctypes.byref(flag)), "timeout flag")
    assert flag.value == 0


# ---------------------------------------------------------------- tcgen05 GEMM (m > 8)
def test_gemm_tcgen05_smoke():
    """One small launch of the tcgen05 GEMM on its own (fp16 operands, tolerance RTOL_BF16)."""
    rng = np.random.default_rng(5)
    m, n, k, g = 16, 128, 128, 1
    w, s, zp = make_lowbit(rng, n, k, 4, g)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = run_linear(x, w, s, zp, n, k, 4, g, path=V.PATH_TCGEN05)
    flag = __import__("ctypes").c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(__import__("ctypes").byref(flag)), "timeout flag")
    assert flag.value == 0
    ref = x.astype(np.float64) @ dequant_np(w, n, k, 4, s, zp, g).T
    err = rel_err(y, ref)
    print(f"gemm smoke err {err:.3e}")
    assert err <= RTOL_BF16


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("m,n,k,g", [(16, 256, 512, 4), (64, 1024, 2048, 16), (130, 384, 1024, 8),
                                     (512, 4096, 4096, 32)])
def test_gemm_tcgen05_matches_oracle(bits, m, n, k, g):
    rng = np.random.default_rng(900 + bits * 10 + m)
    w, s, zp = make_lowbit(rng, n, k, bits, g, sz_f16=(m == 64))
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = run_linear(x, w, s, zp, n, k, bits, g)
    ref = x.astype(np.float64) @ dequant_np(w, n, k, bits, s.astype(np.float32), zp.astype(np.float32), g).T
    err = rel_err(y, ref)
    print(f"gemm bits={bits} m={m} n={n} k={k}: {err:.3e}")
    assert err <= RTOL_BF16


def test_gemm_tcgen05_unsigned_and_fused_epilogues():
    rng = np.random.default_rng(919)
    m, n, k, g = 48, 512, 1024, 8
    w, s, _ = make_lowbit(rng, n, k, 4, g, sz_f16=True, zp_mode="none")
    x = rng.standard_normal((m, k)).astype(np.float32)
    deq = dequant_np(w, n, k, 4, s.astype(np.float32), None, g, unsigned=True, zp_const=8.0)
    full = x.astype(np.float64) @ deq.T
    y = run_linear(x, w, s, None, n, k, 4, g, flags=V.F_UNSIGNED, zp_const=8.0)
    assert rel_err(y, full) <= RTOL_BF16
    res = rng.standard_normal((m, n)).astype(np.float32)
    y = run_linear(x, w, s, None, n, k, 4, g, flags=V.F_UNSIGNED | V.F_RESIDUAL, zp_const=8.0, residual=res)
    assert rel_err(y, full + res) <= RTOL_BF16
    nw = rng.uniform(0.5, 1.5, k).astype(np.float32)
    xh = x.astype(np.float64) / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * nw
    y = run_linear(x, w, s, None, n, k, 4, g, flags=V.F_UNSIGNED | V.F_RMSNORM, zp_const=8.0, norm_w=nw, eps=1e-6)
    assert rel_err(y, xh @ deq.T) <= RTOL_BF16
    gate, up = full[:, : n // 2], full[:, n // 2:]
    y = run_linear(x, w, s, None, n, k, 4, g, flags=V.F_UNSIGNED | V.F_SWIGLU, zp_const=8.0, out_cols=n // 2)
    assert rel_err(y, gate / (1.0 + np.exp(-gate)) * up) <= RTOL_BF16
