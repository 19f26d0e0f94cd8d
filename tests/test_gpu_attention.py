"""GPU parity of the paged GQA decode attention against the oracle (and of the
page-table gather against the reference's own paged cache), through the C ABI."""
import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import RTOL_F32, empty_dev, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu


def make_paged(rng, batch, hkv, d, ctx_lens, pt, dtype=np.float16, extra_pages=3):
    """Seeded pool = sum ceil(ctx/pt) pages (+ spare), page table = seeded permutation."""
    need = [(c + pt - 1) // pt for c in ctx_lens]
    total = sum(need) + extra_pages
    perm = rng.permutation(total).astype(np.int32)
    max_pages = max(1, max(need))
    table = np.zeros((batch, max_pages), dtype=np.int32)
    off = 0
    for b, nb in enumerate(need):
        table[b, :nb] = perm[off:off + nb]
        off += nb
    k = rng.standard_normal((total, pt, hkv, d)).astype(dtype)
    v = rng.standard_normal((total, pt, hkv, d)).astype(dtype)
    return k, v, table, total


def run_attn(q, k, v, table, ctx, hq, hkv, d, pt, scale, kv_dtype, num_pages, max_ctx=None):
    torch = torch_cuda()
    b = q.shape[0]
    dq, dk, dv, dt, dc = to_dev(q), to_dev(k), to_dev(v), to_dev(table), to_dev(ctx)
    out = empty_dev((b, hq, d), torch.float32)
    out.fill_(float("nan"))
    V.paged_attention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dt.data_ptr(), dc.data_ptr(), out.data_ptr(), b,
                      hq, hkv, d, pt, table.shape[1], num_pages, max_ctx if max_ctx is not None else int(ctx.max()),
                      scale, kv_dtype)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("pt", [16, 8, 32])
def test_config3_shape_f16_pages(pt):
    """Config 3 shape (Hq=32, Hkv=8, d=128, fp16 K/V, page table = seeded permutation of
    a shared pool) with a reduced batch and context range the oracle runs in seconds."""
    rng = np.random.default_rng(3 + pt)
    b, hq, hkv, d = 6, 32, 8, 128
    ctx = rng.integers(1, 900, size=b).astype(np.int32)
    ctx[0] = 1
    ctx[1] = 16
    k, v, table, total = make_paged(rng, b, hkv, d, ctx, pt)
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    scale = 1.0 / np.sqrt(d)
    out = run_attn(q, k, v, table, ctx, hq, hkv, d, pt, scale, V.KV_F16, total)
    ref = O.paged_attention(q, k.astype(np.float32), v.astype(np.float32), table, ctx, hq, hkv, d, pt, scale, f64=True)
    ref32 = O.paged_attention(q, k.astype(np.float32), v.astype(np.float32), table, ctx, hq, hkv, d, pt, scale)
    err = rel_err(out, ref)
    print(f"attention pt={pt}: rel err vs f64 {err:.3e}, oracle-f32 vs f64 {rel_err(ref32, ref):.3e}")
    assert err <= RTOL_F32
    for i in range(b):
        assert rel_err(out[i], ref[i]) <= RTOL_F32


def test_long_context_splits_and_uneven_lengths():
    rng = np.random.default_rng(77)
    b, hq, hkv, d, pt = 3, 32, 8, 128, 16
    ctx = np.array([8192, 513, 4097], dtype=np.int32)
    k, v, table, total = make_paged(rng, b, hkv, d, ctx, pt)
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    scale = 1.0 / np.sqrt(d)
    out = run_attn(q, k, v, table, ctx, hq, hkv, d, pt, scale, V.KV_F16, total)
    ref = O.paged_attention(q, k.astype(np.float32), v.astype(np.float32), table, ctx, hq, hkv, d, pt, scale, f64=True)
    assert rel_err(out, ref) <= RTOL_F32


@pytest.mark.parametrize("hq,hkv,d,dtype", [(8, 8, 128, np.float16), (64, 8, 128, np.float16), (16, 2, 128, np.float16),
                                             (8, 2, 64, np.float32), (4, 4, 96, np.float16), (32, 8, 128, np.float32),
                                             (48, 8, 128, np.float16), (32, 2, 128, np.float16), (12, 2, 128, np.float16)])
def test_head_layouts_and_dtypes(hq, hkv, d, dtype):
    rng = np.random.default_rng(hq * 3 + hkv + d)
    b, pt = 4, 16
    ctx = rng.integers(1, 300, size=b).astype(np.int32)
    k, v, table, total = make_paged(rng, b, hkv, d, ctx, pt, dtype=dtype)
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    scale = 1.0 / np.sqrt(d)
    kvd = V.KV_F16 if dtype == np.float16 else V.KV_F32
    out = run_attn(q, k, v, table, ctx, hq, hkv, d, pt, scale, kvd, total)
    ref = O.paged_attention(q, k.astype(np.float32), v.astype(np.float32), table, ctx, hq, hkv, d, pt, scale, f64=True)
    assert rel_err(out, ref) <= RTOL_F32


def test_empty_context_gives_zeros_and_bad_page_is_flagged():
    rng = np.random.default_rng(5)
    b, hq, hkv, d, pt = 2, 8, 2, 128, 16
    ctx = np.array([0, 20], dtype=np.int32)
    k, v, table, total = make_paged(rng, b, hkv, d, [1, 20], pt)
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    assert V.page_fault_flag() in (0, 1)   # clear
    out = run_attn(q, k, v, table, ctx, hq, hkv, d, pt, 0.1, V.KV_F16, total, max_ctx=32)
    assert np.all(out[0] == 0.0)
    assert V.page_fault_flag() == 0
    bad = table.copy()
    bad[1, 1] = total + 5          # out of range: redirected to page 0 and reported
    run_attn(q, k, v, bad, ctx, hq, hkv, d, pt, 0.1, V.KV_F16, total, max_ctx=32)
    assert V.page_fault_flag() == 1
    assert V.page_fault_flag() == 0


@pytest.mark.skipif(O.REF is None, reason="reference CPU library not built")
def test_gather_and_attention_on_reference_built_pages():
    """Pages written by the reference's vspec_kv_paged_append (sessions interleaved):
    GPU gather through each session's pages[] is bit-exact against
    vspec_kv_paged_get_token_ptr, and attention matches the oracle."""
    torch = torch_cuda()
    from test_oracle_pins import _build_interleaved_cache, pool_arrays, session_table
    rng = np.random.default_rng(17)
    pt, maxp, hkv, d = 16, 96, 8, 128
    lens = [300, 45, 16, 129]
    c, ids = _build_interleaved_cache(rng, pt, maxp, hkv, d, lens)
    kp, vp = pool_arrays(c, pt, maxp, hkv, d)
    dk, dv = to_dev(kp), to_dev(vp)
    tables = np.zeros((len(ids), maxp), dtype=np.int32)
    for i, (sid, n) in enumerate(zip(ids, lens)):
        t = session_table(c, sid, maxp)
        tables[i, : len(t)] = t
        rk = np.zeros((n, hkv, d), dtype=np.float32)
        rv = np.zeros((n, hkv, d), dtype=np.float32)
        assert O.REF.ref_paged_gather(c, sid, O.p(rk), O.p(rv)) == 1
        dt = to_dev(t)
        gk = empty_dev((n, hkv, d), torch.float32)
        gv = empty_dev((n, hkv, d), torch.float32)
        V.check(V.lib.vspec_b200_paged_gather(dk.data_ptr(), dv.data_ptr(), dt.data_ptr(), n, pt, hkv, d, V.KV_F32,
                                              gk.data_ptr(), gv.data_ptr(), None), "gather")
        torch.cuda.synchronize()
        assert np.array_equal(gk.cpu().numpy(), rk) and np.array_equal(gv.cpu().numpy(), rv)
    hq = 32
    q = rng.standard_normal((len(ids), hq, d)).astype(np.float32)
    ctx = np.array(lens, dtype=np.int32)
    k4 = kp.reshape(maxp, pt, hkv, d)
    v4 = vp.reshape(maxp, pt, hkv, d)
    out = run_attn(q, k4, v4, tables, ctx, hq, hkv, d, pt, 1.0 / np.sqrt(d), V.KV_F32, maxp)
    ref = O.paged_attention(q, k4, v4, tables, ctx, hq, hkv, d, pt, 1.0 / np.sqrt(d), f64=True)
    assert rel_err(out, ref) <= RTOL_F32
    # and the fp16 mirror of the same pool on the tensor-core path
    out16 = run_attn(q, k4.astype(np.float16), v4.astype(np.float16), tables, ctx, hq, hkv, d, pt, 1.0 / np.sqrt(d),
                     V.KV_F16, maxp)
    ref16 = O.paged_attention(q, k4.astype(np.float16).astype(np.float32), v4.astype(np.float16).astype(np.float32),
                              tables, ctx, hq, hkv, d, pt, 1.0 / np.sqrt(d), f64=True)
    assert rel_err(out16, ref16) <= RTOL_F32
    O.REF.ref_paged_destroy(c)


def test_reference_host_attention_entry_points():
    """vspec_cuda_attention_fused_single_f32 / _flash_ / vspec_cuda_launch_attention_fused
    (host arrays, plain softmax attention per head)."""
    torch_cuda()
    rng = np.random.default_rng(23)
    t, d = 77, 128
    q = rng.standard_normal(d).astype(np.float32)
    k = rng.standard_normal((t, d)).astype(np.float32)
    v = rng.standard_normal((t, d)).astype(np.float32)
    ref = O.paged_attention(q.reshape(1, 1, d), k, v, np.zeros((1, 1), np.int32), np.array([t], np.int32), 1, 1, d, t,
                            1.0 / np.sqrt(d), f64=True).reshape(-1)
    out = np.zeros(d, dtype=np.float32)
    V.lib.vspec_cuda_attention_fused_single_f32(q.ctypes.data, k.ctypes.data, v.ctypes.data, t, d, out.ctypes.data)
    assert rel_err(out, ref) <= RTOL_F32
    out[:] = 0
    V.lib.vspec_attention_flash_single_f32_bridge(q.ctypes.data, k.ctypes.data, v.ctypes.data, t, d, 64,
                                                  out.ctypes.data)
    assert rel_err(out, ref) <= RTOL_F32
    # context launcher over a contiguous VspecKVCache [T][H][d]
    h = 4
    qh = rng.standard_normal(h * d).astype(np.float32)
    kc = rng.standard_normal((t, h, d)).astype(np.float32)
    vc = rng.standard_normal((t, h, d)).astype(np.float32)
    cache = V.KVCache(kc.ctypes.data, vc.ctypes.data, t, h, d, t, 0, None, None, None, None, 0, 0, 0, None, None, 0)
    outh = np.zeros(h * d, dtype=np.float32)
    ctx = V.KernelContext(qh.ctypes.data, __import__("ctypes").addressof(cache), outh.ctypes.data)
    V.lib.vspec_cuda_launch_attention_fused(__import__("ctypes").byref(ctx))
    refh = O.paged_attention(qh.reshape(1, h, d), kc, vc, np.zeros((1, 1), np.int32), np.array([t], np.int32), h, h,
                             d, t, 1.0 / np.sqrt(d), f64=True).reshape(-1)
    assert rel_err(outh, refh) <= RTOL_F32


def test_config3_full_size_sampled_sequences():
    """The paged-attention workload at full size (B=32, Hq=32, Hkv=8, d=128, ctx ~U[512,8192],
    16-token fp16 pages, page table = seeded permutation of the shared pool):
    every output is finite, and the shortest, the longest and one more sequence
    match the f64 oracle (run on just those sequences' pages)."""
    torch = torch_cuda()
    rng = np.random.default_rng(33)
    b, hq, hkv, d, pt = 32, 32, 8, 128, 16
    ctx = rng.integers(512, 8193, size=b).astype(np.int32)
    need = (ctx + pt - 1) // pt
    total = int(need.sum())
    perm = rng.permutation(total).astype(np.int32)
    table = np.zeros((b, int(need.max())), dtype=np.int32)
    off = 0
    for i, nb in enumerate(need):
        table[i, :nb] = perm[off:off + nb]
        off += nb
    g = torch.Generator(device="cuda")
    g.manual_seed(33)
    kp = torch.randn((total, pt, hkv, d), device="cuda", dtype=torch.float16, generator=g)
    vp = torch.randn((total, pt, hkv, d), device="cuda", dtype=torch.float16, generator=g)
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    dq, dt, dc = to_dev(q), to_dev(table), to_dev(ctx)
    out = empty_dev((b, hq, d), torch.float32)
    out.fill_(float("nan"))
    scale = 1.0 / np.sqrt(d)
    V.paged_attention(dq.data_ptr(), kp.data_ptr(), vp.data_ptr(), dt.data_ptr(), dc.data_ptr(), out.data_ptr(), b,
                      hq, hkv, d, pt, table.shape[1], total, int(ctx.max()), scale, V.KV_F16)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    for i in sorted({int(np.argmin(ctx)), int(np.argmax(ctx)), 7}):
        pages = torch.from_numpy(table[i, :need[i]].astype(np.int64)).cuda()
        ks = kp[pages].float().cpu().numpy()
        vs = vp[pages].float().cpu().numpy()
        small = np.arange(need[i], dtype=np.int32)[None, :]
        ref = O.paged_attention(q[i:i + 1], ks, vs, small, ctx[i:i + 1], hq, hkv, d, pt, scale, f64=True)
        assert rel_err(got[i], ref[0]) <= RTOL_F32, (i, int(ctx[i]))
