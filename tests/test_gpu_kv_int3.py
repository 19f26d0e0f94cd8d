"""int3 KV-cache compression on the GPU: the append-time
quantiser bit for bit against the oracle and the reference's own
vspec_kv_cache_append (src/attention/kv_cache.c:64-126,160-226), and paged GQA
attention over int3 pages against the oracle's dequantise-then-attend
(src/kernel/cuda/attention_fused.cu:23-45,232-351), through the C ABI."""
import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import RTOL_F32, empty_dev, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu


def _rows(rng, rows, heads, d):
    x = rng.standard_normal((rows, heads, d)).astype(np.float32)
    x[0, 0, :4] = [1e4, -3e3, 0.0, 0.0]       # one outlier: x / scale beyond int8, wraps before the clip
    x[1 % rows, 1 % heads, :32] = 0.0          # an all-zero block: scale 1
    x[2 % rows, 2 % heads, 5] = -5e6
    x[3 % rows, 3 % heads, :] = 1e-9           # scale clamped to 1e-6
    x[4 % rows, 0, ::2] = x[4 % rows, 0, 1::2]  # ties in |x|
    return x


@pytest.mark.parametrize("block", [16, 32])
def test_int3_quantize_bit_exact(block):
    torch = torch_cuda()
    rng = np.random.default_rng(block)
    rows, heads, d = 37, 8, 128
    x = _rows(rng, rows, heads, d)
    slots = rng.permutation(rows + 11)[:rows].astype(np.int32)   # scattered pool rows
    pool_rows = rows + 11
    pb, nb = d * 3 // 8, d // block
    dc = torch.zeros((pool_rows, heads, pb), dtype=torch.uint8, device="cuda")
    ds = torch.zeros((pool_rows, heads, nb), dtype=torch.float32, device="cuda")
    dx, dsl = to_dev(x), to_dev(slots)
    V.kv_int3_quantize(dx.data_ptr(), dsl.data_ptr(), rows, heads, d, block, dc.data_ptr(), ds.data_ptr())
    torch.cuda.synchronize()
    codes, scales = dc.cpu().numpy()[slots], ds.cpu().numpy()[slots]
    oc, os_ = O.kv_int3_quantize(x, block)
    assert np.array_equal(codes, oc)
    assert np.array_equal(scales.view(np.uint32), os_.view(np.uint32))
    if O.REF is not None:
        rc, rs = O.kv_int3_quantize(x, block, reference=True)
        assert np.array_equal(codes, rc)
        assert np.array_equal(scales.view(np.uint32), rs.view(np.uint32))


def _int3_case(rng, ctx, hq, hkv, d, pt, block, extra_pages=3):
    b = len(ctx)
    need = [(c + pt - 1) // pt for c in ctx]
    pages = sum(need) + extra_pages
    max_pages = max(max(need), 1)
    perm = rng.permutation(pages).astype(np.int32)
    table = np.zeros((b, max_pages), dtype=np.int32)
    o = 0
    for i, n in enumerate(need):
        table[i, :n] = perm[o:o + n]
        o += n
    kf = rng.standard_normal((pages * pt, hkv, d)).astype(np.float32)
    vf = rng.standard_normal((pages * pt, hkv, d)).astype(np.float32)
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    return table, kf, vf, q, pages, max_pages


@pytest.mark.parametrize("block", [32, 16])
@pytest.mark.parametrize("ctx,hq,hkv", [([37, 300], 32, 8), ([1, 16, 17, 600], 8, 2), ([513, 0, 1030], 64, 8),
                                        ([2048], 4, 4)])
def test_int3_paged_attention_matches_oracle(block, ctx, hq, hkv):
    torch = torch_cuda()
    rng = np.random.default_rng(len(ctx) * 100 + hq + block)
    d, pt = 128, 16
    table, kf, vf, q, pages, max_pages = _int3_case(rng, ctx, hq, hkv, d, pt, block)
    # quantise the pools on the GPU (every pool row), check against the oracle, attend
    rows = pages * pt
    pb, nb = d * 3 // 8, d // block
    kc = torch.empty((rows, hkv, pb), dtype=torch.uint8, device="cuda")
    vc = torch.empty((rows, hkv, pb), dtype=torch.uint8, device="cuda")
    ks = torch.empty((rows, hkv, nb), dtype=torch.float32, device="cuda")
    vs = torch.empty((rows, hkv, nb), dtype=torch.float32, device="cuda")
    dk, dv = to_dev(kf), to_dev(vf)
    V.kv_int3_quantize(dk.data_ptr(), None, rows, hkv, d, block, kc.data_ptr(), ks.data_ptr())
    V.kv_int3_quantize(dv.data_ptr(), None, rows, hkv, d, block, vc.data_ptr(), vs.data_ptr())
    torch.cuda.synchronize()
    okc, oks = O.kv_int3_quantize(kf, block)
    assert np.array_equal(kc.cpu().numpy(), okc)
    dq, dt, dctx = to_dev(q), to_dev(table), to_dev(np.array(ctx, dtype=np.int32))
    out = empty_dev((len(ctx), hq, d), torch.float32)
    scale = 1.0 / np.sqrt(d)
    V.paged_attention_int3(dq.data_ptr(), kc.data_ptr(), vc.data_ptr(), ks.data_ptr(), vs.data_ptr(), block,
                           dt.data_ptr(), dctx.data_ptr(), out.data_ptr(), len(ctx), hq, hkv, d, pt, max_pages, pages,
                           max(ctx), scale)
    torch.cuda.synchronize()
    assert V.page_fault_flag() == 0
    ref = O.paged_int3_attention(q, kc.cpu().numpy(), vc.cpu().numpy(), ks.cpu().numpy(), vs.cpu().numpy(), table,
                                 ctx, hq, hkv, d, pt, block, scale)
    got = out.cpu().numpy()
    for i, c in enumerate(ctx):
        if c == 0:
            assert np.all(got[i] == 0.0)
    err = rel_err(got, ref)
    print(f"int3 attention ctx={ctx} hq={hq} hkv={hkv} block={block}: {err:.2e}")
    assert err <= RTOL_F32


def test_int3_attention_rejects_bad_arguments():
    torch = torch_cuda()
    z = torch.zeros(64, dtype=torch.float32, device="cuda")
    t = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(V.VspecB200Error, match="head_dim"):
        V.paged_attention_int3(z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), 32, t.data_ptr(),
                               t.data_ptr(), z.data_ptr(), 1, 8, 8, 64, 16, 1, 1, 16, 0.1)
    with pytest.raises(V.VspecB200Error, match="block_size"):
        V.kv_int3_quantize(z.data_ptr(), None, 1, 1, 128, 24, z.data_ptr(), z.data_ptr())


def test_int3_config3_full_size_sampled_sequences():
    """Config 3 at full size on int3 pages (B=32, Hq=32, Hkv=8, d=128, ctx ~U[512, 8192], 16-token pages,
    block 32, page table = seeded permutation of the shared pool): the pools are quantised on the GPU,
    every output is finite, and the shortest, the longest and one more sequence match the oracle run on
    just those sequences' pages."""
    torch = torch_cuda()
    rng = np.random.default_rng(34)
    b, hq, hkv, d, pt, block = 32, 32, 8, 128, 16, 32
    ctx = rng.integers(512, 8193, size=b).astype(np.int32)
    need = (ctx + pt - 1) // pt
    total = int(need.sum())
    perm = rng.permutation(total).astype(np.int32)
    table = np.zeros((b, int(need.max())), dtype=np.int32)
    off = 0
    for i, nb in enumerate(need):
        table[i, :nb] = perm[off:off + nb]
        off += nb
    rows, pb, nbk = total * pt, d * 3 // 8, d // block
    g = torch.Generator(device="cuda")
    g.manual_seed(34)
    pools = []
    for _ in range(2):
        f = torch.randn((rows, hkv, d), device="cuda", generator=g)
        codes = torch.empty((rows, hkv, pb), dtype=torch.uint8, device="cuda")
        scales = torch.empty((rows, hkv, nbk), dtype=torch.float32, device="cuda")
        V.kv_int3_quantize(f.data_ptr(), None, rows, hkv, d, block, codes.data_ptr(), scales.data_ptr())
        torch.cuda.synchronize()
        del f
        pools.append((codes, scales))
    (kc, ks), (vc, vs) = pools
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    dq, dt, dctx = to_dev(q), to_dev(table), to_dev(ctx)
    out = empty_dev((b, hq, d), torch.float32)
    scale = 1.0 / np.sqrt(d)
    V.paged_attention_int3(dq.data_ptr(), kc.data_ptr(), vc.data_ptr(), ks.data_ptr(), vs.data_ptr(), block,
                           dt.data_ptr(), dctx.data_ptr(), out.data_ptr(), b, hq, hkv, d, pt, table.shape[1], total,
                           int(ctx.max()), scale)
    torch.cuda.synchronize()
    assert V.page_fault_flag() == 0
    got = out.cpu().numpy()
    assert np.all(np.isfinite(got))
    for i in sorted({int(np.argmin(ctx)), int(np.argmax(ctx)), 7}):
        pages_i = table[i, :need[i]]
        sel = torch.from_numpy((pages_i[:, None] * pt + np.arange(pt)[None, :]).reshape(-1).astype(np.int64)).cuda()
        local = np.arange(need[i], dtype=np.int32)[None, :]
        ref = O.paged_int3_attention(q[i:i + 1], kc[sel].cpu().numpy(), vc[sel].cpu().numpy(), ks[sel].cpu().numpy(),
                                     vs[sel].cpu().numpy(), local, ctx[i:i + 1], hq, hkv, d, pt, block, scale)
        err = rel_err(got[i], ref[0])
        print(f"int3 config 3 sequence {i} (ctx {ctx[i]}): {err:.2e}")
        assert err <= RTOL_F32
