"""vspec_b200_kv_paged_sync / vspec_b200_kv_paged_session_view: the device view
of a VspecKVPagedCache built by the reference's own compiled kv_paged_cache.c
(vspec_kv_paged_append, vspec_kv_paged_reuse_prefix), called through the C ABI.

For every session the device page-table row gathers exactly the tokens
vspec_kv_paged_get_token_ptr returns (bit for bit in fp32, fp16-rounded in
fp16), including a session that shares a partly filled prefix page and was
appended past it, and paged attention over the rows matches the oracle.  The
incremental sync copies only the pages written since the previous clock step."""
import ctypes

import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import RTOL_F32, empty_dev, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu

PT, MAXP, HKV, D = 16, 64, 8, 128
SPARE = 4   # spare device pages per batch entry


def _append(c, sid, rng, n):
    stride = HKV * D
    for _ in range(n):
        k = rng.standard_normal(stride).astype(np.float32)
        v = rng.standard_normal(stride).astype(np.float32)
        assert O.REF.vspec_kv_paged_append(c, sid, O.p(k), O.p(v)) == 1


def _build(rng):
    """Sessions 1..5, appends interleaved so page ids mix:
    1: 37 tokens (pages 16 + 16 + 5); 2: 16 tokens (one full page);
    3: reuse_prefix of all of 1 (its short third page shared), then 20 more:
       pages 16, 16, 5 (shared), 16, 4 -- a short page in the middle;
    4: reuse_prefix of 2 (one full shared page), then 3 more;
    5: opened, empty."""
    R = O.REF
    c = R.ref_paged_create(PT, MAXP, HKV, D)
    for sid in (1, 2):
        assert R.vspec_kv_paged_open_session(c, sid) == 1
    for t in range(37):
        _append(c, 1, rng, 1)
        if t < 16:
            _append(c, 2, rng, 1)
    assert R.vspec_kv_paged_reuse_prefix(c, 3, 1, 0) == 1
    assert R.vspec_kv_paged_reuse_prefix(c, 4, 2, 0) == 1
    for t in range(20):
        _append(c, 3, rng, 1)
        if t < 3:
            _append(c, 4, rng, 1)
    assert R.vspec_kv_paged_open_session(c, 5) == 1
    return c


def _ref_tokens(c, sid):
    n = O.REF.vspec_kv_paged_session_tokens(c, sid)
    k = np.zeros((n, HKV, D), dtype=np.float32)
    v = np.zeros((n, HKV, D), dtype=np.float32)
    if n:
        assert O.REF.ref_paged_gather(c, sid, O.p(k), O.p(v)) == 1
    return k, v


def _views(c, sids, dtype, dk, dv, maxpps):
    torch = torch_cuda()
    tab = empty_dev((len(sids), maxpps), torch.int32)
    ctx = empty_dev((len(sids),), torch.int32)
    used = []
    for b, sid in enumerate(sids):
        n, sp = ctypes.c_size_t(0), ctypes.c_size_t(0)
        V.check(V.lib.vspec_b200_kv_paged_session_view(
            c, sid, dtype, dk.data_ptr(), dv.data_ptr(), MAXP + b * SPARE, SPARE, tab[b].data_ptr(), maxpps,
            ctx[b:].data_ptr(), ctypes.byref(n), ctypes.byref(sp), None), "session_view")
        used.append(sp.value)
    return tab, ctx, used


@pytest.mark.parametrize("dtype", [V.KV_F32, V.KV_F16])
def test_session_views_gather_and_attention(dtype):
    torch = torch_cuda()
    if O.REF is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(5 + dtype)
    c = _build(rng)
    sids = [1, 2, 3, 4, 5]
    pages = MAXP + SPARE * len(sids)
    tdt = torch.float32 if dtype == V.KV_F32 else torch.float16
    dk = torch.zeros((pages, PT, HKV, D), dtype=tdt, device="cuda")
    dv = torch.zeros((pages, PT, HKV, D), dtype=tdt, device="cuda")
    step = ctypes.c_uint64(0)
    V.check(V.lib.vspec_b200_kv_paged_sync(c, dtype, dk.data_ptr(), dv.data_ptr(), 0, ctypes.byref(step), None), "sync")
    maxpps = 8
    tab, ctx, used = _views(c, sids, dtype, dk, dv, maxpps)
    # only session 3 has a short page in the middle: two spare pages for its 25 tail tokens
    assert used == [0, 0, 2, 0, 0]
    assert ctx.cpu().numpy().tolist() == [37, 16, 57, 19, 0]
    conv = (lambda a: a) if dtype == V.KV_F32 else (lambda a: a.astype(np.float16).astype(np.float32))
    refs = {}
    for b, sid in enumerate(sids):
        rk, rv = _ref_tokens(c, sid)
        refs[sid] = (conv(rk), conv(rv))
        n = rk.shape[0]
        if n == 0:
            continue
        gk = empty_dev((n, HKV, D), tdt)
        gv = empty_dev((n, HKV, D), tdt)
        V.check(V.lib.vspec_b200_paged_gather(dk.data_ptr(), dv.data_ptr(), tab[b].data_ptr(), n, PT, HKV, D, dtype,
                                              gk.data_ptr(), gv.data_ptr(), None), "gather")
        torch.cuda.synchronize()
        assert np.array_equal(gk.float().cpu().numpy(), refs[sid][0]), sid
        assert np.array_equal(gv.float().cpu().numpy(), refs[sid][1]), sid
    # attention over the rows against the oracle on the reference's token order
    hq = 32
    q = rng.standard_normal((len(sids), hq, D)).astype(np.float32)
    out = empty_dev((len(sids), hq, D), torch.float32)
    V.paged_attention(to_dev(q).data_ptr(), dk.data_ptr(), dv.data_ptr(), tab.data_ptr(), ctx.data_ptr(),
                      out.data_ptr(), len(sids), hq, HKV, D, PT, maxpps, pages, 64, 1.0 / np.sqrt(D), dtype)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert V.page_fault_flag() == 0
    for b, sid in enumerate(sids):
        rk, rv = refs[sid]
        n = rk.shape[0]
        if n == 0:
            assert np.all(got[b] == 0)
            continue
        ref = O.paged_attention(q[b:b + 1], rk, rv, np.zeros((1, 1), np.int32), np.array([n], np.int32), hq, HKV, D,
                                n, 1.0 / np.sqrt(D), f64=True)
        assert rel_err(got[b:b + 1], ref) <= RTOL_F32, sid
    O.REF.ref_paged_destroy(c)


def test_incremental_sync_and_errors():
    torch = torch_cuda()
    if O.REF is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(9)
    c = _build(rng)
    dk = torch.zeros((MAXP, PT, HKV, D), dtype=torch.float32, device="cuda")
    dv = torch.zeros((MAXP, PT, HKV, D), dtype=torch.float32, device="cuda")
    step = ctypes.c_uint64(0)
    V.check(V.lib.vspec_b200_kv_paged_sync(c, V.KV_F32, dk.data_ptr(), dv.data_ptr(), 0, ctypes.byref(step), None),
            "sync")
    first = step.value
    # new tokens for session 2 only (its full page is shared with 4, so a new page opens)
    _append(c, 2, rng, 5)
    dk.fill_(7.0)
    dv.fill_(7.0)
    V.check(V.lib.vspec_b200_kv_paged_sync(c, V.KV_F32, dk.data_ptr(), dv.data_ptr(), first, ctypes.byref(step), None),
            "sync")
    assert step.value > first
    pages = np.zeros(8, dtype=np.uint16)
    n2 = O.REF.ref_paged_session_pages(c, 2, O.p(pages), 8)
    assert n2 == 2
    new_page, shared_page = int(pages[1]), int(pages[0])
    rk, rv = _ref_tokens(c, 2)
    gk = dk.cpu().numpy()
    assert np.array_equal(gk[new_page, :5], rk[16:21])       # the page written since `first`
    assert np.all(gk[shared_page] == 7.0)                     # untouched since `first`: not copied
    # errors: inactive session, row too short, no spare room
    tab = empty_dev((1, 8), torch.int32)
    ctx = empty_dev((1,), torch.int32)
    args = (V.KV_F32, dk.data_ptr(), dv.data_ptr(), MAXP, 0, tab.data_ptr())
    assert V.lib.vspec_b200_kv_paged_session_view(c, 99, *args, 8, ctx.data_ptr(), None, None, None) == 1
    assert "not active" in V.last_error()
    assert V.lib.vspec_b200_kv_paged_session_view(c, 1, *args, 2, ctx.data_ptr(), None, None, None) == 1
    assert V.lib.vspec_b200_kv_paged_session_view(c, 3, *args, 8, ctx.data_ptr(), None, None, None) == 1
    assert "spare" in V.last_error()
    O.REF.ref_paged_destroy(c)
