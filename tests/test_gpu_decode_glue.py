"""The decode step's glue kernels at the Qwen3 shapes (head_dim 128), each
against a numpy restatement of the reference's float32 arithmetic:

  vspec_b200_decode_embed           token embedding row, fp16 -> fp32 (exact)
  vspec_b200_decode_qk_rope_append  per-head q/k RMSNorm (runtime_inference.py:1302-1305),
                                    half-split rotary (:1307-1311) with
                                    inv_freq = 1 / theta ** (i / half) in float32 (:4227)
                                    and cos / sin of fl32(pos * inv_freq) (:1187-1191), the
                                    power and sin / cos correctly rounded to float32;
                                    k and v appended as fp16 at their page slot
  vspec_b200_decode_next_token      _stabilize_logits with the Qwen profile
                                    (:554-567, runtime_compat/profiles.py:67-75: NaN -> 0,
                                    +-inf -> +-clip, clip) then greedy np.argmax
"""
import ctypes

import numpy as np
import pytest

import vspec_b200 as V
from gpu_util import empty_dev, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu
lib = V.lib


def _ref_rms_norm(x, w, eps):
    # runtime_inference.py:587-593 in float32
    x = x.astype(np.float32)
    mean_sq = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (x / np.sqrt(mean_sq + np.float32(eps))) * w.astype(np.float32)


def _inv_freq(theta, d, exact):
    """inv_freq = 1 / theta ** (i / half) in float32 (runtime_inference.py:4227).
    exact: the power correctly rounded to float32 (evaluated in float64, rounded
    once), as the kernel computes it; else numpy's own float32 power, which
    may differ from that by an ulp depending on the host's libm / SIMD."""
    half = d // 2
    e = np.arange(half, dtype=np.float32) / np.float32(half)
    pw = (np.float64(theta) ** e.astype(np.float64)).astype(np.float32) if exact else np.float32(theta) ** e
    return (np.float32(1.0) / pw).astype(np.float32)


def _ref_rotary(v, pos, theta, d, exact=True):
    half = d // 2
    ang = (np.float32(pos) * _inv_freq(theta, d, exact)).astype(np.float32)
    if exact:
        cos = np.cos(ang.astype(np.float64)).astype(np.float32)
        sin = np.sin(ang.astype(np.float64)).astype(np.float32)
    else:
        cos, sin = np.cos(ang), np.sin(ang)
    a, b = v[..., :half], v[..., half:]
    return np.concatenate([a * cos - b * sin, a * sin + b * cos], axis=-1).astype(np.float32)


def test_reference_inv_freq_within_ulps_of_the_correctly_rounded_one():
    """numpy's float32 theta ** (i / half) (the reference's own values on this
    host) is within one ulp of the correctly rounded power the kernel uses, so
    inv_freq within two; an ulp of inv_freq moves the angle at position p by
    about p * 6e-8 * inv_freq, which is what the 1e-3 check against plain numpy
    in test_qk_norm_rope_append absorbs."""
    def ulps(a, b):
        return np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64)).max()
    for d in (64, 128):
        half = d // 2
        e = np.arange(half, dtype=np.float32) / np.float32(half)
        exact = (np.float64(1e6) ** e.astype(np.float64)).astype(np.float32)
        assert ulps(exact, np.float32(1e6) ** e) <= 1
        assert ulps(_inv_freq(1e6, d, True), _inv_freq(1e6, d, False)) <= 2


@pytest.mark.parametrize("hidden,vocab,batch", [(4096, 151936, 8), (5120, 151936, 3)])
def test_embed_exact(hidden, vocab, batch):
    torch = torch_cuda()
    rng = np.random.default_rng(hidden + batch)
    rows = 4096   # a slice of the table is enough to address every token id we draw
    table = rng.uniform(-0.05, 0.05, size=(rows, hidden)).astype(np.float16)
    tok = rng.integers(0, rows, size=batch).astype(np.int32)
    tok[0] = rows - 1
    dt, dtok = to_dev(table.view(np.uint16)), to_dev(tok)
    dx = empty_dev((batch, hidden), torch.float32)
    V.check(lib.vspec_b200_decode_embed(dt.data_ptr(), dtok.data_ptr(), batch, hidden, dx.data_ptr(), None), "embed")
    torch.cuda.synchronize()
    assert np.array_equal(dx.cpu().numpy(), table[tok].astype(np.float32))


@pytest.mark.parametrize("hq,hkv,batch", [(32, 8, 8), (64, 8, 4), (8, 1, 3), (4, 1, 64)])
def test_qk_norm_rope_append(hq, hkv, batch):
    """Positions up to 8191 (angles up to ~8191 rad, where float32 angle
    rounding matters), norm weights not all one, pages from a permuted pool."""
    torch = torch_cuda()
    d, pt, eps, theta = 128, 16, 1e-6, 1e6
    rng = np.random.default_rng(hq * 100 + batch)
    nh = hq + 2 * hkv
    qkv = (rng.standard_normal((batch, nh, d)) * rng.uniform(0.2, 3.0, size=(batch, nh, 1))).astype(np.float32)
    qn = rng.uniform(0.5, 1.5, d).astype(np.float32)
    kn = rng.uniform(0.5, 1.5, d).astype(np.float32)
    pos = rng.integers(0, 8192, size=batch).astype(np.int32)
    pos[0] = 8191
    if batch > 1:
        pos[1] = 0
    max_pages = 512
    n_pages = batch * 2 + 5
    perm = rng.permutation(n_pages).astype(np.int32)
    table = np.full((batch, max_pages), -1, dtype=np.int32)
    for b in range(batch):
        table[b, pos[b] // pt] = perm[b]
    sentinel = np.float16(7.0)
    kp = np.full((n_pages, pt, hkv, d), sentinel, dtype=np.float16)
    vp = np.full((n_pages, pt, hkv, d), sentinel, dtype=np.float16)
    dqkv, dqn, dkn, dpos, dtab = map(to_dev, (qkv, qn, kn, pos, table))
    dkp, dvp = to_dev(kp.view(np.uint16)), to_dev(vp.view(np.uint16))
    dq = empty_dev((batch, hq, d), torch.float32)
    dctx = to_dev(np.zeros(batch, dtype=np.int32))
    V.check(lib.vspec_b200_decode_qk_rope_append(dqkv.data_ptr(), dqn.data_ptr(), dkn.data_ptr(), dpos.data_ptr(),
                                                 batch, hq, hkv, d, eps, theta, dq.data_ptr(), dkp.data_ptr(),
                                                 dvp.data_ptr(), dtab.data_ptr(), max_pages, pt, dctx.data_ptr(), None),
            "qk_rope_append")
    torch.cuda.synchronize()
    q_gpu = dq.cpu().numpy()
    kp_gpu = dkp.cpu().numpy().view(np.float16)
    vp_gpu = dvp.cpu().numpy().view(np.float16)
    assert np.array_equal(dctx.cpu().numpy(), pos + 1)
    touched = np.zeros((n_pages, pt), dtype=bool)
    for b in range(batch):
        qr = _ref_rotary(_ref_rms_norm(qkv[b, :hq], qn, eps), int(pos[b]), theta, d)
        kr = _ref_rotary(_ref_rms_norm(qkv[b, hq:hq + hkv], kn, eps), int(pos[b]), theta, d)
        vr = qkv[b, hq + hkv:]
        # against the reference's float32 formula with correctly rounded power
        # and sin / cos: only the RMSNorm summation order and FMA contraction differ
        assert rel_err(q_gpu[b], qr) <= 4e-6, (b, rel_err(q_gpu[b], qr))
        # against numpy's own float32 power / sin / cos (host-dependent ulps,
        # amplified by the position): the fp32 contract
        qn32 = _ref_rotary(_ref_rms_norm(qkv[b, :hq], qn, eps), int(pos[b]), theta, d, exact=False)
        assert rel_err(q_gpu[b], qn32) <= 1e-3, (b, rel_err(q_gpu[b], qn32))
        page, slot = table[b, pos[b] // pt], pos[b] % pt
        touched[page, slot] = True
        kg = kp_gpu[page, slot].astype(np.float32)
        # fp16 storage: equal to the reference's value rounded to fp16, up to one
        # fp16 step where the float32 values straddle a rounding boundary
        k16 = kr.astype(np.float16).astype(np.float32)
        step = np.abs(np.spacing(kr.astype(np.float16))).astype(np.float32)
        assert np.all(np.abs(kg - k16) <= step), b
        assert np.mean(kg == k16) >= 0.99
        assert np.array_equal(vp_gpu[page, slot], vr.astype(np.float16))
    # nothing else in the pools was written
    assert np.all(kp_gpu[~touched] == sentinel) and np.all(vp_gpu[~touched] == sentinel)


def _stabilized_argmax(lg, clip):
    v = np.nan_to_num(lg.astype(np.float32), nan=0.0, posinf=clip, neginf=-clip)
    return int(np.argmax(np.clip(v, -clip, clip)))


@pytest.mark.parametrize("vocab", [151936, 1000, 7])
def test_next_token_greedy_and_prompt(vocab):
    """Sequences in the prompt take the next prompt token; the others the
    argmax of the cleaned logits, ties to the lowest index (values clipped to
    the same +-24, NaN equal to a 0 logit, +-0, +inf).  Positions advance, the
    token is recorded, and the 12-byte per-sequence state returns to zero."""
    torch = torch_cuda()
    rng = np.random.default_rng(vocab)
    batch, clip, max_prompt, max_steps = 6, 24.0, 5, 40
    lg = (rng.standard_normal((batch, vocab)) * 6).astype(np.float32)
    if vocab > 10:
        lg[0, [3, vocab - 2]] = [30.0, 25.0]              # both clip to 24: index 3 wins
        lg[1, :] = -1.0
        lg[1, [vocab // 2, 5]] = [np.nan, -0.0]          # NaN -> 0 ties with -0: index 5 wins
        lg[2, [9, 11]] = [np.inf, np.inf]                 # +inf -> clip: index 9
        lg[3, :] = -np.inf
        lg[3, vocab - 1] = -5.0
        lg[4, 17] = np.float32(1e30)
    prompt_len = np.array([5, 1, 3, 2, 0, 4], dtype=np.int32)
    prompts = rng.integers(0, vocab, size=(batch, max_prompt)).astype(np.int32)
    pos = np.array([0, 0, 2, 1, 3, 3], dtype=np.int32)   # seq 0 and 5 still in their prompt
    dl, dpr, dpl, dpos = map(to_dev, (lg, prompts, prompt_len, pos))
    dtok = to_dev(np.full(batch, -1, dtype=np.int32))
    dout = to_dev(np.full((batch, max_steps), -1, dtype=np.int32))
    dstate = to_dev(np.zeros(batch * 12 // 4 + 2, dtype=np.int32))
    for it in range(2):
        V.check(lib.vspec_b200_decode_next_token(dl.data_ptr(), batch, vocab, clip, dpr.data_ptr(), dpl.data_ptr(),
                                                 max_prompt, dpos.data_ptr(), dtok.data_ptr(), dout.data_ptr(),
                                                 max_steps, dstate.data_ptr(), None), "next_token")
        torch.cuda.synchronize()
        tok, out, p1 = dtok.cpu().numpy(), dout.cpu().numpy(), dpos.cpu().numpy()
        for b in range(batch):
            p = pos[b] + it
            want = prompts[b, p + 1] if p + 1 < prompt_len[b] else _stabilized_argmax(lg[b], clip)
            assert tok[b] == want, (it, b, tok[b], want)
            assert out[b, p + 1] == want
            assert p1[b] == p + 1
        assert not dstate.cpu().numpy().any()
