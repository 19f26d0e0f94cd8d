"""ctypes loader for the CPU checker libraries.

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, never by the shipped library.

  ORACLE -- liboracle.so, this project's C restatement (oracle.c)
  REF    -- _ref/libvspec_ref.so, Vspec-Engine's own CPU sources compiled from
            the reference tree (None when it was never built)
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_double, c_float, c_int, c_size_t, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libvspec_ref.so")

ORACLE = ctypes.CDLL(ORACLE_PATH)
REF = ctypes.CDLL(REF_PATH) if os.path.exists(REF_PATH) else None

_o = {
    "oracle_row_bytes": ([c_size_t, c_int], c_size_t),
    "oracle_get_code": ([c_void_p, c_size_t, c_int], ctypes.c_int8),
    "oracle_pack_rows": ([c_void_p, c_size_t, c_size_t, c_int, c_void_p], None),
    "oracle_quantize_rowwise": ([c_void_p, c_size_t, c_size_t, c_int, c_int, c_double, c_void_p, c_void_p, c_void_p],
                                c_int),
    "oracle_unpack_rows": ([c_void_p, c_size_t, c_size_t, c_int, c_void_p], None),
    "oracle_group_of": ([c_size_t, c_size_t, c_size_t], c_size_t),
    "oracle_lowbit_matmul_f32": ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_int, c_void_p, c_void_p, c_size_t,
                                  c_void_p], None),
    "oracle_lowbit_matmul_f16sz": ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_int, c_void_p, c_void_p,
                                    c_size_t, c_void_p], None),
    "oracle_lowbit_matmul_f64acc": ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_int, c_void_p, c_void_p,
                                     c_size_t, c_void_p], None),
    "oracle_half_to_float": ([ctypes.c_uint16], c_float),
    "oracle_paged_gather_f32": ([c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_size_t, c_void_p,
                                 c_void_p], None),
    "oracle_paged_gqa_attention_f32": ([c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_size_t,
                                        c_size_t, c_size_t, c_size_t, c_float, c_void_p], None),
    "oracle_clamp_rows_std": ([c_void_p, c_size_t, c_size_t, c_float, c_void_p], None),
    "oracle_attention_ref_f32": ([c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int, c_size_t,
                                  c_void_p], None),
    "oracle_int3_blocknorm_f32": ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p, c_int, c_void_p], None),
    "oracle_paged_gqa_attention_f64": ([c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_size_t,
                                        c_size_t, c_size_t, c_size_t, c_float, c_void_p], None),
}
_o["oracle_kv_int3_quantize"] = ([c_void_p, c_size_t, c_size_t, c_size_t, c_size_t, c_float, c_void_p, c_void_p], None)
_o["oracle_paged_int3_attention_f64"] = ([c_void_p] * 6 + [c_size_t, c_void_p] + [c_size_t] * 6 + [c_float, c_void_p],
                                         None)
_o["oracle_q4k_matmul_f32"] = ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p], None)
for _n, (_a, _r) in _o.items():
    _f = getattr(ORACLE, _n)
    _f.argtypes = _a
    _f.restype = _r


class OracleQwenC(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_int), ("hidden", ctypes.c_int), ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("inter", ctypes.c_int), ("vocab", ctypes.c_int), ("bits", ctypes.c_int),
                ("group", ctypes.c_int), ("eps", ctypes.c_float), ("theta", ctypes.c_float), ("clip", ctypes.c_float),
                ("emb", c_void_p), ("w", c_void_p), ("s", c_void_p), ("w_lm", c_void_p), ("s_lm", c_void_p),
                ("bits_mlp", ctypes.c_int)]


ORACLE.oracle_qwen_generate.argtypes = [ctypes.POINTER(OracleQwenC), c_void_p, ctypes.c_int, ctypes.c_int, c_void_p,
                                        c_void_p]
ORACLE.oracle_qwen_generate.restype = ctypes.c_int
ORACLE.oracle_float_to_half.argtypes = [c_float]
ORACLE.oracle_float_to_half.restype = ctypes.c_uint16


def qwen_generate(cfg: dict, tensors: dict, prompt, gen: int):
    """Greedy decode of one sequence with the C restatement (oracle_qwen_generate).
    tensors: 'emb' (fp16 bits), per layer 'w{l}_{i}' / 's{l}_{i}' (i = 0 qkv, 1 o,
    2 gate+up, 3 down), 'w_lm', 's_lm' as numpy arrays.  Returns (tokens, logits)."""
    L = cfg["num_layers"]
    keep = []

    def ptr(a):
        a = np.ascontiguousarray(a)
        keep.append(a)
        return a.ctypes.data
    wp = (c_void_p * (4 * L))(*[ptr(tensors[f"w{l}_{i}"]) for l in range(L) for i in range(4)])
    sp = (c_void_p * (4 * L))(*[ptr(tensors[f"s{l}_{i}"]) for l in range(L) for i in range(4)])
    q = OracleQwenC(L, cfg["hidden"], cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"], cfg["intermediate"],
                    cfg["vocab"], cfg["bits"], cfg["group"], cfg["rms_eps"], cfg["rope_theta"], cfg["logit_clip"],
                    ptr(tensors["emb"]), ctypes.cast(wp, c_void_p), ctypes.cast(sp, c_void_p), ptr(tensors["w_lm"]),
                    ptr(tensors["s_lm"]), cfg.get("bits_mlp", 0) or 0)
    prompt = np.ascontiguousarray(prompt, dtype=np.int32)
    total = prompt.size + gen
    toks = np.zeros(total, dtype=np.int32)
    logits = np.zeros((total - 1, cfg["vocab"]), dtype=np.float32)
    rc = ORACLE.oracle_qwen_generate(ctypes.byref(q), prompt.ctypes.data, prompt.size, gen, toks.ctypes.data,
                                     logits.ctypes.data)
    if rc != 0:
        raise RuntimeError("oracle_qwen_generate failed")
    return toks, logits

if REF is not None:
    _r = {
        "vspec_quant_packed_bytes": ([c_size_t, ctypes.c_uint8], c_size_t),
        "vspec_quant_pack_signed": ([c_void_p, c_size_t, ctypes.c_uint8, c_void_p], None),
        "vspec_quant_unpack_signed": ([c_void_p, c_size_t, ctypes.c_uint8, c_void_p], None),
        "vspec_quant_get_signed": ([c_void_p, c_size_t, ctypes.c_uint8], ctypes.c_int8),
        "vspec_int4_pack": ([c_void_p, c_size_t, c_void_p], None),
        "vspec_int4_get": ([c_void_p, c_size_t], ctypes.c_int8),
        "vspec_int4_matmul_ref_f32_q4": ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p, c_void_p], None),
        "vspec_int4_compute_zero_points": ([c_void_p, c_size_t, c_size_t, c_void_p], None),
        "vspec_int4_matmul_ref_f32_q4_with_zero_points": ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p,
                                                           c_void_p, c_void_p], None),
        "vspec_int3_matmul_ref_f32_q3": ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p, c_void_p], None),
        "vspec_int3_compute_zero_points": ([c_void_p, c_size_t, c_size_t, c_void_p], None),
        "vspec_int3_matmul_ref_f32_q3_with_zero_points": ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p,
                                                           c_void_p, c_void_p], None),
        "vspec_flash_attention_stub": ([c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_void_p], None),
        "ref_cpu_backend_linear_int4": ([c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p, c_void_p], None),
        "ref_cpu_backend_attention": ([c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p], c_int),
        "ref_paged_create": ([c_size_t, c_size_t, c_size_t, c_size_t], c_void_p),
        "ref_paged_destroy": ([c_void_p], None),
        "ref_paged_key_pool": ([c_void_p], c_void_p),
        "ref_paged_value_pool": ([c_void_p], c_void_p),
        "ref_paged_session_pages": ([c_void_p, c_uint64, c_void_p, c_size_t], c_size_t),
        "ref_paged_page_used": ([c_void_p, c_size_t], c_size_t),
        "ref_paged_gather": ([c_void_p, c_uint64, c_void_p, c_void_p], c_int),
        "vspec_kv_paged_open_session": ([c_void_p, c_uint64], c_int),
        "vspec_kv_paged_close_session": ([c_void_p, c_uint64], c_int),
        "vspec_kv_paged_reuse_prefix": ([c_void_p, c_uint64, c_uint64, c_size_t], c_int),
        "vspec_kv_paged_append": ([c_void_p, c_uint64, c_void_p, c_void_p], c_int),
        "vspec_kv_paged_get_token_ptr": ([c_void_p, c_uint64, c_size_t, c_size_t, POINTER(c_void_p),
                                          POINTER(c_void_p)], c_int),
        "vspec_kv_paged_session_tokens": ([c_void_p, c_uint64], c_size_t),
        "vspec_kv_paged_stats": ([c_void_p, c_void_p], None),
    }
    for _n, (_a, _rt) in _r.items():
        _f = getattr(REF, _n)
        _f.argtypes = _a
        _f.restype = _rt
    for _n in ["ref_sizeof_kernel_context", "ref_sizeof_quant_meta", "ref_sizeof_exec_config", "ref_sizeof_kv_cache",
               "ref_sizeof_kv_paged_cache", "ref_sizeof_backend", "ref_offsetof_ctx_qmeta", "ref_offsetof_ctx_config",
               "ref_offsetof_qmeta_scales", "ref_offsetof_qmeta_scale_count", "ref_offsetof_kv_current_tokens",
               "ref_offsetof_kv_int3", "ref_offsetof_paged_sessions", "ref_offsetof_paged_page_meta"]:
        getattr(REF, _n).restype = c_size_t


def p(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags.c_contiguous
    return a.ctypes.data


def row_bytes(k: int, bits: int) -> int:
    return (k * bits + 7) // 8


# ---------------------------------------------------------------- helpers
def pack_rows(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack int8 codes [n][k] row by row (reference bitstream)."""
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    n, k = codes.shape
    out = np.zeros((n, row_bytes(k, bits)), dtype=np.uint8)
    ORACLE.oracle_pack_rows(p(codes), n, k, bits, p(out))
    return out


def quantize_rowwise(w: np.ndarray, bits: int, block_size: int, percentile: float = 0.999):
    """C restatement of the reference quantizer (oracle_quantize_rowwise).
    Returns (packed [n][row_bytes], scales [n*n_blocks], zero_points)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    nb = (k + block_size - 1) // block_size if block_size > 0 else 1
    packed = np.zeros((n, row_bytes(k, bits)), dtype=np.uint8)
    s = np.zeros(n * nb, dtype=np.float32)
    zp = np.zeros(n * nb, dtype=np.float32)
    if ORACLE.oracle_quantize_rowwise(p(w), n, k, bits, block_size, percentile, p(packed), p(s), p(zp)) != 0:
        raise RuntimeError("oracle_quantize_rowwise failed")
    return packed, s, zp


def unpack_rows(packed: np.ndarray, n: int, k: int, bits: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.zeros((n, k), dtype=np.int8)
    ORACLE.oracle_unpack_rows(p(packed), n, k, bits, p(out))
    return out


def unpack_rows_np(packed: np.ndarray, n: int, k: int, bits: int, unsigned: bool = False) -> np.ndarray:
    """Vectorized numpy decode of the same bitstream (for large matrices)."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8).reshape(n, row_bytes(k, bits))
    bitpos = np.arange(k, dtype=np.int64) * bits
    byte = bitpos >> 3
    shift = (bitpos & 7).astype(np.uint16)
    lo = packed[:, byte].astype(np.uint16)
    hi_idx = np.minimum(byte + 1, packed.shape[1] - 1)
    hi = packed[:, hi_idx].astype(np.uint16)
    v = ((lo | (hi << 8)) >> shift) & ((1 << bits) - 1)
    v = v.astype(np.int16)
    if unsigned:
        return (v - (1 << (bits - 1))).astype(np.int8)
    return np.where(v >= (1 << (bits - 1)), v - (1 << bits), v).astype(np.int8)


def lowbit_matmul(a: np.ndarray, w: np.ndarray, n: int, k: int, bits: int, s: np.ndarray,
                  zp: np.ndarray | None, n_groups: int) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    m = a.shape[0]
    out = np.zeros((m, n), dtype=np.float32)
    if s.dtype == np.float16:
        ORACLE.oracle_lowbit_matmul_f16sz(p(a), m, k, p(np.ascontiguousarray(w)), n, bits,
                                          p(np.ascontiguousarray(s)),
                                          p(np.ascontiguousarray(zp)) if zp is not None else None, n_groups, p(out))
    else:
        ORACLE.oracle_lowbit_matmul_f32(p(a), m, k, p(np.ascontiguousarray(w)), n, bits,
                                        p(np.ascontiguousarray(s, dtype=np.float32)),
                                        p(np.ascontiguousarray(zp, dtype=np.float32)) if zp is not None else None,
                                        n_groups, p(out))
    return out


def lowbit_matmul_f64(a: np.ndarray, w: np.ndarray, n: int, k: int, bits: int, s: np.ndarray,
                      zp: np.ndarray | None, n_groups: int) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    m = a.shape[0]
    out = np.zeros((m, n), dtype=np.float64)
    ORACLE.oracle_lowbit_matmul_f64acc(p(a), m, k, p(np.ascontiguousarray(w)), n, bits,
                                       p(np.ascontiguousarray(s, dtype=np.float32)),
                                       p(np.ascontiguousarray(zp, dtype=np.float32)) if zp is not None else None,
                                       n_groups, p(out))
    return out


def paged_attention(q, k_pages, v_pages, table, ctx_len, hq, hkv, d, pt, scale, f64=False) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    kp = np.ascontiguousarray(k_pages, dtype=np.float32)
    vp = np.ascontiguousarray(v_pages, dtype=np.float32)
    table = np.ascontiguousarray(table, dtype=np.int32)
    ctx = np.ascontiguousarray(ctx_len, dtype=np.int32)
    b = ctx.shape[0]
    out = np.zeros((b, hq, d), dtype=np.float64 if f64 else np.float32)
    fn = ORACLE.oracle_paged_gqa_attention_f64 if f64 else ORACLE.oracle_paged_gqa_attention_f32
    fn(p(q), p(kp), p(vp), p(table), table.shape[1], p(ctx), b, hq, hkv, d, pt, scale, p(out))
    return out


def attention_ref(q, keys, values, module: int, block: int = 64) -> np.ndarray:
    """The CPU backend's attention (attention_ref.c:7-88) on a contiguous cache:
    q [heads][d], keys/values [tokens][heads][d]; module = the 3-bit runtime module."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(keys, dtype=np.float32)
    v = np.ascontiguousarray(values, dtype=np.float32)
    t, h, d = k.shape
    out = np.zeros((h, d), dtype=np.float32)
    ORACLE.oracle_attention_ref_f32(p(q), p(k), p(v), t, h, d, int(module), int(block), p(out))
    return out


def kv_int3_quantize(x: np.ndarray, block: int, percentile: float = 99.5, reference: bool = False):
    """int3 KV compression of rows [rows][heads][d] (kv_cache.c:32-126): codes
    [rows][heads][ceil(3d/8)] uint8 and scales [rows][heads][d/block] fp32.
    reference=True runs the reference's own vspec_kv_cache_append instead
    (percentile fixed at 99.5 there)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, heads, d = x.shape
    codes = np.zeros((rows, heads, row_bytes(d, 3)), dtype=np.uint8)
    scales = np.zeros((rows, heads, (d + block - 1) // block), dtype=np.float32)
    if reference:
        if REF is None:
            raise RuntimeError("oracle/_ref/libvspec_ref.so not built")
        fn = REF.ref_kv_int3_quantize
        fn.argtypes = [c_void_p, c_size_t, c_size_t, c_size_t, c_size_t, c_void_p, c_void_p]
        fn.restype = c_int
        if fn(p(x), rows, heads, d, block, p(codes), p(scales)) != 0:
            raise RuntimeError("ref_kv_int3_quantize failed")
    else:
        ORACLE.oracle_kv_int3_quantize(p(x), rows, heads, d, block, percentile, p(codes), p(scales))
    return codes, scales


def paged_int3_attention(q, k_codes, v_codes, k_scales, v_scales, table, ctx_len, hq, hkv, d, pt, block, scale):
    q = np.ascontiguousarray(q, dtype=np.float32)
    table = np.ascontiguousarray(table, dtype=np.int32)
    ctx = np.ascontiguousarray(ctx_len, dtype=np.int32)
    b = ctx.shape[0]
    out = np.zeros((b, hq, d), dtype=np.float64)
    ORACLE.oracle_paged_int3_attention_f64(p(q), p(np.ascontiguousarray(k_codes)), p(np.ascontiguousarray(v_codes)),
                                           p(np.ascontiguousarray(k_scales, dtype=np.float32)),
                                           p(np.ascontiguousarray(v_scales, dtype=np.float32)), p(table), table.shape[1],
                                           p(ctx), b, hq, hkv, d, pt, block, scale, p(out))
    return out


def q4k_matmul(a: np.ndarray, blocks: np.ndarray, n: int, k: int, reference: bool = False) -> np.ndarray:
    """Q4_K dequant-matmul C = A W^T over [n][k/256] 144-byte blocks
    (q4_k.c:41-134); reference=True runs vspec_q4k_matmul_ref_f32 itself."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    m = a.shape[0]
    out = np.zeros((m, n), dtype=np.float32)
    if reference:
        if REF is None:
            raise RuntimeError("oracle/_ref/libvspec_ref.so not built")
        fn = REF.vspec_q4k_matmul_ref_f32
        fn.argtypes = [c_void_p, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p]
        fn.restype = None
        fn(p(a), m, k, p(blocks), n, p(out))
    else:
        ORACLE.oracle_q4k_matmul_f32(p(a), m, k, p(blocks), n, p(out))
    return out


def random_q4k_blocks(rng, n: int, k: int) -> np.ndarray:
    """Seeded Q4_K rows: fp16 d ~U(0.005, 0.02), dmin ~U(0, 0.1), random 6-bit
    sub-scales / sub-mins and nibbles."""
    nb = k // 256
    blk = rng.integers(0, 256, size=(n, nb, 144), dtype=np.uint8)
    d = rng.uniform(0.005, 0.02, size=(n, nb)).astype(np.float16)
    dmin = rng.uniform(0.0, 0.1, size=(n, nb)).astype(np.float16)
    blk[:, :, 0:2] = d.view(np.uint8).reshape(n, nb, 2)
    blk[:, :, 2:4] = dmin.view(np.uint8).reshape(n, nb, 2)
    return blk


def anf_hybrid(a, w2, s2, w4, s4, zp4, n_blocks: int, hot, n: int, k: int) -> np.ndarray:
    """ANF hybrid linear (fused_linear_hybrid.cu:7-153): int2 draft of every
    column, listed hot columns recomputed from int4 (zero-point added)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    w2 = np.ascontiguousarray(w2, dtype=np.uint8)
    s2 = np.ascontiguousarray(s2, dtype=np.float32)
    hot_arr = np.ascontiguousarray(hot, dtype=np.uint32) if hot is not None else None
    w4 = np.ascontiguousarray(w4, dtype=np.uint8) if w4 is not None else None
    s4 = np.ascontiguousarray(s4, dtype=np.float32) if s4 is not None else None
    zp4 = np.ascontiguousarray(zp4, dtype=np.float32) if zp4 is not None else None
    m = a.shape[0]
    out = np.zeros((m, n), dtype=np.float32)
    fn = ORACLE.oracle_anf_hybrid_f32
    fn.argtypes = [c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                   c_void_p, c_size_t, c_size_t, c_void_p]
    fn.restype = None
    hc = 0 if hot_arr is None else hot_arr.size
    fn(p(a), m, k, p(w2), p(s2), p(w4), p(s4), p(zp4), n_blocks, p(hot_arr) if hc else None, hc, n, p(out))
    return out


class AnfTccState:
    """Host-side temporal selection of the hybrid bridge
    (src/python/cuda_bridge.c:1352-1404): with VSPEC_ENABLE_ANF, VSPEC_ANF_TCC_ENABLE
    and VSPEC_ANF_MODE=active, after `warmup` calls only the hot columns absent
    from the previous call's list are refined, provided they are at most
    `max_changed_ratio` of the list and the list has at least `min_hot` entries."""

    def __init__(self, warmup: int = 4, max_changed_ratio: float = 0.35, min_hot: int = 1):
        self.warmup, self.ratio, self.min_hot = warmup, np.float32(max_changed_ratio), min_hot
        self.steps = 0
        self.prev = None

    def select(self, hot):
        hot = [int(v) for v in hot]
        if not hot:
            return hot
        self.steps += 1
        active = hot
        if self.steps > self.warmup and self.prev and len(hot) >= self.min_hot:
            prev = set(self.prev)
            added = [v for v in hot if v not in prev]
            if np.float32(len(added)) / np.float32(len(hot)) <= self.ratio:
                active = added
        self.prev = list(hot)
        return active
