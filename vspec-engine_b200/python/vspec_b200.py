"""ctypes binding of libvspec_b200.so (the C ABI of include/vspec_b200.h and
include/vspec_b200_compat.h), in the style of the reference's own binding
(Vspec-chat/python/vspec_cuda_bridge.py:9-302).

Device buffers are passed as raw addresses (ints), e.g. a torch tensor's
data_ptr(); host buffers as numpy arrays.  Every native call's status is
checked: a failure raises VspecB200Error with the library's message.  There
is no fallback: if the shared library is missing, importing this module fails.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_size_t, c_uint64, c_void_p

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.abspath(os.path.join(_HERE, "..", "lib", "libvspec_b200.so"))

OK = 0
ERR_ARG = 1
F_SZ_F16 = 0x1
F_UNSIGNED = 0x2
F_RESIDUAL = 0x4
F_RMSNORM = 0x8
F_SWIGLU = 0x10
KV_F32 = 0
KV_F16 = 1
KV_INT3 = 2
PATH_AUTO, PATH_GENERIC, PATH_WARPMMA, PATH_TCGEN05, PATH_RING, PATH_ROWS = 0, 1, 2, 3, 4, 5


class VspecB200Error(RuntimeError):
    pass


class QwenConfig(ctypes.Structure):
    _fields_ = [("num_layers", c_int), ("hidden", c_int), ("num_heads", c_int), ("num_kv_heads", c_int),
                ("head_dim", c_int), ("intermediate", c_int), ("vocab", c_int), ("bits", c_int), ("group", c_int),
                ("rms_eps", c_float), ("rope_theta", c_float), ("logit_clip", c_float), ("page_tokens", c_int),
                ("bits_mlp", c_int)]


# Qwen3-8B shape: 36 layers, hidden 4096, 32/8 heads x 128, SwiGLU 12288, W4 group 128
QWEN3_8B = dict(num_layers=36, hidden=4096, num_heads=32, num_kv_heads=8, head_dim=128, intermediate=12288,
                vocab=151936, bits=4, group=128, rms_eps=1e-6, rope_theta=1e6, logit_clip=24.0, page_tokens=16,
                bits_mlp=0)

# Qwen3-32B shape: 64 layers, hidden 5120, 64/8 heads x 128, SwiGLU 25600; attention and lm_head W4, MLP W3
QWEN3_32B = dict(num_layers=64, hidden=5120, num_heads=64, num_kv_heads=8, head_dim=128, intermediate=25600,
                 vocab=151936, bits=4, group=128, rms_eps=1e-6, rope_theta=1e6, logit_clip=24.0, page_tokens=16,
                 bits_mlp=3)


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libvspec_b200.so not built: {LIB_PATH} (run __graft_entry__.build())")
    return ctypes.CDLL(LIB_PATH)


lib = _load()


class LinearArgs(ctypes.Structure):
    _fields_ = [
        ("d_x", c_void_p), ("d_w", c_void_p), ("d_scales", c_void_p), ("d_zero_points", c_void_p),
        ("zero_point_const", c_float), ("d_y", c_void_p), ("d_residual", c_void_p), ("d_norm_weight", c_void_p),
        ("norm_eps", c_float), ("m", c_size_t), ("n", c_size_t), ("k", c_size_t), ("n_groups", c_size_t),
        ("bits", c_int), ("flags", c_int), ("d_workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


class PagedAttnArgs(ctypes.Structure):
    _fields_ = [
        ("d_q", c_void_p), ("d_k_pages", c_void_p), ("d_v_pages", c_void_p), ("d_page_table", c_void_p),
        ("d_ctx_len", c_void_p), ("d_out", c_void_p),
        ("batch", c_size_t), ("num_q_heads", c_size_t), ("num_kv_heads", c_size_t), ("head_dim", c_size_t),
        ("page_tokens", c_size_t), ("max_pages_per_seq", c_size_t), ("num_pages", c_size_t), ("max_ctx", c_size_t),
        ("scale", c_float), ("kv_dtype", c_int), ("d_workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


# ---- reference ABI structs (include/vspec/quant/quant.h, kernel/context.h, attention/kv_cache.h) ----
class QuantMeta(ctypes.Structure):
    _fields_ = [("schema_version", ctypes.c_uint), ("type", c_int), ("scales", c_void_p), ("scale_count", c_size_t),
                ("special_format", c_int), ("special_data", c_void_p)]


class ExecConfig(ctypes.Structure):
    _fields_ = [("m", c_size_t), ("n", c_size_t), ("k", c_size_t), ("flags", c_size_t)]


class KernelContext(ctypes.Structure):
    _fields_ = [("input", c_void_p), ("weight", c_void_p), ("output", c_void_p), ("qmeta", QuantMeta),
                ("config", ExecConfig)]


class KVCache(ctypes.Structure):
    _fields_ = [
        ("key", c_void_p), ("value", c_void_p), ("max_tokens", c_size_t), ("num_heads", c_size_t),
        ("head_dim", c_size_t), ("current_tokens", c_size_t), ("int3_compressed", c_int), ("key_int3", c_void_p),
        ("value_int3", c_void_p), ("key_scales", c_void_p), ("value_scales", c_void_p), ("block_size", c_size_t),
        ("blocks_per_head", c_size_t), ("packed_head_bytes", c_size_t), ("scratch_key_head", c_void_p),
        ("scratch_value_head", c_void_p), ("owns_int3_buffers", c_int),
    ]


class Backend(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("launch_linear", c_void_p), ("launch_attention", c_void_p)]


QUANT_INT2, QUANT_INT3, QUANT_INT4 = 2, 3, 4

_sigs = {
    "vspec_b200_last_error": ([], ctypes.c_char_p),
    "vspec_b200_version": ([], ctypes.c_char_p),
    "vspec_b200_lowbit_linear": ([POINTER(LinearArgs), c_void_p], c_int),
    "vspec_b200_lowbit_linear_generic": ([POINTER(LinearArgs), c_void_p], c_int),
    "vspec_b200_lowbit_linear_path": ([POINTER(LinearArgs), c_void_p, c_int], c_int),
    "vspec_b200_lowbit_linear_workspace_bytes": ([c_size_t, c_size_t, c_size_t, c_int], c_size_t),
    "vspec_b200_gemv_timeout_flag": ([POINTER(c_int)], c_int),
    "vspec_b200_unpack_codes": ([c_void_p, c_size_t, c_size_t, c_int, c_int, c_void_p, c_int, c_void_p], c_int),
    "vspec_b200_device_info": ([POINTER(c_int), POINTER(c_int), POINTER(c_int), POINTER(c_size_t)], c_int),
    "vspec_b200_dequant_f32": ([c_void_p, c_void_p, c_void_p, c_float, c_int, c_int, c_size_t, c_size_t, c_size_t,
                                c_void_p, c_void_p], c_int),
    "vspec_b200_clamp_rows_std": ([c_void_p, c_void_p, c_size_t, c_size_t, c_float, c_void_p], c_int),
    "vspec_b200_int3_blocknorm_linear": ([c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_int,
                                          c_void_p], c_int),
    "vspec_b200_mean_code_zero_points": ([c_void_p, c_size_t, c_size_t, c_int, c_void_p, c_void_p], c_int),
    "vspec_b200_paged_attention_workspace_bytes": ([c_size_t] * 5, c_size_t),
    "vspec_b200_paged_attention": ([POINTER(PagedAttnArgs), c_void_p], c_int),
    "vspec_b200_attention_ref_workspace_bytes": ([c_size_t, c_size_t, c_size_t], c_size_t),
    "vspec_b200_attention_ref_f32": ([c_void_p] * 3 + [c_size_t] * 3 + [c_int, c_size_t, c_void_p, c_size_t, c_void_p,
                                                                     c_void_p], c_int),
    "vspec_b200_paged_attention_page_fault": ([POINTER(c_int)], c_int),
    "vspec_b200_kv_paged_sync": ([c_void_p, c_int, c_void_p, c_void_p, c_uint64, POINTER(c_uint64), c_void_p], c_int),
    "vspec_b200_kv_paged_session_view": ([c_void_p, c_uint64, c_int, c_void_p, c_void_p, c_size_t, c_size_t, c_void_p,
                                          c_size_t, c_void_p, POINTER(c_size_t), POINTER(c_size_t), c_void_p], c_int),
    "vspec_b200_q4k_linear": ([c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p], c_int),
    "vspec_b200_anf_hybrid_linear": ([c_void_p] * 8 + [c_size_t] * 5 + [c_void_p], c_int),
    "vspec_b200_refine_hot_int4": ([c_void_p] * 6 + [c_size_t] * 5 + [c_void_p], c_int),
    "vspec_cuda_fused_linear_hybrid_device": ([c_void_p] * 8 + [c_size_t] * 5, None),
    "vspec_cuda_fused_linear_hybrid_bridge": ([c_void_p] * 6 + [c_size_t] * 3 + [c_void_p, c_size_t, c_size_t,
                                                                                  c_void_p], c_int),
    "vspec_cuda_fused_linear_hybrid_profile_bridge": ([c_void_p] * 6 + [c_size_t] * 3 +
                                                      [c_void_p, c_size_t, c_size_t] + [c_void_p] * 5, c_int),
    "vspec_b200_kv_int3_quantize": ([c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_size_t, c_float, c_void_p,
                                     c_void_p, c_void_p], c_int),
    "vspec_b200_paged_attention_int3": ([POINTER(PagedAttnArgs), c_void_p, c_void_p, c_size_t, c_void_p], c_int),
    "vspec_b200_paged_gather": ([c_void_p, c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_size_t, c_int, c_void_p,
                                 c_void_p, c_void_p], c_int),
    "vspec_b200_rmsnorm_f32": ([c_void_p, c_void_p, c_float, c_size_t, c_size_t, c_void_p, c_void_p], c_int),
    "vspec_b200_linear_f32": ([c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p, c_void_p], c_int),
    "vspec_b200_silu_f32": ([c_void_p, c_size_t, c_void_p], c_int),
    "vspec_b200_mul_f32": ([c_void_p, c_void_p, c_size_t, c_void_p], c_int),
    "vspec_b200_debug_fail_alloc_after": ([c_int], c_int),
    "vspec_b200_debug_anf_tcc_select": ([c_void_p, c_size_t, c_int, c_void_p, POINTER(c_size_t)], c_int),
    "vspec_b200_lowbit_linear_static": ([POINTER(LinearArgs), c_void_p], c_int),
    "vspec_b200_decode_embed": ([c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p], c_int),
    "vspec_b200_decode_qk_rope_append": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float,
                                          c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p,
                                          c_void_p], c_int),
    "vspec_b200_decode_next_token": ([c_void_p, c_int, c_int, c_float, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                                      c_void_p, c_int, c_void_p, c_void_p], c_int),
    "vspec_b200_random_fill": ([c_void_p, c_size_t, c_int, c_uint64, c_float, c_float, c_void_p], c_int),
    "vspec_b200_random_fill_block": ([c_void_p, c_size_t, c_size_t, c_size_t, c_int, c_uint64, c_size_t, c_size_t,
                                      c_size_t, c_float, c_float, c_void_p], c_int),
    "vspec_b200_quantize_rowwise": ([c_void_p, c_size_t, c_size_t, c_int, c_int, ctypes.c_double, c_void_p, c_void_p,
                                     c_void_p, c_void_p], c_int),
    "vspec_b200_qwen_create": ([POINTER(QwenConfig), c_uint64, c_int, c_int, POINTER(c_void_p)], c_int),
    "vspec_b200_nccl_unique_id": ([c_void_p], c_int),
    "vspec_b200_qwen_create_tp": ([POINTER(QwenConfig), c_uint64, c_int, c_int, c_int, c_int, c_void_p,
                                   POINTER(c_void_p)], c_int),
    "vspec_b200_qwen_destroy": ([c_void_p], None),
    "vspec_b200_qwen_generate": ([c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, POINTER(c_float), c_void_p],
                                 c_int),
    "vspec_b200_qwen_tensor": ([c_void_p, c_int, c_int, c_void_p], c_size_t),
    # reference-named (compat) exports
    "vspec_cuda_fused_available": ([], c_int),
    "vspec_cuda_backend_available": ([], c_int),
    "vspec_cuda_runtime_available": ([], c_int),
    "vspec_make_cuda_backend": ([], Backend),
    "vspec_cuda_launch_linear_impl": ([POINTER(KernelContext)], None),
    "vspec_cuda_launch_attention_impl": ([POINTER(KernelContext)], None),
    "vspec_cuda_launch_fused_linear_int4": ([POINTER(KernelContext)], None),
    "vspec_cuda_launch_fused_linear_int3": ([POINTER(KernelContext)], None),
    "vspec_cuda_launch_fused_linear_int2": ([POINTER(KernelContext)], None),
    "vspec_cuda_launch_fused_linear_int3_storage": ([POINTER(KernelContext)], None),
    "vspec_cuda_launch_attention_fused": ([POINTER(KernelContext)], None),
    "vspec_b200_make_cpu_semantics_backend": ([], Backend),
    "vspec_b200_launch_attention_ref": ([POINTER(KernelContext)], None),
    "vspec_cuda_attention_fused_single_f32": ([c_void_p] * 3 + [c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_attention_flash_single_f32": ([c_void_p] * 3 + [c_size_t, c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_fused_linear_int4_device": ([c_void_p] * 5 + [c_size_t] * 4, None),
    "vspec_cuda_dequant_int4_to_f32_device": ([c_void_p] * 4 + [c_size_t] * 3, None),
    "vspec_cuda_fused_linear_int3_device": ([c_void_p] * 4 + [c_size_t] * 3 + [c_int], None),
    "vspec_cuda_fused_linear_int2_device": ([c_void_p] * 4 + [c_size_t] * 3, None),
    "vspec_cuda_dequant_int2_to_f32_device": ([c_void_p] * 3 + [c_size_t] * 2, None),
    "vspec_cuda_expand_int3_to_int4_device": ([c_void_p] * 2 + [c_size_t] * 2, None),
    "vspec_cuda_rmsnorm_f32": ([c_void_p, c_void_p, c_float, c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_linear_f32": ([c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_gemm_f32": ([c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_attention_single_f32": ([c_void_p] * 3 + [c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_silu_f32": ([c_void_p, c_size_t], None),
    "vspec_cuda_mul_f32": ([c_void_p, c_void_p, c_size_t], None),
    "vspec_cuda_gemm_dispatch_bridge": ([c_void_p] * 5 + [c_size_t] * 4 + [c_int, POINTER(c_int), c_void_p,
                                                                             POINTER(c_int)], c_int),
    "vspec_cuda_fused_linear_int4_register_weight_bridge": ([c_void_p] * 3 + [c_size_t] * 3, c_int),
    "vspec_cuda_fused_linear_int4_cached_bridge": ([c_void_p, c_size_t, c_size_t, c_int, c_size_t, c_void_p], c_int),
    "vspec_cuda_fused_linear_int4_cached_many_bridge": ([c_void_p, c_size_t, c_size_t, c_void_p, c_void_p, c_size_t,
                                                         c_void_p], c_int),
    "vspec_cuda_int4_cached_stats_bridge": ([POINTER(c_uint64)] * 6, c_int),
    "vspec_cuda_fused_linear_int4_bridge": ([c_void_p] * 4 + [c_size_t] * 4 + [c_void_p], c_int),
    "vspec_cuda_fused_linear_int3_bridge": ([c_void_p] * 3 + [c_size_t] * 3 + [c_void_p], c_int),
    "vspec_cuda_rmsnorm_f32_bridge": ([c_void_p, c_void_p, c_float, c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_linear_f32_bridge": ([c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_gemm_f32_bridge": ([c_void_p, c_void_p, c_size_t, c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_attention_single_f32_bridge": ([c_void_p] * 3 + [c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_attention_fused_single_f32_bridge": ([c_void_p] * 3 + [c_size_t, c_size_t, c_void_p], None),
    "vspec_attention_flash_single_f32_bridge": ([c_void_p] * 3 + [c_size_t, c_size_t, c_size_t, c_void_p], None),
    "vspec_cuda_silu_f32_bridge": ([c_void_p, c_size_t], None),
    "vspec_cuda_mul_f32_bridge": ([c_void_p, c_void_p, c_size_t, c_void_p], None),
    "vspec_cuda_mem_info_bridge": ([POINTER(c_size_t), POINTER(c_size_t)], c_int),
    "vspec_cuda_device_capability_bridge": ([POINTER(c_int)] * 3, c_int),
    "vspec_cuda_int4_tensorcore_available_bridge": ([], c_int),
}

for _name, (_args, _res) in _sigs.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = _args
    _fn.restype = _res


def last_error() -> str:
    return lib.vspec_b200_last_error().decode()


def check(rc: int, what: str = "") -> None:
    if rc != OK:
        raise VspecB200Error(f"{what} failed (status {rc}): {last_error()}")


def hptr(a: np.ndarray | None) -> int | None:
    """Host address of a C-contiguous numpy array (None for None)."""
    if a is None:
        return None
    assert a.flags.c_contiguous
    return a.ctypes.data


def lowbit_linear(x: int, w: int, scales: int | None, zp: int | None, y: int, m: int, n: int, k: int, n_groups: int,
                  bits: int, flags: int = 0, zp_const: float = 0.0, residual: int | None = None,
                  norm_weight: int | None = None, eps: float = 1e-6, stream: int = 0, generic: bool = False,
                  workspace: int | None = None, workspace_bytes: int = 0, path: int | None = None) -> None:
    a = LinearArgs(x, w, scales, zp, zp_const, y, residual, norm_weight, eps, m, n, k, n_groups, bits, flags,
                   workspace, workspace_bytes)
    if path is None:
        path = PATH_GENERIC if generic else PATH_AUTO
    check(lib.vspec_b200_lowbit_linear_path(ctypes.byref(a), stream, path), "vspec_b200_lowbit_linear")


def unpack_codes(w: int, n: int, k: int, bits: int, out: int, unsigned: bool = False, fast: bool = True,
                 stream: int = 0) -> None:
    check(lib.vspec_b200_unpack_codes(w, n, k, bits, int(unsigned), out, int(fast), stream), "unpack_codes")


def paged_attention(q: int, k_pages: int, v_pages: int, page_table: int, ctx_len: int, out: int, batch: int, hq: int,
                    hkv: int, d: int, page_tokens: int, max_pages: int, num_pages: int, max_ctx: int, scale: float,
                    kv_dtype: int = KV_F16, workspace: int | None = None, workspace_bytes: int = 0,
                    stream: int = 0) -> None:
    a = PagedAttnArgs(q, k_pages, v_pages, page_table, ctx_len, out, batch, hq, hkv, d, page_tokens, max_pages,
                      num_pages, max_ctx, scale, kv_dtype, workspace, workspace_bytes)
    check(lib.vspec_b200_paged_attention(ctypes.byref(a), stream), "vspec_b200_paged_attention")


def attention_ref(q: int, keys: int, values: int, out: int, tokens: int, heads: int, d: int, module: int = -1,
                  block: int = 0, workspace: int | None = None, workspace_bytes: int = 0, stream: int = 0) -> None:
    """The CPU backend's attention semantics on device buffers (attention_ref.c:7-88);
    module -1 = from the environment, block 0 = VSPEC_3BIT_BLOCK_SIZE."""
    check(lib.vspec_b200_attention_ref_f32(q, keys, values, tokens, heads, d, module, block, workspace,
                                           workspace_bytes, out, stream), "vspec_b200_attention_ref_f32")


def kv_int3_quantize(src: int, slots: int | None, rows: int, heads: int, head_dim: int, block: int, codes: int,
                     scales: int, percentile: float = 99.5, stream: int = 0) -> None:
    check(lib.vspec_b200_kv_int3_quantize(src, slots, rows, heads, head_dim, block, percentile, codes, scales, stream),
          "vspec_b200_kv_int3_quantize")


def paged_attention_int3(q: int, k_codes: int, v_codes: int, k_scales: int, v_scales: int, block: int,
                         page_table: int, ctx_len: int, out: int, batch: int, hq: int, hkv: int, d: int,
                         page_tokens: int, max_pages: int, num_pages: int, max_ctx: int, scale: float,
                         workspace: int | None = None, workspace_bytes: int = 0, stream: int = 0) -> None:
    a = PagedAttnArgs(q, k_codes, v_codes, page_table, ctx_len, out, batch, hq, hkv, d, page_tokens, max_pages,
                      num_pages, max_ctx, scale, KV_INT3, workspace, workspace_bytes)
    check(lib.vspec_b200_paged_attention_int3(ctypes.byref(a), k_scales, v_scales, block, stream),
          "vspec_b200_paged_attention_int3")


def q4k_linear(x: int, blocks: int, y: int, m: int, n: int, k: int, stream: int = 0) -> None:
    check(lib.vspec_b200_q4k_linear(x, blocks, y, m, n, k, stream), "vspec_b200_q4k_linear")


def anf_hybrid_linear(x: int, w2: int, s2: int, w4: int | None, s4: int | None, zp4: int | None, y: int,
                      hot: int | None, hot_count: int, m: int, n: int, k: int, n_blocks_int4: int,
                      stream: int = 0) -> None:
    check(lib.vspec_b200_anf_hybrid_linear(x, w2, s2, w4, s4, zp4, y, hot, hot_count, m, n, k, n_blocks_int4, stream),
          "vspec_b200_anf_hybrid_linear")


def page_fault_flag() -> int:
    v = c_int(0)
    check(lib.vspec_b200_paged_attention_page_fault(ctypes.byref(v)), "page_fault")
    return v.value


def _prefer_wheel_nccl() -> None:
    """Point the library at the NCCL of the `nvidia-nccl` wheel when one is
    installed (the copy PyTorch loads), so that a process which later imports
    torch does not meet an older system NCCL already loaded under the same
    soname.  An explicit VSPEC_B200_NCCL_LIB is kept."""
    if os.environ.get("VSPEC_B200_NCCL_LIB"):
        return
    import importlib.util
    try:
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        spec = None
    for base in (spec.submodule_search_locations or []) if spec else []:
        cand = os.path.join(base, "lib", "libnccl.so.2")
        if os.path.exists(cand):
            os.environ["VSPEC_B200_NCCL_LIB"] = cand
            return


def nccl_unique_id() -> bytes:
    """128-byte NCCL unique id for a tensor-parallel group (made by one rank, shared with all)."""
    _prefer_wheel_nccl()
    buf = ctypes.create_string_buffer(128)
    check(lib.vspec_b200_nccl_unique_id(buf), "vspec_b200_nccl_unique_id")
    return buf.raw


class QwenModel:
    """Random-init Qwen3-shape low-bit decoder on the device (vspec_b200_qwen_*).
    With tp_size > 1 this is one rank's shard of a tensor-parallel group (the
    current CUDA device; every rank constructs it with the same nccl_id)."""

    def __init__(self, cfg: dict, seed: int, max_batch: int, max_ctx: int, tp_size: int = 1, tp_rank: int = 0,
                 nccl_id: bytes | None = None):
        self.cfg = dict(cfg)
        self.cfg.setdefault("bits_mlp", 0)
        self._c = QwenConfig(**self.cfg)
        h = c_void_p()
        if tp_size == 1:
            check(lib.vspec_b200_qwen_create(ctypes.byref(self._c), seed, max_batch, max_ctx, ctypes.byref(h)),
                  "vspec_b200_qwen_create")
        else:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("tensor-parallel shard needs the group's 128-byte nccl_id")
            _prefer_wheel_nccl()
            idbuf = ctypes.create_string_buffer(bytes(nccl_id), 128)
            check(lib.vspec_b200_qwen_create_tp(ctypes.byref(self._c), seed, max_batch, max_ctx, tp_size, tp_rank,
                                                idbuf, ctypes.byref(h)), "vspec_b200_qwen_create_tp")
        self.tp_size, self.tp_rank = tp_size, tp_rank
        self.handle = h

    def close(self) -> None:
        if self.handle:
            lib.vspec_b200_qwen_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def generate(self, prompts: np.ndarray, gen: int, want_logits: bool = False):
        prompts = np.ascontiguousarray(prompts, dtype=np.int32)
        b, plen = prompts.shape
        toks = np.zeros((b, plen + gen), dtype=np.int32)
        ms = c_float(0.0)
        logits = np.zeros((plen + gen - 1, b, self.cfg["vocab"]), dtype=np.float32) if want_logits else None
        check(lib.vspec_b200_qwen_generate(self.handle, b, prompts.ctypes.data, plen, gen, toks.ctypes.data,
                                           ctypes.byref(ms), logits.ctypes.data if logits is not None else None),
              "vspec_b200_qwen_generate")
        return toks, ms.value, logits

    def tensor(self, kind: int, layer: int = 0) -> np.ndarray:
        nbytes = lib.vspec_b200_qwen_tensor(self.handle, kind, layer, None)
        if nbytes == 0:
            raise VspecB200Error(f"no tensor kind={kind} layer={layer}")
        out = np.empty(nbytes, dtype=np.uint8)
        if lib.vspec_b200_qwen_tensor(self.handle, kind, layer, out.ctypes.data) != nbytes:
            raise VspecB200Error("tensor download failed")
        return out
