"""C-ABI checks that need no GPU: the library loads, exports every function
include/*.h declares, its structs are layout-identical to the reference's,
and host-side argument validation rejects bad calls before any CUDA work."""
import ctypes
import os
import re

import numpy as np
import pytest

import oracle as O
import vspec_b200 as V

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"typedef\s+struct.*?\}\s*\w+\s*;", "", text, flags=re.S)
        text = re.sub(r"typedef\s+enum.*?\}\s*\w+\s*;", "", text, flags=re.S)
        for m in re.finditer(r"\b(vspec_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_loads_and_versions():
    assert V.lib.vspec_b200_version().decode().startswith("vspec_b200")


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert len(names) > 50
    missing = [n for n in sorted(names) if not hasattr(V.lib, n)]
    assert not missing, missing


@pytest.mark.skipif(O.REF is None, reason="reference CPU library not built")
def test_struct_layouts_match_reference_headers():
    R = O.REF
    assert ctypes.sizeof(V.KernelContext) == R.ref_sizeof_kernel_context()
    assert ctypes.sizeof(V.QuantMeta) == R.ref_sizeof_quant_meta()
    assert ctypes.sizeof(V.ExecConfig) == R.ref_sizeof_exec_config()
    assert ctypes.sizeof(V.KVCache) == R.ref_sizeof_kv_cache()
    assert ctypes.sizeof(V.Backend) == R.ref_sizeof_backend()
    assert V.KernelContext.qmeta.offset == R.ref_offsetof_ctx_qmeta()
    assert V.KernelContext.config.offset == R.ref_offsetof_ctx_config()
    assert V.QuantMeta.scales.offset == R.ref_offsetof_qmeta_scales()
    assert V.QuantMeta.scale_count.offset == R.ref_offsetof_qmeta_scale_count()
    assert V.KVCache.current_tokens.offset == R.ref_offsetof_kv_current_tokens()
    assert V.KVCache.int3_compressed.offset == R.ref_offsetof_kv_int3()
    # VspecKVPagedCache is 332,904 bytes in the reference headers
    assert R.ref_sizeof_kv_paged_cache() == 332904


def test_c_header_compiles_against_reference_headers(tmp_path):
    """vspec_b200_compat.h must coexist with the reference's own headers (it
    reuses their struct definitions when they are included first)."""
    ref_inc = os.path.join(os.environ.get("VSPEC_REFERENCE", ""), "include")
    if not os.path.isdir(ref_inc):
        pytest.skip("reference headers not present")
    src = tmp_path / "t.c"
    src.write_text('#include "vspec/kernel/backend.h"\n#include "vspec/attention/kv_cache.h"\n'
                   '#include "vspec_b200_compat.h"\n#include "vspec_b200.h"\n'
                   'int main(void){VspecBackend b = vspec_make_cuda_backend(); return b.name == 0;}\n')
    rc = os.system(f"gcc -std=gnu11 -Wall -Werror -c -I{ref_inc} -I{ROOT}/include {src} -o {tmp_path}/t.o")
    assert rc == 0


def _args(**kw):
    base = dict(d_x=None, d_w=None, d_scales=None, d_zero_points=None, zero_point_const=0.0, d_y=None,
                d_residual=None, d_norm_weight=None, norm_eps=0.0, m=1, n=16, k=128, n_groups=1, bits=4, flags=0)
    base.update(kw)
    return V.LinearArgs(**base)


@pytest.mark.parametrize("kw,expect", [
    (dict(), V.OK + 1),                                   # NULL pointers
    (dict(d_x=16, d_w=16, d_y=16, m=0), 1),               # zero dimension
    (dict(d_x=16, d_w=16, d_y=16, bits=5), 1),            # bad bit width
    (dict(d_x=16, d_w=16, d_y=16, flags=V.F_RESIDUAL), 1),  # residual flag without residual
    (dict(d_x=16, d_w=16, d_y=16, flags=V.F_RMSNORM), 1),   # norm flag without weight
    (dict(d_x=16, d_w=16, d_y=16, n_groups=1000), 1),       # more groups than k
    (dict(d_x=16, d_w=16, d_y=16, n=15, flags=V.F_SWIGLU), 1),  # SwiGLU needs even n
])
def test_linear_rejects_bad_arguments_on_host(kw, expect):
    a = _args(**kw)
    rc = V.lib.vspec_b200_lowbit_linear(ctypes.byref(a), None)
    assert rc == V.OK + 1 == expect
    assert V.last_error() != "ok"


def test_attention_rejects_bad_arguments_on_host():
    a = V.PagedAttnArgs()
    assert V.lib.vspec_b200_paged_attention(ctypes.byref(a), None) == 1
    a = V.PagedAttnArgs(16, 16, 16, 16, 16, 16, 1, 6, 4, 128, 16, 4, 4, 64, 0.1, V.KV_F16, None, 0)
    assert V.lib.vspec_b200_paged_attention(ctypes.byref(a), None) == 1   # 6 % 4 != 0
    a = V.PagedAttnArgs(16, 16, 16, 16, 16, 16, 1, 8, 4, 128, 16, 4, 4, 65, 0.1, V.KV_F16, None, 0)
    assert V.lib.vspec_b200_paged_attention(ctypes.byref(a), None) == 1   # max_ctx > 4 pages * 16
    assert "exceeds" in V.last_error()


def test_reference_bridges_fail_closed_on_bad_input():
    # cuda_bridge.c contract: 0 on invalid input, caller falls back
    assert V.lib.vspec_cuda_fused_linear_int4_register_weight_bridge(None, None, None, 128, 16, 1) == 0
    assert V.lib.vspec_cuda_fused_linear_int4_cached_bridge(None, 1, 128, 1, 16, None) == 0
    assert V.lib.vspec_cuda_fused_linear_int4_bridge(None, None, None, None, 1, 128, 16, 1, None) == 0
    assert V.lib.vspec_cuda_gemm_dispatch_bridge(None, None, None, None, None, 0, 0, 0, 0, 4, None, None, None) == 0
    stats = [ctypes.c_uint64() for _ in range(6)]
    assert V.lib.vspec_cuda_int4_cached_stats_bridge(*[ctypes.byref(s) for s in stats]) == 1
    assert stats[2].value >= 1   # the failed cached call counted as a miss


def test_reference_python_bridge_binds_library(tmp_path):
    """The reference's unmodified ctypes bridge (Vspec-chat/python/vspec_cuda_bridge.py)
    loads <root>/build/vspec_cuda_bridge.dll with root = parents[2] of the module
    (vspec_cuda_bridge.py:9-31).  A symlink to this library there must satisfy
    every unconditional binding at import and every optional hasattr probe on the
    path, the ANF hybrid bridge included."""
    import shutil
    import subprocess
    import sys
    ref = os.environ.get("VSPEC_REFERENCE", "")
    src = os.path.join(ref, "Vspec-chat", "python", "vspec_cuda_bridge.py")
    if not os.path.exists(src):
        pytest.skip("reference tree not present")
    pkg = tmp_path / "vspec" / "Vspec-chat" / "python"
    pkg.mkdir(parents=True)
    (tmp_path / "vspec" / "build").mkdir()
    shutil.copy(src, pkg / "vspec_cuda_bridge.py")
    os.symlink(V.LIB_PATH, tmp_path / "vspec" / "build" / "vspec_cuda_bridge.dll")
    names = ["_HAS_FUSED_INT4", "_HAS_FUSED_INT3", "_HAS_INT4_REGISTERED", "_HAS_INT4_REGISTERED_MANY",
             "_HAS_INT4_CACHED_STATS", "_HAS_GEMM_DISPATCH", "_HAS_FUSED_ATTN", "_HAS_FLASH_ATTN",
             "_HAS_DEVICE_CAP", "_HAS_INT4_TENSORCORE", "_HAS_FUSED_HYBRID"]
    code = ("import vspec_cuda_bridge as b; print(b._lib is not None, "
            + ", ".join(f"b.{n}" for n in names) + ")")
    env = dict(os.environ, PYTHONPATH=str(pkg))
    out = subprocess.run([sys.executable, "-c", code], cwd=str(tmp_path), env=env, capture_output=True,
                         text=True, timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    got = dict(zip(["loaded"] + names, out.stdout.split()))
    assert got.pop("loaded") == "True"
    assert all(v == "True" for v in got.values()), got


def test_tensor_parallel_create_rejects_bad_shards_on_host():
    """Shard checks run before any CUDA call: heads, kv heads and intermediate
    must divide by tp_size, the row-parallel slices must be whole scale
    groups, rank must be in range and a group of more than one needs an id."""
    base = dict(num_layers=2, hidden=256, num_heads=4, num_kv_heads=2, head_dim=64, intermediate=512, vocab=1000,
                bits=4, group=128, rms_eps=1e-6, rope_theta=1e6, logit_clip=24.0, page_tokens=16, bits_mlp=3)
    nid = ctypes.create_string_buffer(128)
    h = ctypes.c_void_p()
    cases = [
        (dict(base), 3, 0, nid),                       # 4 heads over 3 ranks
        (dict(base, num_kv_heads=1, num_heads=2), 2, 0, nid),
        (dict(base), 4, 0, nid),                       # q slice 64 columns: not a whole group
        (dict(base, intermediate=384), 2, 0, nid),     # 192-column down slice
        (dict(base), 2, 2, nid),                       # rank out of range
        (dict(base), 2, 0, None),                      # no id
        (dict(base, bits_mlp=5), 1, 0, None),
    ]
    for cfg, tp, rank, idbuf in cases:
        c = V.QwenConfig(**cfg)
        rc = V.lib.vspec_b200_qwen_create_tp(ctypes.byref(c), 1, 4, 64, tp, rank, idbuf, ctypes.byref(h))
        assert rc == 1, (cfg, tp, rank)
        assert not h.value


def test_nccl_unique_id_and_later_torch_import():
    """The tensor-parallel group id comes from the NCCL that PyTorch also
    loads, so importing torch afterwards in the same process still works."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, sys.argv[1]); import vspec_b200 as V; i = V.nccl_unique_id(); "
            "assert len(i) == 128 and any(i); import torch; print('ok')")
    r = subprocess.run([sys.executable, "-c", code, os.path.dirname(V.__file__)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]


def test_q4k_and_hybrid_refuse_bad_arguments_before_any_cuda_call():
    """Argument checks of the Q4_K, hybrid and int4-refine entry points run on
    the host first (no device is touched): status codes and messages, and the
    hybrid bridges' 0 return (cuda_bridge.c:1323-1331)."""
    fake = 0x10000   # never dereferenced on the host
    assert V.lib.vspec_b200_q4k_linear(None, fake, fake, 1, 4, 256, None) == 1
    assert V.lib.vspec_b200_q4k_linear(fake, fake, fake, 1, 4, 200, None) == 3
    assert "multiple of 256" in V.last_error()
    assert V.lib.vspec_b200_q4k_linear(fake + 4, fake, fake, 1, 4, 256, None) == 1
    assert "16-byte aligned" in V.last_error()
    assert V.lib.vspec_b200_q4k_linear(fake, fake, fake, 1, 4, 8448, None) == 3
    assert V.lib.vspec_b200_q4k_linear(fake, fake, fake, 0, 4, 256, None) == 0   # nothing to do
    assert V.lib.vspec_b200_refine_hot_int4(fake, fake, fake, None, fake, fake, 0, 1, 4, 64, 1, None) == 0
    assert V.lib.vspec_b200_refine_hot_int4(fake, None, fake, None, fake, fake, 3, 1, 4, 64, 1, None) == 1
    assert V.lib.vspec_b200_refine_hot_int4(fake, fake, fake, None, fake, fake, 3, 1, 4, 0, 1, None) == 1
    assert V.lib.vspec_b200_anf_hybrid_linear(None, fake, fake, None, None, None, fake, None, 0, 1, 4, 64, 1,
                                              None) == 1
    assert V.lib.vspec_b200_anf_hybrid_linear(fake, fake, fake, None, None, None, fake, None, 0, 0, 4, 64, 1,
                                              None) == 0
    x = np.zeros(64, dtype=np.float32)
    w2 = np.zeros(16, dtype=np.uint8)
    s = np.ones(4, dtype=np.float32)
    hot = np.array([1], dtype=np.uint32)
    out = np.zeros(4, dtype=np.float32)
    bridge = V.lib.vspec_cuda_fused_linear_hybrid_bridge
    assert bridge(None, w2.ctypes.data, s.ctypes.data, None, None, None, 1, 64, 4, None, 0, 1, out.ctypes.data) == 0
    assert bridge(x.ctypes.data, w2.ctypes.data, s.ctypes.data, None, None, None, 1, 64, 4, None, 1, 1,
                  out.ctypes.data) == 0                        # hot_count without a hot list
    assert bridge(x.ctypes.data, w2.ctypes.data, s.ctypes.data, None, None, None, 1, 64, 4, hot.ctypes.data, 1, 1,
                  out.ctypes.data) == 0                        # hot list without int4 weights
    assert bridge(x.ctypes.data, w2.ctypes.data, s.ctypes.data, None, None, None, 0, 64, 4, None, 0, 1,
                  out.ctypes.data) == 0                        # m == 0


def test_int3_kv_entry_points_refuse_bad_arguments_on_host():
    fake = 0x10000
    q = V.lib.vspec_b200_kv_int3_quantize
    assert q(None, None, 1, 1, 128, 32, 99.5, fake, fake, None) == 1
    assert q(fake, None, 0, 1, 128, 32, 99.5, fake, fake, None) == 0          # no rows: nothing to do
    assert q(fake, None, 1, 1, 128, 24, 99.5, fake, fake, None) == 1
    assert "block_size" in V.last_error()
    assert q(fake, None, 1, 1, 136, 32, 99.5, fake, fake, None) == 1          # 136 % 32 != 0
    a = V.PagedAttnArgs(fake, fake, fake, fake, fake, fake, 1, 8, 8, 128, 16, 1, 1, 16, 0.1, V.KV_F16, None, 0)
    assert V.lib.vspec_b200_paged_attention_int3(ctypes.byref(a), fake, fake, 32, None) == 1
    assert "KV_INT3" in V.last_error()
    a = V.PagedAttnArgs(fake, fake, fake, fake, fake, fake, 1, 8, 8, 64, 16, 1, 1, 16, 0.1, V.KV_INT3, None, 0)
    assert V.lib.vspec_b200_paged_attention_int3(ctypes.byref(a), fake, fake, 32, None) == 3
    assert "head_dim 128" in V.last_error()
    a = V.PagedAttnArgs(fake, fake, fake, fake, fake, fake, 1, 32, 2, 128, 16, 1, 1, 16, 0.1, V.KV_INT3, None, 0)
    assert V.lib.vspec_b200_paged_attention_int3(ctypes.byref(a), fake, fake, 32, None) == 1   # 16 q heads per KV head
    a = V.PagedAttnArgs(fake, fake, fake, fake, fake, fake, 1, 8, 8, 128, 16, 1, 1, 17, 0.1, V.KV_INT3, None, 0)
    assert V.lib.vspec_b200_paged_attention_int3(ctypes.byref(a), fake, fake, 32, None) == 1
    assert "exceeds" in V.last_error()


def test_compat_declarations_agree_with_reference_kernel_headers(tmp_path):
    """Every cuda_fused.h / cuda_ops.h function that vspec_b200_compat.h also
    declares (the hybrid and refine launchers among them) must have the same
    signature: one translation unit includes both, and gcc rejects conflicting
    declarations."""
    ref_inc = os.path.join(os.environ.get("VSPEC_REFERENCE", ""), "include")
    if not os.path.isfile(os.path.join(ref_inc, "vspec", "kernel", "cuda_fused.h")):
        pytest.skip("reference headers not present")
    src = tmp_path / "t2.c"
    src.write_text('#include "vspec/kernel/cuda_fused.h"\n#include "vspec/kernel/cuda_ops.h"\n'
                   '#include "vspec_b200_compat.h"\n'
                   'int main(void){ return vspec_cuda_fused_linear_hybrid_device == 0 || '
                   'vspec_cuda_refine_hot_int4_device == 0; }\n')
    rc = os.system(f"gcc -std=gnu11 -Wall -Werror -Wno-address -c -I{ref_inc} -I{ROOT}/include {src} "
                   f"-o {tmp_path}/t2.o")
    assert rc == 0


def test_bridge_declarations_agree_with_reference_bridge(tmp_path):
    """Each VSPEC_CUDA_API export of the reference's src/python/cuda_bridge.c
    (its prototypes read as text) is declared by vspec_b200_compat.h with the
    same signature: the reference prototypes are compiled after the compat
    header in one translation unit."""
    ref = os.environ.get("VSPEC_REFERENCE", "")
    path = os.path.join(ref, "src", "python", "cuda_bridge.c")
    if not os.path.isfile(path):
        pytest.skip("reference tree not present")
    text = open(path).read()
    protos = {}
    for m in re.finditer(r"VSPEC_CUDA_API\s+([\w\s\*]+?)\s*\b(vspec_\w+)\s*\(([^)]*)\)", text):
        protos.setdefault(m.group(2), f"{m.group(1).strip()} {m.group(2)}({' '.join(m.group(3).split())});")
    assert len(protos) >= 20
    compat = open(os.path.join(ROOT, "include", "vspec_b200_compat.h")).read()
    assert [n for n in protos if not re.search(r"\b" + n + r"\s*\(", compat)] == []
    src = tmp_path / "t3.c"
    src.write_text('#include <stddef.h>\n#include <stdint.h>\n#include "vspec_b200_compat.h"\n'
                   + "\n".join(protos.values()) + "\nint main(void){return 0;}\n")
    rc = os.system(f"gcc -std=gnu11 -Wall -Werror -c -I{ROOT}/include {src} -o {tmp_path}/t3.o")
    assert rc == 0


def test_compat_paged_cache_layout_matches_reference(tmp_path):
    """The VspecKVPagedCache restated in vspec_b200_compat.h (read by
    vspec_b200_kv_paged_sync / _session_view) has the reference's size and
    member offsets (include/vspec/attention/kv_paged_cache.h:20-49)."""
    import oracle as O
    if O.REF is None:
        pytest.skip("oracle/_ref not built")
    src = tmp_path / "p.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "vspec_b200_compat.h"\n'
                   'int main(void){printf("%zu %zu %zu", sizeof(VspecKVPagedCache), '
                   'offsetof(VspecKVPagedCache, sessions), offsetof(VspecKVPagedCache, page_meta)); return 0;}\n')
    exe = tmp_path / "p"
    assert os.system(f"gcc -std=gnu11 -Wall -Werror -I{ROOT}/include {src} -o {exe}") == 0
    import subprocess
    size, off_s, off_p = map(int, subprocess.check_output([str(exe)]).split())
    assert size == O.REF.ref_sizeof_kv_paged_cache()
    assert off_s == O.REF.ref_offsetof_paged_sessions()
    assert off_p == O.REF.ref_offsetof_paged_page_meta()
