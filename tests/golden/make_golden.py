"""Generate golden fixtures from Vspec-Engine's own Python runtime.

Run where the reference tree is present (its location in VSPEC_REFERENCE,
which has a default below); the fixtures are committed so that machines without
the tree (the GPU box) only read the .npz files.

    python tests/golden/make_golden.py

Fixtures (all seeded):
  int4_groupwise.npz  -- runtime_lowbit_module._unpack_int4_rowwise on
                         group-wise int4 weights (reference group indexing),
                         plus x @ W^T in float64 from that dequantized W.
  pack_rows.npz       -- runtime_inference._pack_signed_rowwise for bits 2/3/4.
  quantize_w4g128.npz -- runtime_inference._quantize_weight_rowwise with
                         VSPEC_INT4_BLOCK_SIZE=128 (config 4's quantizer).
  quantize_variants.npz -- the same function over block sizes 32/40/64/128
                         (a partial last block), per-row int4/int3/int2 and
                         percentiles 0.97/0.995/0.999/1.0.
  attention_gqa.npz   -- runtime_inference._attention_cpu_batched with GQA 4:1.
"""
from __future__ import annotations

import os
import sys

import numpy as np

REF = os.environ.get("VSPEC_REFERENCE", "")
OUT = os.path.dirname(os.path.abspath(__file__))


def main() -> None:
    if not REF or not os.path.isdir(os.path.join(REF, "Vspec-chat", "python")):
        sys.exit("set VSPEC_REFERENCE to the Vspec-Engine source tree (its Vspec-chat/python modules make the fixtures)")
    sys.path.insert(0, os.path.join(REF, "Vspec-chat", "python"))
    os.environ["VSPEC_INT4_BLOCKWISE_ENABLE"] = "1"
    os.environ["VSPEC_INT4_BLOCK_SIZE"] = "128"
    import runtime_inference as ri  # noqa: E402
    import runtime_lowbit_module as rl  # noqa: E402

    rng = np.random.default_rng(20261201)

    # ---- group-wise int4 dequant (Python reference) ----
    cases = {}
    for name, (n, k, g) in {"a": (24, 256, 2), "b": (16, 384, 3), "c": (8, 512, 1), "d": (40, 1024, 8)}.items():
        packed = rng.integers(0, 256, size=(n, (k + 1) // 2), dtype=np.uint8)
        s = rng.uniform(0.005, 0.02, size=(n * g,)).astype(np.float32)
        zp = rng.integers(-8, 8, size=(n * g,)).astype(np.float32)
        w = rl._unpack_int4_rowwise(packed, s, n, k, zp)
        x = rng.standard_normal((3, k)).astype(np.float32)
        y = x.astype(np.float64) @ w.astype(np.float64).T
        cases.update({f"{name}_packed": packed, f"{name}_s": s, f"{name}_zp": zp, f"{name}_w": w, f"{name}_x": x,
                      f"{name}_y": y, f"{name}_dims": np.array([n, k, g], dtype=np.int64)})
    np.savez_compressed(os.path.join(OUT, "int4_groupwise.npz"), **cases)

    # ---- row packing for bits 2/3/4 ----
    packs = {}
    for bits in (2, 3, 4):
        lo, hi = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
        q = rng.integers(lo, hi + 1, size=(7, 61), dtype=np.int8)
        packs[f"q{bits}"] = q
        packs[f"p{bits}"] = ri._pack_signed_rowwise(q, bits).reshape(7, -1)
    np.savez_compressed(os.path.join(OUT, "pack_rows.npz"), **packs)

    # ---- config-4 quantizer (block 128) ----
    wf = (rng.standard_normal((32, 512)) * 0.02).astype(np.float32)
    packed, s, zp = ri._quantize_weight_rowwise(wf, 4)
    np.savez_compressed(os.path.join(OUT, "quantize_w4g128.npz"), w=wf, packed=packed, s=s, zp=zp)


    # ---- GQA attention (Python CPU reference) ----
    hq, hkv, d, t = 8, 2, 64, 97
    q = rng.standard_normal((hq, d)).astype(np.float32)
    keys = rng.standard_normal((t, hkv, d)).astype(np.float32)
    values = rng.standard_normal((t, hkv, d)).astype(np.float32)
    out = ri._attention_cpu_batched(q, keys, values, hq, hkv, False, hq // hkv, 1.0 / np.sqrt(d), 24.0)
    np.savez_compressed(os.path.join(OUT, "attention_gqa.npz"), q=q, keys=keys, values=values, out=out,
                        dims=np.array([hq, hkv, d, t], dtype=np.int64))
    # ---- quantizer variants: block size, per-row int4/int3/int2, percentile ----
    # (name, bits, n, k, VSPEC_INT4_BLOCKWISE_ENABLE, VSPEC_INT4_BLOCK_SIZE, VSPEC_QUANT_ROW_PERCENTILE)
    variants = [("q4_b32", 4, 12, 320, "1", "32", "0.999"), ("q4_b128_k200", 4, 8, 200, "1", "128", "0.999"),
                ("q4_b64_p995", 4, 8, 256, "1", "64", "0.995"), ("q4_row", 4, 8, 512, "0", "128", "0.999"),
                ("q3_row", 3, 8, 384, "1", "128", "0.999"), ("q3_row_p1", 3, 6, 256, "1", "128", "1.0"),
                ("q2_row", 2, 8, 256, "1", "128", "0.999"), ("q4_b40_outlier", 4, 6, 160, "1", "40", "0.97")]
    qrng = np.random.default_rng(20261202)   # its own stream: the fixtures above stay as committed
    qv = {}
    for name, bits, n, k, enable, block, pct in variants:
        os.environ["VSPEC_INT4_BLOCKWISE_ENABLE"] = enable
        os.environ["VSPEC_INT4_BLOCK_SIZE"] = block
        os.environ["VSPEC_QUANT_ROW_PERCENTILE"] = pct
        wv = (qrng.standard_normal((n, k)) * 0.02).astype(np.float32)
        wv[0, 3] = 0.5     # an outlier above the percentile
        packed, s, zp = ri._quantize_weight_rowwise(wv, bits)
        qv[f"{name}_w"] = wv
        qv[f"{name}_packed"] = np.asarray(packed).reshape(n, -1)
        qv[f"{name}_s"] = np.asarray(s, dtype=np.float32)
        qv[f"{name}_zp"] = np.asarray(zp, dtype=np.float32) if zp is not None else np.zeros(0, np.float32)
        qv[f"{name}_cfg"] = np.array([bits, int(enable), int(block), int(float(pct) * 1e6)], dtype=np.int64)
    np.savez_compressed(os.path.join(OUT, "quantize_variants.npz"), **qv)
    os.environ["VSPEC_INT4_BLOCKWISE_ENABLE"] = "1"
    os.environ["VSPEC_INT4_BLOCK_SIZE"] = "128"
    os.environ.pop("VSPEC_QUANT_ROW_PERCENTILE", None)
    print("fixtures written to", OUT)


if __name__ == "__main__":
    main()
