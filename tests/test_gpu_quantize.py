"""Load-time quantise + pack on the GPU (vspec_b200_quantize_rowwise) against
the reference quantizer's own output (golden fixtures made by
runtime_inference._quantize_weight_rowwise) and, at larger shapes, against
the C restatement pinned to those fixtures: packed codes, scales and
zero-points bit for bit."""
import ctypes

import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import torch_cuda
from test_oracle_pins import GOLDEN, _effective_block

pytestmark = pytest.mark.gpu


def gpu_quantize(w: np.ndarray, bits: int, block: int, pct: float):
    torch = torch_cuda()
    n, k = w.shape
    nb = (k + block - 1) // block if block > 0 else 1
    dw = torch.from_numpy(np.ascontiguousarray(w, dtype=np.float32)).cuda()
    dp = torch.zeros((n, O.row_bytes(k, bits)), dtype=torch.uint8, device="cuda")
    ds = torch.zeros(n * nb, dtype=torch.float32, device="cuda")
    dz = torch.zeros(n * nb, dtype=torch.float32, device="cuda")
    rc = V.lib.vspec_b200_quantize_rowwise(dw.data_ptr(), n, k, bits, block, ctypes.c_double(pct), dp.data_ptr(),
                                           ds.data_ptr(), dz.data_ptr(), None)
    assert rc == 0, V.last_error()
    torch.cuda.synchronize()
    return dp.cpu().numpy(), ds.cpu().numpy(), dz.cpu().numpy()


def test_quantize_matches_reference_fixtures():
    z = np.load(f"{GOLDEN}/quantize_variants.npz")
    for nm in sorted({k.rsplit("_", 1)[0] for k in z.files}):
        bits, enable, block, pct = (int(v) for v in z[nm + "_cfg"])
        packed, s, zp = gpu_quantize(z[nm + "_w"], bits, _effective_block(bits, enable, block), pct / 1e6)
        assert np.array_equal(packed, z[nm + "_packed"]), nm
        assert np.array_equal(s, z[nm + "_s"]), nm
        if z[nm + "_zp"].size:
            assert np.array_equal(zp, z[nm + "_zp"]), nm
    q4 = np.load(f"{GOLDEN}/quantize_w4g128.npz")
    packed, s, zp = gpu_quantize(q4["w"], 4, 128, 0.999)
    assert np.array_equal(packed.reshape(-1), q4["packed"].reshape(-1))
    assert np.array_equal(s, q4["s"]) and np.array_equal(zp, q4["zp"])


@pytest.mark.parametrize("n,k,bits,block,pct", [(64, 4096, 4, 128, 0.999), (48, 4096, 4, 32, 0.999),
                                                (32, 5120, 3, 0, 0.999), (16, 25600, 3, 0, 0.999),
                                                (24, 4096, 2, 0, 0.995), (20, 3000, 4, 0, 0.96),
                                                (12, 12288, 4, 96, 1.0)])
def test_quantize_matches_oracle_at_model_shapes(n, k, bits, block, pct):
    rng = np.random.default_rng(n + k + bits + block)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[1, 7] = 0.4
    w[2, :] = 0.0            # a constant row: span floored at 1e-8
    packed, s, zp = gpu_quantize(w, bits, block, pct)
    rp, rs, rz = O.quantize_rowwise(w, bits, block, pct)
    assert np.array_equal(packed, rp)
    assert np.array_equal(s, rs)
    assert np.array_equal(zp, rz)


def test_quantize_rejects_bad_arguments():
    torch = torch_cuda()
    w = torch.zeros((4, 100), device="cuda")
    out = torch.zeros(400, dtype=torch.uint8, device="cuda")
    s = torch.zeros(16, device="cuda")
    for bits, block in ((5, 32), (4, 40), (1, 0)):
        rc = V.lib.vspec_b200_quantize_rowwise(w.data_ptr(), 4, 100, bits, block, ctypes.c_double(0.999),
                                               out.data_ptr(), s.data_ptr(), None, None)
        assert rc == 1   # VSPEC_B200_ERR_ARG
