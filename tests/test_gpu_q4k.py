"""Q4_K dequant-matmul on the GPU against the oracle, which is
pinned bit for bit to the reference's vspec_q4k_matmul_ref_f32
(src/quant/formats/q4_k.c:41-134), through the C ABI."""
import numpy as np
import pytest

import oracle as O
import vspec_b200 as V
from gpu_util import RTOL_F32, empty_dev, rel_err, to_dev, torch_cuda

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(1, 37, 256), (1, 4096, 4096), (3, 1000, 2048), (8, 640, 1024), (11, 300, 512),
                                   (1, 12288, 4096), (2, 300, 8192), (1, 33, 8192),
                                   (1, 1, 4096), (1, 4097, 2048)])
def test_q4k_linear_matches_oracle(m, n, k):
    torch = torch_cuda()
    rng = np.random.default_rng(m * 1000 + n + k)
    blk = O.random_q4k_blocks(rng, n, k)
    blk[0, 0, 0:2] = [0, 0]            # d = 0
    if n > 1:
        blk[1, 0, 0:2] = [1, 0]        # subnormal d
    x = rng.standard_normal((m, k)).astype(np.float32)
    dx, db = to_dev(x), to_dev(blk)
    dy = empty_dev((m, n), torch.float32)
    V.q4k_linear(dx.data_ptr(), db.data_ptr(), dy.data_ptr(), m, n, k)
    torch.cuda.synchronize()
    ref = O.q4k_matmul(x, blk, n, k)
    err = rel_err(dy.cpu().numpy(), ref)
    print(f"q4k m={m} n={n} k={k}: {err:.2e}")
    assert err <= RTOL_F32


def test_q4k_linear_rejects_bad_k():
    torch = torch_cuda()
    z = torch.zeros(1024, dtype=torch.float32, device="cuda")
    with pytest.raises(V.VspecB200Error, match="multiple of 256"):
        V.q4k_linear(z.data_ptr(), z.data_ptr(), z.data_ptr(), 1, 4, 200)
