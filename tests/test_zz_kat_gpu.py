"""The reference's identity GEMV known answer on the B200, through both GEMM paths:
make_q8_identity(4, 32) with x = 0..31 gives y[i] = i. The reference checks it on its CPU
GEMV (crates/engine/src/q8_gemv.rs:257-281) and on its Metal GEMV
(crates/engine/src/metal_graph.rs:559-598, within 0.01). Every partial sum here is an exact
small integer, so the bar is exact equality."""
import numpy as np
import pytest

from test_oracle_golden import kat_blocks_ident, kats

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [1, 8, 9, 64])
def test_identity_gemv_kat_exact(pkg, cuda, batch):
    torch = cuda
    blocks, x = kat_blocks_ident()
    k = kats()["q8_gemv_ident"]
    w = pkg.Q8Tensor.from_raw(blocks, k["n"], k["m"])
    xd = torch.from_numpy(np.tile(x, (batch, 1))).cuda()
    y = torch.full((batch, k["m"]), -1.0, dtype=torch.float32, device="cuda")
    pkg.q8_gemv(w, xd, y, batch)
    torch.cuda.synchronize()
    exp = np.array(k["expected"], dtype=np.float32)
    for b in range(batch):
        assert np.array_equal(y[b].cpu().numpy(), exp), b
    assert pkg.op_error() == 0
