"""GPU parity of the Q8_0 kernels against the oracle: dequant bit-exact, repack round trip
bit-exact, GEMV/GEMM on the reference KAT (exact) and on the config-4 shapes (tolerance)."""
import numpy as np
import pytest

from conftest import rel_err
from test_oracle_golden import kat_blocks_par, kats

pytestmark = pytest.mark.gpu

# the GEMV/GEMM result tolerance: max|diff| <= tol * max|y_ref| per batch row.
# Batches <= 8 (mma.sync path) keep the weights exact and the activations as an f16 hi/lo
# pair; batches >= 9 (tcgen05 path) round each weight q*d and each activation to f16 once.
TOL = 1e-5
TC_TOL = 3e-3


def tol(batch):
    return TOL if batch <= 8 else TC_TOL


def random_blocks(rng, nb, with_specials=True):
    b = np.empty((nb, 34), dtype=np.uint8)
    b[:, 2:] = rng.integers(-128, 128, size=(nb, 32)).astype(np.int8).view(np.uint8)
    d = np.abs(rng.normal(0, 0.01, size=nb)).astype(np.float16)
    if with_specials and nb >= 4:
        d[0] = 0
        d[1] = np.float16(-0.5)
        d[2] = np.float16(6e-8)     # subnormal
        d[3] = np.float16(65504)    # max finite
    b[:, :2] = d.view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def test_dequant_raw_bit_exact(pkg, oracle, cuda):
    torch = cuda
    rng = np.random.default_rng(1)
    blocks = random_blocks(rng, 4099)
    ref = oracle.q8_dequant(blocks)
    dev = torch.from_numpy(blocks).cuda()
    out = torch.empty(ref.size, dtype=torch.float32, device="cuda")
    pkg.q8_dequant(dev, 4099, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("m,n", [(100, 96), (16, 32), (1, 64), (6144, 2048)])
def test_repack_round_trip_bit_exact(pkg, oracle, cuda, m, n):
    torch = cuda
    rng = np.random.default_rng(m + n)
    blocks = random_blocks(rng, m * n // 32)
    w = pkg.Q8Tensor(blocks, m, n)
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    w.unpack(out)
    torch.cuda.synchronize()
    ref = oracle.q8_dequant(blocks).reshape(m, n)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("batch", [1, 3, 8, 9, 16, 32, 64])
def test_gemv_reference_kat_exact(pkg, cuda, batch):
    # q8_gemv.rs:283-314 inputs; every partial sum is an exact integer so the result is exact
    torch = cuda
    blocks, x = kat_blocks_par()
    w = pkg.Q8Tensor.from_raw(blocks, 1024, 256)
    xd = torch.from_numpy(np.tile(x, (batch, 1))).cuda()
    y = torch.empty((batch, 256), dtype=torch.float32, device="cuda")
    pkg.q8_gemv(w, xd, y, batch)
    torch.cuda.synchronize()
    exp = np.array(kats()["q8_gemv_par"]["expected"], dtype=np.float32)
    for b in range(batch):
        assert np.array_equal(y[b].cpu().numpy(), exp), b
    assert pkg.op_error() == 0


SHAPES = [(6144, 2048), (2048, 6144), (4096, 2048), (151936, 2048), (16, 2048), (8224, 2048)]


@pytest.mark.parametrize("m,n", SHAPES)
@pytest.mark.parametrize("batch", [1, 32])
def test_gemv_matches_oracle(pkg, oracle, synth, cuda, m, n, batch):
    torch = cuda
    rng = np.random.default_rng(m * 7 + n + batch)
    blocks = synth.random_q8_0(rng, m, n, std=0.02)
    w = pkg.Q8Tensor(blocks, m, n)
    x = rng.normal(0, 1, size=(batch, n)).astype(np.float32)
    x = synth.bf16_round(x)          # config 4 activations are bf16 N(0,1)
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    pkg.q8_gemv(w, torch.from_numpy(x).cuda(), y, batch)
    torch.cuda.synchronize()
    yg = y.cpu().numpy()
    rows = range(batch) if batch <= 4 else (0, batch // 2, batch - 1)
    for b in rows:
        ref = oracle.q8_gemv(blocks, m, n, x[b])
        assert rel_err(yg[b], ref) < tol(batch), (b, rel_err(yg[b], ref))
    assert pkg.op_error() == 0


# the tcgen05 path against the oracle's GEMV with the same declared operand rounding (weights
# q*d and inputs rounded once to f16, f32 sums): only the f32 summation order differs
TC_DECLARED_TOL = 2e-5


@pytest.mark.parametrize("m,n", SHAPES)
@pytest.mark.parametrize("batch", [9, 32, 64, 65, 128])  # 65 and 128: the N = 128 form
def test_tc_gemm_matches_declared_rounding(pkg, oracle, synth, cuda, m, n, batch):
    torch = cuda
    rng = np.random.default_rng(m * 3 + n + batch)
    blocks = synth.random_q8_0(rng, m, n, std=0.02)
    w = pkg.Q8Tensor(blocks, m, n)
    x = rng.normal(0, 1, size=(batch, n)).astype(np.float32)
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    pkg.q8_gemv(w, torch.from_numpy(x).cuda(), y, batch)
    torch.cuda.synchronize()
    yg = y.cpu().numpy()
    for b in (0, batch // 2, batch - 1):
        ref = oracle.q8_gemv(blocks, m, n, x[b], f16_operands=True)
        exact = oracle.q8_gemv(blocks, m, n, x[b])
        assert rel_err(yg[b], ref) < TC_DECLARED_TOL, (b, rel_err(yg[b], ref))
        assert rel_err(yg[b], exact) < TC_TOL, (b, rel_err(yg[b], exact))
    assert pkg.op_error() == 0


@pytest.mark.parametrize("batch", [2, 4, 5, 9, 16, 33, 64])
def test_gemm_all_batch_modes(pkg, oracle, synth, cuda, batch):
    torch = cuda
    m, n = 2080, 1024
    rng = np.random.default_rng(batch)
    blocks = synth.random_q8_0(rng, m, n)
    w = pkg.Q8Tensor(blocks, m, n)
    x = rng.normal(0, 1, size=(batch, n)).astype(np.float32)
    y = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    pkg.q8_gemv(w, torch.from_numpy(x).cuda(), y, batch)
    torch.cuda.synchronize()
    yg = y.cpu().numpy()
    W = synth.dequant_q8_0(blocks).reshape(m, n).astype(np.float64)
    ref = x.astype(np.float64) @ W.T
    for b in range(batch):
        assert rel_err(yg[b], ref[b]) < tol(batch), (b, rel_err(yg[b], ref[b]))
    assert pkg.op_error() == 0


def test_gemm_repeated_launches_identical(pkg, oracle, synth, cuda):
    # an lm_head-like shape whose units are never K-split (one unit per CTA, 16 pipeline
    # stages, no reductions), so every launch must give bit-identical outputs; repeating it
    # exposes shared-memory stage hand-off races that only show up on some launches
    torch = cuda
    m, n, batch = 32000, 1024, 9
    rng = np.random.default_rng(21)
    blocks = synth.random_q8_0(rng, m, n)
    w = pkg.Q8Tensor(blocks, m, n)
    x = torch.from_numpy(rng.normal(0, 1, size=(batch, n)).astype(np.float32)).cuda()
    ys = [torch.empty((batch, m), dtype=torch.float32, device="cuda") for _ in range(2)]
    pkg.q8_gemv(w, x, ys[0], batch)
    torch.cuda.synchronize()
    first = ys[0].cpu().numpy()
    W = synth.dequant_q8_0(blocks).reshape(m, n).astype(np.float64)
    ref = x.cpu().numpy().astype(np.float64) @ W.T
    for b in range(batch):
        assert rel_err(first[b], ref[b]) < tol(batch), (b, rel_err(first[b], ref[b]))
    for i in range(120):
        pkg.q8_gemv(w, x, ys[1], batch)
        if i % 8 == 7:
            torch.cuda.synchronize()
            assert torch.equal(ys[1], ys[0]), i
    torch.cuda.synchronize()
    assert torch.equal(ys[1], ys[0])
    assert pkg.op_error() == 0


def test_gemv_rejects_bad_batch(pkg, synth, cuda):
    torch = cuda
    rng = np.random.default_rng(0)
    w = pkg.Q8Tensor(synth.random_q8_0(rng, 32, 64), 32, 64)
    x = torch.zeros((129, 64), device="cuda")
    y = torch.zeros((129, 32), device="cuda")
    with pytest.raises(pkg.Ab2Error) as ei:
        pkg.q8_gemv(w, x, y, 129)
    assert ei.value.code == -6
