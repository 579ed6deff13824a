"""GPU: ab2_q8_gemv_noalloc (scratch in the library's fixed device array) gives the results of
ab2_q8_gemv on the same inputs, on two calls in a row, and rejects batches and shapes whose
scratch does not fit. Collected last so that it also runs after every other GPU test."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-5  # max|diff| <= TOL * max|y| per batch row, the tolerance of the mma.sync path


def blocks_for(rng, m, n):
    nb = m * n // 32
    b = np.empty((nb, 34), dtype=np.uint8)
    b[:, 2:] = rng.integers(-127, 128, size=(nb, 32)).astype(np.int8).view(np.uint8)
    b[:, :2] = np.abs(rng.normal(0, 0.01, size=nb)).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def row_close(got, ref):
    for g, r in zip(got, ref):
        scale = max(float(np.max(np.abs(r))), 1e-30)
        assert float(np.max(np.abs(g.astype(np.float64) - r))) <= TOL * scale


@pytest.mark.parametrize("m,n,batch", [(2048, 6144, 8), (6144, 2048, 3), (4096, 2048, 1), (100, 96, 5),
                                       (16, 131072, 1)])
def test_noalloc_matches_q8_gemv_twice(pkg, cuda, m, n, batch):
    torch = cuda
    rng = np.random.default_rng(m * 7 + n + batch)
    w = pkg.Q8Tensor(blocks_for(rng, m, n), m, n)
    st = torch.cuda.Stream()
    for call in range(2):
        x = torch.from_numpy(rng.normal(size=(batch, n)).astype(np.float32)).cuda()
        y_na = torch.full((batch, m), float("nan"), dtype=torch.float32, device="cuda")
        y_ref = torch.empty((batch, m), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        pkg.q8_gemv_noalloc(w, x, y_na, batch, st)   # first: before the allocating entry point
        st.synchronize()
        pkg.q8_gemv(w, x, y_ref, batch, st)
        st.synchronize()
        got, ref = y_na.cpu().numpy(), y_ref.cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all(), f"call {call}: unwritten outputs"
        row_close(got, ref)


def test_noalloc_allocates_nothing(pkg, cuda):
    """After a device's first call (the one-time address lookup of the fixed array, and the
    first load of the kernels), a call on a shape never seen before leaves the device's free
    memory exactly as it was."""
    torch = cuda
    rng = np.random.default_rng(11)
    st = torch.cuda.Stream()
    warm = pkg.Q8Tensor(blocks_for(rng, 64, 256), 64, 256)
    xw = torch.zeros((7, 256), dtype=torch.float32, device="cuda")
    yw = torch.zeros((7, 64), dtype=torch.float32, device="cuda")
    m, n = 3008, 4096
    w = pkg.Q8Tensor(blocks_for(rng, m, n), m, n)
    x = torch.from_numpy(rng.normal(size=(7, n)).astype(np.float32)).cuda()
    y = torch.empty((7, m), dtype=torch.float32, device="cuda")
    pkg.q8_gemv_noalloc(warm, xw, yw, 7, st)
    st.synchronize()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    pkg.q8_gemv_noalloc(w, x, y, 7, st)
    st.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, (free0, free1)
    ref = torch.empty_like(y)
    pkg.q8_gemv(w, x, ref, 7, st)
    st.synchronize()
    row_close(y.cpu().numpy(), ref.cpu().numpy().astype(np.float64))


def test_noalloc_keeps_the_callers_device(pkg, cuda):
    """A call for a tensor on device 0 from a thread whose current device is 1 leaves the
    thread's current device at 1."""
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    rng = np.random.default_rng(12)
    w = pkg.Q8Tensor(blocks_for(rng, 256, 512), 256, 512)  # device 0
    x = torch.zeros((2, 512), dtype=torch.float32, device="cuda:0")
    y = torch.zeros((2, 256), dtype=torch.float32, device="cuda:0")
    prev = torch.cuda.current_device()
    try:
        torch.cuda.set_device(1)
        pkg.q8_gemv_noalloc(w, x, y, 2)
        assert torch.cuda.current_device() == 1
        pkg.q8_gemv(w, x, y, 2)
        assert torch.cuda.current_device() == 1
    finally:
        torch.cuda.set_device(prev)
    torch.cuda.synchronize(0)


def test_noalloc_rejects_what_does_not_fit(pkg, cuda):
    torch = cuda
    rng = np.random.default_rng(3)
    w = pkg.Q8Tensor(blocks_for(rng, 64, 256), 64, 256)
    x = torch.zeros((9, 256), dtype=torch.float32, device="cuda")
    y = torch.zeros((9, 64), dtype=torch.float32, device="cuda")
    with pytest.raises(pkg.Ab2Error) as e:
        pkg.q8_gemv_noalloc(w, x, y, 9)
    assert e.value.code == -6 and "batch 9" in str(e.value)
    big = pkg.Q8Tensor(blocks_for(rng, 16, 131072), 16, 131072)   # 4 MiB of activations at batch 8
    xb = torch.zeros((8, 131072), dtype=torch.float32, device="cuda")
    yb = torch.zeros((8, 16), dtype=torch.float32, device="cuda")
    with pytest.raises(pkg.Ab2Error) as e:
        pkg.q8_gemv_noalloc(big, xb, yb, 8)
    assert e.value.code == -6 and "scratch" in str(e.value)
    torch.cuda.synchronize()
