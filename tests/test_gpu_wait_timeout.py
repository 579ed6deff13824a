"""GPU: the bounded waits of the pipelined kernels expire cleanly. A test hook arms one launch
to leave one of its asynchronous copies unissued with a 5 ms wait limit (nothing faults: the
mbarrier phase the kernel waits on simply never completes). The kernel must report its error
bit, drain the copies it did issue, free its tensor memory and return, and the next normal
launch must give exactly the results of a launch before the failure."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WAIT_NS = 5_000_000  # 5 ms instead of the production 2 s


@pytest.fixture(autouse=True)
def disarm(pkg):
    """An arm that a failing test did not consume must not reach a later test's launch."""
    yield
    for which in (1, 2, 3):
        pkg.debug_arm_wait_timeout(which, 0, 0)


def test_gemm_weight_copy_timeout(pkg, synth, cuda):
    # an lm_head-like shape with whole-K units (no K split), so normal launches are
    # bit-identical; each CTA's third weight stage is withheld, after two stages went through
    torch = cuda
    m, n, batch = 32000, 1024, 9
    rng = np.random.default_rng(31)
    w = pkg.Q8Tensor(synth.random_q8_0(rng, m, n), m, n)
    x = torch.from_numpy(rng.normal(0, 1, size=(batch, n)).astype(np.float32)).cuda()
    y0 = torch.empty((batch, m), dtype=torch.float32, device="cuda")
    y1 = torch.empty_like(y0)
    assert pkg.op_error() == 0
    pkg.q8_gemv(w, x, y0, batch)
    assert pkg.op_error() == 0
    pkg.debug_arm_wait_timeout(pkg.WAIT_TEST_GEMM, 2, WAIT_NS)
    pkg.q8_gemv(w, x, y1, batch)
    code = pkg.op_error()
    print(f"GEMM error word 0x{code:x}")
    assert code & 128, hex(code)            # the converters' wait for the weight stage
    pkg.q8_gemv(w, x, y1, batch)            # the hook was consumed: a normal launch
    assert pkg.op_error() == 0
    assert torch.equal(y1, y0)


def _attn_inputs(torch, B, ctx, cap, Hq=8, Hkv=2, hd=256):
    g = torch.Generator(device="cuda").manual_seed(5)
    proj = torch.randn(B, Hq * 2 * hd + 2 * Hkv * hd, device="cuda", generator=g)
    kd = torch.randn(B, Hkv, cap, hd, device="cuda", generator=g).to(torch.bfloat16)
    vd = torch.randn(B, Hkv, cap, hd, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.full((B,), ctx - 1, dtype=torch.int32, device="cuda")
    return proj, kd, vd, pos


def test_attention_tile_copy_timeout(pkg, cuda):
    # every CTA's first K/V tile is withheld; appending the new K/V at the same position again
    # writes the same values, so the call can be repeated on the same caches
    torch = cuda
    B, ctx, Hq, Hkv, hd = 4, 2048, 8, 2, 256
    cap = ctx + 8
    proj, kd, vd, pos = _attn_inputs(torch, B, ctx, cap)
    out0 = torch.empty((B, Hq * hd), dtype=torch.float32, device="cuda")
    out1 = torch.empty_like(out0)
    args = (kd, vd, cap, pos, B, Hq, Hkv, hd, True, None, None, 1e7, 64, ctx - 1)
    assert pkg.op_error() == 0
    pkg.attn_decode(proj, *args, out0)
    assert pkg.op_error() == 0
    pkg.debug_arm_wait_timeout(pkg.WAIT_TEST_ATTENTION, 0, WAIT_NS)
    pkg.attn_decode(proj, *args, out1)
    code = pkg.op_error()
    print(f"attention error word 0x{code:x}")
    assert code & 4096, hex(code)
    pkg.attn_decode(proj, *args, out1)
    assert pkg.op_error() == 0
    assert torch.equal(out1, out0)


def test_deltanet_state_copy_timeout(pkg, tiny_gguf, cuda):
    # through the decode step (the DeltaNet kernel runs inside it): the first state copy of
    # every CTA is withheld in the first DeltaNet layer of the step; the step reports the
    # timeout, and after re-seeding the same state a normal step gives the reference logits
    # (B=2 on the exact mma.sync GEMM path, exact_max_batch=2, so the step is deterministic)
    torch = cuda
    B, n_tok = 2, 40
    ctx = pkg.DecodeContext(tiny_gguf, max_batch=B, max_ctx=64, kv_bf16=True, exact_max_batch=2)
    ctx.seed_state(seed=3, n_slots=B, n_tokens=n_tok, dn_std=0.1, conv_std=1.0, kv_std=1.0)
    ref, _ = ctx.decode_step([5, 77])
    ctx.seed_state(seed=3, n_slots=B, n_tokens=n_tok, dn_std=0.1, conv_std=1.0, kv_std=1.0)
    pkg.debug_arm_wait_timeout(pkg.WAIT_TEST_DELTANET, 0, WAIT_NS)
    with pytest.raises(pkg.Ab2Error) as ei:
        ctx.decode_step([5, 77])
    msg = str(ei.value)
    print(msg)
    assert "timed out" in msg and int(msg.split("0x")[1].split(")")[0], 16) & 1024
    ctx.seed_state(seed=3, n_slots=B, n_tokens=n_tok, dn_std=0.1, conv_std=1.0, kv_std=1.0)
    again, _ = ctx.decode_step([5, 77])
    assert np.array_equal(again, ref)
    ctx.close()


def test_attention_timeout_through_the_step(pkg, tiny_gguf, cuda):
    # the same through the decode step's attention layer (tensor-core kernel, bf16 KV)
    B, n_tok = 2, 300
    ctx = pkg.DecodeContext(tiny_gguf, max_batch=B, max_ctx=400, kv_bf16=True, exact_max_batch=2)
    ctx.seed_state(seed=4, n_slots=B, n_tokens=n_tok, dn_std=0.1, conv_std=1.0, kv_std=1.0)
    ref, _ = ctx.decode_step([9, 11])
    ctx.seed_state(seed=4, n_slots=B, n_tokens=n_tok, dn_std=0.1, conv_std=1.0, kv_std=1.0)
    pkg.debug_arm_wait_timeout(pkg.WAIT_TEST_ATTENTION, 1, WAIT_NS)
    with pytest.raises(pkg.Ab2Error) as ei:
        ctx.decode_step([9, 11])
    assert int(str(ei.value).split("0x")[1].split(")")[0], 16) & 4096
    ctx.seed_state(seed=4, n_slots=B, n_tokens=n_tok, dn_std=0.1, conv_std=1.0, kv_std=1.0)
    again, _ = ctx.decode_step([9, 11])
    assert np.array_equal(again, ref)
    ctx.close()

