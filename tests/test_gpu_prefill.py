"""GPU: prefill of a prompt (ab2_prefill: steps of up to 128 tokens, the DeltaNet recurrence in
its chunkwise form over 64 tokens at a time, each token's attention over the slot's cache)
against the oracle's token-by-token qwen35_forward_token, the reference's own prompt loop
(crates/cli/src/main.rs:358-362).

In a context with exact_max_batch = 64 (EXACT below) a prefill step is 64 rows on the
exact-weight path. There the prefill and the oracle differ only in the order of f32 sums
(the 64-row GEMM's K order, the chunkwise recurrence), so the last token's logits and every
state agree to PREFILL_TOL. In a default context a step is 128 rows on the tcgen05 path (its
N = 128 form), whose GEMM operands are rounded to f16, and the decode parity bar applies."""
import numpy as np
import pytest

from conftest import argmax_consistent, rel_err

pytestmark = pytest.mark.gpu

PREFILL_TOL = 1e-4   # max|d| <= PREFILL_TOL * max|ref|: logits and recurrent / conv state
KV_TOL = 1e-2        # bf16 cache entries (one bf16 ulp is 2^-8 relative)
LOGIT_TOL = 1e-2     # tcgen05 path (f16 operands), the decode parity bar
# tcgen05 path, recurrent state after hundreds of tokens: the state integrates every token's
# f16-rounded projections, so it drifts further from the exact path than the logits do
TC_STATE_TOL = 5e-2
EXACT = 64           # exact_max_batch that keeps a 64-row prefill chunk on the exact path


def _oracle_run(model, tokens, seq=None):
    seq = seq or model.new_seq(kv_bf16=True)
    lo = None
    for t in tokens:
        lo = seq.forward(int(t))
    return seq, lo


def _check_states(ctx, seq, n, layers_dn, tol=PREFILL_TOL, slot=0):
    for l, dn in enumerate(layers_dn):
        if dn:
            rec, conv = ctx.get_dn_state(l, slot)
            rr, cr = seq.get_dn(l)
            assert rel_err(rec, rr) < tol, (l, rel_err(rec, rr))
            assert rel_err(conv, cr) < tol, (l, rel_err(conv, cr))
        else:
            k, v = ctx.get_kv(l, slot, n)
            kr, vr = seq.get_kv(l, n)
            assert rel_err(k, kr) < KV_TOL and rel_err(v, vr) < KV_TOL, l


@pytest.mark.parametrize("n", [1, 63, 64, 65, 150])
def test_prefill_tiny_matches_oracle(pkg, oracle, synth, tiny_gguf, tiny_model, n):
    """Prompt lengths around the chunk size: the last token's logits and argmax, the position,
    and every DeltaNet, conv and KV state equal the oracle's after the same prompt; then 16
    greedy decode steps from the prefilled state follow the oracle's."""
    prompt = synth.seeded_tokens(n, 32000, seed=40 + n)
    with pkg.DecodeContext(tiny_gguf, max_batch=1, max_ctx=n + 24, kv_bf16=True, exact_max_batch=EXACT) as ctx:
        lg, nx = ctx.prefill(0, prompt)
        seq, lo = _oracle_run(tiny_model, prompt)
        err = rel_err(lg, lo)
        print(f"n={n}: last-token logit rel err {err:.2e}")
        assert err < PREFILL_TOL
        assert nx == oracle.greedy(lg) and argmax_consistent(nx, lo, lg)
        assert ctx.get_pos(0) == n and seq.pos == n
        _check_states(ctx, seq, n, ctx.layer_is_deltanet)
        tg = to = nx
        for i in range(16):
            lgd, nxd = ctx.decode_step([tg])
            lod = seq.forward(to)
            assert rel_err(lgd[0], lod) < PREFILL_TOL, (i, rel_err(lgd[0], lod))
            tg, to = int(nxd[0]), oracle.greedy(lod)
            assert argmax_consistent(tg, lod, lgd[0]), i
            if tg != to:
                break  # a near tie: the two continuations are no longer comparable


def test_prefill_continues_a_sequence(pkg, oracle, synth, tiny_gguf, tiny_model):
    """Decode 5 tokens, then prefill 70 more from position 5 (a chunk that starts mid-sequence
    and crosses the 64-token boundary), then prefill 3 more."""
    toks = synth.seeded_tokens(78, 32000, seed=7)
    with pkg.DecodeContext(tiny_gguf, max_batch=1, max_ctx=96, kv_bf16=True, exact_max_batch=EXACT) as ctx:
        for t in toks[:5]:
            ctx.decode_step([int(t)])
        ctx.prefill(0, toks[5:75])
        lg, nx = ctx.prefill(0, toks[75:])
        seq, lo = _oracle_run(tiny_model, toks)
        assert rel_err(lg, lo) < PREFILL_TOL
        assert ctx.get_pos(0) == 78
        _check_states(ctx, seq, 78, ctx.layer_is_deltanet)


def test_prefill_matches_stepwise_decode(pkg, synth, tiny_gguf):
    """Prefill of slot 1 against one decode step per token of the same prompt in slot 0 of
    the same context: the same logits to PREFILL_TOL, and slot 1's prefill leaves slot 0 alone."""
    prompt = synth.seeded_tokens(100, 32000, seed=3)
    with pkg.DecodeContext(tiny_gguf, max_batch=2, max_ctx=128, kv_bf16=True, exact_max_batch=EXACT) as ctx:
        lg1, _ = ctx.prefill(1, prompt)
        assert ctx.get_pos(0) == 0
        assert not ctx.get_dn_state(0, 0)[0].any()
        for t in prompt:
            lg0, _ = ctx.decode_step([int(t)])
        assert rel_err(lg1, lg0[0]) < PREFILL_TOL
        for l, dn in enumerate(ctx.layer_is_deltanet):
            if dn:
                assert rel_err(ctx.get_dn_state(l, 1)[0], ctx.get_dn_state(l, 0)[0]) < PREFILL_TOL


def test_prefill_tensor_core_path(pkg, oracle, synth, tiny_gguf, tiny_model):
    """A default context prefills on the tcgen05 GEMM, even with max_batch 1: a 128-row step
    (the GEMM's N = 128 form, the DeltaNet mixer as two 64-token launches) and a 2-row step,
    within the decode parity bar of the oracle."""
    prompt = synth.seeded_tokens(130, 32000, seed=11)
    with pkg.DecodeContext(tiny_gguf, max_batch=1, max_ctx=140, kv_bf16=True) as ctx:
        assert ctx.tensor_core_gemm(64)
        lg, nx = ctx.prefill(0, prompt)
        seq, lo = _oracle_run(tiny_model, prompt)
        err = rel_err(lg, lo)
        print(f"tcgen05 prefill: last-token logit rel err {err:.2e}")
        assert err < LOGIT_TOL
        _check_states(ctx, seq, 130, ctx.layer_is_deltanet, tol=LOGIT_TOL)


def test_prefill_2b_matches_oracle(pkg, oracle, synth):
    """The 2B shape (16 DeltaNet heads, hd-256 attention): 70 prompt tokens (two chunks)."""
    gguf = synth.build_model_gguf(synth.shape_2b(), seed=0)
    prompt = synth.seeded_tokens(70, 151936, seed=5)
    with pkg.DecodeContext(gguf, max_batch=1, max_ctx=80, kv_bf16=True, exact_max_batch=EXACT) as ctx:
        lg, nx = ctx.prefill(0, prompt)
        model = oracle.Model(gguf, ctx_cap=80)
        seq, lo = _oracle_run(model, prompt)
        err = rel_err(lg, lo)
        print(f"2B prefill: last-token logit rel err {err:.2e}")
        assert err < PREFILL_TOL
        assert argmax_consistent(nx, lo, lg)
        _check_states(ctx, seq, 70, ctx.layer_is_deltanet)


def test_prefill_2b_tensor_core_path(pkg, oracle, synth):
    """The 2B shape in a default context: 70 prompt tokens as one 70-row step of the N = 128
    tcgen05 GEMM (rows 70..127 of its operand are padding), then 8 greedy decode steps, all
    within the decode parity bar of the oracle's token-by-token forward."""
    gguf = synth.build_model_gguf(synth.shape_2b(), seed=0)
    prompt = synth.seeded_tokens(70, 151936, seed=6)
    with pkg.DecodeContext(gguf, max_batch=1, max_ctx=90, kv_bf16=True) as ctx:
        lg, nx = ctx.prefill(0, prompt)
        model = oracle.Model(gguf, ctx_cap=90)
        seq, lo = _oracle_run(model, prompt)
        err = rel_err(lg, lo)
        print(f"2B tcgen05 prefill: last-token logit rel err {err:.2e}")
        assert err < LOGIT_TOL
        assert argmax_consistent(nx, lo, lg)
        _check_states(ctx, seq, 70, ctx.layer_is_deltanet, tol=LOGIT_TOL)
        t = nx
        for i in range(8):
            lgd, nxd = ctx.decode_step([t])
            lod = seq.forward(t)  # the GPU's token on both sides: a near tie cannot part them
            assert rel_err(lgd[0], lod) < LOGIT_TOL, (i, rel_err(lgd[0], lod))
            t = int(nxd[0])


@pytest.mark.parametrize("exact", [True, False])
def test_prefill_2b_long_matches_stepwise(pkg, synth, exact):
    """The 2B shape (hd-256 attention), 600 prompt tokens: from the third step on, each query
    block's prefix spans several splits, so the prefill attention kernel's split partials and
    their merge run at hd 256. Against one decode step per token in a second context: the
    last logits and every state. On the exact path both sides keep exact weights, so they
    agree to PREFILL_TOL; a default context prefills on the tcgen05 GEMM (f16 operands) and
    its one-sequence decode steps stay exact, so there the decode parity bar applies to the
    logits (the recurrent state, integrated over 600 tokens, to TC_STATE_TOL)."""
    gguf = synth.build_model_gguf(synth.shape_2b(), seed=0)
    prompt = synth.seeded_tokens(600, 151936, seed=12)
    kw = dict(max_batch=1, max_ctx=640, kv_bf16=True, exact_max_batch=EXACT if exact else 0)
    with pkg.DecodeContext(gguf, **kw) as a, pkg.DecodeContext(gguf, **kw) as b:
        lg_a, _ = a.prefill(0, prompt)
        for t in prompt:
            lg_b, _ = b.decode_step([int(t)])
        tol = PREFILL_TOL if exact else LOGIT_TOL
        err = rel_err(lg_a, lg_b[0])
        print(f"2B 600-token prefill against stepwise decode (exact={exact}): logit rel err {err:.2e}")
        assert err < tol
        assert a.get_pos(0) == b.get_pos(0) == 600
        state_tol = PREFILL_TOL if exact else TC_STATE_TOL
        worst = 0.0
        for l, dn in enumerate(a.layer_is_deltanet):
            if dn:
                e = rel_err(a.get_dn_state(l, 0)[0], b.get_dn_state(l, 0)[0])
                worst = max(worst, e)
                assert e < state_tol, (l, e)
            else:
                ka, va = a.get_kv(l, 0, 600)
                kb, vb = b.get_kv(l, 0, 600)
                assert rel_err(ka, kb) < KV_TOL and rel_err(va, vb) < KV_TOL, l
        print(f"  worst recurrent-state rel err {worst:.2e}")


def test_prefill_rejects_bad_requests(pkg, synth, tiny_gguf):
    with pkg.DecodeContext(tiny_gguf, max_batch=1, max_ctx=32, kv_bf16=True) as ctx:
        with pytest.raises(pkg.Ab2Error) as ei:
            ctx.prefill(0, synth.seeded_tokens(33, 32000))
        assert ei.value.code == -6
        with pytest.raises(pkg.Ab2Error) as ei:
            ctx.prefill(0, np.array([1, 32000], dtype=np.int32))
        assert ei.value.code == -1
        with pytest.raises(pkg.Ab2Error) as ei:
            ctx.prefill(0, np.zeros(0, dtype=np.int32))
        assert ei.value.code == -1
        with pytest.raises(pkg.Ab2Error) as ei:
            ctx.prefill(1, [1, 2])
        assert ei.value.code == -1
        assert ctx.get_pos(0) == 0  # nothing ran
    with pkg.DecodeContext(tiny_gguf, max_batch=1, max_ctx=32, kv_bf16=False) as ctx:
        with pytest.raises(pkg.Ab2Error) as ei:
            ctx.prefill(0, [1, 2])
        assert ei.value.code == -3


def test_prefill_long_prompt_split_attention(pkg, oracle, synth, tiny_gguf, tiny_model):
    """A 700-token prompt (11 chunks): from the fourth chunk on, the tokens' attention spans
    more than one split of the slot's cache, so the per-token split partials and their merge
    run on the shared slot too."""
    prompt = synth.seeded_tokens(700, 32000, seed=77)
    with pkg.DecodeContext(tiny_gguf, max_batch=1, max_ctx=720, kv_bf16=True, exact_max_batch=EXACT) as ctx:
        lg, nx = ctx.prefill(0, prompt)
        seq, lo = _oracle_run(tiny_model, prompt)
        err = rel_err(lg, lo)
        print(f"700-token prefill: last-token logit rel err {err:.2e}")
        assert err < PREFILL_TOL
        assert argmax_consistent(nx, lo, lg)
        _check_states(ctx, seq, 700, ctx.layer_is_deltanet)


@pytest.mark.parametrize("exact", [True, False])
def test_prefill_after_long_seeded_context(pkg, synth, tiny_gguf, exact):
    """Slots seeded with 2000 tokens of state, then 100 more tokens: prefill in one context
    against one decode step per token in another context with the same seeded state. The
    attention of every prompt token reads the long seeded prefix through several splits."""
    prompt = synth.seeded_tokens(100, 32000, seed=8)
    kw = dict(max_batch=1, max_ctx=2112, kv_bf16=True, exact_max_batch=EXACT if exact else 0)
    with pkg.DecodeContext(tiny_gguf, **kw) as a, pkg.DecodeContext(tiny_gguf, **kw) as b:
        for ctx in (a, b):
            ctx.seed_state(seed=3, n_slots=1, n_tokens=2000)
        lg_a, _ = a.prefill(0, prompt)
        for t in prompt:
            lg_b, _ = b.decode_step([int(t)])
        tol = PREFILL_TOL if exact else LOGIT_TOL
        assert rel_err(lg_a, lg_b[0]) < tol
        assert a.get_pos(0) == b.get_pos(0) == 2100
        for l, dn in enumerate(a.layer_is_deltanet):
            if dn:
                assert rel_err(a.get_dn_state(l, 0)[0], b.get_dn_state(l, 0)[0]) < tol
            else:
                ka, va = a.get_kv(l, 0, 2100)
                kb, vb = b.get_kv(l, 0, 2100)
                assert rel_err(ka, kb) < KV_TOL and rel_err(va, vb) < KV_TOL
