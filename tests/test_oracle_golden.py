"""CPU: pin the C++ oracle to the reference's own known-answer tests and cross-check it
against the independent numpy restatement (tests/numpy_ref.py)."""
import json
import os

import numpy as np
import pytest

from conftest import rel_err
import numpy_ref

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_kats.json")


def kats():
    with open(GOLD) as f:
        return json.load(f)


def f16le(v: float) -> np.ndarray:
    return np.array([v], dtype=np.float16).view(np.uint8)


def kat_blocks_ident():
    # crates/engine/src/q8_gemv.rs:258-270: m=4, n=32, d=1, q[r][r] = 1
    blk = np.zeros((4, 34), dtype=np.uint8)
    for r in range(4):
        blk[r, :2] = f16le(1.0)
        blk[r, 2 + r] = 1
    return blk.reshape(-1), np.arange(32, dtype=np.float32)


def kat_blocks_par():
    # crates/engine/src/q8_gemv.rs:285-300: d = 0.5, q = ((row + i) % 256) as i8, x = i % 100
    m, n = 256, 1024
    blk = np.zeros((m, n // 32, 34), dtype=np.uint8)
    blk[:, :, :2] = f16le(0.5)
    i = np.arange(32)
    for row in range(m):
        blk[row, :, 2:] = ((row + i) % 256).astype(np.uint8)
    return blk.reshape(-1), (np.arange(n) % 100).astype(np.float32)


def test_kat_q8_0_dequant(oracle):
    k = kats()["q8_0_dequant"]
    blk = np.zeros(34, dtype=np.uint8)
    blk[:2] = f16le(k["d"])
    blk[2:] = k["q"]
    out = oracle.q8_dequant(blk)
    assert np.all(out == np.float32(k["expected"]))


def test_kat_q8_gemv_identity(oracle):
    k = kats()["q8_gemv_ident"]
    blocks, x = kat_blocks_ident()
    for scalar in (False, True):
        y = oracle.q8_gemv(blocks, 4, 32, x, scalar=scalar)
        assert np.array_equal(y, np.array(k["expected"], dtype=np.float32))


def test_kat_q8_gemv_parallel_equals_scalar(oracle):
    k = kats()["q8_gemv_par"]
    blocks, x = kat_blocks_par()
    yp = oracle.q8_gemv(blocks, 256, 1024, x)
    ys = oracle.q8_gemv(blocks, 256, 1024, x, scalar=True)
    assert np.array_equal(yp, ys)
    assert np.array_equal(yp, np.array(k["expected"], dtype=np.float32))


def test_f16_widening_is_exact(oracle):
    lib = oracle.lib()
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([lib.oracle_f16_to_f32(int(v)) for v in h[::7]], dtype=np.float32)
    r = ref[::7]
    finite = np.isfinite(r)
    assert np.array_equal(got[finite].view(np.uint32), r[finite].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(r)]))


def test_greedy_total_cmp_last_max(oracle):
    x = np.array([0.5, 2.0, -1.0, 2.0, 1.0], dtype=np.float32)
    assert oracle.greedy(x) == 3          # Iterator::max_by keeps the last maximum
    x = np.array([-0.0, 0.0, -0.0], dtype=np.float32)
    assert oracle.greedy(x) == 1          # total_cmp: +0 > -0
    x = np.array([1.0, np.nan, 3.0], dtype=np.float32)
    assert oracle.greedy(x) == 1          # positive NaN sorts above everything


def test_oracle_gemv_matches_numpy(oracle, synth):
    rng = np.random.default_rng(5)
    m, n = 96, 256
    blocks = synth.quantize_q8_0(rng.normal(0, 0.02, size=(m, n)).astype(np.float32))
    x = rng.normal(size=n).astype(np.float32)
    W = synth.dequant_q8_0(blocks).reshape(m, n).astype(np.float64)
    assert rel_err(oracle.q8_gemv(blocks, m, n, x), W @ x) < 1e-5


def test_oracle_gated_delta_matches_numpy(oracle):
    rng = np.random.default_rng(6)
    B, H = 2, 3
    S = rng.normal(0, 0.1, size=(B, H, 128, 128)).astype(np.float32)
    q = rng.normal(size=(B, H, 128)).astype(np.float32)
    k = rng.normal(size=(B, H, 128)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.normal(size=(B, H, 128)).astype(np.float32)
    beta = rng.uniform(0.1, 0.9, size=(B, H)).astype(np.float32)
    decay = rng.uniform(0.5, 1.0, size=(B, H)).astype(np.float32)
    o, S2 = oracle.gated_delta(S, q, k, v, beta, decay)
    for b in range(B):
        for h in range(H):
            on, Sn = numpy_ref.gated_delta(S[b, h].astype(np.float64), q[b, h], k[b, h], v[b, h], beta[b, h],
                                           decay[b, h])
            assert rel_err(o[b, h], on) < 1e-5
            assert rel_err(S2[b, h], Sn) < 1e-5


@pytest.mark.parametrize("rot", [128, 64])
def test_oracle_attention_matches_numpy(oracle, rot):
    rng = np.random.default_rng(7)
    Hq, Hkv, hd, cap, pos = 8, 2, 128, 40, 33
    q = rng.normal(size=(Hq, hd)).astype(np.float32)
    gate = rng.normal(size=(Hq, hd)).astype(np.float32)
    kn = rng.normal(size=(Hkv, hd)).astype(np.float32)
    vn = rng.normal(size=(Hkv, hd)).astype(np.float32)
    kc = rng.normal(size=(Hkv, cap, hd)).astype(np.float32)
    vc = rng.normal(size=(Hkv, cap, hd)).astype(np.float32)
    qn = (1 + rng.normal(0, 0.02, size=hd)).astype(np.float32)
    knw = (1 + rng.normal(0, 0.02, size=hd)).astype(np.float32)
    out, kc2, vc2 = oracle.attn_op(q, gate, kn, vn, kc, vc, pos, 1e7, rot, qn, knw)
    ref = numpy_ref.attn_core(q.astype(np.float64), gate.astype(np.float64), kn.astype(np.float64),
                              vn.astype(np.float64), kc.astype(np.float64), vc.astype(np.float64), pos, 1e7, rot,
                              qn, knw)
    assert rel_err(out, ref) < 2e-5
    assert np.array_equal(kc2[:, :pos], kc[:, :pos])


@pytest.mark.parametrize("kv_bf16", [False, True])
def test_oracle_attn_op_kv_matches_attn_op(oracle, kv_bf16):
    """The persistent-cache form used for CPU op timing computes what attn_op computes,
    step after step as it appends to its own cache."""
    rng = np.random.default_rng(12)
    Hq, Hkv, hd, cap, pos = 8, 2, 64, 24, 9
    kc = rng.normal(size=(Hkv, cap, hd)).astype(np.float32)
    vc = rng.normal(size=(Hkv, cap, hd)).astype(np.float32)
    op = oracle.KvOp(kc, vc)
    for step in range(4):
        q = rng.normal(size=(Hq, hd)).astype(np.float32)
        gate = rng.normal(size=(Hq, hd)).astype(np.float32)
        kn = rng.normal(size=(Hkv, hd)).astype(np.float32)
        vn = rng.normal(size=(Hkv, hd)).astype(np.float32)
        ref, kc, vc = oracle.attn_op(q, gate, kn, vn, kc, vc, pos + step, 1e7, 32, kv_bf16=kv_bf16)
        got = op(q, gate, kn, vn, pos + step, 1e7, 32, kv_bf16=kv_bf16)
        assert np.array_equal(got, ref), step


def test_oracle_forward_matches_numpy(oracle, tiny_gguf, tiny_model):
    ref = numpy_ref.Model(tiny_gguf)
    st = ref.new_state(64)
    seq = tiny_model.new_seq()
    for pos, tok in enumerate([17, 31999, 5, 12345]):
        lo = seq.forward(tok)
        ln = ref.forward(st, tok, pos)
        assert rel_err(lo, ln) < 1e-4, pos


def test_oracle_config_from_gguf(tiny_model, synth):
    s = synth.tiny_shape()
    c = tiny_model.cfg
    assert (c["dim"], c["n_layers"], c["vocab"], c["hidden_dim"]) == (s.dim, s.n_layers, s.vocab, s.ffn)
    assert (c["n_heads"], c["n_kv_heads"], c["head_dim"]) == (s.attn_heads, s.kv_heads, s.head_dim)
    assert (c["ssm_groups"], c["ssm_state"], c["conv_kernel"]) == (s.dn_heads, s.dn_state, s.conv_kernel)
    assert tiny_model.layer_is_dn == [True, True, True, False]


def test_oracle_default_context_cap(oracle, tiny_gguf):
    # ModelConfig::from_gguf caps max_seq_len at 4096 (crates/engine/src/model.rs:50)
    assert oracle.Model(tiny_gguf).cfg["max_seq"] == 4096



def test_oracle_gemv_f16_matches_numpy(oracle, synth):
    """The oracle's GEMV with the batched tensor-core GEMM's declared operand rounding (weights
    q*d and the input rounded once to f16, f32 sums) against numpy with the same rounding."""
    rng = np.random.default_rng(8)
    m, n = 300, 2048
    blocks = synth.random_q8_0(rng, m, n, std=0.02)
    x = rng.normal(size=n).astype(np.float32)
    W16 = numpy_ref.f16(synth.dequant_q8_0(blocks).reshape(m, n).astype(np.float64))
    ref = W16 @ numpy_ref.f16(x.astype(np.float64))
    got = oracle.q8_gemv(blocks, m, n, x, f16_operands=True)
    assert rel_err(got, ref) < 1e-5
    exact = oracle.q8_gemv(blocks, m, n, x)
    assert 1e-5 < rel_err(got, exact) < 3e-3  # the rounding is visible and bounded


def test_f16_operand_rounding_greedy_statistics(tiny_gguf, synth):
    """What the batched tensor-core path's declared rounding (every weight q*d and every GEMM
    input rounded once to f16) does to the reference's logits and greedy picks, measured on
    the float64 restatement of the tiny config (32-token prompt + 64 greedy tokens per
    sequence, teacher-forced with the reference's tokens): the per-step logit error stays far
    inside the 1e-2 bar, and the greedy picks differ only at near-ties, where the reference's
    top-2 gap is below that step's logit error. Rounding alone flips a few picks; the GPU
    tests hold the device to this same characterisation."""
    exact = numpy_ref.Model(tiny_gguf)
    rounded = numpy_ref.Model(tiny_gguf, f16_operands=True)
    worst, flips, total = 0.0, [], 0
    for s in range(3):
        prompt = synth.seeded_tokens(32, 32000, seed=100 + s)
        st, st16 = exact.new_state(128), rounded.new_state(128)
        tok = None
        for i in range(96):
            feed = int(prompt[i]) if i < 32 else tok
            a, b = exact.forward(st, feed, i), rounded.forward(st16, feed, i)
            err = rel_err(b, a)
            worst = max(worst, err)
            if i >= 31:
                total += 1
                ia, ib = int(np.argmax(a)), int(np.argmax(b))
                if ia != ib:
                    gap = (a[ia] - a[ib]) / np.max(np.abs(a))
                    flips.append((s, i, gap, err))
                    assert gap <= 2 * err, (s, i, gap, err)
                tok = ia
    print(f"f16 operand rounding: worst logit rel err {worst:.2e}; {len(flips)} of {total} greedy picks "
          f"differ, at top-2 gaps {[f'{f[2]:.1e}' for f in flips]}")
    assert worst < 1e-2
    assert len(flips) <= total // 50
