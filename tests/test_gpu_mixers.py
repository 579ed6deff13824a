"""GPU parity of the fused DeltaNet and attention kernels against the oracle: the
recurrence op (config 2), the flash-decode op (config 3) and the per-layer mixers."""
import numpy as np
import pytest

from conftest import attn_mma_plan, rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-4   # max|diff| <= TOL * max|ref|


def bf16_bits(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).cuda()


# ---------------------------------------------------------------------------- recurrence op
def config2_inputs(rng, B, H=16):
    S = rng.normal(0, 0.1, size=(B, H, 128, 128)).astype(np.float32)
    q = rng.normal(size=(B, H, 128)).astype(np.float32)
    k = rng.normal(size=(B, H, 128)).astype(np.float32)
    v = rng.normal(size=(B, H, 128)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    beta = (1 / (1 + np.exp(-rng.normal(size=(B, H))))).astype(np.float32)
    decay = np.exp(-np.log1p(np.exp(rng.normal(size=(B, H)))) * np.exp(rng.normal(0, 0.5, size=(B, H))))
    return S, q, k, v, beta, decay.astype(np.float32)


@pytest.mark.parametrize("B", [1, 16, 64, 256])
def test_gated_delta_op(pkg, oracle, synth, cuda, B):
    torch = cuda
    rng = np.random.default_rng(B)
    S, q, k, v, beta, decay = config2_inputs(rng, B)
    q, k, v = synth.bf16_round(q), synth.bf16_round(k), synth.bf16_round(v)
    o_ref, S_ref = oracle.gated_delta(S, q, k, v, beta, decay)
    Sd = torch.from_numpy(S).cuda()
    o = torch.empty((B, 16, 128), dtype=torch.float32, device="cuda")
    pkg.gated_delta(Sd, bf16_bits(torch, q), bf16_bits(torch, k), bf16_bits(torch, v),
                    torch.from_numpy(beta).cuda(), torch.from_numpy(decay).cuda(), o, B, 16)
    torch.cuda.synchronize()
    assert rel_err(o.cpu().numpy(), o_ref) < 1e-5
    assert rel_err(Sd.cpu().numpy(), S_ref) < 1e-5


def test_gated_delta_empty_batch(pkg, cuda):
    torch = cuda
    z = torch.zeros(1, device="cuda")
    pkg.gated_delta(z, z, z, z, z, z, z, 0, 16)   # B = 0 is a no-op


# ---------------------------------------------------------------------------- attention op
def attn_case(rng, synth, B, Hq, Hkv, hd, ctx, cap, kv_bf16):
    proj = rng.normal(size=(B, Hq * 2 * hd + 2 * Hkv * hd)).astype(np.float32)
    kc = rng.normal(size=(B, Hkv, cap, hd)).astype(np.float32)
    vc = rng.normal(size=(B, Hkv, cap, hd)).astype(np.float32)
    if kv_bf16:
        kc, vc = synth.bf16_round(kc), synth.bf16_round(vc)
    pos = np.array([ctx - 1 - (b % 3) for b in range(B)], dtype=np.int32).clip(0)
    return proj, kc, vc, pos


@pytest.mark.parametrize("B,ctx,hd,rot,kv_bf16,norms", [
    (1, 1, 256, 64, True, False),
    (1, 1024, 256, 64, True, False),
    (64, 1024, 256, 64, True, False),
    (1, 4096, 256, 64, True, True),
    (3, 777, 256, 256, True, True),
    (1, 16384, 256, 64, True, False),
    (2, 300, 128, 128, False, True),
    (5, 129, 256, 256, False, False),
])
def test_attn_decode_op(pkg, oracle, synth, cuda, B, ctx, hd, rot, kv_bf16, norms):
    torch = cuda
    Hq, Hkv = 8, 2
    cap = ctx + 8
    rng = np.random.default_rng(ctx + B + hd)
    proj, kc, vc, pos = attn_case(rng, synth, B, Hq, Hkv, hd, ctx, cap, kv_bf16)
    qn = (1 + rng.normal(0, 0.02, size=hd)).astype(np.float32) if norms else None
    kn = (1 + rng.normal(0, 0.02, size=hd)).astype(np.float32) if norms else None
    dt = torch.bfloat16 if kv_bf16 else torch.float32
    kd = torch.from_numpy(kc).to(dt).cuda()
    vd = torch.from_numpy(vc).to(dt).cuda()
    out = torch.empty((B, Hq * hd), dtype=torch.float32, device="cuda")
    pkg.attn_decode(torch.from_numpy(proj).cuda(), kd, vd, cap, torch.from_numpy(pos).cuda(), B, Hq, Hkv, hd, kv_bf16,
                    None if qn is None else torch.from_numpy(qn).cuda(),
                    None if kn is None else torch.from_numpy(kn).cuda(), 1e7, rot, int(pos.max()), out)
    torch.cuda.synchronize()
    og = out.cpu().numpy()
    kg = kd.float().cpu().numpy()
    for b in range(B):
        qf = proj[b, :Hq * 2 * hd].reshape(Hq, 2 * hd)
        kn_ = proj[b, Hq * 2 * hd: Hq * 2 * hd + Hkv * hd].reshape(Hkv, hd)
        vn_ = proj[b, Hq * 2 * hd + Hkv * hd:].reshape(Hkv, hd)
        ref, kc2, _ = oracle.attn_op(qf[:, :hd], qf[:, hd:], kn_, vn_, kc[b], vc[b], int(pos[b]), 1e7, rot, qn, kn,
                                     kv_bf16=kv_bf16)
        assert rel_err(og[b].reshape(Hq, hd), ref) < TOL, b
        p = int(pos[b])
        assert rel_err(kg[b][:, p], kc2[:, p]) < 1e-2 if kv_bf16 else rel_err(kg[b][:, p], kc2[:, p]) < 1e-5
        assert np.array_equal(kg[b][:, :p], kc[b][:, :p])


@pytest.mark.parametrize("B,ctx", [(64, 4096), (64, 16384), (64, 32768), (1, 32768)])
def test_attn_decode_op_config3(pkg, oracle, cuda, B, ctx):
    """The flash-decode cells of BASELINE config 3 (Hq 8, Hkv 2, hd 256, bf16 KV N(0,1), RoPE
    theta 1e7 on the first 64 dims, sigmoid gate N(0,1)) at B=64 and ctx 4K/16K/32K and at B=1,
    ctx 32K. The caches are drawn on the device; sequences 0, B/2 and B-1 (ragged positions)
    are checked against the oracle with their pre-call caches."""
    torch = cuda
    Hq, Hkv, hd, rot = 8, 2, 256, 64
    cap = ctx + 8
    g = torch.Generator(device="cuda").manual_seed(ctx + B)
    proj = torch.randn(B, Hq * 2 * hd + 2 * Hkv * hd, device="cuda", generator=g)
    kd = torch.randn(B, Hkv, cap, hd, device="cuda", generator=g).to(torch.bfloat16)
    vd = torch.randn(B, Hkv, cap, hd, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.tensor([ctx - 1 - (b % 3) for b in range(B)], dtype=torch.int32, device="cuda")
    check = sorted({0, B // 2, B - 1})
    pre = {b: (kd[b].float().cpu().numpy(), vd[b].float().cpu().numpy()) for b in check}
    out = torch.empty((B, Hq * hd), dtype=torch.float32, device="cuda")
    pkg.attn_decode(proj, kd, vd, cap, pos, B, Hq, Hkv, hd, True, None, None, 1e7, rot, int(pos.max().item()), out)
    torch.cuda.synchronize()
    assert pkg.op_error() == 0
    og, pj, ph = out.cpu().numpy(), proj.cpu().numpy(), pos.cpu().numpy()
    for b in check:
        qf = pj[b, :Hq * 2 * hd].reshape(Hq, 2 * hd)
        kn_ = pj[b, Hq * 2 * hd: Hq * 2 * hd + Hkv * hd].reshape(Hkv, hd)
        vn_ = pj[b, Hq * 2 * hd + Hkv * hd:].reshape(Hkv, hd)
        ref, _, _ = oracle.attn_op(qf[:, :hd], qf[:, hd:], kn_, vn_, pre[b][0], pre[b][1], int(ph[b]), 1e7, rot,
                                   kv_bf16=True)
        e = rel_err(og[b].reshape(Hq, hd), ref)
        print(f"B={B} ctx={ctx} seq {b}: rel err {e:.2e}")
        assert e < TOL, b


def test_attn_decode_balanced_partition_ragged(pkg, oracle, cuda):
    """The balanced partition of the tensor-core flash-decode (every pair's tiles laid end to
    end, an equal run per CTA) on a widely ragged batch of 40 sequences (positions 0, 63, 64,
    127, max_pos and seeded values between), with one sequence beyond max_pos that must be
    skipped: a CTA's run then holds many short pairs, long pairs are cut across several
    CTAs, and the device-side plan has to skip the rejected sequence's tiles. Every computed
    sequence is checked against the oracle."""
    torch = cuda
    B, Hq, Hkv, hd, rot, max_pos = 40, 8, 2, 256, 64, 5999
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert attn_mma_plan(B, Hkv, max_pos + 1, sms) == "balanced"
    cap = max_pos + 80
    rng = np.random.default_rng(4040)
    pos_h = rng.integers(0, max_pos + 1, size=B).astype(np.int32)
    pos_h[:6] = [0, 63, 64, 127, max_pos, 1]
    skipped = 17
    pos_h[skipped] = max_pos + 40  # inside the cache, beyond max_pos
    g = torch.Generator(device="cuda").manual_seed(4041)
    proj = torch.randn(B, Hq * 2 * hd + 2 * Hkv * hd, device="cuda", generator=g)
    kd = torch.randn(B, Hkv, cap, hd, device="cuda", generator=g).to(torch.bfloat16)
    vd = torch.randn(B, Hkv, cap, hd, device="cuda", generator=g).to(torch.bfloat16)
    pre = (kd.float().cpu().numpy(), vd.float().cpu().numpy())
    pos = torch.from_numpy(pos_h).cuda()
    out = torch.zeros((B, Hq * hd), dtype=torch.float32, device="cuda")
    assert pkg.op_error() == 0
    pkg.attn_decode(proj, kd, vd, cap, pos, B, Hq, Hkv, hd, True, None, None, 1e7, rot, max_pos, out)
    torch.cuda.synchronize()
    assert pkg.op_error() & 8192
    og, pj = out.cpu().numpy(), proj.cpu().numpy()
    assert float(np.abs(og[skipped]).max()) == 0.0
    worst = 0.0
    for b in range(B):
        if b == skipped:
            continue
        qf = pj[b, :Hq * 2 * hd].reshape(Hq, 2 * hd)
        kn_ = pj[b, Hq * 2 * hd: Hq * 2 * hd + Hkv * hd].reshape(Hkv, hd)
        vn_ = pj[b, Hq * 2 * hd + Hkv * hd:].reshape(Hkv, hd)
        ref, _, _ = oracle.attn_op(qf[:, :hd], qf[:, hd:], kn_, vn_, pre[0][b], pre[1][b], int(pos_h[b]), 1e7, rot,
                                   kv_bf16=True)
        e = rel_err(og[b].reshape(Hq, hd), ref)
        worst = max(worst, e)
        assert e < TOL, (b, int(pos_h[b]), e)
    print(f"balanced partition, 39 ragged sequences: worst rel err {worst:.2e}")


@pytest.mark.parametrize("kv_bf16", [True, False])
def test_attn_decode_rejects_position_above_max_pos(pkg, oracle, synth, cuda, kv_bf16):
    """ab2_attn_decode's device-side position check: a sequence whose pos[b] is above the
    declared max_pos (still inside the cache) is skipped, nothing is appended to its cache,
    and ab2_op_error reports bit 8192; the other sequences are computed as usual."""
    torch = cuda
    B, Hq, Hkv, hd, rot, ctx = 3, 8, 2, 256, 64, 200
    cap = ctx + 64
    rng = np.random.default_rng(77)
    proj, kc, vc, _ = attn_case(rng, synth, B, Hq, Hkv, hd, ctx, cap, kv_bf16)
    max_pos = ctx - 1
    pos = np.array([ctx - 1, ctx + 20, ctx - 2], dtype=np.int32)  # sequence 1 lies beyond max_pos
    dt = torch.bfloat16 if kv_bf16 else torch.float32
    kd, vd = torch.from_numpy(kc).to(dt).cuda(), torch.from_numpy(vc).to(dt).cuda()
    k_before = kd[1].clone()
    out = torch.zeros((B, Hq * hd), dtype=torch.float32, device="cuda")
    assert pkg.op_error() == 0
    pkg.attn_decode(torch.from_numpy(proj).cuda(), kd, vd, cap, torch.from_numpy(pos).cuda(), B, Hq, Hkv, hd, kv_bf16,
                    None, None, 1e7, rot, max_pos, out)
    code = pkg.op_error()
    assert code & 8192, hex(code)
    assert torch.equal(kd[1], k_before)  # no append at the rejected position
    assert float(out[1].abs().max()) == 0.0
    og = out.cpu().numpy()
    for b in (0, 2):
        qf = proj[b, :Hq * 2 * hd].reshape(Hq, 2 * hd)
        kn_ = proj[b, Hq * 2 * hd: Hq * 2 * hd + Hkv * hd].reshape(Hkv, hd)
        vn_ = proj[b, Hq * 2 * hd + Hkv * hd:].reshape(Hkv, hd)
        ref, _, _ = oracle.attn_op(qf[:, :hd], qf[:, hd:], kn_, vn_, kc[b], vc[b], int(pos[b]), 1e7, rot,
                                   kv_bf16=kv_bf16)
        assert rel_err(og[b].reshape(Hq, hd), ref) < TOL, b
    assert pkg.op_error() == 0  # the word was cleared by the read


# ---------------------------------------------------------------------------- model layers
@pytest.fixture(scope="module")
def tiny_ctx(pkg, tiny_gguf, cuda):
    ctx = pkg.DecodeContext(tiny_gguf, max_batch=2, max_ctx=128, kv_bf16=False)
    yield ctx
    ctx.close()


def test_deltanet_layer(tiny_ctx, tiny_model):
    rng = np.random.default_rng(11)
    layer = 1
    rec = rng.normal(0, 0.1, size=(8, 128, 128)).astype(np.float32)
    conv = rng.normal(0, 1, size=(3072, 4)).astype(np.float32)
    seq = tiny_model.new_seq()
    seq.set_dn(layer, rec, conv)
    tiny_ctx.set_dn_state(layer, 1, rec, conv)
    for step in range(3):
        x = rng.normal(size=1024).astype(np.float32)
        ref = seq.mixer(layer, x)
        got = tiny_ctx.mixer_layer(layer, 1, x)
        assert rel_err(got, ref) < TOL, step
    r_ref, c_ref = seq.get_dn(layer)
    r_got, c_got = tiny_ctx.get_dn_state(layer, 1)
    assert rel_err(r_got, r_ref) < 1e-5
    assert rel_err(c_got, c_ref) < 1e-5       # shifted-in columns are the (float) projection output
    assert np.array_equal(c_got[:, 0], conv[:, 3])   # the oldest column is the seeded state, shifted


def test_attention_layer(tiny_ctx, tiny_model):
    rng = np.random.default_rng(12)
    layer = 3
    n = 50
    k = rng.normal(size=(2, n, 128)).astype(np.float32)
    v = rng.normal(size=(2, n, 128)).astype(np.float32)
    seq = tiny_model.new_seq()
    seq.set_kv(layer, k, v)
    seq.pos = n
    tiny_ctx.set_kv(layer, 0, k, v)
    tiny_ctx.set_pos(0, n)
    x = rng.normal(size=1024).astype(np.float32)
    ref = seq.mixer(layer, x)
    got = tiny_ctx.mixer_layer(layer, 0, x)
    assert rel_err(got, ref) < TOL
    kr, vr = seq.get_kv(layer, n + 1)
    kg, vg = tiny_ctx.get_kv(layer, 0, n + 1)
    assert rel_err(kg, kr) < 1e-5 and rel_err(vg, vr) < 1e-5


def test_ffn_layer(tiny_ctx, tiny_model):
    rng = np.random.default_rng(13)
    for layer in (0, 3):
        x = rng.normal(size=1024).astype(np.float32)
        assert rel_err(tiny_ctx.ffn_layer(layer, x), tiny_model.ffn(layer, x)) < TOL
