"""Independent float64 numpy restatement of the reference decode path (test infrastructure).

It follows the same reference functions as oracle/oracle.cpp but shares no code with it
(own GGUF reader, vectorised float64 arithmetic), so agreement between the two is a check
on the C++ restatement for the parts the reference's own tests do not pin:
conv1d + SiLU (crates/engine/src/deltanet_cache.rs:34-54), the gated delta rule and gated
RMSNorm (crates/engine/src/deltanet.rs:429-538), RoPE + SDPA + sigmoid gate
(deltanet.rs:541-675) and the layer/head wrapper (crates/cli/src/main.rs:953-1023).
"""
from __future__ import annotations

import struct

import numpy as np


# ------------------------------------------------------------------------------ GGUF reader
def read_gguf(buf: np.ndarray):
    b = memoryview(np.ascontiguousarray(buf, dtype=np.uint8))
    o = 0

    def rd(fmt):
        nonlocal o
        v = struct.unpack_from("<" + fmt, b, o)
        o += struct.calcsize("<" + fmt)
        return v[0]

    def rstr():
        nonlocal o
        n = rd("Q")
        s = bytes(b[o:o + n]).decode()
        o += n
        return s

    fmts = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "B", 10: "Q", 11: "q", 12: "d"}

    def rval(t):
        if t == 8:
            return rstr()
        if t == 9:
            et, n = rd("I"), rd("Q")
            return [rval(et) for _ in range(n)]
        return rd(fmts[t])

    assert rd("I") == 0x46554747
    ver = rd("I")
    nt, nkv = rd("Q"), rd("Q")
    meta = {}
    for _ in range(nkv):
        k = rstr()
        meta[k] = rval(rd("I"))
    infos = []
    for _ in range(nt):
        name = rstr()
        nd = rd("I")
        dims = [rd("Q") for _ in range(nd)]
        infos.append((name, dims, rd("I"), rd("Q")))
    align = meta.get("general.alignment", 32)
    base = (o + align - 1) // align * align
    tensors = {}
    arr = np.frombuffer(b, dtype=np.uint8)
    for name, dims, t, off in infos:
        ne = int(np.prod(dims))
        if t == 0:
            tensors[name] = arr[base + off: base + off + 4 * ne].view(np.float32).astype(np.float64).reshape(
                list(reversed(dims)))
        elif t == 8:
            nb = ne // 32
            blk = arr[base + off: base + off + 34 * nb].reshape(nb, 34)
            d = blk[:, :2].copy().view(np.float16).astype(np.float64)
            q = blk[:, 2:].view(np.int8).astype(np.float64)
            tensors[name] = (q * d).reshape(dims[1], dims[0])
        else:
            raise ValueError(f"type {t}")
    return ver, meta, tensors


# ------------------------------------------------------------------------------ ops
def rmsnorm(x, w, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * w


def silu(x):
    return x / (1.0 + np.exp(-x))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def gated_delta(S, q, k, v, beta, decay):
    """S [dk][dv]; returns (o [dv], S_new)."""
    S = S * decay
    sk = S.T @ k
    delta = beta * (v - sk)
    S = S + np.outer(k, delta)
    return S.T @ q, S


def rope(x, pos, base, rot):
    x = x.copy()
    i = np.arange(0, rot, 2)
    ang = pos * (1.0 / base ** (i / rot))
    c, s = np.cos(ang), np.sin(ang)
    a0, a1 = x[..., i].copy(), x[..., i + 1].copy()
    x[..., i] = a0 * c - a1 * s
    x[..., i + 1] = a0 * s + a1 * c
    return x


def attn_core(q, gate, k_new, v_new, kc, vc, pos, base, rot, q_norm=None, k_norm=None):
    """q/gate [Hq][hd], k_new/v_new [Hkv][hd], caches [Hkv][cap][hd] (modified)."""
    Hq, hd = q.shape
    Hkv = k_new.shape[0]
    if q_norm is not None:
        q = np.stack([rmsnorm(q[h], q_norm, 1e-6) for h in range(Hq)])
    if k_norm is not None:
        k_new = np.stack([rmsnorm(k_new[h], k_norm, 1e-6) for h in range(Hkv)])
    q = rope(q, pos, base, rot)
    k_new = rope(k_new, pos, base, rot)
    kc[:, pos] = k_new
    vc[:, pos] = v_new
    out = np.empty_like(q)
    g = Hq // Hkv
    for h in range(Hq):
        K = kc[h // g, :pos + 1]
        V = vc[h // g, :pos + 1]
        s = K @ q[h] / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h] = p @ V
    return out * sigmoid(gate)


def f16(a):
    return np.asarray(a).astype(np.float16).astype(np.float64)


class Model:
    """f16_operands: every Q8_0 weight and every GEMM input rounded once to f16 (the batched
    tensor-core GEMM's declared rounding, a test mode; the default is the reference's f32 path)."""

    def __init__(self, gguf, f16_operands=False):
        _, meta, t = read_gguf(gguf)
        self.f16 = f16_operands
        if f16_operands:  # the embedding gather reads exact rows; only GEMM weights are rounded
            t = {k: (f16(v) if k.endswith(".weight") and v.ndim == 2 and "conv1d" not in k
                     and k != "token_embd.weight" else v) for k, v in t.items()}
        a = meta["general.architecture"]
        self.t = t
        self.dim = meta[f"{a}.embedding_length"]
        self.n_layers = meta[f"{a}.block_count"]
        self.hd = meta[f"{a}.attention.key_length"]
        self.Hq = meta[f"{a}.attention.head_count"]
        self.Hkv = meta[f"{a}.attention.head_count_kv"]
        self.H = meta[f"{a}.ssm.group_count"]
        self.K = meta[f"{a}.ssm.conv_kernel"]
        self.eps = meta[f"{a}.attention.layer_norm_rms_epsilon"]
        self.base = meta[f"{a}.rope.freq_base"]
        self.is_dn = [f"blk.{l}.ssm_a" in t for l in range(self.n_layers)]
        self.lm = t.get("output.weight", f16(t["token_embd.weight"]) if f16_operands else t["token_embd.weight"])

    def mv(self, w, x):
        """One Q8_0 GEMV input: W @ x, x rounded to f16 in the f16_operands mode."""
        return w @ (f16(x) if self.f16 else x)

    def new_state(self, cap):
        st = []
        for l in range(self.n_layers):
            if self.is_dn[l]:
                st.append({"S": np.zeros((self.H, 128, 128)), "conv": np.zeros((3 * self.dim, self.K))})
            else:
                st.append({"k": np.zeros((self.Hkv, cap, self.hd)), "v": np.zeros((self.Hkv, cap, self.hd))})
        return st

    def dn_mixer(self, l, x, st):
        t, p, D, H = self.t, f"blk.{l}.", self.dim, self.H
        qkv = self.mv(t[p + "attn_qkv.weight"], x)
        st["conv"] = np.concatenate([st["conv"][:, 1:], qkv[:, None]], axis=1)
        c = silu((st["conv"] * t[p + "ssm_conv1d.weight"]).sum(axis=1))
        q, k, v = c[:D].reshape(H, 128), c[D:2 * D].reshape(H, 128), c[2 * D:].reshape(H, 128)
        q = q / np.sqrt((q * q).sum(1, keepdims=True) + 1e-12) / np.sqrt(128)
        k = k / np.sqrt((k * k).sum(1, keepdims=True) + 1e-12)
        beta = sigmoid(self.mv(t[p + "ssm_beta.weight"], x))
        a = self.mv(t[p + "ssm_alpha.weight"], x) + t[p + "ssm_dt.bias"]
        decay = np.exp(t[p + "ssm_a"] * np.log1p(np.exp(a)))
        o = np.empty((H, 128))
        for h in range(H):
            o[h], st["S"][h] = gated_delta(st["S"][h], q[h], k[h], v[h], beta[h], decay[h])
        gate = self.mv(t[p + "attn_gate.weight"], x)
        normed = np.concatenate([rmsnorm(o[h], t[p + "ssm_norm.weight"], self.eps) for h in range(H)])
        return self.mv(t[p + "ssm_out.weight"], normed * silu(gate))

    def attn_mixer(self, l, x, st, pos):
        t, p, hd = self.t, f"blk.{l}.", self.hd
        qf = self.mv(t[p + "attn_q.weight"], x).reshape(self.Hq, 2 * hd)
        k = self.mv(t[p + "attn_k.weight"], x).reshape(self.Hkv, hd)
        v = self.mv(t[p + "attn_v.weight"], x).reshape(self.Hkv, hd)
        o = attn_core(qf[:, :hd], qf[:, hd:], k, v, st["k"], st["v"], pos, self.base, hd,
                      t[p + "attn_q_norm.weight"], t[p + "attn_k_norm.weight"])
        return self.mv(t[p + "attn_output.weight"], o.reshape(-1))

    def ffn(self, l, x):
        t, p = self.t, f"blk.{l}."
        return self.mv(t[p + "ffn_down.weight"], silu(self.mv(t[p + "ffn_gate.weight"], x)) * self.mv(t[p + "ffn_up.weight"], x))

    def forward(self, st, token, pos):
        t = self.t
        x = t["token_embd.weight"][token].copy()
        for l in range(self.n_layers):
            xn = rmsnorm(x, t[f"blk.{l}.attn_norm.weight"], self.eps)
            x = x + (self.dn_mixer(l, xn, st[l]) if self.is_dn[l] else self.attn_mixer(l, xn, st[l], pos))
            x = x + self.ffn(l, rmsnorm(x, t[f"blk.{l}.post_attention_norm.weight"], self.eps))
        return self.mv(self.lm, rmsnorm(x, t["output_norm.weight"], self.eps))
