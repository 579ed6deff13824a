"""Seeded synthetic Qwen3.5-hybrid models written as GGUF v3 bytes, plus seeded state.

No real checkpoint or dataset is used anywhere in this package: every weight, state and
token id comes from numpy ``Generator(PCG64)`` with a fixed seed scheme
(seed 0 weights, seed 1 recurrent/KV state, seed 2 tokens and activations).

The byte layout is the one the reference parser reads (crates/gguf/src/parser.rs:299-347):
magic "GGUF", version 3, u64 tensor count, u64 metadata count, typed metadata
(U32/F32/String/Array, parser.rs:271-295), tensor infos (name, n_dims, u64 dims with ne0
fastest, ggml type, u64 offset), padding to ``general.alignment`` (32) and the tensor data.
Metadata keys follow the accessors at parser.rs:360-486 with the ``qwen35`` prefix; the
vocabulary size is the length of ``tokenizer.ggml.tokens`` (parser.rs:395-401).
Tensor names follow crates/gguf/src/to_ane.rs:129-163 and crates/cli/src/main.rs:1894-1994.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field

import numpy as np

GGML_F32 = 0
GGML_F16 = 1
GGML_Q8_0 = 8

QK8_0 = 32          # elements per Q8_0 block (crates/engine/src/q8_gemv.rs:23)
Q8_0_BYTES = 34     # [f16 d little-endian][32 x i8] (q8_gemv.rs:24, gguf/src/dequant.rs:29-38)


@dataclass
class HybridShape:
    """Shape of a Qwen3.5 hybrid model (Gated DeltaNet layers + every n-th GQA layer)."""
    n_layers: int = 4
    dim: int = 1024
    vocab: int = 32000
    ffn: int = 3072
    dn_heads: int = 8          # ssm.group_count
    dn_state: int = 128        # ssm.state_size (dk = dv)
    conv_kernel: int = 4       # ssm.conv_kernel
    attn_heads: int = 8        # attention.head_count
    kv_heads: int = 2          # attention.head_count_kv
    head_dim: int = 128        # attention.key_length
    full_attn_interval: int = 4
    rope_base: float = 1e7
    eps: float = 1e-6
    context_length: int = 262144
    tied_embedding: bool = False

    def layer_is_attn(self, l: int) -> bool:
        return (l + 1) % self.full_attn_interval == 0


def tiny_shape() -> HybridShape:
    """Config 1: 4 layers (DN x3 then GQA), hidden 1024, vocab 32000, 8 DN heads, GQA 8/2/128."""
    return HybridShape()


def shape_2b() -> HybridShape:
    """Config 5: 24 layers (every 4th GQA), hidden 2048, vocab 151936, DN 16x128, GQA 8/2/256."""
    return HybridShape(n_layers=24, dim=2048, vocab=151936, ffn=6144, dn_heads=16, dn_state=128,
                       conv_kernel=4, attn_heads=8, kv_heads=2, head_dim=256)


# ----------------------------------------------------------------------------- Q8_0 encode

def f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """Quantise a row-major [m][n] float array to GGUF Q8_0 block bytes [m][n/32][34].

    The rule is llama.cpp's reference Q8_0 quantiser: d = max|w|/127 per 32-element block,
    q = round(w / d) with the f32 d, and d stored as f16.
    """
    w = np.asarray(w, dtype=np.float32)
    m, n = w.shape
    assert n % QK8_0 == 0
    blk = w.reshape(m, n // QK8_0, QK8_0)
    amax = np.abs(blk).max(axis=2)
    d = amax / np.float32(127.0)
    inv = np.where(d > 0, np.float32(1.0) / np.where(d > 0, d, 1), 0).astype(np.float32)
    xs = (blk * inv[..., None]).astype(np.float64)          # f32 product, exact in f64
    q = (np.sign(xs) * np.floor(np.abs(xs) + 0.5)).astype(np.int8)   # C roundf: half away from 0
    out = np.empty((m, n // QK8_0, Q8_0_BYTES), dtype=np.uint8)
    out[..., 0:2] = f16_bits(d).reshape(m, n // QK8_0, 1).view(np.uint8)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(-1)


def random_q8_0(rng: np.random.Generator, m: int, n: int, std: float = 0.02) -> np.ndarray:
    """Random Q8_0 blocks: q uniform in [-127, 127], d = f16(std/73.3 * U[0.75, 1.25]).

    The scale keeps the dequantised weights near N(0, std) in size so activations stay
    finite through many layers. Used for large shapes where quantising N(0, std) floats
    would dominate set-up time.
    """
    nb = m * (n // QK8_0)
    out = np.empty((nb, Q8_0_BYTES), dtype=np.uint8)
    out[:, 2:] = rng.integers(-127, 128, size=(nb, QK8_0), dtype=np.int8).view(np.uint8)
    d = (np.float32(std / 73.3) * rng.uniform(0.75, 1.25, size=nb).astype(np.float32))
    out[:, 0:2] = f16_bits(d).reshape(nb, 1).view(np.uint8)
    return out.reshape(-1)


def dequant_q8_0(blocks: np.ndarray) -> np.ndarray:
    """Exact f32 dequantisation w = (f32)(i8 q) * (f32)(f16 d) (gguf/src/dequant.rs:29-38)."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, Q8_0_BYTES)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(-1)


# ----------------------------------------------------------------------------- GGUF writer

class _Meta:
    def __init__(self):
        self.items: list[bytes] = []

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode()
        return struct.pack("<Q", len(b)) + b

    def u32(self, k, v):
        self.items.append(self._str(k) + struct.pack("<II", 4, v))

    def f32(self, k, v):
        self.items.append(self._str(k) + struct.pack("<If", 6, v))

    def string(self, k, v):
        self.items.append(self._str(k) + struct.pack("<I", 8) + self._str(v))

    def str_array(self, k, values):
        parts = [self._str(k), struct.pack("<IIQ", 9, 8, len(values))]
        parts.extend(self._str(s) for s in values)
        self.items.append(b"".join(parts))


@dataclass
class _Tensor:
    name: str
    dims: tuple          # ne0 first
    gtype: int
    data: np.ndarray     # uint8 bytes


@dataclass
class GgufBuilder:
    alignment: int = 32
    meta: _Meta = field(default_factory=_Meta)
    tensors: list = field(default_factory=list)

    def add_f32(self, name, arr, dims=None):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        dims = dims or tuple(reversed(arr.shape))
        self.tensors.append(_Tensor(name, dims, GGML_F32, arr.view(np.uint8).reshape(-1)))

    def add_q8(self, name, blocks, m, n):
        """Q8_0 tensor of m rows x n cols (GGUF dims ne0=n, ne1=m)."""
        assert blocks.size == m * (n // QK8_0) * Q8_0_BYTES
        self.tensors.append(_Tensor(name, (n, m), GGML_Q8_0, blocks))

    def tobytes(self) -> np.ndarray:
        infos = []
        off = 0
        offsets = []
        for t in self.tensors:
            off = (off + self.alignment - 1) // self.alignment * self.alignment
            offsets.append(off)
            off += t.data.size
        for t, o in zip(self.tensors, offsets):
            nb = t.name.encode()
            infos.append(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(t.dims))
                         + b"".join(struct.pack("<Q", d) for d in t.dims)
                         + struct.pack("<IQ", t.gtype, o))
        head = (struct.pack("<IIQQ", 0x46554747, 3, len(self.tensors), len(self.meta.items))
                + b"".join(self.meta.items) + b"".join(infos))
        data_off = (len(head) + self.alignment - 1) // self.alignment * self.alignment
        total = data_off + off
        buf = np.zeros(total, dtype=np.uint8)
        buf[:len(head)] = np.frombuffer(head, dtype=np.uint8)
        for t, o in zip(self.tensors, offsets):
            buf[data_off + o: data_off + o + t.data.size] = t.data
        return buf


def build_model_gguf(shape: HybridShape, seed: int = 0, exact_quant: bool | None = None,
                     threads: int | None = None) -> np.ndarray:
    """Return the GGUF bytes (uint8 array) of a seeded random Qwen3.5 hybrid model.

    exact_quant=True quantises N(0, 0.02) weights with the Q8_0 rule (config 1);
    False draws random Q8_0 blocks directly (config 5, much faster at 2B shape).
    Default: exact for models under 100M parameters. Every tensor is drawn from its own
    stream PCG64(SeedSequence([seed, tensor index])), so tensors are generated in parallel
    and the bytes do not depend on the thread count.
    """
    s = shape
    nparams = s.vocab * s.dim * 2 + s.n_layers * (4 * s.dim * s.dim + 3 * s.dim * s.ffn)
    if exact_quant is None:
        exact_quant = nparams < 100_000_000

    specs = []   # (name, kind, args): kind q8 -> (m, n); f32 -> (generator name, shape)

    def q8(name, m, n):
        specs.append((name, "q8", (m, n)))

    def f32(name, how, shp):
        specs.append((name, "f32", (how, shp)))

    D, H = s.dim, s.dn_heads
    q8("token_embd.weight", s.vocab, D)
    for l in range(s.n_layers):
        p = f"blk.{l}."
        f32(p + "attn_norm.weight", "norm", D)
        f32(p + "post_attention_norm.weight", "norm", D)
        if s.layer_is_attn(l):
            qd, kvd = s.attn_heads * s.head_dim, s.kv_heads * s.head_dim
            q8(p + "attn_q.weight", 2 * qd, D)
            q8(p + "attn_k.weight", kvd, D)
            q8(p + "attn_v.weight", kvd, D)
            q8(p + "attn_output.weight", D, qd)
            f32(p + "attn_q_norm.weight", "norm", s.head_dim)
            f32(p + "attn_k_norm.weight", "norm", s.head_dim)
        else:
            q8(p + "attn_qkv.weight", 3 * D, D)
            q8(p + "attn_gate.weight", D, D)
            f32(p + "ssm_a", "ssm_a", H)
            q8(p + "ssm_alpha.weight", H, D)
            q8(p + "ssm_beta.weight", H, D)
            f32(p + "ssm_conv1d.weight", "n0.1", (3 * D, s.conv_kernel))
            f32(p + "ssm_dt.bias", "n0.1", H)
            f32(p + "ssm_norm.weight", "norm", s.dn_state)
            q8(p + "ssm_out.weight", D, D)
        q8(p + "ffn_gate.weight", s.ffn, D)
        q8(p + "ffn_up.weight", s.ffn, D)
        q8(p + "ffn_down.weight", D, s.ffn)
    f32("output_norm.weight", "norm", D)
    if not s.tied_embedding:
        q8("output.weight", s.vocab, D)

    def gen(i):
        name, kind, args = specs[i]
        rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, i])))
        if kind == "q8":
            m, n = args
            if exact_quant:
                return quantize_q8_0(rng.normal(0.0, 0.02, size=(m, n)).astype(np.float32))
            return random_q8_0(rng, m, n)
        how, shp = args
        if how == "norm":
            return (1.0 + rng.normal(0.0, 0.02, size=shp)).astype(np.float32)
        if how == "ssm_a":       # negative, so decay = exp(a * softplus(.)) lies in (0, 1)
            return -np.exp(rng.normal(0.0, 0.5, size=shp)).astype(np.float32)
        return rng.normal(0.0, 0.1, size=shp).astype(np.float32)

    import concurrent.futures as cf
    with cf.ThreadPoolExecutor(max_workers=threads or min(32, os.cpu_count() or 4)) as ex:
        data = list(ex.map(gen, range(len(specs))))

    g = GgufBuilder()
    m = g.meta
    a = "qwen35"
    m.string("general.architecture", a)
    m.u32("general.alignment", g.alignment)
    m.u32(f"{a}.embedding_length", s.dim)
    m.u32(f"{a}.block_count", s.n_layers)
    m.u32(f"{a}.feed_forward_length", s.ffn)
    m.u32(f"{a}.context_length", s.context_length)
    m.u32(f"{a}.full_attention_interval", s.full_attn_interval)
    m.u32(f"{a}.attention.head_count", s.attn_heads)
    m.u32(f"{a}.attention.head_count_kv", s.kv_heads)
    m.u32(f"{a}.attention.key_length", s.head_dim)
    m.u32(f"{a}.attention.value_length", s.head_dim)
    m.f32(f"{a}.attention.layer_norm_rms_epsilon", s.eps)
    m.f32(f"{a}.rope.freq_base", s.rope_base)
    m.u32(f"{a}.ssm.state_size", s.dn_state)
    m.u32(f"{a}.ssm.conv_kernel", s.conv_kernel)
    m.u32(f"{a}.ssm.inner_size", s.dim)
    m.u32(f"{a}.ssm.group_count", s.dn_heads)
    m.str_array("tokenizer.ggml.tokens", [f"<t{i}>" for i in range(s.vocab)])
    for (name, kind, args), arr in zip(specs, data):
        if kind == "q8":
            g.add_q8(name, arr, *args)
        else:
            g.add_f32(name, arr)
    return g.tobytes()


# ----------------------------------------------------------------------------- seeded state

def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round f32 to the nearest bf16 (ties to even) and return it as f32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000))
    return r.view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def state_rng(seq: int, layer: int, what: int, seed: int = 1) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64([seed, seq, layer, what]))


def seeded_dn_state(shape: HybridShape, seq: int, layer: int) -> np.ndarray:
    """Recurrent state [H][dk][dv] ~ N(0, 0.1) (config 5)."""
    r = state_rng(seq, layer, 0)
    return r.normal(0.0, 0.1, size=(shape.dn_heads, shape.dn_state, shape.dn_state)).astype(np.float32)


def seeded_conv_state(shape: HybridShape, seq: int, layer: int) -> np.ndarray:
    """Conv state [3*dim][K] ~ N(0, 1) (config 5)."""
    r = state_rng(seq, layer, 1)
    return r.normal(0.0, 1.0, size=(3 * shape.dim, shape.conv_kernel)).astype(np.float32)


def seeded_kv(shape: HybridShape, seq: int, layer: int, n_tokens: int) -> tuple:
    """K and V caches [Hkv][n][hd], N(0,1) rounded to bf16-representable f32 values."""
    r = state_rng(seq, layer, 2)
    k = bf16_round(r.normal(0.0, 1.0, size=(shape.kv_heads, n_tokens, shape.head_dim)).astype(np.float32))
    v = bf16_round(r.normal(0.0, 1.0, size=(shape.kv_heads, n_tokens, shape.head_dim)).astype(np.float32))
    return k, v


def seeded_tokens(n: int, vocab: int, seed: int = 2) -> np.ndarray:
    return np.random.Generator(np.random.PCG64(seed)).integers(0, vocab, size=n).astype(np.int32)
