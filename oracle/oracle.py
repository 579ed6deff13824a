"""ctypes wrapper of liboracle.so, the CPU restatement of the reference decode path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs, never by the product package.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


class OracleConfig(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads",
                                         "head_dim", "vocab", "max_seq")] + \
               [("rope_base", C.c_float), ("eps", C.c_float)] + \
               [(n, C.c_int64) for n in ("interval", "ssm_state", "conv_kernel", "ssm_groups",
                                         "ssm_inner", "n_dn", "n_attn")]


def build() -> str:
    """Compile liboracle.so with the committed Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return os.path.join(_HERE, "liboracle.so")


def lib():
    global _LIB
    if _LIB is not None:
        return _LIB
    path = os.path.join(_HERE, "liboracle.so")
    if not os.path.exists(path):
        build()
    L = C.CDLL(path)
    vp, i64, i32 = C.c_void_p, C.c_int64, C.c_int32
    sig = {
        "oracle_last_error": (C.c_char_p, []),
        "oracle_set_threads": (None, [C.c_int]),
        "oracle_max_threads": (C.c_int, []),
        "oracle_f16_to_f32": (C.c_float, [C.c_uint16]),
        "oracle_q8_dequant": (None, [u8p, i64, f32p]),
        "oracle_q8_gemv": (C.c_int, [u8p, i64, i64, f32p, f32p]),
        "oracle_q8_gemv_scalar": (C.c_int, [u8p, i64, i64, f32p, f32p]),
        "oracle_q8_gemv_f16": (C.c_int, [u8p, i64, i64, f32p, f32p]),
        "oracle_greedy": (i32, [f32p, i64]),
        "oracle_gated_delta": (None, [f32p, f32p, f32p, f32p, f32p, f32p, i64, i64, i64, i64, f32p]),
        "oracle_attn_op": (C.c_int, [f32p, f32p, f32p, f32p, f32p, f32p, i64, i64, i64, i64, i64,
                                     vp, vp, C.c_float, i64, C.c_int, f32p]),
        "oracle_kv_new": (vp, [i64, i64, i64, f32p, f32p]),
        "oracle_kv_free": (None, [vp]),
        "oracle_attn_op_kv": (C.c_int, [vp, f32p, f32p, f32p, f32p, i64, i64, C.c_float, i64, C.c_int, f32p]),
        "oracle_model_load": (vp, [u8p, i64, i64]),
        "oracle_model_free": (None, [vp]),
        "oracle_model_config": (None, [vp, C.POINTER(OracleConfig)]),
        "oracle_layer_is_dn": (C.c_int, [vp, i64]),
        "oracle_seq_new": (vp, [vp, C.c_int]),
        "oracle_seq_free": (None, [vp]),
        "oracle_seq_set_pos": (None, [vp, i64]),
        "oracle_seq_get_pos": (i64, [vp]),
        "oracle_seq_dn_state": (C.c_int, [vp, i64, vp, vp, C.c_int]),
        "oracle_seq_kv": (C.c_int, [vp, i64, vp, vp, i64, C.c_int]),
        "oracle_forward": (C.c_int, [vp, vp, i32, f32p]),
        "oracle_mixer": (C.c_int, [vp, vp, i64, f32p, f32p]),
        "oracle_ffn": (C.c_int, [vp, i64, f32p, f32p]),
        "oracle_embedding_row": (C.c_int, [vp, i32, f32p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = L
    return L


def _err() -> str:
    return lib().oracle_last_error().decode()


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def set_threads(n: int):
    lib().oracle_set_threads(int(n))


def q8_dequant(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    nb = blocks.size // 34
    out = np.empty(nb * 32, dtype=np.float32)
    lib().oracle_q8_dequant(blocks, nb, out)
    return out


def q8_gemv(blocks: np.ndarray, m: int, n: int, x: np.ndarray, scalar: bool = False,
            f16_operands: bool = False) -> np.ndarray:
    """y = W x (q8_gemv.rs:130); f16_operands: the tensor-core GEMM's declared rounding instead."""
    y = np.empty(m, dtype=np.float32)
    fn = lib().oracle_q8_gemv_f16 if f16_operands else (lib().oracle_q8_gemv_scalar if scalar else lib().oracle_q8_gemv)
    if fn(np.ascontiguousarray(blocks, dtype=np.uint8), m, n, np.ascontiguousarray(x, dtype=np.float32), y):
        raise RuntimeError(_err())
    return y


def greedy(logits: np.ndarray) -> int:
    return int(lib().oracle_greedy(np.ascontiguousarray(logits, dtype=np.float32), logits.size))


def gated_delta(S, q, k, v, beta, decay):
    """Returns (o, S_new); S is [B][H][dk][dv], q/k [B][H][dk], v [B][H][dv], beta/decay [B][H]."""
    S = np.array(S, dtype=np.float32, order="C", copy=True)
    B, H, dk, dv = S.shape
    o = np.empty((B, H, dv), dtype=np.float32)
    c = lambda a: np.ascontiguousarray(a, dtype=np.float32)
    lib().oracle_gated_delta(S, c(q), c(k), c(v), c(beta), c(decay), B, H, dk, dv, o)
    return o, S


def attn_op(q, gate, k_new, v_new, k_cache, v_cache, pos, rope_base, rotary_dim,
            q_norm=None, k_norm=None, kv_bf16=False):
    """One sequence: returns (out [Hq][hd], k_cache, v_cache) with caches [Hkv][cap][hd]."""
    q = np.array(q, dtype=np.float32, copy=True)
    k_new = np.array(k_new, dtype=np.float32, copy=True)
    kc = np.array(k_cache, dtype=np.float32, copy=True)
    vc = np.array(v_cache, dtype=np.float32, copy=True)
    Hkv, cap, hd = kc.shape
    Hq = q.size // hd
    out = np.empty(Hq * hd, dtype=np.float32)
    qn = None if q_norm is None else np.ascontiguousarray(q_norm, dtype=np.float32)
    kn = None if k_norm is None else np.ascontiguousarray(k_norm, dtype=np.float32)
    rc = lib().oracle_attn_op(q.reshape(-1), np.ascontiguousarray(gate, dtype=np.float32).reshape(-1),
                              k_new.reshape(-1), np.ascontiguousarray(v_new, dtype=np.float32).reshape(-1),
                              kc, vc, cap, pos, Hq, Hkv, hd, _ptr(qn), _ptr(kn), float(rope_base),
                              rotary_dim, int(kv_bf16), out)
    if rc:
        raise RuntimeError(_err())
    return out.reshape(Hq, hd), kc, vc


class KvOp:
    """attn_op without q/k norms over a cache kept across calls ([Hkv][cap][hd], copied in
    once), for timing the op: each call appends at pos and attends over pos + 1 tokens."""

    def __init__(self, k_cache, v_cache):
        kc = np.ascontiguousarray(k_cache, dtype=np.float32)
        vc = np.ascontiguousarray(v_cache, dtype=np.float32)
        self.n_kv, self.cap, self.hd = kc.shape
        self._h = lib().oracle_kv_new(self.n_kv, self.hd, self.cap, kc, vc)

    def __call__(self, q, gate, k_new, v_new, pos, rope_base, rotary_dim, kv_bf16=False):
        q = np.array(q, dtype=np.float32, copy=True).reshape(-1)
        out = np.empty(q.size, dtype=np.float32)
        rc = lib().oracle_attn_op_kv(self._h, q, np.ascontiguousarray(gate, dtype=np.float32).reshape(-1),
                                     np.array(k_new, dtype=np.float32, copy=True).reshape(-1),
                                     np.ascontiguousarray(v_new, dtype=np.float32).reshape(-1), pos,
                                     q.size // self.hd, float(rope_base), rotary_dim, int(kv_bf16), out)
        if rc:
            raise RuntimeError(_err())
        return out.reshape(-1, self.hd)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().oracle_kv_free(self._h)
            self._h = None


class Model:
    """Reference model (Qwen35ModelWeights + loader) over GGUF bytes."""

    def __init__(self, gguf: np.ndarray, ctx_cap: int = 0):
        """ctx_cap=0 keeps the reference 4096 context cap (model.rs:50); >0 replaces it."""
        self._bytes = np.ascontiguousarray(gguf, dtype=np.uint8)
        self.h = lib().oracle_model_load(self._bytes, self._bytes.size, int(ctx_cap))
        if not self.h:
            raise RuntimeError(_err())
        cfg = OracleConfig()
        lib().oracle_model_config(self.h, C.byref(cfg))
        self.cfg = {n: getattr(cfg, n) for n, _ in OracleConfig._fields_}
        self.layer_is_dn = [bool(lib().oracle_layer_is_dn(self.h, l)) for l in range(self.cfg["n_layers"])]

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_model_free(self.h)
            self.h = None

    def new_seq(self, kv_bf16: bool = False) -> "Seq":
        return Seq(self, kv_bf16)

    def ffn(self, layer: int, x: np.ndarray) -> np.ndarray:
        out = np.empty(self.cfg["dim"], dtype=np.float32)
        lib().oracle_ffn(self.h, layer, np.ascontiguousarray(x, dtype=np.float32), out)
        return out

    def embedding_row(self, token: int) -> np.ndarray:
        out = np.empty(self.cfg["dim"], dtype=np.float32)
        lib().oracle_embedding_row(self.h, int(token), out)
        return out


class Seq:
    """HybridCache for one sequence: DeltaNet/conv states, f32 KV caches, pos."""

    def __init__(self, model: Model, kv_bf16: bool):
        self.m = model
        self.h = lib().oracle_seq_new(model.h, int(kv_bf16))

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_seq_free(self.h)
            self.h = None

    @property
    def pos(self) -> int:
        return int(lib().oracle_seq_get_pos(self.h))

    @pos.setter
    def pos(self, p: int):
        lib().oracle_seq_set_pos(self.h, int(p))

    def set_dn(self, layer: int, rec=None, conv=None):
        rec = None if rec is None else np.ascontiguousarray(rec, dtype=np.float32)
        conv = None if conv is None else np.ascontiguousarray(conv, dtype=np.float32)
        if lib().oracle_seq_dn_state(self.h, layer, _ptr(rec), _ptr(conv), 1):
            raise RuntimeError(_err())

    def get_dn(self, layer: int):
        c = self.m.cfg
        rec = np.empty((c["ssm_groups"], c["ssm_state"], c["ssm_state"]), dtype=np.float32)
        conv = np.empty((3 * c["dim"], c["conv_kernel"]), dtype=np.float32)
        if lib().oracle_seq_dn_state(self.h, layer, _ptr(rec), _ptr(conv), 0):
            raise RuntimeError(_err())
        return rec, conv

    def set_kv(self, layer: int, k: np.ndarray, v: np.ndarray):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        if lib().oracle_seq_kv(self.h, layer, _ptr(k), _ptr(v), k.shape[1], 1):
            raise RuntimeError(_err())

    def get_kv(self, layer: int, n_tokens: int):
        c = self.m.cfg
        k = np.empty((c["n_kv_heads"], n_tokens, c["head_dim"]), dtype=np.float32)
        v = np.empty_like(k)
        if lib().oracle_seq_kv(self.h, layer, _ptr(k), _ptr(v), n_tokens, 0):
            raise RuntimeError(_err())
        return k, v

    def forward(self, token: int) -> np.ndarray:
        logits = np.empty(self.m.cfg["vocab"], dtype=np.float32)
        if lib().oracle_forward(self.m.h, self.h, int(token), logits):
            raise RuntimeError(_err())
        return logits

    def mixer(self, layer: int, x: np.ndarray) -> np.ndarray:
        out = np.empty(self.m.cfg["dim"], dtype=np.float32)
        if lib().oracle_mixer(self.m.h, self.h, layer, np.ascontiguousarray(x, dtype=np.float32), out):
            raise RuntimeError(_err())
        return out
