"""ane_infer_b200 -- B200 decode backend for thebasedcapital/ane-infer's Qwen3.5 hybrid model.

Python host side of the C ABI in include/ab2.h (libab2.so, built for sm_100a by build.py).
The names mirror the reference's Rust interface of the decode path:

    reference (crates/...)                              here
    GpuContext::new + upload_model_weights + HybridCache DecodeContext(gguf_bytes, ...)
    encode_full_token_gpu / qwen35_forward_token         DecodeContext.decode_step(tokens)
    deltanet_decode_step / full_attn_decode_step         DecodeContext.mixer_layer(layer, slot, x)
    ffn_forward                                          DecodeContext.ffn_layer(layer, x)
    Q8Tensor::from_raw                                   Q8Tensor.from_raw(blocks, ne0, ne1)
    q8_gemv                                              q8_gemv(w, x, y)
    dequant_q8_0_block                                   q8_dequant(blocks, out)
    GgufFile::parse + Qwen35Config::from_gguf            inspect_gguf(gguf_bytes)

There is no CPU fallback: if libab2.so is missing or no GPU is present the calls raise.
Device-pointer arguments accept torch CUDA tensors (anything with .data_ptr()) or ints.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

__all__ = ["Ab2Error", "DecodeContext", "Q8Tensor", "inspect_gguf", "q8_gemv", "q8_dequant", "gated_delta",
           "attn_decode", "library_path", "load_library"]

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

AB2_ERR = {-1: "ARG", -2: "FORMAT", -3: "SHAPE", -4: "OOM", -5: "CUDA", -6: "CAPACITY", -7: "DEVICE"}


class Ab2Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"ab2 error {code} ({AB2_ERR.get(code, '?')}): {msg}")
        self.code = code


class Ab2Options(C.Structure):
    _fields_ = [("kv_bf16", C.c_int32), ("rope_dims", C.c_int32), ("exact_max_batch", C.c_int32),
                ("reserved", C.c_int32 * 5)]


class Ab2Config(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("dim", "ffn", "n_layers", "vocab", "n_heads", "n_kv_heads", "head_dim",
                                         "dn_heads", "dn_state", "conv_kernel", "n_dn", "n_attn", "max_batch",
                                         "max_ctx", "context_length")] + \
               [("rope_base", C.c_float), ("eps", C.c_float), ("kv_bf16", C.c_int32), ("rope_dims", C.c_int32)]

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


# every exported symbol of include/ab2.h with its ctypes signature
_vp, _i64, _i32, _u64 = C.c_void_p, C.c_int64, C.c_int32, C.c_uint64
_fp = C.POINTER(C.c_float)
SIGNATURES = {
    "ab2_last_error": (C.c_char_p, []),
    "ab2_gguf_inspect": (C.c_int, [_vp, _u64, C.POINTER(Ab2Config)]),
    "ab2_create": (C.c_int, [_vp, _u64, C.c_int, C.c_int, C.c_int, C.POINTER(Ab2Options), C.POINTER(_vp)]),
    "ab2_destroy": (None, [_vp]),
    "ab2_tp_unique_id": (C.c_int, [_vp, _u64]),
    "ab2_create_tp": (C.c_int, [_vp, _u64, C.c_int, C.c_int, C.c_int, C.POINTER(Ab2Options), C.c_int, C.c_int, _vp,
                                _u64, C.POINTER(_vp)]),
    "ab2_get_tp": (C.c_int, [_vp, C.POINTER(C.c_int32)]),
    "ab2_get_config": (C.c_int, [_vp, C.POINTER(Ab2Config)]),
    "ab2_layer_is_deltanet": (C.c_int, [_vp, C.c_int]),
    "ab2_reset_slot": (C.c_int, [_vp, C.c_int]),
    "ab2_set_pos": (C.c_int, [_vp, C.c_int, _i64]),
    "ab2_get_pos": (C.c_int, [_vp, C.c_int, C.POINTER(_i64)]),
    "ab2_set_dn_state": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp]),
    "ab2_get_dn_state": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp]),
    "ab2_set_kv": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp, _i64]),
    "ab2_get_kv": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp, _i64]),
    "ab2_seed_state": (C.c_int, [_vp, _u64, C.c_int, _i64, C.c_float, C.c_float, C.c_float]),
    "ab2_decode_step": (C.c_int, [_vp, _vp, C.c_int, _vp, _vp]),
    "ab2_decode_step_device": (C.c_int, [_vp, _vp, C.c_int, _vp, _vp, _vp]),
    "ab2_prefill": (C.c_int, [_vp, C.c_int, _vp, _i64, _vp, _vp]),
    "ab2_sync": (C.c_int, [_vp]),
    "ab2_op_error": (C.c_int, [C.POINTER(C.c_uint32)]),
    "ab2_debug_arm_wait_timeout": (C.c_int, [C.c_int, C.c_int, C.c_uint32]),
    "ab2_launches_per_step": (C.c_int, [_vp, C.c_int, C.POINTER(_i64)]),
    "ab2_profile": (C.c_int, [_vp, C.c_int]),
    "ab2_profile_read": (C.c_int, [_vp, C.POINTER(C.c_double), C.POINTER(_i64)]),
    "ab2_step_graph": (C.c_int, [_vp, C.c_int]),
    "ab2_step_graph_captures": (C.c_int, [_vp, C.POINTER(_i64)]),
    "ab2_mixer_layer": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp]),
    "ab2_ffn_layer": (C.c_int, [_vp, C.c_int, _vp, _vp]),
    "ab2_q8_create": (C.c_int, [_vp, _i64, _i64, C.c_int, C.POINTER(_vp)]),
    "ab2_q8_destroy": (None, [_vp]),
    "ab2_q8_gemv": (C.c_int, [_vp, _vp, C.c_int, _vp, _vp]),
    "ab2_q8_gemv_noalloc": (C.c_int, [_vp, _vp, C.c_int, _vp, _vp]),
    "ab2_q8_unpack": (C.c_int, [_vp, _vp, _vp]),
    "ab2_q8_dequant": (C.c_int, [_vp, _i64, _vp, _vp]),
    "ab2_gated_delta": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp]),
    "ab2_attn_decode": (C.c_int, [_vp, _vp, _vp, _i64, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _vp,
                                  _vp, C.c_float, C.c_int, C.c_int, _vp, _vp]),
}


def library_path() -> str:
    return os.path.join(_HERE, "libab2.so")


def load_library():
    """Load libab2.so from this package directory; raise if it has not been built."""
    global _LIB
    if _LIB is None:
        path = library_path()
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing: build it with `python ane-infer_b200/build.py`")
        lib = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def _check(rc: int):
    if rc != 0:
        raise Ab2Error(rc, load_library().ab2_last_error().decode())


def _host(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _hp(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _dp(t):
    """Device pointer of a torch tensor / int / None."""
    if t is None:
        return None
    if isinstance(t, int):
        return C.c_void_p(t)
    return C.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        return None
    if isinstance(stream, int):
        return C.c_void_p(stream)
    return C.c_void_p(stream.cuda_stream)


TP_ID_BYTES = 128


def tp_unique_id() -> bytes:
    """A fresh id for one head-parallel split (made on one rank, passed to every rank)."""
    buf = (C.c_uint8 * TP_ID_BYTES)()
    _check(load_library().ab2_tp_unique_id(C.cast(buf, C.c_void_p), TP_ID_BYTES))
    return bytes(buf)


def inspect_gguf(gguf) -> dict:
    """Parse GGUF bytes on the host and return the derived model configuration."""
    buf = _host(gguf, np.uint8)
    cfg = Ab2Config()
    _check(load_library().ab2_gguf_inspect(_hp(buf), buf.size, C.byref(cfg)))
    return cfg.as_dict()


class DecodeContext:
    """A model resident on one GPU plus per-slot decode state for up to max_batch sequences."""

    def __init__(self, gguf, device: int = 0, max_batch: int = 1, max_ctx: int = 4096, kv_bf16: bool = True,
                 rope_dims: int = 0, exact_max_batch: int = 0, tp=None):
        """exact_max_batch: steps of at most this many sequences multiply the Q8_0 weights exactly
        (mma.sync); larger steps use the tcgen05 path with f16 operands. 0 (default) = 1; -1:
        every step on tcgen05, one sequence included.
        tp: (rank, world, id) to join a head-parallel split of `world` GPUs (id from
        tp_unique_id(), the same on every rank); returns once every rank has joined."""
        lib = load_library()
        buf = _host(gguf, np.uint8)
        opt = Ab2Options(int(kv_bf16), int(rope_dims), int(exact_max_batch))
        self.exact_max_batch = 0 if int(exact_max_batch) < 0 else int(exact_max_batch) or 1
        h = C.c_void_p()
        if tp is None:
            _check(lib.ab2_create(_hp(buf), buf.size, device, max_batch, max_ctx, C.byref(opt), C.byref(h)))
        else:
            rank, world, tp_id = tp
            idb = None if tp_id is None else (C.c_uint8 * len(tp_id)).from_buffer_copy(tp_id)
            _check(lib.ab2_create_tp(_hp(buf), buf.size, device, max_batch, max_ctx, C.byref(opt), int(rank),
                                     int(world), None if idb is None else C.cast(idb, C.c_void_p),
                                     0 if tp_id is None else len(tp_id), C.byref(h)))
        self._h = h
        cfg = Ab2Config()
        _check(lib.ab2_get_config(h, C.byref(cfg)))
        self.config = cfg.as_dict()
        self.layer_is_deltanet = [bool(lib.ab2_layer_is_deltanet(h, l)) for l in range(self.config["n_layers"])]

    def split(self) -> dict:
        """This context's part of a head-parallel split (the whole model when not split)."""
        v = (C.c_int32 * 6)()
        _check(load_library().ab2_get_tp(self._h, v))
        return {"rank": v[0], "world": v[1], "dn_h0": v[2], "dn_heads": v[3], "kv_h0": v[4], "kv_heads": v[5]}

    def tensor_core_gemm(self, batch: int) -> bool:
        """Whether a step of `batch` sequences runs its Q8_0 GEMMs on the tcgen05 path."""
        return batch > self.exact_max_batch

    def close(self):
        if getattr(self, "_h", None):
            load_library().ab2_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # -- state -----------------------------------------------------------------------------
    def reset_slot(self, slot: int):
        _check(load_library().ab2_reset_slot(self._h, slot))

    def set_pos(self, slot: int, pos: int):
        _check(load_library().ab2_set_pos(self._h, slot, pos))

    def get_pos(self, slot: int) -> int:
        v = C.c_int64()
        _check(load_library().ab2_get_pos(self._h, slot, C.byref(v)))
        return v.value

    def set_dn_state(self, layer: int, slot: int, rec=None, conv=None):
        r = None if rec is None else _host(rec, np.float32)
        c = None if conv is None else _host(conv, np.float32)
        _check(load_library().ab2_set_dn_state(self._h, layer, slot, None if r is None else _hp(r),
                                               None if c is None else _hp(c)))

    def get_dn_state(self, layer: int, slot: int):
        cfg = self.config
        # zeros: a head-parallel rank fills its own heads' part only
        rec = np.zeros((cfg["dn_heads"], cfg["dn_state"], cfg["dn_state"]), dtype=np.float32)
        conv = np.zeros((3 * cfg["dim"], cfg["conv_kernel"]), dtype=np.float32)
        _check(load_library().ab2_get_dn_state(self._h, layer, slot, _hp(rec), _hp(conv)))
        return rec, conv

    def set_kv(self, layer: int, slot: int, k, v):
        k = _host(k, np.float32)
        v = _host(v, np.float32)
        _check(load_library().ab2_set_kv(self._h, layer, slot, _hp(k), _hp(v), k.shape[1]))

    def get_kv(self, layer: int, slot: int, n_tokens: int):
        cfg = self.config
        k = np.zeros((cfg["n_kv_heads"], n_tokens, cfg["head_dim"]), dtype=np.float32)
        v = np.zeros_like(k)
        _check(load_library().ab2_get_kv(self._h, layer, slot, _hp(k), _hp(v), n_tokens))
        return k, v

    def seed_state(self, seed: int, n_slots: int, n_tokens: int, dn_std=0.1, conv_std=1.0, kv_std=1.0):
        _check(load_library().ab2_seed_state(self._h, seed, n_slots, n_tokens, dn_std, conv_std, kv_std))

    # -- decode ----------------------------------------------------------------------------
    def decode_step(self, tokens, want_logits: bool = True):
        """One step for slots [0, len(tokens)); returns (logits [B][vocab] or None, next ids [B])."""
        t = _host(tokens, np.int32).reshape(-1)
        B = t.size
        nxt = np.empty(B, dtype=np.int32)
        logits = np.empty((B, self.config["vocab"]), dtype=np.float32) if want_logits else None
        _check(load_library().ab2_decode_step(self._h, _hp(t), B, None if logits is None else _hp(logits),
                                              _hp(nxt)))
        return logits, nxt

    def prefill(self, slot: int, tokens, want_logits: bool = True):
        """Run a prompt through slot `slot` from its position on (steps of 128 tokens on the
        GPU, 64 with exact_max_batch 64); returns (logits of the last token [vocab] or None,
        its argmax)."""
        t = _host(tokens, np.int32).reshape(-1)
        nxt = np.zeros(1, dtype=np.int32)
        logits = np.empty(self.config["vocab"], dtype=np.float32) if want_logits else None
        _check(load_library().ab2_prefill(self._h, slot, _hp(t), t.size, None if logits is None else _hp(logits),
                                          _hp(nxt)))
        return logits, int(nxt[0])

    def decode_step_device(self, tokens_dev, batch: int, logits_dev=None, next_dev=None, stream=None):
        _check(load_library().ab2_decode_step_device(self._h, _dp(tokens_dev), batch, _dp(logits_dev),
                                                     _dp(next_dev), _stream(stream)))

    def sync(self):
        """Wait for queued device work; raises if a tensor-core pipeline wait timed out."""
        _check(load_library().ab2_sync(self._h))

    def launches_per_step(self, batch: int) -> int:
        v = C.c_int64()
        _check(load_library().ab2_launches_per_step(self._h, batch, C.byref(v)))
        return v.value

    def step_graph(self, enable: bool):
        """Replay decode steps from captured CUDA graphs (one per launch plan)."""
        _check(load_library().ab2_step_graph(self._h, int(enable)))

    def step_graph_captures(self) -> int:
        v = C.c_int64()
        _check(load_library().ab2_step_graph_captures(self._h, C.byref(v)))
        return v.value

    def profile(self, enable: bool):
        _check(load_library().ab2_profile(self._h, int(enable)))

    def profile_read(self) -> dict:
        ms = (C.c_double * 4)()
        n = (C.c_int64 * 4)()
        _check(load_library().ab2_profile_read(self._h, ms, n))
        names = ("attention", "deltanet", "q8_gemm", "other")
        return {names[i]: {"ms": ms[i], "launches": n[i]} for i in range(4)}

    # -- per-layer parity entry points -----------------------------------------------------
    def mixer_layer(self, layer: int, slot: int, x) -> np.ndarray:
        x = _host(x, np.float32)
        out = np.empty(self.config["dim"], dtype=np.float32)
        _check(load_library().ab2_mixer_layer(self._h, layer, slot, _hp(x), _hp(out)))
        return out

    def ffn_layer(self, layer: int, x) -> np.ndarray:
        x = _host(x, np.float32)
        out = np.empty(self.config["dim"], dtype=np.float32)
        _check(load_library().ab2_ffn_layer(self._h, layer, _hp(x), _hp(out)))
        return out


class Q8Tensor:
    """A packed Q8_0 weight on a GPU (Q8Tensor::from_raw, crates/engine/src/q8_gemv.rs:33)."""

    def __init__(self, blocks, m: int, n: int, device: int = 0):
        buf = _host(blocks, np.uint8)
        if buf.size != m * (n // 32) * 34:
            raise Ab2Error(-3, f"Quant size mismatch: got {buf.size}, expected {m * (n // 32) * 34}")
        h = C.c_void_p()
        _check(load_library().ab2_q8_create(_hp(buf), m, n, device, C.byref(h)))
        self._h, self.m, self.n = h, m, n

    @classmethod
    def from_raw(cls, data, ne0: int, ne1: int, device: int = 0) -> "Q8Tensor":
        return cls(data, ne1, ne0, device)

    def unpack(self, out, stream=None):
        _check(load_library().ab2_q8_unpack(self._h, _dp(out), _stream(stream)))

    def __del__(self):
        if getattr(self, "_h", None):
            load_library().ab2_q8_destroy(self._h)
            self._h = None


def q8_gemv(w: Q8Tensor, x, y, batch: int = 1, stream=None):
    """y[b][:] = W x[b][:] on device buffers (f32 [batch][n] -> [batch][m])."""
    _check(load_library().ab2_q8_gemv(w._h, _dp(x), batch, _dp(y), _stream(stream)))


def q8_gemv_noalloc(w: Q8Tensor, x, y, batch: int = 1, stream=None):
    """q8_gemv for batch 1..8 with scratch in the library's fixed device array (no device
    allocation); calls that can overlap on the device share that array and race."""
    _check(load_library().ab2_q8_gemv_noalloc(w._h, _dp(x), batch, _dp(y), _stream(stream)))


def op_error() -> int:
    """Synchronise the device; return and clear the op-level tensor-core error word (0 = ok)."""
    v = C.c_uint32()
    _check(load_library().ab2_op_error(C.byref(v)))
    return v.value


# kernel families for debug_arm_wait_timeout
WAIT_TEST_GEMM, WAIT_TEST_ATTENTION, WAIT_TEST_DELTANET = 1, 2, 3


def debug_arm_wait_timeout(which: int, copy_index: int, wait_ns: int):
    """Test hook: the next launch of kernel family `which` (not under stream capture) leaves
    its asynchronous copy number `copy_index` (per CTA) unissued and bounds its waits at
    `wait_ns`, so those waits expire and the kernel reports its error bit and returns.
    wait_ns=0 disarms."""
    _check(load_library().ab2_debug_arm_wait_timeout(int(which), int(copy_index), int(wait_ns)))


def q8_dequant(blocks, n_blocks: int, out, stream=None):
    _check(load_library().ab2_q8_dequant(_dp(blocks), n_blocks, _dp(out), _stream(stream)))


def gated_delta(S, q, k, v, beta, decay, o, B: int, H: int, stream=None):
    """Gated delta rule in place on S [B][H][128][128]; q/k/v bf16 bits (int16/uint16 tensors)."""
    _check(load_library().ab2_gated_delta(_dp(S), _dp(q), _dp(k), _dp(v), _dp(beta), _dp(decay), B, H, 128, 128,
                                          _dp(o), _stream(stream)))


def attn_decode(proj, k_cache, v_cache, cap: int, pos, B: int, Hq: int, Hkv: int, hd: int, kv_bf16: bool,
                q_norm, k_norm, rope_base: float, rope_dims: int, max_pos: int, out, stream=None):
    _check(load_library().ab2_attn_decode(_dp(proj), _dp(k_cache), _dp(v_cache), cap, _dp(pos), B, Hq, Hkv, hd,
                                          int(kv_bf16), _dp(q_norm), _dp(k_norm), float(rope_base), rope_dims,
                                          max_pos, _dp(out), _stream(stream)))
