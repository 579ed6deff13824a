"""CPU: libab2.so loads, exports every entry point of include/ab2.h, and its host-side GGUF
parsing returns the right configuration and the documented error codes."""
import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "ab2.h")


@pytest.fixture(scope="module")
def lib(pkg):
    if not os.path.exists(pkg.library_path()):
        import importlib.util
        spec = importlib.util.spec_from_file_location("ab2_build", os.path.join(ROOT, "ane-infer_b200", "build.py"))
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        m.build()
    return pkg.load_library()


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ab2_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "ab2_create" in syms and "ab2_decode_step" in syms and len(syms) >= 25


def test_library_exports_every_declared_symbol(lib, pkg):
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert set(declared_symbols()) == set(pkg.SIGNATURES), "ctypes signatures out of sync with ab2.h"


def test_build_targets_sm100a():
    import importlib.util
    spec = importlib.util.spec_from_file_location("ab2_build", os.path.join(ROOT, "ane-infer_b200", "build.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    assert m.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_inspect_tiny(pkg, tiny_gguf, synth):
    c = pkg.inspect_gguf(tiny_gguf)
    s = synth.tiny_shape()
    assert (c["dim"], c["n_layers"], c["vocab"], c["ffn"]) == (s.dim, s.n_layers, s.vocab, s.ffn)
    assert (c["n_heads"], c["n_kv_heads"], c["head_dim"]) == (s.attn_heads, s.kv_heads, s.head_dim)
    assert (c["dn_heads"], c["dn_state"], c["conv_kernel"]) == (s.dn_heads, s.dn_state, s.conv_kernel)
    assert (c["n_dn"], c["n_attn"]) == (3, 1)
    assert c["rope_base"] == pytest.approx(1e7) and c["eps"] == pytest.approx(1e-6)


def test_inspect_2b_shape_header_only(pkg, synth):
    # metadata + tensor infos are enough for inspect; build a header-only GGUF of the 2B shape
    s = synth.shape_2b()
    g = synth.GgufBuilder()
    a = "qwen35"
    g.meta.string("general.architecture", a)
    g.meta.u32(f"{a}.embedding_length", s.dim)
    g.meta.u32(f"{a}.block_count", s.n_layers)
    g.meta.u32(f"{a}.feed_forward_length", s.ffn)
    g.meta.u32(f"{a}.attention.head_count", s.attn_heads)
    g.meta.u32(f"{a}.attention.head_count_kv", s.kv_heads)
    g.meta.u32(f"{a}.attention.key_length", s.head_dim)
    g.meta.str_array("tokenizer.ggml.tokens", ["x"] * s.vocab)
    for l in range(s.n_layers):
        if not s.layer_is_attn(l):
            g.add_f32(f"blk.{l}.ssm_a", np.zeros(16, np.float32))
    c = pkg.inspect_gguf(g.tobytes())
    assert (c["n_dn"], c["n_attn"], c["vocab"], c["head_dim"]) == (18, 6, 151936, 256)
    # defaults of Qwen35Config::from_gguf (crates/engine/src/model.rs:72-76)
    assert (c["dn_heads"], c["dn_state"], c["conv_kernel"]) == (16, 128, 4)
    assert c["rope_base"] == pytest.approx(1e4)


def _err(pkg, gguf):
    with pytest.raises(pkg.Ab2Error) as ei:
        pkg.inspect_gguf(gguf)
    return ei.value.code


def test_malformed_gguf_errors(pkg, tiny_gguf):
    g = np.array(tiny_gguf, copy=True)
    assert _err(pkg, g[:3]) == -2                      # truncated magic
    bad = g.copy()
    bad[0] = ord("X")
    assert _err(pkg, bad) == -2                        # bad magic
    v1 = g.copy()
    v1[4:8] = np.frombuffer(struct.pack("<I", 1), np.uint8)
    assert _err(pkg, v1) == -2                         # unsupported version
    assert _err(pkg, g[:200]) == -2                    # truncated metadata
    assert _err(pkg, g[: g.size // 2]) == -2           # tensors outside the file


def test_wrong_architecture(pkg, synth):
    g = synth.GgufBuilder()
    g.meta.string("general.architecture", "llama")
    assert _err(pkg, g.tobytes()) == -2


def test_unsupported_ggml_type(pkg, synth):
    g = synth.GgufBuilder()
    g.meta.string("general.architecture", "qwen35")
    t = synth._Tensor("blk.0.x", (32,), 30, np.zeros(64, np.uint8))   # BF16 is not accepted (parser.rs:93-108)
    g.tensors.append(t)
    assert _err(pkg, g.tobytes()) == -2


def _edit_tensor_info(gguf, name, new_name=None, dims=None):
    """Copy of GGUF bytes with one tensor's info edited in place: its name (same length) or
    its dims (same number of dims)."""
    b = bytearray(np.asarray(gguf, dtype=np.uint8).tobytes())
    key = name.encode()
    i = b.find(struct.pack("<Q", len(key)) + key)
    assert i >= 0, name
    j = i + 8 + len(key)
    if new_name is not None:
        assert len(new_name) == len(name)
        b[i + 8:j] = new_name.encode()
    if dims is not None:
        assert struct.unpack_from("<I", b, j)[0] == len(dims)
        for k, d in enumerate(dims):
            struct.pack_into("<Q", b, j + 4 + 8 * k, d)
    return np.frombuffer(bytes(b), dtype=np.uint8)


def _create_err(pkg, gguf, **kw):
    with pytest.raises(pkg.Ab2Error) as ei:
        pkg.DecodeContext(gguf, max_batch=1, max_ctx=8, **kw)
    return ei.value.code, str(ei.value)


# The model file is checked on the host before any device work, so these fail the same way
# with or without a GPU.
def test_create_rejects_wrong_tensor_shape(pkg, tiny_gguf):
    # ffn_down is D x F (GGUF dims F, D); transposed dims keep the byte size
    code, msg = _create_err(pkg, _edit_tensor_info(tiny_gguf, "blk.2.ffn_down.weight", dims=(1024, 3072)))
    assert code == -3 and "blk.2.ffn_down.weight: shape 3072x1024, expected 1024x3072" in msg
    code, msg = _create_err(pkg, _edit_tensor_info(tiny_gguf, "blk.0.ssm_a", dims=(4,)))
    assert code == -3 and "blk.0.ssm_a: 4 elements, expected 8" in msg


def test_create_rejects_missing_tensor(pkg, tiny_gguf):
    code, msg = _create_err(pkg, _edit_tensor_info(tiny_gguf, "blk.3.attn_k_norm.weight",
                                                   new_name="blk.3.attn_k_xxxx.weight"))
    assert code == -2 and "tensor not found: blk.3.attn_k_norm.weight" in msg


def test_create_rejects_unsupported_shapes(pkg, tiny_gguf, synth):
    g = synth.build_model_gguf(synth.HybridShape(head_dim=64, attn_heads=8, kv_heads=2), seed=1)
    code, msg = _create_err(pkg, g)
    assert code == -3 and "head_dim must be 128 or 256" in msg
    code, msg = _create_err(pkg, tiny_gguf, rope_dims=3)
    assert code == -3 and "rope_dims" in msg


def test_create_without_gpu_fails_cleanly(pkg, tiny_gguf):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(pkg.Ab2Error) as ei:
        pkg.DecodeContext(tiny_gguf, max_batch=1, max_ctx=64)
    assert ei.value.code == -7


def test_bad_arguments(pkg, lib):
    assert lib.ab2_get_config(None, None) == -1
    assert lib.ab2_gguf_inspect(None, 0, None) == -1
    assert "null" in lib.ab2_last_error().decode()
    h = C.c_void_p()
    assert lib.ab2_create(None, 0, 0, 0, 16, None, C.byref(h)) == -1   # max_batch 0


def test_wait_timeout_hook_arguments(pkg):
    """The test hook that arms one pipelined-kernel launch to let its waits expire checks its
    arguments on the host (no device work), and disarming is always accepted."""
    for args in ((0, 0, 1000), (4, 0, 1000), (1, -1, 1000), (1, 0, 10)):
        with pytest.raises(pkg.Ab2Error) as ei:
            pkg.debug_arm_wait_timeout(*args)
        assert ei.value.code == -1
    for which in (1, 2, 3):
        pkg.debug_arm_wait_timeout(which, 0, 0)


def test_create_rejects_bad_exact_max_batch(pkg, tiny_gguf):
    """exact_max_batch is checked before any device work."""
    for bad in (-2, 65):
        with pytest.raises(pkg.Ab2Error) as ei:
            pkg.DecodeContext(tiny_gguf, max_batch=1, max_ctx=8, exact_max_batch=bad)
        assert ei.value.code == -1 and "exact_max_batch" in str(ei.value)


def test_create_tp_rejects_bad_arguments_on_the_host(pkg, tiny_gguf):
    """The head-parallel entry point checks rank, world and id before it loads NCCL or touches
    a device."""
    for tp, what in (((2, 2, bytes(128)), "tp_rank"), ((-1, 2, bytes(128)), "tp_rank"),
                     ((0, 9, bytes(128)), "tp_world"), ((0, 0, bytes(128)), "tp_world"),
                     ((0, 2, None), "tp_id"), ((1, 2, bytes(64)), "tp_id")):
        with pytest.raises(pkg.Ab2Error) as ei:
            pkg.DecodeContext(tiny_gguf, max_batch=1, max_ctx=8, tp=tp)
        assert ei.value.code == -1 and what in str(ei.value), (tp, str(ei.value))
    buf = (C.c_uint8 * 64)()
    assert pkg.load_library().ab2_tp_unique_id(C.cast(buf, C.c_void_p), 64) == -1  # needs 128 bytes
