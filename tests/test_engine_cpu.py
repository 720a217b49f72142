"""Engine library checks that need no GPU: the C ABI loads and exports every
symbol include/sm_engine.h declares; synthetic models and quantizers; errors
are reported through sm_last_error without a device."""
import os
import re

import numpy as np
import pytest

import pyoracle as orc
import smotor
from conftest import ROOT, cuda_available

HEADER = os.path.join(ROOT, "include", "sm_engine.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = set(re.findall(r"^\s*(?:const\s+)?[\w]+\s*\**\s*(sm_\w+)\s*\(", src, flags=re.M))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    L = smotor.lib()
    names = declared_functions()
    assert len(names) >= 30
    for n in names:
        assert hasattr(L, n), n
        assert n in smotor.SIGNATURES, f"binding lacks {n}"
    assert L.sm_abi_version() == 2


def test_rng_seed_matches_reference_rng():
    assert smotor.rng_seed(42) == orc.Rng(42).state


@pytest.mark.parametrize("qt,bs", [(smotor.Q4_K, 256), (smotor.Q6_K, 256), (smotor.Q5_0, 32), (smotor.Q8_0, 32)])
def test_quantizer_roundtrip(qt, bs):
    rng = np.random.default_rng(qt)
    x = rng.normal(0, 1, 16 * bs).astype(np.float32)
    enc = smotor.quantize(qt, x)
    assert len(enc) == len(x) // bs * smotor.BLOCK[qt][1]
    y = orc.dequantize(qt, x.size, enc)
    # relative RMS error of a 4..8-bit block code
    rel = np.sqrt(np.mean((y - x) ** 2)) / np.sqrt(np.mean(x ** 2))
    assert rel < {smotor.Q4_K: 0.12, smotor.Q6_K: 0.03, smotor.Q5_0: 0.05, smotor.Q8_0: 0.01}[qt], rel


def test_quantizer_zero_and_constant_blocks():
    for qt, bs in ((smotor.Q4_K, 256), (smotor.Q6_K, 256), (smotor.Q5_0, 32), (smotor.Q8_0, 32)):
        z = np.zeros(bs, np.float32)
        assert not orc.dequantize(qt, bs, smotor.quantize(qt, z)).any()
        c = np.full(bs, 0.25, np.float32)
        assert np.allclose(orc.dequantize(qt, bs, smotor.quantize(qt, c)), 0.25, rtol=0.05)


def test_synth_is_deterministic_and_seeded(tmp_path):
    s = smotor.synth_spec(n_embd=256, n_layers=1, n_ff=256, vocab=300, seed=7)
    a, b = tmp_path / "a.gguf", tmp_path / "b.gguf"
    smotor.synth_write(s, str(a), threads=1)
    smotor.synth_write(s, str(b), threads=4)
    assert a.read_bytes() == b.read_bytes()
    mem = smotor.SynthBuffer(s, threads=3)
    import ctypes
    assert ctypes.string_at(mem.ptr, mem.len) == a.read_bytes()
    s.seed = 8
    smotor.synth_write(s, str(b))
    assert a.read_bytes() != b.read_bytes()


def test_synth_weights_are_normal_002(tmp_path):
    p = str(tmp_path / "w.gguf")
    smotor.synth_write(smotor.synth_spec(n_embd=512, n_layers=1, n_ff=1024, vocab=256, type_override=0), p)
    w = orc.gguf_tensor_f32(p, "blk.0.ffn_up.weight", 512 * 1024)
    assert abs(w.mean()) < 5e-4 and abs(w.std() - 0.02) < 5e-4
    assert list(orc.gguf_tensor_f32(p, "blk.0.attn_norm.weight", 512)) == [1.0] * 512


def test_preset_shapes_and_q4km_mix(tmp_path):
    s0 = smotor.synth_preset(0)
    assert (s0.n_embd, s0.n_layers, s0.n_heads, s0.n_kv_heads, s0.n_ff, s0.vocab, s0.tied, s0.qkv_bias) == \
        (896, 24, 14, 2, 4864, 151936, 1, 1)
    s2 = smotor.synth_preset(2)
    assert (s2.n_embd, s2.n_layers, s2.n_heads, s2.n_kv_heads, s2.n_ff, s2.vocab) == (3584, 28, 28, 4, 18944, 152064)
    s3 = smotor.synth_preset(3)
    assert (s3.arch, s3.n_embd, s3.n_kv_heads, s3.qkv_bias, np.float32(s3.rope_theta)) == (1, 4096, 8, 0, 5e5)
    s4 = smotor.synth_preset(4)
    assert (s4.n_embd, s4.n_layers, s4.n_heads, s4.n_ff) == (8192, 80, 64, 28672)
    # the Q4_K_M mix with config 0's fallbacks, on a 2-layer copy of its shape
    s0.n_layers, s0.vocab = 2, 512
    p = str(tmp_path / "c0.gguf")
    smotor.synth_write(s0, p)
    types = {t["name"]: t["type"] for t in orc.gguf_info(p)["tensors"]}
    assert types["token_embd.weight"] == smotor.Q8_0 and "output.weight" not in types
    assert types["blk.0.attn_q.weight"] == smotor.Q5_0 and types["blk.0.attn_v.weight"] == smotor.Q8_0
    assert types["blk.0.ffn_down.weight"] == smotor.Q6_K and types["blk.1.ffn_down.weight"] == smotor.Q4_K


def test_preset_size_config2():
    # Qwen2.5-7B shape: 4.38 GB streamed per step + the 0.45 GB embedding table
    n = smotor.synth_size(smotor.synth_preset(2))
    assert 4.75e9 < n < 4.9e9


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU error path")
def test_model_load_without_gpu_fails_cleanly(tmp_path):
    p = str(tmp_path / "t.gguf")
    smotor.synth_write(smotor.synth_spec(), p)
    with pytest.raises(smotor.EngineError) as e:
        smotor.Model.load(p)
    assert e.value.status == 5 and "CUDA" in str(e.value)


def test_model_load_errors(tmp_path):
    with pytest.raises(smotor.EngineError) as e:
        smotor.Model.load(str(tmp_path / "missing.gguf"))
    assert e.value.status == 2
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE0000")
    with pytest.raises(smotor.EngineError) as e:
        smotor.Model.load(str(bad))
    assert e.value.status == 3 and "magic" in str(e.value)


def test_binding_classes_keep_their_methods():
    import smotor
    for cls, names in ((smotor.DWeight, ("gemv", "gemv_noalloc", "gemv_status", "dequant", "nbytes", "free")),
                       (smotor.Model, ("forward_cached", "forward_sample", "decode_batch", "decode_batch_logits",
                                       "decode_run", "embedding", "generate", "free")),
                       (smotor.Cache, ("clone", "truncate", "read_kv", "free"))):
        for n in names:
            assert callable(getattr(cls, n, None)), (cls.__name__, n)
    for n in ("sample", "softmax", "expf_ref", "gemv_noalloc_status", "synth_write", "quantize"):
        assert callable(getattr(smotor, n, None)), n
