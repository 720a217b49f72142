"""CPU ORACLE — test infrastructure only.

ctypes wrapper over oracle/build/liborc.so, the C++ restatement of the
reference's CPU f32 path (s-gguf dequant + GGUF parser, s-models qwen2
forward_cached, SeqState, Sampler/Rng, generate_tokens_seeded). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may use it, and
only as the checker or the timed CPU baseline; the engine never does.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "liborc.so")


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


class orc_config(C.Structure):
    _fields_ = [("n_layers", C.c_uint64), ("n_embd", C.c_uint64), ("n_ff", C.c_uint64),
                ("n_heads", C.c_uint64), ("n_kv_heads", C.c_uint64), ("head_dim", C.c_uint64),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("vocab_size", C.c_uint64)]


class orc_gen_params(C.Structure):
    _fields_ = [("max_tokens", C.c_uint64), ("temperature", C.c_float), ("top_k", C.c_int64),
                ("top_p", C.c_float), ("has_seed", C.c_int32), ("seed", C.c_uint64)]


class orc_gen_result(C.Structure):
    _fields_ = [("n_ids", C.c_uint64), ("finish_stop", C.c_int32), ("prompt_tokens", C.c_uint64),
                ("prefix_reused", C.c_uint64), ("elapsed_secs", C.c_double)]


ON_TOKEN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint32)
MASKER = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_uint8), C.c_size_t)
STOP = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_uint32), C.c_size_t)
ON_PREFILL = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p)

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, SZ, U64 = C.c_void_p, C.c_size_t, C.c_uint64
        sig = {
            "orc_fp16_to_f32": (C.c_float, [C.c_uint16]),
            "orc_dequantize": (C.c_int, [C.c_uint32, U64, P, U64, C.POINTER(C.c_float)]),
            "orc_gguf_info_json": (C.c_long, [C.c_char_p, C.c_char_p, SZ]),
            "orc_gguf_tensor_f32": (C.c_int, [C.c_char_p, C.c_char_p, C.POINTER(C.c_float), U64, C.c_char_p, SZ]),
            "orc_model_load": (P, [C.c_char_p, C.c_int, C.c_char_p, SZ]),
            "orc_model_free": (None, [P]),
            "orc_model_set_threads": (None, [P, C.c_int]),
            "orc_model_config": (None, [P, C.POINTER(orc_config)]),
            "orc_model_embedding": (None, [P, C.c_uint32, C.POINTER(C.c_float)]),
            "orc_cache_new": (P, [P, SZ]),
            "orc_cache_free": (None, [P]),
            "orc_cache_clone": (P, [P]),
            "orc_cache_len": (SZ, [P]),
            "orc_cache_capacity": (SZ, [P]),
            "orc_cache_advance": (None, [P, SZ]),
            "orc_cache_reset": (None, [P]),
            "orc_cache_ensure_capacity": (None, [P, SZ]),
            "orc_cache_truncate": (C.c_int, [P, SZ, C.c_char_p, SZ]),
            "orc_cache_read_kv": (C.c_int, [P, SZ, SZ, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
            "orc_forward_cached": (C.c_int, [P, P, C.POINTER(C.c_uint32), SZ, C.POINTER(C.c_float), C.c_char_p, SZ]),
            "orc_rng_new": (U64, [U64]),
            "orc_rng_next_u64": (U64, [C.POINTER(U64)]),
            "orc_rng_next_f32": (C.c_float, [C.POINTER(U64)]),
            "orc_sample": (SZ, [C.POINTER(C.c_float), C.POINTER(C.c_uint8), SZ, C.c_float, C.c_long, C.c_float,
                                C.POINTER(U64)]),
            "orc_sample_batch": (None, [C.POINTER(C.c_float), SZ, SZ, C.POINTER(C.c_uint8), SZ,
                                         C.POINTER(C.c_float), C.POINTER(C.c_long), C.POINTER(C.c_float),
                                         C.POINTER(U64), C.POINTER(U64), C.c_int]),
            "orc_expf_block": (None, [C.POINTER(C.c_float), C.POINTER(C.c_float), SZ, C.c_int]),
            "orc_softmax": (None, [C.POINTER(C.c_float), SZ]),
            "orc_generate": (C.c_int, [P, C.POINTER(C.c_uint32), SZ, C.POINTER(orc_gen_params),
                                       C.POINTER(C.c_uint32), SZ, ON_TOKEN, MASKER, STOP, ON_PREFILL, P, P, SZ,
                                       C.POINTER(C.c_uint32), C.POINTER(orc_gen_result), C.c_char_p, SZ]),
        }
        for k, (r, a) in sig.items():
            f = getattr(L, k)
            f.restype, f.argtypes = r, a
        _lib = L
    return _lib


def _f32p(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def fp16_to_f32(h: int) -> float:
    return float(lib().orc_fp16_to_f32(h))


def dequantize(qtype: int, n_elements: int, raw: bytes) -> np.ndarray:
    """dequantize() (dequant.rs:209-310)."""
    buf = np.frombuffer(raw, dtype=np.uint8)
    out = np.empty(n_elements, np.float32)
    rc = lib().orc_dequantize(qtype, n_elements, buf.ctypes.data_as(C.c_void_p), buf.size, _f32p(out))
    if rc:
        raise ValueError("dequantize failed")
    return out


def gguf_info(path: str) -> dict:
    n = 1 << 16
    while True:
        buf = C.create_string_buffer(n)
        r = lib().orc_gguf_info_json(path.encode(), buf, n)
        if r < 0:
            raise ValueError(buf.value.decode())
        if r < n:
            return json.loads(buf.value.decode())
        n = r + 1


def gguf_tensor_f32(path: str, name: str, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    err = C.create_string_buffer(512)
    if lib().orc_gguf_tensor_f32(path.encode(), name.encode(), _f32p(out), n, err, 512):
        raise ValueError(err.value.decode())
    return out


class Rng:
    """splitmix64 Rng (sampling.rs:12-41)."""

    def __init__(self, seed: int = 0, state: Optional[int] = None):
        self.s = C.c_uint64(lib().orc_rng_new(seed) if state is None else state)

    def next_u64(self) -> int:
        return int(lib().orc_rng_next_u64(C.byref(self.s)))

    def next_f32(self) -> float:
        return float(lib().orc_rng_next_f32(C.byref(self.s)))

    @property
    def state(self) -> int:
        return self.s.value


def sample(logits, temperature=0.0, top_k=None, top_p=None, rng_state: int = 0, mask=None):
    """Sampler::sample[_masked]; returns (index, new rng state)."""
    lg = np.ascontiguousarray(np.asarray(logits, np.float32))
    st = C.c_uint64(rng_state)
    mk = None
    if mask is not None:
        m8 = np.ascontiguousarray(np.asarray(mask, np.uint8))
        mk = m8.ctypes.data_as(C.POINTER(C.c_uint8))
    idx = lib().orc_sample(_f32p(lg), mk, lg.size, temperature, -1 if top_k is None else top_k,
                           -1.0 if top_p is None else top_p, C.byref(st))
    return int(idx), st.value


def sample_batch(logits, samplers, rng_states, mask=None, shared=False):
    """Many Sampler::sample[_masked] draws (threaded over draws): row i of
    `logits` (or the single row when shared) with samplers[i] = (temperature,
    top_k, top_p) (None allowed) and rng_states[i]; returns (ids, new states)."""
    lg = np.ascontiguousarray(np.asarray(logits, np.float32))
    n = lg.shape[-1]
    rows = len(samplers)
    T = np.array([s[0] for s in samplers], np.float32)
    K = np.array([-1 if s[1] is None else s[1] for s in samplers], np.int64).astype(C.c_long)
    Pp = np.array([-1.0 if s[2] is None else s[2] for s in samplers], np.float32)
    st = np.ascontiguousarray(np.asarray(rng_states, np.uint64))
    out = np.empty(rows, np.uint64)
    mk = None
    if mask is not None:
        m8 = np.ascontiguousarray(np.asarray(mask, np.uint8))
        mk = m8.ctypes.data_as(C.POINTER(C.c_uint8))
    lib().orc_sample_batch(_f32p(lg), 0 if shared else n, n, mk, rows, _f32p(T),
                           K.ctypes.data_as(C.POINTER(C.c_long)), _f32p(Pp), st.ctypes.data_as(C.POINTER(C.c_uint64)),
                           out.ctypes.data_as(C.POINTER(C.c_uint64)), os.cpu_count() or 1)
    return out.astype(np.int64), st


def softmax(x):
    """The sampler's softmax (sampling.rs:157-172) of one row."""
    y = np.array(x, np.float32, copy=True)
    lib().orc_softmax(_f32p(y), y.size)
    return y


def expf_glibc(x):
    """glibc's expf on a float32 array (what Rust's f32::exp calls)."""
    xx = np.ascontiguousarray(np.asarray(x, np.float32))
    y = np.empty_like(xx)
    lib().orc_expf_block(_f32p(xx), _f32p(y), xx.size, os.cpu_count() or 1)
    return y


class SeqState:
    def __init__(self, h, model):
        self.h = C.c_void_p(h)
        self.model = model

    def __len__(self):
        return int(lib().orc_cache_len(self.h))

    @property
    def len(self):
        return len(self)

    def capacity(self):
        return int(lib().orc_cache_capacity(self.h))

    def advance(self, n):
        lib().orc_cache_advance(self.h, n)

    def reset(self):
        lib().orc_cache_reset(self.h)

    def ensure_capacity(self, n):
        lib().orc_cache_ensure_capacity(self.h, n)

    def truncate(self, n):
        err = C.create_string_buffer(256)
        if lib().orc_cache_truncate(self.h, n, err, 256):
            raise ValueError(err.value.decode())

    def clone(self):
        return SeqState(lib().orc_cache_clone(self.h), self.model)

    def read_kv(self, layer, pos):
        kvd = self.model.config.n_kv_heads * self.model.config.head_dim
        k = np.empty(kvd, np.float32)
        v = np.empty(kvd, np.float32)
        if lib().orc_cache_read_kv(self.h, layer, pos, _f32p(k), _f32p(v)):
            raise IndexError("read_kv out of range")
        return k, v

    def __del__(self):
        try:
            if self.h:
                lib().orc_cache_free(self.h)
                self.h = C.c_void_p()
        except Exception:
            pass


class Model:
    """qwen2::Model (CPU, f32), quantized weights dequantized per row on demand."""

    def __init__(self, path: str, threads: int = 0):
        err = C.create_string_buffer(512)
        h = lib().orc_model_load(path.encode(), threads or (os.cpu_count() or 1), err, 512)
        if not h:
            raise ValueError(err.value.decode())
        self.h = C.c_void_p(h)
        cfg = orc_config()
        lib().orc_model_config(self.h, C.byref(cfg))
        self.config = cfg

    def set_threads(self, n: int) -> None:
        lib().orc_model_set_threads(self.h, n)

    def new_cache(self, max_seq: int) -> SeqState:
        return SeqState(lib().orc_cache_new(self.h, max_seq), self)

    def embedding(self, tok: int) -> np.ndarray:
        out = np.empty(self.config.n_embd, np.float32)
        lib().orc_model_embedding(self.h, tok, _f32p(out))
        return out

    def forward_cached(self, cache: SeqState, tokens: Sequence[int]) -> np.ndarray:
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        out = np.empty(self.config.vocab_size, np.float32)
        err = C.create_string_buffer(512)
        if lib().orc_forward_cached(self.h, cache.h, t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size, _f32p(out),
                                    err, 512):
            raise ValueError(err.value.decode())
        return out

    def generate(self, prompt, max_tokens, temperature=0.0, top_k=None, top_p=None, seed=0, eos=(),
                 on_token=None, masker=None, stop=None, on_prefill=None, seed_cache=None, seed_n=0):
        p = np.ascontiguousarray(np.asarray(prompt, np.uint32))
        e = np.ascontiguousarray(np.asarray(list(eos) or [0], np.uint32))
        params = orc_gen_params(max_tokens, temperature, -1 if top_k is None else top_k,
                                -1.0 if top_p is None else top_p, 0 if seed is None else 1,
                                0 if seed is None else seed)
        out = np.zeros(max(1, max_tokens), np.uint32)
        res = orc_gen_result()
        err = C.create_string_buffer(512)
        cb_tok = ON_TOKEN((lambda _u, t: 1 if on_token(t) else 0) if on_token else 0)

        def _mask(_u, ptr, n):
            m = masker()
            if m is None:
                return 0
            C.memmove(ptr, np.ascontiguousarray(np.asarray(m, np.uint8)).ctypes.data, n)
            return 1
        cb_mask = MASKER(_mask if masker else 0)
        cb_stop = STOP((lambda _u, ptr, n: 1 if stop([ptr[i] for i in range(n)]) else 0) if stop else 0)
        cb_pre = ON_PREFILL((lambda _u, c: on_prefill(SeqState(lib().orc_cache_clone(c), self))) if on_prefill
                            else 0)
        rc = lib().orc_generate(self.h, p.ctypes.data_as(C.POINTER(C.c_uint32)), p.size, C.byref(params),
                                e.ctypes.data_as(C.POINTER(C.c_uint32)), len(eos), cb_tok, cb_mask, cb_stop, cb_pre,
                                None, seed_cache.h if seed_cache else None, seed_n,
                                out.ctypes.data_as(C.POINTER(C.c_uint32)), C.byref(res), err, 512)
        if rc:
            raise ValueError(err.value.decode())
        return dict(ids=[int(x) for x in out[:res.n_ids]], finish_reason="stop" if res.finish_stop else "length",
                    prompt_tokens=res.prompt_tokens, prefix_reused=res.prefix_reused,
                    elapsed_secs=res.elapsed_secs)

    def __del__(self):
        try:
            if self.h:
                lib().orc_model_free(self.h)
                self.h = C.c_void_p()
        except Exception:
            pass
