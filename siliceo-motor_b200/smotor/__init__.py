"""Python binding of the siliceo-motor B200 decode engine (libsmotor.so).

A thin ctypes layer over the C ABI in include/sm_engine.h, shaped like the
reference's Rust API for the qwen2/llama path:

    Model            s_models::qwen2::Model / GpuQwen2 (`impl Device`)
    Cache            s_models::state::SeqState (dense, all-KV layers)
    Model.forward_cached(cache, tokens)        Device::forward_cached
    Model.forward_sample / decode_batch        forward + Sampler::sample on device
    generate / generate_with                   generate_tokens_seeded

There is no CPU path: the library must be built (``make -C siliceo-motor_b200``)
and every compute call needs a CUDA device; a missing library raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsmotor.so")

# ggml type codes (crates/s-gguf/src/types.rs)
F32, Q5_0, Q8_0, Q4_K, Q6_K = 0, 6, 8, 12, 14
BLOCK = {Q4_K: (256, 144), Q6_K: (256, 210), Q5_0: (32, 22), Q8_0: (32, 34), F32: (1, 4)}


class EngineError(RuntimeError):
    """A call into libsmotor returned a non-zero sm_status."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"sm_status {status}: {msg}")
        self.status = status


class sm_config(C.Structure):
    _fields_ = [("n_layers", C.c_uint64), ("n_embd", C.c_uint64), ("n_ff", C.c_uint64),
                ("n_heads", C.c_uint64), ("n_kv_heads", C.c_uint64), ("head_dim", C.c_uint64),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("vocab_size", C.c_uint64)]


class sm_load_opts(C.Structure):
    _fields_ = [("device", C.c_int32), ("max_batch", C.c_uint32), ("max_context", C.c_uint32),
                ("tp_rank", C.c_uint32), ("tp_size", C.c_uint32), ("tp_flags", C.c_uint32),
                ("tp_wait_ms", C.c_uint32), ("tp_group", C.c_void_p)]


class sm_tp_shard(C.Structure):
    _fields_ = [("q_head0", C.c_uint64), ("q_heads", C.c_uint64), ("kv_head0", C.c_uint64),
                ("kv_heads", C.c_uint64), ("ff0", C.c_uint64), ("ff", C.c_uint64),
                ("vocab0", C.c_uint64), ("vocab", C.c_uint64)]


TP_ID_BYTES = 128
TP_NCCL = 1  # SM_TP_NCCL: NCCL collectives instead of the engine's peer-memory kernels
ERR_PEER = 9  # SM_ERR_PEER


class sm_sampler(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int64), ("top_p", C.c_float)]


class sm_gen_params(C.Structure):
    _fields_ = [("max_tokens", C.c_uint64), ("temperature", C.c_float), ("top_k", C.c_int64),
                ("top_p", C.c_float), ("has_seed", C.c_int32), ("seed", C.c_uint64)]


class sm_gen_result(C.Structure):
    _fields_ = [("n_ids", C.c_uint64), ("finish_stop", C.c_int32), ("prompt_tokens", C.c_uint64),
                ("prefix_reused", C.c_uint64), ("elapsed_secs", C.c_double)]


class sm_synth_spec(C.Structure):
    _fields_ = [("arch", C.c_int32), ("n_embd", C.c_uint32), ("n_layers", C.c_uint32),
                ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("n_ff", C.c_uint32),
                ("vocab", C.c_uint32), ("rope_theta", C.c_float), ("rms_eps", C.c_float),
                ("qkv_bias", C.c_int32), ("tied", C.c_int32), ("seed", C.c_uint64),
                ("weight_std", C.c_float), ("type_override", C.c_int32)]


ON_TOKEN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint32)
MASKER = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_uint8), C.c_uint64)
STOP = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_uint32), C.c_uint64)
ON_PREFILL = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p)
NEW_CACHE = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint64, C.POINTER(C.c_void_p))
FREE_CACHE = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p)
FWD_SAMPLE = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.POINTER(C.c_uint32), C.c_uint64,
                         C.POINTER(sm_sampler), C.POINTER(C.c_uint64), C.POINTER(C.c_uint8),
                         C.POINTER(C.c_uint32))


class sm_device_vtbl(C.Structure):
    _fields_ = [("new_cache", NEW_CACHE), ("free_cache", FREE_CACHE), ("forward_sample", FWD_SAMPLE)]


# Every symbol include/sm_engine.h declares, with (restype, argtypes).
P, U64, U32, I32, PU32, PU64 = C.c_void_p, C.c_uint64, C.c_uint32, C.c_int32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64)
SIGNATURES = {
    "sm_last_error": (C.c_char_p, []),
    "sm_abi_version": (C.c_int, []),
    "sm_tp_group_id": (C.c_int, [P]),
    "sm_model_tp_abort": (C.c_int, [P]),
    "sm_tp_plan": (C.c_int, [C.POINTER(sm_config), U32, U32, C.POINTER(sm_tp_shard)]),
    "sm_model_load": (C.c_int, [C.c_char_p, C.POINTER(sm_load_opts), C.POINTER(P)]),
    "sm_model_load_memory": (C.c_int, [P, U64, C.POINTER(sm_load_opts), C.POINTER(P)]),
    "sm_model_free": (C.c_int, [P]),
    "sm_model_config": (C.c_int, [P, C.POINTER(sm_config)]),
    "sm_model_weight_bytes": (C.c_int, [P, PU64]),
    "sm_model_stream": (C.c_int, [P, C.POINTER(P)]),
    "sm_model_step_io_bytes": (C.c_int, [P, PU64, PU64]),
    "sm_model_step_launches": (C.c_int, [P, U64, PU64]),
    "sm_cache_new": (C.c_int, [P, U64, C.POINTER(P)]),
    "sm_cache_free": (C.c_int, [P]),
    "sm_cache_len": (C.c_int, [P, PU64]),
    "sm_cache_capacity": (C.c_int, [P, PU64]),
    "sm_cache_advance": (C.c_int, [P, U64]),
    "sm_cache_reset": (C.c_int, [P]),
    "sm_cache_truncate": (C.c_int, [P, U64]),
    "sm_cache_ensure_capacity": (C.c_int, [P, U64]),
    "sm_cache_clone": (C.c_int, [P, C.POINTER(P)]),
    "sm_cache_read_kv": (C.c_int, [P, U64, U64, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
    "sm_model_kv_pages": (C.c_int, [P, PU64, PU64, PU64]),
    "sm_forward_cached": (C.c_int, [P, P, PU32, U64, C.POINTER(C.c_float)]),
    "sm_rng_seed": (C.c_uint64, [U64]),
    "sm_forward_sample": (C.c_int, [P, P, PU32, U64, C.POINTER(sm_sampler), PU64, C.POINTER(C.c_uint8), PU32]),
    "sm_decode_batch": (C.c_int, [P, C.POINTER(P), U64, PU32, C.POINTER(sm_sampler), PU64, PU32]),
    "sm_decode_run": (C.c_int, [P, C.POINTER(P), U64, PU32, C.POINTER(sm_sampler), PU64, U64, PU32, P, P]),
    "sm_decode_batch_logits": (C.c_int, [P, C.POINTER(P), U64, PU32, C.POINTER(sm_sampler), PU64, PU32,
                                         C.POINTER(C.c_float)]),
    "sm_generate_with": (C.c_int, [C.POINTER(sm_device_vtbl), P, U64, PU32, U64, C.POINTER(sm_gen_params),
                                   PU32, U64, ON_TOKEN, MASKER, STOP, ON_PREFILL, P, P, U64, PU32,
                                   C.POINTER(sm_gen_result)]),
    "sm_generate": (C.c_int, [P, PU32, U64, C.POINTER(sm_gen_params), PU32, U64, ON_TOKEN, MASKER, STOP,
                              ON_PREFILL, P, P, U64, PU32, C.POINTER(sm_gen_result)]),
    "sm_dweight_upload": (C.c_int, [U32, P, U64, U64, C.POINTER(P)]),
    "sm_dweight_free": (C.c_int, [P]),
    "sm_dweight_bytes": (C.c_int, [P, PU64]),
    "sm_dequant": (C.c_int, [P, P, P]),
    "sm_gemv": (C.c_int, [P, P, P, U64, P]),
    "sm_gemv_noalloc": (C.c_int, [P, P, P, U64, P]),
    "sm_sample": (C.c_int, [C.POINTER(C.c_float), U64, U64, U64, C.POINTER(C.c_uint8), C.POINTER(sm_sampler),
                            PU64, PU32]),
    "sm_expf_ref": (C.c_int, [P, P, U64, P]),
    "sm_softmax": (C.c_int, [P, U64, U64, P, P]),
    "sm_model_embedding": (C.c_int, [P, U32, C.POINTER(C.c_float)]),
    "sm_gemv_status": (C.c_int, [P, P]),
    "sm_gemv_noalloc_status": (C.c_int, [P]),
    "sm_synth_preset": (C.c_int, [C.c_int, C.POINTER(sm_synth_spec)]),
    "sm_synth_size": (C.c_int, [C.POINTER(sm_synth_spec), PU64]),
    "sm_synth_write": (C.c_int, [C.POINTER(sm_synth_spec), C.c_char_p, C.c_int]),
    "sm_synth_memory": (C.c_int, [C.POINTER(sm_synth_spec), C.c_int, C.POINTER(P), PU64]),
    "sm_synth_free": (None, [P]),
    "sm_quantize": (C.c_int, [U32, C.POINTER(C.c_float), U64, P]),
}

_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    """The loaded engine library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C siliceo-motor_b200`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise EngineError(rc, lib().sm_last_error().decode(errors="replace"))


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(C.POINTER(t))


def rng_seed(seed: int) -> int:
    """The splitmix64 state of Rng::new(seed) (sampling.rs:15-17)."""
    return int(lib().sm_rng_seed(C.c_uint64(seed & 0xFFFFFFFFFFFFFFFF)))


@dataclass
class Sampler:
    """Sampler (sampling.rs:43-60); top_k/top_p None = disabled."""
    temperature: float = 0.0
    top_k: Optional[int] = None
    top_p: Optional[float] = None

    def c(self) -> sm_sampler:
        return sm_sampler(self.temperature, -1 if self.top_k is None else int(self.top_k),
                          -1.0 if self.top_p is None else float(self.top_p))


def sample(logits, samplers, rng_states, mask=None, shared=False):
    """Sampler::sample[_masked] on the device (the decode steps' kernel) for
    host logits: row i (or the single row when shared) with samplers[i] and
    rng_states[i]; returns (ids, new states)."""
    lg = np.ascontiguousarray(np.asarray(logits, np.float32))
    V = lg.shape[-1]
    n = len(samplers)
    sm = (sm_sampler * n)(*[s.c() for s in samplers])
    st = np.ascontiguousarray(np.asarray(rng_states, dtype=np.uint64))
    out = np.empty(n, np.uint32)
    mk = None
    if mask is not None:
        m8 = np.ascontiguousarray(np.asarray(mask, dtype=np.uint8))
        mk = _p(m8, C.c_uint8)
    _check(lib().sm_sample(_p(lg, C.c_float), n, 0 if shared else V, V, mk, sm, _p(st, C.c_uint64),
                           _p(out, C.c_uint32)))
    return out, st


def softmax(x_ptr: int, rows: int, n: int, out_ptr: int, stream: int = 0) -> None:
    """The sampler's softmax (sampling.rs:157-172) of rows x n device floats."""
    _check(lib().sm_softmax(C.c_void_p(x_ptr), rows, n, C.c_void_p(out_ptr), C.c_void_p(stream)))


def expf_ref(x_ptr: int, y_ptr: int, n: int, stream: int = 0) -> None:
    """The sampler's exp (glibc's expf on x <= 0) over n device floats."""
    _check(lib().sm_expf_ref(C.c_void_p(x_ptr), C.c_void_p(y_ptr), n, C.c_void_p(stream)))


class Cache:
    """A sequence state on the device (SeqState for dense models)."""

    def __init__(self, handle: int, model: "Model", owned: bool = True):
        self.h = C.c_void_p(handle)
        self.model = model
        self.owned = owned  # False for a handle lent by the library (on_prefill)

    def __len__(self) -> int:
        v = C.c_uint64()
        _check(lib().sm_cache_len(self.h, C.byref(v)))
        return v.value

    @property
    def len(self) -> int:
        return len(self)

    def capacity(self) -> int:
        v = C.c_uint64()
        _check(lib().sm_cache_capacity(self.h, C.byref(v)))
        return v.value

    def advance(self, n: int) -> None:
        _check(lib().sm_cache_advance(self.h, n))

    def reset(self) -> None:
        _check(lib().sm_cache_reset(self.h))

    def truncate(self, n: int) -> None:
        _check(lib().sm_cache_truncate(self.h, n))

    def ensure_capacity(self, n: int) -> None:
        _check(lib().sm_cache_ensure_capacity(self.h, n))

    def clone(self) -> "Cache":
        out = C.c_void_p()
        _check(lib().sm_cache_clone(self.h, C.byref(out)))
        return Cache(out.value, self.model)

    def read_kv(self, layer: int, pos: int):
        """K and V of one position: the model's KV heads, or with tensor
        parallelism this rank's (sm_tp_plan)."""
        kvd = self.model.kv_width()
        k = np.empty(kvd, np.float32)
        v = np.empty(kvd, np.float32)
        _check(lib().sm_cache_read_kv(self.h, layer, pos, _p(k, C.c_float), _p(v, C.c_float)))
        return k, v

    def free(self) -> None:
        if self.h and self.owned:
            lib().sm_cache_free(self.h)
        self.h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def tp_group_id() -> bytes:
    """A new tensor-parallel group id (an NCCL unique id): made on one rank
    and shared with every rank of the group."""
    buf = (C.c_uint8 * TP_ID_BYTES)()
    _check(lib().sm_tp_group_id(C.cast(buf, C.c_void_p)))
    return bytes(buf)


def tp_plan(config: sm_config, rank: int, size: int) -> sm_tp_shard:
    """The part of the model rank `rank` of a `size`-way group holds."""
    out = sm_tp_shard()
    _check(lib().sm_tp_plan(C.byref(config), rank, size, C.byref(out)))
    return out


def config_of(n_layers, n_embd, n_ff, n_heads, n_kv_heads, vocab, rope_theta=1e6, rms_eps=1e-6) -> sm_config:
    return sm_config(n_layers, n_embd, n_ff, n_heads, n_kv_heads, n_embd // n_heads, rope_theta, rms_eps, vocab)


@dataclass
class TensorParallel:
    """This process's place in a tensor-parallel group (sm_load_opts.tp_*)."""
    rank: int
    size: int
    group_id: bytes
    flags: int = 0
    wait_ms: int = 0

    def __post_init__(self):
        if len(self.group_id) != TP_ID_BYTES:
            raise ValueError(f"group_id must be {TP_ID_BYTES} bytes")
        self._id = (C.c_uint8 * TP_ID_BYTES).from_buffer_copy(self.group_id)

    @classmethod
    def from_process_group(cls, flags: int = 0, wait_ms: int = 0, group=None) -> "TensorParallel":
        """One rank per process of a torch.distributed group: rank 0 makes the
        id and broadcasts it (any backend)."""
        import torch.distributed as dist
        rank, size = dist.get_rank(group), dist.get_world_size(group)
        obj = [tp_group_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(rank, size, obj[0], flags, wait_ms)


class Model:
    """A qwen2/llama GGUF model resident in HBM."""

    tp: Optional[TensorParallel] = None

    def __init__(self, handle: int):
        self.h = C.c_void_p(handle)
        cfg = sm_config()
        _check(lib().sm_model_config(self.h, C.byref(cfg)))
        self.config = cfg

    @staticmethod
    def _opts(device: int, max_batch: int, max_context: int, tp=None) -> sm_load_opts:
        o = sm_load_opts(device, max_batch, max_context, 0, 0, 0, 0, None)
        if tp is not None:
            o.tp_rank, o.tp_size = tp.rank, tp.size
            o.tp_flags, o.tp_wait_ms = tp.flags, tp.wait_ms
            o.tp_group = C.cast(tp._id, C.c_void_p)
        return o

    @classmethod
    def load(cls, path: str, device: int = 0, max_batch: int = 32, max_context: int = 32768,
             tp: Optional["TensorParallel"] = None) -> "Model":
        """tp: this process's rank of a tensor-parallel group (every rank
        loads the same file with its own rank and the same group id)."""
        out = C.c_void_p()
        o = cls._opts(device, max_batch, max_context, tp)
        _check(lib().sm_model_load(path.encode(), C.byref(o), C.byref(out)))
        m = cls(out.value)
        m.tp = tp
        return m

    @classmethod
    def load_memory(cls, buf: int, length: int, device: int = 0, max_batch: int = 32,
                    max_context: int = 32768, tp: Optional["TensorParallel"] = None) -> "Model":
        out = C.c_void_p()
        o = cls._opts(device, max_batch, max_context, tp)
        _check(lib().sm_model_load_memory(C.c_void_p(buf), length, C.byref(o), C.byref(out)))
        m = cls(out.value)
        m.tp = tp
        return m

    def kv_width(self) -> int:
        """Floats per position of this rank's K (and V) cache."""
        c = self.config
        heads = tp_plan(c, self.tp.rank, self.tp.size).kv_heads if self.tp is not None else c.n_kv_heads
        return heads * c.head_dim

    def tp_abort(self) -> None:
        """Mark the tensor-parallel group failed (a peer left): later calls
        raise EngineError(ERR_PEER) without launching, free skips the barrier."""
        _check(lib().sm_model_tp_abort(self.h))

    def weight_bytes(self) -> int:
        v = C.c_uint64()
        _check(lib().sm_model_weight_bytes(self.h, C.byref(v)))
        return v.value

    def kv_pages(self):
        """(pages held by caches, pages allocated, bytes per page) of the
        model's KV pool. Clones share pages until one of them writes."""
        h, a, b = C.c_uint64(), C.c_uint64(), C.c_uint64()
        _check(lib().sm_model_kv_pages(self.h, C.byref(h), C.byref(a), C.byref(b)))
        return h.value, a.value, b.value

    def step_launches(self, n_rows: int) -> int:
        """Kernels one decode_run step of n_rows sequences launches."""
        v = C.c_uint64()
        _check(lib().sm_model_step_launches(self.h, n_rows, C.byref(v)))
        return v.value

    def stream(self) -> int:
        v = C.c_void_p()
        _check(lib().sm_model_stream(self.h, C.byref(v)))
        return v.value or 0

    def embedding(self, token: int) -> np.ndarray:
        """Row `token` of the embedding table as the engine's forward gathers it."""
        out = np.empty(self.config.n_embd, np.float32)
        _check(lib().sm_model_embedding(self.h, token, _p(out, C.c_float)))
        return out

    def new_cache(self, max_seq: int) -> Cache:
        out = C.c_void_p()
        _check(lib().sm_cache_new(self.h, max_seq, C.byref(out)))
        return Cache(out.value, self)

    def forward_cached(self, cache: Cache, tokens: Sequence[int], logits: bool = True) -> Optional[np.ndarray]:
        t = _u32(tokens)
        out = np.empty(self.config.vocab_size, np.float32) if logits else None
        _check(lib().sm_forward_cached(self.h, cache.h, _p(t, C.c_uint32), len(t),
                                       _p(out, C.c_float) if logits else None))
        return out

    def forward_sample(self, cache: Cache, tokens: Sequence[int], sampler: Sampler, rng_state: int,
                       mask: Optional[np.ndarray] = None):
        t = _u32(tokens)
        s = sampler.c()
        st = C.c_uint64(rng_state)
        tok = C.c_uint32()
        mk = None
        if mask is not None:
            m8 = np.ascontiguousarray(np.asarray(mask, dtype=np.uint8))
            mk = _p(m8, C.c_uint8)
        _check(lib().sm_forward_sample(self.h, cache.h, _p(t, C.c_uint32), len(t), C.byref(s), C.byref(st), mk,
                                       C.byref(tok)))
        return tok.value, st.value

    def decode_batch(self, caches: Sequence[Cache], tokens: Sequence[int], samplers: Sequence[Sampler],
                     rng_states: Sequence[int]):
        n = len(caches)
        hs = (C.c_void_p * n)(*[c.h for c in caches])
        t = _u32(tokens)
        sm = (sm_sampler * n)(*[s.c() for s in samplers])
        st = np.ascontiguousarray(np.asarray(rng_states, dtype=np.uint64))
        out = np.empty(n, np.uint32)
        _check(lib().sm_decode_batch(self.h, hs, n, _p(t, C.c_uint32), sm, _p(st, C.c_uint64),
                                     _p(out, C.c_uint32)))
        return out, st

    def decode_batch_logits(self, caches: Sequence[Cache], tokens: Sequence[int], samplers: Sequence[Sampler],
                            rng_states: Sequence[int]):
        """decode_batch, also returning the logits [n, vocab] the step's sampler drew from."""
        n = len(caches)
        hs = (C.c_void_p * n)(*[c.h for c in caches])
        t = _u32(tokens)
        sm = (sm_sampler * n)(*[s.c() for s in samplers])
        st = np.ascontiguousarray(np.asarray(rng_states, dtype=np.uint64))
        out = np.empty(n, np.uint32)
        lg = np.empty((n, self.config.vocab_size), np.float32)
        _check(lib().sm_decode_batch_logits(self.h, hs, n, _p(t, C.c_uint32), sm, _p(st, C.c_uint64),
                                            _p(out, C.c_uint32), _p(lg, C.c_float)))
        return out, st, lg

    def decode_run(self, caches: Sequence[Cache], tokens: Sequence[int], samplers: Sequence[Sampler],
                   rng_states: Sequence[int], n_steps: int, ev_begin: int = 0, ev_end: int = 0):
        """n_steps device-resident decode steps; returns tokens [n_steps, n] and RNG states."""
        n = len(caches)
        hs = (C.c_void_p * n)(*[c.h for c in caches])
        t = _u32(tokens)
        sm = (sm_sampler * n)(*[s.c() for s in samplers])
        st = np.ascontiguousarray(np.asarray(rng_states, dtype=np.uint64))
        out = np.empty((n_steps, n), np.uint32)
        _check(lib().sm_decode_run(self.h, hs, n, _p(t, C.c_uint32), sm, _p(st, C.c_uint64), n_steps,
                                   _p(out, C.c_uint32), C.c_void_p(ev_begin or None), C.c_void_p(ev_end or None)))
        return out, st

    def generate(self, prompt: Sequence[int], max_tokens: int, temperature: float = 0.0,
                 top_k: Optional[int] = None, top_p: Optional[float] = None, seed: Optional[int] = 0,
                 eos: Sequence[int] = (), on_token=None, masker=None, stop=None, on_prefill=None,
                 seed_cache: Optional[Cache] = None, seed_n: int = 0):
        return _generate(lambda *a: lib().sm_generate(self.h, *a), prompt, max_tokens, temperature, top_k, top_p,
                         seed, eos, on_token, masker, stop, on_prefill, seed_cache.h if seed_cache else None,
                         seed_n, self.config.vocab_size, wrap_cache=lambda p: Cache(p, self, owned=False))

    def step_io_bytes(self):
        """(host->device, device->host) bytes one decode step copies."""
        a, b = C.c_uint64(), C.c_uint64()
        _check(lib().sm_model_step_io_bytes(self.h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def free(self) -> None:
        if self.h:
            lib().sm_model_free(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


@dataclass
class Generated:
    """Generated (generate.rs:45-60) minus the text (no tokenizer on this path)."""
    ids: list
    finish_reason: str
    prompt_tokens: int
    prefix_reused: int
    elapsed_secs: float


def _generate(call, prompt, max_tokens, temperature, top_k, top_p, seed, eos, on_token, masker, stop,
              on_prefill, seed_cache_ptr, seed_n, vocab, wrap_cache):
    p = _u32(prompt)
    e = _u32(list(eos)) if len(eos) else np.zeros(1, np.uint32)
    params = sm_gen_params(max_tokens, temperature, -1 if top_k is None else top_k,
                           -1.0 if top_p is None else top_p, 0 if seed is None else 1,
                           0 if seed is None else seed & 0xFFFFFFFFFFFFFFFF)
    out = np.zeros(max(1, max_tokens), np.uint32)
    res = sm_gen_result()
    cb_tok = ON_TOKEN((lambda _u, t: 1 if on_token(t) else 0) if on_token else 0)
    if masker:
        def _mask(_u, ptr, n):
            m = masker()
            if m is None:
                return 0
            C.memmove(ptr, np.ascontiguousarray(np.asarray(m, np.uint8)).ctypes.data, n)
            return 1
        cb_mask = MASKER(_mask)
    else:
        cb_mask = MASKER(0)
    cb_stop = STOP((lambda _u, ptr, n: 1 if stop([ptr[i] for i in range(n)]) else 0) if stop else 0)
    cb_pre = ON_PREFILL((lambda _u, c: on_prefill(wrap_cache(c))) if on_prefill else 0)
    _check(call(_p(p, C.c_uint32), len(p), C.byref(params), _p(e, C.c_uint32), len(eos), cb_tok, cb_mask,
                cb_stop, cb_pre, None, seed_cache_ptr, seed_n, _p(out, C.c_uint32), C.byref(res)))
    return Generated([int(x) for x in out[:res.n_ids]], "stop" if res.finish_stop else "length",
                     res.prompt_tokens, res.prefix_reused, res.elapsed_secs)


def generate_with(device, prompt, max_tokens, vocab, temperature=0.0, top_k=None, top_p=None, seed=0,
                  eos=(), on_token=None, masker=None, stop=None, on_prefill=None, seed_cache=None, seed_n=0):
    """generate_tokens_seeded over a Python device object with
    new_cache(max_seq) -> cache, free_cache(cache), and
    forward_sample(cache, tokens, Sampler, rng_state, mask) -> (token, rng_state)."""
    caches = {}

    def _new(_d, max_seq, out):
        c = device.new_cache(max_seq)
        key = id(c)
        caches[key] = c
        out[0] = key
        return 0

    def _free(_d, key):
        caches.pop(key, None)
        return 0

    def _fwd(_d, key, tp, n, sp, st, mk, out):
        c = caches[key]
        toks = [tp[i] for i in range(n)]
        s = Sampler(sp[0].temperature, None if sp[0].top_k < 0 else sp[0].top_k,
                    None if sp[0].top_p < 0 else sp[0].top_p)
        mask = None if not mk else np.ctypeslib.as_array(mk, shape=(vocab,)).copy()
        tok, new_st = device.forward_sample(c, toks, s, st[0], mask)
        st[0] = new_st
        out[0] = tok
        return 0

    vt = sm_device_vtbl(NEW_CACHE(_new), FREE_CACHE(_free), FWD_SAMPLE(_fwd))
    seed_key = None
    if seed_cache is not None:
        seed_key = id(seed_cache)
        caches[seed_key] = seed_cache
    return _generate(lambda *a: lib().sm_generate_with(C.byref(vt), None, vocab, *a), prompt, max_tokens,
                     temperature, top_k, top_p, seed, eos, on_token, masker, stop, on_prefill, seed_key, seed_n,
                     vocab, wrap_cache=lambda key: caches[key])


class DWeight:
    """One quantized tensor in the engine's HBM layout (kernel-level API)."""

    def __init__(self, qtype: int, data: bytes, n_out: int, n_in: int):
        buf = np.frombuffer(data, dtype=np.uint8)
        out = C.c_void_p()
        _check(lib().sm_dweight_upload(qtype, buf.ctypes.data_as(C.c_void_p), n_out, n_in, C.byref(out)))
        self.h = out
        self.n_out, self.n_in, self.qtype = n_out, n_in, qtype

    def nbytes(self) -> int:
        v = C.c_uint64()
        _check(lib().sm_dweight_bytes(self.h, C.byref(v)))
        return v.value

    def dequant(self, out_ptr: int, stream: int = 0) -> None:
        _check(lib().sm_dequant(self.h, C.c_void_p(out_ptr), C.c_void_p(stream)))

    def gemv(self, x_ptr: int, y_ptr: int, batch: int, stream: int = 0) -> None:
        _check(lib().sm_gemv(self.h, C.c_void_p(x_ptr), C.c_void_p(y_ptr), batch, C.c_void_p(stream)))

    def gemv_noalloc(self, x_ptr: int, y_ptr: int, batch: int, stream: int = 0) -> None:
        """sm_gemv without allocating: its K-split scratch is a fixed library array."""
        _check(lib().sm_gemv_noalloc(self.h, C.c_void_p(x_ptr), C.c_void_p(y_ptr), batch, C.c_void_p(stream)))

    def gemv_status(self, stream: int = 0) -> None:
        """Raises if a bounded wait in an earlier gemv() on this weight gave up."""
        _check(lib().sm_gemv_status(self.h, C.c_void_p(stream)))


    def free(self) -> None:
        if self.h:
            lib().sm_dweight_free(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def gemv_noalloc_status(stream: int = 0) -> None:
    """Raises if a bounded wait in an earlier gemv_noalloc() on the current device gave up."""
    _check(lib().sm_gemv_noalloc_status(C.c_void_p(stream)))


# ------------------------------------------------------------- synthetic ----
def synth_preset(config_index: int) -> sm_synth_spec:
    s = sm_synth_spec()
    _check(lib().sm_synth_preset(config_index, C.byref(s)))
    return s


def synth_spec(arch="qwen2", n_embd=256, n_layers=2, n_heads=4, n_kv_heads=2, n_ff=512, vocab=1024,
               rope_theta=1e6, rms_eps=1e-6, qkv_bias=True, tied=False, seed=0, weight_std=0.02,
               type_override=-1) -> sm_synth_spec:
    return sm_synth_spec(0 if arch == "qwen2" else 1, n_embd, n_layers, n_heads, n_kv_heads, n_ff, vocab,
                         rope_theta, rms_eps, int(qkv_bias), int(tied), seed, weight_std, type_override)


def synth_write(spec: sm_synth_spec, path: str, threads: int = 0) -> None:
    _check(lib().sm_synth_write(C.byref(spec), path.encode(), threads or (os.cpu_count() or 1)))


def synth_size(spec: sm_synth_spec) -> int:
    v = C.c_uint64()
    _check(lib().sm_synth_size(C.byref(spec), C.byref(v)))
    return v.value


class SynthBuffer:
    """A synthetic GGUF image in host memory (freed with the object)."""

    def __init__(self, spec: sm_synth_spec, threads: int = 0):
        p = C.c_void_p()
        n = C.c_uint64()
        _check(lib().sm_synth_memory(C.byref(spec), threads or (os.cpu_count() or 1), C.byref(p), C.byref(n)))
        self.ptr, self.len = p.value, n.value

    def free(self) -> None:
        if self.ptr:
            lib().sm_synth_free(C.c_void_p(self.ptr))
            self.ptr = 0

    def __del__(self):
        self.free()


def quantize(qtype: int, x: np.ndarray) -> bytes:
    """Encode f32 values (whole blocks) as a ggml type."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32).ravel())
    bs, tb = BLOCK[qtype]
    out = np.empty(x.size // bs * tb, np.uint8)
    _check(lib().sm_quantize(qtype, _p(x, C.c_float), x.size, out.ctypes.data_as(C.c_void_p)))
    return out.tobytes()
