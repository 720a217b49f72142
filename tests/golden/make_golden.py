"""Generates tests/golden/dequant_golden.npz (committed).

Seeded random GGUF blocks of each type the decode path reads, with their f32
dequantization by gguf-py (the `gguf` package, the reference implementation
of the GGML block formats that crates/s-gguf/src/dequant.rs:1-6 says it was
verified bit-perfect against). Block scales are drawn from finite fp16
values; the reference's non-finite-scale quirks (NaN half -> Inf, Q6_K block
zeroed) are pinned separately in tests/test_oracle_golden.py.

Run:  python tests/golden/make_golden.py   (needs numpy and gguf)
"""
import importlib.metadata
import os

import gguf
import numpy as np
from gguf import GGMLQuantizationType as T

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dequant_golden.npz")
N_BLOCKS = 8

# byte offsets of the fp16 scale fields inside each block
SCALES = {T.Q4_0: [0], T.Q4_1: [0, 2], T.Q5_0: [0], T.Q8_0: [0], T.Q4_K: [0, 2], T.Q6_K: [208]}


def finite_half(rng, n):
    # magnitudes 2^-14 .. 2^2, random sign: normal halves only
    e = rng.integers(1, 17, size=n)
    m = rng.integers(0, 1024, size=n)
    s = rng.integers(0, 2, size=n)
    return ((s << 15) | (e << 10) | m).astype(np.uint16)


def main():
    rng = np.random.default_rng(20240901)
    arrays = {"gguf_version": np.array([importlib.metadata.version("gguf")])}
    for t, offs in SCALES.items():
        bs, tb = gguf.GGML_QUANT_SIZES[t]
        raw = rng.integers(0, 256, size=(N_BLOCKS, tb), dtype=np.uint8)
        for o in offs:
            h = finite_half(rng, N_BLOCKS)
            raw[:, o] = (h & 0xFF).astype(np.uint8)
            raw[:, o + 1] = (h >> 8).astype(np.uint8)
        deq = gguf.quants.dequantize(raw.reshape(-1), t).astype(np.float32).reshape(-1)
        assert deq.size == N_BLOCKS * bs
        arrays[f"{t.name}_type"] = np.array([int(t)])
        arrays[f"{t.name}_raw"] = raw.reshape(-1)
        arrays[f"{t.name}_f32"] = deq
    np.savez_compressed(OUT, **arrays)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
