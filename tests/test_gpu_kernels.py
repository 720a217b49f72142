"""Kernel-level parity on the GPU, through the C ABI: bit-exact dequant
(crates/s-gguf/src/dequant.rs) and the dequant-fused GEMV on the microbench
shapes (batch 1, 8, 32) within 1e-4 of the exact product, normwise
(max|y - y_ref| / max|y_ref|)."""
import struct

import numpy as np
import pytest

import pyoracle as orc
import smotor

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GEMV_TOL = 1e-4  # "GEMV output within 1e-4 relative"
SHAPES = [(896, 4864), (3584, 18944), (4096, 14336), (8192, 28672)]


def random_blocks(qt, n_out, n_in, seed, special=False):
    """Valid random GGUF rows: random bytes with finite fp16 scales; with
    special=True some scales are NaN/Inf halves (the reference's quirks)."""
    rng = np.random.default_rng(seed)
    bs, tb = smotor.BLOCK[qt]
    nb = n_out * n_in // bs
    raw = rng.integers(0, 256, size=(nb, tb), dtype=np.uint8)
    offs = {smotor.Q4_K: [0, 2], smotor.Q6_K: [208], smotor.Q5_0: [0], smotor.Q8_0: [0]}[qt]
    for o in offs:
        e = rng.integers(1, 12, nb)
        h = ((rng.integers(0, 2, nb) << 15) | (e << 10) | rng.integers(0, 1024, nb)).astype(np.uint16)
        if special:
            pick = rng.random(nb) < 0.05
            h[pick] = rng.choice(np.array([0x7C00, 0xFC00, 0x7E00, 0x0001, 0x0000], np.uint16), pick.sum())
        raw[:, o] = h & 0xFF
        raw[:, o + 1] = h >> 8
    return raw.tobytes()


@pytest.mark.parametrize("qt", [smotor.Q4_K, smotor.Q6_K, smotor.Q5_0, smotor.Q8_0])
@pytest.mark.parametrize("special", [False, True])
def test_dequant_bit_exact(qt, special):
    n_out, n_in = 64, 1024
    raw = random_blocks(qt, n_out, n_in, seed=qt * 7 + special, special=special)
    want = orc.dequantize(qt, n_out * n_in, raw)
    w = smotor.DWeight(qt, raw, n_out, n_in)
    out = torch.empty(n_out * n_in, dtype=torch.float32, device="cuda")
    w.dequant(out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def gemv_check(qt, n_out, n_in, batches, seed, std=1.0, outliers=False):
    rng = np.random.default_rng(seed)
    wf = rng.normal(0, std, n_out * n_in).astype(np.float32)
    raw = smotor.quantize(qt, wf)
    del wf
    wdq = orc.dequantize(qt, n_out * n_in, raw).reshape(n_out, n_in).astype(np.float64)
    w = smotor.DWeight(qt, raw, n_out, n_in)
    assert w.nbytes() == len(raw)
    bmax = max(batches)
    x = rng.normal(0, 1, (bmax, n_in)).astype(np.float32)
    if outliers:  # a few large channels, as activations have: per-block scaling of x must cope
        x[:, ::97] *= 300.0
        x[1::2] *= 1e-3  # and columns of very different magnitude
    y_ref = x.astype(np.float64) @ wdq.T
    xd = torch.from_numpy(x).cuda()
    for b in batches:
        y = torch.full((b, n_out), float("nan"), dtype=torch.float32, device="cuda")
        w.gemv(xd.data_ptr(), y.data_ptr(), b)
        torch.cuda.synchronize()
        got = y.cpu().numpy().astype(np.float64)
        # normwise per column: a column of small values is held to its own scale
        err = (np.abs(got - y_ref[:b]).max(axis=1) / np.abs(y_ref[:b]).max(axis=1)).max()
        assert err <= GEMV_TOL, (qt, n_out, n_in, b, err)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("qt", [smotor.Q4_K, smotor.Q6_K])
def test_gemv_microbench_shapes(qt, shape):
    # N(0,1) weights quantized from seed 1, x ~ N(0,1)
    gemv_check(qt, shape[0], shape[1], [1, 8, 32], seed=1)


@pytest.mark.parametrize("qt", [smotor.Q5_0, smotor.Q8_0])
@pytest.mark.parametrize("batch", [1, 2, 3, 5, 17, 32])
def test_gemv_fallback_types_and_odd_batches(qt, batch):
    gemv_check(qt, 256, 896, [batch], seed=batch)


@pytest.mark.parametrize("batch", [2, 3, 4, 7])
def test_gemv_kquants_odd_batches_and_ragged_rows(batch):
    gemv_check(smotor.Q4_K, 100, 512, [batch], seed=3)
    gemv_check(smotor.Q6_K, 36, 768, [batch], seed=4)


@pytest.mark.parametrize("qt", [smotor.Q4_K, smotor.Q6_K])
@pytest.mark.parametrize("n_out,n_in", [(512, 8192), (4096, 256), (272, 2304)])
def test_gemv_batched_tensor_core_sweep(qt, n_out, n_in):
    # every n-tile count (1, 2, 4, 8 groups of 4 columns) and partial groups;
    # K split many ways (512 x 8192), unsplit (4096 x 256), a ragged last tile
    gemv_check(qt, n_out, n_in, [2, 4, 5, 8, 9, 16, 17, 24, 31, 32], seed=n_out + n_in)


@pytest.mark.parametrize("qt", [smotor.Q4_K, smotor.Q6_K])
def test_gemv_batched_outlier_channels(qt):
    gemv_check(qt, 1024, 4096, [2, 8, 32], seed=9, outliers=True)
    gemv_check(qt, 1024, 4096, [1], seed=9, outliers=True)


def test_gemv_rejects_bad_arguments():
    raw = smotor.quantize(smotor.Q4_K, np.zeros(256 * 8, np.float32))
    w = smotor.DWeight(smotor.Q4_K, raw, 8, 256)
    x = torch.zeros(40 * 256, device="cuda")
    y = torch.zeros(40 * 8, device="cuda")
    with pytest.raises(smotor.EngineError):
        w.gemv(x.data_ptr(), y.data_ptr(), 33)
    with pytest.raises(smotor.EngineError):
        w.gemv(x.data_ptr() + 4, y.data_ptr(), 1)
    with pytest.raises(smotor.EngineError):
        smotor.DWeight(smotor.Q4_K, raw, 16, 128)  # n_in not a multiple of 256
