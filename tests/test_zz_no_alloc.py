"""sm_gemv_noalloc: the GEMV for callers that cannot allocate device memory
(their host hands out all device memory itself, or the call sits on a path
where cudaMalloc's device-wide synchronization is not allowed). The scratch of
its K-split (partial sums and arrival counters) is a fixed array inside the
library. This checks, on two calls in a row with different inputs (the second
finds the counters the first left), that its output equals the exact product
of the oracle's dequantized weights within the GEMV tolerance and sm_gemv's
output on the same inputs; covers rows split several ways (129 blocks: the
planner's slices hold at most 32 blocks, so 5 slices) and many 16-row tiles;
and that a shape whose smallest split overflows the fixed array is refused
with SM_ERR_ARG while sm_gemv still runs it. Collected last on purpose (file
name), so that a run stopping at the first failure has run every other test
first."""
import numpy as np
import pytest

import pyoracle as orc
import smotor

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GEMV_TOL = 1e-4  # the same bar as tests/test_gpu_kernels.py


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max())


def colwise_err(got, want):
    """Normwise per column (row of y): max |got - want| / max |want|."""
    return float((np.abs(got - want).max(axis=-1) / np.abs(want).max(axis=-1)).max())


def check_twice(qt, n_out, n_in, batches, seed):
    rng = np.random.default_rng(seed)
    raw = smotor.quantize(qt, rng.normal(0, 1, n_out * n_in).astype(np.float32))
    wdq = orc.dequantize(qt, n_out * n_in, raw).reshape(n_out, n_in).astype(np.float64)
    w = smotor.DWeight(qt, raw, n_out, n_in)
    for batch in batches:
        for call in range(2):  # two calls in a row; the second reuses the shared scratch
            xh = rng.normal(0, 1, (batch, n_in)).astype(np.float32)
            x = torch.from_numpy(xh).cuda()
            y_ref = torch.full((batch, n_out), float("nan"), device="cuda")
            y = torch.full((batch, n_out), float("nan"), device="cuda")
            w.gemv(x.data_ptr(), y_ref.data_ptr(), batch)
            w.gemv_noalloc(x.data_ptr(), y.data_ptr(), batch)
            torch.cuda.synchronize()
            smotor.gemv_noalloc_status()
            assert not torch.isnan(y).any()
            exact = xh.astype(np.float64) @ wdq.T
            assert colwise_err(y.cpu().numpy().astype(np.float64), exact) <= GEMV_TOL, (qt, batch, call)
            assert rel(y, y_ref) <= GEMV_TOL, (qt, batch, call)
    w.free()


@pytest.mark.parametrize("qt,n_out,n_in", [(smotor.Q4_K, 384, 3584), (smotor.Q6_K, 256, 4864),
                                            (smotor.Q5_0, 128, 896)])
def test_noalloc_matches_oracle_and_gemv_twice(qt, n_out, n_in):
    check_twice(qt, n_out, n_in, (1, 3), seed=qt + n_in)


@pytest.mark.parametrize("qt,n_out,n_in", [(smotor.Q4_K, 64, 32768 + 256), (smotor.Q4_K, 8192, 18944),
                                            (smotor.Q6_K, 512, 14336)])
def test_noalloc_long_rows_and_large_splits(qt, n_out, n_in):
    check_twice(qt, n_out, n_in, (1,), seed=n_out + n_in)


def test_noalloc_refuses_a_split_that_does_not_fit():
    # Q4_K rows of 33 blocks need two slices; 2 x 32784 rows of partial sums
    # exceed the fixed array's 65536 floats. All-zero blocks (d = 0) are valid.
    n_out, n_in = 32784, 33 * 256
    w = smotor.DWeight(smotor.Q4_K, bytes(n_out * (n_in // 256) * 144), n_out, n_in)
    x = torch.ones(n_in, device="cuda")
    y = torch.full((n_out,), float("nan"), device="cuda")
    with pytest.raises(smotor.EngineError) as e:
        w.gemv_noalloc(x.data_ptr(), y.data_ptr(), 1)
    assert e.value.status == 1 and "sm_gemv" in str(e.value)
    w.gemv(x.data_ptr(), y.data_ptr(), 1)  # the allocating entry point runs it
    torch.cuda.synchronize()
    w.gemv_status()
    assert not y.any()
    w.free()
