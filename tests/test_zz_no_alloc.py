"""sm_gemv_noalloc: the GEMV for callers that cannot allocate device memory
(their host hands out all device memory itself, or the call sits on a path
where cudaMalloc's device-wide synchronization is not allowed). The scratch of
its batch-1 K-split (partial sums and arrival counters) is a fixed array inside
the library; this checks that its output equals sm_gemv's within the GEMV
tolerance, on two calls in a row with different inputs (the second finds the
counters the first left), for a row of 129 blocks split 129 ways and a
16-row-tile count that splits K in two. Collected last on purpose (file
name), so that a run stopping at the first failure has run every other test
first."""
import numpy as np
import pytest

import smotor

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GEMV_TOL = 1e-4  # the same bar as tests/test_gpu_kernels.py


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max())


@pytest.mark.parametrize("qt,n_out,n_in", [(smotor.Q4_K, 384, 3584), (smotor.Q6_K, 256, 4864),
                                            (smotor.Q5_0, 128, 896)])
def test_noalloc_matches_gemv_twice(qt, n_out, n_in):
    rng = np.random.default_rng(qt + n_in)
    w = smotor.DWeight(qt, smotor.quantize(qt, rng.normal(0, 1, n_out * n_in).astype(np.float32)), n_out, n_in)
    for batch in (1, 3):
        for call in range(2):  # two calls in a row; the second reuses the shared scratch
            x = torch.from_numpy(rng.normal(0, 1, (batch, n_in)).astype(np.float32)).cuda()
            y_ref = torch.full((batch, n_out), float("nan"), device="cuda")
            y = torch.full((batch, n_out), float("nan"), device="cuda")
            w.gemv(x.data_ptr(), y_ref.data_ptr(), batch)
            w.gemv_noalloc(x.data_ptr(), y.data_ptr(), batch)
            torch.cuda.synchronize()
            assert not torch.isnan(y).any()
            assert rel(y, y_ref) <= GEMV_TOL, (qt, batch, call)
    w.free()


@pytest.mark.parametrize("qt,n_out,n_in", [(smotor.Q4_K, 64, 32768 + 256), (smotor.Q4_K, 8192, 18944)])
def test_noalloc_long_rows_and_large_splits(qt, n_out, n_in):
    rng = np.random.default_rng(n_out + n_in)
    w = smotor.DWeight(qt, smotor.quantize(qt, rng.normal(0, 1, n_out * n_in).astype(np.float32)), n_out, n_in)
    for call in range(2):
        x = torch.from_numpy(rng.normal(0, 1, n_in).astype(np.float32)).cuda()
        y_ref = torch.full((n_out,), float("nan"), device="cuda")
        y = torch.full((n_out,), float("nan"), device="cuda")
        w.gemv(x.data_ptr(), y_ref.data_ptr(), 1)
        w.gemv_noalloc(x.data_ptr(), y.data_ptr(), 1)
        torch.cuda.synchronize()
        assert not torch.isnan(y).any()
        assert rel(y, y_ref) <= GEMV_TOL, (n_out, n_in, call)
    w.free()
