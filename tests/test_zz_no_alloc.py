"""sm_gemv_noalloc: the GEMV for callers that cannot allocate device memory
(their host hands out all device memory itself, or the call sits on a path
where cudaMalloc's device-wide synchronization is not allowed). Its batch-1
scratch is a fixed array inside the library; this checks that its output
equals sm_gemv's within the GEMV tolerance, on two calls in a row with
different inputs, and that it refuses rows longer than that array. Collected
last on purpose (file name), so that a run stopping at the first failure has
run every other test first."""
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


def test_noalloc_rejects_rows_beyond_the_scratch():
    n_in = 32768 + 256
    w = smotor.DWeight(smotor.Q4_K, smotor.quantize(smotor.Q4_K, np.zeros(8 * n_in, np.float32)), 8, n_in)
    x = torch.zeros(n_in, device="cuda")
    y = torch.zeros(8, device="cuda")
    with pytest.raises(smotor.EngineError, match="scratch"):
        w.gemv_noalloc(x.data_ptr(), y.data_ptr(), 1)
    w.free()
