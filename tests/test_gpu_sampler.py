"""The on-device sampler against the reference's Sampler::sample
(crates/s-models/src/sampling.rs:94-172), bit for bit.

- The sampler's exp is glibc's expf on every float of [-104, 0] (exhaustive).
- The sampler's softmax is the reference's softmax, bit for bit (the exact
  left-to-right f32 denominator) on shapes from 1 to 250k values, flat,
  peaked, tied, masked and wide distributions.
- The reference's own sampler tests (sampling.rs:178-230), run on the device.
- Sampled ids and RNG states equal the reference's on >= 10k seeded draws
  over real-shape logits (vocab 152064), and over every mode: top-k only,
  top-p only, neither (the whole vocabulary sorted), k above 1024, k = 0,
  p at 0 and above 1, temperatures from 1e-3 to 100, masks and ties.
"""
import numpy as np
import pytest

import pyoracle as orc
import smotor

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

V = 152064  # Qwen2.5-7B vocabulary


def S(t=0.0, k=None, p=None):
    return smotor.Sampler(t, k, p)


def dev_draws(logits, samplers, states, mask=None, shared=True):
    ids, st = smotor.sample(logits, samplers, states, mask=mask, shared=shared)
    return ids.astype(np.int64), st


def ref_draws(logits, samplers, states, mask=None, shared=True):
    return orc.sample_batch(logits, [(s.temperature, s.top_k, s.top_p) for s in samplers], states, mask=mask,
                            shared=shared)


def check(logits, samplers, states, mask=None, shared=True, what=""):
    di, ds = dev_draws(logits, samplers, states, mask, shared)
    ri, rs = ref_draws(logits, samplers, states, mask, shared)
    bad = np.nonzero((di != ri) | (ds != rs))[0]
    assert bad.size == 0, (f"{what}: {bad.size} of {len(samplers)} draws differ, first at {bad[0]}: "
                           f"device {di[bad[0]]}, reference {ri[bad[0]]}")


def test_expf_is_glibc_on_the_whole_domain():
    lo = -(1 << 31)  # bits 0x80000000: -0.0
    hi = int(np.array([-104.0], np.float32).view(np.int32)[0])  # bits of -104.0, as int32
    step = 1 << 26
    y = torch.empty(step, device="cuda")
    for a in range(lo, hi + 1, step):
        b = min(hi + 1, a + step)
        x = torch.arange(a, b, dtype=torch.int32, device="cuda").view(torch.float32)
        smotor.expf_ref(x.data_ptr(), y.data_ptr(), b - a)
        got = y[:b - a].cpu().numpy()
        want = orc.expf_glibc(x.cpu().numpy())
        bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
        assert bad.size == 0, (hex(a), bad.size, x[int(bad[0])].item())
    edge = np.array([0.0, -0.0, -np.inf, np.nan, -104.5, -150.0, -1e30, -87.3365, -103.97], np.float32)
    xe = torch.from_numpy(edge).cuda()
    ye = torch.empty_like(xe)
    smotor.expf_ref(xe.data_ptr(), ye.data_ptr(), edge.size)
    got, want = ye.cpu().numpy(), orc.expf_glibc(edge)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32))


def softmax_cases():
    r = np.random.default_rng(3)
    yield "one", np.array([0.5], np.float32)
    yield "two", np.array([1.0, 1.0], np.float32)
    yield "flat100", np.full(100, 0.1, np.float32)
    yield "kat", np.array([0.0] * 3 + [20.0] + [0.0] * 6, np.float32)
    for n in (3, 1000, 4099, V, 250000):
        for sd in (0.01, 1.0, 10.0, 50.0):
            yield f"normal n={n} sd={sd}", r.normal(0, sd, n).astype(np.float32)
    x = r.normal(0, 1.2, V).astype(np.float32)
    x[r.integers(0, V, 5000)] = -np.inf  # masked entries
    yield "masked", x
    yield "ties", (np.round(r.normal(0, 2.0, V) * 4) / 4).astype(np.float32)
    yield "one huge", np.where(np.arange(V) == 777, 40.0, r.normal(0, 1, V)).astype(np.float32)
    y = np.zeros(V, np.float32)
    y[::3] = 1e-3
    yield "halfway terms", y  # many equal terms: rounding ties in the running sum
    yield "increasing", np.linspace(-30, 0, V).astype(np.float32)
    yield "decreasing", np.linspace(0, -30, V).astype(np.float32)


def test_softmax_is_the_references_bit_for_bit():
    for name, x in softmax_cases():
        xd = torch.from_numpy(x).cuda()
        out = torch.empty_like(xd)
        smotor.softmax(xd.data_ptr(), 1, x.size, out.data_ptr())
        got = out.cpu().numpy()
        want = orc.softmax(x)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
            (name, int(np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0][0]))


def test_reference_sampler_kats_on_device():
    # sampling.rs:178-230, each through the device sampler
    rs = smotor.rng_seed
    assert dev_draws(np.array([0.1, 5.0, 3.0], np.float32), [S()], [rs(1)])[0][0] == 1
    assert dev_draws(np.array([2.0, 2.0, 1.0], np.float32), [S()], [rs(1)])[0][0] == 0  # tie: lowest index
    assert dev_draws(np.array([-1.0, 9.0, 2.0, 9.0], np.float32), [S(0.0, 40, 0.9)], [rs(42)])[0][0] == 1
    assert dev_draws(np.array([0.2, 0.1, 8.8], np.float32), [S(1.5, 1, None)], [rs(7)])[0][0] == 2
    # seed_stesso_distribuzione_stessa: two samplers with the same seed draw the same 50 tokens
    flat = np.full(100, 0.1, np.float32)
    a, b = rs(123), rs(123)
    for _ in range(50):
        (ta,), (a,) = dev_draws(flat, [S(0.8)], [a])
        (tb,), (b,) = dev_draws(flat, [S(0.8)], [b])
        assert ta == tb
    # topp_piccolo_cola_al_top: top-p 0.01 on a dominant logit picks it
    lg = np.zeros(10, np.float32)
    lg[3] = 20.0
    assert dev_draws(lg, [S(1.0, None, 0.01)], [rs(99)])[0][0] == 3
    # the same draws as the reference implementation, with their RNG states
    check(flat, [S(0.8)] * 50, [rs(123 + i) for i in range(50)], what="flat 0.8")


def real_logits(seed, sd=1.2):
    return np.random.default_rng(seed).normal(0, sd, V).astype(np.float32)


def test_10k_seeded_draws_topk40_topp09_real_shape():
    lg = real_logits(11)
    check(lg, [S(1.0, 40, 0.9)] * 10000, [smotor.rng_seed(i) for i in range(10000)], what="T1 k40 p0.9")


@pytest.mark.parametrize("sampler,n", [
    (S(1.0, None, 0.9), 400), (S(0.8, None, None), 400), (S(1.3, 2000, None), 300), (S(1.0, 1024, 0.5), 1000),
    (S(1.0, 1025, 0.95), 300), (S(0.7, 0, 0.9), 300), (S(1.0, 50, 0.0), 300), (S(1.0, 60, 1.5), 300),
    (S(1e-3, 40, 0.9), 300), (S(100.0, 200, None), 300), (S(1.0, None, 0.999), 200), (S(2.0, 5, None), 1000)])
def test_every_sampler_mode_real_shape(sampler, n):
    lg = real_logits(12, 2.5)
    check(lg, [sampler] * n, [smotor.rng_seed(7000 + i) for i in range(n)],
          what=f"T{sampler.temperature} k{sampler.top_k} p{sampler.top_p}")


def test_ties_masks_and_small_vocabularies():
    r = np.random.default_rng(5)
    tied = (np.round(r.normal(0, 2.0, V) * 2) / 2).astype(np.float32)  # many equal probabilities
    check(tied, [S(1.0, 40, 0.9)] * 2000, [smotor.rng_seed(i) for i in range(2000)], what="ties k40")
    check(tied, [S(1.0, None, 0.8)] * 200, [smotor.rng_seed(i) for i in range(200)], what="ties full")
    mask = (r.random(V) > 0.3).astype(np.uint8)
    check(real_logits(13), [S(1.0, 40, 0.9)] * 1000, [smotor.rng_seed(i) for i in range(1000)], mask=mask,
          what="masked")
    check(real_logits(13), [S()] * 20, [0] * 20, mask=mask, what="masked greedy")
    for n in (1, 2, 3, 7, 33, 1023, 1024, 1025, 5000):
        lg = r.normal(0, 1.0, n).astype(np.float32)
        for smp in (S(), S(1.0, 40, 0.9), S(0.9, None, None), S(1.0, None, 0.5), S(1.1, 3000, 0.99)):
            check(lg, [smp] * 64, [smotor.rng_seed(31 * n + i) for i in range(64)],
                  what=f"n={n} T{smp.temperature} k{smp.top_k} p{smp.top_p}")
    # per-row logits (no sharing)
    rows = r.normal(0, 1.5, (40, 3000)).astype(np.float32)
    check(rows, [S(1.0, 40, 0.9)] * 40, [smotor.rng_seed(i) for i in range(40)], shared=False, what="rows")


def test_greedy_nan_at_index_zero_is_returned():
    lg = np.array([np.nan, 1.0, 5.0, 2.0], np.float32)
    assert dev_draws(lg, [S()], [0])[0][0] == 0  # argmax: x[i] > NaN never holds
    lg = np.array([1.0, np.nan, 5.0, 5.0], np.float32)
    assert dev_draws(lg, [S()], [0])[0][0] == 2
