"""generate_tokens_seeded semantics (crates/s-models/src/generate.rs:339-537)
for the engine's loop (sm_generate_with over a fake device) and, where the
oracle has the same entry point, for the oracle's loop."""
import pytest

import smotor
from fakedev import VOCAB, FakeDevice


def run(dev, prompt, max_tokens, **kw):
    return smotor.generate_with(dev, prompt, max_tokens, VOCAB, **kw)


def test_defaults():
    # generate.rs:263-269: greedy by default, 256 tokens
    assert smotor.Sampler().temperature == 0.0


def test_loop_through_the_device():
    out = run(FakeDevice([3, 9, 15]), [1, 2], 10)
    assert len(out.ids) == 10
    assert out.ids[:3] == [9, 15, 7]
    assert out.finish_reason == "length"
    assert out.prompt_tokens == 2


def test_eos_stops():
    out = run(FakeDevice([3, 9]), [1], 10, eos=[9])
    assert out.ids == [3, 9]
    assert out.finish_reason == "stop"


def test_callback_abort():
    seen = []

    def on_token(t):
        seen.append(t)
        return len(seen) < 2

    out = run(FakeDevice([3, 9, 15]), [1], 10, on_token=on_token)
    assert len(out.ids) == 2 and seen == [3, 9] and out.finish_reason == "stop"


def test_stop_callback():
    out = run(FakeDevice([3, 9, 15, 4]), [1], 10, stop=lambda ids: ids[-2:] == [15, 4])
    assert out.ids == [3, 9, 15, 4] and out.finish_reason == "stop"


def first_pass(dev, prompt, max_tokens):
    snap = {}

    def on_prefill(c):
        snap["c"] = c.clone()

    out = run(dev, prompt, max_tokens, on_prefill=on_prefill)
    return out, snap["c"]


def test_seeded_equals_plain():
    dev = FakeDevice([3, 9, 15])
    base, snapshot = first_pass(dev, [1, 2], 20)
    assert snapshot.len == 2 and base.prefix_reused == 0
    seed = snapshot.clone()
    seed.truncate(1)
    out2 = run(dev, [1, 2], 6, seed_cache=seed, seed_n=1)
    assert out2.prefix_reused == 1
    assert out2.ids == base.ids[:len(out2.ids)]
    ext = [1, 2, 5, 6, 7]
    out3 = run(dev, ext, 6, seed_cache=snapshot.clone(), seed_n=2)
    assert out3.prefix_reused == 2
    assert out3.ids == run(dev, ext, 6).ids


@pytest.mark.parametrize("bad", [0, 5])
def test_unusable_seed_falls_back_to_full_prefill(bad):
    dev = FakeDevice([3, 9, 15])
    _, snapshot = first_pass(dev, [1, 2], 4)
    out = run(dev, [1, 2], 4, seed_cache=snapshot.clone(), seed_n=bad)
    assert out.prefix_reused == 0


def test_on_prefill_once_with_prompt_length():
    calls = []
    run(FakeDevice([3]), [1, 2, 3], 2, on_prefill=lambda c: calls.append(c.len))
    assert calls == [3]


def test_max_tokens_zero_still_prefills():
    calls = []
    out = run(FakeDevice([3]), [1, 2, 3], 0, on_prefill=lambda c: calls.append(c.len))
    assert out.ids == [] and calls == [3] and out.finish_reason == "length"


def test_masker_constrains_sampling():
    mask = [1] * VOCAB
    mask[9] = 0
    out = run(FakeDevice([3, 9, 15]), [1], 3, masker=lambda: mask)
    # position 1 would pick 9 (forbidden): greedy takes the lowest index of the rest (all 0.0)
    assert out.ids == [3, 0, 15]


def test_seeded_sampling_is_reproducible():
    a = run(FakeDevice([3, 9, 15]), [1], 8, temperature=1.0, top_k=4, seed=5)
    b = run(FakeDevice([3, 9, 15]), [1], 8, temperature=1.0, top_k=4, seed=5)
    assert a.ids == b.ids


def test_empty_prompt_rejected():
    with pytest.raises(smotor.EngineError):
        run(FakeDevice([3]), [], 2)
