"""The reference's FakeDevice (crates/s-models/src/generate.rs:274-337): logits
are a function of the position only; sampling goes through the oracle's
Sampler. Drives the generation loop without a model or a GPU."""
import pyoracle as orc

VOCAB = 16


class FakeCache:
    def __init__(self, max_seq):
        self.len, self.max_seq, self.calls = 0, max_seq, 0

    def truncate(self, n):
        assert n <= self.len
        self.len = n

    def clone(self):
        c = FakeCache(self.max_seq)
        c.len, c.calls = self.len, self.calls
        return c


class FakeDevice:
    def __init__(self, sequence):
        self.sequence = list(sequence)

    def new_cache(self, max_seq):
        return FakeCache(max_seq)

    def forward_sample(self, cache, tokens, sampler, rng_state, mask):
        assert len(tokens) > 0
        assert cache.len + len(tokens) <= cache.max_seq
        cache.calls += 1
        cache.len += len(tokens)
        p = cache.len - 1
        winner = self.sequence[p] if p < len(self.sequence) else 7
        logits = [10.0 if i == winner else 0.0 for i in range(VOCAB)]
        return orc.sample(logits, sampler.temperature, sampler.top_k, sampler.top_p, rng_state, mask)
