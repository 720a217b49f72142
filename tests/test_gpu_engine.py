"""Engine vs the CPU oracle on seeded synthetic GGUFs: logits (1e-3 max
relative error, identical top-8), KV cache, greedy token identity, on-device
sampling, batched decode, cache operations."""
import numpy as np
import pytest

import pyoracle as orc
import smotor

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

LOGIT_TOL = 1e-3  # north star: per-step logits within 1e-3 max relative error


def rel_err(got, want):
    return float(np.abs(got.astype(np.float64) - want).max() / np.abs(want).max())


def top8(x):
    return set(np.argsort(-x, kind="stable")[:8].tolist())


SPECS = {
    # qwen2 with biases, GQA 2, std 0.5 so that logits are well spread
    "qwen2_tiny": dict(arch="qwen2", n_embd=512, n_layers=3, n_heads=8, n_kv_heads=2, n_ff=1024, vocab=2048,
                       weight_std=0.5, seed=11),
    # llama, no bias, GQA 4, head_dim 128, untied
    "llama_tiny": dict(arch="llama", n_embd=1024, n_layers=2, n_heads=8, n_kv_heads=2, n_ff=2048, vocab=3000,
                       rope_theta=5e5, rms_eps=1e-5, qkv_bias=False, weight_std=0.3, seed=12),
    # fallback types (Q5_0 / Q8_0) and tied embeddings, like config 0
    "qwen2_fallback": dict(arch="qwen2", n_embd=448, n_layers=2, n_heads=7, n_kv_heads=1, n_ff=768, vocab=1000,
                           tied=True, weight_std=0.4, seed=13),
}


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("gpu")
    out = {}
    for name, kw in SPECS.items():
        p = str(d / f"{name}.gguf")
        smotor.synth_write(smotor.synth_spec(**kw), p)
        out[name] = (smotor.Model.load(p, max_context=4096), orc.Model(p))
    yield out
    for e, _ in out.values():
        e.free()


@pytest.mark.parametrize("name", list(SPECS))
def test_logits_prefill_and_decode_vs_oracle(models, name):
    eng, ora = models[name]
    V = eng.config.vocab_size
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, V, 45).tolist()  # crosses a 32-row prefill chunk and a 64-position tile
    ce, co = eng.new_cache(128), ora.new_cache(128)
    le = eng.forward_cached(ce, prompt)
    lo = ora.forward_cached(co, prompt)
    assert rel_err(le, lo) <= LOGIT_TOL and top8(le) == top8(lo)
    for step in range(30):  # teacher-forced decode across the 64-position tile boundary
        t = int(rng.integers(0, V))
        le = eng.forward_cached(ce, [t])
        lo = ora.forward_cached(co, [t])
        assert rel_err(le, lo) <= LOGIT_TOL, step
        assert top8(le) == top8(lo), step
    assert len(ce) == len(co) == 75
    for layer in (0, eng.config.n_layers - 1):
        for pos in (0, 44, 74):
            ke, ve = ce.read_kv(layer, pos)
            ko, vo = co.read_kv(layer, pos)
            assert rel_err(ke, ko) <= 1e-4 and rel_err(ve, vo) <= 1e-4


@pytest.mark.parametrize("name", list(SPECS))
def test_embedding_row_is_bit_exact(models, name):
    # Q6_K (qwen2_tiny, llama_tiny) and Q8_0 (qwen2_fallback) tables; the
    # engine's embedding kernel must give the oracle's dequantized row bit for bit
    eng, ora = models[name]
    V = eng.config.vocab_size
    for tok in (0, 1, 7, V // 2 + 3, V - 1):
        got, want = eng.embedding(tok), ora.embedding(tok)
        assert got.shape == want.shape == (eng.config.n_embd,)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), tok
    with pytest.raises(smotor.EngineError):
        eng.embedding(V)


@pytest.mark.parametrize("name", list(SPECS))
def test_greedy_generation_identical(models, name):
    eng, ora = models[name]
    prompt = np.random.default_rng(1).integers(0, eng.config.vocab_size, 24).tolist()
    ge = eng.generate(prompt, 64)
    go = ora.generate(prompt, 64)
    assert ge.ids == go["ids"]
    assert ge.finish_reason == go["finish_reason"] == "length"


def test_sampler_on_device_matches_reference(models):
    eng, _ = models["llama_tiny"]
    V = eng.config.vocab_size
    prompt = list(range(10))
    base = eng.new_cache(64)
    eng.forward_cached(base, prompt[:-1], logits=False)
    cases = [smotor.Sampler(1.0, 40, 0.9), smotor.Sampler(0.7, 5, None), smotor.Sampler(1.5, 1000, 0.5),
             smotor.Sampler(0.0, None, None), smotor.Sampler(2.0, 200, None), smotor.Sampler(1.0, None, 0.9),
             smotor.Sampler(0.9, None, None), smotor.Sampler(1.2, 2500, 0.97)]
    for i, s in enumerate(cases):
        for seed in range(8):
            st = smotor.rng_seed(100 * i + seed)
            c1, c2 = base.clone(), base.clone()
            logits = eng.forward_cached(c1, prompt[-1:])
            tok, st_e = eng.forward_sample(c2, prompt[-1:], s, st)
            want, st_o = orc.sample(logits, s.temperature, s.top_k, s.top_p, st)
            assert (tok, st_e) == (want, st_o), (s, seed)
            c1.free()
            c2.free()


def test_masked_sampling(models):
    eng, _ = models["qwen2_tiny"]
    V = eng.config.vocab_size
    c = eng.new_cache(32)
    logits = eng.forward_cached(c.clone(), [1, 2, 3])
    best = int(np.argmax(logits))
    mask = np.ones(V, np.uint8)
    mask[best] = 0
    tok, _ = eng.forward_sample(c, [1, 2, 3], smotor.Sampler(), 0, mask)
    masked = logits.copy()
    masked[best] = -np.inf
    assert tok == int(np.argmax(masked))


def test_batched_decode_matches_single(models):
    eng, ora = models["llama_tiny"]
    V = eng.config.vocab_size
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, V, n).tolist() for n in (5, 17, 40, 66)]
    samplers = [smotor.Sampler(), smotor.Sampler(1.0, 40, 0.9), smotor.Sampler(0.8, 10, None), smotor.Sampler()]
    caches, singles = [], []
    for p in prompts:
        c = eng.new_cache(128)
        eng.forward_cached(c, p[:-1], logits=False)
        caches.append(c)
        singles.append(c.clone())
    toks = [p[-1] for p in prompts]
    states = [smotor.rng_seed(i) for i in range(4)]
    s_toks, s_states = list(toks), list(states)
    for step in range(6):
        out, st = eng.decode_batch(caches, toks, samplers, states)
        for i in range(4):
            t, s_states[i] = eng.forward_sample(singles[i], [s_toks[i]], samplers[i], s_states[i])
            s_toks[i] = t
        assert out.tolist() == s_toks, step
        assert [int(v) for v in st] == s_states
        toks, states = out.tolist(), [int(v) for v in st]
    assert [len(c) for c in caches] == [len(p) - 1 + 6 for p in prompts]


def test_cache_outlives_model_handle(tmp_path):
    p = str(tmp_path / "m.gguf")
    smotor.synth_write(smotor.synth_spec(n_layers=1, vocab=300), p)
    m = smotor.Model.load(p, max_context=256)
    c = m.new_cache(16)
    m.forward_cached(c, [1, 2, 3], logits=False)
    c2 = c.clone()
    m.free()  # the caches keep the model alive
    assert len(c2) == 3
    c.free()
    c2.free()


def test_cache_ops(models):
    eng, _ = models["qwen2_tiny"]
    c = eng.new_cache(40)
    eng.forward_cached(c, [1, 2, 3, 4, 5], logits=False)
    snap = c.clone()
    l1 = eng.forward_cached(c, [6])
    assert len(snap) == 5 and len(c) == 6
    l2 = eng.forward_cached(snap, [6])
    assert np.array_equal(l1, l2)  # same device state, same kernels -> same bits
    c.truncate(5)
    assert np.array_equal(eng.forward_cached(c, [6]), l1)
    with pytest.raises(smotor.EngineError) as e:
        c.truncate(50)
    assert e.value.status == 8
    c.ensure_capacity(100)
    assert c.capacity() == 100 and len(c) == 6
    assert np.array_equal(eng.forward_cached(c, [7]), eng.forward_cached(snap, [7]))
    small = eng.new_cache(3)
    with pytest.raises(smotor.EngineError) as e:
        eng.forward_cached(small, [1, 2, 3, 4])
    assert e.value.status == 7
    with pytest.raises(smotor.EngineError):
        eng.forward_cached(small, [eng.config.vocab_size])  # token out of range


def test_seeded_generation_equals_plain(models):
    eng, _ = models["qwen2_tiny"]
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    base = eng.generate(prompt, 20)
    snap = {}
    eng.generate(prompt, 20, on_prefill=lambda c: snap.setdefault("c", c.clone()))
    seed = snap["c"]
    seed.truncate(5)
    out = eng.generate(prompt, 20, seed_cache=seed, seed_n=5)
    assert out.prefix_reused == 5 and out.ids == base.ids


def test_decode_run_matches_stepwise(models):
    eng, _ = models["llama_tiny"]
    V = eng.config.vocab_size
    prompts = [[5, 6, 7], list(range(40, 110)), [9, 10]]
    samplers = [smotor.Sampler(), smotor.Sampler(1.0, 40, 0.9), smotor.Sampler(0.9, 7, None)]
    runs, steps = [], []
    for p in prompts:
        c = eng.new_cache(128)
        eng.forward_cached(c, p[:-1], logits=False)
        runs.append(c)
        steps.append(c.clone())
    seeds = [smotor.rng_seed(50 + i) for i in range(3)]
    out, st = eng.decode_run(runs, [p[-1] for p in prompts], samplers, seeds, 20)
    for i in range(3):
        tok, s = prompts[i][-1], seeds[i]
        for k in range(20):
            tok, s = eng.forward_sample(steps[i], [tok], samplers[i], s)
            assert out[k, i] == tok, (i, k)
        assert int(st[i]) == s
        assert len(runs[i]) == len(steps[i])


def test_paged_prefix_sharing(models):
    """Clones share KV pages; each writer copies only the page it writes into,
    and every fork still matches the oracle's deep-copied SeqState."""
    eng, ora = models["llama_tiny"]
    prompt = list(range(100, 170))  # 70 positions: pages 0 and 1 full, page 2 holds 64..69
    c = eng.new_cache(256)
    eng.forward_cached(c, prompt, logits=False)
    held0, _, page_bytes = eng.kv_pages()
    assert page_bytes == 2 * eng.config.n_layers * 32 * eng.kv_width() * 4
    forks = [c.clone() for _ in range(3)]
    assert eng.kv_pages()[0] == held0  # nothing copied yet
    co = ora.new_cache(256)
    ora.forward_cached(co, prompt)
    conts = [[7, 8], [9], [10, 11, 12, 13]]
    first = []
    for f, t in zip(forks, conts):
        oc = co.clone()
        want = ora.forward_cached(oc, t)
        got = eng.forward_cached(f, t)
        assert rel_err(got, want) <= LOGIT_TOL and top8(got) == top8(want)
        first.append(got)
    assert eng.kv_pages()[0] == held0 + 3  # one copied page (page 2) per writer
    # the source is untouched by its forks' writes
    for layer in (0, eng.config.n_layers - 1):
        for pos in (0, 63, 64, 69):
            k, v = c.read_kv(layer, pos)
            kw, vw = co.read_kv(layer, pos)
            assert rel_err(k, kw) <= 1e-4 and rel_err(v, vw) <= 1e-4
        k, v = c.read_kv(layer, 70)
        assert not k.any() and not v.any()  # never written here
    # the source now writes its own page 2 in place (no holder shares it), and
    # the same tokens after the same prefix give forks[0]'s bits
    assert np.array_equal(eng.forward_cached(c, conts[0]), first[0])
    assert eng.kv_pages()[0] == held0 + 3
    # truncating inside a page and writing again
    forks[2].truncate(66)
    oc = co.clone()
    oc.truncate(66)
    want = ora.forward_cached(oc, [5, 6])
    got = eng.forward_cached(forks[2], [5, 6])
    assert rel_err(got, want) <= LOGIT_TOL and top8(got) == top8(want)
    for f in forks:
        f.free()
    assert eng.kv_pages()[0] == held0  # back to the source's three pages


def test_batched_decode_over_a_shared_prefix(models):
    """Forks of one prefilled state decoded as a batch: the leading KV pages
    every fork holds are read once for all of them (shared-prefix attention);
    each fork's logits must still match the oracle's deep-copied state."""
    eng, ora = models["llama_tiny"]
    V = eng.config.vocab_size
    rng = np.random.default_rng(21)
    prefix = rng.integers(0, V, 100).tolist()  # pages 0-2 full (shared), page 3 holds 96..99
    base = eng.new_cache(256)
    eng.forward_cached(base, prefix, logits=False)
    ob = ora.new_cache(256)
    ora.forward_cached(ob, prefix)
    conts = [rng.integers(0, V, n).tolist() for n in (1, 5, 9, 30, 2)]
    forks, oforks = [], []
    for c in conts:  # own tokens before the batched steps (the last one is the first step's input)
        f, of = base.clone(), ob.clone()
        if len(c) > 1:
            eng.forward_cached(f, c[:-1], logits=False)
            ora.forward_cached(of, c[:-1])
        forks.append(f)
        oforks.append(of)
    toks = [c[-1] for c in conts]
    n = len(conts)
    for step in range(6):
        out, _, lg = eng.decode_batch_logits(forks, toks, [smotor.Sampler()] * n, [0] * n)
        for i in range(n):
            want = ora.forward_cached(oforks[i], [toks[i]])
            assert rel_err(lg[i], want) <= LOGIT_TOL and top8(lg[i]) == top8(want), (step, i)
            assert int(out[i]) == int(np.argmax(lg[i]))
        toks = out.tolist()
    for f in forks:
        f.free()
    base.free()
