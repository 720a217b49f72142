"""The oracle's model path: SeqState semantics (crates/s-models/src/state.rs
tests), the forward_cached contract (prefill + decode == one prefill,
device.rs:12-16), and its generation loop against the same FakeDevice cases."""
import numpy as np
import pytest

import pyoracle as orc
import smotor


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("m") / "tiny.gguf")
    smotor.synth_write(smotor.synth_spec(n_embd=256, n_layers=2, n_heads=4, n_kv_heads=2, n_ff=512, vocab=512,
                                         weight_std=0.5, seed=3), p)
    return p


def test_config_from_gguf(tiny):
    m = orc.Model(tiny)
    c = m.config
    assert (c.n_layers, c.n_embd, c.n_ff, c.n_heads, c.n_kv_heads, c.head_dim, c.vocab_size) == \
        (2, 256, 512, 4, 2, 64, 512)
    assert np.float32(c.rope_theta) == np.float32(1e6) and np.float32(c.rms_eps) == np.float32(1e-6)


def test_seqstate_semantics(tiny):
    m = orc.Model(tiny)
    st = m.new_cache(16)
    assert len(st) == 0 and st.capacity() == 16
    m.forward_cached(st, [1, 2, 3])
    assert len(st) == 3
    k2, v2 = st.read_kv(1, 2)
    snap = st.clone()
    m.forward_cached(st, [4])
    assert len(snap) == 3 and len(st) == 4
    assert np.array_equal(snap.read_kv(1, 2)[0], k2)
    with pytest.raises(ValueError):
        st.truncate(5)  # truncate refuses to grow (state.rs:493-499)
    st.truncate(1)
    assert len(st) == 1
    st.ensure_capacity(32)
    assert st.capacity() == 32 and len(st) == 1
    st.reset()
    assert len(st) == 0


def test_prefill_plus_decode_equals_single_prefill(tiny):
    m = orc.Model(tiny)
    toks = [5, 17, 300, 2, 99, 7]
    a = m.new_cache(16)
    la = m.forward_cached(a, toks)
    b = m.new_cache(16)
    m.forward_cached(b, toks[:3])
    m.forward_cached(b, toks[3:5])
    lb = m.forward_cached(b, toks[5:])
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    for layer in range(2):
        for pos in range(6):
            assert np.array_equal(a.read_kv(layer, pos)[0], b.read_kv(layer, pos)[0])


def test_threads_do_not_change_results(tiny):
    m1 = orc.Model(tiny, threads=1)
    m8 = orc.Model(tiny, threads=8)
    toks = [1, 2, 3, 4, 5, 6, 7, 8, 9]
    l1 = m1.forward_cached(m1.new_cache(16), toks)
    l8 = m8.forward_cached(m8.new_cache(16), toks)
    assert np.array_equal(l1.view(np.uint32), l8.view(np.uint32))


def test_capacity_overflow_is_an_error(tiny):
    m = orc.Model(tiny)
    c = m.new_cache(2)
    with pytest.raises(ValueError, match="capacity"):
        m.forward_cached(c, [1, 2, 3])


def test_oracle_generate_seeded_equals_plain(tiny):
    m = orc.Model(tiny)
    base = m.generate([1, 2, 3, 4], 12)
    snap = {}
    m.generate([1, 2, 3, 4], 12, on_prefill=lambda c: snap.setdefault("c", c))
    seed = snap["c"]
    seed.truncate(3)
    out = m.generate([1, 2, 3, 4], 12, seed_cache=seed, seed_n=3)
    assert out["prefix_reused"] == 3 and out["ids"] == base["ids"]
