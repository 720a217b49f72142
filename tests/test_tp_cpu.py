"""Tensor parallelism on the host, no GPU: the split plan of the C ABI
(sm_tp_plan), and a two-rank gloo run of the Megatron split it describes
(tests/tpsim.py) against the oracle's single-process forward — the same
heads, FFN columns and output rows per rank, the same all-reduce after
attn_output and ffn_down, and the same gather of the logit slices as the
engine's GPU path. Also the group-id hand-off of smotor.TensorParallel over a
torch.distributed group."""
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

import pyoracle as orc
import smotor


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_partitions_the_70b_shape(world):
    c = smotor.config_of(80, 8192, 28672, 64, 8, 128256, 5e5, 1e-5)
    q, kv, ff, voc = [], [], [], []
    for r in range(world):
        s = smotor.tp_plan(c, r, world)
        q.append((s.q_head0, s.q_heads))
        kv.append((s.kv_head0, s.kv_heads))
        ff.append((s.ff0, s.ff))
        voc.append((s.vocab0, s.vocab))
        assert s.q_heads // s.kv_heads == 8  # GQA groups stay whole on a rank
        assert (s.q_heads * 128) % 256 == 0 and s.ff % 256 == 0  # row-split inputs are whole Q4_K/Q6_K blocks
    for parts, total in ((q, 64), (kv, 8), (ff, 28672), (voc, 128256)):
        pos = 0
        for a, n in parts:
            assert a == pos and n > 0
            pos += n
        assert pos == total


def test_plan_uneven_vocab_and_errors():
    c = smotor.config_of(2, 512, 1024, 4, 2, 1001)
    rows = [smotor.tp_plan(c, r, 2) for r in range(2)]
    assert (rows[0].vocab0, rows[0].vocab, rows[1].vocab0, rows[1].vocab) == (0, 501, 501, 500)
    with pytest.raises(smotor.EngineError):  # 2 kv heads do not split 4 ways
        smotor.tp_plan(c, 0, 4)
    with pytest.raises(smotor.EngineError):
        smotor.tp_plan(c, 2, 2)
    with pytest.raises(smotor.EngineError):
        smotor.tp_plan(smotor.config_of(2, 4096, 8192, 32, 16, 1000), 0, 16)


def _worker(rank, world, port, path, tokens, outdir):
    import torch
    import torch.distributed as dist
    import tpsim
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        tp = smotor.TensorParallel.from_process_group()

        def all_reduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            dist.all_reduce(t)
            return t.numpy()

        def all_gather(a):
            out = [None] * world
            dist.all_gather_object(out, a)
            return out

        logits = tpsim.forward(tpsim.Gguf(path), tokens, rank, world, all_reduce, all_gather)
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), logits=logits, gid=np.frombuffer(tp.group_id, np.uint8),
                 size=tp.size, rank=tp.rank)
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def llama_tiny(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("tp") / "llama_tiny.gguf")
    smotor.synth_write(smotor.synth_spec(arch="llama", n_embd=512, n_layers=2, n_heads=4, n_kv_heads=2, n_ff=1024,
                                         vocab=512, qkv_bias=True, weight_std=0.05, seed=11), p)
    return p


@pytest.mark.parametrize("world", [1, 2])
def test_split_forward_matches_oracle_gloo(llama_tiny, tmp_path, world):
    import torch.multiprocessing as mp
    tokens = [3, 77, 150, 9, 401, 256, 12]
    mp.start_processes(_worker, args=(world, free_port(), llama_tiny, tokens, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    outs = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    ref = orc.Model(llama_tiny)
    want = ref.forward_cached(ref.new_cache(16), tokens).astype(np.float64)
    for r, o in enumerate(outs):
        got = o["logits"]
        assert int(o["rank"]) == r and int(o["size"]) == world
        assert np.array_equal(o["gid"], outs[0]["gid"])  # one group id for every rank
        err = np.abs(got - want).max() / np.abs(want).max()
        assert err < 1e-5, err
        assert set(np.argsort(-got)[:8]) == set(np.argsort(-want)[:8])
        assert np.allclose(got, outs[0]["logits"], rtol=0, atol=1e-9)
