"""One rank of a tensor-parallel engine run, started as a process per GPU by
tests/test_gpu_tp.py. Rank 0 makes the group id and hands it to the other
ranks through a torch.distributed TCPStore on 127.0.0.1.

Modes:
  parity  prefill + teacher-forced decode logits, greedy generation, device
          decode run and seeded sampling; everything goes to rank<r>.npz.
  stall   after one good forward, rank 1 stops taking part (alive, its memory
          still mapped); rank 0's next forward must fail with SM_ERR_PEER
          within the wait bound, later calls at once; then both tear down.
  leave   rank 1 announces on the store that it leaves between steps and
          quits; rank 0 learns it on the host before its next launch and
          aborts its group.
"""
import argparse
import os
import sys
import time
from datetime import timedelta

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "siliceo-motor_b200"))

import smotor  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--path", required=True)
    ap.add_argument("--rank", type=int, required=True)
    ap.add_argument("--world", type=int, required=True)
    ap.add_argument("--port", type=int, required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--flags", type=int, default=0)
    ap.add_argument("--wait-ms", type=int, default=0)
    ap.add_argument("--mode", default="parity", choices=["parity", "stall", "leave"])
    ap.add_argument("--prompt", default="")
    ap.add_argument("--forced", default="")
    a = ap.parse_args()
    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", a.port, a.world, a.rank == 0, timedelta(seconds=120))
    if a.rank == 0:
        store.set("gid", smotor.tp_group_id())
    gid = store.get("gid")
    tp = smotor.TensorParallel(a.rank, a.world, gid, a.flags, a.wait_ms)
    m = smotor.Model.load(a.path, device=a.rank, max_batch=8, max_context=1024, tp=tp)
    prompt = [int(t) for t in a.prompt.split(",") if t]
    forced = [int(t) for t in a.forced.split(",") if t]
    res = {}
    if a.mode == "parity":
        c = m.new_cache(256)
        logits = [m.forward_cached(c, prompt)]
        for t in forced:
            logits.append(m.forward_cached(c, [t]))
        res["logits"] = np.stack(logits)
        L = m.config.n_layers
        res["kv"] = np.stack([np.concatenate(c.read_kv(layer, pos)) for layer in (0, L - 1)
                              for pos in (0, len(prompt) - 1, len(c) - 1)])
        res["greedy"] = np.asarray(m.generate(prompt, 48).ids, np.uint32)
        # device-resident decode of two sequences at once
        cs = [m.new_cache(256), m.new_cache(256)]
        first = []
        for i, cc in enumerate(cs):
            first.append(int(np.argmax(m.forward_cached(cc, prompt[: len(prompt) - i]))))
        toks, _ = m.decode_run(cs, first, [smotor.Sampler()] * 2, [0, 0], 24)
        res["run"] = np.asarray(toks, np.uint32)
        res["run_first"] = np.asarray(first, np.uint32)
        # seeded top-k / top-p sampling (identical on every rank)
        g = m.generate(prompt, 32, temperature=1.0, top_k=40, top_p=0.9, seed=7)
        res["sampled"] = np.asarray(g.ids, np.uint32)
        res["weight_bytes"] = np.uint64(m.weight_bytes())
    elif a.mode == "stall":
        c = m.new_cache(64)
        m.forward_cached(c, prompt[:4])  # every rank takes part
        if a.rank == 0:
            t0 = time.time()
            try:
                m.forward_cached(c, [prompt[4]])
                res["status"] = 0
            except smotor.EngineError as e:
                res["status"] = e.status
            res["fail_s"] = time.time() - t0
            t1 = time.time()
            try:
                m.forward_cached(c, [prompt[5]])
                res["status2"] = 0
            except smotor.EngineError as e:
                res["status2"] = e.status
            res["again_s"] = time.time() - t1
            store.set("failed", b"1")
        else:
            store.wait(["failed"], timedelta(seconds=120))  # stays alive, takes no further part
            m.tp_abort()
            try:
                m.forward_cached(c, [prompt[4]])
                res["status"] = 0
            except smotor.EngineError as e:
                res["status"] = e.status
    else:  # leave
        c = m.new_cache(64)
        m.forward_cached(c, prompt[:4])
        if a.rank == 1:
            store.set("leaving", b"1")  # between steps: nothing of this rank is in flight
            m.tp_abort()
            res["status"] = 0
        else:
            store.wait(["leaving"], timedelta(seconds=120))
            if store.check(["leaving"]):  # learned on the host before the next launch
                m.tp_abort()
            try:
                m.forward_cached(c, [prompt[4]])
                res["status"] = 0
            except smotor.EngineError as e:
                res["status"] = e.status
    m.free()
    np.savez(os.path.join(a.out, f"rank{a.rank}.npz"), **res)
    # the store's server lives in rank 0: it leaves last
    if a.rank == 0:
        store.wait([f"done{r}" for r in range(1, a.world)], timedelta(seconds=120))
    else:
        store.set(f"done{a.rank}", b"1")


if __name__ == "__main__":
    main()
