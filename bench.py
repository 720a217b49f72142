"""Decode benchmark of the siliceo-motor B200 engine (one JSON line on rank 0).

Default workload: Qwen2.5-7B-shaped Q4_K_M GGUF (seeded synthetic weights),
batch 1, 512-token random prompt, greedy decode. A "step" is one decode step
(one token for each sequence). The metric is decode tokens/s, with the
achieved HBM bandwidth against the measured peak in `roofline`.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2|cfg0|cfg3]
  python bench.py --impl reference ...   # the reference CPU path (oracle port)

N > 1 (torchrun): every rank decodes its own replica (the single-sequence
decode path has no partition, so `value` is weak scaling with no
collective); the timed region is bracketed by barriers and the max over
ranks is used. The same job then splits the 70B shape (config 4) over its N
GPUs (tensor parallelism, two all-reduces per layer) and adds that
measurement as `tensor_parallel` to the line (--no-tp-leg skips it).
--workload cfg4 / cfg4b16 make the split model the headline instead.
"""
import argparse
import fcntl
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "siliceo-motor_b200"))

WORKLOADS = {
    # name: (preset, batch, prompt_len, sampler, description)
    "cfg2": (2, 1, 512, "greedy", "Qwen2.5-7B-shape Q4_K_M, batch 1, 512-token prompt, greedy decode"),
    "cfg0": (0, 1, 128, "greedy", "Qwen2.5-0.5B-shape Q4_K_M (Q5_0/Q8_0 fallbacks), batch 1, 128-token prompt"),
    "cfg3": (3, 32, 2048, "topk40_topp0.9",
             "Llama-3-8B-shape Q4_K_M, 32 sequences, 1024 shared + 1024 own prompt tokens, T=1 top-k 40 top-p 0.9"),
    # tensor parallel over every rank of the job (one model split N ways)
    "cfg4": (4, 1, 1024, "greedy", "Llama-3-70B-shape Q4_K_M, tensor parallel, batch 1, 1024-token prompt, greedy"),
    "cfg4b16": (4, 16, 1024, "greedy",
                "Llama-3-70B-shape Q4_K_M, tensor parallel, 16 sequences of 1024-token prompts, greedy"),
}
TP_WORKLOADS = {"cfg4", "cfg4b16"}
HBM_FALLBACK_GBS = 6650.0
GEMV_SHAPES = [(896, 4864), (3584, 18944), (4096, 14336), (8192, 28672)]  # BASELINE config 1 (M x K)


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return HBM_FALLBACK_GBS, "fallback"


def cache_dir(size_hint=0):
    """Where synthetic GGUFs are kept: SM_CACHE_DIR, else RAM-backed /dev/shm
    for a file that fits there with room to spare (a 70B-shape file is written
    at memory speed instead of disk speed), else the temp directory."""
    if os.environ.get("SM_CACHE_DIR"):
        return os.environ["SM_CACHE_DIR"]
    if size_hint:
        try:
            st = os.statvfs("/dev/shm")
            if st.f_bavail * st.f_frsize > 1.5 * size_hint:
                return "/dev/shm/smotor_cache"
        except OSError:
            pass
    return os.path.join(tempfile.gettempdir(), "smotor_cache")


def model_file(preset: int, local_rank: int, barrier, size_hint=0) -> str:
    """The synthetic GGUF of a preset, generated once per machine and reused.
    It is written by a child process, so that the calling process (the
    reference arm among them) never loads the engine's library."""
    d = cache_dir(size_hint)
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"preset{preset}_seed0_v1.gguf")
    if local_rank == 0:
        with open(path + ".lock", "w") as lk:
            fcntl.flock(lk, fcntl.LOCK_EX)
            if not os.path.exists(path):
                code = ("import sys; sys.path.insert(0, %r); import smotor; "
                        "smotor.synth_write(smotor.synth_preset(%d), %r)" % (os.path.join(ROOT, "siliceo-motor_b200"),
                                                                             preset, path + ".part"))
                subprocess.run([sys.executable, "-c", code], check=True)
                os.replace(path + ".part", path)
            fcntl.flock(lk, fcntl.LOCK_UN)
    barrier()
    return path


class Clocks:
    """nvidia-smi samples during the timed region (clocks + throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self, gpus):
        if not self.proc:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        self.f.flush()
        rows = []
        with open(self.f.name) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9 and p[0].isdigit() and int(p[0]) in gpus:
                    rows.append(p)
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def sampler_for(kind):
    import smotor
    return smotor.Sampler() if kind == "greedy" else smotor.Sampler(1.0, 40, 0.9)


def setup_sequences(model, V, batch, prompt_len, kind, extra, prefill=None):
    """Prefill the workload's prompts; returns (caches, next tokens). With
    `prefill` (a dict), a batch-1 prompt's prefill is timed: one untimed pass
    on a scratch cache first, then the measured one (CUDA events on the
    engine's stream around sm_forward_cached)."""
    rng = np.random.default_rng(0)
    cap = prompt_len + extra
    if batch == 1:
        prompt = rng.integers(0, V, prompt_len).tolist()
        if prefill is not None:
            import torch
            scratch = model.new_cache(cap)
            model.forward_cached(scratch, prompt[:-1], logits=False)  # warm-up (kernel set-up, page pool)
            scratch.free()
            ext = torch.cuda.ExternalStream(model.stream())
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c = model.new_cache(cap)
        if prefill is not None:
            torch.cuda.synchronize()
            e0.record(ext)
        model.forward_cached(c, prompt[:-1], logits=False)
        if prefill is not None:
            e1.record(ext)
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            prefill.update({"tokens": prompt_len - 1, "ms": ms, "tok_per_s": (prompt_len - 1) / (ms / 1e3),
                            "api": "sm_forward_cached (32-row chunks on the batched tcgen05 GEMV)"})
        return [c], [prompt[-1]]
    # shared 1024-token prefix prefilled once, cloned per sequence (prefix cache)
    shared = rng.integers(0, V, prompt_len // 2).tolist()
    base = model.new_cache(cap)
    model.forward_cached(base, shared, logits=False)
    caches, toks = [], []
    for i in range(batch):
        own = rng.integers(0, V, prompt_len - len(shared)).tolist()
        c = base.clone()
        model.forward_cached(c, own[:-1], logits=False)
        caches.append(c)
        toks.append(own[-1])
    base.free()
    return caches, toks


def cpu_decode(path, prompt_len, steps, warmup, single_steps):
    """The oracle (the reference's CPU path restated in C++: the same f32
    operations in the same order) decoding greedily at the workload's context:
    the prompt prefilled on all host cores, then `warmup` untimed and `steps`
    timed decode steps on all cores, then `single_steps` timed steps on one
    core (the reference's own execution model: it has no threading)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as orc
    threads = os.cpu_count() or 1
    m = orc.Model(path, threads=threads)
    V = m.config.vocab_size
    prompt = np.random.default_rng(0).integers(0, V, prompt_len).tolist()
    c = m.new_cache(prompt_len + warmup + steps + single_steps + 8)
    tok = int(np.argmax(m.forward_cached(c, prompt)))
    for _ in range(warmup):
        tok = int(np.argmax(m.forward_cached(c, [tok])))
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = int(np.argmax(m.forward_cached(c, [tok])))
    dt = time.perf_counter() - t0
    single = None
    if single_steps:
        m.set_threads(1)
        t1 = time.perf_counter()
        for _ in range(single_steps):
            tok = int(np.argmax(m.forward_cached(c, [tok])))
        ds = (time.perf_counter() - t1) / single_steps
        single = {"s_per_token": ds, "value": 1.0 / ds, "unit": "tok/s", "cores": 1,
                  "sample": f"{single_steps} greedy decode steps on one core, context {prompt_len + warmup + steps + 1}"
                            f"..{prompt_len + warmup + steps + single_steps}"}
    return steps / dt, threads, single


def cpu_baseline(path, prompt_len):
    """Bounded CPU-baseline leg of the engine's line (rank 0, N = 1)."""
    val, threads, single = cpu_decode(path, prompt_len, steps=6, warmup=1, single_steps=2)
    out = {"value": val, "unit": "tok/s", "cores": threads, "kind": "port",
           "sample": f"6 greedy decode steps on {threads} threads after the workload's {prompt_len}-token prompt "
                     f"(context {prompt_len + 2}..{prompt_len + 7})"}
    if single:
        out["single_thread"] = single
    return out


def run_reference(args, rank, world, local_rank, barrier):
    preset, batch, prompt_len, kind, desc = WORKLOADS[args.workload]
    if rank != 0:
        return
    path = model_file(preset, 0, lambda: None)
    val, threads, single = cpu_decode(path, prompt_len, args.steps, args.warmup, 2 if preset != 4 else 0)
    sample = (f"{args.steps} greedy decode steps (batch 1) after a {prompt_len}-token prompt (context "
              f"{prompt_len + args.warmup + 1}..{prompt_len + args.warmup + args.steps}); the reference's f32 "
              f"forward_cached restated in C++ and threaded over independent outputs")
    base = {"value": val, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}
    if single:
        base["single_thread"] = single
    print(json.dumps({
        "impl": "reference", "metric": "decode_tok_per_s", "value": val, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / val,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "description": desc + " (reference CPU path, batch 1)"},
        "cpu_baseline": base,
        "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_gemv(args, rank, world, local_rank, barrier, allmax):
    """Config 1: the dequant-fused GEMV alone, Q4_K and Q6_K, batch 1/8/32.
    Each launch is timed between CUDA events after an L2 flush (a 512 MB
    write), so every launch streams its weights from HBM."""
    import torch
    import smotor
    torch.cuda.set_device(local_rank)
    st = torch.cuda.current_stream()
    # L2 flush by reading 512 MB: leaves clean lines, so no write-back lands in the timed launch
    flush = torch.ones(128 << 20, dtype=torch.float32, device="cuda")
    peak, peak_kind = peaks()
    rng = np.random.default_rng(1)
    rows = []
    only = args.only.split(":") if args.only else None
    for (M, K) in GEMV_SHAPES:
        if only and only[0] != f"{M}x{K}":
            continue
        wf = rng.normal(0, 1, M * K).astype(np.float32)
        for qt, name in ((smotor.Q4_K, "Q4_K"), (smotor.Q6_K, "Q6_K")):
            if only and only[1] != name:
                continue
            w = smotor.DWeight(qt, smotor.quantize(qt, wf), M, K)
            x = torch.randn(32, K, device="cuda")
            y = torch.empty(32, M, device="cuda")
            for b in (1, 8, 32):
                if only and int(only[2]) != b:
                    continue
                times = []
                for it in range(args.warmup + args.steps):
                    flush.sum()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                    w.gemv(x.data_ptr(), y.data_ptr(), b, st.cuda_stream)
                    e1.record(st)
                    e1.synchronize()
                    if it >= args.warmup:
                        times.append(e0.elapsed_time(e1))
                ms = statistics.median(times)
                nbytes = w.nbytes() + 4 * b * (K + M)
                rows.append({"shape": f"{M}x{K}", "type": name, "batch": b, "us": ms * 1e3,
                             "gbs": nbytes / (ms / 1e3) / 1e9, "frac": nbytes / (ms / 1e3) / 1e9 / peak})
            w.free()
    head = ([r for r in rows if r["shape"] == "3584x18944" and r["type"] == "Q4_K" and r["batch"] == 1] or rows)[0]
    print(json.dumps({
        "metric": "gemv_GBps", "value": head["gbs"], "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["us"] / 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (Q4_K/Q6_K weights)", "data": "synthetic N(0,1) weights, seed 1",
        "config": {"workload": "gemv", "headline": "Q4_K 3584x18944 batch 1", "l2": "flushed before every launch",
                   "results": rows},
        "roofline": {"bound": "hbm", "achieved": head["gbs"], "peak": peak, "unit": "GB/s",
                     "frac": head["gbs"] / peak, "traffic": None, "peak_source": peak_kind},
    }), flush=True)


# The dominant kernel of a decode step: the tensor-core batch-1 GEMV, on the
# step's largest launch shape (the interleaved gate/up projection of the 7B
# shape, Q4_K). Its DRAM traffic per launch comes from the ncu capture
# summarised in profiles/ (the bench cannot run ncu itself).
DOMINANT = (37888, 3584, "Q4_K")
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "roofline_traffic.json")


def kernel_roofline(steps, warmup, shape=DOMINANT):
    """Average duration of the dominant kernel over `steps` standalone launches:
    CUDA events on the launching stream, the L2 flushed before each launch by a
    512 MB read that is enqueued first (so the GPU never waits for the host)."""
    import torch
    import smotor
    M, K, tname = shape
    st = torch.cuda.current_stream()
    flush = torch.ones(128 << 20, dtype=torch.float32, device="cuda")
    rng = np.random.default_rng(7)
    qt = getattr(smotor, tname)
    w = smotor.DWeight(qt, smotor.quantize(qt, rng.normal(0, 0.02, M * K).astype(np.float32)), M, K)
    x = torch.randn(K, device="cuda")
    y = torch.empty(M, device="cuda")
    times = []
    for it in range(warmup + steps):
        flush.sum()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        w.gemv(x.data_ptr(), y.data_ptr(), 1, st.cuda_stream)
        e1.record(st)
        e1.synchronize()
        if it >= warmup:
            times.append(e0.elapsed_time(e1))
    nbytes = w.nbytes() + 4 * (K + M)
    w.free()
    del flush
    us = 1e3 * sum(times) / len(times)
    traffic = None
    if os.path.exists(TRAFFIC_FILE):
        with open(TRAFFIC_FILE) as f:
            traffic = json.load(f).get("gemv_tc %dx%d %s batch 1" % shape)
    return nbytes, us, traffic


def tensor_parallel_leg(args, rank, world, local_rank, barrier, allmax):
    """Config 4 (Llama-3-70B shape) split over the job's ranks (tensor
    parallelism with the engine's peer-memory exchanges): batch 1, 1024-token
    prompt, greedy, K timed decode steps. Run by every rank after the replica
    measurement of a multi-GPU job; returns the summary on rank 0."""
    import torch
    import smotor
    preset, batch, prompt_len, kind, desc = WORKLOADS["cfg4"]
    size = smotor.synth_size(smotor.synth_preset(preset))
    path = model_file(preset, local_rank, barrier, size_hint=size)
    extra = args.warmup + 2 * args.steps + 8
    tp = smotor.TensorParallel.from_process_group()
    model = smotor.Model.load(path, device=local_rank, max_batch=32, max_context=prompt_len + extra + 64, tp=tp)
    cfg = model.config
    caches, toks = setup_sequences(model, cfg.vocab_size, 1, prompt_len, kind, extra)
    samplers, states = [smotor.Sampler()], [0]
    ext = torch.cuda.ExternalStream(model.stream())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # recorded once through torch, which otherwise refuses elapsed_time on
    # events that only the engine records
    ev0.record(ext)
    ev1.record(ext)
    torch.cuda.synchronize()
    out, states = model.decode_run(caches, toks, samplers, states, max(args.warmup, 1))
    toks = out[-1].tolist()
    pos0 = len(caches[0])
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks() if rank == 0 else None
    if clocks:
        clocks.start()
    out, states = model.decode_run(caches, toks, samplers, states, args.steps, ev0.cuda_event, ev1.cuda_event)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop(set(range(world))) if clocks else None
    ms = allmax(ev0.elapsed_time(ev1))
    toks = out[-1].tolist()
    # one untimed step through the per-token API first (its step graph is captured there)
    t, states[0] = model.forward_sample(caches[0], [toks[0]], samplers[0], int(states[0]))
    toks = [t]
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        t, states[0] = model.forward_sample(caches[0], [toks[0]], samplers[0], int(states[0]))
        toks = [t]
    torch.cuda.synchronize()
    e2e_s = allmax(time.perf_counter() - t0)
    wbytes = int(allsum(model.weight_bytes()))
    step_kernels = model.step_launches(1)
    model.free()  # every rank at the same point (the group's teardown barrier)
    if rank != 0:
        return None
    kv_bytes = 2 * cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 4 * sum(pos0 + i + 1 for i in range(args.steps))
    alg = args.steps * wbytes + kv_bytes
    peak, peak_kind = peaks()
    achieved = alg / (ms / 1e3) / 1e9
    return {"workload": "cfg4", "description": desc, "tp": world, "value": args.steps / (ms / 1e3),
            "unit": "tok/s", "ms_per_step": ms / args.steps, "steps": args.steps,
            "e2e": {"value": args.steps / e2e_s, "unit": "tok/s", "api": "sm_forward_sample"},
            "exchanges": "peer-memory pushes from the row-split GEMV epilogues (2 all-reduces per layer, one "
                         "logit gather per step)",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak * world, "unit": "GB/s",
                         "frac": achieved / (peak * world), "bytes_per_step": alg / args.steps,
                         "peak_source": peak_kind, "note": "all ranks' weight shards + KV per step / step time, "
                                                           "against %d x the per-GPU peak" % world},
            "gpu_launches": world * args.steps * step_kernels, "clocks": clk}


def run_ours(args, rank, world, local_rank, barrier, allmax):
    import torch
    import smotor

    preset, batch, prompt_len, kind, desc = WORKLOADS[args.workload]
    torch.cuda.set_device(local_rank)
    path = model_file(preset, local_rank, barrier)
    extra = args.warmup + 2 * args.steps + 8
    split = args.workload in TP_WORKLOADS and world > 1
    tp = smotor.TensorParallel.from_process_group(flags=smotor.TP_NCCL if args.tp_nccl else 0) if split else None
    model = smotor.Model.load(path, device=local_rank, max_batch=max(32, batch), max_context=prompt_len + extra + 64,
                              tp=tp)
    cfg = model.config
    V, L, kvd = cfg.vocab_size, cfg.n_layers, cfg.n_kv_heads * cfg.head_dim
    prefill = {} if batch == 1 and not split else None
    caches, toks = setup_sequences(model, V, batch, prompt_len, kind, extra, prefill)
    samplers = [sampler_for(kind)] * batch
    states = [smotor.rng_seed(i) for i in range(batch)]
    ext = torch.cuda.ExternalStream(model.stream())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(ext)
    ev1.record(ext)
    torch.cuda.synchronize()
    # warm-up (graph capture happens here)
    out, states = model.decode_run(caches, toks, samplers, states, max(args.warmup, 1))
    toks = out[-1].tolist()
    pos0 = [len(c) for c in caches]
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks() if rank == 0 else None
    if clocks:
        clocks.start()
    # a profiler started with capture off (ncu --profile-from-start off) sees only the timed steps
    torch.cuda.profiler.start()
    out, states = model.decode_run(caches, toks, samplers, states, args.steps, ev0.cuda_event, ev1.cuda_event)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    barrier()
    clk = clocks.stop(set(range(max(world, 1)))) if clocks else None
    ms = allmax(ev0.elapsed_time(ev1))
    # bytes the whole job streams per step: every rank's shard (tensor parallel) or one replica's weights
    wbytes_job = int(allsum(model.weight_bytes())) if split else model.weight_bytes() * world
    toks = out[-1].tolist()
    # end to end through the per-token public API (host tokens in and out);
    # one untimed step first, in which that API captures its step graph
    def api_step(toks, states):
        if batch == 1:
            t, states[0] = model.forward_sample(caches[0], [toks[0]], samplers[0], int(states[0]))
            return [t], states
        o, states = model.decode_batch(caches, toks, samplers, states)
        return o.tolist(), states

    toks, states = api_step(toks, states)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        toks, states = api_step(toks, states)
    torch.cuda.synchronize()
    e2e_s = allmax(time.perf_counter() - t0)
    barrier()
    h2d, d2h = model.step_io_bytes()
    step_kernels = model.step_launches(batch)  # kernel nodes of the decode-step graph
    model.free()  # every rank at the same point (tensor parallel: the group's teardown barrier)
    for c in caches:
        c.free()
    tp_line = None
    if world > 1 and not split and not args.no_tp_leg:  # the 70B shape split over this job's GPUs
        tp_line = tensor_parallel_leg(args, rank, world, local_rank, barrier, allmax)
    if rank != 0:
        return
    # KV bytes read by attention over the timed steps: positions 0..pos per layer, K and V, f32
    # (the whole model's KV heads: one replica's per rank, or all ranks' shards together)
    kv_positions = sum(sum(p + i + 1 for i in range(args.steps)) for p in pos0)
    kv_bytes = 2 * L * kvd * 4 * kv_positions * (1 if split else world)
    alg_bytes = args.steps * wbytes_job + kv_bytes
    peak, peak_kind = peaks()
    step_achieved = alg_bytes / (ms / 1e3) / 1e9
    step_peak = peak * world
    if split:  # dominant launch of a rank: its gate/up shard
        shape = (2 * cfg.n_ff // world, cfg.n_embd, "Q4_K")
    else:
        shape = DOMINANT
    kbytes, kus, ktraffic = kernel_roofline(max(args.steps, 10), 3, shape)
    achieved = kbytes / (kus / 1e6) / 1e9
    tokens = batch * args.steps * (1 if split else world)
    value = tokens / (ms / 1e3)
    line = {
        "metric": "decode_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if split else "weak",
        "vs_baseline": None, "dtype": "f32 (Q4_K_M weights)", "data": "synthetic (seeded N(0,0.02) GGUF, random ids)",
        "config": {"workload": args.workload, "description": desc, "batch": batch, "prompt_len": prompt_len,
                   "parallelism": (f"tensor parallel x{world} ({'NCCL' if args.tp_nccl else 'peer-memory'} "
                                   f"exchanges)") if split else (f"replicas x{world}" if world > 1 else "single GPU"),
                   "l2": "inputs larger than L2 (%.2f GB of weights streamed per step per GPU)"
                         % (wbytes_job / world / 1e9),
                   "timed": "sm_decode_run: K device-resident graph replays between CUDA events on the engine stream"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": ktraffic, "peak_source": peak_kind,
                     "kernel": "gemv_tc (batch-1 tensor-core GEMV) on %dx%d %s: %.1f us per launch, %d algorithmic "
                               "bytes per launch; standalone launches, L2 flushed" % (shape + (kus, kbytes)),
                     "step": {"achieved": step_achieved, "frac": step_achieved / step_peak,
                              "bytes_per_step": alg_bytes / args.steps, "peak": step_peak,
                              "note": "weights + KV the whole job reads per decode step / step time, against "
                                      "%d x the per-GPU peak" % world}},
        "e2e": {"value": tokens / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": "sm_forward_sample" if batch == 1 else "sm_decode_batch"},
        # per step and rank: embed+norm; per layer QKV (batched: one launch per weight type, 2), attention
        # split, combine, O, gate/up, down; head, sampler, record; tensor parallel adds 2 all-reduce
        # kernels per layer and the logit gather
        "gpu_launches": world * args.steps * step_kernels,
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline and args.workload not in TP_WORKLOADS:
        line["cpu_baseline"] = cpu_baseline(path, prompt_len)
    if prefill:
        line["prefill"] = prefill
    if tp_line is not None:
        line["tensor_parallel"] = tp_line
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg2", choices=list(WORKLOADS) + ["gemv", "dominant"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", default="", help="gemv workload: one MxK:TYPE:batch case, e.g. 3584x18944:Q4_K:1")
    ap.add_argument("--tp-nccl", action="store_true", help="tensor parallel: NCCL collectives instead of the "
                                                            "engine's peer-memory exchange kernels")
    ap.add_argument("--no-tp-leg", action="store_true", help="multi-GPU jobs: skip the tensor-parallel config-4 "
                                                              "measurement added to the replica line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    barrier = lambda: None  # noqa: E731
    allmax = lambda v: v  # noqa: E731
    global allsum
    allsum = lambda v: v  # noqa: E731
    if args.impl == "reference":  # rank 0 alone times the CPU path; other ranks exit
        run_reference(args, rank, world, local_rank, barrier)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))

        def barrier():
            dist.barrier()

        def allmax(v):
            t = torch.tensor([float(v)], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        def allsum(v):
            t = torch.tensor([float(v)], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            return float(t.item())
    try:
        if args.workload == "dominant":  # the roofline kernel alone (what profiles/ captures with ncu)
            import torch
            torch.cuda.set_device(local_rank)
            nbytes, us, traffic = kernel_roofline(args.steps, args.warmup)
            print(json.dumps({"kernel": "gemv_tc %dx%d %s batch 1" % DOMINANT, "us": us, "bytes": nbytes,
                              "gbs": nbytes / us / 1e3, "traffic": traffic}), flush=True)
        else:
            (run_gemv if args.workload == "gemv" else run_ours)(args, rank, world, local_rank, barrier, allmax)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
