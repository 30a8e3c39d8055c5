"""Benchmark of the Q6W hot path: batched greedy decode of the tiny model.

Workload (one "step" = one full pass of the path over one batch): every
rank serves its own 8192 independent requests of the tiny synthetic model
(dim 128, 5 layers, 8 q heads, 4 kv heads, head_dim 16, SwiGLU hidden 384,
vocab 4096, FP32 KV cache of 256 positions; weights N(0, 0.02) from seed
1234, Q6W-quantized), each a 20-token prompt drawn U[3, 4095] (seeded by
rank) prefilled token by token and followed by 128 greedy tokens.  Ranks
share nothing (pure data parallelism, weak scaling).

  python bench.py [--gpus N] [--steps K] [--warmup W]
  python bench.py --impl reference ...   # the reference's CPU path (oracle port), rank 0 only

Prints one JSON line on rank 0.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "tinyllm-pynq-z2_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "generated tok/s (batched greedy decode, tiny Q6W model)"
SEED = 1234
VOCAB_LO = 3


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--n-seqs", type=int, default=8192,
                    help="sequences per GPU (with --split: sequences of the whole job)")
    ap.add_argument("--split", action="store_true",
                    help="strong scaling: the --n-seqs sequences (and the 2048 prefill prompts) are divided "
                         "across the GPUs instead of each GPU serving its own")
    ap.add_argument("--prompt-len", type=int, default=20)
    ap.add_argument("--new-tokens", type=int, default=128)
    ap.add_argument("--cpu-sample-requests", type=int, default=24,
                    help="requests per CPU worker in the CPU baseline (about 10 s of CPU work each)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--verify-sample", type=int, default=512,
                    help="sequences of the timed output teacher-forced against the oracle (all ranks together)")
    ap.add_argument("--verify-all", action="store_true",
                    help="teacher-force every sequence of the timed output against the oracle")
    ap.add_argument("--only-main", action="store_true", help="skip the B=1, GEMV and CPU side measurements")
    ap.add_argument("--profile-gemv", metavar="ROWSxCOLS", default=None,
                    help="only run one B=1 Q6W GEMV of that shape 4 times (a small case for ncu) and exit")
    ap.add_argument("--sweep-only", action="store_true", help="only run the isolated linear sweep and print it")
    ap.add_argument("--profile", choices=("b1", "prefill", "prefill_full", "attn", "sampler", "linear", "quantize"),
                    default=None,
                    help="only run one small case of that path a few times (for an ncu capture) and exit")
    ap.add_argument("--profile-scaled-step", type=int, nargs="?", const=1, default=None, metavar="N",
                    help="only run N short requests (2 + 3 tokens, default N=1) of the 1.1B-shape config and exit")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def make_model_files(d):
    from q6w_b200 import format as fmt

    b, m = Path(d) / "tiny.bin", Path(d) / "tiny.json"
    fmt.write_synthetic(fmt.TINY_ARGS, SEED, b, m)
    return b, m


def prompts_for(rank, n, length):
    import torch

    g = torch.Generator().manual_seed(10_000 + rank)
    return torch.randint(VOCAB_LO, 4096, (n, length), generator=g, dtype=torch.int64).to(torch.int32)


# ---------------------------------------------------------------- CPU side --

def _cpu_worker(args):
    """One process: B=1 greedy requests through the oracle port of the
    reference's CachedTransformer.step loop, single-threaded."""
    bin_path, man_path, prompts, new_tokens = args
    import torch

    torch.set_num_threads(1)
    from oracle.model import OracleModel, greedy_request

    m = OracleModel.from_q6w(bin_path, man_path)
    greedy_request(m, prompts[0], 4)  # warm
    t0 = time.perf_counter()
    n = 0
    for p in prompts:
        n += len(greedy_request(m, p, new_tokens)["generated"])
    return n, time.perf_counter() - t0


def cpu_throughput(bin_path, man_path, prompt_rows, new_tokens, workers, per_worker, pool=None):
    """Aggregate tok/s of `workers` single-threaded processes (one request stream each)."""
    import multiprocessing as mp

    jobs = []
    for w in range(workers):
        rows = [prompt_rows[(w * per_worker + i) % len(prompt_rows)] for i in range(per_worker)]
        jobs.append((str(bin_path), str(man_path), rows, new_tokens))
    own = pool is None
    if own:
        pool = mp.get_context("spawn").Pool(workers)
    try:
        t0 = time.perf_counter()
        res = pool.map(_cpu_worker, jobs)
        wall = time.perf_counter() - t0
    finally:
        if own:
            pool.close()
            pool.join()
    toks = sum(r[0] for r in res)
    busy = max(r[1] for r in res)
    return toks / busy, toks, busy, wall


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def _verify_chunk(job):
    """One process: teacher-forced oracle check of a chunk of device greedy streams."""
    bin_path, man_path, prompts, sampled, new_tokens, threads = job
    import torch

    torch.set_num_threads(threads)
    from oracle.model import BatchScorer, OracleModel

    m = OracleModel.from_q6w(bin_path, man_path)
    return BatchScorer(m).verify_greedy(prompts, sampled, new_tokens, chunk=len(prompts))


def verify_streams(bin_path, man_path, prompts, sampled, new_tokens, workers):
    """Teacher-force device greedy streams through the oracle (BatchScorer) in
    `workers` spawned processes; every pick must be the oracle's argmax or an
    FP32 near-tie within 1e-4 of its maximum, and every stream full length."""
    import multiprocessing as mp

    n = len(prompts)
    workers = max(1, min(workers, n))
    per = (n + workers - 1) // workers
    jobs = [(str(bin_path), str(man_path), prompts[i: i + per], sampled[i: i + per], new_tokens, 1)
            for i in range(0, n, per)]
    with mp.get_context("spawn").Pool(len(jobs)) as pool:
        res = pool.map(_verify_chunk, jobs)
    # failures carry chunk-local sequence indexes: make them indexes into `prompts`
    fails = [(f[0] + c * per,) + tuple(f[1:]) for c, r in enumerate(res) for f in r["failures"]]
    return {"checked": n, "picks": sum(r["picks"] for r in res), "exact": sum(r["exact"] for r in res),
            "near_ties": sum(r["near_ties"] for r in res), "failures": len(fails),
            "first_failures": [list(map(str, f)) for f in fails[:5]],
            "min_margin": min(r["min_margin"] for r in res)}


def _cpu_prefill_worker(job):
    """One single-thread process: the reference's prefill (the cached step over
    every prompt token, torch_benchmark.py:263-264) on a few prompts."""
    bin_path, man_path, prompts = job
    import torch

    torch.set_num_threads(1)
    from oracle.model import OracleModel

    m = OracleModel.from_q6w(bin_path, man_path)
    t0 = time.perf_counter()
    with torch.inference_mode():
        for p in prompts:
            k, v = m.new_cache()
            for pos, tok in enumerate(p):
                m.step(int(tok), pos, k, v)
    return sum(len(p) for p in prompts), time.perf_counter() - t0


def cpu_legs(bin_path, man_path, prompt, new_tokens):
    """CPU baselines of the other configurations, on this host's cores, through
    the oracle port of the reference's code path (bounded samples):
    C1 -- B=1 generate (20-token prompt + 128 tokens) at 1 thread and all cores;
    C3 -- the per-token prefill of a seeded 32-prompt subsample of the 2048
          ragged prompts, one single-thread process per core, extrapolated to
          all 2048 by prompt tokens;
    C5 -- 8 decode steps of the 1.1B-shape config (FP32 weights: the same
          cost as dequantized Q6W) after a 16-token prompt, all cores."""
    import multiprocessing as mp

    import numpy as np
    import torch

    from oracle.model import OracleArgs, OracleModel, greedy_request
    from q6w_b200 import format as fmt

    cores = cpu_cores()
    out = {"cores": cores, "kind": "port"}
    old = torch.get_num_threads()
    orc = OracleModel.from_q6w(bin_path, man_path)
    c1 = {}
    for threads in (1, cores):
        torch.set_num_threads(threads)
        greedy_request(orc, prompt, 4)
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            greedy_request(orc, prompt, new_tokens)
            ts.append(time.perf_counter() - t0)
        c1[f"{threads}_threads_tok_s"] = round(new_tokens / statistics.median(ts), 1)
    out["c1_b1_request"] = {**c1, "sample": f"median of 3 requests ({len(prompt)} + {new_tokens} tokens)"}
    # C3: subsample of the bench's prefill prompts
    rng = np.random.default_rng(2048)
    lens_all = rng.integers(8, 257, 2048)
    ids_all = rng.integers(3, 4096, (2048, 256)).astype(np.int32)
    pick = np.random.default_rng(7).choice(2048, 32, replace=False)
    prompts = [ids_all[i, : lens_all[i]].tolist() for i in pick]
    jobs = [(str(bin_path), str(man_path), prompts[w::cores]) for w in range(min(cores, len(prompts)))]
    with mp.get_context("spawn").Pool(len(jobs)) as pool:
        res = pool.map(_cpu_prefill_worker, jobs)
    toks = sum(r[0] for r in res)
    busy = max(r[1] for r in res)
    tok_s = toks / busy
    out["c3_prefill"] = {"prefill_tok_s": round(tok_s, 1), "extrapolated_ms_for_2048_prompts":
                         round(int(lens_all.sum()) / tok_s * 1e3, 1),
                         "sample": f"32 of the 2048 prompts ({toks} tokens) over {len(jobs)} single-thread processes; "
                                   "the 2048-prompt time is extrapolated by prompt tokens"}
    # C5: 1.1B shape at all cores
    torch.set_num_threads(cores)
    args = OracleArgs.from_model_args(dict(fmt.SCALED_ARGS))
    g = torch.Generator().manual_seed(3)
    shapes = fmt._model_shapes(dict(fmt.SCALED_ARGS))
    state = {k: (torch.randn(v, generator=g) * 0.02 if len(v) == 2 else torch.ones(v)) for k, v in shapes.items()}
    state["output.weight"] = state["tok_embeddings.weight"]
    big = OracleModel(args, state)
    k, v = big.new_cache()
    with torch.inference_mode():
        for pos in range(16):
            big.step(3 + pos, pos, k, v)
        t0 = time.perf_counter()
        for pos in range(16, 24):
            big.step(5 + pos, pos, k, v)
        sec = (time.perf_counter() - t0) / 8
    del big, state, k, v
    out["c5_b1_decode"] = {"ms_per_token": round(sec * 1e3, 2), "tok_s": round(1 / sec, 2),
                           "sample": "8 decode steps after a 16-token prompt, all cores"}
    torch.set_num_threads(old)
    return out


def run_reference(a):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    with tempfile.TemporaryDirectory() as d:
        b, m = make_model_files(d)
        prompts = prompts_for(0, 4096, a.prompt_len).tolist()
        cores = cpu_cores()
        import multiprocessing as mp

        pool = mp.get_context("spawn").Pool(cores)
        try:
            for _ in range(max(0, a.warmup)):
                cpu_throughput(b, m, prompts, a.new_tokens, cores, 1, pool)
            samples = [cpu_throughput(b, m, prompts, a.new_tokens, cores, 1, pool) for _ in range(a.steps)]
        finally:
            pool.close()
            pool.join()
    value = statistics.median(s[0] for s in samples)
    per_step_ms = statistics.median(s[2] for s in samples) * 1e3
    sample = (f"{cores} single-thread processes x 1 request (prompt {a.prompt_len} + {a.new_tokens} greedy "
              f"tokens, B=1 cached-step loop) per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(per_step_ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(a, world),
        "cpu_baseline": {"value": round(value, 2), "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 2), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(a, world):
    split = getattr(a, "split", False)
    per_gpu = -(-a.n_seqs // world) if split else a.n_seqs
    where = f"{a.n_seqs} sequences split across {world} GPU(s)" if split else f"{a.n_seqs} sequences per GPU"
    return {"workload": (f"batched greedy decode, tiny Q6W model (dim 128, 5 layers, 8 q / 4 kv heads, hd 16, "
                         f"hidden 384, vocab 4096, ctx 256): {where} x ({a.prompt_len}-token "
                         f"prompt + {a.new_tokens} generated), FP32 KV cache"),
            "sequences_per_gpu": per_gpu, "prompt_len": a.prompt_len, "new_tokens": a.new_tokens,
            "global_sequences": a.n_seqs if split else a.n_seqs * world,
            "parallelism": f"dp{world} (independent replicas, no collectives)",
            "l2": "inputs larger than L2: per-GPU KV cache 5.4 GB rewritten every step"}


# ---------------------------------------------------------------- GPU side --

class ClockSampler:
    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def run_b200(a):
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())

    from q6w_b200.model import Q6WCudaTransformer

    tmp = tempfile.TemporaryDirectory()
    b, m = make_model_files(tmp.name)
    model = Q6WCudaTransformer.from_q6w(b, m, device=dev)
    P, T = a.prompt_len, a.new_tokens
    if a.split:
        # one 8192-sequence job (prompts from one seed) divided across the ranks
        from q6w_b200 import dp

        lo, hi = dp.shard_range(a.n_seqs, rank, world)
        host_prompts = prompts_for(0, a.n_seqs, P)[lo:hi].contiguous().pin_memory()
        n = hi - lo
        n_job = a.n_seqs
    else:
        n = a.n_seqs
        host_prompts = prompts_for(rank, n, P).pin_memory()
        n_job = n * world
    prompts = host_prompts.to(dev)
    lens = torch.full((n,), P, dtype=torch.int32, device=dev)
    caches = model.new_batch_cache(n)
    out_host = torch.empty((n, T), dtype=torch.int32).pin_memory()

    def one(prompts_dev):
        return model.generate_greedy_device(prompts_dev, lens, P, T, caches=caches)

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up (also captures the step graph)
    for _ in range(max(a.warmup, 1)):
        sampled, n_sampled, stop_reason, _, _, ws = one(prompts)
    model.check_device_status(ws)
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    # ---- device-resident timed region
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(dev.index)
    barrier()
    torch.cuda.synchronize()
    with clk:
        start.record(stream)
        for _ in range(a.steps):
            one(prompts)
        stop.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(stop)
    clocks = clk.summary()

    # ---- end-to-end: pinned host prompts in, generated ids out, every step
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(a.steps):
        pd = host_prompts.to(dev, non_blocking=True)
        sampled, *_ = one(pd)
        out_host.copy_(sampled, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # ---- correctness of the timed output (the last end-to-end step's ids, now in out_host): a seeded
    # sample of the sequences (every sequence with --verify-all) teacher-forced through the oracle
    ok_len = bool((n_sampled == T).all().item())
    import random

    share = n if a.verify_all else min(n, max(1, a.verify_sample // world))
    pick = sorted(random.Random(4242 + rank).sample(range(n), share))
    hp = host_prompts.tolist()
    hs = out_host.tolist()
    t_v = time.perf_counter()
    par = verify_streams(b, m, [hp[i] for i in pick], [hs[i] for i in pick], T,
                         max(1, cpu_cores() // world))
    par["seconds"] = round(time.perf_counter() - t_v, 1)

    # ---- dominant kernel alone: decode attention over this run's caches
    roof = attention_roofline(model, caches, n, P + T - 1, stream)
    # single-GPU side measurements (B=1 latency, GEMV, 1.1B-shape decode, prefill): N=1 runs only, so
    # no rank waits on a collective while rank 0 measures
    side = world == 1 and not a.only_main
    b1 = b1_latency(model, host_prompts[0].tolist(), T, stream) if side else None
    gemv = scaled_gemv(dev, stream) if side else None
    sb1 = scaled_b1(dev, stream) if side else None
    # C3 prefill: at N=1, or in split mode on every rank (2048 prompts balanced by tokens, max over ranks)
    pf = prefill_c3(model, rank, world, stream) if (side or (a.split and not a.only_main)) else None
    sweep = linear_sweep(dev, stream) if side else None

    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    cnt = torch.tensor([par["checked"], par["picks"], par["exact"], par["near_ties"], par["failures"]],
                       dtype=torch.float64, device=dev)
    mm = torch.tensor([par["min_margin"]], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(cnt, op=dist.ReduceOp.SUM)
        dist.all_reduce(mm, op=dist.ReduceOp.MIN)
    ms, e2e_ms = float(t[0]), float(t[1])
    parity = {"checked_sequences": int(cnt[0]), "of_sequences": n_job, "picks": int(cnt[1]),
              "exact": int(cnt[2]), "near_ties": int(cnt[3]), "failures": int(cnt[4]),
              "min_top1_top2_margin": round(float(mm[0]), 6),
              "method": "teacher-forced oracle (BatchScorer) over prompt + all generated tokens; a pick passes "
                        "if it is the oracle argmax or within 1e-4 of the oracle maximum",
              "rank0_first_failures": par["first_failures"], "rank0_seconds": par["seconds"]}
    total_tokens = n_job * T * a.steps
    value = total_tokens / (ms / 1e3)
    e2e_value = total_tokens / (e2e_ms / 1e3)
    launches_per_gen = 1 + (P + T - 1) * (1 + 5 * model.args.n_layers + 2)
    # whole-generation HBM floor: K/V rows read by attention at lengths 1..P+T-1 plus the rows written
    kvb = 2 * model.n_kv_heads * model.head_dim * 4 * model.args.n_layers
    steps_gen = P + T - 1
    gen_bytes = n_job * kvb * (steps_gen * (steps_gen + 1) // 2 + steps_gen)
    peak_hbm, _ = measured_peaks()
    step_hbm = {"kv_bytes_per_generation": gen_bytes,
                "achieved_gbs": round(gen_bytes * a.steps / (ms / 1e3) / world / 1e9, 1),
                "frac": round(gen_bytes * a.steps / (ms / 1e3) / world / 1e9 / peak_hbm, 4),
                "note": "K/V cache bytes a generation must move (reads at every length + writes) over the "
                        "whole timed step, per GPU"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 3), "higher_is_better": True,
            "scaling": "strong" if a.split else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(a, world),
            "e2e": {"value": round(e2e_value, 1), "unit": "tok/s", "h2d_bytes_per_step": int(n * P * 4),
                    "d2h_bytes_per_step": int(n * T * 4)},
            "gpu_launches": launches_per_gen * a.steps,
            "roofline": roof, "step_hbm": step_hbm, "clocks": clocks, "all_sequences_full_length": ok_len,
            "parity": parity,
            "b1": b1, "gemv_scaled": gemv, "scaled_b1": sb1, "prefill": pf, "linear_sweep": sweep,
        }
        if not a.no_cpu_baseline and not a.only_main and world == 1:
            cores = cpu_cores()
            rows = host_prompts[: 4 * cores].tolist()
            v, toks, busy, wall = cpu_throughput(b, m, rows, T, cores, a.cpu_sample_requests)
            line["cpu_baseline"] = {"value": round(v, 2), "unit": "tok/s", "cores": cores, "kind": "port",
                                    "sample": f"{cores} single-thread processes x {a.cpu_sample_requests} requests "
                                              f"({P}+{T} tokens, B=1 cached-step loop of the oracle port); "
                                              f"{toks} tokens in {busy:.1f} s"}
            line["cpu_legs"] = cpu_legs(b, m, host_prompts[0].tolist(), T)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    tmp.cleanup()


def b1_latency(model, prompt, new_tokens, stream, reps=5):
    """B=1 greedy request of the tiny model (20-token prompt + 128 tokens), the
    reference's own headline request shape: device loop, CUDA events."""
    import torch

    dev = model.device
    pr = torch.tensor([prompt], dtype=torch.int32, device=dev)
    ln = torch.tensor([len(prompt)], dtype=torch.int32, device=dev)
    caches = model.new_batch_cache(1)
    for _ in range(3):
        model.generate_greedy_device(pr, ln, len(prompt), new_tokens, caches=caches)
    torch.cuda.synchronize()
    tot, dec = [], []
    for _ in range(reps):
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        e1.record(stream)
        model.generate_greedy_device(pr, ln, len(prompt), new_tokens, caches=caches, prefill_event=e1)
        e2.record(stream)
        torch.cuda.synchronize()
        tot.append(e0.elapsed_time(e2) / 1e3)
        dec.append(e1.elapsed_time(e2) / 1e3)
    t, d = statistics.median(tot), statistics.median(dec)
    steps = len(prompt) + new_tokens - 1
    # Roofline of a model step: the weights it uses (1,178,624 B: packed rows, scales, tied head, norms,
    # one embedding row) plus the K/V rows read (2560 B a position) and written, averaged over the
    # request's steps; against the measured L2 copy rate and the HBM copy peak.  The cluster kernel
    # keeps the weights in shared memory, so these fractions are small by design: the step is
    # latency-bound (about 30 dependent phases a step).
    kv_row = 2 * model.n_kv_heads * model.head_dim * 4 * model.args.n_layers
    step_bytes = 1_178_624 + kv_row * (sum(p + 1 for p in range(steps)) / steps + 1)
    ach = step_bytes / (t / steps) / 1e9
    l2 = l2_copy_gbs(dev, stream)
    hbm, kind = measured_peaks()
    return {"workload": f"B=1 greedy, {len(prompt)}-token prompt + {new_tokens} tokens, tiny model",
            "request_tok_s": round(new_tokens / t, 1), "decode_tok_s": round(new_tokens / d, 1),
            "us_per_model_step": round(t / steps * 1e6, 2), "prefill_ms": round((t - d) * 1e3, 3),
            "roofline": {"bound": "latency", "bytes_per_step": int(step_bytes), "achieved_gbs": round(ach, 1),
                         "l2_copy_gbs": l2, "frac_of_l2": round(ach / l2, 4), "hbm_gbs": hbm,
                         "frac_of_hbm": round(ach / hbm, 4), "peak_kind": f"{kind} hbm_gbs; L2 copy measured here"}}


def scaled_gemv(dev, stream, reps=10):
    """HBM-streaming Q6W GEMV at B=1 on the 1.1B-shape config's matrices
    (22 layers of wq/wk/wv/wo/w1/w2/w3 at dim 2048, hidden 5632, kv 256, plus
    the 32000x2048 vocab): one pass over 777 MB of packed weights per token,
    replayed from a CUDA graph.  Weights are random bytes (every byte pattern
    is a valid Q6W code stream); the cost does not depend on the values."""
    import torch

    from q6w_b200 import _lib

    lib = _lib.load()
    dim, hid, kv, vocab, layers = 2048, 5632, 256, 32000, 22
    shapes = [(dim, dim), (kv, dim), (kv, dim), (dim, dim), (hid, dim), (dim, hid), (hid, dim)] * layers
    shapes.append((vocab, dim))
    nbytes = sum(r * c * 3 // 4 + 4 * r for r, c in shapes)
    blob = torch.randint(0, 256, (nbytes + 256 * len(shapes),), dtype=torch.uint8, device=dev)
    mats, off = [], 0
    for r, c in shapes:
        pb = r * c * 3 // 4
        q = blob[off: off + pb]
        off = (off + pb + 255) // 256 * 256
        sc = blob[off: off + 4 * r].view(torch.float32)
        off = (off + 4 * r + 255) // 256 * 256
        mats.append((q, sc, r, c))
    for _, sc, r, _ in mats:  # finite, positive row scales
        sc.copy_(torch.rand(r, device=dev) * 0.05 + 0.001)
    x = torch.randn(max(dim, hid), device=dev)
    ys = [torch.empty(r, device=dev) for r, _ in shapes]
    def run(st):
        h = _lib.stream_handle(st)
        for (q, sc, r, c), y in zip(mats, ys):
            _lib.check(lib.q6w_linear(q.data_ptr(), sc.data_ptr(), x.data_ptr(), y.data_ptr(), r, c, 1, h))

    run(stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    with torch.cuda.graph(g, stream=side):
        run(side)
    for _ in range(3):
        g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    moved = nbytes + sum(4 * (r + c) for r, c in shapes)
    peak, kind = measured_peaks()
    del g
    # the largest matrix alone (vocab, 49 MB): four copies cycled, so each
    # launch reads its weights from HBM (4 x 49 MB > the 126 MB L2)
    vq, vs, vr, vc = mats[-1]
    copies = [vq] + [torch.randint(0, 256, vq.shape, dtype=torch.uint8, device=dev) for _ in range(3)]
    vy = torch.empty(vr, device=dev)
    gv = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gv, stream=side):
        h = _lib.stream_handle(side)
        for k in range(4 * reps):
            _lib.check(lib.q6w_linear(copies[k % 4].data_ptr(), vs.data_ptr(), x.data_ptr(), vy.data_ptr(), vr, vc, 1, h))
    gv.replay()
    torch.cuda.synchronize()
    e0.record(stream)
    gv.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    vsec = e0.elapsed_time(e1) / 1e3 / (4 * reps)
    vbytes = vr * vc * 3 // 4 + 4 * vr + 4 * (vr + vc)
    del gv, copies
    return {"workload": "B=1 Q6W GEMV pass over the 1.1B-shape matrices (155 launches, CUDA graph)",
            "bytes_per_token": moved, "us_per_token": round(sec * 1e6, 2),
            "achieved_gbs": round(moved / sec / 1e9, 1), "peak_gbs": peak,
            "frac": round(moved / sec / 1e9 / peak, 4), "peak_kind": f"{kind} hbm_gbs",
            "weights_tok_s_ceiling": round(1 / sec, 1),
            "vocab_32000x2048": {"us_per_launch": round(vsec * 1e6, 2), "bytes": vbytes,
                                 "achieved_gbs": round(vbytes / vsec / 1e9, 1),
                                 "frac": round(vbytes / vsec / 1e9 / peak, 4)}}


def l2_copy_gbs(dev, stream, mb=24, reps=50):
    """L2 bandwidth microbenchmark: a copy between two `mb` MB buffers (their
    sum well inside the 126 MB L2), repeated; (read + write bytes) / time."""
    import torch

    a = torch.randn(mb * 262144, device=dev)
    b = torch.empty_like(a)
    for _ in range(5):
        b.copy_(a)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        b.copy_(a)
    e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    del a, b
    return 2 * mb * 2 ** 20 / sec / 1e9


def _graph_time(call, reps, stream):
    """Device seconds per call of `call(stream)`: `reps` calls captured in one
    CUDA graph (no host launch cost between them), replayed after warm-up."""
    import torch

    side = torch.cuda.Stream()
    for _ in range(3):
        call(stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for _ in range(reps):
            call(side)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / 1e3 / reps


SWEEP_SHAPES = [(128, 128), (64, 128), (384, 128), (128, 384), (4096, 128)]
SWEEP_BATCHES = [1, 8, 64, 512, 4096]


def _cpu_linear_ms(w, x, threads, budget_s=0.3):
    """torch CPU FP32 x @ W.T (the reference's nn.Linear on dequantized
    weights) at `threads` threads: median ms of repeated calls."""
    import torch

    old = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        x @ w.T
        times = []
        t_end = time.perf_counter() + budget_s
        while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 50):
            t0 = time.perf_counter()
            x @ w.T
            times.append(time.perf_counter() - t0)
    finally:
        torch.set_num_threads(old)
    return statistics.median(times) * 1e3


def linear_sweep(dev, stream):
    """Isolated Q6W linear sweep on the tiny model's shapes: out x in of
    128x128, 64x128, 384x128, 128x384, 4096x128, activation batch N in
    {1, 8, 64, 512, 4096}; int6 codes U[-32, 31], row scales U(0.001, 0.05),
    x ~ N(0, 1).  Each point times the public linear op (FP32 kernels for
    N <= 8, tcgen05 tensor cores from N = 16) with CUDA events, repeated
    calls on the same (L2-resident) operands.

    Algorithmic work per call: bytes = rows*cols*3/4 + 4*rows + 4*N*cols +
    4*N*rows, flops = 2*N*rows*cols (FP32-equivalent; the tensor-core path
    issues 3x that in bf16 MMAs, one per part of x).  Roofline time =
    max(bytes / measured L2 copy bandwidth, tensor flops / measured bf16
    peak); `frac` = roofline time / measured time.  The CPU leg is torch
    FP32 x @ W.T on the dequantized weights at 1 thread and all cores."""
    import numpy as np
    import torch

    from q6w_b200 import _lib, ops

    lib = _lib.load()
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    l2 = l2_copy_gbs(dev, stream)
    cores = cpu_cores()
    rng = np.random.default_rng(2)
    points = []
    for rows, cols in SWEEP_SHAPES:
        q = rng.integers(-32, 32, size=(rows, cols))
        sc = rng.uniform(0.001, 0.05, size=rows).astype(np.float32)
        u = (q.astype(np.int32) & 0x3F).reshape(rows, -1, 4)
        word = u[..., 0] | (u[..., 1] << 6) | (u[..., 2] << 12) | (u[..., 3] << 18)
        packed = torch.from_numpy(word.astype("<u4").view(np.uint8).reshape(word.shape + (4,))[..., :3].copy()
                                  .reshape(-1)).to(dev)
        scales = torch.from_numpy(sc).to(dev)
        w_cpu = torch.from_numpy(q.astype(np.float32) * sc[:, None])
        for n in SWEEP_BATCHES:
            x_cpu = torch.from_numpy(rng.standard_normal((n, cols)).astype(np.float32))
            x = x_cpu.to(dev)
            y = torch.empty((n, rows), device=dev)
            need = ops.linear_workspace_bytes(rows, cols, n)
            tc = need > 0
            ws = ops._linear_workspace(dev, need) if tc else None
            reps = 200 if n <= 512 else 50

            def call(st, tensor_cores=True):
                h = _lib.stream_handle(st)
                if tensor_cores and tc:
                    _lib.check(lib.q6w_linear_ex(packed.data_ptr(), scales.data_ptr(), x.data_ptr(), y.data_ptr(),
                                                 rows, cols, n, ws.data_ptr(), ws.numel(), h))
                else:
                    _lib.check(lib.q6w_linear(packed.data_ptr(), scales.data_ptr(), x.data_ptr(), y.data_ptr(),
                                              rows, cols, n, h))

            sec = _graph_time(call, reps, stream)
            nbytes = rows * cols * 3 // 4 + 4 * rows + 4 * n * cols + 4 * n * rows
            flops = 2 * n * rows * cols
            tflops_issued = (3 if tc else 1) * flops
            t_roof = max(nbytes / (l2 * 1e9), (tflops_issued / (bf16 * 1e12)) if tc else 0.0)
            pt = {"rows": rows, "cols": cols, "n": n, "kernel": "tcgen05" if tc else "fp32",
                  "us": round(sec * 1e6, 3), "gbs": round(nbytes / sec / 1e9, 1),
                  "tflops_fp32_equiv": round(flops / sec / 1e12, 3),
                  "bound": "tensor" if tc and tflops_issued / (bf16 * 1e12) > nbytes / (l2 * 1e9) else "l2",
                  "frac": round(t_roof / sec, 4)}
            if tc:
                pt["fp32_kernel_us"] = round(_graph_time(lambda st: call(st, False), reps, stream) * 1e6, 3)
            pt["cpu_1t_ms"] = round(_cpu_linear_ms(w_cpu, x_cpu, 1), 4)
            pt["cpu_all_ms"] = round(_cpu_linear_ms(w_cpu, x_cpu, cores), 4)
            points.append(pt)
    return {"workload": "isolated Q6W linear sweep (tiny-model shapes x N in {1, 8, 64, 512, 4096}), "
                        "operands L2-resident across repeated calls",
            "l2_copy_gbs": round(l2, 1), "bf16_peak_tflops": bf16, "cpu_cores": cores, "points": points}


def prefill_c3(model, rank, world, stream, reps=3):
    """Batched ragged prefill of the tiny model: 2048 prompts, lengths
    U[8, 256], ids U[3, 4095] (one seed for all ranks), this rank's share
    balanced by prompt tokens; last-position logits + filled KV caches in
    one q6w_prefill call."""
    import numpy as np
    import torch

    from q6w_b200 import dp

    rng = np.random.default_rng(2048)
    lens_all = rng.integers(8, 257, 2048)
    ids_all = rng.integers(3, 4096, (2048, 256)).astype(np.int32)
    mine = dp.balance_by_tokens(lens_all.tolist(), world)[rank]
    lens = lens_all[mine].astype(np.int32)
    L = int(lens.max())
    pr = torch.from_numpy(np.ascontiguousarray(ids_all[mine, :L])).to(model.device)
    ln = torch.from_numpy(lens).to(model.device)
    total = int(lens.sum())
    caches = model.new_batch_cache(len(mine))
    for _ in range(2):
        _, _, _, ws = model.prefill_batch_device(pr, ln, L, total, caches=caches)
    model.check_device_status(ws)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        model.prefill_batch_device(pr, ln, L, total, caches=caches)
    e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    job_tokens = int(lens_all.sum())
    if world > 1:
        t = torch.tensor([sec], dtype=torch.float64, device=model.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sec = float(t[0])
    del caches
    torch.cuda.empty_cache()
    # roofline: the linears of every prompt token (dim 128 model: 2 x 983,040 flop a token, issued three
    # times as bf16 MMAs on the tensor cores), against the measured sustained bf16 peak
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
    issued = 3 * 2 * 983_040 * job_tokens
    return {"workload": f"batched ragged prefill, tiny model: 2048 prompts, lengths U[8,256], over {world} GPU(s) "
                        f"balanced by tokens (this rank: {len(mine)} prompts, {total} tokens)",
            "prompts": 2048, "tokens": job_tokens, "ms": round(sec * 1e3, 3),
            "prefill_tok_s": round(job_tokens / sec, 1), "prompts_s": round(2048 / sec, 1),
            "roofline": {"bound": "tensor", "achieved": round(issued / sec / 1e12, 2), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(issued / sec / 1e12 / peak / world, 4),
                         "work": "3 x 2 x 983,040 bf16 flop per prompt token (linears; attention and vocab excluded)",
                         "peak_kind": "measured bf16_tflops_sustained per GPU"}}


def scaled_b1(dev, stream, reps=3):
    """B=1 greedy decode of the 1.1B-shape config (dim 2048, 22 layers, 32
    heads / 4 kv heads, hidden 5632, vocab 32000): 128-token prompt + 128
    tokens through the device loop (streaming GEMVs chained by programmatic
    dependent launch inside the step graph).  Random 6-bit codes stand in
    for trained weights (same bytes and shapes, so the same cost)."""
    import torch

    from q6w_b200 import format as fmt
    from q6w_b200.model import Q6WCudaTransformer

    args = dict(fmt.SCALED_ARGS)
    model = Q6WCudaTransformer(fmt.RandomImage(args, seed=7), device=dev)
    P, T = 128, 128
    g = torch.Generator().manual_seed(11)
    pr = torch.randint(3, args["vocab_size"], (1, P), generator=g, dtype=torch.int32).to(dev)
    ln = torch.tensor([P], dtype=torch.int32, device=dev)
    caches = model.new_batch_cache(1)
    for _ in range(2):
        model.generate_greedy_device(pr, ln, P, T, caches=caches)
    torch.cuda.synchronize()
    dec, tot = [], []
    for _ in range(reps):
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        model.generate_greedy_device(pr, ln, P, T, caches=caches, prefill_event=e1)
        e2.record(stream)
        torch.cuda.synchronize()
        tot.append(e0.elapsed_time(e2) / 1e3)
        dec.append(e1.elapsed_time(e2) / 1e3)
    d, t = statistics.median(dec), statistics.median(tot)
    # decode steps: T - 1 model steps after the prefill part (P steps)
    step_s = d / (T - 1)
    # B=64: 64 independent requests of the same shape in one batched loop
    n64 = 64
    pr64 = torch.randint(3, args["vocab_size"], (n64, P), generator=g, dtype=torch.int32).to(dev)
    ln64 = torch.full((n64,), P, dtype=torch.int32, device=dev)
    caches64 = model.new_batch_cache(n64)
    model.generate_greedy_device(pr64, ln64, P, T, caches=caches64)
    torch.cuda.synchronize()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record(stream)
    model.generate_greedy_device(pr64, ln64, P, T, caches=caches64, prefill_event=e1)
    e2.record(stream)
    torch.cuda.synchronize()
    d64, t64 = e1.elapsed_time(e2) / 1e3, e0.elapsed_time(e2) / 1e3
    del caches64
    wbytes = sum(e["data_bytes"] + e.get("scale_bytes", 0) for e in model.image.tensors.values())
    peak, kind = measured_peaks()
    del model, caches
    torch.cuda.empty_cache()
    return {"workload": "B=1 greedy, 1.1B-shape config, 128-token prompt + 128 tokens (random 6-bit codes)",
            "decode_tok_s": round((T - 1) / d, 1), "request_tok_s": round(T / t, 1),
            "us_per_model_step": round(step_s * 1e6, 2), "weight_bytes_per_step": wbytes,
            "weights_gbs": round(wbytes / step_s / 1e9, 1), "frac_of_hbm": round(wbytes / step_s / 1e9 / peak, 4),
            "peak_kind": f"{kind} hbm_gbs",
            "b64": {"decode_tok_s": round(n64 * (T - 1) / d64, 1), "request_tok_s": round(n64 * T / t64, 1),
                    "us_per_model_step": round(d64 / (T - 1) * 1e6, 2)}}


def profile_scaled_step(n=1):
    """n short requests of the 1.1B-shape config (2-token prompts, 3 tokens):
    the launch list of its model steps is the profile of a scaled decode step."""
    import torch

    from q6w_b200 import format as fmt
    from q6w_b200.model import Q6WCudaTransformer

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    model = Q6WCudaTransformer(fmt.RandomImage(dict(fmt.SCALED_ARGS), seed=7), device=dev)
    pr = torch.tensor([[17, 2500]] * n, dtype=torch.int32, device=dev)
    ln = torch.full((n,), 2, dtype=torch.int32, device=dev)
    sampled, n_sampled, *_ = model.generate_greedy_device(pr, ln, 2, 3)
    torch.cuda.synchronize()
    print(json.dumps({"profile_scaled_step": True, "sampled": sampled[0, : int(n_sampled[0])].tolist()}), flush=True)


def profile_gemv(shape):
    """One B=1 GEMV shape, 4 launches on random data: a small case for an
    ncu capture of the streaming GEMV."""
    import torch

    from q6w_b200 import _lib

    rows, cols = (int(v) for v in shape.lower().split("x"))
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    lib = _lib.load()
    q = torch.randint(0, 256, (rows * cols * 3 // 4,), dtype=torch.uint8, device=dev)
    sc = torch.rand(rows, device=dev) * 0.05 + 0.001
    x = torch.randn(cols, device=dev)
    y = torch.empty(rows, device=dev)
    h = _lib.stream_handle()
    for _ in range(4):
        _lib.check(lib.q6w_linear(q.data_ptr(), sc.data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, 1, h))
    torch.cuda.synchronize()
    print(json.dumps({"profile_gemv": shape, "launches": 4, "y_abs_sum": float(y.abs().sum())}), flush=True)


def profile_case(name):
    """Small cases for ncu captures, each run 3 times after one warm-up:
    b1 -- a B=1 request of the tiny model (20 + 128 tokens, the cluster kernel);
    prefill -- 256 of the 2048 ragged prompts in one q6w_prefill;
    prefill_full -- all 2048 ragged prompts (lengths U[8, 256]) in one q6w_prefill;
    attn -- decode attention alone, 8192 sequences (tiny heads) at lengths 20 and 147;
    sampler -- the sampler op on 8192 rows of 4096 logits (top-p 0.9, T 0.8);
    linear -- the 4096 x 128 linear at N = 4096 on the tensor cores;
    quantize -- the device writer on a 5632 x 2048 matrix."""
    import numpy as np
    import torch

    from q6w_b200 import ops
    from q6w_b200.model import Q6WCudaTransformer

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    tmp = tempfile.TemporaryDirectory()
    if name in ("b1", "prefill", "prefill_full"):
        b, m = make_model_files(tmp.name)
        model = Q6WCudaTransformer.from_q6w(b, m, device=dev)
    if name == "b1":
        pr = prompts_for(0, 1, 20).to(dev)
        ln = torch.full((1,), 20, dtype=torch.int32, device=dev)
        run = lambda: model.generate_greedy_device(pr, ln, 20, 128)
    elif name == "prefill":
        rng = np.random.default_rng(2048)
        lens = rng.integers(8, 257, 2048)[:256].astype(np.int32)
        ids = rng.integers(3, 4096, (2048, 256)).astype(np.int32)[:256]
        pr, ln = torch.from_numpy(ids).to(dev), torch.from_numpy(lens).to(dev)
        caches = model.new_batch_cache(256)
        run = lambda: model.prefill_batch_device(pr, ln, 256, int(lens.sum()), caches=caches)
    elif name == "prefill_full":
        rng = np.random.default_rng(2048)
        lens = rng.integers(8, 257, 2048).astype(np.int32)
        ids = rng.integers(3, 4096, (2048, 256)).astype(np.int32)
        pr, ln = torch.from_numpy(ids).to(dev), torch.from_numpy(lens).to(dev)
        caches = model.new_batch_cache(2048)
        run = lambda: model.prefill_batch_device(pr, ln, 256, int(lens.sum()), caches=caches)
    elif name == "attn":
        # decode attention alone (the public op, non-split output), 8192 sequences at lengths 20 and 147
        k = torch.randn(8192, 160, 4, 16, device=dev)
        v = torch.randn(8192, 160, 4, 16, device=dev)
        q = torch.randn(8192, 8, 16, device=dev)
        l20 = torch.full((8192,), 20, dtype=torch.int32, device=dev)
        l147 = torch.full((8192,), 147, dtype=torch.int32, device=dev)

        def run():
            ops.gqa_attention(q, k, v, l20, 2)
            ops.gqa_attention(q, k, v, l147, 2)
    elif name == "sampler":
        g = torch.Generator().manual_seed(1)
        logits = (torch.randn(8192, 4096, generator=g) * 2).to(dev)
        hist = torch.randint(0, 4096, (8192, 32), generator=g, dtype=torch.int32).to(dev)
        hl = torch.full((8192,), 32, dtype=torch.int32, device=dev)
        rng_state = torch.arange(1, 8193, dtype=torch.int64, device=dev)
        run = lambda: ops.sample(logits, hist, hl, rng_state, 0.8, 0.9, repetition_penalty=1.1)
    elif name == "linear":
        rng = np.random.default_rng(4)
        packed = torch.from_numpy(rng.integers(0, 256, 4096 * 96, dtype=np.uint8)).to(dev)
        scales = torch.from_numpy(rng.uniform(0.001, 0.05, 4096).astype(np.float32)).to(dev)
        x = torch.randn(4096, 128, device=dev)
        run = lambda: ops.q6w_linear(x, packed, scales, 4096, 128)
    else:
        w = torch.randn(5632, 2048, device=dev) * 0.02
        run = lambda: ops.quantize_rows(w)
    for _ in range(4):
        run()
    torch.cuda.synchronize()
    tmp.cleanup()
    print(json.dumps({"profile": name, "launches_of_case": 4}), flush=True)


def attention_roofline(model, caches, n, length, stream):
    """Time the decode-attention kernel alone (public op, one layer of this
    run's caches at the final length) and report its HBM roofline.

    Algorithmic bytes per launch = K and V rows read (n * length * kv_heads *
    head_dim * 4 bytes each) + queries in + outputs out.
    """
    import torch

    from q6w_b200 import ops

    k, v = caches
    a = model.args
    H, KV, hd = a.n_heads, model.n_kv_heads, model.head_dim
    kl = k[:, 0]  # layer 0 view: [n, max_seq, KV, hd], sequence stride = whole cache
    vl = v[:, 0]
    q = torch.randn(n, H, hd, device=k.device)
    lens = torch.full((n,), length, dtype=torch.int32, device=k.device)
    for _ in range(3):
        ops.gqa_attention(q, kl, vl, lens, H // KV)
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        ops.gqa_attention(q, kl, vl, lens, H // KV)
    e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    nbytes = 2 * n * length * KV * hd * 4 + 2 * n * H * hd * 4
    peak, kind = measured_peaks()
    ach = nbytes / sec / 1e9
    # over the generation: every 8th attention length 1..length, each weighted as one step (bytes and
    # times summed, so the fraction is the one the whole generation's attention launches reach)
    tb = tt = 0.0
    for ln in sorted(set(list(range(1, length + 1, 8)) + [length])):
        lens.fill_(ln)
        ops.gqa_attention(q, kl, vl, lens, H // KV)
        e0.record(stream)
        for _ in range(5):
            ops.gqa_attention(q, kl, vl, lens, H // KV)
        e1.record(stream)
        torch.cuda.synchronize()
        tt += e0.elapsed_time(e1) / 1e3 / 5
        tb += 2 * n * ln * KV * hd * 4 + 2 * n * H * hd * 4
    over = {"lengths": f"1..{length} every 8th (and {length})", "achieved": round(tb / tt / 1e9, 1),
            "frac": round(tb / tt / 1e9 / peak, 4)}
    # DRAM bytes (read + written) of one launch as ncu measured them on a smaller capture of the same
    # kernel: 2048 sequences at length 147 moved 159.89 MB; traffic grows with the sequence count
    ncu_bytes, ncu_seqs, ncu_len = 159.89e6, 2048, 147
    traffic = int(ncu_bytes * n / ncu_seqs) if length == ncu_len else None
    return {"kernel": "attn_warp_kernel (decode GQA attention, timed alone)", "bound": "hbm",
            "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
            "peak_kind": f"{kind} hbm_gbs (copy, burst)", "traffic": traffic,
            "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at {ncu_seqs} "
                               f"sequences, length {ncu_len}, scaled by sequences ({n})") if traffic else None,
            "bytes_per_launch": nbytes, "us_per_launch": round(sec * 1e6, 2), "over_generation": over}


def main():
    a = parse()
    if a.profile_gemv:
        profile_gemv(a.profile_gemv)
    elif a.profile:
        profile_case(a.profile)
    elif a.sweep_only:
        import torch

        torch.cuda.set_device(0)
        print(json.dumps({"linear_sweep": linear_sweep(torch.device("cuda", 0), torch.cuda.current_stream())}),
              flush=True)
    elif a.profile_scaled_step:
        profile_scaled_step(a.profile_scaled_step)
    elif a.impl == "reference":
        run_reference(a)
    else:
        run_b200(a)


if __name__ == "__main__":
    main()
