"""Benchmark of the paged decode attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Default workload: Llama-3-8B-shape fp16 paged decode (H32/Hkv8/D128, batch
64, context 2048, block size 16, shuffled 8192-block pool).  A step is one
cottus_paged_decode call over the batch with every input already in HBM.
Multi-GPU (torchrun, one process per GPU): each rank decodes its own batch
of sequences (weak scaling, no collective); the long-context config instead
splits every sequence's pages across the ranks and merges LSE partials over
NCCL (strong scaling).  `--impl reference` times the reference's own CPU
pagedAttentionCPU (compiled from its sources into oracle/_ref) on the host
cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "cottus-runtime_b200"))

METRIC = "paged-attn decode KV-read GB/s"
L2_BYTES = 126 * 1024 * 1024


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def describe(w):
    return (f"{w.name}: H{w.H}/Hkv{w.Hkv}/D{w.D}, batch {w.B}, context "
            f"{int(w.ctx.min())}-{int(w.ctx.max())} (sum {int(w.ctx.sum())}), block 16, {w.num_blocks}-block pool")


# -- clocks sampled during the timed region ---------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu, self.rows, self.proc = gpu_index, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "samples": len(rows), "reasons": sorted(reasons)}


# -- CPU baseline (reference pagedAttentionCPU compiled from its sources) --------------------

class ReferenceBatch:
    """The reference's CPU path (oracle/_ref, pagedAttentionCPU) over sequences
    of a workload, one call per sequence, spread over the host threads by the
    library.  Host copies of the pages are made once, outside any timing."""

    def __init__(self, w, t, max_seqs=None):
        from oracle.oracle import Reference
        from cottus_b200.workloads import host_subpool

        self.ref, self.w = Reference(), w
        self.threads = os.cpu_count() or 1
        seqs = list(range(w.B if max_seqs is None else min(w.B, max_seqs)))
        sub, bt, ctx = host_subpool(w, t["kv_pool"], seqs)
        self.q = t["query"][seqs].float().cpu().numpy()
        per = w.block_elems()
        # the reference computes element offsets in int32 (paged_attention_cpu.cpp:63): rebase every
        # sequence onto its own lowest block, or, where its blocks span too far for that, copy its
        # pages into a buffer of their own in table order (identity table)
        self.bases, self.bt, self.keep = [], bt.copy(), [sub]
        for i in range(len(seqs)):
            n = (int(ctx[i]) + w.bs - 1) // w.bs
            lo = int(bt[i, :n].min()) if n else 0
            hi = int(bt[i, :n].max()) if n else 0
            if (hi - lo + 1) * per < 2 ** 31:
                self.bases.append(sub.ctypes.data + 2 * lo * per)
                self.bt[i, :n] -= lo
            else:
                own = np.ascontiguousarray(sub.reshape(-1, per)[bt[i, :n]])
                self.keep.append(own)
                self.bases.append(own.ctypes.data)
                self.bt[i, :n] = np.arange(n, dtype=np.int32)
        self.ctx = ctx
        self.out = np.zeros((len(seqs), w.H * w.D), np.float32)

    def lens(self, n, cap=None):
        c = self.ctx[:n]
        return c if cap is None else np.minimum(c, cap).astype(np.int32)

    def kv_bytes(self, n, cap=None):
        return int(np.sum(self.lens(n, cap).astype(np.int64))) * 2 * self.w.Hkv * self.w.D * 2

    def run(self, n, cap=None):
        """First n sequences; with `cap`, each over its first `cap` tokens only."""
        w = self.w
        self.ref.paged_attention_batch_rebased(self.out[:n], self.q[:n], self.bases[:n], self.bt[:n],
                                               self.lens(n, cap), w.layer, w.H, w.Hkv, w.D, w.bs, w.L, self.threads)


def cpu_reference_rate(w, t, target_s=8.0, max_seqs=None):
    """Times the reference's CPU path on the host cores over a sample of the
    workload's sequences; returns (GB/s, threads, sample description)."""
    rb = ReferenceBatch(w, t, max_seqs)
    n = len(rb.ctx)
    reps, t0 = 0, time.perf_counter()
    while True:
        rb.run(n)
        reps += 1
        el = time.perf_counter() - t0
        if el >= target_s or reps >= 1000:
            break
    return rb.kv_bytes(n) * reps / el / 1e9, rb.threads, f"{n} of {w.B} sequences x {reps} passes ({el:.1f} s wall)"


# -- main --------------------------------------------------------------------------------------

def build_workload(name, rank, batch=None):
    from cottus_b200 import workloads as W

    seed = 1000 + rank
    kw = {"B": batch} if batch else {}
    return W.BUILDERS[name](seed=seed, **kw)


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path, rank 0 only."""
    import torch
    if world > 1 and rank != 0:
        return
    if args.config in ("qkv_llama3_8b", "oproj_llama3_8b", "attn_block_llama3_8b"):
        fn, metric = {"qkv_llama3_8b": (qkv_reference_rate, "fused QKV+RoPE+append tokens/s"),
                      "oproj_llama3_8b": (oproj_reference_rate, "O-projection+residual tokens/s"),
                      "attn_block_llama3_8b": (attn_reference_rate, "attention block tokens/s")}[args.config]
        budget = min(3.0 if fn is attn_reference_rate else 2.0, 60.0 / max(args.steps + args.warmup, 1))
        rates, sample, threads = [], "", 1
        t0 = time.perf_counter()
        for i in range(args.warmup + args.steps):
            r, threads, sample = fn(target_s=budget)
            if i >= args.warmup:
                rates.append(r)
        v = float(np.mean(rates))
        print(json.dumps({"metric": metric, "value": v, "unit": "tokens/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": (time.perf_counter() - t0) / max(args.steps + args.warmup, 1) * 1e3,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                          "data": "synthetic", "config": {"workload": args.config}, "impl": "reference",
                          "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "reference",
                                           "sample": sample},
                          "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return
    from cottus_b200 import workloads as W
    w, config = decode_config(args, world)
    t = W.device_tensors(w, "cpu" if not torch.cuda.is_available() else "cuda")
    # each step is a bounded sample of the workload, sized from one timed sequence so that warm-up and
    # timed steps together take about a minute (a few at most): the first n whole sequences, or, where one
    # sequence alone takes longer than a step may, the first `cap` tokens of one sequence per thread
    rb = ReferenceBatch(w, t, max_seqs=64)
    c0 = int(min(int(rb.ctx[0]), 2048))
    t1 = time.perf_counter()
    rb.run(1, c0)
    per_token = max(time.perf_counter() - t1, 1e-6) / c0
    budget = min(2.0, 60.0 / max(args.steps + args.warmup, 1))  # per step; threads contend, so aim low
    one = per_token * int(rb.ctx[0])
    threads = rb.threads
    if one <= budget:
        n, cap = int(min(len(rb.ctx), (budget // one) * threads)), None
        sample = f"first {n} of {w.B} sequences per step"
    else:
        n, cap = int(min(len(rb.ctx), threads)), int(max(w.bs, budget // per_token))
        sample = f"first {cap} tokens of each of the first {n} of {w.B} sequences per step"
    rates = []
    for _ in range(args.warmup):
        rb.run(n, cap)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ts = time.perf_counter()
        rb.run(n, cap)
        rates.append(rb.kv_bytes(n, cap) / (time.perf_counter() - ts) / 1e9)
    el = time.perf_counter() - t0
    v = float(np.mean(rates))
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": el / max(args.steps, 1) * 1e3, "higher_is_better": True,
            "scaling": "strong" if args.config == "long_ctx_70b" and world > 1 else "weak", "vs_baseline": None,
            "dtype": "f32 (fp16 KV decoded to fp32; the reference's CPU arithmetic)", "data": "synthetic",
            "config": config, "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def start_clocks(local):
    """Starts the SM-clock sampler and lets it come up.  Called before the
    warm-up steps, never between them and the timed region: a GPU left idle
    for a fraction of a second runs its next steps slowly (measured: the
    first step after a 0.3 s pause takes 130-210 us instead of 90 us)."""
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    return sampler


def hold_gpu():
    """Queues a ~1 ms spin on the GPU (torch's bounded sleep kernel) just
    before a timed region, so that the host enqueues the timed steps while
    the GPU is busy: a host stall (other processes, Python) then cannot leave
    the GPU idle inside the region.  The region's first event is recorded
    after the spin, so the spin is not timed."""
    import torch
    torch.cuda._sleep(2_000_000)


def timed_steps(step, args, dev, world, local):
    """W untimed steps, then K steps between CUDA events on the current
    stream with the SM clocks sampled; a synchronize and a barrier (no idle
    pause) between the two; max over ranks.  Returns (ms per step, clocks)."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream(dev)
    sampler = start_clocks(local)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    hold_gpu()
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    return max_over_ranks(e0.elapsed_time(e1) / args.steps, dev, world), clocks


def graph_of_steps(step, n, dev, prerun=True):
    """A CUDA graph of steps 0..n-1 (one per layer's weights): the projection
    kernels take a few microseconds, less than a host-side call through the
    ctypes layer, so the device-timed loop replays the launches as a graph,
    as a decode engine does.  With prerun the steps run once outside the
    capture first (the cached workspace and the kernel attributes are set up
    there); without, the caller has run steps of the same shape already."""
    import torch
    if prerun:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for i in range(n):
                step(i)
        torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n):
            step(i)
    torch.cuda.synchronize(dev)
    return g


def pipelined_e2e(call, host_in, out, args, dev, world):
    """End to end through the public API: every step uploads its inputs from
    pinned host memory (host_in), runs call(i, device_inputs, device_out) and
    reads device_out back into pinned host memory.  Two buffer sets and two
    copy streams pipeline the steps, as a serving loop would: the uploads of
    step i+1 and the read-back of step i-1 run on the copy engines while the
    kernels of step i run.  Returns ms per step between CUDA events on the
    compute stream (max over ranks)."""
    import torch
    stream = torch.cuda.current_stream(dev)
    slots = [dict(ins=[torch.empty(h.shape, dtype=h.dtype, device=dev) for h in host_in], out=out.clone(),
                  hout=torch.empty(out.shape, dtype=out.dtype).pin_memory(),
                  up=torch.cuda.Event(), ran=torch.cuda.Event(), down=torch.cuda.Event())
             for _ in range(2)]
    up_s, down_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def upload(i):
        sl = slots[i % 2]
        with torch.cuda.stream(up_s):
            if i >= 2:
                up_s.wait_event(sl["ran"])  # step i-2 has read this slot's inputs
            for d, h in zip(sl["ins"], host_in):
                d.copy_(h, non_blocking=True)
            sl["up"].record(up_s)

    def run(i):
        sl = slots[i % 2]
        stream.wait_event(sl["up"])
        if i >= 2:
            stream.wait_event(sl["down"])  # step i-2's output has been read back
        call(i, sl["ins"], sl["out"])
        sl["ran"].record(stream)
        with torch.cuda.stream(down_s):
            down_s.wait_event(sl["ran"])
            sl["hout"].copy_(sl["out"], non_blocking=True)
            sl["down"].record(down_s)

    def steps(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            run(i)
        stream.wait_event(slots[(n - 1) % 2]["down"])

    n_e2e = min(max(args.steps, 20), 2000)
    steps(5)
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    up_s.wait_event(a)
    steps(n_e2e)
    b.record(stream)
    torch.cuda.synchronize(dev)
    return max_over_ranks(a.elapsed_time(b) / n_e2e, dev, world)


def max_over_ranks(v, dev, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


QKV = dict(hidden=4096, H=32, Hkv=8, D=128, B=64, layers=4, bs=16, maxb=128)  # Llama-3-8B projection, batch 64


def qkv_inputs(dev, seed=7):
    import torch
    q = QKV
    N = (q["H"] + 2 * q["Hkv"]) * q["D"]
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn((q["B"], q["hidden"]), generator=g)).half()
    ws = [(torch.randn((N, q["hidden"]), generator=g) / q["hidden"] ** 0.5).half() for _ in range(q["layers"])]
    nb = q["B"] * q["maxb"]
    table = torch.randperm(nb, generator=g).int().view(q["B"], q["maxb"])
    pos = torch.randint(0, q["maxb"] * q["bs"], (q["B"],), generator=g).int()
    return N, x, ws, table, pos, nb


def run_qkv(args, rank, world, local):
    """The fused QKV projection + RoPE + KV append (cottus_qkv_rope_append) on
    the Llama-3-8B projection (hidden 4096 -> 6144 rows), batch 64; each step
    one layer, cycling over 4 layers' weights (201 MB > L2) as a decode step
    does.  Replicas per GPU (weak scaling, no collective)."""
    import torch
    import torch.distributed as dist
    import cottus_b200 as cb

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    q = QKV
    N, x, ws, table, pos, nb = qkv_inputs(dev)
    x, table, pos = x.to(dev), table.to(dev), pos.to(dev)
    ws = [w.to(dev) for w in ws]
    tab = cb.rope_cos_sin_table(q["maxb"] * q["bs"], q["D"]).to(dev)
    pool = torch.zeros(nb * 2 * q["layers"] * q["bs"] * q["Hkv"] * q["D"], dtype=torch.int16, device=dev)
    qout = torch.empty((q["B"], q["H"], q["D"]), dtype=torch.float16, device=dev)
    kw = dict(num_heads=q["H"], num_kv_heads=q["Hkv"], head_dim=q["D"], block_size=q["bs"], num_layers=q["layers"],
              num_physical_blocks=nb, query_out=qout)

    def step(i, xx=x):
        cb.qkv_rope_append(xx, ws[i % q["layers"]], pos, tab, pool, table, layer=i % q["layers"], **kw)

    g = graph_of_steps(step, q["layers"], dev)
    reps = max(args.steps // q["layers"], 1)
    args_g = argparse.Namespace(**{**vars(args), "steps": reps, "warmup": max(args.warmup // q["layers"], 3)})
    ms, clocks = timed_steps(lambda i: g.replay(), args_g, dev, world, local)
    ms /= q["layers"]
    steps_timed = reps * q["layers"]
    # end to end: the step's activations from pinned host memory, the rotated query back
    e_ms = pipelined_e2e(lambda i, ins, o: cb.qkv_rope_append(ins[0], ws[i % q["layers"]], pos, tab, pool, table,
                                                              layer=i % q["layers"], **dict(kw, query_out=o)),
                         [x.cpu().pin_memory()], qout, args, dev, world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r, cores, sample = qkv_reference_rate(target_s=6.0)
        cpu = {"value": r, "unit": "tokens/s", "cores": cores, "kind": "reference", "sample": sample}
    if world > 1:
        dist.barrier()
        if rank != 0:
            dist.destroy_process_group()
            return
    peak, peak_kind = peaks()
    wbytes = N * q["hidden"] * 2
    alg = wbytes + x.numel() * 2 + qout.numel() * 2 + q["B"] * 2 * q["Hkv"] * q["D"] * 2 + q["B"] * 8
    line = {
        "metric": "fused QKV+RoPE+append tokens/s", "value": world * q["B"] / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": world, "steps": steps_timed, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 x f16 -> f32",
        "data": "synthetic: seeded N(0,1) activations, N(0, 1/hidden) fp16 weights",
        "config": {"workload": f"qkv_llama3_8b: hidden {q['hidden']} -> {N} rows (H{q['H']}/Hkv{q['Hkv']}/D{q['D']}), "
                               f"batch {q['B']}, one of {q['layers']} layers per step",
                   "l2": f"{q['layers']} layers' weights ({q['layers'] * wbytes / 1e6:.0f} MB) cycled, > 126 MB L2",
                   "parallelism": f"replicas on {world} GPU(s), no collective"},
        "roofline": {"bound": "hbm", "achieved": alg / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": alg / (ms * 1e-3) / 1e9 / peak, "traffic": None, "peak_kind": peak_kind,
                     "kernel": "qkv_proj_kernel + qkv_finish_kernel per step (CUDA graph of 4 layers' steps)",
                     "kernel_ms": ms, "algorithmic_bytes": alg},
        "cpu_baseline": cpu,
        "e2e": {"value": world * q["B"] / (e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": x.numel() * 2,
                "d2h_bytes_per_step": qout.numel() * 2, "ms_per_step": e_ms,
                "api": "cottus_qkv_rope_append (C ABI via ctypes)", "pipelining": "two buffer sets, two copy streams"},
        "gpu_launches": 2 * steps_timed, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    del g
    if world > 1:
        dist.destroy_process_group()


def qkv_reference_rate(target_s=6.0, tokens=None):
    """The reference's CPU step for one token and one layer (gemmCPU x3 as one
    stacked product, ropeCPU on q and k; fp32 weights as the reference keeps
    them), tokens spread over the host threads; returns (tokens/s, threads, sample)."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle.oracle import Reference

    q = QKV
    ref = Reference()
    N = (q["H"] + 2 * q["Hkv"]) * q["D"]
    rng = np.random.default_rng(3)
    wt = (rng.standard_normal((q["hidden"], N), dtype=np.float32) / np.float32(q["hidden"] ** 0.5))
    threads = os.cpu_count() or 1
    n_tok = tokens or threads
    xs = rng.standard_normal((n_tok, q["hidden"]), dtype=np.float32)

    def one(i):
        out = ref.gemm(xs[i:i + 1], wt)
        ref.rope(out[0, :q["H"] * q["D"]], 5, q["H"], q["D"])
        ref.rope(out[0, q["H"] * q["D"]:(q["H"] + q["Hkv"]) * q["D"]], 5, q["Hkv"], q["D"])

    done, t0 = 0, time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        while True:
            list(ex.map(one, range(n_tok)))
            done += n_tok
            el = time.perf_counter() - t0
            if el >= target_s:
                break
    return done / el, threads, f"{done} tokens x 1 layer ({el:.1f} s wall, {threads} threads)"


OPROJ = dict(fin=4096, fout=4096, B=64, layers=8)  # Llama-3-8B output projection, batch 64


def run_oproj(args, rank, world, local):
    """Output projection + residual add (cottus_o_proj_residual) on the
    Llama-3-8B shape (4096 -> 4096), batch 64, in place on the fp32 residual
    stream; each step one layer, cycling over 8 layers' weights (268 MB > L2).
    Replicas per GPU (weak scaling, no collective)."""
    import torch
    import torch.distributed as dist
    import cottus_b200 as cb

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    o = OPROJ
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn((o["B"], o["fin"]), generator=g).half().to(dev)
    ws = [(torch.randn((o["fout"], o["fin"]), generator=g) / o["fin"] ** 0.5).half().to(dev)
          for _ in range(o["layers"])]
    resid = torch.randn((o["B"], o["fout"]), generator=g).to(dev)

    def step(i, xx=x):
        cb.o_proj_residual(xx, ws[i % o["layers"]], resid, out=resid)

    g = graph_of_steps(step, o["layers"], dev)
    reps = max(args.steps // o["layers"], 1)
    args_g = argparse.Namespace(**{**vars(args), "steps": reps, "warmup": max(args.warmup // o["layers"], 3)})
    ms, clocks = timed_steps(lambda i: g.replay(), args_g, dev, world, local)
    ms /= o["layers"]
    steps_timed = reps * o["layers"]
    # end to end: the attention output from pinned host memory, the residual stream back
    o_layers = o["layers"]
    e_ms = pipelined_e2e(lambda i, ins, o: cb.o_proj_residual(ins[0], ws[i % o_layers], o, out=o),
                         [x.cpu().pin_memory()], resid, args, dev, world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r, cores, sample = oproj_reference_rate(target_s=6.0)
        cpu = {"value": r, "unit": "tokens/s", "cores": cores, "kind": "reference", "sample": sample}
    if world > 1:
        dist.barrier()
        if rank != 0:
            dist.destroy_process_group()
            return
    peak, peak_kind = peaks()
    wbytes = o["fout"] * o["fin"] * 2
    alg = wbytes + x.numel() * 2 + 2 * resid.numel() * 4
    line = {
        "metric": "O-projection+residual tokens/s", "value": world * o["B"] / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": world, "steps": steps_timed, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 x f16 -> f32",
        "data": "synthetic: seeded N(0,1) activations and residual, N(0, 1/in) fp16 weights",
        "config": {"workload": f"oproj_llama3_8b: {o['fin']} -> {o['fout']}, batch {o['B']}, "
                               f"one of {o['layers']} layers per step, in place on the fp32 residual",
                   "l2": f"{o['layers']} layers' weights ({o['layers'] * wbytes / 1e6:.0f} MB) cycled, > 126 MB L2",
                   "parallelism": f"replicas on {world} GPU(s), no collective"},
        "roofline": {"bound": "hbm", "achieved": alg / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": alg / (ms * 1e-3) / 1e9 / peak, "traffic": None, "peak_kind": peak_kind,
                     "kernel": "qkv_proj_kernel (GEMM) + oproj_finish_kernel per step (CUDA graph of 8 layers' steps)",
                     "kernel_ms": ms,
                     "algorithmic_bytes": alg},
        "cpu_baseline": cpu,
        "e2e": {"value": world * o["B"] / (e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": x.numel() * 2,
                "d2h_bytes_per_step": resid.numel() * 4, "ms_per_step": e_ms,
                "api": "cottus_o_proj_residual (C ABI via ctypes)", "pipelining": "two buffer sets, two copy streams"},
        "gpu_launches": 2 * steps_timed, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    del g
    if world > 1:
        dist.destroy_process_group()


def oproj_reference_rate(target_s=6.0):
    """The reference's CPU step for one token and one layer: gemmCPU with wo
    (fp32, [in][out]) then residualAddCPU (generic_transformer.cpp:305-327),
    tokens spread over the host threads; returns (tokens/s, threads, sample)."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle.oracle import Reference

    o = OPROJ
    ref = Reference()
    rng = np.random.default_rng(4)
    wt = rng.standard_normal((o["fin"], o["fout"]), dtype=np.float32) / np.float32(o["fin"] ** 0.5)
    threads = os.cpu_count() or 1
    xs = rng.standard_normal((threads, o["fin"]), dtype=np.float32)
    res = rng.standard_normal((threads, o["fout"]), dtype=np.float32)

    def one(i):
        res[i] += ref.gemm(xs[i:i + 1], wt)[0]

    done, t0 = 0, time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        while True:
            list(ex.map(one, range(threads)))
            done += threads
            el = time.perf_counter() - t0
            if el >= target_s:
                break
    return done / el, threads, f"{done} tokens x 1 layer ({el:.1f} s wall, {threads} threads)"


ATTN = dict(hidden=4096, H=32, Hkv=8, D=128, B=64, ctx=2048, layers=4, bs=16)  # Llama-3-8B, batch 64


def run_attn_block(args, rank, world, local):
    """The attention half of one decoder layer per step, for 64 sequences at
    context 2048 (Llama-3-8B shape): QKV projection + RoPE + KV append
    (cottus_qkv_rope_append), paged decode attention over the 2048 tokens
    (cottus_paged_decode), O-projection + residual (cottus_o_proj_residual).
    Four layers' weights (336 MB) and KV (2.1 GB) cycled; the three calls of
    a step issued directly on the stream, their kernels chained by
    programmatic dependent launch.  Replicas per GPU (weak scaling)."""
    import torch
    import torch.distributed as dist
    import cottus_b200 as cb

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    A = ATTN
    H, Hkv, D, B, L, bs = A["H"], A["Hkv"], A["D"], A["B"], A["layers"], A["bs"]
    N, HD = (H + 2 * Hkv) * D, H * D
    g = torch.Generator(device="cpu").manual_seed(13)
    x = torch.randn((B, A["hidden"]), generator=g).half().to(dev)
    wq = [(torch.randn((N, A["hidden"]), generator=g) / A["hidden"] ** 0.5).half().to(dev) for _ in range(L)]
    wo = [(torch.randn((A["hidden"], HD), generator=g) / HD ** 0.5).half().to(dev) for _ in range(L)]
    resid = torch.randn((B, A["hidden"]), generator=g).to(dev)
    pages = A["ctx"] // bs
    nb = B * pages
    gd = torch.Generator(device=dev).manual_seed(14)
    pool = torch.randn(nb * 2 * L * bs * Hkv * D, generator=gd, device=dev).half().view(torch.int16)
    table = torch.randperm(nb, generator=g).int().view(B, pages).to(dev)
    pos = torch.full((B,), A["ctx"] - 1, dtype=torch.int32, device=dev)
    ctx_lens = pos + 1
    tab = cb.rope_cos_sin_table(A["ctx"], D).to(dev)
    q = torch.empty((B, H, D), dtype=torch.float16, device=dev)
    att = torch.empty((B, H, D), dtype=torch.float16, device=dev)

    def step(i, xx=x):
        layer = i % L
        cb.qkv_rope_append(xx, wq[layer], pos, tab, pool, table, num_heads=H, num_kv_heads=Hkv, head_dim=D,
                           block_size=bs, num_layers=L, layer=layer, num_physical_blocks=nb, query_out=q)
        cb.paged_decode(q, pool, table, ctx_lens, num_kv_heads=Hkv, head_dim=D, block_size=bs, num_layers=L,
                        layer=layer, out=att, num_physical_blocks=nb)
        cb.o_proj_residual(att.view(B, HD), wo[layer], resid, out=resid)

    # direct launches: the host issues a step's three calls faster than the GPU runs them
    ms, clocks = timed_steps(step, args, dev, world, local)
    steps_timed = args.steps
    # end to end: the normalised hidden state from pinned host memory, the residual stream back
    def block(i, ins, o):
        layer = i % L
        cb.qkv_rope_append(ins[0], wq[layer], pos, tab, pool, table, num_heads=H, num_kv_heads=Hkv, head_dim=D,
                           block_size=bs, num_layers=L, layer=layer, num_physical_blocks=nb, query_out=q)
        cb.paged_decode(q, pool, table, ctx_lens, num_kv_heads=Hkv, head_dim=D, block_size=bs, num_layers=L,
                        layer=layer, out=att, num_physical_blocks=nb)
        cb.o_proj_residual(att.view(B, HD), wo[layer], o, out=o)

    e_ms = pipelined_e2e(block, [x.cpu().pin_memory()], resid, args, dev, world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r, cores, sample = attn_reference_rate(target_s=9.0)
        cpu = {"value": r, "unit": "tokens/s", "cores": cores, "kind": "reference", "sample": sample}
    if world > 1:
        dist.barrier()
        if rank != 0:
            dist.destroy_process_group()
            return
    peak, peak_kind = peaks()
    wbytes = (N + A["hidden"]) * A["hidden"] * 2
    kv_read = B * A["ctx"] * 2 * Hkv * D * 2
    alg = (wbytes + kv_read + x.numel() * 2 + 2 * q.numel() * 2 + att.numel() * 2 + 2 * resid.numel() * 4 +
           B * 2 * Hkv * D * 2 + table.numel() * 4)
    line = {
        "metric": "attention block tokens/s", "value": world * B / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": world, "steps": steps_timed, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 x f16 -> f32",
        "data": "synthetic: seeded N(0,1) activations, KV and residual, N(0, 1/in) fp16 weights",
        "config": {"workload": f"attn_block_llama3_8b: hidden {A['hidden']}, H{H}/Hkv{Hkv}/D{D}, batch {B}, "
                               f"context {A['ctx']}, one of {L} layers per step (QKV+RoPE+append, paged decode, "
                               f"O-proj+residual)",
                   "l2": f"{L} layers' weights ({L * wbytes / 1e6:.0f} MB) and KV ({L * kv_read / 1e9:.1f} GB) "
                         "cycled, > 126 MB L2",
                   "parallelism": f"replicas on {world} GPU(s), no collective"},
        "roofline": {"bound": "hbm", "achieved": alg / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": alg / (ms * 1e-3) / 1e9 / peak, "traffic": None, "peak_kind": peak_kind,
                     "kernel": "qkv_proj_kernel + qkv_finish_kernel + decode_mma_kernel + qkv_proj_kernel + "
                               "oproj_finish_kernel per step (direct launches, layers cycled)",
                     "kernel_ms": ms, "algorithmic_bytes": alg},
        "cpu_baseline": cpu,
        "e2e": {"value": world * B / (e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": x.numel() * 2,
                "d2h_bytes_per_step": resid.numel() * 4, "ms_per_step": e_ms,
                "api": "cottus_qkv_rope_append + cottus_paged_decode + cottus_o_proj_residual (C ABI via ctypes)",
                "pipelining": "two buffer sets, two copy streams"},
        "gpu_launches": 5 * steps_timed, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def attn_reference_rate(target_s=9.0):
    """The reference's CPU path of the attention block for one token and one
    layer: gemmCPU x3 + ropeCPU (QKV), pagedAttentionCPU over 2048 tokens,
    gemmCPU with wo + residualAddCPU, each phase timed over all host threads;
    the phases run one after the other, so tokens/s = 1 / (sum of the
    phases' seconds per token).  Returns (tokens/s, threads, sample)."""
    import torch
    from cottus_b200 import workloads as W

    r_q, threads, _ = qkv_reference_rate(target_s=target_s / 3)
    r_o, _, _ = oproj_reference_rate(target_s=target_s / 3)
    w = W.llama3_8b(seed=9, B=threads, context=ATTN["ctx"])
    t = W.device_tensors(w, "cpu")
    rb = ReferenceBatch(w, t)
    n, reps, t0 = len(rb.ctx), 0, time.perf_counter()
    while True:
        rb.run(n)
        reps += 1
        el = time.perf_counter() - t0
        if el >= target_s / 3:
            break
    r_a = n * reps / el
    del t, torch
    r = 1.0 / (1.0 / r_q + 1.0 / r_a + 1.0 / r_o)
    return r, threads, (f"per phase, all {threads} threads: QKV {r_q:.0f}, attention over {ATTN['ctx']} tokens "
                        f"{r_a:.0f}, O-proj {r_o:.0f} tokens/s")


# -- decode workloads ---------------------------------------------------------------------

DTYPE_F16 = "f16 (fp16 Q, KV and O; fp16 probabilities on the tensor cores; fp32 accumulation)"
DTYPE_F32 = "f32 out (fp16 KV; fp32 Q/O; fp32-accurate products as fp16 hi+lo pairs on the tensor cores; fp32 accumulation)"


def l2_plan(kv_bytes):
    """How a workload's steps avoid reading KV that an earlier step left in
    L2.  KV of at least 2 x L2 per step: none needed.  Smaller KV: each step
    is one layer of a pool of L layers and the steps cycle through the
    layers, as a decode loop does, with L chosen so that a cycle covers
    3 x L2 (hundreds of layers below 1 MB per layer: a few hundred MB of
    HBM).  Below 8 MB per layer a step's kernel is shorter than one
    host-side call through ctypes, so the K timed steps are captured once
    in a CUDA graph and replayed (graph = True), as a decode engine issues
    its per-layer launches.  Returns (layers, graph)."""
    if kv_bytes >= 2 * L2_BYTES:
        return 1, False
    return -(-3 * L2_BYTES // max(kv_bytes, 1)), kv_bytes < 8 * 1024 * 1024


def l2_text(kv_bytes, layers, graph):
    if layers > 1:
        return (f"{layers} layers' KV cycled ({layers * kv_bytes / 1e6:.0f} MB > 126 MB L2), one layer per step, "
                "no flush" + ("; the timed steps replayed from one CUDA graph" if graph else ""))
    return f"inputs larger than L2 ({kv_bytes / 1e6:.0f} MB KV per GPU vs 126 MB L2), no flush"


def decode_kernel_name(w):
    """The kernel cottus_paged_decode selects for this workload."""
    mma = (w.H // w.Hkv) > 1 and w.D in (64, 128)
    return ("decode_mma_kernel" if mma else "decode_tma_kernel") + (" (RoPE + append fused)" if w.fused else "")


def decode_config(args, world):
    """(workload, the JSON `config` object): the same in both arms."""
    from cottus_b200 import workloads as W
    w = build_workload(args.config, 0, args.batch)
    split = args.config == "long_ctx_70b" and world > 1
    per_gpu = w.kv_bytes() // world if split else w.kv_bytes()
    layers, graph = l2_plan(per_gpu)
    cfg = {"workload": describe(w), "kv": "fp16", "q_out": str(w.q_dtype).replace("torch.", ""),
           "per_gpu_batch": w.B, "kv_bytes_per_step_per_gpu": per_gpu, "l2": l2_text(per_gpu, layers, graph),
           "parallelism": ((f"split-KV over {world} GPUs, " +
                            ("LSE partials read from peer memory over NVLink after a completion flag raised by the "
                             "decode kernel" if args.exchange == "peer" else "NCCL all-gather of LSE partials"))
                           if split else f"sequence-sharded over {world} GPU(s), no collective")}
    del W
    return w, cfg


def run_decode(args, rank, world, local):
    """The five decode workloads: one step = one cottus_paged_decode (or
    cottus_rope_append_decode) launch over the batch; long_ctx_70b on N > 1
    GPUs splits every sequence's pages over the ranks."""
    import dataclasses

    import torch
    import torch.distributed as dist
    import cottus_b200 as cb
    from cottus_b200 import workloads as W

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    split = args.config == "long_ctx_70b" and world > 1
    w, config = decode_config(args, world)
    if not split:
        w = build_workload(args.config, rank, args.batch)
    if split:
        wl = W.shard_long_context(w, rank, world)
    else:
        wl = w
    kv_bytes_rank = wl.kv_bytes()
    layers, graph = l2_plan(kv_bytes_rank)
    if layers > 1:
        w = dataclasses.replace(w, L=layers)
        wl = w
    if split:
        t = W.device_tensors(wl, dev, pool_blocks=wl.meta["pool_range"])
        t["block_table"] = torch.from_numpy(wl.block_table).to(dev)
        t["context_lens"] = torch.from_numpy(wl.ctx).to(dev)
    else:
        t = W.device_tensors(wl, dev)
    if w.fused:
        t["cos_sin"] = cb.rope_cos_sin_table(int(w.positions.max()) + 1, w.D, w.theta).to(dev)

    stream = torch.cuda.current_stream(dev)
    out = torch.empty((w.B, w.H, w.D), dtype=w.out_dtype, device=dev)
    part = torch.empty((w.B, w.H, w.D), dtype=torch.float32, device=dev)
    lse = torch.empty((w.B, w.H), dtype=torch.float32, device=dev)
    pool_snapshot = t["kv_pool"].clone() if w.fused else None  # the fused step appends; restore is not timed

    exchange = None
    if split:
        from cottus_b200 import parallel
        if args.exchange == "peer":
            exchange = parallel.PeerExchange(w.B, w.H, w.D)
    # split over ranks: through peer memory the tensor-core decode kernel also merges the ranks' partials
    # (one launch); through NCCL a decode and an LSE combine launch around the all-gathers
    launches_per_step = (1 if args.exchange == "peer" else 2) if split else 1

    def step(i):
        layer = i % w.L
        if w.fused:
            cb.rope_append_decode(t["query"], t["key"], t["value"], t["positions"], t["cos_sin"], t["kv_pool"],
                                  t["block_table"], num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs,
                                  num_layers=w.L, layer=layer, out=out)
        elif split and exchange is not None:
            # decode kernel (completion flagged to every rank) + combine kernel reading peers over NVLink
            parallel.split_kv_decode_peer(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], exchange,
                                          num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs,
                                          num_physical_blocks=wl.num_blocks, out_dtype=w.out_dtype, out=out)
        elif split:
            parallel.split_kv_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"],
                                     num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs,
                                     num_physical_blocks=wl.num_blocks, out_dtype=w.out_dtype, part=part, lse=lse)
        else:
            cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                            head_dim=w.D, block_size=w.bs, num_layers=w.L, layer=layer, out=out,
                            num_physical_blocks=wl.num_blocks)

    # W warm-up steps right before the K timed ones (no idle pause in between)
    sampler = start_clocks(local)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    # short kernels (see l2_plan): the K timed steps captured as one CUDA graph after the warm-up, without
    # running them first, so that the layers they read were last touched when the pool was written
    timed_graph = graph_of_steps(lambda i: step(args.warmup + i), args.steps, dev, prerun=False) if graph else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    if graph:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        hold_gpu()
        e0.record(stream)
        timed_graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        elapsed_ms = e0.elapsed_time(e1)
    else:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        hold_gpu()
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        elapsed_ms = e0.elapsed_time(e1)
    clocks = sampler.stop()
    ms = max_over_ranks(elapsed_ms, dev, world) / args.steps

    # the dominant kernel alone: one decode launch between each event pair
    ka = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(50)]
    for i, (a, b) in enumerate(ka):
        a.record(stream)
        if w.fused:
            step(i)
        else:
            cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                            head_dim=w.D, block_size=w.bs, num_layers=w.L, layer=i % w.L,
                            out=part if split else out, lse_out=lse if split else None,
                            num_physical_blocks=wl.num_blocks)
        b.record(stream)
    torch.cuda.synchronize(dev)
    k_ms = float(np.mean([a.elapsed_time(b) for a, b in ka]))

    # end to end through the C ABI with host buffers: every step copies its inputs from pinned host
    # memory and reads its output back into pinned host memory (pipelined: the copies of neighbouring
    # steps overlap each kernel)
    e2e = None
    if not args.no_e2e and not split:
        if w.fused:
            host_in = [t["query"].cpu().pin_memory(), t["key"].cpu().pin_memory(), t["value"].cpu().pin_memory(),
                       t["positions"].cpu().pin_memory(), t["block_table"].cpu().pin_memory()]

            def call(i, ins, o):
                cb.rope_append_decode(ins[0], ins[1], ins[2], ins[3], t["cos_sin"], t["kv_pool"], ins[4],
                                      num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs, num_layers=w.L,
                                      layer=i % w.L, out=o)
            api = "cottus_rope_append_decode (C ABI via ctypes)"
        else:
            host_in = [t["query"].cpu().pin_memory(), t["block_table"].cpu().pin_memory(),
                       t["context_lens"].cpu().pin_memory()]

            def call(i, ins, o):
                cb.paged_decode(ins[0], t["kv_pool"], ins[1], ins[2], num_kv_heads=w.Hkv, head_dim=w.D,
                                block_size=w.bs, num_layers=w.L, layer=i % w.L, out=o,
                                num_physical_blocks=wl.num_blocks)
            api = "cottus_paged_decode (C ABI via ctypes)"
        e_ms = pipelined_e2e(call, host_in, out, args, dev, world)
        h2d = sum(h.numel() * h.element_size() for h in host_in)
        d2h = out.numel() * out.element_size()
        e2e = {"value": world * kv_bytes_rank / (e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms, "api": api,
               "pipelining": "two buffer sets; uploads and read-backs on two copy streams overlap the kernels"}
        if graph:
            e2e["launches"] = "direct calls through ctypes (not a graph): bound by the host-side call"

    if pool_snapshot is not None:
        t["kv_pool"].copy_(pool_snapshot)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            wc = dataclasses.replace(w, L=1) if w.L > 1 else w
            tc = W.device_tensors(wc, dev) if w.L > 1 else t
            r, threads, sample = cpu_reference_rate(wc, tc, target_s=8.0,
                                                    max_seqs=1 if w.name == "long_ctx_70b" else None)
            cpu = {"value": r, "unit": "GB/s", "cores": threads, "kind": "reference", "sample": sample}
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "GB/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {ex}"}

    if exchange is not None:
        exchange.close()  # collective: every rank is done with the peer buffers
    del t, pool_snapshot, timed_graph
    torch.cuda.empty_cache()

    extras = {}
    if args.config == "llama3_8b" and not args.no_extras and args.batch is None:
        extras["strong_scaling"] = strong_scaling_extra(args, rank, world, local)
        extras["split_kv"] = split_kv_extra(args, rank, world, local)

    if world > 1:
        dist.barrier()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    peak, peak_kind = peaks()
    total_kv = w.kv_bytes() if split else kv_bytes_rank * world
    value = total_kv / (ms * 1e-3) / 1e9
    alg = kv_bytes_rank + wl.io_bytes()
    # launch duration for the roofline: where a step is one launch of the
    # kernel, the timed region per launch (launches back to back, as a decode
    # loop issues them); otherwise the kernel timed alone between events
    kern_ms = ms if launches_per_step == 1 else k_ms
    achieved = alg / (kern_ms * 1e-3) / 1e9
    traffic = None
    prof = ROOT / "profiles" / "traffic.json"
    if prof.exists():
        tr = json.loads(prof.read_text()).get(w.name)
        traffic = tr.get("bytes_per_launch") if isinstance(tr, dict) else tr
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if split else "weak", "vs_baseline": None,
        "dtype": DTYPE_F16 if w.out_dtype == torch.float16 else DTYPE_F32,
        "data": "synthetic: seeded N(0,1) KV stored via the reference's truncating fp16 encoder",
        "config": config,
        "tokens_per_s": w.B * (1 if split else world) / (ms * 1e-3),
        "pct_hbm_peak": value / world / peak * 100,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_kind": peak_kind,
                     "kernel": decode_kernel_name(w) +
                     ((" with the peer merge in the same launch" if args.exchange == "peer"
                       else " + lse_combine_kernel") if split else "") +
                     ": one decode launch per step",
                     "kernel_ms": kern_ms, "kernel_ms_alone": k_ms, "algorithmic_bytes": alg},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches_per_step * args.steps, "clocks": clocks,
    }
    line.update(extras)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def device_ms(step, args, dev, world):
    """W warm-up steps, then K steps between events on the current stream
    (a synchronize and a barrier between the two); ms per step, max over ranks."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    hold_gpu()
    e0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return max_over_ranks(e0.elapsed_time(e1), dev, world) / args.steps


def strong_scaling_extra(args, rank, world, local):
    """The default workload's fixed batch of 64 sequences partitioned across
    the N ranks (64 / N sequences each, no collective), steps cycling
    through enough layers' KV that no step reads L2-resident KV.  Total
    work fixed as N grows."""
    import dataclasses

    import torch
    import cottus_b200 as cb
    from cottus_b200 import workloads as W

    dev = torch.device("cuda", local)
    B = 64
    per = B // world
    w = W.llama3_8b(seed=3000 + rank, B=per)
    layers, _ = l2_plan(w.kv_bytes())
    w = dataclasses.replace(w, L=layers)
    t = W.device_tensors(w, dev)
    out = torch.empty((w.B, w.H, w.D), dtype=w.out_dtype, device=dev)

    def step(i):
        cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                        head_dim=w.D, block_size=w.bs, num_layers=w.L, layer=i % w.L, out=out,
                        num_physical_blocks=w.num_blocks)

    ms = device_ms(step, args, dev, world)
    peak, _ = peaks()
    total = B * 2048 * 2 * w.Hkv * w.D * 2
    del t
    torch.cuda.empty_cache()
    return {"workload": f"llama3_8b batch {B} partitioned over {world} GPU(s): {per} sequences per GPU, "
                        f"{l2_text(w.kv_bytes(), layers, False)}",
            "scaling": "strong", "ms_per_step": ms, "GB_s": total / (ms * 1e-3) / 1e9,
            "tokens_per_s": B / (ms * 1e-3), "frac_of_n_peaks": total / (ms * 1e-3) / 1e9 / (world * peak),
            "gpu_launches": args.steps}


def split_kv_extra(args, rank, world, local):
    """The long-context workload (H64/Hkv8/D128, batch 8, context 131072,
    4.3 GB of KV) with every sequence's pages split over the N ranks: per
    step a decode of each rank's page range and the merge of the ranks'
    partials, through peer memory (cottus_split_decode) and through NCCL.
    Also times each rank's decode alone, and on rank 0 the un-split decode
    on one GPU, so the line says where the N-GPU step loses to N-fold; and
    the kv-head partition of the same workload (kv_head_partition: each
    rank decodes Hkv/N kv heads of every page, no exchange)."""
    import torch
    import torch.distributed as dist
    import cottus_b200 as cb
    from cottus_b200 import parallel
    from cottus_b200 import workloads as W

    dev = torch.device("cuda", local)
    w = W.long_ctx_70b(seed=4000)
    out = torch.empty((w.B, w.H, w.D), dtype=torch.float16, device=dev)
    peak, _ = peaks()
    res = {"workload": f"long_ctx_70b: H{w.H}/Hkv{w.Hkv}/D{w.D}, batch {w.B}, context {int(w.ctx[0])}, "
                       f"pages of every sequence split over {world} GPU(s)", "scaling": "strong"}
    if world == 1:
        t = W.device_tensors(w, dev)

        def one(i):
            cb.paged_decode(t["query"], t["kv_pool"], t["block_table"], t["context_lens"], num_kv_heads=w.Hkv,
                            head_dim=w.D, block_size=w.bs, out=out, num_physical_blocks=w.num_blocks)
        ms1 = device_ms(one, args, dev, world)
        res.update({"ms_per_step": ms1, "GB_s": w.kv_bytes() / (ms1 * 1e-3) / 1e9,
                    "frac_of_n_peaks": w.kv_bytes() / (ms1 * 1e-3) / 1e9 / peak, "ms_per_step_1gpu": ms1,
                    "efficiency_vs_1gpu": 1.0, "gpu_launches": args.steps,
                    "kv_head_partition": {"workload": f"all {w.Hkv} kv heads on one GPU", "exchange": "none",
                                          "ms_per_step": ms1, "GB_s": w.kv_bytes() / (ms1 * 1e-3) / 1e9,
                                          "frac_of_n_peaks": w.kv_bytes() / (ms1 * 1e-3) / 1e9 / peak,
                                          "efficiency_vs_1gpu": 1.0, "gpu_launches": args.steps}})
        del t
        torch.cuda.empty_cache()
        return res
    s = W.shard_long_context(w, rank, world)
    t = W.device_tensors(s, dev, pool_blocks=s.meta["pool_range"])
    bt, cl = torch.from_numpy(s.block_table).to(dev), torch.from_numpy(s.ctx).to(dev)
    part = torch.empty((w.B, w.H, w.D), dtype=torch.float32, device=dev)
    lse = torch.empty((w.B, w.H), dtype=torch.float32, device=dev)
    kw = dict(num_kv_heads=w.Hkv, head_dim=w.D, block_size=w.bs, num_physical_blocks=s.num_blocks)
    ex = parallel.PeerExchange(w.B, w.H, w.D)
    ms_peer = device_ms(lambda i: parallel.split_kv_decode_peer(t["query"], t["kv_pool"], bt, cl, ex,
                                                                out_dtype=torch.float16, out=out, **kw),
                        args, dev, world)
    ex.close()
    ms_nccl = device_ms(lambda i: parallel.split_kv_decode(t["query"], t["kv_pool"], bt, cl, out_dtype=torch.float16,
                                                           part=part, lse=lse, **kw), args, dev, world)
    ms_dec = device_ms(lambda i: cb.paged_decode(t["query"], t["kv_pool"], bt, cl, out=part, lse_out=lse, **kw),
                       args, dev, world)
    del t
    torch.cuda.empty_cache()
    ms1 = None
    tf = W.device_tensors(w, dev)
    if rank == 0:
        # the same workload un-split on this GPU alone (the other ranks wait at the barrier)
        one_args = argparse.Namespace(**{**vars(args)})

        def one(i):
            cb.paged_decode(tf["query"], tf["kv_pool"], tf["block_table"], tf["context_lens"], num_kv_heads=w.Hkv,
                            head_dim=w.D, block_size=w.bs, out=out, num_physical_blocks=w.num_blocks)
        ms1 = device_ms(one, one_args, dev, 1)
    dist.barrier()
    # the kv-head partition: every rank keeps Hkv/N kv heads of every page and the query heads of their
    # groups, and its outputs are final for those heads (no exchange, no collective in the step)
    sh, sht = W.shard_kv_heads(w, tf, rank, world)
    del tf
    torch.cuda.empty_cache()
    outh = torch.empty((w.B, sh.H, w.D), dtype=torch.float16, device=dev)
    ms_heads = device_ms(lambda i: cb.paged_decode(sht["query"], sht["kv_pool"], sht["block_table"],
                                                   sht["context_lens"], num_kv_heads=sh.Hkv, head_dim=w.D,
                                                   block_size=w.bs, out=outh, num_physical_blocks=sh.num_blocks),
                         args, dev, world)
    del sht
    torch.cuda.empty_cache()
    gbh = w.kv_bytes() / (ms_heads * 1e-3) / 1e9
    res["kv_head_partition"] = {
        "workload": f"kv heads {sh.meta['kv_heads'][0]}.. of {w.Hkv} on rank 0: {sh.Hkv} kv / {sh.H} query heads "
                    f"per GPU, every page", "exchange": "none", "ms_per_step": ms_heads, "GB_s": gbh,
        "frac_of_n_peaks": gbh / (world * peak), "efficiency_vs_1gpu": (ms1 / (world * ms_heads)) if ms1 else None,
        "gpu_launches": args.steps}
    gb = w.kv_bytes() / (ms_peer * 1e-3) / 1e9
    res.update({"exchange": "peer memory over NVLink (cottus_split_decode)", "ms_per_step": ms_peer,
                "GB_s": gb, "frac_of_n_peaks": gb / (world * peak), "ms_per_step_nccl": ms_nccl,
                "ms_decode_alone": ms_dec, "exchange_and_merge_ms": ms_peer - ms_dec, "ms_per_step_1gpu": ms1,
                "efficiency_vs_1gpu": (ms1 / (world * ms_peer)) if ms1 else None,
                "gpu_launches": args.steps})
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="llama3_8b",
                    choices=["tinyllama_f32", "llama3_8b", "ragged_mha", "long_ctx_70b", "fused_tinyllama",
                             "qkv_llama3_8b", "oproj_llama3_8b", "attn_block_llama3_8b"])
    ap.add_argument("--batch", type=int, default=None, help="override the batch size (profiling runs)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the strong-scaling and split-context lines added to the default workload's line")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="split-context partial exchange: peer memory over NVLink, or NCCL all-gather")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    {"qkv_llama3_8b": run_qkv, "oproj_llama3_8b": run_oproj,
     "attn_block_llama3_8b": run_attn_block}.get(args.config, run_decode)(args, rank, world, local)


if __name__ == "__main__":
    main()
