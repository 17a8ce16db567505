"""Benchmark of the B200 decode-attention hot path (tinyllama-engine GQA).

Workload (the largest single-GPU decode case):
256 sequences x 32768 cached positions (pos = 32767, 32768 attended rows),
TinyLlama attention geometry (32 q heads, 4 KV heads, head_dim 64), fp32
KV ~ N(0,1), one layer per step (17.18 GB of K+V per step, far larger than
the 126 MB L2, so no flush is needed).  A step is one fused
rope + append + GQA decode-attention call for every sequence
(tle_decode_batch), i.e. attention() of src/ops.cpp:1317 for 256 sequences.

Multi-GPU (torchrun, one process per GPU): the 256 equal sequences are cut
into contiguous equal blocks (shard.plan), every rank decodes its block from
its own HBM straight into its slot of the all-gather buffer, and the in-place
NCCL all-gather leaves them in sequence order on every rank; the step time is
the max over ranks (strong scaling: the 256-sequence total is fixed).  The same line carries
config 4 at the job's GPU count (`decode_config4`: 64 ragged sequences
LPT-partitioned, 22 layers per step, one all-gather of every layer's
outputs per step).

`--impl reference` times the reference's own CPU attention (src/ops.cpp
compiled unmodified into oracle/_ref) on a bounded sample of the same
workload on all host cores.

Secondary lines (N=1, unless --no-secondary): prefill (config 3), batched
ragged decode (config 4, contiguous and paged), single-sequence decode
(config 1), paged config 5, and end-to-end greedy generation on the device
(config 2: the whole forward pass, tle_forward.h).  `--only NAME` runs one.

Prints ONE JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tinyllama-engine_b200"))

N_SEQS = 256
CTX = 32768
NH, NKV, HD = 32, 4, 64
QD, KVD = NH * HD, NKV * HD
ROW_BYTES = 2 * KVD * 4  # K + V bytes per attended row (all 4 KV heads)
METRIC = "decode-attn KV GB/s"
WORKLOAD = ("config5: 256 seqs x 32768 cached rows (pos 32767), 32q/4kv heads, hd 64, fp32 KV, "
            "1 layer per step, fused rope+append+GQA split-K decode")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["tle", "reference"], default="tle")
    ap.add_argument("--seqs", type=int, default=N_SEQS)
    ap.add_argument("--ctx", type=int, default=CTX)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the config-3 prefill and config-4 ragged-decode lines")
    ap.add_argument("--ctx-rows", type=int, default=4 * 1024 * 1024,
                    help="rows of the single sequence for --only ctxsplit")
    ap.add_argument("--only", choices=["prefill3", "decode4", "decode1", "ctxsplit", "decode5paged", "decode5bf16",
                                       "decode4paged", "generate2", "prompt2"], default=None,
                    help="run one secondary workload alone (--steps/--warmup apply) and print "
                         "its line; for profiling")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="target wall time of the CPU-baseline sample")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1])); smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ------------------------------------------------------------ CPU baseline
def cpu_reference_run(seqs: int, ctx: int, steps: int, warmup: int, target_s: float):
    """Times the reference's attention() (oracle/_ref, compiled from its own
    src/ops.cpp) over a bounded sample of the workload with all host threads.
    Returns (GB/s, dict describing the sample)."""
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    kind = "reference" if oracle.have_reference() else "port"
    lib = oracle.reference() if kind == "reference" else oracle.port()
    threads = os.cpu_count() or 1
    n = max(1, min(seqs, threads, 64))
    g = torch.Generator().manual_seed(1234)
    kcs = [torch.randn((1, ctx, KVD), generator=g).numpy() for _ in range(n)]
    vcs = [torch.randn((1, ctx, KVD), generator=g).numpy() for _ in range(n)]
    q = torch.randn((n, QD), generator=g).numpy()
    k = torch.randn((n, KVD), generator=g).numpy()
    v = torch.randn((n, KVD), generator=g).numpy()
    out = np.zeros((n, QD), np.float32)
    pos = [ctx - 1] * n

    def one():
        lib.decode_batch(kcs, vcs, [ctx] * n, pos, q.copy(), k.copy(), v, out, 0, n_threads=n)

    for _ in range(max(0, warmup)):
        one()
    times = []
    t_end = time.perf_counter() + target_s
    while len(times) < max(1, steps) and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    gbs = n * ctx * ROW_BYTES / med / 1e9
    desc = {"kind": kind, "cores": n,
            "sample": f"{n} of {seqs} sequences x {ctx} rows, 1 layer, rope+attention per sequence "
                      f"on {n} std::threads; median of {len(times)} runs",
            "seconds": round(sum(times), 2), "cpu_model": cpu_model(), "host_threads": threads}
    return gbs, med, len(times), desc


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------- GPU arm
def main_config(args):
    """`config` of the headline line, the same dict in both arms."""
    n = args.gpus
    return {"workload": WORKLOAD, "n_seqs": args.seqs, "ctx": args.ctx, "layers_timed": 1,
            "l2": "inputs larger than L2 (17.2 GB of K+V per step)",
            "parallelism": "sequence partition over %d GPUs + NCCL all-gather" % n if n > 1 else "1 GPU"}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        # Reference arm: rank 0 alone times the reference CPU path.
        if rank != 0:
            return
        gbs, med, runs, desc = cpu_reference_run(args.seqs, args.ctx, args.steps, args.warmup,
                                                 target_s=max(20.0, args.cpu_seconds))
        line = {"metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": runs, "warmup": args.warmup,
                "ms_per_step": round(med * 1e3, 3), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), seeded",
                "config": main_config(args),
                "cpu_baseline": dict(desc, value=round(gbs, 3), unit="GB/s"),
                "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    import tle

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.only == "ctxsplit":
        measure_ctxsplit(args, dev, rank, world, local)
        return
    if args.only:
        fn = {"prefill3": measure_prefill, "decode4": measure_config4, "decode1": measure_config1,
              "decode5paged": measure_paged5, "decode4paged": measure_paged4, "decode5bf16": measure_bf16_5,
              "generate2": measure_config2, "prompt2": measure_prompt2}[args.only]
        kw = {"n_seqs": args.seqs, "ctx": args.ctx} if args.only == "decode5bf16" else {}
        res = fn(dev, load_peaks(), steps=args.steps, warmup=max(3, args.warmup), **kw)
        print(json.dumps(dict(res, impl="tle", n_gpus=1, steps=args.steps,
                              warmup=max(3, args.warmup))), flush=True)
        return
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    peaks = load_peaks()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    r5 = run_config5(args, dev, rank, world, barrier)
    clk = clocks.stop()
    r4 = run_config4_sharded(dev, rank, world, barrier, peaks)
    err_code = tle.device_error()
    if err_code:
        raise RuntimeError(f"device error word 0x{err_code:x}")

    if rank == 0:
        total_bytes = args.seqs * args.ctx * ROW_BYTES
        step_s = r5["t_ms"] / 1e3 / args.steps
        value = total_bytes / step_s / 1e9
        e2e_value = total_bytes / (r5["e2e_ms"] / 1e3 / args.steps) / 1e9
        achieved = r5["local_bytes"] / (r5["kernel_ms"] / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": round(r5["t_ms"] / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic N(0,1) fp32, seeded (no dataset)",
            "config": main_config(args),
            "tok_s_attn_22_layers": round(args.seqs / (step_s * 22), 1),
            "frac_per_gpu": round(value / world / peaks["hbm_gbs"], 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_source": peaks["source"],
                         "traffic": profile_traffic(r5["local_bytes"]),
                         "kernel": "decode_kernel (tle_decode_batch, split-K merge fused), rank 0",
                         "algorithmic_bytes_per_launch": r5["local_bytes"],
                         "kernel_ms": round(r5["kernel_ms"], 4)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": r5["h2d_bytes"], "d2h_bytes_per_step": r5["d2h_bytes"],
                    "ms_per_step": round(r5["e2e_ms"] / args.steps, 4)},
            "decode_config4": r4,
            "gpu_launches": args.steps,   # one decode_kernel per tle_decode_batch call
            "clocks": clk,
        }
        if world == 1 and not args.no_secondary:
            line["secondary"] = {
                "prefill_config3": compact(measure_prefill(dev, peaks)),
                "decode_config4_n1": compact(measure_config4(dev, peaks)),
                "decode_config1": compact(measure_config1(dev, peaks)),
                "decode_config4_paged": compact(measure_paged4(dev, peaks)),
                "decode_config5_paged": compact(measure_paged5(dev, peaks)),
                "decode_config5_bf16": compact(measure_bf16_5(dev, peaks)),
                "generate_config2": compact(measure_config2(dev, peaks, steps=3)),
                "prompt_config2": compact(measure_prompt2(dev, peaks, steps=3))}
        if world == 1 and not args.no_cpu_baseline:
            gbs, med, runs, desc = cpu_reference_run(args.seqs, args.ctx, 1000, 1, args.cpu_seconds)
            line["cpu_baseline"] = dict(desc, value=round(gbs, 3), unit="GB/s")
        print(json.dumps(line), flush=True)

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def compact(d):
    """The few fields of a secondary workload that the one-line record keeps
    (the full record: `bench.py --only NAME`)."""
    out = {"value": d.get("value"), "unit": d.get("unit")}
    for key in ("ms_per_step", "ms_per_token", "value_cold_l2", "tok_s", "prompts"):
        if key in d:
            out[key] = d[key]
    roof = d.get("roofline") or {}
    if "frac" in roof or "frac_cold" in roof:
        out["frac"] = roof.get("frac", roof.get("frac_cold"))
    if "cpu_reference" in d:
        c = d["cpu_reference"]
        out["cpu_reference"] = {k: c[k] for k in ("value", "unit", "cores", "kind") if k in c}
    return out


def run_config5(args, dev, rank, world, barrier):
    """Headline (config 5): every rank decodes its shard of the sequences
    (one tle_decode_batch launch per step) straight into its block of the
    all-gather buffer, then the in-place NCCL all-gather leaves every
    sequence's output in order on every rank.  The gather follows the decode
    on the same stream: run beside the next step's decode it took SMs from
    that grid (one CTA per SM, rows split in advance) and made the step
    slower, not faster.  Two output buffers alternate, so the end-to-end
    loop can read step i back while step i+1 runs.  Returns the max-over-
    ranks times of the device-timed loop and of the end-to-end loop (pinned
    host inputs in, the gathered output back to rank 0's host)."""
    import torch
    import torch.distributed as dist
    import shard
    import tle
    plan = shard.plan([args.ctx] * args.seqs, world)
    mine = plan.mine(rank)
    n = len(mine)
    max_local = plan.max_local
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    kc = torch.randn((n, 1, args.ctx, KVD), generator=gen, device=dev)
    vc = torch.randn((n, 1, args.ctx, KVD), generator=gen, device=dev)
    caches = [(kc[i], vc[i], args.ctx) for i in range(n)]
    batch = tle.DecodeBatch(caches, [args.ctx - 1] * n, tle.tinyllama_shape(1))
    hq = torch.randn((max_local, QD), generator=torch.Generator().manual_seed(7 + rank)).pin_memory()
    hk = torch.randn((max_local, KVD), generator=torch.Generator().manual_seed(8 + rank)).pin_memory()
    hv = torch.randn((max_local, KVD), generator=torch.Generator().manual_seed(9 + rank)).pin_memory()
    q = hq.to(dev); k = hk.to(dev); v = hv.to(dev)
    gathers = [shard.OutputGather(plan, QD, dev) for _ in range(2)]
    outs = [g.local_slot(rank) if world > 1 else torch.zeros((max_local, QD), device=dev)
            for g in gathers]
    stream = torch.cuda.current_stream(dev)
    done = [torch.cuda.Event() for _ in range(2)]

    def finish(b):
        """Gathers buffer b after its decode (same stream); returns the rows
        in sequence order and the event after which they are complete."""
        res = gathers[b](outs[b]) if world > 1 else outs[b]
        done[b].record(stream)
        return res, done[b]

    def step(i, kev=None):
        b = i & 1
        if kev is not None:
            kev[0].record(stream)
        batch.run(q, k, v, outs[b], 0, rotate=True, stream=stream)
        if kev is not None:
            kev[1].record(stream)
        finish(b)

    for i in range(max(3, args.warmup)):
        step(i)
    barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    barrier()
    ev[0].record(stream)
    for i in range(args.steps):
        step(i, kev[i])
    ev[1].record(stream)
    barrier()
    t_ms = ev[0].elapsed_time(ev[1])
    k_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)

    # ---- end to end through the public API with host buffers ----
    # Every step copies its q/k/v from pinned host memory and uploads the
    # per-step descriptor (positions) on a copy stream, double-buffered (two
    # DecodeBatch objects over the same caches), so step i+1's inputs move
    # while step i computes and no copy sits between two decode launches;
    # then it decodes, gathers, and rank 0 reads the gathered output of all
    # sequences back to the host.
    batches = [batch, tle.DecodeBatch(caches, [args.ctx - 1] * n, tle.tinyllama_shape(1))]
    cstream = torch.cuda.Stream(dev)     # host -> device
    dstream = torch.cuda.Stream(dev)     # device -> host (rank 0)
    qb = [torch.empty_like(q) for _ in range(2)]
    kb = [torch.empty_like(k) for _ in range(2)]
    vb = [torch.empty_like(v) for _ in range(2)]
    hout = [torch.zeros((args.seqs, QD)).pin_memory() for _ in range(2)]
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]
    in_free = [None, None]
    out_free = [None, None]
    barrier()
    e2 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    e2[0].record(stream)
    cstream.wait_event(e2[0])
    dstream.wait_event(e2[0])
    for i in range(args.steps):
        b = i & 1
        with torch.cuda.stream(cstream):
            if in_free[b] is not None:
                cstream.wait_event(in_free[b])        # step i-2 finished reading buffers b
            qb[b].copy_(hq, non_blocking=True)
            kb[b].copy_(hk, non_blocking=True)
            vb[b].copy_(hv, non_blocking=True)
            batches[b].upload(cstream)                # per-step descriptor (positions)
            h2d_done[b].record(cstream)
        stream.wait_event(h2d_done[b])
        if out_free[b] is not None:
            stream.wait_event(out_free[b])            # outs[b] gathered and read back
        batches[b].run(qb[b], kb[b], vb[b], outs[b], 0, rotate=True, stream=stream)
        comp_done[b].record(stream)
        in_free[b] = comp_done[b]
        res, ready = finish(b)
        if rank == 0:
            with torch.cuda.stream(dstream):
                dstream.wait_event(ready)
                hout[b].copy_(res, non_blocking=True)
                d2h_done[b].record(dstream)
            out_free[b] = d2h_done[b]
        else:
            out_free[b] = ready
    stream.wait_stream(cstream)
    stream.wait_stream(dstream)
    e2[1].record(stream)
    barrier()
    e2e_ms = e2[0].elapsed_time(e2[1])
    h2d = int(hq[:n].numel() * 4 + hk[:n].numel() * 4 + hv[:n].numel() * 4 + batch.desc_bytes)
    vals = torch.tensor([t_ms, e2e_ms, k_ms, h2d], dtype=torch.float64, device=dev)
    if world > 1:
        mx = vals[:3].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = vals[3:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        vals = torch.cat([mx, tot])
    t_ms, e2e_ms, k_ms, h2d_total = [float(x) for x in vals.cpu()]
    return {"t_ms": t_ms, "e2e_ms": e2e_ms, "kernel_ms": k_ms, "local_bytes": n * args.ctx * ROW_BYTES,
            "h2d_bytes": int(h2d_total), "d2h_bytes": int(args.seqs * QD * 4)}


def run_config4_sharded(dev, rank, world, barrier, peaks, steps=20, warmup=3, n_layers=22):
    """Config 4 at the job's GPU count: the 64 ragged sequences (lengths
    U[128, 2048], seeded) LPT-partitioned over the ranks; a step is one decode
    token for every sequence through all 22 layers (each rank: one CUDA graph
    of its 22 tle_decode_batch launches, TLE_DECODE_KV_READY) and one NCCL
    all-gather of every layer's outputs, reordered into sequence order.
    Time = max over ranks."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import shard
    import tle
    lengths = np.random.default_rng(4).integers(128, 2049, 64)
    plan = shard.plan([int(x) for x in lengths], world)
    mine = plan.mine(rank)
    n, ml = len(mine), plan.max_local
    g = torch.Generator(device=dev).manual_seed(44 + rank)
    caches = [(torch.randn((n_layers, int(lengths[s]), KVD), generator=g, device=dev),
               torch.randn((n_layers, int(lengths[s]), KVD), generator=g, device=dev), int(lengths[s]))
              for s in mine]
    batch = tle.DecodeBatch(caches, [int(lengths[s]) - 1 for s in mine], tle.tinyllama_shape(n_layers))
    q = torch.randn((n, QD), generator=g, device=dev)
    k = torch.randn((n, KVD), generator=g, device=dev)
    v = torch.randn((n, KVD), generator=g, device=dev)
    outs = [torch.zeros((n_layers, ml, QD), device=dev) for _ in range(2)]
    gbufs = [torch.zeros((world, n_layers, ml, QD), device=dev) for _ in range(2)]
    # row of (layer l, sequence s) in a gathered buffer viewed as [world*22*ml][QD]
    local_idx = {s: i for r in range(world) for i, s in enumerate(plan.local[r])}
    index = torch.tensor([(plan.owner[s] * n_layers + l) * ml + local_idx[s]
                          for l in range(n_layers) for s in range(len(lengths))],
                         dtype=torch.long, device=dev)
    stream = torch.cuda.current_stream(dev)
    graphs = []
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    for b in range(2):
        def layers(st, b=b):
            for l in range(n_layers):
                batch.run(q, k, v, outs[b][l], l, True, st, kv_ready=True)
        with torch.cuda.stream(side):
            layers(side)
        torch.cuda.synchronize(dev)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(gr, stream=side):
                layers(side)
        graphs.append(gr)
    torch.cuda.synchronize(dev)

    def step(i):
        b = i & 1
        graphs[b].replay()
        if world > 1:
            dist.all_gather_into_tensor(gbufs[b], outs[b])
            gbufs[b].view(-1, QD).index_select(0, index)

    for i in range(warmup):
        step(i)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for i in range(steps):
        step(i)
    e1.record(stream)
    barrier()
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    del graphs
    kv_bytes = n_layers * int(lengths.sum()) * ROW_BYTES
    gbs = kv_bytes / (ms / 1e3) / 1e9
    return {"value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "tok_s": round(64 / (ms / 1e3), 1), "n_gpus": world,
            "frac_per_gpu": round(gbs / world / peaks["hbm_gbs"], 4)}


def _time_steps(fn, steps, warmup, stream):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _time_graph(fn, steps, warmup, dev):
    """Captures one step (fn) in a CUDA graph and times `steps` replays with
    CUDA events (removes the per-launch host cost of the Python plumbing)."""
    import torch
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            fn(side)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / steps


def measure_prefill(dev, peaks, steps=10, warmup=3):
    """Config 3: causal prefill S=2048 (32 q / 4 kv heads, hd 64) for each of
    22 layers; a step is the 22 tle_prefill calls (distinct per-layer inputs,
    440 MB > L2).  FLOPs are algorithmic: 4*64*32*S(S+1)/2 per layer."""
    import torch
    import tle
    S, n_layers = 2048, 22
    g = torch.Generator(device=dev).manual_seed(33)
    q = torch.randn((n_layers, S, QD), generator=g, device=dev)
    k = torch.randn((n_layers, S, KVD), generator=g, device=dev)
    v = torch.randn((n_layers, S, KVD), generator=g, device=dev)
    kc = torch.zeros((n_layers, S, KVD), device=dev)
    vc = torch.zeros_like(kc)
    out = torch.zeros((S, QD), device=dev)
    shape = tle.tinyllama_shape(n_layers)
    ws = tle.prefill_workspace(S, 0, shape)
    stream = torch.cuda.current_stream(dev)

    def step(st=stream):
        for l in range(n_layers):
            tle.prefill(out, q[l], k[l], v[l], kc, vc, l, 0, S, shape, ws, st)

    ms_eager = _time_steps(step, steps, warmup, stream)
    ms = _time_graph(step, steps, warmup, dev)
    flops = n_layers * 4.0 * HD * NH * S * (S + 1) / 2
    tflops = flops / (ms / 1e3) / 1e12
    cpu = cpu_prefill_reference(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), flops)
    return {"workload": "config3: causal prefill S=2048, 22 layers per step (CUDA graph of the 22 "
                        "tle_prefill calls), bf16 tcgen05 MMA, fp32 softmax, rope+append prep kernel",
            "metric": "prefill attn TFLOP/s", "value": round(tflops, 1), "unit": "TFLOP/s",
            "ms_per_step": round(ms, 4), "ms_per_layer": round(ms / n_layers, 4),
            "ms_per_step_eager": round(ms_eager, 4),
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(tflops / peaks["bf16_tflops"], 4),
                         "peak_source": peaks["source"] + ", burst"},
            "cpu_reference": cpu,
            "gpu_launches": 2 * n_layers * steps}


def _ref_lib():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    kind = "reference" if oracle.have_reference() else "port"
    return (oracle.reference() if kind == "reference" else oracle.port()), kind


def cpu_prefill_reference(q, k, v, flops_22):
    """Config 3 on the host: the reference's own token-at-a-time prefill
    (generate.cpp:56-59: rope + attention for pos 0..2047, oracle/_ref) of
    whole layers, one layer per host thread (ctypes releases the GIL), as
    many layers at once as there are cores up to 22; the 22-layer time is
    extrapolated linearly in layers."""
    import numpy as np
    lib, kind = _ref_lib()
    n_layers, S = q.shape[0], q.shape[1]
    cores = os.cpu_count() or 1
    run = max(1, min(n_layers, cores))
    bufs = []
    for l in range(run):
        bufs.append((np.zeros((S, QD), np.float32), q[l].copy(), k[l].copy(), v[l].copy(),
                     np.zeros((1, S, KVD), np.float32), np.zeros((1, S, KVD), np.float32)))

    def one(b):
        out, qq, kk, vv, kc, vc = b
        lib.prefill(out, qq, kk, vv, kc, vc, 0, 0, S)

    t0 = time.perf_counter()
    th = [threading.Thread(target=one, args=(b,)) for b in bufs]
    for t in th:
        t.start()
    for t in th:
        t.join()
    dt = (time.perf_counter() - t0) * n_layers / run
    return {"value": round(flops_22 / dt / 1e12, 6), "unit": "TFLOP/s", "kind": kind, "cores": run,
            "ms_per_step": round(dt * 1e3, 1),
            "sample": "%d of 22 layers, one per thread, S=2048 token loop each; x22/%d" % (run, run)}


def measure_config4(dev, peaks, steps=20, warmup=3):
    """Config 4: 64 sequences, attended lengths U[128, 2048] (seeded), 22-layer
    fp32 caches; a step is one decode token for every sequence = 22
    tle_decode_batch calls (3.5 GB of KV, > L2).  Timed twice: with
    TLE_DECODE_KV_READY (the headline of this line: each call's previous
    kernel is the decode of another layer, which writes none of the rows the
    call reads, as the QKV projection before attention does in a forward
    pass), and in strict order (every read after the previous kernel)."""
    import numpy as np
    import torch
    import tle
    n_layers = 22
    lengths = np.random.default_rng(4).integers(128, 2049, 64)
    g = torch.Generator(device=dev).manual_seed(44)
    caches = []
    for L in lengths:
        caches.append((torch.randn((n_layers, int(L), KVD), generator=g, device=dev),
                       torch.randn((n_layers, int(L), KVD), generator=g, device=dev), int(L)))
    batch = tle.DecodeBatch(caches, [int(L) - 1 for L in lengths], tle.tinyllama_shape(n_layers))
    q = torch.randn((64, QD), generator=g, device=dev)
    k = torch.randn((64, KVD), generator=g, device=dev)
    v = torch.randn((64, KVD), generator=g, device=dev)
    out = torch.zeros((64, QD), device=dev)
    stream = torch.cuda.current_stream(dev)

    def stepper(kv_ready):
        def step(st=stream):
            for l in range(n_layers):
                batch.run(q, k, v, out, l, True, st, kv_ready=kv_ready)
        return step

    ms_eager = _time_steps(stepper(False), steps, warmup, stream)
    ms_strict = _time_graph(stepper(False), steps, warmup, dev)
    ms = _time_graph(stepper(True), steps, warmup, dev)
    kv_bytes = n_layers * int(lengths.sum()) * ROW_BYTES
    gbs = kv_bytes / (ms / 1e3) / 1e9
    gbs_strict = kv_bytes / (ms_strict / 1e3) / 1e9
    cpu = cpu_config4_reference(lengths, n_layers)
    return {"workload": "config4: 64 seqs, lengths U[128,2048] (sum %d), 22 layers per step "
                        "(CUDA graph of the 22 tle_decode_batch calls, TLE_DECODE_KV_READY)"
                        % int(lengths.sum()),
            "metric": "decode-attn KV GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "tok_s": round(64 / (ms / 1e3), 1), "ms_per_step": round(ms, 4),
            "strict_order": {"ms_per_step": round(ms_strict, 4), "value": round(gbs_strict, 1),
                             "frac": round(gbs_strict / peaks["hbm_gbs"], 4)},
            "ms_per_step_eager_strict": round(ms_eager, 4),
            "n_ctas": batch.n_ctas,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4)},
            "cpu_reference": cpu,
            "gpu_launches": n_layers * steps}


def cpu_config4_reference(lengths, n_layers, sample_layers=2):
    """Config 4 on the host: the reference's rope + attention (oracle/_ref)
    for all 64 sequences, spread over every host thread (independent
    sequences), for `sample_layers` of the 22 layers (the 3.1 GB of fp32
    cache for all layers is not built on the host); the 22-layer time is
    extrapolated linearly in layers."""
    import numpy as np
    lib, kind = _ref_lib()
    cores = os.cpu_count() or 1
    n = len(lengths)
    rng = np.random.default_rng(404)
    kcs = [rng.standard_normal((sample_layers, int(L), KVD), dtype=np.float32) for L in lengths]
    vcs = [rng.standard_normal((sample_layers, int(L), KVD), dtype=np.float32) for L in lengths]
    q = rng.standard_normal((n, QD), dtype=np.float32)
    k = rng.standard_normal((n, KVD), dtype=np.float32)
    v = rng.standard_normal((n, KVD), dtype=np.float32)
    out = np.zeros((n, QD), np.float32)
    lens = [int(L) for L in lengths]
    pos = [L - 1 for L in lens]
    t0 = time.perf_counter()
    for l in range(sample_layers):
        lib.decode_batch(kcs, vcs, lens, pos, q.copy(), k.copy(), v, out, l, n_threads=min(cores, n))
    dt = (time.perf_counter() - t0) * n_layers / sample_layers
    kv_bytes = n_layers * int(np.sum(lengths)) * ROW_BYTES
    return {"value": round(kv_bytes / dt / 1e9, 3), "unit": "GB/s", "kind": kind, "cores": min(cores, n),
            "ms_per_step": round(dt * 1e3, 1),
            "sample": "64 sequences x %d of 22 layers, sequences over %d threads; x22/%d"
                      % (sample_layers, min(cores, n), sample_layers)}


def _paged_setup(dev, lengths, n_layers, page_rows, seed, shuffle=True):
    """Page pools holding every sequence's rows (N(0,1)), pages handed out in
    a shuffled order (or in pool order), and the PagedDecodeBatch over them."""
    import numpy as np
    import torch
    import tle
    need = [-(-int(L) // page_rows) for L in lengths]
    cache = tle.PagedKVCache(sum(need), page_rows, tle.tinyllama_shape(n_layers), device=dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    cache.key_pool.normal_(generator=g)
    cache.value_pool.normal_(generator=g)
    if shuffle:
        cache._free = [int(i) for i in np.random.default_rng(seed).permutation(sum(need))]
    tables = [cache.table(cache.alloc(m)) for m in need]
    batch = tle.PagedDecodeBatch(cache, tables, [int(L) - 1 for L in lengths])
    n = len(lengths)
    q = torch.randn((n, QD), generator=g, device=dev)
    k = torch.randn((n, KVD), generator=g, device=dev)
    v = torch.randn((n, KVD), generator=g, device=dev)
    out = torch.zeros((n, QD), device=dev)
    return cache, batch, q, k, v, out


def measure_paged5(dev, peaks, steps=10, warmup=3, page_rows=256, shuffle=True):
    """Config 5 on a paged cache: 256 sequences x 32768 rows in 256-row pages
    of one shared pool (shuffled), one tle_decode_batch_paged call per step
    (17.2 GB of K+V, > L2)."""
    import torch
    lengths = [CTX] * N_SEQS
    cache, batch, q, k, v, out = _paged_setup(dev, lengths, 1, page_rows, 55, shuffle)
    stream = torch.cuda.current_stream(dev)
    ms = _time_steps(lambda: batch.run(q, k, v, out, 0, True, stream), steps, warmup, stream)
    kv_bytes = N_SEQS * CTX * ROW_BYTES
    gbs = kv_bytes / (ms / 1e3) / 1e9
    del cache
    return {"workload": "config5 paged: 256 seqs x 32768 rows, %d-row pages in one shuffled pool, "
                        "1 layer per step (tle_decode_batch_paged)" % page_rows,
            "metric": "decode-attn KV GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "ms_per_step": round(ms, 4), "n_ctas": batch.n_ctas,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4)},
            "gpu_launches": steps}


def measure_bf16_5(dev, peaks, steps=10, warmup=3, n_seqs=N_SEQS, ctx=CTX):
    """Config 5's shape over bf16 caches: 256 sequences x 32768 rows, one
    tle_decode_batch_bf16 call per step (8.6 GB of K+V, > L2).  The KV bytes
    are the bf16 bytes read; tok/s counts 22 layers per token as the fp32
    line does."""
    import torch
    import tle
    g = torch.Generator(device=dev).manual_seed(56)
    caches = []
    for _ in range(n_seqs):
        kc = torch.randn((1, ctx, KVD), generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn((1, ctx, KVD), generator=g, device=dev).to(torch.bfloat16)
        caches.append((kc, vc, ctx))
    batch = tle.DecodeBatchBf16(caches, [ctx - 1] * n_seqs, tle.tinyllama_shape(1))
    q = torch.randn((n_seqs, QD), generator=g, device=dev)
    k = torch.randn((n_seqs, KVD), generator=g, device=dev)
    v = torch.randn((n_seqs, KVD), generator=g, device=dev)
    out = torch.zeros((n_seqs, QD), device=dev)
    stream = torch.cuda.current_stream(dev)
    ms = _time_steps(lambda: batch.run(q, k, v, out, 0, True, stream), steps, warmup, stream)
    kv_bytes = n_seqs * ctx * KVD * 2 * 2
    gbs = kv_bytes / (ms / 1e3) / 1e9
    assert tle.device_error() == 0
    del caches
    return {"workload": "config5 shape, bf16 KV: %d seqs x %d rows, 1 layer per step "
                        "(tle_decode_batch_bf16, mma.sync m16n8k16)" % (n_seqs, ctx),
            "metric": "decode-attn KV GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "ms_per_step": round(ms, 4), "tok_s_attn_22_layers": round(n_seqs / (22 * ms / 1e3), 1),
            "dtype": "bf16 KV, bf16 q and P on the tensor pipe, fp32 accumulation",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4)},
            "gpu_launches": 2 * steps}


def measure_paged4(dev, peaks, steps=20, warmup=3, page_rows=256, shuffle=True):
    """Config 4 on a paged cache: 64 sequences, lengths U[128, 2048] (the same
    seeded lengths as the contiguous line), 22 layers, 256-row pages; a step
    is 22 tle_decode_batch_paged calls in one CUDA graph, timed with
    TLE_DECODE_KV_READY and in strict order like the contiguous line."""
    import numpy as np
    import torch
    n_layers = 22
    lengths = np.random.default_rng(4).integers(128, 2049, 64)
    cache, batch, q, k, v, out = _paged_setup(dev, lengths, n_layers, page_rows, 44, shuffle)
    stream = torch.cuda.current_stream(dev)

    def stepper(kv_ready):
        def step(st=stream):
            for l in range(n_layers):
                batch.run(q, k, v, out, l, True, st, kv_ready=kv_ready)
        return step

    ms_strict = _time_graph(stepper(False), steps, warmup, dev)
    ms = _time_graph(stepper(True), steps, warmup, dev)
    kv_bytes = n_layers * int(lengths.sum()) * ROW_BYTES
    gbs = kv_bytes / (ms / 1e3) / 1e9
    del cache
    return {"workload": "config4 paged: 64 seqs, lengths U[128,2048] (sum %d), 22 layers per step, "
                        "%d-row pages (CUDA graph of the 22 tle_decode_batch_paged calls, "
                        "TLE_DECODE_KV_READY)" % (int(lengths.sum()), page_rows),
            "metric": "decode-attn KV GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "tok_s": round(64 / (ms / 1e3), 1), "ms_per_step": round(ms, 4),
            "strict_order": {"ms_per_step": round(ms_strict, 4),
                             "value": round(kv_bytes / (ms_strict / 1e3) / 1e9, 1)},
            "n_ctas": batch.n_ctas,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4)},
            "gpu_launches": n_layers * steps}


def cpu_forward_reference(model, tokens, n_threads):
    """The reference's forward() (its own ops.cpp, composed in forward.cpp's
    order by oracle/_ref) on the host: seconds per token over `tokens`."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    kind = "reference" if oracle.have_reference() else "port"
    lib = oracle.reference() if kind == "reference" else oracle.port()
    if kind == "reference":
        lib._fn("set_num_threads", [ctypes_int()])(n_threads)
    hf = oracle.HostForward(model)
    t0 = time.perf_counter()
    for pos, tok in enumerate(tokens):
        lib.forward(hf, int(tok), pos)
    dt = (time.perf_counter() - t0) / len(tokens)
    if kind == "reference":
        lib._fn("set_num_threads", [ctypes_int()])(1)
    return dt, kind


def ctypes_int():
    import ctypes
    return ctypes.c_int


def measure_config2(dev, peaks, steps=1, warmup=1, prompt=128, gen=256, seed=2, cpu_tokens=3):
    """Config 2: end-to-end greedy generation on the device, TinyLlama-1.1B
    shapes with random Q4_0 weights (LM head Q4_0, fp16 embedding table,
    RMSNorm weights 1.0): a 128-token prompt of random ids fed token by token
    (as generate.cpp:56-59 does), then 256 tokens, each the argmax of the
    previous logits, sampled on the device.  Every position runs as one
    CUDA graph (embedding, the 22 layers [RMSNorm+q/k/v, rope+attention,
    output projection+residual, RMSNorm+SwiGLU, down projection+residual] in
    one persistent launch, RMSNorm+LM head, argmax) captured once; the token of step t+1 never leaves the
    device.  Timed with CUDA events over whole generations."""
    import numpy as np
    import torch
    import synth
    import tle
    n_ctx = prompt + gen
    m = synth.make_model(seed=seed, n_layers=22, wtype=synth.Q4_0, output_type=synth.Q4_0,
                         n_ctx=n_ctx)
    dm = tle.DeviceModel(m, device=dev)
    ds = tle.DeviceState(dm, device=dev)
    ids = np.random.default_rng(seed).integers(0, m.n_vocab, prompt)
    toks = torch.zeros(n_ctx + 1, dtype=torch.int32, device=dev)
    toks[:prompt] = torch.from_numpy(ids.astype(np.int32)).to(dev)
    side = torch.cuda.Stream(dev)
    one_launch = lambda p: tle.forward_layers_one_launch(dm, ds, p)  # noqa: E731

    def step(pos, st):
        tle.forward(dm, ds, toks[pos:pos + 1], pos, st)
        if pos >= prompt - 1 and pos + 1 < n_ctx + 1:
            tle.sample_argmax(ds.logits, toks[pos + 1:pos + 2], st)

    # eager (host-launched) generation, also the warm-up
    side.wait_stream(torch.cuda.current_stream(dev))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with torch.cuda.stream(side):
        for pos in range(n_ctx):
            step(pos, side)
        torch.cuda.synchronize(dev)
        ev[0].record(side)
        for pos in range(n_ctx):
            if pos == prompt:
                ev[1].record(side)
            step(pos, side)
        ev[2].record(side)
    torch.cuda.synchronize(dev)
    eager_prompt_ms, eager_gen_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    first = toks[prompt:].cpu().numpy().copy()

    graphs = []
    with torch.cuda.stream(side):
        for pos in range(n_ctx):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                step(pos, side)
            graphs.append(g)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    for pos in range(n_ctx):          # warm replay
        graphs[pos].replay()
    torch.cuda.synchronize(dev)
    runs = max(1, steps)
    pm, gm = [], []
    for _ in range(runs):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        for pos in range(n_ctx):
            if pos == prompt:
                ev[1].record(stream)
            graphs[pos].replay()
        ev[2].record(stream)
        torch.cuda.synchronize(dev)
        pm.append(ev[0].elapsed_time(ev[1]))
        gm.append(ev[1].elapsed_time(ev[2]))
    same = bool(np.array_equal(first, toks[prompt:].cpu().numpy()))
    if tle.device_error():
        raise RuntimeError("device error during generation")
    prompt_ms, gen_ms = statistics.median(pm), statistics.median(gm)
    wbytes = m.weight_bytes_per_token()
    tok_s = gen / (gen_ms / 1e3)
    gbs = wbytes * tok_s / 1e9
    cores = os.cpu_count() or 1
    cpu_s, kind = cpu_forward_reference(m, ids[:cpu_tokens], cores)
    del graphs
    return {"workload": "config2: TinyLlama-1.1B shapes, random Q4_0 weights (LM head Q4_0, fp16 "
                        "embeddings), 128-token random prompt + 256 greedy tokens, batch 1, "
                        "all on the device (one CUDA graph per position)",
            "metric": "generated tok/s", "value": round(tok_s, 1), "unit": "tok/s",
            "ms_per_token": round(gen_ms / gen, 4), "prompt_ms": round(prompt_ms, 3),
            "prompt_tok_s": round(prompt / (prompt_ms / 1e3), 1),
            "eager_ms_per_token": round(eager_gen_ms / gen, 4),
            "eager_prompt_ms": round(eager_prompt_ms, 3),
            "tokens_identical_eager_vs_graph": same,
            "weight_bytes_per_token": wbytes,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                         "note": "weight bytes per token x tok/s"},
            "cpu_reference": {"kind": kind, "cores": cores, "value": round(1.0 / cpu_s, 3),
                              "unit": "tok/s",
                              "sample": "%d prompt tokens through the 22-layer model" % cpu_tokens},
            # per generated token: embedding, the layers (one persistent launch,
            # else 22 x (q/k/v, decode, split-K merge, output projection,
            # gate/up, down)), LM head, argmax
            "gpu_launches": sum(3 + (1 if one_launch(p) else 22 * 6) for p in range(prompt, n_ctx)) * runs}


def measure_prompt2(dev, peaks, steps=5, warmup=3, prompts=(128, 2048), seed=2):
    """Config 2's model with its prompt through the batched prompt pass
    (tle_prompt_forward: every product over all prompt tokens on the tensor
    cores, fp16 weight copy made once beforehand) instead of one forward()
    per prompt token; also a 2048-token prompt.  A step is one whole prompt
    pass (embedding, 22 layers, LM head of the last token), timed with CUDA
    events.  Roofline: the fp16 weight copy must be read once per pass
    (HBM) and the products cost 2 x tokens x weights flops (tensor)."""
    import numpy as np
    import torch
    import synth
    import tle
    m = synth.make_model(seed=seed, n_layers=22, wtype=synth.Q4_0, output_type=synth.Q4_0,
                         n_ctx=max(prompts))
    dm = tle.DeviceModel(m, device=dev)
    ds = tle.DeviceState(dm, device=dev)
    pw = tle.PromptWeights(dm)
    stream = torch.cuda.current_stream(dev)
    lin = sum(m.layers[0][n].rows * m.layers[0][n].cols for n in synth.LAYER_WEIGHTS)
    out = {}
    for S in prompts:
        ids = np.random.default_rng(seed + S).integers(0, m.n_vocab, S).astype(np.int32)
        toks = torch.from_numpy(ids).to(dev)
        scratch = tle.prompt_scratch(dm, S, 0, dev)
        ms = _time_steps(lambda: tle.prompt_forward(dm, ds, pw, toks, 0, scratch, stream),
                         steps, warmup, stream)
        if tle.device_error():
            raise RuntimeError("device error during the prompt pass")
        flops = 22 * (2.0 * S * lin + 4.0 * 64 * 32 * S * (S + 1) / 2)
        wbytes = 22 * 2 * lin
        out[str(S)] = {"ms": round(ms, 4), "tok_s": round(S / (ms / 1e3), 1),
                       "tflops": round(flops / (ms / 1e3) / 1e12, 2),
                       "frac_tensor": round(flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"], 4),
                       "fp16_weight_gbs": round(wbytes / (ms / 1e3) / 1e9, 1),
                       "frac_hbm": round(wbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4)}
    per_pass = 1 + 22 * 9 + 1
    cores = os.cpu_count() or 1
    cpu_s, kind = cpu_forward_reference(m, np.random.default_rng(seed).integers(0, m.n_vocab, 3), cores)
    first, last = out[str(prompts[0])], out[str(prompts[-1])]
    return {"workload": "config2 model (TinyLlama-1.1B shapes, random Q4_0) prompt through "
                        "tle_prompt_forward, %s tokens" % "/".join(str(p) for p in prompts),
            "metric": "prompt tok/s", "value": first["tok_s"], "unit": "tok/s",
            "dtype": "f16 products, fp32 accumulation", "prompts": out,
            "roofline": {"bound": "hbm", "achieved": first["fp16_weight_gbs"], "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": first["frac_hbm"],
                         "note": "%d tokens: the fp16 weight copy read once per pass" % prompts[0]},
            "roofline_long": {"bound": "tensor", "achieved": last["tflops"], "peak": peaks["bf16_tflops"],
                              "unit": "TFLOP/s", "frac": last["frac_tensor"],
                              "note": "%d tokens: products + causal attention flops" % prompts[-1]},
            "cpu_reference": {"kind": kind, "cores": cores, "value": round(1.0 / cpu_s, 3), "unit": "tok/s",
                              "sample": "the reference's prompt loop (one forward() per token, "
                                        "generate.cpp:56-59), 3 tokens of the 22-layer model"},
            "gpu_launches": per_pass * steps * len(prompts)}


def measure_config1(dev, peaks, steps=50, warmup=5, copies=8):
    """Config 1: one sequence, 22 layers, cache capacity 512, rows 0..510
    cached, the new token at pos 511 (L = 512); a step is the 22
    tle_rope_attention calls of one decode token (forward.cpp:192-208 per
    layer), 23.07 MB of K+V.  That fits L2, so the warm number is latency-
    bound; the cold variant rotates `copies` cache copies (184 MB > L2)."""
    import torch
    import tle
    n_layers, n_ctx, pos = 22, 512, 511
    shape = tle.tinyllama_shape(n_layers)
    g = torch.Generator(device=dev).manual_seed(11)
    caches = [(torch.randn((n_layers, n_ctx, KVD), generator=g, device=dev),
               torch.randn((n_layers, n_ctx, KVD), generator=g, device=dev)) for _ in range(copies)]
    q = torch.randn(QD, generator=g, device=dev)
    k = torch.randn(KVD, generator=g, device=dev)
    v = torch.randn(KVD, generator=g, device=dev)
    out = torch.zeros(QD, device=dev)
    ws = tle.attention_workspace(shape, n_ctx)

    def step_on(c, kv_ready=True):
        # kv_ready (TLE_DECODE_KV_READY): each call's previous kernel is the
        # previous layer's call, which writes only that layer's row pos, so
        # this layer's cached rows stream while it finishes (in a forward
        # pass the previous kernel is the q/k/v projection, same contract)
        def step(st):
            kc, vc = caches[c]
            for l in range(n_layers):
                tle.rope_attention(out, q, k, v, kc, vc, l, pos, n_ctx, shape, ws, st,
                                   kv_ready=kv_ready)
        return step

    ms_strict = _time_graph(step_on(0, kv_ready=False), steps, warmup, dev)
    ms_warm = _time_graph(step_on(0), steps, warmup, dev)
    # cold: one captured graph per cache copy, replayed in rotation
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graphs = []
    with torch.cuda.stream(side):
        for c in range(copies):
            step_on(c)(side)
    torch.cuda.synchronize(dev)
    for c in range(copies):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(gr, stream=side):
                step_on(c)(side)
        graphs.append(gr)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    for i in range(copies):
        graphs[i].replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        graphs[i % copies].replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_cold = e0.elapsed_time(e1) / steps
    kv_bytes = n_layers * (pos + 1) * ROW_BYTES
    # the reference's own per-token cost: its rope+attention (oracle/_ref,
    # src/ops.cpp compiled unmodified) for the 22 layers on one host thread
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    kind = "reference" if oracle.have_reference() else "port"
    lib = oracle.reference() if kind == "reference" else oracle.port()
    kc_h, vc_h = caches[0][0].cpu().numpy(), caches[0][1].cpu().numpy()
    q_h, k_h, v_h = q.cpu().numpy()[None], k.cpu().numpy()[None], v.cpu().numpy()[None]
    out_h = np.zeros((1, QD), np.float32)
    ref_times = []
    for _ in range(3):
        t0 = time.perf_counter()
        for l in range(n_layers):
            lib.decode_batch([kc_h], [vc_h], [n_ctx], [pos], q_h.copy(), k_h.copy(), v_h, out_h, l,
                             n_threads=1)
        ref_times.append(time.perf_counter() - t0)
    ref_us = statistics.median(ref_times) * 1e6
    return {"workload": "config1: 1 sequence, 22 layers, L=512 (pos 511, capacity 512); a step is "
                        "the 22 tle_rope_attention calls of one token (CUDA graph)",
            "metric": "decode token latency (22 layers)", "unit": "us", "higher_is_better": False,
            "value": round(ms_warm * 1e3, 2), "value_cold_l2": round(ms_cold * 1e3, 2),
            "value_strict_order": round(ms_strict * 1e3, 2),
            "kv_ready": "value and value_cold_l2 use TLE_DECODE_KV_READY (rows stream before the "
                        "wait on the previous kernel); value_strict_order waits first",
            "kv_gbs_warm": round(kv_bytes / (ms_warm / 1e3) / 1e9, 1),
            "kv_gbs_cold": round(kv_bytes / (ms_cold / 1e3) / 1e9, 1),
            "cold_l2": "%d cache copies rotated (%.0f MB > 126 MB L2)" % (copies, copies * 2 * n_layers * n_ctx * KVD * 4 / 1e6),
            "roofline": {"bound": "latency (23 MB of K+V fits L2)",
                         "achieved_cold_gbs": round(kv_bytes / (ms_cold / 1e3) / 1e9, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac_cold": round(kv_bytes / (ms_cold / 1e3) / 1e9 / peaks["hbm_gbs"], 4)},
            "cpu_reference": {"kind": kind, "cores": 1, "value": round(ref_us, 1), "unit": "us",
                              "sample": "22 layers of rope+attention at L=512, one host thread, "
                                        "median of 3 tokens"},
            "gpu_launches": 3 * n_layers * steps}


def measure_ctxsplit(args, dev, rank, world, local):
    """One sequence of --ctx-rows rows split by rows over the ranks
    (shard.ContextSplitDecode): a step is rope of the new q/k at the global
    position, each rank's tle_attention_lse over its shard, the NCCL
    all-gather of the (out, lse) pairs and tle_merge_lse.  Prints one JSON
    line (rank 0); time is the max over ranks."""
    import torch
    import torch.distributed as dist
    import tle
    import shard
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    L = args.ctx_rows
    pos = L - 1
    plan = shard.context_plan(L, world)
    n_loc = plan.local_rows(rank)
    g = torch.Generator(device=dev).manual_seed(500 + rank)
    kc = torch.randn((1, n_loc + 1, KVD), generator=g, device=dev)
    vc = torch.randn((1, n_loc + 1, KVD), generator=g, device=dev)
    g0 = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn(QD, generator=g0, device=dev)
    k = torch.randn(KVD, generator=g0, device=dev)
    v = torch.randn(KVD, generator=g0, device=dev)
    qw, kw = q.clone(), k.clone()
    shape = tle.tinyllama_shape(1)
    cs = shard.ContextSplitDecode(plan, rank, kc, vc, n_loc + 1, shape, dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        qw.copy_(q)
        kw.copy_(k)
        tle.rope(qw, kw, pos)
        return cs.step(qw, kw, v, 0, pos)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    if rank == 0:
        peaks = load_peaks()
        gbs = L * ROW_BYTES / (ms / 1e3) / 1e9
        print(json.dumps({"metric": "ctx-split decode KV GB/s", "value": round(gbs, 1), "unit": "GB/s",
                          "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
                          "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
                          "dtype": "f32", "data": "synthetic N(0,1) fp32, seeded",
                          "config": {"workload": "1 sequence x %d rows split by rows over %d GPU(s), "
                                                 "1 layer per step (rope + tle_attention_lse per shard + "
                                                 "NCCL all-gather of (out, lse) + tle_merge_lse)" % (L, world)},
                          "per_gpu_frac_hbm": round(gbs / world / peaks["hbm_gbs"], 4),
                          "gpu_launches": 4 * args.steps}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured (MEASURED_PEAKS.json)"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def profile_traffic(local_bytes):
    """DRAM bytes per launch from the committed ncu summary (scaled to this
    launch's rows), or None when no capture has been summarised."""
    p = os.path.join(ROOT, "profiles", "decode_kernel_traffic.txt")
    try:
        for ln in open(p):
            if ln.startswith("dram_bytes_per_algorithmic_byte:"):
                return int(float(ln.split(":", 1)[1]) * local_bytes)
    except OSError:
        pass
    return None


if __name__ == "__main__":
    main()
