"""Benchmark of the DeepSeek-V4.1 decode monokernel path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--rows M] [--impl ours|reference]

Workload: BASELINE config 2 -- one full-size synthetic MoE decode layer (hidden 4096, 64 heads
of 512 + 64 latent dims, 256 experts top-8 + 1 shared, expert intermediate 2048, MXFP4
experts, FP8 block-scaled projections) at KV context 8192, random-init (seed 1). A step is
one decoder layer (K1 + K2, CUDA-graph replayed) over M decode rows; steps alternate
between distinct layer copies and their caches, so no step reads weights another step left
in L2 (each step also reads more than L2 holds). ``value`` = decode tokens/s of the layer
(M rows / layer time, summed over ranks); the sweep over M = 1, 4, 16, 48 and the per-M
fraction of the HBM weight-streaming roofline are in ``config``.

With N > 1 (torchrun), the same layer runs tensor-parallel over the N ranks (TP = N: heads,
wo_a groups, expert and shared-expert intermediates sharded; wqkv_a, the router and the KV
cache replicated), with both all-reduces in-kernel through CUDA IPC peer regions (strong
scaling: the same M rows at every N; ``value`` = M / the max-over-ranks layer time). The
NCCL variant of the all-reduces (all-gather + rank-order sum) and the exchanges alone are
timed beside it, at the headline M.

``config.configs`` carries the other BASELINE configs as sections: 3 (K2i -> top-2048 -> the
sparse layer), 5 (the verify step's pieces) and 4 (a 40-layer decode step, 16 rows at context
16384, chained layers in one CUDA graph; at N > 1 with the NCCL variant beside it).

``--impl reference`` times the reference path's CPU restatement (the repository's oracle:
torch fp32/fp64 on the host cores, all threads) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "decode tokens/s (one config-2 MoE decode layer, K1 + K2)"
UNIT = "tokens/s"
# DRAM bytes (read + write) of the routed-expert stage's two expert_tc_kernel launches per expert
# of the routing union, from one ncu capture (M = 48, ctx 2048, one layer, union 199: gate/up
# 1.774859 GB + 27.11 MB, down 0.887746 GB + 14.77 MB).
EXPERT_DRAM_BYTES_PER_UNIT = (1.774859e9 + 27.109376e6 + 0.887746e9 + 14.774784e6) / 199


REF_SAMPLE_ROWS = 4  # rows of the step's M the reference arm's CPU oracle runs a step
TARGET_LAYERS = 40  # config 5's target model depth
DRAFT_WINDOW = 128  # the draft's attention window (the reference's WINDOW, draft.py:30)


def workload_config(args, world):
    """The workload both arms report, identical for the GPU path and the reference arm (what was
    measured goes to ``detail``)."""
    return {"workload": f"config2: one MoE decode layer (K1 + K2), {args.rows} rows, ctx {args.ctx}",
            "rows": args.rows, "ctx": args.ctx, "tp": world, "parallelism": f"tp{world}",
            "allreduce": "fused in-kernel LL peer stores, rank-order fp32 sum" if world > 1 else "none (tp1)",
            "l2": f"inputs larger than L2: steps alternate {args.layers} layer copies of > 126 MB each"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--rows", type=int, default=48, help="headline decode rows M")
    ap.add_argument("--sweep", default="1,4,16,48")
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--layers", type=int, default=2, help="distinct layer copies stepped round-robin")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--skip-configs", action="store_true", help="skip the config-3 / config-5 sections")
    return ap.parse_args()


# ---------------------------------------------------------------- distributed plumbing
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- clocks during the timed region
class Clocks:
    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.QUERY}",
                                       "--format=csv,noheader,nounits", "-lms", "20"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        # nvidia-smi takes a while to start: wait (at most 3 s) for its first sample, so the
        # samples cover the timed region that follows
        t0 = time.time()
        while self.p is not None and time.time() - t0 < 3.0:
            self.f.flush()
            if os.path.getsize(self.f.name) > 0:
                break
            time.sleep(0.02)

    def mark(self) -> None:
        """The timed region starts: samples before this are dropped."""
        import datetime
        self.t0 = datetime.datetime.now()

    def stop(self) -> dict:
        import datetime
        t1 = datetime.datetime.now()
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows, timed = [], []
        with open(self.f.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 10:
                    rows.append(parts[1:])
                    try:
                        ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                    except ValueError:
                        continue
                    if getattr(self, "t0", None) is not None and self.t0 <= ts <= t1:
                        timed.append(parts[1:])
        os.unlink(self.f.name)
        window = "timed region" if timed else "whole sampler run (no sample fell inside the timed region)"
        rows = timed or rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "window": window}


# ---------------------------------------------------------------- the CPU reference path
def cpu_layer(w, step, shape, rows: int) -> float:
    """Time one layer of the oracle (the reference path's CPU restatement) over ``rows`` rows."""
    from oracle import layer as OL
    from oracle import numerics as N
    W = w
    S = {k: (v[:rows] if torch.is_tensor(v) and k not in ("cache",) else v) for k, v in step.items()}
    cache = step["cache"].clone()
    t0 = time.perf_counter()
    cs = W["cos_sin"][S["pos"]]
    cosv, sinv = cs[:, :32], cs[:, 32:]
    QL, D, nope = shape.q_lora, shape.head_dim, shape.nope
    rn, normed, pre, post, comb = OL.seam(S["res"].float(), S["x"].float(), S["post"], S["comb"], S["pre"],
                                          W["hc_attn_fn"], W["hc_attn_scale"], W["hc_attn_base"], W["attn_norm"])
    x8, x8s = N.mxfp8_quant(normed, "vllm")
    qkv = OL.gemv_x8_fp8(x8, x8s, W["wqkv"], W["wqkv_s"])
    _, qx8, qx8s = OL.q_path(qkv[:, :QL], W["q_norm"])
    nb, rb, codes = OL.kv_record(qkv[:, QL:], W["kv_norm"], cosv, sinv, nope)
    data, sc = OL.record_bytes(nb, rb, codes, 8)
    OL.write_records(cache, S["slot"], data, sc, S["blk"])
    q = OL.rope_q(OL.bf(OL.gemv_x8_fp8(qx8, qx8s, W["wqb"], W["wqb_s"])).view(rows, -1, D), cosv, sinv, nope)
    kt, klen = OL.key_table(S["slot"], S["swa_idx"], S["swa_lens"], None, torch.zeros(rows, dtype=torch.int32),
                            S["swa_idx"].shape[1], 0)
    xo = OL.attention(q, kt, klen, cache, S["blk"], None, 1, W["sink"], cosv, sinv, nope, shape.rope, 8)
    _, x8b, x8bs = OL.wo_a(xo, W["woa"], W["woa_s"], shape.groups_local, shape.o_rank)
    attn = OL.all_reduce([OL.wo_b(x8b, x8bs, W["wob"], W["wob_s"])])
    rn2, normed2, *_ = OL.seam(rn, attn, post, comb, pre, W["hc_ffn_fn"], W["hc_ffn_scale"],
                               W["hc_ffn_base"], W["ffn_norm"])
    OL.moe_partial(normed2, W, shape.route, shape.topk)
    return time.perf_counter() - t0


def cpu_inputs(args, shape, rows):
    """Config-2 weights and a ``rows``-row step on the host (drawn on the GPU when there is one,
    with the GPU arm's seeds: the headline step of layer copy 0)."""
    from sgl_amd_mono_b200.deepseek_v41 import synth
    dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    positions = max(args.ctx, 32768) + 8
    w = synth.make_layer(shape, args.seed, dev, positions=positions)
    step = synth.make_step(shape, rows, args.ctx, args.seed + rows, dev)
    cpu = lambda d: {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in d.items()}  # noqa: E731
    return cpu(w), cpu(step)


def sample_rows(step, rows, first):
    """Rows first .. first + rows (mod M) of a step, as a step of their own (the cache shared)."""
    M = step["res"].shape[0]
    idx = torch.tensor([(first + i) % M for i in range(rows)])
    return {k: (v[idx] if torch.is_tensor(v) and k != "cache" and v.dim() > 0 and v.shape[0] == M else v)
            for k, v in step.items()}


def run_reference(args, world, rank):
    from sgl_amd_mono_b200.deepseek_v41.shapes import CONFIG2
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w, step = cpu_inputs(args, CONFIG2, args.rows)
    k = min(REF_SAMPLE_ROWS, args.rows)
    for i in range(args.warmup):
        cpu_layer(w, sample_rows(step, k, k * i), CONFIG2, k)
    ts = [cpu_layer(w, sample_rows(step, k, k * (args.warmup + i)), CONFIG2, k) for i in range(args.steps)]
    t = sum(ts) / len(ts)
    v = k / t
    sample = (f"{k} of the step's {args.rows} decode rows a step (rotating through the rows), the whole layer "
              f"for them (ctx {args.ctx}); the reference path's CPU restatement (torch fp32/fp64), {threads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic (random-init, seeded)",
        "config": workload_config(args, world),
        "detail": {"reference_kind": "port (the repository's CPU oracle of the reference path: the reference's "
                                     "own kernels are FlyDSL for gfx950 and cannot run here)",
                   "sample_rows": k},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- the GPU path
def run_ours(args, world, rank, local):
    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41 import roofline, synth
    from sgl_amd_mono_b200.deepseek_v41.shapes import CONFIG2
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner, peer_cap

    from sgl_amd_mono_b200.common.peer import PeerBuffer

    dev = torch.device("cuda", local if world > 1 else 0)
    tp = world
    shape = CONFIG2.sharded(tp) if tp > 1 else CONFIG2
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            peaks = json.load(fh)
    except OSError:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    sweep = sorted({int(x) for x in args.sweep.split(",") if x} | {args.rows})
    peers = PeerBuffer(peer_cap(shape, max(sweep)), None, rank, world, dev) if tp > 1 else None
    runner = MonoRunner(shape, dev, rank=rank, peers=peers)
    # every rank draws the same full layer and keeps its shard
    positions = max(args.ctx, 32768) + 8  # config 5's verify rows sit at positions up to 32767
    layers = [runner.bind(synth.make_layer(shape, args.seed + 7919 * i, dev, positions=positions, rank=rank),
                          tag=f"layer{i}") for i in range(args.layers)]
    stream = torch.cuda.current_stream()
    results, graphs_by_m, steps_by_m, bufs_by_m = {}, {}, {}, {}
    launches_per_step = None
    for M in sweep:
        steps = [synth.make_step(shape, M, args.ctx, args.seed + 100 * i + M, dev) for i in range(args.layers)]
        graphs, bufs = [], []
        for L, st in zip(layers, steps):
            b = runner.k1(L, st, M)  # eager: allocates buffers and scratch outside capture
            runner.k2(L, st, M, b)
            c0 = ext.launch_count()
            runner.k1(L, st, M)
            runner.k2(L, st, M, b)
            if launches_per_step is None or M == args.rows:
                launches_per_step = ext.launch_count() - c0
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                runner.k1(L, st, M)
                runner.k2(L, st, M, b)
            graphs.append(g)
            bufs.append(b)
        clocks = Clocks(local if world > 1 else 0) if M == args.rows else None
        for i in range(args.warmup):
            graphs[i % len(graphs)].replay()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        if clocks:
            clocks.mark()
        e0.record(stream)
        for i in range(args.steps):
            graphs[i % len(graphs)].replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        clk = clocks.stop() if clocks else None
        barrier(world)
        ms = max_over_ranks(ms, world)
        # algorithmic bytes of the step (the run's own routing union, the keys read)
        unions = [int(torch.unique(b["ids"]).numel()) for b in bufs]
        keys = [int(b["klen"][:M].sum().item()) for b in bufs]
        lb = [roofline.layer_bytes(shape, u, k)["total"] for u, k in zip(unions, keys)]
        avg_bytes = sum(lb) / len(lb)
        gbs = avg_bytes / (ms * 1e-3) / 1e9
        results[M] = {"us_per_layer": round(ms * 1e3, 2), "tokens_s": round(M / (ms * 1e-3), 1),
                      "algorithmic_MB": round(avg_bytes / 1e6, 1), "union": unions,
                      "GBs": round(gbs, 1), "frac_hbm": round(gbs / hbm_peak, 4)}
        if clk is not None:
            results[M]["clocks"] = clk
        graphs_by_m[M], steps_by_m[M], bufs_by_m[M] = graphs, steps, bufs

    M = args.rows
    ms = results[M]["us_per_layer"] / 1e3
    value = M / (ms * 1e-3)
    runner.check()  # no device-side guard fired during the timed steps
    other = {}
    if not args.skip_configs:
        other["3"] = run_config3(args, runner, layers, world, stream, hbm_peak)
        other["5"] = run_config5(args, runner, layers, world, rank, stream, hbm_peak)
        other["4"] = run_config4(args, runner, layers, world, stream, hbm_peak)
        runner.check()
    tp_extra = tp_comparison(args, runner, layers, steps_by_m[M], bufs_by_m[M], M, world, stream) if tp > 1 else None
    parity = (tp_parity(args, steps_by_m[M][0], bufs_by_m[M][0], M, world, rank, dev, positions) if tp > 1 else
              "tp1: the -m gpu tests check these kernels against the oracle")

    # ---- stage timelines (eager launches, CUDA events at stage boundaries on the stream)
    n1, n2 = len(abi.K1_STAGES), len(abi.K2_STAGES)
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(n1 + 1)]
    ev2 = [torch.cuda.Event(enable_timing=True) for _ in range(n2 + 1)]
    arr1 = (ctypes_events(ev1))
    arr2 = (ctypes_events(ev2))
    reps = max(3, min(args.steps, 10))
    stages_by_m = {}
    for Ms in sweep:
        sm = {k: 0.0 for k in abi.K1_STAGES + abi.K2_STAGES}
        for i in range(reps):
            k = i % len(layers)
            L, st, b = layers[k], steps_by_m[Ms][k], bufs_by_m[Ms][k]
            a1, _ = runner.k1_args(L, st, Ms, events=arr1.addr)
            ext.call("dsv41_k1", a1, stream.cuda_stream)
            a2 = runner.k2_args(L, st, Ms, b, events=arr2.addr)
            ext.call("dsv41_k2", a2, stream.cuda_stream)
            torch.cuda.synchronize()
            for j, name in enumerate(abi.K1_STAGES):
                sm[name] += ev1[j].elapsed_time(ev1[j + 1]) / reps
            for j, name in enumerate(abi.K2_STAGES):
                sm[name] += ev2[j].elapsed_time(ev2[j + 1]) / reps
        stages_by_m[Ms] = sm
        results[Ms]["stages_us"] = {k: round(v * 1e3, 1) for k, v in sm.items()}
    stage_ms = stages_by_m[M]
    union = sum(results[M]["union"]) / len(results[M]["union"])
    exp_bytes = union * roofline.expert_bytes(shape)
    t_exp = stage_ms["routed experts"] * 1e-3
    achieved = exp_bytes / t_exp / 1e9

    # ---- end to end through the C-ABI with host buffers
    names = ("res", "x", "post", "comb", "pre", "pos", "slot", "swa_idx", "swa_lens")
    host_in = [[st[n].cpu().pin_memory() for n in names] for st in steps_by_m[M]]
    host_out = [[torch.empty_like(b[n], device="cpu").pin_memory() for n in ("out", "res2")]
                for b in bufs_by_m[M]]
    h2d = sum(t.numel() * t.element_size() for t in host_in[0])
    d2h = sum(t.numel() * t.element_size() for t in host_out[0])
    graphs = graphs_by_m[M]

    # As a server pipelines them: step i + 1's inputs go host -> device on a copy stream while step i
    # computes (the layer copies alternate, so its buffers are idle), and step i's results go
    # device -> host while step i + 1 computes. Events order each copy after the compute that last
    # used its buffers and each compute after its inputs; every step still copies all its inputs
    # in and its results out inside the timed region.
    copy_stream = torch.cuda.Stream(device=dev)
    nb = len(graphs)
    ev = lambda: [torch.cuda.Event() for _ in range(nb)]
    h2d_done, comp_done, d2h_done = ev(), ev(), ev()
    used = [False] * nb

    def copy_in(i):
        k = i % nb
        with torch.cuda.stream(copy_stream):
            if used[k]:
                copy_stream.wait_event(comp_done[k])  # the step that last read these inputs
            for n, t in zip(names, host_in[k]):
                steps_by_m[M][k][n].copy_(t, non_blocking=True)
            h2d_done[k].record(copy_stream)

    def e2e_run(first, count, start=None):
        if start is not None:
            copy_stream.wait_event(start)  # the first copy inside the timed region too
        copy_in(first)
        for i in range(first, first + count):
            k = i % nb
            stream.wait_event(h2d_done[k])
            if used[k]:
                stream.wait_event(d2h_done[k])  # results of the step that last wrote these buffers
            graphs[k].replay()
            comp_done[k].record(stream)
            used[k] = True
            if i + 1 < first + count:
                copy_in(i + 1)
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(comp_done[k])
                for n, t in zip(("out", "res2"), host_out[k]):
                    t.copy_(bufs_by_m[M][k][n], non_blocking=True)
                d2h_done[k].record(copy_stream)
        stream.wait_stream(copy_stream)

    e2e_run(0, args.warmup)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(args.warmup, args.steps, e0)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        W = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in layers[0].w.items()}
        S = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in steps_by_m[M][0].items()}
        k = min(REF_SAMPLE_ROWS, M)
        cpu_layer(W, sample_rows(S, k, 0), shape, k)
        t_cpu = min(cpu_layer(W, sample_rows(S, k, k * (i + 1)), shape, k) for i in range(2))
        cpu = {"value": k / t_cpu, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{k} of the step's {M} decode rows, the whole layer for them (ctx {args.ctx}), best of 2 "
                         f"after a warm-up; the reference path's CPU restatement (torch), {threads} threads"}
        del W, S

    if rank == 0:
        clk = results[M].get("clocks", {"sm_mhz": None, "sm_max_mhz": None, "reasons": []})
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp8/mxfp4 weights, bf16 activations",
            "data": "synthetic (random-init, seeded)",
            "config": workload_config(args, world),
            "detail": {"algorithmic_MB_per_step": results[M]["algorithmic_MB"],
                       "tp_comparison": tp_extra,
                       "configs": other,
                       "layer_roofline": {"GBs": results[M]["GBs"], "frac": results[M]["frac_hbm"],
                                          "peak_GBs": hbm_peak, "peak": peak_src},
                       "sweep": {str(k): {kk: vv for kk, vv in v.items() if kk != "clocks"}
                                 for k, v in results.items()},
                       "stages_us": {k: round(v * 1e3, 2) for k, v in stage_ms.items()}},
            "parity": parity,
            "roofline": {"bound": "hbm", "kernel": "routed experts (gate/up + act + down)",
                         "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4),
                         "traffic": int(union * EXPERT_DRAM_BYTES_PER_UNIT),
                         "traffic_source": "ncu dram bytes of the stage's two expert_tc_kernel launches "
                                           "(M 48, ctx 2048, union 199) per expert, scaled to this run's union",
                         "algorithmic_bytes": int(exp_bytes), "peak_source": peak_src},
            "cpu_baseline": cpu,
            "e2e": {"value": round(M / (e2e_ms * 1e-3), 1), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    del graphs_by_m, graphs
    torch.cuda.synchronize()
    barrier(world)
    if peers is not None:
        peers.close()


def _graph_time(args, fns, world, stream, reps=None):
    """Capture each callable in a CUDA graph, replay them round-robin after the warm-up, and
    return the max-over-ranks device time of one replay (ms)."""
    graphs = []
    for fn in fns:
        fn()  # eager: buffers and scratch outside the capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        graphs.append(g)
    for i in range(args.warmup):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize()
    barrier(world)
    reps = reps or args.steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps):
        graphs[i % len(graphs)].replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / reps, world)
    del graphs
    return ms


def run_config3(args, runner, layers, world, stream, hbm_peak):
    """the indexer layer -- K2i over 16 rows' FP4 index keys of a 32768-token
    compressed context (64 index heads), the top-2048, then K1 + K2 with the SWA window (128
    keys) and the 2048 selected compressed keys. Timed as one CUDA graph (K2i's walk plan,
    scoring and top-k, K1, K2), and K2i alone; two copies of the step's data alternate. The
    scorer is also timed alone over four copies of the index plane (``k2i_score_us``)."""
    from sgl_amd_mono_b200.deepseek_v41 import roofline, synth
    from sgl_amd_mono_b200.deepseek_v41.sm100a.indexer import K2iRunner

    M, ctx, topk, window, heads = 16, 32768, 2048, 128, 64
    s, dev = runner.s, runner.dev
    k2i = K2iRunner(dev, ctx, topk=topk)
    copies = []
    for i in range(2):
        st = synth.make_step(s, M, window, args.seed + 300 + i, dev)
        sp = synth.make_sparse(s, M, ctx, args.seed + 310 + i, dev, index_heads=heads)
        raw = torch.empty(M, topk, dtype=torch.int32, device=dev)
        page = torch.empty_like(raw)
        lens = torch.clamp(sp["bounds"], max=topk).to(torch.int32)
        copies.append((st, sp, raw, page, lens))

    def select(c):
        st, sp, raw, page, lens = c
        k2i.walk_plan(ratio=1, bounds=sp["bounds"], rows=M, per_req=1)
        k2i.select(kind="full", rows=M, per_req=1, ratio=1, query=(sp["q"], sp["qscale"], sp["w"]),
                   plane=(sp["payload"], sp["kscale"]), page_table=sp["page_table"], bounds=sp["bounds"],
                   raw_out=raw, page_out=page)

    def layer(i):
        c = copies[i]
        st, sp, raw, page, lens = c
        L = layers[i % len(layers)]
        select(c)
        b = runner.k1(L, st, M, topk_width=topk, topk_idx=page, topk_lens=lens)
        runner.k2(L, st, M, b, comp=sp["comp"], comp_stride=sp["comp"].stride(0), comp_blk=sp["comp_blk"])
        return b

    ms_sel = _graph_time(args, [lambda c=c: select(c) for c in copies], world, stream)
    ms_layer = _graph_time(args, [lambda i=i: layer(i) for i in range(2)], world, stream)
    # K2i's scorer alone (each plane's walk plan computed beforehand in its own runner), over four
    # copies of the index plane (4 x 35.7 MB, more than L2)
    planes = [c[1] for c in copies] + [
        synth.make_sparse(s, M, ctx, args.seed + 320 + i, dev, index_heads=heads) for i in range(2)]
    scorers = []
    for sp in planes:
        kr = K2iRunner(dev, ctx, topk=topk)
        kr.walk_plan(ratio=1, bounds=sp["bounds"], rows=M, per_req=1)
        scorers.append((kr, sp))

    def score(kr, sp):
        kr.score(rows=M, per_req=1, ratio=1, query=(sp["q"], sp["qscale"], sp["w"]),
                 plane=(sp["payload"], sp["kscale"]), page_table=sp["page_table"], bounds=sp["bounds"])

    ms_score = _graph_time(args, [lambda kr=kr, sp=sp: score(kr, sp) for kr, sp in scorers], world, stream)
    del planes[2:], scorers
    b = layer(0)
    torch.cuda.synchronize()
    union = int(torch.unique(b["ids"][:M]).numel())
    keys = int(b["klen"][:M].sum().item())
    index_bytes = M * ctx * 68  # 64 B of E2M1 + 4 E8M0 codes a key
    lb = roofline.layer_bytes(s, union, keys)["total"] + index_bytes
    return {"workload": f"config3: K2i (64 heads, ctx {ctx}) -> top-{topk} -> K1 + K2 (window {window} + "
                        f"{topk} compressed keys), {M} rows, tp{runner.s.tp}",
            "rows": M, "us_per_layer": round(ms_layer * 1e3, 2), "tokens_s": round(M / (ms_layer * 1e-3), 1),
            "k2i_select_us": round(ms_sel * 1e3, 2),
            "k2i_index_GBs": round(index_bytes / (ms_sel * 1e-3) / 1e9, 1),
            "k2i_frac_hbm": round(index_bytes / (ms_sel * 1e-3) / 1e9 / hbm_peak, 4),
            "k2i_score_us": round(ms_score * 1e3, 2),
            "k2i_score_frac_hbm": round(index_bytes / (ms_score * 1e-3) / 1e9 / hbm_peak, 4),
            "algorithmic_MB": round(lb / 1e6, 1), "frac_hbm": round(lb / (ms_layer * 1e-3) / 1e9 / hbm_peak, 4),
            "union": union}


def run_config5(args, runner, layers, world, rank, stream, hbm_peak):
    """a speculative-verify step's pieces -- 48 verify rows (8 requests x 6,
    row j of a block seeing its causal prefix of a 32768-token context) through one target
    layer and the one-layer draft (config-2 shapes, their own weights), then the LM head
    (129280 x 4096 bf16, vocab-parallel over the ranks) with the fused argmax and the greedy
    acceptance of each block. Each piece is CUDA-graph timed; the step line sums one target
    layer, the draft and the head."""
    import torch.distributed as dist

    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41 import synth
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi

    M, P, ctx, V = 48, 6, 32768, 129280
    s, dev = runner.s, runner.dev
    steps = [synth.make_step(s, M, ctx, args.seed + 500 + i, dev, per_req=P) for i in range(2)]

    def layer(i):
        L, st = layers[i % len(layers)], steps[i]
        b = runner.k1(L, st, M)
        runner.k2(L, st, M, b)

    ms_layer = _graph_time(args, [lambda i=i: layer(i) for i in range(2)], world, stream, reps=20)
    # the draft: its own layer (config-2 shapes, its own weights) over the same 48 rows, each
    # seeing the draft's window of 128 keys plus its causal prefix of the block (the
    # reference's draft reads WINDOW 128 + the block, draft.py:30-31, 173-195)
    draft_L = runner.bind(synth.make_layer(s, args.seed + 4242, dev, positions=ctx + 8, rank=runner.rank),
                          tag="draft")
    dsteps = [synth.make_step(s, M, DRAFT_WINDOW + P, args.seed + 520 + i, dev, per_req=P) for i in range(2)]

    def draft(i):
        st = dsteps[i]
        b = runner.k1(draft_L, st, M)
        runner.k2(draft_L, st, M, b)

    ms_draft = _graph_time(args, [lambda i=i: draft(i) for i in range(2)], world, stream, reps=20)
    vl = V // world
    g = torch.Generator(device=dev).manual_seed(args.seed + 600)
    heads = [(torch.randn(vl, s.hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(2)]
    x = torch.randn(M, s.hidden, generator=g, device=dev).to(torch.bfloat16)
    best = torch.empty(M, dtype=torch.int64, device=dev)
    ids = torch.empty(M, dtype=torch.int32, device=dev)
    draft_tok = torch.randint(0, V, (M,), generator=g, device=dev, dtype=torch.int32)
    acc = torch.empty(M // P, dtype=torch.int32, device=dev)
    nxt = torch.empty_like(acc)

    def head(i):
        a = abi.LmHeadArgs(M=M, V=vl, K=s.hidden, vbase=rank * vl, w=heads[i].data_ptr(), x=x.data_ptr(), logits=0,
                           best=best.data_ptr(), init=1)
        cur = torch.cuda.current_stream().cuda_stream  # the capturing stream under graph capture
        ext.call("dsv41_lmhead_argmax", a, cur)
        if world > 1:
            dist.all_reduce(best, op=dist.ReduceOp.MAX)
        d = abi.ArgmaxArgs(M=M, best=best.data_ptr(), ids=ids.data_ptr(), vals=0, draft=draft_tok.data_ptr(),
                           per_req=P, accept=acc.data_ptr(), next_tok=nxt.data_ptr())
        ext.call("dsv41_argmax_decode", d, cur)

    ms_head = _graph_time(args, [lambda i=i: head(i) for i in range(2)], world, stream)
    head_bytes = vl * s.hidden * 2
    step_ms = TARGET_LAYERS * ms_layer + ms_draft + ms_head
    del draft_L, dsteps
    return {"workload": f"config5: verify step, {M} rows (8 x {P}), ctx {ctx} causal blocks, a {TARGET_LAYERS}-layer "
                        f"target, the 1-layer draft (window {DRAFT_WINDOW} + the block), LM head {V} x {s.hidden} "
                        f"bf16 + argmax + greedy acceptance, tp{runner.s.tp}",
            "rows": M, "target_layer_us": round(ms_layer * 1e3, 2), "draft_us": round(ms_draft * 1e3, 2),
            "lm_head_argmax_accept_us": round(ms_head * 1e3, 2),
            "lm_head_GBs": round(head_bytes / (ms_head * 1e-3) / 1e9, 1),
            "lm_head_frac_hbm": round(head_bytes / (ms_head * 1e-3) / 1e9 / hbm_peak, 4),
            "verify_step_us": round(step_ms * 1e3, 1),
            "verify_tokens_s": round(M / (step_ms * 1e-3), 1),
            "note": f"verify_step_us = {TARGET_LAYERS} x target_layer_us (each target layer CUDA-graph timed on its own "
                    "copy of the weights) + draft_us + lm_head_argmax_accept_us"}


def run_config4(args, runner, layers, world, stream, hbm_peak):
    """a full 40-layer decode step, 16 rows at KV context 16384, the layers
    chained as the model runs them (layer j + 1's K1 takes layer j's K2 outputs: x, residual,
    post, comb, pre), each layer with its own paged KV cache, the weights cycling over the bound
    layer copies (each larger than L2). One CUDA graph holds the 40 K1 + K2 launches; at TP > 1
    the step is also timed with the NCCL variant of the two all-reduces a layer."""
    from sgl_amd_mono_b200.deepseek_v41 import roofline, synth
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner

    M, ctx, n_layers = 16, 16384, 40
    s, dev = runner.s, runner.dev
    caches = [synth.make_step(s, M, ctx, args.seed + 700 + j, dev) for j in range(n_layers)]

    def chain(r, record=None):
        b = r.buffers(M, ctx)
        for j, st in enumerate(caches):
            if j > 0:
                st = dict(st, res=b["res2"], x=b["out"], post=b["post_f"], comb=b["comb_f"], pre=b["pre_f"])
            r.k1(layers[j % len(layers)], st, M)
            r.k2(layers[j % len(layers)], st, M, b)
            if record is not None:
                record.append((int(torch.unique(b["ids"][:M]).numel()), int(b["klen"][:M].sum().item())))
        return b

    seen = []
    b = chain(runner, seen)  # eager: buffers, scratch and the layers' routing for the byte count
    torch.cuda.synchronize()
    finite = bool(torch.isfinite(b["out"].float()).all().item())
    reps = max(3, min(args.steps, 10))
    ms = _graph_time(args, [lambda: chain(runner)], world, stream, reps=reps)
    step_bytes = sum(roofline.layer_bytes(s, u, k)["total"] for u, k in seen)
    gbs = step_bytes / (ms * 1e-3) / 1e9
    out = {"workload": f"config4: {n_layers}-layer decode step (chained layers, own KV caches, weights cycling "
                       f"over {len(layers)} bound copies), {M} rows, ctx {ctx}, tp{s.tp}",
           "rows": M, "layers": n_layers, "us_per_step": round(ms * 1e3, 1),
           "us_per_layer": round(ms * 1e3 / n_layers, 2), "tokens_s": round(M / (ms * 1e-3), 1),
           "algorithmic_GB_per_step": round(step_bytes / 1e9, 3), "GBs": round(gbs, 1),
           "frac_hbm": round(gbs / hbm_peak, 4), "outputs_finite": finite, "replays": reps}
    if s.tp > 1:
        nccl = MonoRunner(s, dev, rank=runner.rank, group=None, allreduce="nccl")
        ms_n = _graph_time(args, [lambda: chain(nccl)], world, stream, reps=reps)
        out["us_per_step_nccl_variant"] = round(ms_n * 1e3, 1)
        del nccl
    runner.check()
    return out


def tp_parity(args, step, b, M, world, rank, dev, positions):
    """At TP > 1: every rank's layer against a TP = 1 run of the same full layer and step on rank 0,
    stage by stage as the tests compare kernels (each stage from the same input), and every rank's
    output against rank 0's. Attention: the TP = N all-reduced output (the rank-order sum of N bf16
    partials) against TP = 1's single partial, within 1e-2 relative (the reference's wo_b bound,
    1e-3, a partial, plus one bf16 rounding a rank). FFN: TP = 1's FFN half run from the TP = N
    attention output, so the router sees the same row: expert ids identical, the MoE output
    within the reference's ffn.moe.rel (1.5e-2). Also reported: the whole TP = 1 layer from the
    step (its own attention), whose MoE output differs more, as the MXFP8 requantization of the
    FFN input amplifies the attention's rounding."""
    import torch.distributed as dist

    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41 import synth
    from sgl_amd_mono_b200.deepseek_v41.shapes import CONFIG2
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner

    torch.cuda.synchronize()
    out, ids, attn = b["out"][:M].clone(), b["ids"][:M].clone(), b["attn"][:M].clone()
    gathered = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(gathered, out)
    res = None
    if rank == 0:
        rel = lambda a, r: float((a.float() - r.float()).norm() / r.float().norm())  # noqa: E731
        cur = torch.cuda.current_stream().cuda_stream
        r1 = MonoRunner(CONFIG2, dev)
        L1 = r1.bind(synth.make_layer(CONFIG2, args.seed, dev, positions=positions), tag="tp1 parity")
        st = dict(step, cache=step["cache"].clone())
        b1 = r1.k1(L1, st, M)
        r1.k2(L1, st, M, b1)  # the whole TP = 1 layer
        torch.cuda.synchronize()
        whole_rel = rel(out, b1["out"][:M])
        whole_sets = float((ids.sort(1).values == b1["ids"][:M].sort(1).values).all(1).float().mean())
        attn_rel = rel(attn, b1["attn_part"][:M])
        b1["attn"][:M].copy_(attn)  # (tp 1: attn is attn_part) the FFN half from the TP = N attention
        ext.call("dsv41_k2", r1.k2_args(L1, st, M, b1, phase=2), cur)
        torch.cuda.synchronize()
        moe_rel = rel(out, b1["out"][:M])
        ids_equal = bool(torch.equal(ids, b1["ids"][:M]))
        ranks_equal = all(torch.equal(g, out) for g in gathered)
        ok = attn_rel < 1e-2 and moe_rel < 1.5e-2 and ids_equal and ranks_equal
        res = {"status": "ok" if ok else "FAILED", "attention_rel_vs_tp1": round(attn_rel, 6),
               "moe_rel_vs_tp1_same_input": round(moe_rel, 6), "expert_ids_identical": ids_equal,
               "ranks_bit_identical": ranks_equal, "whole_layer_moe_rel_vs_tp1": round(whole_rel, 6),
               "whole_layer_expert_sets_equal_rows": round(whole_sets, 4),
               "bounds": "attention rel < 1e-2; from the same attention: ids identical, moe rel < 1.5e-2; "
                         "ranks identical"}
        del r1, L1, b1, st
        torch.cuda.synchronize()
    dist.barrier()
    return res


def tp_comparison(args, runner, layers, steps, bufs, M, world, stream):
    """At TP > 1: the layer with the NCCL variant of its all-reduces (all-gather + the same
    rank-order sum, CUDA-graph captured like ours), and one exchange of M x hidden bf16 alone
    (ours, the NCCL variant, NCCL's own all_reduce), device-timed, max over ranks."""
    import torch.distributed as dist

    from sgl_amd_mono_b200.common import ext
    from sgl_amd_mono_b200.deepseek_v41.sm100a import abi
    from sgl_amd_mono_b200.deepseek_v41.sm100a.runner import MonoRunner

    def timed(fn, reps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / reps, world) * 1e3

    s = runner.s
    nccl = MonoRunner(s, runner.dev, rank=runner.rank, group=None, allreduce="nccl")
    graphs = []
    for L, st in zip(layers, steps):
        b = nccl.k1(L, st, M)
        nccl.k2(L, st, M, b)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            nccl.k1(L, st, M)
            nccl.k2(L, st, M, b)
        graphs.append(g)
    it = iter(range(1 << 30))
    us_nccl = timed(lambda: graphs[next(it) % len(graphs)].replay(), args.steps)
    del graphs
    torch.cuda.synchronize()
    n = M * s.hidden
    src = torch.randn(n, device=runner.dev).to(torch.bfloat16)
    dst = torch.empty_like(src)
    gathered = torch.empty(world, n, dtype=torch.bfloat16, device=runner.dev)
    pa = abi.AllReduceArgs(n=n, tp=world, rank=runner.rank, peers=runner.peers.table.data_ptr(), cap=runner.peers.cap,
                           src=src.data_ptr(), dst=dst.data_ptr(), deadline_ns=runner.deadline_ns, site=3,
                           skip_push=0)
    ra = abi.RankSumArgs(n=n, tp=world, parts=gathered.data_ptr(), out=dst.data_ptr())
    us_peer = timed(lambda: ext.call("dsv41_allreduce", pa, stream.cuda_stream), 200)
    us_ll = timed(lambda: ext.call("dsv41_allreduce_ll", pa, stream.cuda_stream), 200)
    us_gather = timed(lambda: (dist.all_gather_into_tensor(gathered, src),
                               ext.call("dsv41_rank_sum", ra, stream.cuda_stream)), 200)
    us_ar = timed(lambda: dist.all_reduce(dst), 200)
    runner.check()
    # the layer with the standalone exchange kernels instead of the fused LL exchange
    ext.set_option("fused_allreduce", 0)
    graphs = []
    for L, st, b in zip(layers, steps, bufs):
        runner.k1(L, st, M)
        runner.k2(L, st, M, b)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            runner.k1(L, st, M)
            runner.k2(L, st, M, b)
        graphs.append(g)
    ext.set_option("fused_allreduce", 1)
    it2 = iter(range(1 << 30))
    us_unfused = timed(lambda: graphs[next(it2) % len(graphs)].replay(), args.steps)
    del graphs
    torch.cuda.synchronize()
    runner.check()
    return {"layer_us_nccl_variant": round(us_nccl, 2),
            "layer_us_standalone_exchange": round(us_unfused, 2),
            "exchange_bytes": 2 * n, "nvlink_bytes_out_per_exchange": 2 * n * (world - 1),
            "exchange_us": {"in_kernel_ll": round(us_ll, 2), "in_kernel_flagged": round(us_peer, 2),
                            "nccl_allgather_rank_sum": round(us_gather, 2),
                            "nccl_all_reduce_bf16": round(us_ar, 2)}}


class ctypes_events:
    """A host array of cudaEvent_t handles for the C-ABI's stage events."""

    def __init__(self, events):
        import ctypes
        for e in events:  # torch creates the CUDA event at its first record
            e.record()
        torch.cuda.synchronize()
        self.arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
        self.addr = ctypes.addressof(self.arr)


def main():
    args = parse()
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
