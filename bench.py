#!/usr/bin/env python
"""Benchmark of the HSPMN v2.1 contextual-stream inference path on B200.

Default workload (one JSON line on rank 0): HSPMNBlock eval forward, bf16,
dim=2048, num_heads=16, num_kv_heads=4 (the config default), k=0.2, S=4096,
64 sequences per GPU, x ~ N(0,1), default-init weights (seed 42). A step is
one block forward over the GPU's batch; the router top-K, the row gathers
(with the query RoPE fused), SQDK attention and the residual write-back of
the routed rows inside it are this library's sm_100a kernels; the
projections (cuBLAS), norms, K RoPE and the reflexive stream are stock
PyTorch. Multi-GPU: one process per GPU (torchrun), every rank runs its
own 64 sequences with replicated weights and no data-path collective (weak
scaling); the timed region is bracketed by barriers and the max over ranks is
reported.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload block|sqdk-sweep|sqdk|sqdk-bwd|long]

``--impl reference`` times the reference algorithm's CPU implementation (the
numpy oracle port of HSPMNBlock.forward) on the host cores, one sequence of
the same workload per step; under torchrun only rank 0 runs it.
``--workload sqdk-sweep`` runs the standalone router / gather / SQDK / scatter
sweep (B=8, S=32768, H=Hkv=16, hd=128, k in {0.05, 0.1, 0.2, 0.5}) and
prints one line per k; ``--workload sqdk`` runs the same standalone path at
``--batch/--seq-len/--heads/--kv-heads/--sparsity``. ``--workload long`` runs
one sequence of ``--seq-len`` tokens (262144 for the long-context
configuration) sequence-sharded over the ranks (strong scaling).
``--workload sqdk-bwd`` times the SQDK backward (the training path's
attention gradients) at the block's attention shape.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(REPO, "hspmn-v2.1_b200"), REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "SQDK block tok/s at B=64,S=4096,D=2048,k=0.2; attention TFLOPS % of bf16 peak"
PUBLISHED_TOK_S = 1406304.0  # reference README.md:30, RTX 5090, same block config
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["block", "sqdk-sweep", "sqdk", "sqdk-bwd", "long"], default="block")
    ap.add_argument("--batch", type=int, default=64, help="sequences per GPU")
    ap.add_argument("--seq-len", type=int, default=4096)
    ap.add_argument("--dim", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--sparsity", type=float, default=0.2)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-seconds", type=float, default=12.0)
    a = ap.parse_args()
    if a.warmup < 3:
        ap.error("--warmup must be >= 3")
    return a


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ---------------------------------------------------------------------------
# peaks, traffic, clocks
# ---------------------------------------------------------------------------


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def profiled_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary
    (profiles/<kernel>__<workload>.md, line ``dram_bytes_per_launch = N``)."""
    path = os.path.join(REPO, "profiles", f"{kernel}__{workload}.md")
    try:
        with open(path) as f:
            for line in f:
                if line.strip().startswith("dram_bytes_per_launch"):
                    return float(line.split("=", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = set(gpu_indices)
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="hspmn_clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons, n = [], [], set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                n += 1
                for name, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": n}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port of the reference algorithm on host cores
# ---------------------------------------------------------------------------


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = max((d.get("num_threads", 1) for d in threadpool_info()), default=1)
        return int(n)
    except Exception:  # pragma: no cover
        return os.cpu_count() or 1


def cpu_block_sample(args, seconds: float, max_steps: int | None = None, warmup: int = 1):
    """Time the numpy oracle's HSPMNBlock forward on one sequence of the
    workload. Returns (tok/s, sample description, cores, per-step seconds)."""
    import numpy as np
    import torch

    import oracle
    from hspmn_b200 import HSPMNBlock, HSPMNConfig, seed_everything

    seed_everything(42)
    cfg = HSPMNConfig(dim=args.dim, num_heads=args.heads, num_kv_heads=args.kv_heads,
                      sparsity_k=args.sparsity, max_seq_len=args.seq_len)
    block = HSPMNBlock(cfg).to(torch.bfloat16)
    params = {k: v.float().numpy() for k, v in block.state_dict().items()}
    ts = float(block.router.target_sparsity.item())
    g = torch.Generator().manual_seed(1000)
    x = torch.randn(1, args.seq_len, args.dim, generator=g).to(torch.bfloat16).float().numpy()
    eps = float(torch.finfo(torch.bfloat16).eps)

    def step():
        oracle.block_forward(params, x, args.heads, args.kv_heads, ts, cfg.rope_base, eps, noisy_dtype="bf16")

    for _ in range(warmup):
        step()
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if max_steps is not None and len(times) >= max_steps:
            break
        if max_steps is None and time.perf_counter() - t_start >= seconds:
            break
    per = statistics.mean(times)
    sample = (f"numpy oracle HSPMNBlock.forward (fp32 arithmetic on bf16-valued weights/inputs), one sequence "
              f"S={args.seq_len} D={args.dim} per step, {len(times)} timed step(s) after {warmup} warm-up")
    return args.seq_len / per, sample, cpu_threads(), per


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    steps = max(1, args.steps)
    tok_s, sample, cores, per = cpu_block_sample(args, 0.0, max_steps=steps, warmup=min(args.warmup, 1))
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": tok_s / PUBLISHED_TOK_S, "dtype": "f32",
        "data": "synthetic: x ~ N(0,1), default-init weights (seed 42)",
        "config": workload_config(args),
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------


def workload_config(args, per_gpu_batch=None):
    B = args.batch if per_gpu_batch is None else per_gpu_batch
    return {
        "workload": (f"HSPMNBlock eval forward, bf16, dim={args.dim} heads={args.heads} kv_heads={args.kv_heads} "
                     f"S={args.seq_len} k={args.sparsity}, {B} sequence(s) per GPU"),
        "batch_per_gpu": B, "global_batch": B * args.gpus, "seq_len": args.seq_len, "dim": args.dim,
        "num_heads": args.heads, "num_kv_heads": args.kv_heads, "sparsity_k": args.sparsity,
        "parallelism": f"batch-partitioned x{args.gpus}, no data-path collective",
        "l2": "inputs larger than L2 (x is B*S*D*2 bytes per GPU per step)",
    }


def init_dist(world, local_rank):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    return torch.device("cuda", local_rank)


def barrier(world):
    import torch
    import torch.distributed as dist

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(val: float, world: int, dev) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return val
    t = torch.tensor([val], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_block(args):
    import torch

    from hspmn_b200 import HSPMNBlock, HSPMNConfig, ops, seed_everything

    rank, world, local_rank = dist_env()
    dev = init_dist(world, local_rank)
    seed_everything(42)
    cfg = HSPMNConfig(dim=args.dim, num_heads=args.heads, num_kv_heads=args.kv_heads, sparsity_k=args.sparsity,
                      max_seq_len=args.seq_len)
    model = HSPMNBlock(cfg).to(dev, dtype=torch.bfloat16).eval()
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    B, S, D = args.batch, args.seq_len, args.dim
    x = torch.randn(B, S, D, device=dev, dtype=torch.bfloat16, generator=g)

    with torch.no_grad():
        for _ in range(args.warmup):
            model(x)
        # algorithmic attention FLOPs of one forward (the indices do not change between steps)
        idx = model.router(x).indices
        sqdk_flops = 4.0 * cfg.head_dim * cfg.num_heads * float((idx + 1).sum().item())
        k_sel = idx.shape[1]
        barrier(world)
        clocks = ClockSampler([local_rank] if world == 1 else range(world)) if rank == 0 else None
        if clocks:
            clocks.start()
        launches0 = ops.LaunchStats.launches
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ops.KernelTimer() as kt:
            start.record()
            for _ in range(args.steps):
                model(x)
            end.record()
        torch.cuda.synchronize()
        launches = ops.LaunchStats.launches - launches0
        clock_info = clocks.stop() if clocks else None
        ms_total = max_over_ranks(start.elapsed_time(end), world, dev)
        barrier(world)
        kres = kt.results()

        # end to end through the public API: host x -> device -> forward -> host out, every
        # step. Two-deep pipeline as a server would run it: the upload of step i+1 (copy stream
        # h2d) and the download of step i-1 (copy stream d2h) overlap the forward of step i.
        # The timed region starts before the first upload and ends after the last download.
        e2e = None
        if not args.no_e2e:
            x_host = x.cpu().pin_memory()
            out_host = [torch.empty((B, S, D), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
            aux_host = [torch.empty((), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
            comp = torch.cuda.current_stream(dev)
            h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
            x_dev = [torch.empty_like(x) for _ in range(2)]
            in_ready = [torch.cuda.Event() for _ in range(2)]
            in_free = [torch.cuda.Event() for _ in range(2)]
            out_free = [torch.cuda.Event() for _ in range(2)]

            def run_pipeline(nsteps, start_event):
                h2d.wait_event(start_event)
                with torch.cuda.stream(h2d):
                    x_dev[0].copy_(x_host, non_blocking=True)
                in_ready[0].record(h2d)
                for i in range(nsteps):
                    cur, nxt = i % 2, (i + 1) % 2
                    if i + 1 < nsteps:
                        if i >= 1:
                            h2d.wait_event(in_free[nxt])  # forward i-1 has read x_dev[nxt]
                        with torch.cuda.stream(h2d):
                            x_dev[nxt].copy_(x_host, non_blocking=True)
                        in_ready[nxt].record(h2d)
                    comp.wait_event(in_ready[cur])
                    out, aux = model(x_dev[cur])
                    in_free[cur].record(comp)
                    done = torch.cuda.Event()
                    done.record(comp)
                    d2h.wait_event(done)
                    if i >= 2:
                        d2h.wait_event(out_free[cur])  # host buffer of step i-2 was copied out
                    with torch.cuda.stream(d2h):
                        out_host[cur].copy_(out, non_blocking=True)
                        aux_host[cur].copy_(aux, non_blocking=True)
                    out_free[cur].record(d2h)
                    out.record_stream(d2h)
                    aux.record_stream(d2h)
                comp.wait_stream(d2h)

            for _ in range(2):
                w = torch.cuda.Event()
                w.record(comp)
                run_pipeline(2, w)
            torch.cuda.synchronize()
            barrier(world)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(comp)
            run_pipeline(args.e2e_steps, e0)
            e1.record(comp)
            torch.cuda.synchronize()
            e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
            e2e = {"value": B * S * args.e2e_steps * world / (e2e_ms / 1e3), "unit": "tok/s",
                   "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                   "d2h_bytes_per_step": out_host[0].numel() * out_host[0].element_size() + 2,
                   "pipeline": "2-deep: upload of step i+1 and download of step i-1 overlap forward i",
                   "steps": args.e2e_steps, "ms_per_step": e2e_ms / args.e2e_steps}

        # the opt-in fp32 gate kernel next to the module's cuBLAS gate (nn.Linear(dim, 1)),
        # both over the whole x (larger than L2) of this GPU
        gate_w, gate_b = model.router.gate.weight, model.router.gate.bias
        gate_times = {}
        for name, fn in (("gate_logits", lambda: ops.gate_logits(x, gate_w, gate_b)),
                         ("cublas_gate", lambda: model.router.gate(x))):
            for _ in range(3):
                fn()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record()
            for _ in range(10):
                fn()
            g1.record()
            torch.cuda.synchronize()
            gate_times[name] = g0.elapsed_time(g1) / 10

    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks, peak_src = load_peaks()
    sq = kres.get("sqdk_fwd", {"launches": 0, "ms": float("nan")})
    sq_ms = sq["ms"] / max(1, sq["launches"])
    achieved = sqdk_flops / (sq_ms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    wl_tag = f"B{B}_S{S}_D{D}_H{args.heads}_Hkv{args.kv_heads}"
    traffic = profiled_traffic("sqdk_fwd", wl_tag)
    esz = 2
    kernels = {}
    for name, r in kres.items():
        per = r["ms"] / max(1, r["launches"])
        kernels[name] = {"launches": r["launches"], "ms_per_launch": per}
    if "gather_rows" in kernels:
        gb = 2 * B * k_sel * D * esz + B * k_sel * 8
        kernels["gather_rows"]["GB_s"] = gb / (kernels["gather_rows"]["ms_per_launch"] / 1e3) / 1e9
    if "rope_gather_rows" in kernels:
        # two launches per forward: the K routed query rows (D elements each) and all S key
        # rows (Hkv * hd elements each); each reads its rows and indices and writes its rows
        kv_row = (D // args.heads) * args.kv_heads
        gb_step = (2 * B * k_sel * D * esz + B * k_sel * 8) + (2 * B * S * kv_row * esz + B * S * 8)
        steps_seen = max(1, kernels.get("sqdk_fwd", {}).get("launches", 1))
        per_step = max(1, kernels["rope_gather_rows"]["launches"] // steps_seen)
        kernels["rope_gather_rows"]["GB_s"] = (gb_step / per_step) / (kernels["rope_gather_rows"]["ms_per_launch"] / 1e3) / 1e9
    if "scatter_add_rows" in kernels:
        gb = 3 * B * k_sel * D * esz + B * k_sel * 8
        kernels["scatter_add_rows"]["GB_s"] = gb / (kernels["scatter_add_rows"]["ms_per_launch"] / 1e3) / 1e9
    if "scatter_rows" in kernels:
        gb = B * k_sel * D * esz + B * S * D * esz + B * k_sel * 8
        kernels["scatter_rows"]["GB_s"] = gb / (kernels["scatter_rows"]["ms_per_launch"] / 1e3) / 1e9
    if "router_topk" in kernels:
        gb = B * S * esz + B * k_sel * 8 + B * S
        kernels["router_topk"]["GB_s"] = gb / (kernels["router_topk"]["ms_per_launch"] / 1e3) / 1e9
    if "sqdk_fwd" in kernels:
        kernels["sqdk_fwd"]["TFLOP_s"] = achieved
        kernels["sqdk_fwd"]["algorithmic_flops"] = sqdk_flops
    # gate GEMV: read x and w, write one logit per position (f32 here, bf16 from cuBLAS)
    gate = {}
    for name, out_bytes in (("gate_logits", 4), ("cublas_gate", esz)):
        gb = B * S * D * esz + D * esz + B * S * out_bytes
        ms = gate_times[name]
        gate[name] = {"ms_per_launch": ms, "GB_s": gb / (ms / 1e3) / 1e9,
                      "frac_of_hbm": gb / (ms / 1e3) / 1e9 / float(peaks["hbm_gbs"])}

    value = B * S * args.steps * world / (ms_total / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": value / PUBLISHED_TOK_S, "dtype": "bf16",
        "data": "synthetic: x ~ N(0,1), default-init weights (seed 42)",
        "config": workload_config(args),
        "roofline": {"bound": "tensor", "kernel": "sqdk_fwd", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_src} bf16 dense, sustained (kernel timed inside a long step)",
                     "flops_per_launch": sqdk_flops, "ms_per_launch": sq_ms, "k_selected": k_sel},
        "kernels": kernels,
        "router_gate": dict(gate, note="opt-in fp32 gate (router.fp32_gate) vs the default cuBLAS bf16 gate; "
                                       "outside the timed step"),
        "gpu_launches": launches,
        "clocks": clock_info,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if world == 1 and not args.no_cpu_baseline:
        tok_s, sample, cores, _ = cpu_block_sample(args, args.cpu_sample_seconds)
        line["cpu_baseline"] = {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# standalone SQDK sparsity sweep
# ---------------------------------------------------------------------------


def run_sweep(args, B=8, S=32768, H=16, Hkv=16, fracs=(0.05, 0.1, 0.2, 0.5)):
    import torch

    from hspmn_b200 import ops

    rank, world, local_rank = dist_env()
    dev = init_dist(world, local_rank)
    hd = 128
    peaks, peak_src = load_peaks()
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    q = torch.randn(B, S, H, hd, device=dev, dtype=torch.bfloat16, generator=g)
    k = torch.randn(B, S, Hkv, hd, device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn(B, S, Hkv, hd, device=dev, dtype=torch.bfloat16, generator=g)
    logits = torch.randn(B, S, device=dev, dtype=torch.float32, generator=g)
    for frac in fracs:
        K = max(1, int(S * frac))

        def step():
            idx, _ = ops.router_topk(logits, None, K, torch.float32)
            qs = ops.gather_rows(q, idx)
            o = ops.sqdk_fwd(qs, k, v, idx, hd ** -0.5)
            return ops.scatter_rows(o, idx, S), idx

        with torch.no_grad():
            for _ in range(args.warmup):
                _, idx = step()
            flops = 4.0 * hd * H * float((idx + 1).sum().item())
            barrier(world)
            with ops.KernelTimer() as kt:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(args.steps):
                    step()
                e1.record()
            torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
        res = {n: r["ms"] / r["launches"] for n, r in kt.results().items()}
        if rank == 0:
            tf = flops / (res["sqdk_fwd"] / 1e3) / 1e12
            gather_b = 2 * B * K * H * hd * 2 + B * K * 8  # noqa: E501 (rows are H*hd wide)
            scatter_b = B * K * H * hd * 2 + B * S * H * hd * 2 + B * K * 8
            print(json.dumps({
                "metric": "standalone SQDK: attention TFLOP/s and gather/scatter GB/s", "workload":
                f"B={B} S={S} H={H} Hkv={Hkv} hd={hd} k={frac} (K={K}), router on f32 logits", "n_gpus": world,
                "value": tf, "unit": "TFLOP/s", "frac_of_peak": tf / float(peaks["bf16_tflops"]),
                "peak_source": f"{peak_src} bf16 dense, burst", "ms_per_step": ms / args.steps,
                "router_us": res["router_topk"] * 1e3,
                "gather_GB_s": gather_b / (res["gather_rows"] / 1e3) / 1e9,
                "scatter_GB_s": scatter_b / (res["scatter_rows"] / 1e3) / 1e9,
                "hbm_peak_GB_s": float(peaks["hbm_gbs"]), "sqdk_ms": res["sqdk_fwd"]}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# SQDK backward (training path of the contextual stream)
# ---------------------------------------------------------------------------


def run_sqdk_bwd(args):
    """Backward of the SQDK attention at the block's attention shape
    (--batch/--seq-len/--heads/--kv-heads/--sparsity, hd = dim / heads): the
    selected rows of a random sorted selection, the forward with log-sum-exp
    once, then timed launches of the backward (rowsum(dO*O), the key-block
    kernel, the dq cast). Algorithmic FLOPs: 10 * hd per (row, visible key)
    (S^T, dP^T, dV, dK, dQ), i.e. 2.5 x the forward's."""
    import torch

    from hspmn_b200 import ops

    rank, world, local_rank = dist_env()
    dev = init_dist(world, local_rank)
    B, S, H, Hkv = args.batch, args.seq_len, args.heads, args.kv_heads
    hd = args.dim // H
    K = max(1, int(S * args.sparsity))
    peaks, peak_src = load_peaks()
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    q = torch.randn(B, K, H, hd, device=dev, dtype=torch.bfloat16, generator=g)
    k = torch.randn(B, S, Hkv, hd, device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn(B, S, Hkv, hd, device=dev, dtype=torch.bfloat16, generator=g)
    d_o = torch.randn(B, K, H, hd, device=dev, dtype=torch.bfloat16, generator=g)
    idx = torch.sort(torch.rand(B, S, device=dev, generator=g).argsort(dim=1)[:, :K], dim=1)[0]
    scale = hd ** -0.5
    with torch.no_grad():
        o, lse = ops.sqdk_fwd_lse(q, k, v, idx, scale)
        flops = 10.0 * hd * H * float((idx + 1).sum().item())
        for _ in range(args.warmup):
            ops.sqdk_bwd(q, k, v, idx, o, d_o, lse, scale)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            ops.sqdk_bwd(q, k, v, idx, o, d_o, lse, scale)
        e1.record()
        torch.cuda.synchronize()
        assert ops.device_errors(dev) == 0
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / args.steps
    if rank == 0:
        tf = flops * world / (ms / 1e3) / 1e12
        peak = float(peaks["bf16_tflops"])
        print(json.dumps({
            "metric": "SQDK backward: attention-gradient TFLOP/s", "value": tf, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic: N(0,1) q/k/v/dO, "
            "random sorted selection", "config": {"workload": f"SQDK backward B={B} S={S} H={H} Hkv={Hkv} hd={hd} "
                                                               f"k={args.sparsity} (K={K}) per GPU"},
            "roofline": {"bound": "tensor", "achieved": tf / world, "peak": peak, "unit": "TFLOP/s",
                         "frac": tf / world / peak, "peak_source": f"{peak_src} bf16 dense, burst",
                         "flops_per_launch": flops}}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# long context: one sequence, sequence-sharded over the ranks
# ---------------------------------------------------------------------------


def run_long(args):
    import torch

    from hspmn_b200 import HSPMNBlock, HSPMNConfig, ops, seed_everything
    from hspmn_b200.parallel import SequenceShardedBlock, ZigZagPlan

    rank, world, local_rank = dist_env()
    if world == 1:
        # a one-rank process group keeps the code path identical to N > 1
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29531")
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
        dev = torch.device("cuda", local_rank)
    else:
        dev = init_dist(world, local_rank)
    S = args.seq_len
    seed_everything(42)
    cfg = HSPMNConfig(dim=args.dim, num_heads=args.heads, num_kv_heads=args.kv_heads, sparsity_k=args.sparsity,
                      max_seq_len=S)
    model = HSPMNBlock(cfg).to(dev, dtype=torch.bfloat16).eval()
    plan = ZigZagPlan(S, world)
    sb = SequenceShardedBlock(model, plan)
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    x_local = torch.randn(1, 2 * plan.chunk, args.dim, device=dev, dtype=torch.bfloat16, generator=g)
    with torch.no_grad():
        for _ in range(args.warmup):
            sb.forward(x_local)
        barrier(world)
        launches0 = ops.LaunchStats.launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ops.KernelTimer() as kt:
            e0.record()
            for _ in range(args.steps):
                sb.forward(x_local)
            e1.record()
        torch.cuda.synchronize()
        launches = ops.LaunchStats.launches - launches0
        ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
        kres = kt.results()
        sq = kres.get("sqdk_fwd", {"launches": 1, "ms": float("nan")})
        sq_ms = max_over_ranks(sq["ms"] / max(1, sq["launches"]), world, dev)
    import torch.distributed as dist
    dist.destroy_process_group()
    if rank == 0:
        peaks, peak_src = load_peaks()
        value = S * args.steps / (ms / 1e3)
        print(json.dumps({
            "metric": "long-context HSPMNBlock tok/s (one sequence, sequence-sharded)", "value": value,
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic: x ~ N(0,1), default-init weights (seed 42)",
            "config": {"workload": f"HSPMNBlock eval forward, B=1 S={S} dim={args.dim} heads={args.heads} "
                                   f"kv_heads={args.kv_heads} k={args.sparsity}, zig-zag sequence shards",
                       "seq_len": S, "parallelism": f"sequence-sharded x{world}, all-gather of logits and K/V"},
            "sqdk_ms_per_launch_max_rank": sq_ms, "gpu_launches": launches,
            "kernels_rank0": {n: {"launches": r["launches"], "ms_per_launch": r["ms"] / max(1, r["launches"])}
                              for n, r in kres.items()},
            "peak_source": peak_src}), flush=True)


def main():
    args = parse_args()
    _, world, _ = dist_env()
    if world != args.gpus and world > 1:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    args.gpus = world if world > 1 else args.gpus
    if args.impl == "reference":
        return run_reference(args)
    if args.gpus > 1 and world == 1:
        raise SystemExit("--gpus N>1 needs torchrun: python -m torch.distributed.run --nproc-per-node N bench.py ...")
    if args.workload == "sqdk-sweep":
        return run_sweep(args)
    if args.workload == "long":
        return run_long(args)
    if args.workload == "sqdk":
        return run_sweep(args, args.batch, args.seq_len, args.heads, args.kv_heads, (args.sparsity,))
    if args.workload == "sqdk-bwd":
        return run_sqdk_bwd(args)
    return run_block(args)


if __name__ == "__main__":
    main()
