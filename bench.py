#!/usr/bin/env python
"""Benchmark of the HSPMN v2.1 contextual-stream inference path on B200.

Default workload (one JSON line on rank 0): HSPMNBlock eval forward, bf16,
dim=2048, num_heads=16, num_kv_heads=4 (the config default), k=0.2, S=4096,
64 sequences per GPU, x ~ N(0,1), default-init weights (seed 42). A step is
one block forward over the GPU's batch; the router top-K, the row gathers
(with the query RoPE fused), SQDK attention and the residual write-back of
the routed rows inside it are this library's sm_100a kernels; the
projections (cuBLAS), norms and the reflexive stream are stock PyTorch.
Multi-GPU: one process per GPU (torchrun), every rank runs its own 64
sequences with replicated weights and no data-path collective (weak
scaling); the timed region is bracketed by barriers and the max over ranks is
reported.

After the timed block steps the same run adds, untimed unless stated:
  * ``headline_parity``: two sequences of the timed B=64 SQDK launch against
    the fp32 oracle;
  * ``long_parity``: the sequence-sharded block over all ranks at S=32768
    against the plain one-GPU block forward on rank 0;
  * ``long_context``: the S=262144 single sequence sequence-sharded over all
    ranks (strong scaling), timed, with the K/V exchange timed on its own;
  * at N=1: the standalone sparsity sweep (B=8, S=32768, H=Hkv=16, hd=128,
    k in {0.05, 0.1, 0.2, 0.5}) and library GPU comparators of the SQDK
    attention (torch SDPA with a boolean mask, and the reference's own
    dense-masked PyTorch SQDK pattern run on the GPU);
  * at N=1: ``cpu_baseline``, the reference's PyTorch CPU path (a torch
    restatement of HSPMNBlock.forward with eager FlexAttention, as the
    reference runs without a GPU) on all host cores.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload block|sqdk-sweep|sqdk|sqdk-bwd|long]

``--impl reference`` times the reference's CPU path (the torch restatement
above) on all host cores, one sequence of the block workload per step; under
torchrun only rank 0 runs it. ``--workload sqdk-sweep`` prints the sweep as
one line per k; ``--workload sqdk`` runs the same standalone path at
``--batch/--seq-len/--heads/--kv-heads/--sparsity``; ``--workload long`` runs
only the long-context measurement; ``--workload sqdk-bwd`` times the SQDK
backward (the training path's attention gradients) at the block's attention
shape.
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
LONG_SEQ = 262144
LONG_PARITY_SEQ = 32768


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
    ap.add_argument("--long-steps", type=int, default=5)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="only the timed steps (no parity, long-context, sweep or library comparators)")
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
        sm, smax, pw, reasons, n = [], [], [], set(), 0
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
                try:
                    pw.append(float(parts[3]))
                except ValueError:
                    pass
                n += 1
                for name, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "power_w": statistics.median(pw) if pw else None, "reasons": sorted(reasons), "samples": n}


# ---------------------------------------------------------------------------
# CPU side: the reference's PyTorch CPU path, and the numpy oracle port
# ---------------------------------------------------------------------------


def use_all_host_cores() -> int:
    """torch and the BLAS pools on every host core, whatever OMP_NUM_THREADS
    a launcher set (torchrun sets 1). Returns the thread count in use."""
    import torch

    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(n)
    except Exception:  # pragma: no cover
        pass
    return n


def _cpu_block_setup(args):
    import torch

    from hspmn_b200 import HSPMNBlock, HSPMNConfig, seed_everything

    seed_everything(42)
    cfg = HSPMNConfig(dim=args.dim, num_heads=args.heads, num_kv_heads=args.kv_heads,
                      sparsity_k=args.sparsity, max_seq_len=args.seq_len)
    block = HSPMNBlock(cfg).to(torch.bfloat16)
    g = torch.Generator().manual_seed(1000)
    x = torch.randn(1, args.seq_len, args.dim, generator=g).to(torch.bfloat16)
    return cfg, block, x


def cpu_reference_sample(args, steps: int | None = None, seconds: float = 0.0, warmup: int = 3):
    """Time the reference's PyTorch CPU path (oracle.torch_cpu_ref: the
    reference HSPMNBlock.forward with eager FlexAttention, its path without a
    GPU) on one sequence of the block workload, on all host cores. The first
    two warm-up steps run the module in float32 and in bfloat16; the faster
    dtype is timed. Returns a dict with tok/s, ms/step, dtype, cores and the
    sample description."""
    import warnings

    import torch

    from oracle.torch_cpu_ref import block_forward_torch

    warnings.filterwarnings("ignore", message=".*flex_attention called without torch.compile.*")
    cores = use_all_host_cores()
    cfg, block, x_bf16 = _cpu_block_setup(args)
    sds = {dt: {k: v.to(dt) for k, v in block.state_dict().items()} for dt in (torch.float32, torch.bfloat16)}
    xs = {dt: x_bf16.to(dt) for dt in sds}

    def step(dt):
        t0 = time.perf_counter()
        block_forward_torch(sds[dt], xs[dt], args.heads, args.kv_heads, cfg.rope_base, cfg.block_size)
        return time.perf_counter() - t0

    step(torch.float32)  # first call builds the block mask machinery
    probe = {dt: step(dt) for dt in sds}
    dt = min(probe, key=probe.get)
    for _ in range(max(0, warmup - 2)):
        step(dt)
    times = []
    t_start = time.perf_counter()
    while True:
        times.append(step(dt))
        if steps is not None and len(times) >= steps:
            break
        if steps is None and time.perf_counter() - t_start >= seconds:
            break
    per = statistics.mean(times)
    name = str(dt).replace("torch.", "")
    return {"value": args.seq_len / per, "unit": "tok/s", "cores": cores, "kind": "port",
            "dtype": name, "ms_per_step": per * 1e3,
            "sample": (f"reference HSPMNBlock.forward on its CPU path (eager FlexAttention: dense S x S attention), "
                       f"torch restatement pinned to the reference's block outputs, {name} (faster of f32/bf16 "
                       f"on this host: f32 {probe[torch.float32]:.2f} s, bf16 {probe[torch.bfloat16]:.2f} s), "
                       f"one sequence S={args.seq_len} D={args.dim} per step, {len(times)} timed step(s), "
                       f"{cores} threads")}


def cpu_oracle_sample(args, seconds: float):
    """Time the numpy oracle's HSPMNBlock forward (sparse attention over the
    selected rows only) on one sequence of the workload."""
    import oracle

    cores = use_all_host_cores()
    cfg, block, x = _cpu_block_setup(args)
    params = {k: v.float().numpy() for k, v in block.state_dict().items()}
    ts = float(block.router.target_sparsity.item())
    xn = x.float().numpy()
    eps = 0.0078125  # finfo(bfloat16).eps, the module dtype's

    def step():
        oracle.block_forward(params, xn, args.heads, args.kv_heads, ts, cfg.rope_base, eps, noisy_dtype="bf16")

    step()
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start >= seconds:
            break
    per = statistics.mean(times)
    return {"value": args.seq_len / per, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": (f"numpy oracle HSPMNBlock.forward (attention over the selected rows only, fp32), one "
                       f"sequence S={args.seq_len} D={args.dim} per step, {len(times)} timed step(s)")}


def cpu_sqdk_cfg1(iters: int = 200):
    """The reference's PyTorch SQDK test pattern (test_kernels_v2_1.py:34-65)
    in fp32 at B=2, S=512, H=4, hd=64, K=102 on the host cores: ms per call."""
    import torch

    from oracle.torch_cpu_ref import sqdk_dense_torch

    cores = use_all_host_cores()
    g = torch.Generator().manual_seed(42)
    B, S, H, hd, K = 2, 512, 4, 64, 102
    q, k, v = (torch.randn(B, S, H, hd, generator=g) for _ in range(3))
    idx = torch.stack([torch.sort(torch.randperm(S, generator=g)[:K])[0] for _ in range(B)])
    for _ in range(5):
        sqdk_dense_torch(q, k, v, idx)
    t0 = time.perf_counter()
    for _ in range(iters):
        sqdk_dense_torch(q, k, v, idx)
    return {"ms_per_call": (time.perf_counter() - t0) / iters * 1e3, "cores": cores,
            "sample": f"B={B} S={S} H={H} hd={hd} K={K} fp32, {iters} calls"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    steps = max(1, args.steps)
    ref = cpu_reference_sample(args, steps=steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": ref["value"], "unit": "tok/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ref["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": ref["value"] / PUBLISHED_TOK_S, "dtype": ref["dtype"],
        "data": "synthetic: x ~ N(0,1), default-init weights (seed 42)",
        "config": workload_config(args),
        "cpu_baseline": ref,
        "e2e": {"value": ref["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# distributed helpers
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


def init_dist(world, local_rank, always_group=False):
    """CUDA device of this rank; an NCCL process group when world > 1 (or,
    with ``always_group``, a one-rank group so the collective code path is
    the same at N=1)."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1 or always_group:
        if world == 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", str(29500 + (os.getpid() % 2000)))
            dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=300),
                                    device_id=dev)
        else:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    return dev


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


def free_cuda():
    import gc

    import torch

    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ---------------------------------------------------------------------------
# parity of the timed headline launch
# ---------------------------------------------------------------------------


def headline_parity(model, x):
    """Run one block forward with the SQDK call captured, then compare the
    first and last sequence of that (timed-shape) launch against the fp32
    oracle on the same inputs, and time the same launch on its own (inputs
    larger than L2), which is the kernel's figure against the burst peak."""
    import numpy as np
    import torch

    import oracle
    from hspmn_b200 import ops

    captured = {}
    real = ops.sqdk_fwd

    def capture(q, k, v, idx, scale):
        o = real(q, k, v, idx, scale)
        captured.update(q=q, k=k, v=v, idx=idx, o=o, scale=scale)
        return o

    ops.sqdk_fwd = capture
    try:
        with torch.no_grad():
            model(x)
        torch.cuda.synchronize()
    finally:
        ops.sqdk_fwd = real
    B = captured["q"].shape[0]
    res = {"launch_batch": B, "sequences": [0, B - 1]}
    with torch.no_grad():
        c = captured
        res["standalone_ms"] = _time_cuda(lambda: real(c["q"], c["k"], c["v"], c["idx"], c["scale"]), reps=10, warm=3)
    worst_max, worst_mean = 0.0, 0.0
    for b in (0, B - 1):
        q = captured["q"][b:b + 1].float().cpu().numpy()
        k = captured["k"][b:b + 1].float().cpu().numpy()
        v = captured["v"][b:b + 1].float().cpu().numpy()
        idx = captured["idx"][b:b + 1].cpu().numpy()
        ref = oracle.sqdk_fp32(q, k, v, idx, captured["scale"])
        err = np.abs(captured["o"][b:b + 1].float().cpu().numpy() - ref)
        worst_max, worst_mean = max(worst_max, float(err.max())), max(worst_mean, float(err.mean()))
    res.update(max_abs=worst_max, mean_abs=worst_mean, bar={"max_abs": 2e-2, "mean_abs": 2e-3},
               ok=bool(worst_max <= 2e-2 and worst_mean <= 2e-3))
    return res


# ---------------------------------------------------------------------------
# long context: one sequence, sequence-sharded over the ranks
# ---------------------------------------------------------------------------


def _long_block(args, S, dev, fp32_gate=False):
    import torch

    from hspmn_b200 import HSPMNBlock, HSPMNConfig, seed_everything

    seed_everything(42)
    cfg = HSPMNConfig(dim=args.dim, num_heads=args.heads, num_kv_heads=args.kv_heads, sparsity_k=args.sparsity,
                      max_seq_len=S)
    model = HSPMNBlock(cfg).to(dev, dtype=torch.bfloat16).eval()
    model.router.fp32_gate = fp32_gate
    return model


def long_parity(args, rank, world, dev):
    """Sequence-sharded forward over every rank at S=32768 against the plain
    one-GPU block forward on rank 0 (same weights and input on all ranks).
    The router's fp32 gate kernel is used on both sides: its logits depend
    only on their own row, so both sides select the same positions whatever
    GEMM shapes the projections get."""
    import torch
    import torch.distributed as dist

    from hspmn_b200.parallel import SequenceShardedBlock, ZigZagPlan

    S = LONG_PARITY_SEQ
    model = _long_block(args, S, dev, fp32_gate=True)
    g = torch.Generator(device=dev).manual_seed(3000)
    x = torch.randn(1, S, args.dim, device=dev, dtype=torch.bfloat16, generator=g)
    plan = ZigZagPlan(S, world)
    with torch.no_grad():
        y_local, aux = SequenceShardedBlock(model, plan).forward(plan.shard(x, rank))
        parts = torch.empty((world,) + tuple(y_local.shape), dtype=y_local.dtype, device=dev)
        dist.all_gather_into_tensor(parts, y_local.contiguous())
        res = None
        if rank == 0:
            y_ref, aux_ref = model(x)
            y = plan.unshard(list(parts.unbind(0)))
            err = (y.float() - y_ref.float()).abs()
            res = {"seq_len": S, "ranks": world, "max_abs": err.max().item(), "mean_abs": err.mean().item(),
                   "aux_abs": abs(aux.item() - aux_ref.item()), "bar": {"max_abs": 3e-2, "mean_abs": 1e-3},
                   "router_gate": "fp32 gate kernel (row-independent logits) on both sides"}
            res["ok"] = bool(res["max_abs"] <= 3e-2 and res["mean_abs"] <= 1e-3 and res["aux_abs"] <= 1e-3)
    del model, x, y_local, parts
    return res


def long_context(args, rank, world, dev, steps):
    """Timed S=262144 sequence-sharded forward (strong scaling: the same
    sequence whatever the rank count), then the K/V exchange timed alone."""
    import torch
    import torch.distributed as dist

    from hspmn_b200 import ops
    from hspmn_b200.parallel import SequenceShardedBlock, ZigZagPlan, _all_gather_rows_async

    S = LONG_SEQ
    model = _long_block(args, S, dev)
    plan = ZigZagPlan(S, world)
    sb = SequenceShardedBlock(model, plan)
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    x_local = torch.randn(1, 2 * plan.chunk, args.dim, device=dev, dtype=torch.bfloat16, generator=g)
    with torch.no_grad():
        for _ in range(3):
            sb.forward(x_local)
        barrier(world)
        launches0 = ops.LaunchStats.launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ops.KernelTimer() as kt:
            e0.record()
            for _ in range(steps):
                sb.forward(x_local)
            e1.record()
        torch.cuda.synchronize()
        launches = ops.LaunchStats.launches - launches0
        ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / steps
        kres = kt.results()
        sq = kres.get("sqdk_fwd", {"launches": 1, "ms": float("nan")})
        sq_ms = max_over_ranks(sq["ms"] / max(1, sq["launches"]), world, dev)
        # the K/V exchange alone: both all-gathers of one forward, nothing to overlap
        hd = args.dim // args.heads
        kv = torch.randn(1, 2 * plan.chunk, args.kv_heads, hd, device=dev, dtype=torch.bfloat16, generator=g)
        for _ in range(3):
            _all_gather_rows_async(kv, plan, None)()
        barrier(world)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        a0.record()
        for _ in range(reps):
            fk = _all_gather_rows_async(kv, plan, None)
            fv = _all_gather_rows_async(kv, plan, None)
            fk(), fv()
        a1.record()
        torch.cuda.synchronize()
        ag_ms = max_over_ranks(a0.elapsed_time(a1), world, dev) / reps
    recv_bytes = 2 * (world - 1) * 2 * plan.chunk * args.kv_heads * hd * 2
    res = {"seq_len": S, "ranks": world, "ms_per_forward": ms, "tok_s": S / (ms / 1e3),
           "scaling": "strong", "sqdk_ms_max_rank": sq_ms, "kv_exchange_ms": ag_ms,
           "kv_exchange_GB_s_per_rank": recv_bytes / (ag_ms / 1e3) / 1e9 if world > 1 else None,
           "kv_exchange_note": "K and V of all ranks into local HBM (all-gather + point-to-point), timed alone",
           "steps": steps, "gpu_launches": launches,
           "kernels_rank0": {n: {"launches": r["launches"], "ms_per_launch": r["ms"] / max(1, r["launches"])}
                             for n, r in kres.items()}}
    del model, sb, x_local, kv
    return res


# ---------------------------------------------------------------------------
# standalone SQDK sparsity sweep and GPU comparators
# ---------------------------------------------------------------------------


def _sqdk_flops(idx, H, hd):
    return 4.0 * hd * H * float((idx + 1).sum().item())


def _time_cuda(fn, reps=5, warm=2):
    import torch

    for _ in range(warm):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def gpu_comparators(q_sel, k, v, idx, scale, ours_ms, flops, eager=True):
    """The same SQDK attention through library kernels on this GPU: torch
    SDPA (memory-efficient and cuDNN backends) with a boolean [B,1,K,S] mask,
    and the reference's own dense-masked PyTorch pattern
    (test_kernels_v2_1.py:34-65) in bf16. K/V heads are repeated for grouped
    queries. Each result gives ms, algorithmic TFLOP/s (the same numerator as
    this library's kernel) and this library's speed-up over it."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    B, K, H, hd = q_sel.shape
    S = k.shape[1]
    G = H // k.shape[2]
    qh = q_sel.permute(0, 2, 1, 3)
    kh = k.repeat_interleave(G, dim=2).permute(0, 2, 1, 3) if G > 1 else k.permute(0, 2, 1, 3)
    vh = v.repeat_interleave(G, dim=2).permute(0, 2, 1, 3) if G > 1 else v.permute(0, 2, 1, 3)
    allowed = (torch.arange(S, device=idx.device)[None, None, None, :] <= idx[:, None, :, None])
    out = {}

    def record(name, fn):
        try:
            with torch.no_grad():
                ms = _time_cuda(fn)
            out[name] = {"ms": ms, "TFLOP_s": flops / (ms / 1e3) / 1e12, "ours_speedup": ms / ours_ms}
        except Exception as e:  # a backend that does not take this mask or shape
            out[name] = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:160]}"}
        torch.cuda.synchronize()

    for name, be in (("torch_sdpa_efficient", SDPBackend.EFFICIENT_ATTENTION),
                     ("torch_sdpa_cudnn", SDPBackend.CUDNN_ATTENTION)):
        def run(be=be):
            with sdpa_kernel([be]):
                return F.scaled_dot_product_attention(qh, kh, vh, attn_mask=allowed, scale=scale)
        record(name, run)
    if eager:
        def eager_pattern():
            s = torch.matmul(qh, kh.transpose(-2, -1)) * scale
            s = s.masked_fill(~allowed, float("-inf"))
            return torch.matmul(F.softmax(s, dim=-1), vh)
        record("torch_eager_reference_pattern", eager_pattern)
    out["note"] = ("library kernels on the same inputs and GPU; the reference's Triton kernel cannot be run here "
                   "(the reference is not pip-installable and its sources do not travel to the GPU box)")
    return out


def sqdk_sweep(args, dev, B=8, S=32768, H=16, Hkv=16, fracs=(0.05, 0.1, 0.2, 0.5), steps=None,
               comparators=(0.05, 0.2)):
    """Standalone router / gather / SQDK / scatter at B=8, S=32768, H=Hkv=16,
    hd=128 for each sparsity; returns one dict per k."""
    import torch

    from hspmn_b200 import ops

    hd = 128
    steps = steps or args.steps
    peaks, peak_src = load_peaks()
    g = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn(B, S, H, hd, device=dev, dtype=torch.bfloat16, generator=g)
    k = torch.randn(B, S, Hkv, hd, device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn(B, S, Hkv, hd, device=dev, dtype=torch.bfloat16, generator=g)
    logits = torch.randn(B, S, device=dev, dtype=torch.float32, generator=g)
    rows = []
    for frac in fracs:
        K = max(1, int(S * frac))

        def step():
            idx, _ = ops.router_topk(logits, None, K, torch.float32)
            qs = ops.gather_rows(q, idx)
            o = ops.sqdk_fwd(qs, k, v, idx, hd ** -0.5)
            return ops.scatter_rows(o, idx, S), idx, qs

        with torch.no_grad():
            for _ in range(args.warmup):
                _, idx, qs = step()
            flops = _sqdk_flops(idx, H, hd)
            torch.cuda.synchronize()
            with ops.KernelTimer() as kt:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(steps):
                    step()
                e1.record()
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        res = {n: r["ms"] / r["launches"] for n, r in kt.results().items()}
        tf = flops / (res["sqdk_fwd"] / 1e3) / 1e12
        gather_b = 2 * B * K * H * hd * 2 + B * K * 8
        scatter_b = B * K * H * hd * 2 + B * S * H * hd * 2 + B * K * 8
        router_b = B * S * 4 + B * K * 8 + B * S
        row = {"k": frac, "K": K, "sqdk_ms": res["sqdk_fwd"], "sqdk_TFLOP_s": tf,
               "sqdk_frac_of_burst_peak": tf / float(peaks["bf16_tflops"]),
               "router_us": res["router_topk"] * 1e3, "router_GB_s": router_b / (res["router_topk"] / 1e3) / 1e9,
               "gather_GB_s": gather_b / (res["gather_rows"] / 1e3) / 1e9,
               "scatter_GB_s": scatter_b / (res["scatter_rows"] / 1e3) / 1e9,
               "gather_frac_of_hbm": gather_b / (res["gather_rows"] / 1e3) / 1e9 / float(peaks["hbm_gbs"]),
               "scatter_frac_of_hbm": scatter_b / (res["scatter_rows"] / 1e3) / 1e9 / float(peaks["hbm_gbs"]),
               "ms_per_step": ms / steps}
        if frac in comparators:
            row["gpu_comparator"] = gpu_comparators(qs, k, v, idx, hd ** -0.5, res["sqdk_fwd"], flops,
                                                    eager=frac <= 0.05)
        rows.append(row)
        free_cuda()
    del q, k, v, logits
    return {"workload": f"B={B} S={S} H={H} Hkv={Hkv} hd={hd}, router on f32 logits",
            "peak_source": f"{peak_src} (bf16 burst, HBM copy)", "rows": rows}


# ---------------------------------------------------------------------------
# our arm: the block step
# ---------------------------------------------------------------------------


def run_block(args):
    import torch

    from hspmn_b200 import HSPMNBlock, HSPMNConfig, ops, seed_everything

    rank, world, local_rank = dist_env()
    dev = init_dist(world, local_rank, always_group=not args.no_extras)
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
            e2e_ms_rank = e0.elapsed_time(e1)
            e2e_ms = max_over_ranks(e2e_ms_rank, world, dev)
            bi = x_host.numel() * x_host.element_size()
            bo = out_host[0].numel() * out_host[0].element_size() + 2
            e2e = {"value": B * S * args.e2e_steps * world / (e2e_ms / 1e3), "unit": "tok/s",
                   "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
                   "pipeline": "2-deep: upload of step i+1 and download of step i-1 overlap forward i",
                   "steps": args.e2e_steps, "ms_per_step": e2e_ms / args.e2e_steps,
                   "host_link_GB_s_per_rank": (bi + bo) * args.e2e_steps / (e2e_ms / 1e3) / 1e9,
                   "host_link_GB_s_all_ranks": (bi + bo) * args.e2e_steps * world / (e2e_ms / 1e3) / 1e9}
            del x_host, out_host, x_dev

        # the opt-in fp32 gate kernel next to the module's cuBLAS gate (nn.Linear(dim, 1)),
        # both over the whole x (larger than L2) of this GPU
        gate_w, gate_b = model.router.gate.weight, model.router.gate.bias
        gate_times = {}
        for name, fn in (("gate_logits", lambda: ops.gate_logits(x, gate_w, gate_b)),
                         ("cublas_gate", lambda: model.router.gate(x))):
            gate_times[name] = _time_cuda(fn, reps=10, warm=3)

        extras = {}
        if not args.no_extras:
            if rank == 0:
                extras["headline_parity"] = headline_parity(model, x)
            del model, x
            free_cuda()
            barrier(world)
            extras["long_parity"] = long_parity(args, rank, world, dev)
            free_cuda()
            barrier(world)
            extras["long_context"] = long_context(args, rank, world, dev, args.long_steps)
            free_cuda()
            barrier(world)
            if world == 1:
                sweep = sqdk_sweep(args, dev)
                extras["sqdk_sweep"] = sweep
                free_cuda()
                # comparators at the headline attention shape (B=64, K=820, S=4096, GQA 4)
                extras["gpu_comparator_headline"] = headline_comparators(args, dev)
                free_cuda()
                # the training path's SQDK backward at the same attention shape
                extras["sqdk_bwd"] = sqdk_bwd_measure(args, dev, rank, world, local_rank, 10, 3)
                free_cuda()

    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    elif not args.no_extras:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks, peak_src = load_peaks()
    sq = kres.get("sqdk_fwd", {"launches": 0, "ms": float("nan")})
    sq_ms = sq["ms"] / max(1, sq["launches"])
    achieved = sqdk_flops / (sq_ms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    peak_sus = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    wl_tag = f"B{B}_S{S}_D{D}_H{args.heads}_Hkv{args.kv_heads}"
    traffic = profiled_traffic("sqdk_fwd", wl_tag)
    esz = 2
    kernels = {}
    for name, r in kres.items():
        per = r["ms"] / max(1, r["launches"])
        kernels[name] = {"launches": r["launches"], "ms_per_launch": per}
    hbm = float(peaks["hbm_gbs"])

    def gbs(name, nbytes):
        if name in kernels:
            v = nbytes / (kernels[name]["ms_per_launch"] / 1e3) / 1e9
            kernels[name]["GB_s"] = v
            kernels[name]["frac_of_hbm"] = v / hbm

    gbs("gather_rows", 2 * B * k_sel * D * esz + B * k_sel * 8)
    if "rope_gather_rows" in kernels:
        # the K routed query rows (D elements each, indices read)
        gbs("rope_gather_rows", 2 * B * k_sel * D * esz + B * k_sel * 8)
    if "rope_rows" in kernels:
        # RoPE over all S key rows (Hkv * hd elements each) in one pass, positions implied
        kv_row = (D // args.heads) * args.kv_heads
        gbs("rope_rows", 2 * B * S * kv_row * esz)
    gbs("scatter_add_rows", 3 * B * k_sel * D * esz + B * k_sel * 8)
    gbs("scatter_rows", B * k_sel * D * esz + B * S * D * esz + B * k_sel * 8)
    gbs("router_topk", B * S * esz + B * k_sel * 8 + B * S)
    if "sqdk_fwd" in kernels:
        kernels["sqdk_fwd"]["TFLOP_s"] = achieved
        kernels["sqdk_fwd"]["algorithmic_flops"] = sqdk_flops
    # gate GEMV: read x and w, write one logit per position (f32 here, bf16 from cuBLAS)
    gate = {}
    for name, out_bytes in (("gate_logits", 4), ("cublas_gate", esz)):
        gb = B * S * D * esz + D * esz + B * S * out_bytes
        ms = gate_times[name]
        gate[name] = {"ms_per_launch": ms, "GB_s": gb / (ms / 1e3) / 1e9, "frac_of_hbm": gb / (ms / 1e3) / 1e9 / hbm}

    sm_mhz = clock_info.get("sm_mhz") if clock_info else None
    standalone = None
    hp = extras.get("headline_parity")
    if hp and hp.get("standalone_ms"):
        st_ms = hp["standalone_ms"]
        st_tf = sqdk_flops / (st_ms / 1e3) / 1e12
        standalone = {"ms_per_launch": st_ms, "TFLOP_s": st_tf, "frac_of_burst_peak": st_tf / peak,
                      "note": "the timed launch's own inputs, timed alone (10 launches, inputs larger than L2)"}
    value = B * S * args.steps * world / (ms_total / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": value / PUBLISHED_TOK_S, "dtype": "bf16",
        "data": "synthetic: x ~ N(0,1), default-init weights (seed 42)",
        "config": workload_config(args),
        "roofline": {"bound": "tensor", "kernel": "sqdk_fwd", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_src} bf16 dense, burst (cuBLAS 8192^3 best of 10)",
                     "frac_of_sustained_peak": achieved / peak_sus,
                     "sustained_peak": peak_sus,
                     "sustained_peak_clock_mhz": (peaks.get("clocks_under_load") or {}).get("sm_mhz_median"),
                     "kernel_clock_mhz": sm_mhz,
                     "ms_x_mhz_per_launch": sq_ms * sm_mhz if sm_mhz else None,
                     "standalone": standalone,
                     "flops_per_launch": sqdk_flops, "ms_per_launch": sq_ms, "k_selected": k_sel},
        "kernels": kernels,
        "router_gate": dict(gate, note="opt-in fp32 gate (router.fp32_gate) vs the default cuBLAS bf16 gate; "
                                       "outside the timed step"),
        "gpu_launches": launches,
        "clocks": clock_info,
    }
    if e2e is not None:
        line["e2e"] = e2e
    line.update(extras)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_reference_sample(args, seconds=args.cpu_sample_seconds)
        line["cpu_baseline_oracle"] = cpu_oracle_sample(args, args.cpu_sample_seconds)
        line["cpu_sqdk_cfg1"] = cpu_sqdk_cfg1()
    print(json.dumps(line), flush=True)


def headline_comparators(args, dev):
    """Library comparators at the headline attention shape: this library's
    SQDK vs torch SDPA / the eager reference pattern on the same q_sel, K, V
    and indices (random sorted selection of K = int(S * k) rows)."""
    import torch

    from hspmn_b200 import ops

    B, S, H, Hkv = args.batch, args.seq_len, args.heads, args.kv_heads
    hd = args.dim // H
    K = max(1, int(S * args.sparsity))
    g = torch.Generator(device=dev).manual_seed(13)
    q = torch.randn(B, K, H, hd, device=dev, dtype=torch.bfloat16, generator=g)
    k = torch.randn(B, S, Hkv, hd, device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn(B, S, Hkv, hd, device=dev, dtype=torch.bfloat16, generator=g)
    idx = torch.sort(torch.rand(B, S, device=dev, generator=g).argsort(dim=1)[:, :K], dim=1)[0]
    scale = hd ** -0.5
    with torch.no_grad():
        ours = _time_cuda(lambda: ops.sqdk_fwd(q, k, v, idx, scale), reps=10, warm=3)
    flops = _sqdk_flops(idx, H, hd)
    res = gpu_comparators(q, k, v, idx, scale, ours, flops)
    res["ours"] = {"ms": ours, "TFLOP_s": flops / (ours / 1e3) / 1e12}
    res["workload"] = f"SQDK B={B} K={K} S={S} H={H} Hkv={Hkv} hd={hd} (random sorted selection)"
    return res


# ---------------------------------------------------------------------------
# standalone workloads
# ---------------------------------------------------------------------------


def run_sweep(args, B=8, S=32768, H=16, Hkv=16, fracs=(0.05, 0.1, 0.2, 0.5)):
    rank, world, local_rank = dist_env()
    dev = init_dist(world, local_rank)
    comparators = () if args.no_extras else (fracs if len(fracs) == 1 else (0.05, 0.2))
    res = sqdk_sweep(args, dev, B, S, H, Hkv, fracs, comparators=comparators)
    if rank == 0:
        for row in res["rows"]:
            print(json.dumps({"metric": "standalone SQDK: attention TFLOP/s and gather/scatter GB/s",
                              "workload": res["workload"] + f", k={row['k']} (K={row['K']})", "n_gpus": 1,
                              "value": row["sqdk_TFLOP_s"], "unit": "TFLOP/s", "peak_source": res["peak_source"],
                              **row}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def sqdk_bwd_measure(args, dev, rank, world, local_rank, steps, warmup):
    """Backward of the SQDK attention at the block's attention shape
    (--batch/--seq-len/--heads/--kv-heads/--sparsity, hd = dim / heads): the
    selected rows of a random sorted selection, the forward with log-sum-exp
    once, then timed launches of the backward (rowsum(dO*O), the key-block
    kernel, the dq cast). Algorithmic FLOPs: 10 * hd per (row, visible key)
    (S^T, dP^T, dV, dK, dQ), i.e. 2.5 x the forward's. Returns rank 0's
    figures (max over ranks) and the clocks seen under the same launches."""
    import torch

    from hspmn_b200 import ops

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
        for _ in range(warmup):
            ops.sqdk_bwd(q, k, v, idx, o, d_o, lse, scale)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            ops.sqdk_bwd(q, k, v, idx, o, d_o, lse, scale)
        e1.record()
        torch.cuda.synchronize()
        # clocks and power under the same launches, over about a second (the
        # timed steps alone are shorter than nvidia-smi's sampling period)
        clocks = ClockSampler([local_rank]) if rank == 0 else None
        if clocks:
            clocks.start()
        barrier(world)
        reps = max(1, int(1500.0 / max(e0.elapsed_time(e1) / steps, 0.05)))
        for _ in range(reps):
            ops.sqdk_bwd(q, k, v, idx, o, d_o, lse, scale)
        torch.cuda.synchronize()
        clock_info = clocks.stop() if clocks else None
        assert ops.device_errors(dev) == 0
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / steps
    tf = flops / (ms / 1e3) / 1e12
    peak = float(peaks["bf16_tflops"])
    return {"workload": f"SQDK backward B={B} S={S} H={H} Hkv={Hkv} hd={hd} k={args.sparsity} (K={K}) per GPU",
            "ms_per_launch": ms, "TFLOP_s": tf, "frac_of_burst_peak": tf / peak,
            "frac_of_sustained_peak": tf / float(peaks.get("bf16_tflops_sustained",
                                                            FALLBACK_PEAKS["bf16_tflops_sustained"])),
            "peak": peak, "peak_source": f"{peak_src} bf16 dense, burst", "flops_per_launch": flops,
            "launches_timed": steps, "clocks": clock_info}


def run_sqdk_bwd(args):
    """The SQDK backward alone (see sqdk_bwd_measure), one JSON line."""
    rank, world, local_rank = dist_env()
    dev = init_dist(world, local_rank)
    res = sqdk_bwd_measure(args, dev, rank, world, local_rank, args.steps, args.warmup)
    if rank == 0:
        tf = res["TFLOP_s"] * world
        print(json.dumps({
            "metric": "SQDK backward: attention-gradient TFLOP/s", "value": tf, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_launch"],
            "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic: N(0,1) q/k/v/dO, "
            "random sorted selection", "config": {"workload": res["workload"]},
            "roofline": {"bound": "tensor", "achieved": res["TFLOP_s"], "peak": res["peak"], "unit": "TFLOP/s",
                         "frac": res["frac_of_burst_peak"], "peak_source": res["peak_source"],
                         "frac_of_sustained_peak": res["frac_of_sustained_peak"],
                         "flops_per_launch": res["flops_per_launch"]},
            "clocks": res["clocks"]}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_long(args):
    import torch.distributed as dist

    rank, world, local_rank = dist_env()
    dev = init_dist(world, local_rank, always_group=True)
    par = long_parity(args, rank, world, dev)
    free_cuda()
    barrier(world)
    res = long_context(args, rank, world, dev, args.long_steps)
    barrier(world)
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": "long-context HSPMNBlock tok/s (one sequence, sequence-sharded)", "value": res["tok_s"],
            "unit": "tok/s", "n_gpus": world, "steps": res["steps"], "ms_per_step": res["ms_per_forward"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: x ~ N(0,1), default-init weights (seed 42)",
            "config": {"workload": f"HSPMNBlock eval forward, B=1 S={LONG_SEQ} dim={args.dim} heads={args.heads} "
                                   f"kv_heads={args.kv_heads} k={args.sparsity}, zig-zag sequence shards",
                       "seq_len": LONG_SEQ, "parallelism": f"sequence-sharded x{world}"},
            "long_context": res, "long_parity": par}), flush=True)


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
