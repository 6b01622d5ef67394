"""Multi-process (gloo, CPU) tests of the multi-GPU host logic.

The sequence-sharded forward runs here with the CUDA operators replaced by an
oracle-backed shim (test-only), so the chunk plan, the logits / K/V
all-gathers, the local selection, the halo exchange of the reflexive conv and
the reassembly are checked against the single-process oracle block forward.
"""

import os
import socket
import tempfile
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from hspmn_b200 import HSPMNBlock, HSPMNConfig
from hspmn_b200.parallel import SequenceShardedBlock, ZigZagPlan, batch_slice
from tests.golden.inputs import block_params, normal_f16_exact


class OracleOps:
    """CPU stand-ins for hspmn_b200.ops built on the oracle (tests only)."""

    @staticmethod
    def router_topk(logits, temp, k, noisy_dtype):
        name = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[noisy_dtype]
        noisy = oracle.noisy_logits(logits.float().numpy(), float(temp.float()), name)
        idx, mask = oracle.router_topk(noisy, k, name)
        return torch.from_numpy(idx), torch.from_numpy(mask)

    @staticmethod
    def gather_rows(src, idx):
        return torch.from_numpy(oracle.gather_rows(src.float().numpy(), idx.numpy())).to(src.dtype)

    @staticmethod
    def sqdk_fwd(q, k, v, idx, scale):
        o = oracle.sqdk_fp32(q.float().numpy(), k.float().numpy(), v.float().numpy(), idx.numpy(), scale)
        return torch.from_numpy(o).to(q.dtype)

    @staticmethod
    def scatter_rows(src, idx, S):
        return torch.from_numpy(oracle.scatter_rows(src.float().numpy(), idx.numpy(), S)).to(src.dtype)

    @staticmethod
    def rope_gather_rows(src, idx, cos, sin, by_position):
        hd = src.shape[-1]
        c, s = cos.reshape(-1, hd).float().numpy(), sin.reshape(-1, hd).float().numpy()
        rows = oracle.gather_rows(src.float().numpy(), idx.numpy()) if by_position else src.float().numpy()
        ix = idx.numpy()
        out = np.stack([oracle.rope_rounded(rows[b], c[ix[b]][:, None, :], s[ix[b]][:, None, :], "f32")
                        for b in range(rows.shape[0])])
        return torch.from_numpy(out).to(src.dtype)

    @staticmethod
    def scatter_add_rows_(dst, idx, src):
        for b in range(dst.shape[0]):
            dst[b, idx[b]] += src[b]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make_block(dim, H, Hkv, S, sparsity, seed):
    cfg = HSPMNConfig(dim=dim, num_heads=H, num_kv_heads=Hkv, sparsity_k=sparsity, max_seq_len=S)
    block = HSPMNBlock(cfg).eval()
    shapes = {k: tuple(v.shape) for k, v in block.state_dict().items()}
    params = block_params(shapes, seed)
    sd = block.state_dict()
    sd.update({k: torch.from_numpy(v) for k, v in params.items()})
    block.load_state_dict(sd)
    return block, params


def _sharded_worker(rank, world, port, out_path, dim, H, Hkv, S, sparsity):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        block, _ = _make_block(dim, H, Hkv, S, sparsity, seed=77)
        x = torch.from_numpy(normal_f16_exact(5, (1, S, dim)))
        plan = ZigZagPlan(S, world)
        sb = SequenceShardedBlock(block, plan, ops=OracleOps())
        y_local, aux = sb.forward(plan.shard(x, rank))
        parts = [torch.empty_like(y_local) for _ in range(world)]
        dist.all_gather(parts, y_local)
        if rank == 0:
            torch.save({"y": plan.unshard(parts), "aux": aux}, out_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 4])
def test_sequence_sharded_forward_matches_oracle(world):
    dim, H, Hkv, S, sparsity = 32, 4, 2, 64, 0.25
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "y.pt")
        mp.start_processes(_sharded_worker, args=(world, _free_port(), out, dim, H, Hkv, S, sparsity),
                           nprocs=world, start_method="spawn", join=True)
        res = torch.load(out)
    _, params = _make_block(dim, H, Hkv, S, sparsity, seed=77)
    x = normal_f16_exact(5, (1, S, dim))
    ts = float(torch.tensor(sparsity).item())
    ref, _, _, _ = oracle.block_forward(params, x, H, Hkv, ts, 10000, float(np.finfo(np.float32).eps))
    np.testing.assert_allclose(res["y"].numpy(), ref, atol=2e-5, rtol=1e-4)


def test_zigzag_plan_roundtrip_and_balance():
    plan = ZigZagPlan(4096, 4)
    x = torch.arange(4096).view(1, -1)
    parts = [plan.shard(x, r) for r in range(4)]
    assert torch.equal(plan.unshard(parts), x)
    # causal work per rank (sum of positions) is equal under zig-zag
    work = [int(plan.local_positions(r).sum()) for r in range(4)]
    assert max(work) == min(work)
    with pytest.raises(ValueError):
        ZigZagPlan(100, 3)


def test_batch_slice_covers_batch():
    for gb, w in [(64, 8), (10, 4), (3, 4)]:
        sl = [batch_slice(gb, r, w) for r in range(w)]
        assert sum(s.stop - s.start for s in sl) == gb and sl[0].start == 0 and sl[-1].stop == gb


def _dropout_worker(rank, world, port, flag_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    if rank == 1:
        # this rank leaves between steps, before the next collective
        os._exit(0)
    try:
        out = [torch.empty(4) for _ in range(world)]
        dist.all_gather(out, t)
        status = "no-error"
    except Exception as e:  # the survivor must see an error, not hang
        status = "error:" + type(e).__name__
    with open(flag_path, "w") as f:
        f.write(status)
    os._exit(0)


def test_rank_dropout_surfaces_as_error():
    with tempfile.TemporaryDirectory() as td:
        flag = os.path.join(td, "status")
        ctx = mp.start_processes(_dropout_worker, args=(2, _free_port(), flag), nprocs=2,
                                 start_method="spawn", join=False)
        deadline = time.time() + 120
        while time.time() < deadline and any(p.is_alive() for p in ctx.processes):
            time.sleep(0.2)
        for p in ctx.processes:
            if p.is_alive():
                p.kill()
        assert os.path.exists(flag), "the surviving rank neither finished nor reported an error"
        status = open(flag).read()
    assert status.startswith("error:"), status
