"""Sequence-sharded forward over two GPUs (two NCCL ranks) vs the plain block
forward on one GPU: the routed queries, the all-gathered K/V prefix and the
halo rows of the reflexive stream must reassemble the single-GPU result.
Skipped where fewer than two GPUs are visible."""

import datetime
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hspmn_b200 import HSPMNBlock, HSPMNConfig
from hspmn_b200.parallel import SequenceShardedBlock, ZigZagPlan

pytestmark = pytest.mark.gpu
S, DIM, H, HKV = 8192, 1024, 8, 2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _block(dev):
    torch.manual_seed(3)
    block = HSPMNBlock(HSPMNConfig(dim=DIM, num_heads=H, num_kv_heads=HKV, max_seq_len=S))
    with torch.no_grad():
        block.router.gate.weight.normal_(0, DIM ** -0.5)
    return block.to(dev, dtype=torch.bfloat16).eval()


def _input():
    g = torch.Generator().manual_seed(4)
    return torch.randn(1, S, DIM, generator=g).to(torch.bfloat16)


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        block = _block(dev)
        x = _input().to(dev)
        plan = ZigZagPlan(S, world)
        with torch.no_grad():
            y_local, aux = SequenceShardedBlock(block, plan).forward(plan.shard(x, rank))
        parts = [torch.empty_like(y_local) for _ in range(world)]
        dist.all_gather(parts, y_local.contiguous())
        if rank == 0:
            with torch.no_grad():
                y_ref, aux_ref = block(x)
            err = (plan.unshard(parts).float() - y_ref.float()).abs()
            torch.save({"max": err.max().item(), "mean": err.mean().item(),
                        "aux": abs(aux.item() - aux_ref.item())}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_sequence_sharded_two_gpus_matches_block():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "err.pt")
        mp.start_processes(_worker, args=(2, _port(), out), nprocs=2, start_method="spawn", join=True)
        res = torch.load(out)
    assert res["max"] <= 3e-2 and res["mean"] <= 1e-3, res
    assert res["aux"] <= 1e-3, res
