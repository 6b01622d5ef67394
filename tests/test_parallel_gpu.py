"""Sequence-sharded forward on the GPU (one-rank NCCL group) vs the plain
block forward: the same kernels, so the outputs agree to bf16 rounding."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist

from hspmn_b200 import HSPMNBlock, HSPMNConfig
from hspmn_b200.parallel import SequenceShardedBlock, ZigZagPlan

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_world1_matches_block():
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_port())
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", 0))
    try:
        torch.manual_seed(3)
        S = 4096
        block = HSPMNBlock(HSPMNConfig(dim=1024, num_heads=8, num_kv_heads=2, max_seq_len=S)).cuda()
        block = block.to(torch.bfloat16).eval()
        with torch.no_grad():
            block.router.gate.weight.normal_(0, 1024 ** -0.5)
        x = torch.randn(1, S, 1024, device="cuda", dtype=torch.bfloat16)
        plan = ZigZagPlan(S, 1)
        with torch.no_grad():
            y_ref, aux_ref = block(x)
            y, aux = SequenceShardedBlock(block, plan).forward(plan.shard(x, 0))
        err = (y.float() - y_ref.float()).abs()
        assert err.max().item() <= 3e-2 and err.mean().item() <= 1e-3, (err.max().item(), err.mean().item())
        assert abs(aux.item() - aux_ref.item()) <= 1e-3
    finally:
        dist.destroy_process_group()
