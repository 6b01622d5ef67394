"""Configuration and environment helpers (mirror of utils_v2_1.py).

``HSPMNConfig`` keeps the reference's field names, defaults and derived
fields (utils_v2_1.py:35-54) so configs and checkpoints move across.
"""

from __future__ import annotations

import logging
import random
from dataclasses import dataclass

import numpy as np
import torch


def setup_env() -> None:
    """TF32 matmuls and cuDNN autotuning, as utils_v2_1.py:7-11."""
    torch.set_float32_matmul_precision("high")
    torch.backends.cudnn.benchmark = True
    torch.backends.cuda.matmul.allow_tf32 = True


def get_device() -> torch.device:
    """utils_v2_1.py:13-17."""
    return torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")


def setup_logging(name: str = __name__) -> logging.Logger:
    """utils_v2_1.py:19-26."""
    logging.basicConfig(level=logging.INFO, format="%(asctime)s | %(levelname)s | %(message)s",
                        datefmt="%Y-%m-%d %H:%M:%S")
    return logging.getLogger(name)


def seed_everything(seed: int = 42) -> None:
    """utils_v2_1.py:28-33."""
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    torch.cuda.manual_seed_all(seed)


@dataclass
class HSPMNConfig:
    """Configuration of an HSPMN v2.1 block (utils_v2_1.py:35-54)."""

    dim: int = 768
    num_heads: int = 12
    num_kv_heads: int = 4
    sparsity_k: float = 0.2
    mlp_ratio: int = 4
    max_seq_len: int = 16384
    rope_base: int = 10000
    block_size: int = 128
    router_temp_init: float = 1.0
    router_sparsity_coef: float = 0.1
    router_entropy_coef: float = 0.01

    def __post_init__(self):
        assert self.dim % self.num_heads == 0, "Dim must be divisible by num_heads"
        assert self.num_heads % self.num_kv_heads == 0, "Heads must be divisible by KV heads (GQA)"
        self.head_dim = self.dim // self.num_heads
        self.kv_groups = self.num_heads // self.num_kv_heads
