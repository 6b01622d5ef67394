"""CPU oracle for the HSPMN v2.1 contextual-stream inference path.

TEST INFRASTRUCTURE ONLY. This package restates, in numpy, the reference
algorithm for router top-K -> gather -> sparse-query dense-key (SQDK) causal
attention -> scatter, plus the surrounding HSPMNBlock forward. It is the
reference the CUDA library is tested against: only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm may import it. The product package
(``hspmn_b200``) never imports it and has no CPU fallback.

Parity is pinned against fixtures generated from the reference itself
(``tests/golden/make_golden.py``): its TopKRouter, its dense-masked PyTorch
SQDK test pattern and its eager-Flex HSPMNBlock forward. The one thing the
reference leaves unspecified is the order of tied router logits; the oracle
fixes it as "higher value first, lower position first among equals".
"""

from .sqdk_oracle import (  # noqa: F401
    bf16_round,
    f16_round,
    round_to,
    router_k,
    orderable_keys,
    noisy_logits,
    gate_logits_fp32,
    gate_error_bound,
    router_topk,
    gather_rows,
    scatter_rows,
    sqdk_fp32,
    sqdk_bwd_fp32,
    attention_flops,
    rms_norm,
    rope_tables,
    apply_rope,
    rope_rounded,
    block_forward,
)
