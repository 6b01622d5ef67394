"""Loading helpers for the committed golden fixtures (tests/golden/*.npz)."""

import json
import os

import numpy as np

from tests.golden.inputs import block_params, normal_f16_exact, sha256_of

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def sqdk_inputs(fx):
    """Regenerate q [B,S,H,hd], k, v [B,S,Hkv,hd] of an SQDK fixture and check
    them against the stored hash."""
    seed = int(fx["seed"])
    B, S, H, Hkv, hd = (int(x) for x in fx["shape"])
    q = normal_f16_exact(seed, (B, S, H, hd))
    k = normal_f16_exact(seed + 1, (B, S, Hkv, hd))
    v = normal_f16_exact(seed + 2, (B, S, Hkv, hd))
    assert sha256_of(q, k, v) == fx["qkv_sha"].item().decode(), "input generator drifted"
    return q, k, v


def block_inputs(fx, shapes):
    cfg = json.loads(fx["cfg"].item().decode())
    x = normal_f16_exact(int(fx["seed"]), (cfg["B"], cfg["S"], cfg["dim"]))
    assert sha256_of(x) == fx["x_sha"].item().decode(), "input generator drifted"
    params = block_params(shapes, int(fx["seed"]))
    assert sha256_of(*[params[k] for k in sorted(params)]) == fx["params_sha"].item().decode()
    return cfg, x, params


def block_shapes(dim, num_heads, num_kv_heads, mlp_ratio=4):
    """state_dict names and shapes of an HSPMNBlock (hspmn_v2_1.py:148-166)."""
    hd = dim // num_heads
    kv = num_kv_heads * hd
    hid = dim * mlp_ratio
    return {
        "router.log_temp": (1,), "router.target_sparsity": (),
        "router.gate.weight": (1, dim), "router.gate.bias": (1,),
        "norm.weight": (dim,), "q_proj.weight": (dim, dim), "k_proj.weight": (kv, dim),
        "v_proj.weight": (kv, dim), "o_proj.weight": (dim, dim),
        "reflexive.conv.weight": (dim, 1, 3), "reflexive.norm.weight": (dim,),
        "reflexive.gate_proj.weight": (hid, dim), "reflexive.up_proj.weight": (hid, dim),
        "reflexive.down_proj.weight": (dim, hid),
    }
