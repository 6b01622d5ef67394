"""Seeded input generator shared by the golden-fixture script and the tests.

Values are N(0,1) draws rounded to IEEE half and returned as float32, so the
same numbers are exactly representable in float32, float16 and (after the
kernels' own rounding) comparable across dtypes. The fixtures store the
SHA-256 of what this produced at generation time; ``sha256_of`` recomputes it.
"""

import hashlib

import numpy as np


def normal_f16_exact(seed: int, shape) -> np.ndarray:
    rng = np.random.default_rng(int(seed))
    return rng.standard_normal(size=tuple(shape), dtype=np.float32).astype(np.float16).astype(np.float32)


def sha256_of(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    return h.hexdigest()


def block_params(shapes: dict, seed: int) -> dict:
    """Seeded, fp16-exact values for every HSPMNBlock parameter.

    ``shapes`` maps state_dict names to shapes (identical for the reference
    block and this library's block). Matrices are scaled by a power of two
    near 1/sqrt(fan_in) so the values stay exact; norm weights sit around 1
    and the router temperature parameter is -0.25. The ``target_sparsity``
    buffer is left to the module."""
    out = {}
    for j, name in enumerate(sorted(shapes)):
        shape = tuple(shapes[name])
        if name.endswith("target_sparsity"):
            continue
        a = normal_f16_exact(seed * 1000 + j, shape)
        if name.endswith("norm.weight"):
            a = 1.0 + a * np.float32(0.125)
        elif name.endswith("log_temp"):
            a = np.full(shape, -0.25, dtype=np.float32)
        elif len(shape) >= 2:
            fan_in = int(np.prod(shape[1:]))
            a = a * np.float32(2.0 ** -np.ceil(np.log2(np.sqrt(fan_in))))
        out[name] = a.astype(np.float32)
    return out
