"""The oracle's fp32 router gate (CPU only).

It is pinned three ways before it is trusted for the kernel's bit-exact test:
against the reference TopKRouter's own logits (router fixtures), against a
literal loop over the defined lane/slot order, and its float64 fused
multiply-add emulation against exact rational arithmetic.
"""

from fractions import Fraction

import numpy as np
import pytest

import oracle
from tests import golden_io as G
from tests.golden.inputs import normal_f16_exact, sha256_of


@pytest.mark.parametrize("name", ["router_f32_B2_S512.npz", "router_bf16_B2_S4096.npz"])
def test_gate_against_reference_router_logits(name):
    """The reference gate (nn.Linear(dim, 1) in the module dtype) is the fp32
    gate rounded to that dtype: bf16 logits agree after rounding up to one
    bf16 step where the two sums straddle a rounding boundary; f32 logits
    agree within twice the summation error bound."""
    fx = G.load(name)
    B, S, D = (int(v) for v in fx["shape"])
    dt = "bf16" if fx["dtype"].item().decode() == "bfloat16" else "f32"
    x = normal_f16_exact(int(fx["seed"]), (B, S, D))
    if dt == "bf16":
        x = oracle.bf16_round(x)
    assert sha256_of(x) == fx["x_sha"].item().decode(), "input generator drifted"
    w, b = fx["gate_w"].reshape(-1), float(fx["gate_b"][0])
    got = oracle.gate_logits_fp32(x, w, b, dt)
    ref = fx["logits"]
    if dt == "bf16":
        rounded = oracle.bf16_round(got)
        diff = rounded != ref
        assert diff.mean() <= 1e-3, diff.sum()
        step = np.abs(ref) * 2.0 ** -7
        assert (np.abs(rounded - ref) <= step + 1e-30).all()
    else:
        bound = oracle.gate_error_bound(x, w, b)
        assert (np.abs(got.astype(np.float64) - ref) <= 2 * bound).all()


def _gate_loop(x_row, w, bias, E):
    """The defined order written as plain loops over lanes, vectors and slots."""
    D = len(x_row)
    nvec = D // E
    lanes = []
    for lane in range(32):
        acc = [np.float32(0.0)] * E
        for v in range(lane, nvec, 32):
            for e in range(E):
                d = v * E + e
                acc[e] = np.float32(np.float64(acc[e]) + np.float64(x_row[d]) * np.float64(w[d]))
        if E == 4:
            t = (acc[0] + acc[1]) + (acc[2] + acc[3])
        else:
            t = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]))
        lanes.append(np.float32(t))
    for o in (16, 8, 4, 2, 1):
        lanes = [np.float32(lanes[i] + lanes[i ^ o]) for i in range(32)]
    return np.float32(lanes[0] + np.float32(0.0 if bias is None else bias))


@pytest.mark.parametrize("dt,D", [("bf16", 8), ("bf16", 264), ("f16", 1000), ("f32", 4), ("f32", 260)])
def test_gate_matches_literal_loop(dt, D):
    rng = np.random.default_rng(D)
    x = oracle.round_to(rng.standard_normal((3, D)).astype(np.float32), dt)
    w = oracle.round_to((rng.standard_normal(D) * D ** -0.5).astype(np.float32), dt)
    E = 4 if dt == "f32" else 8
    for bias in (None, 0.375):
        got = oracle.gate_logits_fp32(x, w, bias, dt)
        for r in range(3):
            assert got[r].view(np.uint32) == _gate_loop(x[r], w, bias, E).view(np.uint32)


def _round_f32_exact(q: Fraction) -> np.float32:
    """Round a rational to float32, nearest with ties to even, subnormals and
    overflow included."""
    if q == 0:
        return np.float32(0.0)
    sign = -1 if q < 0 else 1
    a = abs(q)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    if Fraction(2) ** (e + 1) <= a:
        e += 1
    quantum = max(e - 23, -149)
    scaled = a / Fraction(2) ** quantum
    n = scaled.numerator // scaled.denominator
    rem = scaled - n
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2 == 1):
        n += 1
    val = Fraction(n) * Fraction(2) ** quantum
    if val >= Fraction(2) ** 128:
        return np.float32(sign * np.inf)
    return np.float32(sign * float(val))


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_fma_emulation_is_exact_for_16bit_products(dt):
    """float32(float64(acc) + float64(x) * float64(w)) equals the correctly
    rounded acc + x*w for 16-bit x, w and any float32 acc, across exponents
    from the subnormal range to near overflow."""
    rng = np.random.default_rng(7 if dt == "bf16" else 8)
    n = 4000
    lo, hi = (-140, 60) if dt == "bf16" else (-24, 15)
    x = oracle.round_to((rng.standard_normal(n) * 2.0 ** rng.integers(lo, hi, n)).astype(np.float32), dt)
    w = oracle.round_to((rng.standard_normal(n) * 2.0 ** rng.integers(lo, hi, n)).astype(np.float32), dt)
    acc = (rng.standard_normal(n) * 2.0 ** rng.integers(-149, 120, n)).astype(np.float32)
    acc[::7] = (-(x[::7].astype(np.float64) * w[::7].astype(np.float64))).astype(np.float32)  # near-cancellation
    emu = (acc.astype(np.float64) + x.astype(np.float64) * w.astype(np.float64)).astype(np.float32)
    for i in range(n):
        exact = _round_f32_exact(Fraction(float(acc[i])) + Fraction(float(x[i])) * Fraction(float(w[i])))
        assert emu[i] == exact or (np.isinf(exact) and emu[i] == exact), (i, acc[i], x[i], w[i])


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_gate_within_error_bound(dt):
    rng = np.random.default_rng(3)
    D = 2048
    x = oracle.round_to((rng.standard_normal((64, D)) * 3).astype(np.float32), dt)
    w = oracle.round_to((rng.standard_normal(D) * D ** -0.5).astype(np.float32), dt)
    got = oracle.gate_logits_fp32(x, w, -0.25, dt)
    exact = x.astype(np.float64) @ w.astype(np.float64) - 0.25
    assert (np.abs(got - exact) <= oracle.gate_error_bound(x, w, -0.25)).all()
