"""hspmn_sqdk_fwd_noalloc, called through the C ABI, against hspmn_sqdk_fwd
with a caller workspace on the same inputs.

Each case makes two calls in a row on the same shape with different inputs,
so a partial left in the static scratch by the first call would show up in
the second. Tolerance as for the SQDK parity tests: max |diff| <= 2e-2 and
mean |diff| <= 2e-3 (the two entry points run the same kernels and split, so
the results are expected to agree exactly). This file is collected last so
it also runs after every other GPU test in one process.
"""

import ctypes

import pytest
import torch

from hspmn_b200 import _native as N

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_ABS, MEAN_ABS = 2e-2, 2e-3
ERR_SCRATCH = -7
SCRATCH_BYTES = 32 << 20


def _strides(t):
    return N.i64_array(t.stride())


def _inputs(B, S, H, Hkv, hd, K, seed, dtype=torch.bfloat16):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(B, K, H, hd, generator=g, device=DEV).to(dtype)
    k = torch.randn(B, S, Hkv, hd, generator=g, device=DEV).to(dtype)
    v = torch.randn(B, S, Hkv, hd, generator=g, device=DEV).to(dtype)
    idx = torch.stack([torch.randperm(S, generator=g, device=DEV)[:K] for _ in range(B)]).sort(dim=1).values
    return q, k, v, idx.contiguous()


def _call(noalloc, q, k, v, idx, o, S, Hkv, workspace=None):
    B, K, H, hd = q.shape
    lib = N.lib()
    dt = N.HSPMN_BF16 if q.dtype == torch.bfloat16 else N.HSPMN_F16
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [ctypes.c_void_p(q.data_ptr()), _strides(q), ctypes.c_void_p(k.data_ptr()), _strides(k),
            ctypes.c_void_p(v.data_ptr()), _strides(v), ctypes.c_void_p(idx.data_ptr()), idx.stride(0),
            idx.stride(1), ctypes.c_void_p(o.data_ptr()), _strides(o), B, K, S, H, Hkv, hd, dt,
            ctypes.c_float(hd ** -0.5)]
    if noalloc:
        return lib.hspmn_sqdk_fwd_noalloc(*args, st)
    ws_ptr = ctypes.c_void_p(workspace.data_ptr()) if workspace is not None else None
    ws_bytes = workspace.numel() if workspace is not None else 0
    return lib.hspmn_sqdk_fwd(*args, ws_ptr, ws_bytes, st)


def _workspace_bytes(B, K, S, H, Hkv, hd):
    n = N.lib().hspmn_sqdk_workspace_size(B, K, S, H, Hkv, hd)
    assert n >= 0
    return n


@pytest.mark.parametrize("B,S,H,Hkv,hd,K", [
    (1, 4096, 16, 4, 128, 819),   # one sequence: keys split over several CTAs, scratch in use
    (2, 2048, 8, 2, 64, 300),     # split, 64-wide head tile
    (3, 1000, 16, 4, 128, 200),   # split, ragged last tile
    (8, 4096, 16, 4, 128, 819),   # enough tiles for no split: scratch untouched
])
def test_noalloc_matches_workspace_entry(B, S, H, Hkv, hd, K):
    ws_bytes = _workspace_bytes(B, K, S, H, Hkv, hd)
    assert ws_bytes <= SCRATCH_BYTES
    for call in range(2):
        q, k, v, idx = _inputs(B, S, H, Hkv, hd, K, seed=1000 * call + S + K + hd)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV) if ws_bytes else None
        o_ref = torch.empty_like(q)
        o = torch.full_like(q, float("nan"))
        assert _call(False, q, k, v, idx, o_ref, S, Hkv, ws) == 0
        rc = _call(True, q, k, v, idx, o, S, Hkv)
        assert rc == 0, N.strerror(rc)
        torch.cuda.synchronize()
        assert N.device_errors() == 0
        assert torch.isfinite(o).all(), f"call {call}"
        err = (o.float() - o_ref.float()).abs()
        assert err.max().item() <= MAX_ABS and err.mean().item() <= MEAN_ABS, \
            f"call {call}: max={err.max().item():.3e} mean={err.mean().item():.3e}"


def test_noalloc_allocates_nothing():
    B, S, H, Hkv, hd, K = 1, 4096, 16, 4, 128, 819
    assert _workspace_bytes(B, K, S, H, Hkv, hd) > 0
    q, k, v, idx = _inputs(B, S, H, Hkv, hd, K, seed=7)
    o = torch.empty_like(q)
    assert _call(True, q, k, v, idx, o, S, Hkv) == 0  # first split launch on the device: scratch lookup
    torch.cuda.synchronize()

    def calls_leave_memory_alone():
        allocs0 = torch.cuda.memory_stats()["allocation.all.allocated"]
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(2):
            assert _call(True, q, k, v, idx, o, S, Hkv) == 0
        torch.cuda.synchronize()
        # the caching allocator served nothing, and the device's free memory
        # (which other work on the device could also move) did not drop
        assert torch.cuda.memory_stats()["allocation.all.allocated"] == allocs0
        return torch.cuda.mem_get_info()[0] == free0

    assert calls_leave_memory_alone() or calls_leave_memory_alone()
    assert N.device_errors() == 0


def test_noalloc_rejects_shape_beyond_scratch():
    # 256 tiles of 128 rows at hd=128: two key shares each, 34 MB of partials
    # on a 148-SM part. The rule is checked against the workspace size so the
    # test holds on any SM count.
    B, S, H, Hkv, hd, K = 1, 4096, 16, 4, 128, 2048
    need = _workspace_bytes(B, K, S, H, Hkv, hd)
    q, k, v, idx = _inputs(B, S, H, Hkv, hd, K, seed=11)
    o = torch.zeros_like(q)
    rc = _call(True, q, k, v, idx, o, S, Hkv)
    if need > SCRATCH_BYTES:
        assert rc == ERR_SCRATCH
        assert "scratch" in N.strerror(rc)
        torch.cuda.synchronize()
        assert (o == 0).all()  # nothing launched
    else:
        assert rc == 0
