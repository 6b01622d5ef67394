"""The C-ABI library: it loads, exports exactly what include/*.h declares and
rejects bad arguments on the host (no kernel launches; runs without a GPU)."""

import ctypes
import glob
import os
import re

import pytest

from hspmn_b200 import _native as N

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        names |= set(re.findall(r"HSPMN_API\s+[\w\s\*]+?\b(hspmn_\w+)\s*\(", open(h).read()))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"hspmn_router_topk", "hspmn_gate_logits", "hspmn_gather_rows", "hspmn_scatter_rows", "hspmn_sqdk_fwd"} <= names


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(N.EXPORTED) >= declared_symbols()


def test_version_and_strerror():
    lib = N.lib()
    assert lib.hspmn_version() >= 100
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert N.strerror(code)
    assert N.strerror(-99) == "unknown status"


def _i64(*v):
    return N.i64_array(v)


def test_sqdk_validation_rejects_before_launch():
    lib = N.lib()
    st = [64 * 4 * 128, 4 * 128, 128, 1]
    p = ctypes.c_void_p(4096)
    args = dict(q=p, qs=_i64(*st), k=p, ks=_i64(*st), v=p, vs=_i64(*st), idx=p, isb=8, isk=1, o=p,
                os_=_i64(*st), B=1, K=8, S=64, H=4, Hkv=4, hd=128, dt=2, scale=0.088)

    def call(**over):
        a = dict(args, **over)
        return lib.hspmn_sqdk_fwd(a["q"], a["qs"], a["k"], a["ks"], a["v"], a["vs"], a["idx"], a["isb"],
                                  a["isk"], a["o"], a["os_"], a["B"], a["K"], a["S"], a["H"], a["Hkv"],
                                  a["hd"], a["dt"], ctypes.c_float(a["scale"]), None, 0, None)

    assert call(q=ctypes.c_void_p(0)) == -1          # null pointer
    assert call(dt=0) == -2                           # float32 not a tensor-core dtype here
    assert call(hd=136) == -4 and call(hd=20) == -4   # unsupported head_dim
    assert call(Hkv=3) == -4                          # 4 % 3 != 0
    assert call(scale=-1.0) == -1
    assert call(qs=_i64(64 * 4 * 128, 4 * 128, 128, 2)) == -3  # innermost stride must be 1
    assert call(ks=_i64(64 * 4 * 128, 4 * 128, 132, 1)) == -3  # 264-byte head stride
    assert call(B=0) == 0 and call(K=0) == 0          # empty: nothing to do


def test_router_and_rows_validation():
    lib = N.lib()
    p = ctypes.c_void_p(4096)
    # k > S, k < 1, bad dtype
    assert lib.hspmn_router_topk(p, 2, 16, None, 0, 2, 1, 16, 17, p, 17, None, 0, None) == -1
    assert lib.hspmn_router_topk(p, 2, 16, None, 0, 2, 1, 16, 0, p, 1, None, 0, None) == -1
    assert lib.hspmn_router_topk(p, 7, 16, None, 0, 2, 1, 16, 4, p, 4, None, 0, None) == -2
    # gather: null source; odd row bytes cannot be moved
    assert lib.hspmn_gather_rows(None, 0, 0, p, 4, p, 0, 0, 1, 8, 4, 16, None) == -1
    assert lib.hspmn_gather_rows(p, 8 * 3, 3, p, 4, p, 4 * 3, 3, 1, 8, 4, 3, None) == -3
    # scatter: K > S
    assert lib.hspmn_scatter_rows(p, 0, 16, p, 9, p, 0, 16, 1, 8, 9, 16, None) == -1


def test_gate_validation():
    lib = N.lib()
    p = ctypes.c_void_p(4096)
    f32, bf16 = 0, 2

    def gate(x=p, dt=bf16, sb=64 * 256, ss=256, w=p, bias=None, B=1, S=64, D=256, out=p, rs=64):
        return lib.hspmn_gate_logits(x, dt, sb, ss, w, bias, B, S, D, out, rs, None)

    assert gate(x=None) == -1 and gate(w=None) == -1 and gate(out=None) == -1
    assert gate(S=0) == -1 and gate(rs=63) == -1 and gate(sb=-1) == -1
    assert gate(dt=9) == -2
    assert gate(D=12) == -4 and gate(dt=f32, D=6) == -4      # not whole 16-byte vectors
    assert gate(x=ctypes.c_void_p(4098)) == -3                # misaligned row base
    assert gate(ss=260) == -3 and gate(w=ctypes.c_void_p(4104)) == -3
    assert gate(B=0) == 0                                     # empty: nothing to do


def test_sqdk_backward_validation():
    lib = N.lib()
    p = ctypes.c_void_p(4096)
    B, K, S, H, Hkv, hd = 1, 16, 256, 8, 2, 64
    qs = (ctypes.c_int64 * 4)(K * H * hd, H * hd, hd, 1)
    ks = (ctypes.c_int64 * 4)(S * Hkv * hd, Hkv * hd, hd, 1)

    def bwd(k=p, dk=p, q=p, dtype=2, hd_=hd, H_=H, Hkv_=Hkv, K_=K, lse_sb=K * H, ws=p, ws_bytes=1 << 20):
        return lib.hspmn_sqdk_bwd(q, qs, k, ks, k, ks, p, K_, 1, p, qs, p, qs, p, lse_sb, H_, p, qs, dk, ks, dk, ks,
                                  B, K_, S, H_, Hkv_, hd_, dtype, 0.125, ws, ws_bytes, None)

    assert bwd(k=None) == -1 and bwd(dk=None) == -1 and bwd(q=None) == -1
    assert bwd(dtype=0) == -2                      # f32 operands are not supported
    assert bwd(hd_=12) == -4 and bwd(hd_=136) == -4
    assert bwd(H_=6, Hkv_=4) == -4                 # heads not a multiple of kv heads
    assert bwd(lse_sb=K * H + 1) == -1             # lse must be dense [B,K,H]
    assert bwd(ws=None) == -1 and bwd(ws_bytes=16) == -1
    assert bwd(k=ctypes.c_void_p(4100)) == -3
    assert lib.hspmn_sqdk_bwd_workspace_size(1, 16, 8, 64) == 512 + 16 * 8 * 64 * 4
    assert lib.hspmn_sqdk_bwd_workspace_size(1, 0, 8, 64) == 0
    # the forward with log-sum-exp needs somewhere to put it
    assert lib.hspmn_sqdk_fwd_lse(p, qs, p, ks, p, ks, p, K, 1, p, qs, None, K * H, H, B, K, S, H, Hkv, hd, 2,
                                  0.125, None, 0, None) == -1


def test_rope_and_scatter_add_validation():
    lib = N.lib()
    p = ctypes.c_void_p(4096)
    bf16, bad = 2, 9

    def rope(**o):
        a = dict(src=p, src_sb=8 * 2 * 128, src_ss=2 * 128, byp=1, idx=p, idx_sb=4, cos=p, sin=p, tab_ss=128,
                 dst=p, dst_sb=4 * 2 * 128, dst_sk=2 * 128, B=1, S=8, K=4, H=2, hd=128, dt=bf16)
        a.update(o)
        return lib.hspmn_rope_gather_rows(a["src"], a["src_sb"], a["src_ss"], a["byp"], a["idx"], a["idx_sb"],
                                          a["cos"], a["sin"], a["tab_ss"], a["dst"], a["dst_sb"], a["dst_sk"],
                                          a["B"], a["S"], a["K"], a["H"], a["hd"], a["dt"], None)

    assert rope(src=None) == -1                        # null pointer
    assert rope(dt=bad) == -2                          # unknown element type
    assert rope(tab_ss=64) == -1                       # table rows shorter than a head
    assert rope(idx_sb=-1) == -1
    assert rope(hd=12, tab_ss=12, src_ss=24, dst_sk=24) == -4  # a 16-byte group would straddle the head halves
    assert rope(src=ctypes.c_void_p(4098)) == -3       # source not 16-byte aligned
    assert rope(B=0) == 0 and rope(K=0) == 0           # empty: nothing to do

    def rows(**o):
        a = dict(src=p, src_sb=8 * 2 * 128, src_ss=2 * 128, cos=p, sin=p, tab_ss=128, tab_rows=8, pos0=0,
                 dst=p, dst_sb=8 * 2 * 128, dst_ss=2 * 128, B=1, S=8, H=2, hd=128, dt=bf16)
        a.update(o)
        return lib.hspmn_rope_rows(a["src"], a["src_sb"], a["src_ss"], a["cos"], a["sin"], a["tab_ss"],
                                   a["tab_rows"], a["pos0"], a["dst"], a["dst_sb"], a["dst_ss"], a["B"], a["S"],
                                   a["H"], a["hd"], a["dt"], None)

    assert rows(cos=None) == -1                        # null pointer
    assert rows(dt=bad) == -2
    assert rows(pos0=1) == -1                          # positions past the table's last row
    assert rows(pos0=-1) == -1
    assert rows(tab_ss=64) == -1                       # table rows shorter than a head
    assert rows(hd=12, tab_ss=12, src_ss=24, dst_ss=24, src_sb=192, dst_sb=192) == -4
    assert rows(dst=ctypes.c_void_p(4104)) == -3       # destination not 16-byte aligned
    assert rows(B=0) == 0 and rows(S=0, tab_rows=0) == 0

    def sadd(**o):
        a = dict(src=p, src_sb=4 * 2048, src_sk=2048, idx=p, idx_sb=4, dst=p, dst_sb=8 * 2048, dst_ss=2048,
                 B=1, S=8, K=4, row=2048, dt=bf16)
        a.update(o)
        return lib.hspmn_scatter_add_rows(a["src"], a["src_sb"], a["src_sk"], a["idx"], a["idx_sb"], a["dst"],
                                          a["dst_sb"], a["dst_ss"], a["B"], a["S"], a["K"], a["row"], a["dt"], None)

    assert sadd(dst=None) == -1
    assert sadd(dt=bad) == -2
    assert sadd(idx_sb=3) == -1                        # index rows shorter than K
    assert sadd(row=3, src_sk=3, dst_ss=3, src_sb=12, dst_sb=24) == -3  # 6-byte rows
    assert sadd(B=0) == 0 and sadd(K=0) == 0

    assert lib.hspmn_device_errors(None, 0, None) == -1
    # workspace size of a shape the attention rejects: 0, no device query
    assert lib.hspmn_sqdk_workspace_size(1, 8, 64, 4, 3, 128) == 0
    assert lib.hspmn_strerror(-7).decode().startswith("shape needs more split-KV scratch")


def test_ops_reject_cpu_tensors():
    torch = pytest.importorskip("torch")
    from hspmn_b200 import ops
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        ops.router_topk(torch.zeros(1, 8), None, 2, torch.float32)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        ops.gather_rows(torch.zeros(1, 8, 4), torch.zeros(1, 2, dtype=torch.int64))
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        ops.gate_logits(torch.zeros(1, 8, 16), torch.zeros(1, 16), None)
