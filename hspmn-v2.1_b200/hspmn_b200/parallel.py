"""Multi-GPU execution of the contextual-stream inference path.

Two layouts, one process per GPU (``torch.distributed``, NCCL on GPUs):

* Batch partitioning (independent sequences): every rank runs its own
  sequences through an unmodified ``HSPMNBlock``; no collective touches the
  data path. ``batch_slice`` gives a rank's share of a global batch.

* Sequence sharding for one long sequence (the 262,144-token configuration):
  the sequence is cut into ``2W`` equal chunks and rank ``r`` owns chunks ``r``
  and ``2W-1-r`` ("zig-zag"), which balances the causal attention work. Per
  forward there is one real exchange step:

    1. every rank computes gate logits for its rows; an all-gather of the
       logits (2 bytes per position) lets every rank run the same
       deterministic top-K kernel, so the selected positions are identical
       everywhere;
    2. every rank computes K/V (with RoPE) for its rows; an all-gather of
       the first chunks plus point-to-point copies of the second chunks place
       the whole K/V prefix in position order in local HBM (no peer-memory
       loads by the kernels, no reorder copy);
    3. each rank attends the selected queries that fall in its own chunks
       (q_proj on those rows only, RoPE fused into their gather), applies
       o_proj to the attention rows and adds them into its rows of the
       reflexive stream (whose depthwise conv needs one neighbouring row per
       chunk edge, taken from an all-gather of chunk-edge rows).

  The output stays sequence-sharded in the rank's local row order.

The compute operators are looked up on ``self.ops`` (default:
``hspmn_b200.ops``, the CUDA kernels). The reference has no distributed code;
this module follows its single-GPU semantics (hspmn_v2_1.py:95-238) exactly.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import ops as cuda_ops
from .model import HSPMNBlock, RouterOutput, depthwise_conv_seq


def batch_slice(global_batch: int, rank: int, world: int) -> slice:
    """Contiguous share of a global batch for ``rank`` (sizes differ by <= 1)."""
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


@dataclass(frozen=True)
class ZigZagPlan:
    """Zig-zag split of ``seq_len`` positions over ``world`` ranks."""

    seq_len: int
    world: int

    def __post_init__(self):
        if self.seq_len % (2 * self.world) != 0:
            raise ValueError(f"seq_len {self.seq_len} must be a multiple of 2*world ({2 * self.world})")

    @property
    def chunk(self) -> int:
        return self.seq_len // (2 * self.world)

    def chunks(self, rank: int) -> List[Tuple[int, int]]:
        """[start, end) position ranges owned by ``rank``, ascending."""
        c = self.chunk
        a, b = rank, 2 * self.world - 1 - rank
        return [(a * c, (a + 1) * c), (b * c, (b + 1) * c)]

    def local_positions(self, rank: int, device=None) -> torch.Tensor:
        """Global position of each local row (int64 [2*chunk], ascending)."""
        return torch.cat([torch.arange(s, e, device=device) for s, e in self.chunks(rank)])

    def shard(self, x: torch.Tensor, rank: int, dim: int = 1) -> torch.Tensor:
        """This rank's rows of a full-sequence tensor (position dim ``dim``)."""
        return torch.cat([x.narrow(dim, s, e - s) for s, e in self.chunks(rank)], dim=dim)

    def unshard(self, parts: List[torch.Tensor], dim: int = 1) -> torch.Tensor:
        """Inverse of ``shard`` given every rank's local tensor (rank order)."""
        c = self.chunk
        pieces = [None] * (2 * self.world)
        for r, part in enumerate(parts):
            a, b = r, 2 * self.world - 1 - r
            pieces[a] = part.narrow(dim, 0, c)
            pieces[b] = part.narrow(dim, c, c)
        return torch.cat(pieces, dim=dim)


def _all_gather_rows(local: torch.Tensor, plan: ZigZagPlan, group) -> torch.Tensor:
    """All-gather a [B, 2*chunk, ...] local tensor into the full [B, S, ...]
    sequence in position order."""
    return _all_gather_rows_async(local, plan, group)()


def _group_peer(group, group_rank: int) -> int:
    return group_rank if group is None else dist.get_global_rank(group, group_rank)


def _all_gather_rows_async(local: torch.Tensor, plan: ZigZagPlan, group):
    """Start gathering every rank's [B, 2*chunk, ...] rows into one
    position-ordered [B, S, ...] tensor; the returned function makes the
    current stream wait for the transfers and returns that tensor. Work
    queued on the current stream in between overlaps the transfer.

    One sequence (B == 1): the rows land in place, with no reorder copy. The
    first chunks (rank r owns chunk r) arrive in rank order, which is position
    order, by one all-gather into the first half; each rank's second chunk
    (chunk 2W-1-r, i.e. the reverse of rank order) goes point to point
    straight into its slot. Several sequences: one all-gather, then one
    reorder copy."""
    W = plan.world
    B = local.shape[0]
    c = plan.chunk
    tail = tuple(local.shape[2:])
    src = local.contiguous()
    if B != 1:
        flat = torch.empty((W * B,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        work = dist.all_gather_into_tensor(flat, src, group=group, async_op=True)

        def finish_batched(_src=src) -> torch.Tensor:  # _src: the collective reads it until done
            work.wait()
            return plan.unshard(list(flat.view((W, B) + tuple(local.shape[1:])).unbind(0)), dim=1)

        return finish_batched
    rank = dist.get_rank(group)
    full = torch.empty((1, plan.seq_len) + tail, dtype=local.dtype, device=local.device)
    rows = full.view((plan.seq_len,) + tail)
    first, second = src[0, :c], src[0, c:]
    works = [dist.all_gather_into_tensor(rows[: W * c], first, group=group, async_op=True)]
    mine = 2 * W - 1 - rank
    rows[mine * c:(mine + 1) * c].copy_(second)
    ops = []
    for p in range(W):
        if p == rank:
            continue
        slot = 2 * W - 1 - p
        ops.append(dist.P2POp(dist.isend, second, _group_peer(group, p), group))
        ops.append(dist.P2POp(dist.irecv, rows[slot * c:(slot + 1) * c], _group_peer(group, p), group))
    if ops:
        works.extend(dist.batch_isend_irecv(ops))

    def finish(_src=src) -> torch.Tensor:
        for w in works:
            w.wait()
        return full

    return finish


class SequenceShardedBlock:
    """Inference forward of an ``HSPMNBlock`` over one sequence-sharded input.

    ``forward(x_local)`` takes this rank's rows (``plan.shard(x, rank)``,
    [B, 2*chunk, D]) and returns this rank's output rows and the auxiliary
    loss, which every rank computes identically from the gathered logits."""

    def __init__(self, block: HSPMNBlock, plan: ZigZagPlan, group=None, ops=None):
        self.block = block
        self.plan = plan
        self.group = group
        self.ops = ops if ops is not None else cuda_ops
        self.rank = dist.get_rank(group)
        if dist.get_world_size(group) != plan.world:
            raise ValueError("plan.world does not match the process group size")
        self._cache = {}

    # -- router over the gathered logits (hspmn_v2_1.py:95-122, eval) ------
    def _route(self, x_local: torch.Tensor, S: int) -> RouterOutput:
        r = self.block.router
        logits_local = r.gate_logits(x_local)
        logits = _all_gather_rows(logits_local, self.plan, self.group)
        temp = torch.exp(r.log_temp).clamp(0.1, 2.0)
        k = r.num_selected(S)
        noisy_dtype = torch.result_type(logits, temp)
        indices, mask = self.ops.router_topk(logits, temp, k, noisy_dtype)
        probs = torch.sigmoid(logits)
        sparsity_loss = (probs.mean() - r.target_sparsity).pow(2)
        ent = -(probs * (probs + 1e-10).log() + (1.0 - probs) * (1.0 - probs + 1e-10).log())
        aux = r.sparsity_coef * sparsity_loss + r.entropy_coef * ent.mean()
        return RouterOutput(mask, indices, logits, aux)

    def _chunk_tensors(self, device):
        """(chunk bounds [4], local row positions [2*chunk]) on ``device``,
        built once per device."""
        key = str(device)
        if key not in self._cache:
            (s0, e0), (s1, e1) = self.plan.chunks(self.rank)
            self._cache[key] = (torch.tensor([s0, e0, s1, e1], dtype=torch.int64, device=device),
                                self.plan.local_positions(self.rank, device=device))
        return self._cache[key]

    def _selection_bounds_begin(self, indices: torch.Tensor):
        """Where this rank's two chunks start and end in each sorted index row:
        one searchsorted on the device, its [B,4] result copied to host memory
        without waiting. ``_local_selection`` reads it once the independent
        work of the forward is queued, so the host never drains the stream."""
        bounds, _ = self._chunk_tensors(indices.device)
        at = torch.searchsorted(indices, bounds.expand(indices.shape[0], 4).contiguous())
        if not at.is_cuda:
            return at, None
        host = torch.empty(at.shape, dtype=at.dtype, pin_memory=True)
        host.copy_(at, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        return host, ev

    def _local_selection(self, indices: torch.Tensor, pending) -> Tuple[torch.Tensor, torch.Tensor]:
        """Selected positions inside this rank's chunks (ascending, [B, K_r])
        and their local row numbers, from ``_selection_bounds_begin``'s
        result. Requires B == 1 or equal counts per row."""
        host, ev = pending
        if ev is not None:
            ev.synchronize()
        at = host.tolist()
        (s0, _), (s1, _) = self.plan.chunks(self.rank)
        c = self.plan.chunk
        counts = {(r[1] - r[0]) + (r[3] - r[2]) for r in at}
        if len(counts) != 1:
            raise ValueError("per-sequence selection counts differ across the batch on this rank; "
                             "shard one sequence per call")
        pos_list, row_list = [], []
        for b, (lo0, hi0, lo1, hi1) in enumerate(at):
            seg0, seg1 = indices[b, lo0:hi0], indices[b, lo1:hi1]
            pos_list.append(torch.cat([seg0, seg1]))
            row_list.append(torch.cat([seg0 - s0, seg1 - s1 + c]))
        return torch.stack(pos_list), torch.stack(row_list)

    def _halo_rows(self, h_local: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Rows just before / after each local chunk (zeros at sequence ends),
        from an all-gather of every rank's chunk-edge rows. Returns
        (before [B,2,D], after [B,2,D]) for the rank's two chunks."""
        c = self.plan.chunk
        W = self.plan.world
        edges = torch.stack([h_local[:, 0], h_local[:, c - 1], h_local[:, c], h_local[:, 2 * c - 1]], dim=1)
        allg = torch.empty((W * edges.shape[0],) + tuple(edges.shape[1:]), dtype=edges.dtype,
                           device=edges.device)
        dist.all_gather_into_tensor(allg, edges.contiguous(), group=self.group)
        allg = allg.view((W,) + tuple(edges.shape))
        # first/last row of every global chunk
        first = [None] * (2 * W)
        last = [None] * (2 * W)
        for r in range(W):
            a, b = r, 2 * W - 1 - r
            first[a], last[a] = allg[r, :, 0], allg[r, :, 1]
            first[b], last[b] = allg[r, :, 2], allg[r, :, 3]
        zero = torch.zeros_like(h_local[:, 0])
        before, after = [], []
        for ci in (self.rank, 2 * W - 1 - self.rank):
            before.append(last[ci - 1] if ci > 0 else zero)
            after.append(first[ci + 1] if ci < 2 * W - 1 else zero)
        return torch.stack(before, 1), torch.stack(after, 1)

    def _reflexive(self, x_local: torch.Tensor) -> torch.Tensor:
        """ReflexiveStream.forward (hspmn_v2_1.py:141-145) on sharded rows:
        the depthwise conv of each chunk sees its true neighbours."""
        return self._reflexive_end(x_local, *self._reflexive_begin(x_local))

    def _reflexive_begin(self, x_local: torch.Tensor):
        """Norm and the halo exchange (a collective) of the reflexive stream."""
        h = self.block.reflexive.norm(x_local)
        before, after = self._halo_rows(h)
        return h, before, after

    def _reflexive_end(self, x_local: torch.Tensor, h: torch.Tensor, before: torch.Tensor,
                       after: torch.Tensor) -> torch.Tensor:
        """Conv over each chunk with its halo rows, SwiGLU MLP, residual."""
        rf = self.block.reflexive
        c = self.plan.chunk
        outs = []
        for i in range(2):
            seg = torch.cat([before[:, i:i + 1], h[:, i * c:(i + 1) * c], after[:, i:i + 1]], dim=1)
            outs.append(depthwise_conv_seq(seg, rf.conv.weight, padding=0))
        hc = torch.cat(outs, dim=1)
        return x_local + rf.down_proj(F.silu(rf.gate_proj(hc)) * rf.up_proj(hc))

    @torch.no_grad()
    def forward(self, x_local: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        blk = self.block
        B, S_local, D = x_local.shape
        S = self.plan.seq_len
        if S_local != 2 * self.plan.chunk:
            raise ValueError(f"x_local has {S_local} rows; this rank owns {2 * self.plan.chunk}")
        ro = self._route(x_local, S)
        pending = self._selection_bounds_begin(ro.indices)
        H, Hkv, hd = blk.num_heads, blk.num_kv_heads, blk.head_dim
        x_norm = blk.norm(x_local)
        cos, sin = blk.rope(x_local, S)
        pos = self._chunk_tensors(x_local.device)[1].expand(B, S_local)
        # K (RoPE at the rows' global positions) and V of the local rows
        k_loc = self.ops.rope_gather_rows(blk.k_proj(x_norm).view(B, S_local, Hkv, hd), pos, cos, sin, False)
        v_loc = blk.v_proj(x_norm).view(B, S_local, Hkv, hd)
        # the reflexive stream's halo exchange goes first: collectives run in
        # issue order, and it must not queue behind the K/V transfer
        h, before, after = self._reflexive_begin(x_local)
        # the whole sequence's K and V into local HBM (each its own contiguous
        # tensor, which the attention streams fastest), overlapped with the
        # reflexive MLP and the routed-query work
        k_finish = _all_gather_rows_async(k_loc, self.plan, self.group)
        v_finish = _all_gather_rows_async(v_loc, self.plan, self.group)
        y = self._reflexive_end(x_local, h, before, after).contiguous()
        sel_pos, sel_rows = self._local_selection(ro.indices, pending)
        if sel_pos.shape[1] > 0:
            # the routed queries of this rank: q_proj on those rows only, RoPE at
            # their global positions fused into the gather, o_proj on the K
            # attention rows, residual add in place
            x_sel = self.ops.gather_rows(x_norm, sel_rows)
            q_sel = blk.q_proj(x_sel).view(B, -1, H, hd)
            q_sel = self.ops.rope_gather_rows(q_sel, sel_pos, cos, sin, False)
            k_full, v_full = k_finish(), v_finish()
            attn = self.ops.sqdk_fwd(q_sel, k_full, v_full, sel_pos, 1.0 / math.sqrt(hd))
            self.ops.scatter_add_rows_(y, sel_rows, blk.o_proj(attn.reshape(B, -1, D)))
        else:
            k_finish(), v_finish()  # every rank takes part in the collectives and waits for them
        return y, ro.aux_loss
