"""Expert-parallel (EP) prefill of one MoE block over a torch.distributed process group (NCCL, one rank per GPU).

Placement. Every rank holds the router, the RMSNorm weight and the shared-expert slots (data parallel), the
`replicated` experts (the hottest ones: their pairs never leave the rank), and a round-robin share of the
other ("cold") experts: cold expert number c (in id order) lives on rank c % world. With BASELINE's Zipf router
bias six experts take ~80 % of all routed pairs, so sharding them would serialise the step on their owners;
replicating them costs 17 MB per expert of the 180 GB on each GPU.

A prefill step on a rank's own packed tokens:
  1. RMSNorm and routing locally (mv_rmsnorm, mv_route);
  2. the pairs whose expert lives on another rank, sorted by owner rank (stable, so every rank sends in token
     order): pair counts exchanged with one all-to-all, then the token rows (bf16 [H]) and their metadata
     (slot of the expert on its owner, routing weight) with all-to-all-v -- the one exchange step of the block;
  3. ONE tcgen05 grouped-GEMM pass (mv_moe_prefill) over the rank's own tokens and the received rows: an own
     token carries the pairs whose expert this rank holds (the replicated hot experts, its share of the cold
     ones, the shared expert; the other pairs -1, which the expert sort skips), a received row its one pair;
  4. the received rows' weighted outputs travel back (all-to-all-v, the reverse split) and are added at the
     origin in fp32 with the residual and the local output, rounded once.

The exchange sizes are data dependent, so a step synchronises the host once (the split sizes); prefill is not
graph-captured. No kernel reads another GPU's memory: everything remote arrives through NCCL.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import moe


def placement(E: int, world: int, replicated=()):
    """owner[e], slot[e] for every routed expert e: replicated experts -> slot i on every rank (owner -1 =
    "this rank"); cold experts -> rank c % world, slot n_rep + c // world. Also each rank's stack order."""
    rep = list(replicated)
    rset = set(rep)
    cold = [e for e in range(E) if e not in rset]
    owner = [-1] * E
    slot = [0] * E
    for i, e in enumerate(rep):
        slot[e] = i
    for c, e in enumerate(cold):
        owner[e] = c % world
        slot[e] = len(rep) + c // world
    stacks = [rep + [e for c, e in enumerate(cold) if c % world == r] for r in range(world)]
    return owner, slot, stacks


class EPMoeBlock:
    """One rank's part of an expert-parallel MoE block.

    `block` is this rank's MoeBlock: the FULL router / norm, and stacked weights in the order
    placement(E, world, replicated)[2][rank] followed by the shared slots (see shard_block_params).
    `experts_fn(x, ids, wts)` computes weight * expert(x) per row on this rank's stacks (defaults to the CUDA
    grouped GEMM; the CPU tests pass a reference)."""

    def __init__(self, block, E: int, group=None, replicated=(), experts_fn=None):
        self.block = block
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = E
        owner, slot, stacks = placement(E, self.world, replicated)
        self.n_local = len(stacks[self.rank])
        own = torch.tensor(owner, dtype=torch.long)
        self.owner = torch.where(own < 0, torch.full_like(own, self.rank), own)
        self.slot = torch.tensor(slot, dtype=torch.long)
        self.n_shared = len(block.shared_ids)
        self.experts_fn = experts_fn or self._experts_cuda

    # ------------------------------------------------------------------------------------------ pieces
    def _experts_cuda(self, x, ids, wts, residual=None):
        b = self.block
        return moe.experts(x, b.w_gu, b.w_d, ids, wts, s_gu=b.s_gu, s_d=b.s_d, residual=residual)

    def _local(self, xn, ids, wts, x):
        """Sum over this rank's pairs (ids -1 = a pair owned elsewhere, skipped) in one grouped-GEMM pass, plus the
        residual x when x is given (fused, one rounding)."""
        if self.experts_fn == self._experts_cuda:
            return self._experts_cuda(xn, ids, wts, residual=x)
        y = self.experts_fn(xn, ids, wts)
        return y if x is None else (x.float() + y.float()).to(x.dtype)

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    # ------------------------------------------------------------------------------------------ forward
    def forward(self, x):
        """h + MoE(rms_norm(h)) for this rank's N packed tokens x [N, H] bf16."""
        b = self.block
        N, H = x.shape
        K, dev = b.top_k, x.device
        if b.norm_w is not None:
            import fused_ops
            xn = fused_ops.rms_norm(x, b.norm_w, b.eps)
        else:
            xn = x
        ids, wts, _ = b.route(xn)
        if self.owner.device != dev:
            self.owner, self.slot = self.owner.to(dev), self.slot.to(dev)
        routed = ids[:, :K].long()
        own = self.owner[routed]  # [N, K] the rank holding each routed pair's expert
        slot = self.slot[routed]  # its stack index there
        ids_loc = torch.where(own == self.rank, slot, torch.full_like(slot, -1))
        if self.n_shared:
            ids_loc = torch.cat([ids_loc, ids[:, K:].to(ids_loc.dtype)], 1)
        # the pairs of this rank (replicated experts, its share of the cold ones, the shared expert) go through
        # one grouped-GEMM pass over its own tokens. Alone, the residual is fused into it; with remote pairs to
        # add, the sum is completed in fp32 and rounded once.
        ids_loc = ids_loc.to(torch.int32).contiguous()
        if self.world == 1:
            return self._local(xn, ids_loc, wts, x)

        # the other pairs: sorted by owner (stable, so in token order per owner); their counts are exchanged
        # first (the one host synchronisation of the step), then their rows and metadata
        flat_own = own.reshape(-1)
        key = torch.where(flat_own == self.rank, torch.full_like(flat_own, self.world), flat_own)
        order_all = torch.sort(key, stable=True).indices
        # (index_add, not bincount: bincount sizes its output from the data, a host synchronisation on CUDA)
        counts = torch.zeros(self.world + 1, dtype=torch.long, device=dev).index_add_(0, key, torch.ones_like(key))
        counts = counts[: self.world].contiguous()
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        in_splits = counts.tolist()
        out_splits = recv_counts.tolist()
        n_send, R = sum(in_splits), sum(out_splits)

        order = order_all[:n_send]
        tok = torch.div(order, K, rounding_mode="floor")
        send_rows = xn.index_select(0, tok)
        send_meta = torch.stack([slot.reshape(-1)[order].to(torch.float32),
                                 wts[:, :K].reshape(-1)[order].to(torch.float32)], 1)
        recv_rows = torch.empty(R, H, dtype=xn.dtype, device=dev)
        recv_meta = torch.empty(R, 2, dtype=torch.float32, device=dev)
        self._a2a(recv_rows, send_rows, out_splits, in_splits)
        self._a2a(recv_meta, send_meta, out_splits, in_splits)
        # one grouped-GEMM pass over this rank's own tokens and the received rows together: own rows carry their
        # local pairs (others -1), a received row its one (slot, weight) pair in column 0 and -1 elsewhere
        NK = ids_loc.shape[1]
        r_ids = torch.full((R, NK), -1, dtype=torch.int32, device=dev)
        r_wts = torch.zeros(R, NK, dtype=torch.float32, device=dev)
        if R > 0:
            r_ids[:, 0] = recv_meta[:, 0].round().to(torch.int32)
            r_wts[:, 0] = recv_meta[:, 1]
        y_all = self._local(torch.cat([xn, recv_rows]), torch.cat([ids_loc, r_ids]),
                            torch.cat([wts.to(torch.float32), r_wts]), None)
        back = torch.empty(n_send, H, dtype=y_all.dtype, device=dev)
        self._a2a(back, y_all[N:].contiguous(), in_splits, out_splits)
        y32 = x.to(torch.float32, copy=True)  # (never an alias of the caller's tokens)
        y32 += y_all[:N].to(torch.float32)
        if n_send:
            y32.index_add_(0, tok, back.to(torch.float32))
        return y32.to(x.dtype)


def shard_block_params(p: dict, rank: int, world: int, E: int, replicated=()):
    """This rank's stacked weights from a full parameter dict (oracle.make_block_params layout), in the order
    placement() gives, followed by the shared slots; shared_ids re-numbered to follow the routed stacks."""
    _, _, stacks = placement(E, world, replicated)
    sel = stacks[rank] + list(range(E, p["w_gu"].shape[0]))
    q = dict(p)
    for k in ("w_gu", "w_d", "s_gu", "s_d"):
        if q.get(k) is not None:
            q[k] = p[k][sel].contiguous()
    n_loc = len(stacks[rank])
    q["shared_ids"] = tuple(range(n_loc, n_loc + len(p["shared_ids"])))
    return q
