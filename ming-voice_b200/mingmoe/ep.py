"""Expert-parallel (EP) prefill of one MoE block over a torch.distributed process group (NCCL, one rank per GPU).

Placement. Every rank holds the router, the RMSNorm weight and the shared-expert slots (data parallel), the
`replicated` experts (the hottest ones: their pairs never leave the rank), and a share of the other ("cold")
experts dealt in id order as a snake (ranks 0..W-1, then W-1..0, ...), which spreads a popularity that falls with
the expert id evenly over the ranks. With BASELINE's Zipf router
bias six experts take ~80 % of all routed pairs, so sharding them would serialise the step on their owners;
replicating them costs 17 MB per expert of the 180 GB on each GPU.

A prefill step on a rank's own packed tokens (CUDA path, no host synchronisation anywhere: the exchange has a
fixed capacity `cap` of pairs per peer, so the step can be captured in a CUDA graph):
  1. RMSNorm and routing locally (mv_rmsnorm, mv_route);
  2. mv_ep_plan (one CTA) gives every pair whose expert lives here its local slot and every other pair a place in
     its owner's send block (token order kept); mv_ep_pack writes those rows into the send blocks as wire rows
     (H values and a 16-byte (slot, weight, in-use) tail);
  3. one NCCL all-to-all of fixed size moves the wire rows (the one exchange step of the block);
  4. ONE tcgen05 grouped-GEMM pass (mv_moe_prefill_f32, fp32 outputs) over the own rows (local pairs; the rest -1,
     skipped by the expert sort) and the received rows where they landed (their one pair; unused places -1);
     the received rows' outputs go back with a second all-to-all, as bf16 (mv_ep_narrow: each is one weighted
     pair's output, rounded once, which is where the reference's grouped GEMM rounds every pair's output too);
  5. mv_ep_combine adds, per token in fp32, the residual, the local sum and its remote pairs' outputs in pair
     order, rounding once to bf16.
More than `cap` pairs for one peer is an error recorded in the plan's workspace (the excess pairs are dropped);
`plan_capacity` measures what a batch needs. No kernel reads another GPU's memory: everything remote arrives
through NCCL. With an `experts_fn` (the CPU tests) the same step runs on torch tensors with data-dependent
all-to-all sizes instead.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import moe


def placement(E: int, world: int, replicated=()):
    """owner[e], slot[e] for every routed expert e: replicated experts -> slot i on every rank (owner -1 =
    "this rank"); the c-th cold expert -> slot n_rep + c // world on rank c % world in even rounds and
    world - 1 - c % world in odd ones (a snake: with popularity falling with the expert id, as under the Zipf
    router bias, no rank collects the most popular expert of every round). Also each rank's stack order."""
    rep = list(replicated)
    rset = set(rep)
    cold = [e for e in range(E) if e not in rset]
    owner = [-1] * E
    slot = [0] * E
    for i, e in enumerate(rep):
        slot[e] = i

    def rank_of(c):
        rnd, pos = divmod(c, world)
        return pos if rnd % 2 == 0 else world - 1 - pos

    for c, e in enumerate(cold):
        owner[e] = rank_of(c)
        slot[e] = len(rep) + c // world
    stacks = [rep + [e for c, e in enumerate(cold) if rank_of(c) == r] for r in range(world)]
    return owner, slot, stacks


class EPMoeBlock:
    """One rank's part of an expert-parallel MoE block.

    `block` is this rank's MoeBlock: the FULL router / norm, and stacked weights in the order
    placement(E, world, replicated)[2][rank] followed by the shared slots (see shard_block_params).
    `experts_fn(x, ids, wts)` computes weight * expert(x) per row on this rank's stacks (defaults to the CUDA
    grouped GEMM; the CPU tests pass a reference)."""

    def __init__(self, block, E: int, group=None, replicated=(), experts_fn=None, cap=None):
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
        self._owner_raw = torch.tensor(owner, dtype=torch.int32)  # -1 = replicated (held here)
        self.n_shared = len(block.shared_ids)
        self.cuda_path = experts_fn is None
        self.experts_fn = experts_fn or self._experts_cuda
        self.cap = cap
        self._bufs = {}

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

    # ------------------------------------------------------------------------------------------ forward (CUDA)
    def calibrate(self, x, headroom=1.25):
        """Set the per-peer capacity from a representative batch: the largest count of pairs any rank sends to one
        peer (plan_capacity, one host synchronisation), with headroom, rounded up to 16."""
        need = self.plan_capacity(x)
        self.cap = max(16, (int(need * headroom) + 15) // 16 * 16)
        return self.cap

    def plan_capacity(self, x):
        """The largest number of pairs this rank's tokens x send to one peer, over all ranks (one host
        synchronisation and one all-reduce: for sizing `cap` outside the timed or captured path)."""
        b = self.block
        import fused_ops
        xn = fused_ops.rms_norm(x, b.norm_w, b.eps) if b.norm_w is not None else x
        ids, _, _ = b.route(xn)
        own = self.owner.to(x.device)[ids[:, :b.top_k].long()]
        cnt = torch.stack([(own == d).sum() for d in range(self.world) if d != self.rank] or
                          [torch.zeros((), dtype=torch.long, device=x.device)]).max().reshape(1)
        dist.all_reduce(cnt, op=dist.ReduceOp.MAX, group=self.group)
        return int(cnt.item())

    def _buffers(self, N, cap, dev):
        key = (N, cap, dev)
        bf = self._bufs.get(key)
        if bf is None:
            b, W = self.block, self.world
            R, NK, H = W * cap, b.nk, b.H
            bf = dict(
                xn=torch.empty(N, H, dtype=torch.bfloat16, device=dev),
                ids=torch.empty(N, NK, dtype=torch.int32, device=dev),
                wts=torch.empty(N, NK, dtype=torch.float32, device=dev),
                logits=torch.empty(N, b.E, dtype=torch.float32, device=dev),
                ids_all=torch.empty(N + R, NK, dtype=torch.int32, device=dev),  # own rows, then received rows
                wts_all=torch.empty(N + R, NK, dtype=torch.float32, device=dev),
                pos=torch.empty(N, b.top_k, dtype=torch.int32, device=dev),
                send_src=torch.zeros(R, dtype=torch.int32, device=dev),
                send_meta=torch.zeros(W, cap + 1, 2, dtype=torch.int32, device=dev),
                send_rows=torch.zeros(R, H + 8, dtype=torch.bfloat16, device=dev),  # wire rows: H values + tail
                recv_rows=torch.zeros(R, H + 8, dtype=torch.bfloat16, device=dev),
                y32=torch.empty(N + R, H, dtype=torch.float32, device=dev),
                back_send=torch.empty(R, H, dtype=torch.bfloat16, device=dev),  # received rows' outputs, bf16
                back=torch.empty(R, H, dtype=torch.bfloat16, device=dev),
                out=torch.empty(N, H, dtype=torch.bfloat16, device=dev),
                owner=self._owner_raw.to(dev),
                slot=self.slot.to(torch.int32).to(dev),
            )
            self._bufs[key] = bf
        return bf

    PHASES = ("norm+route", "plan+pack", "exchange out", "unpack", "grouped GEMM+narrow", "exchange back", "combine")

    def _forward_cuda(self, x, events=None):
        """The step; `events` (len(PHASES) + 1 CUDA events, or None) are recorded at the phase boundaries."""
        import ctypes as C
        import fused_ops
        from . import _lib as L
        b = self.block
        N, H = x.shape
        if x.dtype != torch.bfloat16 or x.stride(1) != 1:
            raise TypeError("EP prefill: x must be bf16 with a unit inner stride")
        dev = x.device
        cap = self.cap if self.cap is not None else self.calibrate(x)  # (first call without a capacity: measured)
        W, K, NK = self.world, b.top_k, b.nk
        R = W * cap
        bf = self._buffers(N, cap, dev)
        st = L.stream_ptr(dev)
        lib = L.lib()
        xn = bf["xn"]
        mark = (lambda i: events[i].record()) if events is not None else (lambda i: None)
        mark(0)
        if b.norm_w is not None:
            L.check(lib.mv_rmsnorm(L.ptr(x), L.MV_BF16, x.stride(0), L.ptr(b.norm_w), L.MV_BF16, L.ptr(xn), L.MV_BF16,
                                   N, H, C.c_float(b.eps), st), "mv_rmsnorm")
        else:
            xn.copy_(x)
        fused_ops.moe_route(xn, b.router_w, b.router_bias, b.n_group, b.topk_group, K, b.route_scale, bf["logits"],
                            bf["ids"], bf["wts"], mode=b.route_mode, n_shared=len(b.shared_ids),
                            shared_id=b.shared_ids[0] if b.shared_ids else b.E, w_scale=b.router_s)
        mark(1)
        ws = L.workspace("ep", int(lib.mv_ep_workspace_bytes()), dev)
        ids_all, wts_all = bf["ids_all"], bf["wts_all"]
        L.check(lib.mv_ep_plan(L.ptr(bf["ids"]), L.ptr(bf["wts"]), N, NK, K, L.ptr(bf["owner"]), L.ptr(bf["slot"]),
                               self.E, self.rank, W, cap, L.ptr(ids_all), L.ptr(wts_all), L.ptr(bf["pos"]),
                               L.ptr(bf["send_src"]), L.ptr(bf["send_meta"]), L.ptr(ws), ws.numel(), st), "mv_ep_plan")
        L.check(lib.mv_ep_pack(L.ptr(xn), H, H, L.ptr(bf["send_src"]), L.ptr(bf["send_meta"]), W, cap,
                               L.ptr(bf["send_rows"]), st), "mv_ep_pack")
        mark(2)
        # the exchange: rows and their (slot, weight) tails in one all-to-all
        dist.all_to_all_single(bf["recv_rows"], bf["send_rows"], group=self.group)
        mark(3)
        L.check(lib.mv_ep_unpack(L.ptr(bf["recv_rows"]), H, W, cap, NK, L.ptr(ids_all[N:]), L.ptr(wts_all[N:]), st),
                "mv_ep_unpack")
        mark(4)
        # one grouped-GEMM pass: own rows from xn, received rows where they landed (wire row stride H + 8)
        wst = moe.weights_struct(b.w_gu, b.w_d, b.s_gu, b.s_d)
        nbytes = lib.mv_moe_prefill_workspace_bytes(N + R, NK, H, b.I, b.w_gu.shape[0], L.dt(b.w_gu))
        pws = L.workspace("prefill", nbytes, dev)
        y32 = bf["y32"]
        L.check(lib.mv_moe_prefill_f32(C.byref(wst), L.ptr(xn), H, N, L.ptr(bf["recv_rows"]), H + 8, L.ptr(ids_all),
                                       L.MV_I32, L.ptr(wts_all), N + R, NK, None, 0, L.ptr(y32), 0, L.ptr(pws),
                                       pws.numel(), st), "mv_moe_prefill_f32")
        # the received rows' outputs (one weighted pair each) go back as bf16: rounded once, half the bytes
        L.check(lib.mv_ep_narrow(L.ptr(y32[N:]), R * H, L.ptr(bf["back_send"]), st), "mv_ep_narrow")
        mark(5)
        dist.all_to_all_single(bf["back"], bf["back_send"], group=self.group)
        mark(6)
        out = bf["out"]
        L.check(lib.mv_ep_combine(L.ptr(x), x.stride(0), L.ptr(y32), L.ptr(bf["back"]), L.MV_BF16, L.ptr(bf["pos"]),
                                  N, K, H, L.ptr(out), st), "mv_ep_combine")
        mark(7)
        return out

    def phase_times(self, x, reps=20, warmup=3):
        """Device time of each phase of the step (PHASES, microseconds, mean over `reps` replays) on this rank. The
        step is captured in a CUDA graph with event-record nodes at the phase boundaries (as the timed step runs,
        so no host launch gaps count), replayed `reps` times. An exchange phase includes waiting for the slowest
        peer. Every rank must call it with the same arguments (the graph holds the NCCL all-to-alls).
        Host-synchronising: a measurement utility, not for the hot loop."""
        dev = x.device
        for _ in range(warmup):
            self._forward_cuda(x)
        evs = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(self.PHASES) + 1)]
        torch.cuda.synchronize(dev)
        stream = torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            self._forward_cuda(x, events=evs)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                self._forward_cuda(x, events=evs)
        torch.cuda.current_stream(dev).wait_stream(stream)
        tot = [0.0] * len(self.PHASES)
        for _ in range(reps):
            graph.replay()
            torch.cuda.synchronize(dev)
            for i in range(len(self.PHASES)):
                tot[i] += evs[i].elapsed_time(evs[i + 1])
        del graph
        return [v / reps * 1e3 for v in tot]

    def errors(self):
        """Device-side errors of the plan (capacity exceeded: code 3, info = the peer); host-synchronising."""
        from . import _lib as L
        errs = L.all_workspace_errors(clear=True)
        return {k: v for k, v in errs.items() if k[0] == "ep"}

    # ------------------------------------------------------------------------------------------ forward
    def forward(self, x):
        """h + MoE(rms_norm(h)) for this rank's N packed tokens x [N, H] bf16."""
        if self.cuda_path and x.is_cuda:
            return self._forward_cuda(x)
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
