"""Expert-parallel prefill host logic (local pass, all-to-all exchange, combine) on CPU with 2 and 4 gloo ranks.

The experts themselves are the oracle's (this checks the exchange and bookkeeping, not the kernels); each
rank's EP output must equal the single-process block on its own tokens."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, I, E, K = 64, 32, 8, 3


class _RefBlock:
    """The attributes EPMoeBlock uses, with the oracle's router (no RMSNorm: x is already normalised)."""

    def __init__(self, p, shared_ids, bias):
        self.top_k, self.shared_ids, self.norm_w, self.eps = K, shared_ids, None, 1e-6
        self.p, self.bias = p, bias
        self.w_gu = self.w_d = self.s_gu = self.s_d = None

    def route(self, xn):
        from oracle import moe_oracle as O
        ids, wts, logits = O.route_softmax(xn, self.p["router_w"], bias=self.bias, top_k=K,
                                           shared_ids=self.shared_ids)
        return ids.to(torch.int32), wts, logits


def _worker(rank, world, port, seed, replicated, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ming-voice_b200")]
    from mingmoe.ep import EPMoeBlock, shard_block_params
    from oracle import moe_oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p = O.make_block_params(seed=seed, H=H, I=I, E=E, I_s=I, dtype=torch.float32)
        bias = O.zipf_bias(E)
        loc = shard_block_params(p, rank, world, E, replicated)

        def experts_fn(x, ids, wts):  # weight * expert(x) per row, this rank's stacks; id -1 = not here
            ids = ids.long()
            skip = ids < 0
            return O.moe_experts(x, loc["w_gu"], loc["w_d"], torch.where(skip, 0, ids),
                                 torch.where(skip, torch.zeros_like(wts), wts))

        ep = EPMoeBlock(_RefBlock(p, loc["shared_ids"], bias), E, replicated=replicated, experts_fn=experts_fn)
        x = O.make_tokens(13 + 7 * rank, H=H, seed=seed + rank, dtype=torch.float32)
        x0 = x.clone()
        y = ep.forward(x)
        assert torch.equal(x, x0)  # the input is not modified
        ids, wts, _ = O.route_softmax(x, p["router_w"], bias=bias, top_k=K, shared_ids=p["shared_ids"])
        ref = O.moe_experts(x, p["w_gu"], p["w_d"], ids, wts) + x
        q.put((rank, (y.float() - ref).abs().max().item()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("seed,replicated,world", [(0, (), 2), (5, (), 2), (3, (0, 1, 2), 2), (4, (0, 1), 4)])
def test_ep_prefill_ranks_match_single_block(seed, replicated, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seed, replicated, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    res = dict(q.get(timeout=5) for _ in range(world))
    assert all(pr.exitcode == 0 for pr in procs)
    assert all(v < 1e-4 for v in res.values()), res


def test_placement_tables():
    import sys
    sys.path.insert(0, __import__("os").path.join(__import__("os").path.dirname(__file__), "..", "ming-voice_b200"))
    from mingmoe.ep import placement
    owner, slot, stacks = placement(8, 3, replicated=(2, 5))
    assert stacks == [[2, 5, 0, 7], [2, 5, 1, 6], [2, 5, 3, 4]]  # snake: ranks 0 1 2, then 2 1 0
    for r, st in enumerate(stacks):
        for i, e in enumerate(st):
            assert slot[e] == i and owner[e] in (-1, r)
