"""CUDA-graph replay of a block stack: the decode step and padded-bucket prefill.

ming-voice captures its whole decode step once per attention bucket and replays it (engine.py:694-714, replay at
:980), and captures prefill once per padded prompt length (PREFILL_BUCKETS 32 / 64 / 128, engine.py:716-757),
copying a prompt into a static buffer, zeroing the padding and replaying the bucket's graph (:950-961); longer
prompts run eagerly in chunks (:964-970). The same two patterns for a stack of MoE blocks:

  DecodeGraph(blocks, M)     one graph for M tokens through every block (one kernel per block).
  PrefillGraphs(blocks)      one graph per bucket; the padded rows are dropped from the expert GEMMs through a
                             device-side valid-row count (mv_mask_pad_rows), so one graph serves every length up
                             to its bucket.

Graphs are captured on a side stream after two eager warm-up runs (which create the workspaces: none is created
or resized inside a capture) and replayed on the caller's current stream. Results live in static buffers that
the next replay overwrites.
"""
from __future__ import annotations

import torch

PREFILL_BUCKETS = (32, 64, 128)


def _capture(fn, stream, pool):
    for _ in range(2):
        fn()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, pool=pool, stream=stream):
        fn()
    stream.synchronize()
    return g


class DecodeGraph:
    """M tokens through `blocks` (MoeBlock, linked or not) in one graph: x_in [M, H] -> y [M, H] bf16."""

    def __init__(self, blocks, M=1, device=None, ids=None):
        self.blocks = list(blocks)
        dev = torch.device(device) if device is not None else self.blocks[0].w_gu.device
        H = self.blocks[0].H
        self.x_in = torch.zeros(M, H, dtype=torch.bfloat16, device=dev)
        self.bufs = [torch.empty(M, H, dtype=torch.bfloat16, device=dev) for _ in self.blocks]
        # router ids of every block (the aux the reference block returns), [layers, M, top_k + n_shared] int32
        self.ids = torch.empty(len(self.blocks), M, self.blocks[0].nk, dtype=torch.int32, device=dev)

        def step():
            h = self.x_in
            for layer, blk in enumerate(self.blocks):
                blk.decode(h, out=self.bufs[layer], ids=self.ids[layer])
                h = self.bufs[layer]

        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            self.graph = _capture(step, s, torch.cuda.graph_pool_handle())
        torch.cuda.current_stream(dev).wait_stream(s)

    def __call__(self, x):
        self.x_in.copy_(x.reshape(self.x_in.shape), non_blocking=True)
        self.graph.replay()
        return self.bufs[-1]


class PrefillGraphs:
    """Padded-bucket prefill of `blocks`: prompts of up to max(buckets) tokens replay the graph of the smallest
    bucket that holds them; longer ones run eagerly through MoeBlock.prefill."""

    def __init__(self, blocks, buckets=PREFILL_BUCKETS, device=None):
        self.blocks = list(blocks)
        self.buckets = tuple(sorted(buckets))
        dev = torch.device(device) if device is not None else self.blocks[0].w_gu.device
        H = self.blocks[0].H
        tmax = self.buckets[-1]
        self.x = torch.zeros(tmax, H, dtype=torch.bfloat16, device=dev)
        self.y = torch.zeros(tmax, H, dtype=torch.bfloat16, device=dev)
        self.n_valid = torch.zeros(1, dtype=torch.int32, device=dev)
        self.graphs = {}
        pool = torch.cuda.graph_pool_handle()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for tb in self.buckets:
                self.n_valid.fill_(tb)

                def run(tb=tb):
                    h = self.x[:tb]
                    for blk in self.blocks:
                        h = blk.prefill(h, n_valid=self.n_valid)
                    self.y[:tb].copy_(h)

                self.graphs[tb] = _capture(run, s, pool)
        torch.cuda.current_stream(dev).wait_stream(s)

    def bucket(self, T):
        return next((b for b in self.buckets if b >= T), None)

    def __call__(self, x):
        """x [T, H] bf16 -> [T, H] (a view of the static output buffer when a bucket graph ran)."""
        T = x.shape[0]
        tb = self.bucket(T)
        if tb is None:
            h = x
            for blk in self.blocks:
                h = blk.prefill(h)
            return h
        self.x[:T].copy_(x, non_blocking=True)
        self.x[T:tb].zero_()
        self.n_valid.fill_(T)
        self.graphs[tb].replay()
        return self.y[:T]
