"""The MoE block of ming-voice's thinker as one object: RMSNorm -> router -> routed + shared experts -> residual.

Mirrors the patched `BailingMoeV3SparseMoeBlock` forward (ming-voice engine.py:371-386) together with the
post-attention RMSNorm before it (engine.py:229) and the decoder layer's residual after it:

    h_out = h + MoE(rms_norm(h))

decode(x)   M <= 16 tokens: ONE cooperative kernel (mv_block_decode) does all of it.
prefill(x)  any N: RMSNorm kernel, router kernels, then the expert path for N tokens (grouped for large N).

Weights use the reference's stacked layout: w_gu [E1, 2I, H], w_d [E1, H, I] with the routed experts in
slots 0..E-1 and the shared expert in slots shared_ids (one slot of width I as in ming-voice, or several
slots when the shared expert is wider: SwiGLU is separable over its intermediate dimension).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from . import moe

ROUTE_MODES = {"softmax": L.MV_ROUTE_SOFTMAX, "sigmoid_group": L.MV_ROUTE_SIGMOID_GROUP}


class MoeBlock:
    def __init__(self, w_gu, w_d, router_w, norm_w, *, top_k, shared_ids, eps=1e-6, s_gu=None, s_d=None,
                 router_s=None, router_bias=None, route_mode="softmax", n_group=1, topk_group=1, route_scale=1.0):
        L.require_cuda(w_gu, w_d, router_w, norm_w, s_gu, s_d, router_s, router_bias)
        self.w_gu, self.w_d, self.s_gu, self.s_d = w_gu, w_d, s_gu, s_d
        self.router_w = router_w.contiguous()
        self.router_s = None if router_s is None else router_s.contiguous()
        self.router_bias = None if router_bias is None else router_bias.float().contiguous()
        self.norm_w = None if norm_w is None else norm_w.contiguous()
        self.eps = float(eps)
        self.E, self.H = self.router_w.shape
        self.I = w_d.shape[-1]
        self.top_k = int(top_k)
        shared_ids = tuple(int(s) for s in shared_ids)
        if shared_ids and shared_ids != tuple(range(shared_ids[0], shared_ids[0] + len(shared_ids))):
            raise ValueError("shared slots must be consecutive")
        self.shared_ids = shared_ids
        self.route_mode = route_mode
        self.n_group, self.topk_group, self.route_scale = int(n_group), int(topk_group), float(route_scale)
        if self.norm_w is not None and self.norm_w.dtype != torch.bfloat16:
            raise TypeError("norm weight must be bf16")
        self._w = moe.weights_struct(w_gu, w_d, s_gu, s_d)
        b = L.Block()
        b.experts = self._w
        b.norm_w = None if self.norm_w is None else self.norm_w.data_ptr()
        b.router_w = self.router_w.data_ptr()
        b.router_scale = None if self.router_s is None else self.router_s.data_ptr()
        b.router_bias = None if self.router_bias is None else self.router_bias.data_ptr()
        b.eps = self.eps
        b.router_dtype = L.dt(self.router_w)
        b.router_scale_dtype = L.dt(self.router_s) if self.router_s is not None else L.MV_F32
        b.E, b.top_k = self.E, self.top_k
        b.route_mode = ROUTE_MODES[route_mode]
        b.n_group, b.topk_group, b.route_scale = self.n_group, self.topk_group, self.route_scale
        b.n_shared = len(shared_ids)
        b.shared_id = shared_ids[0] if shared_ids else 0
        b.residual_from_x = 1
        self._block = b
        self._next = None
        self.nk = self.top_k + len(shared_ids)

    @classmethod
    def from_params(cls, p, device="cuda", route_mode="softmax", top_k=6, router_bias=None):
        """From a parameter dict of oracle.moe_oracle.make_block_params (tests and benchmarks)."""
        g = {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in p.items()}
        return cls(g["w_gu"], g["w_d"], g["router_w"], g["norm_w"], top_k=top_k, shared_ids=p["shared_ids"],
                   eps=p["eps"], s_gu=g.get("s_gu"), s_d=g.get("s_d"), router_s=g.get("router_s"),
                   router_bias=None if router_bias is None else router_bias.to(device), route_mode=route_mode,
                   n_group=p.get("n_group", 1), topk_group=p.get("topk_group", 1), route_scale=p.get("scale", 1.0))

    def link(self, nxt):
        """Declare the block decoded after this one (None to unlink). While this block's decode kernel runs it
        prefetches the next block's router and RMSNorm weights into L2, so the next block's routing starts from L2.
        A layer stack links block l to block l + 1 (and the last to the first when steps repeat)."""
        self._next = nxt
        self._block.next = None if nxt is None else C.addressof(nxt._block)
        return self

    # ------------------------------------------------------------------------------------------ decode
    def workspace_bytes(self, M=moe.DECODE_MAX_M):
        return L.lib().mv_block_decode_workspace_bytes_tc(C.byref(self._block), M)

    def decode(self, x, out=None, logits=None, ids=None, wts=None):
        """h + MoE(rms_norm(h)) for M <= 16 tokens in one kernel. x [M, H] bf16. Optional router outputs are
        written into `logits` [M, E] fp32, `ids` [M, top_k + n_shared] int32/int64, `wts` fp32."""
        L.require_cuda(x)
        x2 = x.reshape(-1, self.H)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if x2.dtype != torch.bfloat16:
            raise TypeError("decode: x must be bf16")
        M = x2.shape[0]
        if M > moe.DECODE_MAX_M:
            raise ValueError(f"decode handles at most {moe.DECODE_MAX_M} tokens")
        y = torch.empty_like(x2) if out is None else out.view(M, self.H)
        ws = L.workspace("block", self.workspace_bytes(), x.device)
        L.check(L.lib().mv_block_decode(C.byref(self._block), L.ptr(x2), M, L.ptr(y), L.ptr(logits), L.ptr(ids),
                                        L.dt(ids) if ids is not None else L.MV_I64, L.ptr(wts), L.ptr(ws), ws.numel(),
                                        L.stream_ptr(x.device)), "mv_block_decode")
        return y.view(x.shape)

    # ------------------------------------------------------------------------------------------ prefill
    def route(self, xn):
        """Router over normalised tokens: (ids [N, top_k + n_shared] int32, wts fp32, logits [N, E] fp32)."""
        import fused_ops  # the drop-in module (same directory on sys.path)
        N = xn.shape[0]
        ids = torch.empty(N, self.nk, dtype=torch.int32, device=xn.device)
        wts = torch.empty(N, self.nk, dtype=torch.float32, device=xn.device)
        logits = torch.empty(N, self.E, dtype=torch.float32, device=xn.device)
        fused_ops.moe_route(xn, self.router_w, self.router_bias, self.n_group, self.topk_group, self.top_k,
                            self.route_scale, logits, ids, wts, mode=self.route_mode, n_shared=len(self.shared_ids),
                            shared_id=self.shared_ids[0] if self.shared_ids else self.E, w_scale=self.router_s)
        return ids, wts, logits

    def prefill(self, x, n_valid=None):
        """h + MoE(rms_norm(h)) for N packed tokens (any N; sequences are independent per token).

        n_valid: optional device int32 [1]; rows >= n_valid[0] are padding (a prompt padded to a bucket length
        whose graph was captured once): their expert pairs are dropped (mv_mask_pad_rows) and they come out as
        their input."""
        import fused_ops
        x2 = x.reshape(-1, self.H)
        xn = fused_ops.rms_norm(x2, self.norm_w, self.eps) if self.norm_w is not None else x2
        ids, wts, _ = self.route(xn)
        if n_valid is not None:
            L.check(L.lib().mv_mask_pad_rows(L.ptr(ids), L.dt(ids), ids.shape[0], ids.shape[1], L.ptr(n_valid),
                                             L.stream_ptr(x.device)), "mv_mask_pad_rows")
        y = moe.experts(xn, self.w_gu, self.w_d, ids, wts, s_gu=self.s_gu, s_d=self.s_d, residual=x2)
        return y.view(x.shape)
