"""CPU oracle for the Ling-style MoE block hot path of ming-voice.

TEST INFRASTRUCTURE ONLY. Nothing in the product (the `ming-voice_b200` package, its C-ABI library or its
kernels) imports or calls this module. Only `tests/`, `__graft_entry__.smoke()` and the CPU legs of
`bench.py` (`cpu_baseline`, `--impl reference`) use it, and only as the checker / the timed CPU baseline.

It restates, in torch/numpy on the CPU, the reference's algorithm for each function on the path:

  rms_norm            fused_ops.py:16-37       (fp32 statistics, normalise, cast, scale)
  route_sigmoid_group fused_ops.py:40-103       (fp32 gate GEMV, sigmoid + bias, group-limited top-k,
                                                 renormalise (+1e-20), x scale, shared expert appended);
                      engine.py:326-333        (the patched torch gate, same maths for N tokens)
  route_softmax       BASELINE router: softmax(logits [+ bias]) -> top-k -> renormalise
  quantize_rows_int8  fused_moe.py:199-204     (symmetric per-row int8, torch.round = half-to-even)
  align_blocks        fused_moe.py:154-173     (counting sort of (token, slot) pairs by expert, BM padding)
  moe_experts         fused_moe.py:67-83 / :176-196, dev/test_moe_prefill.py:24-38 (per-expert SwiGLU loop,
                      weighted combine)
  small_linear        fastlinear.py:20-62, :142-174

Precision policy. The reference computes in fp32 and rounds several intermediates to bf16
(fused_moe.py:34-38, :60-61, :118-121, :147-148). The oracle has two modes for the expert maths:

  rounding="fp32"       the BASELINE "fp32 reference": every intermediate stays fp32.
  rounding="reference"  mirrors the reference kernels' bf16 rounding points exactly; used to pin the oracle
                        against golden vectors produced by the reference's own kernels.

For the router and the RMSNorm statistics the oracle evaluates the reference's formulas with fp64
internals and rounds to fp32 at the points where the reference holds an fp32 value (the logit, the
score, the weight, the variance). Any correct fp32 implementation lands within its own rounding error of
these values, and they do not depend on a summation order, so top-k selections compare bit-exactly.
Ties in a top-k selection go to the lower expert id, as the reference's argmax loop does
(fused_ops.py:72-86: tl.argmax returns the first maximum).
"""
from __future__ import annotations

import math

import numpy as np
import torch

# ----------------------------------------------------------------------------------------------- helpers


def bf16(t: torch.Tensor) -> torch.Tensor:
    """Round to bf16 (round-to-nearest-even) and return as fp32."""
    return t.to(torch.bfloat16).to(torch.float32)


def _f64(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float64)


# ----------------------------------------------------------------------------------------------- RMSNorm


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """BailingMoeV3RMSNorm as fused_ops.py:16-37 computes it.

    var = mean(x^2) in fp32 (here: exact fp64 sum of the squares, rounded once to fp32);
    y = cast(x * (1 / sqrt(var + eps)), x.dtype); out = cast(w * y, promote(w.dtype, x.dtype)).
    The reference kernel casts the normalised row to bf16 (fused_ops.py:23); for bf16 inputs that is
    the input dtype, which is the cast the HF module performs and the one kept here for every dtype.
    The reciprocal square root is 1/sqrt with both operations correctly rounded, so a GPU kernel that uses
    IEEE sqrt and division reproduces it bit for bit.
    """
    n = x.shape[-1]
    xf = x.float()
    ss = (_f64(xf) * _f64(xf)).sum(-1, keepdim=True)
    var = (ss / n).float()
    r = 1.0 / torch.sqrt(var + torch.tensor(eps, dtype=torch.float32))
    y = (xf * r).to(x.dtype).float()
    out_dtype = torch.promote_types(w.dtype, x.dtype)
    return (w.float() * y).to(out_dtype)


# ----------------------------------------------------------------------------------------------- router


def router_logits(x: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 logits = x @ W^T (fused_ops.py:40-50, engine.py:328), evaluated in fp64 and rounded to fp32.

    `w` may be fp32 (the reference's w32 copy, engine.py:324), bf16, or int8 with a per-row scale
    (`w_scale`, dequantised as q.float() * s.float())."""
    if w.dtype == torch.int8:
        assert w_scale is not None
        wf = dequant_rows_int8(w, w_scale)
    else:
        wf = w.float()
    return (_f64(x.float()) @ _f64(wf).T).float()


def _topk_desc(r: torch.Tensor, k: int) -> torch.Tensor:
    """Indices of the k largest values per row, largest first; equal values: lower index first."""
    # stable sort on -r keeps ascending index order among equal keys
    order = np.argsort(-r.double().numpy(), axis=-1, kind="stable")[..., :k]
    return torch.from_numpy(np.ascontiguousarray(order)).long()


def route_softmax(x, w, bias=None, top_k=6, shared_ids=(), w_scale=None):
    """BASELINE router: logits (+ per-expert bias) -> softmax -> top-k -> renormalise; shared slots appended
    with weight 1.0 (the reference appends its shared expert the same way, fused_ops.py:89-93).

    Returns (ids [M, top_k + n_shared] int64, wts [M, top_k + n_shared] fp32, logits [M, E] fp32).
    Softmax is monotonic, so the selection is made on the biased logits; the weights are
    exp(l_k - l_max) / sum_{j in top-k} exp(l_j - l_max), evaluated in fp64 and rounded to fp32."""
    logits = router_logits(x, w, w_scale)
    r = logits if bias is None else (logits + bias.float())
    idx = _topk_desc(r, top_k)
    r64 = _f64(r)
    mx = r64.max(-1, keepdim=True).values
    e = torch.exp(torch.gather(r64, 1, idx) - mx)
    wts = (e / e.sum(-1, keepdim=True)).float()
    M = x.shape[0]
    if shared_ids:
        sid = torch.tensor(list(shared_ids), dtype=torch.long).expand(M, -1)
        idx = torch.cat([idx, sid], 1)
        wts = torch.cat([wts, torch.ones(M, len(shared_ids))], 1)
    return idx, wts, logits


def route_sigmoid_group(x, w32, bias, n_group, topk_group, top_k, scale, n_shared=1, shared_id=None):
    """The reference router (fused_ops.py:53-93 for one token; engine.py:326-333 for N tokens).

    scores = sigmoid(logits); r = scores + bias; a group's score is the sum of its two largest r
    (fused_ops.py:63-68); the topk_group best groups are kept (:69-76); the top_k experts by r among
    them are taken largest first (:77-86); their *sigmoid scores* are renormalised by (sum + 1e-20)
    and multiplied by `scale` (:87-88); the shared expert (id E by default) follows with weight 1.
    Returns (ids [M, top_k + n_shared], wts fp32, logits fp32)."""
    logits = router_logits(x, w32)
    M, E = logits.shape
    G = n_group
    GS = E // G
    scores64 = 1.0 / (1.0 + torch.exp(-_f64(logits)))
    scores = scores64.float()
    r = scores + bias.float()
    ids_out, wts_out = [], []
    for m in range(M):
        rm = r[m].double().numpy()
        rg = rm.reshape(G, GS)
        gscore = np.empty(G)
        for g in range(G):
            a1 = int(np.argmax(rg[g]))  # first max
            rest = rg[g].copy()
            rest[a1] = -np.inf
            gscore[g] = np.float32(np.float32(rg[g][a1]) + np.float32(rest.max()))
        keep = np.zeros(G, dtype=bool)
        gs = gscore.copy()
        for _ in range(topk_group):
            b = int(np.argmax(gs))
            keep[b] = True
            gs[b] = -np.inf
        masked = np.where(np.repeat(keep, GS), rm, -np.inf)
        sel = []
        for _ in range(top_k):
            e = int(np.argmax(masked))
            sel.append(e)
            masked[e] = -np.inf
        sw = scores[m, sel].double()
        tot = sw.sum()
        wv = (sw / (tot + 1e-20) * float(scale)).float()
        sid = E if shared_id is None else shared_id
        ids_out.append(sel + [sid + j for j in range(n_shared)])
        wts_out.append(torch.cat([wv, torch.ones(n_shared)]))
    return torch.tensor(ids_out, dtype=torch.long), torch.stack(wts_out), logits


# ----------------------------------------------------------------------------------------------- int8


def quantize_rows_int8(w: torch.Tensor, scale_dtype=torch.float32):
    """fused_moe.py:199-204: amax = max|w| per row (fp32, clamp_min 1e-8), scale = amax / 127,
    q = round_half_even(w / scale).clamp(-127, 127). With scale_dtype=bf16 the scale is rounded to bf16
    first and q is computed against the rounded scale (BASELINE's "scale stored bf16")."""
    amax = w.abs().amax(dim=-1).float().clamp_min(1e-8)
    scale = amax / 127.0
    if scale_dtype == torch.bfloat16:
        scale = scale.to(torch.bfloat16)
    q = torch.round(w.float() / scale.float()[..., None]).clamp_(-127, 127).to(torch.int8)
    return q, scale


def dequant_rows_int8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """torch dequantisation: q.float() * s.float() per row (fp32)."""
    return q.float() * scale.float()[..., None]


# ----------------------------------------------------------------------------------------------- align


def align_blocks(flat: np.ndarray, E1: int, BM: int):
    """fused_moe.py:154-173: sort pair indices by expert (stable), pad each expert's run to a multiple of
    BM. Returns (sorted_ids [nb*BM] int32 with P as padding, bexp [nb] int32 with -1 for unused, nb)."""
    flat = np.asarray(flat, dtype=np.int64)
    P = flat.size
    counts = np.bincount(flat, minlength=E1)[:E1]
    padded = (counts + BM - 1) // BM * BM
    pend = np.cumsum(padded)
    pstart = pend - padded
    order = np.argsort(flat, kind="stable")
    se = flat[order]
    cstart = np.cumsum(counts) - counts
    dest = pstart[se] + np.arange(P) - cstart[se]
    nb = (P + E1 * (BM - 1) + BM - 1) // BM
    sorted_ids = np.full(nb * BM, P, dtype=np.int32)
    sorted_ids[dest] = order.astype(np.int32)
    bexp = np.searchsorted(pend, np.arange(nb) * BM, side="right")
    bexp = np.where(bexp < E1, bexp, -1).astype(np.int32)
    return sorted_ids, bexp, nb


# ----------------------------------------------------------------------------------------------- experts


def _expert_weights(w_gu, w_d, s_gu, s_d):
    if s_gu is not None:
        return dequant_rows_int8(w_gu, s_gu), dequant_rows_int8(w_d, s_d)
    return w_gu.float(), w_d.float()


def moe_experts(x, w_gu, w_d, ids, wts, s_gu=None, s_d=None, rounding="fp32"):
    """y[n] = sum_k wts[n,k] * down_e(silu(gate_e(x_n)) * up_e(x_n)), e = ids[n,k].

    Layout as the reference stacks it (engine.py:150-188, fused_moe.py:3-6): w_gu [E1, 2I, H] with gate rows
    [0, I) and up rows [I, 2I); w_d [E1, H, I]; int8 weights carry per-row scales s_gu [E1, 2I], s_d [E1, H].
    rounding="fp32": fp32 throughout, output fp32 (the BASELINE fp32 reference).
    rounding="reference": the reference kernels' rounding (fused_moe.py:31-38, :58-61 for decode and
    :115-121, :144-148, :196 for prefill): gate/up accumulators -> bf16, silu -> bf16, product -> bf16,
    per-expert down output -> bf16, then the weighted sum in fp32; int8 applies the row scale to the fp32
    accumulator (dot(q, x) * s) like the reference kernels do. Returns fp32 [N, H]."""
    N, H = x.shape
    I = w_d.shape[-1]
    ids = ids.reshape(N, -1).long()
    wts = wts.reshape(N, -1).float()
    xf = x.float()
    y = torch.zeros(N, H, dtype=torch.float32)
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    KP1 = ids.shape[1]
    for e in torch.unique(flat).tolist():
        sel = order[flat[order] == e]
        tok = sel // KP1
        xs = xf[tok]
        if rounding == "fp32":
            wgu, wd = _expert_weights(w_gu[e], w_d[e], None if s_gu is None else s_gu[e],
                                      None if s_d is None else s_d[e])
            gu = xs @ wgu.T
            a = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
            o = a @ wd.T
        else:
            if s_gu is not None:
                gu = (xs @ w_gu[e].float().T) * s_gu[e].float()
            else:
                gu = xs @ w_gu[e].float().T
            g = bf16(gu[:, :I])
            u = bf16(gu[:, I:])
            g = bf16(g / (1.0 + torch.exp(-g)))
            a = bf16(g * u)
            if s_d is not None:
                o = (a @ w_d[e].float().T) * s_d[e].float()
            else:
                o = a @ w_d[e].float().T
            o = bf16(o)
        y.index_add_(0, tok, o * wts.reshape(-1)[sel][:, None])
    return y


# ----------------------------------------------------------------------------------------------- small linear


def small_linear(x, w, b=None, act=0, residual=None, norm=None, rounding="reference"):
    """fastlinear.py:20-62: y = act(norm?(x) @ W^T + b) + residual, fp32 accumulate.
    The norm prologue is rstd = 1/sqrt(mean(x^2) + eps), x_n = bf16(bf16(x * rstd) * gamma) (:29-44);
    with an activation, the pre-activation is rounded to bf16 first (:50-57); with a residual, the
    activation output is rounded to bf16 before the add (:59-61). act: 0 none, 1 gelu-tanh, 2 silu."""
    xf = x.float()
    if norm is not None:
        g, eps = norm
        ss = (_f64(xf) * _f64(xf)).sum(-1, keepdim=True)
        var = (ss / xf.shape[-1]).float()
        r = 1.0 / torch.sqrt(var + torch.tensor(float(eps), dtype=torch.float32))
        xf = bf16(bf16(xf * r) * g.float())
    acc = xf @ w.float().T
    if b is not None:
        acc = acc + b.float()
    if act == 1:
        acc = bf16(acc) if rounding == "reference" else acc
        c = 0.7978845608028654 * (acc + 0.044715 * acc * acc * acc)
        acc = 0.5 * acc * (1.0 + torch.tanh(c))
    elif act == 2:
        acc = bf16(acc) if rounding == "reference" else acc
        acc = acc / (1.0 + torch.exp(-acc))
    if residual is not None:
        acc = (bf16(acc) if rounding == "reference" else acc) + residual.float()
    return acc


# ----------------------------------------------------------------------------------------------- block


def moe_block(x, p, rounding="fp32", top_k=6, router="softmax", bias=None):
    """One Ling-style MoE block with residual (the decoder layer's h + MoE(post_attention_layernorm(h))):

      xn  = rms_norm(x, p["norm_w"], p["eps"])                     (bf16 inputs: xn is bf16, as the reference)
      ids, wts = router(xn)                                         (softmax top-k, BASELINE; or sigmoid-group)
      y   = x + sum_k wts_k * expert_{ids_k}(xn)                    (shared-expert slots carry weight 1)

    `p` holds the stacked weights (w_gu [E1, 2I, H], w_d [E1, H, I], optional int8 scales), the router
    weight `router_w` [E, H] (+ `router_s` for int8) and `shared_ids` (the slots appended to every token).
    Returns (y fp32 [M, H], ids, wts, xn)."""
    xn = rms_norm(x, p["norm_w"], p["eps"])
    if router == "softmax":
        ids, wts, _ = route_softmax(xn, p["router_w"], bias=bias, top_k=top_k, shared_ids=p["shared_ids"],
                                    w_scale=p.get("router_s"))
    else:
        ids, wts, _ = route_sigmoid_group(xn, p["router_w"], p["router_bias"], p["n_group"], p["topk_group"],
                                          top_k, p["scale"], n_shared=len(p["shared_ids"]),
                                          shared_id=p["shared_ids"][0])
    y = moe_experts(xn, p["w_gu"], p["w_d"], ids, wts, p.get("s_gu"), p.get("s_d"), rounding=rounding)
    return y + x.float(), ids, wts, xn


# ----------------------------------------------------------------------------------------------- configs

H_BASE, I_BASE, E_BASE, K_BASE, IS_BASE = 2048, 1408, 64, 6, 2816
PREFILL_LENS = (37, 211, 512, 1283)


def zipf_bias(E: int) -> torch.Tensor:
    """BASELINE prefill router bias: b_e = 2 * log(1 / (e + 1)^1.1) (e = 0 .. E-1), fp32."""
    e = torch.arange(E, dtype=torch.float64)
    return (2.0 * torch.log(1.0 / (e + 1.0) ** 1.1)).float()


def make_block_params(seed=0, H=H_BASE, I=I_BASE, E=E_BASE, I_s=IS_BASE, dtype=torch.bfloat16, std=0.02,
                      int8=False, scale_dtype=torch.bfloat16, eps=1e-6):
    """Seeded synthetic block weights: routed experts + a shared SwiGLU expert of
    intermediate I_s, stored as I_s / I extra slots of the stacked tensors (SwiGLU is separable over
    its intermediate dimension, so a 2I-wide shared expert equals two I-wide slots of weight 1)."""
    assert I_s % I == 0
    ns = I_s // I
    g = torch.Generator().manual_seed(seed)
    E1 = E + ns
    w_gu = (torch.randn(E1, 2 * I, H, generator=g) * std)
    w_d = (torch.randn(E1, H, I, generator=g) * std)
    router_w = torch.randn(E, H, generator=g) * std
    if ns > 1:
        # one shared expert of width I_s, split into ns slots: gate/up rows and down columns by block
        sg = torch.randn(I_s, H, generator=g) * std
        su = torch.randn(I_s, H, generator=g) * std
        sd = torch.randn(H, I_s, generator=g) * std
        for j in range(ns):
            w_gu[E + j, :I] = sg[j * I:(j + 1) * I]
            w_gu[E + j, I:] = su[j * I:(j + 1) * I]
            w_d[E + j] = sd[:, j * I:(j + 1) * I]
    p = dict(w_gu=w_gu.to(dtype), w_d=w_d.to(dtype), router_w=router_w.to(dtype),
             norm_w=torch.ones(H, dtype=dtype), eps=eps, shared_ids=tuple(range(E, E1)), E=E, I=I, H=H)
    if int8:
        p["w_gu"], p["s_gu"] = quantize_rows_int8(p["w_gu"], scale_dtype)
        p["w_d"], p["s_d"] = quantize_rows_int8(p["w_d"], scale_dtype)
        p["router_w"], p["router_s"] = quantize_rows_int8(p["router_w"], scale_dtype)
    return p


def make_tokens(M, H=H_BASE, seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed + 1000)
    return torch.randn(M, H, generator=g).to(dtype)


def prefill_cu_seqlens(lens=PREFILL_LENS):
    return [0] + list(np.cumsum(lens).tolist())


def distinct_experts(ids: torch.Tensor) -> int:
    return int(torch.unique(ids.reshape(-1)).numel())


def decode_bytes(U, H=H_BASE, I=I_BASE, E=E_BASE, esz=2, scale_bytes=0, M=1, I_s=IS_BASE):
    """Algorithmic bytes of one decode block step: U routed experts' gate/up/down weights, the shared expert,
    the router, the norm weight and the activations (x in, residual in, y out)."""
    ns = I_s // I
    w = (U + ns) * 3 * I * H * esz + E * H * esz + H * 2
    s = (U + ns) * (2 * I + H) * scale_bytes + (E * scale_bytes if scale_bytes else 0)
    return w + s + 3 * M * H * 2


def prefill_flops(N, H=H_BASE, I=I_BASE, E=E_BASE, K=K_BASE, I_s=IS_BASE):
    """Algorithmic FLOPs of one prefill block pass: 2 * N * (K * 3 * I * H + 3 * I_s * H + E * H)."""
    return 2 * N * (K * 3 * I * H + 3 * I_s * H + E * H)


__all__ = [n for n in dir() if not n.startswith("_")] + ["_topk_desc"]
