"""Generate golden input/output vectors from the reference's own kernels.

Run in a container that has the reference sources (read-only) and Triton:

    python tests/golden/make_golden.py <path of the ming-voice sources>

It imports the reference's `fused_moe.py`, `fused_ops.py` and `fastlinear.py` with TRITON_INTERPRET=1, so the
reference Triton kernels execute on the CPU, feeds them small seeded inputs and saves inputs + outputs to
`tests/golden/*.pt`. The committed fixtures are what the CPU tests pin the oracle against; the GPU box never
runs this script (the reference is not present there).

Shapes are small (H=128, I=32, E=8) because the interpreter is slow; tile configs are set so that every
tile divides its dimension (the reference kernels do not mask ragged tiles, fused_moe.py:24-30), and the
router fixture uses H=256 because `moe_route` hard-codes BK=256 (fused_ops.py:100).

Two interpreter defects of Triton 3.6 are corrected here, in the interpreter, before the reference modules
are imported (the reference sources are not modified):
  * `cast_impl` truncates fp32 -> bf16 and copies an integer's value into the bf16 bit pattern
    (int8 -> bf16); the compiled kernel rounds to nearest even (cvt.rn.bf16.f32) and converts integers by
    value.
  * `create_dot` multiplies the raw uint16 bit patterns of bf16 operands as integers; the compiled kernel
    multiplies the bf16 values with fp32 accumulation.
"""
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"
if len(sys.argv) != 2:
    sys.exit("usage: python tests/golden/make_golden.py <path of the ming-voice sources>")
REF = sys.argv[1]
sys.path.insert(0, REF)
HERE = os.path.dirname(os.path.abspath(__file__))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton.language as tl  # noqa: E402
from triton.runtime import interpreter as _interp  # noqa: E402


def _bf16_bits_to_f32(a):
    return (np.ascontiguousarray(a).astype(np.uint32) << 16).view(np.float32)


_orig_cast = _interp.InterpreterBuilder.cast_impl


def _cast_impl(self, src, dst_type):
    s, d = src.dtype.scalar, dst_type.scalar
    if d == tl.bfloat16 and (s == tl.float32 or s.is_int()):
        t = torch.from_numpy(np.ascontiguousarray(src.data).astype(np.float32)).to(torch.bfloat16)
        return _interp.TensorHandle(t.view(torch.int16).numpy().view(np.uint16), d)
    return _orig_cast(self, src, dst_type)


_orig_dot = _interp.InterpreterBuilder.create_dot


def _create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
    if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
        ad = _bf16_bits_to_f32(a.data) if a.dtype.scalar == tl.bfloat16 else a.data.astype(np.float32)
        bd = _bf16_bits_to_f32(b.data) if b.dtype.scalar == tl.bfloat16 else b.data.astype(np.float32)
        return _interp.TensorHandle(np.matmul(ad, bd, dtype=np.float32) + d.data, d.dtype.scalar)
    return _orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)


_interp.InterpreterBuilder.cast_impl = _cast_impl
_interp.InterpreterBuilder.create_dot = _create_dot

import fastlinear  # noqa: E402
import fused_moe  # noqa: E402
import fused_ops  # noqa: E402


def save(name, **kw):
    path = os.path.join(HERE, name + ".pt")
    torch.save({k: (v.contiguous() if torch.is_tensor(v) else v) for k, v in kw.items()}, path)
    print("wrote", path)


def gen_rms_norm():
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(7, 256, generator=g) * 3).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(256, generator=g)).to(torch.bfloat16)
    y = fused_ops.rms_norm(x, w, 1e-6)
    save("rms_norm", x=x, w=w, eps=1e-6, y=y)


def gen_route():
    g = torch.Generator().manual_seed(12)
    E, H, G, TG, K, scale = 64, 256, 8, 4, 8, 2.5
    w32 = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16).float()
    # exact ties: identical router rows give identical logits; the lower id must come first
    w32[9] = w32[5]
    w32[40] = w32[5]
    bias = (torch.randn(E, generator=g) * 0.01).float()
    bias[9] = bias[5]
    bias[40] = bias[5]
    xs = torch.randn(6, H, generator=g).to(torch.bfloat16)
    xs[5] = (w32[5] * 4.0).to(torch.bfloat16)  # a token that strongly prefers the tied experts
    ids_all, wts_all, logits_all = [], [], []
    for t in range(xs.shape[0]):
        logits = torch.empty(E)
        ids = torch.empty(K + 1, dtype=torch.long)
        wts = torch.empty(K + 1)
        fused_ops.moe_route(xs[t:t + 1], w32, bias, G, TG, K, scale, logits, ids, wts)
        ids_all.append(ids.clone())
        wts_all.append(wts.clone())
        logits_all.append(logits.clone())
    save("moe_route", x=xs, w32=w32, bias=bias, n_group=G, topk_group=TG, top_k=K, scale=scale,
         ids=torch.stack(ids_all), wts=torch.stack(wts_all), logits=torch.stack(logits_all))


def gen_quant():
    g = torch.Generator().manual_seed(13)
    w = (torch.randn(3, 16, 128, generator=g) * 0.02).to(torch.bfloat16)
    w[0, 3] = 0  # an all-zero row: amax clamps to 1e-8
    w[1, 2, :4] = torch.tensor([0.5, -0.5, 1.5, -2.5]).to(torch.bfloat16) * (1.0 / 127.0)
    w[1, 2, 4] = 1.0 / 63.5  # amax row: scale 1/127/63.5... exercises round-half-even on exact halves
    q, s = fused_moe.quantize_rows_int8(w)
    save("quantize_rows_int8", w=w, q=q, scale=s)


def gen_align():
    g = torch.Generator().manual_seed(14)
    E1, BM = 9, 4
    flat = torch.randint(0, E1 - 1, (13 * 4,), generator=g)
    flat[3::4] = E1 - 1
    flat[:8] = 2  # a heavy expert
    sorted_ids, bexp, nb = fused_moe._align_blocks(flat, E1, BM)
    save("align_blocks", flat=flat, E1=E1, BM=BM, sorted_ids=sorted_ids, bexp=bexp, nb=nb)


def moe_weights(seed):
    g = torch.Generator().manual_seed(seed)
    E, H, I = 8, 128, 32
    w_gu = (torch.randn(E + 1, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    w_d = (torch.randn(E + 1, H, I, generator=g) * 0.05).to(torch.bfloat16)
    return g, E, H, I, w_gu, w_d


def gen_decode():
    g, E, H, I, w_gu, w_d = moe_weights(15)
    x = torch.randn(1, H, generator=g).to(torch.bfloat16)
    ids = torch.tensor([3, 6, 1, E])
    wts = torch.tensor([0.5, 0.3, 0.2, 1.0])
    fused_moe.CFG["A"] = dict(BN=16, BK=64, num_warps=4)
    fused_moe.CFG["B"] = dict(BN=16, BK=32, num_warps=4)
    y = fused_moe.fused_moe_decode(x, w_gu, w_d, ids, wts)
    q_gu, s_gu = fused_moe.quantize_rows_int8(w_gu)
    q_d, s_d = fused_moe.quantize_rows_int8(w_d)
    y8 = fused_moe.fused_moe_decode(x, q_gu, q_d, ids, wts, s_gu=s_gu, s_d=s_d)
    save("moe_decode", x=x, w_gu=w_gu, w_d=w_d, ids=ids, wts=wts, y=y,
         q_gu=q_gu, s_gu=s_gu, q_d=q_d, s_d=s_d, y_int8=y8)


def gen_prefill():
    g, E, H, I, w_gu, w_d = moe_weights(16)
    N, K = 13, 3
    x = torch.randn(N, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(N, E, generator=g)
    ids = torch.cat([logits.topk(K, -1).indices, torch.full((N, 1), E)], 1)
    wts = torch.cat([torch.rand(N, K, generator=g), torch.ones(N, 1)], 1)
    fused_moe.GCFG["A"] = dict(BM=32, BN=32, BK=128, num_warps=4)
    fused_moe.GCFG["B"] = dict(BM=32, BN=64, BK=32, num_warps=4)
    y = fused_moe.fused_moe_prefill(x, w_gu, w_d, ids, wts)
    q_gu, s_gu = fused_moe.quantize_rows_int8(w_gu)
    q_d, s_d = fused_moe.quantize_rows_int8(w_d)
    y8 = fused_moe.fused_moe_prefill(x, q_gu, q_d, ids, wts, s_gu=s_gu, s_d=s_d)
    save("moe_prefill", x=x, w_gu=w_gu, w_d=w_d, ids=ids, wts=wts, y=y,
         q_gu=q_gu, s_gu=s_gu, q_d=q_d, s_d=s_d, y_int8=y8)


def gen_small_linear():
    g = torch.Generator().manual_seed(17)
    M, K, N = 3, 128, 96
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    r = torch.randn(M, N, generator=g).to(torch.bfloat16)
    gamma = (1.0 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    cases = {}
    cfg = dict(BN=32, BK=64, num_warps=4)
    for name, kw in {"plain": {}, "bias_gelu_res": dict(b=b, act=1, res=r), "silu": dict(act=2),
                     "norm_bias": dict(b=b, norm=(gamma, 1e-6)), "norm_gelu_res": dict(b=b, act=1, res=r,
                                                                                        norm=(gamma, 1e-6))}.items():
        y = torch.empty(M, N, dtype=torch.bfloat16)
        fastlinear._launch(x, w, kw.get("b"), kw.get("res"), kw.get("act", 0), cfg, y, kw.get("norm"))
        cases[name] = y
    save("small_linear", x=x, w=w, b=b, r=r, gamma=gamma, eps=1e-6, **{"y_" + k: v for k, v in cases.items()})


if __name__ == "__main__":
    torch.manual_seed(0)
    gen_rms_norm()
    gen_route()
    gen_quant()
    gen_align()
    gen_decode()
    gen_prefill()
    gen_small_linear()
