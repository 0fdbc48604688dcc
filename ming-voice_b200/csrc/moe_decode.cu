// Decode MoE block (M <= 16 tokens) in one cooperative kernel.
//
// Replaces fused_moe.fused_moe_decode (ming-voice fused_moe.py:67-83, kernels _moe_gate_up :14-38 and
// _moe_down :42-61), the M = 2..16 use of fused_moe_prefill (engine.py:381-382), and, with the router fused
// in, the whole single-token MoE forward of the patched block (engine.py:371-386: moe_route + fused decode).
//
// The step moves ~U x 17 MB of weights (bf16, H=2048, I=1408) and almost nothing else, so the design goal is
// one uninterrupted stream of large contiguous weight reads across all SMs:
//
//  * gate/up phase: the rows (gate row i + up row i of w_gu[e], 2 x H elements) of the selected experts are
//    split into equal contiguous ranges, one per CTA (one CTA per SM). A CTA computes
//      a[e,t][i] = wts[t,e] * silu(gate_e[i] . xn_t) * (up_e[i] . xn_t)
//    for its rows and the tokens t routed to e, and stores a (fp32) to a small global buffer;
//  * one grid barrier (all CTAs co-resident: cooperative launch; the wait is bounded);
//  * down phase: every CTA owns a contiguous range of output rows h and reads w_d[e][h0:h1][:] (contiguous
//    rows) of every selected expert, y[t][h] = sum_e sum_i w_d[e][h][i] a[e,t][i], then writes
//    out = bf16(y + residual) for its rows. No atomics, no second launch.
//
// A producer warp streams both phases through a ring of 32 KB shared-memory stages with 1-D bulk copies
// (TMA engine, evict-first L2 policy). It does not wait for the grid barrier: the down-projection weights are
// prefetched while the consumers finish the gate/up phase, so HBM sees one continuous stream.
//
// Fused router (mode 1): the shared-expert slots (static ids, weight 1) need no routing, so every CTA
// starts streaming their gate/up rows at once. Meanwhile warp w of CTA b computes the logit of expert w * G + b
// (fp64 accumulation; spread over CTAs so no CTA starts its gate/up share late, and the router rows are
// prefetched into L2 at kernel entry), a first grid barrier publishes them, and every CTA then makes the
// (deterministic, identical) top-k selection itself and continues with the routed experts.
//
// Numerics: fp32 accumulation and intermediates; int8 weights are dequantised per element as
// float(q) * float(scale) (torch's dequantisation, bit-exact); the optional RMSNorm prologue reproduces
// mv_rmsnorm bit for bit.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "decode_common.cuh"

namespace mv {
namespace decode {

// 16 bytes of weights -> VEC fp32 values (int8: dequantised with scale sc)
template <bool INT8>
__device__ __forceinline__ void unpack(const uint4& wv, float sc, float* wf) {
  const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
  if (INT8) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      i8x4_to_f32(ww[q], wf[4 * q], wf[4 * q + 1], wf[4 * q + 2], wf[4 * q + 3]);
#pragma unroll
      for (int z = 0; z < 4; ++z) wf[4 * q + z] = dequant(wf[4 * q + z], sc);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      wf[2 * q] = bf16lo(ww[q]);
      wf[2 * q + 1] = bf16hi(ww[q]);
    }
  }
}

// Offset of element i inside a split row: the VEC-wide chunk c = i / VEC is stored as VEC/4 float4 pieces, piece q
// of every chunk in its own plane of n / (VEC/4) floats. A lane that owns chunk c reads its pieces from
// consecutive 16-byte slots of each plane, so a warp's reads never conflict on shared-memory banks.
template <int VEC>
__device__ __forceinline__ int split_off(int i, int n) {
  constexpr int NQ = VEC / 4;
  return ((i % VEC) / 4) * (n / NQ) + (i / VEC) * 4 + (i & 3);
}

template <bool INT8, int MT, int CW>
__global__ void __launch_bounds__(CW * 32 + 32, 1) moe_decode_kernel(const Params p) {
  using WT = W<INT8>;
  constexpr int kCons = CW * 32;     // consumer threads
  constexpr int kThr = kCons + 32;   // + producer warp
  constexpr int kDG = 4;             // warps per group in the packed down phase
  constexpr bool XF = MT <= 4;       // token activations kept as split fp32 in shared memory
  constexpr int VEC = WT::vec;
  constexpr int NQ = VEC / 4;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int NS = p.n_stages;
  const int H = p.H, I = p.I, M = p.M;
  const int G = gridDim.x;
  const int RG = p.RG, DR = p.DR;
  const int nhc = p.nh_cap;

  // ------------------------------------------------------------------ shared memory
  uint8_t* ring = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(NS) * kStageBytes);
  uint64_t* empty_bar = full_bar + NS;
  uint8_t* region = reinterpret_cast<uint8_t*>(empty_bar + NS);  // x in the gate/up phase, a in the down phase
  uint16_t* xn = reinterpret_cast<uint16_t*>(region);             // [M][H] bf16
  float* xf = reinterpret_cast<float*>(region + ((static_cast<size_t>(M) * H * 2 + 15) & ~size_t(15)));  // split
  float* y_s = reinterpret_cast<float*>(region + p.region_bytes);  // [MT][kNhMax]
  float* gsc = y_s + MT * kNhMax;                                  // [2][gsc_cap] gate / up row scales
  float* dsc = gsc + 2 * p.gsc_cap;                                // [u_max][nh_cap] down row scales
  int* e_id = reinterpret_cast<int*>(dsc + (INT8 ? p.u_max * nhc : 0));
  int* e_ntok = e_id + p.u_max;
  int* e_pbase = e_ntok + p.u_max;
  int* e_tok = e_pbase + p.u_max;                                  // [u_max][MT]
  float* e_w = reinterpret_cast<float*>(e_tok + p.u_max * MT);    // [u_max][MT]
  unsigned int* bitmap = reinterpret_cast<unsigned int*>(e_w + p.u_max * MT);  // [kMaxE1/32]
  int* misc = reinterpret_cast<int*>(bitmap + kMaxE1 / 32);        // [0]=U [1]=abort [3]=pairs
  int* pr_e = misc + 16;                                           // [kMaxM*kMaxNK]
  float* pr_w = reinterpret_cast<float*>(pr_e + kMaxM * kMaxNK);   // [kMaxM*kMaxNK]
  float* sel_r = pr_w + kMaxM * kMaxNK;                            // [M][E_alloc] (router mode)
  float* sel_sc = sel_r + M * p.E_alloc;                           // [M][E_alloc]
  float* sel_gs = sel_sc + M * p.E_alloc;                          // [M][32]
  double* red = reinterpret_cast<double*>((reinterpret_cast<uintptr_t>(sel_gs + M * 32) + 7) & ~uintptr_t(7));
  double* sel_k = red + CW * kMaxM;                                // [M][top_k]
  float* ypart = reinterpret_cast<float*>(sel_k + M * 32);         // [u_max][nh_cap][MT] (packed down phase)

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], CW);
    }
    fence_mbar_init();
    misc[0] = p.router ? p.n_static : 0;
    misc[1] = 0;
  }
  __syncthreads();
  pdl_launch_dependents();  // the next kernel in the stream may be scheduled (it waits for this one)
  pdl_wait();               // the tokens, pairs and workspace are the previous kernel's

  const int n_static = p.router ? p.n_static : 0;
  const long long S = static_cast<long long>(n_static) * I;
  const long long s_lo = S * blockIdx.x / G, s_hi = S * (blockIdx.x + 1) / G;
  const int hd0 = static_cast<int>(static_cast<long long>(H) * blockIdx.x / G);
  const int hd1 = static_cast<int>(static_cast<long long>(H) * (blockIdx.x + 1) / G);
  const int nh = hd1 - hd0;

  if (warp == CW) {
    // ================================================================ producer warp
    const uint64_t pol = policy_evict_first();
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    auto acquire = [&]() -> int {
      if (lane == 0)
        ok = ok && (*reinterpret_cast<volatile int*>(&misc[1]) == 0) &&
             mbar_wait(&empty_bar[stage], phase ^ 1u, p.ws, 0x100u | stage);
      ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
      if (!ok && lane == 0) misc[1] = 1;
      const int s = stage;
      if (++stage == NS) {
        stage = 0;
        phase ^= 1u;
      }
      return s;
    };
    const uint32_t row_b = static_cast<uint32_t>(H) * WT::esz;
    auto gu_stream = [&](GuWalk walk, bool is_static) {
      int u, i0, ni;
      long long r0w;
      while (ok && walk.next(u, i0, ni, r0w)) {
        const int e = is_static ? p.static_id + u : e_id[u];
        const uint8_t* gbase = p.w_gu + static_cast<long long>(e) * p.gu_se * WT::esz;
        for (int s0 = 0; s0 < ni && ok; s0 += RG) {
          const int nr = min(RG, ni - s0);
          const int s = acquire();
          if (!ok) break;
          uint8_t* dst = ring + static_cast<size_t>(s) * kStageBytes;
          if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], 2u * nr * row_b);
          __syncwarp();
          const long long rg = i0 + s0, ru = I + i0 + s0;
          if (p.gu_sr == H) {  // contiguous rows: one copy per half
            if (lane == 0) bulk_g2s(dst, gbase + rg * H * WT::esz, nr * row_b, &full_bar[s], pol);
            if (lane == 1) bulk_g2s(dst + RG * row_b, gbase + ru * H * WT::esz, nr * row_b, &full_bar[s], pol);
          } else if (lane < 2 * nr) {
            const int hf = lane / nr, r = lane % nr;
            bulk_g2s(dst + (hf * RG + r) * row_b, gbase + ((hf ? ru : rg) + r) * p.gu_sr * WT::esz, row_b,
                     &full_bar[s], pol);
          }
        }
      }
    };
    if (p.router) {
      // static (shared-expert) gate/up rows need no routing decision: stream them while the CTA routes
      gu_stream(GuWalk{s_lo, s_hi, I, 0}, true);
    } else {
      // pairs from the caller; this warp builds the expert table
      const int npairs = M * p.NK;
      for (int j = lane; j < npairs; j += 32) {
        const long long e = p.ids_i64 ? reinterpret_cast<const long long*>(p.ids)[j]
                                      : static_cast<long long>(reinterpret_cast<const int*>(p.ids)[j]);
        const bool valid = e >= 0 && e < p.E1;
        pr_e[j] = valid ? static_cast<int>(e) : -1;
        pr_w[j] = p.wts[j];
        if (!valid && e != -1) raise_error(p.ws, kErrBadExpert, static_cast<unsigned int>(j));  // -1: no pair
      }
      __syncwarp();
      if (npairs <= 32)
        table_warp<MT>(pr_e, pr_w, npairs, p.NK, p.E1, 0, 0, M, e_id, e_ntok, e_tok, e_w, e_pbase, misc, p.ws);
      else
        table_bitmap<MT>(pr_e, pr_w, npairs, p.NK, p.E1, 0, 0, M, e_id, e_ntok, e_tok, e_w, e_pbase, misc, bitmap,
                         p.ws, lane, 32, [] { __syncwarp(); });
    }
    named_bar(2, kThr);  // the expert table is published
    const int U = misc[0];
    const long long R = static_cast<long long>(U - n_static) * I;
    const long long T = S + R;
    const long long r_lo = T * blockIdx.x / G - s_lo, r_hi = T * (blockIdx.x + 1) / G - s_hi;
    gu_stream(GuWalk{r_lo, r_hi, I, n_static}, false);
    // down-projection rows of every selected expert
    const uint32_t drow_b = static_cast<uint32_t>(I) * WT::esz;
    if (p.a_all) {
      // packed: stage k holds entries [k*DP, (k+1)*DP) of the (expert, row) sequence, across experts
      const int DP = p.DP;
      const int nent = U * nh;
      for (int e0 = 0; e0 < nent && ok; e0 += DP) {
        const int e1 = min(nent, e0 + DP);
        const int s = acquire();
        if (!ok) break;
        uint8_t* dst = ring + static_cast<size_t>(s) * kStageBytes;
        if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], (e1 - e0) * drow_b);
        __syncwarp();
        if (p.d_sr == I) {
          if (lane == 0) {
            int e = e0;
            while (e < e1) {  // one copy per run of rows of the same expert
              const int u = e / nh, r = e % nh;
              const int n = min(e1 - e, nh - r);
              const uint8_t* src = p.w_d + (static_cast<long long>(e_id[u]) * p.d_se +
                                            static_cast<long long>(hd0 + r) * p.d_sr) * WT::esz;
              bulk_g2s(dst + static_cast<size_t>(e - e0) * drow_b, src, n * drow_b, &full_bar[s], pol);
              e += n;
            }
          }
        } else {
          for (int k = lane; k < e1 - e0; k += 32) {
            const int u = (e0 + k) / nh, r = (e0 + k) % nh;
            const uint8_t* src = p.w_d + (static_cast<long long>(e_id[u]) * p.d_se +
                                          static_cast<long long>(hd0 + r) * p.d_sr) * WT::esz;
            bulk_g2s(dst + static_cast<size_t>(k) * drow_b, src, drow_b, &full_bar[s], pol);
          }
        }
      }
    } else {
      for (int u = 0; u < U && ok; ++u) {
        const int e = e_id[u];
        const uint8_t* dbase =
            p.w_d + (static_cast<long long>(e) * p.d_se + static_cast<long long>(hd0) * p.d_sr) * WT::esz;
        for (int r0 = 0; r0 < nh && ok; r0 += DR) {
          const int nr = min(DR, nh - r0);
          const int s = acquire();
          if (!ok) break;
          uint8_t* dst = ring + static_cast<size_t>(s) * kStageBytes;
          if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], nr * drow_b);
          __syncwarp();
          if (p.d_sr == I) {
            if (lane == 0)
              bulk_g2s(dst, dbase + static_cast<long long>(r0) * I * WT::esz, nr * drow_b, &full_bar[s], pol);
          } else if (lane < nr) {
            bulk_g2s(dst + lane * drow_b, dbase + static_cast<long long>(r0 + lane) * p.d_sr * WT::esz, drow_b,
                     &full_bar[s], pol);
          }
        }
      }
    }
    return;
  }

  // ================================================================== consumers
  // Every consumer warp waits for every stage in ring order and arrives on its empty barrier once: a warp can
  // never wait on a phase more than one ahead of the barrier nor arrive twice in one phase, and no warp idles
  // (every stage's work is spread over all of them).
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  auto wait_full = [&](int s) -> bool {
    bool good = true;
    if (lane == 0) {
      good = (*reinterpret_cast<volatile int*>(&misc[1]) == 0) && mbar_wait(&full_bar[s], phase, p.ws, 0x200u | s);
      if (!good) misc[1] = 1;
    }
    return __shfl_sync(0xffffffffu, good, 0) != 0;
  };
  auto advance = [&]() {
    if (++stage == NS) {
      stage = 0;
      phase ^= 1u;
    }
  };
  auto release = [&](int s) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
  };

  // this thread's first output element's residual, read now rather than after the down phase
  const float res_pre = (p.residual != nullptr && tid < M * nh)
                            ? __uint_as_float(static_cast<uint32_t>(p.residual[(tid / nh) * H + hd0 + tid % nh]) << 16)
                            : 0.f;

  // ---- prologue: token rows (RMSNorm or copy) -> xn (bf16) and, for M <= 4, xf (split fp32)
  {
    // the router row of this warp's logit starts towards L2 before the weight stream fills the memory queues
    if (p.router && lane == 0 && warp * G + static_cast<int>(blockIdx.x) < p.E) {
      const int resz = p.rw_dtype == MV_F32 ? 4 : (p.rw_dtype == MV_BF16 ? 2 : 1);
      bulk_prefetch_l2(static_cast<const uint8_t*>(p.rw) +
                           static_cast<size_t>(warp * G + static_cast<int>(blockIdx.x)) * H * resz,
                       static_cast<uint32_t>(H * resz));
    }
    const int nv = H / 8;  // 16-byte vectors per row
    // the norm weight's first vector per thread is fetched with x, so both latencies overlap
    const uint4 g_pref = (p.norm_w != nullptr && tid < nv) ? reinterpret_cast<const uint4*>(p.norm_w)[tid]
                                                           : make_uint4(0, 0, 0, 0);
    for (int m = 0; m < M; ++m) {
      const uint4* xr = reinterpret_cast<const uint4*>(p.x + m * p.x_stride);
      uint4* xs = reinterpret_cast<uint4*>(xn + m * H);
      double ss = 0.0;
      for (int j = tid; j < nv; j += kCons) {
        const uint4 v = xr[j];
        xs[j] = v;
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const double a = bf16lo(vv[q]), b = bf16hi(vv[q]);
          ss += a * a + b * b;
        }
      }
      if (p.norm_w != nullptr) {
        ss = warp_sum_d(ss);
        if (lane == 0) red[warp * M + m] = ss;
      }
    }
    if (p.norm_w != nullptr) {
      named_bar(1, kCons);
      for (int m = 0; m < M; ++m) {
        double ss = 0.0;
        for (int w = 0; w < CW; ++w) ss += red[w * M + m];
        const float var = static_cast<float>(ss / static_cast<double>(H));
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
        uint4* xs = reinterpret_cast<uint4*>(xn + m * H);
        const uint4* wr = reinterpret_cast<const uint4*>(p.norm_w);
        for (int j = tid; j < nv; j += kCons) {
          const uint4 v = xs[j];
          const uint4 g = j == tid ? g_pref : wr[j];
          const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
          const uint32_t gg4[4] = {g.x, g.y, g.z, g.w};
          uint32_t o[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float y0 = round_bf16(__fmul_rn(bf16lo(vv[q]), r));
            const float y1 = round_bf16(__fmul_rn(bf16hi(vv[q]), r));
            o[q] = static_cast<uint32_t>(f2bf(__fmul_rn(bf16lo(gg4[q]), y0))) |
                   (static_cast<uint32_t>(f2bf(__fmul_rn(bf16hi(gg4[q]), y1))) << 16);
          }
          xs[j] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    named_bar(1, kCons);  // xn complete (written 16 bytes per thread) before it is re-read element-wise
    if (XF) {
      for (int j = tid; j < M * H; j += kCons) {
        const int m = j / H, h = j % H;
        xf[m * H + split_off<VEC>(h, H)] = __uint_as_float(static_cast<uint32_t>(xn[j]) << 16);
      }
    }
    if (INT8) {  // gate / up row scales of this CTA's static rows
      for (long long r = s_lo + tid; r < s_hi; r += kCons) {
        const int u = static_cast<int>(r / I), i = static_cast<int>(r % I);
        const long long b = static_cast<long long>(p.static_id + u) * p.sgu_se;
        gsc[r - s_lo] = ldscale(p.s_gu, b + i, p.s_bf16);
        gsc[p.gsc_cap + (r - s_lo)] = ldscale(p.s_gu, b + I + i, p.s_bf16);
      }
    }
    named_bar(1, kCons);
  }

  // ---- gate/up consumer for one walk. The consumer warps form NG = CW / RG groups; group g owns the ring slots
  // s with s % NG == g and alone waits on and releases their stages (each of its RG arrivals counts CW / RG, so
  // the empty barrier still completes after CW), warp gi of the group computing the complete gate row gi and up
  // row gi, i.e. the activation a[gi] of the expert's tokens (no partial sums). A slot always belongs to one
  // group, so a warp never waits on a phase more than one ahead of the barrier.
  const int gi = warp % RG, gq = warp / RG;
  const int NG = CW / RG;
  auto gu_consume = [&](GuWalk walk, bool is_static, int sc_base) {
    int u, i0, ni;
    long long r0w;
    const long long lo = walk.r;
    while (walk.next(u, i0, ni, r0w)) {
      const int ntok = is_static ? M : e_ntok[u];
      const int pb = is_static ? u * M : e_pbase[u];
      int tok[MT];
      float tw[MT];
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        tok[t] = t < ntok ? (is_static ? t : e_tok[u * MT + t]) : 0;
        tw[t] = t < ntok ? (is_static ? 1.0f : e_w[u * MT + t]) : 0.f;
      }
      for (int s0 = 0; s0 < ni; s0 += RG) {
        const int nr = min(RG, ni - s0);
        const int s = stage;
        const bool grp = (s % NG) == gq;  // the group owning this ring slot consumes the stage
        const bool mine = grp && gi < nr;
        if (grp) ok = wait_full(s) && ok;
        advance();
        if (ok && mine) {
          const uint8_t* st = ring + static_cast<size_t>(s) * kStageBytes;
          const uint8_t* grow = st + static_cast<size_t>(gi) * H * WT::esz;
          const uint8_t* urow = st + static_cast<size_t>(RG + gi) * H * WT::esz;
          float sg = 1.0f, su = 1.0f;
          if (INT8) {
            const int ri = sc_base + static_cast<int>(r0w - lo) + s0 + gi;
            sg = gsc[ri];
            su = gsc[p.gsc_cap + ri];
          }
          float ag[MT][2], au[MT][2];
#pragma unroll
          for (int t = 0; t < MT; ++t) ag[t][0] = ag[t][1] = au[t][0] = au[t][1] = 0.f;
          const int nvec = H / VEC;
#pragma unroll 2
          for (int ch = lane; ch < nvec; ch += 32) {
            const uint4 vg = *reinterpret_cast<const uint4*>(grow + ch * 16);
            const uint4 vu = *reinterpret_cast<const uint4*>(urow + ch * 16);
            const uint32_t wgw[4] = {vg.x, vg.y, vg.z, vg.w};
            const uint32_t wuw[4] = {vu.x, vu.y, vu.z, vu.w};
            if (XF) {
#pragma unroll
              for (int t = 0; t < MT; ++t) {
                if (t >= ntok) break;
                const float* xt = xf + tok[t] * H + ch * 4;
                if (INT8) {
#pragma unroll
                  for (int q = 0; q < 4; ++q) {  // word q = elements 4q..4q+3 = plane q
                    const float4 xv = *reinterpret_cast<const float4*>(xt + q * (H / NQ));
                    float g0, g1, g2, g3, u0, u1, u2, u3;
                    i8x4_to_f32(wgw[q], g0, g1, g2, g3);
                    i8x4_to_f32(wuw[q], u0, u1, u2, u3);
                    fmul2(g0, g1, g0, g1, sg);
                    fmul2(g2, g3, g2, g3, sg);
                    fmul2(u0, u1, u0, u1, su);
                    fmul2(u2, u3, u2, u3, su);
                    ffma2(ag[t][0], ag[t][1], g0, g1, xv.x, xv.y);
                    ffma2(ag[t][0], ag[t][1], g2, g3, xv.z, xv.w);
                    ffma2(au[t][0], au[t][1], u0, u1, xv.x, xv.y);
                    ffma2(au[t][0], au[t][1], u2, u3, xv.z, xv.w);
                  }
                } else {
#pragma unroll
                  for (int q = 0; q < 2; ++q) {  // words 2q, 2q+1 = elements 4q..4q+3 = plane q
                    const float4 xv = *reinterpret_cast<const float4*>(xt + q * (H / NQ));
                    ffma2(ag[t][0], ag[t][1], bf16lo(wgw[2 * q]), bf16hi(wgw[2 * q]), xv.x, xv.y);
                    ffma2(ag[t][0], ag[t][1], bf16lo(wgw[2 * q + 1]), bf16hi(wgw[2 * q + 1]), xv.z, xv.w);
                    ffma2(au[t][0], au[t][1], bf16lo(wuw[2 * q]), bf16hi(wuw[2 * q]), xv.x, xv.y);
                    ffma2(au[t][0], au[t][1], bf16lo(wuw[2 * q + 1]), bf16hi(wuw[2 * q + 1]), xv.z, xv.w);
                  }
                }
              }
            } else {
              float wg[VEC], wu[VEC];
              unpack<INT8>(vg, sg, wg);
              unpack<INT8>(vu, su, wu);
#pragma unroll
              for (int t = 0; t < MT; ++t) {
                if (t < ntok) {
                  const uint16_t* xr = xn + tok[t] * H + ch * VEC;
#pragma unroll
                  for (int q = 0; q < VEC / 8; ++q) {
                    const uint4 xv = *reinterpret_cast<const uint4*>(xr + 8 * q);
                    const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int z = 0; z < 4; ++z) {
                      const float x0 = bf16lo(xx[z]), x1 = bf16hi(xx[z]);
                      ag[t][0] = fmaf(wg[8 * q + 2 * z], x0, ag[t][0]);
                      ag[t][1] = fmaf(wg[8 * q + 2 * z + 1], x1, ag[t][1]);
                      au[t][0] = fmaf(wu[8 * q + 2 * z], x0, au[t][0]);
                      au[t][1] = fmaf(wu[8 * q + 2 * z + 1], x1, au[t][1]);
                    }
                  }
                }
              }
            }
          }
          float gsum[MT], usum[MT];
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            gsum[t] = t < ntok ? warp_sum(ag[t][0] + ag[t][1]) : 0.f;
            usum[t] = t < ntok ? warp_sum(au[t][0] + au[t][1]) : 0.f;
          }
          if (lane == 0) {
            const bool last = true;
            if (last) {
              const int i = i0 + s0 + gi;
#pragma unroll
              for (int t = 0; t < MT; ++t)
                if (t < ntok) {
                  const float g = gsum[t];
                  const float act = g / (1.0f + expf(-g));
                  p.a_g[static_cast<long long>(pb + t) * I + split_off<VEC>(i, I)] = act * usum[t] * tw[t];
                }
            }
          }
        }
        if (grp) {  // the group's RG arrivals count for all CW consumer warps
          __syncwarp();
          if (lane == 0) mbar_arrive_cnt(&empty_bar[s], static_cast<uint32_t>(CW / RG));
        }
      }
    }
  };

  // ---- router logits (mode 1, expert w * G + b on warp w of CTA b), the static (shared-expert) rows, then the
  // routing
  if (p.router) {
    const int e = warp * G + static_cast<int>(blockIdx.x);
    if (e < p.E) {
      double acc[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[m] = 0.0;
      const int resz = p.rw_dtype == MV_F32 ? 4 : (p.rw_dtype == MV_BF16 ? 2 : 1);
      const float rsc = p.rw_dtype == MV_I8 ? ldscale(p.rw_scale, e, p.rw_scale_bf16) : 1.0f;
      route::router_dot<MT>(static_cast<const uint8_t*>(p.rw) + static_cast<size_t>(e) * H * resz, p.rw_dtype, rsc,
                            xn, H, M, acc);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < M) {
          const double v = warp_sum_d(acc[m]);
          if (lane == 0) p.logits_ws[m * p.E + e] = static_cast<float>(v);
        }
      }
    }
    named_bar(1, kCons);
    unsigned long long tgt1 = 0;
    if (tid == 0) tgt1 = grid_arrive_gen(&p.ws->gen1, G);  // (fence + arrive by one thread after the CTA barrier)
    if (tid == 0) grid_wait_gen(&p.ws->gen1, tgt1, p.ws, 0x300u);
    named_bar(1, kCons);
    // every CTA makes the same selection from the published logits, all consumer threads in parallel
    const route::SelectCfg cfg{p.route_mode, p.E, p.top_k, p.n_group, p.topk_group, p.rscale, p.rbias};
    route::select_parallel(cfg, p.logits_ws, M, tid, kCons, [] { named_bar(1, kCons); }, sel_r, sel_sc, sel_k, sel_gs,
                           pr_e, pr_w);
    if (blockIdx.x == 0) {  // router outputs: ids / weights with the static slots appended, logits
      const int NKT = p.top_k + n_static;
      for (int j = tid; j < M * NKT; j += kCons) {
        const int m = j / NKT, k = j % NKT;
        const long long id =
            k < p.top_k ? pr_e[m * p.top_k + k] : static_cast<long long>(p.static_id + k - p.top_k);
        const float wv = k < p.top_k ? pr_w[m * p.top_k + k] : 1.0f;
        if (p.ids_out) {
          if (p.ids_out_i64)
            static_cast<long long*>(p.ids_out)[j] = id;
          else
            static_cast<int*>(p.ids_out)[j] = static_cast<int>(id);
        }
        if (p.wts_out) p.wts_out[j] = wv;
      }
      if (p.logits_out)
        for (int j = tid; j < M * p.E; j += kCons) p.logits_out[j] = ld_cg_f32(p.logits_ws + j);
    }
    const int npairs = M * p.top_k;
    if (npairs <= 32) {
      if (warp == 0)
        table_warp<MT>(pr_e, pr_w, npairs, p.top_k, p.E1, n_static, p.static_id, M, e_id, e_ntok, e_tok, e_w,
                       e_pbase, misc, p.ws);
    } else {
      table_bitmap<MT>(pr_e, pr_w, npairs, p.top_k, p.E1, n_static, p.static_id, M, e_id, e_ntok, e_tok, e_w, e_pbase,
                       misc, bitmap, p.ws, tid, kCons, [] { named_bar(1, kCons); });
    }
  }
  if (p.router) {
    // the table goes to every consumer and, without waiting, to the producer (which streams the static rows
    // first and then waits for it); the routing decision came first, the static rows the ring holds follow
    named_bar(1, kCons);
    named_bar_arrive(2, kThr);
    gu_consume(GuWalk{s_lo, s_hi, I, 0}, true, 0);
  } else {
    named_bar(2, kThr);  // the expert table is published by the producer warp
  }

  const int U = misc[0];
  const long long R = static_cast<long long>(U - n_static) * I;
  const long long T = S + R;
  const long long r_lo = T * blockIdx.x / G - s_lo, r_hi = T * (blockIdx.x + 1) / G - s_hi;
  if (INT8) {  // scales of this CTA's routed gate/up rows and of its down rows of every expert
    const int base = static_cast<int>(s_hi - s_lo);
    for (long long r = r_lo + tid; r < r_hi; r += kCons) {
      const int u = n_static + static_cast<int>(r / I), i = static_cast<int>(r % I);
      const long long b = static_cast<long long>(e_id[u]) * p.sgu_se;
      gsc[base + (r - r_lo)] = ldscale(p.s_gu, b + i, p.s_bf16);
      gsc[p.gsc_cap + base + (r - r_lo)] = ldscale(p.s_gu, b + I + i, p.s_bf16);
    }
    for (int j = tid; j < U * nh; j += kCons) {
      const int u = j / nh, r = j % nh;
      dsc[u * nhc + r] = ldscale(p.s_d, static_cast<long long>(e_id[u]) * p.sd_se + hd0 + r, p.s_bf16);
    }
    named_bar(1, kCons);
  }

  // ---- routed gate/up rows
  gu_consume(GuWalk{r_lo, r_hi, I, n_static}, false, static_cast<int>(s_hi - s_lo));

  // ---- grid barrier: every CTA's activations are in a_g
  named_bar(1, kCons);
  if (tid == 0) {
    const unsigned long long tgt2 = grid_arrive_gen(&p.ws->gen2, G);
    grid_wait_gen(&p.ws->gen2, tgt2, p.ws, 0x400u);
  }
  named_bar(1, kCons);

  // ---- down projection of this CTA's rows [hd0, hd1)
  for (int j = tid; j < MT * kNhMax; j += kCons) y_s[j] = 0.f;
  const int half = p.region_bytes / 2 / 4;  // floats in one half of the region
  float* abuf = reinterpret_cast<float*>(region);
  auto load_a = [&](int u, float* dst) {
    const float* src = p.a_g + static_cast<long long>(e_pbase[u]) * I;
    const int n16 = e_ntok[u] * I / 4;
    for (int j = tid; j < n16; j += kCons) cp_async16(dst + 4 * j, src + 4 * j);
    cp_async_commit();
  };
  auto fits_half = [&](int u) { return e_ntok[u] * I <= half; };
  if (p.a_all) {
    if (nh > 0) {
      const int n16 = misc[3] * I / 4;
      for (int j = tid; j < n16; j += kCons) cp_async16(abuf + 4 * j, p.a_g + 4 * j);
      cp_async_commit();
      cp_async_wait<0>();
    }
  } else if (U > 0 && nh > 0) {
    load_a(0, abuf);
  }
  named_bar(1, kCons);
  // one warp, one w_d row: y[tok][r] += w_d[e][hd0 + r] . a[u, tok] for the tokens of expert u; row r is
  // always computed by warp r % CW, so every y element has a single writer and a fixed summation order
  auto d_row = [&](const uint8_t* row, const float* a_u, int u, int r, float sc, float* part) {
    const int ntok = e_ntok[u];
    float acc[MT][2];
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t][0] = acc[t][1] = 0.f;
    const int nvec = I / VEC;
#pragma unroll 2
    for (int ch = lane; ch < nvec; ch += 32) {
      const uint4 wv = *reinterpret_cast<const uint4*>(row + ch * 16);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        if (t >= ntok) break;
        const float* at = a_u + t * I + ch * 4;
        if (INT8) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 av = *reinterpret_cast<const float4*>(at + q * (I / NQ));
            float w0, w1, w2, w3;
            i8x4_to_f32(ww[q], w0, w1, w2, w3);
            fmul2(w0, w1, w0, w1, sc);
            fmul2(w2, w3, w2, w3, sc);
            ffma2(acc[t][0], acc[t][1], w0, w1, av.x, av.y);
            ffma2(acc[t][0], acc[t][1], w2, w3, av.z, av.w);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const float4 av = *reinterpret_cast<const float4*>(at + q * (I / NQ));
            ffma2(acc[t][0], acc[t][1], bf16lo(ww[2 * q]), bf16hi(ww[2 * q]), av.x, av.y);
            ffma2(acc[t][0], acc[t][1], bf16lo(ww[2 * q + 1]), bf16hi(ww[2 * q + 1]), av.z, av.w);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      if (t < ntok) {
        const float v = warp_sum(acc[t][0] + acc[t][1]);
        if (lane == 0) {
          if (part != nullptr)
            part[t] = v;  // (expert u, row r) has one writer
          else
            y_s[e_tok[u * MT + t] * kNhMax + r] += v;  // row r has one owner warp
        }
      }
    }
  };
  // One token (MT == 1): the expert's activation chunks this lane needs stay in registers across the rows of
  // that expert (kAC floats: the lane's chunks ch = lane + 32 i), so a row costs only its weight reads from
  // shared memory. Same operations in the same order as d_row, so the results are identical.
  constexpr int kAC = 48;
  constexpr int kACIt = kAC / VEC;
  const bool a_regs = MT == 1 && I / VEC <= 32 * kACIt;
  float ac[kACIt][VEC];
  int ac_u = -1;
  auto d_row_m1 = [&](const uint8_t* row, int u, float sc, float* part) {
    const int nvec = I / VEC;
    if (u != ac_u) {
      const float* a_u = abuf + e_pbase[u] * I;
#pragma unroll
      for (int i = 0; i < kACIt; ++i) {
        const int ch = lane + 32 * i;
        if (ch < nvec) {
#pragma unroll
          for (int q = 0; q < NQ; ++q) {
            const float4 av = *reinterpret_cast<const float4*>(a_u + ch * 4 + q * (I / NQ));
            ac[i][4 * q] = av.x;
            ac[i][4 * q + 1] = av.y;
            ac[i][4 * q + 2] = av.z;
            ac[i][4 * q + 3] = av.w;
          }
        }
      }
      ac_u = u;
    }
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int i = 0; i < kACIt; ++i) {
      const int ch = lane + 32 * i;
      if (ch < nvec) {
        const uint4 wv = *reinterpret_cast<const uint4*>(row + ch * 16);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        if (INT8) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float w0, w1, w2, w3;
            i8x4_to_f32(ww[q], w0, w1, w2, w3);
            fmul2(w0, w1, w0, w1, sc);
            fmul2(w2, w3, w2, w3, sc);
            ffma2(acc0, acc1, w0, w1, ac[i][4 * q], ac[i][4 * q + 1]);
            ffma2(acc0, acc1, w2, w3, ac[i][4 * q + 2], ac[i][4 * q + 3]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            ffma2(acc0, acc1, bf16lo(ww[2 * q]), bf16hi(ww[2 * q]), ac[i][4 * q], ac[i][4 * q + 1]);
            ffma2(acc0, acc1, bf16lo(ww[2 * q + 1]), bf16hi(ww[2 * q + 1]), ac[i][4 * q + 2], ac[i][4 * q + 3]);
          }
        }
      }
    }
    const float v = warp_sum(acc0 + acc1);
    if (lane == 0) part[0] = v;
  };
  if (p.a_all) {
    // packed stages, each consumed by one group of kDG warps (the group owning its ring slot; the other warps
    // skip it, and the group's arrivals count for all CW): warp i of the group computes entries i, i + kDG, ...
    // of the stage's slice of the (expert, row) sequence into its own (expert, row) slot of ypart
    const int DP = p.DP;
    const int nent = U * nh;
    const int ngroups = CW / kDG;
    const int dg = warp / kDG, di = warp % kDG;
    for (int e0 = 0; e0 < nent; e0 += DP) {
      const int e1 = min(nent, e0 + DP);
      const int s = stage;
      if (s % ngroups == dg) {
        ok = wait_full(s) && ok;
        if (ok) {
          for (int k = di; k < e1 - e0; k += kDG) {
            const int u = (e0 + k) / nh, r = (e0 + k) % nh;
            const uint8_t* row = ring + static_cast<size_t>(s) * kStageBytes + static_cast<size_t>(k) * I * WT::esz;
            if (a_regs)
              d_row_m1(row, u, INT8 ? dsc[u * nhc + r] : 1.0f, ypart + (u * nhc + r) * MT);
            else
              d_row(row, abuf + e_pbase[u] * I, u, r, INT8 ? dsc[u * nhc + r] : 1.0f, ypart + (u * nhc + r) * MT);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_cnt(&empty_bar[s], static_cast<uint32_t>(CW / kDG));
      }
      advance();
    }
  } else {
    int cur_off = 0;  // float offset of the current expert's a rows in the region
    bool have_next = false;
    int next_off = 0;
    for (int u = 0; u < U && nh > 0; ++u) {
      if (have_next) {
        cur_off = next_off;
      } else if (u > 0) {  // not prefetched: the region is free (barrier at the end of the previous expert)
        load_a(u, abuf);
        cur_off = 0;
      }
      const bool pre = (u + 1 < U) && fits_half(u) && fits_half(u + 1);
      if (pre) {
        next_off = cur_off == 0 ? half : 0;
        load_a(u + 1, abuf + next_off);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      have_next = pre;
      named_bar(1, kCons);
      for (int r0 = 0; r0 < nh; r0 += DR) {
        const int nr = min(DR, nh - r0);
        const int s = stage;
        ok = wait_full(s) && ok;
        advance();
        if (ok) {
          for (int k = 0; k < nr; ++k) {
            if ((r0 + k) % CW != warp) continue;
            const uint8_t* row = ring + static_cast<size_t>(s) * kStageBytes + static_cast<size_t>(k) * I * WT::esz;
            d_row(row, abuf + cur_off, u, r0 + k, INT8 ? dsc[u * nhc + r0 + k] : 1.0f, nullptr);
          }
        }
        release(s);
      }
      named_bar(1, kCons);  // all reads of this expert's a rows finish before the region is reused
    }
  }
  cp_async_wait<0>();
  named_bar(1, kCons);
  for (int j = tid; j < M * nh; j += kCons) {
    const int t = j / nh, r = j % nh;
    float v = y_s[t * kNhMax + r];
    if (p.a_all) {  // packed: the (expert, row) results of token t, added in expert order
      v = 0.f;
      for (int u = 0; u < U; ++u)
        for (int i = 0; i < e_ntok[u]; ++i)
          if (e_tok[u * MT + i] == t) v += ypart[(u * nhc + r) * MT + i];
    }
    if (p.residual != nullptr)
      v += j == tid ? res_pre : __uint_as_float(static_cast<uint32_t>(p.residual[t * H + hd0 + r]) << 16);
    p.out[t * H + hd0 + r] = f2bf(v);
  }
  // (generation grid barriers: nothing to reset for the next call)
}

}  // namespace decode

using decode::Params;

// Token count from which the tensor-core kernel (moe_decode_tc.cu) takes over: below it the step is pure
// weight streaming with little arithmetic, and this CUDA-core kernel's row-granular split (no split-K
// partial sums to combine across CTAs) measured faster at M = 1; from 2 tokens on the tensor cores win
// (16-layer graph, per token: M = 2 45 vs 55 us, M = 4 28 vs 40 us; 3x at 16).
// MINGMOE_DECODE_PATH=classic / =tc forces either kernel.
constexpr int kTcMinM = 2;

#ifdef MV_TRACE
void* g_decode_trace = nullptr;  // phase-timing builds: [G][32] u64 stamps of the next launches
#endif

// Geometry, validation and the cooperative launch; shared by mv_moe_decode and mv_block_decode.
int decode_run(Params& p, const mv_moe_weights* w, void* workspace, size_t workspace_bytes, int nk_pairs,
               cudaStream_t st) {
  using namespace decode;
  const bool int8 = w->w_dtype == MV_I8;
  if (!int8 && w->w_dtype != MV_BF16) return fail(MV_ERR_UNSUPPORTED, "decode: w_dtype must be bf16 or i8");
  if (int8 && (w->s_gu == nullptr || w->s_d == nullptr || (w->s_dtype != MV_F32 && w->s_dtype != MV_BF16)))
    return fail(MV_ERR_INVALID, "decode: int8 weights need f32/bf16 scales s_gu and s_d");
  const int M = p.M, H = w->H, I = w->I, E1 = w->E1;
  if (M < 1 || M > kMaxM) return fail(MV_ERR_INVALID, "decode: M=%d outside [1, %d]", M, kMaxM);
  if (nk_pairs < 1 || nk_pairs > kMaxNK)
    return fail(MV_ERR_INVALID, "decode: %d experts per token outside [1, %d]", nk_pairs, kMaxNK);
  if (E1 < 1 || E1 > kMaxE1) return fail(MV_ERR_INVALID, "decode: E1=%d outside [1, %d]", E1, kMaxE1);
  const int esz = int8 ? 1 : 2, vec = int8 ? 16 : 8;
  if (H < 1 || H > 8192 || I < 1) return fail(MV_ERR_INVALID, "decode: bad H=%d / I=%d", H, I);
  if (I % vec != 0 || H % vec != 0)
    return fail(MV_ERR_INVALID, "decode: H=%d and I=%d must be multiples of %d", H, I, vec);
  const int G = num_sms();
  if ((H + G - 1) / G > kNhMax) return fail(MV_ERR_INVALID, "decode: H=%d too large for %d SMs", H, G);
  const int MT = M == 1 ? 1 : (M <= 4 ? 4 : 16);
  const int CW = MT == 16 ? 8 : 16;  // consumer warps (8 when 16 tokens need the registers)
  int RG = 1;                         // gate (and up) rows per stage: power of two <= 8
  while (RG * 2 <= 8 && 2 * (RG * 2) * H * esz <= kStageBytes) RG *= 2;
  if (2 * RG * H * esz > kStageBytes) return fail(MV_ERR_INVALID, "decode: H=%d too large", H);
  if (static_cast<long long>(I) * esz > kStageBytes) return fail(MV_ERR_UNSUPPORTED, "decode: I=%d too large", I);
  int DR = static_cast<int>(kStageBytes / (static_cast<long long>(I) * esz));  // w_d rows per stage
  if (DR > kNhMax) DR = kNhMax;
  if (!aligned16(w->w_gu) || !aligned16(w->w_d) || !aligned16(p.x) || ((w->gu_se * esz) % 16) ||
      ((w->gu_sr * esz) % 16) || ((w->d_se * esz) % 16) || ((w->d_sr * esz) % 16) || ((p.x_stride * 2) % 16))
    return fail(MV_ERR_ALIGN, "decode: weights, x and their strides must be 16-byte aligned");
  if (p.norm_w != nullptr && !aligned16(p.norm_w)) return fail(MV_ERR_ALIGN, "decode: norm_w must be 16-byte aligned");
  if (p.router) {
    const int resz = p.rw_dtype == MV_F32 ? 4 : (p.rw_dtype == MV_BF16 ? 2 : 1);
    if (!aligned16(p.rw) || (H * resz) % 16) return fail(MV_ERR_ALIGN, "decode: router rows must be 16-byte aligned");
  }
  const size_t need = mv_moe_decode_workspace_bytes(M, nk_pairs, I, p.router ? p.E : 0);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(MV_ERR_WORKSPACE, "decode: workspace of %zu bytes needed", need);

  p.w_gu = static_cast<const uint8_t*>(w->w_gu);
  p.w_d = static_cast<const uint8_t*>(w->w_d);
  p.s_gu = w->s_gu;
  p.s_d = w->s_d;
  p.gu_se = w->gu_se;
  p.gu_sr = w->gu_sr;
  p.d_se = w->d_se;
  p.d_sr = w->d_sr;
  p.sgu_se = w->sgu_se;
  p.sd_se = w->sd_se;
  p.E1 = E1;
  p.H = H;
  p.I = I;
  p.s_bf16 = w->s_dtype == MV_BF16;
  p.ws = static_cast<WsHeader*>(workspace);
#ifdef MV_TRACE
  p.trace = static_cast<unsigned long long*>(g_decode_trace);
#endif
  {  // several tokens with the router fused: the one-token kernel once per token (the block is per-token work). In
    // the 16-layer graph: bf16 M = 2 2 x 36.6 vs 80.9 us per block for the tensor-core kernel (which wins from
    // M = 3); int8 every M, since the general kernel dequantises every weight once per token on the CUDA cores
    // (M = 16: 849 us per block, against 16 x 36.6 here)
    const char* path = getenv("MINGMOE_DECODE_PATH");
    if (M >= 2 && (M == 2 || int8) && p.router && (path == nullptr || path[0] == 'm')) {
      decode::Params q = p;
      q.M = 1;
      const size_t lg1 = (static_cast<size_t>(p.E) * 4 + 255) & ~size_t(255);
      q.logits_ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWsHeaderBytes);
      q.a_g = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWsHeaderBytes + lg1);
      const int id_bytes = p.ids_out_i64 ? 8 : 4;
      int rc = kDecodeM1Unsuitable;
      for (int t = 0; t < M; ++t) {
        q.x = p.x + t * p.x_stride;
        q.residual = p.residual != nullptr ? p.residual + static_cast<long long>(t) * H : nullptr;
        q.out = p.out + static_cast<long long>(t) * H;
        q.ids_out = p.ids_out != nullptr ? static_cast<uint8_t*>(p.ids_out) + static_cast<long long>(t) * nk_pairs * id_bytes
                                         : nullptr;
        q.wts_out = p.wts_out != nullptr ? p.wts_out + static_cast<long long>(t) * nk_pairs : nullptr;
        q.logits_out = p.logits_out != nullptr ? p.logits_out + static_cast<long long>(t) * p.E : nullptr;
        rc = decode_m1_run(q, int8, st);
        if (rc != MV_OK) break;
      }
      if (rc != kDecodeM1Unsuitable) return rc;
    }
  }
  if (!int8) {  // the tensor-core kernel when the shapes and the workspace suit it (M >= kTcMinM)
    const char* path = getenv("MINGMOE_DECODE_PATH");
    const bool force_tc = path != nullptr && path[0] == 't';
    if ((path == nullptr || path[0] != 'c') && (M >= kTcMinM || force_tc)) {
      const int rc = decode_tc_run(p, workspace, workspace_bytes, nk_pairs, st);
      if (rc != kDecodeTcUnsuitable) return rc;
    }
  }
  const size_t lg = (static_cast<size_t>(M) * (p.router ? p.E : 0) * 4 + 255) & ~size_t(255);
  p.logits_ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWsHeaderBytes);
  p.a_g = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWsHeaderBytes + lg);
  {  // one token with the router fused: the dedicated kernel (moe_decode_m1.cu; MINGMOE_DECODE_PATH=classic keeps
    // this kernel)
    const char* path = getenv("MINGMOE_DECODE_PATH");
    const bool want = path == nullptr || path[0] == 'm';
    if (M == 1 && p.router && want) {
      const int rc = decode_m1_run(p, int8, st);
      if (rc != kDecodeM1Unsuitable) return rc;
    }
  }
  p.RG = RG;
  p.DR = DR;
  p.DP = DR;
  p.u_max = p.router ? (p.n_static + (M * p.top_k < E1 ? M * p.top_k : E1)) : (M * p.NK < E1 ? M * p.NK : E1);
  p.E_alloc = p.router ? p.E : 0;
  // region: x (bf16 rows, plus split fp32 rows when M <= 4) in the gate/up phase; the activations of the
  // selected experts in the down phase -- all at once if that leaves a 4-stage ring, else two halves
  const bool XF = MT <= 4;
  const size_t xn_bytes = ((static_cast<size_t>(M) * H * 2 + 15) & ~size_t(15)) + (XF ? static_cast<size_t>(M) * H * 4 : 0);
  size_t a_bytes = static_cast<size_t>(2 * (MT < 8 ? MT : 8)) * I * 4;
  if (static_cast<size_t>(MT) * I * 4 > a_bytes) a_bytes = static_cast<size_t>(MT) * I * 4;
  const size_t all_bytes = static_cast<size_t>(M) * nk_pairs * I * 4;
  p.nh_cap = (H + G - 1) / G;
  p.gsc_cap = int8 ? static_cast<int>((static_cast<long long>(p.u_max) * I + G - 1) / G + 4) : 0;
  const size_t small = static_cast<size_t>(MT) * kNhMax * 4 +
                       2 * static_cast<size_t>(p.gsc_cap) * 4 +
                       (int8 ? static_cast<size_t>(p.u_max) * p.nh_cap * 4 : 0) +
                       static_cast<size_t>(p.u_max) * (3 * 4 + MT * 8) + (kMaxE1 / 32) * 4 + 16 * 4 +
                       kMaxM * kMaxNK * 8 + static_cast<size_t>(M) * p.E_alloc * 8 + static_cast<size_t>(M) * 32 * 4 +
                       8 + static_cast<size_t>(CW) * kMaxM * 8 + static_cast<size_t>(M) * 32 * 8 + 64;
  size_t region = xn_bytes > a_bytes ? xn_bytes : a_bytes;
  const size_t ypart_bytes = static_cast<size_t>(p.u_max) * p.nh_cap * MT * 4;  // packed down-phase results
  p.a_all = 0;
  {
    size_t r_all = xn_bytes > all_bytes ? xn_bytes : all_bytes;
    r_all = (r_all + 31) & ~size_t(31);
    if (4 * (kStageBytes + 16) + r_all + small + ypart_bytes <= 227 * 1024) {
      region = r_all;
      p.a_all = 1;
    }
  }
  region = (region + 31) & ~size_t(31);
  p.region_bytes = static_cast<int>(region);
  const size_t fixed = ((region + small + (p.a_all ? ypart_bytes : 0)) + 15) & ~size_t(15);
  const size_t cap = 227 * 1024;
  // ring depth: 4 x 32 KB stages keep enough bytes in flight per SM (more stages measured slower); an
  // environment override (MINGMOE_DECODE_STAGES=2..8) exists for tuning
  static const int ns_env = [] {
    const char* v = getenv("MINGMOE_DECODE_STAGES");
    const int n = v ? atoi(v) : 0;
    return (n >= 2 && n <= 8) ? n : 4;
  }();
  int NS = ns_env;
  while (NS > 2 && NS * (kStageBytes + 16) + fixed > cap) --NS;
  if (NS * (kStageBytes + 16) + fixed > cap) return fail(MV_ERR_INVALID, "decode: shared memory budget exceeded");
  p.n_stages = NS;
  const size_t smem = NS * (kStageBytes + 16) + fixed;

  void (*kern)(Params);
  if (int8)
    kern = MT == 1 ? moe_decode_kernel<true, 1, 16>
                   : (MT == 4 ? moe_decode_kernel<true, 4, 16> : moe_decode_kernel<true, 16, 8>);
  else
    kern = MT == 1 ? moe_decode_kernel<false, 1, 16>
                   : (MT == 4 ? moe_decode_kernel<false, 4, 16> : moe_decode_kernel<false, 16, 8>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(moe_decode)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(CW * 32 + 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  return cuda_status(e, "moe_decode launch");
}

}  // namespace mv

using namespace mv;

extern "C" size_t mv_moe_decode_workspace_bytes(int M, int NK, int I, int E) {
  M = M > 0 ? M : 1;
  NK = NK > 0 ? NK : 1;
  I = I > 0 ? I : 1;
  E = E > 0 ? E : 0;
  const size_t lg = (static_cast<size_t>(M) * E * 4 + 255) & ~size_t(255);
  return kWsHeaderBytes + lg + static_cast<size_t>(M) * NK * I * sizeof(float);
}

extern "C" size_t mv_moe_decode_workspace_bytes_tc(int M, int NK, int H, int I, int E1) {
  const size_t classic = mv_moe_decode_workspace_bytes(M, NK, I, 0);
  const size_t tc = decode_tc_workspace_bytes(M, NK, H, I, E1, 0, 0);
  return tc > classic ? tc : classic;
}

extern "C" size_t mv_block_decode_workspace_bytes_tc(const mv_block* b, int M) {
  if (b == nullptr) return 0;
  const int nk = b->top_k + b->n_shared;
  const size_t classic = mv_block_decode_workspace_bytes(M, nk, b->experts.I, b->E);
  const size_t tc = decode_tc_workspace_bytes(M, nk, b->experts.H, b->experts.I, b->experts.E1, b->E, b->n_shared);
  return tc > classic ? tc : classic;
}

extern "C" int mv_moe_decode(const mv_moe_weights* w, const void* x, long long x_stride, const void* norm_w,
                             float eps, const void* ids, int ids_dtype, const float* wts, int M, int NK,
                             const void* residual, void* out, void* workspace, size_t workspace_bytes,
                             void* stream) {
  if (w == nullptr || x == nullptr || ids == nullptr || wts == nullptr || out == nullptr)
    return fail(MV_ERR_INVALID, "mv_moe_decode: null pointer argument");
  if (ids_dtype != MV_I32 && ids_dtype != MV_I64) return fail(MV_ERR_INVALID, "mv_moe_decode: ids must be i32 or i64");
  Params p{};
  p.x = static_cast<const uint16_t*>(x);
  p.x_stride = x_stride;
  p.norm_w = static_cast<const uint16_t*>(norm_w);
  p.eps = eps;
  p.M = M;
  p.ids = ids;
  p.ids_i64 = ids_dtype == MV_I64;
  p.wts = wts;
  p.NK = NK;
  p.router = 0;
  p.residual = static_cast<const uint16_t*>(residual);
  p.out = static_cast<uint16_t*>(out);
  return decode_run(p, w, workspace, workspace_bytes, NK, static_cast<cudaStream_t>(stream));
}

extern "C" size_t mv_block_decode_workspace_bytes(int M, int n_experts_per_token, int I, int E) {
  return mv_moe_decode_workspace_bytes(M, n_experts_per_token, I, E);
}

extern "C" int mv_block_decode(const mv_block* b, const void* x, int M, void* out, float* logits_out, void* ids_out,
                               int ids_dtype, float* wts_out, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (b == nullptr || x == nullptr || out == nullptr) return fail(MV_ERR_INVALID, "mv_block_decode: null pointer");
  if (b->router_w == nullptr) return fail(MV_ERR_INVALID, "mv_block_decode: router weight missing");
  if (b->route_mode != MV_ROUTE_SOFTMAX && b->route_mode != MV_ROUTE_SIGMOID_GROUP)
    return fail(MV_ERR_INVALID, "mv_block_decode: bad route_mode");
  if (b->E < 1 || b->E > route::kMaxE || b->top_k < 1 || b->top_k > 32 || b->top_k > b->E)
    return fail(MV_ERR_INVALID, "mv_block_decode: bad E=%d / top_k=%d", b->E, b->top_k);
  if (b->n_shared < 0 || b->top_k + b->n_shared > decode::kMaxNK || b->shared_id < 0 ||
      b->shared_id + b->n_shared > b->experts.E1)
    return fail(MV_ERR_INVALID, "mv_block_decode: bad shared slots %d..%d", b->shared_id,
                b->shared_id + b->n_shared);
  if (b->router_dtype != MV_F32 && b->router_dtype != MV_BF16 && b->router_dtype != MV_I8)
    return fail(MV_ERR_UNSUPPORTED, "mv_block_decode: router weight must be f32, bf16 or i8");
  if (b->router_dtype == MV_I8 && b->router_scale == nullptr)
    return fail(MV_ERR_INVALID, "mv_block_decode: int8 router needs router_scale");
  if (b->route_mode == MV_ROUTE_SIGMOID_GROUP &&
      (b->n_group < 1 || b->n_group > 32 || b->E % b->n_group || b->topk_group < 1 || b->topk_group > b->n_group ||
       (b->n_group > 1 && b->E / b->n_group < 2) || b->top_k > b->topk_group * (b->E / b->n_group)))
    return fail(MV_ERR_INVALID, "mv_block_decode: bad group routing config");
  if (b->E > b->experts.E1) return fail(MV_ERR_INVALID, "mv_block_decode: E exceeds the stacked slots");
  if (ids_out != nullptr && ids_dtype != MV_I32 && ids_dtype != MV_I64)
    return fail(MV_ERR_INVALID, "mv_block_decode: ids must be i32 or i64");
  Params p{};
  p.x = static_cast<const uint16_t*>(x);
  p.x_stride = b->experts.H;
  p.norm_w = static_cast<const uint16_t*>(b->norm_w);
  p.eps = b->eps;
  p.M = M;
  p.router = 1;
  p.route_mode = b->route_mode;
  p.rw = b->router_w;
  p.rw_dtype = b->router_dtype;
  p.rw_scale = b->router_scale;
  p.rw_scale_bf16 = b->router_scale_dtype == MV_BF16;
  p.rbias = b->router_bias;
  p.E = b->E;
  p.top_k = b->top_k;
  p.n_group = b->n_group;
  p.topk_group = b->topk_group;
  p.rscale = b->route_scale;
  p.n_static = b->n_shared;
  p.static_id = b->shared_id;
  p.logits_out = logits_out;
  p.ids_out = ids_out;
  p.ids_out_i64 = ids_dtype == MV_I64;
  p.wts_out = wts_out;
  p.residual = b->residual_from_x ? static_cast<const uint16_t*>(x) : nullptr;
  p.out = static_cast<uint16_t*>(out);
  if (b->next != nullptr && b->next->router_w != nullptr && aligned16(b->next->router_w)) {
    const mv_block* n = b->next;
    const int resz = n->router_dtype == MV_F32 ? 4 : (n->router_dtype == MV_BF16 ? 2 : 1);
    const long long bytes = static_cast<long long>(n->E) * n->experts.H * resz;
    if (bytes > 0 && bytes % 16 == 0) {
      p.nx_rw = static_cast<const uint8_t*>(n->router_w);
      p.nx_rw_bytes = bytes;
      if (n->norm_w != nullptr && aligned16(n->norm_w) && n->experts.H == b->experts.H)
        p.nx_norm = static_cast<const uint16_t*>(n->norm_w);
    }
  }
  return decode_run(p, &b->experts, workspace, workspace_bytes, b->top_k + b->n_shared,
                    static_cast<cudaStream_t>(stream));
}

#ifdef MV_TRACE
extern "C" MV_API void mv_trace_set_decode(void* buf) { mv::g_decode_trace = buf; }
#endif
