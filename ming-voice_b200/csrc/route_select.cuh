// Per-token expert selection (one warp per token), shared by the router kernels and the fused decode kernel.
//
// Follows ming-voice fused_ops.py:53-93 for MV_ROUTE_SIGMOID_GROUP (sigmoid + bias, group top-2 sums, keep
// topk_group groups, top-k by the biased score, weights = sigmoid scores renormalised with +1e-20, x scale)
// and the BASELINE softmax router for MV_ROUTE_SOFTMAX (top-k of logits + bias, weights = softmax renormalised
// over the top-k). Ties go to the lower expert id (tl.argmax returns the first maximum). Sigmoid scores and
// softmax weights are evaluated in fp64 and rounded to fp32.
#pragma once

#include <math.h>

#include "common.cuh"

namespace mv {
namespace route {

constexpr int kMaxE = 512;

struct SelectCfg {
  int mode, E, top_k, n_group, topk_group;
  double scale;
  const float* bias;
};

// Warp argmax over values v[j] of experts lane + 32 j (j < nper); ties to the lower index.
template <int NPER>
__device__ __forceinline__ int warp_argmax(const float (&v)[NPER], int E, float& best_v) {
  const int lane = threadIdx.x & 31;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll
  for (int j = 0; j < NPER; ++j) {
    const int e = lane + 32 * j;
    if (e < E && (v[j] > bv || (v[j] == bv && e < bi))) {
      bv = v[j];
      bi = e;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  best_v = bv;
  return bi;
}

// Selection for token m by one warp. `lg` = the token's fp32 logits [E] (global or shared memory).
// Selection for one token by one warp. `lg` = the token's fp32 logits [E] (global or shared memory), `scr` =
// E floats of shared scratch owned by this warp (may alias lg). Lane 0 writes sel_out[k] / w_out[k], k < top_k.
// Order-preserving 32-bit key of a float (larger float -> larger unsigned key; -inf is the smallest finite key).
__device__ __forceinline__ uint32_t sort_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Arg-max over the warp's E values (lane l holds entries l + 32 j): the largest value, ties to the lower index,
// with two warp reductions (redux.sync) instead of a shuffle tree.
template <int NPER>
__device__ __forceinline__ int warp_argmax_redux(const float (&v)[NPER], int E, float& best_v) {
  const int lane = threadIdx.x & 31;
  uint32_t bk = 0u;
  uint32_t bi = 0xffffffffu;
#pragma unroll
  for (int j = 0; j < NPER; ++j) {
    const int e = lane + 32 * j;
    if (e < E) {
      const uint32_t k = sort_key(v[j]);
      if (k > bk) {  // entries are visited in increasing index: '>' keeps the lower index on ties
        bk = k;
        bi = static_cast<uint32_t>(e);
      }
    }
  }
  const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
  const uint32_t idx = __reduce_min_sync(0xffffffffu, bk == mk ? bi : 0xffffffffu);
  best_v = key_value(mk);
  return static_cast<int>(idx);
}

// Selection for one token by one warp. `lg` = the token's fp32 logits [E] (global or shared memory), `scr` =
// E floats of shared scratch owned by this warp (may alias lg). Lane 0 writes sel_out[k] / w_out[k], k < top_k.
// NPER = ceil(E / 32) values per lane. The configuration is taken by value (a reference would keep it in local
// memory, and every read of it in the unrolled loops would be a memory access).
template <int NPER>
static __device__ __noinline__ void select_core_t(const SelectCfg p, const float* lg, float* scr, int* sel_out,
                                                  float* w_out) {
  const int lane = threadIdx.x & 31;
  const int E = p.E, K = p.top_k;
  float r[NPER];
  float sc[NPER];
#pragma unroll
  for (int j = 0; j < NPER; ++j) {
    const int e = lane + 32 * j;
    r[j] = -INFINITY;
    sc[j] = 0.f;
    if (e < E) {
      const float l = lg[e];
      if (p.mode == MV_ROUTE_SIGMOID_GROUP) {
        sc[j] = static_cast<float>(1.0 / (1.0 + exp(-static_cast<double>(l))));
        r[j] = p.bias ? __fadd_rn(sc[j], p.bias[e]) : sc[j];
      } else {
        r[j] = p.bias ? __fadd_rn(l, p.bias[e]) : l;
      }
      scr[e] = r[j];
    }
  }
  __syncwarp();
  if (p.mode == MV_ROUTE_SIGMOID_GROUP && p.n_group > 1) {
    // group score = sum of the group's two largest r (first maximum removed by index)
    const int G = p.n_group, GS = E / G;
    float gs = -INFINITY;
    if (lane < G) {
      float m1 = -INFINITY;
      int a1 = -1;
      for (int i = 0; i < GS; ++i) {
        const float v = scr[lane * GS + i];
        if (a1 < 0 || v > m1) {
          m1 = v;
          a1 = i;
        }
      }
      float m2 = -INFINITY;
      for (int i = 0; i < GS; ++i)
        if (i != a1) m2 = fmaxf(m2, scr[lane * GS + i]);
      gs = __fadd_rn(m1, m2);
    }
    // keep the topk_group best groups (first maximum wins ties)
    unsigned int keep = 0u;
    for (int t = 0; t < p.topk_group; ++t) {
      const bool live = lane < G && !((keep >> lane) & 1u);
      const uint32_t k = live ? sort_key(gs) : 0u;
      const uint32_t mk = __reduce_max_sync(0xffffffffu, k);
      const uint32_t bi = __reduce_min_sync(0xffffffffu, (live && k == mk) ? static_cast<uint32_t>(lane) : 0xffffffffu);
      if (bi < static_cast<uint32_t>(G)) keep |= 1u << bi;
    }
#pragma unroll
    for (int j = 0; j < NPER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !((keep >> (e / GS)) & 1u)) r[j] = -INFINITY;
    }
  }
  // top-k, largest first, ties to the lower id. The k-th pick lives in lane k's registers (no local arrays).
  int my_sel = 0;
  float my_r = -INFINITY, my_s = 0.f;
  for (int k = 0; k < K; ++k) {
    float bv;
    const int bi = warp_argmax_redux<NPER>(r, E, bv);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NPER; ++j)
      if (lane + 32 * j == bi) {
        s = sc[j];
        r[j] = -INFINITY;
      }
    const float sb = __shfl_sync(0xffffffffu, s, bi & 31);  // the chosen expert's sigmoid score
    if (lane == k) {
      my_sel = bi;
      my_r = bv;
      my_s = sb;
    }
  }
  double wk = 0.0;
  if (p.mode == MV_ROUTE_SIGMOID_GROUP) {
    const double tot = warp_sum_d(lane < K ? static_cast<double>(my_s) : 0.0);
    wk = static_cast<double>(my_s) / (tot + 1e-20) * p.scale;
  } else {
    const double mx = static_cast<double>(__shfl_sync(0xffffffffu, my_r, 0));  // the top-1 logit is the max
    const double ex = lane < K ? exp(static_cast<double>(my_r) - mx) : 0.0;
    const double tot = warp_sum_d(ex);
    wk = ex / tot;
  }
  if (lane < K) {
    sel_out[lane] = my_sel;
    w_out[lane] = static_cast<float>(wk);
  }
}

__device__ __forceinline__ void select_core(const SelectCfg& p, const float* lg, float* scr, int* sel_out,
                                            float* w_out) {
  if (p.E <= 64)
    select_core_t<2>(p, lg, scr, sel_out, w_out);
  else if (p.E <= 128)
    select_core_t<4>(p, lg, scr, sel_out, w_out);
  else if (p.E <= 256)
    select_core_t<8>(p, lg, scr, sel_out, w_out);
  else
    select_core_t<kMaxE / 32>(p, lg, scr, sel_out, w_out);
}

}  // namespace route
}  // namespace mv

namespace mv {
namespace route {

template <int MAXM, int DT>
__device__ __forceinline__ void router_dot_t(const void* w_row, float scale, const uint16_t* xs, int H, int M,
                                             double (&acc)[MAXM]) {
  const int lane = threadIdx.x & 31;
  constexpr int esz = DT == MV_F32 ? 4 : (DT == MV_BF16 ? 2 : 1);
  constexpr int per = 16 / esz;  // elements per 16-byte chunk
  const int nch = H / per;
  const uint8_t* base = static_cast<const uint8_t*>(w_row);
  constexpr int B = 8;
  for (int c0 = 0; c0 < nch; c0 += 32 * B) {
    uint4 buf[B];
#pragma unroll
    for (int j = 0; j < B; ++j) {
      const int c = c0 + lane + 32 * j;
      if (c < nch) buf[j] = ld_nc_v4(base + static_cast<size_t>(c) * 16);
    }
#pragma unroll
    for (int j = 0; j < B; ++j) {
      const int c = c0 + lane + 32 * j;
      if (c >= nch) continue;
      const uint32_t ww[4] = {buf[j].x, buf[j].y, buf[j].z, buf[j].w};
      float wf[per];
      if (DT == MV_F32) {
#pragma unroll
        for (int q = 0; q < 4; ++q) wf[q] = __uint_as_float(ww[q]);
      } else if (DT == MV_BF16) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          wf[2 * q] = bf16lo(ww[q]);
          wf[2 * q + 1] = bf16hi(ww[q]);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f0, f1, f2, f3;
          i8x4_to_f32(ww[q], f0, f1, f2, f3);
          wf[(4 * q) % per] = dequant(f0, scale);
          wf[(4 * q + 1) % per] = dequant(f1, scale);
          wf[(4 * q + 2) % per] = dequant(f2, scale);
          wf[(4 * q + 3) % per] = dequant(f3, scale);
        }
      }
      const int h0 = c * per;
#pragma unroll
      for (int m = 0; m < MAXM; ++m) {
        if (m < M) {
          const uint16_t* xr = xs + m * H + h0;
#pragma unroll
          for (int v = 0; v < per; v += 2) {
            const uint32_t xx = *reinterpret_cast<const uint32_t*>(xr + v);
            acc[m] += static_cast<double>(wf[v]) * static_cast<double>(bf16lo(xx));
            acc[m] += static_cast<double>(wf[v + 1]) * static_cast<double>(bf16hi(xx));
          }
        }
      }
    }
  }
}

// One warp: logits[m] = sum_h xs[m][h] * w_row[h] for m < M (fp64 accumulation of exact products, rounded to
// fp32 by the caller). The row is read 16 bytes per lane, 8 loads in flight per lane before any use.
// xs: bf16 rows in shared memory (row stride H). H % (16 / esz) == 0, w_row 16-byte aligned (host-checked).
template <int MAXM>
__device__ __forceinline__ void router_dot(const void* w_row, int dtype, float scale, const uint16_t* xs, int H,
                                           int M, double (&acc)[MAXM]) {
  if (dtype == MV_F32)
    router_dot_t<MAXM, MV_F32>(w_row, scale, xs, H, M, acc);
  else if (dtype == MV_BF16)
    router_dot_t<MAXM, MV_BF16>(w_row, scale, xs, H, M, acc);
  else
    router_dot_t<MAXM, MV_I8>(w_row, scale, xs, H, M, acc);
}

}  // namespace route
}  // namespace mv

namespace mv {
namespace route {

// Selection for M tokens by NT cooperating threads (thread index t, `sync` = a barrier over those threads),
// in parallel: every expert's rank is the number of experts ahead of it (larger score, or equal score and
// lower id), so the k-th largest is the expert of rank k -- the same order, ties included, as the reference's
// argmax loop, without any serial rounds. Logits come from global memory (written by other CTAs: read through
// L2). r_s, sc_s: M*E floats of scratch; k_s: M*K doubles; gs: M*n_group floats. Outputs sel_e/sel_w [M][K].
template <typename Sync>
__device__ void select_parallel(const SelectCfg& p, const float* logits, int M, int t, int NT, Sync sync, float* r_s,
                                float* sc_s, double* k_s, float* gs, int* sel_e, float* sel_w) {
  const int E = p.E, K = p.top_k;
  for (int i = t; i < M * E; i += NT) {
    const int e = i % E;
    const float l = ld_cg_f32(logits + i);
    float sc = 0.f, r;
    if (p.mode == MV_ROUTE_SIGMOID_GROUP) {
      sc = static_cast<float>(1.0 / (1.0 + exp(-static_cast<double>(l))));
      r = p.bias ? __fadd_rn(sc, p.bias[e]) : sc;
    } else {
      r = p.bias ? __fadd_rn(l, p.bias[e]) : l;
    }
    r_s[i] = r;
    sc_s[i] = sc;
  }
  sync();
  if (p.mode == MV_ROUTE_SIGMOID_GROUP && p.n_group > 1) {
    const int G = p.n_group, GS = E / G;
    for (int i = t; i < M * G; i += NT) {  // group score: its two largest r (first maximum removed by index)
      const float* rg = r_s + (i / G) * E + (i % G) * GS;
      float m1 = -INFINITY;
      int a1 = -1;
      for (int j = 0; j < GS; ++j)
        if (a1 < 0 || rg[j] > m1) {
          m1 = rg[j];
          a1 = j;
        }
      float m2 = -INFINITY;
      for (int j = 0; j < GS; ++j)
        if (j != a1) m2 = fmaxf(m2, rg[j]);
      gs[i] = __fadd_rn(m1, m2);
    }
    sync();
    for (int i = t; i < M * E; i += NT) {  // keep an expert if its group ranks within topk_group
      const int m = i / E, g = (i % E) / GS;
      const float v = gs[m * G + g];
      int rank = 0;
      for (int j = 0; j < G; ++j) {
        const float o = gs[m * G + j];
        rank += (o > v || (o == v && j < g)) ? 1 : 0;
      }
      if (rank >= p.topk_group) sc_s[i] = __int_as_float(0x7fc00000);  // mark (NaN) -> masked below
    }
    sync();
    for (int i = t; i < M * E; i += NT)
      if (sc_s[i] != sc_s[i]) {
        r_s[i] = -INFINITY;
        sc_s[i] = 0.f;
      }
    sync();
  }
  // ranks: `per` consecutive threads (a power of two within a warp) share a candidate, each counting over every
  // per-th competitor, and add their counts with shuffles; every thread runs the same number of rounds
  const int ncand = M * E;
  int per = 1;
  while (per < 32 && per * 2 * ncand <= NT) per *= 2;
  for (int base = 0; base < ncand * per; base += NT) {
    const int i2 = base + t;
    const bool act = i2 < ncand * per;
    const int i = act ? i2 / per : 0, part = i2 % per;
    const int m = i / E, e = i % E;
    const float v = r_s[i];
    int rank = 0;
    if (act) {
      const float* rr = r_s + m * E;
      for (int j = part; j < E; j += per) {
        const float o = rr[j];
        rank += (o > v || (o == v && j < e)) ? 1 : 0;
      }
    }
    for (int o = per >> 1; o > 0; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
    if (act && part == 0 && rank < K && v > -INFINITY) {
      sel_e[m * K + rank] = e;
      k_s[m * K + rank] = p.mode == MV_ROUTE_SIGMOID_GROUP ? static_cast<double>(sc_s[i]) : static_cast<double>(v);
    }
  }
  sync();
  if (p.mode != MV_ROUTE_SIGMOID_GROUP && M * K <= NT) {
    // softmax: each exponential once (exp(v_k - v_0), the rank-0 value is the maximum), then every weight sums
    // the same values in the same order as below
    const double ex = t < M * K ? exp(k_s[t] - k_s[(t / K) * K]) : 0.0;
    sync();
    if (t < M * K) k_s[t] = ex;
    sync();
    if (t < M * K) {
      const double* kv = k_s + (t / K) * K;
      double tot = 0.0;
      for (int j = 0; j < K; ++j) tot += kv[j];
      sel_w[t] = static_cast<float>(ex / tot);
    }
    sync();
    return;
  }
  for (int i = t; i < M * K; i += NT) {
    const int m = i / K, k = i % K;
    const double* kv = k_s + m * K;
    double w;
    if (p.mode == MV_ROUTE_SIGMOID_GROUP) {
      double tot = 0.0;
      for (int j = 0; j < K; ++j) tot += kv[j];
      w = kv[k] / (tot + 1e-20) * p.scale;
    } else {
      const double mx = kv[0];  // the rank-0 logit is the maximum
      double tot = 0.0;
      for (int j = 0; j < K; ++j) tot += exp(kv[j] - mx);
      w = exp(kv[k] - mx) / tot;
    }
    sel_w[i] = static_cast<float>(w);
  }
  sync();
}

}  // namespace route
}  // namespace mv
