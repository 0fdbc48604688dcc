// Shared pieces of the decode kernels: the launch parameters, the expert table builders and small helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "common.cuh"
#include "route_select.cuh"

namespace mv {
namespace decode {

constexpr int kStageBytes = 32768;
constexpr int kMaxM = 16;
constexpr int kMaxNK = 32;
constexpr int kMaxE1 = 4096;
constexpr int kGuSegMax = 256;  // gate/up rows per segment (int8 scale staging)
constexpr int kNhMax = 64;      // output rows per CTA

struct Params {
  const uint8_t* w_gu;
  const uint8_t* w_d;
  const void* s_gu;
  const void* s_d;
  long long gu_se, gu_sr, d_se, d_sr, sgu_se, sd_se;  // element strides
  int E1, H, I;
  int s_bf16;
  const uint16_t* x;
  long long x_stride;
  const uint16_t* norm_w;
  float eps;
  int M;
  // mode 0: pairs given
  const void* ids;
  int ids_i64;
  const float* wts;
  int NK;
  // mode 1: fused router
  int router;
  int route_mode;
  const void* rw;
  int rw_dtype;
  const void* rw_scale;
  int rw_scale_bf16;
  const float* rbias;
  int E, top_k, n_group, topk_group;
  double rscale;
  int n_static, static_id;
  float* logits_out;
  void* ids_out;
  int ids_out_i64;
  float* wts_out;
  // outputs / workspace
  const uint16_t* residual;
  uint16_t* out;
  WsHeader* ws;
  float* logits_ws;  // [M, E]
  float* a_g;        // [pairs, I]
  // geometry (host-computed)
  int n_stages;
  int RG, DR;
  int u_max;
  int region_bytes;  // x / a-buffer union
  int DP;            // w_d rows per packed down stage
  int gsc_cap;       // gate/up scales per CTA (int8)
  int nh_cap;        // output rows per CTA
  int a_all;         // 1: the down phase loads every (expert, token) activation row at once
  int E_alloc;       // selection scratch per warp (router mode)
  // tensor-core path (decode_tc_run)
  float* tc_part_gu;   // [G][2 sequences][8 segments][2][M][128] gate / up pieces of slices cut by range ends
  float* tc_part_d;    // [G * kTcMaxSeg][M][128] down-projection pieces
  uint16_t* tc_abuf;   // [u_max * 32][I] bf16: rows 0..15 = hi(a * w) per token, 16..31 = lo
  int* tc_cnt;         // [(u_max * (I / 128) + H / 128) * 4] arrival counters per 32-row group (zero between calls)
  // next-block L2 prefetch (decode kernels)
  const uint8_t* nx_rw;      // the next block's router weight (NULL: no next block) ...
  long long nx_rw_bytes;     // ... its size in bytes (a multiple of 16)
  const uint16_t* nx_norm;   // the next block's RMSNorm weight [H] bf16, or NULL
#ifdef MV_TRACE
  unsigned long long* trace;  // [G][32] %globaltimer stamps per CTA (phase-timing builds only)
#endif
};

// Phase timestamps for timing studies: compiled only with -DMV_TRACE (a separate build); nothing otherwise.
#ifdef MV_TRACE
#define MV_TRACE_AT(p, k)                                                                   \
  do {                                                                                      \
    if ((p).trace != nullptr) (p).trace[blockIdx.x * 32 + (k)] = globaltimer_ns();          \
  } while (0)
#else
#define MV_TRACE_AT(p, k) \
  do {                    \
  } while (0)
#endif

constexpr int kTcMaxSeg = 4;

template <bool INT8>
struct W;
template <>
struct W<false> {
  static constexpr int esz = 2, vec = 8;
};
template <>
struct W<true> {
  static constexpr int esz = 1, vec = 16;
};

// Rows [r, hi) of a gate/up row space of `ubase`-offset experts, cut into per-expert segments.
struct GuWalk {
  long long r, hi;
  int I, ubase;
  __device__ bool next(int& u, int& i0, int& ni, long long& rpos) {
    if (r >= hi) return false;
    rpos = r;
    u = ubase + static_cast<int>(r / I);
    i0 = static_cast<int>(r % I);
    long long n = hi - r;
    if (n > I - i0) n = I - i0;
    if (n > kGuSegMax) n = kGuSegMax;
    ni = static_cast<int>(n);
    r += n;
    return true;
  }
};

// The ring stages of a gate/up walk in order: each segment of the walk cut into stages of RG rows (gate rows
// [i, i + nr) and the matching up rows). The producer's copies, its L2 lookahead and the consumers all follow
// this one sequence.
struct GuStages {
  GuWalk w;
  int u = 0, i0 = 0, ni = 0, s0 = 0;
  __device__ bool next(int& uu, int& i, int& nr, int RG) {
    if (s0 >= ni) {
      long long r0w;
      if (!w.next(u, i0, ni, r0w)) return false;
      s0 = 0;
    }
    uu = u;
    i = i0 + s0;
    nr = min(RG, ni - s0);
    s0 += RG;
    return true;
  }
};

// The ring stages of the down projection: the (expert u, output row r) entries of a CTA in order, `per` entries
// per stage, a stage either crossing expert boundaries (packed) or ending at them. next() calls f(u, r, n, k) for
// each run of rows of one expert in the stage (k = the run's first entry within the stage).
struct DownStages {
  int u = 0, r = 0;
  template <class F>
  __device__ bool next(int U, int nh, int per, bool cross, F&& f) {
    if (u >= U || nh <= 0) return false;
    int left = per, k = 0;
    while (left > 0 && u < U) {
      const int n = min(left, nh - r);
      f(u, r, n, k);
      left -= n;
      r += n;
      k += n;
      if (r == nh) {
        r = 0;
        ++u;
        if (!cross) break;
      }
    }
    return true;
  }
  // entries in the next stage (0 at the end)
  __device__ int entries(int U, int nh, int per, bool cross) const {
    if (u >= U || nh <= 0) return 0;
    return cross ? min(per, (U - u) * nh - r) : min(per, nh - r);
  }
};

// Sums each of the 8 values v[0..7] over the 32 lanes of the warp in a fixed order; afterwards v[0] of lane l holds
// the sum of value (l >> 2) & 7. Three exchanges that halve the values held (4, 2, 1 shuffles), then two butterfly
// steps: 9 shuffles for 8 sums instead of 40.
__device__ __forceinline__ void reduce8(float (&v)[8]) {
  const int lane = threadIdx.x & 31;
  const bool b4 = (lane & 16) != 0, b3 = (lane & 8) != 0, b2 = (lane & 4) != 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b4 ? v[i] : v[i + 4];
    const float keep = b4 ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? v[i] : v[i + 2];
    const float keep = b3 ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const float send = b2 ? v[0] : v[1];
    const float keep = b2 ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// a{0,1} += the dot of one 16-byte weight chunk (VEC elements in order; int8 dequantised element by element as
// float(q) * sc) with xv[0..VEC): even elements into a0, odd into a1 (packed fp32 FMAs).
template <bool INT8>
__device__ __forceinline__ void chunk_fma(float& a0, float& a1, const uint4& wv, const float* xv, float sc) {
  const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
  if (INT8) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float f0, f1, f2, f3;
      i8x4_to_f32_packed(w[q], f0, f1, f2, f3);
      fmul2(f0, f1, f0, f1, sc);
      fmul2(f2, f3, f2, f3, sc);
      ffma2(a0, a1, f0, f1, xv[4 * q], xv[4 * q + 1]);
      ffma2(a0, a1, f2, f3, xv[4 * q + 2], xv[4 * q + 3]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) ffma2(a0, a1, bf16lo(w[q]), bf16hi(w[q]), xv[2 * q], xv[2 * q + 1]);
  }
}

// The same without the scale: a0 / a1 += float(q) * x (int8, exact products of integers and the fp32 x before
// the fp32 adds) or w * x (bf16). The caller multiplies the row's sum by its scale once.
template <bool INT8>
__device__ __forceinline__ void chunk_fma_unscaled(float& a0, float& a1, const uint4& wv, const float* xv) {
  const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
  if (INT8) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float f0, f1, f2, f3;
      i8x4_to_f32_packed(w[q], f0, f1, f2, f3);
      ffma2(a0, a1, f0, f1, xv[4 * q], xv[4 * q + 1]);
      ffma2(a0, a1, f2, f3, xv[4 * q + 2], xv[4 * q + 3]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) ffma2(a0, a1, bf16lo(w[q]), bf16hi(w[q]), xv[2 * q], xv[2 * q + 1]);
  }
}

__device__ __forceinline__ float ldscale(const void* base, long long idx, int bf16) {
  if (bf16) return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(base)[idx]) << 16);
  return reinterpret_cast<const float*>(base)[idx];
}

__device__ __forceinline__ float router_w(const Params& p, long long e, int h) {
  const long long i = e * p.H + h;
  if (p.rw_dtype == MV_F32) return static_cast<const float*>(p.rw)[i];
  if (p.rw_dtype == MV_BF16) return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(p.rw)[i]) << 16);
  const float s = ldscale(p.rw_scale, e, p.rw_scale_bf16);
  return dequant(static_cast<float>(static_cast<const int8_t*>(p.rw)[i]), s);
}

// Expert table from (expert, weight) pairs, by ONE warp, for at most 32 pairs: lane j holds pair j. Lanes with
// the same expert (and the same expert and token) are found with match.any, so first occurrences, token
// positions and counts are ballot / popc arithmetic; the rank of an expert counts the distinct smaller ids, and
// duplicate (expert, token) weights are summed in pair order.
template <int MT>
__device__ void table_warp(const int* pr_e, const float* pr_w, int npairs, int kp, int E1, int n_static, int static_id,
                           int M, int* e_id, int* e_ntok, int* e_tok, float* e_w, int* e_pbase, int* misc, WsHeader* ws) {
  constexpr unsigned int kFull = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const bool in = lane < npairs;
  const int e = in ? pr_e[lane] : -1;
  const int mj = in ? lane / kp : 0;
  const bool valid = in && e >= 0 && e < E1;
  const unsigned int lt = (1u << lane) - 1u;
  // invalid lanes get keys no other lane has (negative); valid keys are >= 0 (e < kMaxE1, mj < 32)
  const unsigned int same_e = __match_any_sync(kFull, valid ? e : -2 - lane);
  const unsigned int same_em = __match_any_sync(kFull, valid ? e * 32 + mj : -2 - lane);
  const bool first = valid && (same_e & lt) == 0u;
  const bool newtok = valid && (same_em & lt) == 0u;
  const unsigned int fmask = __ballot_sync(kFull, first);
  const unsigned int nmask = __ballot_sync(kFull, newtok);
  int rank = n_static;
  for (unsigned int b = fmask; b != 0u; b &= b - 1u)
    if (pr_e[__ffs(b) - 1] < e) ++rank;
  float wsum = 0.f;
  if (newtok)
    for (unsigned int b = same_em; b != 0u; b &= b - 1u) wsum += pr_w[__ffs(b) - 1];
  const int pos = __popc(nmask & same_e & lt);
  const int ntok = __popc(nmask & same_e);
  for (int u = lane; u < n_static; u += 32) {
    e_id[u] = static_id + u;
    e_ntok[u] = M;
    for (int t = 0; t < M; ++t) {
      e_tok[u * MT + t] = t;
      e_w[u * MT + t] = 1.0f;
    }
  }
  if (first) {
    e_id[rank] = e;
    e_ntok[rank] = ntok < MT ? ntok : MT;
  }
  if (newtok && pos < MT) {
    e_tok[rank * MT + pos] = mj;
    e_w[rank * MT + pos] = wsum;
  }
  if (newtok && pos >= MT) raise_error(ws, kErrOverflow, static_cast<unsigned int>(lane));
  __syncwarp();
  if (lane == 0) {
    const int Ut = n_static + __popc(fmask);
    int pb = 0;
    for (int u = 0; u < Ut; ++u) {
      e_pbase[u] = pb;
      pb += e_ntok[u];
    }
    misc[0] = Ut;
    misc[3] = pb;
  }
  __syncwarp();
}

// Expert table by NT threads (any number of pairs): bitmap of the distinct experts, a warp-0 prefix over its
// words, then one thread per expert collecting its tokens in order.
template <int MT, typename Sync>
__device__ void table_bitmap(const int* pr_e, const float* pr_w, int npairs, int kp, int E1, int n_static,
                             int static_id, int M, int* e_id, int* e_ntok, int* e_tok, float* e_w, int* e_pbase,
                             int* misc, unsigned int* bitmap, WsHeader* ws, int t, int NT, Sync sync) {
  const int lane = t & 31;
  const int nwords = (E1 + 31) >> 5;
  for (int i = t; i < nwords; i += NT) bitmap[i] = 0u;
  sync();
  for (int j = t; j < npairs; j += NT) {
    const int e = pr_e[j];
    if (e >= 0 && e < E1) atomicOr(&bitmap[e >> 5], 1u << (e & 31));
  }
  sync();
  if (t < 32) {
    int base = n_static;
    for (int w0 = 0; w0 < nwords; w0 += 32) {
      const int wd = w0 + lane;
      const int c = wd < nwords ? __popc(bitmap[wd]) : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (wd < nwords) {
        unsigned int b = bitmap[wd];
        int r = base + incl - c;
        while (b) {
          e_id[r++] = (wd << 5) + __ffs(b) - 1;
          b &= b - 1;
        }
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) misc[0] = base;
  }
  for (int u = t; u < n_static; u += NT) {
    e_id[u] = static_id + u;
    e_ntok[u] = M;
    for (int tt = 0; tt < M; ++tt) {
      e_tok[u * MT + tt] = tt;
      e_w[u * MT + tt] = 1.0f;
    }
  }
  sync();
  const int Ut = misc[0];
  for (int u = n_static + t; u < Ut; u += NT) {
    const int e = e_id[u];
    int n = 0;
    for (int j = 0; j < npairs; ++j) {
      if (pr_e[j] != e) continue;
      const int m = j / kp;
      if (n > 0 && e_tok[u * MT + n - 1] == m) {
        e_w[u * MT + n - 1] += pr_w[j];
      } else if (n < MT) {
        e_tok[u * MT + n] = m;
        e_w[u * MT + n] = pr_w[j];
        ++n;
      } else {
        raise_error(ws, kErrOverflow, static_cast<unsigned int>(j));
      }
    }
    e_ntok[u] = n;
  }
  sync();
  if (t == 0) {
    int pb = 0;
    for (int u = 0; u < Ut; ++u) {
      e_pbase[u] = pb;
      pb += e_ntok[u];
    }
    misc[3] = pb;
  }
  sync();
}

}  // namespace decode

// The tensor-core decode path (bf16 weights): workspace need and launch. Returns MV_OK, an error, or
// kDecodeTcUnsuitable when the shapes / workspace do not fit it (the caller then uses the CUDA-core kernel).
constexpr int kDecodeTcUnsuitable = -1;
constexpr int kDecodeM1Unsuitable = -2;

// Whether the decode kernels are launched as programmatic dependents of the previous kernel in the stream (their
// CTAs are scheduled while it finishes; each kernel waits for it before reading the token or the workspace).
// MINGMOE_PDL=0 turns it off.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("MINGMOE_PDL");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}
int decode_m1_run(decode::Params& p, bool int8, cudaStream_t st);
size_t decode_tc_workspace_bytes(int M, int nk, int H, int I, int E1, int E, int n_static);
int decode_tc_run(decode::Params& p, void* workspace, size_t workspace_bytes, int nk_pairs, cudaStream_t st);

}  // namespace mv
