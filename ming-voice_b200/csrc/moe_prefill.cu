// Prefill MoE (any number of tokens) on the 5th-generation tensor cores.
//
// mv_moe_prefill replaces fused_moe.fused_moe_prefill (ming-voice fused_moe.py:176-196; kernels
// _moe_gu_grouped :93-121, _moe_down_grouped :125-148) and mv_moe_align replaces _align_blocks (:154-173).
//
// Pipeline (six launches, no host synchronisation, capture-safe):
//   1. align_*_kernel  stable counting sort of the (token, slot) pairs by expert, each expert's run padded to
//                      128 rows (three launches); the same sorted_ids / bexp arrays the reference builds
//                      (pad id = P, unused block = -1). Pairs with id -1 are left out (expert-parallel prefill
//                      marks the pairs another rank computes that way).
//   2. gather_kernel   xs[r] = x[token of sorted pair r] (bf16, zero rows for pads) and y32 = residual (fp32).
//   3. gemm_kernel     one persistent cooperative launch over two tile sequences:
//                      gate/up tiles, per 128-pair block and 128-column slice of the intermediate dimension:
//                      [gate | up] = xs_blk . W_gu[e]^T as ONE 128 x 256 tcgen05 tile (gate rows n0.., up rows
//                      I+n0.. side by side in shared memory), epilogue a = bf16(silu(gate) * up);
//                      then down tiles, per block and 256-column slice of H: o = a_blk . W_d[e]^T, epilogue
//                      y32[token] += weight * o (fp32 vector reductions; pads skipped). A down tile starts as soon
//                      as its block's gate/up tiles are stored (per-block counters), so the last gate/up wave and
//                      the first down wave overlap.
//   4. finalize_kernel out = bf16(y32).
// The GEMM kernel is warp-specialised: warp 0 issues TMA loads into a 4-deep ring of 48 KB stages (A 128x64,
// B 256x64 bf16, 128-byte swizzle), warp 1 issues tcgen05.mma (M=128, N=256, K=16) into one of two TMEM
// accumulators (2 x 256 fp32 columns), warps 2-5 drain the other accumulator (tcgen05.ld) while the next tile
// accumulates. Every wait is bounded (errors go to the workspace header).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "tc.cuh"

namespace mv {
namespace prefill {

constexpr int kBM = 128;       // sorted pairs per block = MMA M
constexpr int kBK = 64;        // K per stage: one 128-byte swizzle row of bf16
constexpr int kGuHalf = 128;   // gate (and up) columns per gate/up tile: MMA N = 256
constexpr int kDownN = 256;    // output columns per down tile: MMA N = 256
constexpr int kStages = 4;
constexpr int kAStageBytes = kBM * kBK * 2;   // 16 KB
constexpr int kBStageBytes = 256 * kBK * 2;   // 32 KB
constexpr int kStageBytes = kAStageBytes + kBStageBytes;
constexpr int kThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue
constexpr uint32_t kTmemCols = 512;
constexpr int kAlignMaxE1 = 512;
constexpr size_t kGemmSmem = 1024 + kStages * kStageBytes + 256;

__device__ __forceinline__ int load_id(const void* ids, int ids_i64, int p) {
  return ids_i64 ? static_cast<int>(static_cast<const long long*>(ids)[p]) : static_cast<const int*>(ids)[p];
}

// ------------------------------------------------------------------------------------------------ align

// Three launches over chunks of kChunk pairs. Stable: pairs of one expert keep their index order (the
// reference's counting sort), because chunk c's pairs follow chunk c-1's and, inside a chunk, warp w's
// follow warp w-1's and lane order is kept within a warp.
//   align_count_kernel   (one CTA per chunk) per-chunk histogram hist[c][e]
//   align_scan_kernel    (one CTA) hist -> exclusive prefix over chunks, padded run starts, bexp, nb_used,
//                        padding ids (P) for the rows no pair lands on
//   align_scatter_kernel (one CTA per chunk) sorted[start[e] + hist[c][e] + rank] = pair
constexpr int kChunk = 1024;

static size_t align_scratch_bytes(int P, int E1) {
  const size_t nch = static_cast<size_t>(P + kChunk - 1) / kChunk;
  return (nch * E1 + E1) * sizeof(int);
}


__global__ void __launch_bounds__(kChunk) align_count_kernel(const void* __restrict__ ids, int ids_i64, int P, int E1,
                                                             int* __restrict__ hist, WsHeader* ws) {
  extern __shared__ int sh[];
  for (int e = threadIdx.x; e < E1; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int p = blockIdx.x * kChunk + threadIdx.x;
  if (p < P) {
    const int e = load_id(ids, ids_i64, p);
    if (e >= 0 && e < E1)
      atomicAdd(&sh[e], 1);
    else if (e != -1)  // -1: no pair (an expert held by another rank); anything else is an error
      raise_error(ws, kErrBadExpert, static_cast<unsigned int>(p));
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E1; e += blockDim.x) hist[static_cast<long long>(blockIdx.x) * E1 + e] = sh[e];
}

__global__ void __launch_bounds__(1024) align_scan_kernel(int P, int E1, int BM, int nb_max, int nch,
                                                          int* __restrict__ hist, int* __restrict__ start_g,
                                                          int* __restrict__ sorted, int* __restrict__ bexp,
                                                          int* __restrict__ nb_used) {
  extern __shared__ int sh[];
  int* cnt = sh;
  int* start = sh + E1;
  __shared__ int s_total;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E1; e += blockDim.x) {  // exclusive prefix over chunks, per expert
    int acc = 0;
    for (int c = 0; c < nch; ++c) {
      const long long i = static_cast<long long>(c) * E1 + e;
      const int v = hist[i];
      hist[i] = acc;
      acc += v;
    }
    cnt[e] = acc;
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan of the padded run lengths
    const int per = (E1 + 31) / 32;
    const int lo = lane * per, hi = min(lo + per, E1);
    int s = 0;
    for (int e = lo; e < hi; ++e) s += (cnt[e] + BM - 1) / BM * BM;
    int incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int ex = incl - s;
    for (int e = lo; e < hi; ++e) {
      start[e] = ex;
      ex += (cnt[e] + BM - 1) / BM * BM;
    }
    if (lane == 31) s_total = incl;
  }
  __syncthreads();
  const int total = s_total;
  for (int e = tid; e < E1; e += blockDim.x) {
    start_g[e] = start[e];
    const int pad_end = start[e] + (cnt[e] + BM - 1) / BM * BM;
    for (int r = start[e] + cnt[e]; r < pad_end; ++r) sorted[r] = P;
  }
  for (int r = total + tid; r < nb_max * BM; r += blockDim.x) sorted[r] = P;
  for (int b = tid; b < nb_max; b += blockDim.x) {
    int e = -1;
    if (b * BM < total) {  // first expert whose padded run ends after row b*BM
      int lo = 0, hi = E1 - 1;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (start[mid] + (cnt[mid] + BM - 1) / BM * BM > b * BM)
          hi = mid;
        else
          lo = mid + 1;
      }
      e = lo;
    }
    bexp[b] = e;
  }
  if (tid == 0) *nb_used = total / BM;
}

__global__ void __launch_bounds__(kChunk) align_scatter_kernel(const void* __restrict__ ids, int ids_i64, int P,
                                                               int E1, const int* __restrict__ hist,
                                                               const int* __restrict__ start_g,
                                                               int* __restrict__ sorted) {
  extern __shared__ int wcnt[];  // [32][E1]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int p = blockIdx.x * kChunk + tid;
  int e = p < P ? load_id(ids, ids_i64, p) : -1;
  const bool valid = e >= 0 && e < E1;
  if (!valid) e = -1;
  const unsigned int m = __match_any_sync(0xffffffffu, e);
  const unsigned int before = m & ((1u << lane) - 1u);
  for (int i = tid; i < 32 * E1; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  if (valid && before == 0u) wcnt[warp * E1 + e] = __popc(m);
  __syncthreads();
  if (valid) {
    int off = start_g[e] + hist[static_cast<long long>(blockIdx.x) * E1 + e] + __popc(before);
    for (int w2 = 0; w2 < warp; ++w2) off += wcnt[w2 * E1 + e];
    sorted[off] = p;
  }
}

// ------------------------------------------------------------------------------------------------ gather

// One warp per row: rows [0, nb_used*128) of xs from the sorted pairs, then rows [0, N) of y32.
// Rows [0, n_x) of the pass come from x, rows [n_x, N) from x2 (row stride x2_stride): the own and the received
// rows of an expert-parallel pass, read where they lie.
__global__ void __launch_bounds__(256) gather_kernel(const uint16_t* __restrict__ x, long long x_stride, int n_x,
                                                     const uint16_t* __restrict__ x2, long long x2_stride,
                                                     const int* __restrict__ sorted, const int* __restrict__ nb_used,
                                                     int NK, int P, int H, uint16_t* __restrict__ xs,
                                                     const uint16_t* __restrict__ residual, long long r_stride,
                                                     float* __restrict__ y32, int N, int* __restrict__ ready,
                                                     int nb_max) {
  const int lane = threadIdx.x & 31;
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < nb_max; i += blockDim.x) ready[i] = 0;
  const long long rows_xs = static_cast<long long>(*nb_used) * kBM;
  const long long total = rows_xs + N;
  const int nv = H / 8;  // 16-byte vectors per row
  for (long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; row < total;
       row += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    if (row < rows_xs) {
      const int p = sorted[row];
      uint4* dst = reinterpret_cast<uint4*>(xs + row * H);
      if (p < P) {
        const int tok = p / NK;
        const uint4* src = reinterpret_cast<const uint4*>(
            tok < n_x ? x + static_cast<long long>(tok) * x_stride : x2 + static_cast<long long>(tok - n_x) * x2_stride);
        for (int v = lane; v < nv; v += 32) dst[v] = src[v];
      } else {
        for (int v = lane; v < nv; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
      }
    } else {
      const long long t = row - rows_xs;
      float4* dst = reinterpret_cast<float4*>(y32 + t * H);
      if (residual != nullptr) {
        const uint4* src = reinterpret_cast<const uint4*>(residual + t * r_stride);
        for (int v = lane; v < nv; v += 32) {
          const uint4 q = src[v];
          dst[2 * v] = make_float4(bf16lo(q.x), bf16hi(q.x), bf16lo(q.y), bf16hi(q.y));
          dst[2 * v + 1] = make_float4(bf16lo(q.z), bf16hi(q.z), bf16lo(q.w), bf16hi(q.w));
        }
      } else {
        for (int v = lane; v < 2 * nv; v += 32) dst[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
}

__global__ void __launch_bounds__(256) finalize_kernel(const float* __restrict__ y32, long long n4,
                                                       uint16_t* __restrict__ out) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(y32)[i];
    uint2 o;
    o.x = static_cast<uint32_t>(f2bf(v.x)) | (static_cast<uint32_t>(f2bf(v.y)) << 16);
    o.y = static_cast<uint32_t>(f2bf(v.z)) | (static_cast<uint32_t>(f2bf(v.w)) << 16);
    reinterpret_cast<uint2*>(out)[i] = o;
  }
}

// ------------------------------------------------------------------------------------------------ int8 weights

// int8 expert rows -> bf16 rows (exact: |q| <= 127), for the experts the blocks in use refer to; the scales are
// applied to the fp32 products in the GEMM epilogues, as the reference's int8 kernels do (fused_moe.py:115-121).
// Grid: (row groups, E1); a CTA of an expert no block uses returns at once.
__global__ void __launch_bounds__(256) widen_experts_kernel(const int8_t* __restrict__ q, long long q_se, long long q_sr,
                                                            int rows, int K, const int* __restrict__ bexp,
                                                            const int* __restrict__ nb_used, uint16_t* __restrict__ out) {
  const int e = blockIdx.y;
  __shared__ int used;
  if (threadIdx.x == 0) used = 0;
  __syncthreads();
  const int nb = *nb_used;
  for (int b = threadIdx.x; b < nb; b += blockDim.x)
    if (bexp[b] == e) used = 1;
  __syncthreads();
  if (!used) return;
  const int nv = K / 16;  // 16 int8 per 16-byte load
  const int r0 = blockIdx.x * 16;
  for (int i = threadIdx.x; i < 16 * nv; i += blockDim.x) {
    const int r = r0 + i / nv, v = i % nv;
    if (r >= rows) break;
    const uint4 w = *reinterpret_cast<const uint4*>(q + e * q_se + r * q_sr + v * 16);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float f0, f1, f2, f3;
      i8x4_to_f32(ww[k], f0, f1, f2, f3);
      o[2 * k] = static_cast<uint32_t>(f2bf(f0)) | (static_cast<uint32_t>(f2bf(f1)) << 16);
      o[2 * k + 1] = static_cast<uint32_t>(f2bf(f2)) | (static_cast<uint32_t>(f2bf(f3)) << 16);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + (static_cast<long long>(e) * rows + r) * K + v * 16);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// ------------------------------------------------------------------------------------------------ GEMMs

struct GemmArgs {
  const int* sorted;   // [nb_max * 128] pair ids (P = pad)
  const int* bexp;     // [nb_max] expert per block
  const int* nb_used;  // device scalar: blocks in use
  int P, NK, H, I;
  int n_tiles;         // N tiles per block
  int k_steps;         // K / 64
  uint16_t* a_out;     // gate/up: [rows, I] bf16
  float* y32;          // down: [N, H] fp32 accumulator
  const float* wts;    // down: [P] routing weights
  const void* scale;   // int8 weights: per-row scales of the B operand (s_gu [E1, 2I] / s_d [E1, H]), else NULL
  long long scale_se;  // expert stride of `scale` (elements)
  int scale_bf16;      // 1: bf16 scales, 0: f32
  WsHeader* ws;
};

__device__ __forceinline__ float ld_scale(const void* base, long long i, int bf16) {
  return bf16 ? __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(base)[i]) << 16)
              : static_cast<const float*>(base)[i];
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + __expf(-g)) * u; }

// Both GEMMs in one persistent launch. The tile sequence is the gate/up tiles (block-major) followed by the down
// tiles; CTA c takes tiles c, c + G, ... in order. A down tile of block b needs all gate/up tiles of b stored:
// each gate/up epilogue warp counts its 32 rows into ready[b] (release), and the producer waits (acquire,
// bounded) before loading the activation tile. Those gate/up tiles come earlier in the sequence and every CTA
// processes its tiles in order, so with all CTAs resident (cooperative launch) the wait always ends; it lets
// the down tiles start while the last gate/up wave drains instead of after it.
__device__ __forceinline__ void tile_of(int tile, int T0, const GemmArgs& g0, const GemmArgs& g1, int& ph, int& blk,
                                        int& nt) {
  ph = tile >= T0;
  const int local = ph ? tile - T0 : tile;
  const int n = ph ? g1.n_tiles : g0.n_tiles;
  blk = local / n;
  nt = local - blk * n;
}

__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmA0,
                                                           const __grid_constant__ CUtensorMap tmB0,
                                                           const __grid_constant__ CUtensorMap tmA1,
                                                           const __grid_constant__ CUtensorMap tmB1, const GemmArgs g0,
                                                           const GemmArgs g1, int* __restrict__ ready) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stA = smem;
  uint8_t* stB = smem + kStages * kAStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(stB + kStages * kBStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* accf = empty + kStages;
  uint64_t* acce = accf + 2;
  uint64_t* done = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 128);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tmA0);
    tc::prefetch_tmap(&tmB0);
    tc::prefetch_tmap(&tmA1);
    tc::prefetch_tmap(&tmB1);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int nb = *g0.nb_used;
  const int T0 = nb * g0.n_tiles;
  const int total = T0 + nb * g1.n_tiles;
  const unsigned int need = static_cast<unsigned int>(g0.n_tiles) * 4u;  // gate/up epilogue warps per block

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        int ph, blk, nt;
        tile_of(tile, T0, g0, g1, ph, blk, nt);
        const GemmArgs& g = ph ? g1 : g0;
        const int e = g.bexp[blk];
        if (ph) {  // the block's activations are complete (all its gate/up tiles stored)
          const unsigned int* r = reinterpret_cast<const unsigned int*>(ready + blk);
          if (ld_acquire_u32(r) < need) {
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_u32(r) < need) {
              __nanosleep(64);
              if (globaltimer_ns() - t0 > kWaitLimitNs) {
                raise_error(g.ws, kErrTimeout, 0x560u);
                ok = false;
                break;
              }
            }
            if (!ok) break;
          }
          fence_proxy_async_global();  // generic-proxy stores of other CTAs, read by the TMA (async proxy)
        }
        for (int k = 0; k < g.k_steps; ++k) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, g.ws, 0x500u + ph)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          uint8_t* a = stA + stage * kAStageBytes;
          uint8_t* b = stB + stage * kBStageBytes;
          if (ph == 0) {
            tc::tma_load_2d(a, &tmA0, &full[stage], k * kBK, blk * kBM);
            tc::tma_load_3d(b, &tmB0, &full[stage], k * kBK, nt * kGuHalf, e);
            tc::tma_load_3d(b + kBStageBytes / 2, &tmB0, &full[stage], k * kBK, g.I + nt * kGuHalf, e);
          } else {
            tc::tma_load_2d(a, &tmA1, &full[stage], k * kBK, blk * kBM);
            tc::tma_load_3d(b, &tmB1, &full[stage], k * kBK, nt * kDownN, e);
          }
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // copies still in flight land before the CTA exits (immediate when the MMA warp consumed them)
      for (int s = 0; s < kStages && s < issued; ++s) {
        const int last_round = (issued - 1 - s) / kStages;
        mbar_wait(&full[s], static_cast<uint32_t>(last_round & 1), g0.ws, 0x510u);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kBM, 256);
      int stage = 0, j = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++j) {
        int ph, blk, nt;
        tile_of(tile, T0, g0, g1, ph, blk, nt);
        const int k_steps = ph ? g1.k_steps : g0.k_steps;
        const int buf = j & 1;
        const uint32_t aph = static_cast<uint32_t>(j >> 1) & 1u;
        if (!mbar_wait(&acce[buf], aph ^ 1u, g0.ws, 0x520u + ph)) break;
        tc::fence_after_sync();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * 256);
        for (int k = 0; k < k_steps; ++k) {
          if (!mbar_wait(&full[stage], phase, g0.ws, 0x530u + ph)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t ad = tc::sw128_desc(smem_u32(stA + stage * kAStageBytes));
          const uint64_t bd = tc::sw128_desc(smem_u32(stB + stage * kBStageBytes));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc::mma_bf16(d, ad + 2 * kk, bd + 2 * kk, idesc, (k | kk) != 0 ? 1u : 0u);
          tc::mma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) tc::mma_commit(&accf[buf]);
      }
      // every issued MMA retires before the TMEM is released
      tc::mma_commit(done);
      mbar_wait(done, 0u, g0.ws, 0x540u);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int g4 = warp & 3;  // the TMEM lane group this warp may access
    const int row = g4 * 32 + lane;
    int j = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++j) {
      int ph, blk, nt;
      tile_of(tile, T0, g0, g1, ph, blk, nt);
      const GemmArgs& g = ph ? g1 : g0;
      const int buf = j & 1;
      const uint32_t aph = static_cast<uint32_t>(j >> 1) & 1u;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&accf[buf], aph, g.ws, 0x550u + ph));
      if (!ok) break;
      tc::fence_after_sync();
      const long long r = static_cast<long long>(blk) * kBM + row;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(g4 * 32) << 16) + static_cast<uint32_t>(buf * 256);
      if (ph == 0) {
        uint4* dst = reinterpret_cast<uint4*>(g.a_out + r * g.I + nt * kGuHalf);
#pragma unroll 1
        for (int c = 0; c < kGuHalf / 32; ++c) {
          uint32_t gr[32], ur[32];
          tc::tmem_ld32(taddr + c * 32, gr);
          tc::tmem_ld32(taddr + kGuHalf + c * 32, ur);
          tc::tmem_ld_wait();
          if (g.scale != nullptr) {  // int8: the fp32 dot product times the weight row's scale (as the reference)
            const long long sb = static_cast<long long>(g.bexp[blk]) * g.scale_se + nt * kGuHalf + c * 32;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              gr[i] = __float_as_uint(__uint_as_float(gr[i]) * ld_scale(g.scale, sb + i, g.scale_bf16));
              ur[i] = __float_as_uint(__uint_as_float(ur[i]) * ld_scale(g.scale, sb + g.I + i, g.scale_bf16));
            }
          }
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float a0 = silu_mul(__uint_as_float(gr[2 * i]), __uint_as_float(ur[2 * i]));
            const float a1 = silu_mul(__uint_as_float(gr[2 * i + 1]), __uint_as_float(ur[2 * i + 1]));
            pk[i] = static_cast<uint32_t>(f2bf(a0)) | (static_cast<uint32_t>(f2bf(a1)) << 16);
          }
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[c * 4 + v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
        tc::fence_before_sync();
        mbar_arrive(&acce[buf]);
        // this warp's 32 activation rows of block blk are stored: count them for the down tiles (release)
        fence_proxy_async_global();
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(ready + blk, 1);
        continue;
      }
      const int p = g.sorted[r];
      const bool live = p < g.P;
      float w = 0.f;
      float* dst = nullptr;
      if (live) {
        w = g.wts[p];
        dst = g.y32 + static_cast<long long>(p / g.NK) * g.H + nt * kDownN;
      }
#pragma unroll 1
      for (int c = 0; c < kDownN / 32; ++c) {
        uint32_t v[32];
        tc::tmem_ld32(taddr + c * 32, v);
        tc::tmem_ld_wait();
        if (live && g.scale != nullptr) {
          const long long sb = static_cast<long long>(g.bexp[blk]) * g.scale_se + nt * kDownN + c * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * ld_scale(g.scale, sb + i, g.scale_bf16));
        }
        if (live) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            red_add_v4_f32(dst + c * 32 + 4 * i, w * __uint_as_float(v[4 * i]), w * __uint_as_float(v[4 * i + 1]),
                           w * __uint_as_float(v[4 * i + 2]), w * __uint_as_float(v[4 * i + 3]));
        }
      }
      tc::fence_before_sync();
      mbar_arrive(&acce[buf]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------ host

struct Layout {
  int P, nb_max;
  long long rows;
  size_t off_nb, off_ready, off_align, off_sorted, off_bexp, off_xs, off_a, off_y32, off_wgu, off_wd, total;
};

static size_t up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static Layout layout(int N, int NK, int H, int I, int E1, bool int8) {
  Layout L{};
  L.P = N * NK;
  L.nb_max = (L.P + E1 * (kBM - 1) + kBM - 1) / kBM;
  L.rows = static_cast<long long>(L.nb_max) * kBM;
  size_t o = kWsHeaderBytes;
  L.off_nb = o;
  o += 256;
  L.off_ready = o;  // per block: gate/up epilogue warps done (the down tiles wait for them)
  o = up(o + static_cast<size_t>(L.nb_max) * 4, 256);
  L.off_align = o;
  o = up(o + align_scratch_bytes(L.P, E1), 256);
  L.off_sorted = o;
  o = up(o + static_cast<size_t>(L.rows) * 4, 256);
  L.off_bexp = o;
  o = up(o + static_cast<size_t>(L.nb_max) * 4, 256);
  L.off_xs = o;
  o = up(o + static_cast<size_t>(L.rows) * H * 2, 256);
  L.off_a = o;
  o = up(o + static_cast<size_t>(L.rows) * I * 2, 256);
  L.off_y32 = o;
  o = up(o + static_cast<size_t>(N) * H * 4, 256);
  L.off_wgu = L.off_wd = 0;
  if (int8) {  // bf16 copies of the int8 experts in use (same stacked layout, contiguous)
    L.off_wgu = o;
    o = up(o + static_cast<size_t>(E1) * 2 * I * H * 2, 256);
    L.off_wd = o;
    o = up(o + static_cast<size_t>(E1) * H * I * 2, 256);
  }
  L.total = o;
  return L;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// bf16 tensor map, 128-byte swizzle, box inner 64 elements. dims/strides innermost first; strides in bytes.
static int make_tmap(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                     const uint32_t* box, const char* what) {
  auto enc = encode_fn();
  if (enc == nullptr) return fail(MV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
                         reinterpret_cast<const cuuint64_t*>(dims), reinterpret_cast<const cuuint64_t*>(strides),
                         reinterpret_cast<const cuuint32_t*>(box), estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MV_ERR_INVALID, "tensor map for %s rejected (CUresult %d)", what, static_cast<int>(r));
  return MV_OK;
}

// scratch: align_scratch_bytes(P, E1) bytes (hist [nch][E1], start [E1])
static int launch_align(const void* ids, int ids_dtype, int P, int E1, int BM, int nb_max, int* sorted, int* bexp,
                        int* nb_used, int* scratch, WsHeader* ws, cudaStream_t st) {
  const int nch = (P + kChunk - 1) / kChunk;
  int* hist = scratch;
  int* start = scratch + static_cast<size_t>(nch) * E1;
  const size_t sm_scatter = static_cast<size_t>(32) * E1 * sizeof(int);
  cudaError_t e = cudaFuncSetAttribute(align_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(sm_scatter));
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(align)");
  if (nch > 0) {
    align_count_kernel<<<nch, kChunk, E1 * sizeof(int), st>>>(ids, ids_dtype == MV_I64, P, E1, hist, ws);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "align count launch");
  }
  align_scan_kernel<<<1, 1024, 2 * E1 * sizeof(int), st>>>(P, E1, BM, nb_max, nch, hist, start, sorted, bexp, nb_used);
  if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "align scan launch");
  if (nch > 0) {
    align_scatter_kernel<<<nch, kChunk, sm_scatter, st>>>(ids, ids_dtype == MV_I64, P, E1, hist, start, sorted);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "align scatter launch");
  }
  return MV_OK;
}

}  // namespace prefill
}  // namespace mv

using namespace mv;
using namespace mv::prefill;

extern "C" int mv_moe_align(const void* ids, int ids_dtype, int P, int E1, int BM, int* sorted_out, int* bexp_out,
                            int* nb_used_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (ids_dtype != MV_I32 && ids_dtype != MV_I64) return fail(MV_ERR_INVALID, "mv_moe_align: ids must be i32 or i64");
  if (P < 0 || E1 < 1 || E1 > kAlignMaxE1 || BM < 1 || BM > 4096)
    return fail(MV_ERR_INVALID, "mv_moe_align: bad P=%d / E1=%d (<= %d) / BM=%d", P, E1, kAlignMaxE1, BM);
  if ((P > 0 && ids == nullptr) || sorted_out == nullptr || bexp_out == nullptr || nb_used_out == nullptr)
    return fail(MV_ERR_INVALID, "mv_moe_align: null pointer");
  const size_t need = mv_moe_align_workspace_bytes(P, E1);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(MV_ERR_WORKSPACE, "mv_moe_align: workspace of %zu bytes needed", need);
  const long long nb_max = (static_cast<long long>(P) + static_cast<long long>(E1) * (BM - 1) + BM - 1) / BM;
  if (nb_max * BM > 0x7fffffffLL) return fail(MV_ERR_INVALID, "mv_moe_align: too many pairs");
  return launch_align(ids, ids_dtype, P, E1, BM, static_cast<int>(nb_max), sorted_out, bexp_out, nb_used_out,
                      reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + kWsHeaderBytes),
                      static_cast<WsHeader*>(workspace), static_cast<cudaStream_t>(stream));
}

extern "C" size_t mv_moe_align_workspace_bytes(int P, int E1) {
  return kWsHeaderBytes + align_scratch_bytes(P > 0 ? P : 0, E1 > 0 ? E1 : 1);
}

extern "C" size_t mv_moe_prefill_workspace_bytes(int N, int NK, int H, int I, int E1, int w_dtype) {
  if (N < 0 || NK < 1 || H < 1 || I < 1 || E1 < 1) return 0;
  return layout(N, NK, H, I, E1, w_dtype == MV_I8).total;
}

// The pipeline of mv_moe_prefill; with out32 != NULL the fp32 sums are accumulated straight into out32 [N, H]
// (residual added in fp32 when given) and nothing is rounded to bf16.
static int prefill_run(const mv_moe_weights* w, const void* x, long long x_stride, const void* ids, int ids_dtype,
                       const float* wts, int N, int NK, const void* residual, long long residual_stride, void* out,
                       float* out32, void* workspace, size_t workspace_bytes, void* stream, int max_ctas = 0,
                       int n_x = -1, const void* x2 = nullptr, long long x2_stride = 0) {
  if (n_x < 0 || x2 == nullptr) n_x = N;
  if (n_x < N && (!aligned16(x2) || (x2_stride * 2) % 16 || x2_stride < w->H))
    return fail(MV_ERR_ALIGN, "mv_moe_prefill: second row source must be 16-byte aligned with a row stride >= H");
  if (w == nullptr || (N > 0 && (x == nullptr || ids == nullptr || wts == nullptr || (out == nullptr && out32 == nullptr))))
    return fail(MV_ERR_INVALID, "mv_moe_prefill: null pointer argument");
  if (ids_dtype != MV_I32 && ids_dtype != MV_I64) return fail(MV_ERR_INVALID, "mv_moe_prefill: ids must be i32 or i64");
  const bool int8 = w->w_dtype == MV_I8;
  if (!int8 && w->w_dtype != MV_BF16) return fail(MV_ERR_UNSUPPORTED, "mv_moe_prefill: weights must be bf16 or int8");
  if (int8 && (w->s_gu == nullptr || w->s_d == nullptr || (w->s_dtype != MV_F32 && w->s_dtype != MV_BF16)))
    return fail(MV_ERR_INVALID, "mv_moe_prefill: int8 weights need f32/bf16 scales s_gu and s_d");
  const int H = w->H, I = w->I, E1 = w->E1;
  if (N < 0 || NK < 1 || NK > 64) return fail(MV_ERR_INVALID, "mv_moe_prefill: bad N=%d / NK=%d", N, NK);
  if (H % kDownN != 0 || I % kGuHalf != 0 || H > 65536 || I > 65536)
    return fail(MV_ERR_INVALID, "mv_moe_prefill: H=%d must be a multiple of %d and I=%d of %d", H, kDownN, I, kGuHalf);
  if (E1 < 1 || E1 > kAlignMaxE1) return fail(MV_ERR_INVALID, "mv_moe_prefill: E1=%d outside [1, %d]", E1, kAlignMaxE1);
  if (static_cast<long long>(N) * NK > 0x7fffffffLL / 2) return fail(MV_ERR_INVALID, "mv_moe_prefill: too many pairs");
  if (N == 0) return MV_OK;
  const int esz = int8 ? 1 : 2;
  if (!aligned16(w->w_gu) || !aligned16(w->w_d) || !aligned16(x) || (out != nullptr && !aligned16(out)) ||
      (out32 != nullptr && !aligned16(out32)) ||
      (residual != nullptr && (!aligned16(residual) || (residual_stride * 2) % 16)) || (x_stride * 2) % 16 ||
      (w->gu_sr * esz) % 16 || (w->gu_se * esz) % 16 || (w->d_sr * esz) % 16 || (w->d_se * esz) % 16)
    return fail(MV_ERR_ALIGN, "mv_moe_prefill: pointers and row strides must be 16-byte aligned");
  if (x_stride < H || (residual != nullptr && residual_stride < H))
    return fail(MV_ERR_INVALID, "mv_moe_prefill: row stride shorter than H");
  const Layout L = layout(N, NK, H, I, E1, int8);
  if (workspace == nullptr || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(MV_ERR_WORKSPACE, "mv_moe_prefill: 256-byte aligned workspace of %zu bytes needed", L.total);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  WsHeader* hdr = reinterpret_cast<WsHeader*>(ws);
  int* nb_used = reinterpret_cast<int*>(ws + L.off_nb);
  int* ready = reinterpret_cast<int*>(ws + L.off_ready);
  int* sorted = reinterpret_cast<int*>(ws + L.off_sorted);
  int* bexp = reinterpret_cast<int*>(ws + L.off_bexp);
  uint16_t* xs = reinterpret_cast<uint16_t*>(ws + L.off_xs);
  uint16_t* abuf = reinterpret_cast<uint16_t*>(ws + L.off_a);
  float* y32 = out32 != nullptr ? out32 : reinterpret_cast<float*>(ws + L.off_y32);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // int8: the GEMMs read bf16 copies of the experts in use (exact), contiguous in the workspace
  uint16_t* wgu16 = int8 ? reinterpret_cast<uint16_t*>(ws + L.off_wgu) : nullptr;
  uint16_t* wd16 = int8 ? reinterpret_cast<uint16_t*>(ws + L.off_wd) : nullptr;
  const void* gu_base = int8 ? static_cast<const void*>(wgu16) : w->w_gu;
  const void* d_base = int8 ? static_cast<const void*>(wd16) : w->w_d;
  const long long gu_sr = int8 ? H : w->gu_sr, gu_se = int8 ? 2LL * I * H : w->gu_se;
  const long long d_sr = int8 ? I : w->d_sr, d_se = int8 ? static_cast<long long>(H) * I : w->d_se;

  CUtensorMap tm_xs, tm_wgu, tm_a, tm_wd;
  int rc;
  {
    const uint64_t d[2] = {static_cast<uint64_t>(H), static_cast<uint64_t>(L.rows)};
    const uint64_t s[1] = {static_cast<uint64_t>(H) * 2};
    const uint32_t b[2] = {kBK, kBM};
    if ((rc = make_tmap(&tm_xs, xs, 2, d, s, b, "xs")) != MV_OK) return rc;
  }
  {
    const uint64_t d[3] = {static_cast<uint64_t>(H), static_cast<uint64_t>(2 * I), static_cast<uint64_t>(E1)};
    const uint64_t s[2] = {static_cast<uint64_t>(gu_sr) * 2, static_cast<uint64_t>(gu_se) * 2};
    const uint32_t b[3] = {kBK, kGuHalf, 1};
    if ((rc = make_tmap(&tm_wgu, gu_base, 3, d, s, b, "w_gu")) != MV_OK) return rc;
  }
  {
    const uint64_t d[2] = {static_cast<uint64_t>(I), static_cast<uint64_t>(L.rows)};
    const uint64_t s[1] = {static_cast<uint64_t>(I) * 2};
    const uint32_t b[2] = {kBK, kBM};
    if ((rc = make_tmap(&tm_a, abuf, 2, d, s, b, "a")) != MV_OK) return rc;
  }
  {
    const uint64_t d[3] = {static_cast<uint64_t>(I), static_cast<uint64_t>(H), static_cast<uint64_t>(E1)};
    const uint64_t s[2] = {static_cast<uint64_t>(d_sr) * 2, static_cast<uint64_t>(d_se) * 2};
    const uint32_t b[3] = {kBK, kDownN, 1};
    if ((rc = make_tmap(&tm_wd, d_base, 3, d, s, b, "w_d")) != MV_OK) return rc;
  }

  if ((rc = launch_align(ids, ids_dtype, L.P, E1, kBM, L.nb_max, sorted, bexp, nb_used,
                        reinterpret_cast<int*>(ws + L.off_align), hdr, st)) != MV_OK)
    return rc;
  const int G = max_ctas > 0 && max_ctas < num_sms() ? max_ctas : num_sms();  // SMs for the persistent GEMM
  gather_kernel<<<G * 4, 256, 0, st>>>(static_cast<const uint16_t*>(x), x_stride, n_x,
                                       static_cast<const uint16_t*>(x2), x2_stride, sorted, nb_used, NK, L.P, H, xs,
                                       static_cast<const uint16_t*>(residual), residual_stride, y32, N, ready,
                                       L.nb_max);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "gather launch");
  if (int8) {
    widen_experts_kernel<<<dim3((2 * I + 15) / 16, E1), 256, 0, st>>>(static_cast<const int8_t*>(w->w_gu), w->gu_se,
                                                                     w->gu_sr, 2 * I, H, bexp, nb_used, wgu16);
    widen_experts_kernel<<<dim3((H + 15) / 16, E1), 256, 0, st>>>(static_cast<const int8_t*>(w->w_d), w->d_se, w->d_sr,
                                                                 H, I, bexp, nb_used, wd16);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_status(e, "int8 widening launch");
  }

  GemmArgs ga{};
  ga.sorted = sorted;
  ga.bexp = bexp;
  ga.nb_used = nb_used;
  ga.P = L.P;
  ga.NK = NK;
  ga.H = H;
  ga.I = I;
  ga.a_out = abuf;
  ga.y32 = y32;
  ga.wts = wts;
  ga.ws = hdr;
  e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kGemmSmem));
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemm)");
  GemmArgs g1 = ga;
  ga.n_tiles = I / kGuHalf;
  ga.k_steps = H / kBK;
  ga.scale = int8 ? w->s_gu : nullptr;
  ga.scale_se = w->sgu_se;
  ga.scale_bf16 = w->s_dtype == MV_BF16;
  g1.n_tiles = H / kDownN;
  g1.k_steps = I / kBK;
  g1.scale = int8 ? w->s_d : nullptr;
  g1.scale_se = w->sd_se;
  g1.scale_bf16 = w->s_dtype == MV_BF16;
  {  // cooperative: every CTA resident, so a down tile's wait for its block's gate/up tiles always ends
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kGemmSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, gemm_kernel, tm_xs, tm_wgu, tm_a, tm_wd, ga, g1, ready);
    if (e != cudaSuccess) return cuda_status(e, "grouped GEMM launch");
  }
  if (out32 != nullptr) return MV_OK;
  const long long n4 = static_cast<long long>(N) * H / 4;
  long long blocks = (n4 + 255) / 256;
  if (blocks > G * 8) blocks = G * 8;
  finalize_kernel<<<static_cast<unsigned int>(blocks), 256, 0, st>>>(y32, n4, static_cast<uint16_t*>(out));
  return cuda_status(cudaGetLastError(), "finalize launch");
}

extern "C" int mv_moe_prefill(const mv_moe_weights* w, const void* x, long long x_stride, const void* ids,
                              int ids_dtype, const float* wts, int N, int NK, const void* residual,
                              long long residual_stride, void* out, void* workspace, size_t workspace_bytes,
                              void* stream) {
  if (out == nullptr && N > 0) return fail(MV_ERR_INVALID, "mv_moe_prefill: null pointer argument");
  return prefill_run(w, x, x_stride, ids, ids_dtype, wts, N, NK, residual, residual_stride, out, nullptr, workspace,
                     workspace_bytes, stream);
}

extern "C" int mv_moe_prefill_f32(const mv_moe_weights* w, const void* x, long long x_stride, int n_x,
                                  const void* x2, long long x2_stride, const void* ids, int ids_dtype, const float* wts,
                                  int N, int NK, const void* residual, long long residual_stride, float* out32,
                                  int max_ctas, void* workspace, size_t workspace_bytes, void* stream) {
  if (out32 == nullptr && N > 0) return fail(MV_ERR_INVALID, "mv_moe_prefill_f32: null pointer argument");
  if (max_ctas < 0 || n_x < 0 || n_x > N || (n_x < N && x2 == nullptr))
    return fail(MV_ERR_INVALID, "mv_moe_prefill_f32: bad max_ctas / n_x / second row source");
  return prefill_run(w, x, x_stride, ids, ids_dtype, wts, N, NK, residual, residual_stride, nullptr, out32, workspace,
                     workspace_bytes, stream, max_ctas, n_x, x2, x2_stride);
}
