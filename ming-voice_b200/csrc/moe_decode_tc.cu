// Decode MoE block (M <= 16 tokens, bf16 weights) on the 5th-generation tensor cores: one cooperative kernel.
//
// Same contract as the CUDA-core decode kernel (mv_moe_decode / mv_block_decode; reference fused_moe.py:14-83,
// engine.py:371-386); this path runs whenever the weights are bf16, H and I are multiples of 128, H <= 2048
// and the caller's workspace holds what it needs (decode_tc_workspace_bytes), else the CUDA-core kernel runs.
//
// Roles inside each CTA (one CTA per SM, 192 threads):
//   warp 0  TMA producer: streams 32 KB weight tiles (128 rows x 128 K, two 128-byte-swizzled atoms) into a
//           4-deep ring, never waiting for anything but free ring slots (and, once, the expert table and the
//           grid barrier before the down phase);
//   warp 1  MMA issuer (one thread): tcgen05.mma, M = 128 weight rows, N = 16 tokens (gate/up: A = weights,
//           B = the normalised tokens resident in shared memory) or N = 32 (down: B = hi/lo bf16 activations),
//           fp32 accumulators in TMEM (2 x 32 columns, double-buffered);
//   warps 2-5 epilogue: TMEM -> registers -> global partial sums; also the prologue's router and the table.
//
// Work split (every SM gets an equal share of the weight bytes; two sync-light sequences per phase):
//   gate/up  elements (slice z = (expert slot j, 128 rows of the intermediate dimension), 128-K block kb): the
//            gate tile and the up tile of slice z at kb. The shared-expert slots (no routing needed) form one
//            sequence, streamed while the router runs; the routed slots another. Each sequence is cut into G
//            equal contiguous ranges; a CTA accumulates its range slice by slice in TMEM. A slice inside one
//            range is finished at once; a slice cut by a range boundary leaves fp32 pieces, and the last piece
//            to arrive (per-slice arrival counter) adds them in CTA order. Then SiLU(gate) * up * routing weight
//            is stored as two bf16 rows (hi = bf16(v), lo = bf16(v - hi)), so the down projection sees ~16 bits.
//   grid barrier (all activations stored).
//   down     the same scheme over (128-row output slice hs, expert slot j, 128-K block kd) stages: a CTA's range
//            accumulates in TMEM (the expert sum happens inside the accumulator), and the last piece of a slice
//            adds the pieces in CTA order, the hi and lo columns and the residual, and stores bf16.
// Every sum has a fixed order, so results are deterministic. Every wait is bounded (errors in the workspace).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "decode_common.cuh"
#include "tc.cuh"

namespace mv {
namespace dtc {

using decode::Params;
using decode::kMaxE1;
using decode::kMaxM;
using decode::kMaxNK;
using decode::kTcMaxSeg;

constexpr int kThreads = 256;
constexpr int kEpi = 128;          // epilogue threads (warps 2..5)
constexpr int kRt = 64;            // router / table threads (warps 6..7)
constexpr int kStages = 4;
constexpr int kAStage = 32768;     // 128 rows x 128 K bf16
constexpr int kBTile = 8192;       // 32 rows x 128 K bf16 (down-phase B)
constexpr uint32_t kTmemCols = 64;
constexpr int kMaxH = 2048;
constexpr int kMaxPieces = 32;   // CTA ranges that can meet one slice (host-checked)
constexpr int kGuMaxSeg = 8;     // gate/up segments of one CTA in one sequence (host-checked)

struct SmemLayout {
  uint32_t ring, xb, bars, tmem, misc, e_id, e_ntok, e_pbase, e_tok, e_w, wd, bitmap, pr_e, pr_w, sel_r, sel_sc,
      total;
  __host__ __device__ SmemLayout(int H, int u_max, int M, int E_alloc, int top_k) {
    uint32_t o = 0;
    ring = o;
    o += kStages * kAStage;
    xb = o;
    const uint32_t xbb = static_cast<uint32_t>(H) * 32u;  // 16 token rows x H bf16
    o += ((xbb > static_cast<uint32_t>(kStages * kBTile) ? xbb : kStages * kBTile) + 1023u) & ~1023u;
    bars = o;
    o += (2 * kStages + 7) * 8;
    tmem = o;
    o += 16;
    misc = o;
    o += 16 * 4;
    e_id = o;
    o += u_max * 4;
    e_ntok = o;
    o += u_max * 4;
    e_pbase = o;
    o += u_max * 4;
    e_tok = o;
    o += u_max * kMaxM * 4;
    e_w = o;
    o += u_max * kMaxM * 4;
    wd = o;
    o += u_max * kMaxM * 4;
    bitmap = o;
    o += (kMaxE1 / 32) * 4;
    pr_e = o;
    o += kMaxM * kMaxNK * 4;
    pr_w = o;
    o += kMaxM * kMaxNK * 4;
    sel_r = o;
    o += M * E_alloc * 4;
    sel_sc = o;
    o += M * E_alloc * 4;
    total = o;
    (void)top_k;
  }
};

// Pieces of one slice: the CTAs b (in order) whose contiguous range [T*b/G, T*(b+1)/G) of a sequence of T
// elements meets [A, A + Lseg); b wrote its piece to slot (b * nseq + seq) * maxseg + (index of the slice
// among the slices that b's range touches).
__device__ __forceinline__ int first_piece_cta(long long T, long long A, int G) {
  int b0 = static_cast<int>(A * G / T) - 1;
  if (b0 < 0) b0 = 0;
  while (b0 > 0 && T * b0 / G > A) --b0;
  return b0;
}

__device__ __forceinline__ bool meets(long long T, int b, int G, long long A, long long B) {
  const long long lo = T * b / G, hi = T * (b + 1) / G;
  return hi > lo && (lo > A ? lo : A) < (hi < B ? hi : B);
}

__device__ __forceinline__ int count_pieces(long long T, long long A, long long Lseg, int G) {
  int np = 0;
  for (int b = first_piece_cta(T, A, G); b < G && T * b / G < A + Lseg; ++b) np += meets(T, b, G, A, A + Lseg);
  return np;
}

template <typename F>
__device__ __forceinline__ void for_each_piece(long long T, long long A, long long Lseg, int G, int nseq, int seq,
                                               int maxseg, F f) {
  for (int b = first_piece_cta(T, A, G); b < G && T * b / G < A + Lseg; ++b)
    if (meets(T, b, G, A, A + Lseg))
      f((b * nseq + seq) * maxseg + static_cast<int>(A / Lseg - (T * b / G) / Lseg));
}

// byte offset of the 16-byte chunk c (elements 8c..8c+7) of token row t in the swizzled B layout
__device__ __forceinline__ uint32_t xb_off(int t, int c) {
  return static_cast<uint32_t>((c >> 3) * 2048 + t * 128 + (((c & 7) ^ (t & 7)) << 4));
}

__device__ __forceinline__ float ldcg(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}


// The router warps read their expert rows at kernel entry, into registers (16-byte chunks c = lane + 32 i of
// the row), and compute the logits once the tokens are normalised.
constexpr int kRouterChunks = kMaxH * 4 / 16 / 32;  // chunks per lane of an fp32 row at H = kMaxH

__device__ __forceinline__ void router_row_load(const void* w_row, int row_bytes, uint4 (&buf)[kRouterChunks]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < kRouterChunks; ++i) {
    const int c = lane + 32 * i;
    if (c * 16 < row_bytes) buf[i] = ld_nc_v4(static_cast<const uint8_t*>(w_row) + static_cast<size_t>(c) * 16);
  }
}

// fp64 router logits of one expert row (loaded by router_row_load) against the (swizzled) normalised tokens;
// one warp.
template <int DT>
__device__ void router_logits_sw(const uint4 (&buf)[kRouterChunks], float sc, const uint8_t* xb, int H, int M,
                                 double (&acc)[kMaxM]) {
  const int lane = threadIdx.x & 31;
  constexpr int per = DT == MV_F32 ? 4 : (DT == MV_BF16 ? 8 : 16);
  constexpr int kMaxCh = kMaxH / per / 32;  // chunks per lane at H = kMaxH
  const int nch = H / per;
#pragma unroll
  for (int i = 0; i < kMaxCh; ++i) {
    const int c = lane + 32 * i;
    if (c >= nch) break;
    const uint32_t ww[4] = {buf[i].x, buf[i].y, buf[i].z, buf[i].w};
    float wf[per];
    if constexpr (DT == MV_F32) {
#pragma unroll
      for (int q = 0; q < 4; ++q) wf[q] = __uint_as_float(ww[q]);
    } else if constexpr (DT == MV_BF16) {
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
        wf[4 * q] = dequant(f0, sc);
        wf[4 * q + 1] = dequant(f1, sc);
        wf[4 * q + 2] = dequant(f2, sc);
        wf[4 * q + 3] = dequant(f3, sc);
      }
    }
    const int k0 = c * per;
#pragma unroll
    for (int t = 0; t < kMaxM; ++t) {
      if (t >= M) break;
#pragma unroll
      for (int v = 0; v < per; v += 2) {
        const int k = k0 + v;
        const uint32_t xx = *reinterpret_cast<const uint32_t*>(xb + xb_off(t, k >> 3) + (k & 7) * 2);
        acc[t] += static_cast<double>(wf[v]) * static_cast<double>(bf16lo(xx));
        acc[t] += static_cast<double>(wf[v + 1]) * static_cast<double>(bf16hi(xx));
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    moe_decode_tc_kernel(const Params p, const __grid_constant__ CUtensorMap tm_gu,
                         const __grid_constant__ CUtensorMap tm_d, const __grid_constant__ CUtensorMap tm_ab) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SmemLayout Ls(p.H, p.u_max, p.M, p.E_alloc, p.top_k);
  uint8_t* ring = sm + Ls.ring;
  uint8_t* xb = sm + Ls.xb;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Ls.bars);
  uint64_t* empty = full + kStages;
  uint64_t* accf = empty + kStages;
  uint64_t* acce = accf + 2;
  uint64_t* tbl = acce + 2;
  uint64_t* done = tbl + 1;
  uint64_t* rdy = done + 1;  // this CTA's router logits are computed (its weight stream may start)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Ls.tmem);
  int* misc = reinterpret_cast<int*>(sm + Ls.misc);
  int* e_id = reinterpret_cast<int*>(sm + Ls.e_id);
  int* e_ntok = reinterpret_cast<int*>(sm + Ls.e_ntok);
  int* e_pbase = reinterpret_cast<int*>(sm + Ls.e_pbase);
  int* e_tok = reinterpret_cast<int*>(sm + Ls.e_tok);
  float* e_w = reinterpret_cast<float*>(sm + Ls.e_w);
  float* wd = reinterpret_cast<float*>(sm + Ls.wd);
  unsigned int* bitmap = reinterpret_cast<unsigned int*>(sm + Ls.bitmap);
  int* pr_e = reinterpret_cast<int*>(sm + Ls.pr_e);
  float* pr_w = reinterpret_cast<float*>(sm + Ls.pr_w);
  float* sel_r = reinterpret_cast<float*>(sm + Ls.sel_r);
  float* sel_sc = reinterpret_cast<float*>(sm + Ls.sel_sc);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, H = p.H, I = p.I, M = p.M;
  const int S = I / 128, KB = H / 128, KD = I / 128, HS = H / 128;
  const int n_static = p.router ? p.n_static : 0;
  const long long T_s = static_cast<long long>(n_static) * S * KB;  // static gate/up elements
  int* cnt_gu = p.tc_cnt;
  int* cnt_d = p.tc_cnt + p.u_max * S * 4;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], kEpi);
    }
    mbar_init(tbl, 1);
    mbar_init(done, 1);
    mbar_init(rdy, 1);
    fence_mbar_init();
    misc[1] = 0;
    misc[2] = 0;
  }
  pdl_launch_dependents();  // the next kernel in the stream may be scheduled (it waits for this one)
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tm_gu);
    tc::prefetch_tmap(&tm_d);
    tc::prefetch_tmap(&tm_ab);
  }
  // the routing path's reads start first: the norm weights (into L2) and the router warps' expert rows (into
  // registers; warp 6 + w computes expert 2 * CTA + w)
  if (warp == 6 && lane == 0 && p.norm_w != nullptr) bulk_prefetch_l2(p.norm_w, static_cast<uint32_t>(H) * 2u);
  const int r_e = blockIdx.x * 2 + (warp - 6);
  const bool r_has = warp >= 6 && p.router && r_e < p.E;
  const int r_esz = p.rw_dtype == MV_F32 ? 4 : (p.rw_dtype == MV_BF16 ? 2 : 1);
  uint4 r_row[kRouterChunks];
  if (r_has) router_row_load(static_cast<const uint8_t*>(p.rw) + static_cast<size_t>(r_e) * H * r_esz, H * r_esz, r_row);
  // the tokens, the workspace and (on this SM) the tensor memory are the previous kernel's until it completes
  pdl_wait();
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }

  // ---------------------------------------------------------------- prologue: tokens -> swizzled B (all threads)
  {
    const int nch = H / 8;  // 16-byte chunks per token row
    for (int i = tid; i < (kMaxM - M) * nch; i += kThreads) {
      const int t = M + i / nch, c = i % nch;
      *reinterpret_cast<uint4*>(xb + xb_off(t, c)) = make_uint4(0, 0, 0, 0);
    }
    // every token's chunks in flight together (8 loads per thread before any store)
    const int tot = M * nch;
    for (int i0 = tid; i0 < tot; i0 += 8 * kThreads) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * kThreads;
        if (i < tot) v[u] = reinterpret_cast<const uint4*>(p.x + (i / nch) * p.x_stride)[i % nch];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * kThreads;
        if (i < tot) *reinterpret_cast<uint4*>(xb + xb_off(i / nch, i % nch)) = v[u];
      }
    }
    if (p.norm_w != nullptr) {  // one warp per token: fp64 sum of squares (exact), then the normalisation
      __syncthreads();
      const uint4* gw = reinterpret_cast<const uint4*>(p.norm_w);
      for (int m = warp; m < M; m += kThreads / 32) {
        uint4 gpre[kMaxH / 256];  // this lane's norm-weight chunks, in flight during the sum
#pragma unroll
        for (int i = 0; i < kMaxH / 256; ++i)
          if (lane + 32 * i < nch) gpre[i] = gw[lane + 32 * i];
        double ss = 0.0;
        for (int c = lane; c < nch; c += 32) {
          const uint4 v = *reinterpret_cast<const uint4*>(xb + xb_off(m, c));
          const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const double a = bf16lo(vv[q]), b = bf16hi(vv[q]);
            ss += a * a + b * b;
          }
        }
        ss = warp_sum_d(ss);
        const float var = static_cast<float>(ss / static_cast<double>(H));
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
#pragma unroll
        for (int i = 0; i < kMaxH / 256; ++i) {
          const int c = lane + 32 * i;
          if (c >= nch) break;
          uint4* dst = reinterpret_cast<uint4*>(xb + xb_off(m, c));
          const uint4 v = *dst;
          const uint4 g = gpre[i];
          const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
          const uint32_t gg[4] = {g.x, g.y, g.z, g.w};
          uint32_t o[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float y0 = round_bf16(__fmul_rn(bf16lo(vv[q]), r));
            const float y1 = round_bf16(__fmul_rn(bf16hi(vv[q]), r));
            o[q] = static_cast<uint32_t>(f2bf(__fmul_rn(bf16lo(gg[q]), y0))) |
                   (static_cast<uint32_t>(f2bf(__fmul_rn(bf16hi(gg[q]), y1))) << 16);
          }
          *dst = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  fence_proxy_async_smem();  // the tensor core reads xb through the async proxy
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  // down-phase range of this CTA (needs U: computed after the table)
  auto d_range = [&](int U, long long& L, long long& QT, long long& q_lo, long long& q_hi) {
    L = static_cast<long long>(U) * KD;
    QT = HS * L;
    q_lo = QT * blockIdx.x / G;
    q_hi = QT * (blockIdx.x + 1) / G;
  };
  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint64_t pol = policy_evict_first();  // weights are read once per call: keep L2 for the rest
      int used[kStages];       // slot issued at least once
      uint32_t last[kStages];  // parity of its last issue
      for (int s = 0; s < kStages; ++s) used[s] = 0;
      auto acquire = [&]() -> int {
        if (ok) ok = mbar_wait(&empty[stage], ph ^ 1u, p.ws, 0x600u | stage);
        const int s = stage;
        used[s] = 1;
        last[s] = ph;
        if (++stage == kStages) {
          stage = 0;
          ph ^= 1u;
        }
        return s;
      };
      // gate/up: this CTA's contiguous range of the (slice z, k-block) sequence; one element = the gate tile
      // and the up tile of slice z at k-block kb
      auto gu_range = [&](long long T, int zbase, bool is_static) {
        const long long lo = T * blockIdx.x / G, hi = T * (blockIdx.x + 1) / G;
        for (long long q = lo; q < hi && ok; ++q) {
          const int z = zbase + static_cast<int>(q / KB), kb = static_cast<int>(q % KB);
          const int j = z / S, sl = z % S;
          const int e = is_static ? p.static_id + j : e_id[j];
          for (int half = 0; half < 2 && ok; ++half) {
            const int st = acquire();
            if (!ok) return;
            uint8_t* dst = ring + st * kAStage;
            const int row = half * I + sl * 128;
            mbar_arrive_expect_tx(&full[st], kAStage);
            tc::tma_load_3d_hint(dst, &tm_gu, &full[st], kb * 128, row, e, pol);
            tc::tma_load_3d_hint(dst + 16384, &tm_gu, &full[st], kb * 128 + 64, row, e, pol);
          }
        }
      };
      // a CTA computing router logits starts its weight stream after them: the tensor core's shared-memory reads
      // slow the router warps' fp64 dot products several-fold, and the routing decision is the critical path
      if (ok) ok = mbar_wait_lazy(rdy, 0u, p.ws, 0x608u, 256);
      gu_range(T_s, 0, true);
      if (ok) ok = mbar_wait_lazy(tbl, 0u, p.ws, 0x610u, 1024);
      const int U = misc[0];
      gu_range(static_cast<long long>(U - n_static) * S * KB, n_static * S, false);
      long long L, QT, q_lo, q_hi;
      d_range(U, L, QT, q_lo, q_hi);
      auto d_a = [&](long long q, int st) {
        const int hs = static_cast<int>(q / L);
        const int rem = static_cast<int>(q - static_cast<long long>(hs) * L);
        const int j = rem / KD, kd = rem % KD;
        uint8_t* dst = ring + st * kAStage;
        tc::tma_load_3d_hint(dst, &tm_d, &full[st], kd * 128, hs * 128, e_id[j], pol);
        tc::tma_load_3d_hint(dst + 16384, &tm_d, &full[st], kd * 128 + 64, hs * 128, e_id[j], pol);
      };
      auto d_b = [&](long long q, int st) {
        const int rem = static_cast<int>(q % L);
        const int j = rem / KD, kd = rem % KD;
        uint8_t* dst = xb + st * kBTile;
        tc::tma_load_2d(dst, &tm_ab, &full[st], kd * 128, j * 32);
        tc::tma_load_2d(dst + 4096, &tm_ab, &full[st], kd * 128 + 64, j * 32);
      };
      // weight tiles of the first stages run ahead of the grid barrier; their activation tiles follow it
      const long long pre_end = q_lo + kStages < q_hi ? q_lo + kStages : q_hi;
      int pre_slot[kStages];
      int n_pre = 0;
      for (long long q = q_lo; q < pre_end && ok; ++q) {
        const int st = acquire();
        if (!ok) break;
        pre_slot[n_pre++] = st;
        mbar_arrive_expect_tx(&full[st], kAStage + kBTile);
        d_a(q, st);
      }
      const bool bar_ok = grid_wait(&p.ws->bar2, G, p.ws, 0x620u);
      fence_proxy_async_global();
      // the activation tiles of the stages already started are always issued, so every started stage completes
      for (int i = 0; i < n_pre; ++i) d_b(q_lo + i, pre_slot[i]);
      ok = ok && bar_ok;
      for (long long q = pre_end; q < q_hi && ok; ++q) {
        const int st = acquire();
        if (!ok) break;
        mbar_arrive_expect_tx(&full[st], kAStage + kBTile);
        d_a(q, st);
        d_b(q, st);
      }
      // copies in flight land before the CTA exits (immediate when the MMA warp consumed them)
      for (int s = 0; s < kStages; ++s)
        if (used[s]) mbar_wait(&full[s], last[s], p.ws, 0x630u);
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_gu = tc::idesc_bf16_f32(128, 16);
      constexpr uint32_t id_d = tc::idesc_bf16_f32(128, 32);
      int stage = 0, acc_i = 0;
      uint32_t ph = 0;
      bool ok = true;
      auto take = [&](int& buf) -> bool {
        buf = acc_i & 1;
        const uint32_t aph = static_cast<uint32_t>(acc_i >> 1) & 1u;
        ++acc_i;
        if (ok) ok = mbar_wait(&acce[buf], aph ^ 1u, p.ws, 0x640u);
        if (ok) tc::fence_after_sync();
        return ok;
      };
      auto next_full = [&]() -> int {
        if (ok) ok = mbar_wait(&full[stage], ph, p.ws, 0x650u | stage);
        if (ok) tc::fence_after_sync();
        const int s = stage;
        if (++stage == kStages) {
          stage = 0;
          ph ^= 1u;
        }
        return s;
      };
      const uint32_t xb_a = smem_u32(xb);
      auto gu_range = [&](long long T) {
        const long long lo = T * blockIdx.x / G, hi = T * (blockIdx.x + 1) / G;
        for (long long q = lo; q < hi && ok;) {
          const long long seg_end = (q / KB + 1) * KB < hi ? (q / KB + 1) * KB : hi;
          int buf;
          if (!take(buf)) break;
          for (long long q0 = q; q < seg_end && ok; ++q) {
            const int kb = static_cast<int>(q % KB);
            for (int half = 0; half < 2 && ok; ++half) {
              const uint32_t d = tmem + static_cast<uint32_t>(buf * 32 + half * 16);
              const int st = next_full();
              if (!ok) break;
              const uint64_t ad = tc::sw128_desc(smem_u32(ring + st * kAStage));
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                const uint64_t a = ad + (kk >> 2) * (16384 >> 4) + (kk & 3) * 2;
                const uint64_t b = tc::sw128_desc(xb_a + (kb * 2 + (kk >> 2)) * 2048) + (kk & 3) * 2;
                tc::mma_bf16(d, a, b, id_gu, (q != q0 || kk != 0) ? 1u : 0u);
              }
              tc::mma_commit(&empty[st]);
            }
          }
          if (ok) tc::mma_commit(&accf[buf]);
        }
      };
      gu_range(T_s);
      if (ok) ok = mbar_wait_lazy(tbl, 0u, p.ws, 0x660u, 1024);
      const int U = misc[0];
      gu_range(static_cast<long long>(U - n_static) * S * KB);
      long long L, QT, q_lo, q_hi;
      d_range(U, L, QT, q_lo, q_hi);
      for (long long q = q_lo; q < q_hi && ok;) {
        const long long seg_end = (q / L + 1) * L < q_hi ? (q / L + 1) * L : q_hi;
        int buf;
        if (!take(buf)) break;
        const uint32_t d = tmem + static_cast<uint32_t>(buf * 32);
        for (long long q0 = q; q < seg_end && ok; ++q) {
          const int st = next_full();
          if (!ok) break;
          const uint64_t ad = tc::sw128_desc(smem_u32(ring + st * kAStage));
          const uint64_t bd = tc::sw128_desc(xb_a + st * kBTile);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t a = ad + (kk >> 2) * (16384 >> 4) + (kk & 3) * 2;
            const uint64_t b = bd + (kk >> 2) * (4096 >> 4) + (kk & 3) * 2;
            tc::mma_bf16(d, a, b, id_d, (q != q0 || kk != 0) ? 1u : 0u);
          }
          tc::mma_commit(&empty[st]);
        }
        if (ok) tc::mma_commit(&accf[buf]);
      }
      // every issued MMA retires before the TMEM is released
      tc::mma_commit(done);
      mbar_wait_lazy(done, 0u, p.ws, 0x670u, 256);
    }
  } else if (warp >= 6) {
    // ================================================================ router / table (warps 6..7)
    const int rt = tid - 192;
    auto rbar = [] { named_bar(2, kRt); };
    if (!p.router && rt == 0) mbar_arrive(rdy);  // no logits to compute: the weight stream starts at once
    if (p.router) {
      const int e = r_e;
      if (r_has) {
        double acc[kMaxM];
#pragma unroll
        for (int m = 0; m < kMaxM; ++m) acc[m] = 0.0;
        if (p.rw_dtype == MV_F32)
          router_logits_sw<MV_F32>(r_row, 1.0f, xb, H, M, acc);
        else if (p.rw_dtype == MV_BF16)
          router_logits_sw<MV_BF16>(r_row, 1.0f, xb, H, M, acc);
        else
          router_logits_sw<MV_I8>(r_row, decode::ldscale(p.rw_scale, e, p.rw_scale_bf16), xb, H, M, acc);
#pragma unroll
        for (int m = 0; m < kMaxM; ++m) {
          if (m < M) {
            const double v = warp_sum_d(acc[m]);
            if (lane == 0) p.logits_ws[m * p.E + e] = static_cast<float>(v);
          }
        }
      }
      rbar();
      if (rt == 0) mbar_arrive(rdy);
      if (rt == 0) grid_arrive(&p.ws->bar1);
      if (rt == 0) grid_wait(&p.ws->bar1, G, p.ws, 0x680u);
      rbar();
      // one warp per token: the logits (published by other CTAs: read through L2) into shared memory, then
      // the selection (largest first, ties to the lower id) and the weights
      for (int i = rt; i < M * p.E; i += kRt) sel_r[i] = ld_cg_f32(p.logits_ws + i);
      rbar();
      const route::SelectCfg cfg{p.route_mode, p.E, p.top_k, p.n_group, p.topk_group, p.rscale, p.rbias};
      for (int t = warp - 6; t < M; t += kRt / 32)
        route::select_core(cfg, sel_r + t * p.E, sel_sc + t * p.E, pr_e + t * p.top_k, pr_w + t * p.top_k);
      rbar();
      if (blockIdx.x == 0) {  // router outputs: ids / weights with the static slots appended, logits
        const int NKT = p.top_k + n_static;
        for (int j = rt; j < M * NKT; j += kRt) {
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
          for (int j = rt; j < M * p.E; j += kRt) p.logits_out[j] = ld_cg_f32(p.logits_ws + j);
      }
      const int npairs = M * p.top_k;
      if (npairs <= 32) {
        if (warp == 6)
          decode::table_warp<kMaxM>(pr_e, pr_w, npairs, p.top_k, p.E1, n_static, p.static_id, M, e_id, e_ntok, e_tok,
                                    e_w, e_pbase, misc, p.ws);
      } else {
        decode::table_bitmap<kMaxM>(pr_e, pr_w, npairs, p.top_k, p.E1, n_static, p.static_id, M, e_id, e_ntok, e_tok,
                                    e_w, e_pbase, misc, bitmap, p.ws, rt, kRt, rbar);
      }
    } else {
      const int npairs = M * p.NK;
      for (int j = rt; j < npairs; j += kRt) {
        const long long e = p.ids_i64 ? reinterpret_cast<const long long*>(p.ids)[j]
                                      : static_cast<long long>(reinterpret_cast<const int*>(p.ids)[j]);
        const bool valid = e >= 0 && e < p.E1;
        pr_e[j] = valid ? static_cast<int>(e) : -1;
        pr_w[j] = p.wts[j];
        if (!valid && e != -1) raise_error(p.ws, kErrBadExpert, static_cast<unsigned int>(j));  // -1: no pair
      }
      rbar();
      if (npairs <= 32) {
        if (warp == 6)
          decode::table_warp<kMaxM>(pr_e, pr_w, npairs, p.NK, p.E1, 0, 0, M, e_id, e_ntok, e_tok, e_w, e_pbase, misc,
                                    p.ws);
      } else {
        decode::table_bitmap<kMaxM>(pr_e, pr_w, npairs, p.NK, p.E1, 0, 0, M, e_id, e_ntok, e_tok, e_w, e_pbase, misc,
                                    bitmap, p.ws, rt, kRt, rbar);
      }
    }
    rbar();
    const int U = misc[0];
    for (int i = rt; i < U * kMaxM; i += kRt) wd[i] = 0.f;
    rbar();
    for (int j = rt; j < U; j += kRt)
      for (int i = 0; i < e_ntok[j]; ++i) wd[j * kMaxM + e_tok[j * kMaxM + i]] = e_w[j * kMaxM + i];
    rbar();
    if (rt == 0) mbar_arrive(tbl);  // producer, MMA and epilogue warps may read the table now
  } else {
    // ================================================================ epilogue (warps 2..5)
    // Every epilogue warp works on its own 32 TMEM lanes (rows) and its own arrival counters: no CTA-wide
    // barrier inside the loops, so the warps never wait for one another.
    const int et = tid - 64;
    const int g4 = warp & 3;
    const int row = g4 * 32 + lane;
    bool ok = true;
    bool cnt_ready = false;  // the counter-clearing grid barrier has been seen by this warp
    auto counters_ready = [&]() {
      if (!cnt_ready) {
        bool good = true;
        if (lane == 0) good = grid_wait(&p.ws->pad[0], G, p.ws, 0x6a0u);
        ok = ok && __shfl_sync(0xffffffffu, good, 0) != 0;
        cnt_ready = true;
      }
    };
    int acc_i = 0;
    auto take = [&](int& buf) -> bool {
      buf = acc_i & 1;
      const uint32_t aph = static_cast<uint32_t>(acc_i >> 1) & 1u;
      ++acc_i;
      ok = __all_sync(0xffffffffu, ok && mbar_wait_lazy(&accf[buf], aph, p.ws, 0x690u, 256));
      if (ok) tc::fence_after_sync();
      return ok;
    };
    // the arrival counters start from zero in every call (the workspace may hold anything: another call's
    // layout, or the CUDA-core kernel's data): each CTA clears a share, then a grid barrier publishes it. The
    // epilogue warps do it while their first accumulator fills, off the routing path.
    {
      const int ncnt = (p.u_max * S + HS) * 4;
      for (int i = blockIdx.x * kEpi + et; i < ncnt; i += G * kEpi) p.tc_cnt[i] = 0;
      __threadfence();
      named_bar(3, kEpi);
      if (et == 0) grid_arrive(&p.ws->pad[0]);
    }
    const uint32_t tlane = static_cast<uint32_t>(g4 * 32) << 16;
    // SiLU(g) * u * weight as hi / lo bf16 rows of the activation buffer (static slots carry weight 1)
    auto finalize = [&](int j, int sl, const float* g, const float* u) {
      uint16_t* ab = p.tc_abuf + static_cast<long long>(j) * 32 * I + sl * 128 + row;
#pragma unroll
      for (int t = 0; t < kMaxM; ++t) {
        if (t >= M) break;
        const float w = j < n_static ? 1.0f : wd[j * kMaxM + t];
        const float a = g[t] / (1.0f + __expf(-g[t])) * u[t] * w;
        const uint16_t hi = f2bf(a);
        const uint16_t lo = f2bf(a - __uint_as_float(static_cast<uint32_t>(hi) << 16));
        ab[static_cast<long long>(t) * I] = hi;
        ab[static_cast<long long>(16 + t) * I] = lo;
      }
    };
    // one gate/up segment of this CTA's range: a whole slice finalizes at once; a part of a slice writes its
    // partial sums, and the last of the slice's pieces to arrive adds them in CTA order and finalizes
    auto gu_range = [&](long long T, int zbase, int seq) {
      const long long lo = T * blockIdx.x / G, hi = T * (blockIdx.x + 1) / G;
      int seg = 0;
      for (long long q = lo; q < hi && ok; ++seg) {
        const int zl = static_cast<int>(q / KB);
        const long long zs = static_cast<long long>(zl) * KB;
        const long long seg_end = zs + KB < hi ? zs + KB : hi;
        const bool whole = q == zs && seg_end == zs + KB;
        q = seg_end;
        int buf;
        if (!take(buf)) break;
        uint32_t gr[16], ur[16];
        tc::tmem_ld16(tmem + tlane + static_cast<uint32_t>(buf * 32), gr);
        tc::tmem_ld16(tmem + tlane + static_cast<uint32_t>(buf * 32 + 16), ur);
        tc::tmem_ld_wait();
        tc::fence_before_sync();
        mbar_arrive(&acce[buf]);
        float g[kMaxM], u[kMaxM];
#pragma unroll
        for (int t = 0; t < kMaxM; ++t) {
          g[t] = __uint_as_float(gr[t]);
          u[t] = __uint_as_float(ur[t]);
        }
        const int z = zbase + zl, j = z / S, sl = z % S;
        if (whole) {
          finalize(j, sl, g, u);
          continue;
        }
        float* pg = p.tc_part_gu + (static_cast<long long>(blockIdx.x * 2 + seq) * kGuMaxSeg + seg) * 2 * M * 128;
#pragma unroll
        for (int t = 0; t < kMaxM; ++t) {
          if (t >= M) break;
          pg[t * 128 + row] = g[t];
          pg[(M + t) * 128 + row] = u[t];
        }
        __threadfence();
        __syncwarp();
        counters_ready();
        if (!ok) break;
        const int np = count_pieces(T, zs, KB, G);
        int last = 0;
        if (lane == 0) last = atomicAdd(&cnt_gu[z * 4 + g4], 1) == np - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {  // this warp's 32 rows of the slice: add the pieces in CTA order (a piece's loads in flight together)
          __threadfence();
#pragma unroll
          for (int t = 0; t < kMaxM; ++t) g[t] = u[t] = 0.f;
          for_each_piece(T, zs, KB, G, 2, seq, kGuMaxSeg, [&](int slot) {
            const float* pk = p.tc_part_gu + static_cast<long long>(slot) * 2 * M * 128;
            float lg[kMaxM], lu[kMaxM];
#pragma unroll
            for (int t = 0; t < kMaxM; ++t)
              if (t < M) {
                lg[t] = ldcg(pk + t * 128 + row);
                lu[t] = ldcg(pk + (M + t) * 128 + row);
              }
#pragma unroll
            for (int t = 0; t < kMaxM; ++t)
              if (t < M) {
                g[t] += lg[t];
                u[t] += lu[t];
              }
          });
          finalize(j, sl, g, u);
        }
      }
    };
    gu_range(T_s, 0, 0);
    ok = __all_sync(0xffffffffu, ok && mbar_wait_lazy(tbl, 0u, p.ws, 0x6b0u, 1024));
    const int U = misc[0];
    gu_range(static_cast<long long>(U - n_static) * S * KB, n_static * S, 1);
    counters_ready();  // (the down phase uses counters too)
    // all activations of this CTA are stored: arrive on the grid barrier of the down phase
    fence_proxy_async_global();
    __threadfence();
    named_bar(1, kEpi);
    if (et == 0) grid_arrive(&p.ws->bar2);

    long long L, QT, q_lo, q_hi;
    d_range(U, L, QT, q_lo, q_hi);
    for (long long q = q_lo; q < q_hi && ok;) {
      const int hs = static_cast<int>(q / L);
      const long long seg_end = (q / L + 1) * L < q_hi ? (q / L + 1) * L : q_hi;
      q = seg_end;
      int buf;
      if (!take(buf)) break;
      uint32_t v[32];
      tc::tmem_ld32(tmem + tlane + static_cast<uint32_t>(buf * 32), v);
      tc::tmem_ld_wait();
      tc::fence_before_sync();
      mbar_arrive(&acce[buf]);
      const int slot = blockIdx.x * kTcMaxSeg + (hs - static_cast<int>(q_lo / L));
      float* pd = p.tc_part_d + static_cast<long long>(slot) * M * 128;
#pragma unroll
      for (int t = 0; t < kMaxM; ++t)
        if (t < M) pd[t * 128 + row] = __uint_as_float(v[t]) + __uint_as_float(v[16 + t]);
      __threadfence();
      __syncwarp();
      // the CTAs whose ranges meet slice hs, in order; the last to arrive adds their pieces
      const long long A = static_cast<long long>(hs) * L;
      const int np = count_pieces(QT, A, L, G);
      int* cnt = &cnt_d[hs * 4 + g4];
      int last = 0;
      if (lane == 0) last = atomicAdd(cnt, 1) == np - 1;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence();
        float y[kMaxM];
#pragma unroll
        for (int t = 0; t < kMaxM; ++t) y[t] = 0.f;
        for_each_piece(QT, A, L, G, 1, 0, kTcMaxSeg, [&](int pslot) {
          const float* pb = p.tc_part_d + static_cast<long long>(pslot) * M * 128;
          float lv[kMaxM];
#pragma unroll
          for (int t = 0; t < kMaxM; ++t)
            if (t < M) lv[t] = ldcg(pb + t * 128 + row);
#pragma unroll
          for (int t = 0; t < kMaxM; ++t)
            if (t < M) y[t] += lv[t];
        });
        const int col = hs * 128 + row;
#pragma unroll
        for (int t = 0; t < kMaxM; ++t) {
          if (t >= M) break;
          float o = y[t];
          if (p.residual != nullptr) o += __uint_as_float(static_cast<uint32_t>(p.residual[t * H + col]) << 16);
          p.out[t * H + col] = f2bf(o);
        }
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
  // (an epilogue thread, not thread 0: thread 0 is the TMA producer, and its fence would wait on its bulk copies)
  if (tid == 64) {  // the last CTA resets the grid-barrier counters for the next call
    __threadfence();
    if (atomicAdd(&p.ws->counter, 1u) == static_cast<unsigned int>(G - 1)) {
      atomicExch(&p.ws->bar1, 0u);
      atomicExch(&p.ws->bar2, 0u);
      atomicExch(&p.ws->pad[0], 0u);
      atomicExch(&p.ws->counter, 0u);
    }
  }
}

// ------------------------------------------------------------------------------------------------ host

struct WsLayout {
  size_t logits, cnt, part_gu, part_d, abuf, total;
};

static size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

static WsLayout ws_layout(int M, int u_max, int n_static, int u_r_max, int H, int I, int E, int G) {
  WsLayout L{};
  const int S = I / 128, HS = H / 128;
  (void)n_static;
  (void)u_r_max;
  size_t o = kWsHeaderBytes;
  L.logits = o;
  o = up256(o + static_cast<size_t>(M) * (E > 0 ? E : 1) * 4);
  L.cnt = o;
  o = up256(o + static_cast<size_t>(u_max * S + HS) * 4 * 4);
  L.part_gu = o;
  o = up256(o + static_cast<size_t>(G) * 2 * kGuMaxSeg * 2 * M * 128 * 4);
  L.part_d = o;
  o = up256(o + static_cast<size_t>(G) * kTcMaxSeg * M * 128 * 4);
  L.abuf = o;
  o = up256(o + static_cast<size_t>(u_max) * 32 * I * 2);
  L.total = o;
  return L;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

static bool tmap(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                 const uint32_t* box) {
  auto enc = encode_fn();
  if (enc == nullptr) return false;
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
             reinterpret_cast<const cuuint64_t*>(dims), reinterpret_cast<const cuuint64_t*>(strides),
             reinterpret_cast<const cuuint32_t*>(box), estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace dtc

static bool tc_shapes_ok(int H, int I) { return H % 128 == 0 && I % 128 == 0 && H <= dtc::kMaxH && H >= 128; }

size_t decode_tc_workspace_bytes(int M, int nk, int H, int I, int E1, int E, int n_static) {
  if (!tc_shapes_ok(H, I) || M < 1 || M > decode::kMaxM || nk < 1) return 0;
  const int routed = E > 0 ? nk - n_static : nk;  // experts chosen per token by the router (or given)
  int u_r_max = M * (routed > 0 ? routed : 1);
  const int pool = E > 0 ? E : E1;
  if (u_r_max > pool) u_r_max = pool;
  const int ns = E > 0 ? n_static : 0;
  const int u_max = ns + u_r_max;
  return dtc::ws_layout(M, u_max, ns, u_r_max, H, I, E, num_sms()).total;
}

int decode_tc_run(decode::Params& p, void* workspace, size_t workspace_bytes, int nk_pairs, cudaStream_t st) {
  using namespace dtc;
  const int H = p.H, I = p.I, M = p.M, G = num_sms();
  if (!tc_shapes_ok(H, I) || p.w_gu == nullptr) return kDecodeTcUnsuitable;
  const int n_static = p.router ? p.n_static : 0;
  const int routed = p.router ? p.top_k : nk_pairs;
  int u_r_max = M * routed;
  const int pool = p.router ? p.E : p.E1;
  if (u_r_max > pool) u_r_max = pool;
  const int u_max = n_static + u_r_max;
  const WsLayout L = ws_layout(M, u_max, n_static, u_r_max, H, I, p.router ? p.E : 0, G);
  if (workspace_bytes < L.total) return kDecodeTcUnsuitable;
  if ((H / 128 + G - 1) / G + 1 > decode::kTcMaxSeg) return kDecodeTcUnsuitable;
  if ((G + H / 128 - 1) / (H / 128) + 2 > kMaxPieces) return kDecodeTcUnsuitable;
  {  // gate/up: segments per CTA and pieces per slice within their bounds
    const long long KB = H / 128, S = I / 128;
    const long long T_max = static_cast<long long>(u_r_max > n_static ? u_r_max : n_static) * S * KB;
    if ((T_max + G - 1) / G / KB + 2 > kGuMaxSeg || KB + 2 > kMaxPieces) return kDecodeTcUnsuitable;
  }
  const int E_alloc = p.router ? p.E : 0;
  const SmemLayout Ls(H, u_max, M, E_alloc, p.router ? p.top_k : 1);
  const size_t smem = Ls.total + 1024;
  if (smem > 227 * 1024) return kDecodeTcUnsuitable;

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.ws = reinterpret_cast<WsHeader*>(ws);
  p.logits_ws = reinterpret_cast<float*>(ws + L.logits);
  p.tc_cnt = reinterpret_cast<int*>(ws + L.cnt);
  p.tc_part_gu = reinterpret_cast<float*>(ws + L.part_gu);
  p.tc_part_d = reinterpret_cast<float*>(ws + L.part_d);
  p.tc_abuf = reinterpret_cast<uint16_t*>(ws + L.abuf);
  p.u_max = u_max;
  p.E_alloc = E_alloc;
  if (!p.router) p.top_k = 1;  // selection scratch sizing only

  CUtensorMap tm_gu, tm_d, tm_ab;
  {
    const uint64_t d[3] = {static_cast<uint64_t>(H), static_cast<uint64_t>(2 * I), static_cast<uint64_t>(p.E1)};
    const uint64_t s[2] = {static_cast<uint64_t>(p.gu_sr) * 2, static_cast<uint64_t>(p.gu_se) * 2};
    const uint32_t b[3] = {64, 128, 1};
    if (!tmap(&tm_gu, p.w_gu, 3, d, s, b)) return kDecodeTcUnsuitable;
  }
  {
    const uint64_t d[3] = {static_cast<uint64_t>(I), static_cast<uint64_t>(H), static_cast<uint64_t>(p.E1)};
    const uint64_t s[2] = {static_cast<uint64_t>(p.d_sr) * 2, static_cast<uint64_t>(p.d_se) * 2};
    const uint32_t b[3] = {64, 128, 1};
    if (!tmap(&tm_d, p.w_d, 3, d, s, b)) return kDecodeTcUnsuitable;
  }
  {
    const uint64_t d[2] = {static_cast<uint64_t>(I), static_cast<uint64_t>(u_max) * 32};
    const uint64_t s[1] = {static_cast<uint64_t>(I) * 2};
    const uint32_t b[2] = {64, 32};
    if (!tmap(&tm_ab, p.tc_abuf, 2, d, s, b)) return kDecodeTcUnsuitable;
  }
  cudaError_t e = cudaFuncSetAttribute(moe_decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(moe_decode_tc)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, moe_decode_tc_kernel, p, tm_gu, tm_d, tm_ab);
  return cuda_status(e, "moe_decode_tc launch");
}

}  // namespace mv
