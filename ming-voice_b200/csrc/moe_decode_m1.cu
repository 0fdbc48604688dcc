// One-token decode of the MoE block with the router fused (the single-token forward of the patched block,
// ming-voice engine.py:371-386: moe_route followed by fused_moe_decode, kernels fused_moe.py:14-61), in one
// cooperative kernel. This is the configuration a voice decode step runs 16 times per token, so it has its own
// kernel; more tokens, caller-given pairs and other shapes go to moe_decode.cu / moe_decode_tc.cu.
//
// The step streams ~U x 17 MB of expert weights (bf16, H=2048, I=1408) and little else; what limits a
// weight-streaming kernel at this size is how many bytes each SM keeps in flight, and how fast its warps turn a
// landed stage into a free slot. The design:
//
//  * 16 warps = 4 groups of 4 warps, one 40 KB ring slot per group (kSlotBytes). There is no producer warp: the first warp of a
//    group issues the bulk copies (TMA engine, evict-first) of the group's next stage into its own slot right
//    after the group has finished reading it, so a slot never waits for another warp's turn, and without a
//    producer warp the kernel runs 16 warps, i.e. up to 128 registers a thread.
//  * The CTA's stages (its share of the gate/up rows, then of the down rows) are dealt to the groups in turn.
//  * Split K: the 4 warps of a group take the 4 K quarters of every row of a stage, so each lane keeps 8 rows'
//    dot products in flight at once (a warp alone on its SM sub-partition is latency-bound with one or two). The
//    8 partial sums of a warp are reduced with 9 shuffles (reduce8); the quarters of a row meet in shared memory
//    and are added in a fixed order (deterministic results).
//  * Gate/up (row granularity, an equal share of the selected experts' rows per CTA, no split across CTAs):
//    a = wts * silu(gate . xn) * (up . xn) in fp32, stored to the workspace. One grid barrier. Down: each CTA
//    owns output rows [hd0, hd1) of every selected expert; y = sum_e w_d[e][h] . a_e, + residual, bf16.
//  * Routing: the shared-expert (static) rows need no routing, so the first ring-full of them is copied at
//    kernel entry and consumed while the router runs: warps 4q..4q+3 of CTA b compute the K quarters of the
//    logit of expert q * G + b (fp64 dots, added in order and rounded once to fp32), a grid barrier publishes them, and every CTA makes the same selection
//    with all its threads (route::select_parallel: every expert's rank among the biased scores, ties to the
//    lower id, so no serial rounds of arg-max; the router bias was staged in shared memory at entry) and writes
//    its one-token expert table directly (static slots, then the picks in id order). The selection sits on the
//    critical path of every block: made by one warp it took ~3 us of the block's ~48, made by the CTA well
//    under one, and the whole block ran at 39.6 us instead of 48.1 (bf16) and 40.0 instead of 43.1 (int8).
//    Two L2 prefetches of the down rows measured slower and are not used: issued at the routing decision
//    (43.6 us) they delay the routed gate/up stream, issued at the end of the gate/up phase (42.1 us) they
//    delay the slowest CTAs on the grid barrier, and neither shortened the down phase.
//
// Numerics: as moe_decode.cu (fp32 accumulation and intermediates; RMSNorm as mv_rmsnorm), except that an int8
// row's products are float(q) * x and the row's partial sums are multiplied by its scale once (the dequantised
// weight float(q) * float(scale) is never formed: one multiply per row instead of one per weight, ~17 % of the
// consumers' instructions, which bound the int8 kernel; the difference is fp32 rounding, ~1e-7 relative).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "decode_common.cuh"

namespace mv {
namespace decode {
namespace m1 {

constexpr int kGroups = 4;   // ring slots = consuming groups
constexpr int kGW = 4;       // warps per group = K parts of a row
constexpr int kWarps = kGroups * kGW;
constexpr int kThreads = kWarps * 32;
// Ring slot: 40 KB, not the general kernel's 32 KB. A gate/up stage still fills 32 KB of it (RG rows of gate and
// of up), but a down stage takes 14 bf16 rows of 2816 bytes instead of 11, so a CTA's 112 (expert, row) entries
// of the BASELINE block fit 8 stages = two rounds of the 4 groups after the grid barrier instead of three (the
// shared memory has room: 217 KB of 227).
constexpr int kSlotBytes = 40960;

// Shared-memory layout (byte offsets), computed identically on the host (size check) and the device.
struct Layout {
  unsigned int bars, xn, abuf, gsc, dsc, e_id, e_ntok, e_pbase, e_tok, e_w, misc, pr_e, pr_w, sel_r, sel_sc, sel_k,
      sbias, red, gpart, ypart, total;
};

__host__ __device__ inline unsigned int take(unsigned int& o, unsigned int bytes, unsigned int align) {
  o = (o + align - 1) / align * align;
  const unsigned int r = o;
  o += bytes;
  return r;
}

__host__ __device__ inline Layout layout(int H, int I, int E, int u_max, int nhc, int gsc_cap, int RG, bool int8) {
  Layout L;
  unsigned int o = kGroups * kSlotBytes;  // the ring, at offset 0 (1024-byte aligned)
  L.bars = take(o, kGroups * 8, 8);
  L.xn = take(o, H * 2, 16);
  L.abuf = take(o, u_max * I * 4, 16);
  L.gsc = take(o, int8 ? 2 * gsc_cap * 4 : 0, 16);
  L.dsc = take(o, int8 ? u_max * nhc * 4 : 0, 16);
  L.e_id = take(o, u_max * 4, 4);
  L.e_ntok = take(o, u_max * 4, 4);
  L.e_pbase = take(o, u_max * 4, 4);
  L.e_tok = take(o, u_max * 4, 4);
  L.e_w = take(o, u_max * 4, 4);
  L.misc = take(o, 16 * 4, 4);
  L.pr_e = take(o, kMaxNK * 4, 4);
  L.pr_w = take(o, kMaxNK * 4, 4);
  L.sel_r = take(o, E * 4, 16);
  L.sel_sc = take(o, E * 4, 16);
  L.sel_k = take(o, kMaxNK * 8 + 32 * 4, 16);                 // selection: pick values (fp64), group scores
  L.sbias = take(o, E * 4, 16);                               // the router bias, loaded at the start
  L.red = take(o, kWarps * 8, 8);
  L.gpart = take(o, kGroups * 2 * 2 * RG * kGW * 4, 16);
  L.ypart = take(o, u_max * nhc * kGW * 4, 16);
  L.total = o;
  return L;
}

// A ring stage: RG gate rows [i, i + nr) of slot u with the matching up rows, or ne down entries from (du, dr).
struct Stage {
  int down;
  int u, i, nr, walk;  // gate/up: slot index u, first row i, rows nr; walk 1 = routed, else static
  int du, dr, ne;      // down: first (expert, row) entry and the entry count
};

// Gate rows per stage: the largest power of two <= 8 with 2 RG rows (gate + up) in one stage.
__host__ __device__ constexpr int rows_per_stage(int row_bytes) {
  return 2 * 8 * row_bytes <= kSlotBytes ? 8 : (2 * 4 * row_bytes <= kSlotBytes ? 4 : (2 * 2 * row_bytes <= kSlotBytes ? 2 : 1));
}

// Specialised for the hidden size H and the expert width I (the model's, so every offset, trip count and bound
// below is a compile-time constant and the inner loops have no branches).
template <bool INT8, int H, int I>
__global__ void __launch_bounds__(kThreads, 1) decode_m1_kernel(const Params p) {
  using WT = W<INT8>;
  constexpr int VEC = WT::vec;
  constexpr int RG = rows_per_stage(H * WT::esz);
  constexpr int DP0 = kSlotBytes / (I * WT::esz);
  constexpr int DP = DP0 < kNhMax ? DP0 : kNhMax;  // down rows per stage
  constexpr int nvh = H / VEC, nqh = nvh / kGW;    // 16-byte chunks of a gate/up row; of its K quarter
  constexpr int nvi = I / VEC, nqi = nvi / kGW;    // ... of a down row
  constexpr int kXJ = (nqh > nqi ? nqh : nqi) > 32 ? 2 : 1;  // chunks per lane of a K quarter (at most 2)
  static_assert(RG == 4 || RG == 8, "4 or 8 gate rows per stage");
  static_assert(nvh % kGW == 0 && nvi % kGW == 0 && nqh <= 64 && nqi <= 64, "K quarters of at most 64 chunks");
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int grp = warp / kGW;  // group: owns ring slot grp
  const int kq = warp % kGW;   // K quarter of every row this warp takes
  const int G = gridDim.x;
  const int nhc = p.nh_cap;
  const int n_static = p.n_static;
  const Layout Lo = layout(H, I, p.E, p.u_max, nhc, p.gsc_cap, RG, INT8);
  (void)DP0;
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lo.bars);
  uint16_t* xn = reinterpret_cast<uint16_t*>(smem + Lo.xn);
  float* abuf = reinterpret_cast<float*>(smem + Lo.abuf);
  float* gsc = reinterpret_cast<float*>(smem + Lo.gsc);  // [2][gsc_cap] gate / up row scales (int8)
  float* dsc = reinterpret_cast<float*>(smem + Lo.dsc);  // [u_max][nh_cap] down row scales (int8)
  int* e_id = reinterpret_cast<int*>(smem + Lo.e_id);
  int* e_ntok = reinterpret_cast<int*>(smem + Lo.e_ntok);
  int* e_pbase = reinterpret_cast<int*>(smem + Lo.e_pbase);
  int* e_tok = reinterpret_cast<int*>(smem + Lo.e_tok);
  float* e_w = reinterpret_cast<float*>(smem + Lo.e_w);
  int* misc = reinterpret_cast<int*>(smem + Lo.misc);  // [0] = U (experts in the table, static first)
  int* pr_e = reinterpret_cast<int*>(smem + Lo.pr_e);
  float* pr_w = reinterpret_cast<float*>(smem + Lo.pr_w);
  float* sel_r = reinterpret_cast<float*>(smem + Lo.sel_r);
  float* sel_sc = reinterpret_cast<float*>(smem + Lo.sel_sc);
  double* sel_kd = reinterpret_cast<double*>(smem + Lo.sel_k);
  float* sel_gs = reinterpret_cast<float*>(smem + Lo.sel_k + kMaxNK * 8);
  float* sbias = reinterpret_cast<float*>(smem + Lo.sbias);
  double* red = reinterpret_cast<double*>(smem + Lo.red);
  float* gpart = reinterpret_cast<float*>(smem + Lo.gpart);  // [group][2][2 RG][kGW]
  float* ypart = reinterpret_cast<float*>(smem + Lo.ypart);  // [u_max][nh_cap][kGW]

  const long long S = static_cast<long long>(n_static) * I;  // static gate/up rows of the block
  const long long s_lo = S * blockIdx.x / G, s_hi = S * (blockIdx.x + 1) / G;
  const int hd0 = static_cast<int>(static_cast<long long>(H) * blockIdx.x / G);
  const int hd1 = static_cast<int>(static_cast<long long>(H) * (blockIdx.x + 1) / G);
  const int nh = hd1 - hd0;
  const uint32_t row_b = static_cast<uint32_t>(H) * WT::esz;
  const uint32_t drow_b = static_cast<uint32_t>(I) * WT::esz;
  const uint64_t pol = policy_evict_first();
  const bool issuer = kq == 0 && lane == 0;  // issues the copies of the group's slot
  uint8_t* slot = ring + static_cast<size_t>(grp) * kSlotBytes;
  uint64_t* full = bars + grp;
  uint32_t ph = 0;    // parity of the slot's next fill
  int gcount = 0;     // gate/up stages consumed by the group (double-buffered partial sums)
  bool ok = true;

  // The first static stages, one per group (as many as there are), stream before the routing decision; the
  // rest follow the routed rows. s_mid: the first static row after them.
  int n_early = 0;
  long long s_mid = s_lo;
  Stage early{};
  {
    GuStages it{GuWalk{s_lo, s_hi, I, 0}};
    int u, i, nr;
    while (n_early < kGroups && it.next(u, i, nr, RG)) {
      if (n_early == grp) early = Stage{0, u, i, nr, 0, 0, 0, 0};
      s_mid = static_cast<long long>(u) * I + i + nr;
      ++n_early;
    }
  }
  auto issue = [&](const Stage& st) {  // issuer only: the stage's rows into the group's slot
    if (!st.down) {
      const int e = st.walk == 1 ? e_id[st.u] : p.static_id + st.u;
      const uint8_t* gbase = p.w_gu + static_cast<long long>(e) * p.gu_se * WT::esz;
      mbar_arrive_expect_tx(full, 2u * st.nr * row_b);
      if (p.gu_sr == H) {
        bulk_g2s(slot, gbase + static_cast<long long>(st.i) * row_b, st.nr * row_b, full, pol);
        bulk_g2s(slot + RG * row_b, gbase + static_cast<long long>(I + st.i) * row_b, st.nr * row_b, full, pol);
      } else {
        for (int r = 0; r < st.nr; ++r) {
          bulk_g2s(slot + r * row_b, gbase + static_cast<long long>(st.i + r) * p.gu_sr * WT::esz, row_b, full, pol);
          bulk_g2s(slot + (RG + r) * row_b, gbase + static_cast<long long>(I + st.i + r) * p.gu_sr * WT::esz, row_b,
                   full, pol);
        }
      }
    } else {
      mbar_arrive_expect_tx(full, static_cast<uint32_t>(st.ne) * drow_b);
      DownStages c;
      c.u = st.du;
      c.r = st.dr;
      c.next(misc[0], nh, st.ne, true, [&](int u, int r, int n, int k) {
        const uint8_t* src =
            p.w_d + (static_cast<long long>(e_id[u]) * p.d_se + static_cast<long long>(hd0 + r) * p.d_sr) * WT::esz;
        if (p.d_sr == I) {
          bulk_g2s(slot + static_cast<size_t>(k) * drow_b, src, n * drow_b, full, pol);
        } else {
          for (int j = 0; j < n; ++j)
            bulk_g2s(slot + static_cast<size_t>(k + j) * drow_b, src + static_cast<long long>(j) * p.d_sr * WT::esz,
                     drow_b, full, pol);
        }
      });
    }
  };
  auto wait_slot = [&]() {  // every warp of the group: the slot's current fill has landed (skipped once failed)
    bool good = ok;
    if (lane == 0 && good) good = mbar_wait(full, ph, p.ws, 0x500u | grp);
    good = __shfl_sync(0xffffffffu, good, 0) != 0;
    ph ^= 1u;
    ok = ok && good;
  };
  long long r_lo = 0, r_hi = 0;  // this CTA's routed gate/up rows (known after the routing)

  if (tid == 0) {
    MV_TRACE_AT(p, 0);
    for (int s = 0; s < kGroups; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    misc[0] = n_static;
  }
  __syncthreads();
  pdl_launch_dependents();  // the next block's kernel may be scheduled now (it waits for this one to complete)
  if (issuer && grp < n_early) issue(early);
  // the next block's router rows and RMSNorm weight (its routing reads them first): one slice per CTA into L2
  if (tid == 32 && p.nx_rw != nullptr) {
    const long long per = ((p.nx_rw_bytes + G - 1) / G + 15) & ~15LL;
    const long long b0 = per * blockIdx.x;
    if (b0 < p.nx_rw_bytes) bulk_prefetch_l2(p.nx_rw + b0, static_cast<uint32_t>(min(per, p.nx_rw_bytes - b0)));
    if (blockIdx.x == G - 1 && p.nx_norm != nullptr) bulk_prefetch_l2(p.nx_norm, static_cast<uint32_t>(H) * 2u);
  }
  // the logit this warp helps with: expert (warp / 4) * G + b, K quarter warp % 4 (4 warps per logit: a quarter
  // of the dot each, so the logits are published ~4x sooner than with one warp per expert)
  const int e_logit = (warp >> 2) * G + static_cast<int>(blockIdx.x);
  const int lq = warp & 3;
  constexpr int HQ = H / 4;
  const int resz = p.rw_dtype == MV_F32 ? 4 : (p.rw_dtype == MV_BF16 ? 2 : 1);
  if (lane == 0 && e_logit < p.E)
    bulk_prefetch_l2(static_cast<const uint8_t*>(p.rw) + (static_cast<size_t>(e_logit) * H + lq * HQ) * resz,
                     static_cast<uint32_t>(HQ * resz));
  // the router bias into shared memory now: the selection reads it on the critical path, long after this load
  if (p.rbias != nullptr)
    for (int j = tid; j < p.E; j += kThreads) sbias[j] = p.rbias[j];
  // everything above reads weights only; the token and the workspace are the previous kernel's (a programmatic
  // launch may start before it completes)
  pdl_wait();
  // this thread's output element's residual (the token itself), read now rather than at the end
  const float res_pre =
      (p.residual != nullptr && tid < nh) ? __uint_as_float(static_cast<uint32_t>(p.residual[hd0 + tid]) << 16) : 0.f;

  // ---- prologue: RMSNorm of the token (as mv_rmsnorm: fp64 sum of squares, IEEE-rounded 1/sqrt) -> xn bf16
  {
    const int nv = H / 8;
    const uint4* xr = reinterpret_cast<const uint4*>(p.x);
    uint4* xs = reinterpret_cast<uint4*>(xn);
    const uint4 g_pref =
        (p.norm_w != nullptr && tid < nv) ? reinterpret_cast<const uint4*>(p.norm_w)[tid] : make_uint4(0, 0, 0, 0);
    double ss = 0.0;
    for (int j = tid; j < nv; j += kThreads) {
      const uint4 v = xr[j];
      xs[j] = v;
      const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int z = 0; z < 4; ++z) {
        const double a = bf16lo(vv[z]), b = bf16hi(vv[z]);
        ss += a * a + b * b;
      }
    }
    if (p.norm_w != nullptr) {
      ss = warp_sum_d(ss);
      if (lane == 0) red[warp] = ss;
      named_bar(1, kThreads);
      double tot = 0.0;
      for (int w = 0; w < kWarps; ++w) tot += red[w];
      const float var = static_cast<float>(tot / static_cast<double>(H));
      const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
      const uint4* wr = reinterpret_cast<const uint4*>(p.norm_w);
      for (int j = tid; j < nv; j += kThreads) {
        const uint4 v = xs[j];
        const uint4 gw = j == tid ? g_pref : wr[j];
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
        const uint32_t gg[4] = {gw.x, gw.y, gw.z, gw.w};
        uint32_t o[4];
#pragma unroll
        for (int z = 0; z < 4; ++z) {
          const float y0 = round_bf16(__fmul_rn(bf16lo(vv[z]), r));
          const float y1 = round_bf16(__fmul_rn(bf16hi(vv[z]), r));
          o[z] = static_cast<uint32_t>(f2bf(__fmul_rn(bf16lo(gg[z]), y0))) |
                 (static_cast<uint32_t>(f2bf(__fmul_rn(bf16hi(gg[z]), y1))) << 16);
        }
        xs[j] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    if (INT8) {  // gate / up row scales of this CTA's static rows
      for (long long r = s_lo + tid; r < s_hi; r += kThreads) {
        const int u = static_cast<int>(r / I), i = static_cast<int>(r % I);
        const long long b = static_cast<long long>(p.static_id + u) * p.sgu_se;
        gsc[r - s_lo] = ldscale(p.s_gu, b + i, p.s_bf16);
        gsc[p.gsc_cap + (r - s_lo)] = ldscale(p.s_gu, b + I + i, p.s_bf16);
      }
    }
    named_bar(1, kThreads);
    if (tid == 0) MV_TRACE_AT(p, 1);
  }
  // this lane's x values for its K quarter of the gate/up rows: chunks c = kq * nqh + lane + 32 j; a lane past the
  // quarter's end reads the quarter's last chunk with x = 0 (so every lane runs the same branch-free code)
  float xv[kXJ][VEC];
#pragma unroll
  for (int j = 0; j < kXJ; ++j) {
    const bool in = lane + 32 * j < nqh;
    const int c = kq * nqh + (in ? lane + 32 * j : nqh - 1);
#pragma unroll
    for (int e = 0; e < VEC; e += 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(xn + c * VEC + e);
      const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int z = 0; z < 4; ++z) {
        xv[j][e + 2 * z] = in ? bf16lo(vv[z]) : 0.f;
        xv[j][e + 2 * z + 1] = in ? bf16hi(vv[z]) : 0.f;
      }
    }
  }
  int cofs[kXJ];  // byte offset of this lane's chunk j within a gate/up row
#pragma unroll
  for (int j = 0; j < kXJ; ++j) cofs[j] = (kq * nqh + (lane + 32 * j < nqh ? lane + 32 * j : nqh - 1)) * 16;

  // ---- one gate/up stage: split K over the group's warps, SiLU(gate) * up * weight per row -> workspace. All 8
  // rows of a batch are computed (rows past the stage's nr read stale slot data; their sums are never used).
  auto consume_gu = [&](const Stage& st) {
    const bool routed = st.walk == 1;
    const long long rw = static_cast<long long>(st.u - (routed ? n_static : 0)) * I + st.i;  // row in its walk
    // int8 row scales: the CTA's static rows first, then its routed rows
    const int sc0 = routed ? static_cast<int>(s_hi - s_lo + rw - r_lo) : static_cast<int>(rw - s_lo);
    float* gp = gpart + ((grp * 2 + (gcount & 1)) * 2 * RG) * kGW;
    if (ok) {
#pragma unroll
      for (int h = 0; h < RG / 4; ++h) {  // batches of 4 gate rows + the 4 matching up rows
        float acc[8][2];
        float sc[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          acc[r][0] = acc[r][1] = 0.f;
          sc[r] = 1.0f;
          if (INT8) sc[r] = gsc[(r < 4 ? 0 : p.gsc_cap) + sc0 + min(h * 4 + (r & 3), st.nr - 1)];
        }
#pragma unroll
        for (int j = 0; j < kXJ; ++j) {
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const int row = (r < 4 ? 0 : RG) + h * 4 + (r & 3);
            const uint4 wv = *reinterpret_cast<const uint4*>(slot + row * (H * WT::esz) + cofs[j]);
            chunk_fma_unscaled<INT8>(acc[r][0], acc[r][1], wv, xv[j]);
          }
        }
        float v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = INT8 ? (acc[r][0] + acc[r][1]) * sc[r] : acc[r][0] + acc[r][1];
        reduce8(v);
        if ((lane & 3) == 0) {
          const int r = lane >> 2;  // 0..3: gate rows of the batch, 4..7: up rows
          gp[((r < 4 ? 0 : RG) + h * 4 + (r & 3)) * kGW + kq] = v[0];
        }
      }
    }
  };
  auto combine_gu = [&](const Stage& st) {  // warp 0 of the group, one lane per row, after the group barrier
    const float* gp = gpart + ((grp * 2 + (gcount & 1)) * 2 * RG) * kGW;
    if (ok && kq == 0 && lane < st.nr) {
      float g = 0.f, uu = 0.f;
#pragma unroll
      for (int k = 0; k < kGW; ++k) {
        g += gp[lane * kGW + k];
        uu += gp[(RG + lane) * kGW + k];
      }
      const bool routed = st.walk == 1;
      const float tw = routed ? e_w[st.u] : 1.0f;
      const int pb = routed ? e_pbase[st.u] : st.u;
      const float act = g / (1.0f + expf(-g));
      p.a_g[static_cast<long long>(pb) * I + st.i + lane] = act * uu * tw;
    }
  };

  // ---- router logits: warps 4q..4q+3 of CTA b compute the K quarters of expert q * G + b (fp64), thread 0 adds
  // the quarters in order, rounds once to fp32 and publishes
  unsigned long long tgt1 = 0;
  if (e_logit < p.E) {
    double acc[1] = {0.0};
    const float rsc = p.rw_dtype == MV_I8 ? ldscale(p.rw_scale, e_logit, p.rw_scale_bf16) : 1.0f;
    route::router_dot<1>(static_cast<const uint8_t*>(p.rw) + (static_cast<size_t>(e_logit) * H + lq * HQ) * resz,
                         p.rw_dtype, rsc, xn + lq * HQ, HQ, 1, acc);
    const double v = warp_sum_d(acc[0]);
    if (lane == 0) red[warp] = v;
  }
  named_bar(1, kThreads);
  if (tid == 0) {
    for (int q = 0; q < kWarps / 4; ++q) {
      const int e = q * G + static_cast<int>(blockIdx.x);
      if (e < p.E) p.logits_ws[e] = static_cast<float>(((red[4 * q] + red[4 * q + 1]) + red[4 * q + 2]) + red[4 * q + 3]);
    }
    MV_TRACE_AT(p, 2);
    tgt1 = grid_arrive_gen(&p.ws->gen1, G);  // (fence + arrive by the thread that wrote this CTA's logits)
  }

  // ---- the first static stage of each group while the other CTAs' logits arrive
  if (grp < n_early) {
    wait_slot();
    consume_gu(early);
    named_bar(3 + grp, kGW * 32);
    combine_gu(early);
    ++gcount;
  }
  if (tid == 0) MV_TRACE_AT(p, 5);

  // ---- routing: every CTA makes the same selection from the published logits (one warp), then its table
  if (tid == 0) grid_wait_gen(&p.ws->gen1, tgt1, p.ws, 0x300u);
  if (tid == 0) MV_TRACE_AT(p, 3);
  if (tid < kMaxNK) pr_e[tid] = -1;  // a pick the selection leaves unset stays invalid
  named_bar(1, kThreads);
  {  // the selection by all threads: ranks instead of rounds of arg-max (the same picks, ties to the lower id)
    const route::SelectCfg cfg{p.route_mode, p.E, p.top_k, p.n_group, p.topk_group, p.rscale,
                               p.rbias != nullptr ? sbias : nullptr};
    route::select_parallel(cfg, p.logits_ws, 1, tid, kThreads, [] { named_bar(1, kThreads); }, sel_r, sel_sc, sel_kd,
                           sel_gs, pr_e, pr_w);
  }
  if (tid == 0) MV_TRACE_AT(p, 15);
  if (warp == 1 && blockIdx.x == 0) {  // router outputs (beside warp 0's table): ids / weights, static slots, logits
    {
      const int NKT = p.top_k + n_static;
      for (int k = lane; k < NKT; k += 32) {
        const long long id = k < p.top_k ? pr_e[k] : static_cast<long long>(p.static_id + k - p.top_k);
        if (p.ids_out) {
          if (p.ids_out_i64)
            static_cast<long long*>(p.ids_out)[k] = id;
          else
            static_cast<int*>(p.ids_out)[k] = static_cast<int>(id);
        }
        if (p.wts_out) p.wts_out[k] = k < p.top_k ? pr_w[k] : 1.0f;
      }
      if (p.logits_out)
        for (int j = lane; j < p.E; j += 32) p.logits_out[j] = ld_cg_f32(p.logits_ws + j);
    }
  }
  if (warp == 0) {
    {  // the expert table of one token: the static slots, then the valid picks (distinct experts) in id order
      const int K = p.top_k;
      const int pe = lane < K ? pr_e[lane] : -1;
      const bool valid = pe >= 0 && pe < p.E1;
      const int e = valid ? pe : 0x7fffffff;
      const float w = valid ? pr_w[lane] : 0.f;
      int rank = n_static;
      for (int j = 0; j < K; ++j) rank += __shfl_sync(0xffffffffu, e, j) < e ? 1 : 0;
      if (valid) {
        e_id[rank] = e;
        e_w[rank] = w;
      }
      const int Ut = n_static + __popc(__ballot_sync(0xffffffffu, valid));
      for (int u = lane; u < Ut; u += 32) {
        if (u < n_static) {
          e_id[u] = p.static_id + u;
          e_w[u] = 1.0f;
        }
        e_ntok[u] = 1;
        e_tok[u] = 0;
        e_pbase[u] = u;
      }
      if (lane == 0) {
        misc[0] = Ut;
        misc[3] = Ut;
      }
      __syncwarp();
    }
    if (tid == 0) MV_TRACE_AT(p, 17);
  }
  named_bar(1, kThreads);
  if (tid == 0) MV_TRACE_AT(p, 4);
  const int U = misc[0];

  const long long T = S + static_cast<long long>(U - n_static) * I;
  r_lo = T * blockIdx.x / G - s_lo;
  r_hi = T * (blockIdx.x + 1) / G - s_hi;
  if (INT8) {  // scales of this CTA's routed gate/up rows and of its down rows of every expert
    const int base = static_cast<int>(s_hi - s_lo);
    for (long long r = r_lo + tid; r < r_hi; r += kThreads) {
      const int u = n_static + static_cast<int>(r / I), i = static_cast<int>(r % I);
      const long long b = static_cast<long long>(e_id[u]) * p.sgu_se;
      gsc[base + (r - r_lo)] = ldscale(p.s_gu, b + i, p.s_bf16);
      gsc[p.gsc_cap + base + (r - r_lo)] = ldscale(p.s_gu, b + I + i, p.s_bf16);
    }
    for (int j = tid; j < U * nh; j += kThreads) {
      const int u = j / nh, r = j % nh;
      dsc[u * nhc + r] = ldscale(p.s_d, static_cast<long long>(e_id[u]) * p.sd_se + hd0 + r, p.s_bf16);
    }
    named_bar(1, kThreads);
  }

  // ---- the stages after the routing decision, dealt to the groups in turn: routed gate/up rows, the remaining
  // static ones, then the down rows (DP entries per stage, across experts)
  GuStages it_r{GuWalk{r_lo, r_hi, I, n_static}}, it_s{GuWalk{s_mid, s_hi, I, 0}};
  DownStages it_d;
  int seq = n_early;  // index of the next stage of the sequence
  auto next_owned = [&](Stage& st) -> bool {
    while (true) {
      int u, i, nr;
      bool have;
      if (it_r.next(u, i, nr, RG)) {
        st = Stage{0, u, i, nr, 1, 0, 0, 0};
        have = true;
      } else if (it_s.next(u, i, nr, RG)) {
        st = Stage{0, u, i, nr, 0, 0, 0, 0};
        have = true;
      } else {
        const int ne = it_d.entries(U, nh, DP, true);
        have = ne > 0;
        if (have) {
          st = Stage{1, 0, 0, 0, 0, it_d.u, it_d.r, ne};
          it_d.next(U, nh, DP, true, [](int, int, int, int) {});
        }
      }
      if (!have) return false;
      if (seq++ % kGroups == grp) return true;
    }
  };
  Stage cur{};
  bool have = next_owned(cur);
  if (issuer && have) issue(cur);
#ifdef MV_TRACE
  int tj = 0;
#endif
  while (have && !cur.down) {
    wait_slot();
#ifdef MV_TRACE
    if (tid == 0 && tj < 6) MV_TRACE_AT(p, 20 + 2 * tj);
#endif
    consume_gu(cur);
    named_bar(3 + grp, kGW * 32);  // the slot is read: the next stage goes in
    Stage nxt{};
    const bool hn = next_owned(nxt);
    if (issuer && hn && ok) issue(nxt);
#ifdef MV_TRACE
    if (tid == 0 && tj < 6) MV_TRACE_AT(p, 21 + 2 * tj);
    ++tj;
#endif
    combine_gu(cur);
    ++gcount;
    cur = nxt;
    have = hn;
  }
  if (tid == 0) MV_TRACE_AT(p, 6);
  // ---- grid barrier: every CTA's activations are in the workspace; then this CTA loads them all
  named_bar(1, kThreads);
  if (tid == 0) {
    MV_TRACE_AT(p, 7);
    const unsigned long long tgt2 = grid_arrive_gen(&p.ws->gen2, G);
    grid_wait_gen(&p.ws->gen2, tgt2, p.ws, 0x400u);
    MV_TRACE_AT(p, 8);
  }
  named_bar(1, kThreads);
  if (nh > 0) {
    const int n16 = U * I / 4;
    for (int j = tid; j < n16; j += kThreads) cp_async16(abuf + 4 * j, p.a_g + 4 * j);
    cp_async_commit();
    cp_async_wait<0>();
  }
  named_bar(1, kThreads);
  if (tid == 0) MV_TRACE_AT(p, 9);

  // ---- down stages: split K, runs of up to 8 rows of one expert; the K quarters of each (expert, row) to ypart.
  // All 8 rows of a run are computed (rows past the run read other slot or shared data; never used).
  int dofs[kXJ];  // byte offset of this lane's chunk j within a down row
  bool din[kXJ];
#pragma unroll
  for (int j = 0; j < kXJ; ++j) {
    din[j] = lane + 32 * j < nqi;
    dofs[j] = (kq * nqi + (din[j] ? lane + 32 * j : nqi - 1)) * 16;
  }
#ifdef MV_TRACE
  int tk = 0;
#endif
  while (have) {
    wait_slot();
#ifdef MV_TRACE
    if (tid == 0 && tk < 2) MV_TRACE_AT(p, 12 + tk);
    ++tk;
#endif
    if (ok) {
      float av[kXJ][VEC];
      int au = -1;
      DownStages c;
      c.u = cur.du;
      c.r = cur.dr;
      for (int k = 0; k < cur.ne;) {
        const int u = c.u, r0 = c.r;
        const int run = min(8, min(cur.ne - k, nh - r0));
        if (u != au) {  // this lane's activation chunks of expert u (0 past the quarter's end)
          const float* a_u = abuf + e_pbase[u] * I;
#pragma unroll
          for (int j = 0; j < kXJ; ++j) {
#pragma unroll
            for (int e = 0; e < VEC; e += 4) {
              const float4 a4 = *reinterpret_cast<const float4*>(a_u + (dofs[j] / 16) * VEC + e);
              av[j][e] = din[j] ? a4.x : 0.f;
              av[j][e + 1] = din[j] ? a4.y : 0.f;
              av[j][e + 2] = din[j] ? a4.z : 0.f;
              av[j][e + 3] = din[j] ? a4.w : 0.f;
            }
          }
          au = u;
        }
        float acc[8][2];
        float sc[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          acc[r][0] = acc[r][1] = 0.f;
          sc[r] = INT8 ? dsc[u * nhc + r0 + min(r, run - 1)] : 1.0f;
        }
        const uint8_t* rows = slot + k * (I * WT::esz);
#pragma unroll
        for (int j = 0; j < kXJ; ++j) {
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const uint4 wv = *reinterpret_cast<const uint4*>(rows + r * (I * WT::esz) + dofs[j]);
            chunk_fma_unscaled<INT8>(acc[r][0], acc[r][1], wv, av[j]);
          }
        }
        float v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = INT8 ? (acc[r][0] + acc[r][1]) * sc[r] : acc[r][0] + acc[r][1];
        reduce8(v);
        if ((lane & 3) == 0 && (lane >> 2) < run) ypart[(u * nhc + r0 + (lane >> 2)) * kGW + kq] = v[0];
        k += run;
        c.r += run;
        if (c.r == nh) {
          c.r = 0;
          ++c.u;
        }
      }
    }
    named_bar(3 + grp, kGW * 32);  // the slot is read
#ifdef MV_TRACE
    if (tid == 0 && tk <= 2) MV_TRACE_AT(p, 17 + tk);  // group 0's first / second down stage consumed
#endif
    Stage nxt{};
    const bool hn = next_owned(nxt);
    if (issuer && hn && ok) issue(nxt);
    cur = nxt;
    have = hn;
  }
  named_bar(1, kThreads);
  if (tid == 0) MV_TRACE_AT(p, 10);
  // ---- y[h] = sum over experts (in table order) of the K quarters, + residual, bf16
  if (tid < nh) {
    float v = 0.f;
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int k = 0; k < kGW; ++k) v += ypart[(u * nhc + tid) * kGW + k];
    if (p.residual != nullptr) v += res_pre;
    p.out[hd0 + tid] = f2bf(v);
  }
  if (tid == 0) MV_TRACE_AT(p, 11);
}

}  // namespace m1

}  // namespace decode

// Launch of the one-token kernel for the fused block (router mode, M == 1): geometry, shape checks, cooperative
// launch. Returns kDecodeM1Unsuitable when the shapes do not fit it (the caller then runs the general kernel).
int decode_m1_run(decode::Params& p, bool int8, cudaStream_t st) {
  using namespace decode;
  using namespace decode::m1;
  const int H = p.H, I = p.I, esz = int8 ? 1 : 2;
  if (p.M != 1 || !p.router) return kDecodeM1Unsuitable;
  // the instantiated shapes: ming-voice's BASELINE block (H 2048, I 1408) and the released model's (1536, 512)
  void (*kern)(Params) = nullptr;
  if (H == 2048 && I == 1408)
    kern = int8 ? decode_m1_kernel<true, 2048, 1408> : decode_m1_kernel<false, 2048, 1408>;
  else if (H == 1536 && I == 512)
    kern = int8 ? decode_m1_kernel<true, 1536, 512> : decode_m1_kernel<false, 1536, 512>;
  if (kern == nullptr) return kDecodeM1Unsuitable;
  const int G = num_sms();
  if (p.E > (kWarps / 4) * G || p.E > 128 || p.top_k > 32 || p.top_k > p.E) return kDecodeM1Unsuitable;
  const int RG = rows_per_stage(H * esz);
  p.RG = RG;
  p.u_max = p.n_static + (p.top_k < p.E ? p.top_k : p.E);
  p.nh_cap = (H + G - 1) / G;
  if (p.nh_cap > kNhMax) return kDecodeM1Unsuitable;
  p.gsc_cap = int8 ? static_cast<int>((static_cast<long long>(p.u_max) * I + G - 1) / G + 4) : 0;
  const Layout L = layout(H, I, p.E, p.u_max, p.nh_cap, p.gsc_cap, RG, int8);
  if (L.total > 227u * 1024u) return kDecodeM1Unsuitable;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.total));
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(decode_m1)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  // programmatic launch: the kernel starts its weight copies while the previous kernel in the stream finishes
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  return cuda_status(e, "decode_m1 launch");
}

}  // namespace mv
