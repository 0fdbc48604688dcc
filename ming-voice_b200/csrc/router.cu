// MoE router: logits, selection and weights for n tokens.
//
// Replaces fused_ops.moe_route (ming-voice fused_ops.py:96-103; _gate_gemv :40-50, _route :53-93) and the
// patched torch gate (engine.py:326-333) in MV_ROUTE_SIGMOID_GROUP mode, and provides the BASELINE
// softmax-top-k router in MV_ROUTE_SOFTMAX mode.
//
// Logits are dot products of bf16 hidden states with the router rows (fp32 / bf16 / int8-dequantised);
// every product is exact in fp64 and the sum is accumulated in fp64, then rounded once to fp32. The
// selection therefore does not depend on a summation order. Sigmoid scores and softmax weights are
// evaluated in fp64 and rounded to fp32. Top-k takes the largest first, ties to the lower expert id (the
// reference's tl.argmax loop picks the first maximum).
//
// Small n (decode, n <= 16): one kernel; each warp computes one expert's logits for all tokens and the
// last CTA to finish (arrival counter in the workspace) makes the selections. Large n (prefill): a tiled
// fp64 logits kernel followed by a warp-per-token selection kernel.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "route_select.cuh"

namespace mv {
namespace route {

constexpr int kSmallM = 16;

struct Params {
  int mode;
  const uint16_t* x;
  long long x_stride;
  const uint16_t* norm_w;  // optional fused RMSNorm of x (bf16 weight)
  float eps;
  const void* w;
  int w_dtype;
  const void* w_scale;
  int scale_bf16;
  const float* bias;
  int n, H, E, top_k, n_group, topk_group;
  double scale;
  int n_shared, shared_id;
  float* logits;  // [n, E] destination of the logits (caller buffer or workspace)
  void* ids;
  int ids_i64;
  float* wts;
  WsHeader* ws;
};

__device__ __forceinline__ float w_elem(const Params& p, long long e, int h) {
  const long long i = e * p.H + h;
  if (p.w_dtype == MV_F32) return static_cast<const float*>(p.w)[i];
  if (p.w_dtype == MV_BF16) return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(p.w)[i]) << 16);
  const float s = p.scale_bf16
                      ? __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(p.w_scale)[e]) << 16)
                      : static_cast<const float*>(p.w_scale)[e];
  return dequant(static_cast<float>(static_cast<const int8_t*>(p.w)[i]), s);
}

__device__ void select_token(const Params& p, int m, const float* lg, float* scr) {
  const SelectCfg c{p.mode, p.E, p.top_k, p.n_group, p.topk_group, p.scale, p.bias};
  __shared__ int sel_s[8][32];
  __shared__ float w_s[8][32];
  const int warp = (threadIdx.x >> 5) & 7;
  select_core(c, lg, scr, sel_s[warp], w_s[warp]);
  __syncwarp();
  const int K = p.top_k, NKT = K + p.n_shared;
  const int lane = threadIdx.x & 31;
  for (int k = lane; k < NKT; k += 32) {
    const long long id = k < K ? sel_s[warp][k] : static_cast<long long>(p.shared_id + (k - K));
    const float wk = k < K ? w_s[warp][k] : 1.0f;
    if (p.ids_i64)
      static_cast<long long*>(p.ids)[static_cast<long long>(m) * NKT + k] = id;
    else
      static_cast<int*>(p.ids)[static_cast<long long>(m) * NKT + k] = static_cast<int>(id);
    p.wts[static_cast<long long>(m) * NKT + k] = wk;
  }
  __syncwarp();
}

// xn row into shared memory (bf16 bits), optionally through the fused RMSNorm (same arithmetic as
// mv_rmsnorm). Called by all threads of the block.
__device__ void load_xn(const Params& p, uint16_t* xs, double* red) {
  const int nthr = blockDim.x;
  for (int m = 0; m < p.n; ++m) {
    const uint16_t* xr = p.x + m * p.x_stride;
    if (p.norm_w == nullptr) {
      for (int h = threadIdx.x; h < p.H; h += nthr) xs[m * p.H + h] = xr[h];
      continue;
    }
    double ss = 0.0;
    for (int h = threadIdx.x; h < p.H; h += nthr) {
      const double v = __uint_as_float(static_cast<uint32_t>(xr[h]) << 16);
      ss += v * v;
    }
    ss = warp_sum_d(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
    for (int i = 0; i < (nthr >> 5); ++i) tot += red[i];
    __syncthreads();
    const float var = static_cast<float>(tot / static_cast<double>(p.H));
    const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
    for (int h = threadIdx.x; h < p.H; h += nthr) {
      const float y = round_bf16(__fmul_rn(__uint_as_float(static_cast<uint32_t>(xr[h]) << 16), rr));
      xs[m * p.H + h] = f2bf(__fmul_rn(__uint_as_float(static_cast<uint32_t>(p.norm_w[h]) << 16), y));
    }
  }
  __syncthreads();
}

// Small n: grid = ceil(E / 8) CTAs of 8 warps; warp w of CTA b owns expert 8b + w.
__global__ void __launch_bounds__(256) route_small_kernel(const Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);                         // [n][H]
  double* red = reinterpret_cast<double*>(xs + kSmallM * p.H);              // [8]
  float* scr = reinterpret_cast<float*>(red + 8);                           // [8][kMaxE]
  __shared__ int last;
  pdl_launch_dependents();
  load_xn(p, xs, red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  if (e < p.E) {
    double acc[kSmallM];
#pragma unroll
    for (int m = 0; m < kSmallM; ++m) acc[m] = 0.0;
    const int esz = p.w_dtype == MV_F32 ? 4 : (p.w_dtype == MV_BF16 ? 2 : 1);
    const float sc = p.w_dtype == MV_I8
                         ? (p.scale_bf16 ? __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(p.w_scale)[e]) << 16)
                                         : static_cast<const float*>(p.w_scale)[e])
                         : 1.0f;
    router_dot<kSmallM>(static_cast<const uint8_t*>(p.w) + static_cast<size_t>(e) * p.H * esz, p.w_dtype, sc, xs, p.H,
                        p.n, acc);
#pragma unroll
    for (int m = 0; m < kSmallM; ++m) {
      if (m < p.n) {
        const double v = warp_sum_d(acc[m]);
        if (lane == 0) p.logits[static_cast<long long>(m) * p.E + e] = static_cast<float>(v);
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&p.ws->counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // the logits written by the other CTAs are read through L2 (never cached in this SM's L1 before)
  for (int m = warp; m < p.n; m += 8) {
    float* lg = scr + warp * kMaxE;
    for (int i = lane; i < p.E; i += 32) lg[i] = ld_cg_f32(p.logits + static_cast<long long>(m) * p.E + i);
    __syncwarp();
    select_token(p, m, lg, lg);
  }
  __syncthreads();
  if (threadIdx.x == 0) atomicExch(&p.ws->counter, 0u);
}

// Large n: logits tile of 16 tokens x 64 experts per CTA, fp64 accumulation from shared-memory tiles.
constexpr int kTM = 16, kTE = 64, kTK = 64;
__global__ void __launch_bounds__(256) route_logits_kernel(const Params p) {
  __shared__ float xt[kTM][kTK + 1];
  __shared__ float wt[kTE][kTK + 1];
  const int m0 = blockIdx.x * kTM, e0 = blockIdx.y * kTE;
  const int tm = threadIdx.x / 16, te = threadIdx.x % 16;  // thread: token tm, experts te + 16 j
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  for (int k0 = 0; k0 < p.H; k0 += kTK) {
    for (int i = threadIdx.x; i < kTM * kTK; i += 256) {
      const int r = i / kTK, c = i % kTK;
      const int m = m0 + r;
      xt[r][c] = (m < p.n && k0 + c < p.H) ? __uint_as_float(static_cast<uint32_t>(p.x[m * p.x_stride + k0 + c]) << 16) : 0.f;
    }
    for (int i = threadIdx.x; i < kTE * kTK; i += 256) {
      const int r = i / kTK, c = i % kTK;
      const int e = e0 + r;
      wt[r][c] = (e < p.E && k0 + c < p.H) ? w_elem(p, e, k0 + c) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < kTK; ++c) {
      const double xv = xt[tm][c];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] += xv * static_cast<double>(wt[te + 16 * j][c]);
    }
    __syncthreads();
  }
  const int m = m0 + tm;
  if (m < p.n) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + te + 16 * j;
      if (e < p.E) p.logits[static_cast<long long>(m) * p.E + e] = static_cast<float>(acc[j]);
    }
  }
}

// Large n, tensor-core form: fp64 MMA (m16n8k4, exact products, fp64 accumulation) over a tile of 16 tokens
// x 64 experts per pass. The 4 warps split K into quarters; inside a warp, lane t of each quad walks its own
// contiguous run of S = H/16 k-indices (the dot product is a sum over K, so any fixed assignment of k to the
// MMA's k-slots gives the same terms), which lets every lane load 8 (bf16/int8) or 4 (f32) consecutive
// values per row with one vector load. The quarters are added in warp order (deterministic).
constexpr int kDM = 16, kDWarps = 4, kDE = 64;

template <int WDT>  // MV_F32, MV_BF16 or MV_I8
struct RowChunk {
  static constexpr int KG = WDT == MV_F32 ? 4 : 8;  // k-values per vector load
  uint32_t raw[WDT == MV_F32 ? 4 : (WDT == MV_BF16 ? 4 : 2)];
  __device__ __forceinline__ void load(const void* w, long long e, int H, int k) {
    if constexpr (WDT == MV_F32) {
      const uint4 v = *reinterpret_cast<const uint4*>(static_cast<const float*>(w) + e * H + k);
      raw[0] = v.x; raw[1] = v.y; raw[2] = v.z; raw[3] = v.w;
    } else if constexpr (WDT == MV_BF16) {
      const uint4 v = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(w) + e * H + k);
      raw[0] = v.x; raw[1] = v.y; raw[2] = v.z; raw[3] = v.w;
    } else {
      const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const int8_t*>(w) + e * H + k);
      raw[0] = v.x; raw[1] = v.y;
    }
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < static_cast<int>(sizeof(raw) / 4); ++i) raw[i] = 0u;
  }
  // value i of the chunk as the fp32 the oracle uses (int8: dequantised with one rounded multiply)
  __device__ __forceinline__ float get(int i, float sc) const {
    if (WDT == MV_F32) return __uint_as_float(raw[i]);
    if (WDT == MV_BF16) return (i & 1) ? bf16hi(raw[i >> 1]) : bf16lo(raw[i >> 1]);
    const int q = static_cast<int>(static_cast<int8_t>((raw[i >> 2] >> (8 * (i & 3))) & 0xffu));
    return dequant(static_cast<float>(q), sc);
  }
};

__device__ __forceinline__ void dmma_16x8x4(double (&c)[4], double a0, double a1, double b0) {
  asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
               : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
               : "d"(a0), "d"(a1), "d"(b0));
}

template <int WDT>
__global__ void __launch_bounds__(128) route_logits_dmma_kernel(const Params p) {
  constexpr int KG = RowChunk<WDT>::KG;
  __shared__ double part[kDWarps][kDM][kDE + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int m0 = blockIdx.x * kDM;
  const int S = p.H / 16;                          // k-values per lane
  const int kbase = warp * (p.H / 4) + t * S;      // this lane's run
  const int ma = m0 + g, mb = m0 + g + 8;
  const uint16_t* xa = p.x + static_cast<long long>(ma < p.n ? ma : 0) * p.x_stride;
  const uint16_t* xb = p.x + static_cast<long long>(mb < p.n ? mb : 0) * p.x_stride;
  for (int e0 = 0; e0 < p.E; e0 += kDE) {
    double acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0;
    float sc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + 8 * j + g;
      sc[j] = 1.0f;
      if (WDT == MV_I8 && e < p.E)
        sc[j] = p.scale_bf16 ? __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(p.w_scale)[e]) << 16)
                             : static_cast<const float*>(p.w_scale)[e];
    }
    for (int s = 0; s < S; s += KG) {
      const int k = kbase + s;
      double xav[KG], xbv[KG];
      {
        uint32_t ra[KG / 2], rb[KG / 2];
        if constexpr (KG == 8) {
          const uint4 va = ma < p.n ? *reinterpret_cast<const uint4*>(xa + k) : make_uint4(0, 0, 0, 0);
          const uint4 vb = mb < p.n ? *reinterpret_cast<const uint4*>(xb + k) : make_uint4(0, 0, 0, 0);
          ra[0] = va.x; ra[1] = va.y; ra[2] = va.z; ra[3] = va.w;
          rb[0] = vb.x; rb[1] = vb.y; rb[2] = vb.z; rb[3] = vb.w;
        } else {
          const uint2 va = ma < p.n ? *reinterpret_cast<const uint2*>(xa + k) : make_uint2(0, 0);
          const uint2 vb = mb < p.n ? *reinterpret_cast<const uint2*>(xb + k) : make_uint2(0, 0);
          ra[0] = va.x; ra[1] = va.y;
          rb[0] = vb.x; rb[1] = vb.y;
        }
#pragma unroll
        for (int i = 0; i < KG; ++i) {
          xav[i] = static_cast<double>((i & 1) ? bf16hi(ra[i >> 1]) : bf16lo(ra[i >> 1]));
          xbv[i] = static_cast<double>((i & 1) ? bf16hi(rb[i >> 1]) : bf16lo(rb[i >> 1]));
        }
      }
      RowChunk<WDT> wr[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int e = e0 + 8 * j + g;
        if (e < p.E)
          wr[j].load(p.w, e, p.H, k);
        else
          wr[j].zero();
      }
#pragma unroll
      for (int i = 0; i < KG; ++i) {
#pragma unroll
        for (int j = 0; j < 8; ++j) dmma_16x8x4(acc[j], xav[i], xbv[i], static_cast<double>(wr[j].get(i, sc[j])));
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      part[warp][g][8 * j + 2 * t] = acc[j][0];
      part[warp][g][8 * j + 2 * t + 1] = acc[j][1];
      part[warp][g + 8][8 * j + 2 * t] = acc[j][2];
      part[warp][g + 8][8 * j + 2 * t + 1] = acc[j][3];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kDM * kDE; i += blockDim.x) {
      const int r = i / kDE, c = i % kDE;
      const int m = m0 + r, e = e0 + c;
      if (m < p.n && e < p.E) {
        double v = part[0][r][c];
#pragma unroll
        for (int w2 = 1; w2 < kDWarps; ++w2) v += part[w2][r][c];
        p.logits[static_cast<long long>(m) * p.E + e] = static_cast<float>(v);
      }
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(256) route_select_kernel(const Params p) {
  __shared__ float scr[8][kMaxE];
  const int warp = threadIdx.x >> 5;
  const int m = blockIdx.x * 8 + warp;
  if (m >= p.n) return;
  select_token(p, m, p.logits + static_cast<long long>(m) * p.E, scr[warp]);
}

}  // namespace route

// Internal launcher shared with the fused block entry points.
int route_launch(const route::Params& p, cudaStream_t st, bool pdl_primary) {
  using namespace route;
  (void)pdl_primary;
  if (p.n <= kSmallM) {
    const size_t smem = static_cast<size_t>(kSmallM) * p.H * 2 + 8 * 8 + 8 * kMaxE * 4;
    cudaError_t e = cudaFuncSetAttribute(route_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(route_small)");
    route_small_kernel<<<(p.E + 7) / 8, 256, smem, st>>>(p);
    return cuda_status(cudaGetLastError(), "route_small launch");
  }
  if (p.norm_w != nullptr) return fail(MV_ERR_UNSUPPORTED, "route: fused RMSNorm only for n <= 16");
  if (p.H % 128 == 0 && aligned16(p.x) && (p.x_stride * 2) % 16 == 0) {
    const unsigned int blocks = static_cast<unsigned int>((p.n + kDM - 1) / kDM);
    if (p.w_dtype == MV_BF16)
      route_logits_dmma_kernel<MV_BF16><<<blocks, 128, 0, st>>>(p);
    else if (p.w_dtype == MV_F32)
      route_logits_dmma_kernel<MV_F32><<<blocks, 128, 0, st>>>(p);
    else
      route_logits_dmma_kernel<MV_I8><<<blocks, 128, 0, st>>>(p);
  } else {
    dim3 grid((p.n + kTM - 1) / kTM, (p.E + kTE - 1) / kTE);
    route_logits_kernel<<<grid, 256, 0, st>>>(p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "route_logits launch");
  route_select_kernel<<<(p.n + 7) / 8, 256, 0, st>>>(p);
  return cuda_status(cudaGetLastError(), "route_select launch");
}

int route_check(const route::Params& p) {
  if (p.mode != MV_ROUTE_SOFTMAX && p.mode != MV_ROUTE_SIGMOID_GROUP) return fail(MV_ERR_INVALID, "route: bad mode");
  if (p.x == nullptr || p.w == nullptr || p.ids == nullptr || p.wts == nullptr)
    return fail(MV_ERR_INVALID, "route: null pointer");
  if (p.n < 0 || p.H <= 0 || p.E <= 0 || p.E > route::kMaxE)
    return fail(MV_ERR_INVALID, "route: bad sizes n=%d H=%d E=%d (E <= %d)", p.n, p.H, p.E, route::kMaxE);
  if (p.top_k < 1 || p.top_k > p.E || p.top_k > 32 || p.n_shared < 0 || p.top_k + p.n_shared > 32)
    return fail(MV_ERR_INVALID, "route: bad top_k=%d / n_shared=%d", p.top_k, p.n_shared);
  if (p.w_dtype != MV_F32 && p.w_dtype != MV_BF16 && p.w_dtype != MV_I8)
    return fail(MV_ERR_UNSUPPORTED, "route: router weight must be f32, bf16 or i8");
  if (p.w_dtype == MV_I8 && p.w_scale == nullptr) return fail(MV_ERR_INVALID, "route: int8 router needs w_scale");
  if (p.mode == MV_ROUTE_SIGMOID_GROUP) {
    if (p.n_group < 1 || p.n_group > 32 || p.E % p.n_group != 0 || p.topk_group < 1 || p.topk_group > p.n_group)
      return fail(MV_ERR_INVALID, "route: bad n_group=%d / topk_group=%d", p.n_group, p.topk_group);
    if (p.E / p.n_group < 2 && p.n_group > 1) return fail(MV_ERR_INVALID, "route: groups need >= 2 experts");
    if (p.top_k > p.topk_group * (p.E / p.n_group)) return fail(MV_ERR_INVALID, "route: top_k exceeds kept experts");
  }
  {
    const int esz = p.w_dtype == MV_F32 ? 4 : (p.w_dtype == MV_BF16 ? 2 : 1);
    if (!aligned16(p.w) || (static_cast<long long>(p.H) * esz) % 16)
      return fail(MV_ERR_ALIGN, "route: router weight rows must be 16-byte aligned");
  }
  if (p.n <= route::kSmallM && static_cast<size_t>(route::kSmallM) * p.H * 2 + 8 * 8 + 8 * route::kMaxE * 4 > 200 * 1024)
    return fail(MV_ERR_INVALID, "route: H=%d too large", p.H);
  return MV_OK;
}

}  // namespace mv

using namespace mv;

extern "C" size_t mv_route_workspace_bytes(int n_tokens, int E) {
  return kWsHeaderBytes + static_cast<size_t>(n_tokens > 0 ? n_tokens : 1) * (E > 0 ? E : 1) * sizeof(float);
}

extern "C" int mv_route(int mode, const void* x, long long x_stride, const void* w, int w_dtype, const void* w_scale,
                        int scale_dtype, const float* bias, int n_tokens, int H, int E, int top_k, int n_group,
                        int topk_group, double scale, int n_shared, int shared_id, float* logits_out, void* ids_out,
                        int ids_dtype, float* wts_out, void* workspace, size_t workspace_bytes, void* stream) {
  route::Params p{};
  p.mode = mode;
  p.x = static_cast<const uint16_t*>(x);
  p.x_stride = x_stride;
  p.w = w;
  p.w_dtype = w_dtype;
  p.w_scale = w_scale;
  p.scale_bf16 = scale_dtype == MV_BF16;
  p.bias = bias;
  p.n = n_tokens;
  p.H = H;
  p.E = E;
  p.top_k = top_k;
  p.n_group = n_group;
  p.topk_group = topk_group;
  p.scale = scale;
  p.n_shared = n_shared;
  p.shared_id = shared_id;
  p.ids = ids_out;
  p.ids_i64 = ids_dtype == MV_I64;
  p.wts = wts_out;
  int rc = route_check(p);
  if (rc != MV_OK) return rc;
  if (ids_dtype != MV_I32 && ids_dtype != MV_I64) return fail(MV_ERR_INVALID, "mv_route: ids must be i32 or i64");
  if (x_stride < H) return fail(MV_ERR_INVALID, "mv_route: x_stride < H");
  if (workspace == nullptr || workspace_bytes < mv_route_workspace_bytes(n_tokens, E))
    return fail(MV_ERR_WORKSPACE, "mv_route: workspace of %zu bytes needed", mv_route_workspace_bytes(n_tokens, E));
  if (n_tokens == 0) return MV_OK;
  p.ws = static_cast<WsHeader*>(workspace);
  p.logits = logits_out ? logits_out : reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWsHeaderBytes);
  return route_launch(p, static_cast<cudaStream_t>(stream), false);
}
