// Small-M linear layer: y = act(norm?(x) @ W^T + b) + residual for M <= 16 rows.
//
// mv_small_linear replaces fastlinear.small_linear's kernel path (ming-voice fastlinear.py:142-174, Triton
// kernel _small_m_linear :20-62), used for the Talker's Qwen2 step and the shared expert of the thinker.
// The layer is weight streaming: W [N, K] bf16 is read once. The (optionally RMS-normalised) rows of x sit in
// shared memory; each warp owns whole output rows n and reads W[n] with every 16-byte load of the row in
// flight before the first use, accumulating all M rows of x in fp32.
//
// Numerics as the reference (fastlinear.py:29-61): the RMSNorm prologue is rstd = 1/sqrt(mean(x^2) + eps)
// (fp32 statistics; here the sum of squares is fp64, i.e. exact and order-independent), x_n =
// bf16(bf16(x * rstd) * gamma); with an activation the pre-activation (accumulator + bias) is rounded to bf16
// first; with a residual the activation output is rounded to bf16 before the add; the result is bf16.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace mv {
namespace sl {

constexpr int kThreads = 256;
constexpr int kMaxM = 16;
constexpr int kMaxSmem = 200 * 1024;

template <int MT, int NB>  // MT: token rows (>= M); NB: 16-byte chunks of a W row per lane per batch
__global__ void __launch_bounds__(kThreads) small_linear_kernel(const uint16_t* __restrict__ x, long long x_stride,
                                                                const uint16_t* __restrict__ w, long long w_stride,
                                                                const uint16_t* __restrict__ bias,
                                                                const uint16_t* __restrict__ res, long long r_stride,
                                                                const uint16_t* __restrict__ gamma, float eps, int act,
                                                                uint16_t* __restrict__ y, long long y_stride, int M,
                                                                int N, int K) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);  // [M][K] bf16
  __shared__ double red[kThreads / 32][kMaxM];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nch = K / 8;

  // ---- prologue: x (RMS-normalised when gamma is given) into shared memory
  for (int i = tid; i < M * nch; i += kThreads) {
    const int m = i / nch, c = i % nch;
    reinterpret_cast<uint4*>(xs + m * K)[c] = reinterpret_cast<const uint4*>(x + m * x_stride)[c];
  }
  __syncthreads();
  if (gamma != nullptr) {
    for (int m = warp; m < M; m += kThreads / 32) {
      double ss = 0.0;
      for (int c = lane; c < nch; c += 32) {
        const uint4 v = reinterpret_cast<const uint4*>(xs + m * K)[c];
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const double a = bf16lo(vv[q]), b = bf16hi(vv[q]);
          ss += a * a + b * b;
        }
      }
      ss = warp_sum_d(ss);
      if (lane == 0) red[warp][m] = ss;
    }
    __syncthreads();
    for (int i = tid; i < M * nch; i += kThreads) {
      const int m = i / nch, c = i % nch;
      const double ss = red[m % (kThreads / 32)][m];  // (token m was summed by warp m % 8)
      const float var = static_cast<float>(ss / static_cast<double>(K));
      const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
      uint4* p = reinterpret_cast<uint4*>(xs + m * K) + c;
      const uint4 v = *p;
      const uint4 g = reinterpret_cast<const uint4*>(gamma)[c];
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
      *p = make_uint4(o[0], o[1], o[2], o[3]);
    }
    __syncthreads();
  }

  // ---- main loop: one warp per output row
  const int gw = blockIdx.x * (kThreads / 32) + warp;
  const int nw = gridDim.x * (kThreads / 32);
  for (int n = gw; n < N; n += nw) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + static_cast<long long>(n) * w_stride);
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    for (int c0 = 0; c0 < nch; c0 += 32 * NB) {
      uint4 buf[NB];
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const int c = c0 + lane + 32 * j;
        if (c < nch) buf[j] = ld_nc_v4(wr + c);
      }
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const int c = c0 + lane + 32 * j;
        if (c >= nch) break;
        const uint32_t ww[4] = {buf[j].x, buf[j].y, buf[j].z, buf[j].w};
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m >= M) break;
          const uint4 xv = reinterpret_cast<const uint4*>(xs + m * K)[c];
          const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[m] = fmaf(bf16lo(ww[q]), bf16lo(xx[q]), acc[m]);
            acc[m] = fmaf(bf16hi(ww[q]), bf16hi(xx[q]), acc[m]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m >= M) break;
      const float s = warp_sum(acc[m]);
      if (lane == m % 32) {
        float v = s;
        if (bias != nullptr) v += __uint_as_float(static_cast<uint32_t>(bias[n]) << 16);
        if (act == 1) {  // gelu, tanh approximation, on the bf16-rounded pre-activation
          const float a = round_bf16(v);
          const float c = 0.7978845608028654f * (a + 0.044715f * a * a * a);
          v = 0.5f * a * (1.0f + tanhf(c));
        } else if (act == 2) {  // silu on the bf16-rounded pre-activation
          const float a = round_bf16(v);
          v = a / (1.0f + expf(-a));
        }
        if (res != nullptr) v = round_bf16(v) + __uint_as_float(static_cast<uint32_t>(res[m * r_stride + n]) << 16);
        y[m * y_stride + n] = f2bf(v);
      }
    }
  }
}

template <int MT>
static int launch_mt(int NB, unsigned int grid, size_t smem, cudaStream_t st, const uint16_t* x, long long xs,
                     const uint16_t* w, long long ws, const uint16_t* b, const uint16_t* r, long long rs,
                     const uint16_t* g, float eps, int act, uint16_t* y, long long ys, int M, int N, int K) {
  void (*k)(const uint16_t*, long long, const uint16_t*, long long, const uint16_t*, const uint16_t*, long long,
            const uint16_t*, float, int, uint16_t*, long long, int, int, int) =
      NB == 8 ? small_linear_kernel<MT, 8> : small_linear_kernel<MT, 4>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(small_linear)");
  k<<<grid, kThreads, smem, st>>>(x, xs, w, ws, b, r, rs, g, eps, act, y, ys, M, N, K);
  return cuda_status(cudaGetLastError(), "small_linear launch");
}

}  // namespace sl
}  // namespace mv

using namespace mv;

extern "C" int mv_small_linear(const void* x, long long x_stride, const void* w, long long w_stride, const void* bias,
                               const void* residual, long long residual_stride, const void* norm_w, float eps,
                               int act, void* y, long long y_stride, int M, int N, int K, void* stream) {
  if (M == 0 || N == 0) return MV_OK;
  if (x == nullptr || w == nullptr || y == nullptr) return fail(MV_ERR_INVALID, "mv_small_linear: null pointer");
  if (M < 0 || M > sl::kMaxM || N < 0 || K <= 0 || K % 8 != 0)
    return fail(MV_ERR_INVALID, "mv_small_linear: M=%d (<= 16), N=%d, K=%d (multiple of 8)", M, N, K);
  if (act < 0 || act > 2) return fail(MV_ERR_INVALID, "mv_small_linear: act must be 0, 1 or 2");
  if (x_stride < K || w_stride < K || y_stride < N || (residual != nullptr && residual_stride < N))
    return fail(MV_ERR_INVALID, "mv_small_linear: bad strides");
  if (!aligned16(x) || !aligned16(w) || (x_stride * 2) % 16 || (w_stride * 2) % 16 ||
      (norm_w != nullptr && !aligned16(norm_w)))
    return fail(MV_ERR_ALIGN, "mv_small_linear: x, w, norm weight and row strides must be 16-byte aligned");
  const size_t smem = static_cast<size_t>(M) * K * 2;
  if (smem > static_cast<size_t>(sl::kMaxSmem))
    return fail(MV_ERR_UNSUPPORTED, "mv_small_linear: M*K=%d*%d too large for shared memory", M, K);
  const int G = num_sms();
  long long grid = (static_cast<long long>(N) + 7) / 8;
  if (grid > 4LL * G) grid = 4LL * G;
  const int NB = K >= 32 * 8 * 8 ? 8 : 4;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint16_t* xb = static_cast<const uint16_t*>(x);
  const uint16_t* wb = static_cast<const uint16_t*>(w);
  const uint16_t* bb = static_cast<const uint16_t*>(bias);
  const uint16_t* rb = static_cast<const uint16_t*>(residual);
  const uint16_t* gb = static_cast<const uint16_t*>(norm_w);
  uint16_t* yb = static_cast<uint16_t*>(y);
  const unsigned int g = static_cast<unsigned int>(grid);
  if (M == 1) return sl::launch_mt<1>(NB, g, smem, st, xb, x_stride, wb, w_stride, bb, rb, residual_stride, gb, eps, act, yb, y_stride, M, N, K);
  if (M <= 4) return sl::launch_mt<4>(NB, g, smem, st, xb, x_stride, wb, w_stride, bb, rb, residual_stride, gb, eps, act, yb, y_stride, M, N, K);
  if (M <= 8) return sl::launch_mt<8>(NB, g, smem, st, xb, x_stride, wb, w_stride, bb, rb, residual_stride, gb, eps, act, yb, y_stride, M, N, K);
  return sl::launch_mt<16>(NB, g, smem, st, xb, x_stride, wb, w_stride, bb, rb, residual_stride, gb, eps, act, yb, y_stride, M, N, K);
}
