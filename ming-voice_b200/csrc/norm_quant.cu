// RMSNorm and the int8 row quantiser / dequantiser.
//
// mv_rmsnorm replaces fused_ops.rms_norm (ming-voice fused_ops.py:28-37, kernel _rms_norm :16-25).
// mv_quantize_rows_int8 replaces fused_moe.quantize_rows_int8 (fused_moe.py:199-204).
// Both are HBM-bound row kernels: one CTA per row for RMSNorm, one warp per row for the quantiser, 16-byte
// vector loads where the dtype allows.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace mv {

__device__ __forceinline__ float load_as_f32(const void* p, long long i, int dtype) {
  switch (dtype) {
    case MV_BF16:
      return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(p)[i]) << 16);
    case MV_F16:
      return __half2float(static_cast<const __half*>(p)[i]);
    default:
      return static_cast<const float*>(p)[i];
  }
}

// value cast to `dtype` (round to nearest even) and back to fp32
__device__ __forceinline__ float round_to(float v, int dtype) {
  switch (dtype) {
    case MV_BF16:
      return round_bf16(v);
    case MV_F16:
      return __half2float(__float2half_rn(v));
    default:
      return v;
  }
}

__device__ __forceinline__ void store_from_f32(void* p, long long i, float v, int dtype) {
  switch (dtype) {
    case MV_BF16:
      static_cast<uint16_t*>(p)[i] = f2bf(v);
      break;
    case MV_F16:
      static_cast<__half*>(p)[i] = __float2half_rn(v);
      break;
    default:
      static_cast<float*>(p)[i] = v;
  }
}

// y = cast(w * cast(x * (1 / sqrt(fp32(sum x^2 / n) + eps)), x_dtype), y_dtype)
// The sum of squares is accumulated in fp64 (exact for bf16/f16 inputs), and the reciprocal square root
// is 1/sqrt with IEEE-rounded sqrt and division, so the result is independent of the reduction order.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const void* __restrict__ x, int x_dtype, long long x_stride,
                                                      const void* __restrict__ w, int w_dtype, void* __restrict__ y,
                                                      int y_dtype, int n, float eps) {
  __shared__ double red[8];
  const long long row = blockIdx.x;
  const char* xr = static_cast<const char*>(x) + row * x_stride * elem_size_dev(x_dtype);
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const double v = load_as_f32(xr, i, x_dtype);
    ss += v * v;
  }
  ss = warp_sum_d(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  double tot = 0.0;
  for (int i = 0; i < (blockDim.x >> 5); ++i) tot += red[i];
  const float var = static_cast<float>(tot / static_cast<double>(n));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float yv = round_to(__fmul_rn(load_as_f32(xr, i, x_dtype), r), x_dtype);
    store_from_f32(y, row * n + i, __fmul_rn(load_as_f32(w, i, w_dtype), yv), y_dtype);
  }
}

// bf16 in / bf16 weight / bf16 out, n a multiple of 256 and <= 4096: one warp per row, the row held in
// registers (16-byte loads and stores). Same arithmetic as rmsnorm_kernel: the squares of bf16 values are
// exact in fp32 and their sum is taken in fp64, so the result does not depend on the summation order.
template <int NV>  // 16-byte vectors per lane: n = NV * 256
__global__ void __launch_bounds__(256) rmsnorm_bf16_warp_kernel(const uint16_t* __restrict__ x, long long x_stride,
                                                                const uint16_t* __restrict__ w,
                                                                uint16_t* __restrict__ y, int rows, int n, float eps) {
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * x_stride);
  uint4 v[NV];
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = xr[lane + 32 * i];
    const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = bf16lo(u[j]), b = bf16hi(u[j]);
      ss += static_cast<double>(a * a) + static_cast<double>(b * b);
    }
  }
  ss = warp_sum_d(ss);
  const float var = static_cast<float>(ss / static_cast<double>(n));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + row * n);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint4 wv = wr[lane + 32 * i];
    const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __fmul_rn(bf16lo(wu[j]), round_bf16(__fmul_rn(bf16lo(u[j]), r)));
      const float hi = __fmul_rn(bf16hi(wu[j]), round_bf16(__fmul_rn(bf16hi(u[j]), r)));
      o[j] = static_cast<uint32_t>(f2bf(lo)) | (static_cast<uint32_t>(f2bf(hi)) << 16);
    }
    yr[lane + 32 * i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// One warp per row: amax, scale = max(amax, 1e-8) / 127 (f32 or rounded to bf16), q = rint(w / scale).
__global__ void __launch_bounds__(256) quantize_rows_kernel(const void* __restrict__ w, int w_dtype,
                                                            long long w_stride, long long rows, int K,
                                                            int8_t* __restrict__ q, void* __restrict__ scale,
                                                            int scale_dtype) {
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const char* wr = static_cast<const char*>(w) + row * w_stride * elem_size_dev(w_dtype);
  float amax = 0.f;
  for (int i = lane; i < K; i += 32) amax = fmaxf(amax, fabsf(load_as_f32(wr, i, w_dtype)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1e-8f);
  float s = __fdiv_rn(amax, 127.0f);
  if (scale_dtype == MV_BF16) s = round_bf16(s);
  if (lane == 0) store_from_f32(scale, row, s, scale_dtype);
  int8_t* qr = q + row * K;
  for (int i = lane; i < K; i += 32) {
    float v = rintf(__fdiv_rn(load_as_f32(wr, i, w_dtype), s));
    v = fminf(fmaxf(v, -127.f), 127.f);
    qr[i] = static_cast<int8_t>(static_cast<int>(v));
  }
}

__global__ void dequant_rows_kernel(const int8_t* __restrict__ q, const void* __restrict__ scale, int scale_dtype,
                                    long long rows, int K, float* __restrict__ out) {
  const long long n = rows * K;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / K;
    const float s = load_as_f32(scale, r, scale_dtype);
    out[i] = dequant(static_cast<float>(q[i]), s);
  }
}

}  // namespace mv

using namespace mv;

static bool float_dtype(int d) { return d == MV_BF16 || d == MV_F16 || d == MV_F32; }

extern "C" int mv_rmsnorm(const void* x, int x_dtype, long long x_stride, const void* w, int w_dtype, void* y,
                          int y_dtype, int rows, int n, float eps, void* stream) {
  if (rows == 0 && n > 0) return MV_OK;
  if (x == nullptr || w == nullptr || y == nullptr) return fail(MV_ERR_INVALID, "mv_rmsnorm: null pointer");
  if (!float_dtype(x_dtype) || !float_dtype(w_dtype) || !float_dtype(y_dtype))
    return fail(MV_ERR_UNSUPPORTED, "mv_rmsnorm: dtypes must be bf16/f16/f32");
  if (rows < 0 || n <= 0 || x_stride < n) return fail(MV_ERR_INVALID, "mv_rmsnorm: bad shape rows=%d n=%d", rows, n);
  if (rows == 0) return MV_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == MV_BF16 && w_dtype == MV_BF16 && y_dtype == MV_BF16 && n % 256 == 0 && n <= 4096 && aligned16(x) &&
      aligned16(w) && aligned16(y) && (x_stride * 2) % 16 == 0) {
    const unsigned int blocks = static_cast<unsigned int>((rows + 7) / 8);
    const uint16_t* xb = static_cast<const uint16_t*>(x);
    const uint16_t* wb = static_cast<const uint16_t*>(w);
    uint16_t* yb = static_cast<uint16_t*>(y);
    switch (n / 256) {
#define MV_RMS_CASE(NV) \
  case NV:              \
    rmsnorm_bf16_warp_kernel<NV><<<blocks, 256, 0, st>>>(xb, x_stride, wb, yb, rows, n, eps); \
    break;
      MV_RMS_CASE(1) MV_RMS_CASE(2) MV_RMS_CASE(3) MV_RMS_CASE(4) MV_RMS_CASE(5) MV_RMS_CASE(6) MV_RMS_CASE(7)
      MV_RMS_CASE(8) MV_RMS_CASE(9) MV_RMS_CASE(10) MV_RMS_CASE(11) MV_RMS_CASE(12) MV_RMS_CASE(13)
      MV_RMS_CASE(14) MV_RMS_CASE(15) MV_RMS_CASE(16)
#undef MV_RMS_CASE
    }
    return cuda_status(cudaGetLastError(), "mv_rmsnorm launch");
  }
  rmsnorm_kernel<<<rows, 256, 0, st>>>(x, x_dtype, x_stride, w, w_dtype, y, y_dtype, n, eps);
  return cuda_status(cudaGetLastError(), "mv_rmsnorm launch");
}

extern "C" int mv_quantize_rows_int8(const void* w, int w_dtype, long long w_stride, long long rows, int K,
                                     int8_t* q, void* scale, int scale_dtype, void* stream) {
  if (w == nullptr || q == nullptr || scale == nullptr) return fail(MV_ERR_INVALID, "mv_quantize_rows_int8: null");
  if (!float_dtype(w_dtype)) return fail(MV_ERR_UNSUPPORTED, "mv_quantize_rows_int8: w must be bf16/f16/f32");
  if (scale_dtype != MV_F32 && scale_dtype != MV_BF16)
    return fail(MV_ERR_UNSUPPORTED, "mv_quantize_rows_int8: scale must be f32 or bf16");
  if (rows < 0 || K <= 0 || w_stride < K) return fail(MV_ERR_INVALID, "mv_quantize_rows_int8: bad shape");
  if (rows == 0) return MV_OK;
  const long long blocks = (rows + 7) / 8;
  if (blocks > 0x7fffffffLL) return fail(MV_ERR_INVALID, "mv_quantize_rows_int8: too many rows");
  quantize_rows_kernel<<<static_cast<unsigned int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      w, w_dtype, w_stride, rows, K, q, scale, scale_dtype);
  return cuda_status(cudaGetLastError(), "mv_quantize_rows_int8 launch");
}

extern "C" int mv_dequant_rows_int8(const int8_t* q, const void* scale, int scale_dtype, long long rows, int K,
                                    float* out, void* stream) {
  if (q == nullptr || scale == nullptr || out == nullptr) return fail(MV_ERR_INVALID, "mv_dequant_rows_int8: null");
  if (scale_dtype != MV_F32 && scale_dtype != MV_BF16)
    return fail(MV_ERR_UNSUPPORTED, "mv_dequant_rows_int8: scale must be f32 or bf16");
  if (rows < 0 || K <= 0) return fail(MV_ERR_INVALID, "mv_dequant_rows_int8: bad shape");
  if (rows == 0) return MV_OK;
  const long long n = rows * K;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  dequant_rows_kernel<<<static_cast<unsigned int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      q, scale, scale_dtype, rows, K, out);
  return cuda_status(cudaGetLastError(), "mv_dequant_rows_int8 launch");
}
