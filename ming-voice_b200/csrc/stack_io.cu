// Loader and bucket helpers around the MoE block:
//
//  * mv_quantize_into_stack: one expert matrix (a checkpoint tensor as the loader streams it) quantised to int8
//    rows + per-row scales and written straight into its slot of the stacked [E1, rows, K] int8 tensor and the
//    [E1, rows] scale tensor -- the quantise-on-load hook of ming-voice (engine.py:126-147, called by the
//    loader threads of direct_load.py:109-135), without the intermediate q / scale tensors the reference
//    allocates and copies (engine.py:132-135).
//  * mv_mask_pad_rows: marks the expert pairs of padded rows (row >= *n_valid, read on the device) as "no pair"
//    (-1), so a prefill graph captured for a padded bucket length skips the padding in the expert GEMMs (the
//    bucket graphs of engine.py:716-757 / :950-961 run the padded rows through the whole block).
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace mv {
namespace {

template <typename T>
__global__ void mask_pad_rows_kernel(T* ids, int N, int NK, const int* n_valid) {
  const int nv = *n_valid;
  const long long total = static_cast<long long>(N) * NK;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    if (i / NK >= nv) ids[i] = static_cast<T>(-1);
}

}  // namespace
}  // namespace mv

using namespace mv;

extern "C" int mv_quantize_into_stack(const void* w, int w_dtype, long long w_stride, int rows, int K,
                                      int8_t* q_stack, void* s_stack, int s_dtype, int E1, int rows_per_expert,
                                      int e, int row_off, void* stream) {
  if (q_stack == nullptr || s_stack == nullptr || w == nullptr)
    return fail(MV_ERR_INVALID, "mv_quantize_into_stack: null pointer");
  if (s_dtype != MV_F32 && s_dtype != MV_BF16)
    return fail(MV_ERR_UNSUPPORTED, "mv_quantize_into_stack: scales must be f32 or bf16");
  if (E1 <= 0 || rows_per_expert <= 0 || K <= 0 || rows < 0)
    return fail(MV_ERR_INVALID, "mv_quantize_into_stack: bad stack shape");
  if (e < 0 || e >= E1 || row_off < 0 || static_cast<long long>(row_off) + rows > rows_per_expert)
    return fail(MV_ERR_INVALID, "mv_quantize_into_stack: rows [%d, %d) of slot %d outside the [%d, %d, %d] stack",
                row_off, row_off + rows, e, E1, rows_per_expert, K);
  const long long first_row = static_cast<long long>(e) * rows_per_expert + row_off;
  int8_t* q = q_stack + first_row * K;
  void* s = static_cast<uint8_t*>(s_stack) + first_row * (s_dtype == MV_F32 ? 4 : 2);
  return mv_quantize_rows_int8(w, w_dtype, w_stride, rows, K, q, s, s_dtype, stream);
}

extern "C" int mv_mask_pad_rows(void* ids, int ids_dtype, int N, int NK, const int* n_valid, void* stream) {
  if (ids == nullptr || n_valid == nullptr) return fail(MV_ERR_INVALID, "mv_mask_pad_rows: null pointer");
  if (ids_dtype != MV_I32 && ids_dtype != MV_I64) return fail(MV_ERR_INVALID, "mv_mask_pad_rows: ids must be i32/i64");
  if (N < 0 || NK <= 0) return fail(MV_ERR_INVALID, "mv_mask_pad_rows: bad shape N=%d NK=%d", N, NK);
  if (N == 0) return MV_OK;
  const long long total = static_cast<long long>(N) * NK;
  const unsigned int blocks = static_cast<unsigned int>(total / 256 + 1 < 148 ? total / 256 + 1 : 148);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (ids_dtype == MV_I32)
    mask_pad_rows_kernel<int><<<blocks, 256, 0, st>>>(static_cast<int*>(ids), N, NK, n_valid);
  else
    mask_pad_rows_kernel<long long><<<blocks, 256, 0, st>>>(static_cast<long long*>(ids), N, NK, n_valid);
  return cuda_status(cudaGetLastError(), "mv_mask_pad_rows launch");
}
