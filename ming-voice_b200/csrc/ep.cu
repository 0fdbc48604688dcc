// Expert-parallel prefill: the device side of one rank's dispatch and combine (the exchange itself is two NCCL
// all-to-alls of fixed size issued by the host, wire rows out and bf16 outputs back; nothing here synchronises
// the host).
//
// Placement (ming-voice is single-GPU, engine.py:34; expert parallelism is new): every rank holds the router,
// the norm, the shared-expert slots and the replicated hot experts; each other ("cold") expert lives on one rank.
// owner[e] = the rank holding routed expert e (-1: replicated, i.e. this rank), slot[e] = its index in the
// holding rank's stacks.
//
//   mv_ep_plan      (one CTA) every routed pair of this rank's tokens, in token order: a pair whose expert lives
//                   here keeps its local slot id; any other pair gets id -1 locally and a place j < cap in the
//                   send block of its owner d (deterministic: pairs keep their token order per owner). Writes the
//                   per-owner (slot, weight) metadata with the count in entry cap of each block, the source token
//                   of each place, and pos[n, k] = d * cap + j (-1 for local pairs). More than cap pairs for one
//                   owner: the excess pairs are dropped and the capacity error is raised in the workspace.
//   mv_ep_pack      rows of the normalised tokens into the send blocks (one warp per place). A wire row is the H
//                   bf16 values and a 16-byte tail (slot, weight, in-use flag), so rows and their metadata cross
//                   in ONE all-to-all; a place past the count gets only its tail (flag 0).
//   mv_ep_unpack    received tails -> ids / weights of the received rows (id -1 for unused places).
//   mv_ep_narrow    the received rows' fp32 outputs (one weighted pair each) to bf16 for the return exchange.
//   mv_ep_combine   out[n] = bf16(x[n] + y_local[n] + sum over n's remote pairs, in k order, of their returned
//                   outputs), added in fp32 and rounded once.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace mv {
namespace ep {

constexpr int kMaxWorld = 8;
constexpr int kPlanThreads = 1024;

// STAGED: the routed ids and weights, the owner table and the slot table are first copied into shared memory
// (coalesced, 8 loads in flight per thread), so the two per-thread passes over contiguous pair ranges (which keep
// the token order) read shared memory only; unstaged, every pair costs dependent global loads in the pass loops
// (the one-CTA plan took ~45 us for 12 K pairs that way).
template <bool STAGED>
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int* __restrict__ ids, const float* __restrict__ wts,
                                                            int N, int NK, int K, const int* __restrict__ owner,
                                                            const int* __restrict__ slot, int E, int rank, int world,
                                                            int cap, int* __restrict__ ids_local,
                                                            float* __restrict__ wts_local, int* __restrict__ pos,
                                                            int* __restrict__ send_src, int* __restrict__ send_meta,
                                                            WsHeader* ws) {
  __shared__ int s_warp[kPlanThreads / 32][kMaxWorld];
  __shared__ int s_base[kMaxWorld];
  extern __shared__ int s_dyn[];  // STAGED: [E] owner, [E] slot, [N * K] routed ids, [N * K] weights, [N * K] pos
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const long long P = static_cast<long long>(N) * K;
  const long long chunk = (P + kPlanThreads - 1) / kPlanThreads;
  const long long p0 = chunk * t, p1 = min(P, p0 + chunk);
  int* s_owner = s_dyn;
  int* s_slot = s_dyn + E;
  int* s_ids = s_dyn + 2 * E;
  float* s_wts = reinterpret_cast<float*>(s_dyn + 2 * E + P);
  int* s_pos = s_dyn + 2 * E + 2 * P;
  if (STAGED) {
    for (int e = t; e < E; e += kPlanThreads) {
      s_owner[e] = owner[e];
      s_slot[e] = slot[e];
    }
    constexpr int kB = 8;  // loads in flight per thread
    for (long long q0 = t; q0 < P; q0 += kB * kPlanThreads) {
      int iv[kB];
      float wv[kB];
#pragma unroll
      for (int u = 0; u < kB; ++u) {
        const long long q = q0 + static_cast<long long>(u) * kPlanThreads;
        const long long iq = (q / K) * NK + q % K;
        iv[u] = q < P ? ids[iq] : 0;
        wv[u] = q < P ? wts[iq] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kB; ++u) {
        const long long q = q0 + static_cast<long long>(u) * kPlanThreads;
        if (q < P) {
          s_ids[q] = iv[u];
          s_wts[q] = wv[u];
        }
      }
    }
    __syncthreads();
  }
  auto id_at = [&](long long q) { return STAGED ? s_ids[q] : ids[(q / K) * NK + q % K]; };
  auto wt_at = [&](long long q, long long iq) { return STAGED ? s_wts[q] : wts[iq]; };
  auto owner_of = [&](int e) { return STAGED ? s_owner[e] : owner[e]; };
  auto slot_of = [&](int e) { return STAGED ? s_slot[e] : slot[e]; };
  // pass 1: this thread's pairs per owner
  int cnt[kMaxWorld];
#pragma unroll
  for (int d = 0; d < kMaxWorld; ++d) cnt[d] = 0;
  for (long long q = p0; q < p1; ++q) {
    const int e = id_at(q);
    const int d = (e >= 0 && e < E) ? owner_of(e) : -1;
    if (d >= 0 && d != rank) {
#pragma unroll
      for (int dd = 0; dd < kMaxWorld; ++dd) cnt[dd] += dd == d ? 1 : 0;
    }
  }
  // exclusive prefix over threads, per owner (warp shuffles, then the warp totals)
  int pre[kMaxWorld];
#pragma unroll
  for (int d = 0; d < kMaxWorld; ++d) {
    int v = cnt[d];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    pre[d] = v - cnt[d];
    if (lane == 31) s_warp[warp][d] = v;
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int d = 0; d < kMaxWorld; ++d) {
      const int tot = s_warp[lane][d];
      int v = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      s_warp[lane][d] = v - tot;
      if (lane == 31) s_base[d] = v;
    }
  }
  __syncthreads();
  int off[kMaxWorld];
#pragma unroll
  for (int d = 0; d < kMaxWorld; ++d) off[d] = s_warp[warp][d] + pre[d];
  // pass 2: ids / weights of the local pass, places of the remote pairs
  for (long long q = p0; q < p1; ++q) {
    const int n = static_cast<int>(q / K), k = static_cast<int>(q % K);
    const long long iq = static_cast<long long>(n) * NK + k;
    const int e = id_at(q);
    const int d = (e >= 0 && e < E) ? owner_of(e) : rank;
    int pq = -1;
    if (e >= 0 && e < E && d != rank && d >= 0) {
      int j = 0;
#pragma unroll
      for (int dd = 0; dd < kMaxWorld; ++dd)
        if (dd == d) j = off[dd]++;
      if (j < cap) {
        send_src[d * cap + j] = n;
        send_meta[(static_cast<long long>(d) * (cap + 1) + j) * 2] = slot_of(e);
        send_meta[(static_cast<long long>(d) * (cap + 1) + j) * 2 + 1] = __float_as_int(wt_at(q, iq));
        pq = d * cap + j;
      } else {
        raise_error(ws, kErrOverflow, static_cast<unsigned int>(d));
      }
      if (STAGED) {  // in place: this thread has read pair q; the staged arrays are copied out below
        s_ids[q] = -1;
        s_wts[q] = 0.f;
      } else {
        ids_local[iq] = -1;
        wts_local[iq] = 0.f;
      }
    } else {
      const int il = (e >= 0 && e < E) ? slot_of(e) : -1;
      const float wl = wt_at(q, iq);
      if (STAGED) {
        s_ids[q] = il;
        s_wts[q] = wl;
      } else {
        ids_local[iq] = il;
        wts_local[iq] = wl;
      }
    }
    if (STAGED)
      s_pos[q] = pq;
    else
      pos[static_cast<long long>(n) * K + k] = pq;
  }
  if (STAGED) {  // the local ids / weights and the places, copied out coalesced (a thread's pairs are contiguous,
                 // so stores straight from the pass above would touch a different line per lane)
    __syncthreads();
    for (long long q = t; q < P; q += kPlanThreads) {
      const long long iq = (q / K) * NK + q % K;
      ids_local[iq] = s_ids[q];
      wts_local[iq] = s_wts[q];
      pos[q] = s_pos[q];
    }
  }
  // the shared-expert columns (k >= K) keep their (local) ids and weights
  for (long long q = t; q < static_cast<long long>(N) * (NK - K); q += kPlanThreads) {
    const long long iq = (q / (NK - K)) * NK + K + q % (NK - K);
    ids_local[iq] = ids[iq];
    wts_local[iq] = wts[iq];
  }
  if (t < world) send_meta[(static_cast<long long>(t) * (cap + 1) + cap) * 2] = min(s_base[t], cap);
}

// one warp per send place (d, j): row send_src[d, j] of xn and its tail -> wire row d * cap + j of send_rows
// (row stride H + 8 elements); a place past the count gets only a tail with flag 0
__global__ void __launch_bounds__(256) pack_kernel(const uint16_t* __restrict__ xn, long long x_stride, int H,
                                                   const int* __restrict__ send_src, const int* __restrict__ send_meta,
                                                   int world, int cap, uint16_t* __restrict__ send_rows) {
  const int lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(world) * cap;
  const int HW = H + 8;
  for (long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total;
       w += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const int d = static_cast<int>(w / cap), j = static_cast<int>(w % cap);
    const bool used = j < send_meta[(static_cast<long long>(d) * (cap + 1) + cap) * 2];
    uint4* dst = reinterpret_cast<uint4*>(send_rows + w * HW);
    if (used) {
      const uint4* src = reinterpret_cast<const uint4*>(xn + static_cast<long long>(send_src[w]) * x_stride);
      for (int v = lane; v < H / 8; v += 32) dst[v] = src[v];
    }
    if (lane == 0) {
      const long long m = (static_cast<long long>(d) * (cap + 1) + j) * 2;
      dst[H / 8] = used ? make_uint4(static_cast<uint32_t>(send_meta[m]), static_cast<uint32_t>(send_meta[m + 1]), 1u, 0u)
                        : make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// received wire rows' tails -> ids / weights of the received rows: column 0 the pair, the other columns -1
__global__ void __launch_bounds__(256) unpack_kernel(const uint16_t* __restrict__ recv_rows, int H, long long rows,
                                                     int NK, int* __restrict__ ids, float* __restrict__ wts) {
  const long long total = rows * NK;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / NK;
    const int col = static_cast<int>(i % NK);
    const uint4 tail = reinterpret_cast<const uint4*>(recv_rows + row * (H + 8))[H / 8];
    const bool valid = col == 0 && tail.z == 1u;
    ids[i] = valid ? static_cast<int>(tail.x) : -1;
    wts[i] = valid ? __uint_as_float(tail.y) : 0.f;
  }
}

// The remote rows' outputs to bf16 for the return exchange: out[i] = bf16(y[i]), 8 values per thread. A received
// row carries exactly one pair, so this is that pair's weighted output rounded once -- the rounding the
// reference's grouped GEMM applies to every pair's output (its bf16 output cache) -- and it halves the bytes
// that cross NVLink on the way back.
__global__ void __launch_bounds__(256) narrow_kernel(const float* __restrict__ y, long long n8,
                                                     uint4* __restrict__ out) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(y)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(y)[2 * i + 1];
    uint4 o;
    o.x = static_cast<uint32_t>(f2bf(a.x)) | (static_cast<uint32_t>(f2bf(a.y)) << 16);
    o.y = static_cast<uint32_t>(f2bf(a.z)) | (static_cast<uint32_t>(f2bf(a.w)) << 16);
    o.z = static_cast<uint32_t>(f2bf(b.x)) | (static_cast<uint32_t>(f2bf(b.y)) << 16);
    o.w = static_cast<uint32_t>(f2bf(b.z)) | (static_cast<uint32_t>(f2bf(b.w)) << 16);
    out[i] = o;
  }
}

// four returned values of row pq at column group c, as fp32 (fp32 or bf16 rows)
template <bool B16>
__device__ __forceinline__ float4 back4(const void* back, long long pq, int H, int c) {
  if (B16) {
    const uint2 v = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(back) + pq * H)[c];
    return make_float4(bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y));
  }
  return reinterpret_cast<const float4*>(static_cast<const float*>(back) + pq * H)[c];
}

// out[n, 4c..4c+3] = bf16(x + y_local + the returned outputs of n's remote pairs in k order)
template <bool B16>
__global__ void __launch_bounds__(256) combine_kernel(const uint16_t* __restrict__ x, long long x_stride,
                                                      const float* __restrict__ y_local, const void* __restrict__ back,
                                                      const int* __restrict__ pos, int N, int K, int H,
                                                      uint16_t* __restrict__ out) {
  const int h4 = H / 4;
  const long long total = static_cast<long long>(N) * h4;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i / h4), c = static_cast<int>(i % h4);
    const uint2 xv = reinterpret_cast<const uint2*>(x + static_cast<long long>(n) * x_stride)[c];
    const float4 yl = reinterpret_cast<const float4*>(y_local + static_cast<long long>(n) * H)[c];
    float v0 = bf16lo(xv.x) + yl.x, v1 = bf16hi(xv.x) + yl.y, v2 = bf16lo(xv.y) + yl.z, v3 = bf16hi(xv.y) + yl.w;
    for (int k = 0; k < K; ++k) {
      const int pq = pos[static_cast<long long>(n) * K + k];
      if (pq < 0) continue;
      const float4 b = back4<B16>(back, pq, H, c);
      v0 += b.x;
      v1 += b.y;
      v2 += b.z;
      v3 += b.w;
    }
    uint2 o;
    o.x = static_cast<uint32_t>(f2bf(v0)) | (static_cast<uint32_t>(f2bf(v1)) << 16);
    o.y = static_cast<uint32_t>(f2bf(v2)) | (static_cast<uint32_t>(f2bf(v3)) << 16);
    reinterpret_cast<uint2*>(out + static_cast<long long>(n) * H)[c] = o;
  }
}

}  // namespace ep
}  // namespace mv

using namespace mv;

extern "C" size_t mv_ep_workspace_bytes(void) { return kWsHeaderBytes; }

extern "C" int mv_ep_plan(const int* ids, const float* wts, int N, int NK, int K, const int* owner, const int* slot,
                          int E, int rank, int world, int cap, int* ids_local, float* wts_local, int* pos,
                          int* send_src, int* send_meta, void* workspace, size_t workspace_bytes, void* stream) {
  if (ids == nullptr || wts == nullptr || owner == nullptr || slot == nullptr || ids_local == nullptr ||
      wts_local == nullptr || pos == nullptr || send_src == nullptr || send_meta == nullptr)
    return fail(MV_ERR_INVALID, "mv_ep_plan: null pointer argument");
  if (world < 1 || world > ep::kMaxWorld || rank < 0 || rank >= world)
    return fail(MV_ERR_INVALID, "mv_ep_plan: rank %d of world %d (at most %d ranks)", rank, world, ep::kMaxWorld);
  if (N < 0 || K < 1 || NK < K || E < 1 || cap < 1) return fail(MV_ERR_INVALID, "mv_ep_plan: bad shape");
  if (workspace == nullptr || workspace_bytes < kWsHeaderBytes)
    return fail(MV_ERR_WORKSPACE, "mv_ep_plan: workspace of %zu bytes needed", kWsHeaderBytes);
  const size_t dyn = (2 * static_cast<size_t>(E) + 3 * static_cast<size_t>(N) * K) * sizeof(int);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dyn <= 200 * 1024) {  // ids, weights, places, owner and slot tables staged in shared memory
    cudaError_t e = cudaFuncSetAttribute(ep::plan_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(dyn));
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(ep plan)");
    ep::plan_kernel<true><<<1, ep::kPlanThreads, dyn, st>>>(ids, wts, N, NK, K, owner, slot, E, rank, world, cap,
                                                            ids_local, wts_local, pos, send_src, send_meta,
                                                            static_cast<WsHeader*>(workspace));
  } else {
    ep::plan_kernel<false><<<1, ep::kPlanThreads, 0, st>>>(ids, wts, N, NK, K, owner, slot, E, rank, world, cap,
                                                           ids_local, wts_local, pos, send_src, send_meta,
                                                           static_cast<WsHeader*>(workspace));
  }
  return cuda_status(cudaGetLastError(), "mv_ep_plan launch");
}

extern "C" int mv_ep_pack(const void* xn, long long x_stride, int H, const int* send_src, const int* send_meta,
                          int world, int cap, void* send_rows, void* stream) {
  if (xn == nullptr || send_src == nullptr || send_meta == nullptr || send_rows == nullptr)
    return fail(MV_ERR_INVALID, "mv_ep_pack: null pointer argument");
  if (H % 8 || x_stride % 8 || !aligned16(xn) || !aligned16(send_rows))
    return fail(MV_ERR_ALIGN, "mv_ep_pack: 16-byte aligned rows needed");
  if (world < 1 || cap < 1) return fail(MV_ERR_INVALID, "mv_ep_pack: bad world / cap");
  const long long warps = static_cast<long long>(world) * cap;
  const unsigned int blocks = static_cast<unsigned int>((warps + 7) / 8 < 148 * 8 ? (warps + 7) / 8 : 148 * 8);
  ep::pack_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(xn), x_stride, H, send_src, send_meta, world, cap,
      static_cast<uint16_t*>(send_rows));
  return cuda_status(cudaGetLastError(), "mv_ep_pack launch");
}

extern "C" int mv_ep_unpack(const void* recv_rows, int H, int world, int cap, int NK, int* ids, float* wts,
                            void* stream) {
  if (recv_rows == nullptr || ids == nullptr || wts == nullptr) return fail(MV_ERR_INVALID, "mv_ep_unpack: null");
  if (H % 8 || !aligned16(recv_rows)) return fail(MV_ERR_ALIGN, "mv_ep_unpack: 16-byte aligned wire rows needed");
  const long long rows = static_cast<long long>(world) * cap;
  const long long total = rows * NK;
  const unsigned int blocks = static_cast<unsigned int>((total + 255) / 256 < 148 * 4 ? (total + 255) / 256 : 148 * 4);
  ep::unpack_kernel<<<blocks > 0 ? blocks : 1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(recv_rows), H, rows, NK, ids, wts);
  return cuda_status(cudaGetLastError(), "mv_ep_unpack launch");
}

extern "C" int mv_ep_narrow(const float* y, long long n, void* out, void* stream) {
  if (y == nullptr || out == nullptr) return fail(MV_ERR_INVALID, "mv_ep_narrow: null pointer argument");
  if (n < 0 || n % 8 || !aligned16(y) || !aligned16(out)) return fail(MV_ERR_ALIGN, "mv_ep_narrow: 8k values, aligned");
  if (n == 0) return MV_OK;
  const long long n8 = n / 8;
  const unsigned int blocks = static_cast<unsigned int>((n8 + 255) / 256 < 148 * 8 ? (n8 + 255) / 256 : 148 * 8);
  ep::narrow_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, n8, static_cast<uint4*>(out));
  return cuda_status(cudaGetLastError(), "mv_ep_narrow launch");
}

extern "C" int mv_ep_combine(const void* x, long long x_stride, const float* y_local, const void* back,
                             int back_dtype, const int* pos, int N, int K, int H, void* out, void* stream) {
  if (x == nullptr || y_local == nullptr || back == nullptr || pos == nullptr || out == nullptr)
    return fail(MV_ERR_INVALID, "mv_ep_combine: null pointer argument");
  if (back_dtype != MV_F32 && back_dtype != MV_BF16)
    return fail(MV_ERR_UNSUPPORTED, "mv_ep_combine: returned outputs must be f32 or bf16");
  if (H % 4 || x_stride % 4 || !aligned16(y_local) || !aligned16(back))
    return fail(MV_ERR_ALIGN, "mv_ep_combine: aligned rows needed");
  if (N == 0) return MV_OK;
  const long long total = static_cast<long long>(N) * H / 4;
  const unsigned int blocks = static_cast<unsigned int>((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
  if (back_dtype == MV_BF16)
    ep::combine_kernel<true><<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(x), x_stride, y_local, back, pos, N, K, H, static_cast<uint16_t*>(out));
  else
    ep::combine_kernel<false><<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(x), x_stride, y_local, back, pos, N, K, H, static_cast<uint16_t*>(out));
  return cuda_status(cudaGetLastError(), "mv_ep_combine launch");
}
