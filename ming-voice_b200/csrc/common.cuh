// Shared device helpers for the MoE block kernels (sm_100a).
//
// PTX wrappers for mbarriers, 1-D bulk (TMA) copies and bulk reductions, bf16 / int8 unpacking, the exact
// rounding helpers the parity contract relies on, and the bounded-wait policy: every spin on an mbarrier
// gives up after a wall-clock limit, records an error code in the call's workspace header and lets the
// CTA finish, so a bad transaction count can never hang the GPU.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mingmoe_internal.h"

namespace mv {

// ------------------------------------------------------------------------------------------ basic helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ int elem_size_dev(int dtype) {
  return dtype == MV_I8 ? 1 : (dtype == MV_BF16 || dtype == MV_F16) ? 2 : (dtype == MV_I64 ? 8 : 4);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// bf16 bit pattern -> fp32 (exact)
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// fp32 -> bf16 bits, round to nearest even (cvt.rn)
__device__ __forceinline__ uint16_t f2bf(float f) {
  __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&b);
}
__device__ __forceinline__ float round_bf16(float f) { return __uint_as_float(static_cast<uint32_t>(f2bf(f)) << 16); }

// Four signed int8 lanes of a 32-bit word -> exact fp32 values, using the IEEE-754 magic-number method:
// with the sign bit flipped (q ^ 0x80) each byte is an unsigned u = q + 128; placed in the low mantissa
// byte of 2^23 (bits 0x4B0000uu) it reads as 2^23 + u, and subtracting 2^23 + 128 leaves q exactly.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t hi = 0x4B000000u;
  uint32_t b0, b1, b2, b3;
  // selector nibbles pick bytes of {hi(7..4), u(3..0)}: result bytes = [u.byte_i, 0, 0, 0x4B]
  asm("prmt.b32 %0, %1, %2, 0x7540;" : "=r"(b0) : "r"(u), "r"(hi));
  asm("prmt.b32 %0, %1, %2, 0x7541;" : "=r"(b1) : "r"(u), "r"(hi));
  asm("prmt.b32 %0, %1, %2, 0x7542;" : "=r"(b2) : "r"(u), "r"(hi));
  asm("prmt.b32 %0, %1, %2, 0x7543;" : "=r"(b3) : "r"(u), "r"(hi));
  const float bias = 8388736.0f;  // 2^23 + 128
  f0 = __uint_as_float(b0) - bias;
  f1 = __uint_as_float(b1) - bias;
  f2 = __uint_as_float(b2) - bias;
  f3 = __uint_as_float(b3) - bias;
}

// The dequantisation every int8 path uses: torch's q.float() * s.float(), one correctly rounded fp32
// multiply (exported for bit-exact checking through mv_dequant_rows_int8).
__device__ __forceinline__ float dequant(float qf, float s) { return __fmul_rn(qf, s); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Named barrier over `nthreads` threads that also returns the AND of `pred` over them (one decision for all).
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<int>(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Named barrier over `nthreads` threads (a multiple of 32), id 1..15 (0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Arrive on a named barrier without waiting (producer / consumer hand-off: the waiting side uses named_bar).
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------------------------------ error flag

// Workspace header layout (first 256 bytes of every kernel workspace).
struct WsHeader {
  unsigned int counter;   // CTA arrival counter for last-CTA epilogues (reset by the last CTA)
  unsigned int error;     // first error code raised on the device (0 = none); sticky until cleared
  unsigned int err_info;  // where it was raised (kernel-specific)
  unsigned int bar1;      // grid-barrier arrival counters of cooperative kernels (reset by the last CTA)
  unsigned int bar2;
  unsigned int pad[3];
  unsigned long long gen1;  // generation grid barriers: count up by G per call, never reset (grid_arrive_gen)
  unsigned long long gen2;
  unsigned int pad2[52];
};
static_assert(sizeof(WsHeader) == 256, "workspace header must be 256 bytes");

__device__ __forceinline__ void raise_error(WsHeader* h, unsigned int code, unsigned int info) {
  if (h != nullptr && atomicCAS(&h->error, 0u, code) == 0u) atomicExch(&h->err_info, info);
}

// ------------------------------------------------------------------------------------------ mbarriers

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait (the hardware's own short, phase-completion-aware suspend; an explicit suspend-time hint measured
// slower: the waking warp came back late)
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// arrive on behalf of `count` threads / warps
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// d{0,1} = a{0,1} * b{0,1} + d{0,1}: one packed fp32 FMA (Blackwell f32x2), each lane correctly rounded
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rd, {%0, %1};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rd;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// d{0,1} = a{0,1} + b (packed, each lane correctly rounded: the same value as __fadd_rn)
__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1, float b) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b));
}

// Four signed int8 lanes of a 32-bit word -> exact fp32 values as i8x4_to_f32 does (the bytes placed in the low
// mantissa byte of 2^23 by byte permutes), with the bias removed by two packed adds instead of four.
__device__ __forceinline__ void i8x4_to_f32_packed(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t hi = 0x4B000000u;
  uint32_t b0, b1, b2, b3;
  asm("prmt.b32 %0, %1, %2, 0x7540;" : "=r"(b0) : "r"(u), "r"(hi));
  asm("prmt.b32 %0, %1, %2, 0x7541;" : "=r"(b1) : "r"(u), "r"(hi));
  asm("prmt.b32 %0, %1, %2, 0x7542;" : "=r"(b2) : "r"(u), "r"(hi));
  asm("prmt.b32 %0, %1, %2, 0x7543;" : "=r"(b3) : "r"(u), "r"(hi));
  const float nbias = -8388736.0f;  // -(2^23 + 128): exact sums
  fadd2(f0, f1, __uint_as_float(b0), __uint_as_float(b1), nbias);
  fadd2(f2, f3, __uint_as_float(b2), __uint_as_float(b3), nbias);
}

// d{0,1} = a{0,1} * s (packed, each lane correctly rounded: the same value as __fmul_rn)
__device__ __forceinline__ void fmul2(float& d0, float& d1, float a0, float a1, float s) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(s));
}

// Bounded wait for the phase with `parity` to complete. Returns false (and records kErrTimeout) when the
// phase has not completed within kWaitLimitNs of wall-clock time.
static __device__ __noinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, WsHeader* h, unsigned int info) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_error(h, kErrTimeout, info);
      return false;
    }
  }
}

// The same for waits that are expected to be long (a phase of another warp's work, not a ring slot): the
// spinning thread backs off with __nanosleep (64 ns doubling up to max_sleep_ns) so that it leaves the
// SM's issue slots to the warps doing the work.
static __device__ __noinline__ bool mbar_wait_lazy(uint64_t* bar, uint32_t parity, WsHeader* h, unsigned int info,
                                                   unsigned int max_sleep_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  unsigned int ns = 64;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(ns);
    if (ns < max_sleep_ns) ns *= 2;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_error(h, kErrTimeout, info);
      return false;
    }
  }
}

// ------------------------------------------------------------------------------------------ bulk copies

// 1-D bulk copy global -> shared (TMA engine), completion counted on `bar` in bytes. `src`, `dst` 16-byte
// aligned, `bytes` a multiple of 16. Single destination CTA.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Orders this thread's generic-proxy global accesses with async-proxy (TMA) accesses: a writer before it
// publishes data that TMA loads will read, a reader after it has acquired such data and before its TMA loads.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Bulk prefetch of global memory into L2 (no destination, nothing to wait for). `src` 16-byte aligned, `bytes` a
// multiple of 16. Used to start small latency-critical reads (norm weights) before the weight stream fills the
// memory queues.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// fp32 reduction into global memory (relaxed, gpu scope)
__device__ __forceinline__ void red_add_f32(float* addr, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void red_add_v4_f32(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread per CTA: arrive on a grid barrier counter (after a __threadfence by the caller).
__device__ __forceinline__ void grid_arrive(unsigned int* ctr) {
  __threadfence();
  atomicAdd(ctr, 1u);
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Generation grid barrier (one thread per CTA): the counter grows by G in every call and is never reset, so a
// kernel needs no last-CTA epilogue. Arrive returns this call's target: the next multiple of G at or above the
// counter (the counter is a multiple of G between calls).
__device__ __forceinline__ unsigned long long grid_arrive_gen(unsigned long long* ctr, unsigned int G) {
  __threadfence();
  const unsigned long long old = atomicAdd(ctr, 1ull);
  return old - old % G + G;
}

static __device__ __noinline__ bool grid_wait_gen(unsigned long long* ctr, unsigned long long target, WsHeader* h,
                                                  unsigned int info) {
  if (ld_acquire_u64(ctr) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  unsigned int ns = 32;
  while (ld_acquire_u64(ctr) < target) {
    __nanosleep(ns);
    if (ns < 256) ns *= 2;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_error(h, kErrTimeout, info);
      return false;
    }
  }
  return true;
}

// One thread per CTA: wait until `target` CTAs arrived. Bounded: gives up after kWaitLimitNs, records
// kErrTimeout and returns false. Requires all CTAs to be co-resident (cooperative launch).
static __device__ __noinline__ bool grid_wait(unsigned int* ctr, unsigned int target, WsHeader* h, unsigned int info) {
  if (ld_acquire_u32(ctr) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  unsigned int ns = 32;
  while (ld_acquire_u32(ctr) < target) {
    __nanosleep(ns);
    if (ns < 256) ns *= 2;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_error(h, kErrTimeout, info);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ------------------------------------------------------------------------------------------ PDL

// Programmatic dependent launch: let the next kernel in the stream start its prologue, and wait for the
// previous kernel's results. Both are no-ops when the launch did not use the PDL attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace mv
