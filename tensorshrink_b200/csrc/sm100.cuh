// sm_100a building blocks shared by the streaming kernels: mbarriers, TMA
// tensor copies (no cluster multicast anywhere), bounded waits, and host-side
// tensor-map encoding through the driver entry point (no libcuda link).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace ts {

// Upper bound on mbarrier polls before a wait gives up and reports an error
// instead of hanging the GPU (each try_wait may itself suspend briefly).
constexpr uint32_t kMaxWaitPolls = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code` in *err) if the phase with
// `parity` has not completed after kMaxWaitPolls polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  for (uint32_t i = 0; i < kMaxWaitPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  if (err) atomicExch(err, code);
  return false;
}

// 2-D TMA tile load global -> shared, completion signalled on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0),
// completion signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 4-byte asynchronous copy global -> shared (zero-fill when src_bytes == 0).
__device__ __forceinline__ void cp_async4(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// Arrive on `bar` once all of this thread's prior cp.async copies have
// landed (the barrier's expected count must include this arrival).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Named barrier among `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---- host ---------------------------------------------------------------------
// Encode a 2-D row-major tensor map: `inner` elements of `elem_bytes` per row
// (contiguous), `outer` rows `row_stride_bytes` apart, box {box_inner, box_outer}.
int encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner,
                   uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                   CUtensorMapSwizzle swizzle);

}  // namespace ts
