// Shared device helpers for the sm_100a Q8-KV attention / gated-DeltaNet backend.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vxg {

// KvQ8Block (crates/vxg-tensor/src/llm_prefill.rs:17-24): u16 f16-bits scale at byte 0 (LE),
// 32 int8 codes at bytes 2..33.  34 bytes, 2-byte aligned.
constexpr int kBlk = 34;

// Device status word bits (read back by the host after a call).
enum : uint32_t {
  kStatusNonFinite = 1u << 0,  // an attention / DeltaNet output was NaN or +-Inf
  kStatusBadIndex = 1u << 1,   // a sequence id / position outside the KV pool was skipped
  kStatusTimeout = 1u << 2,    // a bounded wait gave up (the kernel returned early)
};

__device__ __forceinline__ float f16bits_to_f32(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

// fp16.rs:33-77 is IEEE binary16 round-to-nearest-even for every non-NaN input, which is what
// __float2half_rn does; the Q8 scale is never NaN (f32::max ignores NaN, fmaxf likewise).
__device__ __forceinline__ uint16_t f32_to_f16bits(float x) {
  return __half_as_ushort(__float2half_rn(x));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- programmatic dependent launch -------------------------------------------------------------
// A kernel launched with programmatic stream serialisation may start while the previous kernel
// of its stream still runs; before it reads that kernel's results it waits for the previous
// grid to complete and its memory to be visible.  The previous kernel lets it start early by
// triggering.  Both are no-ops for kernels launched the ordinary way.
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- mbarrier + 1-D bulk async copy (TMA engine, no tensor map, local source) ---------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Pull the line holding p into L2 (no value is returned, so nothing is read early).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for the completion of the phase of `bar` with parity `parity`, for at most timeout_ns of
// wall-clock time.  Returns false if it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  const uint32_t addr = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 1023u) == 0) {  // the timer is read rarely: polls stay cheap
      const uint64_t t = globaltimer_ns();
      if (i == 0) t0 = t;
      else if (t - t0 > timeout_ns) return false;
    }
  }
}
// global -> shared bulk copy completing on `bar` (bytes and both addresses multiples of 16).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace vxg
