// Exchange of the long-context split-KV partials over NVLink peer memory (one process per GPU).
//
// Every rank owns one exchange buffer, mapped into every other rank by CUDA IPC:
//   float    recv[2][world][per]   packed partials [m (rows) | l (rows) | o (rows x hd)] of each
//                                  rank, double-buffered by step parity
//   uint32   flag[2][world]        step number whose partials rank r has stored in slot r
//   uint32   step                  steps pushed by this rank so far
// A step is two launches on the caller's stream (programmatic dependent launches: each is
// scheduled while the kernel before it runs and waits for that grid to complete first).  peer_push_kernel (one CTA) stores this rank's
// packed partials into slot `rank` of every rank's buffer (its own included) with plain stores
// through the IPC mappings, fences at system scope, then raises flag[p][rank] = step in every
// buffer with a system-scope release store.  peer_combine_kernel (one CTA per row) waits,
// bounded in wall-clock time, until all `world` flags of its own buffer show the step
// (system-scope acquire loads), then merges the parts with the log-sum-exp combine of
// lse_combine_kernel.  The step counter lives in device memory, so a CUDA graph of
// steps replays correctly.  Parity double-buffering makes the reuse of a slot safe: a rank
// pushes step s + 2 only after its combine of step s + 1, which needed every rank's push of
// step s + 1, which each rank issued after its own combine of step s.
// Peer memory is only written with ordinary stores (no TMA).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace vxg {
namespace {
constexpr uint64_t kPeerWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// The step flags are written with release and read with acquire semantics at system scope:
// a reader that sees a flag also sees the partials stored before it, on whichever GPU.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
}  // namespace

size_t peer_buffer_bytes(int world, int per) {
  return (size_t)2 * world * per * sizeof(float) + ((size_t)2 * world + 4) * sizeof(uint32_t);
}

__global__ void __launch_bounds__(512) peer_push_kernel(const float* __restrict__ send, int per,
                                                        PeerTable peers, int world, int rank,
                                                        uint32_t* local_step) {
  __shared__ uint32_t s_step;
  grid_dep_wait();     // the partials (and the step counter) written before this launch
  grid_dep_trigger();  // the combine may be scheduled now; it waits for this grid to complete
  if (threadIdx.x == 0) s_step = ld_volatile(local_step) + 1;
  __syncthreads();
  const uint32_t step = s_step;
  const int p = step & 1;
  const bool vec = (per & 3) == 0;
  for (int d = 0; d < world; ++d) {
    float* dst = peers.buf[d] + ((size_t)p * world + rank) * per;
    if (vec) {
      const float4* s4 = reinterpret_cast<const float4*>(send);
      float4* d4 = reinterpret_cast<float4*>(dst);
      for (int i = threadIdx.x; i < per / 4; i += blockDim.x) d4[i] = s4[i];
    } else {
      for (int i = threadIdx.x; i < per; i += blockDim.x) dst[i] = send[i];
    }
  }
  __threadfence_system();  // this thread's stores reach every GPU before the flags below
  __syncthreads();         // ... and every thread's stores precede thread 0's releases
  if (threadIdx.x == 0) {
    for (int d = 0; d < world; ++d) {
      uint32_t* flags = reinterpret_cast<uint32_t*>(peers.buf[d] + (size_t)2 * world * per);
      st_release_sys(flags + p * world + rank, step);
    }
    *local_step = step;
  }
}

__global__ void __launch_bounds__(256) peer_combine_kernel(const float* buf, int world, int n_rows,
                                                           int hd, const float* gate, float* out,
                                                           uint32_t* status) {
  const int per = n_rows * (hd + 2);
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(buf + (size_t)2 * world * per);
  const uint32_t* local_step = flags + 2 * world;
  __shared__ int s_ok;
  __shared__ uint32_t s_step;
  grid_dep_wait();  // this rank's push has completed before the flags are polled
  if (threadIdx.x == 0) {
    const uint32_t step = ld_volatile(local_step);
    const int p = step & 1;
    int ok = 1;
    uint64_t t0 = 0;
    for (int r = 0; r < world && ok; ++r) {
      for (uint32_t i = 0; ld_acquire_sys(flags + p * world + r) != step; ++i) {
        if ((i & 1023u) == 0) {
          uint64_t t;
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
          if (t0 == 0) t0 = t;
          else if (t - t0 > kPeerWaitNs) {
            ok = 0;
            break;
          }
        }
      }
    }
    s_ok = ok;  // the acquiring loads above order the reads of the parts (after the barrier)
    s_step = step;
  }
  __syncthreads();
  const int row = blockIdx.x;
  if (!s_ok) {
    if (threadIdx.x == 0) atomicOr(status, kStatusTimeout);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) out[(size_t)row * hd + d] = 0.f;
    return;
  }
  const float* parts = buf + (size_t)(s_step & 1) * world * per;
  float M = -INFINITY;
  for (int k = 0; k < world; ++k) M = fmaxf(M, __ldcg(parts + (size_t)k * per + row));
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    if (M != -INFINITY)
      for (int k = 0; k < world; ++k) {
        const float* pk = parts + (size_t)k * per;
        const float mk = __ldcg(pk + row);
        if (mk == -INFINITY) continue;
        const float f = exp2f(mk - M);
        L = fmaf(__ldcg(pk + n_rows + row), f, L);
        O = fmaf(__ldcg(pk + 2 * n_rows + (size_t)row * hd + d), f, O);
      }
    float r = (L > 0.f || L != L) ? O / L : 0.f;  // NaN partials stay NaN
    const size_t oi = (size_t)row * hd + d;
    if (gate) r *= 1.0f / (1.0f + expf(-gate[oi]));
    if (!isfinite(r)) atomicOr(status, kStatusNonFinite);
    out[oi] = r;
  }
}

cudaError_t launch_peer_push(const float* send, int per, const PeerTable& peers, int world,
                             int rank, float* local_buf, cudaStream_t st) {
  uint32_t* local_step =
      reinterpret_cast<uint32_t*>(local_buf + (size_t)2 * world * per) + 2 * world;
  // programmatic dependent launches: the launch overlaps the previous kernel; each kernel
  // waits for its predecessor's grid to complete before it touches memory
  return launch_dependent(peer_push_kernel, dim3(1), dim3(512), 0, st, send, per, peers, world,
                          rank, local_step);
}

cudaError_t launch_peer_combine(const float* local_buf, int world, int n_rows, int hd,
                                const float* gate, float* out, uint32_t* status,
                                cudaStream_t st) {
  if (n_rows == 0) return cudaSuccess;
  return launch_dependent(peer_combine_kernel, dim3(n_rows), dim3(256), 0, st, local_buf, world,
                          n_rows, hd, gate, out, status);
}

}  // namespace vxg
