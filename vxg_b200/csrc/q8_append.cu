// Fused Q8_0 quantise-and-append of new K/V tokens into the device KV pool.
//
// Reference: KvQ8Block::quantize (crates/vxg-tensor/src/llm_prefill.rs:27-42) applied to every
// 32-float block of the new token's K and V and stored at cache index
// pos*n_kv*(hd/32) + kh*(hd/32) + b (llm_prefill.rs:311-324).  Codes and scales are bit-exact
// with the reference: IEEE division for amax/127 and 1/df (no fast-math), binary16 RNE for the
// scale, round-half-even for the codes, NaN -> 0 like Rust's saturating `as i8`.
//
// One warp quantises one 32-value block: lane i owns value i, the block max is a warp
// reduction, lane i writes code byte i and lane 0 writes the 2-byte scale.
#include "kernels.h"

namespace vxg {

__device__ __forceinline__ float load_f32(const float* p) { return *p; }
__device__ __forceinline__ float load_f32(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// T = float or __nv_bfloat16 (bf16 widens to f32 exactly, so the codes are those of the f32 value)
template <typename T>
__global__ void __launch_bounds__(256) q8_append_kernel(const int32_t* __restrict__ seq_ids,
                                                         const int32_t* __restrict__ pos,
                                                         const T* __restrict__ k_new,
                                                         const T* __restrict__ v_new,
                                                         uint8_t* __restrict__ k_pool,
                                                         uint8_t* __restrict__ v_pool,
                                                         int n_batch, int n_tok, int n_seq,
                                                         int cap, int n_kv, int nb,
                                                         uint32_t* status) {
  grid_dep_trigger();  // a decode pass launched after this may start its set-up now
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int per_tok = n_kv * nb;                 // blocks per token in one cache
  const long long per_cache = (long long)n_batch * n_tok * per_tok;
  if (warp >= 2 * per_cache) return;
  const int which = warp >= per_cache;            // 0 = K, 1 = V
  const long long r = warp - which * per_cache;
  const int bt = (int)(r / per_tok);              // (batch, token) index
  const int blk = (int)(r - (long long)bt * per_tok);
  const int b = bt / n_tok;
  const int t = bt - b * n_tok;
  const int s = seq_ids[b];
  const int p = pos[b] + t;
  if (s < 0 || s >= n_seq || p < 0 || p >= cap) {
    if (lane == 0) atomicOr(status, kStatusBadIndex);
    return;
  }
  const T* src = (which ? v_new : k_new) + ((size_t)bt * per_tok + blk) * 32;
  const float x = load_f32(src + lane);
  // amax starts at 0 and ignores NaN (f32::max); fmaxf(0, NaN) = 0 gives the same.
  const float amax = warp_max(fmaxf(0.0f, fabsf(x)));
  const uint16_t dh = f32_to_f16bits(amax / 127.0f);
  const float df = f16bits_to_f32(dh);
  const float inv = df > 0.0f ? 1.0f / df : 0.0f;
  const float rq = rintf(x * inv);
  const int qi = (rq == rq) ? (int)fminf(fmaxf(rq, -127.0f), 127.0f) : 0;
  uint8_t* dst = (which ? v_pool : k_pool) + (((size_t)s * cap + p) * per_tok + blk) * kBlk;
  dst[2 + lane] = (uint8_t)(int8_t)qi;
  if (lane == 0) *reinterpret_cast<uint16_t*>(dst) = dh;
}

cudaError_t launch_q8_append(const int32_t* seq_ids, const int32_t* pos, const float* k_new,
                             const float* v_new, uint8_t* k_pool, uint8_t* v_pool, int n_batch,
                             int n_tok, int n_seq, int cap, int n_kv, int nb, uint32_t* status,
                             cudaStream_t stream) {
  const long long warps = 2LL * n_batch * n_tok * n_kv * nb;
  if (warps == 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  q8_append_kernel<float><<<(unsigned)blocks, threads, 0, stream>>>(
      seq_ids, pos, k_new, v_new, k_pool, v_pool, n_batch, n_tok, n_seq, cap, n_kv, nb, status);
  return cudaGetLastError();
}

cudaError_t launch_q8_append_bf16(const int32_t* seq_ids, const int32_t* pos, const void* k_new,
                                  const void* v_new, uint8_t* k_pool, uint8_t* v_pool, int n_batch,
                                  int n_tok, int n_seq, int cap, int n_kv, int nb, uint32_t* status,
                                  cudaStream_t stream) {
  const long long warps = 2LL * n_batch * n_tok * n_kv * nb;
  if (warps == 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  q8_append_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, stream>>>(
      seq_ids, pos, static_cast<const __nv_bfloat16*>(k_new),
      static_cast<const __nv_bfloat16*>(v_new), k_pool, v_pool, n_batch, n_tok, n_seq, cap, n_kv,
      nb, status);
  return cudaGetLastError();
}

// fp32 pools: one thread per 4 floats of one (batch entry, token) row of K and of V.
__global__ void __launch_bounds__(256) f32_append_kernel(const int32_t* __restrict__ seq_ids,
                                                         const int32_t* __restrict__ pos,
                                                         const float* __restrict__ k_new,
                                                         const float* __restrict__ v_new,
                                                         float* __restrict__ k_pool,
                                                         float* __restrict__ v_pool, int n_batch,
                                                         int n_tok, int n_seq, int cap, int row4,
                                                         uint32_t* status) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long per = (long long)n_batch * n_tok * row4;
  if (i >= per) return;
  const int bt = (int)(i / row4), c = (int)(i - (long long)bt * row4);
  const int b = bt / n_tok, t = bt - b * n_tok;
  const int s = seq_ids[b], p = pos[b] + t;
  if (s < 0 || s >= n_seq || p < 0 || p >= cap) {
    if (c == 0) atomicOr(status, kStatusBadIndex);
    return;
  }
  const size_t dst = ((size_t)s * cap + p) * row4 + c;
  reinterpret_cast<float4*>(k_pool)[dst] = reinterpret_cast<const float4*>(k_new)[i];
  reinterpret_cast<float4*>(v_pool)[dst] = reinterpret_cast<const float4*>(v_new)[i];
}

cudaError_t launch_f32_append(const int32_t* seq_ids, const int32_t* pos, const float* k_new,
                              const float* v_new, float* k_pool, float* v_pool, int n_batch,
                              int n_tok, int n_seq, int cap, int n_kv, int hd, uint32_t* status,
                              cudaStream_t stream) {
  const int row4 = n_kv * hd / 4;
  const long long n = (long long)n_batch * n_tok * row4;
  if (n == 0) return cudaSuccess;
  f32_append_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
      seq_ids, pos, k_new, v_new, k_pool, v_pool, n_batch, n_tok, n_seq, cap, row4, status);
  return cudaGetLastError();
}

}  // namespace vxg
