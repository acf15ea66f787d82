// Fused Q8_0 quantise-and-append of new K/V tokens into the device KV pool.
//
// Reference: KvQ8Block::quantize (crates/vxg-tensor/src/llm_prefill.rs:27-42) applied to every
// 32-float block of the new token's K and V and stored at cache index
// pos*n_kv*(hd/32) + kh*(hd/32) + b (llm_prefill.rs:311-324).  Codes and scales are bit-exact
// with the reference: IEEE division for amax/127 and 1/df (no fast-math), binary16 RNE for the
// scale, round-half-even for the codes, NaN -> 0 like Rust's saturating `as i8`.
//
// Eight lanes quantise one 32-value block, four values each: the block max is a reduction
// over the 8-lane group, each lane writes its four code bytes (two 16-bit stores; records are
// 34 bytes, 2-byte aligned) and the group's first lane the 2-byte scale.  A warp covers four
// consecutive blocks, so loads and stores of neighbouring warps are contiguous.
#include "kernels.h"

namespace vxg {

__device__ __forceinline__ void load4(const float* p, bool vec, float (&x)[4]) {
  if (vec) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = p[i];
  }
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, bool vec, float (&x)[4]) {
  if (vec) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    x[0] = __uint_as_float(v.x << 16); x[1] = __uint_as_float(v.x & 0xFFFF0000u);
    x[2] = __uint_as_float(v.y << 16); x[3] = __uint_as_float(v.y & 0xFFFF0000u);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = __bfloat162float(p[i]);
  }
}

// T = float or __nv_bfloat16 (bf16 widens to f32 exactly, so the codes are those of the f32 value)
// vec: k_new / v_new allow 16-byte (f32) or 8-byte (bf16) loads of four values.
// Division by a divisor fixed for the launch, as a multiply-high, an add and a shift
// (Granlund and Montgomery, "Division by invariant integers using multiplication", 1994):
// with s = ceil(log2 d) and m = floor(2^32 (2^s - d) / d) + 1, n / d = (umulhi(n, m) + n) >> s
// for every 0 <= n < 2^31.
struct Div32 {
  uint32_t d, m, s;
};
Div32 make_div32(uint32_t d) {
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  const uint32_t m = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
  return {d, m, s};
}
__device__ __forceinline__ uint32_t div32(uint32_t n, const Div32& v) {
  return (__umulhi(n, v.m) + n) >> v.s;
}

constexpr int kLaneBits = 2;             // lanes per 32-value block: 4, 8 values each
constexpr int kLanes = 1 << kLaneBits;
constexpr int kVals = 32 / kLanes;       // values per lane

// WIDE: 64-bit block indices (threads >= 2^31); otherwise 32-bit ones with the
// two divisions by per_tok and n_tok done as multiply-shifts.
template <typename T, bool WIDE>
__global__ void __launch_bounds__(256) q8_append_kernel(const int32_t* __restrict__ seq_ids,
                                                         const int32_t* __restrict__ pos,
                                                         const T* __restrict__ k_new,
                                                         const T* __restrict__ v_new,
                                                         uint8_t* __restrict__ k_pool,
                                                         uint8_t* __restrict__ v_pool,
                                                         int n_batch, int n_tok, int n_seq,
                                                         int cap, int n_kv, int nb, bool vec,
                                                         Div32 per_tok_div, Div32 n_tok_div,
                                                         uint32_t* status) {
  grid_dep_trigger();  // a decode pass launched after this may start its set-up now
  // Launched as a programmatic dependent: the launch overlaps the previous kernel's tail, and
  // nothing is read (positions, inputs) or written (the cache a previous pass may still read)
  // before that kernel has completed.
  grid_dep_wait();
  const int sub = threadIdx.x & (kLanes - 1);   // lane in the block's group: kVals values
  const int per_tok = n_kv * nb;                 // blocks per token in one cache
  // every lane takes part in the group reduction; lanes past the end or on a bad index carry 0
  bool ok;
  int which, bt, blk, b, t;
  if constexpr (WIDE) {
    const long long blk_id = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> kLaneBits;
    const long long per_cache = (long long)n_batch * n_tok * per_tok;
    ok = blk_id < 2 * per_cache;
    which = ok && blk_id >= per_cache;           // 0 = K, 1 = V
    const long long r = blk_id - which * per_cache;
    bt = ok ? (int)(r / per_tok) : 0;            // (batch, token) index
    blk = ok ? (int)(r - (long long)bt * per_tok) : 0;
    b = bt / n_tok;
    t = bt - b * n_tok;
  } else {
    const uint32_t blk_id = (blockIdx.x * blockDim.x + threadIdx.x) >> kLaneBits;
    const uint32_t per_cache = (uint32_t)n_batch * (uint32_t)n_tok * (uint32_t)per_tok;
    ok = blk_id < 2 * per_cache;
    which = ok && blk_id >= per_cache;
    const uint32_t r = ok ? blk_id - which * per_cache : 0;
    const uint32_t q = div32(r, per_tok_div);
    bt = (int)q;
    blk = (int)(r - q * (uint32_t)per_tok);
    b = (int)div32(q, n_tok_div);
    t = bt - b * n_tok;
  }
  int s = 0, p = 0;
  if (ok) {
    s = seq_ids[b];
    p = pos[b] + t;
    if (s < 0 || s >= n_seq || p < 0 || p >= cap) {
      if (sub == 0) atomicOr(status, kStatusBadIndex);
      ok = false;
    }
  }
  float x[kVals];
#pragma unroll
  for (int i = 0; i < kVals; ++i) x[i] = 0.f;
  if (ok) {
    const T* src = (which ? v_new : k_new) + ((size_t)bt * per_tok + blk) * 32 + kVals * sub;
#pragma unroll
    for (int i = 0; i < kVals; i += 4) load4(src + i, vec, *reinterpret_cast<float(*)[4]>(&x[i]));
  }
  // amax starts at 0 and ignores NaN (f32::max); fmaxf(0, NaN) = 0 gives the same.
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < kVals; ++i) m = fmaxf(m, fmaxf(0.0f, fabsf(x[i])));
#pragma unroll
  for (int o = 1; o < kLanes; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (!ok) return;
  const uint16_t dh = f32_to_f16bits(m / 127.0f);
  const float df = f16bits_to_f32(dh);
  const float inv = df > 0.0f ? 1.0f / df : 0.0f;
  uint32_t code[kVals];
#pragma unroll
  for (int i = 0; i < kVals; ++i) {
    // round half to even (a NaN product becomes 0, as the reference's cast), then clamp to
    // +-127: a scale that rounded down to a binary16 subnormal can put |x * inv| above 127.5
    const int qi = max(-127, min(127, __float2int_rn(x[i] * inv)));
    code[i] = (uint32_t)qi & 0xFFu;
  }
  uint8_t* dst = (which ? v_pool : k_pool) + (((size_t)s * cap + p) * per_tok + blk) * kBlk;
  uint16_t* d16 = reinterpret_cast<uint16_t*>(dst + 2 + kVals * sub);  // 2-byte aligned codes
#pragma unroll
  for (int i = 0; i < kVals / 2; ++i) d16[i] = (uint16_t)(code[2 * i] | (code[2 * i + 1] << 8));
  if (sub == 0) *reinterpret_cast<uint16_t*>(dst) = dh;
}

cudaError_t launch_q8_append(const int32_t* seq_ids, const int32_t* pos, const float* k_new,
                             const float* v_new, uint8_t* k_pool, uint8_t* v_pool, int n_batch,
                             int n_tok, int n_seq, int cap, int n_kv, int nb, uint32_t* status,
                             cudaStream_t stream) {
  const long long n_blk = 2LL * n_batch * n_tok * n_kv * nb;
  if (n_blk == 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = (n_blk * kLanes + threads - 1) / threads;
  const bool vec = ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15u) == 0;
  const Div32 dp = make_div32((uint32_t)(n_kv * nb)), dt = make_div32((uint32_t)n_tok);
  if (n_blk * kLanes >= (1LL << 31))
    return launch_dependent(q8_append_kernel<float, true>, dim3((unsigned)blocks), dim3(threads),
                            0, stream, seq_ids, pos, k_new, v_new, k_pool, v_pool, n_batch, n_tok,
                            n_seq, cap, n_kv, nb, vec, dp, dt, status);
  return launch_dependent(q8_append_kernel<float, false>, dim3((unsigned)blocks), dim3(threads), 0,
                          stream, seq_ids, pos, k_new, v_new, k_pool, v_pool, n_batch, n_tok,
                          n_seq, cap, n_kv, nb, vec, dp, dt, status);
}

cudaError_t launch_q8_append_bf16(const int32_t* seq_ids, const int32_t* pos, const void* k_new,
                                  const void* v_new, uint8_t* k_pool, uint8_t* v_pool, int n_batch,
                                  int n_tok, int n_seq, int cap, int n_kv, int nb, uint32_t* status,
                                  cudaStream_t stream) {
  const long long n_blk = 2LL * n_batch * n_tok * n_kv * nb;
  if (n_blk == 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = (n_blk * kLanes + threads - 1) / threads;
  const bool vec = ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 7u) == 0;
  const Div32 dp = make_div32((uint32_t)(n_kv * nb)), dt = make_div32((uint32_t)n_tok);
  const auto* kb = static_cast<const __nv_bfloat16*>(k_new);
  const auto* vb = static_cast<const __nv_bfloat16*>(v_new);
  if (n_blk * kLanes >= (1LL << 31))
    return launch_dependent(q8_append_kernel<__nv_bfloat16, true>, dim3((unsigned)blocks),
                            dim3(threads), 0, stream, seq_ids, pos, kb, vb, k_pool, v_pool, n_batch,
                            n_tok, n_seq, cap, n_kv, nb, vec, dp, dt, status);
  return launch_dependent(q8_append_kernel<__nv_bfloat16, false>, dim3((unsigned)blocks),
                          dim3(threads), 0, stream, seq_ids, pos, kb, vb, k_pool, v_pool, n_batch,
                          n_tok, n_seq, cap, n_kv, nb, vec, dp, dt, status);
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
