// Query / key prologue of step_full_gqa_q8 (crates/vxg-tensor/src/llm_prefill.rs:286-309):
// split the gated query (q then gate per head), optional RMSNorm with a [head_dim] weight
// (rms_norm, llm_ops.rs:48-57) and RoPE (apply_rope, llm_ops.rs:81-101) on every query head and
// kv head of one token.
//
// Bit-exact with the reference on the same cos/sin table: the table (cos, sin of pos * freq_i)
// is computed by the host with the C library, exactly the calls the reference makes, and the
// device repeats the reference's operation order with explicitly rounded multiplies / adds (no
// FMA contraction).  The RMSNorm sum of squares is the reference's sequential fma chain.  So
// the K that reaches the quantiser, and therefore its Q8 codes and scales, match bit for bit.
#include "kernels.h"

namespace vxg {

__global__ void gqa_prep_kernel(const float* __restrict__ q_raw, float* __restrict__ k_cur,
                                const float* __restrict__ q_norm, const float* __restrict__ k_norm,
                                int gated, int n_head, int n_kv, int hd,
                                const float2* __restrict__ rope_cs, int rope_half, int neox,
                                float eps, float* __restrict__ q_out,
                                float* __restrict__ gate_out) {
  extern __shared__ float xs[];
  __shared__ float s_scale;
  const int row = blockIdx.x;
  const bool is_q = row < n_head;
  const int h = is_q ? row : row - n_head;
  const float* src = is_q ? q_raw + (size_t)h * (gated ? 2 : 1) * hd : k_cur + (size_t)h * hd;
  for (int i = threadIdx.x; i < hd; i += blockDim.x) {
    xs[i] = src[i];
    if (is_q && gated) gate_out[(size_t)h * hd + i] = src[hd + i];
  }
  __syncthreads();
  const float* w = is_q ? q_norm : k_norm;
  if (w) {
    if (threadIdx.x == 0) {
      float sq = 0.f;
      for (int i = 0; i < hd; ++i) sq = __fmaf_rn(xs[i], xs[i], sq);
      s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, (float)hd), eps)));
    }
    __syncthreads();
    const float sc = s_scale;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], sc), w[i]);
    __syncthreads();
  }
  for (int i = threadIdx.x; i < rope_half; i += blockDim.x) {
    const float c = rope_cs[i].x, s = rope_cs[i].y;
    const int i0 = neox ? i : 2 * i;
    const int i1 = neox ? i + rope_half : 2 * i + 1;
    const float x0 = xs[i0], x1 = xs[i1];
    xs[i0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    xs[i1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
  __syncthreads();
  float* dst = is_q ? q_out + (size_t)h * hd : k_cur + (size_t)h * hd;
  for (int i = threadIdx.x; i < hd; i += blockDim.x) dst[i] = xs[i];
}

cudaError_t launch_gqa_prep(const float* q_raw, float* k_cur, const float* q_norm,
                            const float* k_norm, int gated, int n_head, int n_kv, int hd,
                            const float2* rope_cs, int rope_half, int neox, float eps,
                            float* q_out, float* gate_out, cudaStream_t st) {
  const int threads = hd < 256 ? ((hd + 31) / 32) * 32 : 256;
  gqa_prep_kernel<<<n_head + n_kv, threads, hd * sizeof(float), st>>>(
      q_raw, k_cur, q_norm, k_norm, gated, n_head, n_kv, hd, rope_cs, rope_half, neox, eps, q_out,
      gate_out);
  return cudaGetLastError();
}

}  // namespace vxg
