// Gated-DeltaNet gate arithmetic shared by the DeltaNet kernels (llm_ops.rs:156-165):
//   beta = sigmoid(beta_raw),  log decay = softplus(alpha_raw + dt_bias) * A
// with the reference's piecewise softplus (linear above 20, exp below -20).
#pragma once

namespace vxg {

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float log_decay_of(float alpha_raw, float dt_bias, float A) {
  const float x = alpha_raw + dt_bias;
  const float sp = x > 20.0f ? x : (x < -20.0f ? expf(x) : logf(1.0f + expf(x)));
  return sp * A;
}

}  // namespace vxg
