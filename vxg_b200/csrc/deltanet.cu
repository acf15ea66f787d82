// Gated-DeltaNet recurrent decode step (one token per sequence).
//
// Reference: the per-head core of step_deltanet_recurrent (crates/vxg-tensor/src/llm_ops.rs:
// 139-184): q, k L2-normalised (q scaled by q_scale = 1/sqrt(dk)), beta = sigmoid(beta_raw),
// decay = exp(softplus(alpha_raw + dt_bias) * A) with softplus cut off at +-20, then for every
// state row jv: S[jv,:] *= decay; sk = S[jv,:].k; d = (v[jv] - sk) * beta; S[jv,:] += d * k;
// o[jv] = S[jv,:].q.  The state is [dv][dk] fp32 per (sequence, head).
//
// The step is bound by moving the state: every element is read once and written once.  One CTA
// owns one (sequence, head); 8 lanes own one state row (16 floats each for dk = 128, interleaved
// so 8 lanes cover 128 contiguous bytes per float4 load), 32 rows per pass, and all passes are
// loaded before any arithmetic so a CTA keeps its whole 64 KiB state in flight at once.  Row dot
// products are 3-step shuffle reductions inside the 8-lane group.
#include "kernels.h"

namespace vxg {

template <int DK, int NP>
__global__ void __launch_bounds__(256) deltanet_step_kernel(DeltaNetArgs a) {
  constexpr int LPR = 8;            // lanes per state row
  constexpr int V4 = DK / (LPR * 4);  // float4 per lane per row
  constexpr int RPP = 256 / LPR;    // rows per pass
  const int bh = blockIdx.x;
  const int b = bh / a.n_vh, h = bh - b * a.n_vh;
  const int hk = h / (a.n_vh / a.n_kh);
  const int tid = threadIdx.x;
  const int rip = tid / LPR, sl = tid % LPR;

  // ---- normalised q, k for this lane's dims: dim(k4, i) = 32*k4 + 4*sl + i --------------------
  const float* qg = a.q + ((size_t)b * a.n_kh + hk) * DK;
  const float* kg = a.k + ((size_t)b * a.n_kh + hk) * DK;
  float4 qv[V4], kv[V4];
  float sq = 0.f, sk2 = 0.f;
#pragma unroll
  for (int k4 = 0; k4 < V4; ++k4) {
    qv[k4] = *reinterpret_cast<const float4*>(qg + 32 * k4 + 4 * sl);
    kv[k4] = *reinterpret_cast<const float4*>(kg + 32 * k4 + 4 * sl);
    sq = fmaf(qv[k4].x, qv[k4].x, sq); sq = fmaf(qv[k4].y, qv[k4].y, sq);
    sq = fmaf(qv[k4].z, qv[k4].z, sq); sq = fmaf(qv[k4].w, qv[k4].w, sq);
    sk2 = fmaf(kv[k4].x, kv[k4].x, sk2); sk2 = fmaf(kv[k4].y, kv[k4].y, sk2);
    sk2 = fmaf(kv[k4].z, kv[k4].z, sk2); sk2 = fmaf(kv[k4].w, kv[k4].w, sk2);
  }
#pragma unroll
  for (int o = 1; o < LPR; o <<= 1) {
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
    sk2 += __shfl_xor_sync(0xffffffffu, sk2, o);
  }
  const float qs = a.q_scale / sqrtf(sq + a.eps);   // l2_norm_scaled, llm_ops.rs:70-79
  const float ks = 1.0f / sqrtf(sk2 + a.eps);
#pragma unroll
  for (int k4 = 0; k4 < V4; ++k4) {
    qv[k4].x *= qs; qv[k4].y *= qs; qv[k4].z *= qs; qv[k4].w *= qs;
    kv[k4].x *= ks; kv[k4].y *= ks; kv[k4].z *= ks; kv[k4].w *= ks;
  }
  // ---- gates (llm_ops.rs:156-165) -------------------------------------------------------------
  const float beta = 1.0f / (1.0f + expf(-a.beta_raw[(size_t)b * a.n_vh + h]));
  const float x_sp = a.alpha_raw[(size_t)b * a.n_vh + h] + a.dt_bias[h];
  const float sp = x_sp > 20.0f ? x_sp : (x_sp < -20.0f ? expf(x_sp) : logf(1.0f + expf(x_sp)));
  const float decay = expf(sp * a.ssm_a[h]);

  float* S = a.state + ((size_t)b * a.n_vh + h) * (size_t)a.dv * DK;
  const float* vg = a.v + ((size_t)b * a.n_vh + h) * a.dv;
  float* og = a.o + ((size_t)b * a.n_vh + h) * a.dv;
  bool bad = false;
  for (int r0 = 0; r0 < a.dv; r0 += NP * RPP) {
    float4 st[NP][V4];
    float vv[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int jv = r0 + p * RPP + rip;
      if (jv < a.dv) {
#pragma unroll
        for (int k4 = 0; k4 < V4; ++k4)
          st[p][k4] = __ldcs(reinterpret_cast<const float4*>(S + (size_t)jv * DK + 32 * k4 + 4 * sl));
        vv[p] = vg[jv];
      }
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int jv = r0 + p * RPP + rip;
      if (jv >= a.dv) continue;
      float skp = 0.f;
#pragma unroll
      for (int k4 = 0; k4 < V4; ++k4) {
        st[p][k4].x *= decay; st[p][k4].y *= decay; st[p][k4].z *= decay; st[p][k4].w *= decay;
        skp = fmaf(st[p][k4].x, kv[k4].x, skp); skp = fmaf(st[p][k4].y, kv[k4].y, skp);
        skp = fmaf(st[p][k4].z, kv[k4].z, skp); skp = fmaf(st[p][k4].w, kv[k4].w, skp);
      }
#pragma unroll
      for (int o = 1; o < LPR; o <<= 1) skp += __shfl_xor_sync(0xffffffffu, skp, o);
      const float d = (vv[p] - skp) * beta;
      float op = 0.f;
#pragma unroll
      for (int k4 = 0; k4 < V4; ++k4) {
        st[p][k4].x = fmaf(d, kv[k4].x, st[p][k4].x); st[p][k4].y = fmaf(d, kv[k4].y, st[p][k4].y);
        st[p][k4].z = fmaf(d, kv[k4].z, st[p][k4].z); st[p][k4].w = fmaf(d, kv[k4].w, st[p][k4].w);
        op = fmaf(st[p][k4].x, qv[k4].x, op); op = fmaf(st[p][k4].y, qv[k4].y, op);
        op = fmaf(st[p][k4].z, qv[k4].z, op); op = fmaf(st[p][k4].w, qv[k4].w, op);
        __stcs(reinterpret_cast<float4*>(S + (size_t)jv * DK + 32 * k4 + 4 * sl), st[p][k4]);
      }
#pragma unroll
      for (int o = 1; o < LPR; o <<= 1) op += __shfl_xor_sync(0xffffffffu, op, o);
      if (sl == 0) {
        og[jv] = op;
        bad |= !isfinite(op);
      }
    }
  }
  if (bad) atomicOr(a.status, kStatusNonFinite);
}

cudaError_t launch_deltanet_step(const DeltaNetArgs& a, cudaStream_t st) {
  if (a.n_batch == 0 || a.n_vh == 0) return cudaSuccess;
  const unsigned grid = (unsigned)a.n_batch * a.n_vh;
  switch (a.dk) {
    case 64: deltanet_step_kernel<64, 4><<<grid, 256, 0, st>>>(a); break;
    case 128: deltanet_step_kernel<128, 4><<<grid, 256, 0, st>>>(a); break;
    case 256: deltanet_step_kernel<256, 2><<<grid, 256, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace vxg
