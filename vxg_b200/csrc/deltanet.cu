// Gated DeltaNet: recurrent decode step, multi-token (prefill) recurrence, and the conv1d /
// RMSNorm-SiLU prologue and epilogue of the full reference step.
//
// Reference: step_deltanet_recurrent (crates/vxg-tensor/src/llm_ops.rs:103-193).
//  * prologue (:122-137): causal conv1d of width k_sz over the rolling conv_state, SiLU;
//  * core (:139-184): q, k L2-normalised (q also scaled by q_scale = 1/sqrt(dk)),
//    beta = sigmoid(beta_raw), decay = exp(softplus(alpha_raw + dt_bias) * A) (softplus cut off at
//    +-20), then for every state row jv: S[jv,:] *= decay; sk = S[jv,:].k;
//    d = (v[jv] - sk) * beta; S[jv,:] += d * k; o[jv] = S[jv,:].q   (state [dv][dk] fp32);
//  * epilogue (:186-191): y = RMSNorm(o) * ssm_norm * SiLU(z).
// Prefill in the reference applies the step token by token (llm_prefill.rs:470-480); the
// prefill kernel here does the same recurrence with the state held on chip across all tokens.
//
// Layout of one CTA of the decode step: one (sequence, head); 8 lanes own one state row (16
// floats each at dk = 128, interleaved so 8 lanes cover 128 contiguous bytes per float4 load),
// 32 rows per pass, all passes loaded before any arithmetic so the CTA keeps its whole state in
// flight; row dot products are 3-step shuffle reductions inside the 8-lane group.
#include "dn_gates.cuh"
#include "kernels.h"

#include <algorithm>

namespace vxg {

namespace {
__device__ __forceinline__ float siluf_(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float decay_of(float alpha_raw, float dt_bias, float A) {
  return expf(log_decay_of(alpha_raw, dt_bias, A));
}
}  // namespace

// ---------------------------------------------------------------------------------------------
// Decode step (one token), optionally with the fused RMSNorm * SiLU(z) epilogue.
// ---------------------------------------------------------------------------------------------
template <int DK, int NP>
__global__ void __launch_bounds__(256) deltanet_step_kernel(DeltaNetArgs a) {
  constexpr int LPR = 8;              // lanes per state row
  constexpr int V4 = DK / (LPR * 4);  // float4 per lane per row
  constexpr int RPP = 256 / LPR;      // rows per pass
  __shared__ float s_o[256];          // o of this head (epilogue; dv <= 256)
  __shared__ float s_red[8];
  const int bh = blockIdx.x;
  const int b = bh / a.n_vh, h = bh - b * a.n_vh;
  const int hk = h / (a.n_vh / a.n_kh);
  const int tid = threadIdx.x;
  const int rip = tid / LPR, sl = tid % LPR;

  // ---- normalised q, k for this lane's dims: dim(k4, i) = 32*k4 + 4*sl + i --------------------
  const float* qg = a.q + (size_t)b * a.q_bs + (size_t)hk * DK;
  const float* kg = a.k + (size_t)b * a.k_bs + (size_t)hk * DK;
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
  const size_t gi = (size_t)b * a.g_bs + h;
  const float beta = sigmoidf_(a.beta_raw[gi]);
  const float decay = decay_of(a.alpha_raw[gi], a.dt_bias[h], a.ssm_a[h]);

  float* S = a.state + ((size_t)b * a.n_vh + h) * (size_t)a.dv * DK;
  const float* vg = a.v + (size_t)b * a.v_bs + (size_t)h * a.dv;
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
      if (jv >= a.dv) continue;  // warp-uniform: dv is a multiple of 32
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
        if (a.y) s_o[jv] = op;
        else a.o[(size_t)b * a.o_bs + (size_t)h * a.dv + jv] = op;
        bad |= !isfinite(op);
      }
    }
  }
  if (a.y) {
    // ---- RMSNorm(o) * ssm_norm * SiLU(z), llm_ops.rs:186-191 and :59-68 --------------------
    __syncthreads();
    float part = 0.f;
    for (int j = tid; j < a.dv; j += 256) part = fmaf(s_o[j], s_o[j], part);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if ((tid & 31) == 0) s_red[tid >> 5] = part;
    __syncthreads();
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) sum += s_red[w];
    const float scale = 1.0f / sqrtf(sum / (float)a.dv + a.eps);
    const float* zg = a.z + (size_t)b * a.o_bs + (size_t)h * a.dv;
    float* yg = a.y + (size_t)b * a.o_bs + (size_t)h * a.dv;
    for (int j = tid; j < a.dv; j += 256) {
      const float yv = s_o[j] * scale * a.ssm_norm[j] * siluf_(zg[j]);
      yg[j] = yv;
      bad |= !isfinite(yv);
    }
  }
  if (bad) atomicOr(a.status, kStatusNonFinite);
}

// ---------------------------------------------------------------------------------------------
// Persistent decode step for states up to 64 KiB (dk, dv <= 128): one CTA per SM walks the
// (sequence, head) items; a 2-deep ring of shared-memory stages receives each item's state and
// its q, k, v rows by 1-D bulk async copies, so the next state streams in while the current one
// is updated; updated rows go straight to HBM with streaming stores.
// ---------------------------------------------------------------------------------------------
namespace dn {
constexpr int MAXE = 128 * 128;        // state floats per stage
constexpr int NS = 3;                  // states in flight (3 x 64 KiB ring)
constexpr uint64_t kWaitNs = 2000000000ull;
struct __align__(128) Smem {
  float state[NS][MAXE];
  float q[NS][256], k[NS][256], v[NS][256];
  float o[256];
  float red[8];
  uint64_t full[NS];
};
}  // namespace dn

size_t deltanet_persistent_smem() { return sizeof(dn::Smem); }

template <int DK>
__global__ void __launch_bounds__(256, 1) deltanet_step_persistent(DeltaNetArgs a) {
  constexpr int LPR = 8;
  constexpr int V4 = DK / (LPR * 4);
  extern __shared__ __align__(128) uint8_t smem_raw[];
  dn::Smem& sm = *reinterpret_cast<dn::Smem*>(smem_raw);
  const int tid = threadIdx.x, rip = tid / LPR, sl = tid % LPR;
  const int n_items = a.n_batch * a.n_vh;
  const uint32_t st_bytes = (uint32_t)a.dv * DK * 4;
  grid_dep_trigger();  // the next step's kernel may be scheduled as these CTAs retire
  if (tid == 0) {
    for (int i = 0; i < dn::NS; ++i) mbar_init(&sm.full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  grid_dep_wait();  // every input (the state above all) only after the previous kernel is done
  auto issue = [&](int item, int buf) {
    const int b = item / a.n_vh, h = item - b * a.n_vh;
    const int hk = h / (a.n_vh / a.n_kh);
    const uint32_t qb = DK * 4, vb = (uint32_t)a.dv * 4;
    mbar_arrive_expect_tx(&sm.full[buf], st_bytes + 2 * qb + vb);
    bulk_g2s(sm.state[buf], a.state + (size_t)item * a.dv * DK, st_bytes, &sm.full[buf]);
    bulk_g2s(sm.q[buf], a.q + (size_t)b * a.q_bs + (size_t)hk * DK, qb, &sm.full[buf]);
    bulk_g2s(sm.k[buf], a.k + (size_t)b * a.k_bs + (size_t)hk * DK, qb, &sm.full[buf]);
    bulk_g2s(sm.v[buf], a.v + (size_t)b * a.v_bs + (size_t)h * a.dv, vb, &sm.full[buf]);
  };
  if (tid == 0)
    for (int i = 0; i < dn::NS; ++i)
      if ((int)(blockIdx.x + i * gridDim.x) < n_items) issue(blockIdx.x + i * gridDim.x, i);
  bool bad = false;
  int it = 0;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
    const int buf = it % dn::NS;
    const uint32_t par = (uint32_t)(it / dn::NS) & 1u;
    const int b = item / a.n_vh, h = item - b * a.n_vh;
    const size_t gi = (size_t)b * a.g_bs + h;
    const float beta = sigmoidf_(a.beta_raw[gi]);
    const float decay = decay_of(a.alpha_raw[gi], a.dt_bias[h], a.ssm_a[h]);
    const bool ok = __syncthreads_and(mbar_wait(&sm.full[buf], par, dn::kWaitNs));
    if (!ok) {
      if (tid == 0) atomicOr(a.status, kStatusTimeout);
      // let the copies already in flight land before the CTA leaves
      for (int k = 1; k < dn::NS; ++k)
        if (item + k * (int)gridDim.x < n_items)
          mbar_wait(&sm.full[(it + k) % dn::NS], (uint32_t)((it + k) / dn::NS) & 1u, dn::kWaitNs);
      return;
    }
    float4 qv[V4], kv[V4];
    float sq = 0.f, sk2 = 0.f;
#pragma unroll
    for (int k4 = 0; k4 < V4; ++k4) {
      qv[k4] = *reinterpret_cast<const float4*>(&sm.q[buf][32 * k4 + 4 * sl]);
      kv[k4] = *reinterpret_cast<const float4*>(&sm.k[buf][32 * k4 + 4 * sl]);
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
    const float qs = a.q_scale / sqrtf(sq + a.eps), ks = 1.0f / sqrtf(sk2 + a.eps);
#pragma unroll
    for (int k4 = 0; k4 < V4; ++k4) {
      qv[k4].x *= qs; qv[k4].y *= qs; qv[k4].z *= qs; qv[k4].w *= qs;
      kv[k4].x *= ks; kv[k4].y *= ks; kv[k4].z *= ks; kv[k4].w *= ks;
    }
    float* S = a.state + (size_t)item * a.dv * DK;
    for (int jv = rip; jv < a.dv; jv += 32) {
      float4 st[V4];
#pragma unroll
      for (int k4 = 0; k4 < V4; ++k4)
        st[k4] = *reinterpret_cast<const float4*>(&sm.state[buf][jv * DK + 32 * k4 + 4 * sl]);
      float skp = 0.f;
#pragma unroll
      for (int k4 = 0; k4 < V4; ++k4) {
        st[k4].x *= decay; st[k4].y *= decay; st[k4].z *= decay; st[k4].w *= decay;
        skp = fmaf(st[k4].x, kv[k4].x, skp); skp = fmaf(st[k4].y, kv[k4].y, skp);
        skp = fmaf(st[k4].z, kv[k4].z, skp); skp = fmaf(st[k4].w, kv[k4].w, skp);
      }
#pragma unroll
      for (int o = 1; o < LPR; o <<= 1) skp += __shfl_xor_sync(0xffffffffu, skp, o);
      const float d = (sm.v[buf][jv] - skp) * beta;
      float op = 0.f;
#pragma unroll
      for (int k4 = 0; k4 < V4; ++k4) {
        st[k4].x = fmaf(d, kv[k4].x, st[k4].x); st[k4].y = fmaf(d, kv[k4].y, st[k4].y);
        st[k4].z = fmaf(d, kv[k4].z, st[k4].z); st[k4].w = fmaf(d, kv[k4].w, st[k4].w);
        op = fmaf(st[k4].x, qv[k4].x, op); op = fmaf(st[k4].y, qv[k4].y, op);
        op = fmaf(st[k4].z, qv[k4].z, op); op = fmaf(st[k4].w, qv[k4].w, op);
        __stcs(reinterpret_cast<float4*>(S + (size_t)jv * DK + 32 * k4 + 4 * sl), st[k4]);
      }
#pragma unroll
      for (int o = 1; o < LPR; o <<= 1) op += __shfl_xor_sync(0xffffffffu, op, o);
      if (sl == 0) {
        if (a.y) sm.o[jv] = op;
        else a.o[(size_t)b * a.o_bs + (size_t)h * a.dv + jv] = op;
        bad |= !isfinite(op);
      }
    }
    __syncthreads();  // everyone is done with this stage (and sm.o is complete)
    if (tid == 0 && item + dn::NS * (int)gridDim.x < n_items) issue(item + dn::NS * gridDim.x, buf);
    if (a.y) {
      float part = 0.f;
      for (int j = tid; j < a.dv; j += 256) part = fmaf(sm.o[j], sm.o[j], part);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if ((tid & 31) == 0) sm.red[tid >> 5] = part;
      __syncthreads();
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += sm.red[w];
      const float scale = 1.0f / sqrtf(sum / (float)a.dv + a.eps);
      const float* zg = a.z + (size_t)b * a.o_bs + (size_t)h * a.dv;
      float* yg = a.y + (size_t)b * a.o_bs + (size_t)h * a.dv;
      for (int j = tid; j < a.dv; j += 256) {
        const float yv = sm.o[j] * scale * a.ssm_norm[j] * siluf_(zg[j]);
        yg[j] = yv;
        bad |= !isfinite(yv);
      }
      __syncthreads();  // sm.o and sm.red are reused by the next item
    }
  }
  if (bad) atomicOr(a.status, kStatusNonFinite);
}

// ---------------------------------------------------------------------------------------------
// Prefill: the recurrence over n_tok tokens with the state held in registers.
// Preparation pass: normalised q, k per (b, t, k head) and (beta, decay) per (b, t, v head).
// ---------------------------------------------------------------------------------------------
// One warp per (b, t, k head) with 16-byte accesses (q / k rows are dense and 16-byte aligned:
// the entry points reject misaligned device arrays and dk is 64, 128 or 256); the gates take
// one thread per (b, t, v head).
__global__ void __launch_bounds__(256) deltanet_prep_vec_kernel(DeltaNetArgs a, float* qn,
                                                                float* kn, float2* gates,
                                                                float* lgs, float q_scale) {
  const int lane = threadIdx.x & 31;
  const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w < (long long)a.n_batch * a.n_tok * a.n_kh) {
    const long long bt = w / a.n_kh;
    const int hk = (int)(w - bt * a.n_kh);
    const int b = (int)(bt / a.n_tok), t = (int)(bt - (long long)b * a.n_tok);
    const float* qg = a.q + (size_t)b * a.q_bs + (size_t)t * a.q_ts + (size_t)hk * a.dk;
    const float* kg = a.k + (size_t)b * a.k_bs + (size_t)t * a.k_ts + (size_t)hk * a.dk;
    float4 qv[2], kv[2];
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = 4 * (lane + 32 * u);
      qv[u] = kv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < a.dk) {
        qv[u] = *reinterpret_cast<const float4*>(qg + i);
        kv[u] = *reinterpret_cast<const float4*>(kg + i);
      }
      sq = fmaf(qv[u].x, qv[u].x, sq); sq = fmaf(qv[u].y, qv[u].y, sq);
      sq = fmaf(qv[u].z, qv[u].z, sq); sq = fmaf(qv[u].w, qv[u].w, sq);
      sk = fmaf(kv[u].x, kv[u].x, sk); sk = fmaf(kv[u].y, kv[u].y, sk);
      sk = fmaf(kv[u].z, kv[u].z, sk); sk = fmaf(kv[u].w, kv[u].w, sk);
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    const float qs = q_scale / sqrtf(sq + a.eps), ks = 1.0f / sqrtf(sk + a.eps);
    float* qo = qn + ((size_t)bt * a.n_kh + hk) * a.dk;
    float* ko = kn + ((size_t)bt * a.n_kh + hk) * a.dk;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = 4 * (lane + 32 * u);
      if (i < a.dk) {
        *reinterpret_cast<float4*>(qo + i) =
            make_float4(qv[u].x * qs, qv[u].y * qs, qv[u].z * qs, qv[u].w * qs);
        *reinterpret_cast<float4*>(ko + i) =
            make_float4(kv[u].x * ks, kv[u].y * ks, kv[u].z * ks, kv[u].w * ks);
      }
    }
  }
  const long long gidx = (long long)blockIdx.x * 256 + threadIdx.x;
  if (gidx < (long long)a.n_batch * a.n_tok * a.n_vh) {
    const long long bt = gidx / a.n_vh;
    const int h = (int)(gidx - bt * a.n_vh);
    const int b = (int)(bt / a.n_tok), t = (int)(bt - (long long)b * a.n_tok);
    const size_t gi = (size_t)b * a.g_bs + (size_t)t * a.g_ts + h;
    const float lg = log_decay_of(a.alpha_raw[gi], a.dt_bias[h], a.ssm_a[h]);
    gates[gidx] = make_float2(sigmoidf_(a.beta_raw[gi]), expf(lg));
    if (lgs) lgs[gidx] = lg;
  }
}

// One CTA = (sequence, v head, chunk of 32 state rows); 8 lanes per row, DK/8 dims per lane.
// Rows evolve independently in the recurrence, so chunks of rows run in parallel CTAs; each CTA
// streams the (shared) normalised q, k of every token through L1.
template <int DK>
__global__ void __launch_bounds__(256) deltanet_prefill_kernel(DeltaNetArgs a, const float* qn,
                                                               const float* kn,
                                                               const float2* gates) {
  constexpr int LPR = 8;
  constexpr int V4 = DK / (LPR * 4);
  const int n_chunk = a.dv / 32;
  const int bh = blockIdx.x / n_chunk, chunk = blockIdx.x % n_chunk;
  const int b = bh / a.n_vh, h = bh - b * a.n_vh;
  const int hk = h / (a.n_vh / a.n_kh);
  const int rip = threadIdx.x / LPR, sl = threadIdx.x % LPR;
  const int jv = chunk * 32 + rip;
  float* S = a.state + (((size_t)b * a.n_vh + h) * a.dv + jv) * DK;
  float4 st[V4];
#pragma unroll
  for (int k4 = 0; k4 < V4; ++k4) st[k4] = *reinterpret_cast<const float4*>(S + 32 * k4 + 4 * sl);
  bool bad = false;
  for (int t = 0; t < a.n_tok; ++t) {
    const size_t bt = (size_t)b * a.n_tok + t;
    const float* qg = qn + (bt * a.n_kh + hk) * DK;
    const float* kg = kn + (bt * a.n_kh + hk) * DK;
    const float2 gt = gates[bt * a.n_vh + h];  // (beta, decay)
    const float vj = a.v[(size_t)b * a.v_bs + (size_t)t * a.v_ts + (size_t)h * a.dv + jv];
    float4 kv[V4], qv[V4];
#pragma unroll
    for (int k4 = 0; k4 < V4; ++k4) {
      kv[k4] = __ldg(reinterpret_cast<const float4*>(kg + 32 * k4 + 4 * sl));
      qv[k4] = __ldg(reinterpret_cast<const float4*>(qg + 32 * k4 + 4 * sl));
    }
    float skp = 0.f;
#pragma unroll
    for (int k4 = 0; k4 < V4; ++k4) {
      st[k4].x *= gt.y; st[k4].y *= gt.y; st[k4].z *= gt.y; st[k4].w *= gt.y;
      skp = fmaf(st[k4].x, kv[k4].x, skp); skp = fmaf(st[k4].y, kv[k4].y, skp);
      skp = fmaf(st[k4].z, kv[k4].z, skp); skp = fmaf(st[k4].w, kv[k4].w, skp);
    }
#pragma unroll
    for (int o = 1; o < LPR; o <<= 1) skp += __shfl_xor_sync(0xffffffffu, skp, o);
    const float d = (vj - skp) * gt.x;
    float op = 0.f;
#pragma unroll
    for (int k4 = 0; k4 < V4; ++k4) {
      st[k4].x = fmaf(d, kv[k4].x, st[k4].x); st[k4].y = fmaf(d, kv[k4].y, st[k4].y);
      st[k4].z = fmaf(d, kv[k4].z, st[k4].z); st[k4].w = fmaf(d, kv[k4].w, st[k4].w);
      op = fmaf(st[k4].x, qv[k4].x, op); op = fmaf(st[k4].y, qv[k4].y, op);
      op = fmaf(st[k4].z, qv[k4].z, op); op = fmaf(st[k4].w, qv[k4].w, op);
    }
#pragma unroll
    for (int o = 1; o < LPR; o <<= 1) op += __shfl_xor_sync(0xffffffffu, op, o);
    if (sl == 0) {
      a.o[(size_t)b * a.o_bs + (size_t)t * a.o_ts + (size_t)h * a.dv + jv] = op;
      bad |= !isfinite(op);
    }
  }
#pragma unroll
  for (int k4 = 0; k4 < V4; ++k4) *reinterpret_cast<float4*>(S + 32 * k4 + 4 * sl) = st[k4];
  if (bad) atomicOr(a.status, kStatusNonFinite);
}

// ---------------------------------------------------------------------------------------------
// conv1d + SiLU prologue (llm_ops.rs:122-137): per (sequence, channel), a sequential fma chain
// over the k_sz - 1 history rows and the new input, then the history shifts by one row.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) deltanet_conv_kernel(const float* __restrict__ x,
                                                            const float* __restrict__ w,
                                                            float* __restrict__ conv_state,
                                                            float* __restrict__ out, int n_batch,
                                                            int conv_ch, int k_sz) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)n_batch * conv_ch) return;
  const int b = (int)(idx / conv_ch), c = (int)(idx - (long long)b * conv_ch);
  const int hist = k_sz - 1;
  float* cs = conv_state + (size_t)b * hist * conv_ch;
  const float* wc = w + (size_t)c * k_sz;
  const float xc = x[idx];
  float acc = 0.f;
  for (int t = 0; t < hist; ++t) acc = fmaf(cs[(size_t)t * conv_ch + c], wc[t], acc);
  acc = fmaf(xc, wc[hist], acc);
  for (int t = 0; t + 1 < hist; ++t) cs[(size_t)t * conv_ch + c] = cs[(size_t)(t + 1) * conv_ch + c];
  if (hist > 0) cs[(size_t)(hist - 1) * conv_ch + c] = xc;
  out[idx] = siluf_(acc);
}

// ---------------------------------------------------------------------------------------------
cudaError_t launch_deltanet_step(const DeltaNetArgs& a, cudaStream_t st) {
  if (a.n_batch == 0 || a.n_vh == 0) return cudaSuccess;
  // Persistent ring when the state fits a stage and every bulk copy is 16-byte aligned.
  const bool aligned = ((uintptr_t)a.state | (uintptr_t)a.q | (uintptr_t)a.k | (uintptr_t)a.v) % 16 == 0 &&
                       (a.q_bs % 4) == 0 && (a.k_bs % 4) == 0 && (a.v_bs % 4) == 0;
  if (aligned && (a.dk == 128 || a.dk == 64) && a.dv <= 128) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    static bool attr_set[64] = {};
    if (dev >= 64 || !attr_set[dev]) {
      e = cudaFuncSetAttribute(deltanet_step_persistent<128>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(dn::Smem));
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(deltanet_step_persistent<64>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(dn::Smem));
      if (e != cudaSuccess) return e;
      if (dev < 64) attr_set[dev] = true;
    }
    const int items = a.n_batch * a.n_vh;
    const unsigned grid = (unsigned)std::min(items, sms);
    // chained to the previous kernel of the stream (typically the previous step, whose state it
    // reads): its CTAs are set up as that kernel's CTAs retire
    if (a.dk == 128)
      return launch_dependent(deltanet_step_persistent<128>, dim3(grid), dim3(256),
                              sizeof(dn::Smem), st, a);
    return launch_dependent(deltanet_step_persistent<64>, dim3(grid), dim3(256), sizeof(dn::Smem),
                            st, a);
  }
  const unsigned grid = (unsigned)a.n_batch * a.n_vh;
  switch (a.dk) {
    case 64: deltanet_step_kernel<64, 4><<<grid, 256, 0, st>>>(a); break;
    case 128: deltanet_step_kernel<128, 4><<<grid, 256, 0, st>>>(a); break;
    case 256: deltanet_step_kernel<256, 2><<<grid, 256, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

size_t deltanet_prefill_scratch_bytes(const DeltaNetArgs& a) {
  const size_t bt = (size_t)a.n_batch * a.n_tok;
  return (2 * bt * a.n_kh * a.dk) * sizeof(float) + bt * a.n_vh * (sizeof(float2) + sizeof(float)) +
         256;
}

cudaError_t launch_deltanet_prefill(const DeltaNetArgs& a, void* scratch, int allow_chunk,
                                    cudaStream_t st) {
  if (a.n_batch == 0 || a.n_tok == 0 || a.n_vh == 0) return cudaSuccess;
  // dk = dv = 128 (the Qwen3.5 shape): the tcgen05 / TMEM chunk kernel, which forms the norms
  // and gates itself (no preparation pass)
  if (allow_chunk && deltanet_chunk_tc_supported(a)) return launch_deltanet_chunk_tc(a, st);
  const size_t bt = (size_t)a.n_batch * a.n_tok;
  float* qn = static_cast<float*>(scratch);
  float* kn = qn + bt * a.n_kh * a.dk;
  float2* gates = reinterpret_cast<float2*>(kn + bt * a.n_kh * a.dk);
  float* lgs = reinterpret_cast<float*>(gates + bt * a.n_vh);
  const bool chunked = allow_chunk && deltanet_chunk_supported(a);
  // the chunked kernel takes q unit-normalised (its f16 products want |q| <= 1) and applies
  // q_scale to the products; the sequential kernel takes it folded in
  const float qscale = chunked ? 1.0f : a.q_scale;
  const long long warps = (long long)bt * a.n_kh, gthreads = (long long)bt * a.n_vh;
  const long long blocks = std::max((warps + 7) / 8, (gthreads + 255) / 256);
  deltanet_prep_vec_kernel<<<(unsigned)blocks, 256, 0, st>>>(a, qn, kn, gates,
                                                            chunked ? lgs : nullptr, qscale);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (chunked) {
    e = launch_deltanet_chunk(a, qn, kn, gates, lgs, st);
  } else {
    const unsigned grid = (unsigned)(a.n_batch * a.n_vh * (a.dv / 32));
    switch (a.dk) {
      case 64: deltanet_prefill_kernel<64><<<grid, 256, 0, st>>>(a, qn, kn, gates); break;
      case 128: deltanet_prefill_kernel<128><<<grid, 256, 0, st>>>(a, qn, kn, gates); break;
      case 256: deltanet_prefill_kernel<256><<<grid, 256, 0, st>>>(a, qn, kn, gates); break;
      default: return cudaErrorInvalidValue;
    }
    e = cudaGetLastError();
  }
  return e;
}

cudaError_t launch_deltanet_conv(const float* x, const float* w, float* conv_state, float* out,
                                 int n_batch, int conv_ch, int k_sz, cudaStream_t st) {
  const long long n = (long long)n_batch * conv_ch;
  if (n == 0) return cudaSuccess;
  deltanet_conv_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, w, conv_state, out, n_batch,
                                                                  conv_ch, k_sz);
  return cudaGetLastError();
}

}  // namespace vxg
