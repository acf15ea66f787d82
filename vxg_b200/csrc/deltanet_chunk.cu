// Gated-DeltaNet prompt recurrence in chunked (WY) form on tensor cores.
//
// The reference applies the recurrence token by token (llm_prefill.rs:470-480 over
// llm_ops.rs:139-184): per v-head, S <- g S; d = beta (v - S k); S <- S + d k^T; o = S q.  Write
// w_t = beta_t (v_t - g_t S_{t-1} k_t); then S_t = g_t S_{t-1} + w_t k_t^T, and over a chunk of
// C tokens with cumulative log decay L_t = sum_{i<=t} log g_i (gamma_t = exp L_t):
//   A[t][i] = beta_t exp(L_t - L_i) (k_t . k_i)   (i < t),   T = (I + A)^-1
//   U  = T diag(beta) V,   Wk = T diag(beta gamma) K            (chunk-local)
//   W  = U - Wk S0^T                                            (rows w_t of the chunk)
//   O  = diag(gamma) Q S0^T + (M o Q K^T) W,   M[t][i] = exp(L_t - L_i) for i <= t
//   S_C = gamma_C S0 + W^T diag(exp(L_C - L)) K
// which is the same recurrence re-associated.  One CTA = (sequence, v head, 64 rows of the
// state), chunks in order, state rows on chip.  The products run on mma.sync m16n8k8 TF32 with
// f32 accumulation; the triangular solve's products and the state update use 3xTF32 (hi/lo
// operand splits), which keeps the result within ~4% of the 1e-3 bar of the sequential fp32
// recurrence at 8192 tokens (the single-pass products contribute that; the state update and
// the solve would otherwise dominate).
#include "kernels.h"

namespace vxg {
namespace dnc {

constexpr int C = 64;        // chunk length
constexpr int DK = 128;
constexpr int DS = 64;       // state rows (v dims) per CTA
constexpr int THREADS = 256;
constexpr int LDK = DK + 4;  // row stride of K, Q, S (floats): 4 mod 32
constexpr int LDR = DS + DK + 8;  // R / X = [beta V | beta gamma K] -> [U | Wk] -> [W | Wk]
constexpr int LDA = C + 4;

struct __align__(16) Smem {
  float k[C][LDK];
  float q[C][LDK];
  float s[DS][LDK];
  float r[C][LDR];
  float a[C][LDA];   // A, then T's diagonal blocks in place
  float p[C][LDA];   // M o Q K^T
  float L[C];        // cumulative log decay
  float beta[C];
  float gam[C];      // exp(L_t)
  float rdec[C];     // exp(L_C - L_t)
};

__device__ __forceinline__ uint32_t tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// acc[nt] (+)= A(m0.., k) B(k, n0 + 8 nt ..) over k in [k0, k1), one 16-row tile, NT 8-col tiles.
// fa(m, k) / fb(k, n) read the operands (f32); X3 adds the hi/lo correction products.
template <int NT, bool X3, class FA, class FB>
__device__ __forceinline__ void warp_mma(float (&acc)[NT][4], int m0, int n0, int k0, int k1,
                                         FA fa, FB fb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  for (int k = k0; k < k1; k += 8) {
    const float af[4] = {fa(m0 + g, k + q), fa(m0 + g + 8, k + q), fa(m0 + g, k + q + 4),
                         fa(m0 + g + 8, k + q + 4)};
    uint32_t ah[4], al[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ah[i] = tf32(af[i]);
      if constexpr (X3) al[i] = tf32(af[i] - __uint_as_float(ah[i]));
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = n0 + 8 * nt + g;
      const float b0 = fb(k + q, n), b1 = fb(k + q + 4, n);
      const uint32_t bh0 = tf32(b0), bh1 = tf32(b1);
      if constexpr (X3) {
        const uint32_t bl0 = tf32(b0 - __uint_as_float(bh0)), bl1 = tf32(b1 - __uint_as_float(bh1));
        mma_tf32(acc[nt], al, bh0, bh1);
        mma_tf32(acc[nt], ah, bl0, bl1);
      }
      mma_tf32(acc[nt], ah, bh0, bh1);
    }
  }
}

template <int NT>
__device__ __forceinline__ void zero(float (&acc)[NT][4]) {
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
}

}  // namespace dnc

// grid: n_batch * n_vh * (dv / 64); state rows [64 * slice, 64 * slice + 64) of (b, h).
__global__ void __launch_bounds__(dnc::THREADS, 1)
    deltanet_chunk_kernel(DeltaNetArgs a, const float* qn, const float* kn, const float2* gates,
                          const float* lgs) {
  using namespace dnc;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, qd = lane & 3;
  const int n_sl = a.dv / DS;
  const int bh = blockIdx.x / n_sl, sl = blockIdx.x % n_sl;
  const int b = bh / a.n_vh, h = bh % a.n_vh;
  const int hk = h / (a.n_vh / a.n_kh);
  float* S = a.state + (((size_t)b * a.n_vh + h) * a.dv + (size_t)sl * DS) * DK;

  for (int i = tid; i < DS * DK / 4; i += THREADS) {
    const int r = i / (DK / 4), c4 = (i % (DK / 4)) * 4;
    *reinterpret_cast<float4*>(&sm.s[r][c4]) = *reinterpret_cast<const float4*>(S + r * DK + c4);
  }
  bool bad = false;
  const int n_chunks = (a.n_tok + C - 1) / C;
  const int mt = warp >> 1, half = warp & 1;  // 64 x 64 outputs: m-tile, 4 of the 8 n-tiles

  for (int c = 0; c < n_chunks; ++c) {
    const int t0 = c * C;
    __syncthreads();  // previous chunk's readers of k, q, r are done
    // ---- loads: K, Q (normalised), V slice (raw), beta, log decay -------------------------
    for (int i = tid; i < C * DK / 4; i += THREADS) {
      const int r = i / (DK / 4), c4 = (i % (DK / 4)) * 4;
      const int t = t0 + r;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), qv = kv;
      if (t < a.n_tok) {
        const size_t off = (((size_t)b * a.n_tok + t) * a.n_kh + hk) * DK + c4;
        kv = *reinterpret_cast<const float4*>(kn + off);
        qv = *reinterpret_cast<const float4*>(qn + off);
      }
      *reinterpret_cast<float4*>(&sm.k[r][c4]) = kv;
      *reinterpret_cast<float4*>(&sm.q[r][c4]) = qv;
    }
    for (int i = tid; i < C * DS; i += THREADS) {
      const int r = i / DS, j = i % DS;
      const int t = t0 + r;
      sm.r[r][j] = t < a.n_tok ? a.v[(size_t)b * a.v_bs + (size_t)t * a.v_ts +
                                     (size_t)h * a.dv + sl * DS + j]
                               : 0.f;
    }
    if (warp == 0) {
      // inclusive scan of the log decays (two tokens per lane); padded tokens: beta 0, decay 1
      const int t = t0 + 2 * lane;
      const size_t gi = ((size_t)b * a.n_tok + t) * a.n_vh + h;
      const float l0 = t < a.n_tok ? lgs[gi] : 0.f;
      const float l1 = t + 1 < a.n_tok ? lgs[gi + a.n_vh] : 0.f;
      float s = l0 + l1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      sm.L[2 * lane] = s - l1;
      sm.L[2 * lane + 1] = s;
      sm.beta[2 * lane] = t < a.n_tok ? gates[gi].x : 0.f;
      sm.beta[2 * lane + 1] = t + 1 < a.n_tok ? gates[gi + a.n_vh].x : 0.f;
      const float LC = __shfl_sync(0xffffffffu, s, 31);
      sm.gam[2 * lane] = expf(s - l1);
      sm.gam[2 * lane + 1] = expf(s);
      sm.rdec[2 * lane] = expf(LC - (s - l1));
      sm.rdec[2 * lane + 1] = expf(LC - s);
    }
    __syncthreads();
    // ---- right-hand sides: [beta V | beta gamma K]; G = K K^T -> A; Q K^T -> P -------------
    for (int i = tid; i < C * DK; i += THREADS) {
      const int r = i / DK, j = i % DK;
      sm.r[r][DS + j] = sm.beta[r] * sm.gam[r] * sm.k[r][j];
    }
    for (int i = tid; i < C * DS; i += THREADS) {
      const int r = i / DS, j = i % DS;
      sm.r[r][j] *= sm.beta[r];
    }
    {
      float acc[4][4];
      zero(acc);
      warp_mma<4, false>(acc, 16 * mt, 32 * half, 0, DK,
                         [&](int m, int k) { return sm.k[m][k]; },
                         [&](int k, int n) { return sm.k[n][k]; });
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * mt + g + (e >> 1) * 8, i = 32 * half + 8 * nt + 2 * qd + (e & 1);
          sm.a[t][i] = i < t ? sm.beta[t] * expf(sm.L[t] - sm.L[i]) * acc[nt][e] : 0.f;
        }
      zero(acc);
      warp_mma<4, false>(acc, 16 * mt, 32 * half, 0, DK,
                         [&](int m, int k) { return sm.q[m][k]; },
                         [&](int k, int n) { return sm.k[n][k]; });
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * mt + g + (e >> 1) * 8, i = 32 * half + 8 * nt + 2 * qd + (e & 1);
          sm.p[t][i] = i <= t ? expf(sm.L[t] - sm.L[i]) * acc[nt][e] : 0.f;
        }
    }
    __syncthreads();
    // ---- diagonal 16x16 blocks of T = (I + A)^-1, in place (lane j of a half-warp = column j)
    if (warp < 2) {
      const int blk = 2 * warp + (lane >> 4), j = lane & 15, o = 16 * blk;
      float col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float v = r == j ? 1.f : 0.f;
        if (r > j) {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (i >= j && i < r) v = fmaf(-sm.a[o + r][o + i], col[i], v);
        }
        col[r] = v;
      }
      __syncwarp();
#pragma unroll
      for (int r = 0; r < 16; ++r) sm.a[o + r][o + j] = col[r];
    }
    __syncthreads();
    // ---- blocked forward substitution X = (I + A)^-1 R, each warp owning 24 columns --------
    {
      const int n0 = 24 * warp;
      for (int bi = 0; bi < 4; ++bi) {
        float acc[3][4];
        zero(acc);
        if (bi > 0)
          warp_mma<3, true>(acc, 16 * bi, n0, 0, 16 * bi,
                            [&](int m, int k) { return sm.a[m][k]; },
                            [&](int k, int n) { return sm.r[k][n]; });
        // Y = R_bi - sum_k A_bi,k X_k, written over R_bi (own columns)
#pragma unroll
        for (int nt = 0; nt < 3; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 16 * bi + g + (e >> 1) * 8, n = n0 + 8 * nt + 2 * qd + (e & 1);
            sm.r[t][n] -= acc[nt][e];
          }
        __syncwarp();
        zero(acc);
        warp_mma<3, true>(acc, 16 * bi, n0, 16 * bi, 16 * bi + 16,
                          [&](int m, int k) { return sm.a[m][k]; },
                          [&](int k, int n) { return sm.r[k][n]; });
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < 3; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 16 * bi + g + (e >> 1) * 8, n = n0 + 8 * nt + 2 * qd + (e & 1);
            sm.r[t][n] = acc[nt][e];
          }
        __syncwarp();
      }
    }
    __syncthreads();
    // ---- W = U - Wk S0^T (in place over U) --------------------------------------------------
    {
      float acc[4][4];
      zero(acc);
      warp_mma<4, false>(acc, 16 * mt, 32 * half, 0, DK,
                         [&](int m, int k) { return sm.r[m][DS + k]; },
                         [&](int k, int n) { return sm.s[n][k]; });
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * mt + g + (e >> 1) * 8, j = 32 * half + 8 * nt + 2 * qd + (e & 1);
          sm.r[t][j] -= acc[nt][e];
        }
    }
    __syncthreads();
    // ---- O = diag(gamma) Q S0^T + P W -> global ----------------------------------------------
    {
      float acc[4][4];
      zero(acc);
      warp_mma<4, false>(acc, 16 * mt, 32 * half, 0, DK,
                         [&](int m, int k) { return sm.q[m][k]; },
                         [&](int k, int n) { return sm.s[n][k]; });
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] *= sm.gam[16 * mt + g + (e >> 1) * 8];
      warp_mma<4, false>(acc, 16 * mt, 32 * half, 0, 16 * mt + 16,
                         [&](int m, int k) { return sm.p[m][k]; },
                         [&](int k, int n) { return sm.r[k][n]; });
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int t = t0 + 16 * mt + g + (e >> 1) * 8, j = 32 * half + 8 * nt + 2 * qd;
          if (t < a.n_tok) {
            bad |= !isfinite(acc[nt][e]) || !isfinite(acc[nt][e + 1]);
            *reinterpret_cast<float2*>(a.o + (size_t)b * a.o_bs + (size_t)t * a.o_ts +
                                       (size_t)h * a.dv + sl * DS + j) =
                make_float2(acc[nt][e], acc[nt][e + 1]);
          }
        }
    }
    __syncthreads();  // S0 is read above; now it is updated
    // ---- S = gamma_C S0 + W^T diag(exp(L_C - L)) K  (3xTF32) --------------------------------
    {
      float acc[8][4];
      zero(acc);
      warp_mma<8, true>(acc, 16 * mt, 64 * half, 0, C,
                        [&](int m, int k) { return sm.r[k][m] * sm.rdec[k]; },
                        [&](int k, int n) { return sm.k[k][n]; });
      const float gc = sm.gam[C - 1];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jv = 16 * mt + g + (e >> 1) * 8, kk = 64 * half + 8 * nt + 2 * qd + (e & 1);
          sm.s[jv][kk] = fmaf(gc, sm.s[jv][kk], acc[nt][e]);
        }
    }
  }
  __syncthreads();
  for (int i = tid; i < DS * DK / 4; i += THREADS) {
    const int r = i / (DK / 4), c4 = (i % (DK / 4)) * 4;
    *reinterpret_cast<float4*>(S + r * DK + c4) = *reinterpret_cast<const float4*>(&sm.s[r][c4]);
  }
  if (bad) atomicOr(a.status, kStatusNonFinite);
}

bool deltanet_chunk_supported(const DeltaNetArgs& a) {
  return a.dk == dnc::DK && a.dv % dnc::DS == 0 && a.n_tok >= dnc::C;
}

size_t deltanet_chunk_smem_bytes() { return sizeof(dnc::Smem); }

cudaError_t launch_deltanet_chunk(const DeltaNetArgs& a, const float* qn, const float* kn,
                                  const float2* gates, const float* lgs, cudaStream_t st) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(deltanet_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(dnc::Smem));
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  const unsigned grid = (unsigned)(a.n_batch * a.n_vh * (a.dv / dnc::DS));
  deltanet_chunk_kernel<<<grid, dnc::THREADS, sizeof(dnc::Smem), st>>>(a, qn, kn, gates, lgs);
  return cudaGetLastError();
}

}  // namespace vxg
