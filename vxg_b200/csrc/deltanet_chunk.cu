// Gated-DeltaNet prompt recurrence in chunked (WY) form on tensor cores.
//
// The reference applies the recurrence token by token (llm_prefill.rs:470-480 over
// llm_ops.rs:139-184): per v-head, S <- g S; d = beta (v - S k); S <- S + d k^T; o = S q.  Write
// w_t = beta_t (v_t - g_t S_{t-1} k_t); then S_t = g_t S_{t-1} + w_t k_t^T, and over a chunk of
// C tokens with cumulative log decay L_t = sum_{i<=t} log g_i (gamma_t = exp L_t):
//   A[t][i] = beta_t exp(L_t - L_i) (k_t . k_i)   (i < t),   T = (I + A)^-1
//   W  = T diag(beta) (V - diag(gamma) K S0^T)                  (rows w_t of the chunk)
//   O  = diag(gamma) Q S0^T + (M o Q K^T) W,   M[t][i] = exp(L_t - L_i) for i <= t
//   S_C = gamma_C S0 + W^T diag(exp(L_C - L)) K
// which is the same recurrence re-associated.  One CTA = (sequence, v head, 64 rows of the
// state), chunks in order, state rows on chip.  The products run on mma.sync m16n8k8 TF32 with
// f32 accumulation; the triangular solve's products and the state update use 3xTF32 (hi/lo
// operand splits), which keeps the result within a few % of the 1e-3 bar of the sequential fp32
// recurrence at 8192 tokens (the single-pass products contribute that; the state update and
// the solve would otherwise dominate).
#include "kernels.h"

namespace vxg {
namespace dnc {

constexpr int C = 64;        // chunk length
constexpr int DK = 128;
constexpr int DS = 64;       // state rows (v dims) per CTA
constexpr int THREADS = 256;
// Row strides (floats).  Matrices read along k (contiguous) take 64-bit fragment loads and want
// a stride of 8 mod 32; R, read along its rows by most products, wants 4 mod 32.
constexpr int LDK = DK + 8;       // K, Q, S
constexpr int LDR = DS + 4;       // R: V rows -> right-hand side -> W
constexpr int LDA = C + 8;        // A / T, P

struct __align__(16) Smem {
  float k[2][C][LDK];  // chunk c in k[c & 1]; chunk c + 1 lands in the other while c computes
  float q[C][LDK];     // refilled with chunk c + 1 once chunk c's last Q product is done
  float s[DS][LDK];
  float r[2][C][LDR];  // V rows -> right-hand side -> W; double-buffered like k
  float a[C][LDA];   // A, then T's diagonal blocks in place
  float p[C][LDA];   // M o Q K^T
  float L[C];        // cumulative log decay
  float beta[C];
  float gam[C];      // exp(L_t)
  float rdec[C];     // exp(L_C - L_t)
};

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// f32 -> (hi, lo) with hi the top 19 bits (what the TF32 datapath reads) and lo = x - hi exact
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xFFFFE000u;
  lo = __float_as_uint(x - __uint_as_float(hi));
}

// 16-byte asynchronous global -> shared copy (zero fill when !valid; src must stay a valid
// address), committed as one group per call site and awaited with cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// acc[nt] (+)= A(m0.., k) B(k, n0 + 8 nt ..) over k in [k0, k1): one 16-row tile, NT 8-col
// tiles.  A is [m][k] (AK) or [k][m]; B is [n][k] (BK) or [k][n]; ascale (optional) scales A's
// column k.  Operands go to the TF32 datapath as raw f32 bits (it reads the top 19); X3 adds the
// hi/lo correction products.  Inside each 8-wide k step, fragment slot q holds k + 2q and slot
// q + 4 holds k + 2q + 1 (the same permutation for A and B), so k-contiguous operands load as
// 64-bit pairs.
template <int NT, bool X3, bool AK, bool BK>
__device__ __forceinline__ void warp_mma(float (&acc)[NT][4], const float* A, int lda,
                                         const float* B, int ldb, int m0, int n0, int k0, int k1,
                                         const float* ascale = nullptr) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  // the two correction products accumulate separately: three short dependency chains per tile
  float c1[X3 ? NT : 1][4], c2[X3 ? NT : 1][4];
#pragma unroll
  for (int i = 0; i < (X3 ? NT : 1); ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) c1[i][e] = c2[i][e] = 0.f;
  for (int k = k0; k < k1; k += 8) {
    const int kk = k + 2 * q;
    float a[4];
    if constexpr (AK) {
      const float2 r0 = *reinterpret_cast<const float2*>(A + (m0 + g) * lda + kk);
      const float2 r1 = *reinterpret_cast<const float2*>(A + (m0 + g + 8) * lda + kk);
      a[0] = r0.x; a[2] = r0.y; a[1] = r1.x; a[3] = r1.y;
    } else {
      a[0] = A[kk * lda + m0 + g];
      a[2] = A[(kk + 1) * lda + m0 + g];
      a[1] = A[kk * lda + m0 + g + 8];
      a[3] = A[(kk + 1) * lda + m0 + g + 8];
    }
    if (ascale) {
      const float s0 = ascale[kk], s1 = ascale[kk + 1];
      a[0] *= s0; a[1] *= s0; a[2] *= s1; a[3] *= s1;
    }
    uint32_t ah[4], al[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (X3) split_tf32(a[i], ah[i], al[i]);
      else ah[i] = __float_as_uint(a[i]);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = n0 + 8 * nt + g;
      float b0, b1;
      if constexpr (BK) {
        const float2 r = *reinterpret_cast<const float2*>(B + n * ldb + kk);
        b0 = r.x; b1 = r.y;
      } else {
        b0 = B[kk * ldb + n];
        b1 = B[(kk + 1) * ldb + n];
      }
      if constexpr (X3) {
        uint32_t bh0, bl0, bh1, bl1;
        split_tf32(b0, bh0, bl0);
        split_tf32(b1, bh1, bl1);
        mma_tf32(c1[nt], al, bh0, bh1);
        mma_tf32(c2[nt], ah, bl0, bl1);
        mma_tf32(acc[nt], ah, bh0, bh1);
      } else {
        mma_tf32(acc[nt], ah, __float_as_uint(b0), __float_as_uint(b1));
      }
    }
  }
  if constexpr (X3)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] += c1[nt][e] + c2[nt][e];
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

  // ---- asynchronous chunk loads: K, Q (normalised) and this CTA's V slice ---------------------
  constexpr int NKQ = C * DK / 4 / THREADS, NV = C * DS / 4 / THREADS;
  auto issue_kv = [&](int cc) {  // chunk cc's K rows -> k[cc & 1], V rows -> r[cc & 1]
#pragma unroll
    for (int u = 0; u < NKQ; ++u) {
      const int i = tid + u * THREADS, r = i / (DK / 4), c4 = (i % (DK / 4)) * 4;
      const int t = cc * C + r;
      const bool ok = t < a.n_tok;
      cp_async16(&sm.k[cc & 1][r][c4],
                 kn + (((size_t)b * a.n_tok + (ok ? t : 0)) * a.n_kh + hk) * DK + c4, ok);
    }
#pragma unroll
    for (int u = 0; u < NV; ++u) {
      const int i = tid + u * THREADS, r = i / (DS / 4), j4 = (i % (DS / 4)) * 4;
      const int t = cc * C + r;
      const bool ok = t < a.n_tok;
      cp_async16(&sm.r[cc & 1][r][j4],
                 a.v + (size_t)b * a.v_bs + (size_t)(ok ? t : 0) * a.v_ts + (size_t)h * a.dv +
                     sl * DS + j4,
                 ok);
    }
    cp_async_commit();
  };
  auto issue_q = [&](int cc) {  // chunk cc's Q rows -> q
#pragma unroll
    for (int u = 0; u < NKQ; ++u) {
      const int i = tid + u * THREADS, r = i / (DK / 4), c4 = (i % (DK / 4)) * 4;
      const int t = cc * C + r;
      const bool ok = t < a.n_tok;
      cp_async16(&sm.q[r][c4],
                 qn + (((size_t)b * a.n_tok + (ok ? t : 0)) * a.n_kh + hk) * DK + c4, ok);
    }
    cp_async_commit();
  };
  // warp 0 keeps the next chunk's log decays and betas in registers (two tokens per lane)
  float nl0 = 0.f, nl1 = 0.f, nbe0 = 0.f, nbe1 = 0.f;
  auto load_gates = [&](int cc) {
    const int t = cc * C + 2 * lane;
    const size_t gi = ((size_t)b * a.n_tok + t) * a.n_vh + h;
    nl0 = nl1 = nbe0 = nbe1 = 0.f;
    if (t < a.n_tok) {
      nl0 = lgs[gi];
      nbe0 = gates[gi].x;
    }
    if (t + 1 < a.n_tok) {
      nl1 = lgs[gi + a.n_vh];
      nbe1 = gates[gi + a.n_vh].x;
    }
  };
  issue_kv(0);
  issue_q(0);
  if (warp == 0) load_gates(0);

  for (int c = 0; c < n_chunks; ++c) {
    const int t0 = c * C;
    float(*kb)[LDK] = sm.k[c & 1];
    float(*rb)[LDR] = sm.r[c & 1];
    cp_async_wait_all();
    __syncthreads();  // chunk c's K, Q, V landed; chunk c - 1's readers of k, r are done
    if (c + 1 < n_chunks) issue_kv(c + 1);
    const float l0 = nl0, l1 = nl1, be0 = nbe0, be1 = nbe1;
    if (warp == 0 && c + 1 < n_chunks) load_gates(c + 1);
    if (warp == 0) {
      // inclusive scan of the log decays (two tokens per lane); padded tokens: beta 0, decay 1
      float s = l0 + l1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      sm.L[2 * lane] = s - l1;
      sm.L[2 * lane + 1] = s;
      sm.beta[2 * lane] = be0;
      sm.beta[2 * lane + 1] = be1;
      const float LC = __shfl_sync(0xffffffffu, s, 31);
      sm.gam[2 * lane] = expf(s - l1);
      sm.gam[2 * lane + 1] = expf(s);
      sm.rdec[2 * lane] = expf(LC - (s - l1));
      sm.rdec[2 * lane + 1] = expf(LC - s);
    }
    __syncthreads();
    // ---- G = K K^T -> A;  RHS = beta (V - diag(gamma) K S0^T) over the V rows --------------
    {
      float acc[4][4];
      zero(acc);
      warp_mma<4, false, true, true>(acc, &kb[0][0], LDK, &kb[0][0], LDK, 16 * mt,
                                     32 * half, 0, DK);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * mt + g + (e >> 1) * 8, i = 32 * half + 8 * nt + 2 * qd + (e & 1);
          sm.a[t][i] = i < t ? sm.beta[t] * expf(sm.L[t] - sm.L[i]) * acc[nt][e] : 0.f;
        }
      zero(acc);
      warp_mma<4, false, true, true>(acc, &kb[0][0], LDK, &sm.s[0][0], LDK, 16 * mt,
                                     32 * half, 0, DK);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * mt + g + (e >> 1) * 8, j = 32 * half + 8 * nt + 2 * qd + (e & 1);
          rb[t][j] = sm.beta[t] * (rb[t][j] - sm.gam[t] * acc[nt][e]);
        }
    }
    __syncthreads();
    if (warp < 4) {
      // ---- diagonal 16x16 block `warp` of T = (I + A)^-1 in place; lane j = column j -------
      const int j = lane & 15, o = 16 * warp;
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
      if (lane < 16)
#pragma unroll
        for (int r = 0; r < 16; ++r) sm.a[o + r][o + j] = col[r];
    } else {
      // ---- meanwhile P = M o Q K^T, one 16-row tile per warp ------------------------------------
      const int m = warp - 4;
      float acc[8][4];
      zero(acc);
      warp_mma<8, false, true, true>(acc, &sm.q[0][0], LDK, &kb[0][0], LDK, 16 * m, 0, 0, DK);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * m + g + (e >> 1) * 8, i = 8 * nt + 2 * qd + (e & 1);
          sm.p[t][i] = i <= t ? expf(sm.L[t] - sm.L[i]) * acc[nt][e] : 0.f;
        }
    }
    __syncthreads();
    float o1[8][4];  // warps 4-7: diag(gamma) Q S0^T of their 16-row tile, kept across the sync
    if (warp < 4) {
      // ---- W = (I + A)^-1 RHS by blocked forward substitution, warp w owning 16 columns ------
      const int n0 = 16 * warp;
      for (int bi = 0; bi < 4; ++bi) {
        float acc[2][4];
        zero(acc);
        if (bi > 0)
          warp_mma<2, true, true, false>(acc, &sm.a[0][0], LDA, &rb[0][0], LDR, 16 * bi, n0,
                                         0, 16 * bi);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 16 * bi + g + (e >> 1) * 8, n = n0 + 8 * nt + 2 * qd + (e & 1);
            rb[t][n] -= acc[nt][e];
          }
        __syncwarp();
        zero(acc);
        warp_mma<2, true, true, false>(acc, &sm.a[0][0], LDA, &rb[0][0], LDR, 16 * bi, n0,
                                       16 * bi, 16 * bi + 16);
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 16 * bi + g + (e >> 1) * 8, n = n0 + 8 * nt + 2 * qd + (e & 1);
            rb[t][n] = acc[nt][e];
          }
        __syncwarp();
      }
    } else {
      const int m = warp - 4;
      zero(o1);
      warp_mma<8, false, true, true>(o1, &sm.q[0][0], LDK, &sm.s[0][0], LDK, 16 * m, 0, 0, DK);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o1[nt][e] *= sm.gam[16 * m + g + (e >> 1) * 8];
    }
    __syncthreads();  // W complete; S0 and Q no longer read
    if (c + 1 < n_chunks) issue_q(c + 1);
    if (warp >= 4) {
      // ---- O = diag(gamma) Q S0^T + P W -> global -------------------------------------------
      const int m = warp - 4;
      warp_mma<8, false, true, false>(o1, &sm.p[0][0], LDA, &rb[0][0], LDR, 16 * m, 0, 0,
                                      16 * m + 16);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int t = t0 + 16 * m + g + (e >> 1) * 8, j = 8 * nt + 2 * qd;
          if (t < a.n_tok) {
            bad |= !isfinite(o1[nt][e]) || !isfinite(o1[nt][e + 1]);
            *reinterpret_cast<float2*>(a.o + (size_t)b * a.o_bs + (size_t)t * a.o_ts +
                                       (size_t)h * a.dv + sl * DS + j) =
                make_float2(o1[nt][e], o1[nt][e + 1]);
          }
        }
    }
    // ---- S = gamma_C S0 + W^T diag(exp(L_C - L)) K  (3xTF32), warp w: its 16 x 64 share -------
    {
      float acc[8][4];
      zero(acc);
      warp_mma<8, true, false, false>(acc, &rb[0][0], LDR, &kb[0][0], LDK, 16 * mt,
                                      64 * half, 0, C, sm.rdec);
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
