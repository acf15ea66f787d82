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
// state), chunks in order, state rows on chip.  The products run on mma.sync m16n8k16 with f32
// accumulation, each in the operand format its accuracy needs (measured against the sequential
// f32 recurrence at 8192 tokens): K K^T and Q K^T in f16 (q and k are L2-normalised, |x| <= 1,
// and q's scale is applied to the products); K S0^T in bf16; Q S0^T, P W, the triangular solve
// and the state update in hi/lo-split bf16 (BF16X3), which keeps the f32 exponent range for the
// unbounded state and W.  Operands stay f32 in shared memory and are converted per fragment.
#include "kernels.h"

namespace vxg {
namespace dnc {

constexpr int C = 64;        // chunk length
constexpr int DK = 128;
constexpr int DS = 64;       // state rows (v dims) per CTA
constexpr int THREADS = 256;
// Row strides (floats), chosen for conflict-free fragment loads (see KOrder): K, Q, S (PAIR
// loads, and SPREAD loads along k for the state update) and R (SPREAD loads along k) want 8
// mod 32; A / T and P (SPREAD loads along their rows) want 4 mod 32.
constexpr int LDK = DK + 8;       // K, Q, S
constexpr int LDR = DS + 8;       // R: V rows -> right-hand side -> W
constexpr int LDA = C + 4;        // A / T, P

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

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// two f32 -> one register of two 16-bit values, x0 in the low half (the lower k index)
__device__ __forceinline__ uint32_t pack_f16(float x0, float x1) {
  const __half2 h = __floats2half2_rn(x0, x1);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf16(float x0, float x1) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// (x0, x1) -> bf16 pairs hi = rn(x), lo = rn(x - hi); hi + lo carries 16 significant bits
__device__ __forceinline__ void split_bf16(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16(x0, x1);
  lo = pack_bf16(x0 - __uint_as_float(hi << 16), x1 - __uint_as_float(hi & 0xFFFF0000u));
}

// Operand formats of a product.  F16: one f16 pass, for the normalised q / k (|x| <= 1, so no
// range loss).  BF16: one bf16 pass.  BF16X3: hi/lo bf16 splits of both operands and the three
// products hi.hi + hi.lo + lo.hi (16 significant bits per operand, the f32 exponent range).
enum Fmt { F16, BF16, BF16X3 };
// k orders of a 16-wide k step.  The MMA's k slots of lane quad q are 2q, 2q+1 (a0/a1, b0) and
// 2q+8, 2q+9 (a2/a3, b1); any permutation of k applied to both operands leaves the product
// unchanged.  PAIR keeps slot = k, so a k-contiguous operand loads as 64-bit pairs (row
// strides of 8 mod 32 words are conflict-free).  SPREAD maps slots 2q+j -> q+4j and
// 2q+8+j -> q+8+4j: scalar loads, conflict-free for a [k][m|n] operand with row stride 8 mod 32
// and for an [m|n][k] operand with row stride 4 mod 32.
enum KOrder { PAIR, SPREAD };

// acc[i][nt] (+)= A(m0[i].., k) B(k, n0 + 8 nt ..) over k in [k0, k1) (a multiple of 16): MT
// 16-row tiles sharing each B fragment, NT 8-col tiles of which the first nt_cnt are computed.
// A is [m][k] (AK) or [k][m]; B is [n][k] (BK) or [k][n]; ascale (optional) scales A's column
// k.  SEP keeps the two BF16X3 correction products in their own accumulators (shorter
// dependency chains for small NT).
template <int MT, int NT, Fmt FMT, KOrder KO, bool AK, bool BK, bool SEP = false>
__device__ __forceinline__ void warp_mma_mt(float (&acc)[MT][NT][4], const float* A, int lda,
                                            const int (&m0)[MT], const float* B, int ldb, int n0,
                                            int k0, int k1, const float* ascale = nullptr,
                                            int nt_cnt = NT) {
  static_assert(KO == SPREAD || (AK && BK), "PAIR order needs k-contiguous operands");
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  constexpr bool X3 = FMT == BF16X3;
  constexpr int NC = X3 && SEP ? NT : 1;
  float c1[MT][NC][4], c2[MT][NC][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NC; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) c1[i][j][e] = c2[i][j][e] = 0.f;
  // physical k of slots (2q, 2q+1, 2q+8, 2q+9)
  const int o0 = KO == PAIR ? 2 * q : q, o1 = KO == PAIR ? 2 * q + 1 : q + 4;
  const int o2 = o0 + 8, o3 = o1 + 8;
  for (int k = k0; k < k1; k += 16) {
    // a0 = row g slots 0,1; a1 = row g+8 slots 0,1; a2 = row g slots 2,3; a3 = row g+8 slots 2,3
    uint32_t ah[MT][4], al[MT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      float x[2][4];  // rows g, g + 8; slots 0..3
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int m = m0[i] + g + 8 * h;
        if constexpr (KO == PAIR) {
          const float2 r0 = *reinterpret_cast<const float2*>(A + m * lda + k + o0);
          const float2 r1 = *reinterpret_cast<const float2*>(A + m * lda + k + o2);
          x[h][0] = r0.x; x[h][1] = r0.y; x[h][2] = r1.x; x[h][3] = r1.y;
        } else if constexpr (AK) {
          x[h][0] = A[m * lda + k + o0]; x[h][1] = A[m * lda + k + o1];
          x[h][2] = A[m * lda + k + o2]; x[h][3] = A[m * lda + k + o3];
        } else {
          x[h][0] = A[(k + o0) * lda + m]; x[h][1] = A[(k + o1) * lda + m];
          x[h][2] = A[(k + o2) * lda + m]; x[h][3] = A[(k + o3) * lda + m];
        }
        if (ascale) {
          x[h][0] *= ascale[k + o0]; x[h][1] *= ascale[k + o1];
          x[h][2] *= ascale[k + o2]; x[h][3] *= ascale[k + o3];
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int h = r & 1, s0 = (r >> 1) * 2;
        if constexpr (FMT == F16) ah[i][r] = pack_f16(x[h][s0], x[h][s0 + 1]);
        else if constexpr (FMT == BF16) ah[i][r] = pack_bf16(x[h][s0], x[h][s0 + 1]);
        else split_bf16(x[h][s0], x[h][s0 + 1], ah[i][r], al[i][r]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (nt >= nt_cnt) break;
      const int n = n0 + 8 * nt + g;
      float y[4];
      if constexpr (KO == PAIR) {
        const float2 r0 = *reinterpret_cast<const float2*>(B + n * ldb + k + o0);
        const float2 r1 = *reinterpret_cast<const float2*>(B + n * ldb + k + o2);
        y[0] = r0.x; y[1] = r0.y; y[2] = r1.x; y[3] = r1.y;
      } else if constexpr (BK) {
        y[0] = B[n * ldb + k + o0]; y[1] = B[n * ldb + k + o1];
        y[2] = B[n * ldb + k + o2]; y[3] = B[n * ldb + k + o3];
      } else {
        y[0] = B[(k + o0) * ldb + n]; y[1] = B[(k + o1) * ldb + n];
        y[2] = B[(k + o2) * ldb + n]; y[3] = B[(k + o3) * ldb + n];
      }
      if constexpr (FMT == F16) {
        const uint32_t b0 = pack_f16(y[0], y[1]), b1 = pack_f16(y[2], y[3]);
#pragma unroll
        for (int i = 0; i < MT; ++i) mma_f16(acc[i][nt], ah[i], b0, b1);
      } else if constexpr (FMT == BF16) {
        const uint32_t b0 = pack_bf16(y[0], y[1]), b1 = pack_bf16(y[2], y[3]);
#pragma unroll
        for (int i = 0; i < MT; ++i) mma_bf16(acc[i][nt], ah[i], b0, b1);
      } else {
        uint32_t bh0, bl0, bh1, bl1;
        split_bf16(y[0], y[1], bh0, bl0);
        split_bf16(y[2], y[3], bh1, bl1);
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          if constexpr (SEP) {
            mma_bf16(c1[i][nt], al[i], bh0, bh1);
            mma_bf16(c2[i][nt], ah[i], bl0, bl1);
          } else {
            mma_bf16(acc[i][nt], al[i], bh0, bh1);
            mma_bf16(acc[i][nt], ah[i], bl0, bl1);
          }
          mma_bf16(acc[i][nt], ah[i], bh0, bh1);
        }
      }
    }
  }
  if constexpr (X3 && SEP)
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][nt][e] += c1[i][nt][e] + c2[i][nt][e];
}

// one 16-row tile
template <int NT, Fmt FMT, KOrder KO, bool AK, bool BK, bool SEP = false>
__device__ __forceinline__ void warp_mma(float (&acc)[NT][4], const float* A, int lda,
                                         const float* B, int ldb, int m0, int n0, int k0, int k1,
                                         const float* ascale = nullptr, int nt_cnt = NT) {
  const int mm[1] = {m0};
  warp_mma_mt<1, NT, FMT, KO, AK, BK, SEP>(reinterpret_cast<float(&)[1][NT][4]>(acc), A, lda,
                                           mm, B, ldb, n0, k0, k1, ascale, nt_cnt);
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
    // ---- lower triangles of G = K K^T (warps 0-3, -> A) and Q K^T (warps 4-7, -> P) ---------
    // Only the 16x16 blocks on or below the diagonal are used: 20 8-column tiles per product,
    // dealt 5 to each warp as units (m-tile, first n-tile, count): warp u of a group takes
    // (3, 0, 5) | (3, 5, 3) + (0, 0, 2) | (2, 0, 5) | (2, 5, 1) + (1, 0, 4).
    {
      const int u = warp & 3;
      const bool is_g = warp < 4;
      const float* Aop = is_g ? &kb[0][0] : &sm.q[0][0];
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        const int m = v == 0 ? (u < 2 ? 3 : 2) : (u == 1 ? 0 : 1);
        const int nt0 = v == 0 && (u & 1) ? 5 : 0;
        const int cnt = v == 0 ? ((u & 1) ? (u == 1 ? 3 : 1) : 5) : (u == 1 ? 2 : (u == 3 ? 4 : 0));
        if (cnt == 0) continue;
        float acc[5][4];
        zero(acc);
        warp_mma<5, F16, PAIR, true, true>(acc, Aop, LDK, &kb[0][0], LDK, 16 * m, 8 * nt0, 0, DK,
                                           nullptr, cnt);
#pragma unroll
        for (int nt = 0; nt < 5; ++nt) {
          if (nt >= cnt) break;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 16 * m + g + (e >> 1) * 8, i = 8 * (nt0 + nt) + 2 * qd + (e & 1);
            if (is_g)
              sm.a[t][i] = i < t ? sm.beta[t] * expf(sm.L[t] - sm.L[i]) * acc[nt][e] : 0.f;
            else
              sm.p[t][i] = i <= t ? expf(sm.L[t] - sm.L[i]) * (acc[nt][e] * a.q_scale) : 0.f;
          }
        }
      }
    }
    // ---- RHS = beta (V - diag(gamma) K S0^T) over the V rows, warp (mt, half): 16 x 32 -------
    {
      float acc[4][4];
      zero(acc);
      warp_mma<4, BF16, PAIR, true, true>(acc, &kb[0][0], LDK, &sm.s[0][0], LDK, 16 * mt,
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
    // warps 4-7: q_scale diag(gamma) Q S0^T on the m-tile pair {pm, 3 - pm} (equal shares of the
    // triangular P W below), columns 32 ch .. 32 ch + 31; kept in registers across the sync
    const int pm = (warp >> 1) & 1, ch = warp & 1;
    const int mm[2] = {16 * pm, 16 * (3 - pm)};
    float o1[2][4][4];
    if (warp < 4) {
      // ---- diagonal 16x16 block `warp` of T = (I + A)^-1 in place; lane j = column j -------
      // Right-looking forward substitution: once x[r] is final it updates every later row, so
      // the dependency chain is one FMA per row (entries above row j stay 0 without masking).
      const int j = lane & 15, o = 16 * warp;
      float col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) col[r] = r == j ? 1.f : 0.f;
#pragma unroll
      for (int r = 0; r < 15; ++r)
#pragma unroll
        for (int i = r + 1; i < 16; ++i) col[i] = fmaf(-sm.a[o + i][o + r], col[r], col[i]);
      __syncwarp();
      if (lane < 16)
#pragma unroll
        for (int r = 0; r < 16; ++r) sm.a[o + r][o + j] = col[r];
      asm volatile("bar.sync 1, 128;" ::: "memory");  // warps 0-3: all four blocks inverted
      // ---- W = (I + A)^-1 RHS by blocked forward substitution, warp w owning 16 columns ------
      const int n0 = 16 * warp;
      for (int bi = 0; bi < 4; ++bi) {
        float acc[2][4];
        zero(acc);
        if (bi > 0)
          warp_mma<2, BF16X3, SPREAD, true, false, true>(acc, &sm.a[0][0], LDA, &rb[0][0], LDR,
                                                         16 * bi, n0, 0, 16 * bi);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 16 * bi + g + (e >> 1) * 8, n = n0 + 8 * nt + 2 * qd + (e & 1);
            rb[t][n] -= acc[nt][e];
          }
        __syncwarp();
        zero(acc);
        warp_mma<2, BF16X3, SPREAD, true, false, true>(acc, &sm.a[0][0], LDA, &rb[0][0], LDR,
                                                       16 * bi, n0, 16 * bi, 16 * bi + 16);
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
#pragma unroll
      for (int i = 0; i < 2; ++i) zero(o1[i]);
      warp_mma_mt<2, 4, BF16X3, PAIR, true, true>(o1, &sm.q[0][0], LDK, mm, &sm.s[0][0], LDK,
                                                  32 * ch, 0, DK);
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) o1[i][nt][e] *= sm.gam[mm[i] + g + (e >> 1) * 8] * a.q_scale;
    }
    __syncthreads();  // W complete; S0 and Q no longer read
    if (c + 1 < n_chunks) issue_q(c + 1);
    if (warp >= 4) {
      // ---- O = q_scale diag(gamma) Q S0^T + P W -> global ----------------------------------
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        warp_mma<4, BF16X3, SPREAD, true, false>(o1[i], &sm.p[0][0], LDA, &rb[0][0], LDR, mm[i],
                                                 32 * ch, 0, mm[i] + 16);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int t = t0 + mm[i] + g + (e >> 1) * 8, j = 32 * ch + 8 * nt + 2 * qd;
            if (t < a.n_tok) {
              bad |= !isfinite(o1[i][nt][e]) || !isfinite(o1[i][nt][e + 1]);
              *reinterpret_cast<float2*>(a.o + (size_t)b * a.o_bs + (size_t)t * a.o_ts +
                                         (size_t)h * a.dv + sl * DS + j) =
                  make_float2(o1[i][nt][e], o1[i][nt][e + 1]);
            }
          }
      }
    }
    // ---- S = gamma_C S0 + W^T diag(exp(L_C - L)) K  (BF16X3), warp w: its 16 x 64 share ------
    {
      float acc[8][4];
      zero(acc);
      warp_mma<8, BF16X3, SPREAD, false, false>(acc, &rb[0][0], LDR, &kb[0][0], LDK, 16 * mt,
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
