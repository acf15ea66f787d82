// Gated-DeltaNet prompt recurrence in chunked (WY) form on the 5th-generation tensor cores
// (tcgen05 + tensor memory), dk = dv = 128.
//
// The reference applies the recurrence token by token (llm_prefill.rs:470-480 over
// llm_ops.rs:139-184): per v head, S <- g S; d = beta (v - S k); S <- S + d k^T; o = S q.  Over a
// chunk of C = 64 tokens with cumulative log decays L_t (gamma_t = e^{L_t}, chunk start L = 0;
// kept in log2 units on chip), with S0 the state entering the chunk, it re-associates exactly as
//   A[t][i] = beta_t e^{L_t - L_i} (k_t . k_i)  (i < t),     T = (I + A)^-1
//   R       = diag(beta) (V - diag(gamma) K S0^T),           W = T R
//   O       = diag(q_scale gamma) Q S0^T + P W,   P[t][i] = q_scale e^{L_t - L_i} (q_t . k_i), i <= t
//   S_C     = gamma_C S0 + W^T diag(e^{L_C - L}) K.
//
// One CTA per (sequence, v head) keeps the whole 128 x 128 f32 state in tensor memory, with the
// value dimension on the 128 TMEM lanes, so every state-sized product is one M = 128 MMA:
//   Z  = [K ; Q] K^T        f16 (q and k are unit-normalised)          -> A (rows 0-63), P (64-127)
//   X  = S0 K^T             bf16 x bf16                                -> R
//   Y  = S0 (q_scale gamma Q)^T + W^T P^T    hi/lo-split bf16 (3 MMAs each)  -> O^T
//   W^T = R^T T^T           hi/lo-split bf16                           (the triangular solve)
//   S += W^T (e^{L_C - L} K)  hi/lo-split bf16, after S *= gamma_C      (the state update)
// These are the operand formats of the mma.sync chunk kernel (deltanet_chunk.cu), chosen by a
// model of every product's rounding against the f64 recurrence; T itself is formed from f32 16 x 16
// diagonal blocks (substitution on the CUDA cores) and two merges of block products on mma.sync
// with the same hi/lo-split bf16 operands.
// S0, R^T and W^T enter their MMAs as A operands from tensor memory (bf16 pairs); K, Q, T and P
// are 128-byte-swizzled shared-memory tiles.  Tensor memory (512 columns):
//   S [0,128) f32 | S0 hi [128,192) lo [192,256) | Z [256,320) then W^T hi/lo pairs |
//   X [320,384) then R^T hi/lo pairs | Y [384,448) | W^T accumulator [448,512).
// One thread issues the MMAs; 16 warps share the per-lane phases (a quarter of the columns each);
// every phase ends at a block barrier, and every wait for MMAs is
// bounded in wall-clock time (on timeout the status word's timeout bit is set and the CTA leaves
// its loop, draining its MMAs before it frees the tensor memory).
#include <cuda_bf16.h>

#include "dn_gates.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace vxg {
namespace dntc {

constexpr int C = 64;           // chunk length
constexpr int D = 128;          // dk = dv
constexpr int THREADS = 512;    // 16 warps: 4 per TMEM lane quarter
constexpr int TW = C / (THREADS / 128);   // token columns of a 64-column TMEM region per thread
constexpr int SW = D / (THREADS / 128);   // state columns per thread
constexpr int TILE = C * 128;   // one [64 rows][64 16-bit values] 128-byte-swizzled tile: 8 KB
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t TM_S = 0, TM_S0H = 128, TM_S0L = 192, TM_Z = 256, TM_X = 320, TM_Y = 384,
                   TM_W = 448;

struct __align__(1024) Smem {
  uint8_t kq16[2][2 * TILE];  // [dk block][row: K tokens 0-63, Q tokens 64-127][128 B]  f16
  uint8_t kb16[2][TILE];      // [dk block][token][128 B]  bf16 K
  uint8_t qp[2][2][TILE];     // [hi / lo][dk block][token][128 B]  bf16 q_scale gamma_t q_t
  uint8_t kpp[2][2][TILE];    // [hi / lo][dk block][token][128 B]  bf16 e^{L_C - L_t} k_t
  uint8_t tp[2][TILE];        // [hi / lo][t][128 B over i]  bf16 T
  uint8_t pp[2][TILE];        // [hi / lo][t][128 B over i]  bf16 P
  float af[C][C + 1];         // A (strictly lower triangular)
  float tf[C][C + 1];         // T (lower triangular, unit diagonal)
  float mt[2][16][17];        // block products of the T merges
  float mt32[32][33];
  // gates of chunk c in buffer c & 1 (the next chunk's are formed while this one computes):
  // L2 = cumulative log decay in log2 units
  float L2[2][C], beta[2][C], gam[2][C], rdec[2][C];
  uint64_t mma_bar, drain_bar;
  uint32_t tmem;
  volatile int abort;
};

// kind::f16 instruction descriptor with bf16 A and B (format 1 in bits 7-9 and 10-12).
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool b_mn_major) {
  return tc::idesc_f16(m, n, b_mn_major) | (1u << 7) | (1u << 10);
}

__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// (a, b) -> bf16 pairs hi = rn(x), lo = rn(x - hi): hi + lo carries 16 significant bits.
__device__ __forceinline__ void split_bf16(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16(a, b);
  lo = pack_bf16(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xFFFF0000u));
}
__device__ __forceinline__ void st16(uint8_t* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  *reinterpret_cast<uint4*>(p) = make_uint4(a, b, c, d);
}
// 16-byte asynchronous global -> shared copy (zero fill when !valid; src stays a valid address).
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

// 2^x from the MUFU unit (relative error about 2^-22 for normal results; tiny results flush to
// zero, which is what a decayed weight wants).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(
                   taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
               "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// One warp: acc (16 x 16, two 8-column tiles) += A (16 x K, row-major, leading dimension lda) *
// B (K x 16, leading dimension ldb), both f32 in shared memory, as hi/lo-split bf16 products
// (hi.hi + hi.lo + lo.hi).  acc[nt][e]: row g + 8 (e >> 1), column 8 nt + 2 q + (e & 1).
template <int K>
__device__ __forceinline__ void mma16x16_x3(float (&acc)[2][4], const float* A, int lda,
                                            const float* B, int ldb, int lane) {
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < K; k0 += 16) {
    uint32_t ah[4], al[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {  // a0: row g, k 2q | a1: row g+8 | a2: row g, k 2q+8 | a3
      const float* ap = A + (g + 8 * (r & 1)) * lda + k0 + 2 * q + 8 * (r >> 1);
      split_bf16(ap[0], ap[1], ah[r], al[r]);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const float* bp = B + (k0 + 2 * q) * ldb + 8 * nt + g;
      uint32_t bh0, bl0, bh1, bl1;
      split_bf16(bp[0], bp[ldb], bh0, bl0);
      split_bf16(bp[8 * ldb], bp[9 * ldb], bh1, bl1);
      mma_bf16_16816(acc[nt], al, bh0, bh1);
      mma_bf16_16816(acc[nt], ah, bl0, bl1);
      mma_bf16_16816(acc[nt], ah, bh0, bh1);
    }
  }
}

}  // namespace dntc

// grid: n_batch * n_vh.  Reads the raw q, k, v, beta_raw and alpha_raw of the arguments: the
// L2 norms of q and k and the gates are formed on chip.  The raw K and Q rows of chunk c + 1 are
// copied asynchronously into the space of the K / Q operand tiles (free once the chunk's first
// MMAs are done) while chunk c computes.  16 warps: warp w owns TMEM lanes 32 (w % 4) .. + 32
// and, in each per-lane phase, a quarter (w / 4) of the columns.
__global__ void __launch_bounds__(dntc::THREADS, 1) deltanet_chunk_tc_kernel(DeltaNetArgs a) {
  using namespace dntc;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q4 = warp & 3, wq = warp >> 2;  // TMEM lane quarter, column quarter
  const int row = 32 * q4 + lane;           // this thread's TMEM lane
  const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
  const int b = blockIdx.x / a.n_vh, h = blockIdx.x % a.n_vh;
  const int hk = h / (a.n_vh / a.n_kh);
  const float q_scale = a.q_scale;
  float* Sg = a.state + ((size_t)b * a.n_vh + h) * D * D;
  const int tc0 = TW * wq;  // this thread's tokens [tc0, tc0 + TW) of a 64-column region
  const int sc0 = SW * wq;  // this thread's state columns [sc0, sc0 + SW)

  if (tid == 0) {
    mbar_init(&sm.mma_bar, 1);
    mbar_init(&sm.drain_bar, 1);
    sm.abort = 0;
    fence_mbar_init();
  }

  if (warp == 0) {
    tc::tmem_alloc(&sm.tmem, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = sm.tmem;
  const uint32_t tl = tm + lane_off;  // this warp's lane quarter

  // ---- state columns [sc0, sc0 + SW) of row `row` -> bf16 hi / lo pairs of S0 --------------
  auto put_state_planes = [&](const uint32_t (&s)[SW]) {
    uint32_t hi[SW / 2], lo[SW / 2];
#pragma unroll
    for (int p = 0; p < SW / 2; ++p)
      split_bf16(__uint_as_float(s[2 * p]), __uint_as_float(s[2 * p + 1]), hi[p], lo[p]);
    tc::tmem_st16(tl + TM_S0H + sc0 / 2, hi);
    tc::tmem_st16(tl + TM_S0L + sc0 / 2, lo);
  };
  {
    uint32_t s[SW];
    const float4* src = reinterpret_cast<const float4*>(Sg + (size_t)row * D + sc0);
#pragma unroll
    for (int i = 0; i < SW / 4; ++i) {
      const float4 v = src[i];
      s[4 * i] = __float_as_uint(v.x); s[4 * i + 1] = __float_as_uint(v.y);
      s[4 * i + 2] = __float_as_uint(v.z); s[4 * i + 3] = __float_as_uint(v.w);
    }
    tc::tmem_st32(tl + TM_S + sc0, s);
    put_state_planes(s);
    tc::wait_st();
  }

  const uint32_t id_z = tc::idesc_f16(128, C, false);
  const uint32_t id_x = idesc_bf16(128, C, false);
  const uint32_t id_s = idesc_bf16(128, D, true);
  const int n_chunks = (a.n_tok + C - 1) / C;
  uint32_t mma_phase = 0;
  bool bad = false;
  // All threads wait for the MMAs committed so far; false (uniformly) if the wait gave up.
  auto wait_mma = [&]() -> bool {
    if (!mbar_wait(&sm.mma_bar, mma_phase & 1u, kWaitNs)) {
      sm.abort = 1;
      atomicOr(a.status, kStatusTimeout);
    }
    ++mma_phase;
    __syncthreads();
    tc::fence_after_sync();
    return !sm.abort;
  };
  auto sync_for_mma = [&]() {  // smem tiles and TMEM stores of this thread -> the MMA issuer
    fence_proxy_async_smem();
    tc::wait_st();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  };

  // raw K and Q rows of a chunk: [64][128] f32 each, in the space of kq16 / kb16 / qp
  float* stage_k = reinterpret_cast<float*>(sm.kq16[0]);
  float* stage_q = stage_k + C * D;
  auto issue_stage = [&](int cc) {
#pragma unroll
    for (int u = 0; u < 2 * C * D / 4 / THREADS; ++u) {
      const int i = tid + u * THREADS;          // 16-byte piece
      const int isq = i >> 11, r = (i >> 5) & (C - 1), p = i & 31;
      const int t = cc * C + r;
      const bool ok = t < a.n_tok;
      const float* src = (isq ? a.q : a.k) + (size_t)b * (isq ? a.q_bs : a.k_bs) +
                         (size_t)(ok ? t : 0) * (isq ? a.q_ts : a.k_ts) + (size_t)hk * D + 4 * p;
      cp_async16((isq ? stage_q : stage_k) + r * D + 4 * p, src, ok);
    }
    cp_async_commit();
  };
  issue_stage(0);
  // gates of chunk cc (warp 1): beta, and the inclusive scan of the log2 decays, into buffer
  // cc & 1; padding tokens get beta 0 and decay 1
  const float gA = a.ssm_a[h], gdt = a.dt_bias[h];
  // (warp 1 loads the raw inputs of chunk cc + 1 into registers once chunk cc's are formed)
  float gar0 = 0.f, gar1 = 0.f, gbr0 = 0.f, gbr1 = 0.f;
  auto load_raw_gates = [&](int cc) {
    const int t = cc * C + 2 * lane;
    const size_t gi = (size_t)b * a.g_bs + (size_t)t * a.g_ts + h;
    if (t < a.n_tok) {
      gar0 = a.alpha_raw[gi];
      gbr0 = a.beta_raw[gi];
    }
    if (t + 1 < a.n_tok) {
      gar1 = a.alpha_raw[gi + a.g_ts];
      gbr1 = a.beta_raw[gi + a.g_ts];
    }
  };
  auto form_gates = [&](int cc) {
    const int t = cc * C + 2 * lane, gb = cc & 1;
    float l0 = 0.f, l1 = 0.f, be0 = 0.f, be1 = 0.f;
    if (t < a.n_tok) {
      l0 = log_decay_of(gar0, gdt, gA) * kLog2e;
      be0 = sigmoidf_(gbr0);
    }
    if (t + 1 < a.n_tok) {
      l1 = log_decay_of(gar1, gdt, gA) * kLog2e;
      be1 = sigmoidf_(gbr1);
    }
    float s = l0 + l1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    const float LC = __shfl_sync(0xffffffffu, s, 31);
    sm.L2[gb][2 * lane] = s - l1;
    sm.L2[gb][2 * lane + 1] = s;
    sm.beta[gb][2 * lane] = be0;
    sm.beta[gb][2 * lane + 1] = be1;
    sm.gam[gb][2 * lane] = exp2f(s - l1);
    sm.gam[gb][2 * lane + 1] = exp2f(s);
    sm.rdec[gb][2 * lane] = exp2f(LC - (s - l1));
    sm.rdec[gb][2 * lane + 1] = exp2f(LC - s);
  };
  if (warp == 1) {
    load_raw_gates(0);
    form_gates(0);
    if (n_chunks > 1) load_raw_gates(1);
  }
  // raw V rows of a chunk ([64][128] f32) in the space of A / T, which are dead from the W^T
  // MMA of one chunk to the readout of the next
  float* stage_v = &sm.af[0][0];
  auto issue_stage_v = [&](int cc) {
#pragma unroll
    for (int u = 0; u < C * D / 4 / THREADS; ++u) {
      const int i = tid + u * THREADS;
      const int r = i >> 5, p = i & 31;
      const int t = cc * C + r;
      const bool ok = t < a.n_tok;
      cp_async16(stage_v + r * D + 4 * p,
                 a.v + (size_t)b * a.v_bs + (size_t)(ok ? t : 0) * a.v_ts + (size_t)h * D + 4 * p,
                 ok);
    }
    cp_async_commit();
  };
  issue_stage_v(0);

  for (int c = 0; c < n_chunks; ++c) {
    const int t0 = c * C;
    const int gb = c & 1;   // this chunk's gate buffer
    // ---- K and Q rows of the chunk (staged) -> L2-normalised -> the operand tiles ------------
    //      (8 values = one 16-byte chunk per item; the 16 items of a row sit on 16 adjacent lanes)
    cp_async_wait_all();
    __syncthreads();
    {
      constexpr int NIT = 2 * C * 16 / THREADS;
      float4 raw[NIT][2];
      float inv[NIT];
#pragma unroll
      for (int u = 0; u < NIT; ++u) {
        const int it = tid + u * THREADS;
        const int isq = it >> 10, r = (it >> 4) & (C - 1), ch = it & 15;
        const float4* src =
            reinterpret_cast<const float4*>((isq ? stage_q : stage_k) + r * D + 8 * ch);
        raw[u][0] = src[0];
        raw[u][1] = src[1];
        float sq = raw[u][0].x * raw[u][0].x;
        sq = fmaf(raw[u][0].y, raw[u][0].y, sq); sq = fmaf(raw[u][0].z, raw[u][0].z, sq);
        sq = fmaf(raw[u][0].w, raw[u][0].w, sq); sq = fmaf(raw[u][1].x, raw[u][1].x, sq);
        sq = fmaf(raw[u][1].y, raw[u][1].y, sq); sq = fmaf(raw[u][1].z, raw[u][1].z, sq);
        sq = fmaf(raw[u][1].w, raw[u][1].w, sq);
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        inv[u] = rsqrtf(sq + a.eps);   // q and k unit-normalised (q_scale is applied later)
      }
      __syncthreads();  // the staged rows are read: the tiles may overwrite them
#pragma unroll
      for (int u = 0; u < NIT; ++u) {
        const int it = tid + u * THREADS;
        const int isq = it >> 10, r = (it >> 4) & (C - 1), ch = it & 15;
        const int cb = ch >> 3, cc = ch & 7;
        const float n = inv[u];
        const float x[8] = {raw[u][0].x * n, raw[u][0].y * n, raw[u][0].z * n, raw[u][0].w * n,
                            raw[u][1].x * n, raw[u][1].y * n, raw[u][1].z * n, raw[u][1].w * n};
        const uint32_t off = tc::sw128_off(r, cc);
        const float f = isq ? q_scale * sm.gam[gb][r] : sm.rdec[gb][r];
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) split_bf16(x[2 * p] * f, x[2 * p + 1] * f, hi[p], lo[p]);
        st16(sm.kq16[cb] + (isq ? tc::sw128_off(C + r, cc) : off), pack_f16(x[0], x[1]),
             pack_f16(x[2], x[3]), pack_f16(x[4], x[5]), pack_f16(x[6], x[7]));
        if (isq) {
          st16(sm.qp[0][cb] + off, hi[0], hi[1], hi[2], hi[3]);
          st16(sm.qp[1][cb] + off, lo[0], lo[1], lo[2], lo[3]);
        } else {
          st16(sm.kb16[cb] + off, pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]),
               pack_bf16(x[4], x[5]), pack_bf16(x[6], x[7]));
          st16(sm.kpp[0][cb] + off, hi[0], hi[1], hi[2], hi[3]);
          st16(sm.kpp[1][cb] + off, lo[0], lo[1], lo[2], lo[3]);
        }
      }
    }
    sync_for_mma();
    // ---- Z = [K; Q] K^T, X = S0 K^T, Y = S0 (q_scale gamma Q)^T ------------------------------
    if (tid == 0) {
      const uint64_t dkq = tc::sdesc_sw128(smem_u32(sm.kq16[0]), 16, 1024);
      const uint64_t dkb = tc::sdesc_sw128(smem_u32(sm.kb16[0]), 16, 1024);
      const uint64_t dqh = tc::sdesc_sw128(smem_u32(sm.qp[0][0]), 16, 1024);
      const uint64_t dql = tc::sdesc_sw128(smem_u32(sm.qp[1][0]), 16, 1024);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t o128 = (uint64_t)(((kk >> 2) * 2 * TILE + (kk & 3) * 32) >> 4);
        const uint64_t o64 = (uint64_t)(((kk >> 2) * TILE + (kk & 3) * 32) >> 4);
        const uint32_t acc = kk > 0 ? 1u : 0u;
        tc::mma_ss(tm + TM_Z, dkq + o128, dkq + o128, id_z, acc);
        tc::mma_ts(tm + TM_X, tm + TM_S0H + 8 * kk, dkb + o64, id_x, acc);
        tc::mma_ts(tm + TM_Y, tm + TM_S0H + 8 * kk, dqh + o64, id_x, acc);
        tc::mma_ts(tm + TM_Y, tm + TM_S0H + 8 * kk, dql + o64, id_x, 1u);
        tc::mma_ts(tm + TM_Y, tm + TM_S0L + 8 * kk, dqh + o64, id_x, 1u);
      }
      tc::mma_commit(&sm.mma_bar);
    }
    if (warp == 1 && c + 1 < n_chunks) {  // while the MMAs run
      form_gates(c + 1);
      if (c + 2 < n_chunks) load_raw_gates(c + 2);
    }
    if (!wait_mma()) break;
    if (c + 1 < n_chunks) issue_stage(c + 1);  // the K / Q tiles are consumed
    // ---- Z -> A (lanes 0-63) and P (lanes 64-127); X -> R --------------------------------------
    {
      uint32_t zv[TW], xv[TW];
      tc::tmem_ld16(tl + TM_Z + tc0, zv);
      tc::tmem_ld16(tl + TM_X + tc0, xv);
      float vv[TW];   // V[t][row] of this thread's tokens, from the staged rows
#pragma unroll
      for (int k = 0; k < TW; ++k) vv[k] = stage_v[(tc0 + k) * D + row];
      tc::wait_ld();
      __syncthreads();  // every thread has its V values before A overwrites the staged rows
      if (q4 < 2) {  // A[t][i], t = row
        const int t = row;
        const float Lt = sm.L2[gb][t], bt = sm.beta[gb][t];
#pragma unroll
        for (int k = 0; k < TW; ++k) {
          const int i = tc0 + k;
          sm.af[t][i] = i < t ? bt * ex2(Lt - sm.L2[gb][i]) * __uint_as_float(zv[k]) : 0.f;
        }
      } else {       // P[t][i], t = row - 64
        const int t = row - C;
        const float Lt = sm.L2[gb][t];
#pragma unroll
        for (int m = 0; m < TW / 8; ++m) {
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int k0 = 8 * m + 2 * p, i0 = tc0 + k0;
            const float p0 =
                i0 <= t ? ex2(Lt - sm.L2[gb][i0]) * (__uint_as_float(zv[k0]) * q_scale) : 0.f;
            const float p1 =
                i0 + 1 <= t ? ex2(Lt - sm.L2[gb][i0 + 1]) * (__uint_as_float(zv[k0 + 1]) * q_scale)
                            : 0.f;
            split_bf16(p0, p1, hi[p], lo[p]);
          }
          const uint32_t off = tc::sw128_off(t, tc0 / 8 + m);
          st16(sm.pp[0] + off, hi[0], hi[1], hi[2], hi[3]);
          st16(sm.pp[1] + off, lo[0], lo[1], lo[2], lo[3]);
        }
      }
      // R[t][j] = beta_t (V[t][j] - gamma_t X[j][t]), j = row, this thread's TW tokens
      uint32_t rh[TW / 2], rl[TW / 2];
#pragma unroll
      for (int p = 0; p < TW / 2; ++p) {
        const int t = tc0 + 2 * p;
        const float r0 =
            sm.beta[gb][t] * (vv[2 * p] - sm.gam[gb][t] * __uint_as_float(xv[2 * p]));
        const float r1 = sm.beta[gb][t + 1] *
                         (vv[2 * p + 1] - sm.gam[gb][t + 1] * __uint_as_float(xv[2 * p + 1]));
        split_bf16(r0, r1, rh[p], rl[p]);
      }
      __syncthreads();  // every thread has read X before R^T overwrites it
      tmem_st8(tl + TM_X + tc0 / 2, rh);
      tmem_st8(tl + TM_X + 32 + tc0 / 2, rl);
    }
    __syncthreads();
    // ---- T = (I + A)^-1 -------------------------------------------------------------------
    // Diagonal 16 x 16 blocks by forward substitution, thread = (block, column): warp 0 inverts
    // blocks 0 and 1, warp 1 blocks 2 and 3.  Below the diagonal, by merges of lower-triangular
    // blocks: T [[X, 0], [Y, Z]] has the off-diagonal block -Z Y' X with Y' the off-diagonal block
    // of I + A.  Warp w then merges its pair, T_{2w+1,2w} = -T_{2w+1,2w+1} A_{2w+1,2w} T_{2w,2w},
    // and four warps the 32-row merge T[32:64, 0:32] = -T[32:64, 32:64] A[32:64, 0:32] T[0:32, 0:32],
    // on mma.sync with hi/lo-split bf16 operands.  The upper-right 16 x 16 blocks of the two
    // 32 x 32 diagonal blocks, read by that merge, are zeroed here (the staged V rows of the
    // previous chunk overwrote them).
    if (tid >= 64 && tid < 64 + 2 * 256 / 4) {
      const int i = tid - 64, bi = i >> 6, r = (i >> 2) & 15, c4 = 4 * (i & 3);
      float* z = &sm.tf[32 * bi + r][32 * bi + 16 + c4];
      z[0] = z[1] = z[2] = z[3] = 0.f;
    }
    if (tid < 64) {
      const int o = 16 * (tid >> 4), cl = tid & 15;
      float col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) col[r] = r == cl ? 1.f : 0.f;
#pragma unroll
      for (int r = 0; r < 15; ++r)
#pragma unroll
        for (int i = r + 1; i < 16; ++i) col[i] = fmaf(-sm.af[o + i][o + r], col[r], col[i]);
#pragma unroll
      for (int r = 0; r < 16; ++r) sm.tf[o + r][o + cl] = col[r];
      __syncwarp();
      const int ob = 32 * warp;  // this warp's pair: T_00 at (ob, ob), A_10 at (ob + 16, ob)
      const int g = lane >> 2, q = lane & 3;
      float m[2][4] = {};
      mma16x16_x3<16>(m, &sm.af[ob + 16][ob], C + 1, &sm.tf[ob][ob], C + 1, lane);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sm.mt[warp][g + 8 * (e >> 1)][8 * nt + 2 * q + (e & 1)] = m[nt][e];
      __syncwarp();
      float t2[2][4] = {};
      mma16x16_x3<16>(t2, &sm.tf[ob + 16][ob + 16], C + 1, &sm.mt[warp][0][0], 17, lane);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          sm.tf[ob + 16 + g + 8 * (e >> 1)][ob + 8 * nt + 2 * q + (e & 1)] = -t2[nt][e];
    }
    __syncthreads();
    if (warp < 4) {  // M = A[32:64, 0:32] T[0:32, 0:32], warp = 16 x 16 tile (rt, ct)
      const int rt = warp >> 1, ct = warp & 1, g = lane >> 2, q = lane & 3;
      float m[2][4] = {};
      mma16x16_x3<32>(m, &sm.af[32 + 16 * rt][0], C + 1, &sm.tf[0][16 * ct], C + 1, lane);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          sm.mt32[16 * rt + g + 8 * (e >> 1)][16 * ct + 8 * nt + 2 * q + (e & 1)] = m[nt][e];
    }
    __syncthreads();
    if (warp < 4) {  // T[32:64, 0:32] = -T[32:64, 32:64] M
      const int rt = warp >> 1, ct = warp & 1, g = lane >> 2, q = lane & 3;
      float t2[2][4] = {};
      mma16x16_x3<32>(t2, &sm.tf[32 + 16 * rt][32], C + 1, &sm.mt32[0][16 * ct], 33, lane);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          sm.tf[32 + 16 * rt + g + 8 * (e >> 1)][16 * ct + 8 * nt + 2 * q + (e & 1)] = -t2[nt][e];
    }
    __syncthreads();
    // T -> bf16 hi / lo tiles, row t, 8 values of i per item (zero above the diagonal)
    for (int it = tid; it < C * 8; it += THREADS) {
      const int t = it >> 3, ch = it & 7;
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int i = 8 * ch + 2 * p;
        split_bf16(i <= t ? sm.tf[t][i] : 0.f, i + 1 <= t ? sm.tf[t][i + 1] : 0.f, hi[p], lo[p]);
      }
      const uint32_t off = tc::sw128_off(t, ch);
      st16(sm.tp[0] + off, hi[0], hi[1], hi[2], hi[3]);
      st16(sm.tp[1] + off, lo[0], lo[1], lo[2], lo[3]);
    }
    sync_for_mma();
    // ---- W^T = R^T T^T ------------------------------------------------------------------------
    if (tid == 0) {
      const uint64_t dth = tc::sdesc_sw128(smem_u32(sm.tp[0]), 16, 1024);
      const uint64_t dtl = tc::sdesc_sw128(smem_u32(sm.tp[1]), 16, 1024);
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        const uint64_t o = (uint64_t)((kk * 32) >> 4);
        tc::mma_ts(tm + TM_W, tm + TM_X + 8 * kk, dth + o, id_x, kk > 0 ? 1u : 0u);
        tc::mma_ts(tm + TM_W, tm + TM_X + 8 * kk, dtl + o, id_x, 1u);
        tc::mma_ts(tm + TM_W, tm + TM_X + 32 + 8 * kk, dth + o, id_x, 1u);
      }
      tc::mma_commit(&sm.mma_bar);
    }
    // while the W^T MMAs run (they touch neither): S *= gamma_C, and the next chunk's V rows
    // are staged over A / T (consumed: T is in its tiles)
    {
      uint32_t s[SW];
      tc::tmem_ld32(tl + TM_S + sc0, s);
      tc::wait_ld();
      const float gc = sm.gam[gb][C - 1];
#pragma unroll
      for (int k = 0; k < SW; ++k) s[k] = __float_as_uint(__uint_as_float(s[k]) * gc);
      tc::tmem_st32(tl + TM_S + sc0, s);
    }
    if (c + 1 < n_chunks) issue_stage_v(c + 1);
    if (!wait_mma()) break;
    // ---- W^T -> bf16 hi / lo pairs (over the consumed Z columns) ------------------------------
    {
      uint32_t wv[TW];
      tc::tmem_ld16(tl + TM_W + tc0, wv);
      tc::wait_ld();
      uint32_t wh[TW / 2], wl[TW / 2];
#pragma unroll
      for (int p = 0; p < TW / 2; ++p)
        split_bf16(__uint_as_float(wv[2 * p]), __uint_as_float(wv[2 * p + 1]), wh[p], wl[p]);
      tmem_st8(tl + TM_Z + tc0 / 2, wh);
      tmem_st8(tl + TM_Z + 32 + tc0 / 2, wl);
    }
    sync_for_mma();
    // ---- Y += W^T P^T; S += W^T (e^{L_C - L} K) ---------------------------------------------
    if (tid == 0) {
      const uint64_t dph = tc::sdesc_sw128(smem_u32(sm.pp[0]), 16, 1024);
      const uint64_t dpl = tc::sdesc_sw128(smem_u32(sm.pp[1]), 16, 1024);
      const uint64_t dkh = tc::sdesc_sw128(smem_u32(sm.kpp[0][0]), TILE, 1024);
      const uint64_t dkl = tc::sdesc_sw128(smem_u32(sm.kpp[1][0]), TILE, 1024);
#pragma unroll
      for (int kk = 0; kk < C / 16; ++kk) {
        const uint64_t o = (uint64_t)((kk * 32) >> 4);
        const uint64_t om = (uint64_t)((kk * 16 * 128) >> 4);  // 16 token rows per K-step
        const uint32_t wh = tm + TM_Z + 8 * kk, wl = tm + TM_Z + 32 + 8 * kk;
        tc::mma_ts(tm + TM_Y, wh, dph + o, id_x, 1u);
        tc::mma_ts(tm + TM_Y, wh, dpl + o, id_x, 1u);
        tc::mma_ts(tm + TM_Y, wl, dph + o, id_x, 1u);
        tc::mma_ts(tm + TM_S, wh, dkh + om, id_s, 1u);
        tc::mma_ts(tm + TM_S, wh, dkl + om, id_s, 1u);
        tc::mma_ts(tm + TM_S, wl, dkh + om, id_s, 1u);
      }
      tc::mma_commit(&sm.mma_bar);
    }
    if (!wait_mma()) break;
    // ---- O = Y^T -> global; S -> the next chunk's S0 pairs -----------------------------------
    {
      uint32_t yv[TW], s[SW];
      tc::tmem_ld16(tl + TM_Y + tc0, yv);
      tc::tmem_ld32(tl + TM_S + sc0, s);
      tc::wait_ld();
      float* op = a.o + (size_t)b * a.o_bs + (size_t)(t0 + tc0) * a.o_ts + (size_t)h * D + row;
      const int nt = min(TW, a.n_tok - (t0 + tc0));
#pragma unroll
      for (int k = 0; k < TW; ++k) {
        if (k < nt) {
          const float o = __uint_as_float(yv[k]);
          bad |= !isfinite(o);
          *op = o;
        }
        op += a.o_ts;
      }
      put_state_planes(s);
    }
    tc::wait_st();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }
  // ---- the final state -> global (or, after a timeout, drain the MMAs and leave it) ---------
  if (!sm.abort) {
    uint32_t s[SW];
    tc::tmem_ld32(tl + TM_S + sc0, s);
    tc::wait_ld();
    float4* dst = reinterpret_cast<float4*>(Sg + (size_t)row * D + sc0);
#pragma unroll
    for (int i = 0; i < SW / 4; ++i)
      dst[i] = make_float4(__uint_as_float(s[4 * i]), __uint_as_float(s[4 * i + 1]),
                           __uint_as_float(s[4 * i + 2]), __uint_as_float(s[4 * i + 3]));
  } else if (tid == 0) {
    tc::mma_commit(&sm.drain_bar);
    mbar_wait(&sm.drain_bar, 0, kWaitNs);
  }
  if (bad) atomicOr(a.status, kStatusNonFinite);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 512);
}

bool deltanet_chunk_tc_supported(const DeltaNetArgs& a) {
  // rows of q, k and v are copied in 16-byte pieces: 16-byte aligned bases and strides
  const bool aligned =
      ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
        reinterpret_cast<uintptr_t>(a.v)) & 15u) == 0 &&
      a.q_bs % 4 == 0 && a.q_ts % 4 == 0 && a.k_bs % 4 == 0 && a.k_ts % 4 == 0 &&
      a.v_bs % 4 == 0 && a.v_ts % 4 == 0;
  return aligned && a.dk == dntc::D && a.dv == dntc::D && a.n_tok >= dntc::C;
}

size_t deltanet_chunk_tc_smem_bytes() { return sizeof(dntc::Smem) + 1024; }

cudaError_t launch_deltanet_chunk_tc(const DeltaNetArgs& a, cudaStream_t st) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int smem = (int)deltanet_chunk_tc_smem_bytes();
  if (dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(deltanet_chunk_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  deltanet_chunk_tc_kernel<<<(unsigned)(a.n_batch * a.n_vh), dntc::THREADS, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace vxg
