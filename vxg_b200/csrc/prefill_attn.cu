// Causal GQA prefill attention over the Q8_0 KV cache.
//
// Reference semantics: prefill runs the decode step token by token (llm_prefill.rs:497-517
// calling step_full_gqa_q8, :259-370): token i's K/V are quantised into the cache, then token i's
// query attends to the Q8-dequantised cache [0, pos_i].  Quantising a token never depends on
// other tokens, so this equals: append all prompt tokens, then causal attention over the
// dequantised cache.  That is what runs here:
//   1. q8_append (bit-exact quantiser) for the n_tok new tokens of every sequence;
//   2. dequant: cache tokens [0, pos_base + n_tok) -> two f16 planes hi + lo with
//      hi = f16(code * d), lo = f16(code * d - hi).  code * d is exact in f32 (8-bit code times
//      11-bit scale) and hi + lo reproduces it (the residual has at most 8 significant bits);
//   3. flash attention on tensor cores (mma.sync m16n8k16, f16 x f16 -> f32): per CTA 128 query
//      rows = (128 / G) prompt tokens x the G query heads of one kv head, so each K/V tile is
//      shared by all of them; key tiles double-buffered by cp.async; online softmax in the log2
//      domain; causal mask on the diagonal tiles.
// Accuracy: plain f16 operands put the result only just inside the 1e-3 bar at short contexts
// (rounding K, V and P to 11 bits each moves a 1-2 key softmax by up to ~1e-3).  So every
// product is formed from split operands: S = Qh Kh + Qh Kl (+ Ql Kh for f32 queries; bf16
// queries are exact in f16), O = Ph Vh + Ph Vl + Pl Vh with P = Ph + Pl.  The dropped terms are
// ~2^-22 relative; the result matches the fp32 reference to accumulation-order rounding.
#include "kernels.h"

#include <algorithm>
#include <type_traits>

namespace vxg {

namespace pf {
constexpr int ROWS = 128;          // query rows per CTA
constexpr int THREADS = 256;       // 8 warps x 16 rows
template <int HD, bool QSPLIT>
struct Cfg {
  static constexpr int KT = QSPLIT ? 16 : 32;  // keys per tile (smem: q planes + 2 stages)
  static constexpr int RS = HD + 8;  // row stride in halves (odd multiple of 16 B: ldmatrix rows
                                     // fall in distinct bank groups)
  static constexpr int NQ = QSPLIT ? 2 : 1;
};
template <int HD, bool QSPLIT>
struct __align__(128) Smem {
  using C = Cfg<HD, QSPLIT>;
  __half q[C::NQ][ROWS][C::RS];       // [hi/lo][row][dim]
  __half k[2][2][C::KT][C::RS];       // [stage][hi/lo][key][dim]
  __half v[2][2][C::KT][C::RS];
};
}  // namespace pf

size_t prefill_smem_bytes() { return sizeof(pf::Smem<256, true>); }

// ---- dequantisation of the cache into f16 hi/lo planes -------------------------------------
__global__ void __launch_bounds__(256) q8_dequant_f16_kernel(PrefillArgs a) {
  // one thread per 8 codes (16-byte chunks of each plane)
  const int nb = a.hd / 32;
  const long long per_tok = (long long)a.n_kv * a.hd / 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)a.n_batch * a.lmax * per_tok;
  if (idx >= total) return;
  const int b = (int)(idx / ((long long)a.lmax * per_tok));
  const long long r = idx - (long long)b * a.lmax * per_tok;
  const int t = (int)(r / per_tok);
  const int e = (int)(r - (long long)t * per_tok) * 8;  // element within the token (kv*hd + dim)
  const int s = a.seq_ids[b];
  const int len = a.pos_base[b] + a.n_tok;
  const size_t off = ((size_t)b * a.lmax + t) * a.n_kv * a.hd + e;
  if (t >= len || s < 0 || s >= a.n_seq || a.pos_base[b] < 0 || len > a.cap) {
    for (int p = 0; p < 2; ++p) {
      *reinterpret_cast<uint4*>(a.kd[p] + off) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(a.vd[p] + off) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int kv = e / a.hd, dim = e % a.hd, c = dim / 32, i0 = dim % 32;
  const size_t boff = (((size_t)s * a.cap + t) * a.n_kv * nb + (size_t)kv * nb + c) * kBlk;
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const uint8_t* blk = (which ? a.v_pool : a.k_pool) + boff;
    const float d = f16bits_to_f32(*reinterpret_cast<const uint16_t*>(blk));
    __align__(16) __half hi[8];
    __align__(16) __half lo[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = (float)(int8_t)blk[2 + i0 + j] * d;  // exact
      hi[j] = __float2half_rn(x);
      lo[j] = __float2half_rn(x - __half2float(hi[j]));
    }
    __half* const* dst = which ? a.vd : a.kd;
    *reinterpret_cast<uint4*>(dst[0] + off) = *reinterpret_cast<const uint4*>(hi);
    *reinterpret_cast<uint4*>(dst[1] + off) = *reinterpret_cast<const uint4*>(lo);
  }
}

// ---- helpers -----------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = smem_u32(smem);
  const int n = valid ? 16 : 0;  // 0 source bytes: the 16 destination bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
// (x0, x1) -> f16x2 hi and f16x2 residual lo
__device__ __forceinline__ void h2_split(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = h2(x0 - hf.x, x1 - hf.y);
}
template <typename T>
__device__ __forceinline__ float ld_in(const T* p, size_t i);
template <>
__device__ __forceinline__ float ld_in<float>(const float* p, size_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_in<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) {
  return __bfloat162float(p[i]);
}

// ---- attention -----------------------------------------------------------------------------
// Row r of the CTA's 128 query rows is (prompt token t0 + r / G, query head kh * G + r % G).
template <typename T, int HD, bool QSPLIT>
__global__ void __launch_bounds__(pf::THREADS, 1) prefill_attn_kernel(PrefillArgs a) {
  using namespace pf;
  using C = Cfg<HD, QSPLIT>;
  constexpr int KT = C::KT;
  using S = Smem<HD, QSPLIT>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int G = a.n_head / a.n_kv;
  const int QT = ROWS / G;                    // prompt tokens per CTA
  const int n_qb = (a.n_tok + QT - 1) / QT;
  const int qb = n_qb - 1 - (int)blockIdx.y;  // CTAs start in launch order: heavy (late) query
                                              // blocks of every sequence first
  const int b = blockIdx.x / a.n_kv, kh = blockIdx.x % a.n_kv;
  const int t0 = qb * QT;                     // first prompt token of this CTA
  const int s = a.seq_ids[b];
  const int base = a.pos_base[b];
  const int len = base + a.n_tok;             // keys [0, len)
  const T* qin = static_cast<const T*>(a.q);
  const int r0 = 16 * warp + g, r1 = r0 + 8;  // the two rows of this thread
  const int tq0 = t0 + r0 / G, tq1 = t0 + r1 / G;
  const size_t orow0 = (((size_t)b * a.n_tok + tq0) * a.n_head + kh * G + r0 % G) * HD;
  const size_t orow1 = (((size_t)b * a.n_tok + tq1) * a.n_head + kh * G + r1 % G) * HD;

  if (s < 0 || s >= a.n_seq || base < 0 || len > a.lmax || len > a.cap) {
    // the append flagged (or the host rejected) this entry; its rows are zeroed
    if (tid == 0) atomicOr(a.status, kStatusBadIndex);
    for (int i = 2 * q; i < HD; i += 8) {
      if (tq0 < a.n_tok) *reinterpret_cast<float2*>(a.out + orow0 + i) = make_float2(0.f, 0.f);
      if (tq1 < a.n_tok) *reinterpret_cast<float2*>(a.out + orow1 + i) = make_float2(0.f, 0.f);
    }
    return;
  }
  const int key_end = min(len, base + t0 + QT);  // causal limit of the CTA's last token
  const int n_tiles = (key_end + KT - 1) / KT;

  // ---- Q -> f16 (hi, and lo for f32 queries) in smem -------------------------------------------
  for (int idx = tid; idx < ROWS * (HD / 8); idx += THREADS) {
    const int r = idx / (HD / 8), c8 = (idx % (HD / 8)) * 8;
    const int t = t0 + r / G, h = kh * G + r % G;
    __align__(16) __half vh[8];
    __align__(16) __half vl[8];
    const size_t off = (((size_t)b * a.n_tok + t) * a.n_head + h) * HD + c8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = t < a.n_tok ? ld_in<T>(qin, off + j) : 0.f;
      vh[j] = __float2half_rn(x);
      vl[j] = __float2half_rn(x - __half2float(vh[j]));
    }
    *reinterpret_cast<uint4*>(&sm.q[0][r][c8]) = *reinterpret_cast<const uint4*>(vh);
    if constexpr (QSPLIT)
      *reinterpret_cast<uint4*>(&sm.q[QSPLIT ? 1 : 0][r][c8]) = *reinterpret_cast<const uint4*>(vl);
  }
  auto load_tile = [&](int j, int buf) {
    for (int idx = tid; idx < KT * (HD / 8); idx += THREADS) {
      const int r = idx / (HD / 8), c8 = (idx % (HD / 8)) * 8;
      const int key = j * KT + r;
      const bool valid = key < key_end;
      const size_t off = (((size_t)b * a.lmax + (valid ? key : 0)) * a.n_kv + kh) * HD + c8;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        cp_async16(&sm.k[buf][p][r][c8], a.kd[p] + off, valid);
        cp_async16(&sm.v[buf][p][r][c8], a.vd[p] + off, valid);
      }
    }
    cp_async_commit();
  };
  if (n_tiles > 0) load_tile(0, 0);

  const float sl2 = a.scale * 1.4426950408889634f;
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int qpos0 = base + tq0, qpos1 = base + tq1;
  const int qr = 16 * warp + (lane & 15), qc = 8 * (lane >> 4);

  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_tiles) {
      load_tile(j + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // ---- S = Q K^T: 16 rows x KT keys per warp ----------------------------------------------
    float sc[KT / 8][4];
#pragma unroll
    for (int nt = 0; nt < KT / 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t af[4], afl[4];
      ldsm_x4(af, &sm.q[0][qr][kk * 16 + qc]);
      if constexpr (QSPLIT) ldsm_x4(afl, &sm.q[QSPLIT ? 1 : 0][qr][kk * 16 + qc]);
#pragma unroll
      for (int np = 0; np < KT / 16; ++np) {
        uint32_t bh[4], bl[4];
        // lanes 0-7: keys np*16 + l, dims kk*16; 8-15: same keys, dims +8;
        // 16-23: keys np*16 + 8 + l, dims kk*16; 24-31: those keys, dims +8
        const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(bh, &sm.k[buf][0][key][col]);
        ldsm_x4(bl, &sm.k[buf][1][key][col]);
        mma_f16(sc[2 * np], af, bl[0], bl[1]);
        mma_f16(sc[2 * np + 1], af, bl[2], bl[3]);
        if constexpr (QSPLIT) {
          mma_f16(sc[2 * np], afl, bh[0], bh[1]);
          mma_f16(sc[2 * np + 1], afl, bh[2], bh[3]);
        }
        mma_f16(sc[2 * np], af, bh[0], bh[1]);
        mma_f16(sc[2 * np + 1], af, bh[2], bh[3]);
      }
    }
    // ---- causal mask, online softmax (log2 domain) ------------------------------------------
    const bool diag = (j + 1) * KT > qpos0 + 1;  // some key of the tile may follow a query
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < KT / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j * KT + nt * 8 + 2 * q + (e & 1);
        const int qp = (e & 2) ? qpos1 : qpos0;
        float v = sc[nt][e] * sl2;
        if (diag && key > qp) v = -INFINITY;
        sc[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(m_r[r], mx[r]);
      const float mu = mn == -INFINITY ? 0.f : mn;  // fully masked so far: keep exp2 finite
      alpha[r] = exp2f(m_r[r] - mu);
      m_r[r] = mn;
      mx[r] = mu;
    }
    float ps[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < KT / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        sc[nt][e] = exp2f(sc[nt][e] - mx[e >> 1]);
        ps[e >> 1] += sc[nt][e];
      }
    l_r[0] = l_r[0] * alpha[0] + ps[0];
    l_r[1] = l_r[1] * alpha[1] + ps[1];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    // ---- O += P V with P = Ph + Pl, V = Vh + Vl (Pl Vl dropped) -------------------------------
#pragma unroll
    for (int kk = 0; kk < KT / 16; ++kk) {
      uint32_t ph[4], pl[4];
      h2_split(sc[2 * kk][0], sc[2 * kk][1], ph[0], pl[0]);
      h2_split(sc[2 * kk][2], sc[2 * kk][3], ph[1], pl[1]);
      h2_split(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph[2], pl[2]);
      h2_split(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph[3], pl[3]);
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t vh[4], vl[4];
        // transposed loads (rows = keys): lanes 0-7 keys kk*16 + l, dims dp*16; 8-15 keys +8;
        // 16-23 keys kk*16 + l, dims +8; 24-31 keys +8, dims +8
        const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = dp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(vh, &sm.v[buf][0][key][col]);
        ldsm_x4_t(vl, &sm.v[buf][1][key][col]);
        mma_f16(o[2 * dp], pl, vh[0], vh[1]);
        mma_f16(o[2 * dp + 1], pl, vh[2], vh[3]);
        mma_f16(o[2 * dp], ph, vl[0], vl[1]);
        mma_f16(o[2 * dp + 1], ph, vl[2], vl[3]);
        mma_f16(o[2 * dp], ph, vh[0], vh[1]);
        mma_f16(o[2 * dp + 1], ph, vh[2], vh[3]);
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }

  // ---- normalise, optional sigmoid gate, store --------------------------------------------
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  const T* gin = static_cast<const T*>(a.gate);
  bool bad = false;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if ((r ? tq1 : tq0) >= a.n_tok) continue;
    const size_t off = r ? orow1 : orow0;
    const float inv = (l_r[r] > 0.f || l_r[r] != l_r[r]) ? 1.0f / l_r[r] : 0.f;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      const int d = i * 8 + 2 * q;
      float v0 = o[i][2 * r] * inv, v1 = o[i][2 * r + 1] * inv;
      if (gin) {
        v0 *= 1.0f / (1.0f + expf(-ld_in<T>(gin, off + d)));
        v1 *= 1.0f / (1.0f + expf(-ld_in<T>(gin, off + d + 1)));
      }
      bad |= !isfinite(v0) || !isfinite(v1);
      *reinterpret_cast<float2*>(a.out + off + d) = make_float2(v0, v1);
    }
  }
  if (bad) atomicOr(a.status, kStatusNonFinite);
}

size_t prefill_scratch_bytes(const PrefillArgs& a) {
  return 4 * ((size_t)a.n_batch * a.lmax * a.n_kv * a.hd * sizeof(__half) + 256);
}

template <typename T, int HD>
static cudaError_t run_attn(const PrefillArgs& a, cudaStream_t st) {
  constexpr bool QSPLIT = std::is_same<T, float>::value;
  using S = pf::Smem<HD, QSPLIT>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(prefill_attn_kernel<T, HD, QSPLIT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(S));
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  const int qt = pf::ROWS / (a.n_head / a.n_kv);
  const dim3 grid(a.n_batch * a.n_kv, (a.n_tok + qt - 1) / qt);
  prefill_attn_kernel<T, HD, QSPLIT><<<grid, pf::THREADS, sizeof(S), st>>>(a);
  return cudaGetLastError();
}

bool prefill_supported(int n_head, int n_kv, int hd) {
  if (n_kv <= 0 || n_head % n_kv != 0) return false;
  const int g = n_head / n_kv;
  return (hd == 64 || hd == 128 || hd == 256) && g >= 1 && pf::ROWS % g == 0;
}

cudaError_t launch_prefill(const PrefillArgs& a0, void* scratch, int bf16, int allow_tc,
                           cudaStream_t st, cudaEvent_t ev0, cudaEvent_t ev1) {
  PrefillArgs a = a0;
  if (a.n_batch == 0 || a.n_tok == 0) return cudaSuccess;
  if (!prefill_supported(a.n_head, a.n_kv, a.hd)) return cudaErrorInvalidValue;
  const bool tcpath = allow_tc && prefill_tc_supported(a.n_head, a.n_kv, a.hd, bf16);
  // four 256-byte aligned planes: K hi, K lo, V hi, V lo
  const size_t plane = ((size_t)a.n_batch * a.lmax * a.n_kv * a.hd * sizeof(__half) + 255) &
                       ~size_t(255);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  a.kd[0] = reinterpret_cast<__half*>(base);
  a.kd[1] = reinterpret_cast<__half*>(base + plane);
  a.vd[0] = reinterpret_cast<__half*>(base + 2 * plane);
  a.vd[1] = reinterpret_cast<__half*>(base + 3 * plane);
  // 1. append the prompt's K/V (bit-exact quantiser)
  uint8_t* kp = const_cast<uint8_t*>(a.k_pool);
  uint8_t* vp = const_cast<uint8_t*>(a.v_pool);
  cudaError_t e =
      bf16 ? launch_q8_append_bf16(a.seq_ids, a.pos_base, a.k_new, a.v_new, kp, vp, a.n_batch,
                                   a.n_tok, a.n_seq, a.cap, a.n_kv, a.hd / 32, a.status, st)
           : launch_q8_append(a.seq_ids, a.pos_base, static_cast<const float*>(a.k_new),
                              static_cast<const float*>(a.v_new), kp, vp, a.n_batch, a.n_tok,
                              a.n_seq, a.cap, a.n_kv, a.hd / 32, a.status, st);
  if (e != cudaSuccess) return e;
  if (tcpath) {
    // tensor-memory kernel: dequantises the Q8 records on chip
    if (ev0) cudaEventRecord(ev0, st);
    e = launch_prefill_tc(a, st);
    if (ev1) cudaEventRecord(ev1, st);
    return e;
  }
  // 2. dequantise [0, pos_base + n_tok) into the f16 hi/lo planes
  const long long chunks = (long long)a.n_batch * a.lmax * a.n_kv * a.hd / 8;
  q8_dequant_f16_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(a);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // 3. causal attention
  if (ev0) cudaEventRecord(ev0, st);
  switch (a.hd) {
    case 64: e = bf16 ? run_attn<__nv_bfloat16, 64>(a, st) : run_attn<float, 64>(a, st); break;
    case 128: e = bf16 ? run_attn<__nv_bfloat16, 128>(a, st) : run_attn<float, 128>(a, st); break;
    default: e = bf16 ? run_attn<__nv_bfloat16, 256>(a, st) : run_attn<float, 256>(a, st); break;
  }
  if (ev1) cudaEventRecord(ev1, st);
  return e;
}

}  // namespace vxg
