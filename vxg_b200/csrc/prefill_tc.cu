// Causal GQA prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), bf16 inputs,
// head_dim 256.  Same semantics as prefill_attn.cu (token-by-token step_full_gqa_q8,
// llm_prefill.rs:497-517): the prompt's K/V are first appended to the Q8 cache by the bit-exact
// quantiser, then each query token attends causally to the dequantised cache.
//
// One CTA = 128 query rows (128 / G prompt tokens x the G query heads of one kv head), keys in
// tiles of 32, 16 warps with fixed roles:
//   warp 0       loader: one 2-D TMA tensor copy per cache and tile (this kv head's 272-byte
//                Q8 records of 32 tokens) from the KV pool into a 3-deep raw ring;
//   warp 1       QK MMA issuer (one thread) and TMEM owner; warp 13: PV MMA issuer (one thread);
//   warps 4-7    softmax: thread = query row = TMEM lane; also Q -> TMEM and the epilogue;
//   warps 2, 3, 8, 10 / 11, 12, 14, 15   K / V converters: Q8 records -> f16 hi/lo planes
//                in 128-byte-swizzled shared memory, double-buffered separately for K and V.
// Tensor memory (512 columns): O [0,256) f32, Q [256,384) f16 pairs, S0/S1 [384,512) f32.  The
// K hi and lo planes are stacked as 64 B-rows, so one MMA per K-step gives both halves of S:
//   [S_hi | S_lo] = Q [Kh ; Kl]^T                 (kind::f16, M=128, N=64, 16 K-steps)
//   O += Ph Vh + Ph Vl + Pl Vh                    (kind::f16, M=128, N=256, 3 x 2 K-steps)
// and the softmax reads S = S_hi + S_lo, then writes P (f16 hi and lo halves) over its S buffer;
// both MMAs take A from TMEM.
// bf16 queries are exact in f16, and Kh+Kl, Vh+Vl reproduce code*d exactly, so the products
// match the fp32 reference to ~2^-22 relative plus f32 accumulation rounding.
// The running max used as exponent base is only moved when a tile's max exceeds it by more
// than 8 (log2 units); P then stays <= 256, and O (in TMEM) is rescaled only on those moves.
// Every wait is bounded in wall-clock time; a wait that gives up raises the CTA's abort flag and
// the status word, and all roles leave their loops.
#include <cuda.h>
#include <cuda_bf16.h>

#include "kernels.h"
#include "tc.cuh"

namespace vxg {
namespace pftc {

constexpr int HD = 256;
constexpr int ROWS = 128;
constexpr int KT = 32;            // keys per tile
constexpr int NRAW = 3;           // raw Q8 ring depth
constexpr int REC = 272;          // bytes of one key's blocks for one kv head (8 x 34)
constexpr int THREADS = 512;
constexpr int PLANE = KT * 2 * HD;            // bytes of one f16 plane tile (16 KB)
constexpr uint32_t TM_O = 0, TM_Q = 256, TM_S = 384;  // S buffers: 64 columns each
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr float kRescale = 8.0f;  // log2 units

struct __align__(1024) Smem {
  uint8_t kpl[2][2 * PLANE];      // [stage]: [dim/64 (4)][row (64): Kh keys, then Kl][128 B]
  uint8_t vpl[2][2][PLANE];       // [stage][hi/lo]: [dim/64 (4)][key (32)][128 B]
  uint8_t raw[NRAW][2][KT * REC]; // [stage][K/V][key][272 B]
  uint64_t raw_full[NRAW], raw_empty[NRAW];
  uint64_t kf[2], vf[2];          // K / V planes of stage s written (converters -> issuer)
  uint64_t p_full[2];             // P of tile i written (softmax -> issuer)
  // QK / PV of tile i complete phase i >> 1 of qk_done / pv_done[i & 1]: one commit each tells
  // the softmax that S (resp. O) is ready and the converters that the K (resp. V) planes of
  // stage i & 1 are free
  uint64_t qk_done[2], pv_done[2];
  uint64_t q_full, drain[2];   // drain[0]: QK issuer, drain[1]: PV issuer
  uint32_t tmem;
  volatile int abort;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Smem& sm,
                                              uint32_t* status) {
  const uint32_t addr = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255u) == 0) {
      if (sm.abort) return false;
      const uint64_t t = globaltimer_ns();
      if (i == 0) {
        t0 = t;
      } else if (t - t0 > kWaitNs) {
        sm.abort = 1;
        atomicOr(status, kStatusTimeout);
        return false;
      }
    }
  }
}

// 2-D tiled tensor copy global -> shared completing on `bar` (this GPU's memory only).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Warp w issues on scheduler w % 4.  The converters sit on warps 2, 3, 8, 10, 11, 12, 14, 15, so
// the MMA-issuing warps 1 and 13 share their scheduler only with softmax warp 5 (warp 9 idle).
__device__ __forceinline__ int conv_index(int warp) {
  const int v = (int)((0x76f543f2ffff10ffull >> (4 * warp)) & 0xf);
  return v == 15 ? -1 : v;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// One (key, 32-dim block) item: 34-byte Q8 block at `blk` (2-byte aligned) -> 32 f16 values of
// the hi plane and 32 of the lo plane, written as 4 swizzled 16-byte chunks each.
// All arithmetic is f16x2 and exact where it has to be: the codes become f16 exactly
// (byte ^ 0x80 under the 0x64 exponent is 1024 + code + 128), hi = RN(code * d) is one rounded
// multiply, and lo = RN(code * d - hi) is one fused multiply-add whose result is exact (the
// residual has at most 8 significant bits).
__device__ __forceinline__ void convert_block(const uint8_t* blk, uint8_t* hi_plane,
                                              uint8_t* lo_plane, uint32_t atom_stride, int key,
                                              int c, bool valid) {
  uint32_t a[9];
  if (valid) {
    const uint32_t* wb =
        reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(blk) & ~uintptr_t(3));
    const uint32_t sh = (reinterpret_cast<uintptr_t>(blk) & 2u) ? 16u : 0u;
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = wb[i];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = __funnelshift_r(w[i], w[i + 1], sh);
    a[8] = w[8] >> sh;
  } else {
#pragma unroll
    for (int i = 0; i < 9; ++i) a[i] = 0u;
  }
  // a[0]: scale bits (low half), codes 0-1 (high half); a[i]: codes 4i-2 .. 4i+1
  const uint32_t d2u = __byte_perm(a[0], 0u, 0x1010);
  const __half2 d2 = *reinterpret_cast<const __half2*>(&d2u);
  const __half2 bias = __floats2half2_rn(1152.f, 1152.f);
  const int atom = c >> 1;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int p = 4 * m + q;  // codes 2p, 2p+1 sit in bytes 2p+2, 2p+3 of the stream
      const uint32_t w = a[(p + 1) >> 1] ^ 0x80808080u;
      const uint32_t bu = __byte_perm(w, 0x64646464u, ((p + 1) & 1) ? 0x4342 : 0x4140);
      const __half2 code = __hsub2(*reinterpret_cast<const __half2*>(&bu), bias);  // exact
      const __half2 hi = __hmul2(code, d2);
      const __half2 lo = __hfma2(code, d2, __hneg2(hi));
      h[q] = *reinterpret_cast<const uint32_t*>(&hi);
      l[q] = *reinterpret_cast<const uint32_t*>(&lo);
    }
    const uint32_t off = atom * atom_stride + tc::sw128_off(key, (c & 1) * 4 + m);
    *reinterpret_cast<uint4*>(hi_plane + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo_plane + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

}  // namespace pftc

// kmap / vmap: the K and V pools as 2-D u32 tensors [n_seq * cap rows][token bytes / 4], box
// 68 x 32 (one kv head's 272 bytes of 32 tokens).
__global__ void __launch_bounds__(pftc::THREADS, 1)
    prefill_tc_kernel(PrefillArgs a, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap) {
  using namespace pftc;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.n_head / a.n_kv;
  const int QT = ROWS / G;
  const int n_qb = (a.n_tok + QT - 1) / QT;
  const int qb = n_qb - 1 - (int)blockIdx.y;  // heavy (late) query blocks first
  const int b = blockIdx.x / a.n_kv, kh = blockIdx.x % a.n_kv;
  const int t0 = qb * QT;
  const int s = a.seq_ids[b];
  const int base = a.pos_base[b];
  const int len = base + a.n_tok;

  if (s < 0 || s >= a.n_seq || base < 0 || len > a.cap) {
    // the append flagged this entry; its rows are zeroed (uniform for the CTA)
    if (tid == 0) atomicOr(a.status, kStatusBadIndex);
    for (int r = warp; r < ROWS; r += THREADS / 32) {
      const int t = t0 + r / G;
      if (t >= a.n_tok) continue;
      float* o = a.out + (((size_t)b * a.n_tok + t) * a.n_head + kh * G + r % G) * HD;
      for (int i = lane; i < HD; i += 32) o[i] = 0.f;
    }
    return;
  }
  const int key_end = min(len, base + t0 + QT);
  const int n_tiles = (key_end + KT - 1) / KT;

  if (tid == 0) {
    for (int i = 0; i < NRAW; ++i) {
      mbar_init(&sm.raw_full[i], 1);
      mbar_init(&sm.raw_empty[i], 8);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kf[i], 4);
      mbar_init(&sm.vf[i], 4);
      mbar_init(&sm.qk_done[i], 1);
      mbar_init(&sm.pv_done[i], 1);
      mbar_init(&sm.p_full[i], ROWS);
    }
    mbar_init(&sm.q_full, ROWS);
    mbar_init(&sm.drain[0], 1);
    mbar_init(&sm.drain[1], 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&sm.tmem, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = sm.tmem;
  uint32_t* status = a.status;

  if (warp == 0) {
    // ---------------------------------------------------------------- loader
    if (lane == 0) {
      const int row0 = s * a.cap;
      for (int j = 0; j < n_tiles; ++j) {
        const int rs = j % NRAW;
        if (j >= NRAW && !wait_or_abort(&sm.raw_empty[rs], ((j / NRAW) - 1) & 1, sm, status))
          break;
        // whole boxes always land (rows past the sequence are other tokens or zero fill; the
        // converters ignore keys >= key_end)
        mbar_arrive_expect_tx(&sm.raw_full[rs], (uint32_t)(2 * KT * REC));
        tma_load_2d(sm.raw[rs][0], &kmap, kh * (REC / 4), row0 + j * KT, &sm.raw_full[rs]);
        tma_load_2d(sm.raw[rs][1], &vmap, kh * (REC / 4), row0 + j * KT, &sm.raw_full[rs]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- QK issuer
    // Two threads issue the MMAs: this one the QK products, warp 13's the PV products, each
    // waiting only for its own inputs, so a late P or late V planes do not hold back the next
    // tile's QK (and a late K tile does not hold back a PV).  QK of tile j + 2 overwrites the S
    // buffer that held P of tile j: it waits for that PV to complete first.
    if (lane == 0) {
      const uint32_t id_qk = tc::idesc_f16(128, 2 * KT, false);
      bool ok = wait_or_abort(&sm.q_full, 0, sm, status);
      tc::fence_after_sync();
      // Descriptors are built once; a K-step only adds its byte offset >> 4 to the start-address
      // field (the stage buffers lie far below the field's 256 KB limit), so issuing an MMA
      // costs a few instructions.
      const uint64_t kd0 = tc::sdesc_sw128(smem_u32(sm.kpl[0]), 16, 1024);
      const uint64_t kd1 = tc::sdesc_sw128(smem_u32(sm.kpl[1]), 16, 1024);
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j & 1;
        if (!wait_or_abort(&sm.kf[st], (j >> 1) & 1, sm, status)) break;
        if (j >= 2 && !wait_or_abort(&sm.pv_done[st], ((j >> 1) - 1) & 1, sm, status)) break;
        tc::fence_after_sync();
        const uint64_t kd = st ? kd1 : kd0;
        const uint32_t sd = tm + TM_S + 2 * KT * st;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * (2 * KT * 128) + (kk & 3) * 32;  // compile-time
          tc::mma_ts(sd, tm + TM_Q + kk * 8, kd + (uint64_t)(koff >> 4), id_qk, kk > 0 ? 1u : 0u);
        }
        tc::mma_commit(&sm.qk_done[st]);
      }
      // drain: every MMA issued here is done before the TMEM is released
      tc::mma_commit(&sm.drain[0]);
      mbar_wait(&sm.drain[0], 0, kWaitNs);
    }
    __syncwarp();
  } else if (warp == 13) {
    // ---------------------------------------------------------------- PV issuer
    if (lane == 0) {
      const uint32_t id_pv = tc::idesc_f16(128, HD, true);
      const uint64_t vh0 = tc::sdesc_sw128(smem_u32(sm.vpl[0][0]), KT * 128, 1024);
      const uint64_t vh1 = tc::sdesc_sw128(smem_u32(sm.vpl[1][0]), KT * 128, 1024);
      const uint64_t vl0 = tc::sdesc_sw128(smem_u32(sm.vpl[0][1]), KT * 128, 1024);
      const uint64_t vl1 = tc::sdesc_sw128(smem_u32(sm.vpl[1][1]), KT * 128, 1024);
      for (int i = 0; i < n_tiles; ++i) {
        const int st = i & 1;
        if (!wait_or_abort(&sm.vf[st], (i >> 1) & 1, sm, status)) break;
        if (!wait_or_abort(&sm.p_full[st], (i >> 1) & 1, sm, status)) break;
        tc::fence_after_sync();
        const uint32_t ph = tm + TM_S + 2 * KT * st, pl = ph + 16;
        const uint64_t vh = st ? vh1 : vh0, vl = st ? vl1 : vl0;
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
          // V planes as MN-major B: 64-dim column blocks 4 KB apart, 8-key groups 1 KB apart;
          // K-step kk starts 16 keys (2 KB) further
          const uint64_t dh = vh + (uint64_t)(kk * 2048 >> 4), dl = vl + (uint64_t)(kk * 2048 >> 4);
          tc::mma_ts(tm + TM_O, ph + kk * 8, dh, id_pv, (i > 0 || kk > 0) ? 1u : 0u);
          tc::mma_ts(tm + TM_O, ph + kk * 8, dl, id_pv, 1u);
          tc::mma_ts(tm + TM_O, pl + kk * 8, dh, id_pv, 1u);
        }
        tc::mma_commit(&sm.pv_done[st]);
      }
      tc::mma_commit(&sm.drain[1]);
      mbar_wait(&sm.drain[1], 0, kWaitNs);
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ---------------------------------------------------------------- softmax / Q / epilogue
    const int r = (warp - 4) * 32 + lane;  // query row = TMEM lane
    const uint32_t lane_addr = tm + ((uint32_t)((warp - 4) * 32) << 16);
    const int t = t0 + r / G;
    const int h = kh * G + r % G;
    const bool row_valid = t < a.n_tok;
    const int qpos = base + t;
    const size_t row_off = (((size_t)b * a.n_tok + (row_valid ? t : 0)) * a.n_head + h) * HD;
    const __nv_bfloat16* qrow = static_cast<const __nv_bfloat16*>(a.q) + row_off;
    // Q -> TMEM (f16 pairs; bf16 -> f16 is exact for |q| < 65504)
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch) {
      uint32_t v[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint4 raw = row_valid ? *reinterpret_cast<const uint4*>(qrow + ch * 64 + i * 8)
                              : make_uint4(0, 0, 0, 0);
        const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float lo = __uint_as_float(w4[k] << 16), hi = __uint_as_float(w4[k] & 0xFFFF0000u);
          v[i * 4 + k] = pack_h2(lo, hi);
        }
      }
      tc::tmem_st32(lane_addr + TM_Q + ch * 32, v);
    }
    tc::wait_st();
    tc::fence_before_sync();
    tc::mbar_arrive(&sm.q_full);

    const float sl2 = a.scale * 1.4426950408889634f;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    // PV of tile i done.  A waiter never lags two phases of pv_done[i & 1] behind: PV of tile
    // i + 2 needs this thread's P of tile i + 2 first.
    auto wait_pv = [&](int i) -> bool {
      return wait_or_abort(&sm.pv_done[i & 1], (i >> 1) & 1, sm, status);
    };
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (!wait_or_abort(&sm.qk_done[st], (j >> 1) & 1, sm, status)) { ok = false; break; }
      __syncwarp();
      tc::fence_after_sync();
      uint32_t sv[32], sl[32];
      tc::tmem_ld32(lane_addr + TM_S + 2 * KT * st, sv);       // Q Kh^T
      tc::tmem_ld32(lane_addr + TM_S + 2 * KT * st + KT, sl);  // Q Kl^T
      tc::wait_ld();
      float x[32];
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int key = j * KT + c;
        x[c] = key <= qpos ? (__uint_as_float(sv[c]) + __uint_as_float(sl[c])) * sl2 : -INFINITY;
        mx = fmaxf(mx, x[c]);
      }
      const bool move = mx > m_used + kRescale;
      if (__any_sync(0xffffffffu, move)) {  // warp-uniform: the TMEM accesses are .sync.aligned
        const float m_new = move ? mx : m_used;
        const float alpha = exp2f(m_used - m_new);  // 1 where the base stays, 0 on the first tile
        if (j > 0) {
          // O holds PV of tiles < j: rescale it in TMEM once the last of them is done
          if (!wait_pv(j - 1)) { ok = false; break; }
          __syncwarp();
          tc::fence_after_sync();
#pragma unroll 1
          for (int ch = 0; ch < HD / 32; ++ch) {
            uint32_t ov[32];
            tc::tmem_ld32(lane_addr + TM_O + ch * 32, ov);
            tc::wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tc::tmem_st32(lane_addr + TM_O + ch * 32, ov);
          }
          tc::wait_st();
        }
        l *= alpha;
        m_used = m_new;
      }
      uint32_t ph[16], pl[16];
      float ps = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float p0 = exp2f(x[2 * c] - m_used), p1 = exp2f(x[2 * c + 1] - m_used);
        ps += p0 + p1;
        const __half2 hh = __floats2half2_rn(p0, p1);
        const float2 hf = __half22float2(hh);
        ph[c] = *reinterpret_cast<const uint32_t*>(&hh);
        pl[c] = pack_h2(p0 - hf.x, p1 - hf.y);
      }
      l += ps;
      tc::tmem_st16(lane_addr + TM_S + 2 * KT * st, ph);
      tc::tmem_st16(lane_addr + TM_S + 2 * KT * st + 16, pl);
      tc::wait_st();
      tc::fence_before_sync();
      tc::mbar_arrive(&sm.p_full[st]);
    }
    // ---- epilogue: O / l, optional sigmoid gate, f32 out -----------------------------------
    // PV of the last tile done implies all earlier ones (one issuing thread, in order)
    if (ok && wait_pv(n_tiles - 1)) {
      __syncwarp();
      tc::fence_after_sync();
      const float inv = (l > 0.f || l != l) ? 1.0f / l : 0.f;
      const __nv_bfloat16* grow =
          a.gate ? static_cast<const __nv_bfloat16*>(a.gate) + row_off : nullptr;
      float* orow = a.out + row_off;
      bool bad = false;
#pragma unroll 1
      for (int ch = 0; ch < HD / 32; ++ch) {
        uint32_t ov[32];
        tc::tmem_ld32(lane_addr + TM_O + ch * 32, ov);
        tc::wait_ld();
        if (!row_valid) continue;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          float4 o4 = make_float4(__uint_as_float(ov[i]) * inv, __uint_as_float(ov[i + 1]) * inv,
                                  __uint_as_float(ov[i + 2]) * inv, __uint_as_float(ov[i + 3]) * inv);
          if (grow) {
            const int d = ch * 32 + i;
            o4.x *= 1.0f / (1.0f + expf(-__bfloat162float(grow[d])));
            o4.y *= 1.0f / (1.0f + expf(-__bfloat162float(grow[d + 1])));
            o4.z *= 1.0f / (1.0f + expf(-__bfloat162float(grow[d + 2])));
            o4.w *= 1.0f / (1.0f + expf(-__bfloat162float(grow[d + 3])));
          }
          bad |= !isfinite(o4.x) || !isfinite(o4.y) || !isfinite(o4.z) || !isfinite(o4.w);
          *reinterpret_cast<float4*>(orow + ch * 32 + i) = o4;
        }
      }
      if (bad) atomicOr(status, kStatusNonFinite);
    }
  } else if (conv_index(warp) >= 0) {
    // ---------------------------------------------------------------- converters
    // Converters 0-3 make the K planes, converters 4-7 the V planes, each thread two (key,
    // 32-dim block) items per tile, so K conversion of the next tile does not wait behind V
    // conversion (which waits for the PV that frees its planes).  Lane -> key 8 w + lane % 8 and
    // blocks {0,2,4,6} or {1,3,5,7}: record rows are 68 words apart, so 8 keys start in 8 banks =
    // 0 mod 4 and those four blocks at word offsets 0, 1, 2, 3 mod 4: the 32 lanes read 32
    // distinct banks, and the swizzled 16-byte stores of 8 keys cover all banks once per block.
    const int wc = conv_index(warp);
    const bool is_k = wc < 4;
    const int key = 8 * (wc & 3) + (lane & 7);
    const int c = 2 * (lane >> 3);
    uint64_t* free_bar = is_k ? sm.qk_done : sm.pv_done;
    uint64_t* full_bar = is_k ? sm.kf : sm.vf;
    for (int j = 0; j < n_tiles; ++j) {
      const int rs = j % NRAW, st = j & 1;
      if (!wait_or_abort(&sm.raw_full[rs], (j / NRAW) & 1, sm, status)) break;
      const bool valid = j * KT + key < key_end;
      // the planes of stage st are free once the QK (K) or PV (V) of tile j - 2 is done
      if (j >= 2 && !wait_or_abort(&free_bar[st], ((j >> 1) - 1) & 1, sm, status)) break;
      if (is_k) {
        const uint8_t* rec = sm.raw[rs][0] + key * REC;
        pftc::convert_block(rec + c * kBlk, sm.kpl[st], sm.kpl[st] + KT * 128, 2 * KT * 128, key,
                            c, valid);
        pftc::convert_block(rec + (c + 1) * kBlk, sm.kpl[st], sm.kpl[st] + KT * 128, 2 * KT * 128,
                            key, c + 1, valid);
      } else {
        const uint8_t* rec = sm.raw[rs][1] + key * REC;
        pftc::convert_block(rec + c * kBlk, sm.vpl[st][0], sm.vpl[st][1], KT * 128, key, c,
                            valid);
        pftc::convert_block(rec + (c + 1) * kBlk, sm.vpl[st][0], sm.vpl[st][1], KT * 128, key,
                            c + 1, valid);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&full_bar[st]);
        tc::mbar_arrive(&sm.raw_empty[rs]);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tm, 512);
}

size_t prefill_tc_smem_bytes() { return sizeof(pftc::Smem) + 1024; }

bool prefill_tc_supported(int n_head, int n_kv, int hd, int bf16) {
  // the pool's token rows (n_kv * 272 bytes) must be 16-byte multiples for the tensor map
  if (!bf16 || hd != 256 || n_kv <= 0 || n_head % n_kv != 0 || (n_kv * 272) % 16 != 0)
    return false;
  const int g = n_head / n_kv;
  return g >= 1 && pftc::ROWS % g == 0;
}

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}
// The pool as [n_seq * cap rows][tok_bytes / 4] u32, box = one kv head's record of 32 tokens.
bool encode_pool_map(CUtensorMap* map, const uint8_t* pool, const PrefillArgs& a) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const uint64_t tok_bytes = (uint64_t)a.n_kv * (a.hd / 32) * kBlk;
  const cuuint64_t dims[2] = {tok_bytes / 4, (cuuint64_t)a.n_seq * a.cap};
  const cuuint64_t strides[1] = {tok_bytes};
  const cuuint32_t box[2] = {pftc::REC / 4, pftc::KT};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(pool), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t launch_prefill_tc(const PrefillArgs& a, cudaStream_t st) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int smem = (int)prefill_tc_smem_bytes();
  if (dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  CUtensorMap kmap, vmap;
  if (!encode_pool_map(&kmap, a.k_pool, a) || !encode_pool_map(&vmap, a.v_pool, a))
    return cudaErrorInvalidValue;
  const int qt = pftc::ROWS / (a.n_head / a.n_kv);
  const dim3 grid(a.n_batch * a.n_kv, (a.n_tok + qt - 1) / qt);
  prefill_tc_kernel<<<grid, pftc::THREADS, smem, st>>>(a, kmap, vmap);
  return cudaGetLastError();
}

}  // namespace vxg
