/*
 * vxg_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, statement-for-statement restatement of the vxg-tensor CPU operators on the
 * Q8-KV attention / gated-DeltaNet hot path.  It exists to check the CUDA backend (as the
 * parity oracle) and to time the reference algorithm on host cores (the CPU baseline).
 * Nothing in the product library calls, links or loads this file.
 *
 * Parity status of this restatement:
 *   - f32_to_f16 / f16_to_f32 are PINNED by the reference's own known-answer test
 *     (crates/vxg-tensor/src/fp16.rs:89-108), ported to tests/golden/fp16_kat.json.
 *   - Everything else is UNPINNED against the Rust binary: the reference is Rust, no Rust
 *     toolchain exists on this machine, and the reference ships no operator-level golden
 *     vectors.  It is cross-checked against an independent numpy restatement instead.
 *
 * Equivalences used (Rust -> C):  f32::mul_add -> fmaf;  round_ties_even -> rintf (default
 * FE_TONEAREST);  f32::exp/ln/sqrt/powf/sin/cos -> glibc expf/logf/sqrtf/powf/sinf/cosf;
 * f32::max/min (NaN-ignoring) -> fmaxf/fminf;  `as i8` (saturating, NaN -> 0) -> explicit.
 * Build with -ffp-contract=off: Rust never contracts a*b+c into an FMA on its own.
 *
 * Q8 block layout (crates/vxg-tensor/src/llm_prefill.rs:17-24): #[repr(C)] { d: u16, qs: [i8;32] }
 * = 34 bytes, d = IEEE binary16 bits stored little-endian at byte 0, qs at bytes 2..33.
 * Cache index of (token t, kv head kh, block b) = t*n_kv*(hd/32) + kh*(hd/32) + b
 * (llm_prefill.rs:311-324).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define VXO_BLK 34

/* ---- fp16.rs:6-29 ------------------------------------------------------------------------ */
float vxo_f16_to_f32(uint16_t bits) {
    uint32_t sign = ((uint32_t)(bits & 0x8000u)) << 16;
    uint32_t exp = (uint32_t)((bits >> 10) & 0x1f);
    uint32_t mant = (uint32_t)(bits & 0x03ff);
    uint32_t out;
    if (exp == 0) {
        if (mant == 0) {
            out = sign;
        } else {
            uint32_t m = mant;
            uint32_t e = 127u - 14u;
            while ((m & 0x0400u) == 0) {
                m <<= 1;
                e -= 1;
            }
            m &= 0x03ffu;
            out = sign | (e << 23) | (m << 13);
        }
    } else if (exp == 31) {
        out = sign | 0x7f800000u | (mant << 13);
    } else {
        out = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &out, 4);
    return f;
}

/* ---- fp16.rs:33-77 ----------------------------------------------------------------------- */
uint16_t vxo_f32_to_f16(float val) {
    uint32_t b;
    memcpy(&b, &val, 4);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    int32_t exp = (int32_t)((b >> 23) & 0xffu);
    uint32_t mant = b & 0x007fffffu;
    if (exp == 255) {
        if (mant != 0) return (uint16_t)(sign | 0x7e00u | (uint16_t)(mant >> 13));
        return (uint16_t)(sign | 0x7c00u);
    }
    int32_t unbiased = exp - 127;
    if (unbiased > 15) return (uint16_t)(sign | 0x7c00u);
    if (unbiased < -25) return sign;
    if (unbiased < -14) {
        uint32_t shift = (uint32_t)(-14 - unbiased);
        uint32_t full_mant = mant | 0x00800000u;
        uint32_t round_shift = 13u + shift;
        uint32_t half = 1u << (round_shift - 1);
        uint32_t mask = (1u << round_shift) - 1u;
        uint32_t rem = full_mant & mask;
        uint16_t m16 = (uint16_t)(full_mant >> round_shift);
        if (rem > half || (rem == half && (m16 & 1u) != 0)) m16 += 1;
        return (uint16_t)(sign | m16);
    }
    uint16_t e16 = (uint16_t)(((uint32_t)(unbiased + 15)) << 10);
    uint32_t rem = mant & 0x1fffu;
    uint16_t m16 = (uint16_t)(mant >> 13);
    if (rem > 0x1000u || (rem == 0x1000u && (m16 & 1u) != 0)) {
        m16 += 1;
        if (m16 == 0x0400u) return (uint16_t)(sign | (uint16_t)(e16 + 0x0400u));
    }
    return (uint16_t)(sign | e16 | m16);
}

static inline uint16_t blk_d(const uint8_t* blk) { return (uint16_t)(blk[0] | (blk[1] << 8)); }

/* Rust `x as i8` on an f32 already clamped to [-127, 127]: truncation toward zero, NaN -> 0. */
static inline int8_t sat_i8(float x) {
    if (x != x) return 0;
    return (int8_t)x;
}

/* ---- KvQ8Block::quantize, llm_prefill.rs:27-42 -------------------------------------------- */
void vxo_q8_quantize(const float* src, uint8_t* blk) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(src[i]));
    uint16_t dh = vxo_f32_to_f16(amax / 127.0f);
    float df = vxo_f16_to_f32(dh);
    float inv = df > 0.0f ? 1.0f / df : 0.0f;
    blk[0] = (uint8_t)(dh & 0xff);
    blk[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < 32; ++i) {
        float r = rintf(src[i] * inv);
        /* f32::clamp(-127, 127): NaN passes through */
        if (r < -127.0f) r = -127.0f;
        if (r > 127.0f) r = 127.0f;
        blk[2 + i] = (uint8_t)sat_i8(r);
    }
}

/* ---- KvQ8Block::dot_f32, llm_prefill.rs:45-54 --------------------------------------------- */
float vxo_q8_dot(const uint8_t* blk, const float* q) {
    float sc = vxo_f16_to_f32(blk_d(blk));
    const int8_t* qs = (const int8_t*)(blk + 2);
    float s0 = 0.0f, s1 = 0.0f;
    for (int i = 0; i < 16; ++i) {
        s0 = fmaf((float)qs[2 * i], q[2 * i], s0);
        s1 = fmaf((float)qs[2 * i + 1], q[2 * i + 1], s1);
    }
    return (s0 + s1) * sc;
}

/* ---- KvQ8Block::axpy_f32, llm_prefill.rs:57-62 -------------------------------------------- */
void vxo_q8_axpy(const uint8_t* blk, float weight, float* out) {
    float ws = weight * vxo_f16_to_f32(blk_d(blk));
    const int8_t* qs = (const int8_t*)(blk + 2);
    for (int i = 0; i < 32; ++i) out[i] = fmaf((float)qs[i], ws, out[i]);
}

/* ---- llm_ops.rs:39-46 silu / sigmoid ------------------------------------------------------ */
static inline float silu(float x) { return x / (1.0f + expf(-x)); }
static inline float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

/* ---- rms_norm, llm_ops.rs:48-57 ------------------------------------------------------------ */
void vxo_rms_norm(const float* x, const float* w, float eps, float* out, size_t n) {
    float sq = 0.0f;
    for (size_t i = 0; i < n; ++i) sq = fmaf(x[i], x[i], sq);
    float scale = 1.0f / sqrtf((sq / (float)n) + eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

/* ---- rms_norm_inplace, llm_ops.rs:59-68 ---------------------------------------------------- */
static void rms_norm_inplace(float* x, const float* w, float eps, size_t n) {
    float sq = 0.0f;
    for (size_t i = 0; i < n; ++i) sq = fmaf(x[i], x[i], sq);
    float scale = 1.0f / sqrtf((sq / (float)n) + eps);
    for (size_t i = 0; i < n; ++i) x[i] = x[i] * scale * w[i];
}

/* ---- l2_norm_scaled, llm_ops.rs:70-79 ------------------------------------------------------ */
void vxo_l2_norm_scaled(const float* x, float eps, float mul, float* out, size_t n) {
    float sq = 0.0f;
    for (size_t i = 0; i < n; ++i) sq = fmaf(x[i], x[i], sq);
    float scale = mul / sqrtf(sq + eps);
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * scale;
}

/* ---- apply_rope, llm_ops.rs:81-101 --------------------------------------------------------- */
void vxo_apply_rope(float* vec, size_t n, size_t pos, size_t rope_dim, float freq_base, int neox) {
    size_t rdim = rope_dim < n ? rope_dim : n;
    size_t half = rdim / 2;
    for (size_t i = 0; i < half; ++i) {
        float freq = powf(freq_base, -(2.0f * (float)i) / (float)rdim);
        float theta = (float)pos * freq;
        float sin_t = sinf(theta), cos_t = cosf(theta);
        if (neox) {
            float x0 = vec[i], x1 = vec[i + half];
            vec[i] = x0 * cos_t - x1 * sin_t;
            vec[i + half] = x0 * sin_t + x1 * cos_t;
        } else {
            float x0 = vec[2 * i], x1 = vec[2 * i + 1];
            vec[2 * i] = x0 * cos_t - x1 * sin_t;
            vec[2 * i + 1] = x0 * sin_t + x1 * cos_t;
        }
    }
}

/* ---- append half of step_full_gqa_q8, llm_prefill.rs:311-324 ------------------------------- *
 * k_q8 / v_q8 hold at least (pos+1) tokens (the Vec::resize of the reference is the caller's
 * capacity management here).  k_cur / v_cur are [n_kv][hd] f32 after any norm / RoPE. */
void vxo_q8_append(const float* k_cur, const float* v_cur, size_t n_kv, size_t hd, size_t pos,
                   uint8_t* k_q8, uint8_t* v_q8) {
    size_t blks = hd / 32;
    size_t stride = n_kv * blks;
    size_t base = pos * stride;
    for (size_t kh = 0; kh < n_kv; ++kh) {
        for (size_t b = 0; b < blks; ++b) {
            size_t off = kh * hd + b * 32;
            vxo_q8_quantize(k_cur + off, k_q8 + (base + kh * blks + b) * VXO_BLK);
            vxo_q8_quantize(v_cur + off, v_q8 + (base + kh * blks + b) * VXO_BLK);
        }
    }
}

/* ---- attention half of step_full_gqa_q8, llm_prefill.rs:326-369 ---------------------------- *
 * q_heads: [n_head][hd] prepared queries; gates: [n_head][hd] or NULL; attends to tokens
 * [0, seq_len) of the cache; scale is 1/sqrt(hd) in the reference (passed explicitly).
 * scores: caller scratch of seq_len floats (NULL -> malloc). */
void vxo_q8_attend(const float* q_heads, const float* gates, const uint8_t* k_q8,
                   const uint8_t* v_q8, size_t n_head, size_t n_kv, size_t hd, size_t seq_len,
                   float scale, float* attn_out, float* scores) {
    size_t blks = hd / 32;
    size_t stride = n_kv * blks;
    size_t gqa_mul = n_head / n_kv;
    int own = 0;
    if (!scores) {
        scores = (float*)malloc(sizeof(float) * (seq_len ? seq_len : 1));
        own = 1;
    }
    for (size_t h = 0; h < n_head; ++h) {
        size_t kv_h = h / gqa_mul;
        const float* qh = q_heads + h * hd;
        float max_s = -INFINITY;
        for (size_t t = 0; t < seq_len; ++t) {
            const uint8_t* kb = k_q8 + (t * stride + kv_h * blks) * VXO_BLK;
            float dot = 0.0f;
            for (size_t b = 0; b < blks; ++b) dot += vxo_q8_dot(kb + b * VXO_BLK, qh + b * 32);
            float s = dot * scale;
            scores[t] = s;
            if (s > max_s) max_s = s;
        }
        float sum_exp = 0.0f;
        for (size_t t = 0; t < seq_len; ++t) {
            float e = expf(scores[t] - max_s);
            scores[t] = e;
            sum_exp += e;
        }
        float inv_sum = 1.0f / sum_exp;
        float* out_h = attn_out + h * hd;
        for (size_t i = 0; i < hd; ++i) out_h[i] = 0.0f;
        for (size_t t = 0; t < seq_len; ++t) {
            float w = scores[t] * inv_sum;
            const uint8_t* vb = v_q8 + (t * stride + kv_h * blks) * VXO_BLK;
            for (size_t b = 0; b < blks; ++b) vxo_q8_axpy(vb + b * VXO_BLK, w, out_h + b * 32);
        }
        if (gates) {
            const float* gh = gates + h * hd;
            for (size_t i = 0; i < hd; ++i) out_h[i] *= 1.0f / (1.0f + expf(-gh[i]));
        }
    }
    if (own) free(scores);
}

/* ---- step_full_gqa_q8, llm_prefill.rs:259-370 (whole function) ----------------------------- *
 * q_raw: [n_head][hd] or, when gated_q, [n_head][2*hd] (query then gate per head).
 * k_cur is modified in place (norm + RoPE), as in the reference. q_norm / k_norm may be NULL. */
void vxo_step_full_gqa_q8(const float* q_raw, float* k_cur, const float* v_cur, const float* q_norm,
                          const float* k_norm, int gated_q, size_t n_head, size_t n_kv, size_t hd,
                          size_t pos, size_t rope_pos, size_t rope_dim, float rope_freq_base,
                          int rope_neox, float eps, uint8_t* k_q8, uint8_t* v_q8, float* attn_out) {
    float* q_heads = (float*)malloc(sizeof(float) * n_head * hd);
    float* q_gates = gated_q ? (float*)malloc(sizeof(float) * n_head * hd) : NULL;
    float* tmp = (float*)malloc(sizeof(float) * hd);
    for (size_t h = 0; h < n_head; ++h) {
        float* q_dst = q_heads + h * hd;
        if (gated_q) {
            const float* src = q_raw + h * 2 * hd;
            memcpy(q_dst, src, sizeof(float) * hd);
            memcpy(q_gates + h * hd, src + hd, sizeof(float) * hd);
        } else {
            memcpy(q_dst, q_raw + h * hd, sizeof(float) * hd);
        }
        if (q_norm) {
            memcpy(tmp, q_dst, sizeof(float) * hd);
            vxo_rms_norm(tmp, q_norm, eps, q_dst, hd);
        }
        vxo_apply_rope(q_dst, hd, rope_pos, rope_dim, rope_freq_base, rope_neox);
    }
    for (size_t kh = 0; kh < n_kv; ++kh) {
        float* ks = k_cur + kh * hd;
        if (k_norm) {
            memcpy(tmp, ks, sizeof(float) * hd);
            vxo_rms_norm(tmp, k_norm, eps, ks, hd);
        }
        vxo_apply_rope(ks, hd, rope_pos, rope_dim, rope_freq_base, rope_neox);
    }
    vxo_q8_append(k_cur, v_cur, n_kv, hd, pos, k_q8, v_q8);
    float scale = 1.0f / sqrtf((float)hd);
    vxo_q8_attend(q_heads, q_gates, k_q8, v_q8, n_head, n_kv, hd, pos + 1, scale, attn_out, NULL);
    free(tmp);
    free(q_gates);
    free(q_heads);
}

/* ---- step_full_gqa attention over fp32 caches, llm_ops.rs:255-299 ------------------------ *
 * k_cache / v_cache: [t][n_kv][hd] f32 holding at least seq_len tokens. */
void vxo_f32_attend(const float* q_heads, const float* gates, const float* k_cache,
                    const float* v_cache, size_t n_head, size_t n_kv, size_t hd, size_t seq_len,
                    float scale, float* att_cat, float* scores) {
    size_t kv_stride = n_kv * hd;
    size_t gqa_mul = n_head / n_kv;
    int own = 0;
    if (!scores) {
        scores = (float*)malloc(sizeof(float) * (seq_len ? seq_len : 1));
        own = 1;
    }
    for (size_t h = 0; h < n_head; ++h) {
        size_t kv_h = h / gqa_mul;
        const float* qh = q_heads + h * hd;
        float max_s = -INFINITY;
        for (size_t t = 0; t < seq_len; ++t) {
            const float* kh = k_cache + t * kv_stride + kv_h * hd;
            float dot = 0.0f;
            for (size_t d = 0; d < hd; ++d) dot = fmaf(qh[d], kh[d], dot);
            float s = dot * scale;
            scores[t] = s;
            if (s > max_s) max_s = s;
        }
        float sum_exp = 0.0f;
        for (size_t t = 0; t < seq_len; ++t) {
            scores[t] = expf(scores[t] - max_s);
            sum_exp += scores[t];
        }
        float inv_sum = 1.0f / sum_exp;
        float* out_h = att_cat + h * hd;
        for (size_t d = 0; d < hd; ++d) out_h[d] = 0.0f;
        for (size_t t = 0; t < seq_len; ++t) {
            float w = scores[t] * inv_sum;
            const float* vh = v_cache + t * kv_stride + kv_h * hd;
            for (size_t d = 0; d < hd; ++d) out_h[d] = fmaf(w, vh[d], out_h[d]);
        }
        if (gates) {
            const float* gh = gates + h * hd;
            for (size_t d = 0; d < hd; ++d) out_h[d] *= 1.0f / (1.0f + expf(-gh[d]));
        }
    }
    if (own) free(scores);
}

/* ---- step_full_gqa, llm_ops.rs:196-300 (whole function): the fp32-KV operator ----------- *
 * k_cache / v_cache: [>= pos+1][n_kv][hd]; the token is written at row pos (the reference
 * extends its vectors, so row pos is the new last row). */
void vxo_step_full_gqa(const float* q_raw, float* k_cur, const float* v_cur, const float* q_norm,
                       const float* k_norm, int gated_q, size_t n_head, size_t n_kv, size_t hd,
                       size_t pos, size_t rope_dim, float rope_freq_base, int rope_neox, float eps,
                       float* k_cache, float* v_cache, float* att_cat) {
    float* q_cur = (float*)malloc(sizeof(float) * n_head * hd);
    float* q_gate = gated_q ? (float*)malloc(sizeof(float) * n_head * hd) : NULL;
    float* tmp = (float*)malloc(sizeof(float) * hd);
    for (size_t h = 0; h < n_head; ++h) {
        if (gated_q) {
            memcpy(q_cur + h * hd, q_raw + h * 2 * hd, sizeof(float) * hd);
            memcpy(q_gate + h * hd, q_raw + h * 2 * hd + hd, sizeof(float) * hd);
        } else {
            memcpy(q_cur + h * hd, q_raw + h * hd, sizeof(float) * hd);
        }
    }
    if (q_norm)
        for (size_t h = 0; h < n_head; ++h) {
            memcpy(tmp, q_cur + h * hd, sizeof(float) * hd);
            vxo_rms_norm(tmp, q_norm, eps, q_cur + h * hd, hd);
        }
    if (k_norm)
        for (size_t h = 0; h < n_kv; ++h) {
            memcpy(tmp, k_cur + h * hd, sizeof(float) * hd);
            vxo_rms_norm(tmp, k_norm, eps, k_cur + h * hd, hd);
        }
    for (size_t h = 0; h < n_head; ++h)
        vxo_apply_rope(q_cur + h * hd, hd, pos, rope_dim, rope_freq_base, rope_neox);
    for (size_t h = 0; h < n_kv; ++h)
        vxo_apply_rope(k_cur + h * hd, hd, pos, rope_dim, rope_freq_base, rope_neox);
    memcpy(k_cache + pos * n_kv * hd, k_cur, sizeof(float) * n_kv * hd);
    memcpy(v_cache + pos * n_kv * hd, v_cur, sizeof(float) * n_kv * hd);
    float scale = 1.0f / sqrtf((float)hd);
    vxo_f32_attend(q_cur, q_gate, k_cache, v_cache, n_head, n_kv, hd, pos + 1, scale, att_cat,
                   NULL);
    free(tmp);
    free(q_gate);
    free(q_cur);
}

/* ---- gated-DeltaNet core, llm_ops.rs:139-184 ----------------------------------------------- *
 * q_all/k_all: [n_kh][dk] (before L2 norm); v_all: [n_vh][dv]; state: [n_vh][dv][dk] updated in
 * place; o: [n_vh][dv] = S_new q (before the RMSNorm / SiLU(z) epilogue).  q_scale is
 * 1/sqrt(dk) in the reference (llm_ops.rs:145). */
void vxo_deltanet_core(const float* q_all, const float* k_all, const float* v_all,
                       const float* beta_raw, const float* alpha_raw, const float* ssm_a,
                       const float* dt_bias, size_t n_kh, size_t n_vh, size_t dk, size_t dv,
                       float eps, float q_scale, float* state, float* o) {
    float* q_h = (float*)malloc(sizeof(float) * dk);
    float* k_h = (float*)malloc(sizeof(float) * dk);
    for (size_t h = 0; h < n_vh; ++h) {
        size_t hk = h / (n_vh / n_kh);
        vxo_l2_norm_scaled(q_all + hk * dk, eps, q_scale, q_h, dk);
        vxo_l2_norm_scaled(k_all + hk * dk, eps, 1.0f, k_h, dk);
        const float* v_h = v_all + h * dv;
        float beta = sigmoid(beta_raw[h]);
        float x_sp = alpha_raw[h] + dt_bias[h];
        float sp;
        if (x_sp > 20.0f) sp = x_sp;
        else if (x_sp < -20.0f) sp = expf(x_sp);
        else sp = logf(1.0f + expf(x_sp));
        float decay = expf(sp * ssm_a[h]);
        float* sh = state + h * dv * dk;
        for (size_t jv = 0; jv < dv; ++jv) {
            float* row = sh + jv * dk;
            float sk = 0.0f;
            for (size_t ik = 0; ik < dk; ++ik) {
                float sd = row[ik] * decay;
                row[ik] = sd;
                sk = fmaf(sd, k_h[ik], sk);
            }
            float d_jv = (v_h[jv] - sk) * beta;
            float o_jv = 0.0f;
            for (size_t ik = 0; ik < dk; ++ik) {
                float sn = fmaf(d_jv, k_h[ik], row[ik]);
                row[ik] = sn;
                o_jv = fmaf(sn, q_h[ik], o_jv);
            }
            o[h * dv + jv] = o_jv;
        }
    }
    free(k_h);
    free(q_h);
}

/* ---- step_deltanet_recurrent, llm_ops.rs:103-193 (whole function) -------------------------- */
void vxo_step_deltanet_recurrent(const float* qkv_mixed, size_t conv_ch, const float* z,
                                 const float* alpha_raw, const float* beta_raw,
                                 const float* ssm_conv1d, const float* ssm_a,
                                 const float* ssm_dt_bias, const float* ssm_norm, float* conv_state,
                                 float* ssm_state, size_t n_kh, size_t n_vh, size_t dk, size_t dv,
                                 size_t k_sz, float eps, float* y_concat) {
    size_t hist = k_sz - 1;
    float* conv_silu = (float*)malloc(sizeof(float) * conv_ch);
    for (size_t c = 0; c < conv_ch; ++c) {
        const float* w = ssm_conv1d + c * k_sz;
        float acc = 0.0f;
        for (size_t t = 0; t < hist; ++t) acc = fmaf(conv_state[t * conv_ch + c], w[t], acc);
        acc = fmaf(qkv_mixed[c], w[hist], acc);
        for (size_t t = 0; t + 1 < hist; ++t)
            conv_state[t * conv_ch + c] = conv_state[(t + 1) * conv_ch + c];
        conv_state[(hist - 1) * conv_ch + c] = qkv_mixed[c];
        conv_silu[c] = silu(acc);
    }
    size_t qk_dim = n_kh * dk;
    float* o = (float*)malloc(sizeof(float) * n_vh * dv);
    vxo_deltanet_core(conv_silu, conv_silu + qk_dim, conv_silu + 2 * qk_dim, beta_raw, alpha_raw,
                      ssm_a, ssm_dt_bias, n_kh, n_vh, dk, dv, eps, 1.0f / sqrtf((float)dk),
                      ssm_state, o);
    for (size_t h = 0; h < n_vh; ++h) {
        float* o_h = o + h * dv;
        rms_norm_inplace(o_h, ssm_norm, eps, dv);
        const float* z_h = z + h * dv;
        float* dst_h = y_concat + h * dv;
        for (size_t jv = 0; jv < dv; ++jv) dst_h[jv] = o_h[jv] * silu(z_h[jv]);
    }
    free(o);
    free(conv_silu);
}

/* ======================= batched drivers (CPU baseline / parity harness) ===================== *
 * Device-pool layout shared with the CUDA backend: K pool [n_seq][cap][n_kv][hd/32] blocks, V
 * pool likewise.  Sequences are independent; threads take whole sequences. */

typedef struct {
    size_t n_batch, n_head, n_kv, hd, cap;
    const int32_t* seq_ids;
    const int32_t* pos;
    const float *q, *k_new, *v_new, *gates;
    uint8_t *k_pool, *v_pool;
    float* out;
    float scale;
    int do_append;
    size_t next;
    pthread_mutex_t mu;
} decode_job;

static void* decode_worker(void* arg) {
    decode_job* j = (decode_job*)arg;
    size_t seq_bytes = j->cap * j->n_kv * (j->hd / 32) * VXO_BLK;
    float* scores = (float*)malloc(sizeof(float) * j->cap);
    for (;;) {
        pthread_mutex_lock(&j->mu);
        size_t b = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (b >= j->n_batch) break;
        size_t s = (size_t)j->seq_ids[b];
        size_t p = (size_t)j->pos[b];
        uint8_t* kc = j->k_pool + s * seq_bytes;
        uint8_t* vc = j->v_pool + s * seq_bytes;
        size_t kvd = j->n_kv * j->hd;
        if (j->do_append)
            vxo_q8_append(j->k_new + b * kvd, j->v_new + b * kvd, j->n_kv, j->hd, p, kc, vc);
        size_t qd = j->n_head * j->hd;
        vxo_q8_attend(j->q + b * qd, j->gates ? j->gates + b * qd : NULL, kc, vc, j->n_head,
                      j->n_kv, j->hd, p + 1, j->scale, j->out + b * qd, scores);
    }
    free(scores);
    return NULL;
}

/* One batched decode step: for each b, append (k_new[b], v_new[b]) at pos[b] of sequence
 * seq_ids[b] (if do_append) and attend over tokens [0, pos[b]] -> out[b].  n_threads >= 1. */
void vxo_batch_decode_q8(size_t n_batch, const int32_t* seq_ids, const int32_t* pos,
                         const float* q, const float* k_new, const float* v_new, const float* gates,
                         uint8_t* k_pool, uint8_t* v_pool, size_t cap, size_t n_head, size_t n_kv,
                         size_t hd, float scale, int do_append, float* out, int n_threads) {
    decode_job j;
    memset(&j, 0, sizeof j);
    j.n_batch = n_batch; j.n_head = n_head; j.n_kv = n_kv; j.hd = hd; j.cap = cap;
    j.seq_ids = seq_ids; j.pos = pos; j.q = q; j.k_new = k_new; j.v_new = v_new; j.gates = gates;
    j.k_pool = k_pool; j.v_pool = v_pool; j.out = out; j.scale = scale; j.do_append = do_append;
    pthread_mutex_init(&j.mu, NULL);
    if (n_threads < 1) n_threads = 1;
    pthread_t th[256];
    if (n_threads > 256) n_threads = 256;
    for (int i = 1; i < n_threads; ++i) pthread_create(&th[i], NULL, decode_worker, &j);
    decode_worker(&j);
    for (int i = 1; i < n_threads; ++i) pthread_join(th[i], NULL);
    pthread_mutex_destroy(&j.mu);
}

typedef struct {
    size_t n_batch, n_kh, n_vh, dk, dv;
    const float *q, *k, *v, *beta_raw, *alpha_raw, *ssm_a, *dt_bias;
    float* state;
    float* o;
    float eps, q_scale;
    size_t next;
    pthread_mutex_t mu;
} dnet_job;

static void* dnet_worker(void* arg) {
    dnet_job* j = (dnet_job*)arg;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        size_t b = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (b >= j->n_batch) break;
        vxo_deltanet_core(j->q + b * j->n_kh * j->dk, j->k + b * j->n_kh * j->dk,
                          j->v + b * j->n_vh * j->dv, j->beta_raw + b * j->n_vh,
                          j->alpha_raw + b * j->n_vh, j->ssm_a, j->dt_bias, j->n_kh, j->n_vh,
                          j->dk, j->dv, j->eps, j->q_scale,
                          j->state + b * j->n_vh * j->dv * j->dk, j->o + b * j->n_vh * j->dv);
    }
    return NULL;
}

/* Batched DeltaNet core step over n_batch sequences (state [B][n_vh][dv][dk]). */
void vxo_batch_deltanet(size_t n_batch, const float* q, const float* k, const float* v,
                        const float* beta_raw, const float* alpha_raw, const float* ssm_a,
                        const float* dt_bias, size_t n_kh, size_t n_vh, size_t dk, size_t dv,
                        float eps, float q_scale, float* state, float* o, int n_threads) {
    dnet_job j;
    memset(&j, 0, sizeof j);
    j.n_batch = n_batch; j.n_kh = n_kh; j.n_vh = n_vh; j.dk = dk; j.dv = dv;
    j.q = q; j.k = k; j.v = v; j.beta_raw = beta_raw; j.alpha_raw = alpha_raw;
    j.ssm_a = ssm_a; j.dt_bias = dt_bias; j.state = state; j.o = o; j.eps = eps;
    j.q_scale = q_scale;
    pthread_mutex_init(&j.mu, NULL);
    if (n_threads < 1) n_threads = 1;
    pthread_t th[256];
    if (n_threads > 256) n_threads = 256;
    for (int i = 1; i < n_threads; ++i) pthread_create(&th[i], NULL, dnet_worker, &j);
    dnet_worker(&j);
    for (int i = 1; i < n_threads; ++i) pthread_join(th[i], NULL);
    pthread_mutex_destroy(&j.mu);
}

/* Quantise n_rows rows of 32 floats into n_rows blocks (helper for building caches). */
void vxo_q8_quantize_rows(const float* src, size_t n_rows, uint8_t* dst) {
    for (size_t r = 0; r < n_rows; ++r) vxo_q8_quantize(src + r * 32, dst + r * VXO_BLK);
}
