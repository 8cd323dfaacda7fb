/*
 * concord_oracle.c — CPU restatement of Concord's packed-word hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in concord_b200/; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py load it.  The product path never
 * calls it.
 *
 * It restates, element by element and in the same order, the arithmetic of
 * the reference's Triton kernels (Theophite/Concord concord/packed_b.py):
 *   _hash_uniform                   packed_b.py:109-117
 *   _materialize_packed_bf16_kernel packed_b.py:120-155
 *   _apply_packed_sgd_kernel        packed_b.py:173-312
 *   _apply_packed_adamw_kernel      packed_b.py:422-703
 *   _rebalance_packed_decide_kernel packed_b.py:959-1095 (+ torch medians 1156-1160)
 *   load_weights / _finetune        packed_b.py:1570-1603, 1816-1856
 *   gate_coherence_from_fields      packed_b.py:2081-2106
 *   tl.rand (Triton 3.6 language/random.py: Philox4x32-10 + uint_to_uniform_float)
 * Arithmetic model: every fp32 operation rounds once (compile with
 * -ffp-contract=off, no fast-math); exp2/log2 are correctly rounded
 * (evaluated in x87 extended precision and rounded once to fp32); fp32->bf16
 * is round-to-nearest-even.  The Adafactor v-hat update uses the fixed
 * summation order that the CUDA kernel uses (documented at oracle_vhat).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/concord_b200.h"

/* ---------------- scalar helpers ---------------- */

static inline float f32_of_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_of_f32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* fp32 -> bf16 round-to-nearest-even (NaN kept quiet). */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = bits_of_f32(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}
static inline float bf16_to_f32(uint16_t h) { return f32_of_bits(((uint32_t)h) << 16); }

/* Correctly rounded fp32 log2 / exp2 (x87 extended precision, one rounding). */
float oracle_log2f(float x) { return (float)log2l((long double)x); }
float oracle_exp2f(float y) { return (float)exp2l((long double)y); }

/* numpy-style maximum/minimum: NaN in either operand propagates. */
static inline float np_max(float a, float b) { if (a != a) return a; if (b != b) return b; return a > b ? a : b; }
static inline float np_min(float a, float b) { if (a != a) return a; if (b != b) return b; return a < b ? a : b; }

static inline int32_t shl32(int32_t v, int s) { return (int32_t)((uint32_t)v << s); }

/* fp32 -> int32 truncation as numpy astype does for in-range values. */
static inline int32_t f2i(float f) { return (int32_t)f; }

/* _hash_uniform (packed_b.py:109-117): int32 xorshift, arithmetic >>. */
float oracle_hash_uniform(int32_t x, int32_t pos, int32_t salt) {
    int32_t h = x ^ salt ^ pos;
    h = h ^ shl32(h, 13);
    h = h ^ (h >> 17);
    h = h ^ shl32(h, 5);
    h = h ^ (h >> 7);
    return (float)(h & 0xFFFFFF) * (1.0f / 16777216.0f);
}

/* SR tick: floor(d) + (r < frac(d)), as int32 (packed_b.py:596-598). */
static inline int32_t sr_tick(float d, float r) {
    float fl = floorf(d);
    float fr = d - fl;
    return f2i(fl + (r < fr ? 1.0f : 0.0f));
}

static inline float exp2_int(int32_t e) { return oracle_exp2f((float)e); }

/* Philox4x32-10 keyed (k0, k1) on counter (c0,0,0,0); returns the first output word. */
uint32_t oracle_philox_c0(uint32_t c0, uint32_t k0, uint32_t k1) {
    uint32_t c1 = 0, c2 = 0, c3 = 0;
    for (int r = 0; r < 10; ++r) {
        uint64_t pa = (uint64_t)0xD2511F53u * (uint64_t)c0;
        uint64_t pb = (uint64_t)0xCD9E8D57u * (uint64_t)c2;
        uint32_t n0 = (uint32_t)(pb >> 32) ^ c1 ^ k0;
        uint32_t n2 = (uint32_t)(pa >> 32) ^ c3 ^ k1;
        c1 = (uint32_t)pb;
        c3 = (uint32_t)pa;
        c0 = n0; c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

/* tl.rand(seed:int32, offset:int32) -> fp32 in [0,1). */
float oracle_tl_rand(int32_t seed, int32_t offset) {
    uint64_t s64 = (uint64_t)(int64_t)seed;          /* int32 -> uint64 sign-extends */
    uint32_t x = oracle_philox_c0((uint32_t)offset, (uint32_t)(s64 & 0xffffffffu),
                                  (uint32_t)(s64 >> 32));
    int32_t xi = (int32_t)x;
    if (xi < 0) xi = (int32_t)(~(uint32_t)xi);       /* -x - 1 with int32 wrap */
    return (float)xi * 4.6566127342e-10f;
}

/* ---------------- packed step ---------------- */

static inline int32_t repack(int32_t sf, int32_t ss, int32_t vs) {
    return (int32_t)((((uint32_t)sf & 0xFFFFu) << 16) | (((uint32_t)ss & 0xFFu) << 8) | ((uint32_t)vs & 0xFFu));
}
static inline int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

/*
 * One element of _apply_packed_adamw_kernel (packed_b.py:476-703).
 * Returns the new word; writes the new bf16 weight, the new coh_pre, |m_eff|
 * and the element's coh (NAN if the flags do not compute it).
 */
static int32_t step_adamw_elem(const concord_step_params* P, int32_t packed, float g,
                               int32_t row_e, int32_t col_e, float v_row, float v_col,
                               float sum_v_inv, float* coh_pre_io, float lr, float eps,
                               int32_t salt, int32_t pos, uint16_t* w_out,
                               int32_t* abs_eff_out, float* coh_out) {
    const uint32_t F = P->flags;
    int32_t s_fast = packed >> 16;
    int32_t s_slow = shl32(packed, 16) >> 24;
    int32_t v_slow = shl32(packed, 24) >> 24;
    int32_t s_slow_full = s_slow * 128;
    int32_t v_slow_full = v_slow * 128;

    int32_t te_i = row_e + col_e - P->mantissa_bias;
    float total_exp = (float)te_i;
    float scale_fwd = exp2_int(te_i);
    float scale_inv = oracle_exp2f(-total_exp);

    float d_fs = (float)s_fast;
    float d_sv = (float)(s_slow_full - v_slow_full);
    float noise = d_fs - P->drift_cancel_C * d_sv;
    float noise_in_w = noise * scale_fwd;
    float v_proxy = noise_in_w * noise_in_w * P->v_scale;

    int need_vhat = (F & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) != 0;
    int need_coh = (F & (CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) != 0;
    float v_hat = 0.0f, coh = 0.0f;
    if (need_vhat) v_hat = v_row * v_col * sum_v_inv;
    if (F & CONCORD_F_GF_TRUST) v_proxy = v_proxy + P->gf_trust_delta_sq * v_hat;
    if (need_coh) {
        if (F & CONCORD_F_FIXED_COH) {
            float sig_w = P->drift_cancel_C * d_sv * scale_fwd;
            float sig2 = sig_w * sig_w;
            coh = sig2 / (sig2 + noise_in_w * noise_in_w + 1e-30f);
        } else {
            float mg = P->alpha_v_fast * d_sv * scale_fwd;
            coh = mg * mg / (v_hat + 1e-12f);
        }
        coh = np_min(np_max(coh, 0.0f), 1.0f);
    }
    *coh_out = need_coh ? coh : NAN;

    float denom_p = oracle_exp2f(P->precond_p * oracle_log2f(v_proxy + eps));
    float step_live = g / denom_p;
    step_live = np_min(np_max(step_live, -P->step_cap), P->step_cap);

    float s_fast_in_w = d_fs * scale_fwd;
    float evap = 0.0f;
    int consol = (F & CONCORD_F_GF_CONSOL) != 0;
    if (consol) {
        evap = lr * P->gf_consol * (1.0f - coh) * d_fs;
    } else {
        step_live = step_live + P->weight_decay * s_fast_in_w;
    }
    /* gradient-accumulation gate (prototype_packed_b.py:514-515, 661): the
     * beta1 and evaporation terms only on the consolidate step */
    const int accum = P->consolidate != NULL;
    const float consf = accum ? (float)*P->consolidate : 1.0f;
    float delta_grad = -lr * step_live * scale_inv;
    float delta_t = accum ? delta_grad - consf * (P->beta1 * d_fs) : delta_grad - P->beta1 * d_fs;
    if (consol) delta_t = accum ? delta_t - consf * evap : delta_t - evap;

    float r1 = oracle_hash_uniform(s_fast, pos, salt);
    s_fast = s_fast + sr_tick(delta_t, r1);

    /* ratio floors from device scalars: 1 - floor in fp32 (prototype_packed_b.py:510-511, 691) */
    const float chase_floor = P->ratio_floors ? P->ratio_floors[0] : P->chase_floor;
    const float om_chase_floor = P->ratio_floors ? 1.0f - P->ratio_floors[0] : P->one_minus_chase_floor;
    const float leak_floor = P->ratio_floors ? P->ratio_floors[1] : P->leak_floor;
    const float om_leak_floor = P->ratio_floors ? 1.0f - P->ratio_floors[1] : P->one_minus_leak_floor;
    int32_t new_v = v_slow;
    if (F & CONCORD_F_APPLY_CHASE) {
        float chase_mantissa;
        if (F & CONCORD_F_RATIO_COH) {
            float gate = chase_floor + om_chase_floor * coh;
            chase_mantissa = P->alpha * gate * P->gate_gain * (float)s_fast;
        } else if (F & CONCORD_F_COHPRE) {
            float cp = *coh_pre_io;
            float gate = coh + cp * (1.0f - coh);
            *coh_pre_io = P->one_minus_alpha_v_fast * cp + P->alpha_v_fast * coh;
            chase_mantissa = P->alpha * gate * P->gate_gain * (float)s_fast;
        } else {
            chase_mantissa = P->alpha_gate_gain * (float)s_fast;
        }
        if (accum) chase_mantissa = chase_mantissa * consf;   /* prototype_packed_b.py:695 */
        float chase_i8 = chase_mantissa / 128.0f;
        float r2 = oracle_hash_uniform(s_fast, pos, salt ^ 0x5A5A5A5A);
        int32_t ts = sr_tick(chase_i8, r2);
        s_slow = s_slow + ts;
        s_fast = s_fast - ts * 128;

        float gap = (float)(s_slow * 128 - v_slow_full);
        float delta_v8 = P->alpha_v_fast * gap / 128.0f;
        if (accum) delta_v8 = delta_v8 * consf;                 /* prototype_packed_b.py:709 */
        if (F & CONCORD_F_RATIO_COH)
            delta_v8 = delta_v8 * (leak_floor + om_leak_floor * coh);
        float r3 = oracle_hash_uniform(s_fast, pos, salt ^ 0x33335555);
        int32_t tv = sr_tick(delta_v8, r3);
        new_v = clampi(v_slow + tv, -128, 127);
        if (F & CONCORD_F_MASS_PRESERVE) s_slow = s_slow - (new_v - v_slow);

        int32_t v_full_post = new_v * 128;
        float dsv_post = (float)(s_slow * 128 - v_full_post);
        float wd_sv_d = lr * P->wd_sv * dsv_post / 128.0f;
        if (accum) wd_sv_d = wd_sv_d * consf;                   /* prototype_packed_b.py:726 */
        float r4 = oracle_hash_uniform(s_fast, pos, salt ^ 0x66665555);
        s_slow = s_slow - sr_tick(wd_sv_d, r4);

        int32_t sfl = s_slow * 128 + s_fast;
        float dsf = (float)(sfl - v_full_post);
        float wd_sf_d = lr * P->wd_sf * dsf;
        if (accum) wd_sf_d = wd_sf_d * consf;                   /* prototype_packed_b.py:737 */
        float r5 = oracle_hash_uniform(s_fast, pos, salt ^ 0x77770000);
        s_fast = s_fast - sr_tick(wd_sf_d, r5);
    }

    int32_t sfc = clampi(s_fast, -32768, 32767);
    int32_t ssc = clampi(s_slow, -128, 127);
    int32_t m_new = ssc * 128 + sfc + new_v * 128;
    *w_out = oracle_f32_to_bf16((float)m_new * scale_fwd);
    *abs_eff_out = m_new < 0 ? -m_new : m_new;
    return repack(sfc, ssc, new_v);
}

/* One element of _apply_packed_sgd_kernel (packed_b.py:214-312). */
static int32_t step_sgd_elem(const concord_step_params* P, int32_t packed, float g,
                             int32_t row_e, int32_t col_e, float lr, int32_t salt,
                             int32_t pos, uint16_t* w_out, int32_t* abs_eff_out) {
    int32_t s_fast = packed >> 16;
    int32_t s_slow = shl32(packed, 16) >> 24;
    int32_t v_slow = shl32(packed, 24) >> 24;
    float total_exp = (float)(row_e + col_e - P->mantissa_bias);
    float scale_inv = oracle_exp2f(-total_exp);

    float delta_grad = -lr * g * scale_inv;
    float delta_t = delta_grad - P->beta1 * (float)s_fast;
    float r1 = oracle_hash_uniform(s_fast, pos, salt);
    s_fast = s_fast + sr_tick(delta_t, r1);

    float chase_i8 = P->alpha * (float)s_fast / 128.0f;
    float r2 = oracle_hash_uniform(s_fast, pos, salt ^ 0x5A5A5A5A);
    int32_t ts = sr_tick(chase_i8, r2);
    s_slow = s_slow + ts;
    s_fast = s_fast - ts * 128;

    float gap = (float)(s_slow * 128 - v_slow * 128);
    float delta_v8 = P->alpha_v_fast * gap / 128.0f;
    float r3 = oracle_hash_uniform(s_fast, pos, salt ^ 0x33335555);
    int32_t tv = sr_tick(delta_v8, r3);
    int32_t new_v = clampi(v_slow + tv, -128, 127);
    if (P->flags & CONCORD_F_MASS_PRESERVE) s_slow = s_slow - (new_v - v_slow);

    int32_t sfc = clampi(s_fast, -32768, 32767);
    int32_t ssc = clampi(s_slow, -128, 127);
    int32_t m_new = ssc * 128 + sfc + new_v * 128;
    float scale_fwd = oracle_exp2f(total_exp);
    *w_out = oracle_f32_to_bf16((float)m_new * scale_fwd);
    *abs_eff_out = m_new < 0 ? -m_new : m_new;
    return repack(sfc, ssc, new_v);
}

/*
 * Full packed step over an [N,K] shard starting at global row row0.
 * grad / wbuf are bf16 bit patterns.  row_max/col_max are max-accumulated
 * (caller zeroes them).  coh_stats (nullable) gets += (sum coh, count).
 */
void oracle_step(const concord_step_params* P, int32_t* packed, int64_t ldp,
                 const uint16_t* grad, int64_t ldg, uint16_t* wbuf, int64_t ldw,
                 const int8_t* row_exp, const int8_t* col_exp,
                 int32_t* row_max, int32_t* col_max,
                 const float* v_row, const float* v_col, const float* sum_v_inv,
                 float* coh_pre, int64_t ldc, float lr, float eps, int32_t salt,
                 int64_t N, int64_t K, int64_t row0, double* coh_stats) {
    float svi = sum_v_inv ? *sum_v_inv : 0.0f;
    int track = (P->flags & CONCORD_F_TRACK_REBALANCE) != 0;
    int write_cp = (P->flags & CONCORD_F_COHPRE) && (P->flags & CONCORD_F_APPLY_CHASE)
                   && !(P->flags & CONCORD_F_RATIO_COH) && coh_pre;
    double csum = 0.0, ccnt = 0.0;
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k = 0; k < K; ++k) {
            int32_t gn = (int32_t)(row0 + n);
            int32_t pos = shl32(gn, 16) ^ (int32_t)k;
            int32_t w = packed[n * ldp + k];
            float g = bf16_to_f32(grad[n * ldg + k]);
            uint16_t wb; int32_t ae; float coh = NAN;
            int32_t nw;
            if (P->kind == CONCORD_KIND_SGD) {
                nw = step_sgd_elem(P, w, g, row_exp[n], col_exp[k], lr, salt, pos, &wb, &ae);
            } else {
                float cp = coh_pre ? coh_pre[n * ldc + k] : 1.0f;
                nw = step_adamw_elem(P, w, g, row_exp[n], col_exp[k],
                                     v_row ? v_row[n] : 0.0f, v_col ? v_col[k] : 0.0f, svi,
                                     &cp, lr, eps, salt, pos, &wb, &ae, &coh);
                if (write_cp) coh_pre[n * ldc + k] = cp;
            }
            packed[n * ldp + k] = nw;
            /* weight emit and maxima only on the consolidate step (prototype_packed_b.py:761-782) */
            const int emit = P->kind == CONCORD_KIND_SGD || !P->consolidate || *P->consolidate == 1;
            if (!emit) { if (coh == coh) { csum += coh; ccnt += 1.0; } continue; }
            wbuf[n * ldw + k] = wb;
            if (track) {
                if (ae > row_max[n]) row_max[n] = ae;
                if (ae > col_max[k]) col_max[k] = ae;
            }
            if (coh == coh) { csum += coh; ccnt += 1.0; }
        }
    }
    if (coh_stats && ccnt > 0) { coh_stats[0] += csum; coh_stats[1] += ccnt; }
}

/* ---------------- Adafactor v-hat update ---------------- */

/*
 * Fixed summation order (identical to concord_b200/csrc/vhat.cu):
 *   g2 = g*g in fp32.
 *   row partial (row n, column slab c of 256 columns): lane l (0..31)
 *     sums its 8 columns c*256+8l .. +7 left to right (out-of-range = 0),
 *     then a 32-lane xor butterfly (offsets 16,8,4,2,1: s_l = s_l + s_{l^o}).
 *   col partial (column k, row block b of 128 rows): warp w (0..7) sums
 *     rows b*128 + w + 8i, i = 0..15, in order (out-of-range = 0); then the
 *     8 warp sums are added in order w = 0..7.
 *   row total = partials over slabs added in slab order; col total likewise
 *   over row blocks.  v = b2*v + (1-b2)*total (two roundings, no fma).
 *   sum_v: thread t (0..255) adds v_row[n] for n = t, t+256, ... in order
 *   (starting from 0.0f); then a tree (stride 128,64,..,1: a[t] = a[t] + a[t+s]).
 *   sum_v_inv = 1 / max(sum_v, 1e-30).
 */
#define VH_COLS 256
#define VH_ROWS 128
/* shard mode (concord_vhat_partial): when col_sum_out is non-NULL, the raw
 * column totals go there (v_col untouched) and the v_row sum to *vsum_out
 * (sum_v_inv untouched). */
void oracle_vhat_ex(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K,
                    float* v_row, float* v_col, float* sum_v_inv, float b2, float omb2,
                    float* col_sum_out, float* vsum_out);
void oracle_vhat(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K,
                 float* v_row, float* v_col, float* sum_v_inv, float b2, float omb2) {
    oracle_vhat_ex(grad, ldg, N, K, v_row, v_col, sum_v_inv, b2, omb2, NULL, NULL);
}
void oracle_vhat_ex(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K,
                    float* v_row, float* v_col, float* sum_v_inv, float b2, float omb2,
                    float* col_sum_out, float* vsum_out) {
    int64_t ncs = (K + VH_COLS - 1) / VH_COLS, nrb = (N + VH_ROWS - 1) / VH_ROWS;
    float* rp = (float*)calloc((size_t)(ncs * N + 1), sizeof(float));
    float* cp = (float*)calloc((size_t)(nrb * K + 1), sizeof(float));
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t c = 0; c < ncs; ++c) {
            float s[32];
            for (int l = 0; l < 32; ++l) {
                float acc = 0.0f;
                for (int j = 0; j < 8; ++j) {
                    int64_t k = c * VH_COLS + 8 * l + j;
                    float g = k < K ? bf16_to_f32(grad[n * ldg + k]) : 0.0f;
                    float g2 = g * g;
                    acc = (j == 0) ? g2 : acc + g2;
                }
                s[l] = acc;
            }
            for (int o = 16; o >= 1; o >>= 1) {
                float t[32];
                for (int l = 0; l < 32; ++l) t[l] = s[l] + s[l ^ o];
                memcpy(s, t, sizeof(s));
            }
            rp[c * N + n] = s[0];
        }
    }
    for (int64_t b = 0; b < nrb; ++b) {
        for (int64_t k = 0; k < K; ++k) {
            float tot = 0.0f;
            for (int w = 0; w < 8; ++w) {
                float acc = 0.0f;
                for (int i = 0; i < 16; ++i) {
                    int64_t n = b * VH_ROWS + w + 8 * i;
                    float g = n < N ? bf16_to_f32(grad[n * ldg + k]) : 0.0f;
                    float g2 = g * g;
                    acc = (i == 0) ? g2 : acc + g2;
                }
                tot = (w == 0) ? acc : tot + acc;
            }
            cp[b * K + k] = tot;
        }
    }
    for (int64_t n = 0; n < N; ++n) {
        float t = rp[n];
        for (int64_t c = 1; c < ncs; ++c) t = t + rp[c * N + n];
        v_row[n] = b2 * v_row[n] + omb2 * t;
    }
    for (int64_t k = 0; k < K; ++k) {
        float t = nrb > 0 ? cp[k] : 0.0f;   /* a shard of no rows contributes zero */
        for (int64_t b = 1; b < nrb; ++b) t = t + cp[b * K + k];
        if (col_sum_out) col_sum_out[k] = t;
        else v_col[k] = b2 * v_col[k] + omb2 * t;
    }
    float a[256];
    for (int t = 0; t < 256; ++t) {
        float acc = 0.0f;
        for (int64_t n = t; n < N; n += 256) acc = acc + v_row[n];
        a[t] = acc;
    }
    for (int s = 128; s >= 1; s >>= 1)
        for (int t = 0; t < s; ++t) a[t] = a[t] + a[t + s];
    float sv = a[0];
    if (vsum_out) { *vsum_out = sv; free(rp); free(cp); return; }
    sv = np_max(sv, 1e-30f);
    *sum_v_inv = 1.0f / sv;
    free(rp); free(cp);
}

/* ---------------- rebalance ---------------- */

/* lower median of the 0..128 magnitudes (torch.median semantics). */
static int32_t lower_median_hist(const int64_t* hist, int64_t count) {
    int64_t target = (count - 1) / 2 + 1, run = 0;
    for (int v = 0; v <= 128; ++v) { run += hist[v]; if (run >= target) return v; }
    return 128;
}

/*
 * rebalance_packed + ConcordLinearPackedB.rebalance (packed_b.py:1792-1814,
 * 1129-1190, 959-1095).  Exponent ticks are decided from the pre-call
 * exponents for every element (the reference's kernel can read an exponent
 * another program already incremented).  Philox offsets use global row
 * index row0+n and N_total.
 */
void oracle_rebalance(int32_t* packed, int64_t ldp, int8_t* row_exp, int8_t* col_exp,
                      const int32_t* row_max, const int32_t* col_max,
                      int32_t* row_hwm, int32_t* col_hwm, int32_t* seed,
                      int32_t max_m, int32_t exp_max, int32_t exp_min, int32_t allow_td,
                      int64_t N, int64_t K, int64_t row0, int64_t N_total, int32_t* fired) {
    if (row_hwm) for (int64_t n = 0; n < N; ++n) if (row_max[n] > row_hwm[n]) row_hwm[n] = row_max[n];
    if (col_hwm) for (int64_t k = 0; k < K; ++k) if (col_max[k] > col_hwm[k]) col_hwm[k] = col_max[k];
    *seed = *seed + 1;
    int32_t sd = *seed;
    int32_t* rt = (int32_t*)calloc((size_t)N + 1, sizeof(int32_t));
    int32_t* ct = (int32_t*)calloc((size_t)K + 1, sizeof(int32_t));
    int32_t* rmed = (int32_t*)calloc((size_t)N + 1, sizeof(int32_t));
    int32_t* cmed = (int32_t*)calloc((size_t)K + 1, sizeof(int32_t));
    if (allow_td) {
        int64_t* ch = (int64_t*)calloc((size_t)K * 129, sizeof(int64_t));
        for (int64_t n = 0; n < N; ++n) {
            int64_t rh[129]; memset(rh, 0, sizeof(rh));
            for (int64_t k = 0; k < K; ++k) {
                int32_t w = packed[n * ldp + k];
                int32_t ss = shl32(w, 16) >> 24, vs = shl32(w, 24) >> 24;
                int32_t a = ss < 0 ? -ss : ss, b = vs < 0 ? -vs : vs;
                int32_t m = a > b ? a : b;
                rh[m]++; ch[k * 129 + m]++;
            }
            rmed[n] = lower_median_hist(rh, K);
        }
        for (int64_t k = 0; k < K; ++k) cmed[k] = lower_median_hist(ch + k * 129, N);
        free(ch);
    }
    int any = 0;
    for (int64_t n = 0; n < N; ++n) {
        int up = row_max[n] > max_m && row_exp[n] < exp_max;
        int dn = allow_td && row_max[n] <= max_m && rmed[n] <= 31 && row_exp[n] > exp_min;
        rt[n] = up - dn; any |= (rt[n] != 0);
    }
    for (int64_t k = 0; k < K; ++k) {
        int up = col_max[k] > max_m && col_exp[k] < exp_max;
        int dn = allow_td && col_max[k] <= max_m && cmed[k] <= 31 && col_exp[k] > exp_min;
        ct[k] = up - dn; any |= (ct[k] != 0);
    }
    uint32_t NK = (uint32_t)(N_total * K);
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k = 0; k < K; ++k) {
            int32_t net = rt[n] + ct[k];
            if (net == 0) continue;
            int32_t w = packed[n * ldp + k];
            int32_t sf = w >> 16, ss = shl32(w, 16) >> 24, vs = shl32(w, 24) >> 24;
            int32_t nsf, nss, nvs;
            if (net < 0) {
                int32_t l = -net;
                nsf = shl32(sf, l); nss = shl32(ss, l); nvs = shl32(vs, l);
            } else {
                int32_t rsh = net;
                uint32_t off = (uint32_t)((row0 + n) * K + k);
                float two_pos = exp2_int(rsh);
                int32_t q = sf >> rsh;
                float rem = (float)(sf - shl32(q, rsh));
                int32_t sfs = q + (oracle_tl_rand(sd, (int32_t)off) * two_pos < rem ? 1 : 0);
                int32_t qs = ss >> rsh;
                float rems = (float)(ss - shl32(qs, rsh));
                int32_t ssu = qs + (oracle_tl_rand(sd, (int32_t)(off + NK)) * two_pos < rems ? 1 : 0);
                int32_t sres = shl32(ss, 7 - rsh) - shl32(ssu, 7);
                int32_t qv = vs >> rsh;
                float remv = (float)(vs - shl32(qv, rsh));
                int32_t vu = qv + (oracle_tl_rand(sd, (int32_t)(off + 2u * NK)) * two_pos < remv ? 1 : 0);
                int32_t vres = shl32(vs, 7 - rsh) - shl32(vu, 7);
                nsf = sfs + sres + vres; nss = ssu; nvs = vu;
            }
            packed[n * ldp + k] = repack(clampi(nsf, -32768, 32767), clampi(nss, -128, 127), clampi(nvs, -128, 127));
        }
    }
    for (int64_t n = 0; n < N; ++n) row_exp[n] = (int8_t)(row_exp[n] + rt[n]);
    for (int64_t k = 0; k < K; ++k) col_exp[k] = (int8_t)(col_exp[k] + ct[k]);
    if (fired) *fired = any;
    free(rt); free(ct); free(rmed); free(cmed);
}

/* ---------------- materialize / quantize / coherence ---------------- */

void oracle_materialize(const int32_t* packed, int64_t ldp, const int8_t* row_exp,
                        const int8_t* col_exp, uint16_t* out, int64_t ldo, int64_t N,
                        int64_t K, int32_t mb, int32_t consolidated) {
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {
            int32_t w = packed[n * ldp + k];
            int32_t sf = w >> 16, ss = shl32(w, 16) >> 24, vs = shl32(w, 24) >> 24;
            int32_t m = consolidated ? ss * 128 + vs * 128 : ss * 128 + sf + vs * 128;
            float sc = exp2_int(row_exp[n] + col_exp[k] - mb);
            out[n * ldo + k] = oracle_f32_to_bf16((float)m * sc);
        }
}

void oracle_quantize(const float* W, int64_t ldw, int32_t* packed, int64_t ldp,
                     int8_t* row_exp, int8_t* col_exp, int64_t N, int64_t K, int32_t mb,
                     int32_t exp_min, int32_t exp_max, int32_t finetune) {
    for (int64_t k = 0; k < K; ++k) col_exp[k] = 0;
    for (int64_t n = 0; n < N; ++n) {
        float mx = 0.0f;
        for (int64_t k = 0; k < K; ++k) mx = np_max(mx, fabsf(W[n * ldw + k]));
        mx = np_max(mx, 1e-30f);
        float e = ceilf(oracle_log2f(mx) + 1.0f);
        e = np_min(np_max(e, (float)exp_min), (float)exp_max);
        row_exp[n] = (int8_t)(int32_t)e;
        float scale = exp2_int(row_exp[n] - mb);
        for (int64_t k = 0; k < K; ++k) {
            int32_t m_total = (int32_t)rintf(W[n * ldw + k] / scale);
            int32_t sf, ss = 0, vs = 0;
            if (!finetune) {
                sf = clampi(m_total, -32768, 32767);
            } else {
                int32_t tv = (int32_t)rintf((float)m_total / 2.0f);
                vs = clampi((int32_t)rintf((float)tv / 128.0f), -128, 127);
                int32_t remaining = m_total - vs * 128;
                ss = clampi((int32_t)rintf((float)remaining / 128.0f), -128, 127);
                sf = clampi(remaining - ss * 128, -32768, 32767);
            }
            packed[n * ldp + k] = repack(sf, ss, vs);
        }
    }
}

/* gate_coherence_from_fields summed over the packed state (fp32 per element, double sum). */
void oracle_coherence(const int32_t* packed, int64_t ldp, int64_t N, int64_t K, float C,
                      double* out) {
    double s = 0.0;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {
            int32_t w = packed[n * ldp + k];
            float sf = (float)(w >> 16), ss = (float)(shl32(w, 16) >> 24), vs = (float)(shl32(w, 24) >> 24);
            float d_sv = (ss - vs) * 128.0f;
            float sig = C * d_sv;
            float noise = sf - sig;
            float sig2 = sig * sig;
            s += (double)(sig2 / (sig2 + noise * noise + 1e-30f));
        }
    out[0] = s;
    out[1] = (double)(N * K);
}
