// step.cu — the fused packed-word optimizer step (K1).
//
// Restates _apply_packed_adamw_kernel (concord/packed_b.py:422-703) and
// _apply_packed_sgd_kernel (packed_b.py:173-312) element by element, in the
// same operation order and fp32 rounding, so the words are bit-identical to
// the reference given the same inputs.  The B200 layout is different from
// the reference's 32x64 Triton tile: each thread owns 8 consecutive columns
// of one row at a time (two 16-byte loads of words, one 16-byte load of the
// bf16 gradient, 16-byte stores), walks several rows so its column data
// (col_exp, v_col) stays in registers, reduces |m_eff| per row with warp
// shuffles and per column through shared memory, and issues one atomicMax
// per (row, warp) and per (column, block).
#include <stdlib.h>

#include <cuda_bf16.h>

#include "common.cuh"

namespace concord {

struct StepScalars {
    float lr, eps, svi;
    int32_t salt;
    // gradient accumulation (P.consolidate): consf multiplies the gated terms;
    // emit == false freezes the weight and the row/col maxima
    bool accum, emit;
    float consf;
    // ratio-coherence floors (P.ratio_floors overrides the launch values)
    float chase_floor, om_chase_floor, leak_floor, om_leak_floor;
};

struct ElemOut {
    int32_t word;
    float wval;     // new live weight (fp32; stored as bf16)
    int32_t abs_eff;
    float coh;      // valid when the flags compute coh
    float coh_pre;  // updated coh_pre (when written)
};

// Flag sets with their own kernel instantiation; anything else runs the
// instantiation that reads the flags at run time (FL_DYNAMIC).
constexpr uint32_t FL_DYNAMIC = 0x80000000u;
// set in an instantiation's flag word: wd_sv == wd_sf == 0 (checked at launch)
constexpr uint32_t FL_ZERO_WD = 0x40000000u;
// set in an instantiation's flag word: weight_decay == beta1 == v_scale == 0 and
// gf_trust_delta_sq == gate_gain == 1 (the bare defaults; checked at launch).
// With the exponent range of a SAFE row (|te| <= 46, so every product below is
// finite) the terms they scale are exact no-ops for the ticks.
constexpr uint32_t FL_PLAIN = 0x20000000u;
// set in an instantiation's flag word: the reference-GPU arithmetic
// (CONCORD_ARITH_GPU); FL_DYNAMIC instantiations read P.arith instead
constexpr uint32_t FL_GPU = 0x10000000u;
constexpr uint32_t FL_BARE = CONCORD_F_MASS_PRESERVE | CONCORD_F_APPLY_CHASE | CONCORD_F_TRACK_REBALANCE |
                             CONCORD_F_GF_TRUST | CONCORD_F_COHPRE | CONCORD_F_FIXED_COH | FL_ZERO_WD | FL_PLAIN;
constexpr uint32_t FL_NOCOHPRE = FL_BARE & ~CONCORD_F_COHPRE;

template <uint32_t FL>
__device__ __forceinline__ uint32_t flags_of(const concord_step_params& P) {
    return (FL & FL_DYNAMIC) ? P.flags : (FL & 0xffffu);
}

template <uint32_t FL>
__device__ __forceinline__ bool gpu_of(const concord_step_params& P) {
    return (FL & FL_DYNAMIC) ? P.arith == CONCORD_ARITH_GPU : (FL & FL_GPU) != 0;
}

// a * b + c rounded as the chosen arithmetic does: one fma (GPU) or two roundings (CR)
__device__ __forceinline__ float mad_as(bool gpu, float a, float b, float c) {
    return gpu ? __fmaf_rn(a, b, c) : __fadd_rn(__fmul_rn(a, b), c);
}

// denominator exp2(p * log2(x)) of the chosen arithmetic (one element)
__device__ __forceinline__ float pow2log2_as(bool gpu, float p, float x) {
    return gpu ? ex2_approx(__fmul_rn(p, log2f(x))) : crmath::cr_exp2f(p * crmath::cr_log2f(x));
}

// First half of one AdamW-path element (packed_b.py:476-557): everything up
// to the argument x = v_proxy + eps of the denominator exp2(p*log2(x)).
struct AdamwPre {
    int32_t s_fast, s_slow, v_slow, te;
    float g, d_fs, coh, cp, x;
    float coh_num, coh_den;  // fixed gate: coh = coh_num / coh_den (divided later)
};

// 2^te and 2^-te.  On SAFE elements (|te| <= 46) `te` holds the fp32 bits of
// 2^te itself ((te + 127) << 23, the caller adds a per-row and a per-column
// part), so both are one integer operation at most.
template <bool SAFE>
__device__ __forceinline__ float pow2_exp(int32_t te) {
    return SAFE ? __uint_as_float((uint32_t)te) : exp2i(te);
}
template <bool SAFE>
__device__ __forceinline__ float pow2_inv(int32_t te) {
    return SAFE ? __uint_as_float(0x7F000000u - (uint32_t)te) : exp2i(-te);
}
// the SAFE encoding's per-row and per-column parts of te
__device__ __forceinline__ int32_t safe_row_bits(int32_t row_e, int32_t mantissa_bias) {
    return (int32_t)((uint32_t)(row_e - mantissa_bias + 127) << 23);
}
__device__ __forceinline__ int32_t safe_col_bits(int32_t col_e) { return (int32_t)((uint32_t)col_e << 23); }

template <uint32_t FL, bool SAFE = false>
__device__ __forceinline__ AdamwPre adamw_pre(const concord_step_params& P, int32_t packed, float g,
                                              int32_t row_e, int32_t col_e, float v_row, float v_col,
                                              float cp, const StepScalars& S) {
    const uint32_t F = flags_of<FL>(P);
    const bool gpu = gpu_of<FL>(P);
    AdamwPre e;
    e.s_fast = packed >> 16;
    e.s_slow = shl32(packed, 16) >> 24;
    e.v_slow = shl32(packed, 24) >> 24;
    // SAFE: row_e / col_e arrive as safe_row_bits / safe_col_bits
    e.te = SAFE ? row_e + col_e : row_e + col_e - P.mantissa_bias;
    e.g = g;
    e.cp = cp;
    const float scale_fwd = pow2_exp<SAFE>(e.te);
    e.d_fs = (float)e.s_fast;
    const float d_sv = (float)(e.s_slow * 128 - e.v_slow * 128);
    const float noise = gpu ? __fmaf_rn(-P.drift_cancel_C, d_sv, e.d_fs) : e.d_fs - P.drift_cancel_C * d_sv;
    const float noise_in_w = noise * scale_fwd;
    const bool plain = SAFE && (FL & FL_PLAIN);
    // v_scale == 0: noise_in_w^2 * 0 == +0 (finite for SAFE rows)
    float v_proxy = plain ? 0.0f : noise_in_w * noise_in_w * P.v_scale;
    const bool need_vhat = (F & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) != 0;
    const bool need_coh = (F & (CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) != 0;
    float v_hat = 0.0f, coh = 0.0f;
    if (need_vhat) v_hat = v_row * v_col * S.svi;
    // delta_sq == 1 and v_hat >= +0: 0 + 1 * v_hat == v_hat
    if (plain) v_proxy = v_hat;
    else if (F & CONCORD_F_GF_TRUST) v_proxy = gpu ? __fmaf_rn(P.gf_trust_delta_sq, v_hat, v_proxy)
                                                   : v_proxy + P.gf_trust_delta_sq * v_hat;
    if (need_coh) {
        if (F & CONCORD_F_FIXED_COH) {
            const float sig_w = P.drift_cancel_C * d_sv * scale_fwd;
            const float sig2 = sig_w * sig_w;
            // 0 <= sig2 <= den: the reference's clamp is the identity (NaN propagates)
            e.coh_num = sig2;
            e.coh_den = gpu ? __fmaf_rn(sig_w, sig_w, noise_in_w * noise_in_w) + 1e-30f
                            : sig2 + noise_in_w * noise_in_w + 1e-30f;
            coh = 0.0f;  // = coh_num / coh_den, see fixed_coh_divide
        } else {
            const float mg = P.alpha_v_fast * d_sv * scale_fwd;
            coh = gpu ? clamp_gpu(div_full(mg * mg, v_hat + 1e-12f), 0.0f, 1.0f)
                      : np_min(np_max(mg * mg / (v_hat + 1e-12f), 0.0f), 1.0f);
        }
    }
    e.coh = coh;
    e.x = v_proxy + S.eps;
    return e;
}

// the fixed-gate division of adamw_pre, done separately so that the four
// divisions of a thread sit next to each other
template <uint32_t FL>
__device__ __forceinline__ void fixed_coh_divide(const concord_step_params& P, AdamwPre& e) {
    const uint32_t F = flags_of<FL>(P);
    if ((F & (CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) && (F & CONCORD_F_FIXED_COH))
        e.coh = gpu_of<FL>(P) ? clamp_gpu(div_full(e.coh_num, e.coh_den), 0.0f, 1.0f) : e.coh_num / e.coh_den;
}

// Second half (packed_b.py:558-703), given denom_p = exp2(p*log2(x)).
template <uint32_t FL, bool SAFE = false>
__device__ __forceinline__ ElemOut adamw_post(const concord_step_params& P, const AdamwPre& e,
                                              float step_div, const StepScalars& S, int32_t pos) {
    const uint32_t F = flags_of<FL>(P);
    const bool gpu = gpu_of<FL>(P);
    const float scale_fwd = pow2_exp<SAFE>(e.te);
    const float scale_inv = pow2_inv<SAFE>(e.te);
    const float coh = e.coh, d_fs = e.d_fs;
    int32_t s_fast = e.s_fast, s_slow = e.s_slow;
    const int32_t v_slow = e.v_slow;
    // step_div = g / denom_p
    float step_live = gpu ? clamp_gpu(step_div, -P.step_cap, P.step_cap) : clamp_np(step_div, P.step_cap);
    const bool consol = (F & CONCORD_F_GF_CONSOL) != 0;
    float evap_rate = 0.0f;   // evaporation = evap_rate * d_fs
    if (consol) {
        evap_rate = S.lr * P.gf_consol * (1.0f - coh);
    } else {
        step_live = mad_as(gpu, P.weight_decay, d_fs * scale_fwd, step_live);
    }
    // accumulation (dynamic flags only): the beta1 and evaporation terms are
    // scaled by consf (prototype_packed_b.py:661); consf == 1 changes nothing
    const bool accum = (FL & FL_DYNAMIC) && S.accum;
    const float delta_grad = -S.lr * step_live * scale_inv;
    float delta_t = accum ? delta_grad - S.consf * (P.beta1 * d_fs) : delta_grad - P.beta1 * d_fs;
    if (consol) {
        if (accum) delta_t = delta_t - S.consf * (evap_rate * d_fs);
        else delta_t = gpu ? __fmaf_rn(-evap_rate, d_fs, delta_t) : delta_t - evap_rate * d_fs;
    }

    s_fast = s_fast + sr_tick(delta_t, hash_uniform(s_fast, pos, S.salt));

    int32_t new_v = v_slow;
    float cp_new = e.cp;
    if (F & CONCORD_F_APPLY_CHASE) {
        float chase_mantissa;
        if (F & CONCORD_F_RATIO_COH) {
            const float gate = gpu ? __fmaf_rn(1.0f - S.chase_floor, coh, S.chase_floor)
                                   : S.chase_floor + S.om_chase_floor * coh;
            chase_mantissa = P.alpha * gate * P.gate_gain * (float)s_fast;
        } else if (F & CONCORD_F_COHPRE) {
            const float gate = mad_as(gpu, e.cp, 1.0f - coh, coh);
            cp_new = gpu ? __fmaf_rn(P.alpha_v_fast, coh, (1.0f - P.alpha_v_fast) * e.cp)
                         : P.one_minus_alpha_v_fast * e.cp + P.alpha_v_fast * coh;
            chase_mantissa = (SAFE && (FL & FL_PLAIN)) ? P.alpha * gate * (float)s_fast   // gate_gain == 1
                                                       : P.alpha * gate * P.gate_gain * (float)s_fast;
        } else {
            chase_mantissa = (gpu ? P.alpha * P.gate_gain : P.alpha_gate_gain) * (float)s_fast;
        }
        if (accum) chase_mantissa = chase_mantissa * S.consf;   // prototype_packed_b.py:695
        const int32_t ts = sr_tick(chase_mantissa / 128.0f, hash_uniform(s_fast, pos, S.salt ^ 0x5A5A5A5A));
        s_slow = s_slow + ts;
        s_fast = s_fast - ts * 128;

        float delta_v8 = P.alpha_v_fast * (float)(s_slow * 128 - v_slow * 128) / 128.0f;
        if (accum) delta_v8 = delta_v8 * S.consf;                // prototype_packed_b.py:709
        if (F & CONCORD_F_RATIO_COH)
            delta_v8 = delta_v8 * (gpu ? __fmaf_rn(1.0f - S.leak_floor, coh, S.leak_floor)
                                       : S.leak_floor + S.om_leak_floor * coh);
        const int32_t tv = sr_tick(delta_v8, hash_uniform(s_fast, pos, S.salt ^ 0x33335555));
        new_v = clampi(v_slow + tv, -128, 127);
        if (F & CONCORD_F_MASS_PRESERVE) s_slow = s_slow - (new_v - v_slow);

        const int32_t v_full_post = new_v * 128;
        const bool zero_wd = (FL & FL_ZERO_WD) != 0;
        if (!zero_wd && P.wd_sv != 0.0f) {  // a zero rate gives tick 0 for every finite state
            float d = S.lr * P.wd_sv * (float)(s_slow * 128 - v_full_post) / 128.0f;
            if (accum) d = d * S.consf;                          // prototype_packed_b.py:726
            s_slow = s_slow - sr_tick(d, hash_uniform(s_fast, pos, S.salt ^ 0x66665555));
        }
        if (!zero_wd && P.wd_sf != 0.0f) {
            float d = S.lr * P.wd_sf * (float)(s_slow * 128 + s_fast - v_full_post);
            if (accum) d = d * S.consf;                          // prototype_packed_b.py:737
            s_fast = s_fast - sr_tick(d, hash_uniform(s_fast, pos, S.salt ^ 0x77770000));
        }
    }

    const int32_t sfc = clampi(s_fast, -32768, 32767);
    const int32_t ssc = clampi(s_slow, -128, 127);
    const int32_t m_new = ssc * 128 + sfc + new_v * 128;
    ElemOut o;
    o.word = repack(sfc, ssc, new_v);
    o.wval = (float)m_new * scale_fwd;
    o.abs_eff = abs(m_new);
    o.coh = coh;
    o.coh_pre = cp_new;
    return o;
}

// adamw_post for W elements in lockstep: every stage runs for all W elements
// before the next one, so the W dependent chains (three SR ticks each) sit
// side by side for the scheduler.  Same arithmetic as adamw_post.
template <uint32_t FL, int W>
__device__ __forceinline__ void adamw_post_lockstep(const concord_step_params& P, const AdamwPre (&e)[W],
                                                    const float (&step_div)[W], const StepScalars& S,
                                                    const int32_t (&pos)[W], ElemOut (&o)[W]) {
    const uint32_t F = flags_of<FL>(P);
    const bool gpu = gpu_of<FL>(P);
    const bool plain = (FL & FL_PLAIN) != 0;
    const bool consol = (F & CONCORD_F_GF_CONSOL) != 0;
    const bool accum = (FL & FL_DYNAMIC) && S.accum;   // same gating as adamw_post
    int32_t sf[W], ss[W], nv[W];
    float cpn[W];
#pragma unroll
    for (int j = 0; j < W; ++j) {
        const float scale_fwd = pow2_exp<true>(e[j].te), scale_inv = pow2_inv<true>(e[j].te);
        float step_live = gpu ? clamp_gpu(step_div[j], -P.step_cap, P.step_cap) : clamp_np(step_div[j], P.step_cap);
        float evap_rate = 0.0f;   // evaporation = evap_rate * d_fs
        if (consol) evap_rate = S.lr * P.gf_consol * (1.0f - e[j].coh);
        else if (!plain) step_live = mad_as(gpu, P.weight_decay, e[j].d_fs * scale_fwd, step_live);
        float delta_t = -S.lr * step_live * scale_inv;
        if (!plain) delta_t = accum ? delta_t - S.consf * (P.beta1 * e[j].d_fs) : delta_t - P.beta1 * e[j].d_fs;
        if (consol) {
            if (accum) delta_t = delta_t - S.consf * (evap_rate * e[j].d_fs);
            else delta_t = gpu ? __fmaf_rn(-evap_rate, e[j].d_fs, delta_t) : delta_t - evap_rate * e[j].d_fs;
        }
        sf[j] = e[j].s_fast + sr_tick(delta_t, hash_uniform(e[j].s_fast, pos[j], S.salt));
        ss[j] = e[j].s_slow;
        nv[j] = e[j].v_slow;
        cpn[j] = e[j].cp;
    }
    if (F & CONCORD_F_APPLY_CHASE) {
#pragma unroll
        for (int j = 0; j < W; ++j) {
            const float coh = e[j].coh;
            float chase_mantissa;
            if (F & CONCORD_F_RATIO_COH) {
                const float gate = gpu ? __fmaf_rn(1.0f - S.chase_floor, coh, S.chase_floor)
                                       : S.chase_floor + S.om_chase_floor * coh;
                chase_mantissa = P.alpha * gate * P.gate_gain * (float)sf[j];
            } else if (F & CONCORD_F_COHPRE) {
                const float gate = mad_as(gpu, e[j].cp, 1.0f - coh, coh);
                cpn[j] = gpu ? __fmaf_rn(P.alpha_v_fast, coh, (1.0f - P.alpha_v_fast) * e[j].cp)
                             : P.one_minus_alpha_v_fast * e[j].cp + P.alpha_v_fast * coh;
                chase_mantissa = plain ? P.alpha * gate * (float)sf[j] : P.alpha * gate * P.gate_gain * (float)sf[j];
            } else {
                chase_mantissa = (gpu ? P.alpha * P.gate_gain : P.alpha_gate_gain) * (float)sf[j];
            }
            if (accum) chase_mantissa = chase_mantissa * S.consf;
            const int32_t ts = sr_tick(chase_mantissa / 128.0f, hash_uniform(sf[j], pos[j], S.salt ^ 0x5A5A5A5A));
            ss[j] = ss[j] + ts;
            sf[j] = sf[j] - ts * 128;
        }
#pragma unroll
        for (int j = 0; j < W; ++j) {
            const int32_t v_slow = e[j].v_slow;
            float delta_v8 = P.alpha_v_fast * (float)(ss[j] * 128 - v_slow * 128) / 128.0f;
            if (accum) delta_v8 = delta_v8 * S.consf;
            if (F & CONCORD_F_RATIO_COH)
                delta_v8 = delta_v8 * (gpu ? __fmaf_rn(1.0f - S.leak_floor, e[j].coh, S.leak_floor)
                                           : S.leak_floor + S.om_leak_floor * e[j].coh);
            const int32_t tv = sr_tick(delta_v8, hash_uniform(sf[j], pos[j], S.salt ^ 0x33335555));
            nv[j] = clampi(v_slow + tv, -128, 127);
            if (F & CONCORD_F_MASS_PRESERVE) ss[j] = ss[j] - (nv[j] - v_slow);
        }
        if (!(FL & FL_ZERO_WD)) {
#pragma unroll
            for (int j = 0; j < W; ++j) {
                const int32_t v_full_post = nv[j] * 128;
                if (P.wd_sv != 0.0f) {
                    float d = S.lr * P.wd_sv * (float)(ss[j] * 128 - v_full_post) / 128.0f;
                    if (accum) d = d * S.consf;
                    ss[j] = ss[j] - sr_tick(d, hash_uniform(sf[j], pos[j], S.salt ^ 0x66665555));
                }
                if (P.wd_sf != 0.0f) {
                    float d = S.lr * P.wd_sf * (float)(ss[j] * 128 + sf[j] - v_full_post);
                    if (accum) d = d * S.consf;
                    sf[j] = sf[j] - sr_tick(d, hash_uniform(sf[j], pos[j], S.salt ^ 0x77770000));
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < W; ++j) {
        const int32_t sfc = clampi(sf[j], -32768, 32767);
        const int32_t ssc = clampi(ss[j], -128, 127);
        const int32_t m_new = ssc * 128 + sfc + nv[j] * 128;
        o[j].word = repack(sfc, ssc, nv[j]);
        o[j].wval = (float)m_new * pow2_exp<true>(e[j].te);
        o[j].abs_eff = abs(m_new);
        o[j].coh = e[j].coh;
        o[j].coh_pre = cpn[j];
    }
}

// One element of the AdamW-path step (packed_b.py:476-703).
template <uint32_t FL>
__device__ __forceinline__ ElemOut step_adamw(const concord_step_params& P, int32_t packed, float g,
                                              int32_t row_e, int32_t col_e, float v_row, float v_col,
                                              float cp, const StepScalars& S, int32_t pos) {
    AdamwPre e = adamw_pre<FL>(P, packed, g, row_e, col_e, v_row, v_col, cp, S);
    fixed_coh_divide<FL>(P, e);
    const bool gpu = gpu_of<FL>(P);
    const float denom_p = pow2log2_as(gpu, P.precond_p, e.x);
    return adamw_post<FL>(P, e, gpu ? div_full(e.g, denom_p) : e.g / denom_p, S, pos);
}

// Out-of-line element for rows/columns whose exponents could leave the
// normal fp32 range (never the case for exponents in [EXP_MIN, EXP_MAX]).
template <uint32_t FL>
__device__ __noinline__ ElemOut step_adamw_outlined(const concord_step_params& P, int32_t packed, float g,
                                                   int32_t row_e, int32_t col_e, float v_row, float v_col,
                                                   float cp, const StepScalars& S, int32_t pos) {
    return step_adamw<FL>(P, packed, g, row_e, col_e, v_row, v_col, cp, S, pos);
}

// One element of the SGD-path step (packed_b.py:214-312).
template <uint32_t FL>
__device__ __forceinline__ ElemOut step_sgd(const concord_step_params& P, int32_t packed, float g,
                                            int32_t row_e, int32_t col_e, const StepScalars& S,
                                            int32_t pos) {
    int32_t s_fast = packed >> 16;
    int32_t s_slow = shl32(packed, 16) >> 24;
    int32_t v_slow = shl32(packed, 24) >> 24;
    int32_t te = row_e + col_e - P.mantissa_bias;
    float scale_inv = exp2i(-te);

    float delta_t = -S.lr * g * scale_inv - P.beta1 * (float)s_fast;
    s_fast = s_fast + sr_tick(delta_t, hash_uniform(s_fast, pos, S.salt));

    int32_t ts = sr_tick(P.alpha * (float)s_fast / 128.0f, hash_uniform(s_fast, pos, S.salt ^ 0x5A5A5A5A));
    s_slow = s_slow + ts;
    s_fast = s_fast - ts * 128;

    float delta_v8 = P.alpha_v_fast * (float)(s_slow * 128 - v_slow * 128) / 128.0f;
    int32_t tv = sr_tick(delta_v8, hash_uniform(s_fast, pos, S.salt ^ 0x33335555));
    int32_t new_v = clampi(v_slow + tv, -128, 127);
    if (flags_of<FL>(P) & CONCORD_F_MASS_PRESERVE) s_slow = s_slow - (new_v - v_slow);

    int32_t sfc = clampi(s_fast, -32768, 32767);
    int32_t ssc = clampi(s_slow, -128, 127);
    int32_t m_new = ssc * 128 + sfc + new_v * 128;
    ElemOut o;
    o.word = repack(sfc, ssc, new_v);
    o.wval = (float)m_new * exp2i(te);
    o.abs_eff = abs(m_new);
    o.coh = 0.0f;
    o.coh_pre = 1.0f;
    return o;
}

struct StepArgs {
    concord_step_params P;
    int32_t* packed; int64_t ldp;
    const uint16_t* grad; int64_t ldg;
    uint16_t* wbuf; int64_t ldw;
    const int8_t* row_exp; const int8_t* col_exp;
    int32_t* row_max; int32_t* col_max;
    const float* v_row; const float* v_col; const float* sum_v_inv;
    float* coh_pre; int64_t ldc;
    const float* lr; const float* eps; const int32_t* salt;
    int64_t N, K, row0;
    double* coh_stats;
    const uint64_t* wpeers;  // other ranks' full forward-weight buffers (row stride ldw), or null
    int32_t npeers;
    int32_t rows_per_block;  // vector kernel: rows of one block (a multiple of 8)
};

__device__ __forceinline__ StepScalars load_scalars(const StepArgs& A) {
    StepScalars S;
    S.lr = *A.lr;
    S.eps = A.eps ? *A.eps : 1.0f;
    S.salt = *A.salt;
    const bool need_vhat = (A.P.flags & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) != 0;
    S.svi = (need_vhat && A.P.kind == CONCORD_KIND_ADAMW) ? *A.sum_v_inv : 0.0f;
    S.accum = A.P.consolidate != nullptr && A.P.kind == CONCORD_KIND_ADAMW;
    const int32_t cons = S.accum ? *A.P.consolidate : 1;
    S.consf = (float)cons;
    S.emit = cons == 1;
    if (A.P.ratio_floors) {
        S.chase_floor = A.P.ratio_floors[0];
        S.om_chase_floor = 1.0f - S.chase_floor;
        S.leak_floor = A.P.ratio_floors[1];
        S.om_leak_floor = 1.0f - S.leak_floor;
    } else {
        S.chase_floor = A.P.chase_floor;
        S.om_chase_floor = A.P.one_minus_chase_floor;
        S.leak_floor = A.P.leak_floor;
        S.om_leak_floor = A.P.one_minus_leak_floor;
    }
    return S;
}

}  // namespace concord

namespace concord {


// 4 warps per block, 4 blocks per SM at 128 registers: smaller blocks than
// 8 warps x 64 rows finish more evenly (measured 0.229 against 0.241 ms at
// 10240 x 2048)
constexpr int STEP_THREADS = 128;
constexpr int VEC = 4;                 // consecutive columns per thread
constexpr int STEP_COLS = 32 * VEC;    // columns per block (one warp-width)
// elements computed in lockstep (divides VEC): two pairs keep the kernel at
// 128 registers without spills; one quad spilled
#ifndef CONCORD_STEP_LOCK
#define CONCORD_STEP_LOCK 2
#endif
constexpr int STEP_LOCK = CONCORD_STEP_LOCK;
#ifndef CONCORD_STEP_ROWS
#define CONCORD_STEP_ROWS 32
#endif
constexpr int STEP_ROWS = CONCORD_STEP_ROWS;          // rows per block (8 per warp); fewer on small layers

__device__ __forceinline__ void block_add_coh(double csum, double ccnt, double* coh_stats) {
    __shared__ double red[2][STEP_THREADS / 32];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        csum += __shfl_xor_sync(0xffffffffu, csum, o);
        ccnt += __shfl_xor_sync(0xffffffffu, ccnt, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { red[0][warp] = csum; red[1][warp] = ccnt; }
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0, c = 0.0;
        for (int w = 0; w < STEP_THREADS / 32; ++w) { s += red[0][w]; c += red[1][w]; }
        if (c > 0.0) { atomicAdd(coh_stats, s); atomicAdd(coh_stats + 1, c); }
    }
}

template <int KIND, uint32_t FL>
__device__ __forceinline__ ElemOut step_elem(const concord_step_params& P, int32_t w, float g, int32_t re,
                                             int32_t ce, float vr, float vc, float cp,
                                             const StepScalars& S, int32_t pos) {
    if (KIND == CONCORD_KIND_ADAMW) return step_adamw<FL>(P, w, g, re, ce, vr, vc, cp, S, pos);
    return step_sgd<FL>(P, w, g, re, ce, S, pos);
}

// Vector path: K % 4 == 0, row strides % 4 == 0, 16-byte aligned bases.
// Block = 4 warps; each warp covers 128 columns (4 per lane) of 8 rows.
// The arguments are __grid_constant__: the out-of-line element takes the
// parameters by reference, which for a plain by-value kernel argument made
// every thread copy the 344-byte struct to its stack first (86 local stores
// per thread; measured 0.1509 -> 0.1435 ms at 10240 x 2048).  Smaller edits
// measured on top of this (inputs staged through cp.async 3-8 rows deep,
// integer-to-float and floor through magic-number adds, a per-row hash key,
// pointer increments instead of row products, a persistent grid of one to
// four waves) were all equal or slower.
template <int KIND, uint32_t FL, int MINB>
__global__ void __launch_bounds__(STEP_THREADS, MINB) step_vec_kernel(const __grid_constant__ StepArgs A) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t k0 = (int64_t)blockIdx.x * STEP_COLS + lane * VEC;
    const bool active = k0 < A.K;
    const int rows_pb = A.rows_per_block;
    const int64_t rbase = (int64_t)blockIdx.y * rows_pb;
    const uint32_t F = flags_of<FL>(A.P);
    const bool adamw = KIND == CONCORD_KIND_ADAMW;
    const bool need_vhat = adamw && (F & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH));
    const bool need_coh = adamw && (F & (CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH));
    const bool use_cp = adamw && (F & CONCORD_F_COHPRE) && !(F & CONCORD_F_RATIO_COH) && A.coh_pre;
    const bool write_cp = use_cp && (F & CONCORD_F_APPLY_CHASE);
    const bool track = (F & CONCORD_F_TRACK_REBALANCE) != 0;
    const StepScalars S = load_scalars(A);
    // peer rows start on 16 bytes when the row stride is a multiple of 8 elements
    // (peer buffers are whole allocations, so their bases are aligned)
    const bool peer16 = (A.ldw % 8) == 0;
    // accumulation micro-step (P.consolidate != 1): the weight and the maxima stay frozen
    const bool emit = !(FL & FL_DYNAMIC) || S.emit;

    int32_t ce[VEC];
    float vc[VEC];
    int cmx[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) { ce[j] = 0; vc[j] = 0.0f; cmx[j] = 0; }
    if (active) {
        const uint32_t c4 = *reinterpret_cast<const uint32_t*>(A.col_exp + k0);
#pragma unroll
        for (int j = 0; j < VEC; ++j) ce[j] = (int32_t)(int8_t)(c4 >> (8 * j));
        if (need_vhat) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(A.v_col + k0));
            vc[0] = a.x; vc[1] = a.y; vc[2] = a.z; vc[3] = a.w;
        }
    }
    bool cols_safe = true;
#pragma unroll
    for (int j = 0; j < VEC; ++j) cols_safe &= (uint32_t)(ce[j] + 23) <= 46u;
    int32_t cbits[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) cbits[j] = safe_col_bits(ce[j]);
    float csum = 0.0f;
    int ccnt = 0;
    // rows of this warp: rbase + warp + 8 i; the next row's inputs are loaded
    // before the current row is computed (registers as a 2-stage pipeline)
    int4 nw4 = make_int4(0, 0, 0, 0);
    uint2 ng4 = make_uint2(0, 0);
    float4 ncp = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
    int32_t nre = 0;
    float nvr = 0.0f;
    auto prefetch = [&](int64_t n) {
        if (n < A.N && active) {
            nre = A.row_exp[n];
            nvr = need_vhat ? __ldg(A.v_row + n) : 0.0f;
            nw4 = __ldcs(reinterpret_cast<const int4*>(A.packed + n * A.ldp + k0));
            ng4 = __ldcs(reinterpret_cast<const uint2*>(A.grad + n * A.ldg + k0));
            if (use_cp) ncp = __ldcs(reinterpret_cast<const float4*>(A.coh_pre + n * A.ldc + k0));
        }
    };
    prefetch(rbase + warp);
    for (int r = warp; r < rows_pb; r += STEP_THREADS / 32) {
        const int64_t n = rbase + r;
        if (n >= A.N) break;
        int rml = 0;
        uint2 wb = make_uint2(0u, 0u);
        const int4 w4 = nw4;
        const uint2 g4 = ng4;
        const float4 cpv = ncp;
        const int32_t re = nre;
        const float vr = nvr;
        if (r + STEP_THREADS / 32 < rows_pb) prefetch(n + STEP_THREADS / 32);
        if (active) {
            int32_t* pw = A.packed + n * A.ldp + k0;
            float cp[VEC] = {cpv.x, cpv.y, cpv.z, cpv.w};
            float* pc = use_cp ? A.coh_pre + n * A.ldc + k0 : nullptr;
            int32_t wv[VEC] = {w4.x, w4.y, w4.z, w4.w};
            const uint32_t gw[2] = {g4.x, g4.y};
            float wf[VEC];
            const int32_t posn = shl32((int32_t)(A.row0 + n), 16);
            ElemOut outs[VEC];
            // SAFE rows: |te| <= 46, so 2^te and the products it scales stay finite
            const bool safe = cols_safe && (uint32_t)(re - A.P.mantissa_bias + 23) <= 46u;
            const int32_t rbits = safe_row_bits(re, A.P.mantissa_bias);
            if (KIND == CONCORD_KIND_ADAMW && !safe) {
#pragma unroll
                for (int j = 0; j < VEC; ++j) {
                    const float g = bf16_to_f32((gw[j >> 1] >> ((j & 1) * 16)) & 0xffffu);
                    outs[j] = step_adamw_outlined<FL>(A.P, wv[j], g, re, ce[j], vr, vc[j], cp[j], S,
                                                      posn ^ (int32_t)(k0 + j));
                }
            } else if (KIND == CONCORD_KIND_ADAMW) {
                // LOCK elements at a time: phase 1 up to the denominator's
                // argument; phase 2 the correctly rounded exp2(p*log2(x)) side by
                // side; phase 3 the rest
#pragma unroll
                // the cheap reference-GPU arithmetic runs one element at a time
                // (measured 1-2 % faster); the correctly rounded pow keeps pairs
                constexpr int LK = (FL & FL_GPU) ? 1 : STEP_LOCK;
                for (int h = 0; h < VEC; h += LK) {
                    AdamwPre pre[LK];
                    float xs[LK], den[LK];
                    ElemOut o2[LK];
#pragma unroll
                    for (int u = 0; u < LK; ++u) {
                        const int j = h + u;
                        const float g = bf16_to_f32((gw[j >> 1] >> ((j & 1) * 16)) & 0xffffu);
                        pre[u] = adamw_pre<FL, true>(A.P, wv[j], g, rbits, cbits[j], vr, vc[j], cp[j], S);
                        xs[u] = pre[u].x;
                    }
#pragma unroll
                    for (int u = 0; u < LK; ++u) fixed_coh_divide<FL>(A.P, pre[u]);
                    if (gpu_of<FL>(A.P)) {
#pragma unroll
                        for (int u = 0; u < LK; ++u)
                            den[u] = div_full(pre[u].g, pow2log2_as(true, A.P.precond_p, xs[u]));
                    } else {
                        crmath::cr_pow2log2<LK>(xs, A.P.precond_p, den);
#pragma unroll
                        for (int u = 0; u < LK; ++u) den[u] = pre[u].g / den[u];
                    }
                    int32_t posv[LK];
#pragma unroll
                    for (int u = 0; u < LK; ++u) posv[u] = posn ^ (int32_t)(k0 + h + u);
                    adamw_post_lockstep<FL, LK>(A.P, pre, den, S, posv, o2);
#pragma unroll
                    for (int u = 0; u < LK; ++u) outs[h + u] = o2[u];
                }
            } else {
#pragma unroll
                for (int j = 0; j < VEC; ++j) {
                    const float g = bf16_to_f32((gw[j >> 1] >> ((j & 1) * 16)) & 0xffffu);
                    outs[j] = step_sgd<FL>(A.P, wv[j], g, re, ce[j], S, posn ^ (int32_t)(k0 + j));
                }
            }
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
                const ElemOut& o = outs[j];
                wv[j] = o.word;
                cp[j] = o.coh_pre;
                wf[j] = o.wval;
                if (emit) {
                    rml = max(rml, o.abs_eff);
                    cmx[j] = max(cmx[j], o.abs_eff);
                }
                if (need_coh) csum += o.coh;
            }
            if (need_coh) ccnt += VEC;
            __stcs(reinterpret_cast<int4*>(pw), make_int4(wv[0], wv[1], wv[2], wv[3]));
            __nv_bfloat162 b01 = __floats2bfloat162_rn(wf[0], wf[1]);
            __nv_bfloat162 b23 = __floats2bfloat162_rn(wf[2], wf[3]);
            wb = make_uint2(*reinterpret_cast<uint32_t*>(&b01), *reinterpret_cast<uint32_t*>(&b23));
            if (emit) __stcs(reinterpret_cast<uint2*>(A.wbuf + n * A.ldw + k0), wb);
            if (write_cp) __stcs(reinterpret_cast<float4*>(pc), make_float4(cp[0], cp[1], cp[2], cp[3]));
        }
        if (A.npeers > 0 && emit) {
            // the all-gather of the forward weight: this row's weights into every
            // other rank's buffer, 16 bytes per even lane (its 4 columns and its
            // odd neighbour's), 8 bytes where the neighbour has no columns or the
            // rows are not 16-byte aligned
            const uint32_t hx = __shfl_down_sync(0xffffffffu, wb.x, 1);
            const uint32_t hy = __shfl_down_sync(0xffffffffu, wb.y, 1);
            const bool pair = peer16 && (k0 + VEC) < A.K;
            if (active && (!peer16 || !(lane & 1))) {
                const int64_t off = (A.row0 + n) * A.ldw + k0;
                // each row starts at another peer, spreading the stores over the links
                int q = (int)(n % A.npeers);
                for (int t = 0; t < A.npeers; ++t, q = (q + 1 == A.npeers) ? 0 : q + 1) {
                    uint16_t* dst = reinterpret_cast<uint16_t*>(A.wpeers[q]) + off;
                    if (pair) __stcs(reinterpret_cast<uint4*>(dst), make_uint4(wb.x, wb.y, hx, hy));
                    else __stcs(reinterpret_cast<uint2*>(dst), wb);
                }
            }
        }
        if (track) {
            int m = warp_max(rml);
            if (lane == 0 && m > 0) atomicMax(A.row_max + n, m);
        }
    }
    if (track) {
        __shared__ int cm[STEP_THREADS / 32][STEP_COLS];
#pragma unroll
        for (int j = 0; j < VEC; ++j) cm[warp][lane * VEC + j] = cmx[j];
        __syncthreads();
        for (int c = threadIdx.x; c < STEP_COLS; c += STEP_THREADS) {
            int m = 0;
#pragma unroll
            for (int w = 0; w < STEP_THREADS / 32; ++w) m = max(m, cm[w][c]);
            const int64_t col = (int64_t)blockIdx.x * STEP_COLS + c;
            if (col < A.K && m > 0) atomicMax(A.col_max + col, m);
        }
    }
    if (need_coh && A.coh_stats) block_add_coh((double)csum, (double)ccnt, A.coh_stats);
}

// Generic path: any K and strides, one element per thread (runtime flags).
template <int KIND>
__global__ void __launch_bounds__(STEP_THREADS) step_generic_kernel(const __grid_constant__ StepArgs A) {
    const uint32_t F = A.P.flags;
    const bool adamw = KIND == CONCORD_KIND_ADAMW;
    const bool need_vhat = adamw && (F & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH));
    const bool need_coh = adamw && (F & (CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH));
    const bool use_cp = adamw && (F & CONCORD_F_COHPRE) && !(F & CONCORD_F_RATIO_COH) && A.coh_pre;
    const bool write_cp = use_cp && (F & CONCORD_F_APPLY_CHASE);
    const bool track = (F & CONCORD_F_TRACK_REBALANCE) != 0;
    const StepScalars S = load_scalars(A);
    double csum = 0.0, ccnt = 0.0;
    const int64_t total = A.N * A.K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / A.K, k = i - n * A.K;
        const int32_t pos = shl32((int32_t)(A.row0 + n), 16) ^ (int32_t)k;
        const float g = bf16_to_f32(A.grad[n * A.ldg + k]);
        const float cp = use_cp ? A.coh_pre[n * A.ldc + k] : 1.0f;
        ElemOut o = step_elem<KIND, FL_DYNAMIC>(A.P, A.packed[n * A.ldp + k], g, A.row_exp[n], A.col_exp[k],
                                                need_vhat ? A.v_row[n] : 0.0f, need_vhat ? A.v_col[k] : 0.0f,
                                                cp, S, pos);
        A.packed[n * A.ldp + k] = o.word;
        if (write_cp) A.coh_pre[n * A.ldc + k] = o.coh_pre;
        if (need_coh) { csum += (double)o.coh; ccnt += 1.0; }
        if (!S.emit) continue;   // accumulation micro-step: weight and maxima frozen
        const uint16_t wb = __bfloat16_as_ushort(__float2bfloat16_rn(o.wval));
        A.wbuf[n * A.ldw + k] = wb;
        for (int q = 0; q < A.npeers; ++q)
            reinterpret_cast<uint16_t*>(A.wpeers[q])[(A.row0 + n) * A.ldw + k] = wb;
        if (track && o.abs_eff > 0) {
            atomicMax(A.row_max + n, o.abs_eff);
            atomicMax(A.col_max + k, o.abs_eff);
        }
    }
    if (need_coh && A.coh_stats) block_add_coh(csum, ccnt, A.coh_stats);
}

template <int MINB>
static void launch_vec(bool adamw, uint32_t F, bool has_cp, dim3 grid, cudaStream_t s, const StepArgs& A) {
    const bool zero_wd = A.P.wd_sv == 0.0f && A.P.wd_sf == 0.0f && A.P.weight_decay == 0.0f &&
                         A.P.beta1 == 0.0f && A.P.v_scale == 0.0f && A.P.gf_trust_delta_sq == 1.0f &&
                         A.P.gate_gain == 1.0f && fabsf(A.P.drift_cancel_C) <= 1.0f;
    const bool runtime_scalars = A.P.consolidate != nullptr || A.P.ratio_floors != nullptr;
    const bool gpu = A.P.arith == CONCORD_ARITH_GPU;
    if (!adamw) step_vec_kernel<CONCORD_KIND_SGD, FL_DYNAMIC, MINB><<<grid, STEP_THREADS, 0, s>>>(A);
    else if (runtime_scalars) step_vec_kernel<CONCORD_KIND_ADAMW, FL_DYNAMIC, MINB><<<grid, STEP_THREADS, 0, s>>>(A);
    else if (F == (FL_BARE & 0xffffu) && has_cp && zero_wd && gpu)
        step_vec_kernel<CONCORD_KIND_ADAMW, FL_BARE | FL_GPU, MINB><<<grid, STEP_THREADS, 0, s>>>(A);
    else if (F == (FL_NOCOHPRE & 0xffffu) && zero_wd && gpu)
        step_vec_kernel<CONCORD_KIND_ADAMW, FL_NOCOHPRE | FL_GPU, MINB><<<grid, STEP_THREADS, 0, s>>>(A);
    else if (F == (FL_BARE & 0xffffu) && has_cp && zero_wd) step_vec_kernel<CONCORD_KIND_ADAMW, FL_BARE, MINB><<<grid, STEP_THREADS, 0, s>>>(A);
    else if (F == (FL_NOCOHPRE & 0xffffu) && zero_wd) step_vec_kernel<CONCORD_KIND_ADAMW, FL_NOCOHPRE, MINB><<<grid, STEP_THREADS, 0, s>>>(A);
    else step_vec_kernel<CONCORD_KIND_ADAMW, FL_DYNAMIC, MINB><<<grid, STEP_THREADS, 0, s>>>(A);
}

}  // namespace concord

using namespace concord;

static int step_impl(const concord_step_params* p, int32_t* packed, int64_t ldp,
                     const uint16_t* grad, int64_t ldg, uint16_t* wbuf, int64_t ldw,
                     const int8_t* row_exp, const int8_t* col_exp, int32_t* row_max,
                     int32_t* col_max, const float* v_row, const float* v_col,
                     const float* sum_v_inv, float* coh_pre, int64_t ldc, const float* lr,
                     const float* eps, const int32_t* salt, int64_t N, int64_t K,
                     int64_t row0, double* coh_stats, const uint64_t* wpeers, int32_t npeers,
                     void* stream) {
    if (!p || !packed || !grad || !wbuf || !row_exp || !col_exp || !lr || !salt)
        return fail(CONCORD_EINVAL, "concord_step: null pointer");
    if (npeers < 0 || (npeers > 0 && !wpeers)) return fail(CONCORD_EINVAL, "concord_step_sharded: bad peer list");
    if (N < 0 || K < 0 || ldp < K || ldg < K || ldw < K) return fail(CONCORD_ESHAPE, "concord_step: bad shape/stride");
    if (N == 0 || K == 0) return CONCORD_OK;
    if (p->kind != CONCORD_KIND_ADAMW && p->kind != CONCORD_KIND_SGD)
        return fail(CONCORD_EINVAL, "concord_step: optimizer kind must be adamw or sgd");
    const uint32_t F = p->flags;
    const bool adamw = p->kind == CONCORD_KIND_ADAMW;
    const bool need_vhat = adamw && (F & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH));
    if (adamw && !eps) return fail(CONCORD_EINVAL, "concord_step: eps is required for adamw");
    if (p->step_cap != p->step_cap) return fail(CONCORD_EINVAL, "concord_step: step_cap is NaN");
    if (p->arith != CONCORD_ARITH_GPU && p->arith != CONCORD_ARITH_CR)
        return fail(CONCORD_EINVAL, "concord_step: arith must be CONCORD_ARITH_GPU or CONCORD_ARITH_CR");
    if (need_vhat && (!v_row || !v_col || !sum_v_inv))
        return fail(CONCORD_EINVAL, "concord_step: gf_trust/gf_consol/coh_pre/ratio need v_row, v_col, sum_v_inv");
    if ((F & CONCORD_F_TRACK_REBALANCE) && (!row_max || !col_max))
        return fail(CONCORD_EINVAL, "concord_step: track_rebalance needs row_max and col_max");
    const bool use_cp = adamw && (F & CONCORD_F_COHPRE) && !(F & CONCORD_F_RATIO_COH) && coh_pre;
    if (use_cp && ldc < K) return fail(CONCORD_ESHAPE, "concord_step: bad coh_pre stride");
    if (row0 < 0 || row0 + N > (int64_t)1 << 31) return fail(CONCORD_ESHAPE, "concord_step: row index beyond int32");
    StepArgs A{*p, packed, ldp, grad, ldg, wbuf, ldw, row_exp, col_exp, row_max, col_max,
               v_row, v_col, sum_v_inv, coh_pre, ldc, lr, eps, salt, N, K, row0, coh_stats,
               wpeers, npeers};
    bool vec = (K % VEC == 0) && (ldp % VEC == 0) && (ldg % VEC == 0) && (ldw % VEC == 0) &&
               aligned(packed, 16) && aligned(grad, 8) && aligned(wbuf, 8) && aligned(col_exp, 4);
    if (need_vhat) vec = vec && aligned(v_col, 16);
    if (use_cp) vec = vec && (ldc % VEC == 0) && aligned(coh_pre, 16);
    cudaStream_t s = as_stream(stream);
    if (vec) {
        // 32 rows per block, fewer while the grid would cover under ~4 blocks per SM:
        // a thread walks its rows one after another, so small layers need more blocks
        const int64_t cblocks = (K + STEP_COLS - 1) / STEP_COLS;
        int rpb = STEP_ROWS;
        while (rpb > 8 && cblocks * ((N + rpb - 1) / rpb) < 148 * 4) rpb /= 2;
        A.rows_per_block = rpb;
        dim3 grid((unsigned)cblocks, (unsigned)((N + rpb - 1) / rpb));
        if (grid.y > 65535) return fail(CONCORD_ETOOBIG, "concord_step: too many rows for one launch");
        // resident blocks per SM the register budget targets (default 4 = 16
        // warps; CONCORD_STEP_MINB=5 trades spills for 20 warps)
        static const int minb = [] {
            const char* e = getenv("CONCORD_STEP_MINB");
            return (e && e[0] == '5') ? 5 : 4;
        }();
        if (minb == 4) launch_vec<4>(adamw, F, coh_pre != nullptr, grid, s, A);
        else launch_vec<5>(adamw, F, coh_pre != nullptr, grid, s, A);
    } else {
        int64_t blocks = (N * K + STEP_THREADS - 1) / STEP_THREADS;
        if (blocks > 148 * 64) blocks = 148 * 64;
        if (adamw) step_generic_kernel<CONCORD_KIND_ADAMW><<<(unsigned)blocks, STEP_THREADS, 0, s>>>(A);
        else step_generic_kernel<CONCORD_KIND_SGD><<<(unsigned)blocks, STEP_THREADS, 0, s>>>(A);
    }
    return check_launch("concord_step");
}

extern "C" int concord_step(const concord_step_params* p, int32_t* packed, int64_t ldp,
                            const uint16_t* grad, int64_t ldg, uint16_t* wbuf, int64_t ldw,
                            const int8_t* row_exp, const int8_t* col_exp, int32_t* row_max,
                            int32_t* col_max, const float* v_row, const float* v_col,
                            const float* sum_v_inv, float* coh_pre, int64_t ldc, const float* lr,
                            const float* eps, const int32_t* salt, int64_t N, int64_t K,
                            int64_t row0, double* coh_stats, void* stream) {
    return step_impl(p, packed, ldp, grad, ldg, wbuf, ldw, row_exp, col_exp, row_max, col_max, v_row, v_col,
                     sum_v_inv, coh_pre, ldc, lr, eps, salt, N, K, row0, coh_stats, nullptr, 0, stream);
}

extern "C" int concord_step_sharded(const concord_step_params* p, int32_t* packed, int64_t ldp,
                                    const uint16_t* grad, int64_t ldg, uint16_t* wbuf, int64_t ldw,
                                    const int8_t* row_exp, const int8_t* col_exp, int32_t* row_max,
                                    int32_t* col_max, const float* v_row, const float* v_col,
                                    const float* sum_v_inv, float* coh_pre, int64_t ldc, const float* lr,
                                    const float* eps, const int32_t* salt, int64_t N, int64_t K,
                                    int64_t row0, double* coh_stats, const uint64_t* wbuf_peers,
                                    int32_t n_peers, void* stream) {
    return step_impl(p, packed, ldp, grad, ldg, wbuf, ldw, row_exp, col_exp, row_max, col_max, v_row, v_col,
                     sum_v_inv, coh_pre, ldc, lr, eps, salt, N, K, row0, coh_stats, wbuf_peers, n_peers,
                     stream);
}
