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
#include "common.cuh"

namespace concord {

struct StepScalars {
    float lr, eps, svi;
    int32_t salt;
};

struct ElemOut {
    int32_t word;
    uint16_t wbits;
    int32_t abs_eff;
    float coh;      // valid when the flags compute coh
    float coh_pre;  // updated coh_pre (when written)
};

// One element of the AdamW-path step (packed_b.py:476-703).
__device__ __forceinline__ ElemOut step_adamw(const concord_step_params& P, int32_t packed, float g,
                                              int32_t row_e, int32_t col_e, float v_row, float v_col,
                                              float cp, const StepScalars& S, int32_t pos) {
    const uint32_t F = P.flags;
    int32_t s_fast = packed >> 16;
    int32_t s_slow = shl32(packed, 16) >> 24;
    int32_t v_slow = shl32(packed, 24) >> 24;
    int32_t s_slow_full = s_slow * 128;
    int32_t v_slow_full = v_slow * 128;

    int32_t te = row_e + col_e - P.mantissa_bias;
    float scale_fwd = exp2i(te);
    float scale_inv = exp2i(-te);

    float d_fs = (float)s_fast;
    float d_sv = (float)(s_slow_full - v_slow_full);
    float noise = d_fs - P.drift_cancel_C * d_sv;
    float noise_in_w = noise * scale_fwd;
    float v_proxy = noise_in_w * noise_in_w * P.v_scale;

    const bool need_vhat = (F & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) != 0;
    const bool need_coh = (F & (CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) != 0;
    float v_hat = 0.0f, coh = 0.0f;
    if (need_vhat) v_hat = v_row * v_col * S.svi;
    if (F & CONCORD_F_GF_TRUST) v_proxy = v_proxy + P.gf_trust_delta_sq * v_hat;
    if (need_coh) {
        if (F & CONCORD_F_FIXED_COH) {
            float sig_w = P.drift_cancel_C * d_sv * scale_fwd;
            float sig2 = sig_w * sig_w;
            coh = sig2 / (sig2 + noise_in_w * noise_in_w + 1e-30f);
        } else {
            float mg = P.alpha_v_fast * d_sv * scale_fwd;
            coh = mg * mg / (v_hat + 1e-12f);
        }
        coh = np_min(np_max(coh, 0.0f), 1.0f);
    }

    float denom_p = crmath::cr_exp2f(P.precond_p * crmath::cr_log2f(v_proxy + S.eps));
    float step_live = g / denom_p;
    step_live = np_min(np_max(step_live, -P.step_cap), P.step_cap);

    const bool consol = (F & CONCORD_F_GF_CONSOL) != 0;
    float evap = 0.0f;
    if (consol) {
        evap = S.lr * P.gf_consol * (1.0f - coh) * d_fs;
    } else {
        step_live = step_live + P.weight_decay * (d_fs * scale_fwd);
    }
    float delta_t = -S.lr * step_live * scale_inv - P.beta1 * d_fs;
    if (consol) delta_t = delta_t - evap;

    s_fast = s_fast + sr_tick(delta_t, hash_uniform(s_fast, pos, S.salt));

    int32_t new_v = v_slow;
    float cp_new = cp;
    if (F & CONCORD_F_APPLY_CHASE) {
        float chase_mantissa;
        if (F & CONCORD_F_RATIO_COH) {
            float gate = P.chase_floor + P.one_minus_chase_floor * coh;
            chase_mantissa = P.alpha * gate * P.gate_gain * (float)s_fast;
        } else if (F & CONCORD_F_COHPRE) {
            float gate = coh + cp * (1.0f - coh);
            cp_new = P.one_minus_alpha_v_fast * cp + P.alpha_v_fast * coh;
            chase_mantissa = P.alpha * gate * P.gate_gain * (float)s_fast;
        } else {
            chase_mantissa = P.alpha_gate_gain * (float)s_fast;
        }
        int32_t ts = sr_tick(chase_mantissa / 128.0f, hash_uniform(s_fast, pos, S.salt ^ 0x5A5A5A5A));
        s_slow = s_slow + ts;
        s_fast = s_fast - ts * 128;

        float delta_v8 = P.alpha_v_fast * (float)(s_slow * 128 - v_slow_full) / 128.0f;
        if (F & CONCORD_F_RATIO_COH)
            delta_v8 = delta_v8 * (P.leak_floor + P.one_minus_leak_floor * coh);
        int32_t tv = sr_tick(delta_v8, hash_uniform(s_fast, pos, S.salt ^ 0x33335555));
        new_v = clampi(v_slow + tv, -128, 127);
        if (F & CONCORD_F_MASS_PRESERVE) s_slow = s_slow - (new_v - v_slow);

        int32_t v_full_post = new_v * 128;
        if (P.wd_sv != 0.0f) {  // a zero rate gives tick 0 for every finite state
            float d = S.lr * P.wd_sv * (float)(s_slow * 128 - v_full_post) / 128.0f;
            s_slow = s_slow - sr_tick(d, hash_uniform(s_fast, pos, S.salt ^ 0x66665555));
        }
        if (P.wd_sf != 0.0f) {
            float d = S.lr * P.wd_sf * (float)(s_slow * 128 + s_fast - v_full_post);
            s_fast = s_fast - sr_tick(d, hash_uniform(s_fast, pos, S.salt ^ 0x77770000));
        }
    }

    int32_t sfc = clampi(s_fast, -32768, 32767);
    int32_t ssc = clampi(s_slow, -128, 127);
    int32_t m_new = ssc * 128 + sfc + new_v * 128;
    ElemOut o;
    o.word = repack(sfc, ssc, new_v);
    o.wbits = f32_to_bf16((float)m_new * scale_fwd);
    o.abs_eff = abs(m_new);
    o.coh = coh;
    o.coh_pre = cp_new;
    return o;
}

// One element of the SGD-path step (packed_b.py:214-312).
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
    if (P.flags & CONCORD_F_MASS_PRESERVE) s_slow = s_slow - (new_v - v_slow);

    int32_t sfc = clampi(s_fast, -32768, 32767);
    int32_t ssc = clampi(s_slow, -128, 127);
    int32_t m_new = ssc * 128 + sfc + new_v * 128;
    ElemOut o;
    o.word = repack(sfc, ssc, new_v);
    o.wbits = f32_to_bf16((float)m_new * exp2i(te));
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
};

__device__ __forceinline__ StepScalars load_scalars(const StepArgs& A) {
    StepScalars S;
    S.lr = *A.lr;
    S.eps = A.eps ? *A.eps : 1.0f;
    S.salt = *A.salt;
    const bool need_vhat = (A.P.flags & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) != 0;
    S.svi = (need_vhat && A.P.kind == CONCORD_KIND_ADAMW) ? *A.sum_v_inv : 0.0f;
    return S;
}

}  // namespace concord

namespace concord {

constexpr int STEP_THREADS = 256;
constexpr int STEP_COLS = 256;  // 32 lanes x 8 columns
constexpr int STEP_ROWS = 32;   // rows per block (4 per warp)

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

// Vector path: K % 8 == 0, row strides % 8 == 0, 16-byte aligned bases.
template <int KIND>
__global__ void __launch_bounds__(STEP_THREADS) step_vec_kernel(StepArgs A) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t k0 = (int64_t)blockIdx.x * STEP_COLS + lane * 8;
    const bool active = k0 < A.K;
    const int64_t rbase = (int64_t)blockIdx.y * STEP_ROWS;
    const uint32_t F = A.P.flags;
    const bool adamw = KIND == CONCORD_KIND_ADAMW;
    const bool need_vhat = adamw && (F & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH));
    const bool need_coh = adamw && (F & (CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH));
    const bool use_cp = adamw && (F & CONCORD_F_COHPRE) && !(F & CONCORD_F_RATIO_COH) && A.coh_pre;
    const bool write_cp = use_cp && (F & CONCORD_F_APPLY_CHASE);
    const bool track = (F & CONCORD_F_TRACK_REBALANCE) != 0;
    const StepScalars S = load_scalars(A);

    int32_t ce[8];
    float vc[8];
    int cmx[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { ce[j] = 0; vc[j] = 0.0f; cmx[j] = 0; }
    if (active) {
        int2 c8 = *reinterpret_cast<const int2*>(A.col_exp + k0);
        const int8_t* cb = reinterpret_cast<const int8_t*>(&c8);
#pragma unroll
        for (int j = 0; j < 8; ++j) ce[j] = cb[j];
        if (need_vhat) {
            float4 a = *reinterpret_cast<const float4*>(A.v_col + k0);
            float4 b = *reinterpret_cast<const float4*>(A.v_col + k0 + 4);
            vc[0] = a.x; vc[1] = a.y; vc[2] = a.z; vc[3] = a.w;
            vc[4] = b.x; vc[5] = b.y; vc[6] = b.z; vc[7] = b.w;
        }
    }
    double csum = 0.0, ccnt = 0.0;
    for (int r = warp; r < STEP_ROWS; r += STEP_THREADS / 32) {
        const int64_t n = rbase + r;
        if (n >= A.N) break;
        int rml = 0;
        if (active) {
            const int32_t re = A.row_exp[n];
            const float vr = need_vhat ? A.v_row[n] : 0.0f;
            int32_t* pw = A.packed + n * A.ldp + k0;
            int4 w0 = *reinterpret_cast<const int4*>(pw);
            int4 w1 = *reinterpret_cast<const int4*>(pw + 4);
            uint4 g8 = __ldg(reinterpret_cast<const uint4*>(A.grad + n * A.ldg + k0));
            float cp[8];
            if (use_cp) {
                const float* pc = A.coh_pre + n * A.ldc + k0;
                float4 a = *reinterpret_cast<const float4*>(pc);
                float4 b = *reinterpret_cast<const float4*>(pc + 4);
                cp[0] = a.x; cp[1] = a.y; cp[2] = a.z; cp[3] = a.w;
                cp[4] = b.x; cp[5] = b.y; cp[6] = b.z; cp[7] = b.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) cp[j] = 1.0f;
            }
            int32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            uint32_t gw[4] = {g8.x, g8.y, g8.z, g8.w};
            uint32_t ob[4];
            const int32_t posn = shl32((int32_t)(A.row0 + n), 16);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float g = bf16_to_f32((gw[j >> 1] >> ((j & 1) * 16)) & 0xffffu);
                const int32_t pos = posn ^ (int32_t)(k0 + j);
                ElemOut o = adamw ? step_adamw(A.P, wv[j], g, re, ce[j], vr, vc[j], cp[j], S, pos)
                                  : step_sgd(A.P, wv[j], g, re, ce[j], S, pos);
                wv[j] = o.word;
                cp[j] = o.coh_pre;
                if (j & 1) ob[j >> 1] |= (uint32_t)o.wbits << 16; else ob[j >> 1] = o.wbits;
                rml = max(rml, o.abs_eff);
                cmx[j] = max(cmx[j], o.abs_eff);
                if (need_coh) { csum += (double)o.coh; ccnt += 1.0; }
            }
            *reinterpret_cast<int4*>(pw) = make_int4(wv[0], wv[1], wv[2], wv[3]);
            *reinterpret_cast<int4*>(pw + 4) = make_int4(wv[4], wv[5], wv[6], wv[7]);
            *reinterpret_cast<uint4*>(A.wbuf + n * A.ldw + k0) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
            if (write_cp) {
                float* pc = A.coh_pre + n * A.ldc + k0;
                *reinterpret_cast<float4*>(pc) = make_float4(cp[0], cp[1], cp[2], cp[3]);
                *reinterpret_cast<float4*>(pc + 4) = make_float4(cp[4], cp[5], cp[6], cp[7]);
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
        for (int j = 0; j < 8; ++j) cm[warp][lane * 8 + j] = cmx[j];
        __syncthreads();
        int m = 0;
#pragma unroll
        for (int w = 0; w < STEP_THREADS / 32; ++w) m = max(m, cm[w][threadIdx.x]);
        const int64_t col = (int64_t)blockIdx.x * STEP_COLS + threadIdx.x;
        if (col < A.K && m > 0) atomicMax(A.col_max + col, m);
    }
    if (need_coh && A.coh_stats) block_add_coh(csum, ccnt, A.coh_stats);
}

// Generic path: any K and strides, one element per thread.
template <int KIND>
__global__ void __launch_bounds__(STEP_THREADS) step_generic_kernel(StepArgs A) {
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
        ElemOut o = adamw ? step_adamw(A.P, A.packed[n * A.ldp + k], g, A.row_exp[n], A.col_exp[k],
                                       need_vhat ? A.v_row[n] : 0.0f, need_vhat ? A.v_col[k] : 0.0f,
                                       cp, S, pos)
                          : step_sgd(A.P, A.packed[n * A.ldp + k], g, A.row_exp[n], A.col_exp[k], S, pos);
        A.packed[n * A.ldp + k] = o.word;
        A.wbuf[n * A.ldw + k] = o.wbits;
        if (write_cp) A.coh_pre[n * A.ldc + k] = o.coh_pre;
        if (track && o.abs_eff > 0) {
            atomicMax(A.row_max + n, o.abs_eff);
            atomicMax(A.col_max + k, o.abs_eff);
        }
        if (need_coh) { csum += (double)o.coh; ccnt += 1.0; }
    }
    if (need_coh && A.coh_stats) block_add_coh(csum, ccnt, A.coh_stats);
}

}  // namespace concord

using namespace concord;

extern "C" int concord_step(const concord_step_params* p, int32_t* packed, int64_t ldp,
                            const uint16_t* grad, int64_t ldg, uint16_t* wbuf, int64_t ldw,
                            const int8_t* row_exp, const int8_t* col_exp, int32_t* row_max,
                            int32_t* col_max, const float* v_row, const float* v_col,
                            const float* sum_v_inv, float* coh_pre, int64_t ldc, const float* lr,
                            const float* eps, const int32_t* salt, int64_t N, int64_t K,
                            int64_t row0, double* coh_stats, void* stream) {
    if (!p || !packed || !grad || !wbuf || !row_exp || !col_exp || !lr || !salt)
        return fail(CONCORD_EINVAL, "concord_step: null pointer");
    if (N < 0 || K < 0 || ldp < K || ldg < K || ldw < K) return fail(CONCORD_ESHAPE, "concord_step: bad shape/stride");
    if (N == 0 || K == 0) return CONCORD_OK;
    if (p->kind != CONCORD_KIND_ADAMW && p->kind != CONCORD_KIND_SGD)
        return fail(CONCORD_EINVAL, "concord_step: optimizer kind must be adamw or sgd");
    const uint32_t F = p->flags;
    const bool adamw = p->kind == CONCORD_KIND_ADAMW;
    if (adamw && !eps) return fail(CONCORD_EINVAL, "concord_step: eps is required for adamw");
    if (adamw && (F & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)) &&
        (!v_row || !v_col || !sum_v_inv))
        return fail(CONCORD_EINVAL, "concord_step: gf_trust/gf_consol/coh_pre/ratio need v_row, v_col, sum_v_inv");
    if ((F & CONCORD_F_TRACK_REBALANCE) && (!row_max || !col_max))
        return fail(CONCORD_EINVAL, "concord_step: track_rebalance needs row_max and col_max");
    if (adamw && (F & CONCORD_F_COHPRE) && !(F & CONCORD_F_RATIO_COH) && coh_pre && ldc < K)
        return fail(CONCORD_ESHAPE, "concord_step: bad coh_pre stride");
    if (row0 < 0 || row0 + N > (int64_t)1 << 31) return fail(CONCORD_ESHAPE, "concord_step: row index beyond int32");
    StepArgs A{*p, packed, ldp, grad, ldg, wbuf, ldw, row_exp, col_exp, row_max, col_max,
               v_row, v_col, sum_v_inv, coh_pre, ldc, lr, eps, salt, N, K, row0, coh_stats};
    bool vec = (K % 8 == 0) && (ldp % 8 == 0) && (ldg % 8 == 0) && (ldw % 8 == 0) &&
               aligned(packed, 16) && aligned(grad, 16) && aligned(wbuf, 16) && aligned(col_exp, 8);
    if (adamw && (F & (CONCORD_F_GF_TRUST | CONCORD_F_GF_CONSOL | CONCORD_F_COHPRE | CONCORD_F_RATIO_COH)))
        vec = vec && aligned(v_col, 16);
    if (coh_pre) vec = vec && (ldc % 8 == 0) && aligned(coh_pre, 16);
    cudaStream_t s = as_stream(stream);
    if (vec) {
        dim3 grid((unsigned)((K + STEP_COLS - 1) / STEP_COLS), (unsigned)((N + STEP_ROWS - 1) / STEP_ROWS));
        if (grid.y > 65535) return fail(CONCORD_ETOOBIG, "concord_step: too many rows for one launch");
        if (adamw) step_vec_kernel<CONCORD_KIND_ADAMW><<<grid, STEP_THREADS, 0, s>>>(A);
        else step_vec_kernel<CONCORD_KIND_SGD><<<grid, STEP_THREADS, 0, s>>>(A);
    } else {
        int64_t blocks = (N * K + STEP_THREADS - 1) / STEP_THREADS;
        if (blocks > 148 * 64) blocks = 148 * 64;
        if (adamw) step_generic_kernel<CONCORD_KIND_ADAMW><<<(unsigned)blocks, STEP_THREADS, 0, s>>>(A);
        else step_generic_kernel<CONCORD_KIND_SGD><<<(unsigned)blocks, STEP_THREADS, 0, s>>>(A);
    }
    return check_launch("concord_step");
}
