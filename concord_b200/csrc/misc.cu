// misc.cu — materialize (K0), quantize (load_weights), coherence meter (K4),
// salt bump, and the C-ABI error plumbing.
#include <stdio.h>

#include "common.cuh"

namespace concord {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }
int fail(int code, const std::string& msg) { g_last_error = msg; return code; }
int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
        return CONCORD_ELAUNCH;
    }
    return CONCORD_OK;
}

// _materialize_packed_bf16_kernel (packed_b.py:120-155) / consolidated_weight (1632-1649)
__global__ void materialize_kernel(const int32_t* packed, int64_t ldp, const int8_t* row_exp,
                                   const int8_t* col_exp, uint16_t* out, int64_t ldo, int64_t N,
                                   int64_t K, int32_t mb, int32_t consolidated) {
    const int64_t total = N * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / K, k = i - n * K;
        const int32_t w = packed[n * ldp + k];
        const int32_t sf = w >> 16, ss = shl32(w, 16) >> 24, vs = shl32(w, 24) >> 24;
        const int32_t m = consolidated ? ss * 128 + vs * 128 : ss * 128 + sf + vs * 128;
        out[n * ldo + k] = f32_to_bf16((float)m * exp2i((int32_t)row_exp[n] + col_exp[k] - mb));
    }
}

// load_weights / load_weights_finetune (packed_b.py:1570-1603, 1816-1856):
// one block per row: row max |W| -> row_exp, then quantize the row.
__global__ void quantize_kernel(const float* W, int64_t ldw, int32_t* packed, int64_t ldp,
                                int8_t* row_exp, int64_t K, int32_t mb, int32_t emin,
                                int32_t emax, int32_t finetune) {
    const int64_t n = blockIdx.x;
    __shared__ float red[256];
    float mx = 0.0f;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) mx = np_max(mx, fabsf(W[n * ldw + k]));
    red[threadIdx.x] = mx;
    __syncthreads();
    for (int s = 128; s >= 1; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] = np_max(red[threadIdx.x], red[threadIdx.x + s]);
        __syncthreads();
    }
    mx = np_max(red[0], 1e-30f);
    float e = ceilf(crmath::cr_log2f(mx) + 1.0f);
    e = np_min(np_max(e, (float)emin), (float)emax);
    const int32_t re = (int32_t)e;
    if (threadIdx.x == 0) row_exp[n] = (int8_t)re;
    const float scale = exp2i(re - mb);
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
        const int32_t m_total = __float2int_rz(rintf(W[n * ldw + k] / scale));
        int32_t sf, ss = 0, vs = 0;
        if (!finetune) {
            sf = clampi(m_total, -32768, 32767);
        } else {
            const int32_t tv = __float2int_rz(rintf((float)m_total / 2.0f));
            vs = clampi(__float2int_rz(rintf((float)tv / 128.0f)), -128, 127);
            const int32_t remaining = m_total - vs * 128;
            ss = clampi(__float2int_rz(rintf((float)remaining / 128.0f)), -128, 127);
            sf = clampi(remaining - ss * 128, -32768, 32767);
        }
        packed[n * ldp + k] = repack(sf, ss, vs);
    }
}

// vector form: 4 consecutive columns per thread, a 2-D grid (no 64-bit division)
__global__ void materialize_vec_kernel(const int32_t* packed, int64_t ldp, const int8_t* row_exp,
                                       const int8_t* col_exp, uint16_t* out, int64_t ldo, int64_t N,
                                       int64_t K, int32_t mb, int32_t consolidated) {
    const int64_t k0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (k0 >= K) return;
    const uint32_t c4 = *reinterpret_cast<const uint32_t*>(col_exp + k0);
    for (int64_t n = blockIdx.y; n < N; n += gridDim.y) {
        const int4 w = __ldcs(reinterpret_cast<const int4*>(packed + n * ldp + k0));
        const int32_t re = row_exp[n] - mb;
        const int32_t wv[4] = {w.x, w.y, w.z, w.w};
        float f[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int32_t v = wv[j];
            const int32_t sf = v >> 16, ss = shl32(v, 16) >> 24, vs = shl32(v, 24) >> 24;
            const int32_t m = consolidated ? ss * 128 + vs * 128 : ss * 128 + sf + vs * 128;
            f[j] = (float)m * exp2i(re + (int32_t)(int8_t)(c4 >> (8 * j)));
        }
        const uint32_t lo = (uint32_t)f32_to_bf16(f[0]) | ((uint32_t)f32_to_bf16(f[1]) << 16);
        const uint32_t hi = (uint32_t)f32_to_bf16(f[2]) | ((uint32_t)f32_to_bf16(f[3]) << 16);
        __stcs(reinterpret_cast<uint2*>(out + n * ldo + k0), make_uint2(lo, hi));
    }
}

__global__ void zero_i8_kernel(int8_t* p, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = 0;
}

// gate_coherence_from_fields (packed_b.py:2081-2091) summed in double
__global__ void coherence_kernel(const int32_t* packed, int64_t ldp, int64_t N, int64_t K, float C,
                                 double* out) {
    __shared__ double red[256];
    double acc = 0.0;
    const int64_t total = N * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / K, k = i - n * K;
        const int32_t w = packed[n * ldp + k];
        const float sf = (float)(w >> 16), ss = (float)(shl32(w, 16) >> 24), vs = (float)(shl32(w, 24) >> 24);
        const float d_sv = (ss - vs) * 128.0f;
        const float sig = C * d_sv;
        const float noise = sf - sig;
        const float sig2 = sig * sig;
        acc += (double)(sig2 / (sig2 + noise * noise + 1e-30f));
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int s = 128; s >= 1; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        atomicAdd(out, red[0]);
        if (blockIdx.x == 0) atomicAdd(out + 1, (double)total);
    }
}

// Per-weight garbage fraction (get_garbage_fraction_stats, packed_b.py:1676-1730):
// gf = clamp((noise * 2^te)^2 / (v_hat + 1e-30), 0, 1) with noise the
// drift-cancelled velocity s_fast - C * (128 s_slow - 128 v_slow) and
// v_hat = v_row v_col / sum_v, every operation one fp32 rounding as torch
// evaluates it.  gf is written when gf_out is given; acc[0..2] += sum of gf,
// count of gf < 0.1, count of gf > 0.9 (double, one atomic per block).
__global__ void garbage_fraction_kernel(const int32_t* packed, int64_t ldp, const int8_t* row_exp,
                                        const int8_t* col_exp, const float* v_row, const float* v_col,
                                        const float* sum_v, int64_t N, int64_t K, int32_t mb, float C,
                                        float* gf_out, double* acc) {
    __shared__ double red[3][8];
    const float sv = *sum_v;
    double a0 = 0.0, a1 = 0.0, a2 = 0.0;
    const int64_t total = N * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / K, k = i - n * K;
        const int32_t w = packed[n * ldp + k];
        const float sf = (float)(w >> 16);
        const float ssf = __fmul_rn((float)(shl32(w, 16) >> 24), 128.0f);
        const float vsf = __fmul_rn((float)(shl32(w, 24) >> 24), 128.0f);
        const float noise = __fsub_rn(sf, __fmul_rn(C, __fsub_rn(ssf, vsf)));
        const float nw = __fmul_rn(noise, exp2i((int32_t)row_exp[n] + (int32_t)col_exp[k] - mb));
        const float vh = __fdiv_rn(__fmul_rn(v_row[n], v_col[k]), sv);
        float gf = __fdiv_rn(__fmul_rn(nw, nw), __fadd_rn(vh, 1e-30f));
        gf = fminf(fmaxf(gf, 0.0f), 1.0f);
        if (gf_out) gf_out[i] = gf;
        a0 += (double)gf;
        a1 += gf < 0.1f ? 1.0 : 0.0;
        a2 += gf > 0.9f ? 1.0 : 0.0;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        a0 += __shfl_xor_sync(0xffffffffu, a0, o);
        a1 += __shfl_xor_sync(0xffffffffu, a1, o);
        a2 += __shfl_xor_sync(0xffffffffu, a2, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { red[0][warp] = a0; red[1][warp] = a1; red[2][warp] = a2; }
    __syncthreads();
    if (threadIdx.x < 3) {
        double t = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[threadIdx.x][w];
        atomicAdd(acc + threadIdx.x, t);
    }
}

__global__ void salt_bump_kernel(int32_t* salt) { *salt += 1; }

static unsigned grid_for(int64_t total, int threads) {
    int64_t b = (total + threads - 1) / threads;
    if (b > 148 * 32) b = 148 * 32;
    if (b < 1) b = 1;
    return (unsigned)b;
}

}  // namespace concord

using namespace concord;

extern "C" int concord_abi_version(void) { return CONCORD_ABI_VERSION; }
extern "C" const char* concord_last_error(void) { return g_last_error.c_str(); }

extern "C" int concord_salt_bump(int32_t* salt, void* stream) {
    if (!salt) return fail(CONCORD_EINVAL, "concord_salt_bump: null pointer");
    salt_bump_kernel<<<1, 1, 0, as_stream(stream)>>>(salt);
    return check_launch("concord_salt_bump");
}

extern "C" int concord_materialize(const int32_t* packed, int64_t ldp, const int8_t* row_exp,
                                   const int8_t* col_exp, uint16_t* out, int64_t ldo, int64_t N,
                                   int64_t K, int32_t mantissa_bias, int32_t consolidated, void* stream) {
    if (!packed || !row_exp || !col_exp || !out) return fail(CONCORD_EINVAL, "concord_materialize: null pointer");
    if (N < 0 || K < 0 || ldp < K || ldo < K) return fail(CONCORD_ESHAPE, "concord_materialize: bad shape/stride");
    if (N == 0 || K == 0) return CONCORD_OK;
    if (K % 4 == 0 && ldp % 4 == 0 && ldo % 4 == 0 && aligned(packed, 16) && aligned(out, 8) && aligned(col_exp, 4)) {
        const int64_t tx = (K / 4 + 127) / 128;
        int64_t ty = N < 4096 ? N : 4096;
        materialize_vec_kernel<<<dim3((unsigned)tx, (unsigned)ty), 128, 0, as_stream(stream)>>>(
            packed, ldp, row_exp, col_exp, out, ldo, N, K, mantissa_bias, consolidated);
    } else {
        materialize_kernel<<<grid_for(N * K, 256), 256, 0, as_stream(stream)>>>(packed, ldp, row_exp, col_exp, out,
                                                                              ldo, N, K, mantissa_bias, consolidated);
    }
    return check_launch("concord_materialize");
}

extern "C" int concord_quantize(const float* W, int64_t ldw, int32_t* packed, int64_t ldp, int8_t* row_exp,
                                int8_t* col_exp, int64_t N, int64_t K, int32_t mantissa_bias, int32_t exp_min,
                                int32_t exp_max, int32_t finetune, void* stream) {
    if (!W || !packed || !row_exp || !col_exp) return fail(CONCORD_EINVAL, "concord_quantize: null pointer");
    if (N < 0 || K < 0 || ldw < K || ldp < K) return fail(CONCORD_ESHAPE, "concord_quantize: bad shape/stride");
    if (N == 0 || K == 0) return CONCORD_OK;
    if (N > 0x7fffffff) return fail(CONCORD_ETOOBIG, "concord_quantize: too many rows");
    cudaStream_t s = as_stream(stream);
    zero_i8_kernel<<<grid_for(K, 256), 256, 0, s>>>(col_exp, K);
    quantize_kernel<<<(unsigned)N, 256, 0, s>>>(W, ldw, packed, ldp, row_exp, K, mantissa_bias, exp_min, exp_max,
                                                finetune);
    return check_launch("concord_quantize");
}

extern "C" int concord_coherence(const int32_t* packed, int64_t ldp, int64_t N, int64_t K, float drift_cancel_C,
                                 double* out, void* stream) {
    if (!packed || !out) return fail(CONCORD_EINVAL, "concord_coherence: null pointer");
    if (N < 0 || K < 0 || ldp < K) return fail(CONCORD_ESHAPE, "concord_coherence: bad shape/stride");
    if (N == 0 || K == 0) return CONCORD_OK;
    coherence_kernel<<<grid_for(N * K, 256), 256, 0, as_stream(stream)>>>(packed, ldp, N, K, drift_cancel_C, out);
    return check_launch("concord_coherence");
}

extern "C" int concord_garbage_fraction(const int32_t* packed, int64_t ldp, const int8_t* row_exp,
                                        const int8_t* col_exp, const float* v_row, const float* v_col,
                                        const float* sum_v, int64_t N, int64_t K, int32_t mantissa_bias,
                                        float drift_cancel_C, float* gf_out, double* acc, void* stream) {
    if (!packed || !row_exp || !col_exp || !v_row || !v_col || !sum_v || !acc)
        return fail(CONCORD_EINVAL, "concord_garbage_fraction: null pointer");
    if (N < 0 || K < 0 || ldp < K) return fail(CONCORD_ESHAPE, "concord_garbage_fraction: bad shape/stride");
    if (N == 0 || K == 0) return CONCORD_OK;
    garbage_fraction_kernel<<<grid_for(N * K, 256), 256, 0, as_stream(stream)>>>(
        packed, ldp, row_exp, col_exp, v_row, v_col, sum_v, N, K, mantissa_bias, drift_cancel_C, gf_out, acc);
    return check_launch("concord_garbage_fraction");
}
