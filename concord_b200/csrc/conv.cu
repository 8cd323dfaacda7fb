// conv.cu — the data movement around ConcordConv2dPackedB's convolutions
// when they run as GEMMs: im2col (input -> column matrix) and col2im (column
// gradient -> input gradient).
//
// The reference runs its conv layer through torch's conv2d and its grad
// functions (concord/packed_b.py:2024-2065) on the [O, I*kh*kw] view of the
// packed weight.  Here the convolution is the Linear layer's GEMMs over a
// column matrix whose columns follow that view's order (channel, kernel row,
// kernel column):
//   im2col : cols[m, c*kh*kw + i*kw + j] = x[b, c, ho*sh - ph + i, wo*sw - pw + j]
//            (zero outside the image), m = (b*Ho + ho)*Wo + wo; one pass,
//            transposed through shared memory, 16-byte stores.
//   col2im : dx[b, c, h, w] = sum over (i, j) of dcolsT[c*kh*kw + i*kw + j, m]
//            for the m whose window covers (h, w) at (i, j); the column
//            gradient arrives transposed ([C*kh*kw, B*Ho*Wo], the GEMM writes
//            it that way) so that neighbouring threads read neighbouring
//            addresses; fp32 sum in (i, j) order, one bf16 rounding (RNE).
#include "common.cuh"

namespace concord {

struct ConvGeom {
    int64_t B, C, H, W, Ho, Wo;
    int32_t kh, kw, sh, sw, ph, pw;
};

// One block per tile of IM_TM output positions x IM_TC columns.  A table of
// the tile's columns (input offset and kernel position) is built once per
// block; the gather runs with neighbouring threads on neighbouring positions
// (for stride 1, neighbouring input pixels) into a [column][position] tile,
// and the store runs 16 bytes (8 columns of one position) per thread.
constexpr int IM_TM = 64, IM_TC = 64, IM_THREADS = 256;

__global__ void __launch_bounds__(IM_THREADS) im2col_kernel(const uint16_t* __restrict__ x,
                                                            uint16_t* __restrict__ cols, ConvGeom g) {
    __shared__ uint16_t tile[IM_TC][IM_TM + 2];
    __shared__ int64_t coff[IM_TC];
    __shared__ int32_t cki[IM_TC], ckj[IM_TC];
    const int32_t kk = g.kh * g.kw;
    const int32_t ckk = (int32_t)g.C * kk;
    const int32_t L = (int32_t)(g.Ho * g.Wo);
    const int64_t M = g.B * L;
    const int64_t m0 = (int64_t)blockIdx.x * IM_TM;
    const int32_t c0 = (int32_t)blockIdx.y * IM_TC;
    const int64_t plane = g.H * g.W;
    if (threadIdx.x < IM_TC) {
        const int32_t col = c0 + threadIdx.x;
        int32_t i = -(1 << 29), j = 0;   // columns past the end never pass the bounds test
        int64_t off = 0;
        if (col < ckk) {
            const int32_t c = col / kk, r = col - c * kk;
            i = r / g.kw;
            j = r - i * g.kw;
            off = (int64_t)c * plane + (int64_t)i * g.W + j;
        }
        coff[threadIdx.x] = off; cki[threadIdx.x] = i; ckj[threadIdx.x] = j;
    }
    __syncthreads();
    {
        const int32_t mi = threadIdx.x % IM_TM;
        const int64_t m = m0 + mi;
        const bool mok = m < M;
        const int32_t b = mok ? (int32_t)(m / L) : 0;
        const int32_t p = mok ? (int32_t)(m - (int64_t)b * L) : 0;
        const int32_t ho = p / (int32_t)g.Wo, wo = p - ho * (int32_t)g.Wo;
        const int32_t h0 = mok ? ho * g.sh - g.ph : -(1 << 29), w0 = wo * g.sw - g.pw;
        const int64_t base = (int64_t)b * g.C * plane + (int64_t)h0 * g.W + w0;
#pragma unroll 4
        for (int32_t ci = threadIdx.x / IM_TM; ci < IM_TC; ci += IM_THREADS / IM_TM) {
            const int32_t h = h0 + cki[ci], w = w0 + ckj[ci];
            uint16_t v = 0;
            if ((uint32_t)h < (uint32_t)g.H && (uint32_t)w < (uint32_t)g.W) v = x[base + coff[ci]];
            tile[ci][mi] = v;
        }
    }
    __syncthreads();
    for (int q = threadIdx.x; q < IM_TM * (IM_TC / 8); q += IM_THREADS) {
        const int32_t mi = q >> 3, ch = q & 7;
        const int64_t m = m0 + mi;
        const int32_t col = c0 + ch * 8;
        if (m < M && col < ckk) {
            uint32_t v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                v[e] = (uint32_t)tile[ch * 8 + 2 * e][mi] | ((uint32_t)tile[ch * 8 + 2 * e + 1][mi] << 16);
            *reinterpret_cast<uint4*>(cols + m * ckk + col) = make_uint4(v[0], v[1], v[2], v[3]);
        }
    }
}

// blockIdx.x = (image, channel) plane; 32-bit index arithmetic inside it.
// KH / KW: compile-time kernel size (0: read it from g)
template <bool UNIT_STRIDE, int KH, int KW>
__global__ void col2im_kernel(const uint16_t* __restrict__ dcolsT, uint16_t* __restrict__ dx, ConvGeom g) {
    const int32_t kh = KH ? KH : g.kh, kw = KW ? KW : g.kw;
    const int32_t kk = kh * kw;
    const int64_t M = g.B * g.Ho * g.Wo;
    const int32_t bc = blockIdx.x;
    const int32_t b = bc / (int32_t)g.C, c = bc - b * (int32_t)g.C;
    const int32_t H = (int32_t)g.H, W = (int32_t)g.W, Ho = (int32_t)g.Ho, Wo = (int32_t)g.Wo;
    const int32_t plane = H * W;
    const uint16_t* src = dcolsT + (int64_t)c * kk * M + (int64_t)b * Ho * Wo;
    uint16_t* dst = dx + (int64_t)bc * plane;
    for (int32_t t = blockIdx.y * blockDim.x + threadIdx.x; t < plane; t += gridDim.y * blockDim.x) {
        const int32_t h = t / W, w = t - h * W;
        float acc = 0.0f;
#pragma unroll
        for (int32_t i = 0; i < kh; ++i) {
            int32_t ho = h + g.ph - i;                  // = ho * sh
            if (ho < 0) continue;
            if (!UNIT_STRIDE) {
                if (ho % g.sh) continue;
                ho /= g.sh;
            }
            if (ho >= Ho) continue;
#pragma unroll
            for (int32_t j = 0; j < kw; ++j) {
                int32_t wo = w + g.pw - j;
                if (wo < 0) continue;
                if (!UNIT_STRIDE) {
                    if (wo % g.sw) continue;
                    wo /= g.sw;
                }
                if (wo >= Wo) continue;
                acc = acc + bf16_to_f32(src[(int64_t)(i * kw + j) * M + ho * Wo + wo]);
            }
        }
        dst[t] = f32_to_bf16(acc);
    }
}

// Batched bf16 transpose, in [batches, R, C] -> out [batches, C, R]: the
// NCHW gradient of a convolution as the [B*Ho*Wo, O] rows its dW GEMM reads.
// 32x32 tiles through shared memory (row pitch 34 halves: the column reads
// fall on distinct banks), both sides coalesced.
__global__ void transpose_kernel(const uint16_t* __restrict__ in, uint16_t* __restrict__ out, int64_t R,
                                 int64_t C) {
    __shared__ uint16_t tile[32][34];
    const int64_t b = blockIdx.z;
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    const uint16_t* src = in + b * R * C;
    uint16_t* dst = out + b * R * C;
#pragma unroll
    for (int k = 0; k < 32; k += 8) {
        const int64_t r = r0 + threadIdx.y + k, c = c0 + threadIdx.x;
        if (r < R && c < C) tile[threadIdx.y + k][threadIdx.x] = src[r * C + c];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 32; k += 8) {
        const int64_t c = c0 + threadIdx.y + k, r = r0 + threadIdx.x;
        if (r < R && c < C) dst[c * R + r] = tile[threadIdx.x][threadIdx.y + k];
    }
}

static int make_geom(int64_t B, int64_t C, int64_t H, int64_t W, int32_t kh, int32_t kw, int32_t sh,
                     int32_t sw, int32_t ph, int32_t pw, ConvGeom* g, const char* who) {
    if (B < 0 || C < 0 || H < 0 || W < 0 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 || ph < 0 || pw < 0)
        return fail(CONCORD_EINVAL, std::string(who) + ": bad geometry");
    g->B = B; g->C = C; g->H = H; g->W = W;
    g->kh = kh; g->kw = kw; g->sh = sh; g->sw = sw; g->ph = ph; g->pw = pw;
    g->Ho = (H + 2 * ph - kh) / sh + 1;
    g->Wo = (W + 2 * pw - kw) / sw + 1;
    if (H + 2 * ph < kh || W + 2 * pw < kw) g->Ho = g->Wo = 0;
    return CONCORD_OK;
}

}  // namespace concord

using namespace concord;

extern "C" int concord_im2col(const uint16_t* x, int64_t B, int64_t C, int64_t H, int64_t W, int32_t kh,
                              int32_t kw, int32_t sh, int32_t sw, int32_t ph, int32_t pw, uint16_t* cols,
                              void* stream) {
    ConvGeom g;
    int rc = make_geom(B, C, H, W, kh, kw, sh, sw, ph, pw, &g, "concord_im2col");
    if (rc) return rc;
    if ((C * kh * kw) % 8 != 0) return fail(CONCORD_ESHAPE, "concord_im2col: C*kh*kw must be a multiple of 8");
    if (!aligned(cols, 16)) return fail(CONCORD_EALIGN, "concord_im2col: cols must be 16-byte aligned");
    const int64_t M = B * g.Ho * g.Wo, ckk = C * kh * kw;
    if (M == 0 || ckk == 0) return CONCORD_OK;
    if (!x || !cols) return fail(CONCORD_EINVAL, "concord_im2col: null pointer");
    if (ckk > INT32_MAX || g.Ho * g.Wo > INT32_MAX || C * H * W > INT32_MAX || (M + IM_TM - 1) / IM_TM > INT32_MAX)
        return fail(CONCORD_ESHAPE, "concord_im2col: extents above 32-bit tile indexing");
    const dim3 grid((unsigned)((M + IM_TM - 1) / IM_TM), (unsigned)((ckk + IM_TC - 1) / IM_TC));
    if (grid.y > 65535) return fail(CONCORD_ESHAPE, "concord_im2col: C*kh*kw too large");
    im2col_kernel<<<grid, IM_THREADS, 0, as_stream(stream)>>>(x, cols, g);
    return check_launch("concord_im2col");
}

extern "C" int concord_col2im(const uint16_t* dcols_t, int64_t B, int64_t C, int64_t H, int64_t W, int32_t kh,
                              int32_t kw, int32_t sh, int32_t sw, int32_t ph, int32_t pw, uint16_t* dx,
                              void* stream) {
    ConvGeom g;
    int rc = make_geom(B, C, H, W, kh, kw, sh, sw, ph, pw, &g, "concord_col2im");
    if (rc) return rc;
    const int64_t total = B * C * H * W;
    if (total == 0) return CONCORD_OK;
    if (!dcols_t || !dx) return fail(CONCORD_EINVAL, "concord_col2im: null pointer");
    if (B * C > INT32_MAX || H * W > INT32_MAX || g.Ho * g.Wo > INT32_MAX)
        return fail(CONCORD_ESHAPE, "concord_col2im: extents above 32-bit indexing");
    const int64_t per_plane = (H * W + 255) / 256;
    const dim3 grid((unsigned)(B * C), (unsigned)(per_plane < 64 ? per_plane : 64));
    cudaStream_t st = as_stream(stream);
    const bool unit = sh == 1 && sw == 1;
    if (unit && kh == 3 && kw == 3) col2im_kernel<true, 3, 3><<<grid, 256, 0, st>>>(dcols_t, dx, g);
    else if (unit && kh == 1 && kw == 1) col2im_kernel<true, 1, 1><<<grid, 256, 0, st>>>(dcols_t, dx, g);
    else if (unit) col2im_kernel<true, 0, 0><<<grid, 256, 0, st>>>(dcols_t, dx, g);
    else if (kh == 3 && kw == 3) col2im_kernel<false, 3, 3><<<grid, 256, 0, st>>>(dcols_t, dx, g);
    else col2im_kernel<false, 0, 0><<<grid, 256, 0, st>>>(dcols_t, dx, g);
    return check_launch("concord_col2im");
}

extern "C" int concord_transpose_bf16(const uint16_t* in, int64_t batches, int64_t R, int64_t C, uint16_t* out,
                                      void* stream) {
    if (batches < 0 || R < 0 || C < 0) return fail(CONCORD_EINVAL, "concord_transpose_bf16: negative size");
    if (batches == 0 || R == 0 || C == 0) return CONCORD_OK;
    if (!in || !out) return fail(CONCORD_EINVAL, "concord_transpose_bf16: null pointer");
    if (batches > 65535 || (R + 31) / 32 > 65535 || (C + 31) / 32 > INT32_MAX)
        return fail(CONCORD_ESHAPE, "concord_transpose_bf16: grid too large");
    const dim3 grid((unsigned)((C + 31) / 32), (unsigned)((R + 31) / 32), (unsigned)batches);
    transpose_kernel<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(in, out, R, C);
    return check_launch("concord_transpose_bf16");
}
