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
//            (zero outside the image), m = (b*Ho + ho)*Wo + wo; one pass, one
//            16-byte store of 8 columns per thread.
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

__global__ void im2col_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ cols, ConvGeom g) {
    const int32_t kk = g.kh * g.kw;
    const int64_t ckk = g.C * kk;
    const int64_t groups = ckk / 8;
    const int64_t L = g.Ho * g.Wo;
    const int64_t total = g.B * L * groups;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = t / groups;
        const int64_t col0 = (t - m * groups) * 8;
        const int64_t b = m / L;
        const int64_t p = m - b * L;
        const int64_t ho = p / g.Wo, wo = p - ho * g.Wo;
        const int64_t h0 = ho * g.sh - g.ph, w0 = wo * g.sw - g.pw;
        int64_t c = col0 / kk;
        int32_t r = (int32_t)(col0 - c * kk);
        int32_t i = r / g.kw, j = r - i * g.kw;
        uint32_t v[4];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int64_t h = h0 + i, w = w0 + j;
            uint32_t val = 0;
            if (h >= 0 && h < g.H && w >= 0 && w < g.W) val = x[((b * g.C + c) * g.H + h) * g.W + w];
            if (e & 1) v[e >> 1] |= val << 16;
            else v[e >> 1] = val;
            if (++j == g.kw) { j = 0; if (++i == g.kh) { i = 0; ++c; } }
        }
        reinterpret_cast<uint4*>(cols)[t] = make_uint4(v[0], v[1], v[2], v[3]);
    }
}

__global__ void col2im_kernel(const uint16_t* __restrict__ dcolsT, uint16_t* __restrict__ dx, ConvGeom g) {
    const int32_t kk = g.kh * g.kw;
    const int64_t M = g.B * g.Ho * g.Wo;
    const int64_t total = g.B * g.C * g.H * g.W;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t w = t % g.W;
        const int64_t h = (t / g.W) % g.H;
        const int64_t c = (t / (g.W * g.H)) % g.C;
        const int64_t b = t / (g.W * g.H * g.C);
        float acc = 0.0f;
        for (int32_t i = 0; i < g.kh; ++i) {
            const int64_t hs = h + g.ph - i;           // = ho * sh
            if (hs < 0 || hs % g.sh) continue;
            const int64_t ho = hs / g.sh;
            if (ho >= g.Ho) continue;
            for (int32_t j = 0; j < g.kw; ++j) {
                const int64_t ws = w + g.pw - j;
                if (ws < 0 || ws % g.sw) continue;
                const int64_t wo = ws / g.sw;
                if (wo >= g.Wo) continue;
                const int64_t m = (b * g.Ho + ho) * g.Wo + wo;
                acc = acc + bf16_to_f32(dcolsT[(c * kk + i * g.kw + j) * M + m]);
            }
        }
        dx[t] = f32_to_bf16(acc);
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

static unsigned grid_for(int64_t total, int threads) {
    int64_t blocks = (total + threads - 1) / threads;
    const int64_t cap = 148LL * 16;   // grid-stride beyond 16 blocks per SM
    return (unsigned)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
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
    const int64_t total = B * g.Ho * g.Wo * (C * kh * kw / 8);
    if (total == 0) return CONCORD_OK;
    if (!x || !cols) return fail(CONCORD_EINVAL, "concord_im2col: null pointer");
    im2col_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(x, cols, g);
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
    col2im_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(dcols_t, dx, g);
    return check_launch("concord_col2im");
}
