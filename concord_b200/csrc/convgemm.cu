// convgemm.cu — implicit-GEMM convolutions for ConcordConv2dPackedB on B200.
//
// Replaces the three cuDNN calls of the reference's conv layer
// (concord/packed_b.py:1890 F.conv2d forward, 1939-1947
// torch.nn.grad.conv2d_input / conv2d_weight in the backward) for bf16
// tensors in NHWC order (torch's channels_last), fp32 accumulation, one
// round-to-nearest-even to bf16 per output element:
//   fprop: y[B,Ho,Wo,O]  = conv(x[B,H,W,C], w[O,kh,kw,C])
//   dgrad: dx[B,H,W,C]   = conv_transpose(dy[B,Ho,Wo,O], w)     (stride 1)
//   wgrad: dw[O,kh,kw,C] = sum over B,Ho,Wo of dy (x) x-patches
// No column matrix is built: the activation operand is fetched by TMA in
// im2col mode straight from the NHWC tensor (the tile's pixels and their
// kh x kw neighbourhoods, padding read as zeros), fed to tcgen05.mma through
// a shared-memory ring, accumulated in TMEM and stored by the epilogue warps.
// These are CUTLASS 4's sm100 implicit-GEMM conv collectives, instantiated
// here with a 1x1x1 cluster: every TMA load is a single-CTA load, so the
// same kernels run in multi-GPU jobs.  wgrad reduces over B*Ho*Wo (tens of
// thousands of rows) into a small O x kh*kw*C output; it splits that
// reduction over the SMs (split-K with a deterministic, split-ordered fixup)
// when the output has fewer tiles than the GPU has SMs.
#include <cuda_runtime.h>

#include <stdlib.h>

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/kernel_hardware_info.hpp"
#include "cutlass/conv/collective/collective_builder.hpp"
#include "cutlass/conv/convnd_problem_shape.hpp"
#include "cutlass/conv/device/conv_universal_adapter.hpp"
#include "cutlass/conv/dispatch_policy.hpp"
#include "cutlass/conv/kernel/conv_universal.hpp"
#include "cutlass/epilogue/collective/collective_builder.hpp"

#include "../../include/concord_b200.h"

namespace concord {
int fail(int code, const std::string& msg);
int bind_current_context(const char* name);
}  // namespace concord

namespace {

using namespace cute;

using BF16 = cutlass::bfloat16_t;
using Acc = float;
using ConvTile = Shape<_128, Shape<_128>, Shape<_64>>;
using ConvCluster = Shape<_1, _1, _1>;
constexpr int kAlign = 8;   // 16 bytes of bf16

// The epilogue sees the output in its conv modes: fprop / dgrad write an
// NHWC activation, GEMM modes ((W, H, N), C); wgrad writes the KRSC filter,
// GEMM modes (K, (C, S, R)).
template <cutlass::conv::Operator Op, class Sched>
struct ConvKernels {
    using OutLayout = cute::conditional_t<Op == cutlass::conv::Operator::kWgrad, cutlass::layout::TensorKCSR,
                                          cutlass::layout::TensorNHWC>;
    using Epi = typename cutlass::epilogue::collective::CollectiveBuilder<
        cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, ConvTile, ConvCluster,
        cutlass::epilogue::collective::EpilogueTileAuto, Acc, Acc, BF16, OutLayout, kAlign, BF16, OutLayout,
        kAlign, cutlass::epilogue::TmaWarpSpecialized1Sm>::CollectiveOp;
    using Main = typename cutlass::conv::collective::CollectiveBuilder<
        cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, Op, BF16, cutlass::layout::TensorNHWC, kAlign,
        BF16, cutlass::layout::TensorNHWC, kAlign, Acc, ConvTile, ConvCluster,
        cutlass::conv::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epi::SharedStorage))>,
        cutlass::conv::KernelImplicitTmaWarpSpecialized1SmSm100>::CollectiveOp;
    using Problem = cutlass::conv::ConvProblemShape<Op, Main::DispatchPolicy::NumSpatialDimensions>;
    using Kernel = cutlass::conv::kernel::ConvUniversal<Problem, Main, Epi, Sched>;
    using Conv = cutlass::conv::device::ConvUniversalAdapter<Kernel>;
};

using Fprop = ConvKernels<cutlass::conv::Operator::kFprop, void>::Conv;
using Dgrad = ConvKernels<cutlass::conv::Operator::kDgrad, void>::Conv;
using Wgrad = ConvKernels<cutlass::conv::Operator::kWgrad, cutlass::gemm::StreamKScheduler>::Conv;

struct Geom {
    int B, H, W, C, O, kh, kw, sh, sw, ph, pw, Ho, Wo;
};

int check_geom(const Geom& g, const char* name) {
    if (g.B <= 0 || g.H <= 0 || g.W <= 0 || g.C <= 0 || g.O <= 0 || g.kh <= 0 || g.kw <= 0 || g.sh <= 0 ||
        g.sw <= 0 || g.ph < 0 || g.pw < 0)
        return concord::fail(CONCORD_EINVAL, std::string(name) + ": bad geometry");
    if (g.Ho <= 0 || g.Wo <= 0) return concord::fail(CONCORD_ESHAPE, std::string(name) + ": empty output");
    if (g.C % 8 || g.O % 8)
        return concord::fail(CONCORD_ESHAPE, std::string(name) + ": channel counts must be multiples of 8");
    return CONCORD_OK;
}

// output tiles of the wgrad GEMM (O x kh*kw*C) and the split of its reduction
int wgrad_splits(const Geom& g) {
    const int64_t tiles = ((g.O + 127) / 128) * (((int64_t)g.kh * g.kw * g.C + 127) / 128);
    const int64_t red = (int64_t)g.B * g.Ho * g.Wo;
    int S = 1;
    while (tiles * S * 2 <= 148 && red / (S * 2) >= 2048 && S < 16) S *= 2;
    return S;
}

template <class Conv>
int run_conv(const Geom& g, const void* a, const void* b, void* d, void* ws, size_t ws_bytes, cudaStream_t st,
             bool query, size_t* need, const char* name) {
    using Problem = typename Conv::ConvKernel::ProblemShape;
    constexpr auto Op = Problem::ConvOp;
    Problem shape(cutlass::conv::Mode::kCrossCorrelation, {g.B, g.H, g.W, g.C}, {g.O, g.kh, g.kw, g.C},
                  {g.ph, g.pw}, {g.ph, g.pw}, {g.sh, g.sw}, {1, 1}, 1);
    // packed output strides in the epilogue's modes
    using StrideD = typename Conv::ConvKernel::StrideD;
    StrideD so{};
    if constexpr (Op == cutlass::conv::Operator::kWgrad) {          // (K, (C, S, R)) of [O, kh, kw, C]
        get<0>(so) = (int64_t)g.kh * g.kw * g.C;
        get<1, 1>(so) = g.C;
        get<1, 2>(so) = (int64_t)g.kw * g.C;
    } else {                                                         // ((W, H, N), C) of [N, H, W, C]
        const int64_t c = Op == cutlass::conv::Operator::kFprop ? g.O : g.C;
        const int64_t w = Op == cutlass::conv::Operator::kFprop ? g.Wo : g.W;
        const int64_t h = Op == cutlass::conv::Operator::kFprop ? g.Ho : g.H;
        get<0, 0>(so) = c;
        get<0, 1>(so) = w * c;
        get<0, 2>(so) = h * w * c;
    }
    typename Conv::Arguments args{
        shape,
        {reinterpret_cast<const BF16*>(a), reinterpret_cast<const BF16*>(b)},
        {{1.0f, 0.0f}, reinterpret_cast<const BF16*>(d), so, reinterpret_cast<BF16*>(d), so}};
    if constexpr (Op == cutlass::conv::Operator::kWgrad) {
        using Mode = decltype(args.scheduler.decomposition_mode);
        using Red = decltype(args.scheduler.reduction_mode);
        const int S = wgrad_splits(g);
        args.scheduler.splits = S;
        args.scheduler.decomposition_mode = S > 1 ? Mode::SplitK : Mode::DataParallel;
        args.scheduler.reduction_mode = Red::Deterministic;
    }
    if (query) {
        *need = Conv::get_workspace_size(args);
        return CONCORD_OK;
    }
    Conv conv;
    if (conv.can_implement(args) != cutlass::Status::kSuccess)
        return concord::fail(CONCORD_ESHAPE, std::string(name) + ": convolution not supported by the implicit GEMM");
    if (Conv::get_workspace_size(args) > ws_bytes)
        return concord::fail(CONCORD_EWORKSPACE, std::string(name) + ": workspace too small");
    if (int rc = concord::bind_current_context(name)) return rc;
    if (conv.initialize(args, ws, st) != cutlass::Status::kSuccess)
        return concord::fail(CONCORD_ELAUNCH, std::string(name) + ": initialize failed");
    if (conv.run(st) != cutlass::Status::kSuccess)
        return concord::fail(CONCORD_ELAUNCH, std::string(name) + ": launch failed");
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return concord::fail(CONCORD_ELAUNCH, std::string(name) + ": " + cudaGetErrorString(e));
    return CONCORD_OK;
}

Geom geom(int64_t B, int64_t H, int64_t W, int64_t C, int64_t O, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
          int64_t ph, int64_t pw) {
    Geom g{(int)B, (int)H, (int)W, (int)C, (int)O, (int)kh, (int)kw, (int)sh, (int)sw, (int)ph, (int)pw, 0, 0};
    if (sh > 0 && sw > 0) {
        g.Ho = (int)((H + 2 * ph - kh) >= 0 ? (H + 2 * ph - kh) / sh + 1 : 0);
        g.Wo = (int)((W + 2 * pw - kw) >= 0 ? (W + 2 * pw - kw) / sw + 1 : 0);
    }
    return g;
}

bool fits_int(int64_t B, int64_t H, int64_t W, int64_t C, int64_t O, int64_t kh, int64_t kw) {
    const int64_t lim = (int64_t)1 << 31;
    return B < lim && H < lim && W < lim && C < lim && O < lim && kh < lim && kw < lim &&
           B * H * W * C < lim * 64 && O * kh * kw * C < lim;
}

}  // namespace

extern "C" size_t concord_conv_nhwc_workspace_bytes(int op, int64_t B, int64_t H, int64_t W, int64_t C, int64_t O,
                                                    int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                                                    int64_t pw) {
    if (!fits_int(B, H, W, C, O, kh, kw)) return 0;
    const Geom g = geom(B, H, W, C, O, kh, kw, sh, sw, ph, pw);
    if (g.Ho <= 0 || g.Wo <= 0) return 0;
    size_t need = 0;
    const char* n = "concord_conv_nhwc_workspace_bytes";
    if (op == CONCORD_CONV_FPROP) run_conv<Fprop>(g, nullptr, nullptr, nullptr, nullptr, 0, nullptr, true, &need, n);
    else if (op == CONCORD_CONV_DGRAD) run_conv<Dgrad>(g, nullptr, nullptr, nullptr, nullptr, 0, nullptr, true, &need, n);
    else if (op == CONCORD_CONV_WGRAD) run_conv<Wgrad>(g, nullptr, nullptr, nullptr, nullptr, 0, nullptr, true, &need, n);
    return (need + 255) / 256 * 256;
}

static int conv_entry(int op, const uint16_t* a, const uint16_t* b, uint16_t* d, int64_t B, int64_t H, int64_t W,
                      int64_t C, int64_t O, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                      void* ws, size_t ws_bytes, void* stream, const char* name) {
    if (!a || !b || !d) return concord::fail(CONCORD_EINVAL, std::string(name) + ": null pointer");
    if (!fits_int(B, H, W, C, O, kh, kw)) return concord::fail(CONCORD_ETOOBIG, std::string(name) + ": extents too large");
    const Geom g = geom(B, H, W, C, O, kh, kw, sh, sw, ph, pw);
    if (int rc = check_geom(g, name)) return rc;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(d)) % 16)
        return concord::fail(CONCORD_EALIGN, std::string(name) + ": tensors must be 16-byte aligned");
    if (op == CONCORD_CONV_DGRAD && (sh != 1 || sw != 1))
        return concord::fail(CONCORD_ESHAPE, std::string(name) + ": dgrad supports stride 1 only");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    size_t unused = 0;
    if (op == CONCORD_CONV_FPROP) return run_conv<Fprop>(g, a, b, d, ws, ws_bytes, st, false, &unused, name);
    if (op == CONCORD_CONV_DGRAD) return run_conv<Dgrad>(g, a, b, d, ws, ws_bytes, st, false, &unused, name);
    return run_conv<Wgrad>(g, a, b, d, ws, ws_bytes, st, false, &unused, name);
}

extern "C" int concord_conv_fprop_nhwc(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t B, int64_t H,
                                       int64_t W, int64_t C, int64_t O, int64_t kh, int64_t kw, int64_t sh,
                                       int64_t sw, int64_t ph, int64_t pw, void* workspace, size_t workspace_bytes,
                                       void* stream) {
    return conv_entry(CONCORD_CONV_FPROP, x, w, y, B, H, W, C, O, kh, kw, sh, sw, ph, pw, workspace,
                      workspace_bytes, stream, "concord_conv_fprop_nhwc");
}

extern "C" int concord_conv_dgrad_nhwc(const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t B, int64_t H,
                                       int64_t W, int64_t C, int64_t O, int64_t kh, int64_t kw, int64_t sh,
                                       int64_t sw, int64_t ph, int64_t pw, void* workspace, size_t workspace_bytes,
                                       void* stream) {
    return conv_entry(CONCORD_CONV_DGRAD, dy, w, dx, B, H, W, C, O, kh, kw, sh, sw, ph, pw, workspace,
                      workspace_bytes, stream, "concord_conv_dgrad_nhwc");
}

extern "C" int concord_conv_wgrad_nhwc(const uint16_t* dy, const uint16_t* x, uint16_t* dw, int64_t B, int64_t H,
                                       int64_t W, int64_t C, int64_t O, int64_t kh, int64_t kw, int64_t sh,
                                       int64_t sw, int64_t ph, int64_t pw, void* workspace, size_t workspace_bytes,
                                       void* stream) {
    return conv_entry(CONCORD_CONV_WGRAD, dy, x, dw, B, H, W, C, O, kh, kw, sh, sw, ph, pw, workspace,
                      workspace_bytes, stream, "concord_conv_wgrad_nhwc");
}
