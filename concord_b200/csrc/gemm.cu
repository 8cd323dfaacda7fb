// gemm.cu — the layer's dense GEMMs on B200 tensor cores (tcgen05 / TMEM / TMA).
//
// Replaces the cuBLAS calls of the reference layer (concord/packed_b.py:1219
// forward F.linear, 1263 dX = dY W, 1273 dW = dY^T X):
//   fwd: Y[M,N]  = X[M,K]  * W[N,K]^T       (A row-major,    B K-major)
//   dX : DX[M,K] = DY[M,N] * W[N,K]         (A row-major,    B N-major)
//   dW : DW[N,K] = DY[M,N]^T * X[M,K]       (A column-major, B row-major)
// bf16 operands, fp32 accumulation in tensor memory, bf16 result rounded to
// nearest even — the reference's numerics (its dW is rounded to bf16 before
// the optimizer reads it, packed_b.py:1274-1277).
//
// Each GEMM is a CUTLASS 4 sm100 warp-specialised kernel instantiated here:
// TMA producer warp -> shared-memory ring -> one thread issuing
// tcgen05.mma (cta_group::1, 128x256x64 tiles) into TMEM -> epilogue warps
// reading TMEM with tcgen05.ld and storing through TMA.  A dW whose N x K
// output has fewer tiles than the GPU has SMs splits its reduction into
// slices (a batched GEMM into fp32 partials, summed in slice order and
// rounded once to bf16).  Cluster shape 1x1x1:
// every TMA load is a single-CTA load (the same kernels run in multi-GPU jobs).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <string>

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

#include "../../include/concord_b200.h"

namespace concord {
int fail(int code, const std::string& msg);
int vhat_fold_partials(const float* rp, int64_t ldrp, const float* cp, int64_t ldcp, int64_t N, int64_t K,
                       float* v_row, float* v_col, float* sum_v_inv, float beta2, float one_minus_beta2,
                       int32_t* row_max, int32_t* col_max, int32_t* salt, unsigned* cnt, cudaStream_t st);

__global__ void splitk_reduce_kernel(const float4* __restrict__ part, uint2* __restrict__ out, int64_t n4, int S) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 a = part[i];
        for (int s = 1; s < S; ++s) {
            const float4 b = part[(int64_t)s * n4 + i];
            a.x = a.x + b.x; a.y = a.y + b.y; a.z = a.z + b.z; a.w = a.w + b.w;
        }
        const __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y);
        const __nv_bfloat162 hi = __floats2bfloat162_rn(a.z, a.w);
        out[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    }
}
// The TMA descriptors are encoded through the driver API, which needs a
// current context on the calling host thread.  A thread whose first CUDA work
// is this call (an autograd worker thread running a backward whose first node
// is this layer, for instance) may have none bound yet; encoding then fails
// and the kernel would run with an invalid descriptor.  When the thread has
// no current context, bind the current device's primary context first
// (cudaSetDevice of the device already current).  A thread with a context —
// always the case while a stream capture is running — makes no call that
// could implicitly synchronise.
typedef int (*CuCtxGetCurrentFn)(void**);

int bind_current_context(const char* name) {
    static CuCtxGetCurrentFn get_current = [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<CuCtxGetCurrentFn>(fn);
    }();
    if (get_current) {
        void* ctx = nullptr;
        if (get_current(&ctx) == 0 && ctx != nullptr) return CONCORD_OK;
    }
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);
    if (e != cudaSuccess)
        return concord::fail(CONCORD_ENODEVICE, std::string(name) + ": no usable CUDA device: " + cudaGetErrorString(e));
    return CONCORD_OK;
}

}  // namespace concord

namespace {
using concord::bind_current_context;

using namespace cute;

using BF16 = cutlass::bfloat16_t;
using Acc = float;
using TileMNK = Shape<_128, _256, _64>;
using Cluster = Shape<_1, _1, _1>;

using LayoutC = cutlass::layout::RowMajor;
constexpr int kAlign = 8;  // 16 bytes of bf16

using Epi = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TileMNK, Cluster,
    cutlass::epilogue::collective::EpilogueTileAuto, Acc, Acc, BF16, LayoutC, kAlign, BF16, LayoutC, kAlign,
    cutlass::epilogue::TmaWarpSpecialized1Sm>::CollectiveOp;
constexpr int kEpiSmem = static_cast<int>(sizeof(typename Epi::SharedStorage));

#define CONCORD_DEFINE_GEMM(NAME, LA, LB)                                                                    \
    using NAME##Main = typename cutlass::gemm::collective::CollectiveBuilder<                               \
        cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, BF16, LA, kAlign, BF16, LB, kAlign, Acc,    \
        TileMNK, Cluster, cutlass::gemm::collective::StageCountAutoCarveout<kEpiSmem>,                      \
        cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;                                    \
    using NAME##Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, NAME##Main, Epi, void>; \
    using NAME = cutlass::gemm::device::GemmUniversalAdapter<NAME##Kernel>;

CONCORD_DEFINE_GEMM(GemmFwd, cutlass::layout::RowMajor, cutlass::layout::ColumnMajor)
CONCORD_DEFINE_GEMM(GemmDx, cutlass::layout::RowMajor, cutlass::layout::RowMajor)
CONCORD_DEFINE_GEMM(GemmDw, cutlass::layout::ColumnMajor, cutlass::layout::RowMajor)

// dW split over the reduction (M) as a batch of S slices, fp32 partials
// [S, N, K]; splitk_reduce_kernel sums them in slice order and rounds once.
using EpiF32 = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TileMNK, Cluster,
    cutlass::epilogue::collective::EpilogueTileAuto, Acc, Acc, float, LayoutC, 4, float, LayoutC, 4,
    cutlass::epilogue::TmaWarpSpecialized1Sm>::CollectiveOp;
using GemmDwSplitMain = typename cutlass::gemm::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, BF16, cutlass::layout::ColumnMajor, kAlign, BF16,
    cutlass::layout::RowMajor, kAlign, Acc, TileMNK, Cluster,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename EpiF32::SharedStorage))>,
    cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;
using GemmDwSplitKernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, GemmDwSplitMain, EpiF32, void>;
using GemmDwSplit = cutlass::gemm::device::GemmUniversalAdapter<GemmDwSplitKernel>;

// dW with the v-hat partials in its epilogue.  The epilogue visitor tree
// (CUTLASS's sm90/sm100 EVT nodes) computes, per output element,
// v = float(bf16_rn(acc)) -- the stored dW value itself -- and s = v * v,
// stores bf16(v) (exact: v is already a bf16 value) as dW, and reduces s per
// 128 x 256 output tile into two fixed-order partial arrays in the workspace:
//   ColReduction (sum over the tile's 256 columns): row partial rp[slab][n]
//   RowReduction (sum over the tile's 128 rows):   column partial cp[rblk][k]
// (non-final reductions: each tile writes its own partial, no atomics), the
// same tiling and partial layout as vhat_kernel's tiles, so vhat's
// fixed-order fold turns them into v_row / v_col / sum_v_inv.  The
// in-tile summation order is CUTLASS's (register, then warp-shuffle, then
// shared-memory tree), deterministic but not vhat_kernel's order: the
// v-hat it yields agrees with the standalone kernel's to fp32 rounding, and
// the dW it stores is bit-identical to concord_gemm_dw's.
namespace vhfuse {
using namespace cutlass::epilogue::fusion;
constexpr auto RN = cutlass::FloatRoundStyle::round_to_nearest;

template <class T>
struct RoundBf16 {
    template <int N>
    CUTLASS_DEVICE cutlass::Array<float, N> operator()(cutlass::Array<float, N> const& a) const {
        cutlass::Array<float, N> r;
        CUTLASS_PRAGMA_UNROLL
        for (int i = 0; i < N; ++i) r[i] = __bfloat162float(__float2bfloat16_rn(a[i]));
        return r;
    }
};
template <class T>
struct SquareRn {   // one rounding per square: never contracted into the sum
    template <int N>
    CUTLASS_DEVICE cutlass::Array<float, N> operator()(cutlass::Array<float, N> const& a) const {
        cutlass::Array<float, N> r;
        CUTLASS_PRAGMA_UNROLL
        for (int i = 0; i < N; ++i) r[i] = __fmul_rn(a[i], a[i]);
        return r;
    }
};
template <class T>
struct TakeFirst {
    template <int N>
    CUTLASS_DEVICE cutlass::Array<float, N> operator()(cutlass::Array<float, N> const& a,
                                                       cutlass::Array<float, N> const&) const {
        return a;
    }
};

using Val = Sm90EVT<Sm90Compute<RoundBf16, float, float, RN>, Sm90AccFetch>;
using Sq = Sm90EVT<Sm90Compute<SquareRn, float, float, RN>, Val>;
using RowPart = Sm90ColReduction<cutlass::plus, cutlass::plus, cutlass::plus, 0, TileMNK, float, float, RN,
                                 Stride<_1, _0, _0>, 4, true, false, true>;
using ColPart = Sm90RowReduction<cutlass::plus, cutlass::plus, cutlass::plus, 0, TileMNK, float, float, RN,
                                 Stride<_0, _1, _0>, 4, true, false, true>;
using Parts = Sm90EVT<ColPart, Sm90EVT<RowPart, Sq>>;
using Root = Sm90EVT<Sm90Compute<TakeFirst, cutlass::bfloat16_t, float, RN>, Val, Parts>;   // dW out as bf16
}  // namespace vhfuse

using EpiVhat = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TileMNK, Cluster,
    cutlass::epilogue::collective::EpilogueTileAuto, Acc, Acc, void, LayoutC, kAlign, BF16, LayoutC, kAlign,
    cutlass::epilogue::TmaWarpSpecialized1Sm, vhfuse::Root>::CollectiveOp;
using GemmDwVhatMain = typename cutlass::gemm::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, BF16, cutlass::layout::ColumnMajor, kAlign, BF16,
    cutlass::layout::RowMajor, kAlign, Acc, TileMNK, Cluster,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename EpiVhat::SharedStorage))>,
    cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;
using GemmDwVhatKernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, GemmDwVhatMain, EpiVhat, void>;
using GemmDwVhat = cutlass::gemm::device::GemmUniversalAdapter<GemmDwVhatKernel>;

// Slices for dW[N,K] over a reduction of M: only when the N x K output has
// fewer 128x256 tiles than the GPU has SMs and each slice keeps >= 1024 rows
// (a multiple of 64); 1 means no split.
int dw_slices(int64_t M, int64_t N, int64_t K) {
    const int64_t tiles = ((N + 127) / 128) * ((K + 255) / 256);
    int S = 1;
    while (tiles * S * 2 <= 148 * 2 && M % (64 * S * 2) == 0 && M / (S * 2) >= 1024 && S < 16) S *= 2;
    return tiles >= 148 ? 1 : S;
}

// D[m,n] = sum_k A[m,k] B[k,n]; strides from the problem's layouts.
template <class Gemm, class ElemD = BF16>
int run_gemm(const void* A, const void* B, void* D, int M, int N, int K, void* workspace, size_t ws_bytes,
             cudaStream_t stream, bool query_only, size_t* ws_needed, const char* name, int L = 1) {
    using StrideA = typename Gemm::GemmKernel::StrideA;
    using StrideB = typename Gemm::GemmKernel::StrideB;
    using StrideC = typename Gemm::GemmKernel::StrideC;
    using StrideD = typename Gemm::GemmKernel::StrideD;
    StrideA sa = cutlass::make_cute_packed_stride(StrideA{}, cute::make_shape(M, K, L));
    StrideB sb = cutlass::make_cute_packed_stride(StrideB{}, cute::make_shape(N, K, L));
    StrideC sc = cutlass::make_cute_packed_stride(StrideC{}, cute::make_shape(M, N, L));
    StrideD sd = cutlass::make_cute_packed_stride(StrideD{}, cute::make_shape(M, N, L));
    typename Gemm::Arguments args{
        L == 1 ? cutlass::gemm::GemmUniversalMode::kGemm : cutlass::gemm::GemmUniversalMode::kBatched,
        {M, N, K, L},
        {reinterpret_cast<const BF16*>(A), sa, reinterpret_cast<const BF16*>(B), sb},
        {{1.0f, 0.0f}, reinterpret_cast<const ElemD*>(D), sc, reinterpret_cast<ElemD*>(D), sd}};
    // tile order of the persistent scheduler: swizzled groups of output tiles so
    // that concurrently resident CTAs share operand panels in L2
    static const int swz = [] {
        const char* e = getenv("CONCORD_GEMM_SWIZZLE");
        return e ? atoi(e) : 1;
    }();
    args.scheduler.max_swizzle_size = swz;
    // raster order of the output tiles: 0 CUTLASS's heuristic, 1 along M, 2 along N
    static const int raster = [] {
        const char* e = getenv("CONCORD_GEMM_RASTER");
        return e ? atoi(e) : 0;
    }();
    using RO = decltype(args.scheduler.raster_order);
    args.scheduler.raster_order = raster == 1 ? RO::AlongM : raster == 2 ? RO::AlongN : RO::Heuristic;
    Gemm gemm;
    if (query_only) {
        *ws_needed = Gemm::get_workspace_size(args);
        return CONCORD_OK;
    }
    if (gemm.can_implement(args) != cutlass::Status::kSuccess)
        return concord::fail(CONCORD_ESHAPE, std::string(name) + ": shape/alignment not supported "
                                             "(every extent must be a multiple of 8)");
    if (Gemm::get_workspace_size(args) > ws_bytes)
        return concord::fail(CONCORD_EWORKSPACE, std::string(name) + ": workspace too small");
    if (int rc = bind_current_context(name)) return rc;
    if (gemm.initialize(args, workspace, stream) != cutlass::Status::kSuccess)
        return concord::fail(CONCORD_ELAUNCH, std::string(name) + ": initialize failed");
    if (gemm.run(stream) != cutlass::Status::kSuccess)
        return concord::fail(CONCORD_ELAUNCH, std::string(name) + ": launch failed");
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return concord::fail(CONCORD_ELAUNCH, std::string(name) + ": " + cudaGetErrorString(e));
    return CONCORD_OK;
}

// dW[N,K] = DY^T X with the v-hat partials (GEMM m=N, n=K, k=M): rp receives
// [ceil(K/256)][round_up(N,128)] row partials, cp [ceil(N/128)][round_up(K,256)]
// column partials (fp32 sums of the squared bf16 outputs per tile)
int run_gemm_dw_vhat(const void* dy, const void* x, void* dw, int N, int K, int M, float* rp, float* cp,
                     void* workspace, size_t ws_bytes, cudaStream_t stream, bool query_only, size_t* ws_needed) {
    using Gemm = GemmDwVhat;
    using StrideA = typename Gemm::GemmKernel::StrideA;
    using StrideB = typename Gemm::GemmKernel::StrideB;
    using StrideC = typename Gemm::GemmKernel::StrideC;
    using StrideD = typename Gemm::GemmKernel::StrideD;
    StrideA sa = cutlass::make_cute_packed_stride(StrideA{}, cute::make_shape(N, M, 1));
    StrideB sb = cutlass::make_cute_packed_stride(StrideB{}, cute::make_shape(K, M, 1));
    StrideC sc = cutlass::make_cute_packed_stride(StrideC{}, cute::make_shape(N, K, 1));
    StrideD sd = cutlass::make_cute_packed_stride(StrideD{}, cute::make_shape(N, K, 1));
    using RowPartArgs = typename vhfuse::RowPart::Arguments;
    using ColPartArgs = typename vhfuse::ColPart::Arguments;
    typename Gemm::Arguments args{
        cutlass::gemm::GemmUniversalMode::kGemm,
        {N, K, M, 1},
        {reinterpret_cast<const BF16*>(dy), sa, reinterpret_cast<const BF16*>(x), sb},
        {{{{}, {}},                                                         // v = bf16(acc)
          {{{{{}, {}}, {}}, RowPartArgs{rp, 0.0f, {}}}, ColPartArgs{cp, 0.0f, {}}},  // partials of v*v
          {}},
         nullptr, sc, reinterpret_cast<BF16*>(dw), sd}};
    static const int swz = [] {
        const char* e = getenv("CONCORD_GEMM_SWIZZLE");
        return e ? atoi(e) : 1;
    }();
    args.scheduler.max_swizzle_size = swz;
    Gemm gemm;
    if (query_only) {
        *ws_needed = Gemm::get_workspace_size(args);
        return CONCORD_OK;
    }
    const char* name = "concord_gemm_dw_vhat";
    if (gemm.can_implement(args) != cutlass::Status::kSuccess)
        return concord::fail(CONCORD_ESHAPE, std::string(name) + ": shape/alignment not supported "
                                             "(every extent must be a multiple of 8)");
    if (Gemm::get_workspace_size(args) > ws_bytes)
        return concord::fail(CONCORD_EWORKSPACE, std::string(name) + ": workspace too small");
    if (int rc = bind_current_context(name)) return rc;
    if (gemm.initialize(args, workspace, stream) != cutlass::Status::kSuccess)
        return concord::fail(CONCORD_ELAUNCH, std::string(name) + ": initialize failed");
    if (gemm.run(stream) != cutlass::Status::kSuccess)
        return concord::fail(CONCORD_ELAUNCH, std::string(name) + ": launch failed");
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return concord::fail(CONCORD_ELAUNCH, std::string(name) + ": " + cudaGetErrorString(e));
    return CONCORD_OK;
}

bool bad(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % 16) != 0; }

// which kernels the plain GEMM entry points run: CONCORD_GEMM_2SM (the
// package's own 2-SM kernel, gemm2sm.cu; default) or CONCORD_GEMM_CUTLASS
// (the CUTLASS 1-SM kernels above).  CONCORD_GEMM_IMPL=cutlass in the
// environment changes the default.
std::atomic<int> g_impl{-1};
int gemm_impl() {
    int v = g_impl.load();
    if (v < 0) {
        const char* e = getenv("CONCORD_GEMM_IMPL");
        v = (e && std::string(e) == "cutlass") ? CONCORD_GEMM_CUTLASS : CONCORD_GEMM_2SM;
        int expect = -1;
        g_impl.compare_exchange_strong(expect, v);
        v = g_impl.load();
    }
    return v;
}

}  // namespace

namespace concord {
int gemm2sm(const void* A, int a_mn, int64_t lda, const void* B, int b_mn, int64_t ldb, void* D, int64_t ldd,
            int64_t M, int64_t N, int64_t K, cudaStream_t stream, const char* name, float* rp = nullptr,
            int64_t ldrp = 0, float* cp = nullptr, int64_t ldcp = 0);
}

extern "C" int concord_gemm_set_impl(int32_t impl) {
    if (impl != CONCORD_GEMM_2SM && impl != CONCORD_GEMM_CUTLASS)
        return concord::fail(CONCORD_EINVAL, "concord_gemm_set_impl: impl must be CONCORD_GEMM_2SM or CONCORD_GEMM_CUTLASS");
    g_impl.store(impl);
    return CONCORD_OK;
}

extern "C" int concord_gemm_get_impl(void) { return gemm_impl(); }

// Y[M,N] = X[M,K] W[N,K]^T
extern "C" int concord_gemm_fwd(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t M, int64_t N, int64_t K,
                                void* workspace, size_t workspace_bytes, void* stream) {
    if (bad(x) || bad(w) || bad(y)) return concord::fail(CONCORD_EALIGN, "concord_gemm_fwd: null or unaligned pointer");
    if (M <= 0 || N <= 0 || K <= 0) return concord::fail(CONCORD_ESHAPE, "concord_gemm_fwd: bad shape");
    if (gemm_impl() == CONCORD_GEMM_2SM)      // x K-major [M,K], w K-major [N,K]
        return concord::gemm2sm(x, 0, K, w, 0, K, y, N, M, N, K, reinterpret_cast<cudaStream_t>(stream),
                                "concord_gemm_fwd");
    return run_gemm<GemmFwd>(x, w, y, (int)M, (int)N, (int)K, workspace, workspace_bytes,
                             reinterpret_cast<cudaStream_t>(stream), false, nullptr, "concord_gemm_fwd");
}

// DX[M,K] = DY[M,N] W[N,K]   (GEMM m=M, n=K, k=N)
extern "C" int concord_gemm_dx(const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t M, int64_t N, int64_t K,
                               void* workspace, size_t workspace_bytes, void* stream) {
    if (bad(dy) || bad(w) || bad(dx)) return concord::fail(CONCORD_EALIGN, "concord_gemm_dx: null or unaligned pointer");
    if (M <= 0 || N <= 0 || K <= 0) return concord::fail(CONCORD_ESHAPE, "concord_gemm_dx: bad shape");
    if (gemm_impl() == CONCORD_GEMM_2SM)      // dy K-major [M,N], w MN-major ([N,K]: k=N rows, n=K contiguous)
        return concord::gemm2sm(dy, 0, N, w, 1, K, dx, K, M, K, N, reinterpret_cast<cudaStream_t>(stream),
                                "concord_gemm_dx");
    return run_gemm<GemmDx>(dy, w, dx, (int)M, (int)K, (int)N, workspace, workspace_bytes,
                            reinterpret_cast<cudaStream_t>(stream), false, nullptr, "concord_gemm_dx");
}

// DW[N,K] = DY[M,N]^T X[M,K]   (GEMM m=N, n=K, k=M)
extern "C" int concord_gemm_dw(const uint16_t* dy, const uint16_t* x, uint16_t* dw, int64_t M, int64_t N, int64_t K,
                               void* workspace, size_t workspace_bytes, void* stream) {
    if (bad(dy) || bad(x) || bad(dw)) return concord::fail(CONCORD_EALIGN, "concord_gemm_dw: null or unaligned pointer");
    if (M <= 0 || N <= 0 || K <= 0) return concord::fail(CONCORD_ESHAPE, "concord_gemm_dw: bad shape");
    const int S = dw_slices(M, N, K);
    if (S == 1 && gemm_impl() == CONCORD_GEMM_2SM)   // dy MN-major ([M,N]: k=M rows), x MN-major ([M,K])
        return concord::gemm2sm(dy, 1, N, x, 1, K, dw, K, N, K, M, reinterpret_cast<cudaStream_t>(stream),
                                "concord_gemm_dw");
    if (S == 1)
        return run_gemm<GemmDw>(dy, x, dw, (int)N, (int)K, (int)M, workspace, workspace_bytes,
                                reinterpret_cast<cudaStream_t>(stream), false, nullptr, "concord_gemm_dw");
    // split-K: slice s reduces rows [s*M/S, (s+1)*M/S) into fp32 partial s at
    // the start of the workspace; CUTLASS's own workspace follows it
    const size_t part = (size_t)S * (size_t)N * (size_t)K * sizeof(float);
    if (workspace_bytes < part || (reinterpret_cast<uintptr_t>(workspace) % 16) != 0)
        return concord::fail(CONCORD_EWORKSPACE, "concord_gemm_dw: workspace too small for the split reduction");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int rc = run_gemm<GemmDwSplit, float>(dy, x, workspace, (int)N, (int)K, (int)(M / S),
                                          static_cast<char*>(workspace) + part, workspace_bytes - part, st, false,
                                          nullptr, "concord_gemm_dw", S);
    if (rc) return rc;
    const int64_t n4 = N * K / 4;
    concord::splitk_reduce_kernel<<<(unsigned)std::min<int64_t>((n4 + 255) / 256, 148 * 8), 256, 0, st>>>(
        static_cast<const float4*>(workspace), reinterpret_cast<uint2*>(dw), n4, S);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return concord::fail(CONCORD_ELAUNCH, std::string("concord_gemm_dw: ") + cudaGetErrorString(e));
    return CONCORD_OK;
}

extern "C" size_t concord_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    size_t a = 0, b = 0, c = 0;
    run_gemm<GemmFwd>(nullptr, nullptr, nullptr, (int)M, (int)N, (int)K, nullptr, 0, nullptr, true, &a, "");
    run_gemm<GemmDx>(nullptr, nullptr, nullptr, (int)M, (int)K, (int)N, nullptr, 0, nullptr, true, &b, "");
    run_gemm<GemmDw>(nullptr, nullptr, nullptr, (int)N, (int)K, (int)M, nullptr, 0, nullptr, true, &c, "");
    const int S = dw_slices(M, N, K);
    if (S > 1) {
        size_t d = 0;
        run_gemm<GemmDwSplit, float>(nullptr, nullptr, nullptr, (int)N, (int)K, (int)(M / S), nullptr, 0, nullptr,
                                     true, &d, "", S);
        c = std::max(c, (size_t)S * (size_t)N * (size_t)K * sizeof(float) + d);
    }
    return std::max(a, std::max(b, c));
}

// ---- dW with the v-hat update (the partials in the dW epilogue) ----
namespace {
struct DwVhatLayout {
    int64_t ldrp, ldcp;      // partial strides: N and K rounded up to the tile
    size_t off_rp, off_cp, off_gemm, total;
};
DwVhatLayout dw_vhat_layout(int64_t M, int64_t N, int64_t K) {
    DwVhatLayout L;
    const int64_t ncs = (K + 255) / 256, nrb = (N + 127) / 128;
    L.ldrp = nrb * 128;
    L.ldcp = ncs * 256;
    L.off_rp = 256;   // the fold's arrival counter first
    L.off_cp = L.off_rp + ((size_t)ncs * (size_t)L.ldrp * sizeof(float) + 255) / 256 * 256;
    L.off_gemm = L.off_cp + ((size_t)nrb * (size_t)L.ldcp * sizeof(float) + 255) / 256 * 256;
    size_t g = 0;
    run_gemm_dw_vhat(nullptr, nullptr, nullptr, (int)N, (int)K, (int)M, nullptr, nullptr, nullptr, 0, nullptr, true, &g);
    L.total = L.off_gemm + g;
    return L;
}
}  // namespace

// the epilogue form runs where the dW GEMM fills the GPU with whole output
// tiles (>= 148 tiles of 128 x 256, never split); smaller layers take the
// two-launch path, whose v-hat order the CPU oracle restates
bool dw_vhat_fused(int64_t M, int64_t N, int64_t K) {
    return ((N + 127) / 128) * ((K + 255) / 256) >= 148 && dw_slices(M, N, K) == 1;
}

extern "C" size_t concord_gemm_dw_vhat_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    if (!dw_vhat_fused(M, N, K)) {
        const size_t v = (concord_vhat_workspace_bytes(N, K) + 255) / 256 * 256;
        return v + concord_gemm_workspace_bytes(M, N, K);
    }
    return dw_vhat_layout(M, N, K).total;
}

// dW = DY^T X (bf16, as concord_gemm_dw) followed by the v-hat update of
// concord_vhat_update on it.  On a layer of >= 148 output tiles the squares'
// tile partials come out of the GEMM's epilogue and one fold launch
// finishes; smaller layers run concord_gemm_dw then concord_vhat_update.
extern "C" int concord_gemm_dw_vhat(const uint16_t* dy, const uint16_t* x, uint16_t* dw, int64_t M, int64_t N,
                                    int64_t K, float* v_row, float* v_col, float* sum_v_inv, float beta2,
                                    float one_minus_beta2, int32_t* row_max, int32_t* col_max, int32_t* salt,
                                    void* workspace, size_t workspace_bytes, void* stream) {
    const char* name = "concord_gemm_dw_vhat";
    if (bad(dy) || bad(x) || bad(dw) || bad(workspace))
        return concord::fail(CONCORD_EALIGN, std::string(name) + ": null or unaligned pointer");
    if (!v_row || !v_col || !sum_v_inv) return concord::fail(CONCORD_EINVAL, std::string(name) + ": null v-hat pointer");
    if (M <= 0 || N <= 0 || K <= 0) return concord::fail(CONCORD_ESHAPE, std::string(name) + ": bad shape");
    if (workspace_bytes < concord_gemm_dw_vhat_workspace_bytes(M, N, K))
        return concord::fail(CONCORD_EWORKSPACE, std::string(name) + ": workspace smaller than "
                                                 "concord_gemm_dw_vhat_workspace_bytes(M, N, K)");
    char* ws = static_cast<char*>(workspace);
    if (!dw_vhat_fused(M, N, K)) {
        const size_t v = (concord_vhat_workspace_bytes(N, K) + 255) / 256 * 256;
        if (int rc = concord_gemm_dw(dy, x, dw, M, N, K, ws + v, workspace_bytes - v, stream)) return rc;
        return concord_vhat_update(dw, K, N, K, v_row, v_col, sum_v_inv, beta2, one_minus_beta2, row_max, col_max,
                                   salt, ws, v, stream);
    }
    const DwVhatLayout L = dw_vhat_layout(M, N, K);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    float* rp = reinterpret_cast<float*>(ws + L.off_rp);
    float* cp = reinterpret_cast<float*>(ws + L.off_cp);
    if (gemm_impl() == CONCORD_GEMM_2SM) {
        // the package's 2-SM dW (dy MN-major, x MN-major) with the partials in its epilogue
        if (int rc = concord::gemm2sm(dy, 1, N, x, 1, K, dw, K, N, K, M, st, name, rp, L.ldrp, cp, L.ldcp)) return rc;
    } else if (int rc = run_gemm_dw_vhat(dy, x, dw, (int)N, (int)K, (int)M, rp, cp, ws + L.off_gemm,
                                  workspace_bytes - L.off_gemm, st, false, nullptr))
        return rc;
    return concord::vhat_fold_partials(rp, L.ldrp, cp, L.ldcp, N, K, v_row, v_col, sum_v_inv, beta2,
                                       one_minus_beta2, row_max, col_max, salt, reinterpret_cast<unsigned*>(ws), st);
}
