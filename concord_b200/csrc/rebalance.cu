// rebalance.cu — exponent ratchet (K3) and its gated "anything to do?" check.
//
// Replaces ConcordLinearPackedB.rebalance + rebalance_packed +
// _rebalance_packed_decide_kernel (concord/packed_b.py:1792-1814,
// 1129-1190, 959-1095).  Three launches, none of which waits on another
// block:
//   1. (allow_tickdown only) per-row / per-column histograms of
//      max(|s_slow|,|v_slow|) (0..128) -> exact lower medians, which the
//      reference gets from torch.median (packed_b.py:1156-1160);
//   2. decide: fold row/col max into the high-watermarks, bump the seed,
//      compute each row's and column's tick in {-1,0,+1} from the PRE-launch
//      exponents, write the new exponents, raise a "fired" flag;
//   3. shift: returns at once unless fired; otherwise SR-right-shifts (or
//      left-shifts) only the words whose row+column tick is non-zero, with
//      Philox4x32-10 uniforms at offsets n*K+k + {0, NK, 2NK} (tl.rand).
// Deciding from pre-launch exponents removes a read/write race of the
// reference kernel, in which a program can read an exponent that the
// pid_k==0 program already incremented (it only matters at 6 -> 7).
#include "common.cuh"

namespace concord {

constexpr int RB_THREADS = 256;
constexpr int HB = 129;  // histogram bins 0..128

struct RebArgs {
    int32_t* packed; int64_t ldp;
    int8_t* row_exp; int8_t* col_exp;
    const int32_t* row_max; const int32_t* col_max;
    int32_t* row_hwm; int32_t* col_hwm;
    int32_t* seed;
    int32_t max_m, exp_max, exp_min, allow_td;
    int64_t N, K, row0, N_total;
    int32_t* fired_out;
    int8_t* rt; int8_t* ct; int32_t* fired;   // fired[0] flag, [1] #rows, [2] #cols ticked
    int32_t* rhist; int32_t* chist;
    int32_t* rowlist; int32_t* collist;       // rows / columns whose exponent moved
};

__global__ void reb_hist_kernel(RebArgs A) {
    const int64_t total = A.N * A.K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / A.K, k = i - n * A.K;
        const int32_t w = A.packed[n * A.ldp + k];
        const int32_t ss = abs(shl32(w, 16) >> 24), vs = abs(shl32(w, 24) >> 24);
        const int32_t m = max(ss, vs);
        atomicAdd(A.rhist + n * HB + m, 1);
        atomicAdd(A.chist + k * HB + m, 1);
    }
}

// lower median (torch.median) from a histogram; re-zeroes the bins it read
__device__ int32_t median_and_clear(int32_t* h, int64_t count) {
    const int64_t target = (count - 1) / 2 + 1;
    int64_t run = 0;
    int32_t med = 128;
    bool found = false;
    for (int v = 0; v < HB; ++v) {
        run += h[v];
        if (!found && run >= target) { med = v; found = true; }
        h[v] = 0;
    }
    return med;
}

__global__ void reb_decide_kernel(RebArgs A) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) *A.seed += 1;
    if (i < A.N) {
        const int64_t n = i;
        const int32_t mx = A.row_max[n];
        if (A.row_hwm) A.row_hwm[n] = max(A.row_hwm[n], mx);
        const int32_t e = A.row_exp[n];
        int up = mx > A.max_m && e < A.exp_max;
        int dn = 0;
        if (A.allow_td) {
            int32_t med = median_and_clear(A.rhist + n * HB, A.K);
            dn = mx <= A.max_m && med <= 31 && e > A.exp_min;
        }
        const int t = up - dn;
        A.rt[n] = (int8_t)t;
        if (t) {
            A.row_exp[n] = (int8_t)(e + t);
            atomicOr(A.fired, 1);
            A.rowlist[atomicAdd(A.fired + 1, 1)] = (int32_t)n;
        }
    } else if (i < A.N + A.K) {
        const int64_t k = i - A.N;
        const int32_t mx = A.col_max[k];
        if (A.col_hwm) A.col_hwm[k] = max(A.col_hwm[k], mx);
        const int32_t e = A.col_exp[k];
        int up = mx > A.max_m && e < A.exp_max;
        int dn = 0;
        if (A.allow_td) {
            int32_t med = median_and_clear(A.chist + k * HB, A.N);
            dn = mx <= A.max_m && med <= 31 && e > A.exp_min;
        }
        const int t = up - dn;
        A.ct[k] = (int8_t)t;
        if (t) {
            A.col_exp[k] = (int8_t)(e + t);
            atomicOr(A.fired, 1);
            A.collist[atomicAdd(A.fired + 2, 1)] = (int32_t)k;
        }
    }
}

__device__ __forceinline__ void reb_shift_word(const RebArgs& A, int64_t n, int64_t k, int32_t sd, uint32_t NK) {
    const int32_t net = (int32_t)A.rt[n] + (int32_t)A.ct[k];
    if (net == 0) return;
    int32_t* pw = A.packed + n * A.ldp + k;
    const int32_t w = *pw;
    const int32_t sf = w >> 16, ss = shl32(w, 16) >> 24, vs = shl32(w, 24) >> 24;
    int32_t nsf, nss, nvs;
    if (net < 0) {
        const int l = -net;
        nsf = shl32(sf, l); nss = shl32(ss, l); nvs = shl32(vs, l);
    } else {
        const int rsh = net;
        const uint32_t off = (uint32_t)((A.row0 + n) * A.K + k);
        const float two_pos = exp2i(rsh);
        const int32_t q = sf >> rsh;
        const float rem = (float)(sf - shl32(q, rsh));
        const int32_t sfs = q + (__fmul_rn(tl_rand(sd, off), two_pos) < rem ? 1 : 0);
        const int32_t qs = ss >> rsh;
        const float rems = (float)(ss - shl32(qs, rsh));
        const int32_t ssu = qs + (__fmul_rn(tl_rand(sd, off + NK), two_pos) < rems ? 1 : 0);
        const int32_t sres = shl32(ss, 7 - rsh) - shl32(ssu, 7);
        const int32_t qv = vs >> rsh;
        const float remv = (float)(vs - shl32(qv, rsh));
        const int32_t vu = qv + (__fmul_rn(tl_rand(sd, off + 2u * NK), two_pos) < remv ? 1 : 0);
        const int32_t vres = shl32(vs, 7 - rsh) - shl32(vu, 7);
        nsf = sfs + sres + vres; nss = ssu; nvs = vu;
    }
    *pw = repack(clampi(nsf, -32768, 32767), clampi(nss, -128, 127), clampi(nvs, -128, 127));
}

// Touches only words of a ticked row or a ticked column: first every column of
// the ticked rows, then every other row of the ticked columns.
__global__ void reb_shift_kernel(RebArgs A) {
    const int32_t fired = A.fired[0];
    if (A.fired_out && blockIdx.x == 0 && threadIdx.x == 0) *A.fired_out = fired;
    if (!fired) return;
    const int32_t sd = *A.seed;
    const uint32_t NK = (uint32_t)(A.N_total * A.K);
    const int64_t nr = A.fired[1], nc = A.fired[2];
    const int64_t rows_work = nr * A.K, total = rows_work + A.N * nc;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (i < rows_work) {
            const int64_t n = A.rowlist[i / A.K];
            reb_shift_word(A, n, i % A.K, sd, NK);
        } else {
            const int64_t j = i - rows_work;
            const int64_t n = j / nc;
            if (A.rt[n] != 0) continue;  // done in the row pass
            reb_shift_word(A, n, A.collist[j % nc], sd, NK);
        }
    }
}

}  // namespace concord

using namespace concord;

static size_t al256(size_t x) { return (x + 255) / 256 * 256; }

extern "C" size_t concord_rebalance_workspace_bytes(int64_t N, int64_t K) {
    if (N <= 0 || K <= 0) return 0;
    return 256 + al256((size_t)N) + al256((size_t)K) + al256((size_t)N * HB * 4) + al256((size_t)K * HB * 4) +
           al256((size_t)N * 4) + al256((size_t)K * 4);
}

extern "C" int concord_rebalance(int32_t* packed, int64_t ldp, int8_t* row_exp, int8_t* col_exp,
                                 const int32_t* row_max, const int32_t* col_max, int32_t* row_hwm,
                                 int32_t* col_hwm, int32_t* seed, int32_t max_m, int32_t exp_max,
                                 int32_t exp_min, int32_t allow_tickdown, int64_t N, int64_t K,
                                 int64_t row0, int64_t N_total, int32_t* fired_out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    if (!packed || !row_exp || !col_exp || !row_max || !col_max || !seed)
        return fail(CONCORD_EINVAL, "concord_rebalance: null pointer");
    if (N <= 0 || K <= 0 || ldp < K || row0 < 0 || N_total < row0 + N)
        return fail(CONCORD_ESHAPE, "concord_rebalance: bad shape/stride");
    if (allow_tickdown && N_total != N)
        return fail(CONCORD_EINVAL, "concord_rebalance: tick-down needs the whole matrix (column medians)");
    size_t need = concord_rebalance_workspace_bytes(N, K);
    if (!workspace || workspace_bytes < need)
        return fail(CONCORD_EWORKSPACE, "concord_rebalance: workspace smaller than concord_rebalance_workspace_bytes(N, K)");
    char* ws = static_cast<char*>(workspace);
    RebArgs A;
    A.packed = packed; A.ldp = ldp; A.row_exp = row_exp; A.col_exp = col_exp;
    A.row_max = row_max; A.col_max = col_max; A.row_hwm = row_hwm; A.col_hwm = col_hwm;
    A.seed = seed; A.max_m = max_m; A.exp_max = exp_max; A.exp_min = exp_min;
    A.allow_td = allow_tickdown; A.N = N; A.K = K; A.row0 = row0; A.N_total = N_total;
    A.fired_out = fired_out;
    A.fired = reinterpret_cast<int32_t*>(ws);
    A.rt = reinterpret_cast<int8_t*>(ws + 256);
    A.ct = reinterpret_cast<int8_t*>(ws + 256 + al256((size_t)N));
    A.rhist = reinterpret_cast<int32_t*>(ws + 256 + al256((size_t)N) + al256((size_t)K));
    A.chist = reinterpret_cast<int32_t*>(ws + 256 + al256((size_t)N) + al256((size_t)K) + al256((size_t)N * HB * 4));
    A.rowlist = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(A.chist) + al256((size_t)K * HB * 4));
    A.collist = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(A.rowlist) + al256((size_t)N * 4));
    cudaStream_t s = as_stream(stream);
    if (cudaMemsetAsync(A.fired, 0, 3 * sizeof(int32_t), s) != cudaSuccess) return check_launch("concord_rebalance");
    int64_t blocks = (N * K + RB_THREADS - 1) / RB_THREADS;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (allow_tickdown) reb_hist_kernel<<<(unsigned)blocks, RB_THREADS, 0, s>>>(A);
    reb_decide_kernel<<<(unsigned)((N + K + RB_THREADS - 1) / RB_THREADS), RB_THREADS, 0, s>>>(A);
    reb_shift_kernel<<<148 * 4, RB_THREADS, 0, s>>>(A);
    return check_launch("concord_rebalance");
}
