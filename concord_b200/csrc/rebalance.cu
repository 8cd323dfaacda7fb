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
    unsigned long long* stats;                // optional: [tick-ups, tick-downs, clipped words]
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
        if (A.stats && t) atomicAdd(A.stats + (up ? 0 : 1), 1ull);
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
        if (A.stats && t) atomicAdd(A.stats + (up ? 0 : 1), 1ull);
        A.ct[k] = (int8_t)t;
        if (t) {
            A.col_exp[k] = (int8_t)(e + t);
            atomicOr(A.fired, 1);
            A.collist[atomicAdd(A.fired + 2, 1)] = (int32_t)k;
        }
    }
}

// Diagnostic (only with stats): words whose larger int8 field no longer fits
// in int8 once the net left shift of a tick-down is applied,
// max(|s_slow|, |v_slow|) << max(0, -(rt + ct)) > 127, counted on the
// pre-shift words (a field of -128 counts even without a shift).
__global__ void reb_clip_count_kernel(RebArgs A) {
    unsigned long long c = 0;
    const int64_t total = A.N * A.K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / A.K, k = i - n * A.K;
        const int32_t w = A.packed[n * A.ldp + k];
        const int32_t m = max(abs(shl32(w, 16) >> 24), abs(shl32(w, 24) >> 24));
        const int32_t lsh = max(0, -((int32_t)A.rt[n] + (int32_t)A.ct[k]));
        c += (m << lsh) > 127;
    }
    for (int o = 16; o >= 1; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(A.stats + 2, c);
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
// the ticked rows, then every other row of the ticked columns.  The index
// arithmetic runs in 32 bits when the work fits (it does unless a layer
// holds 2^31 words).
template <typename I>
__device__ __forceinline__ void reb_shift_range(const RebArgs& A, int64_t nr64, int64_t nc64, int32_t sd,
                                                uint32_t NK) {
    const I K = (I)A.K, nc = (I)nc64;
    const I rows_work = (I)nr64 * K, total = rows_work + (I)A.N * nc;
    for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
        if (i < rows_work) {
            const I r = i / K;
            reb_shift_word(A, A.rowlist[r], (int64_t)(i - r * K), sd, NK);
        } else {
            const I j = i - rows_work;
            const I n = j / nc;
            if (A.rt[n] != 0) continue;  // done in the row pass
            reb_shift_word(A, (int64_t)n, A.collist[j - n * nc], sd, NK);
        }
    }
}

__global__ void reb_shift_kernel(RebArgs A) {
    const int32_t fired = A.fired[0];
    if (A.fired_out && blockIdx.x == 0 && threadIdx.x == 0) *A.fired_out = fired;
    if (!fired) return;
    const int32_t sd = *A.seed;
    const uint32_t NK = (uint32_t)(A.N_total * A.K);
    const int64_t nr = A.fired[1], nc = A.fired[2];
    const int64_t total = nr * A.K + A.N * nc;
    if (total + (int64_t)gridDim.x * blockDim.x < ((int64_t)1 << 31))
        reb_shift_range<uint32_t>(A, nr, nc, sd, NK);
    else
        reb_shift_range<int64_t>(A, nr, nc, sd, NK);
}

// ---------------------------------------------------------------------------
// Gated rebalance of many layers (the trainer-side GatedRebalance of the
// reference, notebook/src/concord_winner.py:206-262): when ANY row or column
// maximum of ANY layer exceeds max_m, every layer runs its rebalance (seed
// bump, high-watermark fold, tick-up decisions, SR shift); otherwise none
// does.  The reference decides on the host (one reduction and a device->host
// read per step); here a gate launch writes the decision to device memory and
// two batched launches cover every layer, predicated on it, so the whole
// thing stays on the stream (graph-capturable) and costs three launches
// whatever the number of layers.  Tick-down is not part of this path.
// ---------------------------------------------------------------------------

// gate[0] = 1 if any of the n values of maxima exceeds max_m
__global__ void reb_gate_kernel(const int32_t* rows, int64_t nr, const int32_t* cols, int64_t nc,
                                int32_t max_m, int32_t* gate) {
    int hit = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nr + nc;
         i += (int64_t)gridDim.x * blockDim.x)
        hit |= (i < nr ? rows[i] : cols[i - nr]) > max_m;
    if (__syncthreads_or(hit) && threadIdx.x == 0) atomicOr(gate, 1);
}

__device__ __forceinline__ RebArgs reb_args_of(const concord_reb_layer& L) {
    RebArgs A;
    A.packed = L.packed; A.ldp = L.ldp; A.row_exp = L.row_exp; A.col_exp = L.col_exp;
    A.row_max = L.row_max; A.col_max = L.col_max; A.row_hwm = L.row_hwm; A.col_hwm = L.col_hwm;
    A.seed = L.seed; A.max_m = L.max_m; A.exp_max = L.exp_max; A.exp_min = L.exp_min; A.allow_td = 0;
    A.N = L.N; A.K = L.K; A.row0 = L.row0; A.N_total = L.N_total; A.fired_out = nullptr;
    A.rt = L.rt; A.ct = L.ct; A.fired = L.fired; A.rhist = nullptr; A.chist = nullptr;
    A.rowlist = L.rowlist; A.collist = L.collist; A.stats = nullptr;
    return A;
}

// one thread per row / column of every layer (layer l owns entries
// [L.decide_off, L.decide_off + N + K)); layers found by binary search
__global__ void reb_decide_many_kernel(const concord_reb_layer* layers, int32_t n_layers, int64_t total,
                                       const int32_t* gate) {
    if (*gate == 0) return;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int lo = 0, hi = n_layers - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (layers[mid].decide_off <= i) lo = mid; else hi = mid - 1;
        }
        const concord_reb_layer& L = layers[lo];
        const int64_t j = i - L.decide_off;
        RebArgs A = reb_args_of(L);
        if (j == 0) *A.seed += 1;
        if (j < A.N) {
            const int32_t mx = A.row_max[j];
            if (A.row_hwm) A.row_hwm[j] = max(A.row_hwm[j], mx);
            const int32_t e = A.row_exp[j];
            const int t = mx > A.max_m && e < A.exp_max;
            A.rt[j] = (int8_t)t;
            if (t) {
                A.row_exp[j] = (int8_t)(e + t);
                atomicOr(A.fired, 1);
                A.rowlist[atomicAdd(A.fired + 1, 1)] = (int32_t)j;
            }
        } else {
            const int64_t k = j - A.N;
            const int32_t mx = A.col_max[k];
            if (A.col_hwm) A.col_hwm[k] = max(A.col_hwm[k], mx);
            const int32_t e = A.col_exp[k];
            const int t = mx > A.max_m && e < A.exp_max;
            A.ct[k] = (int8_t)t;
            if (t) {
                A.col_exp[k] = (int8_t)(e + t);
                atomicOr(A.fired, 1);
                A.collist[atomicAdd(A.fired + 2, 1)] = (int32_t)k;
            }
        }
    }
}

// every block walks the layers; a layer with nothing ticked costs one read.
// Afterwards the per-layer counters are cleared for the next call (the last
// block to finish clears them: the counters are read by every block).
__global__ void reb_shift_many_kernel(const concord_reb_layer* layers, int32_t n_layers, const int32_t* gate,
                                      int32_t* fired_out, uint32_t* done) {
    if (*gate != 0) {
        for (int l = 0; l < n_layers; ++l) {
            const concord_reb_layer& L = layers[l];
            const int32_t* f = L.fired;
            if (f[0] == 0) continue;
            RebArgs A = reb_args_of(L);
            const int32_t sd = *A.seed;
            const uint32_t NK = (uint32_t)(A.N_total * A.K);
            const int64_t nr = f[1], nc = f[2];
            const int64_t rows_work = nr * A.K, total = rows_work + A.N * nc;
            for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
                 i += (int64_t)gridDim.x * blockDim.x) {
                if (i < rows_work) {
                    reb_shift_word(A, A.rowlist[i / A.K], i % A.K, sd, NK);
                } else {
                    const int64_t j = i - rows_work;
                    const int64_t n = j / nc;
                    if (A.rt[n] != 0) continue;
                    reb_shift_word(A, n, A.collist[j % nc], sd, NK);
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            if (fired_out) *fired_out = *gate;
            for (int l = 0; l < n_layers; ++l) {
                int32_t* f = layers[l].fired;
                f[0] = 0; f[1] = 0; f[2] = 0;
            }
            *const_cast<int32_t*>(gate) = 0;
            *done = 0;
            __threadfence();
        }
    }
}

}  // namespace concord

using namespace concord;

static size_t al256(size_t x) { return (x + 255) / 256 * 256; }

extern "C" size_t concord_rebalance_gated_layer_workspace_bytes(int64_t N, int64_t K) {
    if (N <= 0 || K <= 0) return 0;
    return 256 + al256((size_t)N) + al256((size_t)K) + al256((size_t)N * 4) + al256((size_t)K * 4);
}

extern "C" int concord_rebalance_gated_layer_layout(int64_t N, int64_t K, void* workspace, concord_reb_layer* layer) {
    if (!workspace || !layer || N <= 0 || K <= 0) return fail(CONCORD_EINVAL, "concord_rebalance_gated_layer_layout: bad arguments");
    char* ws = static_cast<char*>(workspace);
    layer->fired = reinterpret_cast<int32_t*>(ws);
    layer->rt = reinterpret_cast<int8_t*>(ws + 256);
    layer->ct = reinterpret_cast<int8_t*>(ws + 256 + al256((size_t)N));
    layer->rowlist = reinterpret_cast<int32_t*>(ws + 256 + al256((size_t)N) + al256((size_t)K));
    layer->collist = reinterpret_cast<int32_t*>(ws + 256 + al256((size_t)N) + al256((size_t)K) + al256((size_t)N * 4));
    return CONCORD_OK;
}

extern "C" int concord_rebalance_gated(const concord_reb_layer* layers, int32_t n_layers, int64_t total_decide,
                                       const int32_t* row_max_all, int64_t n_rows_all, const int32_t* col_max_all,
                                       int64_t n_cols_all, int32_t gate_max_m, int32_t* gate, int32_t* fired_out,
                                       void* stream) {
    if (!layers || !gate || n_layers <= 0 || total_decide <= 0 || !row_max_all || !col_max_all)
        return fail(CONCORD_EINVAL, "concord_rebalance_gated: bad arguments");
    cudaStream_t s = as_stream(stream);
    int64_t gb = (n_rows_all + n_cols_all + RB_THREADS - 1) / RB_THREADS;
    if (gb > 148 * 4) gb = 148 * 4;
    reb_gate_kernel<<<(unsigned)(gb > 0 ? gb : 1), RB_THREADS, 0, s>>>(row_max_all, n_rows_all, col_max_all,
                                                                      n_cols_all, gate_max_m, gate);
    int64_t db = (total_decide + RB_THREADS - 1) / RB_THREADS;
    if (db > 148 * 8) db = 148 * 8;
    reb_decide_many_kernel<<<(unsigned)db, RB_THREADS, 0, s>>>(layers, n_layers, total_decide, gate);
    reb_shift_many_kernel<<<148 * 4, RB_THREADS, 0, s>>>(layers, n_layers, gate, fired_out,
                                                          reinterpret_cast<uint32_t*>(gate + 1));
    return check_launch("concord_rebalance_gated");
}

extern "C" size_t concord_rebalance_workspace_bytes(int64_t N, int64_t K) {
    if (N < 0 || K <= 0) return 0;
    return 256 + al256((size_t)N) + al256((size_t)K) + al256((size_t)N * HB * 4) + al256((size_t)K * HB * 4) +
           al256((size_t)N * 4) + al256((size_t)K * 4);
}

extern "C" int concord_rebalance(int32_t* packed, int64_t ldp, int8_t* row_exp, int8_t* col_exp,
                                 const int32_t* row_max, const int32_t* col_max, int32_t* row_hwm,
                                 int32_t* col_hwm, int32_t* seed, int32_t max_m, int32_t exp_max,
                                 int32_t exp_min, int32_t allow_tickdown, int64_t N, int64_t K,
                                 int64_t row0, int64_t N_total, int32_t* fired_out,
                                 unsigned long long* stats, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    if (!packed || !row_exp || !col_exp || !row_max || !col_max || !seed)
        return fail(CONCORD_EINVAL, "concord_rebalance: null pointer");
    // N == 0 (a data-parallel rank that owns no rows of the layer): the
    // column decisions still tick the shared column exponents, fold the column
    // high-watermarks and bump the seed; there is no word to shift
    if (N < 0 || K <= 0 || ldp < K || row0 < 0 || N_total < row0 + N || N_total <= 0)
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
    A.stats = stats;
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
    if (blocks < 1) blocks = 1;
    // the histogram bins sit at shape-dependent offsets of a workspace that
    // callers may share between layers of different shapes: clear them first
    if (allow_tickdown &&
        cudaMemsetAsync(A.rhist, 0, al256((size_t)N * HB * 4) + (size_t)K * HB * 4, s) != cudaSuccess)
        return check_launch("concord_rebalance");
    if (allow_tickdown) reb_hist_kernel<<<(unsigned)blocks, RB_THREADS, 0, s>>>(A);
    reb_decide_kernel<<<(unsigned)((N + K + RB_THREADS - 1) / RB_THREADS), RB_THREADS, 0, s>>>(A);
    if (stats) reb_clip_count_kernel<<<(unsigned)blocks, RB_THREADS, 0, s>>>(A);
    reb_shift_kernel<<<148 * 4, RB_THREADS, 0, s>>>(A);
    return check_launch("concord_rebalance");
}
