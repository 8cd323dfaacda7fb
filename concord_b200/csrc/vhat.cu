// vhat.cu — Adafactor rank-1 second-moment update for the packed step.
//
// Replaces the torch ops in FusedConcordLinearPackedB.backward
// (concord/packed_b.py:1288-1303):
//   v_row = b2*v_row + (1-b2)*sum_k g^2;  v_col = b2*v_col + (1-b2)*sum_n g^2;
//   sum_v_inv = 1 / max(sum_n v_row, 1e-30)
// in two launches that read the bf16 gradient once.  The first: tiles of
// (column slabs of 256) x (row blocks of 128), taken by a persistent grid of
// blocks; each tile writes a row partial per (row, slab) and a column partial
// per (column, row block) into the workspace.  The second folds them: v_col
// from the column partials in row-block order, v_row from the row partials
// in slab order, and, in the block that finishes last (an atomic arrival
// counter, so nothing spins), sum_v_inv.  Every sum runs in a fixed order
// (spelled out in oracle/concord_oracle.c:oracle_vhat), so the result is
// deterministic and bit-identical to the CPU restatement.
//
// The first launch also zeroes row_max/col_max and bumps the step salt, which the
// reference does with separate launches before its apply kernel
// (packed_b.py:1281-1283, 910-911).
#include "common.cuh"
#include "peer.cuh"

namespace concord {

constexpr int VH_THREADS = 256;
constexpr int VH_COLS = 256;
constexpr int VH_ROWS = 128;

struct VhatArgs {
    const uint16_t* grad; int64_t ldg;
    int64_t N, K;
    float* v_row; float* v_col; float* sum_v_inv;
    float b2, omb2;
    int32_t* row_max; int32_t* col_max; int32_t* salt;
    float* rp;        // [ncs][N] row partials
    float* cp;        // [nrb][K] column partials
    unsigned* cnt;    // [nrb] row-block arrivals, [ncs] slab arrivals, [1] global
    int ncs, nrb;
    bool vec;
    float* col_sum_out;  // shard mode: raw column sums of g^2 (v_col untouched)
    float* vsum_out;     // shard mode: sum of this shard's updated v_row
    // peer mode (template P >= 1): the gradient rows are the fp32 rank-order
    // sum of P ranks' bf16 rows, rounded to bf16 and written to grad (row
    // stride ldg) as they are read.  Rank q's rows: `own` (this rank's dW rows
    // of its shard) for q == rank, else block q of the receive buffer
    // (recv + q*S*K); row stride K
    const uint16_t* own;
    const uint16_t* recv;
    int64_t S;
    PeerSync sync;
    // fold only: partial strides (0: N for rp, K for cp), and whether the
    // fold zeroes row_max/col_max and bumps the salt (partials made elsewhere)
    int64_t ldrp, ldcp;
    bool fold_resets;
};

// rows of a warp whose loads go out together: 8 for a local gradient, fewer
// when each row is the sum of P ranks' rows
template <int P>
struct VhGroup { static constexpr int G = P == 0 ? 4 : (P <= 4 ? 2 : 1); };

// resident blocks per SM: the local form (P == 0) keeps a whole C2-sized
// layer's tiles (640) resident in one wave (5 x 148 blocks); the peer forms
// hold more sources in flight per thread
template <int P>
struct VhOcc { static constexpr int B = P == 0 ? 5 : 3; };

// Persistent: block b takes tiles b, b + gridDim.x, ...; tile t covers
// column slab t % ncs and row block t / ncs.  Which block computes a tile
// changes nothing in the arithmetic: every partial and every final sum has
// a fixed order.
template <int P>
__global__ void __launch_bounds__(VH_THREADS, VhOcc<P>::B) vhat_kernel(VhatArgs A) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __shared__ float colsm[VH_THREADS / 32][VH_COLS];

    // every rank's push of this epoch has landed in the receive buffer
    if (P > 0 && !peer_wait(A.sync, ld_volatile(A.sync.state))) return;  // leave everything untouched
    const int ntiles = A.ncs * A.nrb;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int cs = tile % A.ncs, rb = tile / A.ncs;
    const int64_t k0 = (int64_t)cs * VH_COLS + lane * 8;
    if (A.salt && cs == 0 && rb == 0 && threadIdx.x == 0) *A.salt += 1;
    if (A.row_max && cs == 0 && threadIdx.x < VH_ROWS) {
        int64_t n = (int64_t)rb * VH_ROWS + threadIdx.x;
        if (n < A.N) A.row_max[n] = 0;
    }
    if (A.col_max && rb == 0) {
        int64_t k = (int64_t)cs * VH_COLS + threadIdx.x;
        if (k < A.K) A.col_max[k] = 0;
    }

    float cacc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) cacc[j] = 0.0f;
    constexpr int G = VhGroup<P>::G;
    const bool vec_ok = A.vec && k0 < A.K;
#pragma unroll
    for (int i0 = 0; i0 < VH_ROWS / 8; i0 += G) {
        // issue the group's loads before any arithmetic (vector path)
        uint4 raw[G];
        if (P == 0) {
            if (vec_ok) {
#pragma unroll
                for (int u = 0; u < G; ++u) {
                    const int64_t n = (int64_t)rb * VH_ROWS + warp + 8 * (i0 + u);
                    raw[u] = n < A.N ? __ldcs(reinterpret_cast<const uint4*>(A.grad + n * A.ldg + k0))
                                     : make_uint4(0, 0, 0, 0);
                }
            }
        } else {
            // sources in chunks of at most 4 (loads of a chunk go out together),
            // added in rank order into fp32 accumulators
            constexpr int PP = P > 0 ? P : 1;
            constexpr int QC = PP < 4 ? PP : 4;
            float acc[G][8];
#pragma unroll
            for (int q0 = 0; q0 < PP; q0 += QC) {
                uint4 pv[G][QC];
#pragma unroll
                for (int u = 0; u < G; ++u) {
                    const int64_t n = (int64_t)rb * VH_ROWS + warp + 8 * (i0 + u);
                    if (n < A.N && k0 < A.K) {
#pragma unroll
                        for (int c = 0; c < QC; ++c) {
                            const int q = q0 + c;
                            if (q < PP) {
                                const uint16_t* src = q == A.sync.rank ? A.own : A.recv + (int64_t)q * A.S * A.K;
                                pv[u][c] = __ldcs(reinterpret_cast<const uint4*>(src + n * A.K + k0));
                            }
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < G; ++u) {
#pragma unroll
                    for (int c = 0; c < QC; ++c) {
                        const int q = q0 + c;
                        if (q == 0) set_bf16x8(acc[u], pv[u][c]);
                        else if (q < PP) add_bf16x8(acc[u], pv[u][c]);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < G; ++u) {
                const int64_t n = (int64_t)rb * VH_ROWS + warp + 8 * (i0 + u);
                raw[u] = make_uint4(0, 0, 0, 0);
                if (n < A.N && k0 < A.K) {
                    raw[u] = pack_bf16x8(acc[u]);
                    __stcs(reinterpret_cast<uint4*>(const_cast<uint16_t*>(A.grad) + n * A.ldg + k0), raw[u]);
                }
            }
        }
        float rs[G];
#pragma unroll
        for (int u = 0; u < G; ++u) {
            const int i = i0 + u;
            const int64_t n = (int64_t)rb * VH_ROWS + warp + 8 * i;
            float g2[8];
            if (n < A.N) {
                const uint16_t* gp = A.grad + n * A.ldg + k0;
                if (P > 0 || vec_ok) {
                    const uint4 v = raw[u];
                    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float g = bf16_to_f32((w[j >> 1] >> ((j & 1) * 16)) & 0xffffu);
                        g2[j] = g * g;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float g = (k0 + j < A.K) ? bf16_to_f32(gp[j]) : 0.0f;
                        g2[j] = g * g;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) g2[j] = 0.0f;
            }
            // row partial: lane sum of 8 columns (the xor butterfly follows for
            // the group's rows side by side)
            float sr = g2[0];
#pragma unroll
            for (int j = 1; j < 8; ++j) sr = sr + g2[j];
            rs[u] = sr;
            // column partial: this warp's rows in order
#pragma unroll
            for (int j = 0; j < 8; ++j) cacc[j] = (i == 0) ? g2[j] : cacc[j] + g2[j];
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
#pragma unroll
            for (int u = 0; u < G; ++u) rs[u] = rs[u] + __shfl_xor_sync(0xffffffffu, rs[u], o);
        }
        if (lane == 0) {
#pragma unroll
            for (int u = 0; u < G; ++u) {
                const int64_t n = (int64_t)rb * VH_ROWS + warp + 8 * (i0 + u);
                if (n < A.N) A.rp[(int64_t)cs * A.N + n] = rs[u];
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) colsm[warp][lane * 8 + j] = cacc[j];
    __syncthreads();
    {
        float tot = colsm[0][threadIdx.x];
#pragma unroll
        for (int w = 1; w < VH_THREADS / 32; ++w) tot = tot + colsm[w][threadIdx.x];
        const int64_t col = (int64_t)cs * VH_COLS + threadIdx.x;
        if (col < A.K) A.cp[(int64_t)rb * A.K + col] = tot;
    }
    __syncthreads();   // shared memory is reused by the next tile
    }
}

// Second launch: the fixed-order folds of the partials (the launch boundary
// orders them after every tile).  Blocks [0, ncb): 256 columns each,
// v_col (or the raw column sums) from the nrb column partials in row-block
// order.  Blocks [ncb, ncb + nrf): 256 rows each, v_row from the ncs row
// partials in slab order; the last of those blocks to finish sums v_row
// (thread t: rows t, t+256, ...; then a tree over the 256 threads) into
// sum_v_inv (or the raw sum).
__global__ void __launch_bounds__(VH_THREADS) vhat_fold_kernel(VhatArgs A, int ncb, const int32_t* err) {
    __shared__ float red[VH_THREADS];
    __shared__ int last;
    if (err && ld_volatile(err) != 0) return;   // the partials were not written
    const int64_t ldrp = A.ldrp ? A.ldrp : A.N, ldcp = A.ldcp ? A.ldcp : A.K;
    if ((int)blockIdx.x < ncb) {
        const int64_t col = (int64_t)blockIdx.x * VH_THREADS + threadIdx.x;
        if (A.fold_resets && A.col_max && col < A.K) A.col_max[col] = 0;
        if (A.fold_resets && A.salt && blockIdx.x == 0 && threadIdx.x == 0) *A.salt += 1;
        if (col < A.K) {
            // fixed order b = 0, 1, ..., nrb-1; the loads of 32 partials go out together
            float t = __ldcg(A.cp + col);
            int b = 1;
            for (; b + 32 <= A.nrb; b += 32) {
                float v[32];
#pragma unroll
                for (int u = 0; u < 32; ++u) v[u] = __ldcg(A.cp + (int64_t)(b + u) * ldcp + col);
#pragma unroll
                for (int u = 0; u < 32; ++u) t = t + v[u];
            }
            for (; b + 8 <= A.nrb; b += 8) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = __ldcg(A.cp + (int64_t)(b + u) * ldcp + col);
#pragma unroll
                for (int u = 0; u < 8; ++u) t = t + v[u];
            }
            for (; b < A.nrb; ++b) t = t + __ldcg(A.cp + (int64_t)b * ldcp + col);
            if (A.col_sum_out) A.col_sum_out[col] = t;
            else A.v_col[col] = A.b2 * A.v_col[col] + A.omb2 * t;
        }
        return;
    }
    const int nrf = (int)gridDim.x - ncb;
    const int64_t n = (int64_t)(blockIdx.x - ncb) * VH_THREADS + threadIdx.x;
    if (A.fold_resets && A.row_max && n < A.N) A.row_max[n] = 0;
    if (n < A.N) {
        float t = __ldcg(A.rp + n);
        for (int c = 1; c < A.ncs; ++c) t = t + __ldcg(A.rp + (int64_t)c * ldrp + n);
        A.v_row[n] = A.b2 * A.v_row[n] + A.omb2 * t;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(A.cnt, 1u) == (unsigned)(nrf - 1);
        __threadfence();
    }
    __syncthreads();
    if (!last) return;
    // fixed order n = t, t+256, t+512, ...; the loads of 32 (then 8) go out together
    float acc = 0.0f;
    int64_t m = threadIdx.x;
    for (; m + 31 * VH_THREADS < A.N; m += 32 * VH_THREADS) {
        float v[32];
#pragma unroll
        for (int u = 0; u < 32; ++u) v[u] = __ldcg(A.v_row + m + u * VH_THREADS);
#pragma unroll
        for (int u = 0; u < 32; ++u) acc = acc + v[u];
    }
    for (; m + 7 * VH_THREADS < A.N; m += 8 * VH_THREADS) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldcg(A.v_row + m + u * VH_THREADS);
#pragma unroll
        for (int u = 0; u < 8; ++u) acc = acc + v[u];
    }
    for (; m < A.N; m += VH_THREADS) acc = acc + __ldcg(A.v_row + m);
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int s = VH_THREADS / 2; s >= 1; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] = red[threadIdx.x] + red[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        if (A.vsum_out) {
            *A.vsum_out = red[0];
        } else {
            float sv = np_max(red[0], 1e-30f);
            *A.sum_v_inv = 1.0f / sv;
        }
        *A.cnt = 0;
    }
}

static void vhat_fold(const VhatArgs& A, const int32_t* err, cudaStream_t st) {
    const int ncb = (int)((A.K + VH_THREADS - 1) / VH_THREADS);
    const int64_t nrf = A.N > 0 ? (A.N + VH_THREADS - 1) / VH_THREADS : 1;
    vhat_fold_kernel<<<(unsigned)(ncb + nrf), VH_THREADS, 0, st>>>(A, ncb, err);
}

// The fold of partials made elsewhere (the dW GEMM's epilogue): rp
// [ceil(K/256)][ldrp], cp [ceil(N/128)][ldcp], cnt one zeroed counter that
// the fold leaves zeroed; also zeroes row_max/col_max and bumps the salt.
int vhat_fold_partials(const float* rp, int64_t ldrp, const float* cp, int64_t ldcp, int64_t N, int64_t K,
                       float* v_row, float* v_col, float* sum_v_inv, float beta2, float one_minus_beta2,
                       int32_t* row_max, int32_t* col_max, int32_t* salt, unsigned* cnt, cudaStream_t st) {
    VhatArgs A{};
    A.N = N; A.K = K;
    A.v_row = v_row; A.v_col = v_col; A.sum_v_inv = sum_v_inv;
    A.b2 = beta2; A.omb2 = one_minus_beta2;
    A.row_max = row_max; A.col_max = col_max; A.salt = salt;
    A.rp = const_cast<float*>(rp); A.cp = const_cast<float*>(cp); A.cnt = cnt;
    A.ncs = (int)((K + VH_COLS - 1) / VH_COLS);
    A.nrb = (int)((N + VH_ROWS - 1) / VH_ROWS);
    A.ldrp = ldrp; A.ldcp = ldcp;
    A.fold_resets = true;
    vhat_fold(A, nullptr, st);
    return check_launch("vhat_fold_partials");
}

// shard mode, after the all-reduce of (column sums, v_row sum) over ranks
__global__ void vhat_finish_kernel(const float* col_sum, const float* vsum, float* v_col, float* sum_v_inv,
                                   int64_t K, float b2, float omb2) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < K; k += (int64_t)gridDim.x * blockDim.x)
        v_col[k] = b2 * v_col[k] + omb2 * col_sum[k];
    if (blockIdx.x == 0 && threadIdx.x == 0) *sum_v_inv = 1.0f / np_max(*vsum, 1e-30f);
}

}  // namespace concord

using namespace concord;

static void vhat_layout(int64_t N, int64_t K, int* ncs, int* nrb, size_t* off_rp, size_t* off_cp,
                        size_t* total) {
    *ncs = (int)((K + VH_COLS - 1) / VH_COLS);
    *nrb = (int)((N + VH_ROWS - 1) / VH_ROWS);
    size_t cnt_bytes = ((size_t)(*nrb + *ncs + 1) * sizeof(unsigned) + 255) / 256 * 256;
    *off_rp = cnt_bytes;
    size_t rp_bytes = ((size_t)(*ncs) * (size_t)N * sizeof(float) + 255) / 256 * 256;
    *off_cp = cnt_bytes + rp_bytes;
    *total = *off_cp + (size_t)(*nrb) * (size_t)K * sizeof(float);
}

// one block per tile up to `per_sm` resident blocks on every SM
static unsigned vhat_grid(int ncs, int nrb, int per_sm) {
    static const int sms = [] {
        int dev = 0, n = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        return n > 0 ? n : 148;
    }();
    const int64_t tiles = (int64_t)ncs * nrb;
    const int64_t cap = (int64_t)sms * per_sm;
    return (unsigned)(tiles < cap ? tiles : cap);
}

extern "C" size_t concord_vhat_workspace_bytes(int64_t N, int64_t K) {
    if (N <= 0 || K <= 0) return 0;
    int ncs, nrb; size_t a, b, t;
    vhat_layout(N, K, &ncs, &nrb, &a, &b, &t);
    return t;
}

static int vhat_launch(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K, float* v_row, float* v_col,
                       float* sum_v_inv, float beta2, float one_minus_beta2, int32_t* row_max, int32_t* col_max,
                       int32_t* salt, float* col_sum_out, float* vsum_out, void* workspace,
                       size_t workspace_bytes, void* stream, const char* name) {
    if (N <= 0 || K <= 0 || ldg < K) return fail(CONCORD_ESHAPE, std::string(name) + ": bad shape/stride");
    int ncs, nrb; size_t off_rp, off_cp, total;
    vhat_layout(N, K, &ncs, &nrb, &off_rp, &off_cp, &total);
    if (!workspace || workspace_bytes < total)
        return fail(CONCORD_EWORKSPACE, std::string(name) + ": workspace smaller than concord_vhat_workspace_bytes(N, K)");
    if ((int64_t)ncs * nrb > INT32_MAX) return fail(CONCORD_ETOOBIG, std::string(name) + ": too many tiles for one launch");
    char* ws = static_cast<char*>(workspace);
    VhatArgs A{grad, ldg, N, K, v_row, v_col, sum_v_inv, beta2, one_minus_beta2, row_max, col_max, salt,
               reinterpret_cast<float*>(ws + off_rp), reinterpret_cast<float*>(ws + off_cp),
               reinterpret_cast<unsigned*>(ws), ncs, nrb,
               (K % 8 == 0) && (ldg % 8 == 0) && aligned(grad, 16), col_sum_out, vsum_out,
               nullptr, nullptr, 0, PeerSync{}};
    vhat_kernel<0><<<vhat_grid(ncs, nrb, VhOcc<0>::B), VH_THREADS, 0, as_stream(stream)>>>(A);
    vhat_fold(A, nullptr, as_stream(stream));
    return check_launch(name);
}

extern "C" int concord_vhat_update(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K,
                                   float* v_row, float* v_col, float* sum_v_inv, float beta2,
                                   float one_minus_beta2, int32_t* row_max, int32_t* col_max,
                                   int32_t* salt, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    if (!grad || !v_row || !v_col || !sum_v_inv) return fail(CONCORD_EINVAL, "concord_vhat_update: null pointer");
    return vhat_launch(grad, ldg, N, K, v_row, v_col, sum_v_inv, beta2, one_minus_beta2, row_max, col_max, salt,
                       nullptr, nullptr, workspace, workspace_bytes, stream, "concord_vhat_update");
}

extern "C" int concord_vhat_partial(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K, float* v_row,
                                    float beta2, float one_minus_beta2, int32_t* row_max, int32_t* col_max,
                                    int32_t* salt, float* col_sum_out, float* vsum_out, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    if (!grad || !v_row || !col_sum_out || !vsum_out) return fail(CONCORD_EINVAL, "concord_vhat_partial: null pointer");
    return vhat_launch(grad, ldg, N, K, v_row, nullptr, nullptr, beta2, one_minus_beta2, row_max, col_max, salt,
                       col_sum_out, vsum_out, workspace, workspace_bytes, stream, "concord_vhat_partial");
}

template <int P>
static void launch_peer_vhat(unsigned grid, cudaStream_t st, const VhatArgs& A) {
    vhat_kernel<P><<<grid, VH_THREADS, 0, st>>>(A);
}

extern "C" int concord_peer_reduce_vhat(const uint16_t* own_rows, const uint16_t* recv, int64_t S, int64_t K,
                                        int64_t n_rows, uint16_t* grad_out, float* v_row, float beta2,
                                        float one_minus_beta2, int32_t* row_max, int32_t* col_max, int32_t* salt,
                                        float* col_sum_out, float* vsum_out, void* workspace,
                                        size_t workspace_bytes, const concord_peer_sync* sync, void* stream) {
    const char* name = "concord_peer_reduce_vhat";
    // a rank without rows (more ranks than rows) passes empty own_rows /
    // grad_out / v_row views, which may be null
    if ((n_rows > 0 && (!own_rows || !recv || !grad_out || !v_row)) || !col_sum_out || !vsum_out || !sync || !sync->flags ||
        !sync->peer_flags || !sync->state)
        return fail(CONCORD_EINVAL, std::string(name) + ": null pointer");
    if (sync->n_ranks < 1 || sync->n_ranks > PEER_MAX_RANKS || sync->rank < 0 || sync->rank >= sync->n_ranks)
        return fail(CONCORD_EINVAL, std::string(name) + ": n_ranks must be 1..8 and rank < n_ranks");
    if (sync->timeout_ns <= 0) return fail(CONCORD_EINVAL, std::string(name) + ": timeout_ns must be > 0");
    if (K <= 0 || K % 8 != 0 || n_rows < 0 || n_rows > S)
        return fail(CONCORD_ESHAPE, std::string(name) + ": K must be a positive multiple of 8 and n_rows <= S");
    if (n_rows > 0 && (!aligned(grad_out, 16) || !aligned(own_rows, 16) || !aligned(recv, 16)))
        return fail(CONCORD_EALIGN, std::string(name) + ": buffers must be 16-byte aligned");
    // a rank with no rows still takes part: one row block of masked rows gives zero partials
    int ncs, nrb; size_t off_rp, off_cp, total;
    vhat_layout(n_rows > 0 ? n_rows : 1, K, &ncs, &nrb, &off_rp, &off_cp, &total);
    if (!workspace || workspace_bytes < total)
        return fail(CONCORD_EWORKSPACE, std::string(name) + ": workspace smaller than "
                                        "concord_vhat_workspace_bytes(max(n_rows, 1), K)");
    if ((int64_t)ncs * nrb > INT32_MAX) return fail(CONCORD_ETOOBIG, std::string(name) + ": too many tiles for one launch");
    char* ws = static_cast<char*>(workspace);
    VhatArgs A{grad_out, K, n_rows, K, v_row, nullptr, nullptr, beta2, one_minus_beta2, row_max, col_max, salt,
               reinterpret_cast<float*>(ws + off_rp), reinterpret_cast<float*>(ws + off_cp),
               reinterpret_cast<unsigned*>(ws), ncs, nrb, true, col_sum_out, vsum_out, own_rows, recv, S,
               PeerSync{sync->flags, sync->peer_flags, sync->state, sync->rank, sync->n_ranks, sync->timeout_ns}};
    const unsigned grid = vhat_grid(ncs, nrb, VhOcc<1>::B);
    cudaStream_t st = as_stream(stream);
    switch (sync->n_ranks) {
        case 1: launch_peer_vhat<1>(grid, st, A); break;
        case 2: launch_peer_vhat<2>(grid, st, A); break;
        case 3: launch_peer_vhat<3>(grid, st, A); break;
        case 4: launch_peer_vhat<4>(grid, st, A); break;
        case 5: launch_peer_vhat<5>(grid, st, A); break;
        case 6: launch_peer_vhat<6>(grid, st, A); break;
        case 7: launch_peer_vhat<7>(grid, st, A); break;
        default: launch_peer_vhat<8>(grid, st, A); break;
    }
    vhat_fold(A, sync->state + 2, st);
    return check_launch(name);
}

extern "C" int concord_vhat_finish(const float* col_sum, const float* vsum, float* v_col, float* sum_v_inv,
                                   int64_t K, float beta2, float one_minus_beta2, void* stream) {
    if (!col_sum || !vsum || !v_col || !sum_v_inv) return fail(CONCORD_EINVAL, "concord_vhat_finish: null pointer");
    if (K <= 0) return fail(CONCORD_ESHAPE, "concord_vhat_finish: bad shape");
    int blocks = (int)((K + 255) / 256);
    if (blocks > 1024) blocks = 1024;
    vhat_finish_kernel<<<blocks, 256, 0, as_stream(stream)>>>(col_sum, vsum, v_col, sum_v_inv, K, beta2, one_minus_beta2);
    return check_launch("concord_vhat_finish");
}

// ---------------------------------------------------------------------------
// Allocation-free form of concord_vhat_update.
//
// For callers that are not allowed to allocate device memory themselves: a
// host framework that hands plugins a fixed device-memory budget and forbids
// cudaMalloc after start-up, or a caller on a latency-critical path where the
// implicit device synchronisation of cudaMalloc/cudaFree would stall other
// streams.  The scratch lives in a file-scope device array that every GPU
// loading this library holds until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

namespace concord {

constexpr size_t VHAT_STATIC_SCRATCH_BYTES = 4u << 20;  // 4 MiB per device
static __device__ __align__(256) unsigned char g_vhat_scratch[VHAT_STATIC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
static void* g_vhat_scratch_ptr[MAX_DEVICES];  // last device address of g_vhat_scratch seen, per device
static std::mutex g_vhat_scratch_mu;

// Every call, with the caller's device current: look up the array's device
// address (the host-side name is only a stand-in; the lookup is a host-side
// table query).  The first call that sees an address for a device, or a new
// address for it (a new CUDA context after cudaDeviceReset, or another
// context made current on the same device), clears the array on the caller's
// stream, because the kernels expect their counters to start at zero and
// leave them at zero when they finish.
static int vhat_scratch_for_current_device(void** out, cudaStream_t stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES)
        return fail(CONCORD_ENODEVICE, "concord_vhat_update_noalloc: no usable current CUDA device");
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_vhat_scratch);
    if (e != cudaSuccess || !p)
        return fail(CONCORD_ELAUNCH, std::string("concord_vhat_update_noalloc: cudaGetSymbolAddress failed: ") +
                                         cudaGetErrorString(e));
    std::lock_guard<std::mutex> lock(g_vhat_scratch_mu);
    if (g_vhat_scratch_ptr[dev] != p) {
        e = cudaMemsetAsync(p, 0, VHAT_STATIC_SCRATCH_BYTES, stream);
        if (e != cudaSuccess)
            return fail(CONCORD_ELAUNCH, std::string("concord_vhat_update_noalloc: clearing scratch failed: ") +
                                         cudaGetErrorString(e));
        g_vhat_scratch_ptr[dev] = p;
    }
    *out = p;
    return CONCORD_OK;
}

}  // namespace concord

extern "C" size_t concord_vhat_noalloc_max_scratch_bytes(void) { return concord::VHAT_STATIC_SCRATCH_BYTES; }

extern "C" int concord_vhat_update_noalloc(const uint16_t* grad, int64_t ldg, int64_t N, int64_t K,
                                           float* v_row, float* v_col, float* sum_v_inv, float beta2,
                                           float one_minus_beta2, int32_t* row_max, int32_t* col_max,
                                           int32_t* salt, void* stream) {
    if (!grad || !v_row || !v_col || !sum_v_inv)
        return fail(CONCORD_EINVAL, "concord_vhat_update_noalloc: null pointer");
    if (N <= 0 || K <= 0 || ldg < K) return fail(CONCORD_ESHAPE, "concord_vhat_update_noalloc: bad shape/stride");
    const size_t need = concord_vhat_workspace_bytes(N, K);
    if (need > concord::VHAT_STATIC_SCRATCH_BYTES)
        return fail(CONCORD_ETOOBIG, "concord_vhat_update_noalloc: N x K needs " + std::to_string(need) +
                                         " bytes of scratch, above the fixed 4 MiB per device; use "
                                         "concord_vhat_update with a caller-provided workspace");
    void* ws = nullptr;
    int rc = concord::vhat_scratch_for_current_device(&ws, as_stream(stream));
    if (rc != CONCORD_OK) return rc;
    return vhat_launch(grad, ldg, N, K, v_row, v_col, sum_v_inv, beta2, one_minus_beta2, row_max, col_max, salt,
                       nullptr, nullptr, ws, concord::VHAT_STATIC_SCRATCH_BYTES, stream,
                       "concord_vhat_update_noalloc");
}
