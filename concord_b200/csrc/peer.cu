// peer.cu — peer memory over NVLink for the row-sharded data-parallel step.
//
// The reference is single-GPU.  Its update needs, for row n, only row n's
// gradient summed over the data-parallel ranks, so the reduce-scatter of the
// bf16 dW is a pull over NVLink: rank r reads rows [row0, row0 + n_rows) of
// every rank's dW (CUDA IPC mappings), adds them in fp32 in rank order and
// rounds once to bf16.  The sum is therefore the same bits on every rank and
// for every rank count (a ring reduction in bf16 is neither).
//
// Ordering: a rank's dW is complete when that rank's stream reaches this
// kernel.  Each block of the kernel announces "epoch e entered" to every
// rank (a release store into that rank's flag array) and waits until every
// rank has announced e (acquire loads of its own flags), then reads.  Each
// wait is bounded by GPU time (globaltimer); when it runs out the block sets
// the error word, skips its work and returns.  The last block to finish
// advances the epoch.  Peer data moves with plain 16-byte loads.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "peer.cuh"

namespace concord {

constexpr int PEER_THREADS = 256;

// Push half of the reduce-scatter: rows of rank q's shard [q*S, min(N, (q+1)*S))
// of this rank's dW go to q's receive buffer, block `rank` (recv_q + rank*S*K),
// for every q != rank, 16 bytes per load and store, four chunks in flight per
// thread.  Nothing waits: when the last block has seen every block's stores
// fenced at system scope, it announces the epoch to every rank.
constexpr int PUSH_UNROLL = 4;

template <typename I>   // index type: 32-bit when the whole gradient has < 2^31 chunks
__device__ __forceinline__ void push_chunk(const uint4* grad, const uint64_t* recv, I c, I kc, I S, int rank,
                                           uint4 v) {
    const I n = c / kc;
    const I q = n / S;
    const int64_t dst = ((int64_t)rank * S + (n - q * S)) * (int64_t)kc + (c - n * kc);
    __stcs(reinterpret_cast<uint4*>(recv[q]) + dst, v);
}

template <typename I>
__global__ void __launch_bounds__(PEER_THREADS) peer_push_kernel(const uint4* grad, int64_t N, int64_t kc64,
                                                                 int64_t S64, const uint64_t* recv, PeerSync s) {
    const int32_t e = ld_volatile(s.state) + 1;
    if (ld_volatile(s.state + 2) == 0) {
        const I kc = (I)kc64, S = (I)S64;
        const I total = (I)(N * kc64);
        // this rank's own rows stay where they are: chunks [own0, own1) are skipped
        const I own0 = (I)min((int64_t)total, (int64_t)s.rank * S64 * kc64);
        const I own1 = (I)min((int64_t)total, ((int64_t)s.rank + 1) * S64 * kc64);
        // the other chunks in the order own1, ..., total-1, 0, ..., own0-1: at any
        // moment rank r writes mostly to rank r+1's shard, rank r+1 to r+2's, and
        // so on, so the ranks' stores spread over every receiver instead of all
        // ranks writing the same receiver's shard at once
        const I work = total - (own1 - own0);
        const I span = (I)gridDim.x * PEER_THREADS;
        for (I i0 = (I)blockIdx.x * PEER_THREADS + threadIdx.x; i0 < work; i0 += span * PUSH_UNROLL) {
            uint4 v[PUSH_UNROLL];
            I cs[PUSH_UNROLL];
#pragma unroll
            for (int u = 0; u < PUSH_UNROLL; ++u) {
                const I i = i0 + (I)u * span;
                I c = own1 + i;
                if (c >= total) c -= total;
                cs[u] = c;
                if (i < work) v[u] = __ldcs(grad + c);
            }
#pragma unroll
            for (int u = 0; u < PUSH_UNROLL; ++u)
                if (i0 + (I)u * span < work) push_chunk<I>(grad, recv, cs[u], kc, S, s.rank, v[u]);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const int blocks = (int)(gridDim.x * gridDim.y * gridDim.z);
        if (atomicAdd(s.state + 1, 1) == blocks - 1) {
            __threadfence_system();
            for (int q = 0; q < s.n_ranks; ++q)
                st_release_sys(reinterpret_cast<int32_t*>(s.peer_flags[q]) + s.rank, e);
            s.state[1] = 0;
            s.state[0] = e;
            __threadfence();
        }
    }
}

// Small all-reduce through peer slots, one block.  Every rank's slot buffer
// holds two halves (epoch parity) of n_ranks rows of slot_count 32-bit
// values.  A rank stores its input into row `rank` of the current half of
// every rank's slots, meets the others, and reduces its own slots in rank
// order.  The two halves make reuse safe: a rank writes a half again only
// after a later rendezvous that every rank enters once it has finished
// reading that half.
constexpr int AR_THREADS = 1024;

__global__ void __launch_bounds__(AR_THREADS) peer_allreduce_kernel(const uint32_t* in, uint32_t* out, int64_t count,
                                                                    int op, const uint64_t* slots, int64_t slot_count,
                                                                    PeerSync s) {
    const int32_t e = ld_volatile(s.state) + 1;
    const int64_t half = (int64_t)(e & 1) * s.n_ranks * slot_count;
    if (ld_volatile(s.state + 2) == 0) {
        for (int64_t i = threadIdx.x; i < count; i += AR_THREADS) {
            const uint32_t v = in[i];
            for (int q = 0; q < s.n_ranks; ++q)
                reinterpret_cast<uint32_t*>(slots[q])[half + (int64_t)s.rank * slot_count + i] = v;
        }
    }
    if (peer_rendezvous(s, e)) {
        const uint32_t* mine = reinterpret_cast<const uint32_t*>(slots[s.rank]) + half;
        for (int64_t i = threadIdx.x; i < count; i += AR_THREADS) {
            if (op == CONCORD_PEER_SUM_F32) {
                float acc = __uint_as_float(__ldcv(mine + i));
                for (int q = 1; q < s.n_ranks; ++q) acc = acc + __uint_as_float(__ldcv(mine + (int64_t)q * slot_count + i));
                out[i] = __float_as_uint(acc);
            } else {
                int32_t acc = (int32_t)__ldcv(mine + i);
                for (int q = 1; q < s.n_ranks; ++q) acc = max(acc, (int32_t)__ldcv(mine + (int64_t)q * slot_count + i));
                out[i] = (uint32_t)acc;
            }
        }
    }
    peer_finish(s, e);
}

}  // namespace concord

using namespace concord;

extern "C" int concord_peer_allreduce(const void* in, void* out, int64_t count, int32_t op, const uint64_t* slots,
                                      int64_t slot_count, const concord_peer_sync* sync, void* stream) {
    if ((count > 0 && (!in || !out)) || !slots || !sync || !sync->flags || !sync->peer_flags || !sync->state)
        return fail(CONCORD_EINVAL, "concord_peer_allreduce: null pointer");
    if (sync->n_ranks < 1 || sync->n_ranks > PEER_MAX_RANKS || sync->rank < 0 || sync->rank >= sync->n_ranks)
        return fail(CONCORD_EINVAL, "concord_peer_allreduce: n_ranks must be 1..8 and rank < n_ranks");
    if (op != CONCORD_PEER_SUM_F32 && op != CONCORD_PEER_MAX_I32)
        return fail(CONCORD_EINVAL, "concord_peer_allreduce: unknown op");
    if (count < 0 || count > slot_count) return fail(CONCORD_ESHAPE, "concord_peer_allreduce: count above slot_count");
    if (sync->timeout_ns <= 0) return fail(CONCORD_EINVAL, "concord_peer_allreduce: timeout_ns must be > 0");
    PeerSync s{sync->flags, sync->peer_flags, sync->state, sync->rank, sync->n_ranks, sync->timeout_ns};
    peer_allreduce_kernel<<<1, AR_THREADS, 0, as_stream(stream)>>>(
        static_cast<const uint32_t*>(in), static_cast<uint32_t*>(out), count, op, slots, slot_count, s);
    return check_launch("concord_peer_allreduce");
}

extern "C" size_t concord_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int concord_peer_alloc(size_t bytes, void** dev_ptr) {
    if (!dev_ptr || bytes == 0) return fail(CONCORD_EINVAL, "concord_peer_alloc: bad arguments");
    *dev_ptr = nullptr;
    cudaError_t e = cudaMalloc(dev_ptr, bytes);
    if (e != cudaSuccess) return fail(CONCORD_ELAUNCH, std::string("concord_peer_alloc: ") + cudaGetErrorString(e));
    e = cudaMemset(*dev_ptr, 0, bytes);
    if (e != cudaSuccess) return fail(CONCORD_ELAUNCH, std::string("concord_peer_alloc: ") + cudaGetErrorString(e));
    return CONCORD_OK;
}

extern "C" int concord_peer_free(void* dev_ptr) {
    if (!dev_ptr) return CONCORD_OK;
    cudaError_t e = cudaFree(dev_ptr);
    if (e != cudaSuccess) return fail(CONCORD_ELAUNCH, std::string("concord_peer_free: ") + cudaGetErrorString(e));
    return CONCORD_OK;
}

extern "C" int concord_ipc_export(void* dev_ptr, void* handle_out) {
    if (!dev_ptr || !handle_out) return fail(CONCORD_EINVAL, "concord_ipc_export: null pointer");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, dev_ptr);
    if (e != cudaSuccess) return fail(CONCORD_ELAUNCH, std::string("concord_ipc_export: ") + cudaGetErrorString(e));
    memcpy(handle_out, &h, sizeof(h));
    return CONCORD_OK;
}

extern "C" int concord_ipc_open(const void* handle, void** dev_ptr) {
    if (!handle || !dev_ptr) return fail(CONCORD_EINVAL, "concord_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *dev_ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(CONCORD_ELAUNCH, std::string("concord_ipc_open: ") + cudaGetErrorString(e));
    return CONCORD_OK;
}

extern "C" int concord_ipc_close(void* dev_ptr) {
    if (!dev_ptr) return CONCORD_OK;
    cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    if (e != cudaSuccess) return fail(CONCORD_ELAUNCH, std::string("concord_ipc_close: ") + cudaGetErrorString(e));
    return CONCORD_OK;
}

extern "C" int concord_peer_push_rows(const uint16_t* grad, int64_t N, int64_t K, int64_t S, const uint64_t* recv,
                                      const concord_peer_sync* sync, void* stream) {
    if (!grad || !recv || !sync || !sync->flags || !sync->peer_flags || !sync->state)
        return fail(CONCORD_EINVAL, "concord_peer_push_rows: null pointer");
    if (sync->n_ranks < 1 || sync->n_ranks > PEER_MAX_RANKS || sync->rank < 0 || sync->rank >= sync->n_ranks)
        return fail(CONCORD_EINVAL, "concord_peer_push_rows: n_ranks must be 1..8 and rank < n_ranks");
    if (N < 0 || K <= 0 || K % 8 != 0 || S <= 0 || S * sync->n_ranks < N)
        return fail(CONCORD_ESHAPE, "concord_peer_push_rows: K must be a positive multiple of 8 and "
                                    "S * n_ranks >= N");
    if (!aligned(grad, 16)) return fail(CONCORD_EALIGN, "concord_peer_push_rows: grad not 16-byte aligned");
    PeerSync s{sync->flags, sync->peer_flags, sync->state, sync->rank, sync->n_ranks, sync->timeout_ns};
    const int64_t kc = K / 8;
    int64_t blocks = (N * kc + PEER_THREADS - 1) / PEER_THREADS;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    if (N * kc < ((int64_t)1 << 31) - (int64_t)blocks * PEER_THREADS * PUSH_UNROLL)
        peer_push_kernel<uint32_t><<<(unsigned)blocks, PEER_THREADS, 0, as_stream(stream)>>>(
            reinterpret_cast<const uint4*>(grad), N, kc, S, recv, s);
    else
        peer_push_kernel<int64_t><<<(unsigned)blocks, PEER_THREADS, 0, as_stream(stream)>>>(
            reinterpret_cast<const uint4*>(grad), N, kc, S, recv, s);
    return check_launch("concord_peer_push_rows");
}
