// peer.cuh — cross-GPU rendezvous over peer memory (CUDA IPC mappings).
//
// A kernel that reads or writes other ranks' memory starts with a
// rendezvous: thread 0 of every block stores this launch's epoch into every
// rank's flag array (a system-scope release store after a system fence, so
// the writes of earlier work on this stream are visible first) and then
// polls its own flag array (acquire loads) until every rank has stored the
// epoch.  The poll is bounded by GPU time (%globaltimer); when the limit
// runs out the block sets the caller's error word and reports failure, and
// every later rendezvous on that state fails at once until the caller
// clears the word.  The last block of the launch advances the epoch.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace concord {

constexpr int PEER_MAX_RANKS = 8;

struct PeerSync {
    int32_t* flags;
    const uint64_t* peer_flags;
    int32_t* state;
    int32_t rank, n_ranks;
    int64_t timeout_ns;
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_volatile(const int32_t* p) {
    return *reinterpret_cast<const volatile int32_t*>(p);
}

// Announce and wait (thread 0 of the block); returns false when the wait ran
// out or the error word was already set.  `e` is this launch's epoch.
static __device__ bool peer_rendezvous(const PeerSync& s, int32_t e) {
    __shared__ int ok;
    __syncthreads();              // the block's earlier writes (e.g. pushes into peers) come first
    if (threadIdx.x == 0) {
        __threadfence_system();   // this block's (and, through the barrier, the launch's) writes first
        for (int q = 0; q < s.n_ranks; ++q)
            st_release_sys(reinterpret_cast<int32_t*>(s.peer_flags[q]) + s.rank, e);
        bool good = ld_volatile(s.state + 2) == 0;
        const uint64_t t0 = globaltimer_ns();
        for (int q = 0; q < s.n_ranks && good; ++q) {
            while ((int32_t)(ld_acquire_sys(s.flags + q) - e) < 0) {
                if (ld_volatile(s.state + 2) != 0) { good = false; break; }
                if ((int64_t)(globaltimer_ns() - t0) > s.timeout_ns) {
                    atomicExch(s.state + 2, 1);
                    good = false;
                    break;
                }
                __nanosleep(64);
            }
        }
        ok = good;
    }
    __syncthreads();
    return ok != 0;
}

// Wait only (thread 0 of the block): every rank has announced epoch e.  Used
// after a launch that announced without waiting (the push of a
// reduce-scatter); false when the wait ran out or the error word is set.
static __device__ bool peer_wait(const PeerSync& s, int32_t e) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        bool good = ld_volatile(s.state + 2) == 0;
        const uint64_t t0 = globaltimer_ns();
        for (int q = 0; q < s.n_ranks && good; ++q) {
            while ((int32_t)(ld_acquire_sys(s.flags + q) - e) < 0) {
                if (ld_volatile(s.state + 2) != 0) { good = false; break; }
                if ((int64_t)(globaltimer_ns() - t0) > s.timeout_ns) {
                    atomicExch(s.state + 2, 1);
                    good = false;
                    break;
                }
                __nanosleep(64);
            }
        }
        ok = good;
    }
    __syncthreads();
    return ok != 0;
}

// The last block of the launch stores the epoch for the next launch.
static __device__ void peer_finish(const PeerSync& s, int32_t e) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const int blocks = (int)(gridDim.x * gridDim.y * gridDim.z);
        if (atomicAdd(s.state + 1, 1) == blocks - 1) {   // every block has started and finished
            s.state[1] = 0;
            s.state[0] = e;
            __threadfence();
        }
    }
}

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], const uint4& v) {
    const uint32_t w[4] = {(uint32_t)v.x, (uint32_t)v.y, (uint32_t)v.z, (uint32_t)v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        acc[2 * j] += __uint_as_float(w[j] << 16);
        acc[2 * j + 1] += __uint_as_float(w[j] & 0xffff0000u);
    }
}
__device__ __forceinline__ void set_bf16x8(float (&acc)[8], const uint4& v) {
    const uint32_t w[4] = {(uint32_t)v.x, (uint32_t)v.y, (uint32_t)v.z, (uint32_t)v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        acc[2 * j] = __uint_as_float(w[j] << 16);
        acc[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
}
__device__ __forceinline__ uint4 pack_bf16x8(const float (&acc)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t*>(&b);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

}  // namespace concord
