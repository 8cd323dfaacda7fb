// common.cuh — shared device helpers and C-ABI plumbing for concord_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/concord_b200.h"
#include "crmath.h"

namespace concord {

// ---- error reporting (per host thread) ----
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- element-level helpers shared by the kernels ----
__device__ __forceinline__ int32_t shl32(int32_t v, int s) { return (int32_t)((uint32_t)v << s); }

// numpy-semantics max/min (NaN propagates), as the reference's kernels see them
__device__ __forceinline__ float np_max(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    return a > b ? a : b;
}
__device__ __forceinline__ float np_min(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    return a < b ? a : b;
}

// numpy minimum(maximum(x, -cap), cap) for a finite cap: a NaN x propagates
__device__ __forceinline__ float clamp_np(float x, float cap) {
    return x != x ? x : fminf(fmaxf(x, -cap), cap);
}

__device__ __forceinline__ int32_t clampi(int32_t v, int32_t lo, int32_t hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

// fp32 -> bf16 bits, round to nearest even (quiet NaN kept)
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
__device__ __forceinline__ float bf16_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// 2^e for an integer exponent (exact; the normal range is built from bits)
__device__ __forceinline__ float exp2i(int32_t e) {
    if (e >= -126 && e <= 127) return __uint_as_float((uint32_t)(e + 127) << 23);
    return crmath::cr_exp2f((float)e);
}

// The reference's xorshift SR uniform (packed_b.py:109-117): int32, arithmetic >>.
__device__ __forceinline__ float hash_uniform(int32_t x, int32_t pos, int32_t salt) {
    int32_t h = x ^ salt ^ pos;
    h = h ^ shl32(h, 13);
    h = h ^ (h >> 17);
    h = h ^ shl32(h, 5);
    h = h ^ (h >> 7);
    return __int2float_rn(h & 0xFFFFFF) * (1.0f / 16777216.0f);
}

// ---- the reference's arithmetic as compiled for NVIDIA GPUs ----
// The reference's kernels are Triton; compiled for sm_100 its fp32 `/` is the
// PTX full-range approximate division, tl.exp2 the hardware approximation
// ex2.approx, tl.log2 the CUDA math library's log2f, and a multiply feeding an
// add is contracted into one fma at the sites the step kernel spells out.
// These were identified by comparing outputs with the compiled reference
// on a B200 (every case of the step bit-identical), not by reading any
// compiled code.
__device__ __forceinline__ float div_full(float a, float b) {
    float r;
    asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
    float r;
    asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
// tl.minimum(tl.maximum(x, lo), hi) as compiled: NaN operands are dropped
__device__ __forceinline__ float clamp_gpu(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

// SR tick: floor(d) + (r < frac(d)) truncated to int32 (packed_b.py:596-598)
__device__ __forceinline__ int32_t sr_tick(float d, float r) {
    float fl = floorf(d);
    float fr = __fsub_rn(d, fl);
    return __float2int_rz(__fadd_rn(fl, r < fr ? 1.0f : 0.0f));
}

// Philox4x32-10 on counter (c0,0,0,0) with key (k0,k1): first output word.
// Round constants and key increments are those of Triton's tl.rand
// (triton/language/random.py), which the reference's rebalance uses.
__device__ __forceinline__ uint32_t philox_c0(uint32_t c0, uint32_t k0, uint32_t k1) {
    uint32_t c1 = 0, c2 = 0, c3 = 0;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        uint32_t hi_a = __umulhi(0xD2511F53u, c0), lo_a = 0xD2511F53u * c0;
        uint32_t hi_b = __umulhi(0xCD9E8D57u, c2), lo_b = 0xCD9E8D57u * c2;
        uint32_t n0 = hi_b ^ c1 ^ k0;
        uint32_t n2 = hi_a ^ c3 ^ k1;
        c1 = lo_b; c3 = lo_a; c0 = n0; c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

// tl.rand(seed:int32, offset:int32) -> uniform fp32 in [0,1)
__device__ __forceinline__ float tl_rand(int32_t seed, uint32_t offset) {
    uint64_t s64 = (uint64_t)(int64_t)seed;
    int32_t x = (int32_t)philox_c0(offset, (uint32_t)s64, (uint32_t)(s64 >> 32));
    if (x < 0) x = (int32_t)(~(uint32_t)x);
    return __fmul_rn(__int2float_rn(x), 4.6566127342e-10f);
}

__device__ __forceinline__ int32_t repack(int32_t sf, int32_t ss, int32_t vs) {
    return (int32_t)((((uint32_t)sf & 0xFFFFu) << 16) | (((uint32_t)ss & 0xFFu) << 8) | ((uint32_t)vs & 0xFFu));
}

// max over the full warp (every lane active): one redux.sync instruction
__device__ __forceinline__ int warp_max(int v) { return __reduce_max_sync(0xffffffffu, v); }

}  // namespace concord
