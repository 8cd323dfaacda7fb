// gemm2sm.cu — the layer's dense GEMMs as 2-SM tcgen05 kernels written here.
//
// D[M,N] (bf16, row-major, leading dimension ldd) = sum_k A(m,k) B(n,k),
// fp32 accumulation in tensor memory, one round-to-nearest-even per output
// (the reference's numerics, concord/packed_b.py:1219, 1263, 1271-1277).
// Each operand is K-major (k contiguous: x and w of the forward, dY of dX)
// or MN-major (m or n contiguous: w of dX, dY and x of dW), described by a
// 2-D TMA tensor map over its global matrix.
//
// Structure: a CTA pair (a 2x1x1 cluster) owns a 256 x 256 output tile and
// walks the reduction in 64-wide k-blocks through a 6-stage shared-memory
// ring.  Each CTA loads its own halves — 128 rows of A and 128 columns of B
// per k-block — with the plain 2-SM form of the TMA tile load (each byte
// lands only in the CTA that issued the copy), whose completion is counted
// on the leader CTA's barrier.
// One thread of the leader issues `tcgen05.mma.cta_group::2` (M=256, N=256,
// K=16) that reads both CTAs' halves and accumulates rows 0-127 into the
// leader's tensor memory and rows 128-255 into the peer's; `tcgen05.commit`
// (multicast to both CTAs' barriers) frees a ring slot once the MMAs reading
// it are done.  Tensor memory holds two 256-column accumulators, so the four
// epilogue warps of each CTA drain one tile (`tcgen05.ld`, bf16 rounding,
// each warp's 32 x 32 pieces staged in shared memory and written by TMA tile
// stores) while the next tile accumulates.  Persistent: pair p takes tiles
// p, p + pairs, ...
//
// Every wait on a barrier is bounded: after 2 s of GPU time it records an
// error word and that role stops; the others then run out too, the pair
// frees its tensor memory and the kernel returns (concord_gemm2sm_error reads
// the word).  No spin without a limit.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "../../include/concord_b200.h"

namespace concord {
int fail(int code, const std::string& msg);
int bind_current_context(const char* name);
}  // namespace concord

namespace g2 {

constexpr int BM = 128;           // rows of A per CTA (256 per pair)
constexpr int BN = 128;           // columns of B per CTA (256 per pair)
constexpr int BK = 64;            // k per stage: 128 bytes of bf16, one swizzle row
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = BN * BK * 2;   // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
// ring depth: 6 stages (192 KB; 7 measured no faster), 5 in the v-hat form
template <bool VHAT>
struct Cfg {
    static constexpr int ST = VHAT ? 5 : 6;
    static constexpr int RING = ST * STAGE_BYTES;
    static constexpr int BAR_OFF = RING;                 // barriers + TMEM slot: 256 B
    static constexpr int VH_OFF = RING + 256;            // v-hat transposition tiles + column sums
    static constexpr int VH_BYTES = VHAT ? (4 * 32 * 33 + 2 * 4 * 256) * 4 : 0;
    static constexpr int STG_OFF = VH_OFF + VH_BYTES;    // output staging: 4 warps x 2 x (32 x 32 bf16)
    static constexpr int STG_BYTES = 4 * 2 * 2048;
    static constexpr size_t SMEM = (size_t)STG_OFF + STG_BYTES + 1024 /* alignment slack */;
};
constexpr int VH_TR_FLOATS = 4 * 32 * 33;
constexpr int THREADS = 192;      // warp 0 TMA, warp 1 MMA / TMEM, warps 2-5 epilogue
constexpr int ACC_COLS = 256;     // fp32 columns of one accumulator
constexpr uint32_t TMEM_COLS = 512;
constexpr uint64_t WAIT_NS = 2000000000ull;   // 2 s of GPU time per wait

struct Params {
    int M, N, K;
    int tiles_m, tiles_n, k_blocks;
    int a_mn, b_mn;        // operand is MN-major
    int n_fastest;         // tile order: n varies fastest
    __nv_bfloat16* D;
    long long ldd;
    int* err;              // error word (0 = fine)
    // v-hat partials of the squared bf16 outputs (VHAT form): rp[n-slab][row]
    // over each row's 256 columns of a tile, cp[128-row block][col] over each
    // CTA's 128 rows
    float* rp;
    float* cp;
    long long ldrp, ldcp;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// bounded wait: false (and the error word set) once WAIT_NS of GPU time have
// passed without the phase completing
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (long long i = 1;; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 255) == 0 && globaltimer_ns() - t0 > WAIT_NS) break;
    }
    atomicCAS(err, 0, code);
    return false;
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// arrive on the barrier at the same offset in CTA `rank` of the cluster
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(bar), "r"(rank));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// 2-SM TMA tile load into this CTA's shared memory; completion bytes are
// counted on the leader's barrier `bar_cluster` (a shared::cluster address)
__device__ __forceinline__ void tma_load_2sm(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                             int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma_2sm(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// arrive once on the barrier at this offset in both CTAs of the pair when
// every MMA issued so far has completed
__device__ __forceinline__ void mma_commit_both(uint32_t bar) {
    const uint16_t mask = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            bar),
        "h"(mask)
        : "memory");
}

// shared-memory matrix descriptor, 128-byte swizzle (sm100 format: start,
// leading / stride byte offsets >> 4, version 1, layout type 2 = SWIZZLE_128B)
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;          // version
    d |= (uint64_t)2 << 61;          // SWIZZLE_128B
    return d;
}

// instruction descriptor: D f32, A/B bf16, majors, N = 256, M = 256
__host__ __device__ constexpr uint32_t instr_desc(int a_mn, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// The operand tile of one CTA and stage: 128 rows (m or n) x 64 k.
// K-major: one TMA box {64 k, 128 rows}: 128 rows of 128 swizzled bytes
//   (8-row groups 1024 B apart: SBO); the k-th 16-wide slice starts 32 B on.
// MN-major: two TMA boxes {64 mn, 64 k} at +0 and +8 KB: 64 k-rows of 128
//   swizzled bytes each (8-row groups 1024 B apart: SBO; the second 64-wide
//   mn block 8 KB on: LBO); the k-th 16-wide slice starts 16 rows = 2 KB on.
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int mn_major, int kk) {
    return mn_major ? smem_desc(base + kk * 2048, 8192, 1024) : smem_desc(base + kk * 32, 16, 1024);
}

__device__ __forceinline__ void load_operand(uint32_t dst, const CUtensorMap* map, int mn_major, uint32_t bar,
                                             int row0, int k0) {
    if (mn_major) {
        tma_load_2sm(dst, map, bar, row0, k0);
        tma_load_2sm(dst + 8192, map, bar, row0 + 64, k0);
    } else {
        tma_load_2sm(dst, map, bar, k0, row0);
    }
}

__device__ __forceinline__ void tile_coords(const Params& P, int t, int& tm, int& tn) {
    if (P.n_fastest) { tn = t % P.tiles_n; tm = t / P.tiles_n; }
    else { tm = t % P.tiles_m; tn = t / P.tiles_m; }
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

template <bool VHAT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm2sm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_d, const __grid_constant__ Params P) {
    using C = Cfg<VHAT>;
    constexpr int STAGES = C::ST;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    // full[STAGES], empty[STAGES], tmem_full[2], tmem_empty[2], then the TMEM base slot
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
    float* vh_tr = reinterpret_cast<float*>(smem + C::VH_OFF);   // VHAT only
    float* vh_cp = vh_tr + VH_TR_FLOATS;
    uint8_t* stg = smem + C::STG_OFF;
    const uint32_t bar0 = smem_u32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto tfull = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto tempty = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();        // 0: leader of the pair
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    const int tiles = P.tiles_m * P.tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(full(s), 1); mbar_init(empty(s), 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(tfull(a), 1); mbar_init(tempty(a), 8); }  // 4 warps x 2 CTAs
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {   // both CTAs' warp 1 allocate the pair's tensor memory together
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t smem_base = smem_u32(smem);

    if (warp == 0) {
        // ---- TMA producer (both CTAs) ----
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            for (int t = pair; t < tiles; t += pairs) {
                int tm, tn;
                tile_coords(P, t, tm, tn);
                const int row_a = tm * 2 * BM + (int)rank * BM;
                const int row_b = tn * 2 * BN + (int)rank * BN;
                for (int kb = 0; kb < P.k_blocks; ++kb) {
                    if (!mbar_wait(empty(s), ph ^ 1, P.err, 1)) goto done;
                    if (rank == 0) mbar_arrive_expect_tx(full(s), 2 * STAGE_BYTES);
                    const uint32_t fb = map_to_rank(full(s), 0);
                    const uint32_t sa = smem_base + s * STAGE_BYTES;
                    load_operand(sa, &map_a, P.a_mn, fb, row_a, kb * BK);
                    load_operand(sa + A_BYTES, &map_b, P.b_mn, fb, row_b, kb * BK);
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issue (leader only) ----
        if (rank == 0 && lane == 0) {
            const uint32_t idesc = instr_desc(P.a_mn, P.b_mn);
            int s = 0;
            uint32_t ph = 0;
            int acc = 0;
            uint32_t aph = 0;
            for (int t = pair; t < tiles; t += pairs) {
                if (!mbar_wait(tempty(acc), aph ^ 1, P.err, 2)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * ACC_COLS);
                for (int kb = 0; kb < P.k_blocks; ++kb) {
                    if (!mbar_wait(full(s), ph, P.err, 3)) goto done;
                    tc_fence_after();
                    const uint32_t sa = smem_base + s * STAGE_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t ad = operand_desc(sa, P.a_mn, kk);
                        const uint64_t bd = operand_desc(sa + A_BYTES, P.b_mn, kk);
                        mma_2sm(d_tmem, ad, bd, idesc, (kb | kk) != 0);
                    }
                    mma_commit_both(empty(s));      // the slot is free once these MMAs are done
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
                mma_commit_both(tfull(acc));        // the accumulator is complete
                if (++acc == 2) { acc = 0; aph ^= 1; }
            }
        }
    } else {
        // ---- epilogue (warps 2-5 of both CTAs): TMEM -> bf16 -> global ----
        const int q = warp & 3;                     // the TMEM lane quadrant this warp may read
        int acc = 0;
        uint32_t aph = 0;
        for (int t = pair; t < tiles; t += pairs) {
            int tm, tn;
            tile_coords(P, t, tm, tn);
            if (!mbar_wait(tfull(acc), aph, P.err, 4)) goto done;
            tc_fence_after();
            const int row = tm * 2 * BM + (int)rank * BM + q * 32 + lane;
            float rsum = 0.0f;
#pragma unroll 1
            for (int c = 0; c < ACC_COLS; c += 32) {
                uint32_t r[32];
                const uint32_t ta = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * ACC_COLS + c);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
                    "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
                    "%30, %31}, [%32];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                      "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                      "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
                      "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
                      "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                    : "r"(ta));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                // the warp's 32 rows x 32 columns as bf16 through a shared staging
                // buffer (two per warp, alternating) and one TMA tile store, which
                // clips what lies beyond M and N
                {
                    uint8_t* sb = stg + (q * 2 + ((c >> 5) & 1)) * 2048;
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                    __syncwarp();
                    uint4* dst = reinterpret_cast<uint4*>(sb + lane * 64);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint4 o;
                        o.x = pack_bf16(__uint_as_float(r[v * 8 + 0]), __uint_as_float(r[v * 8 + 1]));
                        o.y = pack_bf16(__uint_as_float(r[v * 8 + 2]), __uint_as_float(r[v * 8 + 3]));
                        o.z = pack_bf16(__uint_as_float(r[v * 8 + 4]), __uint_as_float(r[v * 8 + 5]));
                        o.w = pack_bf16(__uint_as_float(r[v * 8 + 6]), __uint_as_float(r[v * 8 + 7]));
                        dst[v] = o;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        asm volatile(
                            "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                                reinterpret_cast<uint64_t>(&map_d)),
                            "r"(smem_u32(sb)), "r"(tn * 2 * BN + c), "r"(row - lane)
                            : "memory");
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    }
                }
                if constexpr (VHAT) {
                    // squares of the stored bf16 values (one rounding each); the
                    // row sum in column order; the column sums over this warp's
                    // 32 rows in row order through a transposed tile
                    float* tr = vh_tr + q * (32 * 33);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float v = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[j])));
                        const float sq = __fmul_rn(v, v);
                        rsum = __fadd_rn(rsum, sq);
                        tr[j * 33 + lane] = sq;
                    }
                    __syncwarp();
                    float cs = tr[lane * 33];
#pragma unroll
                    for (int i = 1; i < 32; ++i) cs = __fadd_rn(cs, tr[lane * 33 + i]);
                    vh_cp[(acc * 4 + q) * 256 + c + lane] = cs;
                    __syncwarp();
                }
            }
            tc_fence_before();
            if constexpr (VHAT) {
                const int slab = tn;                     // 256-column slab of the v-hat tiling
                if (row < P.M) P.rp[(long long)slab * P.ldrp + row] = rsum;
                asm volatile("bar.sync 1, 128;" ::: "memory");    // the four epilogue warps' column sums
                const int e = threadIdx.x - 64;
                const int rb = tm * 2 + (int)rank;                // 128-row block of the v-hat tiling
                if (rb * BM < P.M) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int cl = e + h * 128;
                        const float* cpq = vh_cp + acc * 4 * 256 + cl;
                        const float tot = __fadd_rn(__fadd_rn(__fadd_rn(cpq[0], cpq[256]), cpq[512]), cpq[768]);
                        const int gc = tn * 2 * BN + cl;
                        if (gc < P.N) P.cp[(long long)rb * P.ldcp + gc] = tot;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tempty(acc), 0);   // this warp's reads are done
            if (++acc == 2) { acc = 0; aph ^= 1; }
        }
    }
done:
    if (warp >= 2 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // output stores landed
    tc_fence_before();
    __syncthreads();
    cluster_sync();     // no barrier or tensor memory of the pair is used after this
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
    }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// tensor map over a row-major bf16 matrix [rows, cols] (row stride ld
// elements), box {box_inner (cols), box_outer (rows)}, 128-byte swizzle
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_inner,
              int box_outer, bool swizzle = true) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// the error word: a device variable of this module (one per device), found
// by its symbol address on every call, so capture-safe and allocation-free
__device__ int g_err;

int* error_word() {
    int* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_err) != cudaSuccess) return nullptr;
    return p;
}

// CTA pairs of the 2-SM GEMM that can be resident at once (a cluster needs
// two free SMs of one GPC, so this can be below half the SM count)
// Per-device set-up, once per device (a process may drive several GPUs): the
// kernels' shared-memory limit and the number of resident pairs.  Returns the
// pair count, or 0 when the attribute was refused.
constexpr int MAX_DEVICES = 64;
int resident_pairs() {
    static std::atomic<int> pairs_of[MAX_DEVICES];   // 0: not set up yet
    static std::mutex mu;
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= MAX_DEVICES) return 0;
    int n = pairs_of[d].load();
    if (n > 0) return n;
    std::lock_guard<std::mutex> g(mu);
    if ((n = pairs_of[d].load()) > 0) return n;
    if (cudaFuncSetAttribute(gemm2sm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)Cfg<false>::SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(gemm2sm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)Cfg<true>::SMEM) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg<false>::SMEM;
    if (cudaOccupancyMaxActiveClusters(&n, gemm2sm_kernel<false>, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = sms / 2;
    }
    n = std::max(1, std::min(n, sms / 2));
    pairs_of[d].store(n);
    return n;
}

}  // namespace g2

namespace concord {

// D[M,N] = A B^T in the operand layouts described above.  A: K-major [M, K]
// (row stride lda) or MN-major [K, M] (row stride lda); B likewise with N.
// With rp / cp the epilogue also writes the v-hat partials of the squared
// bf16 outputs (rp [ceil(N/256)][ldrp], cp [ceil(M/128)][ldcp]).
int gemm2sm(const void* A, int a_mn, int64_t lda, const void* B, int b_mn, int64_t ldb, void* D, int64_t ldd,
            int64_t M, int64_t N, int64_t K, cudaStream_t stream, const char* name, float* rp, int64_t ldrp,
            float* cp, int64_t ldcp) {
    using namespace g2;
    if (M <= 0 || N <= 0 || K <= 0) return CONCORD_OK;
    if (M % 8 || N % 8 || K % 8 || lda % 8 || ldb % 8 || ldd % 8 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
        return fail(CONCORD_ESHAPE, std::string(name) + ": extents and strides must be multiples of 8");
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(D)) % 16)
        return fail(CONCORD_EALIGN, std::string(name) + ": operands must be 16-byte aligned");
    if (int rc = bind_current_context(name)) return rc;
    CUtensorMap ma, mb, md;
    const bool ok_a = a_mn ? make_map(&ma, A, K, M, lda, 64, 64) : make_map(&ma, A, M, K, lda, 64, 128);
    const bool ok_b = b_mn ? make_map(&mb, B, K, N, ldb, 64, 64) : make_map(&mb, B, N, K, ldb, 64, 128);
    const bool ok_d = make_map(&md, D, M, N, ldd, 32, 32, false);     // output: 32 x 32 tile stores
    if (!ok_a || !ok_b || !ok_d) return fail(CONCORD_ELAUNCH, std::string(name) + ": TMA descriptor encoding failed");
    int* err = error_word();
    if (!err) return fail(CONCORD_ELAUNCH, std::string(name) + ": no error word");
    Params P{};
    P.M = (int)M; P.N = (int)N; P.K = (int)K;
    P.tiles_m = (int)((M + 255) / 256);
    P.tiles_n = (int)((N + 255) / 256);
    P.k_blocks = (int)((K + BK - 1) / BK);
    P.a_mn = a_mn; P.b_mn = b_mn;
    static const int raster = [] {       // 0: n fastest when there are fewer n tiles; 1: m fastest; 2: n fastest
        const char* e = getenv("CONCORD_GEMM2SM_RASTER");
        return e ? atoi(e) : 0;
    }();
    P.n_fastest = raster == 1 ? 0 : raster == 2 ? 1 : (P.tiles_n <= P.tiles_m);
    P.D = reinterpret_cast<__nv_bfloat16*>(D);
    P.ldd = ldd;
    P.err = err;
    P.rp = rp; P.cp = cp; P.ldrp = ldrp; P.ldcp = ldcp;
    const int tiles = P.tiles_m * P.tiles_n;
    const int resident = resident_pairs();
    if (resident <= 0) return fail(CONCORD_ELAUNCH, std::string(name) + ": shared-memory attribute refused");
    const int pairs = std::min(tiles, resident);
    if (rp && cp) gemm2sm_kernel<true><<<2 * pairs, THREADS, Cfg<true>::SMEM, stream>>>(ma, mb, md, P);
    else gemm2sm_kernel<false><<<2 * pairs, THREADS, Cfg<false>::SMEM, stream>>>(ma, mb, md, P);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(CONCORD_ELAUNCH, std::string(name) + ": " + cudaGetErrorString(e));
    return CONCORD_OK;
}

// the error word of the 2-SM GEMMs on the current device (0: no wait ran out)
int gemm2sm_error(int reset) {
    int* err = g2::error_word();
    if (!err) return -1;
    int v = 0;
    cudaMemcpy(&v, err, sizeof(int), cudaMemcpyDeviceToHost);
    if (reset) cudaMemset(err, 0, sizeof(int));
    return v;
}

}  // namespace concord

extern "C" int concord_gemm2sm(const uint16_t* a, int32_t a_mn, int64_t lda, const uint16_t* b, int32_t b_mn,
                                    int64_t ldb, uint16_t* d, int64_t ldd, int64_t M, int64_t N, int64_t K,
                                    void* stream) {
    return concord::gemm2sm(a, a_mn, lda, b, b_mn, ldb, d, ldd, M, N, K, reinterpret_cast<cudaStream_t>(stream),
                            "concord_gemm2sm", nullptr, 0, nullptr, 0);
}

extern "C" int concord_gemm2sm_error(int32_t reset) { return concord::gemm2sm_error(reset); }

extern "C" int concord_gemm2sm_pairs(void) { return g2::resident_pairs(); }
