// ti_gemm2.cu -- K2 on CTA pairs: the residue GEMMs with tcgen05.mma.cta_group::2.
//
// Same products as residue_gemm_kernel (ti_gemm.cu), which restates
// src/tensor_inv/csrc/crt_kernel.cu:17-91: R[i] = (A_i @ B_i^T) mod p_i for every modulus i.
// A cluster of two CTAs (a CTA pair on one TPC) owns a 256 x 256 output tile per unit:
// CTA r loads rows [128r, 128r+128) of the A tile and rows [128r, 128r+128) of the B tile
// (output columns), and one MMA of M = 256, N = 256, K = 32, issued by CTA 0, multiplies the
// pair's operands: each CTA's TMEM receives its own 128 output rows x 256 columns.  Per CTA
// and stage the copies move 32 KB for 128 x 256 x 128 multiply-adds, a third less than the
// 48 KB of a one-CTA 128 x 256 tile; the freed shared memory deepens the ring to 6 stages.
//
// Roles (both CTAs; one pair per TPC, persistent over units (modulus, tile) in
// modulus-major order, tiles rastered 16 row tiles at a time for L2 reuse):
//   warp 0      TMA producer: its CTA's A and B halves per stage, both completing on CTA
//               0's full barrier (cta_group::2 copies, no multicast); CTA 0 arms the
//               barrier with the pair's bytes.
//   warp 1      TMEM allocation for the pair (512 columns: two 256-column accumulators);
//               in CTA 0, lane 0 issues the MMAs and commits to both CTAs' barriers.
//   warps 2..5  epilogue: tcgen05.ld of this CTA's 128 rows, exact mod p, packed stores;
//               each warp then arrives once on CTA 0's accumulator-empty barrier.
// Every mbarrier wait is bounded; on timeout the CTA raises the error word and leaves its
// loops, and both CTAs meet at the closing cluster barrier before freeing TMEM.
#include <atomic>
#include <cstring>

#include "ti_common.cuh"

namespace ti {

bool make_plane_map(CUtensorMap *map, const void *base, int64_t kdim, int64_t rows, int64_t ld,
                    int64_t planes, int box_rows, int64_t plane_stride);

namespace {

constexpr int kPM = 256, kPN = 256, kPK = 128, kPStages = 6;
constexpr int kPHalf = 128;                          // rows of A and of B per CTA
constexpr int kPABytes = kPHalf * kPK, kPBBytes = kPHalf * kPK;
constexpr int kPStageBytes = kPABytes + kPBBytes;    // 32 KB per CTA
constexpr uint32_t kPTxBytes = 2 * kPStageBytes;     // both CTAs' copies of one stage
constexpr int kPEpiWarps = 4;
constexpr int kPThreads = 64 + 32 * kPEpiWarps;      // 192
constexpr uint32_t kPTmemCols = 512;
constexpr int kPGroupM = 16;  // raster: 16 row tiles (4096 rows); 5.6 GB of DRAM reads at
                              // 8192^3 with 16 moduli, against 9.7 GB for 8 and 10.0 GB for 32
constexpr size_t kPSmemBytes = size_t(kPStages) * kPStageBytes + 1024 + 256;

struct PairParams {
    int64_t m, n;
    int num_kb, n_mod;
    int tiles_m, tiles_n;
    int64_t total_units;
    void *out;
    int64_t ldo, plane;
    int out_i32, lower;
    uint32_t idesc;
    ModMagic mm;
    int *err;
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared::cluster address of the variable at local address `a` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t a, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 3-D TMA load into this CTA's shared memory, completing on the barrier at the
// shared::cluster address `bar` (CTA 0's), as one half of a CTA pair's operand.
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *map, uint32_t bar,
                                                 int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on the barrier at this local offset in both CTAs of the pair when the MMAs
// issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)),
        "h"(static_cast<uint16_t>(3))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void pair_decode(const PairParams &P, int64_t r, int &tm, int &tn) {
    const int64_t per_group = int64_t(kPGroupM) * P.tiles_n;
    const int g = static_cast<int>(r / per_group);
    const int first_m = g * kPGroupM;
    const int gsize = min(kPGroupM, P.tiles_m - first_m);
    const int64_t rg = r - int64_t(g) * per_group;
    tm = first_m + static_cast<int>(rg % gsize);
    tn = static_cast<int>(rg / gsize);
}

// Units of the pair (both CTAs walk the same sequence); f(mod, tm, tn) returns false to stop.
template <class F>
__device__ __forceinline__ void pair_units(const PairParams &P, F &&f) {
    const int64_t per_mod = int64_t(P.tiles_m) * P.tiles_n;
    const int64_t pairs = gridDim.x >> 1;
    for (int64_t u = blockIdx.x >> 1; u < P.total_units; u += pairs) {
        const int mod = static_cast<int>(u / per_mod);
        int tm, tn;
        pair_decode(P, u - int64_t(mod) * per_mod, tm, tn);
        if (P.lower && int64_t(tn) * kPN > int64_t(tm) * kPM + (kPM - 1)) continue;
        if (!f(mod, tm, tn)) return;
    }
}

__device__ __forceinline__ void pair_raise(const PairParams &P, volatile int *abort, int code) {
    *abort = 1;
    atomicCAS(P.err, 0, code);
}

__device__ __forceinline__ void pair_drain(const PairParams &P, uint64_t *bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            atomicCAS(P.err, 0, kErrTimeoutDrain);
            return;
        }
    }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    residue_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ PairParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + kPStages * kPABytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kPStages * kPStageBytes);  // CTA 0
    uint64_t *empty = full + kPStages;   // both CTAs: stage free again
    uint64_t *tfull = empty + kPStages;  // [2] both CTAs: accumulator ready
    uint64_t *tempty = tfull + 2;        // [2] CTA 0: accumulator drained by both epilogues
    uint64_t *drain = tempty + 2;        // CTA 0: MMA drain on abort
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 2 * kPEpiWarps);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kPTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers initialised before any copy or arrive targets them
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;
            bool ok = true;
            pair_units(P, [&](int mod, int tm, int tn) {
                for (int kb = 0; kb < P.num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort)) {
                        pair_raise(P, abort, kErrTimeoutProducer);
                        ok = false;
                        return false;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&full[stage], kPTxBytes);
                    const uint32_t fb = map_to_rank(smem_u32(&full[stage]), 0);
                    tma_load_3d_pair(sA + stage * kPABytes, &tmA, fb, kb * kPK,
                                     tm * kPM + static_cast<int>(rank) * kPHalf, mod);
                    tma_load_3d_pair(sB + stage * kPBBytes, &tmB, fb, kb * kPK,
                                     tn * kPN + static_cast<int>(rank) * kPHalf, mod);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == kPStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                return true;
            });
            if (!ok) {
                // Drain: every issued copy lands before the pair may exit.  CTA 0 sees both
                // CTAs' bytes on its full barriers; CTA 1 waits out the same bound.
                if (rank == 0) {
                    for (int s = 0; s < kPStages; ++s)
                        if ((issued_mask >> s) & 1) pair_drain(P, &full[s], (issued_phase >> s) & 1);
                } else {
                    const unsigned long long t0 = globaltimer_ns();
                    while (globaltimer_ns() - t0 < 1000000ull) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (CTA 0) ----------------
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true, any_issued = false;
            int64_t unit = 0;
            pair_units(P, [&](int, int, int) {
                const int acc = static_cast<int>(unit & 1);
                const uint32_t acc_phase = static_cast<uint32_t>((unit >> 1) & 1);
                ++unit;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort)) {
                    pair_raise(P, abort, kErrTimeoutMma);
                    ok = false;
                    return false;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kPN);
                for (int kb = 0; kb < P.num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort)) {
                        pair_raise(P, abort, kErrTimeoutMma);
                        ok = false;
                        return false;
                    }
                    tc_fence_after();
                    const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(sA + stage * kPABytes));
                    const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(sB + stage * kPBBytes));
#pragma unroll
                    for (int kk = 0; kk < kPK / 32; ++kk)
                        umma_i8_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, P.idesc,
                                     (kb | kk) != 0 ? 1u : 0u);
                    any_issued = true;
                    umma_commit_pair(&empty[stage]);
                    if (++stage == kPStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                umma_commit_pair(&tfull[acc]);
                return true;
            });
            if (!ok && any_issued) {
                umma_commit_pair(drain);
                pair_drain(P, drain, 0);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5, both CTAs) ----------------
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int row_in_half = q * 32 + lane;
        int64_t unit = 0;
        pair_units(P, [&](int mod, int tm, int tn) {
            const int acc = static_cast<int>(unit & 1);
            const uint32_t acc_phase = static_cast<uint32_t>((unit >> 1) & 1);
            ++unit;
            if (!mbar_wait(&tfull[acc], acc_phase, abort)) {
                pair_raise(P, abort, kErrTimeoutEpilogue);
                return false;
            }
            tc_fence_after();
            const int64_t row = int64_t(tm) * kPM + int64_t(rank) * kPHalf + row_in_half;
            const uint32_t p = P.mm.p[mod], magic = P.mm.magic[mod], shift = P.mm.shift[mod];
            const uint32_t off = P.mm.off[mod];
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * kPN);
#pragma unroll 1
            for (int c = 0; c < kPN / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tbase + c * 32, v);
                tmem_wait_ld();
                const int64_t col0 = int64_t(tn) * kPN + c * 32;
                if (row >= P.m || col0 >= P.ldo) {
                    // nothing to store for this lane and chunk
                } else if (!P.out_i32) {
                    uint32_t pk[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        uint32_t w = 0;
#pragma unroll
                        for (int b = 0; b < 4; ++b)
                            w |= mod_acc(v[4 * j + b], p, magic, shift, off) << (8 * b);
                        pk[j] = w;
                    }
                    uint8_t *dst = static_cast<uint8_t *>(P.out) + mod * P.plane + row * P.ldo + col0;
                    *reinterpret_cast<uint4 *>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    if (col0 + 16 < P.ldo)
                        *reinterpret_cast<uint4 *>(dst + 16) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                } else {
                    int32_t *dst = static_cast<int32_t *>(P.out) + mod * P.plane + row * P.ldo;
                    const int ip = static_cast<int>(p);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (col0 + j < P.n) {
                            int r = static_cast<int>(v[j]) % ip;
                            dst[col0 + j] = r < 0 ? r + ip : r;
                        }
                    }
                }
            }
            // the whole warp has read its accumulator rows: one arrive per warp on CTA 0
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(map_to_rank(smem_u32(&tempty[acc]), 0));
            return true;
        });
    }

    // Both CTAs leave their loops before either frees TMEM or exits: CTA 0's MMAs read CTA
    // 1's shared memory and CTA 1's epilogue arrives on CTA 0's barriers.
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kPTmemCols);
    }
}

}  // namespace

// Pairs of CTAs that fit at once (0 when the device cannot run the pair kernel).
static int pair_capacity(int dev) {
    static std::atomic<int> cached_dev{-1};
    static std::atomic<int> cached{0};
    if (cached_dev.load() == dev) return cached.load();
    int n = 0;
    if (cudaFuncSetAttribute(residue_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPSmemBytes)) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * 1024);
        cfg.blockDim = dim3(kPThreads);
        cfg.dynamicSmemBytes = kPSmemBytes;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, residue_gemm_pair_kernel, &cfg) != cudaSuccess)
            n = 0;
    }
    cudaGetLastError();  // a refusal above leaves no sticky error
    cached.store(n);
    cached_dev.store(dev);
    return n;
}

// The pair kernel for R[i] = (A_i @ B_i^T) mod p_i (same arguments and output as
// launch_residue_gemm's unfused mode).  Returns cudaErrorNotSupported when the device cannot
// run CTA pairs or when output weights are asked for (the caller then uses the one-CTA
// kernel, which also writes (r_i * weights[i]) mod p_i).
cudaError_t launch_residue_gemm_pair(const int8_t *a_res, const int8_t *b_res, int64_t m,
                                     int64_t n, int64_t kdim, int64_t ld, int n_mod,
                                     const ModMagic &mm, void *out, int64_t ldo, int out_i32,
                                     int *err, cudaStream_t stream, int64_t a_plane,
                                     int64_t b_plane, int64_t out_plane, const uint32_t *weights,
                                     bool unsigned_ops, bool lower) {
    if (m == 0 || n == 0 || n_mod == 0) return cudaSuccess;
    if (kdim <= 0) return cudaErrorInvalidValue;
    if (weights && !out_i32) return cudaErrorNotSupported;
    int dev = 0;
    cudaGetDevice(&dev);
    const int pairs_max = pair_capacity(dev);
    if (pairs_max < 1) return cudaErrorNotSupported;
    CUtensorMap tmA, tmB;
    if (!make_plane_map(&tmA, a_res, kdim, m, ld, n_mod, kPHalf, a_plane ? a_plane : ld * m) ||
        !make_plane_map(&tmB, b_res, kdim, n, ld, n_mod, kPHalf, b_plane ? b_plane : ld * n))
        return cudaErrorInvalidValue;
    PairParams P;
    std::memset(&P, 0, sizeof(P));
    P.m = m;
    P.n = n;
    P.num_kb = static_cast<int>((kdim + kPK - 1) / kPK);
    P.n_mod = n_mod;
    P.tiles_m = static_cast<int>((m + kPM - 1) / kPM);
    P.tiles_n = static_cast<int>((n + kPN - 1) / kPN);
    P.total_units = int64_t(P.tiles_m) * P.tiles_n * n_mod;
    P.out = out;
    P.ldo = ldo;
    P.plane = out_plane ? out_plane : m * ldo;
    P.out_i32 = out_i32;
    P.lower = lower ? 1 : 0;
    P.idesc = unsigned_ops ? make_idesc_u8(kPM, kPN) : make_idesc_i8(kPM, kPN);
    P.mm = mm;
    P.err = err;
    const int64_t pairs = P.total_units < pairs_max ? P.total_units : pairs_max;
    residue_gemm_pair_kernel<<<static_cast<unsigned>(2 * pairs), kPThreads, kPSmemBytes, stream>>>(
        tmA, tmB, P);
    return cudaGetLastError();
}

}  // namespace ti
