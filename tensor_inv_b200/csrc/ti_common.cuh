// ti_common.cuh -- shared device helpers for the sm_100a CRT matmul kernels.
//
// Holds the per-modulus constant blocks passed to every kernel by value, the exact small
// modular reductions, and thin inline-PTX wrappers for mbarriers, TMA and tcgen05 (TMEM
// allocation, UMMA issue/commit, TMEM loads).  All waits are bounded by wall time
// (%globaltimer) so a broken pipeline reports an error instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ti {

constexpr int kMaxModuli = 32;
constexpr int kNonfiniteExp = (-2147483647 - 1);
// A kernel wait that lasts this long is treated as a broken pipeline (device error).
constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;

// Device error codes written to the library's error word.
enum : int {
    kErrNone = 0,
    kErrTimeoutProducer = 0x101,
    kErrTimeoutMma = 0x102,
    kErrTimeoutEpilogue = 0x103,
    kErrTimeoutDrain = 0x104,
    kErrTimeoutGridBarrier = 0x105,
};

// Exact reduction a mod p for a < 2^31 and 3 <= p < 256, p not a power of two:
// q = floor(a * magic / 2^(32+shift)) with magic = ceil(2^(32+shift)/p), shift = floor(log2 p).
// The rounding error of the quotient is below a/2^(32+shift) < 2^-(1+shift) < 1/p.
struct ModMagic {
    uint32_t p[kMaxModuli];
    uint32_t magic[kMaxModuli];
    uint32_t shift[kMaxModuli];
    uint32_t off[kMaxModuli];  // p * ceil(2^31 / p): lifts a signed accumulator to [0, 2^32)
};

__device__ __forceinline__ uint32_t mod_small(uint32_t a, uint32_t p, uint32_t magic,
                                              uint32_t shift) {
    uint32_t q = __umulhi(a, magic) >> shift;
    return a - q * p;
}

// acc mod p in [0, p) for a signed int32 accumulator with |acc| <= 2^31 - 256 (passed as
// its bit pattern).  a = acc + off lies in [0, 2^32); for such a the quotient estimate
// above is at most one too large (error below 2^-shift < 2/p), fixed by one add.
__device__ __forceinline__ uint32_t mod_acc(uint32_t acc, uint32_t p, uint32_t magic,
                                            uint32_t shift, uint32_t off) {
    const uint32_t a = acc + off;
    const int32_t r = static_cast<int32_t>(a - (__umulhi(a, magic) >> shift) * p);
    return static_cast<uint32_t>(r < 0 ? r + static_cast<int32_t>(p) : r);
}

// Constants of the split (scale + residue) kernels.
struct SplitConst {
    int n_mod;
    int bits;
    int symmetric;  // 0: floor-mod residues in [0, p) (the reference's _residues);
                    // 1: symmetric residues in [-(p-1)/2, (p-1)/2] (moduli up to 255)
    ModMagic mm;
    // Every residue is written as (mult * x) mod p: mult = 1 for the reference's residues; the
    // matmul path folds the CRT factor u_i = M_i^-1 mod p_i into A's residues, so the residue
    // GEMM's output is already t_i = (u_i * A_i B_i) mod p_i.
    uint32_t mult[kMaxModuli];
    uint32_t w32[kMaxModuli];   // (2^32 mod p) * mult mod p
    uint32_t w16[kMaxModuli];   // (2^16 mod p) * mult mod p
    uint32_t bigp[kMaxModuli];  // p * ceil(2^30 / p): a multiple of p above any piece sum
                                // (a2*w32 + a1*w16 + a0*mult < 2^21*254 + 2*2^16*254 < 2^30)
    uint32_t offs[kMaxModuli];  // p * ceil(568197120 / p): a multiple of p above any |T|
                                // (T = a2*w32 + a1*w16 + a0*mult of signed pieces)
};

// Constants of the CRT reconstruction.  M = prod p_i < 2^127, M_i = M / p_i.
struct CrtConst {
    int n_mod;
    int two_bits;
    ModMagic mm;
    uint32_t u[kMaxModuli];        // (M_i)^-1 mod p_i
    uint32_t finv[kMaxModuli];     // round(2^32 / p_i)
    uint32_t Mi[kMaxModuli][4];    // M_i, little-endian 32-bit words
    uint32_t M[4];
    uint32_t H[4];                 // (M - 1) / 2
    // Moduli in groups of (up to) three consecutive ones, g = i / 3: with P_g the product of
    // a group, c_g = sum_{i in g} t_i * (P_g / p_i) < 3 P_g < 2^26, and
    //   S = sum_g c_g * (M / P_g),   F = sum_g c_g / P_g   (48-bit fixed point)
    // which equal the per-modulus sums with a third of the 128-bit multiply-adds.
    int n_groups;
    uint32_t coef[kMaxModuli];     // P_g / p_i for the group g of modulus i
    uint32_t Mg[kMaxModuli / 3 + 1][4];
    uint32_t fgl[kMaxModuli / 3 + 1], fgh[kMaxModuli / 3 + 1];  // round(2^48 / P_g), lo/hi words
};

// ---------------------------------------------------------------------------------------
// small PTX helpers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
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

// try_wait that lets the hardware suspend the thread for up to `hint_ns` while the phase is
// incomplete (it resumes as soon as the phase completes), so long waits cost few issue slots.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity,
                                                   uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `bar` with the given parity to complete.  Returns false when the
// wait exceeds limit_ns (kWaitTimeoutNs in every kernel; shorter only in the self-test that
// makes a wait run out) or when another role of the CTA raised *abort.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          unsigned long long limit_ns = kWaitTimeoutNs) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_hint(a, parity, 20000u)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// 3-D tiled TMA load global -> shared, completing on `bar` (no multicast).
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map,
                                            uint64_t *bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// 3-D tiled TMA store shared -> global, in the calling thread's bulk async-group.  Boxes
// that reach past the tensor are clipped by the copy engine.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *smem_src, int c0,
                                             int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::
            "l"(reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until at most N of the calling thread's committed bulk groups still read shared
// memory (their source buffers may then be rewritten).
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until at most N of the calling thread's committed bulk groups are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, TMEM accumulators)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, shapes from idesc.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every tcgen05.mma previously issued by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM words: thread t of the warp receives lane
// (base_lane + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte
// swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked at 1024-byte
// stride (SBO), descriptor version 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t make_sw128_kmajor_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

// Shared-memory matrix descriptor for an MN-major 8-bit operand tile stored with the
// 128-byte swizzle: each 128-byte row holds 128 consecutive M (or N) elements of one k,
// rows of consecutive k at 128-byte stride form 1024-byte atoms of 8 k, atoms stacked at
// 1024-byte stride (SBO).  The tile is exactly one atom wide along M, so the leading
// offset (the stride between atoms along M) is never used; it is set to `lbo_bytes`.
__device__ __forceinline__ uint64_t make_sw128_mnmajor_desc(uint32_t saddr, uint32_t lbo_bytes) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) |
           (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

// Shared-memory matrix descriptor for a K-major 8-bit operand tile without swizzle: core
// matrices of 8 rows x 16 bytes (128 contiguous bytes), `lbo` bytes apart along K and
// `sbo` bytes apart along M (or N).  Layout type 0 (SWIZZLE_NONE), descriptor version 1.
__device__ __forceinline__ uint64_t make_noswizzle_kmajor_desc(uint32_t saddr, uint32_t lbo,
                                                               uint32_t sbo) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1) << 46);
}

// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads
// (tensor-core operand fetches) of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Instruction descriptor of tcgen05.mma.kind::i8: D s32, A and B signed 8-bit, both
// K-major, M x N tile.
__host__ __device__ constexpr uint32_t make_idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// Instruction descriptor of tcgen05.mma.kind::i8 with unsigned 8-bit A stored MN-major and
// unsigned 8-bit B stored K-major, D s32, M x N tile.
__host__ __device__ constexpr uint32_t make_idesc_u8_amn(int M, int N) {
    return (2u << 4) | (1u << 15) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// Work units (a, b), b fastest with nb values, strided over a persistent grid
// (unit u = a * nb + b takes u = blockIdx.x, blockIdx.x + gridDim.x, ...), advanced without
// integer division.
struct GridIter {
    int64_t a, b, step_a, step_b, nb;
    __device__ explicit GridIter(int64_t n_b)
        : a(blockIdx.x / n_b), b(blockIdx.x % n_b), step_a(gridDim.x / n_b),
          step_b(gridDim.x % n_b), nb(n_b) {}
    __device__ __forceinline__ void next() {
        a += step_a;
        b += step_b;
        if (b >= nb) {
            b -= nb;
            ++a;
        }
    }
};

// Instruction descriptor of tcgen05.mma.kind::i8 with unsigned 8-bit A and B, both K-major,
// D s32, M x N tile.
__host__ __device__ constexpr uint32_t make_idesc_u8(int M, int N) {
    return (2u << 4) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// 2-D tiled TMA load global -> shared, completing on `bar` (no multicast).
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map,
                                            uint64_t *bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// cuTensorMapEncodeTiled from the driver, looked up once (null if unavailable).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn get_encode_fn();

}  // namespace ti
