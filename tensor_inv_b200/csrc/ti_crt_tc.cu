// ti_crt_tc.cu -- K3 with the CRT sums on the tensor cores.
//
// Same result, bit for bit, as crt_kernel (ti_crt.cu) on uint8 t-planes; restates
// src/tensor_inv/crt_matmul.py:62-92 (_crt_precompute, _crt_reconstruct).  For one output
// element with t_i = (r_i * u_i) mod p_i (i < n_mod, written by the residue GEMM's epilogue):
//   S = sum_i t_i * M_i  (mod 2^128),     F = sum_i t_i * f_i,   f_i = round(2^48 / p_i),
// then x = S - floor(F / 2^48 + 1/2) * M and the float64 rounding (crt_finish).
// Written in bytes, M_i = sum_j W[i][j] 2^(8j) (j < 16) and f_i = sum_j W[i][16+j] 2^(8j)
// (j < 6), so with D_j = sum_i t_i * W[i][j]:
//   S = sum_{j<16} D_j 2^(8j),    F = sum_{j<6} D_(16+j) 2^(8j).
// D = T x W is an unsigned 8-bit matrix product with 32-bit accumulators: T holds the t
// bytes of 128 consecutive outputs (M = 128) for 32 moduli slots (K = 32, slots at and above
// n_mod are zero), W is the constant 32 x 32 byte matrix (N = 32, bytes 22..31 zero).
// D_j <= 32 * 254 * 255 < 2^21, so every accumulator is exact.  The tensor cores thus do the
// 128-bit multiply-accumulate work that dominates the SIMT kernel; the epilogue only
// assembles S and F from 22 partial sums and runs crt_finish.
//
// Data movement: the t-planes [n_mod][rows][ldr] are read by TMA as boxes of 128 columns
// x 1 row x 32 moduli (out-of-range moduli zero-filled), which land in shared memory as
// [modulus][128 outputs] rows of 128 bytes with the 128-byte swizzle -- an MN-major operand
// (outputs contiguous, moduli at 128-byte stride), so no transpose is needed.
//
// Roles (two CTAs per SM, persistent over units of 4 rows x 128 columns):
//   warp 0       TMA producer, 5-stage ring of 16 KB stages.
//   warp 1       TMEM allocator (256 columns) + single-thread MMA issuer: 4 MMAs of
//                128 x 32 x 32 per unit into one of 2 accumulator buffers.
//   warps 2..9   epilogue: warp w reads TMEM lane quadrant w % 4 of rows (w - 2) / 4 and
//                (w - 2) / 4 + 2 of the unit, two outputs per thread.
// Every wait is bounded; on timeout the CTA raises an error word, drains its in-flight
// copies and MMAs, frees TMEM and exits.
#include <atomic>
#include <cstring>

#include "ti_crt_math.cuh"

namespace ti {

constexpr int kTcRows = 4;                            // output rows per unit
constexpr int kTcCols = 128;                          // output columns per unit (MMA M)
constexpr int kTcK = 32;                              // moduli slots (MMA K)
constexpr int kTcN = 32;                              // weight bytes (MMA N)
constexpr int kTcStages = 5;
constexpr int kTcRowBytes = kTcK * kTcCols;           // 4096: one row's [32][128] tile
constexpr int kTcStageBytes = kTcRows * kTcRowBytes;  // 16384
constexpr int kTcWBytes = kTcN * 128;                 // W: 32 K-major rows of 128 bytes
constexpr int kTcAcc = 2;                             // TMEM accumulator buffers
constexpr uint32_t kTcAccCols = kTcRows * kTcN;       // 128 columns per buffer
constexpr uint32_t kTcTmemCols = kTcAcc * kTcAccCols; // 256: two CTAs per SM share TMEM
#ifndef TI_CRT_TC_ROWS_PER_THREAD
#define TI_CRT_TC_ROWS_PER_THREAD 2
#endif
constexpr int kTcRowsPerThread = TI_CRT_TC_ROWS_PER_THREAD;  // outputs per epilogue thread
constexpr int kTcEpiWarps = 4 * kTcRows / kTcRowsPerThread;  // one per lane quadrant and row set
constexpr int kTcEpiThreads = 32 * kTcEpiWarps;
constexpr int kTcThreads = 64 + kTcEpiThreads;
// Two CTAs fit on one SM (2 x 85 KB of shared memory, 2 x 256 TMEM columns); with the
// residue GEMM (194 KB) a CTA never shares an SM, so TMEM is never oversubscribed.
constexpr size_t kTcSmemBytes = size_t(kTcStages) * kTcStageBytes + kTcWBytes + 1024 + 256;
constexpr uint32_t kTcIdesc = make_idesc_u8_amn(kTcCols, kTcN);

struct CrtTcParams {
    int64_t rows, cols;
    int64_t col_blocks, row_blocks;
    const int32_t *row_exp, *col_exp;
    double *C;
    int64_t ldc;
    int out_mode;  // 0 store, 1 subtract, 2 add
    int lower;     // skip units entirely above the diagonal
    int *err;
    CrtConst K;
};

// A unit (4 rows x 128 columns) lies entirely above the diagonal: all roles skip it.
__device__ __forceinline__ bool tc_skip(const CrtTcParams &P, int64_t rb, int64_t cb) {
    return P.lower && cb * kTcCols > rb * kTcRows + (kTcRows - 1);
}

__device__ __forceinline__ void tc_raise(const CrtTcParams &P, volatile int *abort, int code) {
    *abort = 1;
    atomicCAS(P.err, 0, code);
}

// Waits (bounded) for a barrier phase that an earlier operation of this CTA will complete,
// so that nothing is in flight when the CTA exits after an abort.
__device__ __forceinline__ void tc_drain_wait(const CrtTcParams &P, uint64_t *bar,
                                              uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            atomicCAS(P.err, 0, kErrTimeoutDrain);
            return;
        }
    }
}

// x = (w3:w2:w1:w0) - q * M  (mod 2^128), with 32-bit carry chains.
__device__ __forceinline__ void sub_q_times_m(uint32_t &w0, uint32_t &w1, uint32_t &w2,
                                              uint32_t &w3, uint32_t q, const uint32_t (&M)[4]) {
    asm("{\n\t.reg .u32 l0, l1, l2, l3, h0, h1, h2;\n\t"
        "mul.lo.u32 l0, %4, %5;\n\t"
        "mul.hi.u32 h0, %4, %5;\n\t"
        "mad.lo.cc.u32 l1, %4, %6, h0;\n\t"
        "madc.hi.u32 h1, %4, %6, 0;\n\t"
        "mad.lo.cc.u32 l2, %4, %7, h1;\n\t"
        "madc.hi.u32 h2, %4, %7, 0;\n\t"
        "mad.lo.u32 l3, %4, %8, h2;\n\t"
        "sub.cc.u32 %0, %0, l0;\n\t"
        "subc.cc.u32 %1, %1, l1;\n\t"
        "subc.cc.u32 %2, %2, l2;\n\t"
        "subc.u32 %3, %3, l3;\n\t}"
        : "+r"(w0), "+r"(w1), "+r"(w2), "+r"(w3)
        : "r"(q), "r"(M[0]), "r"(M[1]), "r"(M[2]), "r"(M[3]));
}

// The float64 output from the MMA's byte sums D[0..21] (each < 2^21) and the exponent sum
// e2 = row_exp + col_exp - 2*bits.  Same value as crt_finish<48> on the same S and F:
//   S = sum_{j<16} D_j 2^(8j) (mod 2^128),  F = sum_{j<6} D_(16+j) 2^(8j),
//   q = floor(F / 2^48 + 1/2),  x = S - q*M (mod 2^128).
// F / 2^48 is within 4064 / 2^48 < 2^-36 of S / M, and S / M is never a half-integer (M is
// odd), so q = round(S / M) unless (F + 2^47) mod 2^48 lies within 2^14 of a multiple of
// 2^48; only then is the exact range check on x (lift_symmetric) needed.  float(x) is rounded
// to nearest-even from its top 64 bits plus a sticky bit, then scaled by 2^e2 with gradual
// underflow.
__device__ __forceinline__ double crt_from_byte_sums(const uint32_t (&D)[32], int e2,
                                                     const CrtConst &K) {
    // S = sum_j (A_j + G_j 2^16) 2^(32j) with A_j = D_4j + D_(4j+1) 2^8 and
    // G_j = D_(4j+2) + D_(4j+3) 2^8 (both < 2^30): the 128-bit sum of A and of G shifted
    // left by 16 bits, added with one carry chain.
    uint32_t A[4], G[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        A[j] = D[4 * j] + (D[4 * j + 1] << 8);
        G[j] = D[4 * j + 2] + (D[4 * j + 3] << 8);
    }
    const uint32_t H0 = G[0] << 16, H1 = __funnelshift_l(G[0], G[1], 16),
                   H2 = __funnelshift_l(G[1], G[2], 16), H3 = __funnelshift_l(G[2], G[3], 16);
    uint32_t w0, w1, w2, w3;
    asm("{\n\tadd.cc.u32 %0, %4, %8;\n\taddc.cc.u32 %1, %5, %9;\n\t"
        "addc.cc.u32 %2, %6, %10;\n\taddc.u32 %3, %7, %11;\n\t}"
        : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
        : "r"(A[0]), "r"(A[1]), "r"(A[2]), "r"(A[3]), "r"(H0), "r"(H1), "r"(H2), "r"(H3));
    // t = F + 2^47 + 2^14 as (thi:tlo), F = Fa + Fb 2^16 + Fc 2^32
    const uint32_t Fa = D[16] + (D[17] << 8), Fb = D[18] + (D[19] << 8),
                   Fc = D[20] + (D[21] << 8);
    uint32_t tlo, thi;
    asm("{\n\tadd.cc.u32 %0, %2, %3;\n\taddc.u32 %1, %4, 0;\n\t}"
        : "=r"(tlo), "=r"(thi)
        : "r"(Fa + (1u << 14)), "r"(Fb << 16), "r"(Fc + (Fb >> 16) + (1u << 15)));
    const uint32_t q = thi >> 16;
    const bool near = tlo < (1u << 15) && (thi & 0xFFFFu) == 0u;
    sub_q_times_m(w0, w1, w2, w3, q, K.M);
    if (near) lift_symmetric(w0, w1, w2, w3, K);
    // |x| and its sign
    const bool neg = (w3 >> 31) != 0;
    uint32_t n0, n1, n2, n3;
    asm("{\n\tsub.cc.u32 %0, %8, %4;\n\tsubc.cc.u32 %1, %8, %5;\n\t"
        "subc.cc.u32 %2, %8, %6;\n\tsubc.u32 %3, %8, %7;\n\t}"
        : "=r"(n0), "=r"(n1), "=r"(n2), "=r"(n3)
        : "r"(w0), "r"(w1), "r"(w2), "r"(w3), "r"(0u));
    const uint32_t a0 = neg ? n0 : w0, a1 = neg ? n1 : w1, a2 = neg ? n2 : w2,
                   a3 = neg ? n3 : w3;
    // top 64 bits below the leading one (|x| < 2^126, so the leading limb is a3 or lower)
    const bool c3 = a3 != 0u;
    const uint32_t top = c3 ? a3 : a2, mid = c3 ? a2 : a1, low = c3 ? a1 : a0;
    const uint32_t rest = c3 ? a0 : 0u;
    const uint32_t sh = static_cast<uint32_t>(__clz(top));  // 32 when |x| < 2^64
    const uint32_t th = __funnelshift_lc(mid, top, sh);
    const uint32_t tl = __funnelshift_lc(low, mid, sh);
    const uint32_t dropped = (low & __funnelshift_rc(0xFFFFFFFFu, 0u, sh)) | rest;
    const uint64_t T = (static_cast<uint64_t>(th) << 32) | tl | (dropped != 0u ? 1u : 0u);
    double d = __ull2double_rn(T);
    if (neg) d = -d;
    const int sc = (c3 ? 64 : 32) - static_cast<int>(sh) + e2;
    // Fast path: with a nonzero top limb T's leading one is bit 63, so d's biased exponent is
    // 1086 (1087 if the rounding carried); if 1086 + sc stays within [2, 2045] the scaled value
    // is normal and exact, and adding sc to the exponent field is the whole ldexp.
    if (top != 0u && sc >= 2 - 1086 && sc <= 2045 - 1086)
        return __longlong_as_double(__double_as_longlong(d) + (static_cast<long long>(sc) << 52));
    return scale_pow2_rne(d, sc);
}

template <int kOutMode>  // 0 store, 1 subtract, 2 add
__global__ void __launch_bounds__(kTcThreads, 2)
    crt_tc_kernel(const __grid_constant__ CUtensorMap tmT, const __grid_constant__ CrtTcParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sT = smem;
    uint8_t *sW = smem + kTcStages * kTcStageBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(sW + kTcWBytes);
    uint64_t *empty = full + kTcStages;
    uint64_t *tfull = empty + kTcStages;  // [kTcAcc] accumulator written
    uint64_t *tempty = tfull + kTcAcc;    // [kTcAcc] accumulator read by the epilogue
    uint64_t *drain = tempty + kTcAcc;    // MMA drain on abort
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // W (K-major, 128-byte swizzle): row n = weight byte, column k = modulus slot.
    for (int i = threadIdx.x; i < kTcWBytes / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(sW)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    for (int i = threadIdx.x; i < kTcN * kTcK; i += blockDim.x) {
        const int n = i / kTcK, k = i - (i / kTcK) * kTcK;
        uint32_t v = 0;
        if (k < P.K.n_mod) {
            if (n < 16) {
                v = (P.K.Mi[k][n >> 2] >> (8 * (n & 3))) & 0xFFu;
            } else if (n < 22) {
                const uint64_t p = P.K.mm.p[k];
                const uint64_t f = ((uint64_t(1) << 48) + p / 2) / p;  // round(2^48 / p)
                v = static_cast<uint32_t>(f >> (8 * (n - 16))) & 0xFFu;
            }
        }
        sW[(n >> 3) * 1024 + (n & 7) * 128 + ((((k >> 4) ^ (n & 7))) << 4) + (k & 15)] =
            static_cast<uint8_t>(v);
    }
    fence_proxy_async_smem();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < kTcAcc; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kTcEpiThreads);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmT);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTcTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, issued_phase = 0;
            bool ok = true;
            for (GridIter it(P.col_blocks); it.a < P.row_blocks; it.next()) {
                if (tc_skip(P, it.a, it.b)) continue;
                const int64_t cb = it.b, r0 = it.a * kTcRows;
                const int nr = P.rows - r0 < kTcRows ? static_cast<int>(P.rows - r0) : kTcRows;
                if (!mbar_wait(&empty[stage], phase ^ 1, abort)) {
                    tc_raise(P, abort, kErrTimeoutProducer);
                    ok = false;
                    break;
                }
                // rows past the matrix are not loaded (their stale bytes give outputs that
                // the epilogue skips); moduli slots >= n_mod are zero-filled by the copy
                mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(nr * kTcRowBytes));
                for (int r = 0; r < nr; ++r)
                    tma_load_3d(sT + stage * kTcStageBytes + r * kTcRowBytes, &tmT, &full[stage],
                                static_cast<int>(cb * kTcCols), static_cast<int>(r0 + r), 0);
                issued_mask |= 1u << stage;
                issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == kTcStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok)
                for (int s = 0; s < kTcStages; ++s)
                    if ((issued_mask >> s) & 1) tc_drain_wait(P, &full[s], (issued_phase >> s) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(sW));
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true, any_issued = false;
            int64_t local = 0;
            for (GridIter it(P.col_blocks); it.a < P.row_blocks; it.next()) {
                if (tc_skip(P, it.a, it.b)) continue;
                const int acc = static_cast<int>(local % kTcAcc);
                const uint32_t acc_phase = static_cast<uint32_t>((local / kTcAcc) & 1);
                ++local;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort) ||
                    !mbar_wait(&full[stage], phase, abort)) {
                    tc_raise(P, abort, kErrTimeoutMma);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(sT + stage * kTcStageBytes);
#pragma unroll
                for (int r = 0; r < kTcRows; ++r)
                    umma_i8(tmem_base + static_cast<uint32_t>(acc) * kTcAccCols + r * kTcN,
                            make_sw128_mnmajor_desc(a0 + r * kTcRowBytes, kTcRowBytes), bdesc,
                            kTcIdesc, 0u);
                any_issued = true;
                umma_commit(&empty[stage]);
                umma_commit(&tfull[acc]);
                if (++stage == kTcStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok && any_issued) {
                umma_commit(drain);
                tc_drain_wait(P, drain, 0);
            }
        }
    } else {
        // ---------------- epilogue (warps 2 .. 2 + kTcEpiWarps) ----------------
        // warp w reads TMEM lane quadrant w % 4 (the unit's columns 32q .. 32q + 31) for the
        // rows r0, r0 + kRowStep, ... of the unit, one output per row and thread.  The
        // exponents of the next unit are loaded while this one is reconstructed, and when C
        // is updated the next unit's outputs are prefetched into L2, so reading their old
        // values does not wait on DRAM (no registers held: K3 is at its register cap).
        constexpr int kRowStep = kTcRows / kTcRowsPerThread;
        const int r0 = (warp - 2) >> 2;
        const int q = warp & 3;
        const int m = q * 32 + lane;  // column within the unit (TMEM lane)
        const CrtConst &K = P.K;
        GridIter it(P.col_blocks);
        while (it.a < P.row_blocks && tc_skip(P, it.a, it.b)) it.next();
        int ce_n = kNonfiniteExp, re_n[kTcRowsPerThread];
        auto load_next = [&](const GridIter &u) {
            const int64_t col = u.b * kTcCols + m;
            ce_n = col < P.cols ? __ldg(P.col_exp + col) : kNonfiniteExp;
#pragma unroll
            for (int k = 0; k < kTcRowsPerThread; ++k) {
                const int64_t row = u.a * kTcRows + r0 + k * kRowStep;
                re_n[k] = row < P.rows ? __ldg(P.row_exp + row) : kNonfiniteExp;
                if (kOutMode != 0 && row < P.rows && col < P.cols)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(P.C + row * P.ldc + col));
            }
        };
        if (it.a < P.row_blocks) load_next(it);
        int64_t local = 0;
        while (it.a < P.row_blocks) {
            const int64_t ua = it.a, ub = it.b;
            const int ce = ce_n;
            int re[kTcRowsPerThread];
#pragma unroll
            for (int k = 0; k < kTcRowsPerThread; ++k) re[k] = re_n[k];
            do {
                it.next();
            } while (it.a < P.row_blocks && tc_skip(P, it.a, it.b));
            if (it.a < P.row_blocks) load_next(it);
            const int acc = static_cast<int>(local % kTcAcc);
            const uint32_t acc_phase = static_cast<uint32_t>((local / kTcAcc) & 1);
            ++local;
            if (!mbar_wait(&tfull[acc], acc_phase, abort)) {
                tc_raise(P, abort, kErrTimeoutEpilogue);
                break;
            }
            tc_fence_after();
            const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                  static_cast<uint32_t>(acc) * kTcAccCols;
            uint32_t D[kTcRowsPerThread][32];
#pragma unroll
            for (int k = 0; k < kTcRowsPerThread; ++k)
                tmem_ld_32x32b_x32(tacc + (r0 + k * kRowStep) * kTcN, D[k]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            const int64_t col = ub * kTcCols + m;
#pragma unroll
            for (int k = 0; k < kTcRowsPerThread; ++k) {
                const int64_t row = ua * kTcRows + r0 + k * kRowStep;
                if (row >= P.rows || col >= P.cols) continue;
                double *dst = P.C + row * P.ldc + col;
                double old = 0.0;
                if (kOutMode != 0) old = *dst;
                const double v = (re[k] == kNonfiniteExp || ce == kNonfiniteExp)
                                     ? nan_value()
                                     : crt_from_byte_sums(D[k], re[k] + ce - K.two_bits, K);
                if (kOutMode == 0) *dst = v;
                else if (kOutMode == 1) *dst = __dsub_rn(old, v);
                else *dst = __dadd_rn(old, v);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, kTcTmemCols);
    }
}

static cudaError_t configure_tc(int dev) {
    static std::atomic<int> configured{-1};  // last device configured
    if (configured.load() == dev) return cudaSuccess;
    for (auto fn : {crt_tc_kernel<0>, crt_tc_kernel<1>, crt_tc_kernel<2>}) {
        const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(kTcSmemBytes));
        if (e != cudaSuccess) return e;
    }
    configured.store(dev);
    return cudaSuccess;
}

// C (op)= CRT of the uint8 t-planes R[i][row][ldr] (plane bytes apart), rows x cols outputs.
// R, ldr and plane must be multiples of 16 bytes.  Returns cudaErrorInvalidValue when the
// tensor map cannot be built.
cudaError_t launch_crt_tc(const uint8_t *R, int64_t ldr, int64_t plane, int64_t rows,
                          int64_t cols, const int32_t *row_exp, const int32_t *col_exp, double *C,
                          int64_t ldc, int out_mode, const CrtConst &K, int *err, int num_sms,
                          cudaStream_t stream, bool lower) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(R) & 15) || (ldr & 15) || (plane & 15) || K.n_mod > kTcK)
        return cudaErrorInvalidValue;
    const EncodeTiledFn enc = get_encode_fn();
    if (!enc) return cudaErrorInvalidValue;
    CUtensorMap tm;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(K.n_mod)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ldr), static_cast<cuuint64_t>(plane)};
    const cuuint32_t box[3] = {kTcCols, 1, kTcK};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(R), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = configure_tc(dev);
    if (e != cudaSuccess) return e;
    CrtTcParams P;
    std::memset(&P, 0, sizeof(P));
    P.rows = rows;
    P.cols = cols;
    P.col_blocks = (cols + kTcCols - 1) / kTcCols;
    P.row_blocks = (rows + kTcRows - 1) / kTcRows;
    const int64_t units = P.row_blocks * P.col_blocks;
    P.row_exp = row_exp;
    P.col_exp = col_exp;
    P.C = C;
    P.ldc = ldc;
    P.out_mode = out_mode;
    P.lower = lower ? 1 : 0;
    P.err = err;
    P.K = K;
    const int64_t grid = units < 2 * int64_t(num_sms) ? units : 2 * int64_t(num_sms);
    const dim3 g(static_cast<unsigned>(grid));
    if (out_mode == 0) crt_tc_kernel<0><<<g, kTcThreads, kTcSmemBytes, stream>>>(tm, P);
    else if (out_mode == 1) crt_tc_kernel<1><<<g, kTcThreads, kTcSmemBytes, stream>>>(tm, P);
    else crt_tc_kernel<2><<<g, kTcThreads, kTcSmemBytes, stream>>>(tm, P);
    return cudaGetLastError();
}

}  // namespace ti
