// ti_split_tc.cu -- K1 with the residue arithmetic on the tensor cores.
//
// Same residues, bit for bit, as split_rows_kernel / split_cols_kernel with symmetric
// residues (ti_split.cu); restates src/tensor_inv/crt_matmul.py:32-46 (_scale_to_int,
// _residues) with the representative of each residue in [-(p-1)/2, (p-1)/2].
//
// Per element the scaled integer v = round_half_even(x * 2^(bits - e)), |v| <= 2^53, is
// written as eight unsigned digits: b_0..b_6, the bytes of v mod 2^56, and b_7 = [v < 0], so
//   v = sum_{j<7} b_j 2^(8j) - 2^56 b_7.
// With c_(j,i) = m_i 2^(8j) mod p_i (j < 7) and c_(7,i) = -m_i 2^56 mod p_i, all in [0, p_i)
// (m_i the factor folded into the residues, 1 for plain ones),
//   T_i = sum_j b_j c_(j,i) == m_i v (mod p_i),   0 <= T_i < 8 * 255 * 255 < 2^19,
// an unsigned 8-bit matrix product with 32-bit accumulation.  G element groups share one
// MMA through a block-diagonal weight matrix W[(i, g)][(g', j)] = [g == g'] c_(j,i)
// (M = 128 rows = 128/G moduli slots x G groups, row m = i * G + g; K = 8G bytes) times the
// digit matrix B[(g', j)][n] = digit j of element (g', n) (N = 256).  D[m][n] = T_i of
// element (g, n) lands in TMEM lane m, so each epilogue thread owns one modulus of one group
// and reduces consecutive elements of one vector:
//   symmetric:  r = T - p * round(T / p)  in [-(p-1)/2, (p-1)/2].  The quotient comes from
//               two float32 operations on pairs of lanes: the bit pattern of T read as a
//               float32 is the subnormal T * 2^-149; times 2^100 it is T * 2^-49 exactly,
//               and fma(T * 2^-49, c, 1.5 * 2^23) with c = 2^49 / p rounded to float32
//               (relative error below 2^-23) rounds T / p (1 + e), |e| < 2^-23, to the
//               nearest integer q, held as the low bits of 1.5 * 2^23 + q.  That is exact:
//               T / p is never closer than 1 / (2p) to a half-integer (p is odd) and the
//               error is below T * 2^-23 / p < 1 / (16 p).  Then
//               r = T - p * bits(1.5 * 2^23 + q) (mod 2^8), one integer multiply-add,
//               because bits(1.5 * 2^23) = 0x4B400000 is a multiple of 2^8.
//   floor-mod:  r = T - p * floor(T / p) in [0, p) with the integer quotient
//               umulhi(T, ceil(2^32 / p)), exact for arguments below 2^24.
//
// G = 8 (up to 16 moduli; K = 64, two MMAs of K = 32) or G = 4 (up to 32 moduli; K = 32).
// A unit is G vectors x 256 consecutive k: G rows of a k-contiguous operand or G columns of
// an outer-contiguous one, loaded by one 2-D TMA box of float64 (zero-filled past the
// matrix).  Both operand tiles use the no-swizzle K-major layout: core matrices of 8 rows x
// 16 bytes, 128 bytes apart along K, 8*K bytes apart along M/N.
//
// The residues of a unit leave by TMA: the epilogue writes them to a shared-memory box
// [modulus][vector][128 k] per half unit, rows of 128 bytes in TMEM-lane order with the
// 128-byte swizzle (conflict-free for the row-per-lane writes), and one thread stores both
// halves with 3-D tensor copies that clip rows and columns past the residue planes.
//
// Roles (one CTA per SM, persistent over units; vector blocks outer, k blocks fastest):
//   warp 0       TMA producer: float64 tiles, 4-stage ring.
//   warp 1       TMEM allocator (512 columns) + MMA issuer, 2 accumulators of 256 columns.
//   warps 2..9   digits: scale each element, split it into 8 digits, store the B operand
//                (2-stage ring); two groups of four warps take alternate units.
//   warps 10..25 epilogue: warp w reads TMEM lane quadrant w % 4, column quarter
//                (w - 10) / 4, into a double-buffered staging box; warp 10's lane 0 issues
//                the stores.  (TI_SPLIT_EPI_WARPS=8 at compile time gives 8 warps with
//                column halves: 7 % fewer instructions, no faster at 8192^3: 335 / 352 us
//                against 325 / 364 us for A / B.)
// Every wait is bounded; on timeout the CTA raises an error word, drains its in-flight
// copies and MMAs, frees TMEM and exits.
#include <atomic>
#include <cstring>

#include "ti_scale.cuh"

namespace ti {

constexpr int kSpBoxBytes = 128 * 128;         // staged residues of half a unit
constexpr int kSpStageBytes = 2 * kSpBoxBytes;  // one unit

template <int kG>
struct SplitTcCfg {
    static constexpr int kSlots = 128 / kG;          // moduli slots per element group
    static constexpr int kK = 8 * kG;                // digit bytes per B column (MMA K)
    static constexpr int kN = 256;                   // elements per vector per unit (MMA N)
    static constexpr int kXStages = 4;
    static constexpr int kXBytes = kG * kN * 8;      // float64 tile
    static constexpr int kBStages = 2;
    static constexpr int kBBytes = kN * kK;          // digit tile
    static constexpr int kWBytes = 128 * kK;         // weights
    static constexpr uint32_t kSbo = kK * 8;         // stride of 8-row groups
    static constexpr int kPairs = kG;                // element pairs per digit thread per unit
    static constexpr size_t kUsed = size_t(kXStages) * kXBytes + size_t(kBStages) * kBBytes +
                                    kWBytes + 2 * kSpStageBytes + 1024 + 256;
    // at least 120 KB, so a second CTA (of this kernel, which takes all 512 TMEM columns)
    // never lands on the same SM and waits for TMEM
    static constexpr size_t kSmem = kUsed > 120 * 1024 ? kUsed : 120 * 1024;
};

constexpr int kSpDigitThreads = 128;  // per group; two groups alternate units
#ifndef TI_SPLIT_EPI_WARPS
#define TI_SPLIT_EPI_WARPS 16
#endif
constexpr int kSpEpiWarps = TI_SPLIT_EPI_WARPS;         // a multiple of 4 (lane quadrants)
constexpr int kSpEpiThreads = 32 * kSpEpiWarps;
constexpr int kSpEpiCols = 256 / (kSpEpiWarps / 4);     // unit columns per epilogue thread
constexpr int kSpThreads = 64 + 2 * kSpDigitThreads + kSpEpiThreads;
constexpr uint32_t kSpTmemCols = 512;
constexpr uint32_t kSpIdesc = make_idesc_u8(128, 256);

struct SplitTcParams {
    int64_t outer, kdim, ld_res, plane;
    int64_t vec_blocks, k_blocks;
    const int32_t *exps;
    int8_t *res;
    int bits, n_mod;
    int *err;
    uint32_t p[kMaxModuli];
    uint32_t mult[kMaxModuli];  // factor folded into every residue (1: none)
    float pinv[kMaxModuli];     // 2^49 / p rounded to float32 (p = 3 in the unused slots)
};

__device__ __forceinline__ void sp_raise(const SplitTcParams &P, volatile int *abort, int code) {
    *abort = 1;
    atomicCAS(P.err, 0, code);
}

__device__ __forceinline__ void sp_drain_wait(const SplitTcParams &P, uint64_t *bar,
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

// 2^k as a float64, -1022 <= k <= 1023.
__device__ __forceinline__ double pow2_normal(int k) {
    return __longlong_as_double(static_cast<long long>(k + 1023) << 52);
}

// The eight digits of the scaled element as one little-endian word (0 for a vector with a
// non-finite entry, whose residues are all zero).
// v = round_half_even(x * 2^n), n = bits - e, in float64 arithmetic: |x| < 2^e, so
// |x * 2^n| < 2^bits <= 2^53 and -1016 <= n <= 1049.  For n >= 0 the two power-of-two
// factors (2^min(n,1023), then the rest) only scale up, so both products are exact (no
// overflow; a subnormal x scales exactly).  For n < 0 the single product is exact unless it
// is below 2^-1022, and then both it and the exact value round to 0.  The conversion rounds
// to nearest-even, so v equals the integer-arithmetic result of scaled_magnitude.
__device__ __forceinline__ uint64_t digits8(double x, int bits, int e) {
    if (e == kNonfiniteExp) return 0;
    const int n = bits - e;
    const int n1 = n < 1023 ? n : 1023;
    const double y = (x * pow2_normal(n1)) * pow2_normal(n - n1);
    const long long v = __double2ll_rn(y);
    return (static_cast<uint64_t>(v) & 0x00FFFFFFFFFFFFFFull) | (v < 0 ? (1ull << 56) : 0ull);
}

template <int kG, bool kRows, bool kFloorMod>
__global__ void __launch_bounds__(kSpThreads, 1)
    split_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmR,
                    const __grid_constant__ SplitTcParams P) {
    using Cfg = SplitTcCfg<kG>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // operand tiles first (weights, digits), then the float64 ring, the staged residues
    // (1024-byte aligned: every region before it is a multiple of 1024 bytes) and the barriers
    uint8_t *sW = smem;
    uint8_t *sB = sW + Cfg::kWBytes;
    uint8_t *sX = sB + Cfg::kBStages * Cfg::kBBytes;
    uint8_t *sS = sX + Cfg::kXStages * Cfg::kXBytes;  // [2][kSpStageBytes]
    uint64_t *xfull = reinterpret_cast<uint64_t *>(sS + 2 * kSpStageBytes);
    uint64_t *xempty = xfull + Cfg::kXStages;
    uint64_t *bfull = xempty + Cfg::kXStages;
    uint64_t *bempty = bfull + Cfg::kBStages;
    uint64_t *tfull = bempty + Cfg::kBStages;  // [2]
    uint64_t *tempty = tfull + 2;              // [2]
    uint64_t *sfull = tempty + 2;              // [2] staging box written
    uint64_t *sfree = sfull + 2;               // [2] staging box read by its stores
    uint64_t *drain = sfree + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // weights: row m = i * kG + g, column k = g * 8 + j (zero outside the diagonal blocks
    // and for slots i >= n_mod)
    for (int i = threadIdx.x; i < Cfg::kWBytes / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(sW)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    for (int idx = threadIdx.x; idx < 128 * 8; idx += blockDim.x) {
        const int m = idx >> 3, j = idx & 7;
        const int g = m % kG, i = m / kG;
        if (i >= P.n_mod) continue;
        const uint32_t p = P.p[i];
        uint32_t t = 1;
        for (int s = 0; s < (j < 7 ? j : 7); ++s) t = (t * 256u) % p;  // 2^(8 min(j,7)) mod p
        uint32_t c = j < 7 ? t : (t == 0 ? 0u : p - t);                // j = 7: (-2^56) mod p
        c = (c * P.mult[i]) % p;                                       // the folded factor
        const int k = g * 8 + j;
        sW[(m >> 3) * Cfg::kSbo + (k >> 4) * 128 + (m & 7) * 16 + (k & 15)] =
            static_cast<uint8_t>(c);
    }
    fence_proxy_async_smem();

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kXStages; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&xempty[s], kSpDigitThreads);
        }
        for (int s = 0; s < Cfg::kBStages; ++s) {
            mbar_init(&bfull[s], kSpDigitThreads);
            mbar_init(&bempty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kSpEpiThreads);
            mbar_init(&sfull[a], kSpEpiThreads);
            mbar_init(&sfree[a], 1);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmX);
        prefetch_tensormap(&tmR);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kSpTmemCols);
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
            for (GridIter it(P.k_blocks); it.a < P.vec_blocks; it.next()) {
                const int64_t o0 = it.a * kG, l0 = it.b * Cfg::kN;
                if (!mbar_wait(&xempty[stage], phase ^ 1, abort)) {
                    sp_raise(P, abort, kErrTimeoutProducer);
                    ok = false;
                    break;
                }
                if (l0 < P.kdim) {
                    mbar_arrive_expect_tx(&xfull[stage], Cfg::kXBytes);
                    if (kRows)
                        tma_load_2d(sX + stage * Cfg::kXBytes, &tmX, &xfull[stage],
                                    static_cast<int>(l0), static_cast<int>(o0));
                    else
                        tma_load_2d(sX + stage * Cfg::kXBytes, &tmX, &xfull[stage],
                                    static_cast<int>(o0), static_cast<int>(l0));
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                } else {
                    mbar_arrive(&xfull[stage]);  // padding columns only: no copy, zero digits
                }
                if (++stage == Cfg::kXStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok)
                for (int s = 0; s < Cfg::kXStages; ++s)
                    if ((issued_mask >> s) & 1) sp_drain_wait(P, &xfull[s], (issued_phase >> s) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            const uint32_t w_addr = smem_u32(sW);
            int bs = 0;
            uint32_t bph = 0;
            bool ok = true, any_issued = false;
            int64_t local = 0;
            for (GridIter it(P.k_blocks); it.a < P.vec_blocks; it.next(), ++local) {
                const int acc = static_cast<int>(local & 1);
                const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort) ||
                    !mbar_wait(&bfull[bs], bph, abort)) {
                    sp_raise(P, abort, kErrTimeoutMma);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t b_addr = smem_u32(sB + bs * Cfg::kBBytes);
#pragma unroll
                for (int kk = 0; kk < Cfg::kK / 32; ++kk)  // K = 32 bytes = 2 core matrices
                    umma_i8(tmem_base + static_cast<uint32_t>(acc) * 256u,
                            make_noswizzle_kmajor_desc(w_addr + kk * 256, 128, Cfg::kSbo),
                            make_noswizzle_kmajor_desc(b_addr + kk * 256, 128, Cfg::kSbo),
                            kSpIdesc, kk > 0 ? 1u : 0u);
                any_issued = true;
                umma_commit(&bempty[bs]);
                umma_commit(&tfull[acc]);
                if (++bs == Cfg::kBStages) {
                    bs = 0;
                    bph ^= 1;
                }
            }
            if (!ok && any_issued) {
                umma_commit(drain);
                sp_drain_wait(P, drain, 0);
            }
        }
    } else if (warp < 10) {
        // ---------------- digits (warps 2..9) ----------------
        const int group = (warp - 2) >> 2;                     // takes units j with j % 2 == group
        const int dt = (threadIdx.x - 64) & (kSpDigitThreads - 1);
        int64_t j = 0;
        for (GridIter it(P.k_blocks); it.a < P.vec_blocks; it.next(), ++j) {
            if ((j & 1) != group) continue;
            const int xs = static_cast<int>(j % Cfg::kXStages);
            const uint32_t xph = static_cast<uint32_t>((j / Cfg::kXStages) & 1);
            const int bs = static_cast<int>(j % Cfg::kBStages);
            const uint32_t bph = static_cast<uint32_t>((j / Cfg::kBStages) & 1);
            const int64_t o0 = it.a * kG, l0 = it.b * Cfg::kN;
            if (!mbar_wait(&xfull[xs], xph, abort) || !mbar_wait(&bempty[bs], bph ^ 1, abort)) {
                sp_raise(P, abort, kErrTimeoutEpilogue);
                break;
            }
            const double *X = reinterpret_cast<const double *>(sX + xs * Cfg::kXBytes);
            uint8_t *Bt = sB + bs * Cfg::kBBytes;
            const bool live = l0 < P.kdim;
            // exponents of the groups this thread touches: all kG (rows: a = jp / 2) or the
            // pair 2a, 2a+1 with a = dt % (kG/2) fixed (columns)
            int ex[kG];
#pragma unroll
            for (int g = 0; g < kG; ++g) {
                const bool mine = kRows || (g >> 1) == dt % (kG / 2);
                ex[g] = (mine && o0 + g < P.outer) ? __ldg(P.exps + o0 + g) : kNonfiniteExp;
            }
#pragma unroll
            for (int jp = 0; jp < Cfg::kPairs; ++jp) {
                // element pair (groups 2a and 2a+1, column n): 16 bytes of one B row
                const int pi = dt + kSpDigitThreads * jp;
                const int a = kRows ? (pi >> 8) : (pi % (kG / 2));
                const int n = kRows ? (pi & 255) : (pi / (kG / 2));
                uint64_t d0 = 0, d1 = 0;
                if (live) {
                    double x0, x1;
                    if (kRows) {
                        x0 = X[(2 * a) * Cfg::kN + n];
                        x1 = X[(2 * a + 1) * Cfg::kN + n];
                    } else {
                        const double2 v = *reinterpret_cast<const double2 *>(X + n * kG + 2 * a);
                        x0 = v.x;
                        x1 = v.y;
                    }
                    int e0, e1;
                    if (kRows) {  // a is a compile-time function of jp
                        e0 = ex[2 * (jp >> 1)];
                        e1 = ex[2 * (jp >> 1) + 1];
                    } else {      // a = dt % (kG/2) for every j
                        e0 = kNonfiniteExp;
                        e1 = kNonfiniteExp;
#pragma unroll
                        for (int g = 0; g < kG; g += 2)
                            if ((g >> 1) == a) {
                                e0 = ex[g];
                                e1 = ex[g + 1];
                            }
                    }
                    d0 = digits8(x0, P.bits, e0);
                    d1 = digits8(x1, P.bits, e1);
                }
                *reinterpret_cast<uint4 *>(Bt + (n >> 3) * Cfg::kSbo + a * 128 + (n & 7) * 16) =
                    make_uint4(static_cast<uint32_t>(d0), static_cast<uint32_t>(d0 >> 32),
                               static_cast<uint32_t>(d1), static_cast<uint32_t>(d1 >> 32));
            }
            fence_proxy_async_smem();  // digit stores before the tensor core reads them
            mbar_arrive(&xempty[xs]);
            mbar_arrive(&bfull[bs]);
        }
    } else {
        // ---------------- epilogue (warps 10..25) ----------------
        const int q = warp & 3;                // TMEM lane quadrant this warp may access
        const int col0 = ((warp - 10) >> 2) * kSpEpiCols;  // this warp's columns of the unit
        const int L = q * 32 + lane;           // TMEM lane = weight row m = i * kG + g
        const int slot = L / kG;               // modulus slot i of this lane
        const uint32_t p = slot < P.n_mod ? P.p[slot] : 3u;
        const uint32_t magic = static_cast<uint32_t>(((uint64_t(1) << 32) + p - 1) / p);
        const uint32_t negp = 0u - p;
        const float2 pinv = make_float2(P.pinv[slot], P.pinv[slot]);
        const float2 two100 = make_float2(0x1p100f, 0x1p100f);
        const float2 round23 = make_float2(0x1.8p23f, 0x1.8p23f);
        // this lane's 128-byte row of its half-unit box; 16-byte chunk j of the row sits at
        // chunk j ^ (L & 7) (the store's 128-byte swizzle; L & 7 == lane & 7)
        const int box = col0 >> 7, chunk0 = (col0 & 127) >> 4;
        const bool issuer = warp == 10 && lane == 0;
        int64_t local = 0;
        for (GridIter it(P.k_blocks); it.a < P.vec_blocks; it.next(), ++local) {
            const int acc = static_cast<int>(local & 1);  // accumulator and staging buffer
            const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
            if (!mbar_wait(&tfull[acc], acc_phase, abort) ||
                !mbar_wait(&sfree[acc], acc_phase ^ 1, abort)) {
                sp_raise(P, abort, kErrTimeoutEpilogue);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc) * 256u + col0;
            uint8_t *row = sS + acc * kSpStageBytes + box * kSpBoxBytes + L * 128;
#pragma unroll 1
            for (int c = 0; c < kSpEpiCols / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tbase + c * 32, v);
                tmem_wait_ld();
                if (c == kSpEpiCols / 32 - 1) {  // the accumulator is fully read
                    tc_fence_before();
                    mbar_arrive(&tempty[acc]);
                }
                uint32_t pk[8];
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    uint32_t r[4];
                    if (kFloorMod) {
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const uint32_t T = v[4 * w + b];
                            r[b] = T - __umulhi(T, magic) * p;  // low byte
                        }
                    } else {
#pragma unroll
                        for (int b = 0; b < 4; b += 2) {
                            const float2 x = make_float2(__uint_as_float(v[4 * w + b]),
                                                         __uint_as_float(v[4 * w + b + 1]));
                            const float2 qv = __ffma2_rn(__fmul2_rn(x, two100), pinv, round23);
                            r[b] = v[4 * w + b] + negp * __float_as_uint(qv.x);  // low byte
                            r[b + 1] = v[4 * w + b + 1] + negp * __float_as_uint(qv.y);
                        }
                    }
                    pk[w] = __byte_perm(__byte_perm(r[0], r[1], 0x0040),
                                        __byte_perm(r[2], r[3], 0x0040), 0x5410);
                }
                const int j0 = chunk0 + 2 * c;
                *reinterpret_cast<uint4 *>(row + ((j0 ^ (lane & 7)) << 4)) =
                    make_uint4(pk[0], pk[1], pk[2], pk[3]);
                *reinterpret_cast<uint4 *>(row + (((j0 + 1) ^ (lane & 7)) << 4)) =
                    make_uint4(pk[4], pk[5], pk[6], pk[7]);
            }
            fence_proxy_async_smem();  // staged residues before the copy engine reads them
            mbar_arrive(&sfull[acc]);
            if (issuer) {
                if (!mbar_wait(&sfull[acc], acc_phase, abort)) {
                    sp_raise(P, abort, kErrTimeoutEpilogue);
                    break;
                }
                const int x0 = static_cast<int>(it.b * Cfg::kN);
                const int y0 = static_cast<int>(it.a * kG);
                uint8_t *box0 = sS + acc * kSpStageBytes;
                tma_store_3d(&tmR, box0, x0, y0, 0);
                if (x0 + 128 < P.ld_res) tma_store_3d(&tmR, box0 + kSpBoxBytes, x0 + 128, y0, 0);
                bulk_commit_group();
                bulk_wait_group_read<1>();  // the previous unit's boxes are read
                if (local > 0) mbar_arrive(&sfree[acc ^ 1]);
            }
        }
        if (issuer) bulk_wait_group<0>();  // every store complete before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, kSpTmemCols);
    }
}

template <int kG, bool kRows, bool kFloorMod>
static cudaError_t launch_split_tc_t(const CUtensorMap &tm, const CUtensorMap &tr,
                                     const SplitTcParams &P, int num_sms, cudaStream_t stream) {
    static std::atomic<int> configured{-1};  // last device configured
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured.load() != dev) {
        const cudaError_t e = cudaFuncSetAttribute(split_tc_kernel<kG, kRows, kFloorMod>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(SplitTcCfg<kG>::kSmem));
        if (e != cudaSuccess) return e;
        configured.store(dev);
    }
    const int64_t units = P.vec_blocks * P.k_blocks;
    const int64_t grid = units < num_sms ? units : num_sms;
    split_tc_kernel<kG, kRows, kFloorMod><<<static_cast<unsigned>(grid), kSpThreads,
                                            SplitTcCfg<kG>::kSmem, stream>>>(tm, tr, P);
    return cudaGetLastError();
}

// Residues of one operand (exponents already in `exps`) on the tensor cores: symmetric, or
// floor-mod in [0, p) as unsigned bytes when C.symmetric is 0.
// X is outer vectors of kdim elements, element (o, l) at X[o*s_outer + l*s_k], with either
// s_k == 1 (rows) or s_outer == 1 (columns).  Writes res[i*plane + o*ld_res + l] for
// l < ld_res (zero for l >= kdim).  Returns cudaErrorNotSupported when the layout does not
// suit the 2-D copies (misaligned base or odd stride): the SIMT kernels cover that case.
cudaError_t launch_split_tc(const double *X, int64_t outer, int64_t kdim, int64_t s_outer,
                            int64_t s_k, const SplitConst &C, const int32_t *exps, int8_t *res,
                            int64_t ld_res, int64_t plane, int *err, int num_sms,
                            cudaStream_t stream) {
    if (outer == 0) return cudaSuccess;
    const bool rows = (s_k == 1);
    const int64_t stride = rows ? s_outer : s_k;
    if (C.n_mod > kMaxModuli || kdim < 1 ||
        (reinterpret_cast<uintptr_t>(X) & 15) || (stride & 1) || stride < 2 ||
        stride >= (int64_t(1) << 36) || (!rows && s_outer != 1) || (ld_res & 15) ||
        (plane & 15) || (reinterpret_cast<uintptr_t>(res) & 15) || ld_res >= (int64_t(1) << 30) ||
        outer >= (int64_t(1) << 30) || plane >= (int64_t(1) << 39))
        return cudaErrorNotSupported;
    const EncodeTiledFn enc = get_encode_fn();
    if (!enc) return cudaErrorNotSupported;
    const int G = C.n_mod <= 16 ? 8 : 4;
    CUtensorMap tm;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(rows ? kdim : outer),
                                static_cast<cuuint64_t>(rows ? outer : kdim)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 8};
    const cuuint32_t box[2] = {rows ? 256u : static_cast<cuuint32_t>(G),
                               rows ? static_cast<cuuint32_t>(G) : 256u};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double *>(X), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorNotSupported;
    // residue planes [modulus][outer][ld_res] bytes, stored by boxes of 128 k x G vectors x
    // all moduli
    CUtensorMap tr;
    const cuuint64_t rdims[3] = {static_cast<cuuint64_t>(ld_res), static_cast<cuuint64_t>(outer),
                                 static_cast<cuuint64_t>(C.n_mod)};
    const cuuint64_t rstrides[2] = {static_cast<cuuint64_t>(ld_res),
                                    static_cast<cuuint64_t>(plane)};
    const cuuint32_t rbox[3] = {128u, static_cast<cuuint32_t>(G),
                                static_cast<cuuint32_t>(C.n_mod)};
    const cuuint32_t restr[3] = {1, 1, 1};
    if (enc(&tr, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, res, rdims, rstrides, rbox, restr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorNotSupported;
    SplitTcParams P;
    std::memset(&P, 0, sizeof(P));
    P.outer = outer;
    P.kdim = kdim;
    P.ld_res = ld_res;
    P.plane = plane;
    P.vec_blocks = (outer + G - 1) / G;
    P.k_blocks = (ld_res + 255) / 256;
    P.exps = exps;
    P.res = res;
    P.bits = C.bits;
    P.n_mod = C.n_mod;
    P.err = err;
    for (int i = 0; i < kMaxModuli; ++i) {
        const uint32_t pi = i < C.n_mod ? C.mm.p[i] : 3u;
        P.p[i] = i < C.n_mod ? pi : 0u;
        P.mult[i] = i < C.n_mod ? C.mult[i] : 0u;
        P.pinv[i] = static_cast<float>(0x1p49 / static_cast<double>(pi));
    }
#define TI_SPLIT_TC(GG, FM)                                                               \
    return rows ? launch_split_tc_t<GG, true, FM>(tm, tr, P, num_sms, stream)             \
                : launch_split_tc_t<GG, false, FM>(tm, tr, P, num_sms, stream);
    if (G == 8) {
        if (C.symmetric) { TI_SPLIT_TC(8, false) }
        TI_SPLIT_TC(8, true)
    }
    if (C.symmetric) { TI_SPLIT_TC(4, false) }
    TI_SPLIT_TC(4, true)
#undef TI_SPLIT_TC
}

}  // namespace ti
