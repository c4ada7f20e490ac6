// ti_gemm.cu -- K2: the per-modulus residue GEMMs as one persistent tcgen05 kernel, with an
// optional fused CRT stage (K2+K3).
//
// Restates src/tensor_inv/csrc/crt_kernel.cu:17-91 (cuBLASLt batched int8 GEMM followed by
// the mod_reduce kernel, crt_kernel.cu:6-15):
//   R[i] = (A_i @ B_i^T) mod p_i   for every modulus i,
// with A_i (rows x K) and B_i (cols x K) int8 residue planes stored K-major.
//
// Roles (one CTA per SM, persistent):
//   warp 0      TMA producer: 128x128-byte A tile + 256x128-byte B tile per stage,
//               4-stage mbarrier ring, 128-byte swizzle, no multicast.
//   warp 1      TMEM allocator + single-thread tcgen05.mma.kind::i8 issuer, M=128 N=256
//               K=32 per instruction, int32 accumulators in TMEM, double-buffered
//               (2 x 256 columns = all 512 TMEM columns).
//   warps 2..9  epilogue: tcgen05.ld 32 rows x 32 columns at a time, exact mod p, pack.  With
//               a short K loop (k <= 512, e.g. the trailing updates of LU and Cholesky) the
//               epilogue and not the MMA bounds a tile, so all 8 warps work, two per TMEM lane
//               quadrant with 128 columns each; otherwise warps 2..5 take whole tile rows and
//               warps 6..9 idle (fewer warps polling beside the MMA issuer).
//   warps 10..13 (fused mode only) CRT: exact reconstruction of a finished output tile.
//
// Unfused mode: work units are (modulus, tile) in modulus-major order; the epilogue writes
// uint8 residue planes R[i][m][ldo] (or int32 planes) that K3 (ti_crt.cu) consumes.
// Fused mode: each CTA takes whole 128x256 output tiles and runs all N moduli of a tile
// back to back.  The epilogue stores t_i = (r_i * u_i) mod p_i for every modulus into one
// of two per-CTA scratch slots ([N][128][256] bytes); after the last modulus the CRT warps
// rebuild the float64 tile from that slot while the tensor cores move on to the next tile,
// so the reconstruction hides behind the MMA.
//
// Every wait is bounded; on timeout the CTA raises an error word, drains its in-flight
// copies and MMAs, frees TMEM and exits.
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "ti_crt_math.cuh"

namespace ti {

constexpr int kBM = 128, kBN = 256, kBK = 128, kStages = 4;
constexpr int kABytes = kBM * kBK, kBBytes = kBN * kBK, kStageBytes = kABytes + kBBytes;
constexpr int kEpiThreads = 256, kCrtThreads = 128;
constexpr int kEpiWarpEnd = 2 + kEpiThreads / 32;  // epilogue warps are 2 .. kEpiWarpEnd-1
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kIdesc = make_idesc_i8(kBM, kBN);
constexpr int kGroupM = 16;  // tile raster: 16 row-tiles per group for L2 reuse
constexpr size_t kGemmSmemBytes = size_t(kStages) * kStageBytes + 1024 /*align*/ + 256 /*bars*/;
constexpr int64_t kSlotPlaneBytes = int64_t(kBM) * kBN;  // one modulus of one tile, uint8

__host__ __device__ constexpr int gemm_threads(bool fused) {
    return 64 + kEpiThreads + (fused ? kCrtThreads : 0);
}

struct GemmParams {
    int64_t m, n;      // output rows / columns per modulus
    int num_kb;        // K blocks of 128 bytes
    int n_mod;
    int tiles_m, tiles_n;
    int64_t total_units;  // n_mod * tiles_m * tiles_n
    // unfused output
    void *out;         // uint8 [n_mod][m][ldo] or int32 [n_mod][m][ldo]
    int64_t ldo;       // elements; multiple of 16 for uint8 output
    int64_t plane;     // elements between moduli planes
    int out_i32;       // 0: uint8 residues (|accumulator| <= 2^31 - 256); 1: int32, any int8
    int store_t;       // uint8 output holds t = (r * crt.u[i]) mod p instead of r
    uint32_t idesc;    // MMA instruction descriptor: signed or unsigned 8-bit operands
    int lower;         // unfused: skip output tiles entirely above the diagonal
    int epi_warps;     // 8 when the K loop is short (the epilogue bounds the tile), else 4
    // |accumulator| < 2^22 - 256 (short K loops): r = acc mod p from a rounded float32
    // quotient of T = acc + qofs[i] (0 <= T < 2^23): q = round(T / p) from
    // fma(T * 2^-49, qinv[i], qmagic[i]) (T read as the subnormal T * 2^-149, times 2^100;
    // qinv = 2^49 / p correctly rounded, so the quotient is exact for T < 2^23), and
    // r = T - p * bits(q) (mod 2^8), qmagic = 1.5 * 2^23 + kappa with p * kappa == -h
    // (mod 2^8) so the byte is (acc + qofs + h) - p * q = acc mod p, h = (p - 1) / 2.
    int small_acc;
    uint32_t qofs[kMaxModuli];
    float qinv[kMaxModuli];
    float qmagic[kMaxModuli];
    // fused output
    uint8_t *scratch;  // 2 slots x n_mod x 128 x 256 bytes per CTA
    const int32_t *row_exp, *col_exp;
    double *C;
    int64_t ldc;
    int out_mode;      // 0 store, 1 subtract, 2 add
    ModMagic mm;
    CrtConst crt;      // fused mode: reconstruction constants (crt.u also used by epilogue)
    int *err;
};

__device__ __forceinline__ void decode_tile(const GemmParams &P, int64_t r, int &tm, int &tn) {
    const int64_t per_group = int64_t(kGroupM) * P.tiles_n;
    const int g = static_cast<int>(r / per_group);
    const int first_m = g * kGroupM;
    const int gsize = min(kGroupM, P.tiles_m - first_m);
    const int64_t rg = r - int64_t(g) * per_group;
    tm = first_m + static_cast<int>(rg % gsize);
    tn = static_cast<int>(rg / gsize);
}

// Work-unit order seen by every role of one CTA.  Unfused: units strided over the grid in
// modulus-major order.  Fused: output tiles strided over the grid, all moduli of a tile
// consecutively.  f(mod, tm, tn, tile_local) returns false to stop.
template <bool kFused, class F>
__device__ __forceinline__ void for_each_unit(const GemmParams &P, F &&f) {
    if (!kFused) {
        const int64_t per_mod = int64_t(P.tiles_m) * P.tiles_n;
        for (int64_t u = blockIdx.x; u < P.total_units; u += gridDim.x) {
            const int mod = static_cast<int>(u / per_mod);
            int tm, tn;
            decode_tile(P, u - int64_t(mod) * per_mod, tm, tn);
            // every role skips the same tiles (first column past the last row)
            if (P.lower && int64_t(tn) * kBN > int64_t(tm) * kBM + (kBM - 1)) continue;
            if (!f(mod, tm, tn, int64_t(0))) return;
        }
    } else {
        const int64_t tiles = int64_t(P.tiles_m) * P.tiles_n;
        int64_t local = 0;
        for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
            int tm, tn;
            decode_tile(P, t, tm, tn);
            for (int mod = 0; mod < P.n_mod; ++mod)
                if (!f(mod, tm, tn, local)) return;
        }
    }
}

__device__ __forceinline__ void raise_error(const GemmParams &P, volatile int *abort, int code) {
    *abort = 1;
    atomicCAS(P.err, 0, code);
}

// CRT of one finished 128 x 256 tile from scratch slot `slot` ([n_mod][128][256] bytes of t_i).
// CRT thread ct (0..127): warp w = ct / 32 takes rows w, w+4, ...; lane l takes 4 columns.
__device__ __forceinline__ void crt_tile(const GemmParams &P, const uint8_t *slot, int tm, int tn,
                                         int ct) {
    const int w = ct >> 5, lane = ct & 31;
    const CrtConst &K = P.crt;
    const bool vec_out = ((reinterpret_cast<uintptr_t>(P.C) & 15) == 0) && ((P.ldc & 1) == 0);
#pragma unroll 1
    for (int it = w; it < kBM * 2; it += 4) {
        const int r = it >> 1, half = it & 1;
        const int64_t row = int64_t(tm) * kBM + r;
        if (row >= P.m) continue;  // warp-uniform
        const int cl = half * 128 + lane * 4;
        const int64_t col = int64_t(tn) * kBN + cl;
        if (col >= P.n) continue;
        const uint8_t *src = slot + r * kBN + cl;
        // all moduli's residue words in flight at once (the slot is read once, from L2)
        uint32_t w4[kMaxModuli];
#pragma unroll
        for (int i = 0; i < kMaxModuli; ++i)
            w4[i] = i < K.n_mod ? __ldcg(reinterpret_cast<const unsigned int *>(src + i * kSlotPlaneBytes))
                                : 0u;
        uint64_t s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0}, s2[4] = {0, 0, 0, 0},
                 s3[4] = {0, 0, 0, 0}, f[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < kMaxModuli; ++i) {
            if (i >= K.n_mod) break;
            const uint32_t m0 = K.Mi[i][0], m1 = K.Mi[i][1], m2 = K.Mi[i][2], m3 = K.Mi[i][3];
            const uint32_t fi = K.finv[i];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t t = (w4[i] >> (8 * e)) & 0xFFu;
                s0[e] += static_cast<uint64_t>(t) * m0;
                s1[e] += static_cast<uint64_t>(t) * m1;
                s2[e] += static_cast<uint64_t>(t) * m2;
                s3[e] += static_cast<uint64_t>(t) * m3;
                f[e] += static_cast<uint64_t>(t) * fi;
            }
        }
        const int re = P.row_exp[row];
        const int nc = P.n - col < 4 ? static_cast<int>(P.n - col) : 4;
        double outv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int ce = e < nc ? P.col_exp[col + e] : 0;
            outv[e] = (re == kNonfiniteExp || ce == kNonfiniteExp)
                          ? nan_value()
                          : crt_finish(s0[e], s1[e], s2[e], s3[e], f[e], re + ce - K.two_bits, K);
        }
        double *dst = P.C + row * P.ldc + col;
        if (nc == 4 && vec_out && P.out_mode == 0) {
            reinterpret_cast<double2 *>(dst)[0] = make_double2(outv[0], outv[1]);
            reinterpret_cast<double2 *>(dst)[1] = make_double2(outv[2], outv[3]);
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < nc) write_mode(dst + e, outv[e], P.out_mode);
        }
    }
}

template <bool kFused>
__global__ void __launch_bounds__(gemm_threads(kFused), 1)
    residue_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ GemmParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + kStages * kABytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
    uint64_t *empty = full + kStages;
    uint64_t *tfull = empty + kStages;   // [2] accumulator ready
    uint64_t *tempty = tfull + 2;        // [2] accumulator drained by the epilogue
    uint64_t *drain = tempty + 2;        // MMA drain on abort
    uint64_t *sfull = drain + 1;         // [2] scratch slot complete (fused)
    uint64_t *sempty = sfull + 2;        // [2] scratch slot consumed by the CRT warps (fused)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sempty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 32 * P.epi_warps);
            mbar_init(&sfull[a], 32 * P.epi_warps);
            mbar_init(&sempty[a], kCrtThreads);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
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
            uint32_t phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;
            bool ok = true;
            for_each_unit<kFused>(P, [&](int mod, int tm, int tn, int64_t) {
                for (int kb = 0; kb < P.num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort)) {
                        raise_error(P, abort, kErrTimeoutProducer);
                        ok = false;
                        return false;
                    }
                    mbar_arrive_expect_tx(&full[stage], kStageBytes);
                    tma_load_3d(sA + stage * kABytes, &tmA, &full[stage], kb * kBK, tm * kBM, mod);
                    tma_load_3d(sB + stage * kBBytes, &tmB, &full[stage], kb * kBK, tn * kBN, mod);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                return true;
            });
            if (!ok) {
                // Drain: every issued copy must land before the CTA may exit.
                for (int s = 0; s < kStages; ++s) {
                    if (!((issued_mask >> s) & 1)) continue;
                    const uint32_t a = smem_u32(&full[s]);
                    const unsigned long long t0 = globaltimer_ns();
                    while (!mbar_try_wait(a, (issued_phase >> s) & 1)) {
                        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                            atomicCAS(P.err, 0, kErrTimeoutDrain);
                            break;
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true, any_issued = false;
            int64_t unit = 0;
            for_each_unit<kFused>(P, [&](int, int, int, int64_t) {
                const int acc = static_cast<int>(unit & 1);
                const uint32_t acc_phase = static_cast<uint32_t>((unit >> 1) & 1);
                ++unit;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort)) {
                    raise_error(P, abort, kErrTimeoutMma);
                    ok = false;
                    return false;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
                for (int kb = 0; kb < P.num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort)) {
                        raise_error(P, abort, kErrTimeoutMma);
                        ok = false;
                        return false;
                    }
                    tc_fence_after();
                    const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(sA + stage * kABytes));
                    const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(sB + stage * kBBytes));
#pragma unroll
                    for (int kk = 0; kk < kBK / 32; ++kk) {
                        // advance the start address by 32 bytes (2 x 16-byte units) per K step
                        umma_i8(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, P.idesc,
                                (kb | kk) != 0 ? 1u : 0u);
                    }
                    any_issued = true;
                    umma_commit(&empty[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                umma_commit(&tfull[acc]);
                return true;
            });
            if (!ok && any_issued) {
                umma_commit(drain);
                const uint32_t a = smem_u32(drain);
                const unsigned long long t0 = globaltimer_ns();
                while (!mbar_try_wait(a, 0)) {
                    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                        atomicCAS(P.err, 0, kErrTimeoutDrain);
                        break;
                    }
                }
            }
        }
    } else if (warp < 2 + P.epi_warps) {
        // ---------------- epilogue (warps 2..9) ----------------
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int row_in_tile = q * 32 + lane;
        // 8 warps: two per quadrant, 4 column chunks each; 4 warps: all 8 chunks
        const int c_count = P.epi_warps == 8 ? kBN / 64 : kBN / 32;
        const int c_begin = ((warp - 2) >> 2) * c_count;
        int64_t unit = 0;
        for_each_unit<kFused>(P, [&](int mod, int tm, int tn, int64_t tile_local) {
            const int acc = static_cast<int>(unit & 1);
            const uint32_t acc_phase = static_cast<uint32_t>((unit >> 1) & 1);
            ++unit;
            const int slot_idx = static_cast<int>(tile_local & 1);
            const uint32_t slot_phase = static_cast<uint32_t>((tile_local >> 1) & 1);
            if (kFused && mod == 0) {  // the slot must have been consumed by the CRT warps
                if (!mbar_wait(&sempty[slot_idx], slot_phase ^ 1, abort)) {
                    raise_error(P, abort, kErrTimeoutEpilogue);
                    return false;
                }
            }
            if (!mbar_wait(&tfull[acc], acc_phase, abort)) {
                raise_error(P, abort, kErrTimeoutEpilogue);
                return false;
            }
            tc_fence_after();
            const int64_t row = int64_t(tm) * kBM + row_in_tile;
            const uint32_t p = P.mm.p[mod], magic = P.mm.magic[mod], shift = P.mm.shift[mod];
            const uint32_t off = P.mm.off[mod];
            const uint32_t u = kFused ? P.crt.u[mod] : 0u;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * kBN);
            uint8_t *slot_row =
                kFused ? P.scratch + (int64_t(blockIdx.x) * 2 + slot_idx) * P.n_mod * kSlotPlaneBytes +
                             int64_t(mod) * kSlotPlaneBytes + int64_t(row_in_tile) * kBN
                       : nullptr;
#pragma unroll 1
            for (int c = c_begin; c < c_begin + c_count; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tbase + c * 32, v);
                tmem_wait_ld();
                const int64_t col0 = int64_t(tn) * kBN + c * 32;
                if (kFused) {
                    // t = (r * u) mod p with r = acc mod p; the whole tile row is stored (rows
                    // and columns past the matrix are skipped by the CRT warps)
                    uint32_t pk[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        uint32_t w = 0;
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const uint32_t r = mod_acc(v[4 * j + b], p, magic, shift, off);
                            w |= mod_small(r * u, p, magic, shift) << (8 * b);
                        }
                        pk[j] = w;
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(slot_row + c * 32);
                    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                } else if (row < P.m && col0 < P.ldo) {
                    if (!P.out_i32) {
                        uint32_t pk[8];
                        if (P.store_t) {  // t = (r * u) mod p
                            const uint32_t wt = P.crt.u[mod];
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                uint32_t w = 0;
#pragma unroll
                                for (int b = 0; b < 4; ++b) {
                                    const uint32_t r = mod_acc(v[4 * j + b], p, magic, shift, off);
                                    w |= mod_small(r * wt, p, magic, shift) << (8 * b);
                                }
                                pk[j] = w;
                            }
                        } else if (P.small_acc) {  // r itself, float32 quotient (see GemmParams)
                            const uint32_t qofs = P.qofs[mod], negp = 0u - p;
                            const float2 qinv = make_float2(P.qinv[mod], P.qinv[mod]);
                            const float2 qmag = make_float2(P.qmagic[mod], P.qmagic[mod]);
                            const float2 two100 = make_float2(0x1p100f, 0x1p100f);
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                uint32_t r[4];
#pragma unroll
                                for (int b = 0; b < 4; b += 2) {
                                    const uint32_t t0 = v[4 * j + b] + qofs;
                                    const uint32_t t1 = v[4 * j + b + 1] + qofs;
                                    const float2 q = __ffma2_rn(
                                        __fmul2_rn(make_float2(__uint_as_float(t0),
                                                               __uint_as_float(t1)), two100),
                                        qinv, qmag);
                                    r[b] = t0 + negp * __float_as_uint(q.x);  // low byte
                                    r[b + 1] = t1 + negp * __float_as_uint(q.y);
                                }
                                pk[j] = __byte_perm(__byte_perm(r[0], r[1], 0x0040),
                                                    __byte_perm(r[2], r[3], 0x0040), 0x5410);
                            }
                        } else {  // r itself (the matmul path folds u into A's residues)
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                uint32_t w = 0;
#pragma unroll
                                for (int b = 0; b < 4; ++b)
                                    w |= mod_acc(v[4 * j + b], p, magic, shift, off) << (8 * b);
                                pk[j] = w;
                            }
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
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            if (kFused && mod == P.n_mod - 1) {
                __threadfence();  // slot bytes visible at L2 before the CRT warps read them
                mbar_arrive(&sfull[slot_idx]);
            }
            return true;
        });
    } else if (kFused && warp >= kEpiWarpEnd) {
        // ---------------- CRT warps (10..13, fused mode) ----------------
        const int ct = threadIdx.x - (64 + kEpiThreads);
        const int64_t tiles = int64_t(P.tiles_m) * P.tiles_n;
        int64_t local = 0;
        for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
            int tm, tn;
            decode_tile(P, t, tm, tn);
            const int slot_idx = static_cast<int>(local & 1);
            const uint32_t slot_phase = static_cast<uint32_t>((local >> 1) & 1);
            if (!mbar_wait(&sfull[slot_idx], slot_phase, abort)) {
                raise_error(P, abort, kErrTimeoutEpilogue);
                break;
            }
            const uint8_t *slot =
                P.scratch + (int64_t(blockIdx.x) * 2 + slot_idx) * P.n_mod * kSlotPlaneBytes;
            crt_tile(P, slot, tm, tn, ct);
            mbar_arrive(&sempty[slot_idx]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
EncodeTiledFn get_encode_fn() {
    // one lookup, safe under concurrent first calls (static local initialisation)
    static const EncodeTiledFn fn = []() -> EncodeTiledFn {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(p);
        return nullptr;
    }();
    return fn;
}

// 3-D map over int8 residue planes [planes][rows][ld] with dims (kdim, rows, planes) and a
// box of (128, box_rows, 1) using the 128-byte swizzle.
bool make_plane_map(CUtensorMap *map, const void *base, int64_t kdim, int64_t rows,
                           int64_t ld, int64_t planes, int box_rows, int64_t plane_stride) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(kdim), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(planes)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld), static_cast<cuuint64_t>(plane_stride)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Sets the kernel's dynamic shared-memory limit once per device (kept per device, so calls on
// several devices from several host threads each set up their own; threads racing on the
// first call of a device both set the same attribute, which is harmless).
template <bool kFused>
static cudaError_t configure(int dev) {
    constexpr int kMaxDev = 64;
    static std::atomic<int> configured[kMaxDev];
    if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
    if (configured[dev].load(std::memory_order_acquire)) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(residue_gemm_kernel<kFused>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kGemmSmemBytes));
    if (e == cudaSuccess) configured[dev].store(1, std::memory_order_release);
    return e;
}

static cudaError_t fill_common(GemmParams &P, CUtensorMap &tmA, CUtensorMap &tmB,
                               const int8_t *a_res, const int8_t *b_res, int64_t m, int64_t n,
                               int64_t kdim, int64_t ld, int n_mod, const ModMagic &mm, int *err,
                               int64_t a_plane, int64_t b_plane, bool unsigned_ops) {
    // kdim == 0 is handled by the callers; a map needs at least one column
    const int64_t kd = kdim > 0 ? kdim : 1;
    if (!make_plane_map(&tmA, a_res, kd, m, ld, n_mod, kBM, a_plane ? a_plane : ld * m))
        return cudaErrorInvalidValue;
    if (!make_plane_map(&tmB, b_res, kd, n, ld, n_mod, kBN, b_plane ? b_plane : ld * n))
        return cudaErrorInvalidValue;
    std::memset(&P, 0, sizeof(P));
    P.m = m;
    P.n = n;
    P.num_kb = static_cast<int>((kdim + kBK - 1) / kBK);
    P.epi_warps = P.num_kb <= 4 ? 8 : 4;
    P.n_mod = n_mod;
    P.tiles_m = static_cast<int>((m + kBM - 1) / kBM);
    P.tiles_n = static_cast<int>((n + kBN - 1) / kBN);
    P.total_units = int64_t(P.tiles_m) * P.tiles_n * n_mod;
    P.mm = mm;
    P.err = err;
    P.idesc = unsigned_ops ? make_idesc_u8(kBM, kBN) : kIdesc;
    // the float32 quotient when every accumulator is below 2^22 - 256 in magnitude
    const int64_t amax = unsigned_ops ? 254 : 127;
    if (kdim * amax * amax < (int64_t(1) << 22) - 256) {
        P.small_acc = 1;
        for (int i = 0; i < n_mod; ++i) {
            const uint32_t p = mm.p[i], h = (p - 1) / 2;
            const uint32_t off = p * (((uint32_t(1) << 22) + p - 1) / p);  // multiple of p >= 2^22
            P.qofs[i] = off - h;
            P.qinv[i] = 562949953421312.0f / static_cast<float>(p);  // 2^49 / p, rounded once
            uint32_t pinv8 = 1;  // p^-1 mod 2^8 (p odd): Newton steps double the correct bits
            for (int it = 0; it < 4; ++it) pinv8 *= 2u - p * pinv8;
            const uint32_t kappa = ((256u - (h & 255u)) * pinv8) & 255u;  // p * kappa == -h
            P.qmagic[i] = 12582912.0f + static_cast<float>(kappa);       // 1.5 * 2^23 + kappa
        }
    }
    return P.num_kb > 0 ? cudaSuccess : cudaErrorInvalidValue;
}

int gemm_smem_bytes() { return static_cast<int>(kGemmSmemBytes); }

cudaError_t launch_residue_gemm_pair(const int8_t *a_res, const int8_t *b_res, int64_t m,
                                     int64_t n, int64_t kdim, int64_t ld, int n_mod,
                                     const ModMagic &mm, void *out, int64_t ldo, int out_i32,
                                     int *err, cudaStream_t stream, int64_t a_plane,
                                     int64_t b_plane, int64_t out_plane, const uint32_t *weights,
                                     bool unsigned_ops, bool lower);

// The CTA-pair kernel (ti_gemm2.cu) takes products with K >= 1024 and at least one 256 x 256
// tile; shorter K loops (the trailing updates of LU and Cholesky) are bounded by the
// epilogue, where the one-CTA kernel's eight epilogue warps serve better.  TI_GEMM_PAIR=0
// in the environment selects the one-CTA kernel throughout.
static bool use_pair_kernel(int64_t m, int64_t n, int64_t kdim) {
    const char *env = std::getenv("TI_GEMM_PAIR");
    if (env && env[0] == '0') return false;
    return kdim >= 1024 && m >= 256 && n >= 256;
}

// Launch R[i] = (A_i @ B_i^T) mod p_i over n_mod planes.
//   a_res: [n_mod][m][ld] int8, b_res: [n_mod][n][ld] int8 (K-major, ld % 16 == 0)
//   out:   uint8 [n_mod][m][ldo] (ldo % 16 == 0) or int32 [n_mod][m][ldo]
// Returns cudaErrorInvalidValue if a tensor map cannot be built.
// a_plane / b_plane: bytes between the residue planes of A / B (0: ld * m / ld * n);
// out_plane: elements between output planes (0: m * ldo).  Row bands of larger operands
// pass their full operands' strides.
// weights: if not null, the uint8 output holds t_i = (r_i * weights[i]) mod p_i.
// unsigned_ops: the residue planes hold unsigned bytes (floor-mod residues up to 254)
// instead of signed ones.  lower: output tiles entirely above the diagonal are skipped.
cudaError_t launch_residue_gemm(const int8_t *a_res, const int8_t *b_res, int64_t m, int64_t n,
                                int64_t kdim, int64_t ld, int n_mod, const ModMagic &mm,
                                void *out, int64_t ldo, int out_i32, int *err, int num_sms,
                                cudaStream_t stream, int64_t a_plane, int64_t b_plane,
                                int64_t out_plane, const uint32_t *weights, bool unsigned_ops,
                                bool lower) {
    if (m == 0 || n == 0 || n_mod == 0) return cudaSuccess;
    if (use_pair_kernel(m, n, kdim)) {
        const cudaError_t pe = launch_residue_gemm_pair(a_res, b_res, m, n, kdim, ld, n_mod, mm,
                                                        out, ldo, out_i32, err, stream, a_plane,
                                                        b_plane, out_plane, weights, unsigned_ops,
                                                        lower);
        if (pe != cudaErrorNotSupported) return pe;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = configure<false>(dev);
    if (e != cudaSuccess) return e;
    CUtensorMap tmA, tmB;
    GemmParams P;
    e = fill_common(P, tmA, tmB, a_res, b_res, m, n, kdim, ld, n_mod, mm, err, a_plane, b_plane,
                    unsigned_ops);
    if (e != cudaSuccess) return e;
    P.out = out;
    P.ldo = ldo;
    P.plane = out_plane ? out_plane : m * ldo;
    P.out_i32 = out_i32;
    P.lower = lower ? 1 : 0;
    if (weights && !out_i32) {
        P.store_t = 1;
        for (int i = 0; i < n_mod; ++i) P.crt.u[i] = weights[i];
    }
    const int64_t grid = P.total_units < num_sms ? P.total_units : num_sms;
    residue_gemm_kernel<false><<<static_cast<unsigned>(grid), gemm_threads(false), kGemmSmemBytes,
                                 stream>>>(tmA, tmB, P);
    return cudaGetLastError();
}

// Output tiles of 128 x 256 for an m x n product.
int64_t gemm_output_tiles(int64_t m, int64_t n) {
    return ((m + kBM - 1) / kBM) * ((n + kBN - 1) / kBN);
}

// Scratch bytes of the fused kernel: 2 slots of n_mod x 128 x 256 bytes per CTA.
size_t fused_scratch_bytes(int n_mod, int num_ctas) {
    return size_t(num_ctas) * 2 * size_t(n_mod) * size_t(kSlotPlaneBytes);
}

// Fused K2+K3: C (op)= CRT(A_i @ B_i^T mod p_i) with the exponent scaling.  `grid` CTAs,
// scratch of fused_scratch_bytes(n_mod, grid).
cudaError_t launch_fused_gemm_crt(const int8_t *a_res, const int8_t *b_res, int64_t m, int64_t n,
                                  int64_t kdim, int64_t ld, const CrtConst &K,
                                  const int32_t *row_exp, const int32_t *col_exp, double *C,
                                  int64_t ldc, int out_mode, uint8_t *scratch, int grid, int *err,
                                  cudaStream_t stream, bool unsigned_ops) {
    if (m == 0 || n == 0) return cudaSuccess;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = configure<true>(dev);
    if (e != cudaSuccess) return e;
    CUtensorMap tmA, tmB;
    GemmParams P;
    e = fill_common(P, tmA, tmB, a_res, b_res, m, n, kdim, ld, K.n_mod, K.mm, err, 0, 0,
                    unsigned_ops);
    if (e != cudaSuccess) return e;
    P.scratch = scratch;
    P.row_exp = row_exp;
    P.col_exp = col_exp;
    P.C = C;
    P.ldc = ldc;
    P.out_mode = out_mode;
    P.crt = K;
    residue_gemm_kernel<true><<<static_cast<unsigned>(grid), gemm_threads(true), kGemmSmemBytes,
                                stream>>>(tmA, tmB, P);
    return cudaGetLastError();
}

}  // namespace ti
