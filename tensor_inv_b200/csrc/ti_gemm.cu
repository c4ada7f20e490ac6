// ti_gemm.cu -- K2: the per-modulus residue GEMMs as one persistent tcgen05 kernel.
//
// Restates src/tensor_inv/csrc/crt_kernel.cu:17-91 (cuBLASLt batched int8 GEMM followed
// by the mod_reduce kernel, crt_kernel.cu:6-15) as a single sm_100a kernel:
//   R[i] = (A_i @ B_i^T) mod p_i   for every modulus i,
// with A_i (rows x K) and B_i (cols x K) int8 residue planes stored K-major.
//
// Design (one CTA per SM, persistent over (modulus, tile_m, tile_n) work units):
//   warp 0      TMA producer: 128x128-byte A tile + 256x128-byte B tile per stage,
//               4-stage mbarrier ring, 128-byte swizzle, no multicast.
//   warp 1      TMEM allocator + single-thread tcgen05.mma.kind::i8 issuer,
//               M=128 N=256 K=32 per instruction, int32 accumulators in TMEM,
//               double-buffered (2 x 256 columns = all 512 TMEM columns).
//   warps 2..5  epilogue: tcgen05.ld 32 rows x 32 columns at a time, exact mod p, pack,
//               store.  The epilogue of tile t overlaps the main loop of tile t+1.
// Every wait is bounded; on timeout the CTA raises an error word, drains its in-flight
// copies and MMAs, frees TMEM and exits.
#include "ti_common.cuh"

namespace ti {

constexpr int kBM = 128, kBN = 256, kBK = 128, kStages = 4;
constexpr int kABytes = kBM * kBK, kBBytes = kBN * kBK, kStageBytes = kABytes + kBBytes;
constexpr int kGemmThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kIdesc = make_idesc_i8(kBM, kBN);
constexpr int kGroupM = 16;  // tile raster: 16 row-tiles per group for L2 reuse
constexpr size_t kGemmSmemBytes = size_t(kStages) * kStageBytes + 1024 /*align*/ + 256 /*bars*/;

struct GemmParams {
    int64_t m, n;      // output rows / columns per modulus
    int num_kb;        // K blocks of 128 bytes
    int n_mod;
    int tiles_m, tiles_n;
    int64_t total_tiles;
    void *out;         // uint8 [n_mod][m][ldo] or int32 [n_mod][m][ldo]
    int64_t ldo;       // elements; multiple of 16 for uint8 output
    int64_t plane;     // elements between moduli planes
    int out_i32;       // 0: uint8 residues (inputs in [0, p)); 1: int32, any int8 inputs
    ModMagic mm;
    int *err;
};

__device__ __forceinline__ void decode_tile(const GemmParams &P, int64_t t, int &mod, int &tm,
                                            int &tn) {
    const int64_t per_mod = int64_t(P.tiles_m) * P.tiles_n;
    mod = static_cast<int>(t / per_mod);
    const int64_t r = t - int64_t(mod) * per_mod;
    const int64_t per_group = int64_t(kGroupM) * P.tiles_n;
    const int g = static_cast<int>(r / per_group);
    const int first_m = g * kGroupM;
    const int gsize = min(kGroupM, P.tiles_m - first_m);
    const int64_t rg = r - int64_t(g) * per_group;
    tm = first_m + static_cast<int>(rg % gsize);
    tn = static_cast<int>(rg / gsize);
}

__device__ __forceinline__ void raise_error(const GemmParams &P, volatile int *abort, int code) {
    *abort = 1;
    atomicCAS(P.err, 0, code);
}

__global__ void __launch_bounds__(kGemmThreads, 1)
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
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 128);
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
            for (int64_t t = blockIdx.x; t < P.total_tiles && ok; t += gridDim.x) {
                int mod, tm, tn;
                decode_tile(P, t, mod, tm, tn);
                for (int kb = 0; kb < P.num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort)) {
                        raise_error(P, abort, kErrTimeoutProducer);
                        ok = false;
                        break;
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
            }
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
            int64_t local = 0;
            for (int64_t t = blockIdx.x; t < P.total_tiles && ok; t += gridDim.x, ++local) {
                const int acc = static_cast<int>(local & 1);
                const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort)) {
                    raise_error(P, abort, kErrTimeoutMma);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
                for (int kb = 0; kb < P.num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort)) {
                        raise_error(P, abort, kErrTimeoutMma);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(sA + stage * kABytes));
                    const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(sB + stage * kBBytes));
#pragma unroll
                    for (int kk = 0; kk < kBK / 32; ++kk) {
                        // advance the start address by 32 bytes (2 x 16-byte units) per K step
                        umma_i8(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, kIdesc,
                                (kb | kk) != 0 ? 1u : 0u);
                    }
                    any_issued = true;
                    umma_commit(&empty[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (ok) umma_commit(&tfull[acc]);
            }
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
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int row_in_tile = q * 32 + lane;
        int64_t local = 0;
        for (int64_t t = blockIdx.x; t < P.total_tiles; t += gridDim.x, ++local) {
            int mod, tm, tn;
            decode_tile(P, t, mod, tm, tn);
            const int acc = static_cast<int>(local & 1);
            const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
            if (!mbar_wait(&tfull[acc], acc_phase, abort)) {
                raise_error(P, abort, kErrTimeoutEpilogue);
                break;
            }
            tc_fence_after();
            const int64_t row = int64_t(tm) * kBM + row_in_tile;
            const uint32_t p = P.mm.p[mod], magic = P.mm.magic[mod], shift = P.mm.shift[mod];
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * kBN);
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tbase + c * 32, v);
                tmem_wait_ld();
                const int64_t col0 = int64_t(tn) * kBN + c * 32;
                if (row < P.m && col0 < P.ldo) {
                    if (!P.out_i32) {
                        uint32_t pk[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            uint32_t w = 0;
#pragma unroll
                            for (int b = 0; b < 4; ++b)
                                w |= mod_small(v[4 * j + b], p, magic, shift) << (8 * b);
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
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
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
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 3-D map over int8 residue planes [planes][rows][ld] with dims (kdim, rows, planes) and a
// box of (128, box_rows, 1) using the 128-byte swizzle.
static bool make_plane_map(CUtensorMap *map, const void *base, int64_t kdim, int64_t rows,
                           int64_t ld, int64_t planes, int box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(kdim), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(planes)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld), static_cast<cuuint64_t>(ld * rows)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int gemm_smem_bytes() { return static_cast<int>(kGemmSmemBytes); }

// Launch R[i] = (A_i @ B_i^T) mod p_i over n_mod planes.
//   a_res: [n_mod][m][ld] int8, b_res: [n_mod][n][ld] int8 (K-major, ld % 16 == 0)
//   out:   uint8 [n_mod][m][ldo] (ldo % 16 == 0) or int32 [n_mod][m][ldo]
// Returns cudaErrorInvalidValue if a tensor map cannot be built.
cudaError_t launch_residue_gemm(const int8_t *a_res, const int8_t *b_res, int64_t m, int64_t n,
                                int64_t kdim, int64_t ld, int n_mod, const ModMagic &mm,
                                void *out, int64_t ldo, int out_i32, int *err, int num_sms,
                                cudaStream_t stream) {
    if (m == 0 || n == 0 || n_mod == 0) return cudaSuccess;
    static int configured_device = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_device != dev) {
        cudaError_t e = cudaFuncSetAttribute(residue_gemm_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kGemmSmemBytes));
        if (e != cudaSuccess) return e;
        configured_device = dev;
    }
    CUtensorMap tmA, tmB;
    // kdim == 0 still needs a valid map: describe one zero column (never loaded).
    const int64_t kd = kdim > 0 ? kdim : 1;
    if (!make_plane_map(&tmA, a_res, kd, m, ld, n_mod, kBM)) return cudaErrorInvalidValue;
    if (!make_plane_map(&tmB, b_res, kd, n, ld, n_mod, kBN)) return cudaErrorInvalidValue;
    GemmParams P;
    P.m = m;
    P.n = n;
    P.num_kb = static_cast<int>((kdim + kBK - 1) / kBK);
    P.n_mod = n_mod;
    P.tiles_m = static_cast<int>((m + kBM - 1) / kBM);
    P.tiles_n = static_cast<int>((n + kBN - 1) / kBN);
    P.total_tiles = int64_t(P.tiles_m) * P.tiles_n * n_mod;
    P.out = out;
    P.ldo = ldo;
    P.plane = m * ldo;
    P.out_i32 = out_i32;
    P.mm = mm;
    P.err = err;
    if (P.num_kb == 0) return cudaErrorInvalidValue;  // callers handle k == 0
    int64_t grid = P.total_tiles < num_sms ? P.total_tiles : num_sms;
    residue_gemm_kernel<<<static_cast<unsigned>(grid), kGemmThreads, kGemmSmemBytes, stream>>>(
        tmA, tmB, P);
    return cudaGetLastError();
}

}  // namespace ti
