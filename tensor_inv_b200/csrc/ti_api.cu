// ti_api.cu -- the extern "C" entry points of libtensor_inv_crt.so (include/tensor_inv_crt.h).
//
// Host-side planning for the CRT matmul: the modulus count (crt_matmul.py:20 _n_moduli),
// the per-modulus constants every kernel receives by value, the workspace layout, and the
// stage sequence K1 (split) -> K2 (tcgen05 residue GEMM) -> K3 (exact CRT).
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "tensor_inv_crt.h"
#include "ti_common.cuh"

namespace ti {
cudaError_t launch_split(const double *X, int64_t outer, int64_t kdim, int64_t s_outer,
                         int64_t s_k, const SplitConst &C, int32_t *exp_out, int8_t *res,
                         int64_t ld_res, int num_sms, cudaStream_t stream, int64_t plane = 0,
                         int blocks_per_sm = 8, int *err = nullptr, bool exps_given = false);
cudaError_t launch_residue_gemm(const int8_t *a_res, const int8_t *b_res, int64_t m, int64_t n,
                                int64_t kdim, int64_t ld, int n_mod, const ModMagic &mm,
                                void *out, int64_t ldo, int out_i32, int *err, int num_sms,
                                cudaStream_t stream, int64_t a_plane = 0, int64_t b_plane = 0,
                                int64_t out_plane = 0, const uint32_t *weights = nullptr,
                                bool unsigned_ops = false, bool lower = false);
cudaError_t launch_crt(const void *R, bool in_u8, int64_t ldr, int64_t plane, int64_t rows,
                       int64_t cols, const int32_t *row_exp, const int32_t *col_exp, double *C,
                       int64_t ldc, int out_mode, const CrtConst &K, int num_sms,
                       cudaStream_t stream, int blocks_per_sm = 8, bool lower = false);
cudaError_t launch_split_tc(const double *X, int64_t outer, int64_t kdim, int64_t s_outer,
                            int64_t s_k, const SplitConst &C, const int32_t *exps, int8_t *res,
                            int64_t ld_res, int64_t plane, int *err, int num_sms,
                            cudaStream_t stream);
cudaError_t launch_crt_tc(const uint8_t *R, int64_t ldr, int64_t plane, int64_t rows,
                          int64_t cols, const int32_t *row_exp, const int32_t *col_exp, double *C,
                          int64_t ldc, int out_mode, const CrtConst &K, int *err, int num_sms,
                          cudaStream_t stream, bool lower);
int64_t gemm_output_tiles(int64_t m, int64_t n);
size_t fused_scratch_bytes(int n_mod, int num_ctas);
cudaError_t launch_fused_gemm_crt(const int8_t *a_res, const int8_t *b_res, int64_t m, int64_t n,
                                  int64_t kdim, int64_t ld, const CrtConst &K,
                                  const int32_t *row_exp, const int32_t *col_exp, double *C,
                                  int64_t ldc, int out_mode, uint8_t *scratch, int grid, int *err,
                                  cudaStream_t stream, bool unsigned_ops);

// The fused GEMM+CRT kernel (K2+K3 in one launch) is opt-in (TI_CRT_PATH=fused): measured
// on B200 at 8192^3 its tile-major order (all moduli of one tile back to back) costs the
// GEMM ~20% in L2 reuse, more than the separate reconstruction kernel it hides.
// Scratch of the fused kernel is sized for at most this many CTAs (one per SM).
constexpr int kFusedMaxCtas = 192;

// TI_CRT_PATH=fused selects the fused kernel (default: K2 then K3), for tests and tuning.
// Read on every call so one process can exercise both paths.
static int path_override() {
    const char *e = getenv("TI_CRT_PATH");
    return (e && !strcmp(e, "fused")) ? 1 : (e && !strcmp(e, "unfused")) ? 0 : -1;
}

static bool use_fused(int64_t m, int64_t n) {
    return path_override() == 1 && gemm_output_tiles(m, n) >= 1;
}

// K3 on uint8 t-planes: the tensor-core kernel (ti_crt_tc.cu) by default; TI_CRT_K3=simt
// selects the SIMT kernel (ti_crt.cu), which gives the same bits, for comparisons.  `sms`
// caps the CTAs (a share of the SMs when the launch runs beside a GEMM).
static cudaError_t launch_k3(const uint8_t *R, int64_t ldr, int64_t plane, int64_t rows,
                             int64_t cols, const int32_t *rexp, const int32_t *cexp, double *C,
                             int64_t ldc, int out_mode, const CrtConst &K, int *err, int sms,
                             cudaStream_t s, int blocks_per_sm = 8, bool lower = false) {
    const char *e = getenv("TI_CRT_K3");
    if (e && !strcmp(e, "simt"))
        return launch_crt(R, true, ldr, plane, rows, cols, rexp, cexp, C, ldc, out_mode, K, sms,
                          s, blocks_per_sm, lower);
    int ctas = sms * blocks_per_sm / 8;
    if (ctas < 1) ctas = 1;
    return launch_crt_tc(R, ldr, plane, rows, cols, rexp, cexp, C, ldc, out_mode, K, err, ctas, s,
                         lower);
}

// The device error word: kernels record a bounded wait that ran out here.
__device__ int g_device_error = 0;

static const int32_t kPrimes[30] = {3,  5,  7,  11, 13, 17, 19, 23, 29,  31,  37,  41,  43,  47,  53,
                                    59, 61, 67, 71, 73, 79, 83, 89, 97, 101, 103, 107, 109, 113, 127};
// Pairwise-coprime odd moduli up to 255, largest first (each taken greedily when coprime
// with all larger ones).  Sixteen of them multiply to 2^124.95.
static const int32_t kWide[16] = {255, 253, 251, 247, 241, 239, 233, 229,
                                  227, 223, 217, 211, 199, 197, 193, 191};
constexpr int kMaxPrimesModuli = 25;  // prod(first 25 primes) = 2^126.5 < 2^127
constexpr int kMaxWideModuli = 16;    // prod(16 wide moduli) = 2^124.95 < 2^127
// |symmetric residue| <= 127 for the wide moduli: 127*127*k < 2^31 - 256
constexpr int64_t kMaxKWide = 133144;

typedef unsigned __int128 u128;

static inline int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }
static inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---------------------------------------------------------------------------------------
// modulus count: exact comparison of prod(p) with 2*k*2^(2*bits) on 32-bit words
// ---------------------------------------------------------------------------------------
static int n_moduli_exact(int64_t k, int bits) {
    if (k < 0 || bits < 1 || bits > 64) return -1;
    uint32_t target[10] = {0}, prod[10] = {0};
    // target = k << (2*bits + 1)
    const int sh = 2 * bits + 1;
    u128 kk = static_cast<u128>(static_cast<uint64_t>(k));
    for (int w = 0; w < 10; ++w) {
        // bit range [32w, 32w+32) of kk << sh
        const int lo = 32 * w - sh;
        uint32_t word = 0;
        for (int b = 0; b < 32; ++b) {
            const int src = lo + b;
            if (src >= 0 && src < 128 && ((kk >> src) & 1)) word |= 1u << b;
        }
        target[w] = word;
    }
    prod[0] = 1;
    for (int i = 0; i < 30; ++i) {
        uint64_t carry = 0;
        for (int w = 0; w < 10; ++w) {
            const uint64_t t = static_cast<uint64_t>(prod[w]) * kPrimes[i] + carry;
            prod[w] = static_cast<uint32_t>(t);
            carry = t >> 32;
        }
        int cmp = 0;
        for (int w = 9; w >= 0 && cmp == 0; --w)
            if (prod[w] != target[w]) cmp = prod[w] > target[w] ? 1 : -1;
        if (cmp > 0) return i + 1;
    }
    return -1;
}

// ---------------------------------------------------------------------------------------
// moduli plan: which moduli, how many, and the precision kept
// ---------------------------------------------------------------------------------------
struct Plan {
    int n_mod;
    int bits;        // precision actually kept (<= the requested bits)
    bool wide;
    int32_t moduli[kMaxModuli];
};

// Largest b <= bits with prod(moduli[:n]) > 2*k*2^(2b), or 0 if none.  Exact (u128).
static int bits_for(const int32_t *moduli, int n, int64_t k, int bits) {
    u128 M = 1;
    for (int i = 0; i < n; ++i) M *= static_cast<uint32_t>(moduli[i]);
    for (int b = bits; b >= 1; --b)
        if ((static_cast<u128>(static_cast<uint64_t>(k)) << (2 * b + 1)) < M) return b;
    return 0;
}

static int make_plan(int64_t k, int bits, const ti_crt_options_t *opt, Plan &P) {
    const int kind = opt ? opt->moduli : TI_MODULI_PRIMES;
    const int want = opt ? opt->n_moduli : 0;
    if (kind != TI_MODULI_PRIMES && kind != TI_MODULI_WIDE) return TI_ERR_INVALID_ARGUMENT;
    if (want < 0) return TI_ERR_INVALID_ARGUMENT;
    P.wide = kind == TI_MODULI_WIDE;
    const int32_t *set = P.wide ? kWide : kPrimes;
    const int max_n = P.wide ? kMaxWideModuli : kMaxPrimesModuli;
    if (k > (P.wide ? kMaxKWide : int64_t(TI_MAX_K))) return TI_ERR_UNSUPPORTED;
    if (want > max_n) return TI_ERR_UNSUPPORTED;
    if (want == 0 && !P.wide) {
        P.n_mod = n_moduli_exact(k, bits);  // crt_matmul.py:20-29
        P.bits = bits;
        if (P.n_mod < 0 || P.n_mod > max_n) return TI_ERR_UNSUPPORTED;
    } else if (want == 0) {
        P.n_mod = -1;
        for (int n = 1; n <= max_n; ++n)
            if (bits_for(set, n, k, bits) == bits) {
                P.n_mod = n;
                break;
            }
        if (P.n_mod < 0) return TI_ERR_UNSUPPORTED;
        P.bits = bits;
    } else {
        P.n_mod = want;
        P.bits = bits_for(set, want, k, bits);
        if (P.bits < 1) return TI_ERR_UNSUPPORTED;
    }
    for (int i = 0; i < P.n_mod; ++i) P.moduli[i] = set[i];
    return TI_OK;
}

// ---------------------------------------------------------------------------------------
// per-modulus constants
// ---------------------------------------------------------------------------------------
static bool is_pow2(uint32_t x) { return (x & (x - 1)) == 0; }

static bool make_magic(const int32_t *moduli, int n, ModMagic &mm) {
    if (n < 1 || n > kMaxModuli) return false;
    std::memset(&mm, 0, sizeof(mm));
    for (int i = 0; i < n; ++i) {
        const uint32_t p = static_cast<uint32_t>(moduli[i]);
        if (moduli[i] < 2 || p >= 256) return false;
        uint32_t sh = 0;
        while ((2u << sh) <= p) ++sh;  // floor(log2 p)
        mm.p[i] = p;
        mm.shift[i] = sh;
        // ceil(2^(32+sh) / p) < 2^32 for p not a power of two; powers of two use
        // magic = 2^32 / p * 2^sh exactly -- not needed by the int8 paths, kept valid anyway
        const u128 num = static_cast<u128>(1) << (32 + sh);
        u128 mg = (num + p - 1) / p;
        if (is_pow2(p)) mg = (static_cast<u128>(1) << 32) - 1;  // unused (uint8 path is odd p)
        mm.magic[i] = static_cast<uint32_t>(mg);
        mm.off[i] = p * (((uint32_t(1) << 31) + p - 1) / p);
    }
    return true;
}

// mult: a factor folded into every residue ((mult_i * x) mod p_i), or null for none.
static bool make_split_const(const int32_t *moduli, int n_mod, int bits, bool symmetric,
                             const uint32_t *mult, SplitConst &C) {
    std::memset(&C, 0, sizeof(C));
    C.n_mod = n_mod;
    C.bits = bits;
    C.symmetric = symmetric ? 1 : 0;
    if (!make_magic(moduli, n_mod, C.mm)) return false;
    for (int i = 0; i < n_mod; ++i) {
        const uint64_t p = static_cast<uint32_t>(moduli[i]);
        const uint64_t m = mult ? mult[i] % p : 1;
        C.mult[i] = static_cast<uint32_t>(m);
        C.w32[i] = static_cast<uint32_t>((((uint64_t(1) << 32) % p) * m) % p);
        C.w16[i] = static_cast<uint32_t>((((uint64_t(1) << 16) % p) * m) % p);
        C.bigp[i] = static_cast<uint32_t>(p * (((uint64_t(1) << 30) + p - 1) / p));
        C.offs[i] = static_cast<uint32_t>(p * ((uint64_t(568197120) + p - 1) / p));
    }
    return true;
}

// Residue representative on the matmul path: symmetric residues in [-(p-1)/2, (p-1)/2]
// (signed bytes, a signed residue GEMM).  The products mod p, and so every output bit, are
// the same for any representative; the symmetric one is the cheaper for the tensor-core
// split (a rounded float32 quotient) and keeps the GEMM accumulator below k * 127^2.

static bool make_crt_const(const int32_t *moduli, int n_mod, int bits, CrtConst &K);

// Split constants of the matmul path: A's residues carry the CRT factor u_i (so the residue
// GEMM writes t_i = (u_i A_i B_i) mod p_i with one reduction), B's are plain.
static bool make_matmul_consts(const Plan &PL, SplitConst &SCA, SplitConst &SCB, CrtConst &KC) {
    return make_crt_const(PL.moduli, PL.n_mod, PL.bits, KC) &&
           make_split_const(PL.moduli, PL.n_mod, PL.bits, true, KC.u, SCA) &&
           make_split_const(PL.moduli, PL.n_mod, PL.bits, true, nullptr, SCB);
}

// Pairwise-coprime moduli with product below 2^127 (so every lifted value fits 128 bits).
static bool make_crt_const(const int32_t *moduli, int n_mod, int bits, CrtConst &K) {
    std::memset(&K, 0, sizeof(K));
    if (!make_magic(moduli, n_mod, K.mm)) return false;
    K.n_mod = n_mod;
    K.two_bits = 2 * bits;
    u128 M = 1;
    for (int i = 0; i < n_mod; ++i) {
        const u128 p = static_cast<uint32_t>(moduli[i]);
        if (M > (static_cast<u128>(1) << 127) / p) return false;
        M *= p;
    }
    if (M >= (static_cast<u128>(1) << 127)) return false;
    for (int i = 0; i < n_mod; ++i) {
        const uint32_t p = static_cast<uint32_t>(moduli[i]);
        const u128 Mi = M / p;
        const uint32_t red = static_cast<uint32_t>(Mi % p);
        uint32_t inv = 0;
        for (uint32_t t = 1; t < p; ++t)
            if ((static_cast<uint64_t>(red) * t) % p == 1) {
                inv = t;
                break;
            }
        if (!inv) return false;  // not coprime
        K.u[i] = inv;
        K.finv[i] = static_cast<uint32_t>(((uint64_t(1) << 32) + p / 2) / p);
        for (int w = 0; w < 4; ++w) K.Mi[i][w] = static_cast<uint32_t>(Mi >> (32 * w));
    }
    const u128 H = (M - 1) / 2;
    for (int w = 0; w < 4; ++w) {
        K.M[w] = static_cast<uint32_t>(M >> (32 * w));
        K.H[w] = static_cast<uint32_t>(H >> (32 * w));
    }
    // groups of three consecutive moduli (P_g <= 255^3 < 2^24, so c_g < 3 P_g < 2^26)
    K.n_groups = (n_mod + 2) / 3;
    for (int g = 0; g < K.n_groups; ++g) {
        uint64_t Pg = 1;
        for (int i = 3 * g; i < 3 * g + 3 && i < n_mod; ++i) Pg *= static_cast<uint32_t>(moduli[i]);
        for (int i = 3 * g; i < 3 * g + 3 && i < n_mod; ++i)
            K.coef[i] = static_cast<uint32_t>(Pg / static_cast<uint32_t>(moduli[i]));
        const u128 Mg = M / Pg;
        for (int w = 0; w < 4; ++w) K.Mg[g][w] = static_cast<uint32_t>(Mg >> (32 * w));
        const uint64_t finv = ((uint64_t(1) << 48) + Pg / 2) / Pg;  // round(2^48 / P_g)
        K.fgl[g] = static_cast<uint32_t>(finv);
        K.fgh[g] = static_cast<uint32_t>(finv >> 32);
    }
    return true;
}

// ---------------------------------------------------------------------------------------
// device bookkeeping
// ---------------------------------------------------------------------------------------
struct DevInfo {
    int num_sms;
    int *err;
};

static int device_info(DevInfo &d);

// SM count and device error word of the current device, for kernels in other files.
int device_context(int *num_sms, int **err) {
    DevInfo d;
    const int rc = device_info(d);
    if (rc != TI_OK) return rc;
    *num_sms = d.num_sms;
    *err = d.err;
    return TI_OK;
}

static int device_info(DevInfo &d) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return TI_ERR_NO_DEVICE;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return TI_ERR_NO_DEVICE;
    if (major != 10) return TI_ERR_NO_DEVICE;
    if (cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return TI_ERR_CUDA;
    if (cudaGetSymbolAddress(reinterpret_cast<void **>(&d.err), g_device_error) != cudaSuccess)
        return TI_ERR_CUDA;
    return TI_OK;
}

static int cuda_status(cudaError_t e) { return e == cudaSuccess ? TI_OK : TI_ERR_CUDA; }

// ---------------------------------------------------------------------------------------
// per-device streams and events of the banded pipeline (created once, kept until exit)
// ---------------------------------------------------------------------------------------
constexpr int kMaxBands = 16;
constexpr int kMaxDevices = 64;
constexpr int kSideBlocksPerSm = 2;  // split/CRT blocks per SM while a GEMM is resident

struct Pipeline {
    std::mutex mu;                   // held while a call records and waits on the events
    bool ready = false;
    cudaStream_t hi = nullptr;       // GEMMs (highest priority)
    cudaStream_t lo = nullptr;       // splits and reconstructions (lowest priority)
    cudaEvent_t fork = nullptr, hi_done = nullptr, lo_done = nullptr;
    cudaEvent_t split_done[kMaxBands] = {}, gemm_done[kMaxBands] = {};
    // host-operand pipeline: copy engines on their own streams
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaEvent_t b_in = nullptr, a_in[kMaxBands] = {}, c_ready[kMaxBands] = {};
};

static Pipeline g_pipe[kMaxDevices];

static int pipeline_for_device(int dev, Pipeline *&out) {
    if (dev < 0 || dev >= kMaxDevices) return TI_ERR_UNSUPPORTED;
    Pipeline &P = g_pipe[dev];
    out = &P;
    if (P.ready) return TI_OK;
    int least = 0, greatest = 0;
    if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) return TI_ERR_CUDA;
    if (cudaStreamCreateWithPriority(&P.hi, cudaStreamNonBlocking, greatest) != cudaSuccess ||
        cudaStreamCreateWithPriority(&P.lo, cudaStreamNonBlocking, least) != cudaSuccess)
        return TI_ERR_CUDA;
    cudaEvent_t *evs[] = {&P.fork, &P.hi_done, &P.lo_done};
    for (cudaEvent_t *e : evs)
        if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return TI_ERR_CUDA;
    for (int b = 0; b < kMaxBands; ++b)
        if (cudaEventCreateWithFlags(&P.split_done[b], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&P.gemm_done[b], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&P.a_in[b], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&P.c_ready[b], cudaEventDisableTiming) != cudaSuccess)
            return TI_ERR_CUDA;
    if (cudaStreamCreateWithFlags(&P.h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&P.d2h, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&P.b_in, cudaEventDisableTiming) != cudaSuccess)
        return TI_ERR_CUDA;
    P.ready = true;
    return TI_OK;
}

// Automatic banding of device-resident operands: one band.  Measured on B200 at 8192^3,
// splits and reconstructions sharing SMs with the GEMM slow it by more (5.6 -> 8.7 ms) than
// the integer work they hide (3.5 ms), so overlap is opt-in (options.bands > 1).
static int auto_bands(int64_t) { return 1; }

// ---------------------------------------------------------------------------------------
// int8 repacking for the reference-layout batched GEMM entry point
// ---------------------------------------------------------------------------------------
// dst[b][r][0..ld) = src[b][r][0..K) followed by zeros
__global__ void pad_rows_i8_kernel(const int8_t *__restrict__ src, int64_t batch, int64_t rows,
                                   int64_t K, int8_t *__restrict__ dst, int64_t ld) {
    const int64_t total = batch * rows * ld;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t br = i / ld, c = i - br * ld;
        dst[i] = c < K ? src[br * K + c] : 0;
    }
}

// dst[b][n][0..ld) = src[b][0..K)[n] followed by zeros (transpose of each K x N plane)
__global__ void transpose_i8_kernel(const int8_t *__restrict__ src, int64_t batch, int64_t K,
                                    int64_t N, int8_t *__restrict__ dst, int64_t ld) {
    __shared__ int8_t tile[64][65];
    const int64_t tk = (ld + 63) / 64, tn = (N + 63) / 64;
    for (int64_t t = blockIdx.x; t < batch * tk * tn; t += gridDim.x) {
        const int64_t b = t / (tk * tn), r = t - b * tk * tn;
        const int64_t k0 = (r / tn) * 64, n0 = (r % tn) * 64;
        for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
            const int kk = i / 64, nn = i % 64;
            const int64_t k = k0 + kk, n = n0 + nn;
            tile[kk][nn] = (k < K && n < N) ? src[(b * K + k) * N + n] : 0;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
            const int nn = i / 64, kk = i % 64;
            const int64_t k = k0 + kk, n = n0 + nn;
            if (n < N && k < ld) dst[(b * N + n) * ld + k] = tile[kk][nn];
        }
        __syncthreads();
    }
}

}  // namespace ti

using namespace ti;

// =======================================================================================
// C ABI
// =======================================================================================
extern "C" {

const char *ti_status_string(int status) {
    switch (status) {
        case TI_OK: return "ok";
        case TI_ERR_INVALID_ARGUMENT: return "invalid argument";
        case TI_ERR_UNSUPPORTED: return "unsupported size (inner dimension or moduli)";
        case TI_ERR_WORKSPACE: return "workspace too small or misaligned";
        case TI_ERR_CUDA: return "CUDA error";
        case TI_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case TI_ERR_NO_DEVICE: return "no sm_100 device";
        case TI_ERR_SCRATCH_LIMIT:
            return "problem needs more scratch than the no-alloc entry point's static 64 MiB";
        default: return "unknown status";
    }
}

const char *ti_version(void) { return "0.1.0"; }

const int32_t *ti_primes(void) { return kPrimes; }

int ti_n_moduli(int64_t k, int bits, int *n_out) {
    if (!n_out) return TI_ERR_INVALID_ARGUMENT;
    const int n = n_moduli_exact(k, bits);
    if (n < 0) return TI_ERR_UNSUPPORTED;
    *n_out = n;
    return TI_OK;
}

// Workspace layout of ti_crt_matmul (each piece 256-byte aligned):
//   row_exp int32[m] | col_exp int32[n] | A residues int8[N][m][ldk] |
//   B residues int8[N][n][ldk] | product residues uint8[N][m][ldr] (K2 then K3)
//                                or per-CTA slots uint8[CTAs][2][N][128][256] (fused)
struct CrtLayout {
    int n_mod;
    Plan plan;
    int64_t ldk, ldr;
    size_t off_rexp, off_cexp, off_a, off_b, off_r, total;
};

static int crt_layout(int64_t m, int64_t n, int64_t k, int bits, const ti_crt_options_t *opt,
                      CrtLayout &L) {
    if (m < 0 || n < 0 || k < 0) return TI_ERR_INVALID_ARGUMENT;
    if (bits != 8 && bits != 11 && bits != 24 && bits != 53) return TI_ERR_INVALID_ARGUMENT;
    const int rc = make_plan(k, bits, opt, L.plan);
    if (rc != TI_OK) return rc;
    L.n_mod = L.plan.n_mod;
    L.ldk = round_up(k > 0 ? k : 1, 16);
    L.ldr = round_up(n > 0 ? n : 1, 16);
    size_t off = 0;
    L.off_rexp = off; off += align256(sizeof(int32_t) * size_t(m));
    L.off_cexp = off; off += align256(sizeof(int32_t) * size_t(n));
    L.off_a = off; off += align256(size_t(L.n_mod) * size_t(m) * size_t(L.ldk));
    L.off_b = off; off += align256(size_t(L.n_mod) * size_t(n) * size_t(L.ldk));
    L.off_r = off;
    const size_t planes = align256(size_t(L.n_mod) * size_t(m) * size_t(L.ldr));
    const size_t slots = align256(fused_scratch_bytes(L.n_mod, kFusedMaxCtas));
    off += use_fused(m, n) ? slots : planes;
    L.total = off;
    return TI_OK;
}

int ti_crt_workspace_size_ex(int64_t m, int64_t n, int64_t k, int bits,
                             const ti_crt_options_t *opt, size_t *bytes) {
    if (!bytes) return TI_ERR_INVALID_ARGUMENT;
    CrtLayout L;
    const int rc = crt_layout(m, n, k, bits, opt, L);
    if (rc != TI_OK) return rc;
    *bytes = L.total;
    return TI_OK;
}

int ti_crt_workspace_size(int64_t m, int64_t n, int64_t k, int bits, size_t *bytes) {
    return ti_crt_workspace_size_ex(m, n, k, bits, nullptr, bytes);
}

int ti_crt_plan(int64_t k, int bits, const ti_crt_options_t *opt, int *n_mod_out,
                int *bits_eff_out, int32_t *moduli_out) {
    if (k < 0 || bits < 1 || bits > 53) return TI_ERR_INVALID_ARGUMENT;
    Plan P;
    const int rc = make_plan(k, bits, opt, P);
    if (rc != TI_OK) return rc;
    if (n_mod_out) *n_mod_out = P.n_mod;
    if (bits_eff_out) *bits_eff_out = P.bits;
    if (moduli_out)
        for (int i = 0; i < P.n_mod; ++i) moduli_out[i] = P.moduli[i];
    return TI_OK;
}

int ti_crt_split(const double *X, int64_t outer, int64_t kdim, int64_t s_outer, int64_t s_k,
                 int bits, int n_mod, int32_t *exp_out, int8_t *res_out, int64_t ld_res,
                 void *stream) {
    if (outer < 0 || kdim < 1 || n_mod < 1 || n_mod > 30) return TI_ERR_INVALID_ARGUMENT;
    if (bits < 1 || bits > 53) return TI_ERR_INVALID_ARGUMENT;
    if (ld_res < kdim || (ld_res & 15) || (reinterpret_cast<uintptr_t>(res_out) & 15))
        return TI_ERR_INVALID_ARGUMENT;
    if (!(s_k == 1 || s_outer == 1)) return TI_ERR_INVALID_ARGUMENT;
    if (outer == 0) return TI_OK;
    if (!X || !exp_out || !res_out) return TI_ERR_INVALID_ARGUMENT;
    DevInfo d;
    int rc = device_info(d);
    if (rc != TI_OK) return rc;
    SplitConst C;
    if (!make_split_const(kPrimes, n_mod, bits, false, nullptr, C)) return TI_ERR_INVALID_ARGUMENT;
    // s_k == 1 selects the k-contiguous kernels (also for a 1-long outer stride)
    const int64_t sk = (s_k == 1) ? 1 : s_k;
    const int64_t so = (s_k == 1) ? s_outer : 1;
    return cuda_status(launch_split(X, outer, kdim, so, sk, C, exp_out, res_out, ld_res,
                                    d.num_sms, static_cast<cudaStream_t>(stream)));
}

int ti_crt_residue_partial_workspace_size(int64_t m, int64_t n, int64_t k, int n_mod,
                                          size_t *bytes) {
    if (!bytes || m < 0 || n < 0 || k < 0 || n_mod < 1 || n_mod > 30)
        return TI_ERR_INVALID_ARGUMENT;
    const int64_t ldk = round_up(k > 0 ? k : 1, 16);
    *bytes = align256(size_t(n_mod) * size_t(m) * size_t(ldk)) +
             align256(size_t(n_mod) * size_t(n) * size_t(ldk));
    return TI_OK;
}

int ti_crt_residue_partial(const double *A, int64_t sa0, int64_t sa1, const double *B,
                           int64_t sb0, int64_t sb1, int64_t m, int64_t n, int64_t k, int bits,
                           int n_mod, const int32_t *row_exp, const int32_t *col_exp,
                           int32_t *out, void *workspace, size_t workspace_bytes, void *stream) {
    if (m < 0 || n < 0 || k < 0 || n_mod < 1 || n_mod > 30) return TI_ERR_INVALID_ARGUMENT;
    if (bits < 1 || bits > 53) return TI_ERR_INVALID_ARGUMENT;
    if (k > int64_t(TI_MAX_K)) return TI_ERR_UNSUPPORTED;
    if (m == 0 || n == 0) return TI_OK;
    if (!out || !row_exp || !col_exp) return TI_ERR_INVALID_ARGUMENT;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (k == 0)  // an empty slice contributes zero residues
        return cuda_status(cudaMemsetAsync(out, 0, sizeof(int32_t) * n_mod * m * n, s));
    if (!A || !B) return TI_ERR_INVALID_ARGUMENT;
    if (!(sa1 == 1 || sa0 == 1) || !(sb0 == 1 || sb1 == 1)) return TI_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    ti_crt_residue_partial_workspace_size(m, n, k, n_mod, &need);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return TI_ERR_WORKSPACE;
    DevInfo d;
    int rc = device_info(d);
    if (rc != TI_OK) return rc;
    SplitConst SC;  // the reference's floor-mod residues of the first n_mod primes
    if (!make_split_const(kPrimes, n_mod, bits, false, nullptr, SC)) return TI_ERR_INVALID_ARGUMENT;
    const int64_t ldk = round_up(k, 16);
    int8_t *ares = static_cast<int8_t *>(workspace);
    int8_t *bres = ares + align256(size_t(n_mod) * size_t(m) * size_t(ldk));
    int32_t *rexp = const_cast<int32_t *>(row_exp), *cexp = const_cast<int32_t *>(col_exp);
    cudaError_t e;
    if (sa1 == 1) e = launch_split(A, m, k, sa0, 1, SC, rexp, ares, ldk, d.num_sms, s, 0, 8, d.err, true);
    else e = launch_split(A, m, k, 1, sa1, SC, rexp, ares, ldk, d.num_sms, s, 0, 8, d.err, true);
    if (e != cudaSuccess) return TI_ERR_CUDA;
    if (sb0 == 1) e = launch_split(B, n, k, sb1, 1, SC, cexp, bres, ldk, d.num_sms, s, 0, 8, d.err, true);
    else e = launch_split(B, n, k, 1, sb0, SC, cexp, bres, ldk, d.num_sms, s, 0, 8, d.err, true);
    if (e != cudaSuccess) return TI_ERR_CUDA;
    e = launch_residue_gemm(ares, bres, m, n, k, ldk, n_mod, SC.mm, out, n, 1, d.err, d.num_sms, s);
    if (e != cudaSuccess) return e == cudaErrorInvalidValue ? TI_ERR_NO_DEVICE : TI_ERR_CUDA;
    return TI_OK;
}

int ti_batched_gemm_workspace_size(int64_t batch, int64_t M, int64_t K, int64_t N,
                                   size_t *bytes) {
    if (!bytes || batch < 0 || M < 0 || K < 0 || N < 0) return TI_ERR_INVALID_ARGUMENT;
    const int64_t ld = round_up(K > 0 ? K : 1, 16);
    *bytes = align256(size_t(batch) * size_t(M) * size_t(ld)) +
             align256(size_t(batch) * size_t(N) * size_t(ld));
    return TI_OK;
}

int ti_batched_int8_gemm_mod(const int8_t *a, const int8_t *b, const int32_t *moduli,
                             int64_t batch, int64_t M, int64_t K, int64_t N, int32_t *c,
                             void *workspace, size_t workspace_bytes, void *stream) {
    if (batch < 0 || M < 0 || K < 0 || N < 0) return TI_ERR_INVALID_ARGUMENT;
    if (batch > kMaxModuli) return TI_ERR_UNSUPPORTED;
    if (K > 131071) return TI_ERR_UNSUPPORTED;  // 128*128*K < 2^31
    if (batch == 0 || M == 0 || N == 0) return TI_OK;
    if (!a || !b || !moduli || !c) return TI_ERR_INVALID_ARGUMENT;
    ModMagic mm;
    if (!make_magic(moduli, static_cast<int>(batch), mm)) return TI_ERR_INVALID_ARGUMENT;
    DevInfo d;
    int rc = device_info(d);
    if (rc != TI_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (K == 0) return cuda_status(cudaMemsetAsync(c, 0, sizeof(int32_t) * batch * M * N, s));
    size_t need = 0;
    ti_batched_gemm_workspace_size(batch, M, K, N, &need);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return TI_ERR_WORKSPACE;
    const int64_t ld = round_up(K, 16);
    int8_t *ap = static_cast<int8_t *>(workspace);
    int8_t *bp = ap + align256(size_t(batch) * size_t(M) * size_t(ld));
    {
        const int64_t total = batch * M * ld;
        int64_t blocks = (total + 255) / 256;
        if (blocks > int64_t(d.num_sms) * 8) blocks = int64_t(d.num_sms) * 8;
        pad_rows_i8_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(a, batch, M, K, ap, ld);
        int64_t tb = batch * ((ld + 63) / 64) * ((N + 63) / 64);
        if (tb > int64_t(d.num_sms) * 8) tb = int64_t(d.num_sms) * 8;
        transpose_i8_kernel<<<static_cast<unsigned>(tb), 256, 0, s>>>(b, batch, K, N, bp, ld);
        if (cudaGetLastError() != cudaSuccess) return TI_ERR_CUDA;
    }
    return cuda_status(launch_residue_gemm(ap, bp, M, N, K, ld, static_cast<int>(batch), mm, c,
                                           N, 1, d.err, d.num_sms, s));
}

int ti_crt_reconstruct(const int32_t *residues, const int32_t *moduli, int n_mod, int bits,
                       const int32_t *row_exp, const int32_t *col_exp, int64_t rows,
                       int64_t cols, double *out, int64_t ldo, void *stream) {
    if (rows < 0 || cols < 0 || n_mod < 1 || n_mod > kMaxModuli || ldo < cols)
        return TI_ERR_INVALID_ARGUMENT;
    if (bits < 1 || bits > 53) return TI_ERR_INVALID_ARGUMENT;
    if (rows == 0 || cols == 0) return TI_OK;
    if (!residues || !moduli || !row_exp || !col_exp || !out) return TI_ERR_INVALID_ARGUMENT;
    CrtConst K;
    if (!make_crt_const(moduli, n_mod, bits, K)) return TI_ERR_INVALID_ARGUMENT;
    DevInfo d;
    int rc = device_info(d);
    if (rc != TI_OK) return rc;
    return cuda_status(launch_crt(residues, false, cols, rows * cols, rows, cols, row_exp, col_exp,
                                  out, ldo, 0, K, d.num_sms, static_cast<cudaStream_t>(stream)));
}

static void record(void *const *ev, int i, cudaStream_t s) {
    if (ev && ev[i]) cudaEventRecord(static_cast<cudaEvent_t>(ev[i]), s);
}

// The banded pipeline: A split into row bands of band_rows (a multiple of 128).
//   hi: K1(B), K1(A_0) | GEMM(0) | GEMM(1) | ... each GEMM(b) after split_done[b]
//   lo: K1(A_{b+1}) -> split_done[b+1]; wait gemm_done[b]; K3(b)     for b = 0 .. bands-1
// so the GEMM of band b (tensor cores) overlaps the integer work of the split of band b+1
// and the reconstruction of band b-1.  Both streams fork from and join back to `s`.
static int crt_matmul_banded(const double *A, int64_t sa0, int64_t sa1, const double *B,
                             int64_t sb0, int64_t sb1, double *C, int64_t ldc, int64_t m,
                             int64_t n, int64_t k, int out_mode, void *const *ev,
                             cudaStream_t s, const CrtLayout &L, const SplitConst &SCA,
                             const SplitConst &SC,
                             const CrtConst &KC, const DevInfo &d, int bands, int64_t band_rows,
                             int32_t *rexp, int32_t *cexp, int8_t *ares, int8_t *bres,
                             uint8_t *R) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return TI_ERR_CUDA;
    Pipeline *PP = nullptr;
    std::lock_guard<std::mutex> lock(g_pipe[dev < 0 || dev >= kMaxDevices ? 0 : dev].mu);
    int rc = pipeline_for_device(dev, PP);
    if (rc != TI_OK) return rc;
    Pipeline &P = *PP;
    const int64_t a_plane = m * L.ldk, b_plane = n * L.ldk, r_plane = m * L.ldr;
    auto split_a = [&](int b, cudaStream_t st, int bps) {
        const int64_t r0 = int64_t(b) * band_rows;
        const int64_t rows = m - r0 < band_rows ? m - r0 : band_rows;
        const double *Ab = A + r0 * sa0;
        if (sa1 == 1)
            return launch_split(Ab, rows, k, sa0, 1, SCA, rexp + r0, ares + r0 * L.ldk, L.ldk,
                                d.num_sms, st, a_plane, bps, d.err);
        return launch_split(Ab, rows, k, 1, sa1, SCA, rexp + r0, ares + r0 * L.ldk, L.ldk,
                            d.num_sms, st, a_plane, bps, d.err);
    };
    record(ev, 0, s);
    if (cudaEventRecord(P.fork, s) != cudaSuccess) return TI_ERR_CUDA;
    if (cudaStreamWaitEvent(P.hi, P.fork, 0) != cudaSuccess ||
        cudaStreamWaitEvent(P.lo, P.fork, 0) != cudaSuccess)
        return TI_ERR_CUDA;
    // hi: B and the first band of A, at full occupancy (nothing to overlap yet)
    cudaError_t e;
    if (sb0 == 1) e = launch_split(B, n, k, sb1, 1, SC, cexp, bres, L.ldk, d.num_sms, P.hi, 0, 8, d.err);
    else e = launch_split(B, n, k, 1, sb0, SC, cexp, bres, L.ldk, d.num_sms, P.hi, 0, 8, d.err);
    if (e != cudaSuccess) return TI_ERR_CUDA;
    if (split_a(0, P.hi, 8) != cudaSuccess) return TI_ERR_CUDA;
    if (cudaEventRecord(P.split_done[0], P.hi) != cudaSuccess) return TI_ERR_CUDA;
    // lo waits for B's residues before any band split (the split of A needs nothing from B,
    // but sharing SMs with K1(B) would only delay the first GEMM)
    if (cudaStreamWaitEvent(P.lo, P.split_done[0], 0) != cudaSuccess) return TI_ERR_CUDA;
    record(ev, 1, P.hi);
    for (int b = 0; b < bands; ++b) {
        const int64_t r0 = int64_t(b) * band_rows;
        const int64_t rows = m - r0 < band_rows ? m - r0 : band_rows;
        // hi: GEMM(b)
        if (b > 0 && cudaStreamWaitEvent(P.hi, P.split_done[b], 0) != cudaSuccess)
            return TI_ERR_CUDA;
        e = launch_residue_gemm(ares + r0 * L.ldk, bres, rows, n, k, L.ldk, L.n_mod, SC.mm,
                                R + r0 * L.ldr, L.ldr, 0, d.err, d.num_sms, P.hi, a_plane,
                                b_plane, r_plane, nullptr, !SC.symmetric);
        if (e != cudaSuccess) return e == cudaErrorInvalidValue ? TI_ERR_NO_DEVICE : TI_ERR_CUDA;
        if (cudaEventRecord(P.gemm_done[b], P.hi) != cudaSuccess) return TI_ERR_CUDA;
        // lo: split of the next band, then the reconstruction of this one
        if (b + 1 < bands) {
            if (split_a(b + 1, P.lo, kSideBlocksPerSm) != cudaSuccess) return TI_ERR_CUDA;
            if (cudaEventRecord(P.split_done[b + 1], P.lo) != cudaSuccess) return TI_ERR_CUDA;
        }
        if (cudaStreamWaitEvent(P.lo, P.gemm_done[b], 0) != cudaSuccess) return TI_ERR_CUDA;
        if (b == bands - 1) record(ev, 2, P.lo);
        e = launch_k3(R + r0 * L.ldr, L.ldr, r_plane, rows, n, rexp + r0, cexp, C + r0 * ldc,
                      ldc, out_mode, KC, d.err, d.num_sms, P.lo,
                      b == bands - 1 ? 8 : kSideBlocksPerSm);
        if (e != cudaSuccess) return TI_ERR_CUDA;
    }
    if (cudaEventRecord(P.hi_done, P.hi) != cudaSuccess ||
        cudaEventRecord(P.lo_done, P.lo) != cudaSuccess ||
        cudaStreamWaitEvent(s, P.hi_done, 0) != cudaSuccess ||
        cudaStreamWaitEvent(s, P.lo_done, 0) != cudaSuccess)
        return TI_ERR_CUDA;
    record(ev, 3, s);
    return TI_OK;
}

int ti_crt_matmul(const double *A, int64_t sa0, int64_t sa1, const double *B, int64_t sb0,
                  int64_t sb1, double *C, int64_t ldc, int64_t m, int64_t n, int64_t k,
                  int bits, int out_mode, void *workspace, size_t workspace_bytes,
                  void *stream) {
    return ti_crt_matmul_ex(A, sa0, sa1, B, sb0, sb1, C, ldc, m, n, k, bits, out_mode,
                            workspace, workspace_bytes, stream, nullptr);
}

int ti_crt_matmul_events(const double *A, int64_t sa0, int64_t sa1, const double *B,
                         int64_t sb0, int64_t sb1, double *C, int64_t ldc, int64_t m, int64_t n,
                         int64_t k, int bits, int out_mode, void *workspace,
                         size_t workspace_bytes, void *stream, void *const *ev) {
    ti_crt_options_t o;
    std::memset(&o, 0, sizeof(o));
    for (int i = 0; i < 4 && ev; ++i) o.stage_events[i] = ev[i];
    return ti_crt_matmul_ex(A, sa0, sa1, B, sb0, sb1, C, ldc, m, n, k, bits, out_mode,
                            workspace, workspace_bytes, stream, &o);
}

int ti_crt_matmul_ex(const double *A, int64_t sa0, int64_t sa1, const double *B, int64_t sb0,
                     int64_t sb1, double *C, int64_t ldc, int64_t m, int64_t n, int64_t k,
                     int bits, int out_mode, void *workspace, size_t workspace_bytes,
                     void *stream, const ti_crt_options_t *opt) {
    if (out_mode < TI_OUT_STORE || out_mode > TI_OUT_ADD) return TI_ERR_INVALID_ARGUMENT;
    void *const *ev = opt ? opt->stage_events : nullptr;
    CrtLayout L;
    int rc = crt_layout(m, n, k, bits, opt, L);
    if (rc != TI_OK) return rc;
    if (m == 0 || n == 0) return TI_OK;
    if (!C || ldc < n) return TI_ERR_INVALID_ARGUMENT;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DevInfo d;
    rc = device_info(d);
    if (rc != TI_OK) return rc;
    if (k == 0) {  // empty sum: C = 0 (store) or C unchanged
        if (out_mode != TI_OUT_STORE) return TI_OK;
        return cuda_status(cudaMemset2DAsync(C, sizeof(double) * ldc, 0, sizeof(double) * n, m, s));
    }
    if (!A || !B) return TI_ERR_INVALID_ARGUMENT;
    if (!(sa1 == 1 || sa0 == 1) || !(sb0 == 1 || sb1 == 1)) return TI_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return TI_ERR_WORKSPACE;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    int32_t *rexp = reinterpret_cast<int32_t *>(ws + L.off_rexp);
    int32_t *cexp = reinterpret_cast<int32_t *>(ws + L.off_cexp);
    int8_t *ares = reinterpret_cast<int8_t *>(ws + L.off_a);
    int8_t *bres = reinterpret_cast<int8_t *>(ws + L.off_b);
    uint8_t *R = ws + L.off_r;

    SplitConst SCA, SC;
    CrtConst KC;
    const Plan &PL = L.plan;
    // symmetric residues (the products mod p do not depend on the representative; the stage
    // entry ti_crt_split keeps the reference's floor-mod bytes)
    if (!make_matmul_consts(PL, SCA, SC, KC)) return TI_ERR_UNSUPPORTED;

    int bands = opt && opt->bands > 0 ? opt->bands : auto_bands(m);
    if (bands > kMaxBands) bands = kMaxBands;
    int64_t band_rows = (m + bands - 1) / bands;
    band_rows = (band_rows + 127) / 128 * 128;
    bands = static_cast<int>((m + band_rows - 1) / band_rows);
    if (bands > 1 && !use_fused(m, n))
        return crt_matmul_banded(A, sa0, sa1, B, sb0, sb1, C, ldc, m, n, k, out_mode, ev, s, L,
                                 SCA, SC, KC, d, bands, band_rows, rexp, cexp, ares, bres, R);

    // K1: A as m vectors along k (rows), B as n vectors along k (columns)
    cudaError_t e;
    record(ev, 0, s);
    if (sa1 == 1) e = launch_split(A, m, k, sa0, 1, SCA, rexp, ares, L.ldk, d.num_sms, s, 0, 8, d.err);
    else e = launch_split(A, m, k, 1, sa1, SCA, rexp, ares, L.ldk, d.num_sms, s, 0, 8, d.err);
    if (e != cudaSuccess) return TI_ERR_CUDA;
    if (sb0 == 1) e = launch_split(B, n, k, sb1, 1, SC, cexp, bres, L.ldk, d.num_sms, s, 0, 8, d.err);
    else e = launch_split(B, n, k, 1, sb0, SC, cexp, bres, L.ldk, d.num_sms, s, 0, 8, d.err);
    if (e != cudaSuccess) return TI_ERR_CUDA;
    record(ev, 1, s);
    if (use_fused(m, n)) {
        // K2+K3 fused: residue GEMMs with the CRT of each finished tile in the same kernel
        int64_t grid = gemm_output_tiles(m, n);
        if (grid > d.num_sms) grid = d.num_sms;
        if (grid > kFusedMaxCtas) grid = kFusedMaxCtas;
        CrtConst KF = KC;  // A's residues already carry u_i: the epilogue multiplies by 1
        for (int i = 0; i < KF.n_mod; ++i) KF.u[i] = 1;
        e = launch_fused_gemm_crt(ares, bres, m, n, k, L.ldk, KF, rexp, cexp, C, ldc, out_mode, R,
                                  static_cast<int>(grid), d.err, s, !SC.symmetric);
        record(ev, 2, s);
        record(ev, 3, s);
        if (e != cudaSuccess) return e == cudaErrorInvalidValue ? TI_ERR_NO_DEVICE : TI_ERR_CUDA;
        return TI_OK;
    }
    // K2: per-modulus residue GEMMs, mod-reduced to uint8 planes
    const bool lower = opt && opt->lower;
    e = launch_residue_gemm(ares, bres, m, n, k, L.ldk, L.n_mod, SC.mm, R, L.ldr, 0, d.err,
                            d.num_sms, s, 0, 0, 0, nullptr, !SC.symmetric, lower);
    if (e != cudaSuccess) return e == cudaErrorInvalidValue ? TI_ERR_NO_DEVICE : TI_ERR_CUDA;
    // K3: exact CRT + inverse scaling
    record(ev, 2, s);
    e = launch_k3(R, L.ldr, m * L.ldr, m, n, rexp, cexp, C, ldc, out_mode, KC, d.err, d.num_sms, s,
                  8, lower);
    record(ev, 3, s);
    return cuda_status(e);
}

// ---------------------------------------------------------------------------------------
// host operands: copies pipelined against the kernels in row bands of A
// ---------------------------------------------------------------------------------------
// One row band of C = A @ B, all stages in order on `s`, inside the workspace laid out for
// the full product (L).  B's exponents and residues are produced when split_b and reused by
// the following bands.
// B's column exponents and residues (once per product, before the first band).
static int crt_split_b(const double *B, int64_t sb0, int64_t sb1, int64_t n, int64_t k,
                       const CrtLayout &L, const SplitConst &SC, uint8_t *ws, cudaStream_t s,
                       const DevInfo &d) {
    int32_t *cexp = reinterpret_cast<int32_t *>(ws + L.off_cexp);
    int8_t *bres = reinterpret_cast<int8_t *>(ws + L.off_b);
    const cudaError_t e =
        sb0 == 1 ? launch_split(B, n, k, sb1, 1, SC, cexp, bres, L.ldk, d.num_sms, s, 0, 8, d.err)
                 : launch_split(B, n, k, 1, sb0, SC, cexp, bres, L.ldk, d.num_sms, s, 0, 8, d.err);
    return cuda_status(e);
}

// One row band of C = A @ B, B already split (crt_split_b).
static int crt_band_compute(const double *A, int64_t sa0, int64_t sa1, double *C, int64_t ldc,
                            int64_t rows, int64_t n, int64_t k, const CrtLayout &L,
                            const SplitConst &SCA, const SplitConst &SC, const CrtConst &KC,
                            uint8_t *ws, cudaStream_t s, const DevInfo &d) {
    int32_t *rexp = reinterpret_cast<int32_t *>(ws + L.off_rexp);
    int32_t *cexp = reinterpret_cast<int32_t *>(ws + L.off_cexp);
    int8_t *ares = reinterpret_cast<int8_t *>(ws + L.off_a);
    int8_t *bres = reinterpret_cast<int8_t *>(ws + L.off_b);
    uint8_t *R = ws + L.off_r;
    cudaError_t e;
    if (sa1 == 1) e = launch_split(A, rows, k, sa0, 1, SCA, rexp, ares, L.ldk, d.num_sms, s, 0, 8, d.err);
    else e = launch_split(A, rows, k, 1, sa1, SCA, rexp, ares, L.ldk, d.num_sms, s, 0, 8, d.err);
    if (e != cudaSuccess) return TI_ERR_CUDA;
    e = launch_residue_gemm(ares, bres, rows, n, k, L.ldk, L.n_mod, SC.mm, R, L.ldr, 0, d.err,
                            d.num_sms, s, 0, 0, 0, nullptr, !SC.symmetric);
    if (e != cudaSuccess) return e == cudaErrorInvalidValue ? TI_ERR_NO_DEVICE : TI_ERR_CUDA;
    e = launch_k3(R, L.ldr, rows * L.ldr, rows, n, rexp, cexp, C, ldc, TI_OUT_STORE, KC, d.err,
                  d.num_sms, s);
    return cuda_status(e);
}
// Device copies of A, B and C ahead of the ti_crt_matmul_ex workspace, 256-byte aligned.
static int host_layout(int64_t m, int64_t n, int64_t k, int bits, const ti_crt_options_t *opt,
                       size_t &off_a, size_t &off_b, size_t &off_c, size_t &off_ws,
                       size_t &ws_inner, size_t &total) {
    const int rc = ti_crt_workspace_size_ex(m, n, k, bits, opt, &ws_inner);
    if (rc != TI_OK) return rc;
    size_t off = 0;
    off_a = off; off += align256(sizeof(double) * size_t(m) * size_t(k));
    off_b = off; off += align256(sizeof(double) * size_t(k) * size_t(n));
    off_c = off; off += align256(sizeof(double) * size_t(m) * size_t(n));
    off_ws = off; off += ws_inner;
    total = off;
    return TI_OK;
}

int ti_crt_host_workspace_size(int64_t m, int64_t n, int64_t k, int bits,
                               const ti_crt_options_t *opt, size_t *bytes) {
    if (!bytes) return TI_ERR_INVALID_ARGUMENT;
    size_t oa, ob, oc, ow, wi, total;
    const int rc = host_layout(m, n, k, bits, opt, oa, ob, oc, ow, wi, total);
    if (rc != TI_OK) return rc;
    *bytes = total;
    return TI_OK;
}

// Row bands of the host-operand pipeline: band b is rows [r0[b], r0[b] + rows[b]).  The
// copies are PCIe-bound: all of B, then A, in; C out.  C starts out once B and A's first band
// are in and computed, and ends after A's last band is in, computed and out; while A comes in,
// C goes out at the same byte rate, about one band behind.  So for m >= 4096 the first band
// is short (256 rows), the middle ones about 1024 rows and the last ones shrink (512, 256,
// 128 rows) to shorten the tail.  n > 0 in options.bands asks for n equal bands instead.
// Returns the band count.
static int host_bands(int64_t m, const ti_crt_options_t *opt, int64_t (&r0)[kMaxBands],
                      int64_t (&rows)[kMaxBands]) {
    int count = 0;
    auto push = [&](int64_t r) {
        r0[count] = count ? r0[count - 1] + rows[count - 1] : 0;
        rows[count++] = r;
    };
    auto equal = [&](int nb) {
        if (nb > kMaxBands) nb = kMaxBands;
        if (nb < 1) nb = 1;
        int64_t br = (m + nb - 1) / nb;
        br = (br + 127) / 128 * 128;
        for (int64_t r = 0; r < m; r += br) push(m - r < br ? m - r : br);
        return count;
    };
    if (opt && opt->bands > 0) return equal(opt->bands);
    if (m < 1024) return equal(1);
    if (m < 4096) return equal(4);
    constexpr int64_t kHead = 256, kTail[3] = {512, 256, 128};
    const int64_t mid = m - kHead - (kTail[0] + kTail[1] + kTail[2]);
    int64_t nmid = (mid + 1023) / 1024;
    if (nmid > kMaxBands - 4) nmid = kMaxBands - 4;
    int64_t br = (mid + nmid - 1) / nmid;
    br = (br + 127) / 128 * 128;
    push(kHead);
    for (int64_t r = 0; r < mid; r += br) push(mid - r < br ? mid - r : br);
    for (int64_t t : kTail) push(t);
    return count;
}

// Host band copy of rows [r0, r0+rows) of an m x k operand with strides (s0, s1), one of
// them 1, into its dense device copy of the same orientation.
static cudaError_t copy_rows_h2d(double *dst, const double *src, int64_t m, int64_t k, int64_t s0,
                                 int64_t s1, int64_t r0, int64_t rows, cudaStream_t st) {
    if (rows == 0 || k == 0) return cudaSuccess;
    if (s1 == 1)  // row-major rows: rows x k, pitch s0
        return cudaMemcpy2DAsync(dst + r0 * k, sizeof(double) * k, src + r0 * s0,
                                 sizeof(double) * s0, sizeof(double) * k, rows,
                                 cudaMemcpyHostToDevice, st);
    // column-major: k columns of `rows` contiguous elements, pitch s1
    return cudaMemcpy2DAsync(dst + r0, sizeof(double) * m, src + r0, sizeof(double) * s1,
                             sizeof(double) * rows, k, cudaMemcpyHostToDevice, st);
}

int ti_crt_matmul_host(const double *A, int64_t sa0, int64_t sa1, const double *B, int64_t sb0,
                       int64_t sb1, double *C, int64_t ldc, int64_t m, int64_t n, int64_t k,
                       int bits, void *workspace, size_t workspace_bytes, void *stream,
                       const ti_crt_options_t *opt) {
    size_t off_a, off_b, off_c, off_ws, ws_inner, total;
    int rc = host_layout(m, n, k, bits, opt, off_a, off_b, off_c, off_ws, ws_inner, total);
    if (rc != TI_OK) return rc;
    if (m == 0 || n == 0) return TI_OK;
    if (!C || ldc < n) return TI_ERR_INVALID_ARGUMENT;
    if (k > 0 && (!A || !B)) return TI_ERR_INVALID_ARGUMENT;
    if (k > 0 && (!(sa1 == 1 || sa0 == 1) || !(sb0 == 1 || sb1 == 1)))
        return TI_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < total || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return TI_ERR_WORKSPACE;
    DevInfo d;
    rc = device_info(d);
    if (rc != TI_OK) return rc;
    CrtLayout L;
    rc = crt_layout(m, n, k, bits, opt, L);
    if (rc != TI_OK) return rc;
    SplitConst SCA, SC;
    CrtConst KC;
    if (k > 0 && !make_matmul_consts(L.plan, SCA, SC, KC)) return TI_ERR_UNSUPPORTED;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TI_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_pipe[dev].mu);
    Pipeline *PP = nullptr;
    rc = pipeline_for_device(dev, PP);
    if (rc != TI_OK) return rc;
    Pipeline &P = *PP;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    double *dA = reinterpret_cast<double *>(ws + off_a);
    double *dB = reinterpret_cast<double *>(ws + off_b);
    double *dC = reinterpret_cast<double *>(ws + off_c);
    // device strides of the dense copies (same orientation as the host operands)
    const int64_t da0 = (sa1 == 1) ? k : 1, da1 = (sa1 == 1) ? 1 : m;
    const int64_t db0 = (sb1 == 1) ? n : 1, db1 = (sb1 == 1) ? 1 : k;
    int64_t band_r0[kMaxBands], band_rows[kMaxBands];
    const int bands = host_bands(m, opt, band_r0, band_rows);

    if (cudaEventRecord(P.fork, s) != cudaSuccess ||
        cudaStreamWaitEvent(P.h2d, P.fork, 0) != cudaSuccess ||
        cudaStreamWaitEvent(P.d2h, P.fork, 0) != cudaSuccess)
        return TI_ERR_CUDA;
    // copy engine in: all of B (its column exponents need every row), then A band by band
    if (k > 0) {
        cudaError_t e = (sb1 == 1)
            ? cudaMemcpy2DAsync(dB, sizeof(double) * n, B, sizeof(double) * sb0,
                                sizeof(double) * n, k, cudaMemcpyHostToDevice, P.h2d)
            : cudaMemcpy2DAsync(dB, sizeof(double) * k, B, sizeof(double) * sb1,
                                sizeof(double) * k, n, cudaMemcpyHostToDevice, P.h2d);
        if (e != cudaSuccess || cudaEventRecord(P.b_in, P.h2d) != cudaSuccess) return TI_ERR_CUDA;
        for (int b = 0; b < bands; ++b) {
            const int64_t r0 = band_r0[b], rows = band_rows[b];
            if (copy_rows_h2d(dA, A, m, k, sa0, sa1, r0, rows, P.h2d) != cudaSuccess ||
                cudaEventRecord(P.a_in[b], P.h2d) != cudaSuccess)
                return TI_ERR_CUDA;
        }
        // B is split as soon as it is in, while A's first band is still arriving
        if (cudaStreamWaitEvent(s, P.b_in, 0) != cudaSuccess) return TI_ERR_CUDA;
        rc = crt_split_b(dB, db0, db1, n, k, L, SC, ws + off_ws, s, d);
        if (rc != TI_OK) return rc;
    }
    // kernels on the caller's stream, one band at a time; each band's C goes out as soon as
    // it is reconstructed
    for (int b = 0; b < bands; ++b) {
        const int64_t r0 = band_r0[b], rows = band_rows[b];
        if (k > 0) {
            if (cudaStreamWaitEvent(s, P.a_in[b], 0) != cudaSuccess) return TI_ERR_CUDA;
            // band b of C = A[r0:r0+rows] @ B
            rc = crt_band_compute(dA + r0 * da0, da0, da1, dC + r0 * n, n, rows, n, k, L, SCA,
                                  SC, KC, ws + off_ws, s, d);
            if (rc != TI_OK) return rc;
        } else if (cudaMemsetAsync(dC + r0 * n, 0, sizeof(double) * rows * n, s) != cudaSuccess) {
            return TI_ERR_CUDA;  // empty sum
        }
        if (cudaEventRecord(P.c_ready[b], s) != cudaSuccess ||
            cudaStreamWaitEvent(P.d2h, P.c_ready[b], 0) != cudaSuccess ||
            cudaMemcpy2DAsync(C + r0 * ldc, sizeof(double) * ldc, dC + r0 * n, sizeof(double) * n,
                              sizeof(double) * n, rows, cudaMemcpyDeviceToHost, P.d2h) != cudaSuccess)
            return TI_ERR_CUDA;
    }
    if (cudaEventRecord(P.lo_done, P.d2h) != cudaSuccess ||
        cudaEventRecord(P.hi_done, P.h2d) != cudaSuccess ||
        cudaStreamWaitEvent(s, P.lo_done, 0) != cudaSuccess ||
        cudaStreamWaitEvent(s, P.hi_done, 0) != cudaSuccess)
        return TI_ERR_CUDA;
    return TI_OK;
}

int ti_device_error(int *code_out, int reset) {
    if (!code_out) return TI_ERR_INVALID_ARGUMENT;
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return TI_ERR_CUDA;
    *code_out = v;
    if (reset) {
        const int z = 0;
        if (cudaMemcpyToSymbol(g_device_error, &z, sizeof(int)) != cudaSuccess) return TI_ERR_CUDA;
    }
    return TI_OK;
}

}  // extern "C"
