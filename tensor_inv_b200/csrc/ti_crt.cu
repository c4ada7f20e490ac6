// ti_crt.cu -- K3: exact CRT reconstruction + inverse power-of-two scaling to float64.
//
// Restates src/tensor_inv/crt_matmul.py:68-98 (_crt_precompute, _crt_reconstruct) exactly:
//   x   = sum_i r_i * M_i * (M_i^-1 mod p_i)  mod M,   lifted to (-M/2, M/2]
//   out = math.ldexp(float(x), row_exp + col_exp - 2*bits)
// and so replaces the reference's double-double approximation (crt_kernel.cu:93-125).
//
// Per element, with t_i = (r_i * u_i) mod p_i and u_i = M_i^-1 mod p_i:
//   S = sum_i t_i * M_i  (== x mod M, 0 <= S < n_mod * M)   accumulated mod 2^128,
//   F = sum_i t_i / p_i  (== S / M)                        in 32.32 fixed point,
//   q = floor(F + 1/2),  x = S - q*M  (exact mod 2^128; |x| < 2^126).
// The fixed-point error of F is below 1600 * 2^-32; a final exact range check on x
// (lift_symmetric) corrects the quotient in the rare case the estimate is off by one.
// float(x) is rounded to nearest-even from the top 64 bits plus a sticky bit; the final
// scaling reproduces ldexp's gradual underflow (a second rounding for subnormal results).
#include "ti_common.cuh"

namespace ti {

// x * 2^e for a float64 x that is zero or normal, rounded to nearest-even with gradual
// underflow, +-inf on overflow: the semantics of C ldexp (and Python math.ldexp for
// results in range).  Written from the IEEE-754 encoding.
__device__ __forceinline__ double scale_pow2_rne(double x, int e) {
    const uint64_t b = static_cast<uint64_t>(__double_as_longlong(x));
    const uint64_t sign = b & 0x8000000000000000ull;
    const int be = static_cast<int>((b >> 52) & 0x7FF);
    if (be == 0) return x;  // +-0
    const int nbe = be + e;
    if (nbe >= 2047) return __longlong_as_double(static_cast<long long>(sign | 0x7FF0000000000000ull));
    const uint64_t frac = b & 0x000FFFFFFFFFFFFFull;
    if (nbe >= 1)
        return __longlong_as_double(
            static_cast<long long>(sign | (static_cast<uint64_t>(nbe) << 52) | frac));
    // subnormal result: significand (2^52 + frac) * 2^(nbe-1) in units of 2^-1074
    const uint64_t sig = frac | 0x0010000000000000ull;
    const int sh = 1 - nbe;
    if (sh > 63) return __longlong_as_double(static_cast<long long>(sign));
    uint64_t q = sig >> sh;
    const uint64_t rem = sig & ((1ull << sh) - 1);
    const uint64_t half = 1ull << (sh - 1);
    q += (rem > half) || (rem == half && (q & 1));
    return __longlong_as_double(static_cast<long long>(sign | q));
}

// Correctly rounded float64 of the signed 128-bit integer (w3:w2:w1:w0), times 2^e.
__device__ __forceinline__ double int128_ldexp(uint32_t w0, uint32_t w1, uint32_t w2,
                                               uint32_t w3, int e) {
    uint64_t lo = (static_cast<uint64_t>(w1) << 32) | w0;
    uint64_t hi = (static_cast<uint64_t>(w3) << 32) | w2;
    const bool neg = (hi >> 63) != 0;
    if (neg) {  // two's complement negate
        lo = ~lo + 1;
        hi = ~hi + (lo == 0 ? 1 : 0);
    }
    double d;
    int e2;
    if (hi == 0) {
        d = __ull2double_rn(lo);
        e2 = 0;
    } else {
        const int lz = __clzll(static_cast<long long>(hi));
        const uint64_t top = lz ? ((hi << lz) | (lo >> (64 - lz))) : hi;
        const uint64_t rest = lz ? (lo << lz) : lo;
        d = __ull2double_rn(top | (rest != 0 ? 1ull : 0ull));
        e2 = 64 - lz;
    }
    if (neg) d = -d;
    return scale_pow2_rne(d, e2 + e);
}

// Exact guard on the quotient estimate: the lifted value must lie in [-H, H] with
// H = (M-1)/2.  A quotient off by one (possible only when x is within ~2^-21 M of +-M/2)
// leaves |x| just above H; moving it by M makes the result exact for any residues.
__device__ __forceinline__ void lift_symmetric(uint32_t &w0, uint32_t &w1, uint32_t &w2,
                                               uint32_t &w3, const CrtConst &K) {
    const bool neg = (w3 >> 31) != 0;
    uint32_t a0 = w0, a1 = w1, a2 = w2, a3 = w3;  // |x|
    if (neg) {
        a0 = ~a0; a1 = ~a1; a2 = ~a2; a3 = ~a3;
        uint64_t c = static_cast<uint64_t>(a0) + 1; a0 = static_cast<uint32_t>(c);
        c = (c >> 32) + a1; a1 = static_cast<uint32_t>(c);
        c = (c >> 32) + a2; a2 = static_cast<uint32_t>(c);
        c = (c >> 32) + a3; a3 = static_cast<uint32_t>(c);
    }
    const bool gt = (a3 != K.H[3]) ? a3 > K.H[3]
                  : (a2 != K.H[2]) ? a2 > K.H[2]
                  : (a1 != K.H[1]) ? a1 > K.H[1]
                  : a0 > K.H[0];
    if (!gt) return;
    // x -= M (x > H) or x += M (x < -H)
    uint64_t c;
    if (!neg) {
        uint64_t bw = 0;
        c = static_cast<uint64_t>(w0) - K.M[0]; w0 = static_cast<uint32_t>(c); bw = (c >> 63) & 1;
        c = static_cast<uint64_t>(w1) - K.M[1] - bw; w1 = static_cast<uint32_t>(c); bw = (c >> 63) & 1;
        c = static_cast<uint64_t>(w2) - K.M[2] - bw; w2 = static_cast<uint32_t>(c); bw = (c >> 63) & 1;
        c = static_cast<uint64_t>(w3) - K.M[3] - bw; w3 = static_cast<uint32_t>(c);
    } else {
        c = static_cast<uint64_t>(w0) + K.M[0]; w0 = static_cast<uint32_t>(c);
        c = (c >> 32) + w1 + K.M[1]; w1 = static_cast<uint32_t>(c);
        c = (c >> 32) + w2 + K.M[2]; w2 = static_cast<uint32_t>(c);
        c = (c >> 32) + w3 + K.M[3]; w3 = static_cast<uint32_t>(c);
    }
}

template <int kOutMode>
__device__ __forceinline__ void write_out(double *dst, double v) {
    if (kOutMode == 0) *dst = v;
    else if (kOutMode == 1) *dst = __dsub_rn(*dst, v);
    else *dst = __dadd_rn(*dst, v);
}

// Residues in: uint8 planes R[i][row][ldr] (values in [0, p_i)) when kInU8, else int32
// planes (any value, reduced here).  Each thread reconstructs 4 consecutive columns.
template <bool kInU8, int kOutMode>
__global__ void __launch_bounds__(256) crt_kernel(
    const void *__restrict__ Rv, int64_t ldr, int64_t plane, int64_t rows, int64_t cols,
    const int32_t *__restrict__ row_exp, const int32_t *__restrict__ col_exp,
    double *__restrict__ C, int64_t ldc, const __grid_constant__ CrtConst K) {
    // t = (r * u_i) mod p_i as a table over r in [0, 128) for every modulus
    __shared__ uint8_t lut[kMaxModuli][128];
    for (int idx = threadIdx.x; idx < K.n_mod * 128; idx += blockDim.x) {
        const int i = idx >> 7, r = idx & 127;
        lut[i][r] = static_cast<uint8_t>((static_cast<uint32_t>(r) * K.u[i]) % K.mm.p[i]);
    }
    __syncthreads();

    const int64_t groups = (cols + 3) >> 2;
    const int64_t total = rows * groups;
    const bool vec_out = ((reinterpret_cast<uintptr_t>(C) & 15) == 0) && ((ldc & 1) == 0);
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = idx / groups;
        const int64_t col = (idx - row * groups) << 2;
        const int nc = cols - col < 4 ? static_cast<int>(cols - col) : 4;

        uint64_t s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0}, s2[4] = {0, 0, 0, 0},
                 s3[4] = {0, 0, 0, 0}, f[4] = {0, 0, 0, 0};
        for (int i = 0; i < K.n_mod; ++i) {
            uint32_t r4[4];
            if (kInU8) {
                const uint8_t *src = static_cast<const uint8_t *>(Rv) + i * plane + row * ldr + col;
                const uint32_t w = *reinterpret_cast<const uint32_t *>(src);  // ldr % 16 == 0
#pragma unroll
                for (int e = 0; e < 4; ++e) r4[e] = (w >> (8 * e)) & 0xFFu;
            } else {
                const int32_t *src = static_cast<const int32_t *>(Rv) + i * plane + row * ldr + col;
                const int ip = static_cast<int>(K.mm.p[i]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    int v = e < nc ? src[e] % ip : 0;
                    r4[e] = static_cast<uint32_t>(v < 0 ? v + ip : v);
                }
            }
            const uint32_t m0 = K.Mi[i][0], m1 = K.Mi[i][1], m2 = K.Mi[i][2], m3 = K.Mi[i][3];
            const uint32_t fi = K.finv[i];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t t = lut[i][r4[e] & 127];
                s0[e] += static_cast<uint64_t>(t) * m0;
                s1[e] += static_cast<uint64_t>(t) * m1;
                s2[e] += static_cast<uint64_t>(t) * m2;
                s3[e] += static_cast<uint64_t>(t) * m3;
                f[e] += static_cast<uint64_t>(t) * fi;
            }
        }
        const int re = row_exp[row];
        double outv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int ce = e < nc ? col_exp[col + e] : 0;
            if (re == kNonfiniteExp || ce == kNonfiniteExp) {
                outv[e] = __longlong_as_double(0x7FF8000000000000ll);
                continue;
            }
            // carry-propagate the four 64-bit column sums into 128 bits
            uint64_t c = s0[e];
            uint32_t w0 = static_cast<uint32_t>(c);
            c = (c >> 32) + s1[e];
            uint32_t w1 = static_cast<uint32_t>(c);
            c = (c >> 32) + s2[e];
            uint32_t w2 = static_cast<uint32_t>(c);
            c = (c >> 32) + s3[e];
            uint32_t w3 = static_cast<uint32_t>(c);
            // x = S - q*M  (mod 2^128)
            const uint32_t qv = static_cast<uint32_t>((f[e] + 0x80000000ull) >> 32);
            uint64_t b = static_cast<uint64_t>(qv) * K.M[0];
            uint64_t d = static_cast<uint64_t>(w0) - static_cast<uint32_t>(b);
            w0 = static_cast<uint32_t>(d);
            uint64_t borrow = (d >> 63) & 1;
            b = (b >> 32) + static_cast<uint64_t>(qv) * K.M[1];
            d = static_cast<uint64_t>(w1) - static_cast<uint32_t>(b) - borrow;
            w1 = static_cast<uint32_t>(d);
            borrow = (d >> 63) & 1;
            b = (b >> 32) + static_cast<uint64_t>(qv) * K.M[2];
            d = static_cast<uint64_t>(w2) - static_cast<uint32_t>(b) - borrow;
            w2 = static_cast<uint32_t>(d);
            borrow = (d >> 63) & 1;
            b = (b >> 32) + static_cast<uint64_t>(qv) * K.M[3];
            d = static_cast<uint64_t>(w3) - static_cast<uint32_t>(b) - borrow;
            w3 = static_cast<uint32_t>(d);
            lift_symmetric(w0, w1, w2, w3, K);
            outv[e] = int128_ldexp(w0, w1, w2, w3, re + ce - K.two_bits);
        }
        double *dst = C + row * ldc + col;
        if (nc == 4 && vec_out && kOutMode == 0) {
            reinterpret_cast<double2 *>(dst)[0] = make_double2(outv[0], outv[1]);
            reinterpret_cast<double2 *>(dst)[1] = make_double2(outv[2], outv[3]);
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (e < nc) write_out<kOutMode>(dst + e, outv[e]);
        }
    }
}

template <bool kInU8>
static cudaError_t launch_crt_t(const void *R, int64_t ldr, int64_t plane, int64_t rows,
                                int64_t cols, const int32_t *row_exp, const int32_t *col_exp,
                                double *C, int64_t ldc, int out_mode, const CrtConst &K,
                                int num_sms, cudaStream_t stream) {
    const int64_t total = rows * ((cols + 3) >> 2);
    int64_t blocks = (total + 255) / 256;
    if (blocks > int64_t(num_sms) * 8) blocks = int64_t(num_sms) * 8;
    const unsigned g = static_cast<unsigned>(blocks);
    if (out_mode == 0)
        crt_kernel<kInU8, 0><<<g, 256, 0, stream>>>(R, ldr, plane, rows, cols, row_exp, col_exp, C, ldc, K);
    else if (out_mode == 1)
        crt_kernel<kInU8, 1><<<g, 256, 0, stream>>>(R, ldr, plane, rows, cols, row_exp, col_exp, C, ldc, K);
    else
        crt_kernel<kInU8, 2><<<g, 256, 0, stream>>>(R, ldr, plane, rows, cols, row_exp, col_exp, C, ldc, K);
    return cudaGetLastError();
}

cudaError_t launch_crt(const void *R, bool in_u8, int64_t ldr, int64_t plane, int64_t rows,
                       int64_t cols, const int32_t *row_exp, const int32_t *col_exp, double *C,
                       int64_t ldc, int out_mode, const CrtConst &K, int num_sms,
                       cudaStream_t stream) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    if (in_u8)
        return launch_crt_t<true>(R, ldr, plane, rows, cols, row_exp, col_exp, C, ldc, out_mode, K,
                                  num_sms, stream);
    return launch_crt_t<false>(R, ldr, plane, rows, cols, row_exp, col_exp, C, ldc, out_mode, K,
                               num_sms, stream);
}

}  // namespace ti
