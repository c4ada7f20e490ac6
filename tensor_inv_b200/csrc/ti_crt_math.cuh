// ti_crt_math.cuh -- exact CRT finish for one output element, shared by the standalone
// reconstruction kernel (K3) and the fused GEMM+CRT kernel.
//
// Given, for one element, the four 64-bit column sums of S = sum_i t_i * M_i (t_i =
// (r_i * u_i) mod p_i, M_i = M / p_i) and the 32.32 fixed-point F = sum_i t_i / p_i, it
// forms x = S - floor(F + 1/2) * M mod 2^128 (exact), lifts x into [-(M-1)/2, (M-1)/2] as
// the reference's `x > M // 2 -> x - M` does (crt_matmul.py:87-89), rounds float(x) to
// nearest-even and applies ldexp(., row_exp + col_exp - 2*bits) with gradual underflow
// (crt_matmul.py:90).
#pragma once

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

// One element: column sums s0..s3 of S, F = S / M in fixed point with kFracBits fraction
// bits, exponent sum e2 = re + ce - 2*bits.
template <int kFracBits = 32>
__device__ __forceinline__ double crt_finish(uint64_t s0, uint64_t s1, uint64_t s2, uint64_t s3,
                                             uint64_t f, int e2, const CrtConst &K) {
    // carry-propagate the four 64-bit column sums into 128 bits
    uint64_t c = s0;
    uint32_t w0 = static_cast<uint32_t>(c);
    c = (c >> 32) + s1;
    uint32_t w1 = static_cast<uint32_t>(c);
    c = (c >> 32) + s2;
    uint32_t w2 = static_cast<uint32_t>(c);
    c = (c >> 32) + s3;
    uint32_t w3 = static_cast<uint32_t>(c);
    // x = S - q*M  (mod 2^128)
    const uint32_t qv = static_cast<uint32_t>((f + (1ull << (kFracBits - 1))) >> kFracBits);
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
    return int128_ldexp(w0, w1, w2, w3, e2);
}

__device__ __forceinline__ double nan_value() {
    return __longlong_as_double(0x7FF8000000000000ll);
}

// out_mode 0: store, 1: *dst - v, 2: *dst + v (one IEEE operation, as `C -= product`).
__device__ __forceinline__ void write_mode(double *dst, double v, int out_mode) {
    if (out_mode == 0) *dst = v;
    else if (out_mode == 1) *dst = __dsub_rn(*dst, v);
    else *dst = __dadd_rn(*dst, v);
}

}  // namespace ti
