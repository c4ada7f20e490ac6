// ti_scale.cuh -- the reference's power-of-two scaling of one float64, in exact integer
// arithmetic, shared by the split kernels (ti_split.cu, ti_split_tc.cu).
//
// Restates src/tensor_inv/crt_matmul.py:32-38 (_scale_to_int): per vector the frexp exponent
// e of max(max |x|, 1e-300), then v = round_half_even(x * 2^(bits - e)) for every element.
#pragma once

#include "ti_common.cuh"

namespace ti {

__device__ __forceinline__ uint64_t abs_bits(double x) {
    return static_cast<uint64_t>(__double_as_longlong(x)) & 0x7FFFFFFFFFFFFFFFull;
}

// frexp exponent of max(m, 1e-300) from the bit pattern of m = max |x| (non-negative).
__device__ __forceinline__ int exp_from_maxbits(uint64_t mb) {
    if (mb >= 0x7FF0000000000000ull) return kNonfiniteExp;  // inf or NaN in the vector
    if (mb < 0x0010000000000000ull) return -996;             // zero or subnormal: clamp
    int e = static_cast<int>(mb >> 52) - 1022;               // frexp exponent
    return e < -996 ? -996 : e;                               // clamp(min=1e-300)
}

// round_half_even(|x| * 2^(bits - e)) for |x| < 2^e; also returns the sign of x.
__device__ __forceinline__ uint64_t scaled_magnitude(double x, int bits, int e, bool &neg) {
    const uint64_t u = static_cast<uint64_t>(__double_as_longlong(x));
    neg = (u >> 63) != 0;
    const int be = static_cast<int>((u >> 52) & 0x7FF);
    const uint64_t f = u & 0x000FFFFFFFFFFFFFull;
    uint64_t sig;
    int ex;  // |x| = sig * 2^ex
    if (be == 0) {
        sig = f;
        ex = -1074;
    } else {
        sig = f | 0x0010000000000000ull;
        ex = be - 1075;
    }
    int sh = e - bits - ex;  // right shift, >= 0 because |x| < 2^e
    if (sh <= 0) return sig << (-sh);  // sh == 0 only (kept general)
    if (sh > 63) sh = 63;              // sig < 2^53: shifts >= 54 all round to zero
    const uint64_t q = sig >> sh;
    const uint64_t rem = sig & ((1ull << sh) - 1);
    const uint64_t half = 1ull << (sh - 1);
    return q + ((rem > half) || (rem == half && (q & 1)));
}

}  // namespace ti
