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
#include "ti_crt_math.cuh"

namespace ti {

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
    // t = (r * u_i) mod p_i as a table over r in [0, 256) for every modulus
    __shared__ uint8_t lut[kMaxModuli][256];
    for (int idx = threadIdx.x; idx < K.n_mod * 256; idx += blockDim.x) {
        const int i = idx >> 8, r = idx & 255;
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
                const uint32_t t = lut[i][r4[e] & 255];
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
            outv[e] = crt_finish(s0[e], s1[e], s2[e], s3[e], f[e], re + ce - K.two_bits, K);
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
                                int num_sms, cudaStream_t stream, int blocks_per_sm) {
    const int64_t total = rows * ((cols + 3) >> 2);
    int64_t blocks = (total + 255) / 256;
    if (blocks > int64_t(num_sms) * blocks_per_sm) blocks = int64_t(num_sms) * blocks_per_sm;
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
                       cudaStream_t stream, int blocks_per_sm) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    if (in_u8)
        return launch_crt_t<true>(R, ldr, plane, rows, cols, row_exp, col_exp, C, ldc, out_mode, K,
                                  num_sms, stream, blocks_per_sm);
    return launch_crt_t<false>(R, ldr, plane, rows, cols, row_exp, col_exp, C, ldc, out_mode, K,
                               num_sms, stream, blocks_per_sm);
}

}  // namespace ti
