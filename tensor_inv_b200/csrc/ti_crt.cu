// ti_crt.cu -- K3: exact CRT reconstruction + inverse power-of-two scaling to float64.
//
// Restates src/tensor_inv/crt_matmul.py:62-92 (_crt_precompute, _crt_reconstruct) exactly:
//   x   = sum_i r_i * M_i * (M_i^-1 mod p_i)  mod M,   lifted to (-M/2, M/2]
//   out = math.ldexp(float(x), row_exp + col_exp - 2*bits)
// and so replaces the reference's double-double approximation (crt_kernel.cu:93-125).
//
// Per element, with t_i = (r_i * u_i) mod p_i and u_i = M_i^-1 mod p_i:
//   S = sum_i t_i * M_i  (== x mod M, 0 <= S < n_mod * M)   accumulated mod 2^128,
//   F = sum_i t_i / p_i  (== S / M)                        in 48-bit fixed point,
//   q = floor(F + 1/2),  x = S - q*M  (exact mod 2^128; |x| < 2^126).
// Both sums run over groups of three moduli (CrtConst::coef/Mg/fgl/fgh), one 128-bit
// multiply-add per group.  The fixed-point error of F is below 2^-20; a final exact range
// check on x (lift_symmetric) corrects the quotient if the estimate is ever off by one.
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

// Residues in: uint8 planes R[i][row][ldr] of t_i = (r_i * u_i) mod p_i (written so by the
// residue GEMM) when kInU8, else int32 planes of residues r_i (any value, reduced and
// weighted here).  Each thread reconstructs 4 consecutive columns of one row; blocks walk
// rows with blockIdx.y and column groups with blockIdx.x (no integer division).
// kMaxM bounds the moduli count at compile time (16 for the wide set, 32 otherwise) so the
// per-thread residue words fit in fewer registers.
template <bool kInU8, int kOutMode, int kMaxM>
__global__ void __launch_bounds__(256, 3) crt_kernel(
    const void *__restrict__ Rv, int64_t ldr, int64_t plane, int64_t rows, int64_t cols,
    const int32_t *__restrict__ row_exp, const int32_t *__restrict__ col_exp,
    double *__restrict__ C, int64_t ldc, int lower, const __grid_constant__ CrtConst K) {
    const int64_t groups = (cols + 3) >> 2;
    const bool vec_out = ((reinterpret_cast<uintptr_t>(C) & 15) == 0) && ((ldc & 1) == 0);
    for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
        const int re = row_exp[row];
        for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
             g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            const int64_t col = g << 2;
            if (lower && col > row) continue;  // the group lies above the diagonal
            const int nc = cols - col < 4 ? static_cast<int>(cols - col) : 4;
            // t bytes of every modulus, 4 columns per word, all loads in flight at once
            uint32_t w[kMaxM];
            if (kInU8) {
                const uint8_t *src = static_cast<const uint8_t *>(Rv) + row * ldr + col;
#pragma unroll
                for (int i = 0; i < kMaxM; ++i)
                    w[i] = i < K.n_mod
                               ? __ldg(reinterpret_cast<const unsigned int *>(src + i * plane))
                               : 0u;
            } else {
                const int32_t *src = static_cast<const int32_t *>(Rv) + row * ldr + col;
#pragma unroll 1
                for (int i = 0; i < K.n_mod; ++i) {
                    const int ip = static_cast<int>(K.mm.p[i]);
                    uint32_t word = 0;
                    for (int e = 0; e < 4; ++e) {
                        int v = e < nc ? src[i * plane + e] % ip : 0;
                        v = v < 0 ? v + ip : v;
                        word |= ((static_cast<uint32_t>(v) * K.u[i]) % K.mm.p[i]) << (8 * e);
                    }
                    w[i] = word;
                }
            }
            uint64_t s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0}, s2[4] = {0, 0, 0, 0},
                     s3[4] = {0, 0, 0, 0}, f[4] = {0, 0, 0, 0};
#pragma unroll
            for (int gi = 0; gi < (kMaxM + 2) / 3; ++gi) {
                if (gi >= K.n_groups) break;
                uint32_t c[4] = {0, 0, 0, 0};
#pragma unroll
                for (int j = 0; j < 3; ++j) {
                    const int i = 3 * gi + j;
                    if (i < kMaxM && i < K.n_mod) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) c[e] += ((w[i] >> (8 * e)) & 0xFFu) * K.coef[i];
                    }
                }
                const uint32_t m0 = K.Mg[gi][0], m1 = K.Mg[gi][1], m2 = K.Mg[gi][2],
                               m3 = K.Mg[gi][3], fl = K.fgl[gi], fh = K.fgh[gi];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    s0[e] += static_cast<uint64_t>(c[e]) * m0;
                    s1[e] += static_cast<uint64_t>(c[e]) * m1;
                    s2[e] += static_cast<uint64_t>(c[e]) * m2;
                    s3[e] += static_cast<uint64_t>(c[e]) * m3;
                    f[e] += static_cast<uint64_t>(c[e]) * fl + (static_cast<uint64_t>(c[e] * fh) << 32);
                }
            }
            double outv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int ce = e < nc ? col_exp[col + e] : 0;
                outv[e] = (re == kNonfiniteExp || ce == kNonfiniteExp)
                              ? nan_value()
                              : crt_finish<48>(s0[e], s1[e], s2[e], s3[e], f[e],
                                               re + ce - K.two_bits, K);
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
}

template <bool kInU8>
static cudaError_t launch_crt_t(const void *R, int64_t ldr, int64_t plane, int64_t rows,
                                int64_t cols, const int32_t *row_exp, const int32_t *col_exp,
                                double *C, int64_t ldc, int out_mode, const CrtConst &K,
                                int num_sms, cudaStream_t stream, int blocks_per_sm, int lower) {
    const int64_t groups = (cols + 3) >> 2;
    int64_t gx = (groups + 255) / 256;
    int64_t cap = int64_t(num_sms) * blocks_per_sm;
    if (gx > cap) gx = cap;
    int64_t gy = cap / gx;
    if (gy < 1) gy = 1;
    if (gy > rows) gy = rows;
    if (gy > 65535) gy = 65535;
    const dim3 g(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
    const bool small = K.n_mod <= 16;
#define TI_CRT_LAUNCH(MODE)                                                                      \
    if (small)                                                                                   \
        crt_kernel<kInU8, MODE, 16><<<g, 256, 0, stream>>>(R, ldr, plane, rows, cols, row_exp,  \
                                                           col_exp, C, ldc, lower, K);           \
    else                                                                                         \
        crt_kernel<kInU8, MODE, kMaxModuli><<<g, 256, 0, stream>>>(R, ldr, plane, rows, cols,   \
                                                                   row_exp, col_exp, C, ldc,    \
                                                                   lower, K);
    if (out_mode == 0) {
        TI_CRT_LAUNCH(0)
    } else if (out_mode == 1) {
        TI_CRT_LAUNCH(1)
    } else {
        TI_CRT_LAUNCH(2)
    }
#undef TI_CRT_LAUNCH
    return cudaGetLastError();
}

cudaError_t launch_crt(const void *R, bool in_u8, int64_t ldr, int64_t plane, int64_t rows,
                       int64_t cols, const int32_t *row_exp, const int32_t *col_exp, double *C,
                       int64_t ldc, int out_mode, const CrtConst &K, int num_sms,
                       cudaStream_t stream, int blocks_per_sm, bool lower) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    if (in_u8)
        return launch_crt_t<true>(R, ldr, plane, rows, cols, row_exp, col_exp, C, ldc, out_mode, K,
                                  num_sms, stream, blocks_per_sm, lower ? 1 : 0);
    return launch_crt_t<false>(R, ldr, plane, rows, cols, row_exp, col_exp, C, ldc, out_mode, K,
                               num_sms, stream, blocks_per_sm, lower ? 1 : 0);
}

}  // namespace ti
