// ti_split.cu -- K1: fused power-of-two scaling + int8 residue split of one operand.
//
// Restates src/tensor_inv/crt_matmul.py:32-46 (_scale_to_int, _residues) in exact integer
// arithmetic.  An operand is `outer` vectors of length `kdim` (rows of A or columns of B)
// with element (o, l) at X[o*s_outer + l*s_k].  Two passes:
//   1. exponent: e_o = frexp(max(max_l |x_ol|, 1e-300)).exponent (or kNonfiniteExp)
//   2. split:    v = round_half_even(x * 2^(bits - e_o)) computed from the float64 bits,
//                r_i = v mod p_i in [0, p_i) (the reference's floor mod; or, for the
//                opt-in wide moduli up to 255, the symmetric residue in
//                [-(p_i-1)/2, (p_i-1)/2]), written K-major as res[i][o][l] (int8).
// Two layouts of the source are handled without copies: k contiguous (s_k == 1, "rows")
// and outer contiguous (s_outer == 1, "cols", a transposed view), the latter through a
// shared-memory transpose.  Both write 8 consecutive residues per thread and modulus
// as one 8-byte store, so a warp writes whole 32-byte sectors.
#include <cstdlib>
#include <cstring>

#include "ti_scale.cuh"

namespace ti {

// Residue bytes of 8 signed values (magnitudes mag[j] < 2^53, signs neg[j]) mod p_i,
// packed little-endian into two 32-bit words: floor-mod residues in [0, p).
__device__ __forceinline__ uint2 residues8(const uint32_t (&a2)[8], const uint32_t (&a1)[8],
                                           const uint32_t (&a0)[8], uint32_t negmask,
                                           const SplitConst &C, int i) {
    const uint32_t p = C.mm.p[i], magic = C.mm.magic[i], shift = C.mm.shift[i];
    const uint32_t w32 = C.w32[i], w16 = C.w16[i], bigp = C.bigp[i], mult = C.mult[i];
    uint32_t out[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        // mag = a2*2^32 + a1*2^16 + a0  ==>  t == mult * mag (mod p), t < 2^30
        uint32_t t = a2[j] * w32 + a1[j] * w16 + a0[j] * mult;
        t = ((negmask >> j) & 1u) ? bigp - t : t;  // -mag (mod p), bigp - t < 2^31
        const uint32_t r = mod_small(t, p, magic, shift);
        out[j >> 2] |= r << (8 * (j & 3));
    }
    return make_uint2(out[0], out[1]);
}

// Symmetric residues of 8 signed values given as signed pieces (v = a2*2^32 + a1*2^16 + a0
// with every piece carrying the sign of v): T = a2*w32 + a1*w16 + a0*mult == mult*v (mod p)
// with |T| < 568197120; u = T + offs (a multiple of p above |T|, so 0 <= u < 2^31);
// q = floor((u + h) / p) exactly, and u - q*p is the residue in [-h, h], h = (p-1)/2.
__device__ __forceinline__ uint2 residues8_sym(const uint32_t (&a2)[8], const uint32_t (&a1)[8],
                                               const uint32_t (&a0)[8], const SplitConst &C,
                                               int i) {
    const uint32_t p = C.mm.p[i], magic = C.mm.magic[i], shift = C.mm.shift[i];
    const uint32_t w32 = C.w32[i], w16 = C.w16[i], offs = C.offs[i], h = p >> 1;
    const uint32_t mult = C.mult[i];
    uint32_t r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t u = a2[j] * w32 + a1[j] * w16 + (a0[j] * mult + offs);
        const uint32_t q = __umulhi(u + h, magic) >> shift;
        r[j] = u - q * p;  // low byte is the two's-complement residue
    }
    const uint32_t lo = __byte_perm(__byte_perm(r[0], r[1], 0x0040), __byte_perm(r[2], r[3], 0x0040),
                                    0x5410);
    const uint32_t hi = __byte_perm(__byte_perm(r[4], r[5], 0x0040), __byte_perm(r[6], r[7], 0x0040),
                                    0x5410);
    return make_uint2(lo, hi);
}

// Negate the pieces of negative values (two's complement), once per element.
__device__ __forceinline__ void sign_pieces(uint32_t (&a2)[8], uint32_t (&a1)[8],
                                            uint32_t (&a0)[8], uint32_t negmask) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if ((negmask >> j) & 1u) {
            a2[j] = 0u - a2[j];
            a1[j] = 0u - a1[j];
            a0[j] = 0u - a0[j];
        }
    }
}

__device__ __forceinline__ void decompose8(const double (&x)[8], int bits, int e,
                                           uint32_t (&a2)[8], uint32_t (&a1)[8],
                                           uint32_t (&a0)[8], uint32_t &negmask) {
    negmask = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        bool neg;
        const uint64_t mag = (e == kNonfiniteExp) ? 0ull : scaled_magnitude(x[j], bits, e, neg);
        if (e == kNonfiniteExp) neg = false;
        const uint32_t lo = static_cast<uint32_t>(mag);
        a2[j] = static_cast<uint32_t>(mag >> 32);
        a1[j] = lo >> 16;
        a0[j] = lo & 0xFFFFu;
        negmask |= (neg && mag != 0 ? 1u : 0u) << j;
    }
}

// ---------------------------------------------------------------------------------------
// pass 1: exponents
// ---------------------------------------------------------------------------------------

// k contiguous: one warp per vector.
__global__ void exp_rows_kernel(const double *__restrict__ X, int64_t outer, int64_t kdim,
                                int64_t s_outer, int32_t *__restrict__ exp_out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t o = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
         o < outer; o += warps) {
        const double *x = X + o * s_outer;
        uint64_t mb = 0;
        int64_t l = lane;
        for (; l + 96 < kdim; l += 128) {
            const uint64_t b0 = abs_bits(__ldg(x + l)), b1 = abs_bits(__ldg(x + l + 32));
            const uint64_t b2 = abs_bits(__ldg(x + l + 64)), b3 = abs_bits(__ldg(x + l + 96));
            mb = max(mb, max(max(b0, b1), max(b2, b3)));
        }
        for (; l < kdim; l += 32) mb = max(mb, abs_bits(__ldg(x + l)));
#pragma unroll
        for (int off = 16; off; off >>= 1) mb = max(mb, __shfl_xor_sync(0xFFFFFFFFu, mb, off));
        if (lane == 0) exp_out[o] = exp_from_maxbits(mb);
    }
}

// outer contiguous: a 32 x 32 thread block owns 32 vectors, threads stride over k.
__global__ void exp_cols_kernel(const double *__restrict__ X, int64_t outer, int64_t kdim,
                                int64_t s_k, int32_t *__restrict__ exp_out) {
    __shared__ uint64_t red[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int64_t o = static_cast<int64_t>(blockIdx.x) * 32 + tx;
    uint64_t mb = 0;
    if (o < outer) {
        int64_t l = ty;
        for (; l + 96 < kdim; l += 128) {
            const uint64_t b0 = abs_bits(__ldg(X + l * s_k + o));
            const uint64_t b1 = abs_bits(__ldg(X + (l + 32) * s_k + o));
            const uint64_t b2 = abs_bits(__ldg(X + (l + 64) * s_k + o));
            const uint64_t b3 = abs_bits(__ldg(X + (l + 96) * s_k + o));
            mb = max(mb, max(max(b0, b1), max(b2, b3)));
        }
        for (; l < kdim; l += 32) mb = max(mb, abs_bits(__ldg(X + l * s_k + o)));
    }
    red[ty][tx] = mb;
    __syncthreads();
    if (ty == 0) {
        for (int r = 1; r < 32; ++r) mb = max(mb, red[r][tx]);
        if (o < outer) exp_out[o] = exp_from_maxbits(mb);
    }
}

// Outer contiguous, long vectors: two passes.  Block (g, s) takes 64 consecutive vectors
// (each lane two neighbours, one 16-byte load per k) over the s-th of kExpColSplit slices
// of k, 8 warps striding the slice with 4 loads in flight each, and writes the slice's
// maximum bit patterns to part[s][o]; exp_cols_finish_kernel reduces the slices.  The
// one-pass kernel above gives only outer / 32 blocks of 1024 threads (256 at outer = 8192,
// fewer than two per SM) with 8-byte loads.
constexpr int kExpColSplit = 8;

__global__ void __launch_bounds__(256)
    exp_cols_partial_kernel(const double *__restrict__ X, int64_t outer, int64_t kdim,
                            int64_t s_k, uint64_t *__restrict__ part) {
    __shared__ uint64_t red[8][64];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t o = int64_t(blockIdx.x) * 64 + 2 * lane;
    const int64_t per = (kdim + kExpColSplit - 1) / kExpColSplit;
    const int64_t l0 = int64_t(blockIdx.y) * per;
    const int64_t l1 = l0 + per < kdim ? l0 + per : kdim;
    uint64_t m0 = 0, m1 = 0;
    if (o + 1 < outer) {
        int64_t l = l0 + warp;
        for (; l + 24 < l1; l += 32) {
            double2 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                v[u] = __ldg(reinterpret_cast<const double2 *>(X + (l + 8 * u) * s_k + o));
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                m0 = max(m0, abs_bits(v[u].x));
                m1 = max(m1, abs_bits(v[u].y));
            }
        }
        for (; l < l1; l += 8) {
            const double2 v = __ldg(reinterpret_cast<const double2 *>(X + l * s_k + o));
            m0 = max(m0, abs_bits(v.x));
            m1 = max(m1, abs_bits(v.y));
        }
    } else if (o < outer) {  // the last vector when outer is odd
        for (int64_t l = l0 + warp; l < l1; l += 8) m0 = max(m0, abs_bits(__ldg(X + l * s_k + o)));
    }
    red[warp][2 * lane] = m0;
    red[warp][2 * lane + 1] = m1;
    __syncthreads();
    if (threadIdx.x < 64) {
        uint64_t m = red[0][threadIdx.x];
#pragma unroll
        for (int w = 1; w < 8; ++w) m = max(m, red[w][threadIdx.x]);
        const int64_t oc = int64_t(blockIdx.x) * 64 + threadIdx.x;
        if (oc < outer) part[int64_t(blockIdx.y) * outer + oc] = m;
    }
}

__global__ void exp_cols_finish_kernel(const uint64_t *__restrict__ part, int64_t outer,
                                       int32_t *__restrict__ exp_out) {
    for (int64_t o = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; o < outer;
         o += int64_t(gridDim.x) * blockDim.x) {
        uint64_t m = part[o];
#pragma unroll
        for (int s = 1; s < kExpColSplit; ++s) m = max(m, part[int64_t(s) * outer + o]);
        exp_out[o] = exp_from_maxbits(m);
    }
}

// ---------------------------------------------------------------------------------------
// pass 2: scale + residues
// ---------------------------------------------------------------------------------------

// k contiguous.  Each thread owns 8 consecutive elements of one vector.
template <bool kSym>
__global__ void __launch_bounds__(256) split_rows_kernel(
    const double *__restrict__ X, int64_t outer, int64_t kdim, int64_t s_outer,
    const int32_t *__restrict__ exps, int8_t *__restrict__ res, int64_t ld_res,
    int64_t plane, const __grid_constant__ SplitConst C) {
    const int64_t chunks_per_vec = ld_res >> 3;
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(X) & 15) == 0) && ((s_outer & 1) == 0);
    // vectors by blockIdx.y, 8-element chunks of a vector by blockIdx.x (no division)
    for (int64_t o = blockIdx.y; o < outer; o += gridDim.y)
    for (int64_t ch = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
         ch < chunks_per_vec; ch += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t l0 = ch << 3;
        const double *x = X + o * s_outer + l0;
        double v[8];
        if (vec_ok && l0 + 8 <= kdim) {
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                const double2 t = __ldg(reinterpret_cast<const double2 *>(x + j));
                v[j] = t.x;
                v[j + 1] = t.y;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = (l0 + j < kdim) ? __ldg(x + j) : 0.0;
        }
        const int e = exps[o];
        uint32_t a2[8], a1[8], a0[8], negmask;
        decompose8(v, C.bits, e, a2, a1, a0, negmask);
        int8_t *dst = res + o * ld_res + l0;
        if (kSym) sign_pieces(a2, a1, a0, negmask);
        for (int i = 0; i < C.n_mod; ++i) {
            const uint2 w = kSym ? residues8_sym(a2, a1, a0, C, i)
                                 : residues8(a2, a1, a0, negmask, C, i);
            *reinterpret_cast<uint2 *>(dst + i * plane) = w;
        }
    }
}

// outer contiguous (a transposed view).  A block loads a 64 (k) x 32 (outer) tile with
// coalesced reads, transposes it through shared memory, and each thread then owns 8
// consecutive k of one vector.
constexpr int kColTileK = 64, kColTileO = 32, kColPad = 66;  // row pitch in doubles

template <bool kSym>
__global__ void __launch_bounds__(256) split_cols_kernel(
    const double *__restrict__ X, int64_t outer, int64_t kdim, int64_t s_k,
    const int32_t *__restrict__ exps, int8_t *__restrict__ res, int64_t ld_res,
    int64_t plane, const __grid_constant__ SplitConst C) {
    __shared__ __align__(16) double tile[kColTileO * kColPad];  // [o][k]
    const int tid = threadIdx.x;
    const int64_t tiles_o = (outer + kColTileO - 1) / kColTileO;
    const int64_t tiles_k = (ld_res + kColTileK - 1) / kColTileK;
    for (int64_t t = blockIdx.x; t < tiles_o * tiles_k; t += gridDim.x) {
        const int64_t to = t / tiles_k, tk = t - to * tiles_k;
        const int64_t o0 = to * kColTileO, l0 = tk * kColTileK;
        {   // coalesced load: warp w reads rows l0 + w + 8r, 32 consecutive outer indices
            const int tx = tid & 31, ty = tid >> 5;
            const int64_t o = o0 + tx;
#pragma unroll
            for (int r = 0; r < kColTileK / 8; ++r) {
                const int64_t l = l0 + ty + 8 * r;
                tile[tx * kColPad + ty + 8 * r] =
                    (o < outer && l < kdim) ? __ldg(X + l * s_k + o) : 0.0;
            }
        }
        __syncthreads();
        const int oo = tid >> 3, kc = tid & 7;
        const int64_t o = o0 + oo;
        const int64_t lc = l0 + kc * 8;
        if (o < outer && lc < ld_res) {
            double v[8];
            const double2 *src = reinterpret_cast<const double2 *>(tile + oo * kColPad + kc * 8);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const double2 d = src[j];
                v[2 * j] = d.x;
                v[2 * j + 1] = d.y;
            }
            const int e = exps[o];
            uint32_t a2[8], a1[8], a0[8], negmask;
            decompose8(v, C.bits, e, a2, a1, a0, negmask);
            int8_t *dst = res + o * ld_res + lc;
            if (kSym) sign_pieces(a2, a1, a0, negmask);
            for (int i = 0; i < C.n_mod; ++i) {
                const uint2 w = kSym ? residues8_sym(a2, a1, a0, C, i)
                                     : residues8(a2, a1, a0, negmask, C, i);
                *reinterpret_cast<uint2 *>(dst + i * plane) = w;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------------------
cudaError_t launch_split_tc(const double *X, int64_t outer, int64_t kdim, int64_t s_outer,
                            int64_t s_k, const SplitConst &C, const int32_t *exps, int8_t *res,
                            int64_t ld_res, int64_t plane, int *err, int num_sms,
                            cudaStream_t stream);

// Residues go to the tensor-core kernel (ti_split_tc.cu) when `err` (the device error word
// its bounded waits report to) is given and the layout suits its copies;
// TI_SPLIT=simt keeps them on the SIMT kernels below, which give the same bytes, and
// TI_SPLIT=tc reports an unsuitable layout as an error instead of falling back (tests).
static int split_mode() {  // 0 simt, 1 tensor cores with fallback, 2 tensor cores only
    const char *e = getenv("TI_SPLIT");
    if (e && !strcmp(e, "simt")) return 0;
    if (e && !strcmp(e, "tc")) return 2;
    return 1;
}

// plane: bytes between the residue planes of consecutive moduli (0: outer * ld_res, the
// operand's own planes; a row band of a larger operand passes the full operand's stride).
// exps_given: exp_out already holds the exponents (for example reduced over the inner
// dimension of several ranks), so they are read, not computed.
// blocks_per_sm caps the grid so the kernel can share SMs with a concurrent GEMM.
cudaError_t launch_split(const double *X, int64_t outer, int64_t kdim, int64_t s_outer,
                         int64_t s_k, const SplitConst &C, int32_t *exp_out, int8_t *res,
                         int64_t ld_res, int num_sms, cudaStream_t stream, int64_t plane,
                         int blocks_per_sm, int *err, bool exps_given) {
    if (outer == 0) return cudaSuccess;
    if (plane == 0) plane = outer * ld_res;
    const int64_t cap = int64_t(num_sms) * blocks_per_sm;
    const int mode = err ? split_mode() : 0;
    const bool try_tc = mode != 0;
    int tc_ctas = static_cast<int>(cap / 8);
    if (tc_ctas < 1) tc_ctas = 1;
    if (s_k == 1) {
        const int64_t warps_needed = outer;
        int64_t blocks = (warps_needed + 7) / 8;
        if (blocks > int64_t(num_sms) * 16) blocks = int64_t(num_sms) * 16;
        if (!exps_given)
            exp_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(X, outer, kdim,
                                                                               s_outer, exp_out);
        if (try_tc) {
            const cudaError_t e = launch_split_tc(X, outer, kdim, s_outer, 1, C, exp_out, res,
                                                  ld_res, plane, err, tc_ctas, stream);
            if (e != cudaErrorNotSupported || mode == 2) return e;
        }
        const int64_t chunks = ld_res >> 3;
        int64_t gx = (chunks + 255) / 256;
        if (gx > cap) gx = cap;
        int64_t gy = cap / gx;
        if (gy > outer) gy = outer;
        if (gy > 65535) gy = 65535;
        if (gy < 1) gy = 1;
        const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
        if (C.symmetric)
            split_rows_kernel<true><<<grid, 256, 0, stream>>>(X, outer, kdim, s_outer, exp_out,
                                                              res, ld_res, plane, C);
        else
            split_rows_kernel<false><<<grid, 256, 0, stream>>>(X, outer, kdim, s_outer, exp_out,
                                                               res, ld_res, plane, C);
    } else {
        const int64_t blocks = (outer + 31) / 32;
        // two passes for long vectors, their partial maxima parked in the first residue plane
        // (kExpColSplit * outer * 8 bytes <= outer * ld_res; the split overwrites it next)
        const bool two_pass = kdim >= 1024 && ld_res >= 8 * kExpColSplit &&
                              (reinterpret_cast<uintptr_t>(X) & 15) == 0 && (s_k & 1) == 0 &&
                              (reinterpret_cast<uintptr_t>(res) & 7) == 0 &&
                              (outer + 63) / 64 <= 65535 * 1024;
        if (!exps_given && two_pass) {
            uint64_t *part = reinterpret_cast<uint64_t *>(res);
            exp_cols_partial_kernel<<<dim3(static_cast<unsigned>((outer + 63) / 64), kExpColSplit),
                                      256, 0, stream>>>(X, outer, kdim, s_k, part);
            int64_t fb = (outer + 255) / 256;
            if (fb > int64_t(num_sms) * 8) fb = int64_t(num_sms) * 8;
            exp_cols_finish_kernel<<<static_cast<unsigned>(fb), 256, 0, stream>>>(part, outer,
                                                                                 exp_out);
        } else if (!exps_given) {
            exp_cols_kernel<<<static_cast<unsigned>(blocks), 1024, 0, stream>>>(X, outer, kdim,
                                                                                s_k, exp_out);
        }
        if (try_tc) {
            const cudaError_t e = launch_split_tc(X, outer, kdim, 1, s_k, C, exp_out, res,
                                                  ld_res, plane, err, tc_ctas, stream);
            if (e != cudaErrorNotSupported || mode == 2) return e;
        }
        const int64_t tiles = ((outer + kColTileO - 1) / kColTileO) *
                              ((ld_res + kColTileK - 1) / kColTileK);
        int64_t sblocks = tiles;
        if (sblocks > cap) sblocks = cap;
        if (C.symmetric)
            split_cols_kernel<true><<<static_cast<unsigned>(sblocks), 256, 0, stream>>>(
                X, outer, kdim, s_k, exp_out, res, ld_res, plane, C);
        else
            split_cols_kernel<false><<<static_cast<unsigned>(sblocks), 256, 0, stream>>>(
                X, outer, kdim, s_k, exp_out, res, ld_res, plane, C);
    }
    return cudaGetLastError();
}

}  // namespace ti
