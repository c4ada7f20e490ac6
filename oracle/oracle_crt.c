/*
 * oracle_crt.c -- CPU restatement of tensor_inv's CRT-emulated matmul.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path in
 * tensor_inv_b200: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference leg may load it.  The product never calls it.
 *
 * Every function restates one step of the reference algorithm with plain
 * exact CPU arithmetic (multi-word integers, libm frexp/ldexp/nearbyint):
 *
 *   or_n_moduli          src/tensor_inv/crt_matmul.py:20-29   (_n_moduli)
 *   or_split             src/tensor_inv/crt_matmul.py:32-46   (_scale_to_int + _residues)
 *   or_residue_gemm      src/tensor_inv/crt_matmul.py:49-59   (_matmul_residues, CPU branch)
 *   or_crt_reconstruct   src/tensor_inv/crt_matmul.py:62-92   (_crt_precompute + _crt_reconstruct)
 *   or_crt_matmul        src/tensor_inv/crt_matmul.py:95-120 (crt_matmul, CPU branch)
 *   or_crt_matmul_moduli the same path with a caller-chosen moduli set and precision
 *                        (the opt-in wide-moduli scheme; the steps are unchanged)
 *
 * Parity is pinned against fixtures produced by the reference itself
 * (tests/golden/make_golden.py) and checked in tests/test_oracle_golden.py.
 *
 * Divergences (documented, deliberate):
 *   - Python's math.ldexp raises OverflowError when the result overflows;
 *     C ldexp returns +-inf, which is what this oracle returns.
 *   - Non-finite inputs: the reference casts NaN/inf to int64 (undefined
 *     behaviour in C++).  The oracle defines the output row (for A) or column
 *     (for B) that holds a non-finite value as NaN; or_split flags it with
 *     exponent OR_NONFINITE_EXP.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_NONFINITE_EXP (-2147483647 - 1)
#define OR_MAX_MODULI 30
#define BN_WORDS 8 /* 256-bit unsigned integers: every quantity here is < 2^200 */

static const int OR_PRIMES[OR_MAX_MODULI] = {3,  5,  7,  11, 13, 17, 19, 23, 29,  31,
                                             37, 41, 43, 47, 53, 59, 61, 67, 71,  73,
                                             79, 83, 89, 97, 101, 103, 107, 109, 113, 127};

/* ------------------------------------------------------------------------ */
/* tiny fixed-width unsigned bigint, little-endian 32-bit words              */
/* ------------------------------------------------------------------------ */
typedef struct {
    uint32_t w[BN_WORDS];
} bn_t;

static void bn_zero(bn_t *a) { memset(a, 0, sizeof(*a)); }

static void bn_set_u64(bn_t *a, uint64_t v) {
    bn_zero(a);
    a->w[0] = (uint32_t)v;
    a->w[1] = (uint32_t)(v >> 32);
}

static void bn_mul_small(bn_t *a, uint32_t m) {
    uint64_t carry = 0;
    for (int i = 0; i < BN_WORDS; ++i) {
        uint64_t t = (uint64_t)a->w[i] * m + carry;
        a->w[i] = (uint32_t)t;
        carry = t >> 32;
    }
}

static void bn_add(bn_t *a, const bn_t *b) {
    uint64_t carry = 0;
    for (int i = 0; i < BN_WORDS; ++i) {
        uint64_t t = (uint64_t)a->w[i] + b->w[i] + carry;
        a->w[i] = (uint32_t)t;
        carry = t >> 32;
    }
}

/* a -= b, requires a >= b */
static void bn_sub(bn_t *a, const bn_t *b) {
    int64_t borrow = 0;
    for (int i = 0; i < BN_WORDS; ++i) {
        int64_t t = (int64_t)a->w[i] - b->w[i] - borrow;
        borrow = t < 0;
        a->w[i] = (uint32_t)(t + (borrow ? ((int64_t)1 << 32) : 0));
    }
}

static int bn_cmp(const bn_t *a, const bn_t *b) {
    for (int i = BN_WORDS - 1; i >= 0; --i) {
        if (a->w[i] != b->w[i]) return a->w[i] > b->w[i] ? 1 : -1;
    }
    return 0;
}

static int bn_bitlen(const bn_t *a) {
    for (int i = BN_WORDS - 1; i >= 0; --i)
        if (a->w[i]) return 32 * i + 32 - __builtin_clz(a->w[i]);
    return 0;
}

static void bn_shl(bn_t *r, const bn_t *a, int s) {
    bn_t t;
    bn_zero(&t);
    int ws = s / 32, bs = s % 32;
    for (int i = BN_WORDS - 1; i >= ws; --i) {
        uint64_t v = (uint64_t)a->w[i - ws] << bs;
        if (bs && i - ws - 1 >= 0) v |= (uint64_t)a->w[i - ws - 1] >> (32 - bs);
        t.w[i] = (uint32_t)v;
    }
    *r = t;
}

static void bn_shr1(bn_t *a) {
    for (int i = 0; i < BN_WORDS; ++i) {
        uint32_t hi = (i + 1 < BN_WORDS) ? a->w[i + 1] : 0;
        a->w[i] = (a->w[i] >> 1) | (hi << 31);
    }
}

/* a = a mod m (shift-and-subtract long division) */
static void bn_mod(bn_t *a, const bn_t *m) {
    int la = bn_bitlen(a), lm = bn_bitlen(m);
    if (la < lm) return;
    bn_t sh;
    bn_shl(&sh, m, la - lm);
    for (int s = la - lm; s >= 0; --s) {
        if (bn_cmp(a, &sh) >= 0) bn_sub(a, &sh);
        bn_shr1(&sh);
    }
}

static uint32_t bn_mod_small(const bn_t *a, uint32_t m) {
    uint64_t r = 0;
    for (int i = BN_WORDS - 1; i >= 0; --i) r = ((r << 32) | a->w[i]) % m;
    return (uint32_t)r;
}

/* correctly rounded (round-half-even) conversion of a non-negative bigint to
   double: the top 64 bits with every lower bit ORed into bit 0 round exactly
   like the full value (the sticky bit sits below the rounding position). */
static double bn_to_double(const bn_t *a) {
    int L = bn_bitlen(a);
    if (L <= 64) {
        uint64_t v = (uint64_t)a->w[0] | ((uint64_t)a->w[1] << 32);
        return (double)v;
    }
    int sh = L - 64;
    uint64_t top = 0;
    for (int b = 0; b < 64; ++b) {
        int bit = sh + b;
        if ((a->w[bit / 32] >> (bit % 32)) & 1u) top |= (uint64_t)1 << b;
    }
    int sticky = 0;
    for (int bit = 0; bit < sh && !sticky; ++bit)
        if ((a->w[bit / 32] >> (bit % 32)) & 1u) sticky = 1;
    top |= (uint64_t)sticky;
    return ldexp((double)top, sh);
}

/* ------------------------------------------------------------------------ */
/* crt_matmul.py:20-29  _n_moduli(k, bits)                                   */
/* smallest N with prod(first N primes) > 2*k*2^(2*bits); -1 if none         */
/* ------------------------------------------------------------------------ */
/* Threads of the oracle's parallel loops (OpenMP); overrides OMP_NUM_THREADS. */
void or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int or_n_moduli(int64_t k, int bits) {
    if (k < 0 || bits < 0 || 2 * bits + 1 + 64 > 32 * BN_WORDS - 8) return -1;
    bn_t target, prod;
    bn_set_u64(&target, (uint64_t)k);
    bn_shl(&target, &target, 2 * bits + 1);
    bn_set_u64(&prod, 1);
    for (int i = 0; i < OR_MAX_MODULI; ++i) {
        bn_mul_small(&prod, (uint32_t)OR_PRIMES[i]);
        if (bn_cmp(&prod, &target) > 0) return i + 1;
    }
    return -1;
}

const int *or_primes(void) { return OR_PRIMES; }

/* ------------------------------------------------------------------------ */
/* crt_matmul.py:32-46  _scale_to_int + _residues for ONE operand.           */
/* The operand is viewed as `outer` vectors of length `kdim` (rows of A, or  */
/* columns of B); element (o, l) lives at X[o*s_outer + l*s_k].              */
/*   exp_out[o]            = frexp(max(max_l |x|, 1e-300)).exponent          */
/*   v                     = nearbyint(ldexp(x, bits - exp_out[o]))          */
/*   res_out[i][o][l]      = v mod moduli[i]   (floor mod, in [0, p))        */
/* ------------------------------------------------------------------------ */
void or_split(const double *X, int64_t outer, int64_t kdim, int64_t s_outer, int64_t s_k,
              int bits, int n_mod, const int32_t *moduli, int32_t *exp_out, int8_t *res_out) {
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < outer; ++o) {
        const double *x = X + o * s_outer;
        double mx = 0.0;
        int nonfinite = 0;
        for (int64_t l = 0; l < kdim; ++l) {
            double a = fabs(x[l * s_k]);
            if (!isfinite(a)) nonfinite = 1;
            if (a > mx) mx = a;
        }
        int e;
        if (nonfinite) {
            exp_out[o] = OR_NONFINITE_EXP;
        } else {
            if (mx < 1e-300) mx = 1e-300; /* .clamp(min=1e-300) */
            (void)frexp(mx, &e);
            exp_out[o] = e;
        }
        for (int64_t l = 0; l < kdim; ++l) {
            int64_t v = 0;
            if (!nonfinite) v = (int64_t)nearbyint(ldexp(x[l * s_k], bits - exp_out[o]));
            for (int i = 0; i < n_mod; ++i) {
                int64_t p = moduli[i];
                int64_t r = v % p;
                if (r < 0) r += p;
                res_out[((int64_t)i * outer + o) * kdim + l] = (int8_t)r;
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* crt_matmul.py:49-59  _matmul_residues (CPU branch):                       */
/*   c[i] = (a_res[i].int() @ b_res[i].int()) % moduli[i]                    */
/* a_res: [n_mod][m][k], b_res: [n_mod][k][n] (the reference layout),       */
/* c: [n_mod][m][n] int32.  Accumulation is int32, as in torch's int matmul; */
/* callers keep 127*127*k below 2^31.                                         */
/* ------------------------------------------------------------------------ */
__attribute__((target_clones("avx512f", "avx2", "default"))) void
or_residue_gemm(const int8_t *a_res, const int8_t *b_res, int n_mod, const int32_t *moduli,
                int64_t m, int64_t n, int64_t k, int32_t *c) {
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int i = 0; i < n_mod; ++i) {
        for (int64_t r = 0; r < m; ++r) {
            const int8_t *a = a_res + ((int64_t)i * m + r) * k;
            const int8_t *b = b_res + (int64_t)i * k * n;
            int32_t *acc = c + ((int64_t)i * m + r) * n;
            for (int64_t j = 0; j < n; ++j) acc[j] = 0;
            for (int64_t l = 0; l < k; ++l) {
                int32_t av = a[l];
                const int8_t *brow = b + l * n;
                for (int64_t j = 0; j < n; ++j) acc[j] += av * (int32_t)brow[j];
            }
            int32_t p = moduli[i];
            for (int64_t j = 0; j < n; ++j) {
                int32_t v = acc[j] % p;
                acc[j] = v < 0 ? v + p : v;
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* crt_matmul.py:62-92  _crt_precompute + _crt_reconstruct                  */
/*   x = sum_i r_i * M_i * (M_i^-1 mod m_i)  mod M;  x > M//2 -> x - M        */
/*   out = ldexp(float(x), row_exp + col_exp - 2*bits)                        */
/* residues: [n_mod][rows][cols] int32; out: rows x cols, leading dim ldo.   */
/* Returns 0, or -1 for bad moduli.                                           */
/* ------------------------------------------------------------------------ */
int or_crt_reconstruct(const int32_t *residues, int n_mod, const int32_t *moduli, int bits,
                       const int32_t *row_exp, const int32_t *col_exp, int64_t rows, int64_t cols,
                       double *out, int64_t ldo) {
    if (n_mod < 1 || n_mod > OR_MAX_MODULI) return -1;
    bn_t M, half, W[OR_MAX_MODULI];
    bn_set_u64(&M, 1);
    for (int i = 0; i < n_mod; ++i) {
        if (moduli[i] < 2) return -1;
        bn_mul_small(&M, (uint32_t)moduli[i]);
    }
    for (int i = 0; i < n_mod; ++i) {
        /* M_i = M / m_i, built as the product of the other moduli */
        bn_t Mi;
        bn_set_u64(&Mi, 1);
        for (int j = 0; j < n_mod; ++j)
            if (j != i) bn_mul_small(&Mi, (uint32_t)moduli[j]);
        uint32_t mi = (uint32_t)moduli[i];
        uint32_t red = bn_mod_small(&Mi, mi), inv = 0;
        for (uint32_t t = 1; t < mi; ++t)
            if ((uint64_t)red * t % mi == 1) {
                inv = t;
                break;
            }
        if (!inv) return -1; /* moduli not pairwise coprime */
        W[i] = Mi;
        bn_mul_small(&W[i], inv);
    }
    half = M;
    bn_shr1(&half); /* M // 2 */

#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t c = 0; c < cols; ++c) {
            double val;
            if (row_exp[r] == OR_NONFINITE_EXP || col_exp[c] == OR_NONFINITE_EXP) {
                val = NAN;
            } else {
                bn_t x, t;
                bn_zero(&x);
                for (int i = 0; i < n_mod; ++i) {
                    int64_t ri = residues[((int64_t)i * rows + r) * cols + c];
                    int64_t p = moduli[i];
                    ri %= p; /* Python's % on the bigint sum makes this a no-op */
                    if (ri < 0) ri += p;
                    t = W[i];
                    bn_mul_small(&t, (uint32_t)ri);
                    bn_add(&x, &t);
                }
                bn_mod(&x, &M);
                int neg = 0;
                if (bn_cmp(&x, &half) > 0) { /* x > M//2 -> x - M, i.e. -(M - x) */
                    bn_t y = M;
                    bn_sub(&y, &x);
                    x = y;
                    neg = 1;
                }
                double d = bn_to_double(&x);
                if (neg) d = -d;
                val = ldexp(d, row_exp[r] + col_exp[c] - 2 * bits);
            }
            out[r * ldo + c] = val;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* crt_matmul.py:95-120 with an explicit moduli set and precision: the     */
/* same four steps (scale + residues, per-modulus int32 GEMM mod m_i,       */
/* bigint CRT, ldexp) for any pairwise-coprime moduli < 256.  bits is used  */
/* exactly as the reference uses _PRECISION_BITS[dtype].                    */
/* Returns 0, -2 on allocation failure, -1 for bad moduli.                  */
/* ------------------------------------------------------------------------ */
int or_crt_matmul_moduli(const double *A, int64_t sa0, int64_t sa1, const double *B,
                         int64_t sb0, int64_t sb1, int64_t m, int64_t n, int64_t k,
                         const int32_t *moduli, int n_mod, int bits, double *C, int64_t ldc) {
    if (n_mod < 1 || n_mod > OR_MAX_MODULI) return -1;
    size_t na = (size_t)n_mod * (size_t)m * (size_t)k, nb = (size_t)n_mod * (size_t)k * (size_t)n;
    int8_t *ar = (int8_t *)malloc(na ? na : 1);
    int8_t *br_t = (int8_t *)malloc(nb ? nb : 1);
    int8_t *br = (int8_t *)malloc(nb ? nb : 1);
    int32_t *re = (int32_t *)malloc(sizeof(int32_t) * (m ? m : 1));
    int32_t *ce = (int32_t *)malloc(sizeof(int32_t) * (n ? n : 1));
    int32_t *cr = (int32_t *)malloc(sizeof(int32_t) * (size_t)n_mod * (size_t)m * (size_t)n + 4);
    int rc = 0;
    if (!ar || !br_t || !br || !re || !ce || !cr) {
        rc = -2;
        goto done;
    }
    /* residues are stored as int8 of the floor-mod value; moduli above 128 keep the same
       bits in a uint8 view, so the GEMM below reads them back as unsigned */
    or_split(A, m, k, sa0, sa1, bits, n_mod, moduli, re, ar);
    or_split(B, n, k, sb1, sb0, bits, n_mod, moduli, ce, br_t);
    for (int i = 0; i < n_mod; ++i)
        for (int64_t j = 0; j < n; ++j)
            for (int64_t l = 0; l < k; ++l)
                br[((int64_t)i * k + l) * n + j] = br_t[((int64_t)i * n + j) * k + l];
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int i = 0; i < n_mod; ++i) {
        for (int64_t r = 0; r < m; ++r) {
            const uint8_t *a = (const uint8_t *)ar + ((int64_t)i * m + r) * k;
            const uint8_t *b = (const uint8_t *)br + (int64_t)i * k * n;
            int32_t *acc = cr + ((int64_t)i * m + r) * n;
            for (int64_t j = 0; j < n; ++j) acc[j] = 0;
            for (int64_t l = 0; l < k; ++l) {
                int32_t av = a[l];
                const uint8_t *brow = b + l * n;
                /* partial sums stay exact: reduce every 16384 steps (255*255*16384 < 2^31) */
                for (int64_t j = 0; j < n; ++j) acc[j] += av * (int32_t)brow[j];
                if ((l & 16383) == 16383)
                    for (int64_t j = 0; j < n; ++j) acc[j] %= moduli[i];
            }
            for (int64_t j = 0; j < n; ++j) acc[j] %= moduli[i];
        }
    }
    rc = or_crt_reconstruct(cr, n_mod, moduli, bits, re, ce, m, n, C, ldc);
done:
    free(ar), free(br_t), free(br), free(re), free(ce), free(cr);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* crt_matmul.py:95-120  crt_matmul, CPU branch, for float64 operands.     */
/* A element (i,l) at A[i*sa0 + l*sa1]; B element (l,j) at B[l*sb0 + j*sb1]. */
/* bits: 53 fp64, 24 fp32, 11 fp16, 8 bf16 (_PRECISION_BITS).                */
/* Returns 0, -1 when no modulus count covers k, -2 on allocation failure.   */
/* ------------------------------------------------------------------------ */
int or_crt_matmul(const double *A, int64_t sa0, int64_t sa1, const double *B, int64_t sb0,
                  int64_t sb1, int64_t m, int64_t n, int64_t k, int bits, double *C, int64_t ldc) {
    int n_mod = or_n_moduli(k, bits);
    if (n_mod < 0) return -1;
    int32_t moduli[OR_MAX_MODULI];
    for (int i = 0; i < n_mod; ++i) moduli[i] = OR_PRIMES[i];
    size_t na = (size_t)n_mod * (size_t)m * (size_t)k, nb = (size_t)n_mod * (size_t)k * (size_t)n;
    int8_t *ar = (int8_t *)malloc(na ? na : 1);
    int8_t *br_t = (int8_t *)malloc(nb ? nb : 1); /* [n_mod][n][k]: columns of B */
    int8_t *br = (int8_t *)malloc(nb ? nb : 1);   /* [n_mod][k][n]: reference layout */
    int32_t *re = (int32_t *)malloc(sizeof(int32_t) * (m ? m : 1));
    int32_t *ce = (int32_t *)malloc(sizeof(int32_t) * (n ? n : 1));
    int32_t *cr = (int32_t *)malloc(sizeof(int32_t) * (size_t)n_mod * (size_t)m * (size_t)n + 4);
    if (!ar || !br_t || !br || !re || !ce || !cr) {
        free(ar), free(br_t), free(br), free(re), free(ce), free(cr);
        return -2;
    }
    or_split(A, m, k, sa0, sa1, bits, n_mod, moduli, re, ar);
    or_split(B, n, k, sb1, sb0, bits, n_mod, moduli, ce, br_t);
    for (int i = 0; i < n_mod; ++i)
        for (int64_t j = 0; j < n; ++j)
            for (int64_t l = 0; l < k; ++l)
                br[((int64_t)i * k + l) * n + j] = br_t[((int64_t)i * n + j) * k + l];
    or_residue_gemm(ar, br, n_mod, moduli, m, n, k, cr);
    int rc = or_crt_reconstruct(cr, n_mod, moduli, bits, re, ce, m, n, C, ldc);
    free(ar), free(br_t), free(br), free(re), free(ce), free(cr);
    return rc;
}
