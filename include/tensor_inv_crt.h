/*
 * tensor_inv_crt.h -- C ABI of libtensor_inv_crt.so, the B200 (sm_100a) implementation
 * of tensor_inv's CRT-emulated float64 matmul ("Ozaki scheme II" with the first N odd
 * primes as moduli).
 *
 * Conventions
 *   - Every pointer marked "device" is CUDA device memory on the current device.
 *   - Every call is asynchronous on `stream` (a cudaStream_t passed as void*; NULL is the
 *     legacy default stream) and returns a ti_status_t.  Nothing allocates device memory:
 *     calls that need scratch space take a caller-owned workspace.
 *   - Matrices are described by element strides: element (i, j) of an m x n matrix X
 *     lives at X[i*s0 + j*s1].  One of the two strides must be 1.
 *   - bits is the number of significand bits kept per input element (the reference's
 *     _PRECISION_BITS: 53 float64, 24 float32, 11 float16, 8 bfloat16).
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   ti_n_moduli               src/tensor_inv/crt_matmul.py:20      _n_moduli(k, bits)
 *   ti_crt_split              src/tensor_inv/crt_matmul.py:32,41   _scale_to_int + _residues
 *   ti_batched_int8_gemm_mod  src/tensor_inv/csrc/crt_kernel.cu:17 batched_int8_gemm_mod
 *   ti_crt_reconstruct        src/tensor_inv/csrc/crt_kernel.cu:127 crt_reconstruct
 *   ti_crt_matmul             src/tensor_inv/crt_matmul.py:95     crt_matmul (CUDA branch)
 */
#ifndef TENSOR_INV_CRT_H
#define TENSOR_INV_CRT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    TI_OK = 0,
    TI_ERR_INVALID_ARGUMENT = 1, /* bad shape, stride, dtype bits or null pointer */
    TI_ERR_UNSUPPORTED = 2,      /* k beyond the int32 accumulator bound or the moduli set */
    TI_ERR_WORKSPACE = 3,        /* workspace too small or misaligned */
    TI_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed */
    TI_ERR_DEVICE_TIMEOUT = 5,   /* a kernel gave up on a bounded wait (see ti_device_error) */
    TI_ERR_NO_DEVICE = 6,        /* no sm_100 device, or the driver entry point is missing */
    TI_ERR_SCRATCH_LIMIT = 7     /* problem needs more than ti_crt_matmul_noalloc's scratch */
} ti_status_t;

/* Row/column exponent value that marks a row of A (or column of B) holding a NaN or an
   infinity; the matching output row (column) is NaN. */
#define TI_NONFINITE_EXP (-2147483647 - 1)

/* Largest inner dimension: 126*126*k must stay below 2^31 in the int32 accumulators. */
#define TI_MAX_K 135263

/* Human-readable name of a status code (static string). */
const char *ti_status_string(int status);

/* Library version, e.g. "0.1.0". */
const char *ti_version(void);

/* Replaces crt_matmul.py:20 _n_moduli: smallest N with prod(first N odd primes) >
   2*k*2^(2*bits).  Writes N to *n_out; TI_ERR_UNSUPPORTED if no N <= 30 works. */
int ti_n_moduli(int64_t k, int bits, int *n_out);

/* The 30 moduli (3, 5, 7, ..., 127), in order. */
const int32_t *ti_primes(void);

/* Workspace bytes ti_crt_matmul needs for an m x k by k x n product at `bits`. */
int ti_crt_workspace_size(int64_t m, int64_t n, int64_t k, int bits, size_t *bytes);

/*
 * Replaces crt_matmul.py:32 _scale_to_int + crt_matmul.py:41 _residues for one operand.
 * The operand is `outer` vectors of length `kdim` (rows of A, or columns of B); element
 * (o, l) is X[o*s_outer + l*s_k] (device, float64).
 *   exp_out[o]   (device int32[outer]) = frexp(max(max_l |x|, 1e-300)).exponent,
 *                or TI_NONFINITE_EXP
 *   res_out      (device int8, [n_mod][outer][ld_res]) = nearbyint(x * 2^(bits-exp)) mod p_i,
 *                in [0, p_i); columns kdim..ld_res-1 are written as 0.
 * ld_res must be a multiple of 16 and >= kdim; res_out must be 16-byte aligned.
 */
int ti_crt_split(const double *X, int64_t outer, int64_t kdim, int64_t s_outer, int64_t s_k,
                 int bits, int n_mod, int32_t *exp_out, int8_t *res_out, int64_t ld_res,
                 void *stream);

/*
 * Replaces crt_kernel.cu:17 batched_int8_gemm_mod (cuBLASLt int8 GEMM + mod_reduce):
 *   c[i] = (a[i] @ b[i]) mod moduli[i], with the result in [0, moduli[i]).
 * a: device int8 (batch, M, K) row-major; b: device int8 (batch, K, N) row-major;
 * c: device int32 (batch, M, N) row-major; moduli: HOST int32[batch], each in [2, 256).
 * Unlike the reference, M, K and N need no padding.  Runs on tcgen05 tensor cores.
 * workspace: device scratch of ti_batched_gemm_workspace_size() bytes, 256-byte aligned.
 */
int ti_batched_gemm_workspace_size(int64_t batch, int64_t M, int64_t K, int64_t N,
                                   size_t *bytes);
int ti_batched_int8_gemm_mod(const int8_t *a, const int8_t *b, const int32_t *moduli,
                             int64_t batch, int64_t M, int64_t K, int64_t N, int32_t *c,
                             void *workspace, size_t workspace_bytes, void *stream);

/*
 * Replaces crt_kernel.cu:127 crt_reconstruct.  Exact integer CRT (not the reference GPU
 * kernel's double-double approximation): x = sum_i r_i M_i (M_i^-1 mod p_i) mod M, lifted
 * to (-M/2, M/2], then out = ldexp((double)x, row_exp[r] + col_exp[c] - 2*bits) with the
 * rounding of Python's float(int) followed by math.ldexp.  Bit-identical to the
 * reference's CPU path (crt_matmul.py:73-92).
 * residues: device int32 (n_mod, rows, cols); moduli: HOST int32[n_mod], pairwise coprime,
 * each in [2, 256), product below 2^127; row_exp/col_exp: device int32; out: device
 * float64 rows x cols with leading dimension ldo.
 */
int ti_crt_reconstruct(const int32_t *residues, const int32_t *moduli, int n_mod, int bits,
                       const int32_t *row_exp, const int32_t *col_exp, int64_t rows,
                       int64_t cols, double *out, int64_t ldo, void *stream);

/*
 * One rank's share of a product whose inner dimension is split across ranks, C = sum_r A_r B_r
 * (the contractions over the row-sharded dimension of a distributed rSVD, A^T Q and Q^T A).
 * With the exponents of the whole product given (row_exp: frexp exponents of max |A[i, :]|
 * over every rank's columns, col_exp likewise for B's columns; TI_NONFINITE_EXP for a
 * non-finite row/column), writes this rank's residue products (A_r B_r) mod p_i as int32 planes
 * out[i][m][n] in [0, p_i), for the first n_mod primes (n_mod = ti_n_moduli of the WHOLE inner
 * dimension).  The element-wise sum of all ranks' planes (an int32 all-reduce; below
 * ranks * 127) passed to ti_crt_reconstruct with the same exponents and moduli gives the
 * crt_matmul of the whole product bit for bit.  A: m x k (this rank's k), B: k x n, strides
 * in elements with one of each pair 1.  No counterpart in the reference, which runs on one
 * device; it splits crt_matmul.py:95-120 at _matmul_residues.
 * workspace: ti_crt_residue_partial_workspace_size() bytes, 256-byte aligned.
 */
int ti_crt_residue_partial_workspace_size(int64_t m, int64_t n, int64_t k, int n_mod,
                                          size_t *bytes);
int ti_crt_residue_partial(const double *A, int64_t sa0, int64_t sa1, const double *B,
                           int64_t sb0, int64_t sb1, int64_t m, int64_t n, int64_t k, int bits,
                           int n_mod, const int32_t *row_exp, const int32_t *col_exp,
                           int32_t *out, void *workspace, size_t workspace_bytes, void *stream);

/* Moduli sets.  TI_MODULI_PRIMES is the reference's (the first N odd primes, 3..127,
   N from _n_moduli).  TI_MODULI_WIDE is an opt-in extension:
   pairwise-coprime odd moduli up to 255 (255, 253, 251, 247, 241, 239, 233, 229, 227, 223,
   217, 211, 199, 197, 193, 191), at most 16.  With the automatic count, WIDE keeps every
   bit of the input precision, so its outputs are bit-identical to PRIMES with about a
   third fewer residue GEMMs (16 instead of 25 at k = 8192). */
#define TI_MODULI_PRIMES 0
#define TI_MODULI_WIDE 1

/* Options of the *_ex entry points.  A NULL options pointer means all defaults. */
typedef struct ti_crt_options {
    int moduli;             /* TI_MODULI_PRIMES (default) or TI_MODULI_WIDE */
    int n_moduli;           /* 0: automatic (PRIMES: the reference's _n_moduli; WIDE: the
                               fewest moduli that keep `bits`).  Otherwise exactly this many
                               (PRIMES <= 25, WIDE <= 16); when they cannot hold 2*k*2^(2*bits)
                               the precision is lowered to the largest b with
                               prod(moduli) > 2*k*2^(2*b) (a moduli-count sweep) */
    void *stage_events[4];  /* optional cudaEvent_t, recorded before K1, before the first K2,
                               after the last K2 (before the last K3) and at the end; NULL
                               entries are skipped */
    int bands;              /* 0 or 1: one band, all stages in order on `stream`.  n > 1 splits
                               A into n row bands pipelined over two internal streams: the GEMM
                               of band b overlaps the split of band b+1 and the reconstruction
                               of band b-1 (opt-in: on B200 the shared SMs slow the GEMM more
                               than the overlap saves) */
    int lower;              /* 0: every element of C.  1: only elements C[r][c] with r >= c are
                               guaranteed (a symmetric update such as Cholesky's
                               W -= L21 L21^T, which reads only the lower triangle): output tiles
                               entirely above the diagonal are skipped by the residue GEMM and
                               the reconstruction, and those elements may or may not be written.
                               Honoured by the single-band device path; otherwise ignored (every
                               element is computed) */
} ti_crt_options_t;

/* The moduli count, the precision actually kept, and (if moduli_out != NULL, room for 32)
   the moduli that ti_crt_matmul_ex will use for inner dimension k at `bits`. */
int ti_crt_plan(int64_t k, int bits, const ti_crt_options_t *opt, int *n_mod_out,
                int *bits_eff_out, int32_t *moduli_out);

/* Workspace bytes of ti_crt_matmul_ex with these options. */
int ti_crt_workspace_size_ex(int64_t m, int64_t n, int64_t k, int bits,
                             const ti_crt_options_t *opt, size_t *bytes);

/* Output modes of ti_crt_matmul. */
#define TI_OUT_STORE 0    /* C  = A @ B  */
#define TI_OUT_SUBTRACT 1 /* C -= A @ B  (C - round(A@B), as `W -= crt_matmul(...)`) */
#define TI_OUT_ADD 2      /* C += A @ B  */

/*
 * Replaces crt_matmul.py:95 crt_matmul for float64 operands on the device:
 *   A (m x k): element (i, l) at A[i*sa0 + l*sa1];  B (k x n): (l, j) at B[l*sb0 + j*sb1];
 *   C (m x n) row-major with leading dimension ldc.
 * Output bits equal the reference CPU path for finite inputs.  Stages: split A and B into
 * int8 residues (K1), one tcgen05 int8 GEMM per modulus with the mod-reduce in its
 * epilogue (K2), exact CRT reconstruction + inverse scaling (K3).
 * workspace: device scratch of ti_crt_workspace_size() bytes, 256-byte aligned.
 */
int ti_crt_matmul(const double *A, int64_t sa0, int64_t sa1, const double *B, int64_t sb0,
                  int64_t sb1, double *C, int64_t ldc, int64_t m, int64_t n, int64_t k,
                  int bits, int out_mode, void *workspace, size_t workspace_bytes,
                  void *stream);

/*
 * ti_crt_matmul with options (moduli set, moduli count, profiling events).  With the
 * defaults it is ti_crt_matmul.  No counterpart in the reference, which has no options:
 * it extends crt_matmul.py:95 with an opt-in moduli set and moduli count.
 */
int ti_crt_matmul_ex(const double *A, int64_t sa0, int64_t sa1, const double *B, int64_t sb0,
                     int64_t sb1, double *C, int64_t ldc, int64_t m, int64_t n, int64_t k,
                     int bits, int out_mode, void *workspace, size_t workspace_bytes,
                     void *stream, const ti_crt_options_t *opt);

/*
 * crt_matmul on HOST operands (the reference's CPU-tensor call, crt_matmul.py:95), with
 * the copies pipelined against the kernels: all of B goes to the device first, then A in
 * row bands; each band is split, multiplied and reconstructed on `stream` as soon as it has
 * arrived, and its rows of C are copied back while the next band computes.  The three copy
 * streams run on the copy engines, so the transfers overlap the kernels.  Host memory
 * should be pinned (page-locked) for the copies to overlap; pageable memory still works,
 * serially.  A (m x k) element (i,l) at A[i*sa0 + l*sa1], B (k x n) at B[l*sb0 + j*sb1] (one
 * stride of each 1); C row-major host, leading dimension ldc; C = A @ B (store).  The call
 * is asynchronous on `stream`: synchronize it before reading C.
 * workspace: device scratch of ti_crt_host_workspace_size() bytes, 256-byte aligned.
 */
int ti_crt_host_workspace_size(int64_t m, int64_t n, int64_t k, int bits,
                               const ti_crt_options_t *opt, size_t *bytes);
int ti_crt_matmul_host(const double *A, int64_t sa0, int64_t sa1, const double *B, int64_t sb0,
                       int64_t sb1, double *C, int64_t ldc, int64_t m, int64_t n, int64_t k,
                       int bits, void *workspace, size_t workspace_bytes, void *stream,
                       const ti_crt_options_t *opt);

/*
 * ti_crt_matmul that also records four caller-created CUDA events (cudaEvent_t, passed as
 * void*; NULL entries are skipped) on `stream`: stage_events[0] before K1 (split),
 * [1] before K2 (residue GEMM), [2] before K3 (CRT), [3] after K3.  For profiling; the
 * events add no synchronisation.
 */
int ti_crt_matmul_events(const double *A, int64_t sa0, int64_t sa1, const double *B,
                         int64_t sb0, int64_t sb1, double *C, int64_t ldc, int64_t m, int64_t n,
                         int64_t k, int bits, int out_mode, void *workspace,
                         size_t workspace_bytes, void *stream, void *const *stage_events);

/* Bytes of the library's static device scratch used by ti_crt_matmul_noalloc (64 MiB). */
#define TI_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)

/*
 * ti_crt_matmul without a workspace, for callers that cannot allocate device memory: a host
 * program whose own allocator already owns the GPU's memory pool, or a latency-critical
 * caller that cannot afford cudaMalloc's implicit device synchronisation.  No counterpart
 * in the reference (its crt_matmul allocates through torch).  It calls no cudaMalloc,
 * cudaFree or allocating library routine; its scratch is a static device array of
 * TI_NOALLOC_SCRATCH_BYTES per device, held by every GPU that loads it until the process
 * exits.  Problems whose ti_crt_workspace_size() exceeds that return TI_ERR_SCRATCH_LIMIT
 * (about m = n = k = 940 at float64).  The first call on each device with a non-empty
 * output looks up the array's device address and should come before any stream capture.
 * All calls on a device share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  It always runs the reference's primes on the default path (no
 * ti_crt_options_t: no wide moduli, no fixed moduli count); with the tuning switch
 * TI_CRT_PATH=fused set in the environment every call returns TI_ERR_SCRATCH_LIMIT, because
 * that kernel's scratch holds one slot per SM.
 */
int ti_crt_matmul_noalloc(const double *A, int64_t sa0, int64_t sa1, const double *B,
                          int64_t sb0, int64_t sb1, double *C, int64_t ldc, int64_t m, int64_t n,
                          int64_t k, int bits, int out_mode, void *stream);

/*
 * Self-test of the kernels' bounded waits, for tests: launches a wait that nothing completes
 * (which = 0: an mbarrier of a one-CTA pipeline whose producer never arrives; which = 1: the
 * LU panel's grid barrier, waited on for one CTA more than arrive) with a limit of limit_ns
 * (1e3..1e10) instead of the kernels' 2 s, synchronises `stream` and returns
 * TI_ERR_DEVICE_TIMEOUT when the wait ran out and recorded its code in the device error word
 * (left set; read and clear it with ti_device_error).  No counterpart in the reference, whose
 * kernels have no bounded waits.
 */
int ti_selftest_bounded_wait(int which, long long limit_ns, void *stream);

/*
 * Reads (and, if reset != 0, clears) the current device's kernel error word.  Kernels set
 * it instead of hanging when a bounded wait runs out; 0 means no error.  Synchronous.
 */
int ti_device_error(int *code_out, int reset);

/*
 * The unblocked LU panel with partial pivoting of src/tensor_inv/lu.py:24-34 (the loop over
 * k in [j, jb) inside `lu`), in one launch on `stream`: for each column k the first index p of
 * max |W[i, k]| over i >= k, the swap of rows k and p of W (all n columns) and of piv[k], piv[p],
 * then, if |W[k, k]| > 1e-15, W[i, k] /= W[k, k] and W[i, c] -= W[i, k] * W[k, c] (product
 * rounded first) for i > k, k < c < jb.  Bit-identical to the reference's torch loop.
 * W: n x n float64, row-major with leading dimension ldw >= n; piv: int64 [n] (device).
 * jb - j <= 1024.  workspace: ti_lu_panel_workspace_size() bytes of device memory, 256-byte
 * aligned (its first bytes are cleared on `stream` by the call).  Returns TI_ERR_CUDA if the
 * cooperative launch fails; a grid barrier that runs out sets the device error word.
 */
int ti_lu_panel_workspace_size(size_t *bytes);
int ti_lu_panel(double *W, int64_t ldw, int64_t n, int64_t j, int64_t jb, int64_t *piv,
                void *workspace, size_t workspace_bytes, void *stream);

/*
 * ti_lu_panel on a panel that sits at any column of a rectangular W: the panel is rows
 * [j, n) of W's columns [pc, pc + jb - j), W has n rows and `ncols` columns (leading
 * dimension ldw >= ncols), and every row swap exchanges all ncols columns.  Column k of the
 * reference loop is W's column pc + (k - j); rows keep their global indices, as do piv's
 * entries.  ti_lu_panel(W, ldw, n, j, jb, ...) is ti_lu_panel_ex(W, ldw, n, n, j, jb, j, ...).
 * It serves a rank that holds only some block columns of the matrix (the block-cyclic LU of
 * tensor_inv_b200.distributed): the panel owner factorises its panel in its local columns.
 */
int ti_lu_panel_ex(double *W, int64_t ldw, int64_t n, int64_t ncols, int64_t j, int64_t jb,
                   int64_t pc, int64_t *piv, void *workspace, size_t workspace_bytes,
                   void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TENSOR_INV_CRT_H */
