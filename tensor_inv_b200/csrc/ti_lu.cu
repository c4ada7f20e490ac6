// ti_lu.cu -- the unblocked LU panel with partial pivoting as one cooperative kernel.
//
// Restates the panel loop of src/tensor_inv/lu.py:24-34 with the same IEEE operations in the
// same order, so P, L and U are bit-identical to the reference's torch loop:
//   for k in [j, jb):
//     p = first index of the maximum of |W[i, k]| over i >= k    (torch argmax)
//     if p != k: swap rows k and p of W (all its columns) and entries k and p of piv
//     if |W[k, k]| > 1e-15:
//       W[i, k] = W[i, k] / W[k, k]                            for i > k
//       W[i, c] = W[i, c] - round(W[i, k] * W[k, c])           for i > k, k < c < jb
// The product is rounded before the subtraction, as the reference's separate `@` (a K = 1
// matrix product) and `-=`; nothing is contracted into a fused multiply-add.
//
// One launch per panel replaces the reference's 8 small launches and 2 host round trips per
// column.  CTAs (launched cooperatively, so all are resident at once) own contiguous row
// ranges of the panel.  In the global-memory variant each column takes two grid barriers:
// after the per-CTA argmax candidates (every CTA then reduces the same candidates in the same
// total order, so all agree on p), and after the row swap (the update reads the pivot row).
// The shared-memory variant below needs one per column.  The barriers' words live in the
// caller's workspace; every wait is bounded in time, and on timeout the kernel records an
// error and all CTAs return.  All accesses to W bypass L1 (ld/st .cg), so
// a CTA never reads a stale copy of a row that another CTA swapped or updated.
#include <atomic>
#include <cstring>

#include "tensor_inv_crt.h"
#include "ti_common.cuh"

namespace ti {

int device_context(int *num_sms, int **err);

constexpr int kLuThreads = 256;
constexpr int kLuMaxCtas = 1024;
constexpr int kLuMaxPanel = 1024;  // columns per panel

struct LuSync {
    unsigned count;
    unsigned gen;
    int abort;
    int pad;
};

struct LuCand {
    double v;   // |W[i, k]|
    long long i;
};

// a is a better argmax candidate than b: larger, or NaN over a number, or equal with the
// smaller index (torch.argmax returns the first maximal element; NaN counts as maximal)
__device__ __forceinline__ bool lu_better(double av, long long ai, double bv, long long bi) {
    const bool an = av != av, bn = bv != bv;
    if (an != bn) return an;
    if (!an && av != bv) return av > bv;
    return ai < bi;
}

// Grid-wide barrier over `nblocks` co-resident CTAs.  Returns false (in every thread of the
// CTA) if a wait ran out or another CTA gave up.
__device__ __forceinline__ unsigned lu_atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ unsigned lu_ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void lu_st_release(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid-wide barrier over `nblocks` co-resident CTAs.  Returns false (in every thread of the
// CTA) if a wait ran out or another CTA gave up.  Thread 0 arrives with an acquire-release
// add on the counter (after the CTA barrier, so it carries the CTA's writes); the last
// arrival resets the counter and releases the generation word, which the others poll with
// acquire loads.
__device__ bool lu_grid_sync(LuSync *s, unsigned nblocks, unsigned &gen_local, int *err) {
    __shared__ int ok_sh;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned target = gen_local + 1;
        if (lu_atom_add_acq_rel(&s->count, 1u) == nblocks - 1) {
            s->count = 0u;  // ordered before the release below
            lu_st_release(&s->gen, target);
        } else {
            const unsigned long long t0 = globaltimer_ns();
            while (lu_ld_acquire(&s->gen) != target) {
                if (*reinterpret_cast<volatile int *>(&s->abort)) {
                    ok = 0;
                    break;
                }
                if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
                    atomicExch(&s->abort, 1);
                    atomicCAS(err, 0, kErrTimeoutGridBarrier);
                    ok = 0;
                    break;
                }
            }
        }
        gen_local = target;
        ok_sh = ok;
    }
    __syncthreads();
    return ok_sh != 0;
}

// A split grid barrier on a count of arrivals that only grows during a launch (the host zeroes
// it first): barrier t is complete once the count reaches t * G.  Thread 0 arrives with a
// release reduction (no value returned, so it does not wait for the L2 round trip) after a CTA
// barrier, so the arrival carries the CTA's writes; waiters poll the count with acquire loads.
// A CTA can only arrive at barrier t + 1 after its own wait for t, so the count is below
// (t + 2) * G while any CTA waits for t.
__device__ __forceinline__ void lu_red_release_add(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// lu_grid_arrive: called by every thread after the CTA's writes that the other CTAs read;
// advances `target` to the count that completes this barrier.
__device__ __forceinline__ void lu_grid_arrive(LuSync *s, unsigned nblocks, unsigned &target) {
    __syncthreads();
    if (threadIdx.x == 0) lu_red_release_add(&s->count, 1u);
    target += nblocks;
}

// lu_grid_wait: until the count of arrivals reaches `target` (bounded by limit_ns; false in
// every thread if the wait ran out or another CTA gave up).  Ends with a CTA barrier.
__device__ bool lu_grid_wait(LuSync *s, unsigned target, int *err,
                             unsigned long long limit_ns = kWaitTimeoutNs) {
    __shared__ int ok_sh;
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned long long t0 = globaltimer_ns();
        while (static_cast<int>(lu_ld_acquire(&s->count) - target) < 0) {
            if (*reinterpret_cast<volatile int *>(&s->abort)) {
                ok = 0;
                break;
            }
            if (globaltimer_ns() - t0 > limit_ns) {
                atomicExch(&s->abort, 1);
                atomicCAS(err, 0, kErrTimeoutGridBarrier);
                ok = 0;
                break;
            }
        }
        ok_sh = ok;
    }
    __syncthreads();
    return ok_sh != 0;
}

// The best of the eight warps' candidates in red_*, computed by every warp: lanes 0..7 take one
// warp's candidate each and an xor-shuffle tree over them leaves the best in lane 0, which is
// broadcast.  The order (NaN first, then value, then the smaller index) is strict and total on
// distinct rows, so every warp, and every CTA reducing the same values, picks the same one as
// any other reduction order would.  red_b may be null (no CTA indices).
__device__ __forceinline__ void lu_reduce_warps(const double *red_v, const long long *red_i,
                                                const int *red_b, double &bv, long long &bi,
                                                int &bb) {
    constexpr int kW = kLuThreads / 32;
    const int lane = threadIdx.x & 31;
    bv = lane < kW ? red_v[lane] : -1.0;
    bi = lane < kW ? red_i[lane] : LLONG_MAX;
    bb = lane < kW && red_b ? red_b[lane] : 0;
#pragma unroll
    for (int off = kW / 2; off; off >>= 1) {
        const double ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
        const long long oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
        const int ob = __shfl_xor_sync(0xFFFFFFFFu, bb, off);
        if (oi != LLONG_MAX && (bi == LLONG_MAX || lu_better(ov, oi, bv, bi))) {
            bv = ov;
            bi = oi;
            bb = ob;
        }
    }
    bv = __shfl_sync(0xFFFFFFFFu, bv, 0);
    bi = __shfl_sync(0xFFFFFFFFu, bi, 0);
    bb = __shfl_sync(0xFFFFFFFFu, bb, 0);
}

// The global pivot from the G published candidates: thread t loads candidate t (all loads in
// flight at once), then a warp reduction and, in every warp, the reduction of the eight warps'
// results (lu_reduce_warps).  Every CTA reduces the same values in the same total order, so all
// agree.  Returns the row and the publishing CTA in every thread.  red_* are read after the CTA
// barrier inside; the caller passes another CTA barrier before they are written again.
__device__ __forceinline__ void lu_global_pivot(const LuCand *cands, unsigned G, long long &row,
                                                int &cta, double *red_v, long long *red_i,
                                                int *red_b) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    double bv = -1.0;
    long long bi = LLONG_MAX;
    int bb = 0;
    for (unsigned q = tid; q < G; q += kLuThreads) {
        const double v = __ldcg(&cands[q].v);
        const long long i = __ldcg(&cands[q].i);
        if (i != LLONG_MAX && (bi == LLONG_MAX || lu_better(v, i, bv, bi))) {
            bv = v;
            bi = i;
            bb = static_cast<int>(q);
        }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const double ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
        const long long oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
        const int ob = __shfl_xor_sync(0xFFFFFFFFu, bb, off);
        if (oi != LLONG_MAX && (bi == LLONG_MAX || lu_better(ov, oi, bv, bi))) {
            bv = ov;
            bi = oi;
            bb = ob;
        }
    }
    if (lane == 0) {
        red_v[warp] = bv;
        red_i[warp] = bi;
        red_b[warp] = bb;
    }
    __syncthreads();
    lu_reduce_warps(red_v, red_i, red_b, bv, bi, bb);
    row = bi;
    cta = bb;
}

__global__ void __launch_bounds__(kLuThreads)
    lu_panel_kernel(double *__restrict__ W, int64_t ldw, int64_t n, int64_t ncols, int64_t j,
                    int64_t jb, int64_t dc, int64_t *__restrict__ piv, LuSync *sync, LuCand *cand,
                    int *err) {
    __shared__ double urow[kLuMaxPanel];  // W[k, k+1 .. jb-1] of the current column
    __shared__ double red_v[kLuThreads / 32];
    __shared__ long long red_i[kLuThreads / 32];
    __shared__ int red_b[kLuThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned G = gridDim.x;
    const int64_t rows = n - j;
    const int64_t per = (rows + G - 1) / G;
    const int64_t r0 = j + int64_t(blockIdx.x) * per;
    const int64_t r1 = r0 + per < n ? r0 + per : n;  // owned rows [r0, r1)
    unsigned gen = 0;

    for (int64_t k = j; k < jb; ++k) {
        // ---- A: this CTA's argmax candidate over owned rows >= k (column k)
        double bv = -1.0;
        long long bi = LLONG_MAX;
        for (int64_t i = (r0 > k ? r0 : k) + tid; i < r1; i += kLuThreads) {
            const double v = fabs(__ldcg(W + i * ldw + k + dc));
            if (bi == LLONG_MAX || lu_better(v, i, bv, bi)) {
                bv = v;
                bi = i;
            }
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            const double ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
            const long long oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
            if (oi != LLONG_MAX && (bi == LLONG_MAX || lu_better(ov, oi, bv, bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            red_v[warp] = bv;
            red_i[warp] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < kLuThreads / 32; ++w)
                if (red_i[w] != LLONG_MAX &&
                    (bi == LLONG_MAX || lu_better(red_v[w], red_i[w], bv, bi))) {
                    bv = red_v[w];
                    bi = red_i[w];
                }
            cand[blockIdx.x].v = bv;
            cand[blockIdx.x].i = bi;
        }
        if (!lu_grid_sync(sync, G, gen, err)) return;

        // ---- B: the global pivot, then the row swap
        long long p_row;
        int p_cta;
        lu_global_pivot(cand, G, p_row, p_cta, red_v, red_i, red_b);
        const int64_t p = p_row;
        if (p != k) {
            const int64_t per_c = (ncols + G - 1) / G;
            const int64_t c0 = int64_t(blockIdx.x) * per_c;
            const int64_t c1 = c0 + per_c < ncols ? c0 + per_c : ncols;
            for (int64_t c = c0 + tid; c < c1; c += kLuThreads) {
                const double a = __ldcg(W + k * ldw + c), b = __ldcg(W + p * ldw + c);
                __stcg(W + k * ldw + c, b);
                __stcg(W + p * ldw + c, a);
            }
            if (blockIdx.x == 0 && tid == 0) {
                const int64_t t = piv[k];
                piv[k] = piv[p];
                piv[p] = t;
            }
        }
        if (!lu_grid_sync(sync, G, gen, err)) return;

        // ---- C: scale column k and update the panel, owned rows > k
        const double d = __ldcg(W + k * ldw + k + dc);
        if (!(fabs(d) > 1e-15)) continue;  // the reference skips this column
        const int64_t nc = jb - k - 1;
        for (int64_t c = tid; c < nc; c += kLuThreads)
            urow[c] = __ldcg(W + k * ldw + k + dc + 1 + c);
        __syncthreads();
        for (int64_t i = (r0 > k + 1 ? r0 : k + 1) + warp; i < r1; i += kLuThreads / 32) {
            double *wi = W + i * ldw + dc;  // panel column k of row i at wi[k]
            const double l = __ddiv_rn(__ldcg(wi + k), d);
            for (int64_t c0 = 0; c0 < nc; c0 += 256) {  // 8 loads in flight per lane
                double x[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int64_t c = c0 + lane + 32 * u;
                    x[u] = c < nc ? __ldcg(wi + k + 1 + c) : 0.0;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int64_t c = c0 + lane + 32 * u;
                    if (c < nc) __stcg(wi + k + 1 + c, __dsub_rn(x[u], __dmul_rn(l, urow[c])));
                }
            }
            if (lane == 0) __stcg(wi + k, l);
        }
        __syncthreads();  // urow is rewritten in the next column
    }
}

// ---------------------------------------------------------------------------------------
// Shared-memory variant: each CTA keeps its panel rows (all b columns) in shared memory for
// the whole panel, so the column updates never touch global memory, and one grid barrier per
// column suffices.  Before column k's barrier every CTA publishes its argmax candidate (with
// the candidate row's values at columns k and k+1) and that candidate's panel row, and the
// owner of row k publishes row k and, apart, its values at columns k and k+1 (all
// double-buffered by column parity: a CTA can only write column k+1's slots after every CTA
// has passed column k's barrier, and it reads column k's slots before arriving at column
// k+1's).  After the barrier every CTA reduces the candidates to the pivot row p; those loads
// also bring the pivot W[p, k], W[p, k+1] and old row k's W[k, k], W[k, k+1], which are all
// that the multipliers and the update of column k+1 need, so those run while the full pivot
// row (and, for the owner of p, old row k) are still on their way from L2 into registers.
// The barrier is split into an arrival and a wait, and column k+1's candidate is found ahead
// of the rest of column k's update: each CTA divides its rows' multipliers and updates
// column k+1 only, takes its candidate for column k+1, places the swapped rows, finishes the
// two rows it may publish (the candidate and row k+1), publishes and arrives; the rest of the
// rank-1 update (columns k+2 ..) and the swap of the columns outside the panel (in global
// memory, each CTA always on the same column slice, so its swaps stay in program order) run
// while the other CTAs arrive.  Every element receives the same operations in the same order.
// ---------------------------------------------------------------------------------------
constexpr int kLuSmemMaxPanel = 256;
constexpr int kLuSmemMaxCtas = 256;
static_assert(kLuSmemMaxPanel <= kLuThreads && kLuSmemMaxCtas <= kLuThreads,
              "one thread per panel column and per candidate");

struct LuCandRow {
    double d;      // the candidate row's W[i, k]; |d| ranks the candidates
    long long i;   // the row, LLONG_MAX if the CTA has no rows >= k
    double u1;     // the candidate row's W[i, k + 1] (0 past the panel)
    double pad;
};

struct LuSlots {
    LuCandRow cand[2][kLuSmemMaxCtas];
    double khead[2][2];  // W[k, k], W[k, k + 1] of row k before the swap
    double krow[2][kLuSmemMaxPanel];
    double crow[2][kLuSmemMaxCtas][kLuSmemMaxPanel];
};

// This CTA's argmax candidate for column k (panel column kc of P) over its rows >= k, returned
// in every thread.  red_* are read after the CTA barrier inside; the caller passes another CTA
// barrier before they are written again.
__device__ __forceinline__ long long lu_cta_candidate(const double *P, int pitch, int64_t r0,
                                                      int64_t r1, int64_t k, int kc,
                                                      double *red_v, long long *red_i) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    double bv = -1.0;
    long long bi = LLONG_MAX;
    for (int64_t i = (r0 > k ? r0 : k) + tid; i < r1; i += kLuThreads) {
        const double v = fabs(P[(i - r0) * pitch + kc]);
        if (bi == LLONG_MAX || lu_better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const double ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
        const long long oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
        if (oi != LLONG_MAX && (bi == LLONG_MAX || lu_better(ov, oi, bv, bi))) {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0) {
        red_v[warp] = bv;
        red_i[warp] = bi;
    }
    __syncthreads();
    int unused;
    lu_reduce_warps(red_v, red_i, nullptr, bv, bi, unused);
    return bi;
}

// Column k's slots (panel column kc): the candidate `mine` with its values at kc and kc+1,
// its panel row, and (owner of row k) row k with, apart, its values at kc and kc+1.
__device__ __forceinline__ void lu_publish(LuSlots *slots, int par, const double *P, int pitch,
                                           int b, int64_t r0, int64_t r1, int64_t k, int kc,
                                           long long mine) {
    const int tid = threadIdx.x;
    const bool own_k = k >= r0 && k < r1;
    if (mine != LLONG_MAX)
        for (int c = tid; c < b; c += kLuThreads)
            __stcg(&slots->crow[par][blockIdx.x][c], P[(mine - r0) * pitch + c]);
    if (own_k)
        for (int c = tid; c < b; c += kLuThreads)
            __stcg(&slots->krow[par][c], P[(k - r0) * pitch + c]);
    if (tid == 0) {
        LuCandRow *s = &slots->cand[par][blockIdx.x];
        const double *pm = mine != LLONG_MAX ? P + (mine - r0) * pitch : nullptr;
        __stcg(&s->d, pm ? pm[kc] : 0.0);
        __stcg(&s->i, mine);
        __stcg(&s->u1, pm && kc + 1 < b ? pm[kc + 1] : 0.0);
    }
    if (tid == 32 && own_k) {
        const double *pk = P + (k - r0) * pitch;
        __stcg(&slots->khead[par][0], pk[kc]);
        __stcg(&slots->khead[par][1], kc + 1 < b ? pk[kc + 1] : 0.0);
    }
}

// The pivot from column k's G published candidates (thread t loads candidate t), with the
// pivot row's values at columns k and k+1 and old row k's (from the header slot), in every
// thread.  `bc` is 4 doubles of shared memory.  Every CTA reduces the same values in the same
// total order, so all agree.  red_* and bc are read after the CTA barriers inside; the caller
// passes another CTA barrier before they are written again.
__device__ __forceinline__ void lu_smem_pivot(const LuCandRow *cands, const double *khead,
                                              unsigned G, long long &row, int &cta, double &d,
                                              double &u1, double &k0, double &k1, double *red_v,
                                              long long *red_i, int *red_b, double *bc) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    double bv = -1.0, dv = 0.0, uv = 0.0;
    long long bi = LLONG_MAX;
    int bb = 0;
    if (tid < static_cast<int>(G)) {
        const long long i = __ldcg(&cands[tid].i);
        dv = __ldcg(&cands[tid].d);
        uv = __ldcg(&cands[tid].u1);
        if (i != LLONG_MAX) {
            bv = fabs(dv);
            bi = i;
            bb = tid;
        }
    }
    if (tid == kLuThreads - 1) {
        bc[2] = __ldcg(&khead[0]);
        bc[3] = __ldcg(&khead[1]);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const double ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
        const long long oi = __shfl_xor_sync(0xFFFFFFFFu, bi, off);
        const int ob = __shfl_xor_sync(0xFFFFFFFFu, bb, off);
        if (oi != LLONG_MAX && (bi == LLONG_MAX || lu_better(ov, oi, bv, bi))) {
            bv = ov;
            bi = oi;
            bb = ob;
        }
    }
    if (lane == 0) {
        red_v[warp] = bv;
        red_i[warp] = bi;
        red_b[warp] = bb;
    }
    __syncthreads();
    lu_reduce_warps(red_v, red_i, red_b, bv, bi, bb);
    if (tid == bb) {  // the thread that loaded the winner holds its values
        bc[0] = dv;
        bc[1] = uv;
    }
    __syncthreads();
    row = bi;
    cta = bb;
    d = bc[0];
    u1 = bc[1];
    k0 = bc[2];
    k1 = bc[3];
}

__global__ void __launch_bounds__(kLuThreads, 1)
    lu_panel_smem_kernel(double *__restrict__ W, int64_t ldw, int64_t n, int64_t ncols, int64_t j,
                         int64_t jb, int64_t col0, int64_t *__restrict__ piv, LuSync *sync,
                         LuSlots *slots, int *err) {
    extern __shared__ double P[];            // [per][b + 1]: owned rows, panel columns
    __shared__ double urow[kLuSmemMaxPanel];  // the pivot row (after the swap), panel columns
    __shared__ double red_v[kLuThreads / 32];
    __shared__ long long red_i[kLuThreads / 32];
    __shared__ int red_b[kLuThreads / 32];
    __shared__ double bc[4];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned G = gridDim.x;
    const int b = static_cast<int>(jb - j), pitch = b + 1;
    const int64_t per = (n - j + G - 1) / G;
    const int64_t r0 = j + int64_t(blockIdx.x) * per;
    const int64_t r1 = r0 + per < n ? r0 + per : n;
    const int nr = r1 > r0 ? static_cast<int>(r1 - r0) : 0;
    unsigned arrivals = 0;  // the count of arrivals that completes the next barrier

    for (int e = tid; e < nr * b; e += kLuThreads) {
        const int r = e / b, c = e - r * b;
        P[r * pitch + c] = __ldcg(W + (r0 + r) * ldw + col0 + c);
    }
    // columns outside the panel, this CTA's slice of them (for the row swaps)
    const int64_t nout = ncols - b;
    const int64_t per_c = (nout + G - 1) / G;
    const int64_t t0 = int64_t(blockIdx.x) * per_c;
    const int64_t t1 = t0 + per_c < nout ? t0 + per_c : nout;
    __syncthreads();

    // column j's slots, published before the first barrier
    {
        const long long mine = lu_cta_candidate(P, pitch, r0, r1, j, 0, red_v, red_i);
        lu_publish(slots, static_cast<int>(j & 1), P, pitch, b, r0, r1, j, 0, mine);
    }
    lu_grid_arrive(sync, G, arrivals);

    for (int64_t k = j; k < jb; ++k) {
        const int kc = static_cast<int>(k - j);  // panel column of k
        const int par = static_cast<int>(k & 1);
        if (!lu_grid_wait(sync, arrivals, err)) return;

        // ---- B: the pivot and the values the multipliers need; the full pivot row and (owner
        // of p) old row k start towards registers
        long long p_row;
        int pcta;
        double d, u1, k0, k1;
        lu_smem_pivot(slots->cand[par], slots->khead[par], G, p_row, pcta, d, u1, k0, k1, red_v,
                      red_i, red_b, bc);
        const int64_t p = p_row;
        const bool own_k = k >= r0 && k < r1;
        const bool own_p = p != k && p >= r0 && p < r1;
        double ru = 0.0, rk = 0.0;
        if (tid < b) {
            ru = __ldcg(&slots->crow[par][pcta][tid]);
            if (own_p) rk = __ldcg(&slots->krow[par][tid]);
        }

        // ---- C1: every owned row > k: its multiplier l = W[i, k] / d, then its column k + 1
        // (one row per thread, the divisions in parallel).  Row p already holds old row k
        // here: its two values come from the header slot.
        const bool upd = fabs(d) > 1e-15;  // the reference skips this column otherwise
        const int64_t i0 = r0 > k + 1 ? r0 : k + 1;
        if (upd) {
            for (int64_t i = i0 + tid; i < r1; i += kLuThreads) {
                double *pi = P + (i - r0) * pitch;
                const bool sw = i == p;
                const double l = __ddiv_rn(sw ? k0 : pi[kc], d);
                pi[kc] = l;
                if (kc + 1 < b)
                    pi[kc + 1] = __dsub_rn(sw ? k1 : pi[kc + 1], __dmul_rn(l, u1));
            }
        } else if (own_p && tid == 0) {
            double *pp = P + (p - r0) * pitch;
            pp[kc] = k0;
            if (kc + 1 < b) pp[kc + 1] = k1;
        }
        __syncthreads();

        // ---- A of column k + 1, ahead of the rest of column k's update: column k + 1 is final
        // in every row, so the candidate is too
        const long long mine =
            k + 1 < jb ? lu_cta_candidate(P, pitch, r0, r1, k + 1, kc + 1, red_v, red_i)
                       : LLONG_MAX;

        // ---- the swap: row k takes the pivot row, row p old row k (its columns k and k + 1
        // were written above)
        if (tid < b) {
            urow[tid] = ru;
            if (own_k && p != k) P[(k - r0) * pitch + tid] = ru;
            if (own_p && tid != kc && tid != kc + 1) P[(p - r0) * pitch + tid] = rk;
        }
        if (p != k && blockIdx.x == 0 && tid == 0) {
            const int64_t t = piv[k];
            piv[k] = piv[p];
            piv[p] = t;
        }
        __syncthreads();

        // ---- the two rows other CTAs may read (the candidate and row k + 1) are finished
        // first, published, and the CTA arrives
        long long done_a = LLONG_MAX, done_b = LLONG_MAX;  // rows already fully updated
        if (k + 1 < jb) {
            const bool own1 = k + 1 >= r0 && k + 1 < r1;
            if (upd) {
                const int64_t fin = warp == 0 ? mine : (warp == 1 && own1 && k + 1 != mine)
                                                           ? k + 1 : LLONG_MAX;
                if (fin != LLONG_MAX) {
                    double *pi = P + (fin - r0) * pitch;
                    const double l = pi[kc];
                    for (int c = kc + 2 + lane; c < b; c += 32)
                        pi[c] = __dsub_rn(pi[c], __dmul_rn(l, urow[c]));
                }
            }
            __syncthreads();
            lu_publish(slots, par ^ 1, P, pitch, b, r0, r1, k + 1, kc + 1, mine);
            lu_grid_arrive(sync, G, arrivals);
            done_a = mine;
            done_b = own1 ? k + 1 : LLONG_MAX;
        }

        // ---- C2: the rest of the rank-1 update (columns k + 2 ..), a warp per row, and the
        // swap of the columns outside the panel (this CTA's slice), while the others arrive
        if (upd) {
            for (int64_t i = i0 + warp; i < r1; i += kLuThreads / 32) {
                if (i == done_a || i == done_b) continue;
                double *pi = P + (i - r0) * pitch;
                const double l = pi[kc];
                for (int c = kc + 2 + lane; c < b; c += 32)
                    pi[c] = __dsub_rn(pi[c], __dmul_rn(l, urow[c]));
            }
        }
        if (p != k) {
            for (int64_t t = t0 + tid; t < t1; t += kLuThreads) {
                const int64_t c = t < col0 ? t : t + b;
                const double x = __ldcg(W + k * ldw + c), y = __ldcg(W + p * ldw + c);
                __stcg(W + k * ldw + c, y);
                __stcg(W + p * ldw + c, x);
            }
        }
        // the next column's wait ends with a CTA barrier before P or urow is touched again
    }
    __syncthreads();

    for (int e = tid; e < nr * b; e += kLuThreads) {
        const int r = e / b, c = e - r * b;
        __stcg(W + (r0 + r) * ldw + col0 + c, P[r * pitch + c]);
    }
}

size_t lu_smem_bytes(int64_t rows_per_cta, int64_t b) {
    return size_t(rows_per_cta) * size_t(b + 1) * sizeof(double);
}

// ---------------------------------------------------------------------------------------
// Self-test of the bounded waits (ti_selftest_bounded_wait): waits that nothing will ever
// complete, with a short limit, so the path by which a broken pipeline becomes an error code
// instead of a hung GPU actually runs.  Both use the library's own wait primitives.
// ---------------------------------------------------------------------------------------

// One CTA: an mbarrier that expects one arrival which never comes (the wait of an MMA or
// epilogue warp whose producer died).
__global__ void __launch_bounds__(32) selftest_mbar_timeout_kernel(unsigned long long limit_ns,
                                                                   int *err) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        abort_flag = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0 && !mbar_wait(&bar, 0, &abort_flag, limit_ns))
        atomicCAS(err, 0, kErrTimeoutMma);
}

// `ctas` CTAs: each arrives once at the LU panel's grid barrier and waits for one arrival more
// than there are CTAs (a CTA that never arrives).
__global__ void __launch_bounds__(32) selftest_grid_timeout_kernel(LuSync *sync,
                                                                   unsigned long long limit_ns,
                                                                   int *err) {
    unsigned target = 0;
    lu_grid_arrive(sync, gridDim.x, target);
    lu_grid_wait(sync, target + 1, err, limit_ns);
}

__device__ LuSync g_selftest_sync;

}  // namespace ti

using namespace ti;

// Largest dynamic shared memory of lu_panel_smem_kernel on each device (0: not yet set up).
constexpr int kLuMaxDevices = 64;
static std::atomic<size_t> g_lu_max_dyn[kLuMaxDevices];

extern "C" {

// Workspace: the barrier words (256 bytes), the candidates of the global-memory kernel, then
// the slots of the shared-memory kernel.
static size_t lu_cand_offset() { return 256; }
static size_t lu_slots_offset() {
    return (256 + sizeof(LuCand) * kLuMaxCtas + 255) / 256 * 256;
}

int ti_lu_panel_workspace_size(size_t *bytes) {
    if (!bytes) return TI_ERR_INVALID_ARGUMENT;
    *bytes = lu_slots_offset() + sizeof(LuSlots);
    return TI_OK;
}

int ti_lu_panel(double *W, int64_t ldw, int64_t n, int64_t j, int64_t jb, int64_t *piv,
                void *workspace, size_t workspace_bytes, void *stream) {
    return ti_lu_panel_ex(W, ldw, n, n, j, jb, j, piv, workspace, workspace_bytes, stream);
}

int ti_lu_panel_ex(double *W, int64_t ldw, int64_t n, int64_t ncols, int64_t j, int64_t jb,
                   int64_t pc, int64_t *piv, void *workspace, size_t workspace_bytes,
                   void *stream) {
    if (!W || !piv || n < 1 || ncols < 1 || ldw < ncols || j < 0 || jb <= j || jb > n ||
        jb - j > kLuMaxPanel || pc < 0 || pc + (jb - j) > ncols)
        return TI_ERR_INVALID_ARGUMENT;
    int64_t dc = pc - j;  // column shift of the panel (a kernel argument, so not const)
    size_t need = 0;
    ti_lu_panel_workspace_size(&need);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return TI_ERR_WORKSPACE;
    int num_sms = 0;
    int *err = nullptr;
    int rc = device_context(&num_sms, &err);
    if (rc != TI_OK) return rc;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lu_panel_kernel, kLuThreads, 0) !=
            cudaSuccess ||
        per_sm < 1)
        return TI_ERR_CUDA;
    // at least 32 rows per CTA; every CTA resident at once (cooperative launch)
    int64_t grid = (n - j + 31) / 32;
    if (grid > num_sms) grid = num_sms;
    if (grid > int64_t(per_sm) * num_sms) grid = int64_t(per_sm) * num_sms;
    if (grid > kLuMaxCtas) grid = kLuMaxCtas;
    if (grid < 1) grid = 1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    LuSync *sync = reinterpret_cast<LuSync *>(ws);
    if (cudaMemsetAsync(sync, 0, sizeof(LuSync), s) != cudaSuccess) return TI_ERR_CUDA;
    // shared-memory variant when the CTAs' panel rows fit (one CTA per SM)
    const int64_t b = jb - j;
    int64_t g_smem = (n - j + 31) / 32;
    if (g_smem > num_sms) g_smem = num_sms;
    if (g_smem > kLuSmemMaxCtas) g_smem = kLuSmemMaxCtas;
    const int64_t per = (n - j + g_smem - 1) / g_smem;
    const size_t smem = lu_smem_bytes(per, b);
    // the largest dynamic shared memory a CTA may take: the opt-in limit less the kernel's
    // static arrays (at b = 256 this holds 111 rows per CTA: n = 16384 on 148 SMs)
    // (kept per device, set up once on each; threads racing on the first call of a device
    // both set the same attribute, which is harmless)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kLuMaxDevices)
        return TI_ERR_NO_DEVICE;
    size_t max_dyn = g_lu_max_dyn[dev].load(std::memory_order_acquire);
    if (max_dyn == 0) {
        cudaFuncAttributes fa;
        int optin = 0;
        if (cudaFuncGetAttributes(&fa, lu_panel_smem_kernel) != cudaSuccess ||
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
                cudaSuccess ||
            optin <= static_cast<int>(fa.sharedSizeBytes))
            return TI_ERR_CUDA;
        max_dyn = size_t(optin) - fa.sharedSizeBytes;
        if (cudaFuncSetAttribute(lu_panel_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(max_dyn)) != cudaSuccess)
            return TI_ERR_CUDA;
        g_lu_max_dyn[dev].store(max_dyn, std::memory_order_release);
    }
    if (b <= kLuSmemMaxPanel && smem <= max_dyn) {
        int per_sm_s = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_s, lu_panel_smem_kernel,
                                                          kLuThreads, smem) == cudaSuccess &&
            int64_t(per_sm_s) * num_sms >= g_smem) {
            LuSlots *slots = reinterpret_cast<LuSlots *>(ws + lu_slots_offset());
            void *args[] = {&W, &ldw, &n, &ncols, &j, &jb, &pc, &piv, &sync, &slots, &err};
            if (cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(lu_panel_smem_kernel),
                                            dim3(static_cast<unsigned>(g_smem)), dim3(kLuThreads),
                                            args, smem, s) != cudaSuccess)
                return TI_ERR_CUDA;
            return TI_OK;
        }
    }
    LuCand *cand = reinterpret_cast<LuCand *>(ws + lu_cand_offset());
    void *args[] = {&W, &ldw, &n, &ncols, &j, &jb, &dc, &piv, &sync, &cand, &err};
    if (cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(lu_panel_kernel),
                                    dim3(static_cast<unsigned>(grid)), dim3(kLuThreads), args, 0,
                                    s) != cudaSuccess)
        return TI_ERR_CUDA;
    return TI_OK;
}

// Test entry: see tensor_inv_crt.h.  Synchronous; the waits run out after limit_ns.
int ti_selftest_bounded_wait(int which, long long limit_ns, void *stream) {
    if ((which != 0 && which != 1) || limit_ns < 1000 || limit_ns > 10000000000ll)
        return TI_ERR_INVALID_ARGUMENT;
    int num_sms = 0;
    int *err = nullptr;
    int rc = device_context(&num_sms, &err);
    if (rc != TI_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned long long lim = static_cast<unsigned long long>(limit_ns);
    if (which == 0) {
        selftest_mbar_timeout_kernel<<<1, 32, 0, s>>>(lim, err);
    } else {
        LuSync *sync = nullptr;
        if (cudaGetSymbolAddress(reinterpret_cast<void **>(&sync), g_selftest_sync) != cudaSuccess ||
            cudaMemsetAsync(sync, 0, sizeof(LuSync), s) != cudaSuccess)
            return TI_ERR_CUDA;
        selftest_grid_timeout_kernel<<<4, 32, 0, s>>>(sync, lim, err);
    }
    if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess)
        return TI_ERR_CUDA;
    int code = 0;
    if (cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return TI_ERR_CUDA;
    return code != 0 ? TI_ERR_DEVICE_TIMEOUT : TI_OK;
}

}  // extern "C"
