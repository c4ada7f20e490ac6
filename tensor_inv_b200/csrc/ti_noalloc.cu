// ti_noalloc.cu -- ti_crt_matmul_noalloc: the CRT matmul for callers that cannot allocate.
//
// Some callers of this library cannot call cudaMalloc, or must not at call time:
//   * a host application whose own allocator has already reserved the GPU's memory as a
//     pool, so a stray cudaMalloc either fails or fragments memory it does not own;
//   * latency-critical callers, because cudaMalloc/cudaFree may synchronise the device
//     and take driver-wide locks, stalling every other stream of the process.
// For them this entry point runs the same three stages as ti_crt_matmul (split, tcgen05
// residue GEMM, exact CRT) with the scratch taken from a fixed array in device memory
// that belongs to the library: kNoallocScratchBytes (64 MiB) per device, reserved when
// this module is loaded on that device and held until the process exits.
//
// The array's name is only a host-side stand-in in host code, never a device address.
// The device address is fetched once per device with cudaGetSymbolAddress, with that
// device current, by the first call made on the device; that first call should therefore
// come before any stream capture.  Every call on a device shares the one array and it
// keeps the previous call's contents.  Nothing in it has to start at zero: every byte a
// call reads was written earlier by the same call.  Calls whose kernels overlap on the
// GPU (different streams, or host threads) race on the array and must be serialised by
// the caller.
//
// It always runs the reference's 25-prime scheme through the default single-band path: it
// takes no ti_crt_options_t, so the wide moduli, a fixed moduli count and the stage events
// are not available here.  The opt-in fused GEMM+CRT kernel (TI_CRT_PATH=fused in the
// environment, a tuning switch) sizes its scratch for one slot per SM, about 150-300 MB, so
// with that switch set every call here returns TI_ERR_SCRATCH_LIMIT.
#include <atomic>

#include "tensor_inv_crt.h"

namespace {

constexpr size_t kNoallocScratchBytes = TI_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::atomic<void *> g_scratch_ptr[kMaxDevices];

// Device address of g_noalloc_scratch on the current device (set up on first use).
int scratch_for_current_device(void **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return TI_ERR_NO_DEVICE;
    if (dev >= kMaxDevices) return TI_ERR_UNSUPPORTED;
    void *p = g_scratch_ptr[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) return TI_ERR_CUDA;
        g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return TI_OK;
}

}  // namespace

extern "C" int ti_crt_matmul_noalloc(const double *A, int64_t sa0, int64_t sa1, const double *B,
                                     int64_t sb0, int64_t sb1, double *C, int64_t ldc, int64_t m,
                                     int64_t n, int64_t k, int bits, int out_mode, void *stream) {
    size_t need = 0;
    int rc = ti_crt_workspace_size(m, n, k, bits, &need);
    if (rc != TI_OK) return rc;
    if (need > kNoallocScratchBytes) return TI_ERR_SCRATCH_LIMIT;
    // An empty output needs no scratch: the shapes are checked and nothing is launched, so an
    // empty call never looks the array up (and may come first, even inside a capture).
    if (m == 0 || n == 0)
        return ti_crt_matmul(A, sa0, sa1, B, sb0, sb1, C, ldc, m, n, k, bits, out_mode, nullptr,
                             0, stream);
    void *scratch = nullptr;
    rc = scratch_for_current_device(&scratch);
    if (rc != TI_OK) return rc;
    return ti_crt_matmul(A, sa0, sa1, B, sb0, sb1, C, ldc, m, n, k, bits, out_mode, scratch,
                         kNoallocScratchBytes, stream);
}
