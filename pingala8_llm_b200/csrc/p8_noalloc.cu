// p8_noalloc.cu -- a batch-1 GEMV entry point that allocates nothing and needs no caller workspace.
//
// For callers that cannot allocate device memory when they run the op and have no scratch buffer to lend it: for
// example a host application that plans every device allocation up front and gives this op only its weight, input and
// output buffers, or a code path that must not call cudaMalloc (which can synchronise the device and can fail under
// memory pressure). The scratch the GEMV needs (the row partials per 256-column block, and x' of an input op) lives
// in one fixed device array of this file instead of a caller workspace.
//
// The array is kNoAllocScratchBytes (6 MiB). It is placed on a device when this file's device module is loaded there,
// and with CUDA's default lazy module loading that happens inside the first p8_mul_mat_vec_noalloc call on that
// device: that first call makes the 6 MiB device allocation (the driver's, not this library's) and can fail like one
// (P8_ERR_NOALLOC_SCRATCH), and it must not run inside a stream capture. Make one call on every device during set-up,
// outside any capture; from then on every GPU that loaded the array holds it until the process exits.
// A tensor whose GEMV needs more scratch than that (p8_workspace_size(t, 1) > 6 MiB: 4 bytes per row and 256-column
// block plus 4 bytes per column, e.g. more than 1.5 M rows x blocks) is rejected with P8_ERR_WORKSPACE.
//
// All calls share the array and it keeps the previous call's contents: every partial a call reads is written by the
// same call first, so no state leaks between calls and nothing needs clearing. Calls that can overlap on the GPU
// (other streams, other host threads) race on the array and must be serialised by the caller.
#include <cuda_runtime.h>

#include "p8_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)6 << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array in the current device's context. In host code the array's name is only a
// host-side stand-in, so the address is looked up with the device current. It is looked up on every call (cheap once
// the module is loaded) rather than cached, so a context that was torn down and re-created (cudaDeviceReset) never sees
// an address of the old one.
p8_status scratch_for_current_device(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return P8_ERR_CUDA;
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
        (void)cudaGetLastError();  // the failed module load is reported through the status, not left pending
        return P8_ERR_NOALLOC_SCRATCH;
    }
    *out = p;
    return P8_OK;
}

}  // namespace

extern "C" {

size_t p8_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

p8_status p8_mul_mat_vec_noalloc(const p8_tensor *t, const float *x, float *y, void *stream) {
    if (!t || t->magic != kTensorMagic) return P8_ERR_NOT_PREPARED;
    if (!x || !y || ((uintptr_t)x & 15)) return P8_ERR_ARG;
    if (p8::gemv_workspace(t, 1) > kNoAllocScratchBytes) return P8_ERR_WORKSPACE;
    void *scratch = nullptr;
    p8_status st = scratch_for_current_device(&scratch);
    if (st) return st;
    return p8::launch_gemv(t, x, 1, t->K, y, t->rows, scratch, kNoAllocScratchBytes, (cudaStream_t)stream);
}

}  // extern "C"
