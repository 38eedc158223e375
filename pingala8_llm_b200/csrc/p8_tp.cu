// p8_tp.cu -- C ABI of the row-parallel exchange: per-rank exchange buffers, their peer mappings, and the fused
// GEMV + all-reduce (p8_tp_gemv_allreduce). The kernel side is the GEMV's epilogue (tp_exchange_row, p8_kernels.cu).
#include <cuda_runtime.h>
#include <string.h>

#include "p8_internal.h"

using namespace p8;

struct p8_tp_comm {
    uint32_t magic;
    int device, rank, world;
    int64_t cap;                              // output rows per (parity, rank) section
    uint64_t timeout_ns;
    unsigned long long *buf;                  // this rank's exchange buffer: 2 * world * cap entries
    unsigned int *epoch;                      // this rank's call counter (not shared)
    unsigned long long *peer[kTpMaxWorld];    // peer q's exchange buffer as mapped in this process
    bool mapped[kTpMaxWorld];                 // peer[q] came from an IPC handle (unmapped at destroy)
};

namespace {
constexpr uint32_t kCommMagic = 0x50385443u;
constexpr int64_t kMaxCap = int64_t(1) << 24;

bool valid_comm(const p8_tp_comm *c) { return c && c->magic == kCommMagic; }
size_t buf_bytes(const p8_tp_comm *c) { return (size_t)2 * c->world * (size_t)c->cap * 8; }

bool on_device(int dev) {
    int cur = -1;
    return cudaGetDevice(&cur) == cudaSuccess && cur == dev;
}
}  // namespace

extern "C" {

p8_status p8_tp_comm_create(int rank, int world, int64_t max_rows, uint32_t timeout_ms, p8_tp_comm **out) {
    if (!out) return P8_ERR_ARG;
    *out = nullptr;
    if (world < 1 || world > kTpMaxWorld || rank < 0 || rank >= world || max_rows < 1 || max_rows > kMaxCap ||
        timeout_ms < 1 || timeout_ms > 600000)
        return P8_ERR_ARG;
    p8_tp_comm *c = new p8_tp_comm();
    c->magic = kCommMagic;
    c->rank = rank;
    c->world = world;
    c->cap = max_rows;
    c->timeout_ns = (uint64_t)timeout_ms * 1000000ull;
    if (cudaGetDevice(&c->device) != cudaSuccess || cudaMalloc((void **)&c->buf, buf_bytes(c)) != cudaSuccess ||
        cudaMalloc((void **)&c->epoch, sizeof(unsigned int)) != cudaSuccess ||
        cudaMemset(c->buf, 0, buf_bytes(c)) != cudaSuccess || cudaMemset(c->epoch, 0, sizeof(unsigned int)) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(c->buf);
        cudaFree(c->epoch);
        c->magic = 0;
        delete c;
        return P8_ERR_CUDA;
    }
    c->peer[rank] = c->buf;
    *out = c;
    return P8_OK;
}

p8_status p8_tp_comm_destroy(p8_tp_comm *c) {
    if (!valid_comm(c)) return P8_ERR_ARG;
    for (int q = 0; q < c->world; ++q)
        if (c->mapped[q]) cudaIpcCloseMemHandle(c->peer[q]);
    cudaFree(c->buf);
    cudaFree(c->epoch);
    c->magic = 0;
    delete c;
    return P8_OK;
}

p8_status p8_tp_comm_ipc_handle(const p8_tp_comm *c, void *handle, size_t handle_bytes) {
    if (!valid_comm(c) || !handle || handle_bytes < sizeof(cudaIpcMemHandle_t)) return P8_ERR_ARG;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, c->buf) != cudaSuccess) return P8_ERR_CUDA;
    memcpy(handle, &h, sizeof(h));
    return P8_OK;
}

p8_status p8_tp_comm_open_peer(p8_tp_comm *c, int q, const void *handle, size_t handle_bytes) {
    if (!valid_comm(c) || q < 0 || q >= c->world || q == c->rank || c->peer[q] || !handle ||
        handle_bytes < sizeof(cudaIpcMemHandle_t))
        return P8_ERR_ARG;
    if (!on_device(c->device)) return P8_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return P8_ERR_CUDA;
    c->peer[q] = static_cast<unsigned long long *>(p);
    c->mapped[q] = true;
    return P8_OK;
}

p8_status p8_tp_comm_set_peer(p8_tp_comm *c, int q, void *dev_buffer) {
    if (!valid_comm(c) || q < 0 || q >= c->world || q == c->rank || c->peer[q] || !dev_buffer || ((uintptr_t)dev_buffer & 7))
        return P8_ERR_ARG;
    c->peer[q] = static_cast<unsigned long long *>(dev_buffer);
    return P8_OK;
}

p8_status p8_tp_comm_buffer(const p8_tp_comm *c, void **dev_buffer, size_t *nbytes) {
    if (!valid_comm(c)) return P8_ERR_ARG;
    if (dev_buffer) *dev_buffer = c->buf;
    if (nbytes) *nbytes = buf_bytes(c);
    return P8_OK;
}

p8_status p8_tp_comm_epoch(const p8_tp_comm *c, uint32_t *epoch) {
    if (!valid_comm(c) || !epoch) return P8_ERR_ARG;
    return cudaMemcpy(epoch, c->epoch, sizeof(uint32_t), cudaMemcpyDeviceToHost) == cudaSuccess ? P8_OK : P8_ERR_CUDA;
}

p8_status p8_tp_comm_reset(p8_tp_comm *c, void *stream) {
    if (!valid_comm(c)) return P8_ERR_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(c->buf, 0, buf_bytes(c), s) != cudaSuccess ||
        cudaMemsetAsync(c->epoch, 0, sizeof(unsigned int), s) != cudaSuccess)
        return P8_ERR_CUDA;
    return P8_OK;
}

p8_status p8_tp_gemv_allreduce(const p8_tensor *t, const float *x, float *y, p8_tp_comm *c, void *workspace,
                               size_t workspace_bytes, void *stream) {
    if (!t || t->magic != kTensorMagic) return P8_ERR_NOT_PREPARED;
    if (!valid_comm(c) || !x || !y || ((uintptr_t)x & 15)) return P8_ERR_ARG;
    if (t->rows > c->cap || t->device != c->device || !on_device(c->device)) return P8_ERR_ARG;
    TpExchange tp;
    memset(&tp, 0, sizeof(tp));
    for (int q = 0; q < c->world; ++q) {
        if (!c->peer[q]) return P8_ERR_ARG;  // every peer's buffer must be attached
        tp.peer[q] = c->peer[q];
    }
    tp.epoch = c->epoch;
    tp.cap = c->cap;
    tp.timeout_ns = c->timeout_ns;
    tp.tag_rows = (uint32_t)t->rows >> 5;
    tp.rank = c->rank;
    tp.world = c->world;
    return launch_gemv_tp(t, x, y, tp, c->epoch, workspace, workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"
