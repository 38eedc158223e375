// p8_api.cu -- C ABI entry points: tensor preparation, registry and the compute calls.
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <mutex>
#include <vector>

#include "p8_internal.h"

using namespace p8;

namespace p8 {
unsigned int read_and_clear_device_error();
}

namespace {
std::mutex g_mu;
std::map<const void *, p8_tensor *> g_reg;  // slot pointer -> prepared tensor (as the reference's g_vr registry, CU:2548)

bool valid(const p8_tensor *t) { return t && t->magic == kTensorMagic; }

template <typename T>
cudaError_t dmalloc_copy(T **dst, const T *src, size_t count) {
    *dst = nullptr;
    if (!count) return cudaSuccess;
    cudaError_t e = cudaMalloc((void **)dst, sizeof(T) * count);
    if (e != cudaSuccess) return e;
    return cudaMemcpy(*dst, src, sizeof(T) * count, cudaMemcpyHostToDevice);
}

void free_tensor(p8_tensor *t) {
    if (!t) return;
    cudaFree(t->ic);
    cudaFree(t->cp);
    cudaFree(t->cc);
    cudaFree(t->cv);
    cudaFree(t->rsc);
    t->magic = 0;
    delete t;
}
}  // namespace

extern "C" {

p8_status p8_prepare(const void *dev_slot, size_t nbytes, int64_t K, int64_t rows, void *stream, p8_tensor **out) {
    if (!dev_slot || !out || ((uintptr_t)dev_slot & 15)) return P8_ERR_ARG;  // kernels stream the slot in 16-byte units
    *out = nullptr;
    p8_status st = check_shape(K, rows);
    if (st) return st;
    const size_t nb = (size_t)K / 256, ng = (size_t)rows / 32, nt = nb * ng;
    if (nbytes < 4096 || nbytes < offD(nt)) return P8_ERR_TRAILER;
    cudaStream_t s = (cudaStream_t)stream;
    const uint8_t *base = (const uint8_t *)dev_slot;
    // device -> host reads of the small parts (as vr_prepare_native, CU:3050-3053)
    Trailer tr;
    std::vector<uint8_t> hdr(kHdrBytes);
    std::vector<uint32_t> M(nt);
    if (cudaMemcpyAsync(&tr, base + nbytes - 32, 32, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyAsync(hdr.data(), base, kHdrBytes, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyAsync(M.data(), base + kHdrBytes, 4 * nt, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return P8_ERR_CUDA;
    if (tr.magic0 != kMagic0 || tr.magic1 != kMagic1 || tr.rows != (uint32_t)rows || tr.K != (uint32_t)K || tr.ns != kNS)
        return P8_ERR_TRAILER;
    if (tr.nd > nbytes) return P8_ERR_DELTA;
    const SideOffsets so = side_offsets(nbytes, (size_t)rows, (size_t)K, tr.nd);
    if (so.E >= nbytes || so.E < offD(nt)) return P8_ERR_PAYLOAD;
    std::vector<uint8_t> side(nbytes - so.E);  // E .. end: delta, c16, prm, pinv, signs, trailer
    if (cudaMemcpyAsync(side.data(), base + so.E, side.size(), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return P8_ERR_CUDA;
    auto at = [&](size_t off) { return side.data() + (off - so.E); };
    SlotView v;
    v.n = nbytes;
    v.hdr = hdr.data();
    v.M = M.data();
    v.tr = &tr;
    v.sg = (const int8_t *)at(so.SG);
    v.prm = (const int16_t *)at(so.P);
    v.pinv = (const int16_t *)at(so.Q);
    v.drow = (const uint16_t *)at(so.E);
    v.dcol = v.drow + tr.nd;
    v.c16 = (const uint16_t *)at(so.C);
    size_t kb = 0;
    uint32_t cm = 0;
    uint64_t hist[8];
    st = validate_slot(v, K, rows, &kb, &cm, hist);
    if (st) return st;
    p8_tensor *t = new p8_tensor();
    t->magic = kTensorMagic;
    cudaGetDevice(&t->device);
    t->slot = base; t->nbytes = nbytes; t->kbytes = kb; t->nt = nt;
    t->rows = (int)rows; t->K = (int)K; t->nb = (int)nb; t->ng = (int)ng; t->nsl = (int)(K / 128); t->nd = (int)tr.nd;
    t->A = (const uint32_t *)base;
    t->M = (const uint32_t *)(base + kHdrBytes);
    t->S = (const uint16_t *)(base + offS(nt));
    t->D = (const uint32_t *)(base + offD(nt));
    t->c16 = (const uint16_t *)(base + so.C);
    t->prm = (const int16_t *)(base + so.P);
    t->pinv = (const int16_t *)(base + so.Q);
    memcpy(&t->cs, hdr.data() + 2048, 4);
    t->class_mask = cm;
    {   // uniform layout: one class everywhere, payloads back to back in tile order (single-class writers, VR3)
        const int c0 = (int)(M[0] >> 29);
        bool uni = c0 != 0;
        for (size_t i = 0; uni && i < nt; ++i) uni = M[i] == ((uint32_t)(i * 64 * NW(c0)) | ((uint32_t)c0 << 29));
        t->uniform_class = uni ? c0 : 0;
    }
    memcpy(t->hist, hist, sizeof(hist));
    t->A_host.assign((const uint32_t *)hdr.data(), (const uint32_t *)hdr.data() + 256);
    // sgn / c per column, float division as vrc_init (CP:264)
    std::vector<float> ic((size_t)K);
    for (int64_t k = 0; k < K; ++k) ic[(size_t)k] = (float)v.sg[k & 255] / half_bits_to_float(v.c16[k]);
    // clamp-delta CSR by original row, entries in slot order within a row (CP:266-273)
    std::vector<int> cp((size_t)rows + 1, 0);
    std::vector<uint16_t> cc(tr.nd);
    std::vector<float> cv(tr.nd);
    const float *dval = (const float *)at(so.E + 4 * (size_t)tr.nd);
    memset(t->delta_blocks, 0, sizeof(t->delta_blocks));
    for (uint32_t e = 0; e < tr.nd; ++e) {
        cp[v.drow[e] + 1]++;
        t->delta_blocks[(v.drow[e] >> 8) >> 5] |= 1u << ((v.drow[e] >> 8) & 31);
    }
    for (int64_t r = 0; r < rows; ++r) cp[(size_t)r + 1] += cp[(size_t)r];
    std::vector<int> fill(cp.begin(), cp.end() - 1);
    for (uint32_t e = 0; e < tr.nd; ++e) {
        const int q = fill[v.drow[e]]++;
        cc[(size_t)q] = v.dcol[e];
        memcpy(&cv[(size_t)q], dval + e, 4);
    }
    {  // content hash of everything the prepared activation depends on (as the reference's c hash, CP:261)
        uint64_t h = 1469598103934665603ull;
        auto mix = [&h](const void *p, size_t n) {
            const uint8_t *b = (const uint8_t *)p;
            for (size_t i = 0; i < n; ++i) { h ^= b[i]; h *= 1099511628211ull; }
        };
        mix(ic.data(), 4 * ic.size());
        mix(hdr.data(), 1024);
        mix(hdr.data() + 2048, 4);
        t->act_hash = h;
    }
    if (dmalloc_copy(&t->ic, ic.data(), ic.size()) != cudaSuccess || dmalloc_copy(&t->cp, cp.data(), cp.size()) != cudaSuccess ||
        dmalloc_copy(&t->cc, cc.data(), cc.size()) != cudaSuccess || dmalloc_copy(&t->cv, cv.data(), cv.size()) != cudaSuccess) {
        free_tensor(t);
        return P8_ERR_CUDA;
    }
    if ((st = gemm_prepare(t, s)) != P8_OK) {
        free_tensor(t);
        return st;
    }
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_reg.find(dev_slot);
        if (it != g_reg.end()) {  // re-prepare of the same slot replaces the old handle's registration
            it->second = t;
        } else {
            g_reg[dev_slot] = t;
        }
    }
    *out = t;
    return P8_OK;
}

p8_status p8_release(p8_tensor *t) {
    if (!valid(t)) return P8_ERR_NOT_PREPARED;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_reg.find(t->slot);
        if (it != g_reg.end() && it->second == t) g_reg.erase(it);
    }
    free_tensor(t);
    return P8_OK;
}

int p8_active(const void *dev_slot) {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_reg.count(dev_slot) ? 1 : 0;
}

p8_status p8_tensor_info(const p8_tensor *t, int64_t *rows, int64_t *K, int64_t *nd, uint64_t *class_hist) {
    if (!valid(t)) return P8_ERR_NOT_PREPARED;
    if (rows) *rows = t->rows;
    if (K) *K = t->K;
    if (nd) *nd = t->nd;
    if (class_hist) memcpy(class_hist, t->hist, sizeof(t->hist));
    return P8_OK;
}

size_t p8_workspace_size(const p8_tensor *t, int64_t ncols) {
    if (!valid(t) || ncols <= 0) return 0;
    size_t w = gemv_workspace(t, ncols);
    if (gemm_supported(t, ncols)) {
        const size_t g = gemm_workspace(t, ncols);
        if (g > w) w = g;
    }
    return w;
}

p8_status p8_mul_mat_vec(const p8_tensor *t, const float *x, float *y, void *workspace, size_t workspace_bytes, void *stream) {
    if (!valid(t)) return P8_ERR_NOT_PREPARED;
    if (!x || !y || ((uintptr_t)x & 15)) return P8_ERR_ARG;
    return launch_gemv(t, x, 1, t->K, y, t->rows, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t p8_workspace_size_group(const p8_tensor *const *ts, int n, int64_t ncols) {
    if (!ts || n < 1 || n > 4 || ncols <= 0) return 0;
    for (int i = 0; i < n; ++i)
        if (!valid(ts[i])) return 0;
    return gemv_group_workspace(ts, n, ncols);
}

p8_status p8_mul_mat_vec_group(const p8_tensor *const *ts, int n, const float *x, float *const *ys, void *workspace,
                               size_t workspace_bytes, void *stream) {
    if (!ts || !ys || n < 1 || n > 4 || !x || ((uintptr_t)x & 15)) return P8_ERR_ARG;
    int64_t ld[4];
    for (int i = 0; i < n; ++i) {
        if (!valid(ts[i])) return P8_ERR_NOT_PREPARED;
        if (!ys[i]) return P8_ERR_ARG;
        ld[i] = ts[i]->rows;
    }
    return launch_gemv_group(ts, n, x, 1, ts[0]->K, ys, ld, workspace, workspace_bytes, (cudaStream_t)stream);
}

p8_status p8_mul_mat_vec_group_ex(const p8_tensor *const *ts, int n, const float *x, const p8_prologue *pro, float *const *ys,
                                  void *workspace, size_t workspace_bytes, void *stream) {
    if (!ts || !ys || n < 1 || n > 4 || !x || ((uintptr_t)x & 15)) return P8_ERR_ARG;
    for (int i = 0; i < n; ++i) {
        if (!valid(ts[i])) return P8_ERR_NOT_PREPARED;
        if (!ys[i]) return P8_ERR_ARG;
    }
    if (pro) {
        if (pro->kind == P8_PROLOGUE_RMSNORM) {
            if (!pro->w || ((uintptr_t)pro->w & 15) || !(pro->eps >= 0.f)) return P8_ERR_ARG;
        } else if (pro->kind == P8_PROLOGUE_SWIGLU) {
            if (!pro->x2 || ((uintptr_t)pro->x2 & 15)) return P8_ERR_ARG;
        } else if (pro->kind != P8_PROLOGUE_NONE) {
            return P8_ERR_ARG;
        }
    }
    return launch_gemv_group_pro(ts, n, x, pro, ys, workspace, workspace_bytes, (cudaStream_t)stream);
}

p8_status p8_mul_mat(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, float *Y, int64_t ldy, void *workspace,
                     size_t workspace_bytes, void *stream) {
    if (!valid(t)) return P8_ERR_NOT_PREPARED;
    if (!X || !Y || ncols <= 0 || ldx < t->K || ldy < t->rows || ((uintptr_t)X & 15) || (ldx & 3)) return P8_ERR_ARG;
    if (gemm_supported(t, ncols)) return launch_gemm(t, X, ncols, ldx, Y, ldy, workspace, workspace_bytes, (cudaStream_t)stream);
    return launch_gemv(t, X, ncols, ldx, Y, ldy, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t p8_workspace_size_ex(const p8_tensor *t, int64_t ncols, int kind) {
    if (!valid(t) || ncols <= 0) return 0;
    size_t w = gemv_workspace(t, ncols);
    if (gemm_supported(t, ncols)) {
        const size_t g = gemm_workspace(t, ncols, kind != P8_PROLOGUE_NONE);
        if (g > w) w = g;
    }
    return w;
}

p8_status p8_mul_mat_ex(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, const p8_prologue *pro, float *Y,
                        int64_t ldy, void *workspace, size_t workspace_bytes, void *stream) {
    if (!valid(t)) return P8_ERR_NOT_PREPARED;
    if (!X || !Y || ncols <= 0 || ldx < t->K || ldy < t->rows || ((uintptr_t)X & 15) || (ldx & 3)) return P8_ERR_ARG;
    if (pro) {
        if (pro->kind == P8_PROLOGUE_RMSNORM) {
            if (!pro->w || ((uintptr_t)pro->w & 15) || !(pro->eps >= 0.f)) return P8_ERR_ARG;
        } else if (pro->kind == P8_PROLOGUE_SWIGLU) {
            if (!pro->x2 || ((uintptr_t)pro->x2 & 15)) return P8_ERR_ARG;
        } else if (pro->kind != P8_PROLOGUE_NONE) {
            return P8_ERR_ARG;
        }
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (gemm_supported(t, ncols)) return launch_gemm(t, X, ncols, ldx, Y, ldy, workspace, workspace_bytes, s, pro);
    // below the GEMM's column count: the batch-1 GEMV, two columns per call where it can
    return launch_gemv_cols(&t, 1, X, ncols, ldx, pro, &Y, &ldy, workspace, workspace_bytes, s);
}

size_t p8_workspace_size_group_ex(const p8_tensor *const *ts, int n, int64_t ncols, int kind) {
    if (!ts || n < 1 || n > 4 || ncols <= 0) return 0;
    for (int i = 0; i < n; ++i)
        if (!valid(ts[i])) return 0;
    size_t w = gemv_group_workspace(ts, n, ncols);
    int nsup = 0;
    for (int i = 0; i < n; ++i) {
        const size_t g = gemv_workspace(ts[i], ncols);
        if (g > w) w = g;
        if (gemm_supported(ts[i], ncols)) {
            ++nsup;
            const size_t h = gemm_workspace(ts[i], ncols, kind != P8_PROLOGUE_NONE);
            if (h > w) w = h;
        }
    }
    if (nsup == n) {
        const size_t h = gemm_group_workspace(ts, n, ncols, kind != P8_PROLOGUE_NONE);
        if (h > w) w = h;
    }
    return w;
}

p8_status p8_mul_mat_group(const p8_tensor *const *ts, int n, const float *X, int64_t ncols, int64_t ldx, const p8_prologue *pro,
                           float *const *Ys, const int64_t *ldys, void *workspace, size_t workspace_bytes, void *stream) {
    if (!ts || !Ys || !ldys || n < 1 || n > 4) return P8_ERR_ARG;
    for (int i = 0; i < n; ++i)
        if (!valid(ts[i])) return P8_ERR_NOT_PREPARED;
    if (!X || ncols <= 0 || ldx < ts[0]->K || ((uintptr_t)X & 15) || (ldx & 3)) return P8_ERR_ARG;
    int nsup = 0;
    for (int i = 0; i < n; ++i) {
        if (!Ys[i] || ldys[i] < ts[i]->rows) return P8_ERR_ARG;
        if (ts[i]->K != ts[0]->K || ts[i]->act_hash != ts[0]->act_hash) return P8_ERR_ARG;
        nsup += gemm_supported(ts[i], ncols) ? 1 : 0;
    }
    if (pro) {
        if (pro->kind == P8_PROLOGUE_RMSNORM) {
            if (!pro->w || ((uintptr_t)pro->w & 15) || !(pro->eps >= 0.f)) return P8_ERR_ARG;
        } else if (pro->kind == P8_PROLOGUE_SWIGLU) {
            if (!pro->x2 || ((uintptr_t)pro->x2 & 15)) return P8_ERR_ARG;
        } else if (pro->kind != P8_PROLOGUE_NONE) {
            return P8_ERR_ARG;
        }
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (nsup == n) return launch_gemm_group(ts, n, X, ncols, ldx, Ys, ldys, workspace, workspace_bytes, s, pro);
    if (nsup == 0)  // below the GEMM's column count: the grouped batch-1 GEMV, two columns per call where it can
        return launch_gemv_cols(ts, n, X, ncols, ldx, pro, Ys, ldys, workspace, workspace_bytes, s);
    for (int i = 0; i < n; ++i) {  // tensors on different paths: one call each
        const p8_status st = p8_mul_mat_ex(ts[i], X, ncols, ldx, pro, Ys[i], ldys[i], workspace, workspace_bytes, stream);
        if (st) return st;
    }
    return P8_OK;
}

p8_status p8_get_rows(const p8_tensor *t, const int32_t *ids, int64_t n, float *out, int64_t ldo, void *stream) {
    if (!valid(t)) return P8_ERR_NOT_PREPARED;
    if (n < 0 || (n && (!ids || !out)) || ldo < t->K || ((uintptr_t)out & 15) || (ldo & 3)) return P8_ERR_ARG;
    return launch_get_rows(t, ids, n, out, ldo, (cudaStream_t)stream) == cudaSuccess ? P8_OK : P8_ERR_CUDA;
}

p8_status p8_dequant_f32(const p8_tensor *t, float *out, void *stream) {
    if (!valid(t)) return P8_ERR_NOT_PREPARED;
    if (!out || ((uintptr_t)out & 15)) return P8_ERR_ARG;
    return launch_dequant(t, out, (cudaStream_t)stream) == cudaSuccess ? P8_OK : P8_ERR_CUDA;
}

p8_status p8_decode_int(const p8_tensor *t, int16_t *out, void *stream) {
    if (!valid(t)) return P8_ERR_NOT_PREPARED;
    if (!out) return P8_ERR_ARG;
    return launch_decode_int(t, out, (cudaStream_t)stream) == cudaSuccess ? P8_OK : P8_ERR_CUDA;
}

p8_status p8_chain_create(const p8_chain_step *steps, int nsteps, p8_chain **out) { return chain_create(steps, nsteps, out); }
size_t p8_chain_workspace_size(const p8_chain *c) { return chain_workspace(c); }
p8_status p8_chain_run(const p8_chain *c, void *workspace, size_t workspace_bytes, void *stream) {
    static const int pf = [] {  // units per warp asked of L2 ahead of the warp's current unit (P8_CHAIN_PF; tuning knob)
        const char *e = getenv("P8_CHAIN_PF");
        return e ? atoi(e) : 2;
    }();
    return chain_run(c, workspace, workspace_bytes, (cudaStream_t)stream, pf);
}
p8_status p8_chain_destroy(p8_chain *c) { return chain_destroy(c); }
p8_status p8_chain_trace(p8_chain *c, uint64_t *dev_buf, size_t words) {
    return chain_trace(c, reinterpret_cast<unsigned long long *>(dev_buf), words);
}

/* 1 if a kernel since the last call gave up on a bounded wait (results of that launch are invalid). Synchronous. */
int p8_device_error(void) { return (int)read_and_clear_device_error(); }

const char *p8_build_info(void) { return "pingala8_b200 sm_100a (tcgen05/TMA), C ABI v1"; }

}  // extern "C"
