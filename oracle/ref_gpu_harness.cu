/*
 * ref_gpu_harness.cu -- TEST INFRASTRUCTURE ONLY (the same-box comparison arm; never part of the product path).
 *
 * Launches the reference's OWN batch-1 GEMV kernels on this GPU: k_vr_qx_real (CU:3003-3018: x' = FWHT256(x sgn / c)/16,
 * int8 per 128 columns) and k_vr<RL, V, 8, 108> (CU:2662-2727: table decode + dp4a LUT dot, atomicAdd into y[prm[r]],
 * clamp delta fused at entry). oracle/build_ref.py cuts their source from the patch text (vr49.cuh, a new file of
 * patches/llama_cuda_vs_7ac59a6.patch) into oracle/_ref/vr49_kvr.cuh and oracle/_ref/vr49_qx.cuh, never committed.
 *
 * The host side restates what the reference's ggml glue does for one native Pingala-8 tensor:
 *   refgpu_set_tables = vr_prepare_native (CU:3045-3102): codebook A (words 0-255), B (256-511) and coset c (word 512)
 *                       into c_vrA / c_vrB / c_vrcs; the slot's Hadamard signs as floats into c_vr_sgn and g_vr_sgn_d.
 *   refgpu_gemv       = vr_mul_mat_vec (CU:3177-3232) in native ("real") mode: k_vr_qx_real into an int8 x' and its
 *                       per-128 scales, y = 0, then k_vr with prm, c16 and the f32 clamp delta at the trailer's offsets
 *                       (vrn_offsets, CU:36-43). RL (GGML_VR_RL, default 1) and V (GGML_VRC_V: 5 as shipped, 7 the
 *                       code default) are arguments; NWP = 8 and NS = 108 as the native file fixes them.
 */
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <map>
#include <mutex>

typedef uint32_t u32;
// the cut-out source uses these two names only inside vr_init_sgn, the timing-only random fill, which this harness
// never calls (the signs come from the slot, as in the native prepare)
#define CUDA_CHECK(call) do { const cudaError_t e_ = (call); if (e_ != cudaSuccess) { fprintf(stderr, "%s\n", cudaGetErrorString(e_)); abort(); } } while (0)
static uint64_t f44_sm64(uint64_t &s) { return ++s; }

#include "ggml-vr-native.h"
#include "vr49_kvr.cuh"
#include "vr49_qx.cuh"

extern "C" {

int refgpu_set_tables(const uint32_t *hdr513, const int8_t *signs) {
    float sg[256];
    for (int i = 0; i < 256; ++i) sg[i] = (float)signs[i];
    cudaError_t e = cudaMemcpyToSymbol(c_vrA, hdr513, 1024);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_vrB, hdr513 + 256, 1024);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_vrcs, hdr513 + 512, 4);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_vr_sgn, sg, sizeof(sg));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_vr_sgn_d, sg, sizeof(sg));
    return (int)e;
}

/* one GEMV; xq (K bytes, 8-byte aligned) and xs (K/128 floats) are the caller's scratch. Returns 0, a CUDA error code,
   or -1 for arguments the kernels do not cover (shape, alignment, variant). */
int refgpu_gemv(const unsigned char *slot, size_t nbytes, int rows, int K, int nd, const float *x, float *y, int8_t *xq,
                float *xs, int V, int RL, void *stream) {
    if (rows <= 0 || K <= 0 || rows % 32 || K % 256 || rows >= 32768 || nd < 0 || ((uintptr_t)slot & 15) ||
        ((uintptr_t)x & 15) || ((uintptr_t)xq & 7) || (V != 5 && V != 7) || (RL != 1 && RL != 2 && RL != 4))
        return -1;
    const int nb = K / 256, ng = rows / 32;
    const size_t nt = (size_t)nb * ng;
    const size_t offM = 2064, offS = offM + 4 * nt, offD = (offS + 64 * nt + 15) & ~(size_t)15;
    size_t offE, offC, offP, offQ, offSG, offT;
    if (nbytes < vrn_need(offD, rows, K, nd)) return -1;
    vrn_offsets(nbytes, rows, K, nd, &offE, &offC, &offP, &offQ, &offSG, &offT);
    cudaStream_t st = (cudaStream_t)stream;

    k_vr_qx_real<<<(K / 256 + 7) / 8, 256, 0, st>>>(x, (const half *)(slot + offC), xq, xs, K);
    cudaError_t e = cudaMemsetAsync(y, 0, (size_t)rows * sizeof(float), st);
    if (e != cudaSuccess) return (int)e;

    vr_args a;
    a.D = (const u32 *)(slot + offD);
    a.M = (const u32 *)(slot + offM);
    a.S = (const half *)(slot + offS);
    a.X = xq;
    a.XS = xs;
    a.y = y;
    a.rows = rows;
    a.nsl = K / 128;
    a.nb = nb;
    a.ng = ng;
    a.prm = (const short *)(slot + offP);
    a.drow = (const unsigned short *)(slot + offE);
    a.dcol = (const unsigned short *)(slot + offE + 2 * (size_t)nd);
    a.dval = (const float *)(slot + offE + 4 * (size_t)nd);
    a.nd = nd;
    a.xraw = x;
    const dim3 grid(((ng + 8 * RL - 1) / (8 * RL)) * a.nsl);
    if (V == 5) {
        if (RL == 1) k_vr<1, 5, 8, 108><<<grid, 256, 0, st>>>(a);
        else if (RL == 2) k_vr<2, 5, 8, 108><<<grid, 256, 0, st>>>(a);
        else k_vr<4, 5, 8, 108><<<grid, 256, 0, st>>>(a);
    } else {
        if (RL == 1) k_vr<1, 7, 8, 108><<<grid, 256, 0, st>>>(a);
        else if (RL == 2) k_vr<2, 7, 8, 108><<<grid, 256, 0, st>>>(a);
        else k_vr<4, 7, 8, 108><<<grid, 256, 0, st>>>(a);
    }
    return (int)cudaGetLastError();
}

const char *refgpu_error_string(int e) { return e < 0 ? "bad arguments" : cudaGetErrorString((cudaError_t)e); }

}  // extern "C"
