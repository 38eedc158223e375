// p8_device.cuh -- device helpers shared by the Pingala-8 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "p8_format.h"

namespace p8 {

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ---------------------------------------------------------------------------------------------------------------
// FWHT-256 over one warp: lane l holds elements 8l..8l+7. Index bits 0-2 live in registers, bits 3-7 across lanes.
// Every butterfly is (a + b, a - b) of the same operands in the same stage order (h = 1, 2, ..., 128) as the scalar
// reference (vrc_fwht256, CP:536-540), so the result is bit-identical; the final scale by 1/16 is separate.
__device__ __forceinline__ void fwht256_warp(float (&v)[8], int lane) {
#pragma unroll
    for (int h = 1; h < 8; h <<= 1) {
#pragma unroll
        for (int m = 0; m < 8; ++m)
            if (!(m & h)) {
                const float a = v[m], b = v[m | h];
                v[m] = __fadd_rn(a, b);
                v[m | h] = __fsub_rn(a, b);
            }
    }
#pragma unroll
    for (int msk = 1; msk < 32; msk <<= 1) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const float p = __shfl_xor_sync(0xffffffffu, v[m], msk);
            v[m] = (lane & msk) ? __fsub_rn(p, v[m]) : __fadd_rn(v[m], p);
        }
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) v[m] = __fmul_rn(v[m], 0.0625f);
}

// W-bit field at bit W*k of the word array starting at word wb (LSB first, may straddle two words).
template <int NWA>
__device__ __forceinline__ uint32_t field(const uint32_t (&w)[NWA], int wb, int W, int k) {
    const int pos = W * k, wi = wb + (pos >> 5), bb = pos & 31;
    uint32_t v = w[wi] >> bb;
    if (bb + W > 32) v |= w[wi + 1] << (32 - bb);
    return v & ((1u << W) - 1u);
}

// z bits of one lane-slice in STEP order (bit k = stage-1 MSB of the chunk at step k).
template <int C, int NWA>
__device__ __forceinline__ uint32_t zbits(const uint32_t (&w)[NWA]) {
    if (W1(C) == 8) {
        uint32_t pm = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) pm |= (((w[i] & 0x80808080u) * 0x00204081u) >> 28) << (4 * i);
        return pm;
    }
    return w[0];
}

// stage-1 index at step k (whole byte for W1 = 8; MSB word + (W1-1)-bit fields otherwise)
template <int C, int NWA>
__device__ __forceinline__ uint32_t f1_at(const uint32_t (&w)[NWA], int k) {
    if (W1(C) == 8) return field(w, 0, 8, k);
    return field(w, 1, W1(C) - 1, k) | (((w[0] >> k) & 1u) << (W1(C) - 1));
}

// Exact integer weights of the chunk at step k (chunk t = (j + k) & 31 of lane j) from the lane's words (coset folded
// in, no int8 wrap: the tables are checked at prepare time). A is a shared-memory copy of the codebook.
template <int C, int NWA>
__device__ __forceinline__ void chunk_ints_step(const uint32_t (&w)[NWA], const uint32_t *A, uint32_t cs, uint32_t H, int k, int t,
                                                int (&v)[4]) {
    const int h = (H >> t) & 1u;
    const uint32_t a1 = A[f1_at<C>(w, k)];
    const uint32_t a2 = W2(C) ? A[field(w, W1(C), W2(C) ? W2(C) : 1, k)] : 0u;
    const uint32_t a3 = W3(C) ? A[field(w, W1(C) + W2(C), 8, k)] : 0u;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int ce = h ? (int)(int8_t)(cs >> (8 * e)) : 0;
        int x = ((int)(int8_t)(a1 >> (8 * e)) + ce) * (1 << SH1(C));
        if (W2(C)) x += ((int)(int8_t)(a2 >> (8 * e)) + ce) * (1 << SH2(C));
        if (W3(C)) x += (int)(int8_t)(a3 >> (8 * e)) + ce;
        v[e] = x;
    }
}
// the same for chunk t of lane j (step k = (t - j) & 31)
template <int C, int NWA>
__device__ __forceinline__ void chunk_ints(const uint32_t (&w)[NWA], const uint32_t *A, uint32_t cs, uint32_t H, int j, int t,
                                           int (&v)[4]) {
    chunk_ints_step<C>(w, A, cs, H, (t - j) & 31, t, v);
}

// lane words of half-slice hs: word i of lane j at D[off + hs*NW*32 + (i>>1)*64 + 2j + (i&1)]
template <int C, int NWA>
__device__ __forceinline__ void load_lane_words(const uint32_t *p0, int hs, int j, uint32_t (&w)[NWA]) {
    constexpr int nw = NW(C);
    const uint2 *q = reinterpret_cast<const uint2 *>(p0) + (size_t)hs * nw * 16 + j;
#pragma unroll
    for (int i = 0; i < nw / 2; ++i) {
        const uint2 u = __ldg(q + i * 32);
        w[2 * i] = u.x;
        w[2 * i + 1] = u.y;
    }
#pragma unroll
    for (int i = nw; i < NWA; ++i) w[i] = 0;
}

// ---------------------------------------------------------------------------------------------------------------
// mbarrier + bulk-copy helpers (cp.async.bulk, no multicast)
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after max_iter polls (each try_wait itself suspends for a short, hardware-bounded time).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase, uint32_t max_iter) {
    for (uint32_t i = 0; i < max_iter; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}
// global -> shared bulk copy completing on an mbarrier (16-byte aligned addresses, size a multiple of 16)
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

}  // namespace p8
