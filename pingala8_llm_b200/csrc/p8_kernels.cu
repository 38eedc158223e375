// p8_kernels.cu -- Pingala-8 decode / dequant / get_rows and the batch-1 table GEMV for sm_100a.
//
// One translation unit holds every kernel of the library (the tcgen05 GEMM is included from p8_gemm.cuh).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "p8_device.cuh"
#include "p8_internal.h"

namespace p8 {

// device-side error word: bit 0 = a bounded wait timed out (that launch's results are invalid)
__device__ unsigned int g_p8_device_error = 0;

// ================================================================================================================
// 1. Tile decode and f32 dequant (bit-identical to vrc_decode_tile_int / vrc_dequant_f32, CP:992-1027)
// ================================================================================================================
struct TileArgs {
    const uint32_t *A, *M, *D;
    const uint16_t *S;
    const int16_t *prm;
    const float *ic;
    const int *cp;
    const uint16_t *cc;
    const float *cv;
    uint32_t cs;
    int rows, K, nb;
};

constexpr int kXiStride = 256 + 8;  // int16 per decoded row in shared memory

// lane j decodes row j of half-slice hs of tile (g, b) into xi[j][hs*128 + 4t + e]
template <int C>
__device__ __forceinline__ void decode_lane_to_smem(const TileArgs &a, const uint32_t *p0, const uint32_t *A_s, int hs, int j,
                                                    int16_t *xi) {
    uint32_t w[25];
    load_lane_words<C>(p0, hs, j, w);
    const uint32_t H = pingala8_h(__funnelshift_l(zbits<C>(w), zbits<C>(w), j));
#pragma unroll
    for (int t = 0; t < 32; ++t) {
        int v[4];
        chunk_ints<C>(w, A_s, a.cs, H, j, t, v);
        int16_t *o = xi + j * kXiStride + hs * 128 + 4 * t;
        o[0] = (int16_t)v[0]; o[1] = (int16_t)v[1]; o[2] = (int16_t)v[2]; o[3] = (int16_t)v[3];
    }
}

__device__ __forceinline__ void decode_tile_to_smem(const TileArgs &a, int g, int b, const uint32_t *A_s, int16_t *xi) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t mt = a.M[(size_t)g * a.nb + b];
    const int c = (int)(mt >> 29);
    const uint32_t *p0 = a.D + (mt & 0x1FFFFFFFu);
    if (warp < 2) {
        const int hs = warp;
        switch (c) {
            case 0:
                for (int i = 0; i < 128; ++i) xi[lane * kXiStride + hs * 128 + i] = 0;
                break;
            case 1: decode_lane_to_smem<1>(a, p0, A_s, hs, lane, xi); break;
            case 2: decode_lane_to_smem<2>(a, p0, A_s, hs, lane, xi); break;
            case 3: decode_lane_to_smem<3>(a, p0, A_s, hs, lane, xi); break;
            case 4: decode_lane_to_smem<4>(a, p0, A_s, hs, lane, xi); break;
            case 5: decode_lane_to_smem<5>(a, p0, A_s, hs, lane, xi); break;
            case 6: decode_lane_to_smem<6>(a, p0, A_s, hs, lane, xi); break;
            default: decode_lane_to_smem<7>(a, p0, A_s, hs, lane, xi); break;
        }
    }
}

// grid (nb, ng), 256 threads: decoded ints of tile (g, b) -> out[r][K] (sorted rows)
__global__ void __launch_bounds__(256) k_decode_int(TileArgs a, int16_t *out) {
    __shared__ uint32_t A_s[256];
    __shared__ __align__(16) int16_t xi[32 * kXiStride];
    const int b = blockIdx.x, g = blockIdx.y;
    A_s[threadIdx.x] = a.A[threadIdx.x];
    __syncthreads();
    decode_tile_to_smem(a, g, b, A_s, xi);
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * 256; i += 256) {
        const int j = i >> 8, col = i & 255;
        out[(size_t)(g * 32 + j) * a.K + b * 256 + col] = xi[j * kXiStride + col];
    }
}

// W[ro][b*256 + i] = (FWHT(int * S)[i] / 16) * ic + delta, per warp and row: the reference order of float operations
__device__ __forceinline__ void dequant_row_block(const TileArgs &a, int r, int b, const int16_t *ints, float *dst) {
    const int lane = threadIdx.x & 31;
    const float sc = h2f(a.S[(size_t)b * a.rows + r]);
    float v[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) v[m] = __fmul_rn((float)ints[8 * lane + m], sc);
    fwht256_warp(v, lane);
    const float4 i0 = *reinterpret_cast<const float4 *>(a.ic + b * 256 + 8 * lane);
    const float4 i1 = *reinterpret_cast<const float4 *>(a.ic + b * 256 + 8 * lane + 4);
    const float icv[8] = {i0.x, i0.y, i0.z, i0.w, i1.x, i1.y, i1.z, i1.w};
#pragma unroll
    for (int m = 0; m < 8; ++m) v[m] = __fmul_rn(v[m], icv[m]);
    const int ro = a.prm[r];
    for (int e = a.cp[ro]; e < a.cp[ro + 1]; ++e) {  // clamp delta of this row inside this block (CSR order)
        const int col = (int)a.cc[e] - b * 256 - 8 * lane;
#pragma unroll
        for (int m = 0; m < 8; ++m)
            if (col == m) v[m] = __fadd_rn(v[m], a.cv[e]);
    }
    float4 *o = reinterpret_cast<float4 *>(dst + 8 * lane);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// grid (nb, ng), 256 threads
__global__ void __launch_bounds__(256) k_dequant(TileArgs a, float *W) {
    __shared__ uint32_t A_s[256];
    __shared__ __align__(16) int16_t xi[32 * kXiStride];
    const int b = blockIdx.x, g = blockIdx.y, warp = threadIdx.x >> 5;
    A_s[threadIdx.x] = a.A[threadIdx.x];
    __syncthreads();
    decode_tile_to_smem(a, g, b, A_s, xi);
    __syncthreads();
    for (int j = warp; j < 32; j += 8) {
        const int r = g * 32 + j;
        dequant_row_block(a, r, b, xi + j * kXiStride, W + (size_t)a.prm[r] * a.K + b * 256);
    }
}

// get_rows: grid (n), 256 threads; warp w handles blocks b = w, w + 8, ... of row ids[i] (ORIGINAL row).
// Lane l needs chunks 2l', 2l'+1 (l' = l & 15) of half-slice l >> 4; it decodes them from the row's lane words.
template <int C>
__device__ __forceinline__ void row_chunk_ints(const TileArgs &a, const uint32_t *p0, const uint32_t *A_s, int j, int lane,
                                               int (&out)[8]) {
    uint32_t w[25];
    const int hs = lane >> 4;
    constexpr int nw = NW(C);
    const uint32_t *q = p0 + (size_t)hs * nw * 32 + 2 * j;
#pragma unroll
    for (int i = 0; i < nw; ++i) w[i] = __ldg(q + (i >> 1) * 64 + (i & 1));
#pragma unroll
    for (int i = nw; i < 25; ++i) w[i] = 0;
    const uint32_t H = pingala8_h(__funnelshift_l(zbits<C>(w), zbits<C>(w), j));
    const int t0 = 2 * (lane & 15);
    int v[4];
    chunk_ints<C>(w, A_s, a.cs, H, j, t0, v);
    out[0] = v[0]; out[1] = v[1]; out[2] = v[2]; out[3] = v[3];
    chunk_ints<C>(w, A_s, a.cs, H, j, t0 + 1, v);
    out[4] = v[0]; out[5] = v[1]; out[6] = v[2]; out[7] = v[3];
}

__global__ void __launch_bounds__(256) k_get_rows(TileArgs a, const int16_t *pinv, const int32_t *ids, float *out, int64_t ldo) {
    __shared__ uint32_t A_s[256];
    __shared__ __align__(16) int16_t xs[8][256];
    A_s[threadIdx.x] = a.A[threadIdx.x];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ro = ids[blockIdx.x];
    if (ro < 0 || ro >= a.rows) return;  // ids are range-checked on the host side of the C ABI as well
    const int r = pinv[ro], g = r >> 5, j = r & 31;
    for (int b = warp; b < a.nb; b += 8) {
        const uint32_t mt = a.M[(size_t)g * a.nb + b];
        const int c = (int)(mt >> 29);
        const uint32_t *p0 = a.D + (mt & 0x1FFFFFFFu);
        int v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        switch (c) {
            case 0: break;
            case 1: row_chunk_ints<1>(a, p0, A_s, j, lane, v); break;
            case 2: row_chunk_ints<2>(a, p0, A_s, j, lane, v); break;
            case 3: row_chunk_ints<3>(a, p0, A_s, j, lane, v); break;
            case 4: row_chunk_ints<4>(a, p0, A_s, j, lane, v); break;
            case 5: row_chunk_ints<5>(a, p0, A_s, j, lane, v); break;
            case 6: row_chunk_ints<6>(a, p0, A_s, j, lane, v); break;
            default: row_chunk_ints<7>(a, p0, A_s, j, lane, v); break;
        }
        // lanes hold natural positions 8l..8l+7 already: (l & 15) * 8 + 128 * (l >> 4) == 8l
#pragma unroll
        for (int m = 0; m < 8; ++m) xs[warp][8 * lane + m] = (int16_t)v[m];
        __syncwarp();
        dequant_row_block(a, r, b, xs[warp], out + (size_t)blockIdx.x * ldo + b * 256);
        __syncwarp();
    }
}

static TileArgs tile_args(const p8_tensor *t) {
    TileArgs a;
    a.A = t->A; a.M = t->M; a.D = t->D; a.S = t->S; a.prm = t->prm; a.ic = t->ic; a.cp = t->cp; a.cc = t->cc; a.cv = t->cv;
    a.cs = t->cs; a.rows = t->rows; a.K = t->K; a.nb = t->nb;
    return a;
}

cudaError_t launch_decode_int(const p8_tensor *t, int16_t *out, cudaStream_t st) {
    k_decode_int<<<dim3(t->nb, t->ng), 256, 0, st>>>(tile_args(t), out);
    return cudaGetLastError();
}
cudaError_t launch_dequant(const p8_tensor *t, float *out, cudaStream_t st) {
    k_dequant<<<dim3(t->nb, t->ng), 256, 0, st>>>(tile_args(t), out);
    return cudaGetLastError();
}
cudaError_t launch_get_rows(const p8_tensor *t, const int32_t *ids, int64_t n, float *out, int64_t ldo, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_get_rows<<<(unsigned)n, 256, 0, st>>>(tile_args(t), t->pinv, ids, out, ldo);
    return cudaGetLastError();
}

// ================================================================================================================
// 2. Batch-1 GEMV (table form).
//
// y[prm[r]] = sum_b S[b][r] * sum_hs d[hs] * ( sum_k T[f_k][hs][t_k] << SH  +  MC * sum_t h_t <c, q_t> ) + (Delta x)
// with q = x16 activation (14-bit ints per 128-col half-slice, the reference CPU default) and the table
// T[f][hs][t] = <A[f], q_t> (exact int32). The integer sums equal the reference's exact integer dot products, so the
// only difference to the CPU result is float rounding in the final scale-and-sum.
//
//   k_act_prep   grid (nb, ncols), 256 thr : x -> FWHT(x sgn/c)/16 -> q, d; tables T (64 KB per 256-col block),
//                                            coset nibble tables G (8 groups x 16 per half-slice)
//   k_gemv       grid (nb * chunks, ncols), 512 thr : one 256-col block x (32 * 16 * tpw) rows per CTA. The block's
//                                            T and G arrive by one bulk copy (TMA engine, mbarrier); each lane owns one
//                                            row and walks its 2 x 32 chunks: 1 PRMT (field byte + rotated chunk
//                                            offset -> table address) + 1 LDS + 1 add per chunk.
//   k_gemv_reduce grid (rows/256, ncols)    : fixed-order sum over blocks, clamp delta, un-permute (deterministic)
// ================================================================================================================
constexpr int kTabInts = 256 * 64;          // T ints per 256-column block: [f][hs][t]
constexpr int kTabBytes = kTabInts * 4;      // 64 KB
constexpr int kGInts = 128;                  // per half-slice: 8 nibble groups x 16
constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr uint32_t kWaitPolls = 1u << 20;  // a healthy table copy lands within a few polls

struct PrepArgs {
    const float *X;
    int64_t ldx;
    const float *ic;
    const uint32_t *A;
    uint32_t cs;
    int K, nb, nsl;
    int *T;     // [ncols][nb][16384]
    int *G;     // [ncols][nsl][128]
    float *d;   // [ncols][nsl]
};

__global__ void __launch_bounds__(256) k_act_prep(PrepArgs a) {
    __shared__ int q_s[256];
    __shared__ uint32_t A_s[256];
    __shared__ int cx_s[64];
    const int b = blockIdx.x, n = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    A_s[tid] = a.A[tid];
    if (tid < 32) {
        const float *x = a.X + (size_t)n * a.ldx + b * 256 + 8 * lane;
        const float *ic = a.ic + b * 256 + 8 * lane;
        float v[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) v[m] = __fmul_rn(x[m], ic[m]);
        fwht256_warp(v, lane);
        float am = 0.f;
#pragma unroll
        for (int m = 0; m < 8; ++m) am = fmaxf(am, fabsf(v[m]));
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));  // per 16-lane half
        const float d = __fdiv_rn(am, 8191.f), id = d > 0.f ? __fdiv_rn(1.f, d) : 0.f;
#pragma unroll
        for (int m = 0; m < 8; ++m) q_s[8 * lane + m] = __float2int_rn(__fmul_rn(v[m], id));
        if ((lane & 15) == 0) a.d[(size_t)n * a.nsl + 2 * b + (lane >> 4)] = d;
    }
    __syncthreads();
    if (tid < 64) {  // <c, q_t> for the 64 chunks of the block
        int cx = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) cx += (int)(int8_t)(a.cs >> (8 * e)) * q_s[4 * tid + e];
        cx_s[tid] = cx;
    }
    __syncthreads();
    {
        const int hs = tid >> 7, grp = (tid >> 4) & 7, m = tid & 15;
        int gsum = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if ((m >> i) & 1) gsum += cx_s[hs * 32 + 4 * grp + i];
        a.G[((size_t)n * a.nsl + 2 * b + hs) * kGInts + grp * 16 + m] = gsum;
    }
    const int ht = tid & 63;  // (hs, t) of this thread
    const int q0 = q_s[4 * ht], q1 = q_s[4 * ht + 1], q2 = q_s[4 * ht + 2], q3 = q_s[4 * ht + 3];
    int *T = a.T + ((size_t)n * a.nb + b) * kTabInts;
#pragma unroll 8
    for (int f = tid >> 6; f < 256; f += 4) {
        const uint32_t w = A_s[f];
        T[f * 64 + ht] = (int)(int8_t)w * q0 + (int)(int8_t)(w >> 8) * q1 + (int)(int8_t)(w >> 16) * q2 + (int)(int8_t)(w >> 24) * q3;
    }
}

struct GemvArgs {
    const uint32_t *M, *D;
    const uint16_t *S;
    const int *T, *G;
    const float *d;
    float *part;  // [ncols][nb][rows]
    int rows, nb, ng, nsl, tpw, chunks;
};

// PRMT selector for step k: result byte 0 = chunk offset byte (k % 3) of po[k / 3], byte 1 = field byte (k % 4) of the
// word, bytes 2-3 = po's zero byte 3 -> (field << 8) | (((lane + k) & 31) * 4) = byte offset into T[f][hs][t].
template <int k>
struct Sel {
    static constexpr uint32_t v = (uint32_t)(4 + k % 3) | ((uint32_t)(k % 4) << 4) | 0x7700u;
};

template <int C, int k>
__device__ __forceinline__ int stage_sum_step(const uint32_t (&w)[24], const uint32_t (&po)[11], const char *Th, int lane, int stage) {
    constexpr int w1 = W1(C), w2 = W2(C), w3 = W3(C);
    const int W = stage == 0 ? w1 : stage == 1 ? w2 : w3;
    const int wb = stage == 0 ? 0 : stage == 1 ? w1 : w1 + w2;
    uint32_t addr;
    if (W == 8) {
        addr = __byte_perm(w[wb + k / 4], po[k / 3], Sel<k>::v);
    } else {
        const uint32_t off = ((uint32_t)(lane + k) & 31u) << 2;
        uint32_t f;
        if (stage == 0) f = ((w[1 + ((w1 - 1) * k) / 32] >> (((w1 - 1) * k) % 32)) |
                             ((((w1 - 1) * k) % 32 + (w1 - 1) > 32) ? (w[2 + ((w1 - 1) * k) / 32] << (32 - ((w1 - 1) * k) % 32)) : 0u)) &
                            ((1u << (w1 - 1)) - 1u);
        else f = (w[wb + (W * k) / 32] >> ((W * k) % 32)) & ((1u << W) - 1u);
        if (stage == 0) f |= ((w[0] >> k) & 1u) << (w1 - 1);
        addr = (f << 8) | off;
    }
    return *reinterpret_cast<const int *>(Th + addr);
}

template <int C, int k>
struct StepLoop {
    static __device__ __forceinline__ void run(const uint32_t (&w)[24], const uint32_t (&po)[11], const char *Th, int lane, int &a1, int &a2,
                                               int &a3) {
        a1 += stage_sum_step<C, k>(w, po, Th, lane, 0);
        if (W2(C)) a2 += stage_sum_step<C, k>(w, po, Th, lane, 1);
        if (W3(C)) a3 += stage_sum_step<C, k>(w, po, Th, lane, 2);
        StepLoop<C, k + 1>::run(w, po, Th, lane, a1, a2, a3);
    }
};
template <int C>
struct StepLoop<C, 32> {
    static __device__ __forceinline__ void run(const uint32_t (&)[24], const uint32_t (&)[11], const char *, int, int &, int &, int &) {}
};

// integer total of one lane-slice: sum of table entries per stage << SH + MC * coset term
template <int C>
__device__ __forceinline__ int lane_slice_dot(const uint32_t (&w)[24], const uint32_t (&po)[11], const char *Th, const int *Gh, int lane) {
    const uint32_t pm = zbits<C>(w);
    const uint32_t H = pingala8_h(__funnelshift_l(pm, pm, lane));
    int cs = 0;
#pragma unroll
    for (int grp = 0; grp < 8; ++grp) cs += Gh[grp * 16 + ((H >> (4 * grp)) & 15u)];
    int a1 = 0, a2 = 0, a3 = 0;
    StepLoop<C, 0>::run(w, po, Th, lane, a1, a2, a3);
    return a1 * (1 << SH1(C)) + a2 * (1 << SH2(C)) + a3 + MC(C) * cs;
}

template <int C>
__device__ __forceinline__ float tile_row_dot(const uint32_t *p0, const uint32_t (&po)[11], const char *Ts, const int *Gs, int lane, float d0,
                                              float d1) {
    uint32_t w0[24], w1[24];
    load_lane_words<C>(p0, 0, lane, w0);
    load_lane_words<C>(p0, 1, lane, w1);
    const int i0 = lane_slice_dot<C>(w0, po, Ts, Gs, lane);
    const int i1 = lane_slice_dot<C>(w1, po, Ts + 128, Gs + kGInts, lane);
    return __fadd_rn(__fmul_rn((float)i0, d0), __fmul_rn((float)i1, d1));
}

__global__ void __launch_bounds__(kGemvThreads, 2) k_gemv(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    int *Ts = reinterpret_cast<int *>(sm);
    int *Gs = Ts + kTabInts;
    uint64_t *bar = reinterpret_cast<uint64_t *>(Gs + 2 * kGInts);
    const int b = blockIdx.x % a.nb, chunk = blockIdx.x / a.nb, n = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_expect_tx(bar, kTabBytes + 2 * kGInts * 4);
        bulk_g2s(Ts, a.T + ((size_t)n * a.nb + b) * kTabInts, kTabBytes, bar);
        bulk_g2s(Gs, a.G + ((size_t)n * a.nsl + 2 * b) * kGInts, 2 * kGInts * 4, bar);
    }
    const int g_first = chunk * kGemvWarps * a.tpw + warp;
    if (lane == 0) {  // stream this warp's tile payloads toward L2 while the tables arrive
        for (int i = 0; i < a.tpw; ++i) {
            const int g = g_first + kGemvWarps * i;
            if (g >= a.ng) break;
            const uint32_t mt = __ldg(a.M + (size_t)g * a.nb + b);
            const int c = (int)(mt >> 29);
            if (c) bulk_prefetch_l2(a.D + (mt & 0x1FFFFFFFu), (uint32_t)NW(c) * 256u);
        }
    }
    uint32_t po[11];
#pragma unroll
    for (int q = 0; q < 11; ++q) {
        uint32_t r = 0;
#pragma unroll
        for (int i = 0; i < 3; ++i)
            if (3 * q + i < 32) r |= (((uint32_t)(lane + 3 * q + i) & 31u) << 2) << (8 * i);
        po[q] = r;
    }
    const float d0 = a.d[(size_t)n * a.nsl + 2 * b], d1 = a.d[(size_t)n * a.nsl + 2 * b + 1];
    if (!mbar_wait_bounded(bar, 0, kWaitPolls)) {
        if (lane == 0) atomicOr(&g_p8_device_error, 1u);
        mbar_wait_bounded(bar, 0, kWaitPolls);  // the copy must land before the CTA's shared memory goes away
        return;
    }
    const char *Tc = reinterpret_cast<const char *>(Ts);
    for (int i = 0; i < a.tpw; ++i) {
        const int g = g_first + kGemvWarps * i;
        if (g >= a.ng) break;
        const uint32_t mt = __ldg(a.M + (size_t)g * a.nb + b);
        const int c = (int)(mt >> 29);
        const uint32_t *p0 = a.D + (mt & 0x1FFFFFFFu);
        float acc = 0.f;
        switch (c) {
            case 0: break;
            case 1: acc = tile_row_dot<1>(p0, po, Tc, Gs, lane, d0, d1); break;
            case 2: acc = tile_row_dot<2>(p0, po, Tc, Gs, lane, d0, d1); break;
            case 3: acc = tile_row_dot<3>(p0, po, Tc, Gs, lane, d0, d1); break;
            case 4: acc = tile_row_dot<4>(p0, po, Tc, Gs, lane, d0, d1); break;
            case 5: acc = tile_row_dot<5>(p0, po, Tc, Gs, lane, d0, d1); break;
            case 6: acc = tile_row_dot<6>(p0, po, Tc, Gs, lane, d0, d1); break;
            default: acc = tile_row_dot<7>(p0, po, Tc, Gs, lane, d0, d1); break;
        }
        const int r = g * 32 + lane;
        a.part[((size_t)n * a.nb + b) * a.rows + r] = __fmul_rn(acc, h2f(a.S[(size_t)b * a.rows + r]));
    }
}

struct ReduceArgs {
    const float *part;
    const int16_t *prm;
    const int *cp;
    const uint16_t *cc;
    const float *cv;
    const float *X;
    int64_t ldx;
    float *Y;
    int64_t ldy;
    int rows, nb;
};

__global__ void __launch_bounds__(256) k_gemv_reduce(ReduceArgs a) {
    const int r = blockIdx.x * 256 + threadIdx.x, n = blockIdx.y;
    if (r >= a.rows) return;
    const float *p = a.part + (size_t)n * a.nb * a.rows + r;
    float s = 0.f;
    for (int b = 0; b < a.nb; ++b) s = __fadd_rn(s, p[(size_t)b * a.rows]);
    const int ro = a.prm[r];
    const float *x = a.X + (size_t)n * a.ldx;
    for (int e = a.cp[ro]; e < a.cp[ro + 1]; ++e) s = __fadd_rn(s, __fmul_rn(a.cv[e], x[a.cc[e]]));
    a.Y[(size_t)n * a.ldy + ro] = s;
}

// workspace layout (bytes, each part 256-aligned): T | G | d | partials
struct GemvWs {
    size_t T, G, d, part, total;
};
static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }
static GemvWs gemv_ws_layout(const p8_tensor *t, int64_t ncols) {
    GemvWs w;
    w.T = 0;
    w.G = w.T + al256((size_t)ncols * t->nb * kTabBytes);
    w.d = w.G + al256((size_t)ncols * t->nsl * kGInts * 4);
    w.part = w.d + al256((size_t)ncols * t->nsl * 4);
    w.total = w.part + al256((size_t)ncols * t->nb * t->rows * 4);
    return w;
}
size_t gemv_workspace(const p8_tensor *t, int64_t ncols) { return gemv_ws_layout(t, ncols).total; }

static int gemv_tpw(const p8_tensor *t) {
    // rows per CTA = 512 * tpw: aim at >= 2 CTAs per SM in flight without shrinking a CTA below 512 rows
    const int sms = 148;
    int tpw = 1;
    while (tpw < 4 && (size_t)t->nb * ((t->ng + kGemvWarps * (tpw * 2) - 1) / (kGemvWarps * (tpw * 2))) >= (size_t)2 * sms) tpw *= 2;
    return tpw;
}

p8_status launch_gemv(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, float *Y, int64_t ldy, void *ws, size_t ws_bytes,
                      cudaStream_t st) {
    const GemvWs L = gemv_ws_layout(t, ncols);
    if (!ws || ws_bytes < L.total) return P8_ERR_WORKSPACE;
    if (ncols > 65535) return P8_ERR_ARG;
    uint8_t *w = static_cast<uint8_t *>(ws);
    PrepArgs pa;
    pa.X = X; pa.ldx = ldx; pa.ic = t->ic; pa.A = t->A; pa.cs = t->cs; pa.K = t->K; pa.nb = t->nb; pa.nsl = t->nsl;
    pa.T = reinterpret_cast<int *>(w + L.T);
    pa.G = reinterpret_cast<int *>(w + L.G);
    pa.d = reinterpret_cast<float *>(w + L.d);
    k_act_prep<<<dim3(t->nb, (unsigned)ncols), 256, 0, st>>>(pa);
    GemvArgs ga;
    ga.M = t->M; ga.D = t->D; ga.S = t->S; ga.T = pa.T; ga.G = pa.G; ga.d = pa.d;
    ga.part = reinterpret_cast<float *>(w + L.part);
    ga.rows = t->rows; ga.nb = t->nb; ga.ng = t->ng; ga.nsl = t->nsl;
    ga.tpw = gemv_tpw(t);
    ga.chunks = (t->ng + kGemvWarps * ga.tpw - 1) / (kGemvWarps * ga.tpw);
    const size_t smem = kTabBytes + 2 * kGInts * 4 + 16;
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return P8_ERR_CUDA;
        attr_set = true;
    }
    k_gemv<<<dim3((unsigned)(t->nb * ga.chunks), (unsigned)ncols), kGemvThreads, smem, st>>>(ga);
    ReduceArgs ra;
    ra.part = ga.part; ra.prm = t->prm; ra.cp = t->cp; ra.cc = t->cc; ra.cv = t->cv; ra.X = X; ra.ldx = ldx; ra.Y = Y; ra.ldy = ldy;
    ra.rows = t->rows; ra.nb = t->nb;
    k_gemv_reduce<<<dim3((unsigned)((t->rows + 255) / 256), (unsigned)ncols), 256, 0, st>>>(ra);
    return cudaGetLastError() == cudaSuccess ? P8_OK : P8_ERR_CUDA;
}

unsigned int read_and_clear_device_error() {
    unsigned int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_p8_device_error, sizeof(v));
    cudaMemcpyToSymbol(g_p8_device_error, &z, sizeof(z));
    return v;
}

}  // namespace p8
