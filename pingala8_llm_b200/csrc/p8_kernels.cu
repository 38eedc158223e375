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
//   k_act_prep  grid (nb, 8, ncols), 256 thr: x -> FWHT(x sgn/c)/16 -> q, d (per 128-col half-slice); 1/8 of the
//               table T[b] (64 KB per 256-col block) per CTA; coset nibble tables G; zeroes the accumulators.
//   k_gemv      grid (items, ncols), 512 thr: an item is one 256-col block b x 512 * tpw sorted rows of one tensor
//               (up to 4 tensors sharing x run in one launch: q/k/v, gate/up). The block's T and G arrive by one bulk
//               copy (TMA engine, mbarrier) while the warps load their first payload words; each lane owns one row
//               and walks its 2 x 32 chunks: 1 PRMT (field byte + rotated chunk offset -> table address) + 1 LDS +
//               1 add per chunk. Row partials go to int64 fixed-point accumulators with integer atomics (exact, so
//               the result does not depend on arrival order); the last item of a row range (arrival counter)
//               converts, adds the clamp delta and scatters y[prm[r]].
// Both kernels use programmatic dependent launch: a GEMV's CTAs start while the previous kernel drains, stream
// their weight tiles toward L2, and only then wait for the activation tables.
// ================================================================================================================
constexpr int kTabInts = 256 * 64;          // T ints per 256-column block: [f][hs][t]
constexpr int kTabBytes = kTabInts * 4;      // 64 KB
constexpr int kGInts = 128;                  // per half-slice: 8 nibble groups x 16
constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kMaxGroup = 4;
constexpr uint32_t kWaitPolls = 1u << 20;  // a healthy table copy lands within a few polls
constexpr double kFixScale = 4294967296.0; // fixed-point accumulators: 2^32 units per 1.0

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

struct GemvTensor {
    const uint32_t *M, *D;
    const uint16_t *S;
    const int16_t *prm;
    const int *cp;
    const uint16_t *cc;
    const float *cv;
    float *Y;
    int64_t ldy;
    unsigned long long *acc;  // [ncols][rows]
    unsigned int *cnt;        // [ncols][chunks]
    int rows, ng, chunks, item0;
};

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
    unsigned long long *zero64;  // accumulators to clear
    size_t nzero64;
    unsigned int *zero32;        // arrival counters to clear
    size_t nzero32;
};

__global__ void __launch_bounds__(256) k_act_prep(PrepArgs a) {
    __shared__ int q_s[256];
    __shared__ uint32_t A_s[32];
    __shared__ int cx_s[64];
    const int b = blockIdx.x, fg = blockIdx.y, n = blockIdx.z, tid = threadIdx.x, lane = tid & 31;
    pdl_launch_dependents();
    if (tid < 32) A_s[tid] = a.A[32 * fg + tid];
    pdl_wait();  // x and the workspace belong to the previous kernel until it completes
    {
        const size_t nthreads = (size_t)gridDim.x * gridDim.y * gridDim.z * 256;
        const size_t id = (((size_t)n * gridDim.y + fg) * gridDim.x + b) * 256 + tid;
        for (size_t i = id; i < a.nzero64; i += nthreads) a.zero64[i] = 0ull;
        for (size_t i = id; i < a.nzero32; i += nthreads) a.zero32[i] = 0u;
    }
    if (tid < 32) {
        const float *x = a.X + (size_t)n * a.ldx + b * 256 + 8 * lane;
        const float *ic = a.ic + b * 256 + 8 * lane;
        const float4 x0 = *reinterpret_cast<const float4 *>(x), x1 = *reinterpret_cast<const float4 *>(x + 4);
        const float4 i0 = *reinterpret_cast<const float4 *>(ic), i1 = *reinterpret_cast<const float4 *>(ic + 4);
        float v[8] = {__fmul_rn(x0.x, i0.x), __fmul_rn(x0.y, i0.y), __fmul_rn(x0.z, i0.z), __fmul_rn(x0.w, i0.w),
                      __fmul_rn(x1.x, i1.x), __fmul_rn(x1.y, i1.y), __fmul_rn(x1.z, i1.z), __fmul_rn(x1.w, i1.w)};
        fwht256_warp(v, lane);
        float am = 0.f;
#pragma unroll
        for (int m = 0; m < 8; ++m) am = fmaxf(am, fabsf(v[m]));
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));  // per 16-lane half
        const float d = __fdiv_rn(am, 8191.f), id = d > 0.f ? __fdiv_rn(1.f, d) : 0.f;
#pragma unroll
        for (int m = 0; m < 8; ++m) q_s[8 * lane + m] = __float2int_rn(__fmul_rn(v[m], id));
        if (fg == 0 && (lane & 15) == 0) a.d[(size_t)n * a.nsl + 2 * b + (lane >> 4)] = d;
    }
    __syncthreads();
    if (fg == 0) {
        if (tid < 64) {  // <c, q_t> for the 64 chunks of the block
            int cx = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) cx += (int)(int8_t)(a.cs >> (8 * e)) * q_s[4 * tid + e];
            cx_s[tid] = cx;
        }
        __syncthreads();
        const int hs = tid >> 7, grp = (tid >> 4) & 7, m = tid & 15;
        int gsum = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if ((m >> i) & 1) gsum += cx_s[hs * 32 + 4 * grp + i];
        a.G[((size_t)n * a.nsl + 2 * b + hs) * kGInts + grp * 16 + m] = gsum;
    }
    // this CTA's 32 codebook entries x 64 (hs, t): thread = (f-quarter, hs, t), 8 entries each, coalesced stores
    const int ht = tid & 63;
    const int q0 = q_s[4 * ht], q1 = q_s[4 * ht + 1], q2 = q_s[4 * ht + 2], q3 = q_s[4 * ht + 3];
    int *T = a.T + ((size_t)n * a.nb + b) * kTabInts + (32 * fg) * 64;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int f = (tid >> 6) + 4 * i;
        const uint32_t w = A_s[f];
        T[f * 64 + ht] = (int)(int8_t)w * q0 + (int)(int8_t)(w >> 8) * q1 + (int)(int8_t)(w >> 16) * q2 + (int)(int8_t)(w >> 24) * q3;
    }
}

struct GemvArgs {
    GemvTensor t[kMaxGroup];
    int ntensors;
    const int *T, *G;
    const float *d;
    const float *X;
    int64_t ldx;
    int nb, nsl, tpw;
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

__device__ __forceinline__ float tile_row_any(int c, const uint32_t *p0, const uint32_t (&po)[11], const char *Ts, const int *Gs, int lane,
                                              float d0, float d1) {
    switch (c) {
        case 0: return 0.f;
        case 1: return tile_row_dot<1>(p0, po, Ts, Gs, lane, d0, d1);
        case 2: return tile_row_dot<2>(p0, po, Ts, Gs, lane, d0, d1);
        case 3: return tile_row_dot<3>(p0, po, Ts, Gs, lane, d0, d1);
        case 4: return tile_row_dot<4>(p0, po, Ts, Gs, lane, d0, d1);
        case 5: return tile_row_dot<5>(p0, po, Ts, Gs, lane, d0, d1);
        case 6: return tile_row_dot<6>(p0, po, Ts, Gs, lane, d0, d1);
        default: return tile_row_dot<7>(p0, po, Ts, Gs, lane, d0, d1);
    }
}

__global__ void __launch_bounds__(kGemvThreads, 2) k_gemv(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    int *Ts = reinterpret_cast<int *>(sm);
    int *Gs = Ts + kTabInts;
    uint64_t *bar = reinterpret_cast<uint64_t *>(Gs + 2 * kGInts);
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, n = blockIdx.y;
    // item -> (tensor, block, row chunk)
    int ti = 0;
#pragma unroll
    for (int i = 1; i < kMaxGroup; ++i)
        if (i < a.ntensors && (int)blockIdx.x >= a.t[i].item0) ti = i;
    const GemvTensor &T = a.t[ti];
    const int item = blockIdx.x - T.item0, b = item % a.nb, chunk = item / a.nb;
    const int g_first = chunk * kGemvWarps * a.tpw + warp;
    pdl_launch_dependents();
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    if (lane == 0) {  // stream this warp's tile payloads toward L2 before waiting on the producer of x
        for (int i = 0; i < a.tpw; ++i) {
            const int g = g_first + kGemvWarps * i;
            if (g >= T.ng) break;
            const uint32_t mt = __ldg(T.M + (size_t)g * a.nb + b);
            const int c = (int)(mt >> 29);
            if (c) bulk_prefetch_l2(T.D + (mt & 0x1FFFFFFFu), (uint32_t)NW(c) * 256u);
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
    pdl_wait();  // tables, accumulators and x are written by the preceding prep kernel
    __syncthreads();
    if (tid == 0) {
        mbar_expect_tx(bar, kTabBytes + 2 * kGInts * 4);
        bulk_g2s(Ts, a.T + ((size_t)n * a.nb + b) * kTabInts, kTabBytes, bar);
        bulk_g2s(Gs, a.G + ((size_t)n * a.nsl + 2 * b) * kGInts, 2 * kGInts * 4, bar);
    }
    const float d0 = a.d[(size_t)n * a.nsl + 2 * b], d1 = a.d[(size_t)n * a.nsl + 2 * b + 1];
    if (!mbar_wait_bounded(bar, 0, kWaitPolls)) {
        if (lane == 0) atomicOr(&g_p8_device_error, 1u);
        mbar_wait_bounded(bar, 0, kWaitPolls);  // the copy must land before the CTA's shared memory goes away
        return;
    }
    const char *Tc = reinterpret_cast<const char *>(Ts);
    unsigned long long *acc = T.acc + (size_t)n * T.rows;
    for (int i = 0; i < a.tpw; ++i) {
        const int g = g_first + kGemvWarps * i;
        if (g >= T.ng) break;
        const uint32_t mt = __ldg(T.M + (size_t)g * a.nb + b);
        const float part = tile_row_any((int)(mt >> 29), T.D + (mt & 0x1FFFFFFFu), po, Tc, Gs, lane, d0, d1);
        const int r = g * 32 + lane;
        const float v = __fmul_rn(part, h2f(T.S[(size_t)b * T.rows + r]));
        atomicAdd(acc + r, (unsigned long long)__double2ll_rn((double)v * kFixScale));
    }
    // arrival counter of this row chunk; the last of its nb items finishes the rows
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(T.cnt + (size_t)n * T.chunks + chunk, 1u);
        s_last = prev == (unsigned)(a.nb - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int r0 = chunk * kGemvWarps * a.tpw * 32, r1 = min(T.rows, r0 + kGemvWarps * a.tpw * 32);
    const float *x = a.X + (size_t)n * a.ldx;
    for (int r = r0 + tid; r < r1; r += kGemvThreads) {
        const long long s = (long long)__ldcg(acc + r);
        float v = (float)((double)s * (1.0 / kFixScale));
        const int ro = T.prm[r];
        for (int e = T.cp[ro]; e < T.cp[ro + 1]; ++e) v = __fadd_rn(v, __fmul_rn(T.cv[e], x[T.cc[e]]));
        T.Y[(size_t)n * T.ldy + ro] = v;
    }
}

// workspace layout (bytes, each part 256-aligned): T | G | d | acc (int64 per row) | counters
struct GemvWs {
    size_t T, G, d, acc, cnt, total;
};
static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }
static int gemv_tpw_for(int ng_total, int nb) {
    // rows per item = 512 * tpw: the largest that still leaves ~2 items per SM (148 SMs) in the launch
    int tpw = 1;
    while (tpw < 8 && (size_t)nb * (size_t)((ng_total + kGemvWarps * tpw * 2 - 1) / (kGemvWarps * tpw * 2)) >= 296) tpw *= 2;
    return tpw;
}
static GemvWs gemv_ws_layout(const p8_tensor *const *ts, int nt, int64_t ncols, int tpw) {
    const p8_tensor *t = ts[0];
    size_t rows = 0, chunks = 0;
    for (int i = 0; i < nt; ++i) {
        rows += (size_t)ts[i]->rows;
        chunks += (size_t)((ts[i]->ng + kGemvWarps * tpw - 1) / (kGemvWarps * tpw));
    }
    GemvWs w;
    w.T = 0;
    w.G = w.T + al256((size_t)ncols * t->nb * kTabBytes);
    w.d = w.G + al256((size_t)ncols * t->nsl * kGInts * 4);
    w.acc = w.d + al256((size_t)ncols * t->nsl * 4);
    w.cnt = w.acc + al256((size_t)ncols * rows * 8);
    w.total = w.cnt + al256((size_t)ncols * chunks * 4);
    return w;
}
size_t gemv_workspace(const p8_tensor *t, int64_t ncols) {
    // sized for the smallest row chunk (tpw = 1): covers every tpw choice
    return gemv_ws_layout(&t, 1, ncols, 1).total;
}
size_t gemv_group_workspace(const p8_tensor *const *ts, int nt, int64_t ncols) { return gemv_ws_layout(ts, nt, ncols, 1).total; }

static cudaError_t launch_pdl(const void *fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void **args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

p8_status launch_gemv_group(const p8_tensor *const *ts, int nt, const float *X, int64_t ncols, int64_t ldx, float *const *Ys,
                            const int64_t *ldys, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (nt < 1 || nt > kMaxGroup) return P8_ERR_ARG;
    const p8_tensor *t0 = ts[0];
    int ng_total = 0;
    for (int i = 0; i < nt; ++i) {
        // tensors of one launch share x and its table: same K, column scales, signs and codebook (content hash)
        if (ts[i]->K != t0->K || ts[i]->act_hash != t0->act_hash) return P8_ERR_ARG;
        ng_total += ts[i]->ng;
    }
    if (ncols > 65535) return P8_ERR_ARG;
    const int tpw = gemv_tpw_for(ng_total, t0->nb);
    const GemvWs L = gemv_ws_layout(ts, nt, ncols, tpw);
    if (!ws || ws_bytes < L.total) return P8_ERR_WORKSPACE;
    uint8_t *w = static_cast<uint8_t *>(ws);
    PrepArgs pa;
    pa.X = X; pa.ldx = ldx; pa.ic = t0->ic; pa.A = t0->A; pa.cs = t0->cs; pa.K = t0->K; pa.nb = t0->nb; pa.nsl = t0->nsl;
    pa.T = reinterpret_cast<int *>(w + L.T);
    pa.G = reinterpret_cast<int *>(w + L.G);
    pa.d = reinterpret_cast<float *>(w + L.d);
    pa.zero64 = reinterpret_cast<unsigned long long *>(w + L.acc);
    pa.nzero64 = (L.cnt - L.acc) / 8;
    pa.zero32 = reinterpret_cast<unsigned int *>(w + L.cnt);
    pa.nzero32 = (L.total - L.cnt) / 4;
    {
        void *args[] = {&pa};
        if (launch_pdl((const void *)k_act_prep, dim3(t0->nb, 8, (unsigned)ncols), dim3(256), 0, st, args) != cudaSuccess)
            return P8_ERR_CUDA;
    }
    GemvArgs ga;
    memset(&ga, 0, sizeof(ga));
    ga.ntensors = nt; ga.T = pa.T; ga.G = pa.G; ga.d = pa.d; ga.X = X; ga.ldx = ldx;
    ga.nb = t0->nb; ga.nsl = t0->nsl; ga.tpw = tpw;
    int item0 = 0;
    size_t acc_off = 0, cnt_off = 0;
    for (int i = 0; i < nt; ++i) {
        const p8_tensor *t = ts[i];
        GemvTensor &g = ga.t[i];
        g.M = t->M; g.D = t->D; g.S = t->S; g.prm = t->prm; g.cp = t->cp; g.cc = t->cc; g.cv = t->cv;
        g.Y = Ys[i]; g.ldy = ldys[i];
        g.rows = t->rows; g.ng = t->ng;
        g.chunks = (t->ng + kGemvWarps * tpw - 1) / (kGemvWarps * tpw);
        g.item0 = item0;
        g.acc = pa.zero64 + acc_off * ncols;
        g.cnt = pa.zero32 + cnt_off * ncols;
        acc_off += (size_t)t->rows;
        cnt_off += (size_t)g.chunks;
        item0 += g.chunks * t->nb;
    }
    const size_t smem = kTabBytes + 2 * kGInts * 4 + 16;
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return P8_ERR_CUDA;
        attr_set = true;
    }
    void *args[] = {&ga};
    if (launch_pdl((const void *)k_gemv, dim3((unsigned)item0, (unsigned)ncols), dim3(kGemvThreads), smem, st, args) != cudaSuccess)
        return P8_ERR_CUDA;
    return P8_OK;
}

p8_status launch_gemv(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, float *Y, int64_t ldy, void *ws, size_t ws_bytes,
                      cudaStream_t st) {
    return launch_gemv_group(&t, 1, X, ncols, ldx, &Y, &ldy, ws, ws_bytes, st);
}

unsigned int read_and_clear_device_error() {
    unsigned int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_p8_device_error, sizeof(v));
    cudaMemcpyToSymbol(g_p8_device_error, &z, sizeof(z));
    return v;
}

}  // namespace p8
