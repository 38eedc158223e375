// p8_kernels.cu -- Pingala-8 decode / dequant / get_rows and the batch-1 table GEMV for sm_100a.
//
// One translation unit holds every kernel of the library (the tcgen05 GEMM is included from p8_gemm.cuh).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <algorithm>
#include <type_traits>
#include <atomic>

#include "p8_device.cuh"
#include "p8_internal.h"

namespace p8 {

// device-side error word (that launch's results are invalid): bit 2 GEMM pipeline wait timed out, bit 3 row-parallel
// exchange wait timed out, bit 4 exchange entry with a foreign tag (bits 0, 1 and 5 unused)
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
// T[f][hs][t] = <A[f], q_t> (an exact integer, |T| < 2^23, stored as a float: exact). The lane sums run in fp32 on the
// FP32 pipe, which leaves the integer ALU to the address PRMTs; they equal the reference's exact integer dot products
// up to fp32 rounding of the running sum (<= 2^-24 relative per add), as does the final scale-and-sum.
//
//   k_gemv         at most one 512-thread CTA per SM. The work is the list of (block b, tile g) units of up to four
//                  tensors that read the same x, ordered block-major and cut into contiguous CTA ranges balanced on
//                  the host (a CTA touches one or two blocks). After the wait for the producer of x, each CTA builds
//                  the tables of its blocks in its own shared memory: x -> input op -> FWHT(x sgn/c)/16 -> x16 ints
//                  and scales per half-slice -> T (64 KB per block) and the coset nibble tables G. No table goes
//                  through global memory and no second kernel sits between x and the units. The payload words of a
//                  warp's next unit are loaded into registers while the current unit computes; each lane owns one
//                  row: per chunk 1 PRMT (field byte + rotated chunk offset -> table byte address) + 1 LDS + 1 FADD.
//                  A unit stores its 32 row partials at the rows' original positions ([b][rows]).
//   k_gemv_reduce  the rows, in original order: y[ro] = sum_b part[b][ro] in block order + clamp delta (coalesced;
//                  deterministic, no float
//                  atomics); the row-parallel exchange for the fused tensor-parallel call.
// Both kernels use programmatic dependent launch: each is resident and waiting before its predecessor ends, and a
// call is two kernel hand-offs (producer of x -> k_gemv -> k_gemv_reduce) with no grid barrier.
// ================================================================================================================
constexpr int kTabInts = 256 * 64;          // T ints per 256-column block: [f][hs][t]
constexpr int kTabBytes = kTabInts * 4;      // 64 KB
constexpr int kGInts = 128;                  // per half-slice: 8 nibble groups x 16
constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kMaxGroup = 4;
constexpr int kGemvMaxCtas = 256;           // CTA ranges carried in the launch arguments
// dynamic shared memory of k_gemv: two table buffers, two G buffers (both half-slices)
constexpr int kSmemT0 = 0, kSmemT1 = kTabBytes, kSmemG0 = 2 * kTabBytes, kSmemG1 = kSmemG0 + 2 * kGInts * 4,
              kGemvSmem = kSmemG1 + 2 * kGInts * 4;

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
    float *part;          // [nb][rows] row partials per block
    const float *res;     // chained calls: residual added to the output (nullptr: none)
    int rows, ng, g0, row0;  // g0: first unit index of this tensor inside one block; row0: first row in the group
    int ucls;                // uniform class (payload of tile i at word i * 64 NW), 0 if the M words must be read
};

// Chained calls (p8_chain): a step's input may be an output y of the previous step, read straight from that step's
// partials while the tables are built; the previous step's other outputs are reduced by this step's CTAs in equal
// shares. Either way a previous output row is
//     y[ro] = ((sum over 16-block slices, in order, of the slice's partials in block order) + clamp delta on x'_prev)
//             * scale_prev + res[ro]
// the same order as k_gemv_reduce, so a row's value does not depend on which kernel or CTA reduced it. scale_prev is
// the previous step's deferred RMSNorm scale (1 / sqrt(sum of its blocks' x^2 / K + eps)) or 1.
struct ChainSrc {
    const float *part;    // the tensor's partials [nb][rows] (original row positions); nullptr: not from partials
    const int *cp;        // its clamp-delta CSR by original row
    const uint16_t *cc;
    const float *cv;
    const float *res;     // residual added to its output (nullptr: none)
    float *Y;             // its output (the reducing CTA writes it)
    int rows;
};
struct ChainIn {
    ChainSrc x, x2;            // sources of this step's x and of the SwiGLU up (part == nullptr: from memory)
    ChainSrc unc[kMaxGroup];   // previous-step outputs this step does not read
    int nunc, unc_rows;
    const float *xv;           // the previous step's x' (its outputs' clamp-delta term)
    const float *ss;           // the previous step's per-block sums of x^2 when its RMSNorm scale is deferred, else nullptr
    int nb, K;                 // the previous step's blocks and K
    float eps;
    int chained;               // 1: there is a previous step (the fields above are valid)
    float *ss_out;             // this step's input comes from partials with RMSNorm: per-block sums of x^2 (the scale
                               // is deferred to the outputs); nullptr otherwise
    unsigned long long *trace; // optional phase stamps: [CTA][8] globaltimer ns (nullptr: off)
};

struct GemvArgs {
    GemvTensor t[kMaxGroup];
    int rows_total;
    int ntensors;
    // the group's one input: x, column scales sgn/c, codebook, coset word, input op
    const float *X;
    const float *ic;
    const uint32_t *A;
    uint32_t cs;
    int K, nb, nsl, ng_total;
    long long units;       // nb * ng_total
    const float *pw, *x2;  // input op (k_gemv<PRO>): RMSNorm weight / SwiGLU up
    float eps;
    float *xv;             // x' of the input op for the clamp-delta term (written by the first CTA of each block)
    unsigned int *epoch;   // row-parallel exchange: this rank's call counter (advanced by CTA 0), else nullptr
    int ustart[kGemvMaxCtas + 1];  // CTA c takes the units [ustart[c], ustart[c + 1]) of the block-major list
    long long ldx;         // k_gemv2: column 1's x (and SwiGLU up) at X + ldx (x2 + ldx)
};

// the row reduction after k_gemv: y[ro] = sum_b part[b][ro] (block order) + clamp delta (+ row-parallel exchange)
struct ReduceArgs {
    GemvTensor t[kMaxGroup];
    int rows_total, ntensors, nb;
    const float *X;  // x, or x' of the input op: the clamp delta multiplies it
    TpExchange tp;   // row-parallel exchange (tp.world > 1), single tensor only
    const float *ss; // the last chain step's deferred RMSNorm: per-block sums of x^2 (nullptr: scale 1)
    int ssK;
    float eps;
};

// the deferred RMSNorm scale from nb per-block sums of squares (one thread; fixed order)
__device__ __forceinline__ float deferred_scale(const float *ss, int nb, int K, float eps) {
    float v = 0.f;
#pragma unroll 8
    for (int i = 0; i < nb; ++i) v = __fadd_rn(v, __ldcg(ss + i));
    return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, (float)K), eps)));
}

// the 16-block slice sums of row ro of a [nb][rows] partial array (slice j: blocks 16 j .. 16 j + 15 in block order)
__device__ __forceinline__ float slice_sum(const float *part, int rows, int nb, int ro, int j) {
    const int b0 = 16 * j, n = min(16, nb - b0);
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = k < n ? __ldcg(part + (size_t)(b0 + k) * rows + ro) : 0.f;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k)
        if (k < n) s = __fadd_rn(s, v[k]);
    return s;
}
// y of a chained output row from its slice sums sl[0 .. S) (k_gemv_reduce's order), clamp delta, scale, residual
__device__ __forceinline__ float chain_row_value(const ChainSrc &T, int ro, float y, const float *xv, float scale) {
    const int e1 = __ldg(T.cp + ro + 1);
    for (int e = __ldg(T.cp + ro); e < e1; ++e) y = __fadd_rn(y, __fmul_rn(__ldg(T.cv + e), __ldcg(xv + __ldg(T.cc + e))));
    y = __fmul_rn(y, scale);
    if (T.res) y = __fadd_rn(y, __ldcg(T.res + ro));
    return y;
}

// x'[i] = (x[i] * scale) * w[i], scale = 1 / sqrt(mean(x^2) + eps): ggml's rms_norm (sum of squares, mean by float
// division, 1 / sqrtf) followed by the weight multiply. Every CTA sums the whole vector in the same fixed order
// (per-thread strided float4 sums, a butterfly over each warp, then the warp sums in warp order: one barrier), so all
// CTAs get the same scale.
template <int NT>
__device__ __forceinline__ float rms_scale(const float *x, int K, float eps, float *red) {
    const int tid = threadIdx.x;
    float ss = 0.f;
    for (int k = 4 * tid; k < K; k += 4 * NT) {
        const float4 v = *reinterpret_cast<const float4 *>(x + k);
        ss = __fmaf_rn(v.x, v.x, ss);
        ss = __fmaf_rn(v.y, v.y, ss);
        ss = __fmaf_rn(v.z, v.z, ss);
        ss = __fmaf_rn(v.w, v.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));  // every lane: the warp sum
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float t = red[0];
#pragma unroll
    for (int w = 1; w < NT / 32; ++w) t = __fadd_rn(t, red[w]);
    const float mean = __fdiv_rn(t, (float)K);
    return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

extern __shared__ __align__(1024) uint8_t g_smem[];

__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Row-parallel exchange of one output row (layout and protocol: TpExchange). Each 8-byte entry carries the value and
// its tag in one single-copy-atomic store, so an entry that reads as tagged holds its value: no flag, no fence. The
// peers' entries are loaded together (one round trip for all ranks) and only the missing ones are polled again.
// Returns the sum over ranks in rank order (the same bits on every rank); on a wait past the deadline or a mismatched
// tag it sets the device error word (bit 3 / bit 4) and the row's result is invalid.
__device__ __forceinline__ float tp_exchange_row(const TpExchange &x, unsigned int par, int row, int orig_row, float y,
                                                 unsigned long long deadline, bool &ok) {
    const unsigned int tag = 0x80000000u | ((unsigned int)orig_row << 16) | x.tag_rows;
    const unsigned long long v = ((unsigned long long)tag << 32) | __float_as_uint(y);
    const long long sec = (long long)par * x.world;
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q)
        if (q < x.world && q != x.rank) st_relaxed_sys(x.peer[q] + (sec + x.rank) * x.cap + row, v);
    unsigned long long *own = x.peer[x.rank] + sec * x.cap + row;
    unsigned long long e[kTpMaxWorld];
    unsigned int missing = 0;  // bit q: rank q's entry not seen yet
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q) {
        e[q] = 0ull;
        if (ok && q < x.world && q != x.rank) e[q] = ld_relaxed_sys(own + q * x.cap);
    }
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q)
        if (q < x.world && q != x.rank && (unsigned int)(e[q] >> 32) == 0u) missing |= 1u << q;
    while (ok && missing) {
        if (global_ns() > deadline) {
            atomicOr(&g_p8_device_error, 8u);
            ok = false;
            break;
        }
        __nanosleep(32);
#pragma unroll
        for (int q = 0; q < kTpMaxWorld; ++q)
            if ((missing >> q) & 1u) {
                e[q] = ld_relaxed_sys(own + q * x.cap);
                if ((unsigned int)(e[q] >> 32) != 0u) missing &= ~(1u << q);
            }
    }
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kTpMaxWorld; ++q) {
        if (q >= x.world) break;
        float yq = y;
        if (q != x.rank) {
            if (ok && (unsigned int)(e[q] >> 32) != tag) atomicOr(&g_p8_device_error, 16u);
            if (ok) own[q * x.cap] = 0ull;  // consumed; the peer writes this half again two calls later
            yq = __uint_as_float((unsigned int)e[q]);
        }
        s = q == 0 ? yq : __fadd_rn(s, yq);
    }
    return s;
}

// table byte address of the chunk at step k: PRMT places the field byte (k % 4 of word k / 4) in bits 8-15 and the
// lane's rotated chunk offset ((lane + k) & 31) * 4 (byte k % 3 of po[k / 3]; po byte 3 is zero) in bits 0-7.
template <int k>
struct Sel {
    static constexpr uint32_t v = (uint32_t)(4 + k % 3) | ((uint32_t)(k % 4) << 4) | 0x7700u;
};

// shared-memory int at a compile-time offset plus a register byte offset: indexing the extern __shared__ symbol
// directly lets the compiler fold the offset into the load's immediate (no address add per lookup)
template <int OFF, typename V = int>
__device__ __forceinline__ V lds_at(uint32_t byte_off) {
    return *reinterpret_cast<const V *>(g_smem + OFF + byte_off);
}

template <int C, int k>
__device__ __forceinline__ uint32_t stage_addr(const uint32_t (&w)[24], const uint32_t (&po)[11], int lane, int stage) {
    constexpr int w1 = W1(C), w2 = W2(C), w3 = W3(C);
    const int W = stage == 0 ? w1 : stage == 1 ? w2 : w3;
    const int wb = stage == 0 ? 0 : stage == 1 ? w1 : w1 + w2;
    if (W == 8) return __byte_perm(w[wb + k / 4], po[k / 3], Sel<k>::v);
    const uint32_t off = ((uint32_t)(lane + k) & 31u) << 2;
    uint32_t f;
    if (stage == 0) {
        constexpr int we = w1 > 1 ? w1 - 1 : 1, pos = we * k, bb = pos % 32;
        f = w[1 + pos / 32] >> bb;
        if (bb + we > 32) f |= w[2 + pos / 32] << ((32 - bb) & 31);
        f = (f & ((1u << we) - 1u)) | (((w[0] >> k) & 1u) << we);
    } else {
        f = (w[wb + (W * k) / 32] >> ((W * k) % 32)) & ((1u << W) - 1u);
    }
    return (f << 8) | off;
}

// V = int: exact integer tables (the chain kernel); V = float: the same integers stored as floats (k_gemv), so the
// per-chunk accumulate runs on the FP32 pipe instead of the integer ALU that the address PRMT already occupies. Stage 1
// alternates two accumulators (even / odd steps) to halve the dependent-add chain; the order is fixed, so the result
// is deterministic.
template <int C, int TOFF, int k, typename V>
struct StepLoop {
    static __device__ __forceinline__ void run(const uint32_t (&w)[24], const uint32_t (&po)[11], int lane, V &a1, V &a1b, V &a2,
                                               V &a3) {
        if (k & 1) a1b += lds_at<TOFF, V>(stage_addr<C, k>(w, po, lane, 0));
        else a1 += lds_at<TOFF, V>(stage_addr<C, k>(w, po, lane, 0));
        if (W2(C)) a2 += lds_at<TOFF, V>(stage_addr<C, k>(w, po, lane, 1));
        if (W3(C)) a3 += lds_at<TOFF, V>(stage_addr<C, k>(w, po, lane, 2));
        StepLoop<C, TOFF, k + 1, V>::run(w, po, lane, a1, a1b, a2, a3);
    }
};
template <int C, int TOFF, typename V>
struct StepLoop<C, TOFF, 32, V> {
    static __device__ __forceinline__ void run(const uint32_t (&)[24], const uint32_t (&)[11], int, V &, V &, V &, V &) {}
};

// z bits (stage-1 MSBs) in step order. For W1 = 8: the byte MSBs of words 2p+1 (bits 7, 15, 23, 31) and 2p (shifted to
// bits 3, 11, 19, 27) are merged, and one multiply by 0x00204081 gathers them into bits 24-27 (word 2p, steps 8p..8p+3)
// and 28-31 (word 2p+1) without carries: every partial-product bit lands on a distinct position.
template <int C>
__device__ __forceinline__ uint32_t zbits_fast(const uint32_t (&w)[24]) {
    if (W1(C) != 8) return w[0];
    uint32_t pm = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const uint32_t x = (w[2 * p + 1] & 0x80808080u) | ((w[2 * p] >> 4) & 0x08080808u);
        pm |= ((x * 0x00204081u) >> 24) << (8 * p);
    }
    return pm;
}

// total of one lane-slice (integer tables: exact; float tables: the same integers summed in fp32, |entry| < 2^22, so each
// add rounds by at most 2^-24 of the running sum); TOFF / GOFF: shared-memory byte offsets of its table and coset tables
template <int C, int TOFF, int GOFF, typename V = int>
__device__ __forceinline__ V lane_slice_dot(const uint32_t (&w)[24], const uint32_t (&po)[11], int lane) {
    const uint32_t pm = zbits_fast<C>(w);
    const uint32_t H = pingala8_h(__funnelshift_l(pm, pm, lane));
    // coset term: nibble grp of H indexes a 16-entry table of group grp; (H >> (4 grp - 2)) & 0x3C is that nibble
    // times 4 (two ops), and grp * 64 folds into the load's offset
    V cs = 0;
#pragma unroll
    for (int grp = 0; grp < 8; ++grp) {
        const uint32_t sh = grp == 0 ? (H << 2) : (H >> (4 * grp - 2));
        cs += lds_at<GOFF, V>((sh & 0x3Cu) + grp * 64);
    }
    V a1 = 0, a1b = 0, a2 = 0, a3 = 0;
    StepLoop<C, TOFF, 0, V>::run(w, po, lane, a1, a1b, a2, a3);
    return (a1 + a1b) * (V)(1 << SH1(C)) + a2 * (V)(1 << SH2(C)) + a3 + (V)MC(C) * cs;
}

// k_gemv's lane-slice sums come from float tables (V = float); the result is scaled by the half-slice scales d0, d1
template <int C, int BUF>
__device__ __forceinline__ float tile_row_dot_w(const uint32_t (&w0)[24], const uint32_t (&w1)[24], const uint32_t (&po)[11], int lane, float d0,
                                                float d1) {
    constexpr int T0 = BUF ? kSmemT1 : kSmemT0, G0 = BUF ? kSmemG1 : kSmemG0;
    const float i0 = lane_slice_dot<C, T0, G0, float>(w0, po, lane);
    const float i1 = lane_slice_dot<C, T0 + 128, G0 + kGInts * 4, float>(w1, po, lane);
    return __fadd_rn(__fmul_rn(i0, d0), __fmul_rn(i1, d1));
}

template <int C, int BUF>
__device__ __noinline__ float tile_row_dot(const uint32_t *p0, const uint32_t (&po)[11], int lane, float d0, float d1) {
    constexpr int T0 = BUF ? kSmemT1 : kSmemT0, G0 = BUF ? kSmemG1 : kSmemG0;
    uint32_t w[24];
    load_lane_words<C>(p0, 0, lane, w);
    const float i0 = lane_slice_dot<C, T0, G0, float>(w, po, lane);
    load_lane_words<C>(p0, 1, lane, w);
    const float i1 = lane_slice_dot<C, T0 + 128, G0 + kGInts * 4, float>(w, po, lane);
    return __fadd_rn(__fmul_rn(i0, d0), __fmul_rn(i1, d1));
}

template <int BUF>
__device__ __forceinline__ float tile_row_other(int c, const uint32_t *p0, const uint32_t (&po)[11], int lane, float d0, float d1) {
    switch (c) {
        case 1: return tile_row_dot<1, BUF>(p0, po, lane, d0, d1);
        case 2: return tile_row_dot<2, BUF>(p0, po, lane, d0, d1);
        case 4: return tile_row_dot<4, BUF>(p0, po, lane, d0, d1);
        case 5: return tile_row_dot<5, BUF>(p0, po, lane, d0, d1);
        case 6: return tile_row_dot<6, BUF>(p0, po, lane, d0, d1);
        case 7: return tile_row_dot<7, BUF>(p0, po, lane, d0, d1);
        default: return 0.f;
    }
}

// class-3 payload of one tile row (both half-slices): 8 words each
__device__ __forceinline__ void load3(const uint32_t *p0, int lane, uint32_t (&v)[16]) {
    const uint2 *q = reinterpret_cast<const uint2 *>(p0) + lane;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint2 u = __ldg(q + i * 32);  // hs 0: i < 4, hs 1: i >= 4 (hs stride = 8 words * 32 lanes = 128 uint2)
        v[2 * i] = u.x;
        v[2 * i + 1] = u.y;
    }
}

__device__ __forceinline__ int tensor_of(const GemvArgs &a, int rr) {
    int ti = 0;
#pragma unroll
    for (int i = 1; i < kMaxGroup; ++i)
        if (i < a.ntensors && rr >= a.t[i].g0) ti = i;
    return ti;
}

// the warp's units of a CTA: per block b (segment), units rr = first + warp + 16 j of [rr_begin(b), rr_end(b)); a
// unit is tile g = rr - g0 of tensor tensor_of(rr). Pure integer bookkeeping, no divisions.
struct WarpCursor {
    int b, rr;  // current unit (256-column block, row tile of the group); exhausted once past the CTA's range
};

// table-build scratch of one k_gemv CTA (static shared memory): x16 ints and coset dot products of up to two blocks,
// the codebook, the per-half-slice scales of each table buffer, the RMSNorm reduction
struct __align__(16) BuildSmem {
    float4 Af[256];  // the codebook as floats (entry f: its four int8 values)
    int q[2][256];
    int cx[2][64];
    float d[2][2];   // [buffer][half-slice]
    float red[kGemvThreads];
};

// chain steps only: the blocks' input values (and SwiGLU up), reduced from the previous step's partials or loaded;
// read as float4 by build_tables, so 16-byte aligned
struct __align__(16) ChainSmem {
    float xin[2][256], x2in[2][256];
};

// The activation tables of blocks bA .. bA + nbld - 1 (nbld <= 2) into table buffers 0 .. nbld - 1 of this CTA's
// shared memory; every thread of the CTA takes part (CTA-uniform call). Per block: x' = x (after the input op) times
// sgn/c, FWHT256 / 16, x16 quantisation per 128-column half-slice (d = amax / 8191, q = rint(x' / d): the reference CPU
// default, vrc_prep_block16 CP:584-616), then
//   T[f][hs][t] = <A[f], q_t> as a float (exact: |T| < 2^23), four fp32 FMAs on the float codebook copy
//   G[hs][grp][m] = sum over the set bits i of nibble m of <c, q_{4 grp + i}> (coset nibble tables, exact)
// The first CTA of a block (the one holding the block's first unit) stores x' for the clamp-delta term.
template <int PRO, bool CH>
__device__ __forceinline__ void build_tables(const GemvArgs &a, BuildSmem &s, const ChainSmem *cs, float *ss_out, int bA, int nbld,
                                             float scale, long long u0, long long u1) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp < nbld) {
        const int i = warp, b = bA + i;
        const float *x = CH ? &cs->xin[i][8 * lane] : a.X + b * 256 + 8 * lane;
        float4 x0 = *reinterpret_cast<const float4 *>(x), x1 = *reinterpret_cast<const float4 *>(x + 4);
        const long long bu = (long long)b * a.ng_total;  // the block's first unit
        if (PRO == P8_PROLOGUE_RMSNORM && CH && ss_out) {  // deferred RMSNorm: the block's sum of x^2 (fixed order)
            float q2 = 0.f;
            q2 = __fmaf_rn(x0.x, x0.x, q2); q2 = __fmaf_rn(x0.y, x0.y, q2); q2 = __fmaf_rn(x0.z, x0.z, q2);
            q2 = __fmaf_rn(x0.w, x0.w, q2); q2 = __fmaf_rn(x1.x, x1.x, q2); q2 = __fmaf_rn(x1.y, x1.y, q2);
            q2 = __fmaf_rn(x1.z, x1.z, q2); q2 = __fmaf_rn(x1.w, x1.w, q2);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) q2 = __fadd_rn(q2, __shfl_down_sync(0xffffffffu, q2, o));
            if (lane == 0 && u0 <= bu && bu < u1) ss_out[b] = q2;
        }
        const float *icp = a.ic + b * 256 + 8 * lane;
        const float4 i0 = *reinterpret_cast<const float4 *>(icp), i1 = *reinterpret_cast<const float4 *>(icp + 4);
        if (PRO == P8_PROLOGUE_RMSNORM) {
            const float4 w0 = *reinterpret_cast<const float4 *>(a.pw + b * 256 + 8 * lane);
            const float4 w1 = *reinterpret_cast<const float4 *>(a.pw + b * 256 + 8 * lane + 4);
            x0 = make_float4(__fmul_rn(__fmul_rn(x0.x, scale), w0.x), __fmul_rn(__fmul_rn(x0.y, scale), w0.y),
                             __fmul_rn(__fmul_rn(x0.z, scale), w0.z), __fmul_rn(__fmul_rn(x0.w, scale), w0.w));
            x1 = make_float4(__fmul_rn(__fmul_rn(x1.x, scale), w1.x), __fmul_rn(__fmul_rn(x1.y, scale), w1.y),
                             __fmul_rn(__fmul_rn(x1.z, scale), w1.z), __fmul_rn(__fmul_rn(x1.w, scale), w1.w));
        } else if (PRO == P8_PROLOGUE_SWIGLU) {  // silu(gate) * up = gate / (1 + exp(-gate)) * up
            const float *x2p = CH ? &cs->x2in[i][8 * lane] : a.x2 + b * 256 + 8 * lane;
            const float4 u0v = *reinterpret_cast<const float4 *>(x2p);
            const float4 u1v = *reinterpret_cast<const float4 *>(x2p + 4);
            auto sw = [](float g, float u) { return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u); };
            x0 = make_float4(sw(x0.x, u0v.x), sw(x0.y, u0v.y), sw(x0.z, u0v.z), sw(x0.w, u0v.w));
            x1 = make_float4(sw(x1.x, u1v.x), sw(x1.y, u1v.y), sw(x1.z, u1v.z), sw(x1.w, u1v.w));
        }
        if (PRO != P8_PROLOGUE_NONE && u0 <= bu && bu < u1) {
            *reinterpret_cast<float4 *>(a.xv + b * 256 + 8 * lane) = x0;
            *reinterpret_cast<float4 *>(a.xv + b * 256 + 8 * lane + 4) = x1;
        }
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
        for (int m = 0; m < 8; ++m) s.q[i][8 * lane + m] = __float2int_rn(__fmul_rn(v[m], id));
        if ((lane & 15) == 0) s.d[i][lane >> 4] = d;
    }
    __syncthreads();
    if (tid < 64 * nbld) {  // <c, q_t> for the 64 chunks of each block
        const int i = tid >> 6, t = tid & 63;
        int cx = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) cx += (int)(int8_t)(a.cs >> (8 * e)) * s.q[i][4 * t + e];
        s.cx[i][t] = cx;
    }
    __syncthreads();
    if (tid < 256 * nbld) {  // a 16-entry group table spans 16 banks: the lookups never conflict (equal m broadcast)
        const int i = tid >> 8, hs = (tid >> 7) & 1, grp = (tid >> 4) & 7, m = tid & 15;
        int gsum = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if ((m >> k) & 1) gsum += s.cx[i][hs * 32 + 4 * grp + k];
        reinterpret_cast<float *>(g_smem + (i ? kSmemG1 : kSmemG0))[hs * kGInts + grp * 16 + m] = (float)gsum;
    }
    // thread = (f mod 8, hs, t): 32 codebook entries f = tid / 64 + 8 j per block, consecutive threads consecutive t.
    // fp32 FMAs on integer values: every product (< 2^20) and partial sum (< 2^23) is exact, so T is the exact integer
    const int ht = tid & 63, f0 = tid >> 6;
    for (int i = 0; i < nbld; ++i) {
        const float q0 = (float)s.q[i][4 * ht], q1 = (float)s.q[i][4 * ht + 1], q2 = (float)s.q[i][4 * ht + 2],
                    q3 = (float)s.q[i][4 * ht + 3];
        float *T = reinterpret_cast<float *>(g_smem + (i ? kSmemT1 : kSmemT0));
#pragma unroll 8
        for (int j = 0; j < 32; ++j) {
            const int f = f0 + 8 * j;
            const float4 w = s.Af[f];
            T[f * 64 + ht] = __fmaf_rn(w.x, q0, __fmaf_rn(w.y, q1, __fmaf_rn(w.z, q2, __fmul_rn(w.w, q3))));
        }
    }
    __syncthreads();
}

// Chained step: the input values of blocks bA .. bA + nbld - 1 into s.xin (and the SwiGLU up into s.x2in), each
// either reduced from the previous step's partials (the block's first CTA also writes those rows of the previous
// output) or loaded from memory. Pass 1 sums the 16-block slices of every (source, block, row) with each slice's loads
// in flight (the slice sums go to the table region, free until the tables are built); pass 2 adds the slices in order
// and applies the clamp delta, the previous step's scale and residual. Every thread of the CTA takes part.
template <int PRO>
__device__ __forceinline__ void chain_inputs(const GemvArgs &a, const ChainIn &ch, ChainSmem &s, int bA, int nbld, float scale_prev,
                                             long long u0, long long u1) {
    const int tid = threadIdx.x;
    const bool px = ch.x.part != nullptr, px2 = PRO == P8_PROLOGUE_SWIGLU && ch.x2.part != nullptr;
    const int S = (ch.nb + 15) / 16;
    float *sl = reinterpret_cast<float *>(g_smem + kSmemT0);  // [src][blk][slice][256]
    const int per_src = nbld * 256 * S;
    const int items = (px ? per_src : 0) + (px2 ? per_src : 0);
    for (int it = tid; it < items; it += kGemvThreads) {
        const int src = px ? (it >= per_src ? 1 : 0) : 1;
        const int r = px ? (it >= per_src ? it - per_src : it) : it;
        const int blk = r / (256 * S), rem = r - blk * 256 * S, j = rem >> 8, i = rem & 255;
        const ChainSrc &T = src ? ch.x2 : ch.x;
        sl[((src * 2 + blk) * S + j) * 256 + i] = slice_sum(T.part, T.rows, ch.nb, 256 * (bA + blk) + i, j);
    }
    for (int it = tid; it < nbld * 256; it += kGemvThreads) {  // sources in memory
        const int blk = it >> 8, i = it & 255, col = 256 * (bA + blk) + i;
        if (!px) s.xin[blk][i] = __ldcg(a.X + col);
        if (PRO == P8_PROLOGUE_SWIGLU && !px2) s.x2in[blk][i] = __ldcg(a.x2 + col);
    }
    __syncthreads();
    const int n2 = (px ? nbld * 256 : 0) + (px2 ? nbld * 256 : 0);
    for (int it = tid; it < n2; it += kGemvThreads) {
        const int src = px ? (it >= nbld * 256 ? 1 : 0) : 1;
        const int r = px ? (it >= nbld * 256 ? it - nbld * 256 : it) : it;
        const int blk = r >> 8, i = r & 255, ro = 256 * (bA + blk) + i;
        const ChainSrc &T = src ? ch.x2 : ch.x;
        const float *q = sl + (src * 2 + blk) * S * 256 + i;
        float y = q[0];
        for (int j = 1; j < S; ++j) y = __fadd_rn(y, q[j * 256]);
        y = chain_row_value(T, ro, y, ch.xv, scale_prev);
        (src ? s.x2in : s.xin)[blk][i] = y;
        const long long bu = (long long)(bA + blk) * a.ng_total;
        if (u0 <= bu && bu < u1) T.Y[ro] = y;  // the block's first CTA writes the previous step's output
    }
    __syncthreads();
}

// Chained step: this CTA's equal share of the previous step's outputs that this step does not read (one thread per
// row, the k_gemv_reduce order)
__device__ __forceinline__ void chain_unconsumed(const ChainIn &ch, float scale_prev) {
    const int ra = (int)((long long)ch.unc_rows * blockIdx.x / gridDim.x), rb = (int)((long long)ch.unc_rows * (blockIdx.x + 1) / gridDim.x);
    const int S = (ch.nb + 15) / 16;
    for (int r = ra + (int)threadIdx.x; r < rb; r += kGemvThreads) {
        int ti = 0, ro = r;
        while (ti + 1 < ch.nunc && ro >= ch.unc[ti].rows) ro -= ch.unc[ti++].rows;
        const ChainSrc &T = ch.unc[ti];
        float y = slice_sum(T.part, T.rows, ch.nb, ro, 0);
        for (int j = 1; j < S; ++j) y = __fadd_rn(y, slice_sum(T.part, T.rows, ch.nb, ro, j));
        T.Y[ro] = chain_row_value(T, ro, y, ch.xv, scale_prev);
    }
}

// One CTA per SM at most (512 threads, 104 registers: 16 warps leave room for a k_gemv_reduce CTA beside it). Each
// CTA takes the contiguous range [ustart[c], ustart[c + 1]) of the block-major unit list (host-balanced: a unit
// counts one, every extra block touched counts the cost of building its table) and builds the tables of the blocks
// it touches in its own shared memory, two at a time; warp w takes units u0 + w, u0 + w + 16, ... The row partials
// go to part[b][ro] (original row ro = prm[r]); k_gemv_reduce (the next kernel) sums them.
template <int PRO, bool CH>
__device__ __forceinline__ void gemv_body(const GemvArgs &a, const ChainIn *chp) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ BuildSmem bs;
    ChainSmem *cs = nullptr;
    if constexpr (CH) {
        __shared__ ChainSmem chs;
        cs = &chs;
    }
    const long long u0 = a.ustart[blockIdx.x], u1 = a.ustart[blockIdx.x + 1];
    pdl_launch_dependents();
    if (u1 <= u0) return;
    const int b_first = (int)(u0 / a.ng_total), b_last = (int)((u1 - 1) / a.ng_total);
    const int rr_first = (int)(u0 - (long long)b_first * a.ng_total);             // first unit's rr in block b_first
    const int rr_last_end = (int)(u1 - (long long)b_last * a.ng_total);           // end rr in block b_last
    const int nseg = b_last - b_first + 1;
    uint32_t po[11];
#pragma unroll
    for (int q = 0; q < 11; ++q) {
        uint32_t r = 0;
#pragma unroll
        for (int i = 0; i < 3; ++i)
            if (3 * q + i < 32) r |= (((uint32_t)(lane + 3 * q + i) & 31u) << 2) << (8 * i);
        po[q] = r;
    }
    if (tid < 256) {  // the codebook belongs to the tensors: converted before the wait
        const uint32_t w = __ldg(a.A + tid);
        bs.Af[tid] = make_float4((float)(int8_t)w, (float)(int8_t)(w >> 8), (float)(int8_t)(w >> 16), (float)(int8_t)(w >> 24));
    }
    // ---- this warp's cursor (global order) and its first units' M words, payload and scale. The weights are not
    // written by earlier kernels of the stream, so these loads are issued before the wait for the producer of x.
    auto in_range = [&](const WarpCursor &c) { return c.b < b_last || (c.b == b_last && c.rr < rr_last_end); };
    auto advance = [&](WarpCursor c) -> WarpCursor {
        c.rr += kGemvWarps;
        while (c.rr >= a.ng_total) {
            c.rr -= a.ng_total;
            ++c.b;
        }
        return c;
    };
    auto m_of = [&](const WarpCursor &c) -> uint32_t {
        const int ti = tensor_of(a, c.rr);
        const uint32_t tile = (uint32_t)(c.rr - a.t[ti].g0) * (uint32_t)a.nb + (uint32_t)c.b;
        const int uc = a.t[ti].ucls;
        if (uc) return (tile * (uint32_t)(64 * NW(uc))) | ((uint32_t)uc << 29);
        return __ldg(a.t[ti].M + tile);
    };
    uint32_t nxt[16];
    uint32_t mt_n = 0, mt_nn = 0;
    uint16_t s_n = 0;
    int16_t p_n = 0;
    auto fetch = [&](const WarpCursor &c, uint32_t mt) {  // payload + row scale of unit c (its M word known)
        const int ti = tensor_of(a, c.rr), g = c.rr - a.t[ti].g0;
        if ((mt >> 29) == 3) load3(a.t[ti].D + (mt & 0x1FFFFFFFu), lane, nxt);
        s_n = __ldg(a.t[ti].S + (size_t)c.b * a.t[ti].rows + g * 32 + lane);
        p_n = __ldg(a.t[ti].prm + g * 32 + lane);  // the row's original position: partials are stored there
    };
    WarpCursor nc = {b_first, rr_first + warp};
    while (nc.rr >= a.ng_total) {
        nc.rr -= a.ng_total;
        ++nc.b;
    }
    WarpCursor nc2 = nc;
    if (in_range(nc)) {
        mt_n = m_of(nc);
        fetch(nc, mt_n);
        nc2 = advance(nc);
        if (in_range(nc2)) mt_nn = m_of(nc2);
    }
    pdl_wait();  // x (and the row-parallel call counter) belong to the preceding kernel until it completes
    if (a.epoch && blockIdx.x == 0 && tid == 0) *a.epoch += 1u;  // k_gemv_reduce reads it after this kernel completes
    __shared__ float s_scale_prev;
    if (CH && tid == 0) s_scale_prev = chp->ss ? deferred_scale(chp->ss, chp->nb, chp->K, chp->eps) : 1.f;
    // chain phase stamps (read from the parameters when taken: no register held across the unit loop)
    auto stamp = [&](int k) {
        if constexpr (CH)
            if (chp->trace && threadIdx.x == 0) chp->trace[(size_t)blockIdx.x * 8 + k] = global_ns();
    };
    stamp(0);
    float scale = 1.f;  // a deferred RMSNorm (ss_out) builds the tables from x * w and scales the outputs later
    if (PRO == P8_PROLOGUE_RMSNORM && !(CH && chp->ss_out)) scale = rms_scale<kGemvThreads>(a.X, a.K, a.eps, bs.red);
    // segments (blocks) two at a time: build their tables (buffers 0, 1), run the warp's units in them; a CTA spans
    // more than two blocks only when nb > the number of CTAs
    for (int ph = 0; 2 * ph < nseg; ++ph) {
        if (ph > 0) __syncthreads();  // every warp is done with the previous pair of tables
        if (CH) {
            if (ph == 0) __syncthreads();  // s_scale_prev
            chain_inputs<PRO>(a, *chp, *cs, b_first + 2 * ph, nseg - 2 * ph < 2 ? nseg - 2 * ph : 2, s_scale_prev, u0, u1);
        }
        if (ph == 0) stamp(1), stamp(2);
        build_tables<PRO, CH>(a, bs, cs, CH ? chp->ss_out : nullptr, b_first + 2 * ph, nseg - 2 * ph < 2 ? nseg - 2 * ph : 2, scale, u0,
                              u1);
        if (ph == 0) stamp(3);
        const int seg_end = 2 * ph + 2;
        while (in_range(nc) && nc.b - b_first < seg_end) {
            const int seg = nc.b - b_first;
            const int b = nc.b, rr = nc.rr;
            const float d0 = bs.d[seg & 1][0], d1 = bs.d[seg & 1][1];
            const uint32_t mt = mt_n;
            const uint16_t sc = s_n;
            const int ro = p_n;
            uint32_t cur[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) cur[i] = nxt[i];
            nc = nc2;
            mt_n = mt_nn;
            if (in_range(nc)) {
                fetch(nc, mt_n);  // possibly in the next segment
                nc2 = advance(nc);
                if (in_range(nc2)) mt_nn = m_of(nc2);
            }
            const GemvTensor &T = a.t[tensor_of(a, rr)];
            const int c = (int)(mt >> 29);
            float part;
            if (c == 3) {
                uint32_t w0[24], w1[24];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    w0[2 * i] = cur[2 * i]; w0[2 * i + 1] = cur[2 * i + 1];
                    w1[2 * i] = cur[8 + 2 * i]; w1[2 * i + 1] = cur[8 + 2 * i + 1];
                }
#pragma unroll
                for (int i = 8; i < 24; ++i) { w0[i] = 0; w1[i] = 0; }
                part = (seg & 1) ? tile_row_dot_w<3, 1>(w0, w1, po, lane, d0, d1) : tile_row_dot_w<3, 0>(w0, w1, po, lane, d0, d1);
            } else {
                const uint32_t *p0 = T.D + (mt & 0x1FFFFFFFu);
                part = (seg & 1) ? tile_row_other<1>(c, p0, po, lane, d0, d1) : tile_row_other<0>(c, p0, po, lane, d0, d1);
            }
            T.part[(size_t)b * T.rows + ro] = __fmul_rn(part, h2f(sc));
        }
    }
    if constexpr (CH) {
        if (chp->trace) {
            __syncthreads();
            stamp(4);
        }
        if (chp->nunc) chain_unconsumed(*chp, s_scale_prev);
        stamp(5);
    }
}

template <int PRO>
__global__ void __maxnreg__(104) k_gemv(const __grid_constant__ GemvArgs a) {
    gemv_body<PRO, false>(a, nullptr);
}
// a chain step (p8_chain.cuh): the same kernel with the previous step's outputs as its input
template <int PRO>
__global__ void __maxnreg__(104) k_gemv_chain(const __grid_constant__ GemvArgs a, const __grid_constant__ ChainIn ch) {
    gemv_body<PRO, true>(a, &ch);
}

// One thread per (row, block slice): a row's blocks are cut into S = ceil(nb / 16) slices of 16 (the last one
// shorter); slice j sums blocks [16 j, 16 j + 16) of its row in block order with all its loads in flight, then one
// thread adds the S slice sums in slice order, adds the clamp delta sum_e val_e x[col_e] and stores y[ro] (with
// the row-parallel exchange first for TPX). The summation order depends on nb alone -- not on the grid, the group or
// the rows per CTA -- so every entry point that computes a row gets the same bits.
constexpr int kRedThreads = 256;
constexpr int kRedRowsPerCta = 32;
constexpr int kRedSlice = 16;

// CHN: a chain's last step (its deferred RMSNorm scale and residuals); a separate instantiation, so the per-op reduce
// carries none of it
template <bool TPX, bool CHN = false>
__global__ void __launch_bounds__(kRedThreads, 5) k_gemv_reduce(const __grid_constant__ ReduceArgs a) {
    const int tid = threadIdx.x;
    __shared__ float red[kRedThreads];
    pdl_launch_dependents();
    const int r0 = (int)((long long)a.rows_total * blockIdx.x / gridDim.x), r1 = (int)((long long)a.rows_total * (blockIdx.x + 1) / gridDim.x);
    const int n_rows = r1 - r0;
    const int S = (a.nb + kRedSlice - 1) / kRedSlice;  // <= 16 for K <= 65536
    const int R = min(n_rows, kRedThreads / S);         // rows per pass
    const int rl = R > 0 ? tid % R : 0, sl = R > 0 ? tid / R : S;
    // the combining threads' row metadata (permutation, clamp-delta range) belongs to the tensors: loaded before the wait
    int c_ti = 0, c_ro = 0, c_e0 = 0, c_e1 = 0;
    if (tid < R) {
        const int rt = r0 + tid;
#pragma unroll
        for (int i = 1; i < kMaxGroup; ++i)
            if (i < a.ntensors && rt >= a.t[i].row0) c_ti = i;
        const GemvTensor &T = a.t[c_ti];
        c_ro = rt - T.row0;
        c_e0 = T.cp[c_ro];
        c_e1 = T.cp[c_ro + 1];
    }
    pdl_wait();  // the partials (and x' of an input op) come from k_gemv
    __shared__ float s_scale;
    if (CHN && a.ss && tid == 0) s_scale = deferred_scale(a.ss, a.nb, a.ssK, a.eps);  // read after the loop's first barrier
    constexpr bool tpx = TPX;
    const unsigned int par = tpx ? (__ldcg(a.tp.epoch) & 1u) : 0u;  // advanced by this call's k_gemv
    const unsigned long long deadline = tpx ? global_ns() + a.tp.timeout_ns : 0ull;
    bool tp_ok = true;
    const int b_lo = kRedSlice * sl, b_hi = min(a.nb, kRedSlice * (sl + 1));
    for (int base = r0; base < r1; base += R) {
        const int rt = base + rl;
        float s = 0.f;
        if (sl < S && rt < r1) {
            int ti = 0;
#pragma unroll
            for (int i = 1; i < kMaxGroup; ++i)
                if (i < a.ntensors && rt >= a.t[i].row0) ti = i;
            const GemvTensor &T = a.t[ti];
            const float *p = T.part + (rt - T.row0);
            int bb = b_lo;
            for (; bb + 16 <= b_hi; bb += 16) {
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __ldcg(p + (size_t)(bb + j) * T.rows);
#pragma unroll
                for (int j = 0; j < 16; ++j) s = __fadd_rn(s, v[j]);
            }
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = bb + j < b_hi ? __ldcg(p + (size_t)(bb + j) * T.rows) : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (bb + j < b_hi) s = __fadd_rn(s, v[j]);
        }
        if (sl < S) red[sl * R + rl] = s;
        __syncthreads();
        if (tid < R && base + tid < r1) {
            float y = red[tid];
            for (int j = 1; j < S; ++j) y = __fadd_rn(y, red[j * R + tid]);
            const int rt2 = base + tid;
            if (base != r0) {  // rows past the first pass: metadata loaded here
                c_ti = 0;
#pragma unroll
                for (int i = 1; i < kMaxGroup; ++i)
                    if (i < a.ntensors && rt2 >= a.t[i].row0) c_ti = i;
                const GemvTensor &T = a.t[c_ti];
                c_ro = rt2 - T.row0;
                c_e0 = T.cp[c_ro];
                c_e1 = T.cp[c_ro + 1];
            }
            const GemvTensor &T = a.t[c_ti];
            for (int e = c_e0; e < c_e1; ++e) y = __fadd_rn(y, __fmul_rn(T.cv[e], a.X[T.cc[e]]));
            if (CHN) {  // a chain's last step: its deferred RMSNorm scale and its residual
                if (a.ss) y = __fmul_rn(y, s_scale);
                if (T.res) y = __fadd_rn(y, __ldcg(T.res + c_ro));
            }
            if (tpx) y = tp_exchange_row(a.tp, par, c_ro, c_ro, y, deadline, tp_ok);
            T.Y[c_ro] = y;
        }
        __syncthreads();
    }
}

// ================================================================================================================
// Two columns at once (batched decode of 2 or 3 sequences): the weights are decoded once for both columns. The two
// columns' tables of a block are interleaved as float2, T2[hs][f][t] (64 KiB per half-slice, both half-slices = the
// two table buffers of k_gemv), so one PRMT-built address and one 64-bit lookup per 4-weight chunk serve both columns;
// the coset tables likewise (G2[hs][grp][m]). A CTA works on one block at a time. Class-3 tensors in the uniform
// layout only (the synthetic and class-3 model files); other tensors take the per-column path.
// ================================================================================================================
constexpr int kG2Off = 2 * 65536;                  // G2 after the two half-slice tables
constexpr int kGemv2Smem = kG2Off + 2 * 1024;       // G2: [hs][8 groups][16][2] floats

struct __align__(16) Build2Smem {
    float4 Af[256];     // the codebook as floats
    int q[2][256];      // x16 ints per column
    int cx[2][64];      // <c, q_t> per column
    float d[2][2];      // [column][half-slice]
    float red[kGemvThreads];
};

// the lane's chunk offsets for the float2 tables: po byte i of word q = ((lane + 3 q + i) & 31) * 8
__device__ __forceinline__ void po2_init(uint32_t (&po)[11], int lane) {
#pragma unroll
    for (int q = 0; q < 11; ++q) {
        uint32_t r = 0;
#pragma unroll
        for (int i = 0; i < 3; ++i)
            if (3 * q + i < 32) r |= (((uint32_t)(lane + 3 * q + i) & 31u) << 3) << (8 * i);
        po[q] = r;
    }
}

// half-slice HS of a class-3 unit row for both columns: table sum (steps alternate two accumulators) + coset term
template <int HS, int k>
struct Step2 {
    static __device__ __forceinline__ void run(const uint32_t (&w)[16], const uint32_t (&po)[11], float2 &a, float2 &b) {
        const float2 v = *reinterpret_cast<const float2 *>(g_smem + HS * 65536 + __byte_perm(w[8 * HS + k / 4], po[k / 3], Sel<k>::v));
        if (k & 1) { b.x += v.x; b.y += v.y; } else { a.x += v.x; a.y += v.y; }
        Step2<HS, k + 1>::run(w, po, a, b);
    }
};
template <int HS>
struct Step2<HS, 32> {
    static __device__ __forceinline__ void run(const uint32_t (&)[16], const uint32_t (&)[11], float2 &, float2 &) {}
};
template <int HS>
__device__ __forceinline__ float2 slice2(const uint32_t (&w)[16], const uint32_t (&po)[11], int lane) {
    uint32_t pm = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {  // z bits in step order (as zbits_fast)
        const uint32_t x = (w[8 * HS + 2 * p + 1] & 0x80808080u) | ((w[8 * HS + 2 * p] >> 4) & 0x08080808u);
        pm |= ((x * 0x00204081u) >> 24) << (8 * p);
    }
    const uint32_t H = pingala8_h(__funnelshift_l(pm, pm, lane));
    float2 cs = make_float2(0.f, 0.f);
#pragma unroll
    for (int grp = 0; grp < 8; ++grp) {  // nibble grp of H times 8 bytes
        const uint32_t sh = grp == 0 ? (H << 3) : (H >> (4 * grp - 3));
        const float2 v = *reinterpret_cast<const float2 *>(g_smem + kG2Off + HS * 1024 + grp * 128 + (sh & 0x78u));
        cs.x += v.x;
        cs.y += v.y;
    }
    float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
    Step2<HS, 0>::run(w, po, a, b);
    return make_float2((a.x + b.x) + cs.x, (a.y + b.y) + cs.y);  // class 3: one stage, no shift, coset multiplicity 1
}

// both columns' tables of block b: warp c (c < 2) prepares column c's x16 ints; then coset and the interleaved table
template <int PRO>
__device__ __forceinline__ void build_tables2(const GemvArgs &a, Build2Smem &s, int b, const float (&scale)[2], long long u0,
                                              long long u1) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp < 2) {
        const int c = warp;
        const float *x = a.X + (size_t)c * a.ldx + b * 256 + 8 * lane;
        float4 x0 = *reinterpret_cast<const float4 *>(x), x1 = *reinterpret_cast<const float4 *>(x + 4);
        const float *icp = a.ic + b * 256 + 8 * lane;
        const float4 i0 = *reinterpret_cast<const float4 *>(icp), i1 = *reinterpret_cast<const float4 *>(icp + 4);
        if (PRO == P8_PROLOGUE_RMSNORM) {
            const float sc = scale[c];
            const float4 w0 = *reinterpret_cast<const float4 *>(a.pw + b * 256 + 8 * lane);
            const float4 w1 = *reinterpret_cast<const float4 *>(a.pw + b * 256 + 8 * lane + 4);
            x0 = make_float4(__fmul_rn(__fmul_rn(x0.x, sc), w0.x), __fmul_rn(__fmul_rn(x0.y, sc), w0.y),
                             __fmul_rn(__fmul_rn(x0.z, sc), w0.z), __fmul_rn(__fmul_rn(x0.w, sc), w0.w));
            x1 = make_float4(__fmul_rn(__fmul_rn(x1.x, sc), w1.x), __fmul_rn(__fmul_rn(x1.y, sc), w1.y),
                             __fmul_rn(__fmul_rn(x1.z, sc), w1.z), __fmul_rn(__fmul_rn(x1.w, sc), w1.w));
        } else if (PRO == P8_PROLOGUE_SWIGLU) {
            const float *x2p = a.x2 + (size_t)c * a.ldx + b * 256 + 8 * lane;
            const float4 u0v = *reinterpret_cast<const float4 *>(x2p), u1v = *reinterpret_cast<const float4 *>(x2p + 4);
            auto sw = [](float g, float u) { return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u); };
            x0 = make_float4(sw(x0.x, u0v.x), sw(x0.y, u0v.y), sw(x0.z, u0v.z), sw(x0.w, u0v.w));
            x1 = make_float4(sw(x1.x, u1v.x), sw(x1.y, u1v.y), sw(x1.z, u1v.z), sw(x1.w, u1v.w));
        }
        const long long bu = (long long)b * a.ng_total;
        if (PRO != P8_PROLOGUE_NONE && u0 <= bu && bu < u1) {
            float *xv = a.xv + (size_t)c * a.K + b * 256 + 8 * lane;
            *reinterpret_cast<float4 *>(xv) = x0;
            *reinterpret_cast<float4 *>(xv + 4) = x1;
        }
        float v[8] = {__fmul_rn(x0.x, i0.x), __fmul_rn(x0.y, i0.y), __fmul_rn(x0.z, i0.z), __fmul_rn(x0.w, i0.w),
                      __fmul_rn(x1.x, i1.x), __fmul_rn(x1.y, i1.y), __fmul_rn(x1.z, i1.z), __fmul_rn(x1.w, i1.w)};
        fwht256_warp(v, lane);
        float am = 0.f;
#pragma unroll
        for (int m = 0; m < 8; ++m) am = fmaxf(am, fabsf(v[m]));
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const float d = __fdiv_rn(am, 8191.f), id = d > 0.f ? __fdiv_rn(1.f, d) : 0.f;
#pragma unroll
        for (int m = 0; m < 8; ++m) s.q[c][8 * lane + m] = __float2int_rn(__fmul_rn(v[m], id));
        if ((lane & 15) == 0) s.d[c][lane >> 4] = d;
    }
    __syncthreads();
    if (tid < 128) {
        const int c = tid >> 6, t = tid & 63;
        int cx = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) cx += (int)(int8_t)(a.cs >> (8 * e)) * s.q[c][4 * t + e];
        s.cx[c][t] = cx;
    }
    __syncthreads();
    {  // G2[hs][grp][m][c]: thread (c, hs, grp, m)
        const int c = tid >> 8, hs = (tid >> 7) & 1, grp = (tid >> 4) & 7, m = tid & 15;
        int gsum = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if ((m >> k) & 1) gsum += s.cx[c][hs * 32 + 4 * grp + k];
        reinterpret_cast<float *>(g_smem + kG2Off)[((hs * 8 + grp) * 16 + m) * 2 + c] = (float)gsum;
    }
    // T2[hs][f][t] = (<A[f], q0_t>, <A[f], q1_t>): thread (chunk ht, f mod 8), 32 entries, one 8-byte store each
    const int ht = tid & 63, f0 = tid >> 6, hs = ht >> 5, t = ht & 31;
    const float q00 = (float)s.q[0][4 * ht], q01 = (float)s.q[0][4 * ht + 1], q02 = (float)s.q[0][4 * ht + 2], q03 = (float)s.q[0][4 * ht + 3];
    const float q10 = (float)s.q[1][4 * ht], q11 = (float)s.q[1][4 * ht + 1], q12 = (float)s.q[1][4 * ht + 2], q13 = (float)s.q[1][4 * ht + 3];
    uint8_t *T = g_smem + hs * 65536 + t * 8;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
        const int f = f0 + 8 * j;
        const float4 w = s.Af[f];
        *reinterpret_cast<float2 *>(T + f * 256) =
            make_float2(__fmaf_rn(w.x, q00, __fmaf_rn(w.y, q01, __fmaf_rn(w.z, q02, __fmul_rn(w.w, q03)))),
                        __fmaf_rn(w.x, q10, __fmaf_rn(w.y, q11, __fmaf_rn(w.z, q12, __fmul_rn(w.w, q13)))));
    }
    __syncthreads();
}

// Two-column GEMV: the k_gemv unit loop with both columns' sums per unit; partials [column][b][rows] per tensor
// (column 1 at part + nb * rows), rows at their original positions. A CTA's blocks one at a time.
template <int PRO>
__global__ void __maxnreg__(104) k_gemv2(const __grid_constant__ GemvArgs a) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ Build2Smem bs;
    const long long u0 = a.ustart[blockIdx.x], u1 = a.ustart[blockIdx.x + 1];
    pdl_launch_dependents();
    if (u1 <= u0) return;
    const int b_first = (int)(u0 / a.ng_total), b_last = (int)((u1 - 1) / a.ng_total);
    const int rr_first = (int)(u0 - (long long)b_first * a.ng_total);
    const int rr_last_end = (int)(u1 - (long long)b_last * a.ng_total);
    uint32_t po[11];
    po2_init(po, lane);
    if (tid < 256) {  // the codebook belongs to the tensors: converted before the wait
        const uint32_t w = __ldg(a.A + tid);
        bs.Af[tid] = make_float4((float)(int8_t)w, (float)(int8_t)(w >> 8), (float)(int8_t)(w >> 16), (float)(int8_t)(w >> 24));
    }
    auto in_range = [&](const WarpCursor &c) { return c.b < b_last || (c.b == b_last && c.rr < rr_last_end); };
    auto advance = [&](WarpCursor c) -> WarpCursor {
        c.rr += kGemvWarps;
        while (c.rr >= a.ng_total) {
            c.rr -= a.ng_total;
            ++c.b;
        }
        return c;
    };
    uint32_t nxt[16];
    uint16_t s_n = 0;
    int16_t p_n = 0;
    auto fetch = [&](const WarpCursor &c) {  // class-3 uniform: payload of tile g * nb + b at word tile * 512
        const int ti = tensor_of(a, c.rr), g = c.rr - a.t[ti].g0;
        const uint32_t tile = (uint32_t)g * (uint32_t)a.nb + (uint32_t)c.b;
        load3(a.t[ti].D + (size_t)tile * 512, lane, nxt);
        s_n = __ldg(a.t[ti].S + (size_t)c.b * a.t[ti].rows + g * 32 + lane);
        p_n = __ldg(a.t[ti].prm + g * 32 + lane);
    };
    WarpCursor nc = {b_first, rr_first + warp};
    while (nc.rr >= a.ng_total) {
        nc.rr -= a.ng_total;
        ++nc.b;
    }
    if (in_range(nc)) fetch(nc);
    pdl_wait();  // x belongs to the preceding kernel until it completes
    float scale[2] = {1.f, 1.f};
    if (PRO == P8_PROLOGUE_RMSNORM) {
        scale[0] = rms_scale<kGemvThreads>(a.X, a.K, a.eps, bs.red);
        __syncthreads();
        scale[1] = rms_scale<kGemvThreads>(a.X + a.ldx, a.K, a.eps, bs.red);
    }
    for (int b = b_first; b <= b_last; ++b) {
        if (b > b_first) __syncthreads();  // every warp is done with the previous block's tables
        build_tables2<PRO>(a, bs, b, scale, u0, u1);
        const float d00 = bs.d[0][0], d01 = bs.d[0][1], d10 = bs.d[1][0], d11 = bs.d[1][1];
        while (in_range(nc) && nc.b == b) {
            const int rr = nc.rr;
            const uint16_t sc = s_n;
            const int ro = p_n;
            uint32_t cur[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) cur[i] = nxt[i];
            nc = advance(nc);
            if (in_range(nc)) fetch(nc);
            const GemvTensor &T = a.t[tensor_of(a, rr)];
            const float2 i0 = slice2<0>(cur, po, lane), i1 = slice2<1>(cur, po, lane);
            const float s = h2f(sc);
            T.part[(size_t)b * T.rows + ro] = __fmul_rn(__fadd_rn(__fmul_rn(i0.x, d00), __fmul_rn(i1.x, d01)), s);
            T.part[(size_t)(a.nb + b) * T.rows + ro] = __fmul_rn(__fadd_rn(__fmul_rn(i0.y, d10), __fmul_rn(i1.y, d11)), s);
        }
    }
}

// the rows of a two-column call: virtual row r of [0, 2 rows_total) is column r / rows_total; the same slice order as
// k_gemv_reduce, so each column's outputs equal a one-column call's bit for bit
struct Reduce2Args {
    ReduceArgs r;          // column 0's view (X: column 0's x or x')
    long long ldy[kMaxGroup];
    const float *X1;       // column 1's x or x'
};
__global__ void __launch_bounds__(kRedThreads, 5) k_gemv_reduce2(const __grid_constant__ Reduce2Args A) {
    const ReduceArgs &a = A.r;
    const int tid = threadIdx.x;
    __shared__ float red[kRedThreads];
    pdl_launch_dependents();
    const int total = 2 * a.rows_total;
    const int r0 = (int)((long long)total * blockIdx.x / gridDim.x), r1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
    const int n_rows = r1 - r0;
    const int S = (a.nb + kRedSlice - 1) / kRedSlice;
    const int R = min(n_rows, kRedThreads / S);
    const int rl = R > 0 ? tid % R : 0, sl = R > 0 ? tid / R : S;
    pdl_wait();  // the partials (and x' of an input op) come from k_gemv2
    const int b_lo = kRedSlice * sl, b_hi = min(a.nb, kRedSlice * (sl + 1));
    auto locate = [&](int vr, int &c, int &ti, int &ro) {
        c = vr >= a.rows_total ? 1 : 0;
        const int rt = vr - c * a.rows_total;
        ti = 0;
#pragma unroll
        for (int i = 1; i < kMaxGroup; ++i)
            if (i < a.ntensors && rt >= a.t[i].row0) ti = i;
        ro = rt - a.t[ti].row0;
    };
    for (int base = r0; base < r1; base += R) {
        const int vr = base + rl;
        float s = 0.f;
        if (sl < S && vr < r1) {
            int c, ti, ro;
            locate(vr, c, ti, ro);
            const GemvTensor &T = a.t[ti];
            const float *p = T.part + (size_t)c * a.nb * T.rows + ro;
            int bb = b_lo;
            for (; bb + 16 <= b_hi; bb += 16) {
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __ldcg(p + (size_t)(bb + j) * T.rows);
#pragma unroll
                for (int j = 0; j < 16; ++j) s = __fadd_rn(s, v[j]);
            }
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = bb + j < b_hi ? __ldcg(p + (size_t)(bb + j) * T.rows) : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (bb + j < b_hi) s = __fadd_rn(s, v[j]);
        }
        if (sl < S) red[sl * R + rl] = s;
        __syncthreads();
        if (tid < R && base + tid < r1) {
            float y = red[tid];
            for (int j = 1; j < S; ++j) y = __fadd_rn(y, red[j * R + tid]);
            int c, ti, ro;
            locate(base + tid, c, ti, ro);
            const GemvTensor &T = a.t[ti];
            const float *X = c ? A.X1 : a.X;
            const int e1 = T.cp[ro + 1];
            for (int e = T.cp[ro]; e < e1; ++e) y = __fadd_rn(y, __fmul_rn(T.cv[e], X[T.cc[e]]));
            T.Y[(size_t)c * A.ldy[ti] + ro] = y;
        }
        __syncthreads();
    }
}

// workspace layout (bytes, each part 256-aligned): x' of an input op | partials ([nb][rows] per tensor)
struct GemvWs {
    size_t xv, part, total;
};
static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }
// nc = 2: the two-column kernel's x' of both columns and partials [column][nb][rows] per tensor
static GemvWs gemv_ws_layout(const p8_tensor *const *ts, int nt, int nc = 1) {
    const p8_tensor *t = ts[0];
    size_t part = 0;
    for (int i = 0; i < nt; ++i) part += al256((size_t)nc * ts[i]->nb * ts[i]->rows * 4);
    GemvWs w;
    w.xv = 0;
    w.part = w.xv + al256((size_t)nc * t->K * 4);
    w.total = w.part + part;
    return w;
}
size_t gemv_workspace(const p8_tensor *t, int64_t ncols) { return gemv_ws_layout(&t, 1, ncols >= 2 ? 2 : 1).total; }
size_t gemv_group_workspace(const p8_tensor *const *ts, int nt, int64_t ncols) {
    return gemv_ws_layout(ts, nt, ncols >= 2 ? 2 : 1).total;
}

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

// SM count of the current device; the first call on a device also raises the GEMV kernels' shared-memory limit there.
// The cache entry is published only after the attributes are set, so a second host thread never launches before them
// (two threads racing on a first call both set the attributes, which is harmless).
static int sm_count() {
    static std::atomic<int> n[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    int v = n[dev].load(std::memory_order_acquire);
    if (!v) {
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        if (v <= 0) v = 148;
        cudaFuncSetAttribute(k_gemv<P8_PROLOGUE_NONE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmem);
        cudaFuncSetAttribute(k_gemv2<P8_PROLOGUE_NONE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemv2Smem);
        cudaFuncSetAttribute(k_gemv2<P8_PROLOGUE_RMSNORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemv2Smem);
        cudaFuncSetAttribute(k_gemv2<P8_PROLOGUE_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemv2Smem);
        cudaFuncSetAttribute(k_gemv_chain<P8_PROLOGUE_NONE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmem);
        cudaFuncSetAttribute(k_gemv<P8_PROLOGUE_RMSNORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmem);
        cudaFuncSetAttribute(k_gemv_chain<P8_PROLOGUE_RMSNORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmem);
        cudaFuncSetAttribute(k_gemv<P8_PROLOGUE_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmem);
        cudaFuncSetAttribute(k_gemv_chain<P8_PROLOGUE_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmem);
        n[dev].store(v, std::memory_order_release);
    }
    return v;
}

// Cut the block-major list of `units` units (ng per block) into at most P contiguous CTA ranges that minimise the
// largest CTA cost, cost = units taken + kTableCost per block touched (a table build costs about that many units of
// work). Greedy filling under a bound, binary search on the bound. Returns the CTAs used; ustart[0 .. used] is filled.
// The weight was measured on the Llama-3.1-8B decode step: 5 -> 763, 8 -> 789, 11 -> 788, 14 -> 783 tok/s (the small
// q/k/v and o calls gain most: fewer CTAs build two tables).
constexpr int kTableCost = 8;
static int partition_units(long long units, long long ng, int P, int *ustart, int tcost = kTableCost) {
    auto fill = [&](long long C, int *out) -> int {  // CTAs needed under bound C (P + 1 if more than P)
        long long s = 0;
        int c = 0;
        if (out) out[0] = 0;
        while (s < units) {
            if (c == P) return P + 1;
            long long e = s, cost = 0;
            while (e < units) {
                const long long blk_end = std::min(units, (e / ng + 1) * ng);
                if (cost + tcost + 1 > C) break;
                const long long take = std::min(blk_end - e, C - cost - tcost);
                e += take;
                cost += tcost + take;
                if (e < blk_end) break;
            }
            if (e == s) return P + 1;
            s = e;
            ++c;
            if (out) out[c] = (int)s;
        }
        return c;
    };
    long long lo = (units + P - 1) / P + tcost, hi = units + tcost * (units / ng + 2);
    while (lo < hi) {
        const long long mid = (lo + hi) / 2;
        if (fill(mid, nullptr) <= P) hi = mid;
        else lo = mid + 1;
    }
    return fill(lo, ustart);
}

// one column: k_gemv (tables, units, partials) + k_gemv_reduce (rows), both with programmatic dependent launch
static p8_status launch_gemv_col(const p8_tensor *const *ts, int nt, const float *x, float *const *Ys, void *ws, size_t ws_bytes,
                                 cudaStream_t st, const TpExchange *tp = nullptr, unsigned int *epoch = nullptr,
                                 const p8_prologue *pro = nullptr) {
    const p8_tensor *t0 = ts[0];
    const GemvWs L = gemv_ws_layout(ts, nt);
    if (!ws || ws_bytes < L.total) return P8_ERR_WORKSPACE;
    uint8_t *w = static_cast<uint8_t *>(ws);
    const int nsm = sm_count();
    const int pk = pro ? pro->kind : P8_PROLOGUE_NONE;
    GemvArgs ga;
    memset(&ga, 0, sizeof(ga));
    ReduceArgs ra;
    memset(&ra, 0, sizeof(ra));
    ga.ntensors = nt;
    ga.X = x;
    ga.ic = t0->ic;
    ga.A = t0->A;
    ga.cs = t0->cs;
    ga.K = t0->K;
    ga.nb = t0->nb;
    ga.nsl = t0->nsl;
    if (pk != P8_PROLOGUE_NONE) {
        ga.pw = pro->w;
        ga.x2 = pro->x2;
        ga.eps = pro->eps;
        ga.xv = reinterpret_cast<float *>(w + L.xv);
    }
    ga.epoch = tp ? epoch : nullptr;
    size_t poff = L.part;
    int g0 = 0;
    for (int i = 0; i < nt; ++i) {
        const p8_tensor *t = ts[i];
        GemvTensor &g = ga.t[i];
        g.M = t->M; g.D = t->D; g.S = t->S; g.prm = t->prm; g.cp = t->cp; g.cc = t->cc; g.cv = t->cv;
        g.Y = Ys[i];
        g.part = reinterpret_cast<float *>(w + poff);
        poff += al256((size_t)t->nb * t->rows * 4);
        g.rows = t->rows; g.ng = t->ng; g.g0 = g0; g.row0 = ga.rows_total; g.ucls = t->uniform_class;
        g0 += t->ng;
        ga.rows_total += t->rows;
        ra.t[i] = g;
    }
    ga.ng_total = g0;
    ga.units = (long long)g0 * t0->nb;
    const int P = (int)std::min<long long>(ga.units, std::min(nsm, kGemvMaxCtas));
    const int grid = partition_units(ga.units, g0, P, ga.ustart);
    if (grid < 1 || grid > P) return P8_ERR_ARG;
    {
        void *args[] = {&ga};
        const void *fn = pk == P8_PROLOGUE_RMSNORM ? (const void *)k_gemv<P8_PROLOGUE_RMSNORM>
                         : pk == P8_PROLOGUE_SWIGLU  ? (const void *)k_gemv<P8_PROLOGUE_SWIGLU>
                                                     : (const void *)k_gemv<P8_PROLOGUE_NONE>;
        if (launch_pdl(fn, dim3(grid), dim3(kGemvThreads), kGemvSmem, st, args) != cudaSuccess) return P8_ERR_CUDA;
    }
    ra.rows_total = ga.rows_total;
    ra.ntensors = nt;
    ra.nb = t0->nb;
    ra.X = pk != P8_PROLOGUE_NONE ? ga.xv : x;
    if (tp) ra.tp = *tp;
    // at most one CTA per SM: each one beside a k_gemv CTA (256 threads, <= 48 registers fit next to its 16 warps),
    // resident and waiting before k_gemv ends
    const int rgrid = std::max(1, std::min((ra.rows_total + kRedRowsPerCta - 1) / kRedRowsPerCta, nsm));
    void *args[] = {&ra};
    const void *fn = tp ? (const void *)k_gemv_reduce<true> : (const void *)k_gemv_reduce<false>;
    if (launch_pdl(fn, dim3(rgrid), dim3(kRedThreads), 0, st, args) != cudaSuccess) return P8_ERR_CUDA;
    return P8_OK;
}

// two columns (x at x and x + ldx; outputs at Ys[i] and Ys[i] + ldys[i]): k_gemv2 + k_gemv_reduce2
static p8_status launch_gemv2(const p8_tensor *const *ts, int nt, const float *x, int64_t ldx, const p8_prologue *pro,
                              float *const *Ys, const int64_t *ldys, void *ws, size_t ws_bytes, cudaStream_t st) {
    const p8_tensor *t0 = ts[0];
    const GemvWs L = gemv_ws_layout(ts, nt, 2);
    if (!ws || ws_bytes < L.total) return P8_ERR_WORKSPACE;
    uint8_t *w = static_cast<uint8_t *>(ws);
    const int nsm = sm_count();
    const int pk = pro ? pro->kind : P8_PROLOGUE_NONE;
    GemvArgs ga;
    memset(&ga, 0, sizeof(ga));
    ga.ntensors = nt;
    ga.X = x;
    ga.ldx = ldx;
    ga.ic = t0->ic; ga.A = t0->A; ga.cs = t0->cs; ga.K = t0->K; ga.nb = t0->nb; ga.nsl = t0->nsl;
    if (pk != P8_PROLOGUE_NONE) {
        ga.pw = pro->w;
        ga.x2 = pro->x2;
        ga.eps = pro->eps;
        ga.xv = reinterpret_cast<float *>(w + L.xv);
    }
    size_t poff = L.part;
    int g0 = 0;
    for (int i = 0; i < nt; ++i) {
        const p8_tensor *t = ts[i];
        GemvTensor &g = ga.t[i];
        g.M = t->M; g.D = t->D; g.S = t->S; g.prm = t->prm; g.cp = t->cp; g.cc = t->cc; g.cv = t->cv;
        g.Y = Ys[i];
        g.part = reinterpret_cast<float *>(w + poff);
        poff += al256((size_t)2 * t->nb * t->rows * 4);
        g.rows = t->rows; g.ng = t->ng; g.g0 = g0; g.row0 = ga.rows_total; g.ucls = t->uniform_class;
        g0 += t->ng;
        ga.rows_total += t->rows;
    }
    ga.ng_total = g0;
    ga.units = (long long)g0 * t0->nb;
    const int P = (int)std::min<long long>(ga.units, std::min(nsm, kGemvMaxCtas));
    const int grid = partition_units(ga.units, g0, P, ga.ustart, 2 * kTableCost);  // two tables per block
    if (grid < 1 || grid > P) return P8_ERR_ARG;
    {
        void *args[] = {&ga};
        const void *fn = pk == P8_PROLOGUE_RMSNORM ? (const void *)k_gemv2<P8_PROLOGUE_RMSNORM>
                         : pk == P8_PROLOGUE_SWIGLU  ? (const void *)k_gemv2<P8_PROLOGUE_SWIGLU>
                                                     : (const void *)k_gemv2<P8_PROLOGUE_NONE>;
        if (launch_pdl(fn, dim3(grid), dim3(kGemvThreads), kGemv2Smem, st, args) != cudaSuccess) return P8_ERR_CUDA;
    }
    Reduce2Args ra;
    memset(&ra, 0, sizeof(ra));
    for (int i = 0; i < nt; ++i) {
        ra.r.t[i] = ga.t[i];
        ra.ldy[i] = ldys[i];
    }
    ra.r.rows_total = ga.rows_total;
    ra.r.ntensors = nt;
    ra.r.nb = t0->nb;
    ra.r.X = pk != P8_PROLOGUE_NONE ? ga.xv : x;
    ra.X1 = pk != P8_PROLOGUE_NONE ? ga.xv + t0->K : x + ldx;
    const int rgrid = std::max(1, std::min((2 * ga.rows_total + kRedRowsPerCta - 1) / kRedRowsPerCta, nsm));
    void *args[] = {&ra};
    if (launch_pdl((const void *)k_gemv_reduce2, dim3(rgrid), dim3(kRedThreads), 0, st, args) != cudaSuccess) return P8_ERR_CUDA;
    return P8_OK;
}

// ncols columns (x_n = X + n ldx, the SwiGLU up at pro->x2 + n ldx; y_i of column n at Ys[i] + n ldys[i]): pairs of
// columns through the two-column kernel when every tensor is uniform class 3, the rest one column at a time
p8_status launch_gemv_cols(const p8_tensor *const *ts, int nt, const float *X, int64_t ncols, int64_t ldx, const p8_prologue *pro,
                           float *const *Ys, const int64_t *ldys, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (nt < 1 || nt > kMaxGroup) return P8_ERR_ARG;
    const p8_tensor *t0 = ts[0];
    bool two = ncols >= 2 && (ldx & 3) == 0;
    for (int i = 0; i < nt; ++i) {
        if (ts[i]->K != t0->K || ts[i]->act_hash != t0->act_hash) return P8_ERR_ARG;
        if (ts[i]->uniform_class != 3) two = false;
    }
    (void)sm_count();
    int64_t n = 0;
    for (; two && n + 1 < ncols; n += 2) {
        p8_prologue pn;
        if (pro) {
            pn = *pro;
            if (pn.x2) pn.x2 += n * ldx;
        }
        float *Yn[kMaxGroup];
        for (int i = 0; i < nt; ++i) Yn[i] = Ys[i] + n * ldys[i];
        const p8_status s = launch_gemv2(ts, nt, X + n * ldx, ldx, pro ? &pn : nullptr, Yn, ldys, ws, ws_bytes, st);
        if (s) return s;
    }
    for (; n < ncols; ++n) {
        p8_prologue pn;
        if (pro) {
            pn = *pro;
            if (pn.x2) pn.x2 += n * ldx;
        }
        float *Yn[kMaxGroup];
        for (int i = 0; i < nt; ++i) Yn[i] = Ys[i] + n * ldys[i];
        const p8_status s = launch_gemv_col(ts, nt, X + n * ldx, Yn, ws, ws_bytes, st, nullptr, nullptr, pro ? &pn : nullptr);
        if (s) return s;
    }
    return P8_OK;
}

p8_status launch_gemv_group(const p8_tensor *const *ts, int nt, const float *X, int64_t ncols, int64_t ldx, float *const *Ys,
                            const int64_t *ldys, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (nt < 1 || nt > kMaxGroup) return P8_ERR_ARG;
    const p8_tensor *t0 = ts[0];
    for (int i = 0; i < nt; ++i)  // tensors of one launch share x and its table: same K, column scales, signs and codebook
        if (ts[i]->K != t0->K || ts[i]->act_hash != t0->act_hash) return P8_ERR_ARG;
    // ncols > 1 (below the GEMM's column count): pairs of columns through the two-column kernel
    return launch_gemv_cols(ts, nt, X, ncols, ldx, nullptr, Ys, ldys, ws, ws_bytes, st);
}

p8_status launch_gemv_group_pro(const p8_tensor *const *ts, int nt, const float *x, const p8_prologue *pro, float *const *Ys,
                                void *ws, size_t ws_bytes, cudaStream_t st) {
    if (nt < 1 || nt > kMaxGroup) return P8_ERR_ARG;
    for (int i = 0; i < nt; ++i)
        if (ts[i]->K != ts[0]->K || ts[i]->act_hash != ts[0]->act_hash) return P8_ERR_ARG;
    (void)sm_count();
    return launch_gemv_col(ts, nt, x, Ys, ws, ws_bytes, st, nullptr, nullptr, pro);
}

p8_status launch_gemv(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, float *Y, int64_t ldy, void *ws, size_t ws_bytes,
                      cudaStream_t st) {
    return launch_gemv_group(&t, 1, X, ncols, ldx, &Y, &ldy, ws, ws_bytes, st);
}

p8_status launch_gemv_tp(const p8_tensor *t, const float *x, float *y, const TpExchange &tp, unsigned int *epoch, void *ws,
                         size_t ws_bytes, cudaStream_t st) {
    (void)sm_count();
    if (tp.world < 2) return launch_gemv_col(&t, 1, x, &y, ws, ws_bytes, st);
    return launch_gemv_col(&t, 1, x, &y, ws, ws_bytes, st, &tp, epoch);
}

unsigned int read_and_clear_device_error() {
    unsigned int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_p8_device_error, sizeof(v));
    cudaMemcpyToSymbol(g_p8_device_error, &z, sizeof(z));
    return v;
}

// ================================================================================================================
// 3. Batched GEMM (tcgen05)
// ================================================================================================================
#include "p8_gemm.cuh"

// ================================================================================================================
// 4. Chained batch-1 GEMVs in one persistent launch
// ================================================================================================================
#include "p8_chain.cuh"

}  // namespace p8
