// p8_chain.cuh -- a chain of batch-1 GEMVs in one persistent launch (included by p8_kernels.cu, namespace p8).
//
// A decode step runs a fixed sequence of projections, each reading an earlier one's output: o -> gate/up -> down ->
// q/k/v of the next layer. The per-op path (p8_mul_mat_vec_group) pays, per projection, two kernel boundaries (prep
// kernel, GEMV), a grid barrier inside the GEMV and a separate row reduce. Here one launch of one CTA per SM runs the
// whole sequence with ONE grid barrier per projection:
//
//   prep(s)   every CTA builds, in its own shared memory, the activation tables of the (at most two, usually one)
//             256-column blocks its units touch. A block's input values come straight from the previous projection's
//             row partials: the CTA sums the partials of those 256 rows itself (8 fixed block slices, then the slices
//             in order), adds the clamp delta, the output scale and the residual, applies the input op (RMSNorm weight
//             or SwiGLU), then the FWHT and the x16 quantisation (as k_act_prep), the coset tables and the 64 KiB
//             table T[f][hs][t] = <A[f], q_t> with two dp4a per entry (q = 128 hi + lo, |lo|, |hi| <= 64: exact).
//             The CTA that owns a block (it holds the block's first unit) writes those rows of the previous output,
//             the block's x' and its sum of squares. Rows of the previous projection that this one does not read
//             (k and v after q/k/v) are reduced by all CTAs in equal shares, in the same slice order.
//   units(s)  the table GEMV (the k_gemv unit loop) over the CTA's equal, contiguous share of the block-major
//             (block, tile) units; a unit stores its 32 row partials at the rows' ORIGINAL positions, so that the
//             next prep reads the 256 rows of a block as contiguous float4s.
//   barrier   every partial of step s is visible; then prep(s + 1). Before it, each CTA asks L2 for the payload of
//             its first units of step s + 1 (bulk prefetch), so HBM keeps streaming through the barrier and prep.
//   final     after the last barrier, the last projection's rows are reduced in equal shares.
//
// RMSNorm's scale 1 / sqrt(mean(x^2) + eps) is one positive scalar per vector and the product is linear, so the chain
// applies it to the projection's OUTPUT: tables and clamp-delta term use x * w, and the output reduce one barrier
// later, when every block's sum of squares is known, multiplies by the scale. The x16 quantisation is per 128
// columns relative to their largest value, so it is the same up to float rounding of the scaled inputs.
//
// Workspace: partials of two consecutive steps (ping-pong), x' and per-block sums of squares likewise. The plan
// (device step descriptors and the two barrier words) is built once by chain_create; a run reads nothing from the
// host. Barrier words are zero between launches: each launch counts its arrivals upwards and the last CTA to finish
// resets both words.

constexpr int kChainThreads = 512;
constexpr int kChainWarps = kChainThreads / 32;
constexpr int kChainMaxSteps = 4096;
// dynamic shared memory: the GEMV's table and coset regions (T0, T1, G0, G1 at the k_gemv offsets, so the unit loop's
// compile-time addresses are shared), then the step descriptors and the prep staging
constexpr int kChSteps = kSmemG1 + 2 * kGInts * 4;          // 133120: two ChainStep copies
constexpr int kChStepBytes = 1024;
constexpr int kChA = kChSteps + 2 * kChStepBytes;           // codebook copy u32[256]
constexpr int kChX = kChA + 1024;                           // x values [2][256] f32
constexpr int kChX2 = kChX + 2048;                          // SwiGLU up values [2][256] f32
constexpr int kChQ = kChX2 + 2048;                          // q [2][256] i32
constexpr int kChCx = kChQ + 2048;                          // <c, q_t> [2][64] i32
constexpr int kChD = kChCx + 512;                           // d [2][2] f32, ss partials [2][8] f32
constexpr int kChSmem = kChD + 256;
// the prep's reduce staging lives in the table region (free until the tables are built): [2][8][256] f32 per input
constexpr int kChRed = 0, kChRed2 = 16384, kChRedShare = 32768;

struct ChainTensor {
    const uint32_t *M, *D;
    const uint16_t *S;
    const int16_t *prm;
    const int *cp;
    const uint16_t *cc;
    const float *cv;
    float *Y;
    const float *res;
    unsigned long long part_off;  // byte offset of the tensor's partials [nb][rows] inside the step's partial buffer
    int rows, ng, g0, ucls;
};

struct ChainStep {
    ChainTensor t[kMaxGroup];
    const uint32_t *A;            // codebook of the step's tensors (device)
    const float *ic, *x, *x2, *pw;
    uint32_t cs;
    float eps;
    int nt, K, nb, ng_total, pro;
    int xsrc, x2src;              // -1: read x / x2 from memory; i >= 0: output of tensor i of the previous step
    int nunc, unc_rows;           // tensors whose rows the next step does not read (all of them for the last step)
    int unc[kMaxGroup];
    long long units;
};
static_assert(sizeof(ChainStep) <= kChStepBytes, "ChainStep outgrew its shared-memory slot");

struct ChainArgs {
    const ChainStep *steps;
    unsigned int *sync;           // [0] barrier arrivals of this launch, [1] exits; zero between launches
    uint8_t *ws;
    unsigned long long part[2], xv[2], ss[2];  // workspace byte offsets (ping-pong by step parity)
    int nsteps;
    int pf;                       // units per CTA whose payload is prefetched into L2 before each step
};

__device__ __forceinline__ float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }

// grid barrier number `n` (0-based) of this launch: every CTA arrives once per barrier whether or not it still waits,
// so the counts stay consistent after a timeout (bit 5 of the device error word; the launch's results are invalid)
__device__ __forceinline__ void chain_barrier(unsigned int *cnt, unsigned int target, int *s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(cnt, 1u);
        if (*s_ok) {
            const unsigned long long dl = global_ns() + kGridWaitNs;
            unsigned int v;
            for (;;) {
                asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
                if (v >= target) break;
                if (global_ns() > dl) {
                    atomicOr(&g_p8_device_error, 32u);
                    *s_ok = 0;
                    break;
                }
            }
        }
        __threadfence();
    }
    __syncthreads();
}

// y of one output row of step `P` (tensor T): the slice-ordered sum of its partials `sum`, then the clamp delta on x'
// (in CSR order), the output scale (RMSNorm of the step's input), the residual
__device__ __forceinline__ float chain_row_out(const ChainTensor &T, int ro, float sum, const float *xv, float scale) {
    float y = sum;
    const int e1 = __ldg(T.cp + ro + 1);
    for (int e = __ldg(T.cp + ro); e < e1; ++e) y = __fadd_rn(y, __fmul_rn(__ldg(T.cv + e), __ldcg(xv + __ldg(T.cc + e))));
    y = __fmul_rn(y, scale);
    if (T.res) y = __fadd_rn(y, __ldcg(T.res + ro));
    return y;
}

// 8 slices of the partial sums of rows [r0, r0 + 256) of a tensor with `nb` blocks: slice k sums blocks k, k + 8, ...
// in order; red[k][r]. Thread (quad j, slice k) loads float4s.
__device__ __forceinline__ void chain_slices_256(const float *part, int rows, int nb, int r0, float *red) {
    const int j = threadIdx.x & 63, k = threadIdx.x >> 6;
    const float *p = part + r0 + 4 * j;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int bb = k;
    for (; bb + 24 < nb; bb += 32) {
        const float4 v0 = ldcg4(p + (size_t)bb * rows), v1 = ldcg4(p + (size_t)(bb + 8) * rows);
        const float4 v2 = ldcg4(p + (size_t)(bb + 16) * rows), v3 = ldcg4(p + (size_t)(bb + 24) * rows);
        acc.x = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc.x, v0.x), v1.x), v2.x), v3.x);
        acc.y = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc.y, v0.y), v1.y), v2.y), v3.y);
        acc.z = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc.z, v0.z), v1.z), v2.z), v3.z);
        acc.w = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc.w, v0.w), v1.w), v2.w), v3.w);
    }
    for (; bb < nb; bb += 8) {
        const float4 v = ldcg4(p + (size_t)bb * rows);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    *reinterpret_cast<float4 *>(red + k * 256 + 4 * j) = acc;
}

__device__ __forceinline__ float chain_sum_slices(const float *red, int stride, int r) {
    float y = red[r];
#pragma unroll
    for (int k = 1; k < 8; ++k) y = __fadd_rn(y, red[k * stride + r]);
    return y;
}

// RMSNorm output scale of step P (1 without RMSNorm) from its per-block sums of squares (one warp, fixed order)
__device__ __forceinline__ float chain_scale(const ChainStep &P, const float *ss) {
    const int lane = threadIdx.x & 31;
    float v = 0.f;
    for (int i = lane; i < P.nb; i += 32) v = __fadd_rn(v, __ldcg(ss + i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
    const float mean = __fdiv_rn(v, (float)P.K);
    return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, P.eps)));
}

// Rows [ra, rb) of the concatenated not-read-next tensors of step P, reduced and written (equal shares per CTA).
__device__ void chain_share_reduce(const ChainStep &P, const ChainArgs &a, int pp, long long ra, long long rb, float scale) {
    float *red = reinterpret_cast<float *>(g_smem + kChRedShare);  // [8][64]
    const float *xv = reinterpret_cast<const float *>(a.ws + a.xv[pp]);
    const uint8_t *pbase = a.ws + a.part[pp];
    const int r = threadIdx.x & 63, k = threadIdx.x >> 6;
    for (long long base = ra; base < rb; base += 64) {
        const long long i = base + r;
        int ti = -1, ro = 0;
        if (i < rb) {
            long long off = i;
            for (int q = 0; q < P.nunc; ++q) {
                const int t = P.unc[q];
                if (off < P.t[t].rows) {
                    ti = t;
                    ro = (int)off;
                    break;
                }
                off -= P.t[t].rows;
            }
        }
        float acc = 0.f;
        if (ti >= 0) {
            const ChainTensor &T = P.t[ti];
            const float *p = reinterpret_cast<const float *>(pbase + T.part_off) + ro;
            for (int bb = k; bb < P.nb; bb += 8) acc = __fadd_rn(acc, __ldcg(p + (size_t)bb * T.rows));
        }
        red[k * 64 + r] = acc;
        __syncthreads();
        if (k == 0 && ti >= 0) {
            const ChainTensor &T = P.t[ti];
            T.Y[ro] = chain_row_out(T, ro, chain_sum_slices(red, 64, r), xv, scale);
        }
        __syncthreads();
    }
}

// input values of blocks pb .. pb + nsg - 1 of step C from source src (-1: memory at xext; else tensor src of the
// previous step P, reduced here) into dst[seg][256]; the block's owner writes the reduced rows to the output
__device__ void chain_input(const ChainStep &C, const ChainStep *P, const ChainArgs &a, int s, int src, const float *xext,
                            int pb, int nsg, unsigned own_mask, float scale, float *dst) {
    const int tid = threadIdx.x;
    if (src < 0) {
        if (tid < 256 * nsg) dst[tid] = __ldcg(xext + 256 * pb + tid);
        return;
    }
    const int pp = (s - 1) & 1;
    const ChainTensor &T = P->t[src];
    const float *part = reinterpret_cast<const float *>(a.ws + a.part[pp] + T.part_off);
    float *red = reinterpret_cast<float *>(g_smem + kChRed);  // [2][8][256]
    for (int sg = 0; sg < nsg; ++sg) chain_slices_256(part, T.rows, P->nb, 256 * (pb + sg), red + sg * 2048);
    __syncthreads();
    if (tid < 256 * nsg) {
        const int sg = tid >> 8, r = tid & 255, ro = 256 * (pb + sg) + r;
        const float *xv = reinterpret_cast<const float *>(a.ws + a.xv[pp]);
        const float y = chain_row_out(T, ro, chain_sum_slices(red + sg * 2048, 256, r), xv, scale);
        dst[tid] = y;
        if ((own_mask >> sg) & 1u) T.Y[ro] = y;
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kChainThreads, 1) k_chain(const __grid_constant__ ChainArgs a) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ int s_ok;
    __shared__ float s_scale;
    float *xs = reinterpret_cast<float *>(g_smem + kChX);
    float *x2s = reinterpret_cast<float *>(g_smem + kChX2);
    int *q_s = reinterpret_cast<int *>(g_smem + kChQ);
    int *cx_s = reinterpret_cast<int *>(g_smem + kChCx);
    float *d_s = reinterpret_cast<float *>(g_smem + kChD);
    float *ssp = d_s + 4;  // [2][8] per-warp partial sums of squares
    uint32_t *A_s = reinterpret_cast<uint32_t *>(g_smem + kChA);
    pdl_launch_dependents();
    uint32_t po[11];
#pragma unroll
    for (int q = 0; q < 11; ++q) {
        uint32_t r = 0;
#pragma unroll
        for (int i = 0; i < 3; ++i)
            if (3 * q + i < 32) r |= (((uint32_t)(lane + 3 * q + i) & 31u) << 2) << (8 * i);
        po[q] = r;
    }
    if (tid == 0) s_ok = 1;
    pdl_wait();  // inputs, workspace and barrier words belong to earlier kernels until they complete
    for (int s = 0; s <= a.nsteps; ++s) {
        // ---- descriptors: step s into slot s & 1 (step s - 1 is already in the other slot)
        ChainStep *Cs = reinterpret_cast<ChainStep *>(g_smem + kChSteps + (s & 1) * kChStepBytes);
        const ChainStep *P = s > 0 ? reinterpret_cast<const ChainStep *>(g_smem + kChSteps + ((s - 1) & 1) * kChStepBytes) : nullptr;
        if (s < a.nsteps) {
            const uint32_t *src = reinterpret_cast<const uint32_t *>(a.steps + s);
            uint32_t *dst = reinterpret_cast<uint32_t *>(Cs);
            for (int i = tid; i < (int)(sizeof(ChainStep) / 4); i += kChainThreads) dst[i] = __ldg(src + i);
        }
        if (tid < 32) {  // output scale of the previous step (its input's RMSNorm), from its blocks' sums of squares
            float sc = 1.f;
            if (P && P->pro == P8_PROLOGUE_RMSNORM) sc = chain_scale(*P, reinterpret_cast<const float *>(a.ws + a.ss[(s - 1) & 1]));
            if (lane == 0) s_scale = sc;
        }
        __syncthreads();
        const float scale_p = s_scale;
        const int pp = (s - 1) & 1;
        if (s == a.nsteps) {  // final phase: the last step's rows in equal shares
            if (P && s_ok) {
                const long long R = P->unc_rows;
                chain_share_reduce(*P, a, pp, R * blockIdx.x / gridDim.x, R * (blockIdx.x + 1) / gridDim.x, scale_p);
            }
            break;
        }
        const ChainStep &C = *Cs;
        const int cp_ = s & 1;
        // ---- this CTA's units of step s: [u0, u1) of the block-major list; warp w takes u0 + w, u0 + w + 16, ...
        const long long u0 = C.units * blockIdx.x / gridDim.x, u1 = C.units * (blockIdx.x + 1) / gridDim.x;
        const int ngt = C.ng_total;
        const int b_first = u1 > u0 ? (int)(u0 / ngt) : 0, b_last = u1 > u0 ? (int)((u1 - 1) / ngt) : -1;
        const int rr_first = (int)(u0 - (long long)b_first * ngt);
        long long un = u0 + warp;
        int cb = (int)(un / ngt), crr = (int)(un - (long long)cb * ngt);
        auto advance = [&]() {
            un += kChainWarps;
            crr += kChainWarps;
            while (crr >= ngt) {
                crr -= ngt;
                ++cb;
            }
        };
        auto tensor_of_rr = [&](int rr) {
            int ti = 0;
#pragma unroll
            for (int i = 1; i < kMaxGroup; ++i)
                if (i < C.nt && rr >= C.t[i].g0) ti = i;
            return ti;
        };
        auto m_of = [&](int b, int rr) -> uint32_t {
            const ChainTensor &T = C.t[tensor_of_rr(rr)];
            const uint32_t tile = (uint32_t)(rr - T.g0) * (uint32_t)C.nb + (uint32_t)b;
            if (T.ucls) return (tile * (uint32_t)(64 * NW(T.ucls))) | ((uint32_t)T.ucls << 29);
            return __ldg(T.M + tile);
        };
        uint32_t nxt[16];
        uint32_t mt_n = 0;
        uint16_t s_n = 0;
        int pr_n = 0;
        auto fetch = [&]() {  // payload, scale and output row of the warp's unit (cb, crr)
            const ChainTensor &T = C.t[tensor_of_rr(crr)];
            const int g = crr - T.g0;
            mt_n = m_of(cb, crr);
            if ((mt_n >> 29) == 3) load3(T.D + (mt_n & 0x1FFFFFFFu), lane, nxt);
            s_n = __ldg(T.S + (size_t)cb * T.rows + g * 32 + lane);
            pr_n = __ldg(T.prm + g * 32 + lane);
        };
        if (un < u1) fetch();  // weights only: the first unit's loads overlap the prep below
        // ---- rows of the previous step that this step does not read: equal shares
        if (P && s_ok && P->nunc) {
            const long long R = P->unc_rows;
            chain_share_reduce(*P, a, pp, R * blockIdx.x / gridDim.x, R * (blockIdx.x + 1) / gridDim.x, scale_p);
        }
        for (int i = tid; i < 256; i += kChainThreads) A_s[i] = __ldg(C.A + i);
        float *xv_c = reinterpret_cast<float *>(a.ws + a.xv[cp_]);
        float *ss_c = reinterpret_cast<float *>(a.ws + a.ss[cp_]);
        for (int pb = b_first; pb <= b_last; pb += 2) {
            const int nsg = b_last - pb + 1 < 2 ? b_last - pb + 1 : 2;
            unsigned own = 0;  // blocks whose first unit is this CTA's
            for (int sg = 0; sg < nsg; ++sg)
                if (pb + sg > b_first || rr_first == 0) own |= 1u << sg;
            // ---- (a) input values of the pair's blocks (fused reduce of the previous step, or memory)
            if (s_ok) {
                chain_input(C, P, a, s, C.xsrc, C.x, pb, nsg, own, scale_p, xs);
                if (C.pro == P8_PROLOGUE_SWIGLU) chain_input(C, P, a, s, C.x2src, C.x2, pb, nsg, own, scale_p, x2s);
            }
            __syncthreads();
            // ---- (b) input op: x' (RMSNorm: x * w, its scale goes to the output; SwiGLU: silu(x) * up); the owner
            // writes x' (clamp-delta term of this step's outputs) and the block's sum of x^2 (RMSNorm scale)
            if (tid < 256 * nsg) {
                const int sg = tid >> 8, col = 256 * (pb + sg) + (tid & 255);
                const float x = xs[tid];
                float xp = x;
                if (C.pro == P8_PROLOGUE_RMSNORM) {
                    xp = __fmul_rn(x, __ldg(C.pw + col));
                    float q2 = __fmul_rn(x, x);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) q2 = __fadd_rn(q2, __shfl_down_sync(0xffffffffu, q2, o));
                    if (lane == 0) ssp[(tid >> 5)] = q2;  // warp (tid >> 5) = 8 sg + w
                } else if (C.pro == P8_PROLOGUE_SWIGLU) {
                    const float u = x2s[tid];
                    xp = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.f, expf(-x))), u);
                }
                xs[tid] = xp;
                if ((own >> sg) & 1u) xv_c[col] = xp;
            }
            __syncthreads();
            if (C.pro == P8_PROLOGUE_RMSNORM && tid < nsg && ((own >> tid) & 1u)) {
                float v = ssp[8 * tid];
                for (int w = 1; w < 8; ++w) v = __fadd_rn(v, ssp[8 * tid + w]);
                ss_c[pb + tid] = v;
            }
            // ---- (c) FWHT(x' sgn/c) / 16 and the x16 quantisation per 128 columns (warp sg: block pb + sg)
            if (warp < nsg) {
                const float *icp = C.ic + 256 * (pb + warp) + 8 * lane;
                const float4 i0 = __ldg(reinterpret_cast<const float4 *>(icp)), i1 = __ldg(reinterpret_cast<const float4 *>(icp + 4));
                const float *xp = xs + 256 * warp + 8 * lane;
                float v[8] = {__fmul_rn(xp[0], i0.x), __fmul_rn(xp[1], i0.y), __fmul_rn(xp[2], i0.z), __fmul_rn(xp[3], i0.w),
                              __fmul_rn(xp[4], i1.x), __fmul_rn(xp[5], i1.y), __fmul_rn(xp[6], i1.z), __fmul_rn(xp[7], i1.w)};
                fwht256_warp(v, lane);
                float am = 0.f;
#pragma unroll
                for (int m = 0; m < 8; ++m) am = fmaxf(am, fabsf(v[m]));
#pragma unroll
                for (int o = 1; o < 16; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                const float d = __fdiv_rn(am, 8191.f), id = d > 0.f ? __fdiv_rn(1.f, d) : 0.f;
#pragma unroll
                for (int m = 0; m < 8; ++m) q_s[256 * warp + 8 * lane + m] = __float2int_rn(__fmul_rn(v[m], id));
                if ((lane & 15) == 0) d_s[2 * warp + (lane >> 4)] = d;
            }
            __syncthreads();
            if (tid < 64 * nsg) {  // <c, q_t> per chunk
                int cx = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e) cx += (int)(int8_t)(C.cs >> (8 * e)) * q_s[4 * tid + e];
                cx_s[tid] = cx;
            }
            __syncthreads();
            if (tid < 256 * nsg) {  // coset nibble tables: G[hs][grp][m] = sum over set bits i of m of <c, q_(32 hs + 4 grp + i)>
                const int sg = tid >> 8, e = tid & 255, hs = e >> 7, grp = (e >> 4) & 7, m = e & 15;
                int gs = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if ((m >> i) & 1) gs += cx_s[64 * sg + 32 * hs + 4 * grp + i];
                reinterpret_cast<int *>(g_smem + (sg ? kSmemG1 : kSmemG0))[hs * kGInts + grp * 16 + m] = gs;
            }
            // ---- (d) the 64 KiB table of each block: T[f][hs * 32 + t] = <A[f], q_(hs, t)>, four consecutive (hs, t)
            // per thread and 16-byte stores; q = 128 hi + lo with hi, lo in int8 range, so two dp4a per entry are exact
            {
                const int h4 = tid & 15, fr = tid >> 4;
                for (int sg = 0; sg < nsg; ++sg) {
                    int H[4], Lo[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int4 qv = *reinterpret_cast<const int4 *>(q_s + 256 * sg + 4 * (4 * h4 + j));
                        const int qq[4] = {qv.x, qv.y, qv.z, qv.w};
                        uint32_t hp = 0, lp = 0;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int hi = (qq[e] + 64) >> 7, lo = qq[e] - 128 * hi;
                            hp |= ((uint32_t)hi & 0xffu) << (8 * e);
                            lp |= ((uint32_t)lo & 0xffu) << (8 * e);
                        }
                        H[j] = (int)hp;
                        Lo[j] = (int)lp;
                    }
                    int *T = reinterpret_cast<int *>(g_smem + (sg ? kSmemT1 : kSmemT0));
#pragma unroll 2
                    for (int i = 0; i < 8; ++i) {
                        const int f = fr + 32 * i;
                        const int av = (int)A_s[f];
                        int4 o;
                        o.x = __dp4a(av, H[0], 0) * 128 + __dp4a(av, Lo[0], 0);
                        o.y = __dp4a(av, H[1], 0) * 128 + __dp4a(av, Lo[1], 0);
                        o.z = __dp4a(av, H[2], 0) * 128 + __dp4a(av, Lo[2], 0);
                        o.w = __dp4a(av, H[3], 0) * 128 + __dp4a(av, Lo[3], 0);
                        *reinterpret_cast<int4 *>(T + f * 64 + 4 * h4) = o;
                    }
                }
            }
            __syncthreads();
            // ---- (e) units of the pair's blocks
            while (s_ok && un < u1 && cb < pb + nsg) {
                const int sg = cb - pb, b = cb, rr = crr;
                const float d0 = d_s[2 * sg], d1 = d_s[2 * sg + 1];
                const uint32_t mt = mt_n;
                const uint16_t sc = s_n;
                const int ro = pr_n;
                uint32_t cur[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) cur[i] = nxt[i];
                advance();
                if (un < u1) fetch();
                const ChainTensor &T = C.t[tensor_of_rr(rr)];
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
                    part = sg ? tile_row_dot_w<3, 1>(w0, w1, po, lane, d0, d1) : tile_row_dot_w<3, 0>(w0, w1, po, lane, d0, d1);
                } else {
                    const uint32_t *p0 = T.D + (mt & 0x1FFFFFFFu);
                    part = sg ? tile_row_other<1>(c, p0, po, lane, d0, d1) : tile_row_other<0>(c, p0, po, lane, d0, d1);
                }
                float *pt = reinterpret_cast<float *>(a.ws + a.part[cp_] + T.part_off);
                pt[(size_t)b * T.rows + ro] = __fmul_rn(part, h2f(sc));
            }
            __syncthreads();
        }
        // ---- ask L2 for the payload of this CTA's first units of the next step (weights: no dependency)
        if (warp == 0 && s + 1 < a.nsteps && a.pf > 0) {
            const ChainStep *N = a.steps + s + 1;
            const long long nu = __ldg(&N->units);
            const long long v0 = nu * blockIdx.x / gridDim.x, v1 = nu * (blockIdx.x + 1) / gridDim.x;
            const int ng2 = __ldg(&N->ng_total), nb2 = __ldg(&N->nb), nt2 = __ldg(&N->nt);
            for (long long u = v0 + lane; u < v1 && u < v0 + a.pf; u += 32) {
                const int b = (int)(u / ng2), rr = (int)(u - (long long)b * ng2);
                int ti = 0;
                for (int i = 1; i < nt2; ++i)
                    if (rr >= __ldg(&N->t[i].g0)) ti = i;
                const ChainTensor *T = N->t + ti;  // plan memory: written once at creation, read with plain loads
                const uint32_t tile = (uint32_t)(rr - T->g0) * (uint32_t)nb2 + (uint32_t)b;
                const int uc = T->ucls;
                const uint32_t mt = uc ? ((tile * (uint32_t)(64 * NW(uc))) | ((uint32_t)uc << 29)) : __ldg(T->M + tile);
                const int c = (int)(mt >> 29);
                if (c) bulk_prefetch_l2(T->D + (mt & 0x1FFFFFFFu), (uint32_t)(256 * NW(c)));
            }
        }
        chain_barrier(a.sync, (unsigned int)(s + 1) * gridDim.x, &s_ok);
    }
    // ---- exit: the last CTA out resets the barrier words for the next launch (every CTA has passed every barrier)
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned int old = atomicAdd(a.sync + 1, 1u);
        if (old == gridDim.x - 1) {
            a.sync[0] = 0u;
            a.sync[1] = 0u;
            __threadfence();
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------- host
}  // namespace p8

struct p8_chain {
    uint32_t magic;
    int device, nsteps;
    p8::ChainStep *d_steps;
    unsigned int *d_sync;
    unsigned long long part[2], xv[2], ss[2];
    size_t ws_bytes;
};

namespace p8 {

constexpr uint32_t kChainMagic = 0x50384348u;

static bool overlaps(const void *a, size_t na, const void *b, size_t nb) {
    const uintptr_t x = (uintptr_t)a, y = (uintptr_t)b;
    return na && nb && x < y + nb && y < x + na;
}

p8_status chain_create(const p8_chain_step *st, int n, p8_chain **out) {
    if (!out || !st || n < 1 || n > kChainMaxSteps) return P8_ERR_ARG;
    *out = nullptr;
    std::vector<ChainStep> hs((size_t)n);
    size_t part_max = 0, k_max = 0, nb_max = 0;
    int dev = -1;
    for (int s = 0; s < n; ++s) {
        const p8_chain_step &q = st[s];
        ChainStep &c = hs[(size_t)s];
        memset(&c, 0, sizeof(c));
        if (q.n < 1 || q.n > kMaxGroup || !q.x || ((uintptr_t)q.x & 15)) return P8_ERR_ARG;
        for (int i = 0; i < q.n; ++i) {
            const p8_tensor *t = q.t[i];
            if (!t || t->magic != kTensorMagic) return P8_ERR_NOT_PREPARED;
            if (t->K != q.t[0]->K || t->act_hash != q.t[0]->act_hash || !q.y[i]) return P8_ERR_ARG;
            if (dev < 0) dev = t->device;
            if (t->device != dev) return P8_ERR_ARG;
            if (q.res[i] && overlaps(q.res[i], 4 * (size_t)t->rows, q.y[i], 4 * (size_t)t->rows)) return P8_ERR_ARG;
        }
        const p8_tensor *t0 = q.t[0];
        const int pk = q.pro.kind;
        if (pk == P8_PROLOGUE_RMSNORM) {
            if (!q.pro.w || ((uintptr_t)q.pro.w & 15) || !(q.pro.eps >= 0.f)) return P8_ERR_ARG;
        } else if (pk == P8_PROLOGUE_SWIGLU) {
            if (!q.pro.x2 || ((uintptr_t)q.pro.x2 & 15)) return P8_ERR_ARG;
        } else if (pk != P8_PROLOGUE_NONE) {
            return P8_ERR_ARG;
        }
        c.A = t0->A; c.ic = t0->ic; c.cs = t0->cs; c.x = q.x; c.x2 = pk == P8_PROLOGUE_SWIGLU ? q.pro.x2 : nullptr;
        c.pw = pk == P8_PROLOGUE_RMSNORM ? q.pro.w : nullptr; c.eps = q.pro.eps; c.pro = pk;
        c.nt = q.n; c.K = t0->K; c.nb = t0->nb;
        size_t poff = 0;
        int g0 = 0;
        for (int i = 0; i < q.n; ++i) {
            const p8_tensor *t = q.t[i];
            ChainTensor &T = c.t[i];
            T.M = t->M; T.D = t->D; T.S = t->S; T.prm = t->prm; T.cp = t->cp; T.cc = t->cc; T.cv = t->cv;
            T.Y = q.y[i]; T.res = q.res[i]; T.part_off = poff;
            T.rows = t->rows; T.ng = t->ng; T.g0 = g0; T.ucls = t->uniform_class;
            poff += ((size_t)t->nb * t->rows * 4 + 255) & ~(size_t)255;
            g0 += t->ng;
        }
        c.ng_total = g0;
        c.units = (long long)g0 * c.nb;
        part_max = poff > part_max ? poff : part_max;
        k_max = (size_t)c.K > k_max ? (size_t)c.K : k_max;
        nb_max = (size_t)c.nb > nb_max ? (size_t)c.nb : nb_max;
        // input sources: the previous step's output is read through the fused reduce; any other overlap with it is
        // refused (its rows are written only during this step's prep)
        c.xsrc = c.x2src = -1;
        if (s > 0) {
            const p8_chain_step &pq = st[s - 1];
            auto source = [&](const float *p, int &src) -> bool {
                for (int i = 0; i < pq.n; ++i) {
                    if (p == pq.y[i]) {
                        if (pq.t[i]->rows != c.K) return false;
                        src = i;
                        return true;
                    }
                    if (overlaps(p, 4 * (size_t)c.K, pq.y[i], 4 * (size_t)pq.t[i]->rows)) return false;
                }
                return true;
            };
            if (!source(c.x, c.xsrc)) return P8_ERR_ARG;
            if (c.x2 && !source(c.x2, c.x2src)) return P8_ERR_ARG;
        }
    }
    for (int s = 0; s < n; ++s) {  // tensors whose rows the next step does not read
        ChainStep &c = hs[(size_t)s];
        c.nunc = 0;
        c.unc_rows = 0;
        for (int i = 0; i < c.nt; ++i) {
            const bool read = s + 1 < n && (hs[(size_t)s + 1].xsrc == i || hs[(size_t)s + 1].x2src == i);
            if (!read) {
                c.unc[c.nunc++] = i;
                c.unc_rows += c.t[i].rows;
            }
        }
    }
    p8_chain *p = new p8_chain();
    p->magic = kChainMagic;
    p->device = dev;
    p->nsteps = n;
    size_t o = 0;
    for (int i = 0; i < 2; ++i) { p->part[i] = o; o += part_max; }
    for (int i = 0; i < 2; ++i) { p->xv[i] = o; o += (4 * k_max + 255) & ~(size_t)255; }
    for (int i = 0; i < 2; ++i) { p->ss[i] = o; o += (4 * nb_max + 255) & ~(size_t)255; }
    p->ws_bytes = o;
    if (cudaMalloc((void **)&p->d_steps, sizeof(ChainStep) * (size_t)n) != cudaSuccess ||
        cudaMalloc((void **)&p->d_sync, 256) != cudaSuccess ||
        cudaMemcpy(p->d_steps, hs.data(), sizeof(ChainStep) * (size_t)n, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(p->d_sync, 0, 256) != cudaSuccess) {
        cudaFree(p->d_steps);
        cudaFree(p->d_sync);
        delete p;
        return P8_ERR_CUDA;
    }
    *out = p;
    return P8_OK;
}

p8_status chain_destroy(p8_chain *p) {
    if (!p || p->magic != kChainMagic) return P8_ERR_ARG;
    cudaFree(p->d_steps);
    cudaFree(p->d_sync);
    p->magic = 0;
    delete p;
    return P8_OK;
}

size_t chain_workspace(const p8_chain *p) { return p && p->magic == kChainMagic ? p->ws_bytes : 0; }

p8_status chain_run(const p8_chain *p, void *ws, size_t ws_bytes, cudaStream_t st, int pf) {
    if (!p || p->magic != kChainMagic) return P8_ERR_ARG;
    if (!ws || ws_bytes < p->ws_bytes || ((uintptr_t)ws & 255)) return P8_ERR_WORKSPACE;
    static std::atomic<bool> attr[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return P8_ERR_CUDA;
    if (dev != p->device) return P8_ERR_ARG;
    if (dev < 0 || dev >= 64 || !attr[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(k_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, kChSmem) != cudaSuccess) return P8_ERR_CUDA;
        if (dev >= 0 && dev < 64) attr[dev].store(true, std::memory_order_release);
    }
    ChainArgs a;
    memset(&a, 0, sizeof(a));
    a.steps = p->d_steps;
    a.sync = p->d_sync;
    a.ws = static_cast<uint8_t *>(ws);
    for (int i = 0; i < 2; ++i) { a.part[i] = p->part[i]; a.xv[i] = p->xv[i]; a.ss[i] = p->ss[i]; }
    a.nsteps = p->nsteps;
    a.pf = pf < 0 ? 0 : pf;
    void *args[] = {&a};
    return launch_pdl((const void *)k_chain, dim3((unsigned)sm_count()), dim3(kChainThreads), kChSmem, st, args) == cudaSuccess
               ? P8_OK
               : P8_ERR_CUDA;
}
