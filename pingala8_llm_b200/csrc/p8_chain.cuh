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
//             next prep reads the 256 rows of a block as contiguous float4s. Each warp keeps its next unit's payload
//             in registers and asks L2 (bulk prefetch) for the payload, scales and row order of the units after it.
//   barrier   every partial of step s is visible; then prep(s + 1).
//   final     after the last barrier, the last projection's rows are reduced in equal shares.
//
// Nothing a prep needs waits on DRAM after the barrier: the step descriptors sit in shared memory a step ahead
// (three slots), the next step's codebook, column scales and norm weight for the CTA's blocks are copied into shared
// memory by cp.async while the CTA waits at the barrier, every warp asks L2 for its first units of the next step, and
// row epilogues read clamp-delta data only in 256-row blocks that hold entries (a per-tensor block mask).
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
// The unit loop picks the table of a unit's block by data, not by code: the lane's lookup-address registers carry the
// block's buffer index (0 / 1), which the PRMT that builds a lookup address places at bits 16-23, so
// the tables sit 64 KiB apart (T0 at 0, T1 at 64 KiB) and the coset tables likewise (G0 at 128 KiB, G1 at 192 KiB);
// one copy of the loop serves both buffers.
constexpr int kChG0 = 131072, kChG1 = kChG0 + 65536;        // coset tables [hs][8][16] i32 per buffer
constexpr int kChSteps = kChG0 + 2 * kGInts * 4;            // three ChainStep slots (step s in slot s % 3)
constexpr int kChStepBytes = 1024;
constexpr int kChA = kChSteps + 3 * kChStepBytes;           // codebook copy u32[256]
constexpr int kChIc = kChA + 1024;                          // column scales sgn/c of the first pair [2][256] f32
constexpr int kChPw = kChIc + 2048;                         // RMSNorm weight of the first pair [2][256] f32
constexpr int kChX = kChPw + 2048;                          // x values [2][256] f32
constexpr int kChX2 = kChX + 2048;                          // SwiGLU up values [2][256] f32
constexpr int kChHL = kChX2 + 2048;                         // x16 ints as int8x4 hi / lo words per chunk [2][64] uint2
constexpr int kChCx = kChHL + 1024;                         // <c, q_t> [2][64] i32
constexpr int kChD = kChCx + 512;                           // d [2][2] f32, ss partials [2][8] f32
constexpr int kChSmem = kChG1 + 2 * kGInts * 4;
static_assert(kChD + 256 <= kChG1, "chain staging overlaps the second coset table");
// the prep's reduce staging lives in the table region (free until the tables are built)
constexpr int kChRed = 0, kChRedShare = 32768;

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
    uint32_t dmask[4];            // bit b: original rows [256 b, 256 b + 256) hold clamp-delta entries
};

struct alignas(16) ChainStep {
    ChainTensor t[kMaxGroup];
    const uint32_t *A;            // codebook of the step's tensors (device)
    const float *ic, *x, *x2, *pw;
    uint32_t cs;
    float eps;
    int nt, K, nb, ng_total, pro;
    int xsrc, x2src;              // -1: read x / x2 from memory; i >= 0: output of tensor i of the previous step
    int nunc, unc_rows;           // tensors whose rows the next step does not read (all of them for the last step)
    int unc[kMaxGroup];
    unsigned int units;           // nb * ng_total (< 2^20)
    const uint2 *cuts;            // [CTAs] each CTA's contiguous unit range [x, y) of this step (host-balanced)
};
constexpr int kChRangeOff = 1016;  // a slot holds the descriptor, and this CTA's unit range (uint2) at this byte
static_assert(sizeof(ChainStep) <= kChRangeOff && sizeof(ChainStep) % 16 == 0, "ChainStep slot");

struct ChainArgs {
    const ChainStep *steps;
    unsigned int *sync;           // [0] barrier arrivals of this launch, [1] exits; zero between launches
    uint8_t *ws;
    unsigned long long part[2], xv[2], ss[2];  // workspace byte offsets (ping-pong by step parity)
    int nsteps;
    int pf;                       // units per warp whose payload is asked of L2 ahead of the warp's current unit
    int s_begin, s_end;           // this launch runs phases s_begin .. s_end (phase nsteps: the last step's rows)
    unsigned long long *trace;    // optional phase trace: [step][cta][8] globaltimer stamps (NULL: off)
    const uint2 *cuts;            // [nsteps][CTAs] unit ranges (ChainStep::cuts of step s = cuts + s * CTAs)
};

__device__ __forceinline__ float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }
__device__ __forceinline__ void cp_async16(void *smem, const void *g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__device__ __forceinline__ const ChainStep *chain_slot(int s) {
    return reinterpret_cast<const ChainStep *>(g_smem + kChSteps + (s % 3) * kChStepBytes);
}
// step s's descriptor into its slot, asynchronously (cp.async; the caller waits before reading it)
__device__ __forceinline__ void chain_load_step(const ChainArgs &a, int s) {
    constexpr int n16 = (int)(sizeof(ChainStep) / 16);
    const uint8_t *src = reinterpret_cast<const uint8_t *>(a.steps + s);
    uint8_t *dst = g_smem + kChSteps + (s % 3) * kChStepBytes;
    for (int i = (int)threadIdx.x - 32; i < n16; i += kChainThreads - 32)  // warps 1..: none in flight on thread 0
        if (i >= 0) cp_async16(dst + 16 * i, src + 16 * i);
}
// this CTA's unit range of step s into the slot (the plan's cuts array; 8-byte cp.async)
__device__ __forceinline__ void chain_load_range(const ChainArgs &a, int s, const uint2 *cuts_of_step) {
    if (threadIdx.x == kChainThreads - 1) {
        uint8_t *dst = g_smem + kChSteps + (s % 3) * kChStepBytes + kChRangeOff;
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(cuts_of_step + blockIdx.x) : "memory");
    }
}

// this CTA's unit range of a step and its first block pair
struct ChainRange {
    unsigned int u0, u1;
    int b_first, b_last;
};
__device__ __forceinline__ ChainRange chain_range(const ChainStep &C) {
    const uint2 u = *reinterpret_cast<const uint2 *>(reinterpret_cast<const uint8_t *>(&C) + kChRangeOff);
    ChainRange r;
    r.u0 = u.x;
    r.u1 = u.y;
    r.b_first = r.u1 > r.u0 ? (int)(r.u0 / (unsigned int)C.ng_total) : 0;
    r.b_last = r.u1 > r.u0 ? (int)((r.u1 - 1) / (unsigned int)C.ng_total) : -1;
    return r;
}

// the step's constants for blocks pb .. pb + nsg - 1 into shared memory, asynchronously: codebook, column scales,
// RMSNorm weight (16-byte cp.async chunks; every source is 16-byte aligned)
__device__ __forceinline__ void chain_stage_consts(const ChainStep &C, int pb, int nsg) {
    const int tid = threadIdx.x - 32;  // warps 1..: thread 0 keeps no copies in flight (it fences at the barrier)
    if (tid < 0) return;
    if (tid < 64) {
        cp_async16(g_smem + kChA + 16 * tid, C.A + 4 * tid);
    } else if (tid < 64 + 64 * nsg) {
        const int i = tid - 64;
        cp_async16(g_smem + kChIc + 16 * i, C.ic + 256 * pb + 4 * i);
    } else if (C.pro == P8_PROLOGUE_RMSNORM && tid < 64 + 128 * nsg) {
        const int i = tid - 64 - 64 * nsg;
        cp_async16(g_smem + kChPw + 16 * i, C.pw + 256 * pb + 4 * i);
    }
}

// ask L2 for unit (block b, row tile rr) of step C (payload, the unit's 32 row scales and row order)
__device__ __forceinline__ void chain_prefetch_br(const ChainStep &C, int b, int rr) {
    int ti = 0;
#pragma unroll
    for (int i = 1; i < kMaxGroup; ++i)
        if (i < C.nt && rr >= C.t[i].g0) ti = i;
    const ChainTensor &T = C.t[ti];
    const int g = rr - T.g0;
    const uint32_t tile = (uint32_t)g * (uint32_t)C.nb + (uint32_t)b;
    const uint32_t mt = T.ucls ? ((tile * (uint32_t)(64 * NW(T.ucls))) | ((uint32_t)T.ucls << 29)) : __ldg(T.M + tile);
    const int c = (int)(mt >> 29);
    if (c) bulk_prefetch_l2(T.D + (mt & 0x1FFFFFFFu), (uint32_t)(256 * NW(c)));
    prefetch_l2(T.S + (size_t)b * T.rows + g * 32);
    prefetch_l2(T.prm + g * 32);
}
__device__ __forceinline__ void chain_prefetch_unit(const ChainStep &C, unsigned int u) {
    const int b = (int)(u / (unsigned int)C.ng_total);
    chain_prefetch_br(C, b, (int)(u - (unsigned int)b * (unsigned int)C.ng_total));
}

// grid barrier: every CTA arrives once per barrier whether or not it still waits, so the counts stay consistent after
// a timeout (bit 5 of the device error word; the launch's results are invalid)
__device__ __forceinline__ void chain_barrier(unsigned int *cnt, unsigned int target, int *s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        // release: the CTA's partial stores (ordered before this thread by the CTA barrier) are visible before the
        // arrival is counted; acquire after the wait: the other CTAs' partials are visible to the loads that follow
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
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
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
    }
    __syncthreads();
}

// y of one output row of step `P` (tensor T): the slice-ordered sum of its partials `sum`, then the clamp delta on x'
// (in CSR order; only in blocks whose mask bit is set), the output scale (RMSNorm of the step's input), the residual
__device__ __forceinline__ float chain_row_out(const ChainTensor &T, int ro, float sum, const float *xv, float scale) {
    float y = sum;
    if ((T.dmask[ro >> 13] >> ((ro >> 8) & 31)) & 1u) {
        const int e1 = __ldg(T.cp + ro + 1);
        for (int e = __ldg(T.cp + ro); e < e1; ++e) y = __fadd_rn(y, __fmul_rn(__ldg(T.cv + e), __ldcg(xv + __ldg(T.cc + e))));
    }
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

// ---- the unit loop (class 3 in registers, other classes from memory)
// The chain's lookup-address registers pq[j] hold the lane's rotated chunk offsets of steps 2j and 2j + 1 in bytes 0
// and 1, the table buffer (0 / 1) of the unit's block in byte 2 and zero in byte 3. The PRMT selector of step k takes
// offset byte k % 2 -> bits 0-7, field byte k % 4 of word k / 4 -> bits 8-15, the buffer -> bits 16-23, zero -> 24-31.
template <int k>
struct SelBuf {
    static constexpr uint32_t v = (uint32_t)(4 + (k & 1)) | ((uint32_t)(k % 4) << 4) | 0x7600u;
};
template <int HS, int k>
struct ChStep3 {
    static __device__ __forceinline__ void run(const uint32_t (&w)[16], const uint32_t (&pq)[16], int &a) {
        a += lds_at<HS * 128>(__byte_perm(w[8 * HS + k / 4], pq[k / 2], SelBuf<k>::v));
        ChStep3<HS, k + 1>::run(w, pq, a);
    }
};
template <int HS>
struct ChStep3<HS, 32> {
    static __device__ __forceinline__ void run(const uint32_t (&)[16], const uint32_t (&)[16], int &) {}
};
// integer total of half-slice HS of a class-3 unit row: table sum + coset term (class 3: one stage, no shift, MC = 1);
// gbuf = buffer << 16 selects the coset table of the unit's block
template <int HS>
__device__ __forceinline__ int chain_slice3(const uint32_t (&w)[16], const uint32_t (&pq)[16], int lane, uint32_t gbuf) {
    uint32_t pm = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {  // z bits in step order (zbits_fast on this half-slice's words)
        const uint32_t x = (w[8 * HS + 2 * p + 1] & 0x80808080u) | ((w[8 * HS + 2 * p] >> 4) & 0x08080808u);
        pm |= ((x * 0x00204081u) >> 24) << (8 * p);
    }
    const uint32_t H = pingala8_h(__funnelshift_l(pm, pm, lane));
    int cs = 0;
#pragma unroll
    for (int grp = 0; grp < 8; ++grp) {
        const uint32_t sh = grp == 0 ? (H << 2) : (H >> (4 * grp - 2));
        cs += lds_at<kChG0 + HS * kGInts * 4>(((sh & 0x3Cu) | gbuf) + grp * 64);  // grp * 64 folds into the offset
    }
    int a = 0;
    ChStep3<HS, 0>::run(w, pq, a);
    return a + cs;
}
// other classes: lane words from memory, the generic lane-slice dot on the buffer's tables
template <int C, int BUF>
__device__ __noinline__ float chain_row_cls(const uint32_t *p0, int lane, float d0, float d1) {
    constexpr int T0 = BUF ? kSmemT1 : kSmemT0, G0 = BUF ? kChG1 : kChG0;
    uint32_t po[11];  // the generic loop's layout: three rotated chunk offsets per register
#pragma unroll
    for (int q = 0; q < 11; ++q) {
        uint32_t r = 0;
#pragma unroll
        for (int i = 0; i < 3; ++i)
            if (3 * q + i < 32) r |= (((uint32_t)(lane + 3 * q + i) & 31u) << 2) << (8 * i);
        po[q] = r;
    }
    uint32_t w[24];
    load_lane_words<C>(p0, 0, lane, w);
    const int i0 = lane_slice_dot<C, T0, G0>(w, po, lane);
    load_lane_words<C>(p0, 1, lane, w);
    const int i1 = lane_slice_dot<C, T0 + 128, G0 + kGInts * 4>(w, po, lane);
    return __fadd_rn(__fmul_rn((float)i0, d0), __fmul_rn((float)i1, d1));
}
template <int BUF>
__device__ __forceinline__ float chain_row_other(int c, const uint32_t *p0, int lane, float d0, float d1) {
    switch (c) {
        case 1: return chain_row_cls<1, BUF>(p0, lane, d0, d1);
        case 2: return chain_row_cls<2, BUF>(p0, lane, d0, d1);
        case 3: return chain_row_cls<3, BUF>(p0, lane, d0, d1);
        case 4: return chain_row_cls<4, BUF>(p0, lane, d0, d1);
        case 5: return chain_row_cls<5, BUF>(p0, lane, d0, d1);
        case 6: return chain_row_cls<6, BUF>(p0, lane, d0, d1);
        case 7: return chain_row_cls<7, BUF>(p0, lane, d0, d1);
        default: return 0.f;
    }
}

// one fetched unit of a warp: class-3 payload in registers (both half-slices), where its partial goes, its row scale
struct ChainUnit {
    uint32_t w[16];
    const uint32_t *p0;  // payload (other classes read it from here)
    float *dst;          // this lane's partial: block b, the row's ORIGINAL position
    uint32_t mt;         // class << 29 | payload word offset
    int b;
    uint16_t sc;
};
// fields of the tensor the warp's units currently belong to (reloaded from the descriptor when a unit leaves it)
struct ChainTensorCache {
    const uint32_t *M, *D;
    const uint16_t *S;
    const int16_t *prm;
    float *part;
    int rows, ucls, lo, hi;  // the tensor's row tiles are rr in [lo, hi) of the step's group
};
__device__ __forceinline__ void chain_tcache(const ChainStep &C, const uint8_t *pbase, int rr, ChainTensorCache &R) {
    int ti = 0;
#pragma unroll
    for (int i = 1; i < kMaxGroup; ++i)
        if (i < C.nt && rr >= C.t[i].g0) ti = i;
    const ChainTensor &T = C.t[ti];
    R.M = T.M; R.D = T.D; R.S = T.S; R.prm = T.prm; R.part = reinterpret_cast<float *>(const_cast<uint8_t *>(pbase) + T.part_off);
    R.rows = T.rows; R.ucls = T.ucls; R.lo = T.g0; R.hi = T.g0 + T.ng;
}
__device__ __forceinline__ void chain_fetch(const ChainStep &C, const uint8_t *pbase, ChainTensorCache &R, int b, int rr, int lane,
                                            ChainUnit &u) {
    if (rr < R.lo || rr >= R.hi) chain_tcache(C, pbase, rr, R);
    const int g = rr - R.lo;
    const uint32_t tile = (uint32_t)g * (uint32_t)C.nb + (uint32_t)b;
    u.mt = R.ucls ? ((tile * (uint32_t)(64 * NW(R.ucls))) | ((uint32_t)R.ucls << 29)) : __ldg(R.M + tile);
    u.p0 = R.D + (u.mt & 0x1FFFFFFFu);
    if ((u.mt >> 29) == 3) load3(u.p0, lane, u.w);
    u.sc = __ldg(R.S + (size_t)b * R.rows + g * 32 + lane);
    u.dst = R.part + (size_t)b * R.rows + __ldg(R.prm + g * 32 + lane);
    u.b = b;
}
// the unit's partial: its table buffer comes from pq byte 2 / gbuf (set for block pb + buf by the caller)
__device__ __forceinline__ void chain_do_unit(const ChainUnit &u, const uint32_t (&pq)[16], int lane, int buf, const float *d_s) {
    const float d0 = d_s[2 * buf], d1 = d_s[2 * buf + 1];
    const int c = (int)(u.mt >> 29);
    float part;
    if (c == 3) {
        const uint32_t gbuf = (uint32_t)buf << 16;
        const int i0 = chain_slice3<0>(u.w, pq, lane, gbuf), i1 = chain_slice3<1>(u.w, pq, lane, gbuf);
        part = __fadd_rn(__fmul_rn((float)i0, d0), __fmul_rn((float)i1, d1));
    } else {
        part = buf ? chain_row_other<1>(c, u.p0, lane, d0, d1) : chain_row_other<0>(c, u.p0, lane, d0, d1);
    }
    *u.dst = __fmul_rn(part, h2f(u.sc));
}

// row i of the concatenation of step P's not-passed-on tensors -> (tensor, row); ti = -1 past the end
__device__ __forceinline__ void chain_unc_row(const ChainStep &P, int i, int &ti, int &ro) {
    ti = -1;
    ro = 0;
    int off = i;
    for (int q = 0; q < P.nunc; ++q) {
        const int t = P.unc[q];
        if (off < P.t[t].rows) {
            ti = t;
            ro = off;
            return;
        }
        off -= P.t[t].rows;
    }
}

// The prep's reduction of step P's partials with every load in flight before one shared-memory exchange:
//   rows [ra, rb) of P's not-passed-on tensors, reduced and written to their outputs, up to 256 per round (thread
//   (r, k) sums rows ra + r + 64 j, j < 4, over blocks k, k + 8, ...);
//   in the first round, the input blocks pb .. pb + nsg - 1 of this step from sources xsrc / x2src (a tensor of P, or
//   -1 for memory at xext / x2ext) into dst / dst2 (8 slices x 64 float4 columns per block); the owner of a block
//   writes its reduced rows to the output.
// Slices are summed in slice order, so a row's value does not depend on which CTA reduced it.
__device__ void chain_reduce(const ChainStep *P, const ChainArgs &a, int pp, int ra, int rb, int xsrc, const float *xext,
                             int x2src, const float *x2ext, int pb, int nsg, unsigned own, float scale, float *dst,
                             float *dst2) {
    const int tid = threadIdx.x, j4 = tid & 63, k = tid >> 6;
    float *red_x = reinterpret_cast<float *>(g_smem + kChRed);            // [2][8][256]
    float *red_x2 = reinterpret_cast<float *>(g_smem + kChRed + 16384);   // [2][8][256]
    float *red_sh = reinterpret_cast<float *>(g_smem + kChRedShare);      // [8][256]
    const float *xv = P ? reinterpret_cast<const float *>(a.ws + a.xv[pp]) : nullptr;
    const uint8_t *pbase = a.ws + a.part[pp];
    for (int base = ra;; base += 256) {
        const bool first = base == ra;
        // ---- loads: the share rows' slices, then the input blocks' slices
        if (P && base < rb) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                int ti, ro;
                float acc = 0.f;
                if (base + j4 + 64 * j < rb) {
                    chain_unc_row(*P, base + j4 + 64 * j, ti, ro);
                    if (ti >= 0) {
                        const ChainTensor &T = P->t[ti];
                        const float *p = reinterpret_cast<const float *>(pbase + T.part_off) + ro;
                        for (int bb = k; bb < P->nb; bb += 8) acc = __fadd_rn(acc, __ldcg(p + (size_t)bb * T.rows));
                    }
                }
                red_sh[k * 256 + j4 + 64 * j] = acc;
            }
        }
        if (first && P) {
            for (int sg = 0; sg < nsg; ++sg) {
                if (xsrc >= 0) {
                    const ChainTensor &T = P->t[xsrc];
                    chain_slices_256(reinterpret_cast<const float *>(pbase + T.part_off), T.rows, P->nb, 256 * (pb + sg), red_x + sg * 2048);
                }
                if (x2src >= 0) {
                    const ChainTensor &T = P->t[x2src];
                    chain_slices_256(reinterpret_cast<const float *>(pbase + T.part_off), T.rows, P->nb, 256 * (pb + sg), red_x2 + sg * 2048);
                }
            }
        }
        __syncthreads();
        // ---- epilogues
        if (P && tid < rb - base && tid < 256) {
            int ti, ro;
            chain_unc_row(*P, base + tid, ti, ro);
            if (ti >= 0) {
                const ChainTensor &T = P->t[ti];
                T.Y[ro] = chain_row_out(T, ro, chain_sum_slices(red_sh, 256, tid), xv, scale);
            }
        }
        if (first && tid < 256 * nsg) {
            const int sg = tid >> 8, r = tid & 255, ro = 256 * (pb + sg) + r;
            if (xsrc >= 0) {
                const ChainTensor &T = P->t[xsrc];
                const float y = chain_row_out(T, ro, chain_sum_slices(red_x + sg * 2048, 256, r), xv, scale);
                dst[tid] = y;
                if ((own >> sg) & 1u) T.Y[ro] = y;
            } else if (xext) {
                dst[tid] = __ldcg(xext + 256 * pb + tid);
            }
            if (x2src >= 0) {
                const ChainTensor &T = P->t[x2src];
                const float y = chain_row_out(T, ro, chain_sum_slices(red_x2 + sg * 2048, 256, r), xv, scale);
                dst2[tid] = y;
                if ((own >> sg) & 1u) T.Y[ro] = y;
            } else if (x2ext) {
                dst2[tid] = __ldcg(x2ext + 256 * pb + tid);
            }
        }
        __syncthreads();
        if (base + 256 >= rb) break;
    }
}

__global__ void __launch_bounds__(kChainThreads, 1) k_chain(const __grid_constant__ ChainArgs a) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ int s_ok;
    __shared__ float s_scale;
    float *xs = reinterpret_cast<float *>(g_smem + kChX);
    float *x2s = reinterpret_cast<float *>(g_smem + kChX2);
    int *cx_s = reinterpret_cast<int *>(g_smem + kChCx);
    float *d_s = reinterpret_cast<float *>(g_smem + kChD);
    float *ssp = d_s + 4;  // [2][8] per-warp partial sums of squares
    const uint32_t *A_s = reinterpret_cast<const uint32_t *>(g_smem + kChA);
    const float *ic_s = reinterpret_cast<const float *>(g_smem + kChIc);
    const float *pw_s = reinterpret_cast<const float *>(g_smem + kChPw);
    pdl_launch_dependents();
    uint32_t pq[16];  // lookup-address registers (SelBuf): chunk offsets of steps 2j, 2j + 1, table buffer, zero
#pragma unroll
    for (int j = 0; j < 16; ++j)
        pq[j] = ((((uint32_t)(lane + 2 * j) & 31u) << 2)) | ((((uint32_t)(lane + 2 * j + 1) & 31u) << 2) << 8);
    int cur_buf = 0;  // the table buffer in pq byte 2
    if (tid == 0) s_ok = 1;
    // ---- before the wait for the previous kernel: the descriptors of the previous, first and second phase of this
    // launch, the first step's constants and first units (all of it the plan's and the weights', which no earlier
    // kernel writes)
    const int s0 = a.s_begin;
    if (s0 >= 1) chain_load_step(a, s0 - 1);
    if (s0 < a.nsteps) chain_load_step(a, s0);
    if (s0 + 1 < a.nsteps && a.s_end > s0) chain_load_step(a, s0 + 1);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    if (s0 < a.nsteps) chain_load_range(a, s0, a.cuts + (size_t)s0 * gridDim.x);
    if (s0 + 1 < a.nsteps && a.s_end > s0) chain_load_range(a, s0 + 1, a.cuts + (size_t)(s0 + 1) * gridDim.x);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    if (s0 < a.nsteps) {
        const ChainRange r0 = chain_range(*chain_slot(s0));
        if (r0.b_last >= r0.b_first) chain_stage_consts(*chain_slot(s0), r0.b_first, r0.b_last - r0.b_first + 1 < 2 ? 1 : 2);
        cp_async_commit();
        for (int j = 0; j < a.pf; ++j)
            if (lane == 1 && r0.u0 + warp + kChainWarps * j < r0.u1) chain_prefetch_unit(*chain_slot(s0), r0.u0 + warp + kChainWarps * j);
    }
    pdl_wait();  // inputs, workspace and barrier words belong to earlier kernels until they complete
    for (int s = s0; s <= a.s_end; ++s) {
        const ChainStep *P = s > 0 ? chain_slot(s - 1) : nullptr;
        cp_async_wait_all();  // this step's constants (and the descriptor of step s + 1 copied during step s - 1)
        if (tid < 32) {       // output scale of the previous step (its input's RMSNorm), from its blocks' sums of squares
            float sc = 1.f;
            if (P && P->pro == P8_PROLOGUE_RMSNORM) sc = chain_scale(*P, reinterpret_cast<const float *>(a.ws + a.ss[(s - 1) & 1]));
            if (lane == 0) s_scale = sc;
        }
        __syncthreads();
        const float scale_p = s_scale;
        const int pp = (s - 1) & 1;
        unsigned long long *tr = a.trace && s < a.nsteps ? a.trace + ((size_t)s * gridDim.x + blockIdx.x) * 8 : nullptr;
        if (tr && tid == 0) tr[0] = global_ns();
        if (s == a.nsteps) {  // final phase: the last step's rows in equal shares
            if (P && s_ok) {
                const int R = P->unc_rows;
                chain_reduce(P, a, pp, (int)((long long)R * blockIdx.x / gridDim.x), (int)((long long)R * (blockIdx.x + 1) / gridDim.x),
                             -1, nullptr, -1, nullptr, 0, 0, 0u, scale_p, nullptr, nullptr);
            }
            break;
        }
        const ChainStep &C = *chain_slot(s);
        const int cp_ = s & 1;
        // ---- this CTA's units of step s: [u0, u1) of the block-major list; warp w takes u0 + w, u0 + w + 16, ...
        const ChainRange rg = chain_range(C);
        const unsigned int u0 = rg.u0, u1 = rg.u1;
        const int b_first = rg.b_first, b_last = rg.b_last;
        const unsigned int ngt = (unsigned int)C.ng_total;
        const int rr_first = (int)(u0 - (unsigned int)b_first * ngt);
        unsigned int un = u0 + warp;  // the warp's next unit to fetch: block cb, row tile crr of the group
        int cb = (int)(un / ngt), crr = (int)(un - (unsigned int)cb * ngt);
        auto advance = [&]() {
            un += kChainWarps;
            crr += kChainWarps;
            while (crr >= (int)ngt) {
                crr -= (int)ngt;
                ++cb;
            }
        };
        unsigned int pun = un + kChainWarps * (unsigned int)a.pf;  // the unit the warp asks L2 for next
        int pcb = (int)(pun / ngt), pcrr = (int)(pun - (unsigned int)pcb * ngt);
        auto pf_step = [&]() {
            if (lane == 1 && pun < u1) chain_prefetch_br(C, pcb, pcrr);
            pun += kChainWarps;
            pcrr += kChainWarps;
            while (pcrr >= (int)ngt) {
                pcrr -= (int)ngt;
                ++pcb;
            }
        };
        const uint8_t *pbase = a.ws + a.part[cp_];
        ChainTensorCache R;
        R.lo = R.hi = 0;  // loaded by the first fetch
        ChainUnit uA, uB;
        bool fa = false, fb = false;
        if (un < u1) {  // weights only: the first unit's loads overlap the prep below
            chain_fetch(C, pbase, R, cb, crr, lane, uA);
            fa = true;
            advance();
        }
        // rows of the previous step that this step does not read: equal shares (reduced with the first block pair)
        const int sh_r = P ? P->unc_rows : 0;
        const int sh_a = (int)((long long)sh_r * blockIdx.x / gridDim.x), sh_b = (int)((long long)sh_r * (blockIdx.x + 1) / gridDim.x);
        float *xv_c = reinterpret_cast<float *>(a.ws + a.xv[cp_]);
        float *ss_c = reinterpret_cast<float *>(a.ws + a.ss[cp_]);
        if (b_last < b_first && s_ok && sh_b > sh_a)  // no units this step: only the share of rows
            chain_reduce(P, a, pp, sh_a, sh_b, -1, nullptr, -1, nullptr, 0, 0, 0u, scale_p, nullptr, nullptr);
        for (int pb = b_first; pb <= b_last; pb += 2) {
            const int nsg = b_last - pb + 1 < 2 ? b_last - pb + 1 : 2;
            if (pb != b_first) {  // later pairs (only when a CTA's units span more than two blocks): constants now
                chain_stage_consts(C, pb, nsg);
                cp_async_commit();
                cp_async_wait_all();
                __syncthreads();
            }
            unsigned own = 0;  // blocks whose first unit is this CTA's
            for (int sg = 0; sg < nsg; ++sg)
                if (pb + sg > b_first || rr_first == 0) own |= 1u << sg;
            // ---- (a) input values of the pair's blocks (fused reduce of the previous step, or memory), with the
            // previous step's not-passed-on rows of this CTA's share in the same loads-then-exchange round
            if (s_ok) {
                const bool sw = C.pro == P8_PROLOGUE_SWIGLU;
                chain_reduce(P, a, pp, pb == b_first ? sh_a : 0, pb == b_first ? sh_b : 0, C.xsrc, C.x, sw ? C.x2src : -1,
                             sw ? C.x2 : nullptr, pb, nsg, own, scale_p, xs, x2s);
            }
            __syncthreads();
            if (tr && tid == 0 && pb == b_first) tr[1] = global_ns();
            // ---- (b) input op: x' (RMSNorm: x * w, its scale goes to the output; SwiGLU: silu(x) * up); the owner
            // writes x' (clamp-delta term of this step's outputs) and the block's sum of x^2 (RMSNorm scale)
            if (tid < 256 * nsg) {
                const int sg = tid >> 8, col = 256 * (pb + sg) + (tid & 255);
                const float x = xs[tid];
                float xp = x;
                if (C.pro == P8_PROLOGUE_RMSNORM) {
                    xp = __fmul_rn(x, pw_s[tid]);
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
            // ---- (c) FWHT(x' sgn/c) / 16 and the x16 quantisation per 128 columns (warp sg: block pb + sg). Lane l holds
            // columns 8l .. 8l + 7 = chunks 2l and 2l + 1: it packs each chunk's ints as int8x4 hi / lo words (q = 128 hi
            // + lo, both within int8) for the table's dp4a, and computes the chunks' coset products <c, q_t>.
            if (warp < nsg) {
                const float *icp = ic_s + 256 * warp + 8 * lane;
                const float *xp = xs + 256 * warp + 8 * lane;
                float v[8];
#pragma unroll
                for (int m = 0; m < 8; ++m) v[m] = __fmul_rn(xp[m], icp[m]);
                fwht256_warp(v, lane);
                float am = 0.f;
#pragma unroll
                for (int m = 0; m < 8; ++m) am = fmaxf(am, fabsf(v[m]));
#pragma unroll
                for (int o = 1; o < 16; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                const float d = __fdiv_rn(am, 8191.f), id = d > 0.f ? __fdiv_rn(1.f, d) : 0.f;
                uint32_t hl[4] = {0u, 0u, 0u, 0u};  // chunk 2l: hi, lo; chunk 2l + 1: hi, lo
                int cx[2] = {0, 0};
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    const int q = __float2int_rn(__fmul_rn(v[m], id));
                    const int hi = (q + 64) >> 7, lo = q - 128 * hi;
                    hl[2 * (m >> 2)] |= ((uint32_t)hi & 0xffu) << (8 * (m & 3));
                    hl[2 * (m >> 2) + 1] |= ((uint32_t)lo & 0xffu) << (8 * (m & 3));
                    cx[m >> 2] += (int)(int8_t)(C.cs >> (8 * (m & 3))) * q;
                }
                *reinterpret_cast<uint4 *>(g_smem + kChHL + 512 * warp + 16 * lane) = make_uint4(hl[0], hl[1], hl[2], hl[3]);
                *reinterpret_cast<int2 *>(cx_s + 64 * warp + 2 * lane) = make_int2(cx[0], cx[1]);
                if ((lane & 15) == 0) d_s[2 * warp + (lane >> 4)] = d;
            }
            __syncthreads();
            if (tr && tid == 0 && pb == b_first) tr[2] = global_ns();
            if (tid < 256 * nsg) {  // coset nibble tables: G[hs][grp][m] = sum over set bits i of m of <c, q_(32 hs + 4 grp + i)>
                const int sg = tid >> 8, e = tid & 255, hs = e >> 7, grp = (e >> 4) & 7, m = e & 15;
                int gs = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if ((m >> i) & 1) gs += cx_s[64 * sg + 32 * hs + 4 * grp + i];
                reinterpret_cast<int *>(g_smem + (sg ? kChG1 : kChG0))[hs * kGInts + grp * 16 + m] = gs;
            }
            // ---- (d) the 64 KiB table of each block: T[f][hs * 32 + t] = <A[f], q_(hs, t)> = 128 dp4a(A[f], hi) +
            // dp4a(A[f], lo), exact; four consecutive chunks per thread and 16-byte stores
            {
                const int h4 = tid & 15, fr = tid >> 4;
                for (int sg = 0; sg < nsg; ++sg) {
                    const uint4 p0 = *reinterpret_cast<const uint4 *>(g_smem + kChHL + 512 * sg + 32 * h4);
                    const uint4 p1 = *reinterpret_cast<const uint4 *>(g_smem + kChHL + 512 * sg + 32 * h4 + 16);
                    const int H[4] = {(int)p0.x, (int)p0.z, (int)p1.x, (int)p1.z}, Lo[4] = {(int)p0.y, (int)p0.w, (int)p1.y, (int)p1.w};
                    int *T = reinterpret_cast<int *>(g_smem + (sg ? kSmemT1 : kSmemT0));
#pragma unroll 4
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
            if (tr && tid == 0 && pb == b_first) tr[3] = global_ns();
            // ---- (e) units of the pair's blocks, two register buffers in turn (the next unit's loads are in flight
            // while one computes); each warp keeps pf units ahead of itself asked of L2
            if (!fa && un < u1 && cb < pb + nsg) {
                chain_fetch(C, pbase, R, cb, crr, lane, uA);
                fa = true;
                advance();
            }
            auto set_buf = [&](int buf) {  // table buffer of the unit's block into pq byte 2
                if (buf != cur_buf) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) pq[j] = (pq[j] & 0x0000FFFFu) | ((uint32_t)buf << 16);
                    cur_buf = buf;
                }
            };
            while (s_ok) {
                if (!fa || uA.b >= pb + nsg) break;
                fb = un < u1 && cb < pb + nsg;
                if (fb) {
                    chain_fetch(C, pbase, R, cb, crr, lane, uB);
                    advance();
                }
                pf_step();
                set_buf(uA.b - pb);
                chain_do_unit(uA, pq, lane, uA.b - pb, d_s);
                fa = false;
                if (!fb) break;
                fa = un < u1 && cb < pb + nsg;
                if (fa) {
                    chain_fetch(C, pbase, R, cb, crr, lane, uA);
                    advance();
                }
                pf_step();
                set_buf(uB.b - pb);
                chain_do_unit(uB, pq, lane, uB.b - pb, d_s);
                fb = false;
                if (!fa) break;
            }
            __syncthreads();
        }
        if (tr && tid == 0) tr[4] = global_ns();
        if (s == a.s_end) break;  // the next phase is the next launch: the kernel boundary is its barrier
        // ---- the next steps, while this CTA waits at the barrier. Step s + 2's descriptor goes to the slot of step
        // s - 1, which nothing reads any more; step s + 1's (copied during step s - 1) is here: ask L2 for every
        // warp's first units and copy the step's constants for this CTA's blocks into shared memory
        if (s + 2 < a.nsteps) {
            chain_load_step(a, s + 2);
            chain_load_range(a, s + 2, a.cuts + (size_t)(s + 2) * gridDim.x);
        }
        if (s + 1 < a.nsteps) {
            const ChainStep &N = *chain_slot(s + 1);
            const ChainRange rn = chain_range(N);
            if (lane == 1)  // lane 1: thread 0 keeps no prefetch in flight when it fences at the barrier
                for (int j = 0; j < a.pf; ++j)
                    if (rn.u0 + warp + kChainWarps * j < rn.u1) chain_prefetch_unit(N, rn.u0 + warp + kChainWarps * j);
            if (rn.b_last >= rn.b_first) chain_stage_consts(N, rn.b_first, rn.b_last - rn.b_first + 1 < 2 ? 1 : 2);
            cp_async_commit();
        }
        chain_barrier(a.sync, (unsigned int)(s + 1) * gridDim.x, &s_ok);
        if (tr && tid == 0) tr[5] = global_ns();
    }
    // ---- exit: the last CTA out resets the barrier words for the next launch (every CTA has passed every barrier);
    // a one-phase launch met no barrier
    cp_async_wait_all();
    __syncthreads();
    if (tid == 0 && a.s_end > a.s_begin) {
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
    int device, nsteps, ctas;
    uint2 *d_cuts;              // [nsteps][ctas] unit ranges
    unsigned long long *trace;  // optional phase trace buffer (device), set by p8_chain_trace
    p8::ChainStep *d_steps;
    unsigned int *d_sync;
    unsigned long long part[2], xv[2], ss[2];
    size_t ws_bytes;
};

namespace p8 {

constexpr uint32_t kChainMagic = 0x50384348u;

// Contiguous ranges of a step's block-major unit list for G CTAs that minimise the largest per-CTA cost: a unit counts
// 1 and each 256-column block a CTA touches counts tc more (the table it builds and the block's input it reduces).
// Binary search on the cost bound with greedy packing; every CTA of the result holds a contiguous, possibly empty range.
static void chain_partition(unsigned units, unsigned ngt, int G, unsigned tc, uint2 *out) {
    auto pack = [&](unsigned cap, uint2 *o) -> bool {
        unsigned a = 0;
        for (int c = 0; c < G; ++c) {
            unsigned e = a, cost = 0;
            while (e < units && cost + tc < cap) {
                const unsigned bend = (e / ngt + 1) * ngt;
                const unsigned take = std::min(cap - cost - tc, bend - e);
                e += take;
                cost += tc + take;
                if (e < bend) break;
            }
            if (o) o[c] = make_uint2(a, e);
            a = e;
        }
        return a >= units;
    };
    unsigned lo = 1, hi = units + tc * (units / ngt + 1) + 1;  // one CTA holding everything fits hi
    while (lo < hi) {
        const unsigned mid = lo + (hi - lo) / 2;
        if (pack(mid, nullptr)) hi = mid; else lo = mid + 1;
    }
    pack(lo, out);
}

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
            memcpy(T.dmask, t->delta_blocks, sizeof(T.dmask));
            poff += ((size_t)t->nb * t->rows * 4 + 255) & ~(size_t)255;
            g0 += t->ng;
        }
        c.ng_total = g0;
        c.units = (unsigned int)g0 * (unsigned int)c.nb;  // <= 4092 tiles x 255 blocks
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
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != dev) return P8_ERR_ARG;  // the tensors' device must be current
    const int G = sm_count();
    const unsigned tc = [] {  // table cost in units for the range balance (P8_CHAIN_TC; tuning knob)
        const char *e = getenv("P8_CHAIN_TC");
        return e ? (unsigned)atoi(e) : 10u;
    }();
    std::vector<uint2> cuts((size_t)n * G);
    for (int s = 0; s < n; ++s)
        chain_partition(hs[(size_t)s].units, (unsigned)hs[(size_t)s].ng_total, G, tc, cuts.data() + (size_t)s * G);
    p8_chain *p = new p8_chain();
    p->magic = kChainMagic;
    p->device = dev;
    p->nsteps = n;
    p->ctas = G;
    size_t o = 0;
    for (int i = 0; i < 2; ++i) { p->part[i] = o; o += part_max; }
    for (int i = 0; i < 2; ++i) { p->xv[i] = o; o += (4 * k_max + 255) & ~(size_t)255; }
    for (int i = 0; i < 2; ++i) { p->ss[i] = o; o += (4 * nb_max + 255) & ~(size_t)255; }
    p->ws_bytes = o;
    p->d_steps = nullptr;
    p->d_sync = nullptr;
    p->d_cuts = nullptr;
    p->trace = nullptr;
    bool ok = cudaMalloc((void **)&p->d_cuts, sizeof(uint2) * cuts.size()) == cudaSuccess;
    for (int s = 0; ok && s < n; ++s) hs[(size_t)s].cuts = p->d_cuts + (size_t)s * G;
    ok = ok && cudaMalloc((void **)&p->d_steps, sizeof(ChainStep) * (size_t)n) == cudaSuccess &&
         cudaMalloc((void **)&p->d_sync, 256) == cudaSuccess &&
         cudaMemcpy(p->d_cuts, cuts.data(), sizeof(uint2) * cuts.size(), cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(p->d_steps, hs.data(), sizeof(ChainStep) * (size_t)n, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemset(p->d_sync, 0, 256) == cudaSuccess;
    if (!ok) {
        cudaFree(p->d_steps);
        cudaFree(p->d_sync);
        cudaFree(p->d_cuts);
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
    cudaFree(p->d_cuts);
    p->magic = 0;
    delete p;
    return P8_OK;
}

size_t chain_workspace(const p8_chain *p) { return p && p->magic == kChainMagic ? p->ws_bytes : 0; }

p8_status chain_trace(p8_chain *p, unsigned long long *buf, size_t words) {
    if (!p || p->magic != kChainMagic) return P8_ERR_ARG;
    if (buf && words < (size_t)p->nsteps * (size_t)p->ctas * 8) return P8_ERR_WORKSPACE;
    p->trace = buf;
    return P8_OK;
}

p8_status chain_run(const p8_chain *p, void *ws, size_t ws_bytes, cudaStream_t st, int pf) {
    if (!p || p->magic != kChainMagic) return P8_ERR_ARG;
    if (!ws || ws_bytes < p->ws_bytes || ((uintptr_t)ws & 255)) return P8_ERR_WORKSPACE;
    static std::atomic<bool> attr[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return P8_ERR_CUDA;
    if (dev != p->device || sm_count() != p->ctas) return P8_ERR_ARG;
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
    a.trace = p->trace;
    a.cuts = p->d_cuts;
    // one launch per phase (steps, then the last step's rows), each waiting on the previous one with programmatic
    // dependent launch: a kernel boundary costs less than a grid barrier (measured ~0.9 us against ~1.6 us after the
    // last arrival), and a launch starts while the previous one's last CTAs still run
    for (int s = 0; s <= p->nsteps; ++s) {
        a.s_begin = a.s_end = s;
        void *args[] = {&a};
        if (launch_pdl((const void *)k_chain, dim3((unsigned)p->ctas), dim3(kChainThreads), kChSmem, st, args) != cudaSuccess)
            return P8_ERR_CUDA;
    }
    return P8_OK;
}
