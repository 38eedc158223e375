// p8_gemm.cuh -- batched (prefill) Pingala-8 matmul on the 5th-generation tensor cores: tcgen05 MMA with the
// accumulator in tensor memory (TMEM), operands in shared memory written by decoder warps (weights) and by bulk copies
// (activations). Included by p8_kernels.cu, so it shares that file's device error word and launch helpers.
//
// The reference batch path (ggml_cuda_f44_mul_mat_q8, CU:1014-1054; the CPU batch path CP:1201-1262) computes
//     Y[n][ro] = sum_k W[ro][k] X[n][k],   W = H256(int * S) / 16 * (sgn / c) + Delta        (vrc_dequant_f32)
// The 256-point Walsh-Hadamard transform H is symmetric, sum_i H(u)_i v_i = sum_i u_i H(v)_i, so the transform moves to
// the activations:
//     Y[n][prm[r]] = sum_b sum_i (int[r][b,i] * S[b][r]) * Xr[n][b,i]  +  (Delta X)[n][prm[r]]
//     Xr[n][b, :]  = H256(X[n][b, :] * sgn/c) / 16
// and the weight operand is the decoded integer times its tile scale: the decoder writes MMA operands straight from the
// payload, with no transform on the weight side.
//
// Operands are fp16, accumulation fp32 (kind::f16). Power-of-two scales keep both operands in range and are multiplied
// out exactly in the epilogue: per sorted row 2^sigma_r with max_b |S[b][r]| * max|int| * 2^sigma_r < 2^15 (computed at
// prepare time, rsc), per token 2^tau_n with max |Xr[n]| < 2^14. The only rounding besides fp32 accumulation is fp16
// rounding of the two operands (about 3e-4 relative L2 error against the exact product).
//
//   k_gx_max   grid (Npad, K/2048 rounded up), 256 thr: partial max |X[n] * sgn/c| over 2048 columns.
//   k_gx_prep  grid (Npad/8, nb/4 rounded up), 256 thr, warp = token: tau from the partial maxima; Xr as fp16 in the
//              operand layout below ([half-slice][token group of 8][16 core matrices][8 tokens][8 columns]), so the
//              GEMM moves one B stage with one bulk copy.
//   k_gemm     grid (rows/128 rounded up, Npad/BN), 320 thr, 1 CTA per SM:
//              warps 0-7  decoders: warp (q, hs) decodes half-slice hs of row tile q (32 rows) of every 256-column
//                         block into the A stage as fp16 int * S * 2^sigma; then the epilogue (TMEM -> registers,
//                         scales, clamp delta, y[n][prm[r]]);
//              warp 8     one lane bulk-copies each B stage (BN tokens x 128 columns) onto the stage's mbarrier;
//              warp 9     allocates TMEM; one lane issues 8 MMAs (M = 128, N = BN, K = 16) per stage and commits them to
//                         the stage's 'empty' barrier, and after the last stage to the accumulator barrier.
// One stage = one 128-column half-slice: A 128 x 128 fp16 (32 KB), B BN x 128 fp16. Shared-memory operand layout,
// both operands (UMMA K-major, no swizzle): a core matrix is 8 rows x 8 fp16, 16 B per row, 128 B contiguous;
//     byte(row, col) = (row >> 3) * 2048 + (col >> 3) * 128 + (row & 7) * 16 + (col & 7) * 2
// so descriptor LBO (next core matrix along K) = 128 B and SBO (next group of 8 rows) = 2048 B. A decoder lane owns
// one row and writes 16 B (two 4-column chunks) per store; eight lanes cover the 32 banks, so stores are conflict-free.
//
// Every mbarrier wait is bounded; a wait that gives up sets bit 2 (value 4) of the device error word, the kernel
// still drains its own copies and MMAs, frees its TMEM and returns (results of that launch are invalid).

constexpr int kGemmThreads = 320;
constexpr int kGemmStageA = 32768;                  // 128 rows x 128 columns fp16
constexpr int kGemmOperandBudget = 196608;          // bytes of shared memory for the stage ring
constexpr int kGemmMaxStages = 8;
constexpr int kGemmAH = 512 * 8;                    // fp16 (codebook + h * coset) table for the one-stage classes
constexpr uint32_t kGemmPolls = 1u << 22;
constexpr int kGemmMinCols = 8;                     // below this the per-column table GEMV is faster

struct GemmArgs {
    const uint32_t *A, *M, *D;
    const uint16_t *S;
    const int16_t *prm;
    const float2 *rsc;     // per sorted row {2^sigma, 2^-sigma}
    const int *cp;
    const uint16_t *cc;
    const float *cv;
    const float *X;
    float *Y;
    const uint8_t *Xh;     // prepared activations (operand layout)
    const float *tdown;    // per token 2^-tau
    long long ldx, ldy;
    uint32_t cs;
    int rows, nb, ng, ncols, npad, bn, nst, ucls;
};

struct GxArgs {
    const float *X;
    const float *ic;
    float *pmax;           // [npad][nkc]
    uint8_t *Xh;
    float *tdown;
    long long ldx;
    int K, nb, ncols, npad, nkc;
};

// ---------------------------------------------------------------------------------------------------------------
// tcgen05 / TMEM wrappers (PTX ISA 8.6+, sm_100a)
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_alloc(uint32_t *slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, both K-major; accumulate = 0 overwrites D
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// arrive on the mbarrier once every MMA this thread issued so far has completed
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 32 TMEM lanes (one per thread of the warp) x 16 consecutive 32-bit columns
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];\n"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// shared-memory matrix descriptor: no swizzle, K-major, LBO 128 B, SBO 2048 B, descriptor version 1 (sm_100)
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128u >> 4) << 16) | ((uint64_t)(2048u >> 4) << 32) |
           ((uint64_t)1 << 46);
}
// instruction descriptor: D f32, A = B = f16, both K-major, N = bn, M = 128
__host__ __device__ constexpr uint32_t umma_idesc_f16(int bn) {
    return (1u << 4) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }  // e in [-126, 127]
// smallest e with |v| < 2^e, for finite v > 0 (normal or subnormal)
__device__ __forceinline__ int exp_above(float v) { return (int)((__float_as_uint(v) >> 23) & 0xFFu) - 126; }

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// ---------------------------------------------------------------------------------------------------------------
// per-row weight scale 2^sigma_r (prepare time): max_b |S[b][r]| * bint * 2^sigma < 2^15, bint = max |int| of the tensor
__global__ void __launch_bounds__(256) k_row_scale(const uint16_t *S, int rows, int nb, float bint, float2 *rsc) {
    const int r = blockIdx.x * 256 + threadIdx.x;
    if (r >= rows) return;
    float m = 0.f;
    for (int b = 0; b < nb; ++b) m = fmaxf(m, fabsf(h2f(S[(size_t)b * rows + r])));
    const float v = m * bint;
    int sg = 0;
    if (v > 0.f && v <= 3.0e38f) sg = min(126, max(-126, 15 - exp_above(v)));
    rsc[r] = make_float2(pow2f(sg), pow2f(-sg));
}

// ---------------------------------------------------------------------------------------------------------------
// activation prep
__global__ void __launch_bounds__(256) k_gx_max(const GxArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float red[8];
    const int n = blockIdx.x, col = blockIdx.y * 2048 + threadIdx.x * 8;
    float m = 0.f;
    if (n < a.ncols && col < a.K) {
        const float4 *xp = reinterpret_cast<const float4 *>(a.X + (size_t)n * a.ldx + col);
        const float4 *ip = reinterpret_cast<const float4 *>(a.ic + col);
        const float4 x0 = xp[0], x1 = xp[1], i0 = ip[0], i1 = ip[1];
        m = fmaxf(fmaxf(fmaxf(fabsf(x0.x * i0.x), fabsf(x0.y * i0.y)), fmaxf(fabsf(x0.z * i0.z), fabsf(x0.w * i0.w))),
                  fmaxf(fmaxf(fabsf(x1.x * i1.x), fabsf(x1.y * i1.y)), fmaxf(fabsf(x1.z * i1.z), fabsf(x1.w * i1.w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = red[0];
        for (int i = 1; i < 8; ++i) v = fmaxf(v, red[i]);
        a.pmax[(size_t)n * a.nkc + blockIdx.y] = v;
    }
}

__global__ void __launch_bounds__(256) k_gx_prep(const GxArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + warp;
    float m = lane < a.nkc ? a.pmax[(size_t)n * a.nkc + lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // |Xr| <= 16 max|x * sgn/c| < 16 * 2^e  ->  tau = 10 - e gives |Xr * 2^tau| < 2^14
    int tau = 0;
    if (m > 0.f && m <= 3.0e38f) tau = min(126, max(-126, 10 - exp_above(m)));
    const float up = pow2f(tau);
    if (blockIdx.y == 0 && lane == 0) a.tdown[n] = pow2f(-tau);
    const size_t panel = (size_t)a.npad * 256;
    for (int i = 0; i < 4; ++i) {
        const int b = blockIdx.y * 4 + i;
        if (b >= a.nb) break;
        float v[8];
        if (n < a.ncols) {
            const float4 *xp = reinterpret_cast<const float4 *>(a.X + (size_t)n * a.ldx + b * 256 + 8 * lane);
            const float4 *ip = reinterpret_cast<const float4 *>(a.ic + b * 256 + 8 * lane);
            const float4 x0 = xp[0], x1 = xp[1], i0 = ip[0], i1 = ip[1];
            v[0] = __fmul_rn(x0.x, i0.x); v[1] = __fmul_rn(x0.y, i0.y); v[2] = __fmul_rn(x0.z, i0.z); v[3] = __fmul_rn(x0.w, i0.w);
            v[4] = __fmul_rn(x1.x, i1.x); v[5] = __fmul_rn(x1.y, i1.y); v[6] = __fmul_rn(x1.z, i1.z); v[7] = __fmul_rn(x1.w, i1.w);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = 0.f;
        }
        fwht256_warp(v, lane);  // lane holds columns 8 lane .. 8 lane + 7 of the block, already / 16
        uint4 o;
        o.x = h2u(__floats2half2_rn(v[0] * up, v[1] * up));
        o.y = h2u(__floats2half2_rn(v[2] * up, v[3] * up));
        o.z = h2u(__floats2half2_rn(v[4] * up, v[5] * up));
        o.w = h2u(__floats2half2_rn(v[6] * up, v[7] * up));
        // column 8 lane + e of block b: half-slice 2b + (lane >> 4), core matrix (lane & 15), token row n & 7
        uint8_t *dst = a.Xh + (size_t)(2 * b + (lane >> 4)) * panel + (size_t)(n >> 3) * 2048 + (lane & 15) * 128 + (n & 7) * 16;
        *reinterpret_cast<uint4 *>(dst) = o;
    }
}

// ---------------------------------------------------------------------------------------------------------------
// decoders: one lane = one row of a 32-row tile, one 128-column half-slice, written as fp16 into the A stage row
// (arow = stage + row offset; chunk t = columns 4t..4t+3 lands at (t >> 1) * 128 + (t & 1) * 8).

// One-stage class 3 (W1 = 8): the lane's 8 words are loaded with the byte stream rotated by j words' worth at load
// time (word i <- stored word (i - j/4) & 7); the remaining j & 3 bytes are rotated in registers, after which byte t is
// the field of chunk t (stored at step k = (t - j) & 31).
__device__ __forceinline__ void load_c3_rotated(const uint32_t *p0, int hs, int j, uint32_t (&w)[24]) {
    const uint32_t *q = p0 + (size_t)hs * 8 * 32 + 2 * j;
    const int a = j >> 2;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int s = (i - a) & 7;
        w[i] = __ldg(q + (s >> 1) * 64 + (s & 1));
    }
}

__device__ __forceinline__ void decode_c3(const uint32_t (&w)[24], int j, const uint2 *AH, float sc, uint8_t *arow) {
    uint32_t rw[8];
    const int sh = 8 * (j & 3);
#pragma unroll
    for (int i = 0; i < 8; ++i) rw[i] = __funnelshift_l(w[(i + 7) & 7], w[i], sh);
    const uint32_t H = pingala8_h(zbits<3>(rw));
    const __half2 s2 = __float2half2_rn(sc);
#pragma unroll
    for (int p = 0; p < 16; ++p) {
        uint2 e[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int t = 2 * p + u;
            const uint32_t f = (rw[t >> 2] >> (8 * (t & 3))) & 0xFFu;
            e[u] = AH[(f << 1) | ((H >> t) & 1u)];
        }
        uint4 o;
        o.x = h2u(__hmul2(u2h(e[0].x), s2));
        o.y = h2u(__hmul2(u2h(e[0].y), s2));
        o.z = h2u(__hmul2(u2h(e[1].x), s2));
        o.w = h2u(__hmul2(u2h(e[1].y), s2));
        *reinterpret_cast<uint4 *>(arow + p * 128) = o;
    }
}

// any class: exact integers per step (chunk_ints_step), then fp16(int * sc)
template <int C>
__device__ __forceinline__ void decode_generic(const uint32_t (&w)[24], int j, const uint32_t *A_s, uint32_t cs, float sc,
                                               uint8_t *arow) {
    const uint32_t z = zbits<C>(w);
    const uint32_t H = pingala8_h(__funnelshift_l(z, z, j));
#pragma unroll
    for (int k = 0; k < 32; ++k) {
        const int t = (j + k) & 31;
        int v[4];
        chunk_ints_step<C>(w, A_s, cs, H, k, t, v);
        uint2 o;
        o.x = h2u(__floats2half2_rn(__fmul_rn((float)v[0], sc), __fmul_rn((float)v[1], sc)));
        o.y = h2u(__floats2half2_rn(__fmul_rn((float)v[2], sc), __fmul_rn((float)v[3], sc)));
        *reinterpret_cast<uint2 *>(arow + (t >> 1) * 128 + (t & 1) * 8) = o;
    }
}

__device__ __forceinline__ void load_tile_words(int c, const uint32_t *p0, int hs, int j, uint32_t (&w)[24]) {
    switch (c) {
        case 0: break;
        case 1: load_lane_words<1>(p0, hs, j, w); break;
        case 2: load_lane_words<2>(p0, hs, j, w); break;
        case 3: load_c3_rotated(p0, hs, j, w); break;
        case 4: load_lane_words<4>(p0, hs, j, w); break;
        case 5: load_lane_words<5>(p0, hs, j, w); break;
        case 6: load_lane_words<6>(p0, hs, j, w); break;
        default: load_lane_words<7>(p0, hs, j, w); break;
    }
}

__device__ __forceinline__ void decode_tile(int c, const uint32_t (&w)[24], int j, const uint2 *AH, const uint32_t *A_s,
                                            uint32_t cs, float sc, uint8_t *arow) {
    switch (c) {
        case 0:
#pragma unroll
            for (int p = 0; p < 16; ++p) *reinterpret_cast<uint4 *>(arow + p * 128) = make_uint4(0u, 0u, 0u, 0u);
            break;
        case 1: decode_generic<1>(w, j, A_s, cs, sc, arow); break;
        case 2: decode_generic<2>(w, j, A_s, cs, sc, arow); break;
        case 3: decode_c3(w, j, AH, sc, arow); break;
        case 4: decode_generic<4>(w, j, A_s, cs, sc, arow); break;
        case 5: decode_generic<5>(w, j, A_s, cs, sc, arow); break;
        case 6: decode_generic<6>(w, j, A_s, cs, sc, arow); break;
        default: decode_generic<7>(w, j, A_s, cs, sc, arow); break;
    }
}

// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm(const __grid_constant__ GemmArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nst = a.nst, bn = a.bn;
    const int stageB = bn * 256;
    uint8_t *sA = g_smem;
    uint8_t *sB = g_smem + (size_t)nst * kGemmStageA;
    uint2 *AH = reinterpret_cast<uint2 *>(sB + (size_t)nst * stageB);
    uint32_t *A_s = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(AH) + kGemmAH);
    uint64_t *full_a = reinterpret_cast<uint64_t *>(A_s + 256);
    uint64_t *full_b = full_a + kGemmMaxStages;
    uint64_t *empty = full_b + kGemmMaxStages;
    uint64_t *acc_bar = empty + kGemmMaxStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_bar + 1);
    const uint32_t tcols = bn < 32 ? 32u : (uint32_t)bn;
    const int nhs = 2 * a.nb;  // stages = half-slices

    if (threadIdx.x == 0) {
        for (int i = 0; i < nst; ++i) {
            mbar_init(full_a + i, 4);  // the four decoder warps of the stage's half-slice
            mbar_init(full_b + i, 1);
            mbar_init(empty + i, 1);   // tcgen05.commit
        }
        mbar_init(acc_bar, 1);
        fence_mbar_init();
    }
    if (warp == 9) tmem_alloc(tmem_slot, tcols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // everything below may read memory written by earlier work in the stream
    for (int i = threadIdx.x; i < 512; i += kGemmThreads) {  // (codebook + h * coset) as fp16, exact (|v| <= 256)
        const uint32_t av = a.A[i >> 1];
        const int h = i & 1;
        int v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = (int)(int8_t)(av >> (8 * e)) + (h ? (int)(int8_t)(a.cs >> (8 * e)) : 0);
        AH[i] = make_uint2(h2u(__halves2half2(__int2half_rn(v[0]), __int2half_rn(v[1]))),
                           h2u(__halves2half2(__int2half_rn(v[2]), __int2half_rn(v[3]))));
    }
    for (int i = threadIdx.x; i < 256; i += kGemmThreads) A_s[i] = a.A[i];
    __syncthreads();

    bool ok = true;
    if (warp < 8) {
        // ------------------------------------------------------------------ decoders
        const int q = warp & 3, hs = warp >> 2;
        const int R = q * 32 + lane;
        const int g = blockIdx.x * 4 + q;
        const bool tile = g < a.ng;
        const int r = g * 32 + lane;
        uint8_t *arow0 = sA + (R >> 3) * 2048 + (R & 7) * 16;
        const float up = tile ? a.rsc[r].x : 0.f;
        auto mword = [&](int b) -> uint32_t {
            if (!tile) return 0u;
            const size_t ti = (size_t)g * a.nb + b;
            if (a.ucls) return (uint32_t)(ti * 64 * NW(a.ucls)) | ((uint32_t)a.ucls << 29);
            return __ldg(a.M + ti);
        };
        uint32_t w[24], wn[24];
        uint32_t m_cur = mword(0), m_next = a.nb > 1 ? mword(1) : 0u;
        load_tile_words((int)(m_cur >> 29), a.D + (m_cur & 0x1FFFFFFFu), hs, lane, w);
        float s_cur = tile ? h2f(a.S[r]) : 0.f;
        for (int b = 0; b < a.nb; ++b) {
            // prefetch: payload and scale of block b + 1, M word of block b + 2
            float s_next = 0.f;
            uint32_t m_n2 = 0u;
            if (b + 1 < a.nb) {
                load_tile_words((int)(m_next >> 29), a.D + (m_next & 0x1FFFFFFFu), hs, lane, wn);
                if (tile) s_next = h2f(a.S[(size_t)(b + 1) * a.rows + r]);
                if (b + 2 < a.nb) m_n2 = mword(b + 2);
            }
            const int s = 2 * b + hs, slot = s % nst;
            const uint32_t ph = (uint32_t)(s / nst) & 1u;
            if (!mbar_wait_bounded(empty + slot, ph ^ 1u, kGemmPolls)) ok = false;
            decode_tile((int)(m_cur >> 29), w, lane, AH, A_s, a.cs, __fmul_rn(s_cur, up), arow0 + (size_t)slot * kGemmStageA);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(full_a + slot);
#pragma unroll
            for (int i = 0; i < 24; ++i) w[i] = wn[i];
            s_cur = s_next;
            m_cur = m_next;
            m_next = m_n2;
        }
    } else if (warp == 8) {
        // ------------------------------------------------------------------ activation tiles
        if (lane == 0) {
            const uint8_t *src = a.Xh + (size_t)blockIdx.y * stageB;
            const size_t panel = (size_t)a.npad * 256;
            for (int s = 0; s < nhs; ++s) {
                const int slot = s % nst;
                const uint32_t ph = (uint32_t)(s / nst) & 1u;
                if (!mbar_wait_bounded(empty + slot, ph ^ 1u, kGemmPolls)) ok = false;
                mbar_expect_tx(full_b + slot, (uint32_t)stageB);
                bulk_g2s(sB + (size_t)slot * stageB, src + (size_t)s * panel, (uint32_t)stageB, full_b + slot);
            }
            // drain: every copy issued has landed before the CTA may exit
            for (int s = nhs - nst < 0 ? 0 : nhs - nst; s < nhs; ++s)
                if (!mbar_wait_bounded(full_b + s % nst, (uint32_t)(s / nst) & 1u, kGemmPolls)) ok = false;
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ MMA issue
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(bn);
            for (int s = 0; s < nhs; ++s) {
                const int slot = s % nst;
                const uint32_t ph = (uint32_t)(s / nst) & 1u;
                bool st_ok = mbar_wait_bounded(full_a + slot, ph, kGemmPolls);
                st_ok = mbar_wait_bounded(full_b + slot, ph, kGemmPolls) && st_ok;
                tc_fence_after();
                if (st_ok) {
                    const uint64_t da = smem_desc(smem_u32(sA + (size_t)slot * kGemmStageA));
                    const uint64_t db = smem_desc(smem_u32(sB + (size_t)slot * stageB));
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)  // K = 16 per MMA: two core matrices (256 B) further along K
                        umma_f16(tmem, da + (uint64_t)(16 * kk), db + (uint64_t)(16 * kk), idesc, (s | kk) != 0);
                } else {
                    ok = false;
                }
                umma_commit(empty + slot);
            }
            umma_commit(acc_bar);
            if (!mbar_wait_bounded(acc_bar, 0, kGemmPolls)) ok = false;  // own MMAs done before TMEM is freed
        }
        __syncwarp();
    }

    if (warp < 8) {
        // ------------------------------------------------------------------ epilogue
        pdl_launch_dependents();
        bool acc_ok = mbar_wait_bounded(acc_bar, 0, kGemmPolls);
        acc_ok = __all_sync(0xffffffffu, acc_ok);
        tc_fence_after();
        if (!acc_ok) ok = false;
        const int q = warp & 3, half = warp >> 2;
        const int r = blockIdx.x * 128 + q * 32 + lane;
        const bool row = r < a.rows;
        const int ro = row ? a.prm[r] : 0;
        const float down = row ? a.rsc[r].y : 0.f;
        const int e0 = row ? a.cp[ro] : 0, e1 = row ? a.cp[ro + 1] : 0;
        const int n0 = blockIdx.y * bn;
        const int cw = bn >> 1;
        for (int c0 = half * cw; acc_ok && c0 < (half + 1) * cw; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
            if (row) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n = n0 + c0 + i;
                    if (n < a.ncols) {
                        float y = __fmul_rn(__fmul_rn(__uint_as_float(v[i]), down), a.tdown[n]);
                        const float *xn = a.X + (size_t)n * a.ldx;
                        for (int e = e0; e < e1; ++e) y = __fadd_rn(y, __fmul_rn(a.cv[e], xn[a.cc[e]]));
                        a.Y[(size_t)n * a.ldy + ro] = y;
                    }
                }
            }
        }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && lane == 0) atomicOr(&g_p8_device_error, 4u);
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, tcols);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// host side
struct GemmPlan {
    int bn, nst, npad, nkc, mt, nnt;
    size_t xh, pmax, tdown, total, smem;
};

static int gemm_stages(int bn) {
    const int s = kGemmOperandBudget / (kGemmStageA + bn * 256);
    return s > kGemmMaxStages ? kGemmMaxStages : s;
}
static size_t gemm_smem(int bn) {
    return (size_t)gemm_stages(bn) * (kGemmStageA + bn * 256) + kGemmAH + 1024 + 8 * (3 * kGemmMaxStages + 1) + 16;
}

static GemmPlan gemm_plan(const p8_tensor *t, int64_t ncols) {
    const int nsm = sm_count();
    GemmPlan p;
    p.mt = (t->rows + 127) / 128;
    // tile width: fewest waves, weighting a tile's time as its MMA share (BN) plus the decode it cannot hide
    int best = 256;
    long long best_cost = -1;
    for (int bn = 256; bn >= 32; bn >>= 1) {
        const long long tiles = (long long)p.mt * ((ncols + bn - 1) / bn);
        const long long waves = (tiles + nsm - 1) / nsm;
        const long long cost = waves * ((bn > 64 ? bn : 64) + 32);
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = bn; }
    }
    p.bn = best;
    p.nst = gemm_stages(best);
    p.nnt = (int)((ncols + best - 1) / best);
    p.npad = p.nnt * best;
    p.nkc = (t->K + 2047) / 2048;
    p.xh = 0;
    p.pmax = al256((size_t)t->K * p.npad * 2);
    p.tdown = p.pmax + al256((size_t)p.npad * p.nkc * 4);
    p.total = p.tdown + al256((size_t)p.npad * 4);
    p.smem = gemm_smem(best);
    return p;
}

bool gemm_supported(const p8_tensor *t, int64_t ncols) {
    return ncols >= kGemmMinCols && t->K <= 65536 && t->rsc != nullptr;
}

size_t gemm_workspace(const p8_tensor *t, int64_t ncols) { return gemm_plan(t, ncols).total; }

p8_status launch_gemm(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, float *Y, int64_t ldy, void *ws,
                      size_t ws_bytes, cudaStream_t st) {
    const GemmPlan p = gemm_plan(t, ncols);
    if (!ws || ws_bytes < p.total || ((uintptr_t)ws & 255)) return P8_ERR_WORKSPACE;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        size_t mx = 0;
        for (int bn = 32; bn <= 256; bn <<= 1) mx = gemm_smem(bn) > mx ? gemm_smem(bn) : mx;
        if (cudaFuncSetAttribute(k_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mx) != cudaSuccess) return P8_ERR_CUDA;
        attr_set[dev] = true;
    }
    uint8_t *w = static_cast<uint8_t *>(ws);
    GxArgs xa;
    xa.X = X; xa.ic = t->ic; xa.ldx = ldx; xa.K = t->K; xa.nb = t->nb; xa.ncols = (int)ncols; xa.npad = p.npad; xa.nkc = p.nkc;
    xa.Xh = w + p.xh;
    xa.pmax = reinterpret_cast<float *>(w + p.pmax);
    xa.tdown = reinterpret_cast<float *>(w + p.tdown);
    {
        void *args[] = {&xa};
        if (launch_pdl((const void *)k_gx_max, dim3(p.npad, p.nkc), dim3(256), 0, st, args) != cudaSuccess) return P8_ERR_CUDA;
        if (launch_pdl((const void *)k_gx_prep, dim3(p.npad / 8, (t->nb + 3) / 4), dim3(256), 0, st, args) != cudaSuccess)
            return P8_ERR_CUDA;
    }
    GemmArgs ga;
    ga.A = t->A; ga.M = t->M; ga.D = t->D; ga.S = t->S; ga.prm = t->prm; ga.rsc = t->rsc; ga.cp = t->cp; ga.cc = t->cc;
    ga.cv = t->cv; ga.X = X; ga.Y = Y; ga.Xh = xa.Xh; ga.tdown = xa.tdown; ga.ldx = ldx; ga.ldy = ldy; ga.cs = t->cs;
    ga.rows = t->rows; ga.nb = t->nb; ga.ng = t->ng; ga.ncols = (int)ncols; ga.npad = p.npad; ga.bn = p.bn; ga.nst = p.nst;
    ga.ucls = t->uniform_class;
    void *args[] = {&ga};
    if (launch_pdl((const void *)k_gemm, dim3(p.mt, p.nnt), dim3(kGemmThreads), p.smem, st, args) != cudaSuccess)
        return P8_ERR_CUDA;
    return P8_OK;
}

// prepare-time part: per-row weight scales. bint = max |int| over the classes the tensor uses.
p8_status gemm_prepare(p8_tensor *t, cudaStream_t st) {
    int m1 = 0;
    for (int f = 0; f < 256; ++f)
        for (int e = 0; e < 4; ++e)
            for (int h = 0; h < 2; ++h) {
                const int v = (int)(int8_t)(t->A_host[f] >> (8 * e)) + (h ? (int)(int8_t)(t->cs >> (8 * e)) : 0);
                if (v > m1) m1 = v;
                if (-v > m1) m1 = -v;
            }
    int bint = 0;
    for (int c = 1; c < 8; ++c)
        if ((t->class_mask >> c) & 1u) bint = bint > m1 * MC(c) ? bint : m1 * MC(c);
    if (cudaMalloc((void **)&t->rsc, sizeof(float2) * (size_t)t->rows) != cudaSuccess) {
        t->rsc = nullptr;
        return P8_ERR_CUDA;
    }
    k_row_scale<<<(t->rows + 255) / 256, 256, 0, st>>>(t->S, t->rows, t->nb, (float)bint, t->rsc);
    if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) return P8_ERR_CUDA;
    return P8_OK;
}
