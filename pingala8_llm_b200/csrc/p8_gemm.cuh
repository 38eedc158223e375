// p8_gemm.cuh -- batched (prefill) Pingala-8 matmul on the 5th-generation tensor cores: tcgen05 MMA with the weight
// operand and the accumulator in tensor memory (TMEM), the activation operand in shared memory. Included by
// p8_kernels.cu, so it shares that file's device error word and launch helpers.
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
//   k_gx_prep  grid (Npad/8, nb), 256 thr, warp = token: tau from the partial maxima; Xr as fp16 in the
//              operand layout below ([half-slice][token group of 8][16 core matrices][8 tokens][8 columns]), so the
//              GEMM moves one B stage with one bulk copy.
//   k_gemm     grid (rows/128 rounded up, Npad/BN), 352 thr, 1 CTA per SM. One stage = one 128-column half-slice.
//              warp 8     stages the packed payload: per stage, one bulk copy per row tile (NW words x 32 lanes of its
//                         half-slice) into a ring of up to 8 shared-memory slots, several stages ahead of the decoders;
//              warps 0-7  decoders: warp (q, hs) decodes half-slice hs of row tile q (32 rows) of every 256-column
//                         block from the staged words into a TMEM A slot (4 slots, 64 columns each) as fp16
//                         int * S * 2^sigma with tcgen05.st (lane = row); then the epilogue (TMEM -> registers,
//                         scales, clamp delta, y[n][prm[r]]);
//              warp 10    bulk-copies each B stage (BN tokens x 128 columns) into a shared-memory ring;
//              warp 9     allocates TMEM; one lane issues 8 MMAs (M = 128, N = BN, K = 16, A from TMEM) per stage and
//                         commits them to the stage's A-slot and B-slot 'empty' barriers, after the last stage to the
//                         accumulator barrier.
//   k_splitk_reduce  (split-K only) one thread per output: the splits' raw partials summed in split order, scaled,
//                    clamp delta, y[n][prm[r]].
//   k_unpermute      (single split, >= 64 tokens) the epilogue stores finished outputs in sorted-row order with 16-byte
//                    stores; this kernel writes Y[n][ro] from row pinv[ro] with coalesced stores (Y's rows are the
//                    permuted ones, so direct stores would scatter one 4-byte store per output).
// The loader and MMA warps run their loops as whole warps (every lane polls, one or four lanes issue): a single active
// lane with 31 parked at a warp barrier was starved behind the decoders' shared-memory traffic.
// Keeping A in TMEM leaves shared-memory bandwidth to the B tile (written once by the copy, read once by the MMA). The
// codebook lookup table is a lane-private copy (entry f of lane l at word 32 f + l), so a warp's lookups never share a
// bank. B operand layout (UMMA K-major, no swizzle): a core matrix is 8 rows x 8 fp16, 16 B per row, 128 B contiguous;
//     byte(row, col) = (row >> 3) * 2048 + (col >> 3) * 128 + (row & 7) * 16 + (col & 7) * 2
// so descriptor LBO (next core matrix along K) = 128 B and SBO (next group of 8 rows) = 2048 B.
//
// Every mbarrier wait is bounded; a wait that gives up sets bit 2 (value 4) of the device error word, the kernel
// drains its own copies and MMAs, frees its TMEM and returns (results of that launch are invalid).

constexpr int kGemmThreads = 352;                   // 8 decoder warps, payload loader, MMA, activation loader
constexpr int kGemmCbk = 256 * 32 * 4;              // lane-private codebook copy (32 KB)
constexpr int kGemmASlots = 4;                      // A operand stages in TMEM, 64 columns each
constexpr int kGemmAColBase = 256;                  // TMEM columns [0, 256): accumulator; [256, 512): A stages
constexpr uint32_t kGemmTmemCols = 512;
constexpr int kGemmMaxB = 4, kGemmMaxP = 8;         // activation / payload ring depths
constexpr int kGemmSmemMax = 227 * 1024;            // shared memory per CTA (sm_100 opt-in maximum)
constexpr int kGemmSmemDyn = kGemmSmemMax - 1024;   // dynamic part (the kernel's static shared memory takes 1 KB)
constexpr uint32_t kGemmPolls = 1u << 22;
constexpr int kGemmMinCols = 4;                     // below this the per-column table GEMV is faster (measured crossover)
constexpr int kGemmMinColsC3 = 6;                   // uniform class-3 tensors: below this the two-column table GEMV (pairs)
                                                    // is faster (Llama-3.1-8B decode chain: bs 4 3.4 vs 5.1 ms, bs 5 4.7 vs
                                                    // 5.1, bs 6 5.1 vs 5.1, bs 7 6.4 vs 5.2 ms per step)
constexpr int kGemmStagedMinCols = 64;              // from here (single split) outputs go out in sorted-row order first

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
    int rows, nb, ng, ncols, npad, bn, nbs, np, tileb, ucls;
    int xpad;              // token count of Xh's panels (the prep's padding: >= npad when a group shares the prep)
    int rs;                // sorted rows >= rs come from split-K partials: k_splitk_reduce covers [rs, rows),
                           // k_unpermute [0, rs); partial rows are indexed from rs
    int ksplit, mtr;       // split-K: CTAs per output tile along K; rows of the partials
    float *kpart;          // split-K partial accumulators [ksplit][npad][mtr] (raw fp32)
    float *Yt;             // (single split, many tokens) outputs in sorted-row order [mtr][npad], un-permuted after
    const int16_t *pinv;   // original row -> sorted row
};

// 256-column blocks per k_gx_prep CTA: one, so that a token's blocks are converted in parallel (each warp's load ->
// FWHT -> store chain is latency-bound; with several blocks per warp they ran one after another)
constexpr int kGxBlocksPerCta = 1;

struct GxArgs {
    const float *X;
    const float *ic;
    float *pmax;           // [npad][nkc]
    uint8_t *Xh;
    float *tdown;
    long long ldx;
    int K, nb, ncols, npad, nkc;
    // activation prologue (k_gx_*<PRO>, PRO != P8_PROLOGUE_NONE): x' per token from x and w (RMSNorm weight [K]) or
    // x2 (SwiGLU up, [ncols][ldx]); ss [npad][nkc] partial sums of squares; x' f32 to xv [npad][K] for the delta term
    const float *pw, *x2;
    float eps;
    float *ss, *xv;
};

// the prologue's x' of one element (x = the input, w / u = the weight or up value, scale = the token's RMSNorm scale),
// the same formulas as the batch-1 prep: (x * scale) * w, or x / (1 + exp(-x)) * u
template <int PRO>
__device__ __forceinline__ float pro_val(float x, float wu, float scale) {
    if (PRO == P8_PROLOGUE_RMSNORM) return __fmul_rn(__fmul_rn(x, scale), wu);
    if (PRO == P8_PROLOGUE_SWIGLU) return __fmul_rn(__fdiv_rn(x, __fadd_rn(1.f, expf(-x))), wu);
    return x;
}

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
template <int PRO>
__global__ void __launch_bounds__(256) k_gx_max(const GxArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float red[8];
    __shared__ float red2[8];
    const int n = blockIdx.x, col = blockIdx.y * 2048 + threadIdx.x * 8;
    float m = 0.f, sq = 0.f;
    if (n < a.ncols && col < a.K) {
        const float4 *xp = reinterpret_cast<const float4 *>(a.X + (size_t)n * a.ldx + col);
        const float4 *ip = reinterpret_cast<const float4 *>(a.ic + col);
        float4 x0 = xp[0], x1 = xp[1];
        const float4 i0 = ip[0], i1 = ip[1];
        if (PRO == P8_PROLOGUE_RMSNORM) {  // sum of squares of x; the bound uses x * w (the scale is a positive scalar)
            const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) sq = __fmaf_rn(xs[e], xs[e], sq);
            const float4 w0 = *reinterpret_cast<const float4 *>(a.pw + col), w1 = *reinterpret_cast<const float4 *>(a.pw + col + 4);
            x0 = make_float4(x0.x * w0.x, x0.y * w0.y, x0.z * w0.z, x0.w * w0.w);
            x1 = make_float4(x1.x * w1.x, x1.y * w1.y, x1.z * w1.z, x1.w * w1.w);
        } else if (PRO == P8_PROLOGUE_SWIGLU) {
            const float4 *up = reinterpret_cast<const float4 *>(a.x2 + (size_t)n * a.ldx + col);
            const float4 u0 = up[0], u1 = up[1];
            x0 = make_float4(pro_val<PRO>(x0.x, u0.x, 1.f), pro_val<PRO>(x0.y, u0.y, 1.f), pro_val<PRO>(x0.z, u0.z, 1.f),
                             pro_val<PRO>(x0.w, u0.w, 1.f));
            x1 = make_float4(pro_val<PRO>(x1.x, u1.x, 1.f), pro_val<PRO>(x1.y, u1.y, 1.f), pro_val<PRO>(x1.z, u1.z, 1.f),
                             pro_val<PRO>(x1.w, u1.w, 1.f));
        }
        m = fmaxf(fmaxf(fmaxf(fabsf(x0.x * i0.x), fabsf(x0.y * i0.y)), fmaxf(fabsf(x0.z * i0.z), fabsf(x0.w * i0.w))),
                  fmaxf(fmaxf(fabsf(x1.x * i1.x), fabsf(x1.y * i1.y)), fmaxf(fabsf(x1.z * i1.z), fabsf(x1.w * i1.w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    if (PRO == P8_PROLOGUE_RMSNORM) {  // fixed-order tree: the same partial sums on every call
#pragma unroll
        for (int o = 16; o; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
        if ((threadIdx.x & 31) == 0) red2[threadIdx.x >> 5] = sq;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = red[0];
        for (int i = 1; i < 8; ++i) v = fmaxf(v, red[i]);
        a.pmax[(size_t)n * a.nkc + blockIdx.y] = v;
        if (PRO == P8_PROLOGUE_RMSNORM) {
            float t = red2[0];
            for (int i = 1; i < 8; ++i) t = __fadd_rn(t, red2[i]);
            a.ss[(size_t)n * a.nkc + blockIdx.y] = t;
        }
    }
}

template <int PRO>
__global__ void __launch_bounds__(256) k_gx_prep(const GxArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + warp;
    float m = lane < a.nkc ? a.pmax[(size_t)n * a.nkc + lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float scale = 1.f;
    if (PRO == P8_PROLOGUE_RMSNORM) {  // 1 / sqrt(sum(x^2) / K + eps), chunk sums added in chunk order
        float t = 0.f;
        for (int y = 0; y < a.nkc; ++y) t = __fadd_rn(t, a.ss[(size_t)n * a.nkc + y]);
        scale = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)a.K), a.eps)));
        m = m * scale;  // the bound of |x' * sgn/c| (the 2 spare bits of the fp16 range absorb its rounding)
    }
    // |Xr| <= 16 max|x * sgn/c| < 16 * 2^e  ->  tau = 10 - e gives |Xr * 2^tau| < 2^14
    int tau = 0;
    if (m > 0.f && m <= 3.0e38f) tau = min(126, max(-126, 10 - exp_above(m)));
    const float up = pow2f(tau);
    if (blockIdx.y == 0 && lane == 0) a.tdown[n] = pow2f(-tau);
    const size_t panel = (size_t)a.npad * 256;
    for (int i = 0; i < kGxBlocksPerCta; ++i) {
        const int b = blockIdx.y * kGxBlocksPerCta + i;
        if (b >= a.nb) break;
        float v[8];
        if (n < a.ncols) {
            const float4 *xp = reinterpret_cast<const float4 *>(a.X + (size_t)n * a.ldx + b * 256 + 8 * lane);
            const float4 *ip = reinterpret_cast<const float4 *>(a.ic + b * 256 + 8 * lane);
            float4 x0 = xp[0], x1 = xp[1];
            const float4 i0 = ip[0], i1 = ip[1];
            if (PRO != P8_PROLOGUE_NONE) {
                const float *wu = PRO == P8_PROLOGUE_RMSNORM ? a.pw + b * 256 + 8 * lane : a.x2 + (size_t)n * a.ldx + b * 256 + 8 * lane;
                const float4 u0 = *reinterpret_cast<const float4 *>(wu), u1 = *reinterpret_cast<const float4 *>(wu + 4);
                x0 = make_float4(pro_val<PRO>(x0.x, u0.x, scale), pro_val<PRO>(x0.y, u0.y, scale), pro_val<PRO>(x0.z, u0.z, scale),
                                 pro_val<PRO>(x0.w, u0.w, scale));
                x1 = make_float4(pro_val<PRO>(x1.x, u1.x, scale), pro_val<PRO>(x1.y, u1.y, scale), pro_val<PRO>(x1.z, u1.z, scale),
                                 pro_val<PRO>(x1.w, u1.w, scale));
                float4 *xo = reinterpret_cast<float4 *>(a.xv + (size_t)n * a.K + b * 256 + 8 * lane);  // x' for the delta term
                xo[0] = x0;
                xo[1] = x1;
            }
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
// decoders: one lane = one row of a 32-row tile, one 128-column half-slice, written as fp16 into the TMEM A slot of
// the stage (row = TMEM lane, column c of the slot holds columns 2c, 2c + 1 of the half-slice as a half2).
//
// Chunk order: the payload stores chunk t of lane j at step k = (t - j) & 31, i.e. every field stream of the lane is
// rotated by j fields. Reading the lane's words from shared memory with the word rotation applied at load time and
// the bit rotation by a funnel shift puts chunk t's fields at static bit positions t * width, so each class decodes
// straight into registers in chunk order, eight chunks (16 columns) per tcgen05.st.

// lane words of one half-slice in the staging slot: word i of lane j at pw[(i >> 1) * 64 + 2 j + (i & 1)]
__device__ __forceinline__ uint32_t slot_word(const uint32_t *pw, int lane, int i) { return pw[(i >> 1) * 64 + 2 * lane + (i & 1)]; }

// the W-word stream at words [wbase, wbase + W) rotated left by rbits (< 32 W) bits: out bit p = stream bit p - rbits
template <int W>
__device__ __forceinline__ void rot_stream(const uint32_t *pw, int wbase, int lane, int rbits, uint32_t (&out)[W]) {
    const int qw = rbits >> 5, o = rbits & 31;
    uint32_t r[W];
#pragma unroll
    for (int i = 0; i < W; ++i) {
        int s = i - qw;
        if (s < 0) s += W;
        r[i] = slot_word(pw, lane, wbase + s);
    }
#pragma unroll
    for (int i = 0; i < W; ++i) out[i] = __funnelshift_l(r[(i + W - 1) % W], r[i], o);
}

// width-bit field at static bit position pos of a word array
template <int N>
__device__ __forceinline__ uint32_t sfield(const uint32_t (&w)[N], int pos, int width) {
    const int wi = pos >> 5, bb = pos & 31;
    uint32_t v = w[wi] >> bb;
    if (bb + width > 32) v |= w[wi + 1] << (32 - bb);
    return v & ((1u << width) - 1u);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16};\n" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]^T, B K-major; accumulate = 0 overwrites D
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

constexpr uint32_t kHalf2M1152 = 0xE480E480u;  // half2(-1152, -1152)

// Class 3 (one 8-bit stage). The codebook copy holds A[f] ^ 0x80808080 (bytes a + 128). PRMT places two bytes u under
// the fp16 exponent pattern 0x64 (giving 1024 + u exactly); adding -1152 (h = 0) or c_e - 1152 (h = 1) gives the exact
// integer a + h c, and one multiply by the row scale rounds it to fp16 once.
__device__ __forceinline__ void decode_c3_tmem(const uint32_t *pw, int lane, const uint32_t *cl, float sc, uint32_t dlo,
                                               uint32_t dhi, uint32_t tA) {
    uint32_t rw[8];
    rot_stream<8>(pw, 0, lane, 8 * lane, rw);
    const uint32_t H = pingala8_h(zbits<3>(rw));
    const __half2 s2 = __float2half2_rn(sc);
#pragma unroll
    for (int gq = 0; gq < 4; ++gq) {
        uint32_t o[16];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int t = 8 * gq + u;
            const uint32_t f = (rw[t >> 2] >> (8 * (t & 3))) & 0xFFu;
            const uint32_t v = cl[f * 32];
            const uint32_t hm = (uint32_t)((int32_t)(H << (31 - t)) >> 31);
            const uint32_t lo = __byte_perm(v, 0x64646464u, 0x5140), hi = __byte_perm(v, 0x64646464u, 0x7362);
            o[2 * u] = h2u(__hmul2(__hadd2(u2h(lo), u2h((hm & dlo) ^ kHalf2M1152)), s2));
            o[2 * u + 1] = h2u(__hmul2(__hadd2(u2h(hi), u2h((hm & dhi) ^ kHalf2M1152)), s2));
        }
        tmem_st16(tA + 16 * gq, o);
    }
}

// any class: exact integers sum_s (A[f_s] + h c) << SH_s per element, then fp16(int * sc)
template <int C>
__device__ __forceinline__ void decode_gen_tmem(const uint32_t *pw, int lane, const uint32_t *cl, uint32_t cs, float sc,
                                                uint32_t tA) {
    constexpr int w1 = W1(C), w2 = W2(C), w3 = W3(C);
    constexpr int n1 = w1 == 8 ? 8 : w1 - 1;
    uint32_t s1[n1], s2[w2 > 0 ? w2 : 1], s3[8], z;
    if constexpr (w1 == 8) {
        rot_stream<8>(pw, 0, lane, 8 * lane, s1);
        z = zbits<3>(s1);
    } else {
        uint32_t m0[1];
        rot_stream<1>(pw, 0, lane, lane, m0);  // stage-1 MSB word: bit k = z of step k
        z = m0[0];
        rot_stream<n1>(pw, 1, lane, n1 * lane, s1);
    }
    if constexpr (w2 > 0) rot_stream<(w2 > 0 ? w2 : 1)>(pw, w1, lane, w2 * lane, s2);
    if constexpr (w3 > 0) rot_stream<8>(pw, w1 + w2, lane, 8 * lane, s3);
    const uint32_t H = pingala8_h(z);
#pragma unroll
    for (int gq = 0; gq < 4; ++gq) {
        uint32_t o[16];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int t = 8 * gq + u;
            uint32_t f1;
            if constexpr (w1 == 8) f1 = (s1[t >> 2] >> (8 * (t & 3))) & 0xFFu;
            else f1 = sfield(s1, (w1 - 1) * t, w1 - 1) | (((z >> t) & 1u) << (w1 - 1));
            const uint32_t a1 = cl[f1 * 32] ^ 0x80808080u;
            uint32_t a2 = 0, a3 = 0;
            if constexpr (w2 > 0) a2 = cl[sfield(s2, w2 * t, w2) * 32] ^ 0x80808080u;
            if constexpr (w3 > 0) a3 = cl[((s3[t >> 2] >> (8 * (t & 3))) & 0xFFu) * 32] ^ 0x80808080u;
            const int h = (H >> t) & 1u;
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int ce = h ? (int)(int8_t)(cs >> (8 * e)) : 0;
                int x = ((int)(int8_t)(a1 >> (8 * e)) + ce) * (1 << SH1(C));
                if (w2 > 0) x += ((int)(int8_t)(a2 >> (8 * e)) + ce) * (1 << SH2(C));
                if (w3 > 0) x += (int)(int8_t)(a3 >> (8 * e)) + ce;
                v[e] = __fmul_rn((float)x, sc);
            }
            o[2 * u] = h2u(__floats2half2_rn(v[0], v[1]));
            o[2 * u + 1] = h2u(__floats2half2_rn(v[2], v[3]));
        }
        tmem_st16(tA + 16 * gq, o);
    }
}

__device__ __forceinline__ void decode_tile_tmem(int c, const uint32_t *pw, int lane, const uint32_t *cl, uint32_t cs, float sc,
                                                 uint32_t dlo, uint32_t dhi, uint32_t tA) {
    switch (c) {
        case 0: {
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = 0u;
#pragma unroll
            for (int gq = 0; gq < 4; ++gq) tmem_st16(tA + 16 * gq, o);
            break;
        }
        case 1: decode_gen_tmem<1>(pw, lane, cl, cs, sc, tA); break;
        case 2: decode_gen_tmem<2>(pw, lane, cl, cs, sc, tA); break;
        case 3: decode_c3_tmem(pw, lane, cl, sc, dlo, dhi, tA); break;
        case 4: decode_gen_tmem<4>(pw, lane, cl, cs, sc, tA); break;
        case 5: decode_gen_tmem<5>(pw, lane, cl, cs, sc, tA); break;
        case 6: decode_gen_tmem<6>(pw, lane, cl, cs, sc, tA); break;
        default: decode_gen_tmem<7>(pw, lane, cl, cs, sc, tA); break;
    }
}

// ---------------------------------------------------------------------------------------------------------------
// shared-memory layout of k_gemm (bytes from the dynamic base), shared by host and device
struct GemmSmem {
    int cbk, B, P, Mw, bars, tslot, total;
};
__host__ __device__ inline GemmSmem gemm_smem_layout(int bn, int nbs, int np, int tileb, int nb) {
    GemmSmem L;
    L.cbk = 0;
    L.B = kGemmCbk;
    L.P = L.B + nbs * bn * 256;
    L.Mw = L.P + np * 4 * tileb;
    L.bars = L.Mw + 16 * nb;  // 4 tiles x nb words
    L.tslot = L.bars + 8 * (2 * kGemmMaxP + 2 * kGemmMaxB + 2 * kGemmASlots + 1);
    L.total = L.tslot + 16;
    return L;
}

// One k_gemm launch covers row tiles of one tensor, or of two tensors of one shape and plan that read the same
// operand (the second's row tiles follow the first's, so both fill the same waves): global row tile gt =
// blockIdx.x + mt0, tensor 1 from gt >= mtA. A launch can start past row tile 0 (the split-K tail of a tail split).
template <int NT>
struct GemmLaunch {
    GemmArgs t[NT];
    int mt0, mtA;
};

// the CTA's work on row tile mtile of one tensor; inlined once per tensor of the launch, so that every field of
// the tensor's arguments is read at a fixed parameter offset
__device__ __forceinline__ void gemm_cta(const GemmArgs &a, const int mtile) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bn = a.bn, nbs = a.nbs, np = a.np;
    const int stageB = bn * 256, stageP = 4 * a.tileb;
    const GemmSmem L = gemm_smem_layout(bn, nbs, np, a.tileb, a.nb);
    uint32_t *cbk = reinterpret_cast<uint32_t *>(g_smem + L.cbk);
    uint8_t *sB = g_smem + L.B;
    uint8_t *sP = g_smem + L.P;
    uint32_t *sM = reinterpret_cast<uint32_t *>(g_smem + L.Mw);
    uint64_t *p_full = reinterpret_cast<uint64_t *>(g_smem + L.bars);
    uint64_t *p_empty = p_full + kGemmMaxP, *b_full = p_empty + kGemmMaxP, *b_empty = b_full + kGemmMaxB;
    uint64_t *a_full = b_empty + kGemmMaxB, *a_empty = a_full + kGemmASlots, *acc_bar = a_empty + kGemmASlots;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(g_smem + L.tslot);
    // split-K: this CTA's 256-column blocks [b0, b1); local stage ls = 2 (b - b0) + hs indexes every ring
    const int b0 = a.nb * (int)blockIdx.z / a.ksplit, b1 = a.nb * ((int)blockIdx.z + 1) / a.ksplit;
    const int nls = 2 * (b1 - b0);

    if (threadIdx.x == 0) {
        for (int i = 0; i < np; ++i) {
            mbar_init(p_full + i, 4);   // one arrival (with its byte count) per row tile, then the bytes
            mbar_init(p_empty + i, 4);  // the four decoder warps of the stage have read the slot
        }
        for (int i = 0; i < nbs; ++i) {
            mbar_init(b_full + i, 1);
            mbar_init(b_empty + i, 1);  // tcgen05.commit
        }
        for (int i = 0; i < kGemmASlots; ++i) {
            mbar_init(a_full + i, 4);
            mbar_init(a_empty + i, 1);
        }
        mbar_init(acc_bar, 1);
        fence_mbar_init();
    }
    if (warp == 9) tmem_alloc(tmem_slot, kGemmTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // The codebook, M words, payload and row scales belong to the tensor (no kernel of the stream writes them), so the
    // set-up, the payload ring and the decoders run before the wait for the preceding kernels; the two roles that read
    // what those kernels write wait first: the activation-tile loader (prepared operand) and the epilogue (x, the
    // per-token scales, the outputs).
    // lane-private codebook (entry f of lane l at word 32 f + l: a warp's lookups never share a bank), bytes + 128;
    // written as 16-byte groups (group i = words 4i..4i+3, all of entry i / 8): one load and one store per group
    for (int i = threadIdx.x; i < 256 * 8; i += kGemmThreads) {
        const uint32_t v = __ldg(a.A + (i >> 3)) ^ 0x80808080u;
        reinterpret_cast<uint4 *>(cbk)[i] = make_uint4(v, v, v, v);
    }
    // M words of the CTA's four row tiles (arithmetic for uniform single-class layouts)
    for (int i = threadIdx.x; i < 4 * a.nb; i += kGemmThreads) {
        const int q = i / a.nb, b = i - q * a.nb, g = mtile * 4 + q;
        uint32_t m = 0u;
        if (g < a.ng) {
            const size_t ti = (size_t)g * a.nb + b;
            m = a.ucls ? ((uint32_t)(ti * 64 * NW(a.ucls)) | ((uint32_t)a.ucls << 29)) : __ldg(a.M + ti);
        }
        sM[i] = m;
    }
    __syncthreads();

    bool ok = true;
    if (warp < 8) {
        // ------------------------------------------------------------------ decoders
        const int q = warp & 3, hs = warp >> 2;
        const int g = mtile * 4 + q;
        const bool tile = g < a.ng;
        const int r = g * 32 + lane;
        const float up = tile ? a.rsc[r].x : 0.f;
        const int c0 = (int)(int8_t)a.cs, c1 = (int)(int8_t)(a.cs >> 8), c2 = (int)(int8_t)(a.cs >> 16), c3 = (int)(int8_t)(a.cs >> 24);
        const uint32_t dlo = h2u(__floats2half2_rn((float)(c0 - 1152), (float)(c1 - 1152))) ^ kHalf2M1152;
        const uint32_t dhi = h2u(__floats2half2_rn((float)(c2 - 1152), (float)(c3 - 1152))) ^ kHalf2M1152;
        const uint32_t *cl = cbk + lane;
        const uint32_t tA0 = tmem + ((uint32_t)(q * 32) << 16) + kGemmAColBase;
        float s_next = tile ? h2f(a.S[(size_t)b0 * a.rows + r]) : 0.f;
        for (int b = b0; b < b1 && ok; ++b) {
            const int s = 2 * (b - b0) + hs;
            const float s_cur = s_next;
            if (tile && b + 1 < b1) s_next = h2f(a.S[(size_t)(b + 1) * a.rows + r]);
            const int ps = s % np, as = s & (kGemmASlots - 1);
            bool w = mbar_wait_bounded(p_full + ps, (uint32_t)(s / np) & 1u, kGemmPolls);
            w = mbar_wait_bounded(a_empty + as, ((uint32_t)(s / kGemmASlots) & 1u) ^ 1u, kGemmPolls) && w;
            if (!__all_sync(0xffffffffu, w)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t m = sM[q * a.nb + b];
            const uint32_t *pw = reinterpret_cast<const uint32_t *>(sP + (size_t)ps * stageP + q * a.tileb);
            decode_tile_tmem((int)(m >> 29), pw, lane, cl, a.cs, __fmul_rn(s_cur, up), dlo, dhi, tA0 + 64 * as);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(p_empty + ps);
                mbar_arrive(a_full + as);
            }
        }
    } else if (warp == 8) {
        // ------------------------------------------------------------------ payload staging (bulk copies, deep ring)
        // The whole warp runs the loop (no lane parked on a divergent path behind the decoders' shared-memory traffic):
        // every lane polls the barrier; lanes 0-3 each own one row tile: each arrives on the stage's barrier with its
        // own byte count (count 4) and issues its copy, with no cross-lane step. The M word of the next stage is read
        // one iteration ahead.
        int last = -1;
        uint32_t m = lane < 4 ? sM[lane * a.nb + b0] : 0u;
        for (int s = 0; s < nls; ++s) {
            const int b = b0 + (s >> 1), hs = s & 1, ps = s % np;
            const bool w = mbar_wait_bounded(p_empty + ps, ((uint32_t)(s / np) & 1u) ^ 1u, kGemmPolls);
            if (!__all_sync(0xffffffffu, w)) {
                ok = false;
                break;
            }
            const int nw = NW((int)(m >> 29));
            if (lane < 4) {
                if (nw) {
                    mbar_expect_tx(p_full + ps, (uint32_t)nw * 128u);
                    bulk_g2s(sP + (size_t)ps * stageP + lane * a.tileb, a.D + (m & 0x1FFFFFFFu) + (size_t)hs * nw * 32,
                             (uint32_t)nw * 128u, p_full + ps);
                } else {
                    mbar_arrive(p_full + ps);
                }
            }
            if (hs && lane < 4 && b + 1 < b1) m = sM[lane * a.nb + b + 1];
            last = s;
        }
        for (int s = last - np + 1 < 0 ? 0 : last - np + 1; s <= last; ++s)  // drain: every copy has landed
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(p_full + s % np, (uint32_t)(s / np) & 1u, kGemmPolls))) ok = false;
    } else if (warp == 10) {
        // ------------------------------------------------------------------ activation tiles (whole warp, lane 0 copies)
        pdl_wait();  // the operand comes from the preceding prep kernel
        const uint8_t *src = a.Xh + (size_t)blockIdx.y * stageB;
        const size_t panel = (size_t)a.xpad * 256;
        int last = -1;
        for (int s = 0; s < nls; ++s) {
            const int bs = s % nbs;
            const bool w = mbar_wait_bounded(b_empty + bs, ((uint32_t)(s / nbs) & 1u) ^ 1u, kGemmPolls);
            if (!__all_sync(0xffffffffu, w)) {
                ok = false;
                break;
            }
            if (lane == 0) {
                mbar_expect_tx(b_full + bs, (uint32_t)stageB);
                bulk_g2s(sB + (size_t)bs * stageB, src + (size_t)(2 * b0 + s) * panel, (uint32_t)stageB, b_full + bs);
            }
            __syncwarp();
            last = s;
        }
        for (int s = last - nbs + 1 < 0 ? 0 : last - nbs + 1; s <= last; ++s)
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(b_full + s % nbs, (uint32_t)(s / nbs) & 1u, kGemmPolls))) ok = false;
    } else {
        // ------------------------------------------------------------------ MMA issue (warp 9; lane 0 issues)
        const uint32_t idesc = umma_idesc_f16(bn);
        for (int s = 0; s < nls; ++s) {
            const int as = s & (kGemmASlots - 1), bs = s % nbs;
            bool st = mbar_wait_bounded(a_full + as, (uint32_t)(s / kGemmASlots) & 1u, kGemmPolls);
            st = mbar_wait_bounded(b_full + bs, (uint32_t)(s / nbs) & 1u, kGemmPolls) && st;
            tc_fence_after();
            if (!__all_sync(0xffffffffu, st)) {
                ok = false;
                break;
            }
            if (lane == 0) {
                const uint64_t db = smem_desc(smem_u32(sB + (size_t)bs * stageB));
                const uint32_t ta = tmem + kGemmAColBase + 64 * as;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)  // K = 16 per MMA: 8 TMEM columns of A, two core matrices (256 B) of B
                    umma_f16_ts(tmem, ta + 8 * kk, db + (uint64_t)(16 * kk), idesc, (s | kk) != 0);
                umma_commit(a_empty + as);
                umma_commit(b_empty + bs);
            }
            __syncwarp();
        }
        if (lane == 0) umma_commit(acc_bar);
        __syncwarp();
        // own MMAs done before TMEM is freed
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(acc_bar, 0, kGemmPolls))) ok = false;
    }

    if (warp < 8) {
        // ------------------------------------------------------------------ epilogue
        pdl_wait();  // x and the token scales come from earlier kernels; outputs and partials are shared too
        pdl_launch_dependents();
        bool acc_ok = ok && mbar_wait_bounded(acc_bar, 0, kGemmPolls);
        acc_ok = __all_sync(0xffffffffu, acc_ok);
        tc_fence_after();
        if (!acc_ok) ok = false;
        const int q = warp & 3, half = warp >> 2;
        const int r = mtile * 128 + q * 32 + lane;
        const bool row = r < a.rows;
        const int ro = row ? a.prm[r] : 0;
        const float down = row ? a.rsc[r].y : 0.f;
        const int e0 = row ? a.cp[ro] : 0, e1 = row ? a.cp[ro + 1] : 0;
        const int n0 = blockIdx.y * bn;
        const int cw = bn >> 1;
        if (a.ksplit > 1) {  // raw accumulators of this K range -> partials (k_splitk_reduce finishes them)
            const int rp = r - a.rs;
            for (int cc0 = half * cw; acc_ok && cc0 < (half + 1) * cw; cc0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)cc0, v);
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    a.kpart[((size_t)blockIdx.z * a.npad + n0 + cc0 + i) * a.mtr + rp] = __uint_as_float(v[i]);
            }
        }
        for (int cc0 = half * cw; acc_ok && a.ksplit == 1 && a.Yt && cc0 < (half + 1) * cw; cc0 += 16) {
            // sorted-row order: the lane's 16 tokens as four 16-byte stores (the permuted rows of Y would take one
            // scattered 4-byte store per output); k_unpermute writes Y from here with coalesced stores
            uint32_t v[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)cc0, v);
            if (row) {
                float yv[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n = n0 + cc0 + i;
                    float y = 0.f;
                    if (n < a.ncols) {
                        y = __fmul_rn(__fmul_rn(__uint_as_float(v[i]), down), a.tdown[n]);
                        const float *xn = a.X + (size_t)n * a.ldx;
                        for (int e = e0; e < e1; ++e) y = __fadd_rn(y, __fmul_rn(a.cv[e], xn[a.cc[e]]));
                    }
                    yv[i] = y;
                }
                float4 *o = reinterpret_cast<float4 *>(a.Yt + (size_t)r * a.npad + n0 + cc0);
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i] = make_float4(yv[4 * i], yv[4 * i + 1], yv[4 * i + 2], yv[4 * i + 3]);
            }
        }
        for (int cc0 = half * cw; acc_ok && a.ksplit == 1 && !a.Yt && cc0 < (half + 1) * cw; cc0 += 16) {
            uint32_t v[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)cc0, v);
            if (row) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n = n0 + cc0 + i;
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
        tmem_dealloc(tmem, kGemmTmemCols);
    }
}

template <int NT>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm(const __grid_constant__ GemmLaunch<NT> gl) {
    const int gt = (int)blockIdx.x + gl.mt0;  // uniform per CTA
    if (NT > 1 && gt >= gl.mtA)
        gemm_cta(gl.t[NT - 1], gt - gl.mtA);
    else
        gemm_cta(gl.t[0], gt);
}

// Outputs staged in sorted-row order (Yt) to Y: thread = (original row ro, 8 tokens); reads the 8 tokens of sorted row
// pinv[ro] (32 contiguous bytes), writes Y[n][ro] (a warp's 32 consecutive rows: one coalesced store per token).
__global__ void __launch_bounds__(256) k_unpermute(const __grid_constant__ GemmArgs a) {
    pdl_wait();  // Yt comes from k_gemm
    pdl_launch_dependents();
    const int ro = blockIdx.x * 256 + threadIdx.x, n8 = blockIdx.y * 8;
    if (ro >= a.rows) return;
    const int r = a.pinv[ro];
    if (r >= a.rs) return;  // a row of the split-K tail
    const float4 *src = reinterpret_cast<const float4 *>(a.Yt + (size_t)r * a.npad + n8);
    const float4 u0 = __ldcg(src), u1 = __ldcg(src + 1);
    const float v[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (n8 + i < a.ncols) a.Y[(size_t)(n8 + i) * a.ldy + ro] = v[i];
}

// Split-K reduction (ksplit > 1), the kernel after k_gemm: one thread per output (token n, sorted row r), r fastest
// (coalesced partial reads). y[n][prm[r]] = (sum over splits z in order of the raw partials) * 2^-sigma_r * 2^-tau_n
// + the row's clamp delta -- the same operations in the same order as the single-split epilogue. A kernel of its own
// instead of the last CTA of each tile: no fence / counter chain at the tail of the GEMM, and every SM takes part.
__global__ void __launch_bounds__(256) k_splitk_reduce(const __grid_constant__ GemmArgs a) {
    pdl_wait();  // the partials come from k_gemm
    pdl_launch_dependents();
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    const int nr = a.rows - a.rs;
    if (i >= (long long)nr * a.ncols) return;
    const int n = (int)(i / nr), rr = (int)(i - (long long)n * nr), r = a.rs + rr;
    float acc = 0.f;
    for (int z = 0; z < a.ksplit; ++z) acc = __fadd_rn(acc, __ldcg(a.kpart + ((size_t)z * a.npad + n) * a.mtr + rr));
    const int ro = a.prm[r];
    float y = __fmul_rn(__fmul_rn(acc, a.rsc[r].y), a.tdown[n]);
    const float *xn = a.X + (size_t)n * a.ldx;
    for (int e = a.cp[ro]; e < a.cp[ro + 1]; ++e) y = __fadd_rn(y, __fmul_rn(a.cv[e], xn[a.cc[e]]));
    a.Y[(size_t)n * a.ldy + ro] = y;
}

// ---------------------------------------------------------------------------------------------------------------
// host side
struct GemmPlan {
    int bn, nbs, np, tileb, npad, nkc, mt, nnt, ks;
    int nten;        // tensors in one launch: 1, or 2 of one shape whose row tiles fill the same waves
    int mh, kt;      // tail split (kt > 1): row tiles [0, mh) of the launch single-split in whole waves, the rest split kt
                     // ways along K (with two tensors the tail lies in the second)
    long long cost;  // modelled time
    size_t ss, xv;   // prologue only: partial sums of squares [npad][nkc], x' [npad][K]
    bool staged;     // single split, >= kGemmStagedMinCols tokens: outputs staged in sorted-row order, then un-permuted
    size_t xh, pmax, tdown, prep;  // the activation prep's part [0, prep)
    size_t kpart, yt, own;         // the launch's own part (offsets from its start; own = its size): split-K
                                   // partials, then staged outputs [mt * 128][npad] per tensor
    size_t total, smem;
};

static int gemm_tile_bytes(const p8_tensor *t) {  // staging bytes of one tile's half-slice: the largest class present
    int m = 1;
    for (int c = 1; c < 8; ++c)
        if (((t->class_mask >> c) & 1u) && NW(c) > m) m = NW(c);
    return m * 128;
}

static GemmPlan gemm_plan(const p8_tensor *t, int64_t ncols, bool pro = false, int nten = 1) {
    const int nsm = sm_count();
    GemmPlan p;
    p.nten = nten;
    p.mt = (t->rows + 127) / 128;
    const int mtg = nten * p.mt;  // row tiles of the launch
    // Tile width and K split: the lowest estimated time. A tile's time is modelled as BN + 200 (the MMA share plus
    // the decode and fixed part; the 200 is fitted to measured 128- and 256-wide tiles of the same projection).
    // Tiles that leave at least half the SMs idle are split along K (ks CTAs per tile, at least two 256-column blocks
    // each; time / ks). More tiles than SMs take whole waves, or a tail split: the row tiles of the full waves as
    // one launch, the remaining row tiles as a second launch split kt ways along K (one wave of 1/kt-long tiles),
    // charged 32 more for the extra launch and reduction. Widths below 64 are not used (no better in this model).
    const int kmax = t->nb / 2 > 1 ? t->nb / 2 : 1;
    int best = 256;
    long long best_cost = -1;
    p.ks = 1;
    p.mh = 0;
    p.kt = 1;
    for (int bn = 256; bn >= 64; bn >>= 1) {
        const long long nnt = (ncols + bn - 1) / bn, tiles = (long long)mtg * nnt, c = (long long)(bn + 200) * 64;
        long long cost;
        int ks = 1, mh = 0, kt = 1;
        if (2 * tiles <= nsm) {
            ks = (int)(nsm / tiles);
            if (ks > kmax) ks = kmax;
            cost = c / ks;
        } else {
            cost = (tiles + nsm - 1) / nsm * c;
            if (tiles > nsm && tiles % nsm) {
                const long long full = tiles / nsm;
                const int h = (int)(full * nsm / nnt);
                const long long tt = (long long)(mtg - h) * nnt;
                int k = h > 0 && tt > 0 ? (int)(nsm / tt) : 1;
                if (k > kmax) k = kmax;
                const long long ct = ((long long)h * nnt + nsm - 1) / nsm * c + c / (k > 1 ? k : 1) + 32 * 64;
                if (k >= 2 && ct < cost) { cost = ct; mh = h; kt = k; }
            }
        }
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = bn; p.ks = ks; p.mh = mh; p.kt = kt; }
    }
    p.cost = best_cost;
    p.bn = best;
    p.tileb = gemm_tile_bytes(t);
    p.nbs = best >= 256 ? 2 : best >= 128 ? 3 : kGemmMaxB;
    p.np = kGemmMaxP;
    while (p.np > 2 && gemm_smem_layout(p.bn, p.nbs, p.np, p.tileb, t->nb).total > kGemmSmemDyn) --p.np;
    while (p.nbs > 2 && gemm_smem_layout(p.bn, p.nbs, p.np, p.tileb, t->nb).total > kGemmSmemDyn) --p.nbs;
    p.smem = (size_t)gemm_smem_layout(p.bn, p.nbs, p.np, p.tileb, t->nb).total;
    p.nnt = (int)((ncols + best - 1) / best);
    p.npad = p.nnt * best;
    p.nkc = (t->K + 2047) / 2048;
    // workspace: the activation prep's part first (shared by the tensors of a group), then the launch's own part
    p.xh = 0;
    p.pmax = al256((size_t)t->K * p.npad * 2);
    p.tdown = p.pmax + al256((size_t)p.npad * p.nkc * 4);
    p.ss = p.tdown + al256((size_t)p.npad * 4);
    p.xv = p.ss + (pro ? al256((size_t)p.npad * p.nkc * 4) : 0);
    p.prep = p.xv + (pro ? al256((size_t)p.npad * t->K * 4) : 0);
    p.staged = p.ks == 1 && ncols >= kGemmStagedMinCols;
    p.kpart = 0;
    p.yt = p.kpart + (p.ks > 1   ? al256((size_t)p.ks * p.npad * mtg * 128 * 4)
                      : p.kt > 1 ? al256((size_t)p.kt * p.npad * (mtg - p.mh) * 128 * 4)
                                 : 0);
    p.own = p.yt + (p.staged ? (size_t)nten * al256((size_t)p.mt * 128 * p.npad * 4) : 0);
    p.total = p.prep + p.own;
    return p;
}

bool gemm_supported(const p8_tensor *t, int64_t ncols) {
    return ncols >= (t->uniform_class == 3 ? kGemmMinColsC3 : kGemmMinCols) && t->K <= 65536 && t->rsc != nullptr &&
           (size_t)gemm_plan(t, ncols).smem <= (size_t)kGemmSmemDyn;
}

size_t gemm_workspace(const p8_tensor *t, int64_t ncols, bool pro) { return gemm_plan(t, ncols, pro).total; }

// A group's tensors (equal K and prepared-activation hash) share one activation prep and run as launches of one
// tensor, or of two consecutive tensors of one shape (gate/up, k/v) when their row tiles together fill the waves
// better than apart. A pair shares a launch only where both tensors alone would run single-split without a tail, so
// that every row keeps its K order except the rows of a shared launch's tail split (then summed over kt splits).
// The launches' plans may pad the tokens differently (the tile width follows the row count), so the prep pads to
// the largest npad: Xh's panels carry that token count (GemmArgs::xpad) and each launch reads its first npad
// tokens, which are the same as its own prep's. The launches' own parts follow the prep's part, one after another.
struct GemmItem {
    int i0;
    GemmPlan p;
};

static int gemm_group_items(const p8_tensor *const *ts, int n, int64_t ncols, bool pro, GemmItem *it) {
    int m = 0;
    for (int i = 0; i < n;) {
        const GemmPlan p1 = gemm_plan(ts[i], ncols, pro);
        if (i + 1 < n && ts[i + 1]->rows == ts[i]->rows && gemm_tile_bytes(ts[i + 1]) == gemm_tile_bytes(ts[i])) {
            const GemmPlan p2 = gemm_plan(ts[i + 1], ncols, pro);
            const GemmPlan pp = gemm_plan(ts[i], ncols, pro, 2);
            if (p1.ks == 1 && p1.kt == 1 && p2.ks == 1 && p2.kt == 1 && pp.ks == 1 && (pp.kt == 1 || pp.mh >= pp.mt) &&
                pp.smem <= (size_t)kGemmSmemDyn && pp.cost < p1.cost + p2.cost) {
                it[m].i0 = i;
                it[m++].p = pp;
                i += 2;
                continue;
            }
        }
        it[m].i0 = i;
        it[m++].p = p1;
        ++i;
    }
    return m;
}

static int gemm_items_prep(const GemmItem *it, int m, size_t *own) {
    int j = 0;
    *own = 0;
    for (int i = 0; i < m; ++i) {
        if (it[i].p.npad > it[j].p.npad) j = i;
        if (it[i].p.own > *own) *own = it[i].p.own;
    }
    return j;
}

size_t gemm_group_workspace(const p8_tensor *const *ts, int n, int64_t ncols, bool pro) {
    if (n < 1 || n > 4) return 0;
    GemmItem it[4];
    const int m = gemm_group_items(ts, n, ncols, pro, it);
    size_t own = 0;
    const int j = gemm_items_prep(it, m, &own);
    return it[j].p.prep + own;
}

static void launch_args(GemmArgs &ga, const p8_tensor *t, const GemmPlan &p, const GxArgs &xa, int pk, const float *X,
                        int64_t ncols, int64_t ldx, float *Y, int64_t ldy) {
    ga.A = t->A; ga.M = t->M; ga.D = t->D; ga.S = t->S; ga.prm = t->prm; ga.rsc = t->rsc; ga.cp = t->cp; ga.cc = t->cc;
    ga.cv = t->cv; ga.Y = Y; ga.Xh = xa.Xh; ga.tdown = xa.tdown; ga.ldy = ldy; ga.cs = t->cs;
    ga.X = pk != P8_PROLOGUE_NONE ? xa.xv : X;  // the clamp-delta term multiplies x'
    ga.ldx = pk != P8_PROLOGUE_NONE ? t->K : ldx;
    ga.rows = t->rows; ga.nb = t->nb; ga.ng = t->ng; ga.ncols = (int)ncols; ga.npad = p.npad; ga.bn = p.bn; ga.nbs = p.nbs;
    ga.np = p.np; ga.tileb = p.tileb; ga.ucls = t->uniform_class;
    ga.xpad = xa.npad;
    ga.pinv = t->pinv;
}

// one launch of NT (1 or 2) tensors: k_gemm (with a tail split: the full waves, then the split-K tail), then the
// epilogue kernels (un-permute of staged outputs per tensor, split-K reduction)
template <int NT>
static p8_status launch_gemm_item(const p8_tensor *const *ts, const GemmPlan &p, const GxArgs &xa, int pk, const float *X,
                                  int64_t ncols, int64_t ldx, float *const *Ys, const int64_t *ldys, uint8_t *own,
                                  cudaStream_t st) {
    GemmLaunch<NT> gl;
    memset(&gl, 0, sizeof(gl));
    const int mtg = NT * p.mt, last = NT - 1;
    for (int i = 0; i < NT; ++i) {
        GemmArgs &ga = gl.t[i];
        launch_args(ga, ts[i], p, xa, pk, X, ncols, ldx, Ys[i], ldys[i]);
        ga.ksplit = p.ks;
        ga.mtr = p.mt * 128;
        ga.rs = p.ks > 1 ? 0 : ts[i]->rows;
        ga.kpart = reinterpret_cast<float *>(own + p.kpart);
        ga.Yt = p.staged ? reinterpret_cast<float *>(own + p.yt + (size_t)i * al256((size_t)p.mt * 128 * p.npad * 4)) : nullptr;
    }
    gl.mt0 = 0;
    gl.mtA = NT > 1 ? p.mt : mtg;
    const void *fn = (const void *)k_gemm<NT>;
    void *args[] = {&gl};
    GemmLaunch<NT> tl = gl;
    if (p.kt > 1) {
        gl.t[last].rs = (p.mh - last * p.mt) * 128;  // the tail's first row in the last tensor
        tl = gl;
        tl.mt0 = p.mh;
        tl.t[last].ksplit = p.kt;
        tl.t[last].mtr = (mtg - p.mh) * 128;
        void *targs[] = {&tl};
        if (launch_pdl(fn, dim3(p.mh, p.nnt, 1), dim3(kGemmThreads), p.smem, st, args) != cudaSuccess ||
            launch_pdl(fn, dim3(mtg - p.mh, p.nnt, p.kt), dim3(kGemmThreads), p.smem, st, targs) != cudaSuccess)
            return P8_ERR_CUDA;
    } else if (launch_pdl(fn, dim3(mtg, p.nnt, p.ks), dim3(kGemmThreads), p.smem, st, args) != cudaSuccess) {
        return P8_ERR_CUDA;
    }
    for (int i = 0; p.staged && i < NT; ++i) {
        void *uargs[] = {&gl.t[i]};
        if (launch_pdl((const void *)k_unpermute, dim3((unsigned)((ts[i]->rows + 255) / 256), (unsigned)((ncols + 7) / 8)), dim3(256),
                       0, st, uargs) != cudaSuccess)
            return P8_ERR_CUDA;
    }
    if (p.ks > 1 || p.kt > 1) {
        GemmArgs *ra = p.kt > 1 ? &tl.t[last] : &gl.t[0];
        void *rargs[] = {ra};
        const long long outs = (long long)(ra->rows - ra->rs) * ncols;
        if (launch_pdl((const void *)k_splitk_reduce, dim3((unsigned)((outs + 255) / 256)), dim3(256), 0, st, rargs) != cudaSuccess)
            return P8_ERR_CUDA;
    }
    return P8_OK;
}

// tensors reading the same X (equal K and activation hash, checked by the caller): one activation prep, then the
// group's launches
p8_status launch_gemm_group(const p8_tensor *const *ts, int n, const float *X, int64_t ncols, int64_t ldx, float *const *Ys,
                            const int64_t *ldys, void *ws, size_t ws_bytes, cudaStream_t st, const p8_prologue *pro) {
    if (n < 1 || n > 4) return P8_ERR_ARG;
    const int pk = pro ? pro->kind : P8_PROLOGUE_NONE;
    for (int i = 0; i < n; ++i)
        if (ts[i]->K != ts[0]->K) return P8_ERR_ARG;
    GemmItem it[4];
    const int m = gemm_group_items(ts, n, ncols, pk != P8_PROLOGUE_NONE, it);
    for (int i = 0; i < m; ++i)
        if (it[i].p.smem > (size_t)kGemmSmemDyn) return P8_ERR_UNSUPPORTED;
    size_t own = 0;
    const GemmPlan &p = it[gemm_items_prep(it, m, &own)].p;
    if (!ws || ws_bytes < p.prep + own || ((uintptr_t)ws & 255)) return P8_ERR_WORKSPACE;
    static std::atomic<bool> attr_set[64];  // published after the attributes are set (see sm_count)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(k_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmemDyn) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemm<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmemDyn) != cudaSuccess)
            return P8_ERR_CUDA;
        if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
    }
    const p8_tensor *t = ts[0];
    uint8_t *w = static_cast<uint8_t *>(ws);
    GxArgs xa;
    memset(&xa, 0, sizeof(xa));
    if (pk != P8_PROLOGUE_NONE) {
        xa.pw = pro->w;
        xa.x2 = pro->x2;
        xa.eps = pro->eps;
        xa.ss = reinterpret_cast<float *>(w + p.ss);
        xa.xv = reinterpret_cast<float *>(w + p.xv);
    }
    xa.X = X; xa.ic = t->ic; xa.ldx = ldx; xa.K = t->K; xa.nb = t->nb; xa.ncols = (int)ncols; xa.npad = p.npad; xa.nkc = p.nkc;
    xa.Xh = w + p.xh;
    xa.pmax = reinterpret_cast<float *>(w + p.pmax);
    xa.tdown = reinterpret_cast<float *>(w + p.tdown);
    {
        void *args[] = {&xa};
        const void *fm = pk == P8_PROLOGUE_RMSNORM ? (const void *)k_gx_max<P8_PROLOGUE_RMSNORM>
                         : pk == P8_PROLOGUE_SWIGLU  ? (const void *)k_gx_max<P8_PROLOGUE_SWIGLU>
                                                     : (const void *)k_gx_max<P8_PROLOGUE_NONE>;
        const void *fp = pk == P8_PROLOGUE_RMSNORM ? (const void *)k_gx_prep<P8_PROLOGUE_RMSNORM>
                         : pk == P8_PROLOGUE_SWIGLU  ? (const void *)k_gx_prep<P8_PROLOGUE_SWIGLU>
                                                     : (const void *)k_gx_prep<P8_PROLOGUE_NONE>;
        if (launch_pdl(fm, dim3(p.npad, p.nkc), dim3(256), 0, st, args) != cudaSuccess) return P8_ERR_CUDA;
        if (launch_pdl(fp, dim3(p.npad / 8, (t->nb + kGxBlocksPerCta - 1) / kGxBlocksPerCta), dim3(256), 0, st, args) !=
            cudaSuccess)
            return P8_ERR_CUDA;
    }
    for (int i = 0; i < m; ++i) {
        const int i0 = it[i].i0;
        const p8_status r =
            it[i].p.nten > 1 ? launch_gemm_item<2>(ts + i0, it[i].p, xa, pk, X, ncols, ldx, Ys + i0, ldys + i0, w + p.prep, st)
                             : launch_gemm_item<1>(ts + i0, it[i].p, xa, pk, X, ncols, ldx, Ys + i0, ldys + i0, w + p.prep, st);
        if (r) return r;
    }
    return P8_OK;
}

p8_status launch_gemm(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, float *Y, int64_t ldy, void *ws,
                      size_t ws_bytes, cudaStream_t st, const p8_prologue *pro) {
    return launch_gemm_group(&t, 1, X, ncols, ldx, &Y, &ldy, ws, ws_bytes, st, pro);
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
