// p8_encode.cu -- offline trellis encoder on the GPU: one 128-column slice of the LDLQ Viterbi that turns the
// FWHT-domain weights of a tensor into Pingala-8 codes (the reference encoder, research/detail/r48k.py: encode
// r48k.py:105, vit_k r48k.py:57, best_cw r48k.py:33, zero_ldlq r48k.py:97; trellis mode with the 8 gana states).
//
// Per row of the slice (128 columns = 32 steps of 4 weights) the encoder keeps one survivor per trellis state: its path
// metric and its residual weights (earlier steps' quantisation errors fed forward through the Cholesky block Hb). A
// step finds, for every (state, stored half bit) pair, the codeword nearest to the state's residual in the
// A4[t]-transformed metric, adds it to the path metric, keeps the better of the two transitions into each state,
// and updates the survivors' residuals. The last step's best state is traced back to the codes.
//
// Layout on the GPU: a half-warp per row (16 lanes: lane = (state, half) pair during the search, columns during the
// residual update), two rows per warp, rows independent. Per-row state lives in shared memory; the step tables
// TA[t][i] = A[i] @ A4[t] (every class's stage tables are power-of-two multiples of them) come from a small pre-kernel.
// Float operations follow the reference's formulas and order where it defines one (x / S - off, then @ Am; squared
// differences summed in index order; ties to the first index; the first of the two transitions into a state on a tie),
// so the codes match the reference except where two candidates' metrics differ in the last bits.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <atomic>
#include <string.h>

#include "p8_internal.h"

namespace p8 {
namespace {

constexpr int kVitRowsPerCta = 8;  // 4 warps, 2 rows each
constexpr int kSteps = 32;         // 4-weight steps per 128-column slice
constexpr int kNS = 8;             // trellis states

// per-row shared memory (floats unless noted)
struct RowSmem {
    float xs[2][kNS][132];      // survivors' residuals (double buffered; rows padded so the 8 states sit in different banks)
    float xn[kSteps][kNS][4];   // residual of the chosen source per step and state (for the error in the traceback)
    float e[kNS][4];            // this step's transformed errors per destination state
    uint8_t src[kSteps][kNS];   // chosen source state
    uint8_t id[kSteps][kNS][4]; // chosen (i1, i2, i3)
    int srcd[kNS];
    int path[kSteps];
};

struct VitArgs {
    const float *X;      long long ldx;  // slice of the (residual-updated) weights, row r at X + r * ldx
    const float *Hb;     long long ldh;  // Cholesky block of the slice (upper triangular), row-major
    const float *A4;                     // [32][4][4] inverses of Hb's diagonal 4 x 4 blocks
    const float *TA;                     // [32][256][4] codebook rows times A4[t]
    const int8_t *A;                     // codebook [256][4]
    const uint8_t *cls;  long long ldc;  // class of row r: cls[r * ldc]
    const float *S;      long long lds;  // scale of row r: S[r * lds]
    int rows;
    float *Q;            long long ldq;  // out: quantised values (int units x S)
    float *E;            long long lde;  // out: errors in the A4-transformed metric (the encoder's feedback term)
    uint8_t *IDX;        long long ldi;  // out: (i1, i2, i3) of step t at IDX + r * ldi + 3 t
    float cvec[4];                       // coset vector c
};

__device__ __forceinline__ uint32_t ux_of(int s) { return (uint32_t)((s ^ (s >> 2)) & 1); }  // parity(s & 0b101)
__device__ __forceinline__ float z0_of(int s) { return (float)((s >> 1) & 1); }             // parity(s & 0b010)

// squared distance of the 4-vector (x - sc * t), summed in index order, no fused operations (the reference's
// (x - T).pow(2).sum(-1))
__device__ __forceinline__ float dist4(const float (&x)[4], float4 t, float sc) {
    const float d0 = __fsub_rn(x[0], __fmul_rn(sc, t.x)), d1 = __fsub_rn(x[1], __fmul_rn(sc, t.y));
    const float d2 = __fsub_rn(x[2], __fmul_rn(sc, t.z)), d3 = __fsub_rn(x[3], __fmul_rn(sc, t.w));
    return __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(d0, d0), __fmul_rn(d1, d1)), __fmul_rn(d2, d2)), __fmul_rn(d3, d3));
}

__device__ __forceinline__ float4 ta_at(const float *TAt, int i) { return __ldg(reinterpret_cast<const float4 *>(TAt) + i); }

// insert (v, i) into the ascending top-4 list (equal values keep scan order)
__device__ __forceinline__ void top4_insert(float (&v)[4], int (&ix)[4], float d, int i) {
    if (!(d < v[3])) return;
    if (d < v[2]) {
        v[3] = v[2]; ix[3] = ix[2];
        if (d < v[1]) {
            v[2] = v[1]; ix[2] = ix[1];
            if (d < v[0]) {
                v[1] = v[0]; ix[1] = ix[0];
                v[0] = d; ix[0] = i;
            } else {
                v[1] = d; ix[1] = i;
            }
        } else {
            v[2] = d; ix[2] = i;
        }
    } else {
        v[3] = d; ix[3] = i;
    }
}

// Best codeword of class C in half H (stage-1 MSB) for the transformed target xa (best_cw): cost and (i1, i2, i3).
// Stage tables: t1 = 2^SH1 A[0 .. 2^W1), t2 = 2^SH2 A[0 .. 2^W2), t3 = A[0 .. 2^W3), each times A4[t] = TA scaled.
// One stage: the nearest entry of the half. More stages: the 4 nearest stage-1 entries of the half, then for each the
// nearest stage-2 entry to the residual (two stages), or the 4 nearest stage-2 entries and for each the nearest
// stage-3 entry (three stages); the smallest final distance wins, the first on ties in (stage-1 rank, stage-2 rank).
template <int C>
__device__ __forceinline__ void best_cw(const float (&xa)[4], const float *TAt, int H, float &cost, int &i1, int &i2, int &i3) {
    constexpr int K1 = 1 << W1(C), hs = K1 / 2;
    const float sc1 = (float)(1 << SH1(C)), sc2 = (float)(1 << SH2(C));
    i2 = 0;
    i3 = 0;
    if (NST(C) == 1) {
        float best = INFINITY;
        int bi = H * hs;
#pragma unroll 8
        for (int m = 0; m < hs; ++m) {
            const int i = H * hs + m;
            const float d = dist4(xa, ta_at(TAt, i), sc1);
            if (d < best) { best = d; bi = i; }
        }
        cost = best;
        i1 = bi;
        return;
    }
    float v1[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
    int t1i[4] = {H * hs, H * hs, H * hs, H * hs};
#pragma unroll 8
    for (int m = 0; m < hs; ++m) {
        const int i = H * hs + m;
        top4_insert(v1, t1i, dist4(xa, ta_at(TAt, i), sc1), i);
    }
    constexpr int K2 = 1 << W2(C);
    float best = INFINITY;
    int b1 = t1i[0], b2 = 0, b3 = 0;
#pragma unroll 1
    for (int T = 0; T < 4; ++T) {
        const float4 a = ta_at(TAt, t1i[T]);
        const float r1[4] = {__fsub_rn(xa[0], __fmul_rn(sc1, a.x)), __fsub_rn(xa[1], __fmul_rn(sc1, a.y)),
                             __fsub_rn(xa[2], __fmul_rn(sc1, a.z)), __fsub_rn(xa[3], __fmul_rn(sc1, a.w))};
        if (NST(C) == 2) {
            float c2 = INFINITY;
            int j2 = 0;
#pragma unroll 8
            for (int i = 0; i < K2; ++i) {
                const float d = dist4(r1, ta_at(TAt, i), sc2);
                if (d < c2) { c2 = d; j2 = i; }
            }
            if (c2 < best) { best = c2; b1 = t1i[T]; b2 = j2; }
        } else {
            float v2[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
            int t2i[4] = {0, 0, 0, 0};
#pragma unroll 8
            for (int i = 0; i < K2; ++i) top4_insert(v2, t2i, dist4(r1, ta_at(TAt, i), sc2), i);
            constexpr int K3 = 1 << W3(C);
#pragma unroll 1
            for (int u = 0; u < 4; ++u) {
                const float4 b = ta_at(TAt, t2i[u]);
                const float r2[4] = {__fsub_rn(r1[0], __fmul_rn(sc2, b.x)), __fsub_rn(r1[1], __fmul_rn(sc2, b.y)),
                                     __fsub_rn(r1[2], __fmul_rn(sc2, b.z)), __fsub_rn(r1[3], __fmul_rn(sc2, b.w))};
                float c3 = INFINITY;
                int j3 = 0;
#pragma unroll 8
                for (int i = 0; i < K3; ++i) {
                    const float d = dist4(r2, ta_at(TAt, i), 1.f);
                    if (d < c3) { c3 = d; j3 = i; }
                }
                if (c3 < best) { best = c3; b1 = t1i[T]; b2 = t2i[u]; b3 = j3; }
            }
        }
    }
    cost = best;
    i1 = b1;
    i2 = b2;
    i3 = b3;
}

// integer-unit codeword of class C for (i1, i2, i3): t1[i1] + t2[i2] + t3[i3], summed in that order
template <int C>
__device__ __forceinline__ void cw_of(const int8_t *A, int i1, int i2, int i3, float (&cw)[4]) {
    const float sc1 = (float)(1 << SH1(C)), sc2 = (float)(1 << SH2(C));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float v = __fmul_rn((float)A[4 * i1 + k], sc1);
        if (W2(C)) v = __fadd_rn(v, __fmul_rn((float)A[4 * i2 + k], sc2));
        if (W3(C)) v = __fadd_rn(v, (float)A[4 * i3 + k]);
        cw[k] = v;
    }
}

// TA[t][i] = A[i] @ A4[t] (row vector times 4 x 4), one thread per (t, i)
__global__ void __launch_bounds__(256) k_vit_tables(const int8_t *A, const float *A4, float *TA) {
    const int t = blockIdx.x, i = threadIdx.x;
    const float *m = A4 + 16 * t;
    float a[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) a[k] = (float)A[4 * i + k];
    float4 o;
    float *op = reinterpret_cast<float *>(&o);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        float v = __fmul_rn(a[0], m[c]);
#pragma unroll
        for (int k = 1; k < 4; ++k) v = __fmaf_rn(a[k], m[4 * k + c], v);
        op[c] = v;
    }
    reinterpret_cast<float4 *>(TA)[t * 256 + i] = o;
}

// x @ m for a row 4-vector and a row-major 4 x 4 matrix, k in order (first product, then fused adds)
__device__ __forceinline__ void vecmat4(const float (&x)[4], const float *m, float (&o)[4]) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        float v = __fmul_rn(x[0], m[c]);
#pragma unroll
        for (int k = 1; k < 4; ++k) v = __fmaf_rn(x[k], m[4 * k + c], v);
        o[c] = v;
    }
}

// class-0 rows (zero_ldlq): nothing is quantised; the whole row is error, fed forward step by step
__device__ void zero_row(const VitArgs &a, int r, RowSmem &sm, int h, unsigned hmask) {
    float *x = sm.xs[0][0];
    for (int c = h; c < 128; c += 16) x[c] = a.X[(long long)r * a.ldx + c];
    __syncwarp(hmask);
    for (int t = 0; t < kSteps; ++t) {
        const int j = 4 * t;
        if (h == 0) {
            const float xv[4] = {x[j], x[j + 1], x[j + 2], x[j + 3]};
            float e[4];
            vecmat4(xv, a.A4 + 16 * t, e);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                sm.e[0][k] = e[k];
                a.E[(long long)r * a.lde + j + k] = e[k];
                a.Q[(long long)r * a.ldq + j + k] = 0.f;
            }
        }
        __syncwarp(hmask);
        for (int c = j + 4 + h; c < 128; c += 16) {
            const float *hb = a.Hb + (long long)j * a.ldh + c;
            float v = __fmul_rn(sm.e[0][0], __ldg(hb));
#pragma unroll
            for (int k = 1; k < 4; ++k) v = __fmaf_rn(sm.e[0][k], __ldg(hb + k * a.ldh), v);
            x[c] = __fsub_rn(x[c], v);
        }
        __syncwarp(hmask);
    }
}

template <int C>
__device__ void vit_row(const VitArgs &a, int r, RowSmem &sm, int h, unsigned hmask) {
    const float S = a.S[(long long)r * a.lds];
    const int s = h >> 1, H = h & 1;  // search pair of this lane
    const float mcz = (float)MC(C);
    float off_s[4];  // coset offset of state s: z0(s) * (MC * c)
#pragma unroll
    for (int k = 0; k < 4; ++k) off_s[k] = __fmul_rn(z0_of(s), __fmul_rn(mcz, a.cvec[k]));
    for (int c = h; c < 128; c += 16) {
        const float v = a.X[(long long)r * a.ldx + c];
#pragma unroll
        for (int q = 0; q < kNS; ++q) sm.xs[0][q][c] = v;
    }
    float pm = (h == 0) ? 0.f : INFINITY;  // lane d < 8 holds the path metric of state d
    __syncwarp(hmask);
    int cur = 0;
    for (int t = 0; t < kSteps; ++t) {
        const int j = 4 * t;
        const float *Am = a.A4 + 16 * t;
        const float *TAt = a.TA + (size_t)t * 256 * 4;
        // search: xa = (x_s / S - off_s) @ Am, then the best codeword of half H
        float xa[4];
        {
            float v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __fsub_rn(__fdiv_rn(sm.xs[cur][s][j + k], S), off_s[k]);
            vecmat4(v, Am, xa);
        }
        float cost;
        int i1, i2, i3;
        best_cw<C>(xa, TAt, H, cost, i1, i2, i3);
        const float pm_s = __shfl_sync(hmask, pm, s, 16);
        const float cand = __fadd_rn(pm_s, cost);
        // each state d has two sources: s1 = d >> 1 and s2 = s1 | 4, with half bit b = (d & 1) ^ ux(s)
        const int d = h & 7, s1 = d >> 1, s2 = s1 | 4;
        const int q1 = 2 * s1 + (int)((uint32_t)(d & 1) ^ ux_of(s1)), q2 = 2 * s2 + (int)((uint32_t)(d & 1) ^ ux_of(s2));
        const float c1 = __shfl_sync(hmask, cand, q1, 16), c2 = __shfl_sync(hmask, cand, q2, 16);
        const int q = (c2 < c1) ? q2 : q1;  // the first source on a tie
        const int g1 = __shfl_sync(hmask, i1, q, 16), g2 = __shfl_sync(hmask, i2, q, 16), g3 = __shfl_sync(hmask, i3, q, 16);
        if (h < kNS) {
            pm = (c2 < c1) ? c2 : c1;
            const int src = q >> 1;
            float cw[4];
            cw_of<C>(a.A, g1, g2, g3, cw);
            const float z = z0_of(src);
            float u[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float offk = __fmul_rn(z, __fmul_rn(mcz, a.cvec[k]));
                const float xn = sm.xs[cur][src][j + k];
                sm.xn[t][h][k] = xn;
                u[k] = __fsub_rn(xn, __fmul_rn(__fadd_rn(cw[k], offk), S));  // xn - (cw + off) * S
            }
            float e[4];
            vecmat4(u, Am, e);
#pragma unroll
            for (int k = 0; k < 4; ++k) sm.e[h][k] = e[k];
            sm.src[t][h] = (uint8_t)src;
            sm.srcd[h] = src;
            sm.id[t][h][0] = (uint8_t)g1;
            sm.id[t][h][1] = (uint8_t)g2;
            sm.id[t][h][2] = (uint8_t)g3;
        }
        __syncwarp(hmask);
        if (t + 1 < kSteps) {  // survivors' residuals: x_d[c] = x_src[c] - e_d @ Hb[j .. j+3][c]
            const int nxt = cur ^ 1;
            for (int c = j + 4 + h; c < 128; c += 16) {
                const float *hb = a.Hb + (long long)j * a.ldh + c;
                const float h0 = __ldg(hb), h1 = __ldg(hb + a.ldh), h2 = __ldg(hb + 2 * a.ldh), h3 = __ldg(hb + 3 * a.ldh);
#pragma unroll
                for (int dd = 0; dd < kNS; ++dd) {
                    float v = __fmul_rn(sm.e[dd][0], h0);
                    v = __fmaf_rn(sm.e[dd][1], h1, v);
                    v = __fmaf_rn(sm.e[dd][2], h2, v);
                    v = __fmaf_rn(sm.e[dd][3], h3, v);
                    sm.xs[nxt][dd][c] = __fsub_rn(sm.xs[cur][sm.srcd[dd]][c], v);
                }
            }
            cur = nxt;
        }
        __syncwarp(hmask);
    }
    // best final state (the first on a tie), then the path back through the recorded sources
    float best = __shfl_sync(hmask, pm, 0, 16);
    int bs = 0;
#pragma unroll
    for (int dd = 1; dd < kNS; ++dd) {
        const float v = __shfl_sync(hmask, pm, dd, 16);
        if (v < best) { best = v; bs = dd; }
    }
    if (h == 0) {
        int st = bs;
        for (int t = kSteps - 1; t >= 0; --t) {
            sm.path[t] = st;
            st = sm.src[t][st];
        }
    }
    __syncwarp(hmask);
    for (int t = h; t < kSteps; t += 16) {
        const int st = sm.path[t], src = sm.src[t][st], j = 4 * t;
        const int g1 = sm.id[t][st][0], g2 = sm.id[t][st][1], g3 = sm.id[t][st][2];
        float cw[4], u[4], e[4], qv[4];
        cw_of<C>(a.A, g1, g2, g3, cw);
        const float z = z0_of(src);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            qv[k] = __fmul_rn(__fadd_rn(cw[k], __fmul_rn(z, __fmul_rn(mcz, a.cvec[k]))), S);
            u[k] = __fsub_rn(sm.xn[t][st][k], qv[k]);
        }
        vecmat4(u, a.A4 + 16 * t, e);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            a.Q[(long long)r * a.ldq + j + k] = qv[k];
            a.E[(long long)r * a.lde + j + k] = e[k];
        }
        uint8_t *o = a.IDX + (long long)r * a.ldi + 3 * t;
        o[0] = (uint8_t)g1;
        o[1] = (uint8_t)g2;
        o[2] = (uint8_t)g3;
    }
}

extern __shared__ __align__(16) uint8_t g_enc_smem[];

__global__ void __launch_bounds__(128) k_vit(const __grid_constant__ VitArgs a) {
    const int lane = threadIdx.x & 31, h = lane & 15, slot = threadIdx.x >> 4;
    const unsigned hmask = 0xFFFFu << (lane & 16);
    const int r = blockIdx.x * kVitRowsPerCta + slot;
    if (r >= a.rows) return;  // whole half-warps leave together
    RowSmem &sm = reinterpret_cast<RowSmem *>(g_enc_smem)[slot];
    switch (a.cls[(long long)r * a.ldc]) {
        case 0: zero_row(a, r, sm, h, hmask); break;
        case 1: vit_row<1>(a, r, sm, h, hmask); break;
        case 2: vit_row<2>(a, r, sm, h, hmask); break;
        case 3: vit_row<3>(a, r, sm, h, hmask); break;
        case 4: vit_row<4>(a, r, sm, h, hmask); break;
        case 5: vit_row<5>(a, r, sm, h, hmask); break;
        case 6: vit_row<6>(a, r, sm, h, hmask); break;
        default: vit_row<7>(a, r, sm, h, hmask); break;
    }
}

}  // namespace
}  // namespace p8

using namespace p8;

extern "C" {

size_t p8_encode_workspace(void) { return (size_t)32 * 256 * 4 * sizeof(float); }

p8_status p8_encode_slice(const float *X, int64_t ldx, const float *Hb, int64_t ldh, const float *A4, const int8_t *codebook,
                          const int8_t *coset, const uint8_t *cls, int64_t ldc, const float *S, int64_t lds, int64_t rows, float *Q,
                          int64_t ldq, float *E, int64_t lde, uint8_t *IDX, int64_t ldi, void *workspace, size_t workspace_bytes,
                          void *stream) {
    if (rows < 0 || rows > (int64_t)1 << 30) return P8_ERR_ARG;
    if (rows == 0) return P8_OK;
    if (!X || !Hb || !A4 || !codebook || !coset || !cls || !S || !Q || !E || !IDX || ldx < 128 || ldh < 128 || ldq < 128 ||
        lde < 128 || ldi < 96 || ldc < 0 || lds < 0)
        return P8_ERR_ARG;
    if (!workspace || workspace_bytes < p8_encode_workspace() || ((uintptr_t)workspace & 15)) return P8_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    float *TA = static_cast<float *>(workspace);
    k_vit_tables<<<kSteps, 256, 0, st>>>(codebook, A4, TA);
    if (cudaGetLastError() != cudaSuccess) return P8_ERR_CUDA;
    VitArgs a;
    memset(&a, 0, sizeof(a));
    a.X = X; a.ldx = ldx; a.Hb = Hb; a.ldh = ldh; a.A4 = A4; a.TA = TA; a.A = codebook; a.cls = cls; a.ldc = ldc; a.S = S;
    a.lds = lds; a.rows = (int)rows; a.Q = Q; a.ldq = ldq; a.E = E; a.lde = lde; a.IDX = IDX; a.ldi = ldi;
    for (int k = 0; k < 4; ++k) a.cvec[k] = (float)coset[k];
    const size_t smem = sizeof(RowSmem) * kVitRowsPerCta;
    static std::atomic<bool> attr[64];  // the attribute is per device; published after it is set
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return P8_ERR_CUDA;
    if (dev < 0 || dev >= 64 || !attr[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(k_vit, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return P8_ERR_CUDA;
        if (dev >= 0 && dev < 64) attr[dev].store(true, std::memory_order_release);
    }
    const unsigned grid = (unsigned)((rows + kVitRowsPerCta - 1) / kVitRowsPerCta);
    k_vit<<<grid, 128, smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? P8_OK : P8_ERR_CUDA;
}

}  // extern "C"
