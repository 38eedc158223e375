/*
 * ref_harness.c -- TEST INFRASTRUCTURE ONLY (the timed CPU baseline and a second checker).
 *
 * Thin glue around the reference's OWN CPU core `vr-native-cpu-core.h` (patches/llama_cpu_vs_7ac59a6.patch CP:144-1027),
 * which oracle/build_ref.py extracts from the patch text into oracle/_ref/ (never committed). The ggml glue of the
 * reference (vr-native-cpu.c, CP:1028-1312) needs ggml internals (threadpool, barriers, tensors), so its two compute
 * paths are restated here with OpenMP in place of the ggml threadpool:
 *   ref_gemv_x16    = vrc_tg (CP:1161-1199): x16 planes, vrc_prep_cx, vrc_tile_v4x per 32-row group, CSR delta.
 *   ref_mul_mat_x16 = ggml_vr_cpu_mul_mat batch path (CP:1201-1262) with x16 on (GGML_VR_CPU_X16 semantics), vrc_tile_ls.
 * Work is split by 32-row groups (the reference's dynamic chunks), each output element written once.
 */
#include "vr-native-cpu-core.h"
#include "ggml-vr-native.h"
#include "llama-vr3.h"
#include <omp.h>
#include <stdio.h>

size_t ref_meta_size(void) { return sizeof(vrc_meta); }
int ref_init(vrc_meta *m, const uint8_t *base, size_t n, int rows, int K) { return vrc_init(m, base, n, rows, K); }
void ref_free(vrc_meta *m) { vrc_free(m); }
void ref_decode_tile_int(const vrc_meta *m, int g, int b, int16_t *xi) { vrc_decode_tile_int(m, g, b, xi); }
void ref_dequant_f32(const vrc_meta *m, float *W) { vrc_dequant_f32(m, W); }
int ref_threads(void) { return omp_get_max_threads(); }
/* all host cores for the timed baseline, whatever OMP_NUM_THREADS says (torchrun sets it to 1) */
void ref_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
int ref_has_v4(void) {
#if defined(VRC_V4)
    return 1;
#else
    return 0;
#endif
}
const char *ref_isa(void) {
#if defined(__AVXVNNI__)
    return "AVX2+AVX-VNNI";
#elif defined(__AVX2__)
    return "AVX2";
#else
    return "scalar";
#endif
}

/* contract helpers (ggml-vr-native.h CU:25-51, llama-vr3.h CU:3630-3660) */
size_t ref_need(size_t kbytes, size_t rows, size_t K, size_t nd) { return vrn_need(kbytes, rows, K, nd); }
void ref_offsets(size_t n, size_t rows, size_t K, size_t nd, size_t *o6) {
    vrn_offsets(n, rows, K, nd, &o6[0], &o6[1], &o6[2], &o6[3], &o6[4], &o6[5]);
}
size_t ref_vr3_rows(size_t fbytes, size_t K, uint32_t w515, size_t *kbytes) { return vrn3_rows(fbytes, K, w515, kbytes); }
void ref_vr3_expand(const uint8_t *f, size_t fbytes, size_t rows, size_t K, uint8_t *dst) { vrn3_expand(f, fbytes, rows, K, dst); }

/* batch path (CP:1201-1262), x16 on: virtual columns 2n (hi plane) and 2n+1 (lo plane) */
#if defined(__AVX2__)
void ref_mul_mat_x16(const vrc_meta *m, const float *X, int N, int ldx, float *Y, int ldy) {
    const int nsl = m->nsl, nb = m->nb, NV = 2 * N;
    int8_t *X2 = (int8_t *)aligned_alloc(64, ((size_t)NV * nsl * 256 + 63) & ~(size_t)63);
    float *XS = (float *)malloc(sizeof(float) * (size_t)NV * nsl);
    int32_t *SX = (int32_t *)malloc(sizeof(int32_t) * (size_t)NV * nsl);
#pragma omp parallel for schedule(static)
    for (int u = 0; u < N * nb; ++u) {
        const int n = u / nb, b = u % nb;
        const float *xc = X + (size_t)n * ldx;
        vrc_prep_block16(m, xc, b, X2 + ((size_t)(2 * n) * nsl + 2 * b) * 256, XS + (size_t)(2 * n) * nsl + 2 * b, SX + (size_t)(2 * n) * nsl + 2 * b,
                         X2 + ((size_t)(2 * n + 1) * nsl + 2 * b) * 256, XS + (size_t)(2 * n + 1) * nsl + 2 * b, SX + (size_t)(2 * n + 1) * nsl + 2 * b);
    }
    const int ncb = 64, ncblk = (NV + ncb - 1) / ncb, items = m->ng * ncblk;
#pragma omp parallel
    {
        __m256i tbv[96], acci[64];
        float *accY = (float *)aligned_alloc(64, sizeof(float) * 64 * 32);
#pragma omp for schedule(dynamic, 1)
        for (int it = 0; it < items; ++it) {
            const int g = it % m->ng, cb = it / m->ng, n0 = cb * ncb, nc = NV - n0 < ncb ? NV - n0 : ncb;
            memset(accY, 0, sizeof(float) * 32 * nc);
            for (int b = 0; b < nb; ++b) vrc_tile_ls(m, g, b, nc, X2 + (size_t)n0 * nsl * 256, XS + (size_t)n0 * nsl, SX + (size_t)n0 * nsl, accY, tbv, acci);
            for (int j = 0; j < 32; ++j) {
                const int ro = m->prm[g * 32 + j], e0 = m->cp[ro], e1 = m->cp[ro + 1];
                for (int nn = 0; nn < nc; nn += 2) {
                    float a = accY[nn * 32 + j] + accY[(nn + 1) * 32 + j];
                    const int col = (n0 + nn) / 2;
                    const float *xr = X + (size_t)col * ldx;
                    for (int e = e0; e < e1; ++e) a += m->cv[e] * xr[m->cc[e]];
                    Y[(size_t)col * ldy + ro] = a;
                }
            }
        }
        free(accY);
    }
    free(X2); free(XS); free(SX);
}
#endif

/* tg path (CP:1161-1199), x16 (2 planes); falls back to the batch path when the core has no v4 kernel (no AVX-VNNI) */
void ref_gemv_x16(const vrc_meta *m, const float *x, float *y) {
#if defined(VRC_V4)
    const int nb = m->nb, nsl = m->nsl;
    const size_t xps = (size_t)nsl * 256, sps = (size_t)nsl, lhs = (size_t)nsl * 16;
    int8_t *X = (int8_t *)aligned_alloc(64, 2 * xps);
    float *XS = (float *)malloc(sizeof(float) * 2 * sps);
    int32_t *SX = (int32_t *)malloc(sizeof(int32_t) * 2 * sps);
    uint32_t *LH = (uint32_t *)aligned_alloc(64, sizeof(uint32_t) * 2 * lhs);
#pragma omp parallel for schedule(static)
    for (int b = 0; b < nb; ++b) {
        vrc_prep_block16(m, x, b, X + (size_t)2 * b * 256, XS + 2 * b, SX + 2 * b, X + xps + (size_t)2 * b * 256, XS + sps + 2 * b, SX + sps + 2 * b);
        for (int p = 0; p < 2; ++p)
            for (int hs = 0; hs < 2; ++hs) vrc_prep_cx(m->cs, X + p * xps + (size_t)(2 * b + hs) * 256, LH + p * lhs + (size_t)(2 * b + hs) * 16);
    }
#pragma omp parallel for schedule(dynamic, 1)
    for (int g = 0; g < m->ng; ++g) {
        _Alignas(64) float accY[32];
        memset(accY, 0, sizeof accY);
        for (int b = 0; b < nb; ++b) vrc_tile_v4x(m, g, b, X, xps, XS, SX, sps, LH, lhs, accY);
        for (int j = 0; j < 32; ++j) {
            const int ro = m->prm[g * 32 + j];
            float a = accY[j];
            for (int e = m->cp[ro]; e < m->cp[ro + 1]; ++e) a += m->cv[e] * x[m->cc[e]];
            y[ro] = a;
        }
    }
    free(X); free(XS); free(SX); free(LH);
#elif defined(__AVX2__)
    ref_mul_mat_x16(m, x, 1, m->K, y, m->rows);
#else
#error "the reference CPU core needs AVX2 for its x16 paths"
#endif
}
