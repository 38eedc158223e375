// p8_internal.h -- library-internal declarations (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "pingala8.h"
#include "p8_format.h"

// A prepared tensor: device pointers into the caller's slot plus the small device arrays built at prepare time.
struct p8_tensor {
    uint32_t magic;  // kTensorMagic while alive
    int device;
    const uint8_t *slot;
    size_t nbytes, kbytes, nt;
    int rows, K, nb, ng, nsl, nd;
    // device pointers into the slot
    const uint32_t *A;  // codebook (header words 0..255)
    const uint32_t *M;
    const uint16_t *S;
    const uint32_t *D;
    const uint16_t *c16;
    const int16_t *prm, *pinv;
    // owned device arrays
    float *ic;   // sgn/c per column, float division on the host as vrc_init (CP:264)
    int *cp;     // clamp-delta CSR by ORIGINAL row (rows + 1), entries in slot order within a row (CP:266-273)
    uint16_t *cc;
    float *cv;
    float2 *rsc;  // per sorted row {2^sigma, 2^-sigma}: power-of-two weight scale that keeps the GEMM's fp16 operand in range
    // host copies
    uint32_t cs;              // coset word
    uint32_t class_mask;      // bit c set if some tile has class c
    int uniform_class;        // c if every tile has class c and tile i's payload starts at word i * 64 NW(c), else 0
    uint64_t hist[8];
    uint32_t delta_blocks[4]; // bit b: some clamp-delta entry lies in original rows [256 b, 256 b + 256)
    uint64_t act_hash;        // FNV-1a of (sgn/c per column, codebook, coset): tensors with equal hashes share a prepared x
    std::vector<uint32_t> A_host;
};

constexpr uint32_t kTensorMagic = 0x50385454u;

namespace p8 {
// host-side validation of a slot image (used by p8_prepare on the device-side reads, and by p8_slot_check)
struct SlotView {
    const uint8_t *hdr;       // >= 2064 bytes
    const uint32_t *M;        // nt words
    const Trailer *tr;
    const int8_t *sg;         // 256
    const int16_t *prm, *pinv;
    const uint16_t *drow, *dcol;
    const uint16_t *c16;
    size_t n;
};
p8_status validate_slot(const SlotView &v, int64_t K, int64_t rows, size_t *kbytes_out, uint32_t *class_mask,
                        uint64_t *hist);
p8_status check_shape(int64_t K, int64_t rows);

// launchers (p8_kernels.cu)
cudaError_t launch_decode_int(const p8_tensor *t, int16_t *out, cudaStream_t st);
cudaError_t launch_dequant(const p8_tensor *t, float *out, cudaStream_t st);
cudaError_t launch_get_rows(const p8_tensor *t, const int32_t *ids, int64_t n, float *out, int64_t ldo, cudaStream_t st);
size_t gemv_workspace(const p8_tensor *t, int64_t ncols);
size_t gemv_group_workspace(const p8_tensor *const *ts, int nt, int64_t ncols);
p8_status launch_gemv_group(const p8_tensor *const *ts, int nt, const float *X, int64_t ncols, int64_t ldx, float *const *Ys,
                            const int64_t *ldys, void *ws, size_t ws_bytes, cudaStream_t st);
p8_status launch_gemv(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, float *Y, int64_t ldy, void *ws,
                      size_t ws_bytes, cudaStream_t st);
p8_status launch_gemv_group_pro(const p8_tensor *const *ts, int nt, const float *x, const p8_prologue *pro, float *const *Ys,
                                void *ws, size_t ws_bytes, cudaStream_t st);
p8_status launch_gemv_cols(const p8_tensor *const *ts, int nt, const float *X, int64_t ncols, int64_t ldx, const p8_prologue *pro,
                           float *const *Ys, const int64_t *ldys, void *ws, size_t ws_bytes, cudaStream_t st);
// Fused row-parallel exchange of the GEMV's row reduce (one-shot all-reduce over peer memory). Every rank owns an
// exchange buffer of u64 entries: entry (parity s, source rank q, output row ro) at index (s * world + q) * cap + ro
// holds (tag << 32) | float bits of rank q's partial y[ro], 0 when empty; tag = 0x80000000 | ro << 16 | rows / 32.
// The reduce kernel's threads take consecutive output rows, so a warp's 32 entries are one coalesced write per peer;
// the row count in the tag checks that the ranks run the same tensor. A rank stores its partials into every peer's buffer
// (plain 8-byte stores over NVLink), then polls its own buffer for the peers' partials (bounded by timeout_ns), sums
// the ranks' values in rank order and clears the entries it consumed. The parity s = epoch & 1 alternates per call, so
// a rank one call ahead writes the other half while a slow peer still reads this one.
constexpr int kTpMaxWorld = 8;
struct TpExchange {
    unsigned long long *peer[kTpMaxWorld];  // each rank's exchange buffer as mapped here (peer[rank] = own)
    const unsigned int *epoch;              // this rank's call counter, advanced by the call's k_gemv
    long long cap;                          // output rows per (parity, rank) section
    unsigned long long timeout_ns;
    unsigned int tag_rows;                  // rows / 32 (tag bits 0-15); an entry with another non-zero tag is a mismatch
    int rank, world;
};
p8_status launch_gemv_tp(const p8_tensor *t, const float *x, float *y, const TpExchange &tp, unsigned int *epoch, void *ws,
                         size_t ws_bytes, cudaStream_t st);

size_t gemm_workspace(const p8_tensor *t, int64_t ncols, bool pro = false);
p8_status launch_gemm(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, float *Y, int64_t ldy, void *ws,
                      size_t ws_bytes, cudaStream_t st, const p8_prologue *pro = nullptr);
bool gemm_supported(const p8_tensor *t, int64_t ncols);
size_t gemm_group_workspace(const p8_tensor *const *ts, int n, int64_t ncols, bool pro = false);
p8_status launch_gemm_group(const p8_tensor *const *ts, int n, const float *X, int64_t ncols, int64_t ldx, float *const *Ys,
                            const int64_t *ldys, void *ws, size_t ws_bytes, cudaStream_t st, const p8_prologue *pro = nullptr);
p8_status gemm_prepare(p8_tensor *t, cudaStream_t st);  // prepare-time per-row scales (rsc)

// chained batch-1 GEMVs (p8_chain.cuh)
p8_status chain_create(const p8_chain_step *steps, int n, p8_chain **out);
p8_status chain_destroy(p8_chain *c);
size_t chain_workspace(const p8_chain *c);
p8_status chain_run(const p8_chain *c, void *ws, size_t ws_bytes, cudaStream_t st, int pf);
p8_status chain_trace(p8_chain *c, unsigned long long *buf, size_t words);
}  // namespace p8
