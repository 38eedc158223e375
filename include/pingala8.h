/*
 * pingala8.h -- C ABI of the B200 (sm_100a) Pingala-8 quantized-weight matmul path.
 *
 * Drop-in boundary for the reference's ggml hooks (Genrius-AI/pingala8-llm, patches/llama_cuda_vs_7ac59a6.patch = CU,
 * patches/llama_cpu_vs_7ac59a6.patch = CP). Plain pointers, sizes and status codes; no ggml or torch types.
 * The reference aborts (GGML_ABORT / GGML_ASSERT) or throws std::runtime_error where these functions return a status.
 *
 * Tensor memory ("slot") is the reference's in-memory contract byte for byte (ggml-vr-native.h, CU:1-51): kernel bytes
 * (A | B | c, NS, TRL | M | S | D), then, top-down from the end, clamp delta E, c16, prm, pinv, Hadamard signs and a
 * 32-byte trailer "VVRN" "RI51". Logical shape [K, rows] (ggml ne0 = K, ne1 = rows).
 *
 * Every compute entry point enqueues on the given stream, does not synchronise and allocates nothing: scratch comes
 * from the caller (p8_workspace_size), as ggml's pool allocations do, so calls are capturable into CUDA graphs.
 * p8_prepare is the one-time set-up (device->host reads, small device allocations) and must run before capture,
 * as ggml_cuda_f44_prepare_graph does (CU:1351).
 */
#ifndef PINGALA8_H
#define PINGALA8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum p8_status {
    P8_OK = 0,
    P8_ERR_ARG = -1,        /* null pointer, bad shape or size argument */
    P8_ERR_TRAILER = -2,    /* trailer magic / rows / K / NS mismatch (reference: "bad trailer/header", CU:3058-3061) */
    P8_ERR_HEADER = -3,     /* header NS != 108 or TRL != 2 (CU:3547) */
    P8_ERR_PAYLOAD = -4,    /* kernel bytes != size implied by the M words, or a tile outside the payload (CU:3553-3556) */
    P8_ERR_PERM = -5,       /* prm is not a permutation / pinv inconsistent (CU:3563-3568) */
    P8_ERR_DELTA = -6,      /* clamp-delta index out of range (CU:3573) */
    P8_ERR_SIGNS = -7,      /* Hadamard signs not +-1 (CU:3576) */
    P8_ERR_TABLES = -8,     /* A + c leaves int8 range (the coset add must not wrap) */
    P8_ERR_SHAPE = -9,      /* K % 256, rows % 32, rows >= 32768 (CU:3481) */
    P8_ERR_CUDA = -10,      /* a CUDA runtime call failed */
    P8_ERR_WORKSPACE = -11, /* workspace missing or too small */
    P8_ERR_NOT_PREPARED = -12, /* tensor handle unknown / released (reference: GGML_ABORT, CU:3172) */
    P8_ERR_UNSUPPORTED = -13,  /* valid request this build does not serve */
    P8_ERR_TIMEOUT = -14,   /* a bounded device-side wait gave up (kernel returned early, results invalid) */
    P8_ERR_SLOT = -15,      /* no slot type is large enough (loader: "no slot type fits", CU:3498) */
    P8_ERR_FILE = -16,      /* model file: I/O error, not a GGUF file (v2/v3), or a malformed container */
    P8_ERR_MODEL = -17,     /* model file: Pingala-8 keys or tensors missing or inconsistent (vr_native_init) */
    P8_ERR_NOALLOC_SCRATCH = -18 /* p8_mul_mat_vec_noalloc: the library's fixed scratch array could not be placed on
                                    this device (its module is loaded, and the array allocated, at the first call) */
} p8_status;

typedef struct p8_tensor p8_tensor;

/* ---------------------------------------------------------------- tensor life cycle ----------------------------- */

/* Validate a slot resident in device memory and build its device-side aux data (sgn/c per column, CSR clamp delta).
 * Replaces vr_native_probe + vr_prepare_native (CU:666-676, CU:3046-3101), i.e. ggml_cuda_f44_prepare_graph
 * (CU:678-715) for one tensor. Reads the header, M, side data and trailer to the host (synchronises `stream`). */
p8_status p8_prepare(const void *dev_slot, size_t nbytes, int64_t K, int64_t rows, void *stream, p8_tensor **out);

/* Release a prepared tensor (the reference never frees its CSR arrays, CU:3094-3098). */
p8_status p8_release(p8_tensor *t);

/* 1 if dev_slot was prepared and not released, else 0. Replaces ggml_cuda_f44_active (CU:223-232). */
int p8_active(const void *dev_slot);

/* Shape and stats of a prepared tensor: rows, K, nd (delta entries), class histogram (8 entries, may be NULL). */
p8_status p8_tensor_info(const p8_tensor *t, int64_t *rows, int64_t *K, int64_t *nd, uint64_t *class_hist);

/* ---------------------------------------------------------------- compute -------------------------------------- */

/* Scratch bytes needed by p8_mul_mat_vec / p8_mul_mat for `ncols` activation columns (ggml pool allocations in the
 * reference, CU:3182-3184; CPU: ggml_vr_cpu_wsize, CP:1080-1088). */
size_t p8_workspace_size(const p8_tensor *t, int64_t ncols);

/* y[rows] = W x, x f32[K] (16-byte aligned). Batch-1 decode GEMV. Replaces ggml_cuda_f44_mul_mat_vec (CU:277) ->
 * vr_mul_mat_vec (CU:3177-3232). Activations x16 (14-bit per 128-column half-slice, the reference CPU default),
 * deterministic (no float atomics). */
p8_status p8_mul_mat_vec(const p8_tensor *t, const float *x, float *y, void *workspace, size_t workspace_bytes, void *stream);

/* Several tensors that read the same x (q/k/v, gate/up): y_i = W_i x for i < n (n <= 4), one prepared activation and
 * one launch. The tensors need equal K, column scales c, signs and codebook (else P8_ERR_ARG). The reference prepares
 * x once for consecutive tensors with the same input and c (vrc_tg activation cache, CP:1171-1180); ggml itself has no
 * grouped op, so this entry point is an extension. */
size_t p8_workspace_size_group(const p8_tensor *const *ts, int n, int64_t ncols);
p8_status p8_mul_mat_vec_group(const p8_tensor *const *ts, int n, const float *x, float *const *ys, void *workspace,
                               size_t workspace_bytes, void *stream);

/* Activation prologue fused into the GEMV's activation prep, for the op that produces a projection's input in a
 * llama-style layer (each a separate ggml op, and kernel, in the reference):
 *   P8_PROLOGUE_RMSNORM  x' = (x * scale) * w, scale = 1 / sqrt(sum(x^2) / K + eps)   (ggml rms_norm, then mul by the
 *                        norm weight w[K]; the q/k/v and gate/up inputs)
 *   P8_PROLOGUE_SWIGLU   x' = x / (1 + exp(-x)) * x2                                    (ggml swiglu: silu(gate) * up
 *                        with x = gate, x2 = up[K]; the down projection's input)
 * x' is computed in fp32 and is what the GEMV multiplies (clamp-delta term included); it is not written back. The
 * stock llama.cpp fuses the GLU into its own quantized GEMV (ggml_cuda_should_fuse_mul_mat_vec_q); the reference turns
 * that off for Pingala-8 tensors (CU:1319-1321). */
typedef enum p8_prologue_kind { P8_PROLOGUE_NONE = 0, P8_PROLOGUE_RMSNORM = 1, P8_PROLOGUE_SWIGLU = 2 } p8_prologue_kind;
typedef struct p8_prologue {
    int kind;          /* p8_prologue_kind */
    const float *w;    /* RMSNORM: norm weight [K] (16-byte aligned) */
    const float *x2;   /* SWIGLU: up [K] (16-byte aligned) */
    float eps;         /* RMSNORM */
} p8_prologue;
/* p8_mul_mat_vec_group with a prologue (pro NULL or kind NONE: the plain call); workspace as p8_workspace_size_group */
p8_status p8_mul_mat_vec_group_ex(const p8_tensor *const *ts, int n, const float *x, const p8_prologue *pro, float *const *ys,
                                  void *workspace, size_t workspace_bytes, void *stream);
/* p8_mul_mat (prefill / batched) with a prologue applied to every token: RMSNORM per token (its own sum of squares)
 * with the shared weight w[K]; SWIGLU with up rows at pro->x2 + n * ldx. Workspace p8_workspace_size_ex(t, ncols, kind)
 * (the tcgen05 path keeps x' [ncols][K] f32 for the clamp-delta term). */
size_t p8_workspace_size_ex(const p8_tensor *t, int64_t ncols, int kind);
p8_status p8_mul_mat_ex(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, const p8_prologue *pro, float *Y,
                        int64_t ldy, void *workspace, size_t workspace_bytes, void *stream);

/* p8_mul_mat_ex for several tensors that read the same X (q/k/v, gate/up; n <= 4, requirements as
 * p8_mul_mat_vec_group, else P8_ERR_ARG): the activation prep, prologue included, runs once and each tensor's product
 * reads it; Y_i [ncols][ldys[i]]. Two consecutive tensors of one shape (gate/up) may share one GEMM launch when
 * their row tiles fill the SMs' waves better together. Results are bit-identical to separate p8_mul_mat_ex calls,
 * except the rows of a shared launch's last, K-split row tiles (same products, fp32 sums in another order). The reference's
 * activation cache (vrc_tg, CP:1171-1180) reuses a prepared x across consecutive tensors the same way; ggml has no
 * grouped op, so this entry point is an extension. Workspace p8_workspace_size_group_ex(ts, n, ncols, kind). */
size_t p8_workspace_size_group_ex(const p8_tensor *const *ts, int n, int64_t ncols, int kind);
p8_status p8_mul_mat_group(const p8_tensor *const *ts, int n, const float *X, int64_t ncols, int64_t ldx, const p8_prologue *pro,
                           float *const *Ys, const int64_t *ldys, void *workspace, size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------- chained batch-1 GEMVs -------------------------- */

/* A decode step evaluates a fixed run of MUL_MAT nodes, each reading an earlier one's output, with RMS_NORM + MUL,
 * SWIGLU and ADD nodes between them (ggml_backend_cuda_graph_compute walking the graph, each MUL_MAT through
 * ggml_cuda_mul_mat, CU:1330-1342). A chain runs such a run of batch-1 Pingala-8 products with ONE GEMV launch per
 * product (plus one row reduce after the last), instead of a GEMV and a row reduce per product: a step whose input is
 * an output of the previous step reads it straight from that step's partial sums while it builds its tables; an
 * extension, the reference launches every op separately. Step s computes, for its n tensors (equal K and column
 * tables, as p8_mul_mat_vec_group):
 *     y_i = W_i x' (+ res_i),  x' = pro(x)
 * pro as p8_prologue (NONE, RMSNORM with w and eps, SWIGLU with x2 = up). x (and x2) may be any device buffer of K
 * floats, or exactly an output y_j of the previous step (then the chain reads it straight from that step's partial
 * sums); any other overlap with the previous step's outputs is refused. An earlier step's output (two or more steps
 * back) may be read as x, x2 or res. res_i must not overlap y_i. Results equal the separate calls up to float
 * rounding where a step's RMSNorm input comes from the previous step (the scale then multiplies the product instead
 * of its input; the integer table sums are exact), and bit for bit elsewhere.
 * A plan holds the launch arguments of every step (buffers are fixed at creation, like a captured graph):
 * p8_chain_create is set-up time; p8_chain_run only enqueues the launches on the stream and is capturable; runs of
 * one plan must not overlap on the GPU. Workspace: p8_chain_workspace_size bytes, 256-byte aligned. */
typedef struct p8_chain_step {
    int n;                   /* tensors reading the same input, 1..4 */
    const p8_tensor *t[4];
    const float *x;          /* input [K] (16-byte aligned) */
    p8_prologue pro;         /* kind 0: none */
    float *y[4];             /* outputs [rows_i] */
    const float *res[4];     /* optional residual [rows_i] added to y_i (NULL: none) */
} p8_chain_step;
typedef struct p8_chain p8_chain;
p8_status p8_chain_create(const p8_chain_step *steps, int nsteps, p8_chain **out);
size_t p8_chain_workspace_size(const p8_chain *c);
p8_status p8_chain_run(const p8_chain *c, void *workspace, size_t workspace_bytes, void *stream);
p8_status p8_chain_destroy(p8_chain *c);
/* Profiling aid: record, in later runs, per step (after the first) and CTA, globaltimer stamps (ns) into the device
 * buffer dev_buf (nsteps x CTAs x 8 words, CTAs = the device's SM count; [0] after the wait for the previous launch,
 * [1] and [2] input values ready, [3] tables built, [4] units done, [5] the previous step's unread rows reduced).
 * NULL turns it off. */
p8_status p8_chain_trace(p8_chain *c, uint64_t *dev_buf, size_t words);

/* y = W x like p8_mul_mat_vec, but with no workspace argument and no allocation by this library: the scratch is a
 * fixed 6 MiB device array inside the library, for callers that cannot allocate device memory at call time and have
 * no buffer to lend (e.g. a host framework that plans all device memory up front). No counterpart in the reference.
 * Limit: tensors with p8_workspace_size(t, 1) <= p8_noalloc_scratch_bytes() (else P8_ERR_WORKSPACE).
 * The array is placed on a device when the library's module is loaded there, which under CUDA's default lazy loading
 * is the first call on that device: that call makes the 6 MiB device allocation, can fail like one
 * (P8_ERR_NOALLOC_SCRATCH) and must not be inside a stream capture, so make one call per device during set-up. From
 * then on the GPU holds the array until the process exits. Calls share it, so calls that can overlap on the GPU race
 * and must be serialised by the caller. */
size_t p8_noalloc_scratch_bytes(void);
p8_status p8_mul_mat_vec_noalloc(const p8_tensor *t, const float *x, float *y, void *stream);

/* Y[n][ldy] (rows per column) = W X[n][ldx], n < ncols. ncols > 1: batched decode / prefill. Replaces
 * ggml_cuda_f44_mul_mat_q8 (CU:1014-1054). From 4 columns (6 for a tensor whose tiles are all class 3) the
 * tensor-core product runs (fp16 operands, fp32 accumulate, within 1e-3 of the exact product); below that the
 * batch-1 GEMV, two columns per launch for class-3 tensors (the weights decoded once per pair; each column equal to
 * the one-column call bit for bit). Deterministic. Calls on the same workspace must not overlap on the GPU. */
p8_status p8_mul_mat(const p8_tensor *t, const float *X, int64_t ncols, int64_t ldx, float *Y, int64_t ldy,
                     void *workspace, size_t workspace_bytes, void *stream);

/* out[i][ldo] = row ids[i] (ORIGINAL row index) of W in f32, bit-identical to vrc_dequant_f32 (CP:1012-1027).
 * The get_rows / embedding lookup entry. */
p8_status p8_get_rows(const p8_tensor *t, const int32_t *ids, int64_t n, float *out, int64_t ldo, void *stream);

/* W (rows x K, row-major by ORIGINAL row) in f32, bit-identical to vrc_dequant_f32 (CP:1012-1027); ggml to_fp32. */
p8_status p8_dequant_f32(const p8_tensor *t, float *out, void *stream);

/* Exact integer weights (sorted rows x K, natural columns) = vrc_decode_tile_int (CP:992-1010) over all tiles. */
p8_status p8_decode_int(const p8_tensor *t, int16_t *out, void *stream);

/* ---------------------------------------------------------------- host format helpers ---------------------------- */

/* vrn_need (CU:27-29): bytes a slot needs for the given kernel bytes, shape and delta count. */
size_t p8_slot_need(size_t kbytes, size_t rows, size_t K, size_t nd);

/* vrn_offsets (CU:30-37): offE, offC, offP, offQ, offSG, offT of a slot of n bytes (out6 = 6 entries). */
void p8_slot_offsets(size_t n, size_t rows, size_t K, size_t nd, size_t *out6);

/* vrn_kbytes(rows, K, vrn_payload_words(M)) (CU:41-51). */
size_t p8_kbytes_from_m(size_t rows, size_t K, const uint32_t *M);

/* Slot size the loader picks: smallest of IQ2_XXS, Q2_K..Q6_K holding `need` bytes (CU:3493-3497). 0 if none. */
size_t p8_slot_nbytes(size_t rows, size_t K, size_t need, int *slot_type_index);

/* Assemble a slot in host memory from kernel bytes and side tensors, as vr_native_load does (CU:3527-3580):
 * c16 fp16[K], prm int16[rows] (NULL = identity, VR3), delta rows/cols u16[nd] + vals f32[nd], signs int8[256].
 * `out` must hold p8_slot_nbytes(...) bytes; *out_n receives that size. All the loader's checks apply. */
p8_status p8_slot_assemble(const uint8_t *kbytes, size_t kb_n, int64_t rows, int64_t K, const uint16_t *c16,
                           const int16_t *prm, const uint16_t *drow, const uint16_t *dcol, const float *dval, int64_t nd,
                           const int8_t *signs, uint8_t *out, size_t out_cap, size_t *out_n);

/* Validate a slot held in HOST memory (every check p8_prepare does). */
p8_status p8_slot_check(const uint8_t *slot, size_t nbytes, int64_t K, int64_t rows);

/* VR3 file layout (llama-vr3.h, CU:3621-3661): rows of a VR3 tensor from its file size, K and header word 515
 * (0 if inconsistent; *kbytes = expanded v2 kernel bytes), and the expansion to the v2 in-memory bytes. */
size_t p8_vr3_rows(size_t fbytes, size_t K, uint32_t w515, size_t *kbytes);
p8_status p8_vr3_expand(const uint8_t *f, size_t fbytes, size_t rows, size_t K, uint8_t *dst, size_t dst_cap);

/* ---------------------------------------------------------------- tensor parallel (no reference counterpart) ---- */

/* Column-parallel shard (q/k/v/gate/up): the ORIGINAL output rows [r0, r1) (r1 - r0 a multiple of 32) as a standalone
 * slot. The selected rows keep their sorted order and are re-tiled (a row moved to another lane of a tile has its steps
 * rotated, since step k holds chunk (lane + k) & 31); the shard's prm maps to original row - r0. Needs one class per
 * new tile-block (always true for single-class tensors), else P8_ERR_UNSUPPORTED. orig_rows (optional, r1 - r0
 * entries) receives the original row of each shard row. Host memory in and out. */
p8_status p8_tp_shard_rows(const uint8_t *slot, size_t nbytes, int64_t K, int64_t rows, int64_t r0, int64_t r1,
                           uint8_t *out, size_t out_cap, size_t *out_n, int32_t *orig_rows /* [r1-r0] or NULL */);

/* Row-parallel shard (o/down): the slot of 256-column blocks [b0, b1) (columns [256 b0, 256 b1)) as a standalone
 * slot; every rank keeps all rows, partial outputs are summed by an all-reduce. */
p8_status p8_tp_shard_cols(const uint8_t *slot, size_t nbytes, int64_t K, int64_t rows, int64_t b0, int64_t b1,
                           uint8_t *out, size_t out_cap, size_t *out_n);

/* Fused row-parallel product: y = sum over ranks of (rank's column shard) x (rank's slice of x), computed by one GEMV
 * launch per rank whose epilogue exchanges the partial rows over peer memory (NVLink stores, no collective library):
 * each rank stores its partial y into every peer's exchange buffer, polls its own buffer for the peers' partials and
 * sums the ranks' values in rank order, so every rank gets the same bits. A wait is bounded by the communicator's
 * timeout; past it the launch gives up, p8_device_error reports bit 3 (8), the result is invalid and every rank must
 * p8_tp_comm_reset its communicator (between steps, then a host barrier) before the next call. An entry whose tag
 * names another row count or another original row (the ranks called different tensors, or shards whose row order
 * differs) sets bit 4 (16).
 *
 * Exchange buffer of rank r: 2 * world * max_rows u64 entries; entry (parity s, source rank q, output row ro) at index
 * (s * world + q) * max_rows + ro holds (tag << 32) | float bits of rank q's partial y[ro], tag = 0x80000000 |
 * ro << 16 | rows / 32; 0 = empty.
 * Parity s = the communicator's call count & 1 (the first call is 1). Peers' buffers must have the same world and
 * max_rows. All ranks make the same sequence of p8_tp_gemv_allreduce calls on their communicators, each with its
 * column shard of one tensor (same rows); a rank with no columns cannot take part (use a collective instead).
 * The exchange runs in the call's row-reduce kernel, whose CTAs (at most one per SM) wait for their peers: while a
 * fused call may be in flight, run no other kernel on the GPU that waits for other ranks (an NCCL collective on another
 * stream): its CTAs can keep a reduce CTA from becoming resident while the peers' wait for this rank. Synchronise the
 * device before such a collective. */
typedef struct p8_tp_comm p8_tp_comm;
#define P8_IPC_HANDLE_BYTES 64
/* rank of world (1..8) on the current device, up to max_rows output rows per call, waits bounded by timeout_ms */
p8_status p8_tp_comm_create(int rank, int world, int64_t max_rows, uint32_t timeout_ms, p8_tp_comm **out);
p8_status p8_tp_comm_destroy(p8_tp_comm *c);
/* CUDA IPC handle (P8_IPC_HANDLE_BYTES) of this rank's exchange buffer, for the other processes' p8_tp_comm_open_peer */
p8_status p8_tp_comm_ipc_handle(const p8_tp_comm *c, void *handle, size_t handle_bytes);
/* map peer q's exchange buffer from its IPC handle (one process per GPU) */
p8_status p8_tp_comm_open_peer(p8_tp_comm *c, int q, const void *handle, size_t handle_bytes);
/* or attach it by device pointer (one process driving several GPUs, peer access enabled by the caller) */
p8_status p8_tp_comm_set_peer(p8_tp_comm *c, int q, void *dev_buffer);
p8_status p8_tp_comm_buffer(const p8_tp_comm *c, void **dev_buffer, size_t *nbytes);
/* calls made so far (synchronous device read) */
p8_status p8_tp_comm_epoch(const p8_tp_comm *c, uint32_t *epoch);
/* zero the exchange buffer and the call count (enqueued on stream) */
p8_status p8_tp_comm_reset(p8_tp_comm *c, void *stream);
/* the fused call: t = this rank's column shard (p8_tp_shard_cols), x its input slice, y [rows]; workspace as
 * p8_workspace_size(t, 1). Enqueues on stream, capturable into a CUDA graph (the call count lives on the device). */
p8_status p8_tp_gemv_allreduce(const p8_tensor *t, const float *x, float *y, p8_tp_comm *c, void *workspace,
                               size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------- offline encoder ------------------------------- */

/* One 128-column slice of the trellis encoder (the reference's LDLQ Viterbi, research/detail/r48k.py encode / vit_k /
 * best_cw / zero_ldlq, r48k.py:33-120, trellis mode with 8 states) for all rows, on the GPU. Device pointers unless
 * noted; row r of each array at base + r * ld:
 *   X    [rows][128] f32   the slice of the FWHT-domain weights after the earlier slices' error feedback
 *   Hb   [128][128]  f32   the slice's diagonal block of the upper Cholesky factor Uc (Hi = Uc^T Uc)
 *   A4   [32][4][4]  f32   inverses of Hb's diagonal 4 x 4 blocks (row-major)
 *   codebook [256][4] i8   the codebook A (header bytes 0..1023); coset: 4 i8 in HOST memory
 *   cls  u8 per row (stride ldc), S f32 per row (stride lds): the class and scale of the row's 256-column block
 *   Q    [rows][128] f32   out: quantised values (integer codeword x S); E [rows][128] f32 out: the errors in the
 *        A4-transformed metric (the caller subtracts E @ Uc[slice, later columns] from the later columns)
 *   IDX  [rows][32][3] u8  out: (f1, f2, f3) per 4-weight step (rows of class 0 are not written)
 * workspace: p8_encode_workspace() bytes (16-byte aligned). Rows are independent and the result is deterministic;
 * codes equal the reference's except where two candidates' metrics differ only in their last bits. */
size_t p8_encode_workspace(void);
p8_status p8_encode_slice(const float *X, int64_t ldx, const float *Hb, int64_t ldh, const float *A4, const int8_t *codebook,
                          const int8_t *coset, const uint8_t *cls, int64_t ldc, const float *S, int64_t lds, int64_t rows, float *Q,
                          int64_t ldq, float *E, int64_t lde, uint8_t *IDX, int64_t ldi, void *workspace, size_t workspace_bytes,
                          void *stream);

/* ---------------------------------------------------------------- model files (GGUF) ---------------------------- */

/* A GGUF file holding a Pingala-8 ("VR native") model, opened and checked as llama_model_loader::vr_native_init does
 * (CU:3411-3508): KV vr.format, vr.ns = 108, vr.trl = 2, vr.n_linear (= 7 x <arch>.block_count when present),
 * vr.layout 2 (kernel bytes + vr_prm) or 3 (VR3 file tensors, natural rows); per linear <base>.weight (I8),
 * <base>.vr_c (F16 [K]), <base>.vr_prm (I16 [rows], layout 2), optional <base>.vr_didx (I16 [nd, 2]) and
 * <base>.vr_dval (F32 [nd]); vr.had_signs (I8 [256]). Host memory only; one handle is not safe for concurrent use. */
typedef struct p8_gguf p8_gguf;
p8_status p8_gguf_open(const char *path, p8_gguf **out);
void p8_gguf_close(p8_gguf *g);
/* linears in name order */
int64_t p8_gguf_n_linear(const p8_gguf *g);
p8_status p8_gguf_linear_info(const p8_gguf *g, int64_t i, const char **name, int64_t *K, int64_t *rows, int64_t *nd,
                              size_t *slot_nbytes, int *layout);
/* Linear i as the slot the reference builds in device memory (vr_native_load, CU:3527-3580): kernel bytes (VR3
 * expanded), c16, permutation (identity for VR3) and its inverse, clamp delta, signs and trailer, assembled in `out`
 * (slot_nbytes bytes) with every loader check; every linear must carry the first one's codebook and coset. Upload
 * the bytes and p8_prepare them. */
p8_status p8_gguf_load_linear(p8_gguf *g, int64_t i, uint8_t *out, size_t out_cap, size_t *out_n);

/* Non-zero if a kernel since the last call gave up (that launch's results are invalid), then clears the word. Bits:
 * 4 GEMM pipeline wait timed out, 8 row-parallel exchange wait timed out, 16 exchange entry with a foreign tag (1, 2
 * and 32 are unused). Synchronises the device. */
int p8_device_error(void);

const char *p8_status_str(p8_status s);
const char *p8_build_info(void);

#ifdef __cplusplus
}
#endif
#endif /* PINGALA8_H */
