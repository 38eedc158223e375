// p8_host.cpp -- host-side format library: validation, slot assembly, VR3 expansion, tensor-parallel shards.
//
// The checks are the reference loader's and CUDA prepare's (llama-model-loader.cpp vr_native_init / vr_native_load,
// CU:3411-3580; vr49.cuh vr_prepare_native, CU:3046-3101), returned as status codes instead of throw / GGML_ABORT,
// plus bounds checks the kernels rely on (every tile's payload lies inside D; the coset add never wraps int8).
#include <string.h>

#include <algorithm>
#include <vector>

#include "p8_internal.h"

using namespace p8;

namespace p8 {

p8_status check_shape(int64_t K, int64_t rows) {
    if (K <= 0 || rows <= 0 || K % 256 || rows % 32 || rows > kMaxRows || K > 65535) return P8_ERR_SHAPE;
    return P8_OK;
}

p8_status validate_slot(const SlotView &v, int64_t K, int64_t rows, size_t *kbytes_out, uint32_t *class_mask,
                        uint64_t *hist) {
    p8_status st = check_shape(K, rows);
    if (st) return st;
    const size_t nb = (size_t)K / 256, ng = (size_t)rows / 32, nt = ng * nb;
    if (v.n < 4096 || v.n < offD(nt)) return P8_ERR_TRAILER;  // vrc_probe: n >= 4096 (CP:227)
    const Trailer &tr = *v.tr;
    if (tr.magic0 != kMagic0 || tr.magic1 != kMagic1 || tr.rows != (uint32_t)rows || tr.K != (uint32_t)K || tr.ns != kNS)
        return P8_ERR_TRAILER;
    uint32_t hw[3];
    memcpy(hw, v.hdr + 2052, 12);
    if (hw[0] != kNS || hw[1] != kTRL) return P8_ERR_HEADER;
    // payload size implied by the M words == trailer kbytes, inside the slot below the side data (CU:3553-3556, CU:3072)
    size_t words = 0;
    uint32_t cm = 0;
    uint64_t hh[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t i = 0; i < nt; ++i) {
        const int c = (int)(v.M[i] >> 29);
        words += (size_t)64 * NW(c);
        cm |= 1u << c;
        hh[c]++;
    }
    const size_t kb = offD(nt) + 4 * words;
    if (kb != tr.kbytes) return P8_ERR_PAYLOAD;
    if (tr.nd > (uint32_t)v.n) return P8_ERR_DELTA;
    const SideOffsets so = side_offsets(v.n, (size_t)rows, (size_t)K, tr.nd);
    if (so.E > v.n || kb > so.E) return P8_ERR_PAYLOAD;
    // every tile's payload [off, off + 64 NW) inside the payload words (kernels read D at these offsets)
    for (size_t i = 0; i < nt; ++i) {
        const int c = (int)(v.M[i] >> 29);
        if (!c) continue;
        const size_t off = v.M[i] & 0x1FFFFFFFu;
        if (off + (size_t)64 * NW(c) > words) return P8_ERR_PAYLOAD;
        if (off % 4) return P8_ERR_PAYLOAD;  // tiles start on 16 bytes (the writer packs 64 NW-word tiles back to back)
    }
    // prm a permutation, pinv its inverse (CU:3563-3568)
    std::vector<uint8_t> seen((size_t)rows, 0);
    for (int64_t r = 0; r < rows; ++r) {
        const int p = v.prm[r];
        if (p < 0 || p >= rows || seen[(size_t)p]++) return P8_ERR_PERM;
    }
    for (int64_t r = 0; r < rows; ++r)
        if (v.pinv[v.prm[r]] != (int16_t)r) return P8_ERR_PERM;
    for (uint32_t e = 0; e < tr.nd; ++e)
        if (v.drow[e] >= rows || v.dcol[e] >= K) return P8_ERR_DELTA;  // CU:3573
    for (int i = 0; i < 256; ++i)
        if (v.sg[i] != 1 && v.sg[i] != -1) return P8_ERR_SIGNS;  // CU:3576
    // the coset add A[f] + c must stay inside int8 (the GEMV's table split relies on it; the shipped tables do)
    uint32_t A[256], cs;
    memcpy(A, v.hdr, 1024);
    memcpy(&cs, v.hdr + 2048, 4);
    for (int f = 0; f < 256; ++f)
        for (int e = 0; e < 4; ++e) {
            const int s = (int)(int8_t)(A[f] >> (8 * e)) + (int)(int8_t)(cs >> (8 * e));
            if (s < -128 || s > 127) return P8_ERR_TABLES;
        }
    for (size_t k = 0; k < (size_t)K; ++k) {  // c16 finite and non-zero (sgn / c is taken per column)
        const uint16_t h = v.c16[k];
        if ((h & 0x7fffu) == 0 || (h & 0x7c00u) == 0x7c00u) return P8_ERR_ARG;
    }
    if (kbytes_out) *kbytes_out = kb;
    if (class_mask) *class_mask = cm;
    if (hist) memcpy(hist, hh, sizeof(hh));
    return P8_OK;
}

}  // namespace p8

static const int kSlotBPB[6] = {66, 84, 110, 144, 176, 210};  // IQ2_XXS, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K bytes per 256

extern "C" {

size_t p8_slot_need(size_t kbytes, size_t rows, size_t K, size_t nd) { return slot_need(kbytes, rows, K, nd); }

void p8_slot_offsets(size_t n, size_t rows, size_t K, size_t nd, size_t *out6) {
    if (!out6) return;
    const SideOffsets o = side_offsets(n, rows, K, nd);
    out6[0] = o.E; out6[1] = o.C; out6[2] = o.P; out6[3] = o.Q; out6[4] = o.SG; out6[5] = o.T;
}

size_t p8_kbytes_from_m(size_t rows, size_t K, const uint32_t *M) {
    const size_t nt = (rows / 32) * (K / 256);
    size_t w = 0;
    for (size_t i = 0; i < nt; ++i) w += (size_t)64 * NW((int)(M[i] >> 29));
    return offD(nt) + 4 * w;
}

size_t p8_slot_nbytes(size_t rows, size_t K, size_t need, int *slot_type_index) {
    for (int i = 0; i < 6; ++i) {
        const size_t n = rows * (K / 256) * (size_t)kSlotBPB[i];
        if (n >= need) {
            if (slot_type_index) *slot_type_index = i;
            return n;
        }
    }
    if (slot_type_index) *slot_type_index = -1;
    return 0;
}

p8_status p8_slot_check(const uint8_t *slot, size_t nbytes, int64_t K, int64_t rows) {
    if (!slot) return P8_ERR_ARG;
    p8_status st = check_shape(K, rows);
    if (st) return st;
    const size_t nt = (size_t)(rows / 32) * (size_t)(K / 256);
    if (nbytes < 4096 || nbytes < offD(nt)) return P8_ERR_TRAILER;
    SlotView v;
    v.n = nbytes;
    v.hdr = slot;
    v.M = (const uint32_t *)(slot + kHdrBytes);
    v.tr = (const Trailer *)(slot + nbytes - 32);
    if (v.tr->nd > nbytes) return P8_ERR_DELTA;
    const SideOffsets so = side_offsets(nbytes, (size_t)rows, (size_t)K, v.tr->nd);
    if (so.E >= nbytes || so.E < offD(nt)) return P8_ERR_PAYLOAD;
    v.sg = (const int8_t *)(slot + so.SG);
    v.prm = (const int16_t *)(slot + so.P);
    v.pinv = (const int16_t *)(slot + so.Q);
    v.drow = (const uint16_t *)(slot + so.E);
    v.dcol = v.drow + v.tr->nd;
    v.c16 = (const uint16_t *)(slot + so.C);
    return validate_slot(v, K, rows, nullptr, nullptr, nullptr);
}

p8_status p8_slot_assemble(const uint8_t *kb, size_t kb_n, int64_t rows, int64_t K, const uint16_t *c16,
                           const int16_t *prm, const uint16_t *drow, const uint16_t *dcol, const float *dval, int64_t nd,
                           const int8_t *signs, uint8_t *out, size_t out_cap, size_t *out_n) {
    if (!kb || !c16 || !signs || !out || nd < 0 || (nd && (!drow || !dcol || !dval))) return P8_ERR_ARG;
    p8_status st = check_shape(K, rows);
    if (st) return st;
    const size_t nt = (size_t)(rows / 32) * (size_t)(K / 256);
    if (kb_n < offD(nt)) return P8_ERR_PAYLOAD;
    uint32_t hw[3];
    memcpy(hw, kb + 2052, 12);
    if (hw[0] != kNS || hw[1] != kTRL) return P8_ERR_HEADER;                                       // CU:3547
    if (p8_kbytes_from_m((size_t)rows, (size_t)K, (const uint32_t *)(kb + kHdrBytes)) != kb_n) return P8_ERR_PAYLOAD;  // CU:3553
    const size_t need = slot_need(kb_n, (size_t)rows, (size_t)K, (size_t)nd);
    const size_t n = p8_slot_nbytes((size_t)rows, (size_t)K, need, nullptr);
    if (!n) return P8_ERR_SLOT;
    if (out_n) *out_n = n;
    if (out_cap < n) return P8_ERR_ARG;
    memset(out, 0, n);
    memcpy(out, kb, kb_n);
    const SideOffsets o = side_offsets(n, (size_t)rows, (size_t)K, (size_t)nd);
    if (kb_n > o.E) return P8_ERR_PAYLOAD;
    memcpy(out + o.C, c16, 2 * (size_t)K);
    int16_t *P = (int16_t *)(out + o.P), *Q = (int16_t *)(out + o.Q);
    std::vector<uint8_t> seen((size_t)rows, 0);
    for (int64_t r = 0; r < rows; ++r) {
        const int16_t p = prm ? prm[r] : (int16_t)r;  // VR3: identity (CU:3562)
        if (p < 0 || p >= rows || seen[(size_t)p]++) return P8_ERR_PERM;
        P[r] = p;
    }
    for (int64_t r = 0; r < rows; ++r) Q[P[r]] = (int16_t)r;
    if (nd) {
        uint16_t *er = (uint16_t *)(out + o.E), *ec = er + nd;
        float *ev = (float *)(out + o.E + 4 * (size_t)nd);
        for (int64_t e = 0; e < nd; ++e) {
            if (drow[e] >= rows || dcol[e] >= K) return P8_ERR_DELTA;
            er[e] = drow[e];
            ec[e] = dcol[e];
            ev[e] = dval[e];
        }
    }
    for (int i = 0; i < 256; ++i) {
        if (signs[i] != 1 && signs[i] != -1) return P8_ERR_SIGNS;
        out[o.SG + i] = (uint8_t)signs[i];
    }
    const Trailer tr = {kMagic0, kMagic1, (uint32_t)kb_n, (uint32_t)nd, (uint32_t)rows, (uint32_t)K, kNS, 1u};
    memcpy(out + o.T, &tr, sizeof(tr));
    return P8_OK;
}

size_t p8_vr3_rows(size_t fbytes, size_t K, uint32_t w515, size_t *kbytes) {
    const uint32_t c = w515 & 7u;
    if ((w515 & 0xFFFFFFF8u) != kVR3Tag || c == 0 || K == 0 || K % 256 || fbytes < kHdrBytes) return 0;
    const size_t tw = (size_t)64 * NW((int)c), per = 64 + 4 * tw, nb = K / 256;
    if ((fbytes - kHdrBytes) % per) return 0;
    const size_t nt = (fbytes - kHdrBytes) / per;
    if (nt == 0 || nt % nb || nt * tw >= ((size_t)1 << 29)) return 0;
    const size_t rows = 32 * (nt / nb);
    if (rows > (size_t)kMaxRows) return 0;
    if (kbytes) *kbytes = offD(nt) + 4 * nt * tw;
    return rows;
}

p8_status p8_vr3_expand(const uint8_t *f, size_t fbytes, size_t rows, size_t K, uint8_t *dst, size_t dst_cap) {
    if (!f || !dst || fbytes < kHdrBytes) return P8_ERR_ARG;
    uint32_t w515;
    memcpy(&w515, f + 2060, 4);
    size_t kb = 0;
    if (p8_vr3_rows(fbytes, K, w515, &kb) != rows || rows == 0) return P8_ERR_ARG;
    if (dst_cap < kb) return P8_ERR_ARG;
    const uint32_t c = w515 & 7u;
    const size_t nt = (rows / 32) * (K / 256), tw = (size_t)64 * NW((int)c), od = offD(nt);
    memcpy(dst, f, 2060);
    memset(dst + 2060, 0, 4);  // a v2 file carries word 515 = 0
    for (size_t i = 0; i < nt; ++i) {
        const uint32_t m = (uint32_t)(i * tw) | (c << 29);
        memcpy(dst + kHdrBytes + 4 * i, &m, 4);
    }
    memcpy(dst + offS(nt), f + kHdrBytes, 64 * nt);
    memset(dst + kHdrBytes + 68 * nt, 0, od - (kHdrBytes + 68 * nt));
    memcpy(dst + od, f + kHdrBytes + 64 * nt, fbytes - kHdrBytes - 64 * nt);
    return P8_OK;
}

// ------------------------------------------------------------------------------------------ tensor-parallel shards
namespace {
struct HostSlot {
    const uint8_t *s;
    size_t n, nt, nb, ng;
    int64_t rows, K;
    const Trailer *tr;
    SideOffsets so;
    const uint32_t *M, *D;
    const uint16_t *S, *c16, *drow, *dcol;
    const float *dval;
    const int16_t *prm;
    const int8_t *sg;
};
p8_status open_host(const uint8_t *slot, size_t n, int64_t K, int64_t rows, HostSlot &h) {
    p8_status st = p8_slot_check(slot, n, K, rows);
    if (st) return st;
    h.s = slot; h.n = n; h.K = K; h.rows = rows;
    h.nb = (size_t)K / 256; h.ng = (size_t)rows / 32; h.nt = h.nb * h.ng;
    h.tr = (const Trailer *)(slot + n - 32);
    h.so = side_offsets(n, (size_t)rows, (size_t)K, h.tr->nd);
    h.M = (const uint32_t *)(slot + kHdrBytes);
    h.S = (const uint16_t *)(slot + offS(h.nt));
    h.D = (const uint32_t *)(slot + offD(h.nt));
    h.c16 = (const uint16_t *)(slot + h.so.C);
    h.drow = (const uint16_t *)(slot + h.so.E);
    h.dcol = h.drow + h.tr->nd;
    h.dval = (const float *)(slot + h.so.E + 4 * (size_t)h.tr->nd);
    h.prm = (const int16_t *)(slot + h.so.P);
    h.sg = (const int8_t *)(slot + h.so.SG);
    return P8_OK;
}

// lane fields of one half-slice in STEP order: stage s, step k -> field; z (stage-1 MSB) handled with stage 0
struct LaneFields {
    uint32_t f[3][32];
};
uint32_t get_bits(const uint32_t *w, int pos, int W) {
    uint32_t v = 0;
    for (int q = 0; q < W; ++q) v |= ((w[(pos + q) >> 5] >> ((pos + q) & 31)) & 1u) << q;
    return v;
}
void put_bits(uint32_t *w, int pos, int W, uint32_t v) {
    for (int q = 0; q < W; ++q) {
        const int p = pos + q;
        w[p >> 5] = (w[p >> 5] & ~(1u << (p & 31))) | (((v >> q) & 1u) << (p & 31));
    }
}
void read_lane(const uint32_t *p0, int c, int hs, int j, LaneFields &lf) {
    const int nw = NW(c), w1 = W1(c), w2 = W2(c), w3 = W3(c);
    uint32_t w[24];
    for (int i = 0; i < nw; ++i) w[i] = p0[(size_t)hs * nw * 32 + (size_t)(i >> 1) * 64 + 2 * j + (i & 1)];
    for (int k = 0; k < 32; ++k) {
        if (w1 == 8) lf.f[0][k] = get_bits(w, 8 * k, 8);
        else lf.f[0][k] = get_bits(w + 1, (w1 - 1) * k, w1 - 1) | (((w[0] >> k) & 1u) << (w1 - 1));
        lf.f[1][k] = w2 ? get_bits(w + w1, w2 * k, w2) : 0;
        lf.f[2][k] = w3 ? get_bits(w + w1 + w2, w3 * k, w3) : 0;
    }
}
void write_lane(uint32_t *p0, int c, int hs, int j, const LaneFields &lf) {
    const int nw = NW(c), w1 = W1(c), w2 = W2(c), w3 = W3(c);
    uint32_t w[24] = {0};
    for (int k = 0; k < 32; ++k) {
        if (w1 == 8) put_bits(w, 8 * k, 8, lf.f[0][k]);
        else {
            put_bits(w + 1, (w1 - 1) * k, w1 - 1, lf.f[0][k] & ((1u << (w1 - 1)) - 1u));
            w[0] |= ((lf.f[0][k] >> (w1 - 1)) & 1u) << k;
        }
        if (w2) put_bits(w + w1, w2 * k, w2, lf.f[1][k]);
        if (w3) put_bits(w + w1 + w2, w3 * k, w3, lf.f[2][k]);
    }
    for (int i = 0; i < nw; ++i) p0[(size_t)hs * nw * 32 + (size_t)(i >> 1) * 64 + 2 * j + (i & 1)] = w[i];
}

p8_status finish_shard(const HostSlot &h, const std::vector<uint32_t> &M, const std::vector<uint16_t> &S,
                       const std::vector<uint32_t> &D, int64_t rows, int64_t K, const uint16_t *c16, const int16_t *prm,
                       const std::vector<uint16_t> &dr, const std::vector<uint16_t> &dc, const std::vector<float> &dv,
                       uint8_t *out, size_t out_cap, size_t *out_n) {
    const size_t nt = (size_t)(rows / 32) * (size_t)(K / 256);
    std::vector<uint8_t> kb(offD(nt) + 4 * D.size(), 0);
    memcpy(kb.data(), h.s, kHdrBytes);
    memcpy(kb.data() + kHdrBytes, M.data(), 4 * nt);
    memcpy(kb.data() + offS(nt), S.data(), 2 * S.size());
    if (!D.empty()) memcpy(kb.data() + offD(nt), D.data(), 4 * D.size());
    return p8_slot_assemble(kb.data(), kb.size(), rows, K, c16, prm, dr.data(), dc.data(), dv.data(), (int64_t)dv.size(),
                            h.sg, out, out_cap, out_n);
}
}  // namespace

p8_status p8_tp_shard_cols(const uint8_t *slot, size_t nbytes, int64_t K, int64_t rows, int64_t b0, int64_t b1,
                           uint8_t *out, size_t out_cap, size_t *out_n) {
    HostSlot h;
    p8_status st = open_host(slot, nbytes, K, rows, h);
    if (st) return st;
    if (b0 < 0 || b1 <= b0 || b1 > (int64_t)h.nb) return P8_ERR_ARG;
    const size_t nb2 = (size_t)(b1 - b0), nt2 = h.ng * nb2;
    std::vector<uint32_t> M(nt2), D;
    std::vector<uint16_t> S(nb2 * (size_t)rows);
    for (size_t g = 0; g < h.ng; ++g)
        for (size_t b = 0; b < nb2; ++b) {
            const uint32_t mt = h.M[g * h.nb + b0 + b];
            const int c = (int)(mt >> 29);
            M[g * nb2 + b] = (uint32_t)D.size() | ((uint32_t)c << 29);
            const size_t w = (size_t)64 * NW(c);
            D.insert(D.end(), h.D + (mt & 0x1FFFFFFFu), h.D + (mt & 0x1FFFFFFFu) + w);
        }
    memcpy(S.data(), h.S + (size_t)b0 * rows, 2 * S.size());
    std::vector<uint16_t> dr, dc;
    std::vector<float> dv;
    for (uint32_t e = 0; e < h.tr->nd; ++e)
        if (h.dcol[e] >= 256 * b0 && h.dcol[e] < 256 * b1) {
            dr.push_back(h.drow[e]);
            dc.push_back((uint16_t)(h.dcol[e] - 256 * b0));
            dv.push_back(h.dval[e]);
        }
    return finish_shard(h, M, S, D, rows, 256 * (int64_t)nb2, h.c16 + 256 * b0, h.prm, dr, dc, dv, out, out_cap, out_n);
}

p8_status p8_tp_shard_rows(const uint8_t *slot, size_t nbytes, int64_t K, int64_t rows, int64_t r0, int64_t r1,
                           uint8_t *out, size_t out_cap, size_t *out_n, int32_t *orig_rows) {
    // Shard on ORIGINAL rows [r0, r1): the sorted rows whose prm lies in the range, kept in sorted order and re-tiled.
    // A row moved from lane j to lane j' has its steps rotated (step k holds chunk (lane + k) & 31).
    HostSlot h;
    p8_status st = open_host(slot, nbytes, K, rows, h);
    if (st) return st;
    if (r0 < 0 || r1 <= r0 || r1 > rows || (r1 - r0) % 32) return P8_ERR_ARG;
    const int64_t R = r1 - r0;
    std::vector<int> src;  // sorted source rows of the shard, in sorted order
    for (int64_t r = 0; r < rows; ++r)
        if (h.prm[r] >= r0 && h.prm[r] < r1) src.push_back((int)r);
    const size_t ng2 = (size_t)R / 32, nt2 = ng2 * h.nb;
    std::vector<uint32_t> M(nt2), D;
    std::vector<uint16_t> S(h.nb * (size_t)R);
    LaneFields lf, lf2;
    for (size_t g2 = 0; g2 < ng2; ++g2)
        for (size_t b = 0; b < h.nb; ++b) {
            int c = -1;
            for (int j2 = 0; j2 < 32; ++j2) {
                const int r = src[g2 * 32 + j2];
                const int cr = (int)(h.M[(size_t)(r / 32) * h.nb + b] >> 29);
                if (c < 0) c = cr;
                else if (c != cr) return P8_ERR_UNSUPPORTED;  // re-tiling needs one class per new tile-block
            }
            const size_t w = (size_t)64 * NW(c), base = D.size();
            M[g2 * h.nb + b] = (uint32_t)base | ((uint32_t)c << 29);
            D.resize(base + w, 0);
            for (int j2 = 0; j2 < 32; ++j2) {
                const int r = src[g2 * 32 + j2], j = r % 32;
                S[b * (size_t)R + g2 * 32 + j2] = h.S[b * (size_t)rows + r];
                if (!c) continue;
                const uint32_t *p0 = h.D + (h.M[(size_t)(r / 32) * h.nb + b] & 0x1FFFFFFFu);
                for (int hs = 0; hs < 2; ++hs) {
                    read_lane(p0, c, hs, j, lf);
                    for (int k2 = 0; k2 < 32; ++k2) {
                        const int k = (k2 + j2 - j) & 31;  // same chunk t = (j2 + k2) & 31 = (j + k) & 31
                        for (int s = 0; s < 3; ++s) lf2.f[s][k2] = lf.f[s][k];
                    }
                    write_lane(D.data() + base, c, hs, j2, lf2);
                }
            }
        }
    std::vector<int16_t> prm2((size_t)R);
    for (int64_t r2 = 0; r2 < R; ++r2) {
        prm2[(size_t)r2] = (int16_t)(h.prm[src[(size_t)r2]] - r0);
        if (orig_rows) orig_rows[r2] = h.prm[src[(size_t)r2]];
    }
    std::vector<uint16_t> dr, dc;
    std::vector<float> dv;
    for (uint32_t e = 0; e < h.tr->nd; ++e)
        if (h.drow[e] >= r0 && h.drow[e] < r1) {
            dr.push_back((uint16_t)(h.drow[e] - r0));
            dc.push_back(h.dcol[e]);
            dv.push_back(h.dval[e]);
        }
    return finish_shard(h, M, S, D, R, K, h.c16, prm2.data(), dr, dc, dv, out, out_cap, out_n);
}

const char *p8_status_str(p8_status s) {
    switch (s) {
        case P8_OK: return "ok";
        case P8_ERR_ARG: return "invalid argument";
        case P8_ERR_TRAILER: return "bad trailer (magic, rows, K or NS)";
        case P8_ERR_HEADER: return "bad header (NS must be 108, TRL 2)";
        case P8_ERR_PAYLOAD: return "payload size does not match the M words";
        case P8_ERR_PERM: return "prm is not a permutation";
        case P8_ERR_DELTA: return "delta index out of range";
        case P8_ERR_SIGNS: return "Hadamard signs must be +-1";
        case P8_ERR_TABLES: return "codebook + coset leaves int8 range";
        case P8_ERR_SHAPE: return "bad shape (K % 256, rows % 32, rows < 32768)";
        case P8_ERR_CUDA: return "CUDA runtime error";
        case P8_ERR_WORKSPACE: return "workspace too small";
        case P8_ERR_NOT_PREPARED: return "tensor not prepared";
        case P8_ERR_UNSUPPORTED: return "unsupported request";
        case P8_ERR_TIMEOUT: return "device wait timed out";
        case P8_ERR_SLOT: return "no slot type fits";
        case P8_ERR_FILE: return "model file unreadable, not GGUF v2/v3, or malformed";
        case P8_ERR_MODEL: return "model file: Pingala-8 keys or tensors missing or inconsistent";
        case P8_ERR_NOALLOC_SCRATCH: return "the fixed no-allocation scratch array could not be placed on this device";
    }
    return "unknown status";
}

}  // extern "C"
