// p8_gguf.cpp -- GGUF reader and Pingala-8 ("VR native") model loader, host side.
//
// Follows the reference loader (llama_model_loader::vr_native_init / vr_native_load, CU:3411-3580): the file KV
// vr.format, vr.ns = 108, vr.trl = 2, vr.n_linear, vr.layout (2 = slot kernel bytes + row permutation, 3 = VR3 file
// tensors with natural rows); per linear <base>.weight (I8, 1-D kernel or VR3 bytes), <base>.vr_c (F16 [K]),
// <base>.vr_prm (I16 [rows], layout 2 only), optionally <base>.vr_didx (I16 [nd, 2]) + <base>.vr_dval (F32 [nd]);
// vr.had_signs (I8 [256]) shared. Each linear becomes the slot the reference builds in device memory (smallest of
// IQ2_XXS, Q2_K..Q6_K rows that holds it), assembled in host memory by p8_slot_assemble with all of its checks.
//
// The GGUF container (versions 2 and 3) is parsed by bounded reads: every length and offset is checked against the
// file size before use. Errors: P8_ERR_FILE (I/O, not GGUF, malformed container), P8_ERR_MODEL (VR keys or tensors
// missing or inconsistent), and the slot statuses of p8_slot_assemble.
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "p8_format.h"
#include "pingala8.h"

using namespace p8;

namespace {

enum GgufType : uint32_t {  // GGUF value types
    U8 = 0, I8 = 1, U16 = 2, I16 = 3, U32 = 4, I32 = 5, F32 = 6, BOOL = 7, STR = 8, ARR = 9, U64 = 10, I64 = 11, F64 = 12
};
enum GgmlType : uint32_t { G_F32 = 0, G_F16 = 1, G_I8 = 24, G_I16 = 25 };

struct Kv {
    uint32_t type = 0;
    uint64_t u = 0;   // integer scalars
    std::string s;    // strings
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> ne;
    uint32_t type = 0;
    uint64_t offset = 0;  // from the start of the data section
    uint64_t nbytes = 0;  // 0 for types this loader does not read
};

struct Reader {
    FILE *f = nullptr;
    uint64_t size = 0, pos = 0;
    bool ok = true;
    bool read(void *dst, uint64_t n) {
        if (!ok || n > size - pos) return ok = false;
        if (n && fread(dst, 1, (size_t)n, f) != (size_t)n) return ok = false;
        pos += n;
        return true;
    }
    bool skip(uint64_t n) {
        if (!ok || n > size - pos) return ok = false;
        if (fseeko(f, (off_t)(pos + n), SEEK_SET) != 0) return ok = false;
        pos += n;
        return true;
    }
    template <typename T>
    T get() {
        T v{};
        read(&v, sizeof(T));
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > size - pos || n > (1u << 20)) {  // keys and string values are short; a huge length is corruption
            ok = false;
            return std::string();
        }
        std::string s((size_t)n, '\0');
        read(&s[0], n);
        return s;
    }
};

uint64_t scalar_bytes(uint32_t t) {
    switch (t) {
        case U8: case I8: case BOOL: return 1;
        case U16: case I16: return 2;
        case U32: case I32: case F32: return 4;
        case U64: case I64: case F64: return 8;
        default: return 0;
    }
}

bool read_value(Reader &r, uint32_t t, Kv *kv, int depth) {
    if (t == STR) {
        std::string s = r.str();
        if (kv) kv->s = std::move(s);
        return r.ok;
    }
    if (t == ARR) {
        if (depth > 0) return r.ok = false;  // nested arrays do not occur in model files
        const uint32_t et = r.get<uint32_t>();
        const uint64_t n = r.get<uint64_t>();
        if (!r.ok) return false;
        if (et == STR) {
            for (uint64_t i = 0; i < n && r.ok; ++i) (void)r.str();
            return r.ok;
        }
        const uint64_t es = scalar_bytes(et);
        if (!es || n > (r.size - r.pos) / es) return r.ok = false;
        return r.skip(n * es);
    }
    const uint64_t es = scalar_bytes(t);
    if (!es) return r.ok = false;
    uint64_t v = 0;
    r.read(&v, es);
    if (kv) kv->u = v;
    return r.ok;
}

bool ends_with(const std::string &s, const char *suf) {
    const size_t n = strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

}  // namespace

struct p8_linear {
    std::string name;  // <base>.weight
    const TensorInfo *w = nullptr, *c = nullptr, *prm = nullptr, *didx = nullptr, *dval = nullptr;
    int64_t K = 0, rows = 0, nd = 0;
    size_t fbytes = 0, kbytes = 0, slot_n = 0;
};

struct p8_gguf {
    Reader r;
    uint64_t data_off = 0;
    uint32_t layout = 2;
    std::map<std::string, Kv> kv;
    std::vector<TensorInfo> tensors;
    std::map<std::string, size_t> by_name;
    std::vector<p8_linear> linears;
    const TensorInfo *signs = nullptr;
    std::vector<uint8_t> hdr0;  // A, B, c of the first linear loaded (every linear must carry the same tables)
};

namespace {

bool read_at(p8_gguf *g, uint64_t off, void *dst, uint64_t n) {
    if (off > g->r.size || n > g->r.size - off) return false;
    if (fseeko(g->r.f, (off_t)off, SEEK_SET) != 0) return false;
    return !n || fread(dst, 1, (size_t)n, g->r.f) == (size_t)n;
}
bool read_tensor(p8_gguf *g, const TensorInfo *t, void *dst, uint64_t n) {
    return t && n <= t->nbytes && read_at(g, g->data_off + t->offset, dst, n);
}
const TensorInfo *find(const p8_gguf *g, const std::string &name) {
    const auto it = g->by_name.find(name);
    return it == g->by_name.end() ? nullptr : &g->tensors[it->second];
}
bool kv_u32(const p8_gguf *g, const char *key, uint32_t *v) {
    const auto it = g->kv.find(key);
    if (it == g->kv.end() || it->second.type != U32) return false;
    *v = (uint32_t)it->second.u;
    return true;
}

p8_status parse(p8_gguf *g) {
    Reader &r = g->r;
    const uint32_t magic = r.get<uint32_t>(), version = r.get<uint32_t>();
    if (!r.ok || magic != 0x46554747u || (version != 2 && version != 3)) return P8_ERR_FILE;  // "GGUF", v2 / v3
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) return P8_ERR_FILE;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        std::string key = r.str();
        Kv v;
        v.type = r.get<uint32_t>();
        if (!r.ok || !read_value(r, v.type, &v, 0)) return P8_ERR_FILE;
        g->kv[key] = std::move(v);
    }
    g->tensors.resize((size_t)n_tensors);
    for (uint64_t i = 0; i < n_tensors; ++i) {
        TensorInfo &t = g->tensors[(size_t)i];
        t.name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (!r.ok || nd == 0 || nd > 4) return P8_ERR_FILE;
        t.ne.resize(nd);
        uint64_t ne = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            t.ne[d] = r.get<uint64_t>();
            if (t.ne[d] == 0 || ne > (1ull << 40) / t.ne[d]) return P8_ERR_FILE;
            ne *= t.ne[d];
        }
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        if (!r.ok) return P8_ERR_FILE;
        const uint64_t es = t.type == G_F32 ? 4 : (t.type == G_F16 || t.type == G_I16) ? 2 : t.type == G_I8 ? 1 : 0;
        t.nbytes = ne * es;
        g->by_name[t.name] = (size_t)i;
    }
    uint32_t align = 32;
    {
        const auto it = g->kv.find("general.alignment");
        if (it != g->kv.end() && it->second.type == U32) align = (uint32_t)it->second.u;
        if (align == 0 || (align & (align - 1))) return P8_ERR_FILE;
    }
    g->data_off = (r.pos + align - 1) / align * align;
    for (const TensorInfo &t : g->tensors)  // every tensor this loader reads lies inside the file
        if (t.nbytes && (t.offset > r.size || g->data_off > r.size - t.offset || t.nbytes > r.size - g->data_off - t.offset))
            return P8_ERR_FILE;
    return P8_OK;
}

// vr_native_init (CU:3411-3508)
p8_status init_vr(p8_gguf *g) {
    if (!g->kv.count("vr.format")) return P8_ERR_MODEL;
    uint32_t ns = 0, trl = 0, n_linear = 0;
    if (!kv_u32(g, "vr.ns", &ns) || ns != kNS) return P8_ERR_MODEL;
    if (!kv_u32(g, "vr.trl", &trl) || trl != kTRL || !kv_u32(g, "vr.n_linear", &n_linear)) return P8_ERR_MODEL;
    if (g->kv.count("vr.layout") && !kv_u32(g, "vr.layout", &g->layout)) return P8_ERR_MODEL;
    if (g->layout != 2 && g->layout != 3) return P8_ERR_MODEL;
    for (const TensorInfo &t : g->tensors) {
        if (!ends_with(t.name, ".vr_c")) continue;
        const std::string b = t.name.substr(0, t.name.size() - 5);
        p8_linear L;
        L.name = b + ".weight";
        L.w = find(g, L.name);
        L.c = &t;
        if (!L.w || L.w->type != G_I8 || L.w->ne.size() != 1) return P8_ERR_MODEL;
        if (L.c->type != G_F16 || L.c->ne.size() != 1) return P8_ERR_MODEL;
        L.K = (int64_t)L.c->ne[0];
        L.fbytes = (size_t)L.w->ne[0];
        if (g->layout == 2) {
            L.prm = find(g, b + ".vr_prm");
            if (!L.prm || L.prm->type != G_I16 || L.prm->ne.size() != 1) return P8_ERR_MODEL;
            L.rows = (int64_t)L.prm->ne[0];
            L.kbytes = L.fbytes;
        } else {  // VR3: rows from the file size, K and header word 515; natural rows, no permutation tensor
            if (find(g, b + ".vr_prm")) return P8_ERR_MODEL;
            uint32_t w515 = 0;
            if (L.fbytes < kHdrBytes) return P8_ERR_MODEL;
            if (!read_at(g, g->data_off + L.w->offset + 2060, &w515, 4)) return P8_ERR_FILE;
            size_t kb = 0;
            L.rows = (int64_t)p8_vr3_rows(L.fbytes, (size_t)L.K, w515, &kb);
            if (!L.rows) return P8_ERR_MODEL;
            L.kbytes = kb;
        }
        if (L.K <= 0 || L.K % 256 || L.rows <= 0 || L.rows % 32 || L.rows > kMaxRows || L.K > 65535) return P8_ERR_SHAPE;
        L.didx = find(g, b + ".vr_didx");
        L.dval = find(g, b + ".vr_dval");
        if (!L.didx != !L.dval) return P8_ERR_MODEL;
        if (L.dval) {
            if (L.didx->type != G_I16 || L.dval->type != G_F32 || L.dval->ne.size() != 1 || L.didx->ne.size() != 2 ||
                L.didx->ne[0] != L.dval->ne[0] || L.didx->ne[1] != 2)
                return P8_ERR_MODEL;
            L.nd = (int64_t)L.dval->ne[0];
        }
        const size_t need = p8_slot_need(L.kbytes, (size_t)L.rows, (size_t)L.K, (size_t)L.nd);
        int ti = -1;
        L.slot_n = p8_slot_nbytes((size_t)L.rows, (size_t)L.K, need, &ti);
        if (!L.slot_n) return P8_ERR_SLOT;
        g->linears.push_back(L);
    }
    g->signs = find(g, "vr.had_signs");
    if (!g->signs || g->signs->type != G_I8 || g->signs->ne.size() != 1 || g->signs->ne[0] != 256) return P8_ERR_MODEL;
    // load-time count check: vr.n_linear linears, and 7 per block where the architecture states its block count
    if (g->linears.size() != n_linear) return P8_ERR_MODEL;
    const auto ia = g->kv.find("general.architecture");
    if (ia != g->kv.end() && ia->second.type == STR) {
        uint32_t blocks = 0;
        if (kv_u32(g, (ia->second.s + ".block_count").c_str(), &blocks) && n_linear != 7u * blocks) return P8_ERR_MODEL;
    }
    std::sort(g->linears.begin(), g->linears.end(), [](const p8_linear &a, const p8_linear &b) { return a.name < b.name; });
    return P8_OK;
}

}  // namespace

extern "C" {

p8_status p8_gguf_open(const char *path, p8_gguf **out) {
    if (!path || !out) return P8_ERR_ARG;
    *out = nullptr;
    p8_gguf *g = new p8_gguf();
    g->r.f = fopen(path, "rb");
    if (!g->r.f) {
        delete g;
        return P8_ERR_FILE;
    }
    if (fseeko(g->r.f, 0, SEEK_END) != 0 || (g->r.size = (uint64_t)ftello(g->r.f)) == (uint64_t)-1 ||
        fseeko(g->r.f, 0, SEEK_SET) != 0) {
        fclose(g->r.f);
        delete g;
        return P8_ERR_FILE;
    }
    p8_status st = parse(g);
    if (st == P8_OK) st = init_vr(g);
    if (st != P8_OK) {
        fclose(g->r.f);
        delete g;
        return st;
    }
    *out = g;
    return P8_OK;
}

void p8_gguf_close(p8_gguf *g) {
    if (!g) return;
    if (g->r.f) fclose(g->r.f);
    delete g;
}

int64_t p8_gguf_n_linear(const p8_gguf *g) { return g ? (int64_t)g->linears.size() : 0; }

p8_status p8_gguf_linear_info(const p8_gguf *g, int64_t i, const char **name, int64_t *K, int64_t *rows, int64_t *nd,
                              size_t *slot_nbytes, int *layout) {
    if (!g || i < 0 || i >= (int64_t)g->linears.size()) return P8_ERR_ARG;
    const p8_linear &L = g->linears[(size_t)i];
    if (name) *name = L.name.c_str();
    if (K) *K = L.K;
    if (rows) *rows = L.rows;
    if (nd) *nd = L.nd;
    if (slot_nbytes) *slot_nbytes = L.slot_n;
    if (layout) *layout = (int)g->layout;
    return P8_OK;
}

// vr_native_load (CU:3527-3580), into host memory
p8_status p8_gguf_load_linear(p8_gguf *g, int64_t i, uint8_t *out, size_t out_cap, size_t *out_n) {
    if (!g || !out || i < 0 || i >= (int64_t)g->linears.size()) return P8_ERR_ARG;
    const p8_linear &L = g->linears[(size_t)i];
    if (out_cap < L.slot_n) return P8_ERR_ARG;
    std::vector<uint8_t> kb(L.kbytes);
    if (g->layout == 2) {
        if (!read_tensor(g, L.w, kb.data(), L.kbytes)) return P8_ERR_FILE;
    } else {
        std::vector<uint8_t> f3(L.fbytes);
        if (!read_tensor(g, L.w, f3.data(), L.fbytes)) return P8_ERR_FILE;
        const p8_status st = p8_vr3_expand(f3.data(), L.fbytes, (size_t)L.rows, (size_t)L.K, kb.data(), kb.size());
        if (st) return st;
    }
    if (g->hdr0.empty()) {
        g->hdr0.assign(kb.begin(), kb.begin() + 2052);
    } else if (memcmp(g->hdr0.data(), kb.data(), 2052) != 0) {
        return P8_ERR_TABLES;  // every linear of a model carries the same codebook and coset
    }
    std::vector<uint16_t> c16((size_t)L.K);
    std::vector<int16_t> prm;
    std::vector<uint16_t> didx((size_t)L.nd * 2);
    std::vector<float> dval((size_t)L.nd);
    std::vector<int8_t> signs(256);
    if (!read_tensor(g, L.c, c16.data(), 2 * c16.size()) || !read_tensor(g, g->signs, signs.data(), 256)) return P8_ERR_FILE;
    if (L.prm) {
        prm.resize((size_t)L.rows);
        if (!read_tensor(g, L.prm, prm.data(), 2 * prm.size())) return P8_ERR_FILE;
    }
    if (L.nd && (!read_tensor(g, L.didx, didx.data(), 2 * didx.size()) || !read_tensor(g, L.dval, dval.data(), 4 * dval.size())))
        return P8_ERR_FILE;
    return p8_slot_assemble(kb.data(), kb.size(), L.rows, L.K, c16.data(), L.prm ? prm.data() : nullptr,
                            L.nd ? didx.data() : nullptr, L.nd ? didx.data() + L.nd : nullptr, L.nd ? dval.data() : nullptr,
                            L.nd, signs.data(), out, out_cap, out_n);
}

}  // extern "C"
