// p8_chain.cuh -- chained batch-1 GEMVs (included by p8_kernels.cu, namespace p8).
//
// A decode step runs a fixed sequence of projections, each reading an earlier one's output: o -> gate/up -> down ->
// q/k/v of the next layer. As separate calls every projection costs k_gemv, a hand-off, k_gemv_reduce and a second
// hand-off. A chain runs each projection as ONE k_gemv launch in chained mode:
//
//   * a step whose input x (or SwiGLU up) is an output of the previous step reads it straight from that step's row
//     partials while it builds its tables (chain_inputs: the 16-block slices of the block's 256 rows, then clamp
//     delta, the previous step's output scale and residual); the CTA that holds a block's first unit writes those rows
//     of the previous output;
//   * the previous step's outputs that this step does not read (k and v after q/k/v) are reduced by this step's CTAs
//     in equal shares after their units (chain_unconsumed);
//   * an RMSNorm on an input that comes from partials is applied to the step's OUTPUT: its scale 1 / sqrt(mean(x^2) +
//     eps) is one positive scalar per vector and the product is linear, so the tables use x * w and the reduce of the
//     step's partials one launch later (the next step or the final k_gemv_reduce), when every block's sum of squares
//     is known, multiplies by the scale. The x16 quantisation is per 128 columns relative to their largest value, so
//     it is the same up to float rounding of the scaled inputs;
//   * after the last step one k_gemv_reduce (chain semantics: scale and residual) writes its outputs.
//
// Every launch waits on the previous one with programmatic dependent launch, so a chain of n steps is n + 1 kernels
// and n + 1 hand-offs, against 2 n of each for separate calls. A row's reduction order is k_gemv_reduce's in every
// place it is reduced, so a chained output differs from the separate call only where RMSNorm's scale moved.
//
// Workspace: partials of two consecutive steps (ping-pong), x' and per-block sums of squares likewise. The plan (the
// launch arguments of every step, with workspace offsets) is built once by chain_create; a run patches the workspace
// address into a copy and enqueues the launches.

constexpr int kChainMaxSteps = 4096;

// one step's launch: the k_gemv arguments with workspace-relative pointers kept as offsets (bound per run)
struct ChainPlanStep {
    GemvArgs a;
    ChainIn ch;
    int pro, grid;
    long long part_off[kMaxGroup];  // this step's partials per tensor
    long long xv_off;               // this step's x' (input op), -1: none
    long long ss_off;               // this step's per-block sums of squares (deferred RMSNorm), -1: none
    long long x_off, x2_off;        // sources of x / x2 among the previous step's partials, -1: memory
    long long unc_off[kMaxGroup];   // the previous step's unread outputs' partials
    long long chxv_off;             // the previous step's x' in the workspace, -1: ch.xv is a caller buffer
    long long chss_off;             // the previous step's sums of squares, -1: none
};

}  // namespace p8

struct p8_chain {
    uint32_t magic;
    int device, nsteps, ctas;
    std::vector<p8::ChainPlanStep> steps;
    p8::ReduceArgs fin;             // the last step's rows (partials and x' / ss bound per run)
    long long fin_part_off[p8::kMaxGroup], fin_xv_off, fin_ss_off;
    int fin_grid;
    size_t ws_bytes;
    unsigned long long *trace;      // optional phase stamps (device), set by p8_chain_trace
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
    // ---- validation (the step rules of p8_chain_create)
    int dev = -1;
    std::vector<int> xsrc((size_t)n, -1), x2src((size_t)n, -1);
    for (int s = 0; s < n; ++s) {
        const p8_chain_step &q = st[s];
        if (q.n < 1 || q.n > kMaxGroup || !q.x || ((uintptr_t)q.x & 15)) return P8_ERR_ARG;
        for (int i = 0; i < q.n; ++i) {
            const p8_tensor *t = q.t[i];
            if (!t || t->magic != kTensorMagic) return P8_ERR_NOT_PREPARED;
            if (t->K != q.t[0]->K || t->act_hash != q.t[0]->act_hash || !q.y[i]) return P8_ERR_ARG;
            if (dev < 0) dev = t->device;
            if (t->device != dev) return P8_ERR_ARG;
            if (q.res[i] && overlaps(q.res[i], 4 * (size_t)t->rows, q.y[i], 4 * (size_t)t->rows)) return P8_ERR_ARG;
        }
        const int pk = q.pro.kind;
        if (pk == P8_PROLOGUE_RMSNORM) {
            if (!q.pro.w || ((uintptr_t)q.pro.w & 15) || !(q.pro.eps >= 0.f)) return P8_ERR_ARG;
        } else if (pk == P8_PROLOGUE_SWIGLU) {
            if (!q.pro.x2 || ((uintptr_t)q.pro.x2 & 15)) return P8_ERR_ARG;
        } else if (pk != P8_PROLOGUE_NONE) {
            return P8_ERR_ARG;
        }
        // input sources: exactly an output of the previous step is read from its partials; any other overlap with
        // the previous step's outputs is refused (their rows are written only during this step)
        if (s > 0) {
            const p8_chain_step &pq = st[s - 1];
            const int K = q.t[0]->K;
            auto source = [&](const float *p, int &src) -> bool {
                for (int i = 0; i < pq.n; ++i) {
                    if (p == pq.y[i]) {
                        if (pq.t[i]->rows != K) return false;
                        src = i;
                        return true;
                    }
                    if (overlaps(p, 4 * (size_t)K, pq.y[i], 4 * (size_t)pq.t[i]->rows)) return false;
                }
                return true;
            };
            if (!source(q.x, xsrc[(size_t)s])) return P8_ERR_ARG;
            if (pk == P8_PROLOGUE_SWIGLU && !source(q.pro.x2, x2src[(size_t)s])) return P8_ERR_ARG;
        }
    }
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != dev) return P8_ERR_ARG;  // the tensors' device must be current
    const int nsm = sm_count();
    // ---- workspace: partials / x' / sums of squares of two consecutive steps
    size_t part_max = 0, k_max = 0, nb_max = 0;
    std::vector<std::vector<size_t>> poff((size_t)n);
    for (int s = 0; s < n; ++s) {
        size_t o = 0;
        for (int i = 0; i < st[s].n; ++i) {
            poff[(size_t)s].push_back(o);
            o += ((size_t)st[s].t[i]->nb * st[s].t[i]->rows * 4 + 255) & ~(size_t)255;
        }
        part_max = std::max(part_max, o);
        k_max = std::max(k_max, (size_t)st[s].t[0]->K);
        nb_max = std::max(nb_max, (size_t)st[s].t[0]->nb);
    }
    long long PART[2], XV[2], SS[2];
    size_t o = 0;
    for (int i = 0; i < 2; ++i) { PART[i] = (long long)o; o += part_max; }
    for (int i = 0; i < 2; ++i) { XV[i] = (long long)o; o += (4 * k_max + 255) & ~(size_t)255; }
    for (int i = 0; i < 2; ++i) { SS[i] = (long long)o; o += (4 * nb_max + 255) & ~(size_t)255; }
    auto deferred = [&](int s) { return s > 0 && xsrc[(size_t)s] >= 0 && st[s].pro.kind == P8_PROLOGUE_RMSNORM; };
    auto read_by_next = [&](int s, int i) { return s + 1 < n && (xsrc[(size_t)s + 1] == i || x2src[(size_t)s + 1] == i); };
    p8_chain *p = new p8_chain();
    p->magic = kChainMagic;
    p->device = dev;
    p->nsteps = n;
    p->ctas = nsm;
    p->ws_bytes = o;
    p->trace = nullptr;
    p->steps.resize((size_t)n);
    for (int s = 0; s < n; ++s) {
        const p8_chain_step &q = st[s];
        const p8_tensor *t0 = q.t[0];
        ChainPlanStep &P = p->steps[(size_t)s];
        memset(&P, 0, sizeof(P));
        GemvArgs &g = P.a;
        g.ntensors = q.n;
        g.X = q.x;
        g.ic = t0->ic; g.A = t0->A; g.cs = t0->cs; g.K = t0->K; g.nb = t0->nb; g.nsl = t0->nsl;
        P.pro = q.pro.kind;
        if (P.pro == P8_PROLOGUE_RMSNORM) { g.pw = q.pro.w; g.eps = q.pro.eps; }
        if (P.pro == P8_PROLOGUE_SWIGLU) g.x2 = q.pro.x2;
        int g0 = 0;
        for (int i = 0; i < q.n; ++i) {
            const p8_tensor *t = q.t[i];
            GemvTensor &T = g.t[i];
            T.M = t->M; T.D = t->D; T.S = t->S; T.prm = t->prm; T.cp = t->cp; T.cc = t->cc; T.cv = t->cv;
            T.Y = q.y[i]; T.res = q.res[i];
            T.rows = t->rows; T.ng = t->ng; T.g0 = g0; T.row0 = g.rows_total; T.ucls = t->uniform_class;
            P.part_off[i] = PART[s & 1] + (long long)poff[(size_t)s][(size_t)i];
            g0 += t->ng;
            g.rows_total += t->rows;
        }
        g.ng_total = g0;
        g.units = (long long)g0 * t0->nb;
        P.xv_off = P.pro != P8_PROLOGUE_NONE ? XV[s & 1] : -1;
        P.ss_off = deferred(s) ? SS[s & 1] : -1;
        P.x_off = P.x2_off = P.chxv_off = P.chss_off = -1;
        for (int i = 0; i < kMaxGroup; ++i) P.unc_off[i] = -1;
        if (s > 0) {
            const p8_chain_step &pq = st[s - 1];
            const ChainPlanStep &PP = p->steps[(size_t)s - 1];
            ChainIn &c = P.ch;
            c.chained = 1;
            auto src_of = [&](int i) {
                ChainSrc r;
                r.part = nullptr;
                r.cp = pq.t[i]->cp; r.cc = pq.t[i]->cc; r.cv = pq.t[i]->cv;
                r.res = pq.res[i]; r.Y = pq.y[i]; r.rows = pq.t[i]->rows;
                return r;
            };
            if (xsrc[(size_t)s] >= 0) { c.x = src_of(xsrc[(size_t)s]); P.x_off = PP.part_off[xsrc[(size_t)s]]; }
            if (x2src[(size_t)s] >= 0) { c.x2 = src_of(x2src[(size_t)s]); P.x2_off = PP.part_off[x2src[(size_t)s]]; }
            for (int i = 0; i < pq.n; ++i)
                if (!read_by_next(s - 1, i)) {
                    P.unc_off[c.nunc] = PP.part_off[i];
                    c.unc[c.nunc++] = src_of(i);
                    c.unc_rows += pq.t[i]->rows;
                }
            // the previous step's x' (its outputs' clamp-delta term): its input op's output, else its input itself
            if (pq.pro.kind != P8_PROLOGUE_NONE) P.chxv_off = PP.xv_off;
            else c.xv = pq.x;
            P.chss_off = PP.ss_off;
            c.nb = pq.t[0]->nb;
            c.K = pq.t[0]->K;
            c.eps = pq.pro.eps;
        }
        const int Pm = (int)std::min<long long>(g.units, std::min(nsm, kGemvMaxCtas));
        P.grid = partition_units(g.units, g0, Pm, g.ustart);
        if (P.grid < 1) {
            delete p;
            return P8_ERR_ARG;
        }
    }
    // ---- the final reduce: every output of the last step
    {
        const int L = n - 1;
        const p8_chain_step &q = st[L];
        const ChainPlanStep &PL = p->steps[(size_t)L];
        ReduceArgs &r = p->fin;
        memset(&r, 0, sizeof(r));
        r.ntensors = q.n;
        r.nb = q.t[0]->nb;
        for (int i = 0; i < q.n; ++i) {
            r.t[i] = PL.a.t[i];
            p->fin_part_off[i] = PL.part_off[i];
        }
        r.rows_total = PL.a.rows_total;
        r.X = q.x;  // replaced by the workspace x' when the step has an input op
        p->fin_xv_off = PL.xv_off;
        p->fin_ss_off = PL.ss_off;
        r.ssK = q.t[0]->K;
        r.eps = q.pro.eps;
        p->fin_grid = std::max(1, std::min((r.rows_total + kRedRowsPerCta - 1) / kRedRowsPerCta, nsm));
    }
    *out = p;
    return P8_OK;
}

p8_status chain_destroy(p8_chain *p) {
    if (!p || p->magic != kChainMagic) return P8_ERR_ARG;
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

p8_status chain_run(const p8_chain *p, void *ws, size_t ws_bytes, cudaStream_t st, int) {
    if (!p || p->magic != kChainMagic) return P8_ERR_ARG;
    if (!ws || ws_bytes < p->ws_bytes || ((uintptr_t)ws & 255)) return P8_ERR_WORKSPACE;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return P8_ERR_CUDA;
    if (dev != p->device || sm_count() != p->ctas) return P8_ERR_ARG;
    uint8_t *w = static_cast<uint8_t *>(ws);
    auto at = [&](long long off) { return off < 0 ? nullptr : reinterpret_cast<float *>(w + off); };
    for (int s = 0; s < p->nsteps; ++s) {
        const ChainPlanStep &P = p->steps[(size_t)s];
        GemvArgs g = P.a;  // bind the workspace
        ChainIn c = P.ch;
        for (int i = 0; i < g.ntensors; ++i) g.t[i].part = at(P.part_off[i]);
        g.xv = at(P.xv_off);
        c.ss_out = at(P.ss_off);
        c.x.part = at(P.x_off);
        c.x2.part = at(P.x2_off);
        for (int i = 0; i < c.nunc; ++i) c.unc[i].part = at(P.unc_off[i]);
        if (P.chxv_off >= 0) c.xv = at(P.chxv_off);
        c.ss = at(P.chss_off);
        c.trace = p->trace ? p->trace + (size_t)s * p->ctas * 8 : nullptr;
        // the first step reads its input from memory and has no previous step: the plain GEMV kernel; the others the
        // chain-step kernel (a RMSNorm whose input comes from partials is deferred: c.ss_out)
        const bool chained = c.chained != 0;
        void *args1[] = {&g};
        void *args2[] = {&g, &c};
        const void *fn = P.pro == P8_PROLOGUE_RMSNORM ? (chained ? (const void *)k_gemv_chain<P8_PROLOGUE_RMSNORM> : (const void *)k_gemv<P8_PROLOGUE_RMSNORM>)
                         : P.pro == P8_PROLOGUE_SWIGLU ? (chained ? (const void *)k_gemv_chain<P8_PROLOGUE_SWIGLU> : (const void *)k_gemv<P8_PROLOGUE_SWIGLU>)
                                                       : (chained ? (const void *)k_gemv_chain<P8_PROLOGUE_NONE> : (const void *)k_gemv<P8_PROLOGUE_NONE>);
        if (launch_pdl(fn, dim3((unsigned)P.grid), dim3(kGemvThreads), kGemvSmem, st, chained ? args2 : args1) != cudaSuccess)
            return P8_ERR_CUDA;
    }
    ReduceArgs r = p->fin;
    for (int i = 0; i < r.ntensors; ++i) r.t[i].part = at(p->fin_part_off[i]);
    if (p->fin_xv_off >= 0) r.X = at(p->fin_xv_off);
    r.ss = at(p->fin_ss_off);
    void *args[] = {&r};
    return launch_pdl((const void *)k_gemv_reduce<false, true>, dim3((unsigned)p->fin_grid), dim3(kRedThreads), 0, st, args) == cudaSuccess
               ? P8_OK
               : P8_ERR_CUDA;
}
