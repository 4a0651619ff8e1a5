// C ABI of liblmoe.so (declared in include/lmoe.h).  Host-side validation,
// workspace layout and kernel sequencing; no allocation, no host sync.
#include <cstring>
#include <mutex>

#include "../../include/lmoe.h"
#include "lmoe_kernels.cuh"

using namespace lmoe;

namespace {

// bit widths and group sizes of the decode GEMVs
bool gemv_ok(int bits, int gs) {
    return (bits == 2 && (gs == 64 || gs == 128)) ||
           ((bits == 4 || bits == 8) && (gs == 32 || gs == 64 || gs == 128));
}
// ... and of the arena arrays a layer accepts: 3-bit projections run on the
// prefill (tcgen05) kernels at every token count
bool quant_ok(int bits, int gs) { return gemv_ok(bits, gs) || (bits == 3 && (gs == 32 || gs == 64 || gs == 128)); }

size_t al(size_t v) { return (v + 255) & ~size_t(255); }

#ifdef LMOE_PROFILE_TRACE
// profiling timeline of the gate/up kernel (lmoe_profile_trace, profiling
// builds only)
uint64_t *g_trace = nullptr;
int32_t g_trace_units = 0;
#endif

struct Layout {
    size_t status = 0, partial = 0, idx = 0, w = 0, sorted = 0, counts = 0, roff = 0,
           nchunks = 0, chunks = 0, xpanel = 0, xsum = 0, hpanel = 0, hsum = 0, yw = 0,
           cnt = 0, dblk = 0, total = 0;
    int max_chunks = 0;
    // single-token kernel (lmoe_vec.cu): its counter (right after cnt, so the
    // per-call zeroing covers it: zero_end) and the int8 pieces of h and x
    size_t vcnt = 0, vhq = 0, vhs = 0, zero_end = 0;
    // prefill path: tiled activation panels of the tcgen05 grouped GEMM
    size_t pfx = 0, pfh = 0;
    int pf_rows = 0, pf_chunks = 0;
    bool prefill = false;
};

int max_chunks_for(int buckets, int R) {
    const int distinct = buckets < R ? buckets : R;
    return distinct + R + 1;  // any chunk size >= 1
}

// Layout shared by all entry points.  x_rows: rows of the input panel;
// R: routes; K: input width; I: intermediate width (0 if unused);
// H_out: output width of the combine (0 if unused); T: tokens.
// Scratch of the single-token kernel (zero sizes: not used by the layout):
// counter words (right after cnt, so the per-call zeroing covers them), the
// int8 pieces of h then x, and their (sum, factor) arrays.
struct VecSizes {
    size_t cnt_words = 0, hq_bytes = 0, hs_bytes = 0;
};

Layout make_layout(int T, int R, int K, int I, int H_out, int buckets, int E_router,
                   int ksplit, int x_rows, const VecSizes &vs = VecSizes()) {
    Layout L;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += al(bytes);
        return o;
    };
    L.status = take(256);
    // The regions that must start at zero (status word and router counter
    // above, combine counters here) sit at fixed offsets at the start, so a
    // workspace zeroed once serves calls with any token count that fits:
    // every call restores the counters it used, and a smaller call uses a
    // prefix of the same zero region.  Everything after is rewritten by each
    // call before it is read.
    L.cnt = take((size_t)T * (H_out / 16) * 4);
    if (vs.cnt_words) L.vcnt = take(vs.cnt_words * 4);
    L.zero_end = off;
    // logits, then (score, biased score) per (token, expert)
    L.partial = take((size_t)ksplit * T * E_router * 4 + 8 + (size_t)T * E_router * 8);
    L.idx = take((size_t)R * 4);
    L.w = take((size_t)R * 4);
    L.sorted = take((size_t)R * 4);
    L.counts = take((size_t)(buckets + 1) * 4);
    L.roff = take((size_t)(buckets + 1) * 4);
    L.nchunks = take(16);
    L.max_chunks = max_chunks_for(buckets, R);
    L.chunks = take((size_t)L.max_chunks * sizeof(Chunk));
    L.dblk = take((size_t)((R + 255) / 256) * buckets * 4);
    L.xpanel = take((size_t)x_rows * K * 2);
    L.xsum = take((size_t)x_rows * (K / 16) * 8);
    L.hpanel = take((size_t)R * I * 2);
    L.hsum = take((size_t)R * (I / 16) * 8);
    L.yw = take((size_t)R * H_out * 2);
    if (vs.hq_bytes) {
        L.vhq = take(vs.hq_bytes);
        L.vhs = take(vs.hs_bytes);
    }
    L.total = off;
    return L;
}

// shared: one more route per token for the block's shared expert (its
// routes follow the T * top_k routed ones)
// Single-token layers whose geometry the integer tensor-pipe kernel
// (lmoe_vec.cu) covers: gate and up alike, one group size for all three
// projections, the stream format's geometry, at most 32 routes.  Whether the
// stream copies exist is checked per call; the workspace is sized on the
// geometry alone.
bool vec_geometry(const lmoe_layer *l, int R, VecCfg *cfg) {
    const lmoe_experts &ex = l->experts;
    if (ex.gate.bits != ex.up.bits || ex.gate.group_size != ex.up.group_size) return false;
    VecCfg c;
    if (!vec_layer_config(ex.hidden, ex.inter, ex.gate.bits, ex.gate.group_size, ex.down.bits, ex.down.group_size,
                          R, &c))
        return false;
    if (cfg) *cfg = c;
    return true;
}

VecSizes vec_sizes(const lmoe_layer *l, int T, int R) {
    VecSizes vs;
    VecCfg c;
    if (T != 1 || !vec_geometry(l, R, &c)) return vs;
    const lmoe_experts &ex = l->experts;
    vs.cnt_words = (size_t)R * c.dn.nck;  // finished gate/up units per (route, down K chunk)
    vs.hq_bytes = al((size_t)R * ex.inter * 2) + al((size_t)ex.hidden * 2);
    vs.hs_bytes = al((size_t)R * (ex.inter / 32) * 8 + 16) + al((size_t)(ex.hidden / ex.gate.group_size) * 8 + 16);
    return vs;
}

Layout layer_layout(const lmoe_layer *l, int T, bool shared = false) {
    const int H = l->experts.hidden, I = l->experts.inter;
    const int R = T * l->router.top_k + (shared ? T : 0);
    return make_layout(T, R, H, I, H, l->router.n_experts + 1, l->router.n_experts,
                       router_ksplit(T, l->router.n_experts, H, l->experts.dtype == LMOE_F16), T,
                       vec_sizes(l, T, R));
}

// Layout of the prefill path: the shared routing regions and the y*w rows
// of make_layout (no GEMV panels), then the two tiled activation panels.
Layout prefill_layout(const lmoe_layer *l, int T, bool shared = false) {
    const int H = l->experts.hidden, I = l->experts.inter;
    const int R = T * l->router.top_k + (shared ? T : 0);
    const int buckets = l->router.n_experts + 1 + (shared ? 1 : 0);
    Layout L = make_layout(T, R, H, 0, H, buckets, l->router.n_experts,
                           router_ksplit(T, l->router.n_experts, H, l->experts.dtype == LMOE_F16), 0);
    L.prefill = true;
    L.pf_chunks = pf_max_chunks(buckets, R);
    L.pf_rows = pf_panel_rows(R, L.pf_chunks);
    size_t off = (L.total + 1023) & ~size_t(1023);
    L.pfx = off;
    off += (((size_t)L.pf_rows * H * 2) + 1023) & ~size_t(1023);
    L.pfh = off;
    off += (((size_t)L.pf_rows * I * 2) + 1023) & ~size_t(1023);
    L.total = off;
    return L;
}

template <typename P>
P *at(void *ws, size_t off) {
    return reinterpret_cast<P *>(static_cast<uint8_t *>(ws) + off);
}

QView view(const lmoe_qproj &p, int n_slots, int rows, int cols) {
    QView v;
    v.w = p.weight;
    v.s = static_cast<const uint16_t *>(p.scales);
    v.b = static_cast<const uint16_t *>(p.biases);
    v.words_per_row = cols * p.bits / 32;
    v.groups_per_row = cols / p.group_size;
    v.w_slot_stride = (int64_t)rows * v.words_per_row;
    v.sb_slot_stride = (int64_t)rows * v.groups_per_row;
    v.rows = rows;
    v.cols = cols;
    // the pre-tiled copy is in the stream format (StreamGeo); without its
    // geometry there is no copy to read
    StreamGeo sg;
    const bool sok = gemv_ok(p.bits, p.group_size) && stream_geo(rows, cols, p.bits, p.group_size, &sg) &&
                     sg.tg.SB == 16;
    v.tiles = sok ? static_cast<const uint8_t *>(p.tiles) : nullptr;
    v.tile_slot_stride = sok ? sg.slot : 0;
    (void)n_slots;
    return v;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_proj(const lmoe_qproj &p, int rows, int cols) {
    if (p.tiles) {
        if (!aligned16(p.tiles)) return LMOE_EINVAL;
    } else if (!p.weight || !p.scales || !p.biases) {
        return LMOE_EINVAL;
    }
    if (!quant_ok(p.bits, p.group_size)) return LMOE_EUNSUPPORTED;
    if (rows % 16 != 0 || cols % p.group_size != 0) return LMOE_EUNSUPPORTED;
    return LMOE_OK;
}

int check_experts(const lmoe_experts *e) {
    if (!e) return LMOE_EINVAL;
    if (e->n_slots < 1 || e->hidden <= 0 || e->inter <= 0) return LMOE_EINVAL;
    if (e->dtype != LMOE_BF16 && e->dtype != LMOE_F16) return LMOE_EUNSUPPORTED;
    int rc;
    if ((rc = check_proj(e->gate, e->inter, e->hidden))) return rc;
    if ((rc = check_proj(e->up, e->inter, e->hidden))) return rc;
    if ((rc = check_proj(e->down, e->hidden, e->inter))) return rc;
    if (e->gate.bits != e->up.bits || e->gate.group_size != e->up.group_size) return LMOE_EUNSUPPORTED;
    return LMOE_OK;
}

int check_layer(const lmoe_layer *l) {
    if (!l) return LMOE_EINVAL;
    int rc = check_experts(&l->experts);
    if (rc) return rc;
    const lmoe_router &r = l->router;
    if (r.n_experts < 1 || r.top_k < 1 || r.top_k > 16 || r.top_k > r.n_experts) return LMOE_EINVAL;
    if (r.n_experts > 32 * kRouterMaxEPL) return LMOE_EUNSUPPORTED;
    if (r.scoring < 0 || r.scoring > 2) return LMOE_EUNSUPPORTED;
    if (l->swiglu_mode != LMOE_SWIGLU_FUSED && l->swiglu_mode != LMOE_SWIGLU_STOCK) return LMOE_EUNSUPPORTED;
    if (!l->expert_slot) return LMOE_EINVAL;
    return LMOE_OK;
}

int cuda_rc(cudaError_t e) {
    if (e == cudaSuccess) return LMOE_OK;
    if (e == cudaErrorInvalidValue) return LMOE_EUNSUPPORTED;
    return LMOE_ECUDA;
}

// Runs dispatch for R routes into buckets [0, n_experts) (+ zero bucket).
int run_dispatch(const Layout &L, void *ws, const int32_t *idx, int R, int n_experts,
                 const int32_t *expert_slot, int n_slots, int chunk_tok, cudaStream_t st, bool drop_zero = false) {
    DispatchIn din;
    din.idx = idx;
    din.R = R;
    din.chunk_tok = chunk_tok;
    din.n_experts = n_experts;
    din.expert_slot = expert_slot;
    din.n_slots = n_slots;
    din.drop_zero = drop_zero ? 1 : 0;
    DispatchOut dout;
    dout.sorted_routes = at<int32_t>(ws, L.sorted);
    dout.chunks = at<Chunk>(ws, L.chunks);
    dout.n_chunks = at<int32_t>(ws, L.nchunks);
    dout.counts = at<int32_t>(ws, L.counts);
    dout.route_off = at<int32_t>(ws, L.roff);
    dout.blk = at<int32_t>(ws, L.dblk);
    int32_t *err = at<int32_t>(ws, L.status);
    if (R <= kDispatchSmallMaxRoutes && n_experts + 1 <= kDispatchSmallMaxBuckets)
        return cuda_rc(launch_dispatch_small(din, dout, err, st));
    return cuda_rc(launch_dispatch_large(din, dout, err, st));
}

GemvArgs gemv_base(const Layout &L, void *ws, int n_slots, int ntok_max) {
    GemvArgs a;
    std::memset(&a, 0, sizeof(a));
    a.chunks = at<Chunk>(ws, L.chunks);
    a.n_chunks = at<int32_t>(ws, L.nchunks);
    a.sorted_routes = at<int32_t>(ws, L.sorted);
    a.n_slots = n_slots;
    a.ntok_max = ntok_max;
    a.err = at<int32_t>(ws, L.status);
    return a;
}

// Largest chunk (routes of one expert per unit, at most one MMA n-tile of 8)
// whose shared-memory stages fit, capped by the routes one expert can get.
int chunk_for(int mode, int bits, int gs, int K, int cap) {
    int c = cap < kChunkTok ? cap : kChunkTok;
    GemvCfg cfg;
    while (c > 1 && !gemv_config(mode, bits, gs, K, c, &cfg)) --c;
    if (c < 1 || !gemv_config(mode, bits, gs, K, c, &cfg)) return 0;
    return c;
}

// The stream GEMVs run a projection when its pre-tiled copy is present (in
// the stream format; view() keeps the pointer only for that geometry); the
// row-major bulk-copy GEMV runs it otherwise.
// ntok: routes per chunk the launch serves; prow: panel rows it may read
// (tokens for gate/up, routes for down), resident in shared memory.
bool gateup_streamed(const lmoe_experts &ex, int ntok, int prow, StreamCfg *c) {
    const QView g = view(ex.gate, ex.n_slots, ex.inter, ex.hidden), u = view(ex.up, ex.n_slots, ex.inter, ex.hidden);
    return g.tiles && u.tiles && ex.gate.bits == ex.up.bits && ex.gate.group_size == ex.up.group_size &&
           stream_config(SMODE_GATEUP, ex.inter, ex.hidden, ex.gate.bits, ex.gate.group_size, false, ntok, prow, c);
}
bool down_streamed(const lmoe_experts &ex, bool local, int ntok, int prow, StreamCfg *c) {
    return view(ex.down, ex.n_slots, ex.hidden, ex.inter).tiles &&
           stream_config(SMODE_PAIR, ex.hidden, ex.inter, ex.down.bits, ex.down.group_size, local, ntok, prow, c);
}

// Routes per chunk: up to 8 (one MMA n-tile), also bounded by the stage plan
// of the row-major GEMV for the projections it runs.
int layer_chunk(const lmoe_layer *l, int T) {
    const lmoe_experts &ex = l->experts;
    StreamCfg sc;
    int c = T < kChunkTok ? T : kChunkTok;
    if (!gateup_streamed(ex, c, T, &sc)) {
        const int a = chunk_for(MODE_GATEUP, ex.gate.bits, ex.gate.group_size, ex.hidden, T);
        if (a < c) c = a;
    }
    if (c >= 1 && !down_streamed(ex, false, c, T * (l->router.top_k + 1), &sc)) {
        const int b = chunk_for(MODE_DOWN, ex.down.bits, ex.down.group_size, ex.inter, T);
        if (b < c) c = b;
    }
    return c;
}

// What the combine adds after the routed sum: the shared expert's rows
// (routes shared_base + t, when shared_base > 0) and a residual.
struct Extra {
    int shared_base = 0;
    const uint16_t *residual = nullptr;
    uint16_t *yw = nullptr;  // caller buffer for the per-route rows (default: the workspace's)
    // single token: the gate/up kernel selects the routing from the
    // router's scores (route_impl ran without its finisher)
    const float2 *tk_scores = nullptr;
    int32_t *idx_user = nullptr;
    float *w_user = nullptr;
    // the layer's natural activation rows (single-token kernel), or nullptr,
    // and whether the router already wrote their int8 pieces
    const uint16_t *x = nullptr;
    bool x_ready = false;
};

// The single-token kernel runs this call: its scratch is in the layout, x
// is 16-byte aligned and every projection has its stream copy.
bool vec_ready(const lmoe_layer *l, const Layout &L, const void *x, int shared_base, VecCfg *cfg) {
    const lmoe_experts &ex = l->experts;
    const int k = l->router.top_k, R = k + (shared_base > 0 ? 1 : 0);
    if (!x || !aligned16(x) || !L.vhq) return false;
    if (shared_base > 0 && shared_base != k) return false;
    if (!view(ex.gate, ex.n_slots, ex.inter, ex.hidden).tiles || !view(ex.up, ex.n_slots, ex.inter, ex.hidden).tiles ||
        !view(ex.down, ex.n_slots, ex.hidden, ex.inter).tiles)
        return false;
    return vec_geometry(l, R, cfg);
}
// x's int8 pieces and (sum, factor) follow those of h in their regions
uint8_t *vec_xq(const Layout &L, const lmoe_layer *l, int R, void *ws) {
    return at<uint8_t>(ws, L.vhq) + al((size_t)R * l->experts.inter * 2);
}
float2 *vec_xs(const Layout &L, const lmoe_layer *l, int R, void *ws) {
    return reinterpret_cast<float2 *>(at<uint8_t>(ws, L.vhs) + al((size_t)R * (l->experts.inter / 32) * 8 + 16));
}

// Single-token layer on the integer tensor-pipe kernel (lmoe_vec.cu): gate/up
// + SwiGLU into h (natural layout, in the h panel's region) and its int8
// pieces, then down + combine, in one launch.  Returns 1 (not taken) when the
// layer or call does not qualify: the caller then runs the stream / bulk-copy
// GEMVs.
int run_vec(const lmoe_layer *l, const Layout &L, void *ws, const float *route_w, void *out, cudaStream_t st,
            cudaEvent_t ev_gateup, const Extra &extra) {
    const lmoe_experts &ex = l->experts;
    const int H = ex.hidden, I = ex.inter, k = l->router.top_k;
    const int R = k + (extra.shared_base > 0 ? 1 : 0);
    VecCfg c;
    if (!vec_ready(l, L, extra.x, extra.shared_base, &c)) return 1;
    const QView qg = view(ex.gate, ex.n_slots, I, H), qu = view(ex.up, ex.n_slots, I, H);
    const QView qd = view(ex.down, ex.n_slots, H, I);
    VecArgs a;
    std::memset(&a, 0, sizeof(a));
    a.q0 = qg;
    a.q1 = qu;
    a.q2 = qd;
    a.x = extra.x;
    a.chunks = at<Chunk>(ws, L.chunks);
    a.n_chunks = at<int32_t>(ws, L.nchunks);
    a.sorted_routes = at<int32_t>(ws, L.sorted);
    a.n_slots = ex.n_slots;
    a.max_chunks = L.max_chunks;
    a.routes = R;
    a.shared_base = extra.shared_base;
    if (extra.tk_scores) {
        const lmoe_router &r = l->router;
        a.tk_scores = extra.tk_scores;
        a.tk_E = r.n_experts;
        a.tk_k = k;
        a.tk_norm = r.norm_topk;
        a.tk_scaling = r.routed_scaling;
        a.tk_expert_slot = l->expert_slot;
        a.tk_idx = at<int32_t>(ws, L.idx);
        a.tk_w = at<float>(ws, L.w);
        a.tk_idx_user = extra.idx_user;
        a.tk_w_user = extra.w_user;
        a.tk_sorted = at<int32_t>(ws, L.sorted);
        a.tk_chunks = at<Chunk>(ws, L.chunks);
        a.tk_nchunks = at<int32_t>(ws, L.nchunks);
    }
    a.hq = at<uint8_t>(ws, L.vhq);
    a.hs = at<float2>(ws, L.vhs);
    a.xq = vec_xq(L, l, R, ws);
    a.xs = vec_xs(L, l, R, ws);
    a.x_ready = extra.x_ready ? 1 : 0;
    a.limit = l->swiglu_limit;
    a.swiglu_mode = l->swiglu_mode;
    a.route_w = route_w;
    a.top_k = k;
    a.residual = extra.residual;
    a.out = static_cast<uint16_t *>(out);
    // per-route rows when asked for, or when there is no combined output
    a.yw = extra.yw ? extra.yw : (out ? nullptr : at<uint16_t>(ws, L.yw));
    a.hready = at<uint32_t>(ws, L.vcnt);
    a.err = at<int32_t>(ws, L.status);
    const int rc = cuda_rc(launch_vec_layer(ex.dtype == LMOE_F16, ex.gate.bits, ex.down.bits, ex.gate.group_size, a,
                                            c, st));
    if (rc) return rc;
    // one launch covers both projections: the gate/up event follows it
    if (ev_gateup && cudaEventRecord(ev_gateup, st) != cudaSuccess) return LMOE_ECUDA;
    return LMOE_OK;
}

// gate/up + SwiGLU then down + combine over an already dispatched layer.
// out == nullptr: the down kernel leaves the rounded y*w rows of every
// computed route in the workspace and combines nothing.
int run_experts(const lmoe_layer *l, const Layout &L, void *ws, int T, const float *route_w,
                void *out, cudaStream_t st, cudaEvent_t ev_gateup = nullptr, Extra extra = Extra()) {
    const lmoe_experts &ex = l->experts;
    const int H = ex.hidden, I = ex.inter, k = l->router.top_k;
    if (T == 1) {
        const int vr = run_vec(l, L, ws, route_w, out, st, ev_gateup, extra);
        if (vr <= 0) return vr;  // ran (or failed); 1: not taken
        if (extra.x_ready) return LMOE_EINVAL;  // the router wrote pieces, not the panel
    }
    const int ntok_max = layer_chunk(l, T);
    if (ntok_max < 1) return LMOE_EUNSUPPORTED;
    GemvArgs gu = gemv_base(L, ws, ex.n_slots, ntok_max);
    gu.q0 = view(ex.gate, ex.n_slots, I, H);
    gu.q1 = view(ex.up, ex.n_slots, I, H);
    gu.panel = at<uint16_t>(ws, L.xpanel);
    gu.sum16 = at<float>(ws, L.xsum);
    gu.route_div = k;
    gu.out = at<uint16_t>(ws, L.hpanel);
    gu.out_sum16 = at<float>(ws, L.hsum);
    gu.out_panel = 1;
    gu.out_bits = ex.down.bits;
    gu.out_gs = ex.down.group_size;
    gu.limit = l->swiglu_limit;
    gu.swiglu_mode = l->swiglu_mode;
    gu.shared_base = extra.shared_base;  // the shared expert's routes read token rows
    gu.chunks_est = T * k + (extra.shared_base > 0 ? T : 0);
#ifdef LMOE_PROFILE_TRACE
    gu.trace = g_trace;
    gu.trace_units = g_trace_units;
#endif
    const int f16 = ex.dtype == LMOE_F16;
    int rc;
    StreamCfg sc;
    if (gateup_streamed(ex, ntok_max, T, &sc)) {
        if (extra.tk_scores) {
            const lmoe_router &r = l->router;
            gu.tk_scores = extra.tk_scores;
            gu.tk_E = r.n_experts;
            gu.tk_k = k;
            gu.tk_norm = r.norm_topk;
            gu.tk_scaling = r.routed_scaling;
            gu.tk_expert_slot = l->expert_slot;
            gu.tk_idx = at<int32_t>(ws, L.idx);
            gu.tk_w = at<float>(ws, L.w);
            gu.tk_idx_user = extra.idx_user;
            gu.tk_w_user = extra.w_user;
            gu.tk_sorted = at<int32_t>(ws, L.sorted);
            gu.tk_chunks = at<Chunk>(ws, L.chunks);
            gu.tk_nchunks = at<int32_t>(ws, L.nchunks);
        }
        rc = cuda_rc(launch_stream(SMODE_GATEUP, f16, ex.gate.bits, ex.gate.group_size, gu, sc, L.max_chunks, st));
    } else {
        if (extra.tk_scores) return LMOE_EINVAL;  // fusion is only planned for the stream kernel
        // row-major arrays through the bulk-copy GEMV
        if (!ex.gate.weight || !ex.up.weight) return LMOE_EINVAL;
        gu.q0.tiles = gu.q1.tiles = nullptr;
        rc = cuda_rc(launch_gemv(MODE_GATEUP, f16, ex.gate.bits, ex.gate.group_size, gu, L.max_chunks, st));
    }
    if (rc) return rc;
    if (ev_gateup && cudaEventRecord(ev_gateup, st) != cudaSuccess) return LMOE_ECUDA;
    GemvArgs dn = gemv_base(L, ws, ex.n_slots, ntok_max);
    dn.q0 = view(ex.down, ex.n_slots, H, I);
    dn.panel = at<uint16_t>(ws, L.hpanel);
    dn.sum16 = at<float>(ws, L.hsum);
    dn.route_div = 1;
    dn.out = extra.yw ? extra.yw : at<uint16_t>(ws, L.yw);
    dn.route_w = route_w;
    dn.top_k = k;
    dn.counters = out ? at<uint32_t>(ws, L.cnt) : nullptr;
    dn.combined = static_cast<uint16_t *>(out);
    dn.n_tok = T;
    dn.shared_base = extra.shared_base;
    dn.residual = extra.residual;
    dn.chunks_est = gu.chunks_est;
    const int dprow = T * k + (extra.shared_base > 0 ? T : 0);  // h panel rows: routed + shared routes
    if (down_streamed(ex, false, ntok_max, dprow, &sc)) {
        // Few tokens: blocks own row pairs and combine locally.  More
        // tokens (or no combine): units spread over every SM, then the
        // route-order combine kernel (the same arithmetic).
        StreamCfg lc;
        const int grid = down2_grid(sc.pairs);
        if (out && T <= kDown2MaxTokens && grid > 0 && down_streamed(ex, true, ntok_max, dprow, &lc)) {
            lc.grid = grid;
            dn.counters = nullptr;
            return cuda_rc(launch_stream(SMODE_PAIR, f16, ex.down.bits, ex.down.group_size, dn, lc, L.max_chunks, st));
        }
        dn.counters = nullptr;
        dn.combined = nullptr;
        rc = cuda_rc(launch_stream(SMODE_PAIR, f16, ex.down.bits, ex.down.group_size, dn, sc, L.max_chunks, st));
        if (rc || !out) return rc;
        return cuda_rc(launch_pf_combine(f16, dn.out, T, H, k, static_cast<uint16_t *>(out), st, extra.shared_base,
                                         extra.residual));
    }
    if (!ex.down.weight) return LMOE_EINVAL;
    dn.q0.tiles = nullptr;  // row-major arrays through the bulk-copy GEMV
    // Few tokens: blocks own row pairs and combine locally (no device-wide
    // counters or fences at the tail).  More tokens: row tiles spread over
    // every SM and the counter-based combine.  Without a combine the paired
    // tiles serve any token count.
    GemvCfg d2;
    const int mode = ((T <= kDown2MaxTokens || !out) && H % 32 == 0 && down2_grid(H / 32) > 0 &&
                      gemv_config(MODE_DOWN2, ex.down.bits, ex.down.group_size, I, ntok_max, &d2))
                         ? MODE_DOWN2
                         : MODE_DOWN;
    if (mode == MODE_DOWN2) dn.q1 = dn.q0;
    return cuda_rc(launch_gemv(mode, ex.dtype == LMOE_F16, ex.down.bits, ex.down.group_size, dn, L.max_chunks, st));
}

// Prefill path over an already dispatched layer (chunks of at most kPfNmax
// routes): x rows -> tiled panel, gate/up + SwiGLU on tcgen05 (h straight
// into the down panel), down on tcgen05 (y*w rows), combine per token.
int run_experts_pf(const lmoe_layer *l, const Layout &L, void *ws, const void *x, int T, const float *route_w,
                   void *out, cudaStream_t st, cudaEvent_t ev_gateup = nullptr, int x_stride = 0,
                   Extra extra = Extra()) {
    const lmoe_experts &ex = l->experts;
    const int H = ex.hidden, I = ex.inter, k = l->router.top_k;
    const int f16 = ex.dtype == LMOE_F16;
    PfPanelArgs pa;
    std::memset(&pa, 0, sizeof(pa));
    pa.x = static_cast<const uint16_t *>(x);
    pa.K = H;
    pa.x_stride = x_stride;
    pa.shared_base = extra.shared_base;
    pa.route_div = k;
    pa.chunks = at<Chunk>(ws, L.chunks);
    pa.n_chunks = at<int32_t>(ws, L.nchunks);
    pa.sorted_routes = at<int32_t>(ws, L.sorted);
    pa.panel = at<uint8_t>(ws, L.pfx);
    pa.prow = L.pf_rows;
    pa.bits = ex.gate.bits;
    int rc = cuda_rc(launch_pf_panel(pa, L.pf_chunks, st));
    if (rc) return rc;
    PfArgs g;
    std::memset(&g, 0, sizeof(g));
    const QView qg = view(ex.gate, ex.n_slots, I, H), qu = view(ex.up, ex.n_slots, I, H);
    rc = cuda_rc(pf_prepare(g, PF_GATEUP, qg, qu, ex.gate.bits, ex.gate.group_size, ex.n_slots));
    if (rc) return rc;
    g.panel = pa.panel;
    g.prow = L.pf_rows;
    g.K = H;
    g.chunks = pa.chunks;
    g.n_chunks = pa.n_chunks;
    g.sorted_routes = pa.sorted_routes;
    g.rbn = I / 128;
    g.hpanel = at<uint8_t>(ws, L.pfh);
    g.hprow = L.pf_rows;
    g.hbits = ex.down.bits;
    g.limit = l->swiglu_limit;
    g.swiglu_mode = l->swiglu_mode;
    g.err = at<int32_t>(ws, L.status);
    rc = cuda_rc(launch_pf_gemm(PF_GATEUP, f16, ex.gate.bits, ex.gate.group_size, g, st));
    if (rc) return rc;
    if (ev_gateup && cudaEventRecord(ev_gateup, st) != cudaSuccess) return LMOE_ECUDA;
    PfArgs d = g;
    const QView qd = view(ex.down, ex.n_slots, H, I);
    rc = cuda_rc(pf_prepare(d, PF_DOWN, qd, qd, ex.down.bits, ex.down.group_size, ex.n_slots));
    if (rc) return rc;
    d.panel = g.hpanel;
    d.K = I;
    d.rbn = H / 256;
    d.hpanel = nullptr;
    d.yw = at<uint16_t>(ws, L.yw);
    d.H = H;
    d.route_w = route_w;
    rc = cuda_rc(launch_pf_gemm(PF_DOWN, f16, ex.down.bits, ex.down.group_size, d, st));
    if (rc || !out) return rc;  // out == nullptr: the caller combines the y*w rows
    return cuda_rc(launch_pf_combine(f16, d.yw, T, H, k, static_cast<uint16_t *>(out), st, extra.shared_base,
                                     extra.residual));
}

// The prefill kernels read the row-major arena arrays in 16-byte pieces.
bool layer_pf_ok(const lmoe_layer *l) {
    const lmoe_experts &ex = l->experts;
    const lmoe_qproj *ps[3] = {&ex.gate, &ex.up, &ex.down};
    for (const lmoe_qproj *p : ps)
        if (!p->weight || !p->scales || !p->biases || !aligned16(p->weight) || !aligned16(p->scales) ||
            !aligned16(p->biases))
            return false;
    return pf_supported(ex.hidden, ex.inter, ex.gate.bits, ex.gate.group_size, PF_GATEUP) &&
           pf_supported(ex.inter, ex.hidden, ex.down.bits, ex.down.group_size, PF_DOWN);
}

// The decode GEMVs need supported bit widths and, for both projections, a
// shared-memory plan with at least two stages of one route (the tile layout
// needs a power-of-two number of 16-byte chunks per code row).
bool layer_gemv_ok(const lmoe_layer *l) {
    const lmoe_experts &ex = l->experts;
    return gemv_ok(ex.gate.bits, ex.gate.group_size) && gemv_ok(ex.up.bits, ex.up.group_size) &&
           gemv_ok(ex.down.bits, ex.down.group_size) && layer_chunk(l, 1) >= 1;
}

// Router kernels: 16-byte column loads over 256-column warp chunks (the last
// may be partial) and 64-column tensor-core stages for many tokens.
bool router_hidden_ok(int hidden) { return hidden > 0 && hidden % 64 == 0; }

// 1 = prefill grouped GEMM, 0 = decode GEMVs, -1 = the requested path is unavailable
int choose_path(const lmoe_layer *l, int T, int path) {
    const bool dec = layer_gemv_ok(l);
    if (path == LMOE_PATH_DECODE) return dec ? 0 : -1;
    const bool ok = layer_pf_ok(l);
    if (path == LMOE_PATH_PREFILL) return ok ? 1 : -1;
    if (path != LMOE_PATH_AUTO) return -1;
    if (!dec) return ok ? 1 : -1;
    const long routes = (long)T * l->router.top_k;
    return ok && routes >= LMOE_PREFILL_MIN_ROUTES &&
           4 * routes >= (long)LMOE_PREFILL_ROUTES_PER_4_EXPERTS * l->router.n_experts;
}

// ---- expert-parallel receive side
// The local layer: the rank's experts, its slot table and the route width;
// its router is never evaluated (n_experts = local experts, top_k may exceed it).
int check_ep_local(const lmoe_layer *l) {
    if (!l) return LMOE_EINVAL;
    int rc = check_experts(&l->experts);
    if (rc) return rc;
    const lmoe_router &r = l->router;
    if (r.n_experts < 1 || r.top_k < 1 || r.top_k > 16) return LMOE_EINVAL;
    if (r.n_experts + 1 > kDispatchSmallMaxBuckets) return LMOE_EUNSUPPORTED;
    if (l->swiglu_mode != LMOE_SWIGLU_FUSED && l->swiglu_mode != LMOE_SWIGLU_STOCK) return LMOE_EUNSUPPORTED;
    if (!l->expert_slot) return LMOE_EINVAL;
    return LMOE_OK;
}

// Path of the received routes: AUTO applies the layer rule to the routes a
// rank receives on average, rows * top_k / world (each rank sends its
// tokens' top_k routes spread over the world).
int ep_path(const lmoe_layer *l, int rows, int world, int path) {
    const bool dec = layer_gemv_ok(l);
    if (path == LMOE_PATH_DECODE) return dec ? 0 : -1;
    const bool ok = layer_pf_ok(l);
    if (path == LMOE_PATH_PREFILL) return ok ? 1 : -1;
    if (path != LMOE_PATH_AUTO) return -1;
    if (!dec) return ok ? 1 : -1;
    const long routes = (long)rows * l->router.top_k / world;
    return ok && routes >= LMOE_PREFILL_MIN_ROUTES &&
           4 * routes >= (long)LMOE_PREFILL_ROUTES_PER_4_EXPERTS * l->router.n_experts;
}

// Workspace of the receive side: the routing regions over rows * top_k
// route slots (no router logits), the decode panels or the prefill panels,
// and the y*w rows.
Layout ep_layout(const lmoe_layer *l, int rows, bool pf) {
    const int H = l->experts.hidden, I = l->experts.inter;
    const int R = rows * l->router.top_k;
    const int buckets = l->router.n_experts + 1;
    if (!pf) return make_layout(rows, R, H, I, H, buckets, 1, 1, rows);
    Layout L = make_layout(rows, R, H, 0, H, buckets, 1, 1, 0);
    L.prefill = true;
    L.pf_chunks = pf_max_chunks(buckets, R);
    L.pf_rows = pf_panel_rows(R, L.pf_chunks);
    size_t off = (L.total + 1023) & ~size_t(1023);
    L.pfx = off;
    off += (((size_t)L.pf_rows * H * 2) + 1023) & ~size_t(1023);
    L.pfh = off;
    off += (((size_t)L.pf_rows * I * 2) + 1023) & ~size_t(1023);
    L.total = off;
    return L;
}

}  // namespace

extern "C" {

int lmoe_version(void) { return LMOE_ABI_VERSION; }

#ifdef LMOE_PROFILE_TRACE
// Profiling builds only (not declared in lmoe.h): while buf is non-NULL,
// every gate/up GEMV records %globaltimer stamps into
// buf[block][unit][8] (device memory owned by the caller).
void lmoe_profile_trace(uint64_t *buf, int32_t units_per_block) {
    g_trace = buf;
    g_trace_units = buf ? units_per_block : 0;
}
#endif

const char *lmoe_strerror(int status) {
    switch (status) {
        case LMOE_OK: return "ok";
        case LMOE_EINVAL: return "invalid argument";
        case LMOE_EUNSUPPORTED: return "unsupported geometry, bit width or group size";
        case LMOE_EINDEX: return "expert id or arena slot out of range";
        case LMOE_ECUDA: return "CUDA error";
        case LMOE_EWORKSPACE: return "workspace too small";
        default: return "unknown status";
    }
}

size_t lmoe_workspace_size(const lmoe_layer *layer, int32_t max_tokens) {
    return lmoe_workspace_size_path(layer, max_tokens, LMOE_PATH_AUTO);
}

size_t lmoe_workspace_size_routes(int32_t max_routes, int32_t hidden, int32_t inter, int32_t n_slots) {
    if (max_routes < 0 || hidden <= 0 || n_slots < 1) return 0;
    const int R = max_routes > 0 ? max_routes : 1;
    const int K = hidden > inter ? hidden : inter;
    return make_layout(R, R, K, 0, 0, n_slots + 1, 1, 1, R).total;
}

int lmoe_workspace_init(void *workspace, size_t bytes, void *stream) {
    if (!workspace || bytes == 0) return LMOE_EINVAL;
    return cuda_rc(cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)));
}

int lmoe_workspace_status(void *workspace, void *stream) {
    if (!workspace) return LMOE_EINVAL;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t host = 0;
    cudaError_t e = cudaMemcpyAsync(&host, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return LMOE_ECUDA;
    if (host != 0) {
        e = cudaMemsetAsync(workspace, 0, sizeof(int32_t), st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return LMOE_ECUDA;
        return host;
    }
    return LMOE_OK;
}

// Router (+ top-k, + dispatch when `l` is given).  In the decode regime the
// router kernel's last block runs top-k (and dispatch) itself: one launch.
// Element-wise scores (score, score + bias) follow the logit partials.
static float2 *router_scores(const Layout &L, void *ws, int ksplit, int T, int E) {
    return reinterpret_cast<float2 *>(at<float>(ws, L.partial) + (((size_t)ksplit * T * E + 1) & ~size_t(1)));
}

// Single-token decode whose top-k runs inside the stream gate/up kernel:
// element-wise scoring (no softmax over the experts, no hash routing), one
// logit split, no shared-expert routes, and the streamed gate/up kernel.
static bool topk_fusable(const lmoe_layer *l, int T, const int32_t *hash_idx, bool shared, int pf) {
    if (T != 1 || hash_idx || shared || pf) return false;
    const lmoe_router &r = l->router;
    if (r.scoring == LMOE_SCORE_SOFTMAX || r.n_experts > 32 * kRouterMaxEPL || r.top_k > 16) return false;
    if (router_ksplit(1, r.n_experts, l->experts.hidden, l->experts.dtype == LMOE_F16) != 1) return false;
    StreamCfg sc;
    return gateup_streamed(l->experts, layer_chunk(l, 1), 1, &sc);
}

// fused: the top-k and dispatch are left to the stream gate/up kernel
// (topk_fusable holds); only the logit blocks run here.
// vec_shared_base >= 0: the layer call's shared-expert route base (0: none);
// when the single-token kernel will run the call, the router writes x's int8
// pieces for it instead of the GEMV panel (*x_pieces = true).
static int route_impl(const lmoe_router &r, int H, int dtype, const lmoe_layer *l, const Layout &L, const void *x,
                      int T, int32_t *idx_user, float *w_user, void *ws, cudaStream_t st,
                      const int32_t *hash_idx = nullptr, bool fused = false, int vec_shared_base = -1,
                      bool *x_pieces = nullptr) {
    if (x_pieces) *x_pieces = false;
    const int k = r.top_k;
    const int R = T * k;
    const int ksplit = router_ksplit(T, r.n_experts, H, dtype == LMOE_F16);
    const int chunk_tok = l ? (L.prefill ? kPfNmax : layer_chunk(l, T)) : kChunkTok;
    if (chunk_tok < 1) return LMOE_EUNSUPPORTED;
    RouterArgs a;
    std::memset(&a, 0, sizeof(a));
    a.x = static_cast<const uint16_t *>(x);
    a.T = T;
    a.H = H;
    a.wg = static_cast<const uint16_t *>(r.weight);
    a.bias = r.bias;
    a.E = r.n_experts;
    a.top_k = k;
    a.scoring = r.scoring;
    a.norm_topk = r.norm_topk;
    a.scaling = r.routed_scaling;
    a.partial = at<float>(ws, L.partial);
    a.ksplit = ksplit;
    // element-wise scorings are finished by the logit blocks themselves,
    // unless the logits are split over the hidden dimension (then the top-k
    // sums the splits and scores)
    a.scores = (r.scoring == LMOE_SCORE_SOFTMAX || ksplit > 1) ? nullptr
                                                                 : router_scores(L, ws, ksplit, T, r.n_experts);
    if (l) {
        // this call's combine counters start at zero whatever the workspace
        // held before (another token count or entry point)
        a.zero = at<uint32_t>(ws, L.cnt);
        a.zero_words = static_cast<int32_t>((L.zero_end - L.cnt) / 4);  // combine and unit counters
        if (!L.prefill) {  // the decode GEMVs read x through the router's panel
            a.xpanel = at<uint16_t>(ws, L.xpanel);
            a.xsum16 = at<float>(ws, L.xsum);
            a.pbits = l->experts.gate.bits;
            a.pgs = l->experts.gate.group_size;
            if (T == 1 && vec_shared_base >= 0 && vec_ready(l, L, x, vec_shared_base, nullptr)) {
                // the single-token kernel reads x's int8 pieces instead
                const int Rv = r.top_k + (vec_shared_base > 0 ? 1 : 0);
                a.xq = vec_xq(L, l, Rv, ws);
                a.xs = vec_xs(L, l, Rv, ws);
                a.xpanel = nullptr;
                a.xsum16 = nullptr;
                if (x_pieces) *x_pieces = true;
            }
        }
    }
    a.act_f16 = dtype == LMOE_F16;
    a.hash_idx = hash_idx;
    a.counter = at<uint32_t>(ws, L.status) + 1;
    a.idx_ws = at<int32_t>(ws, L.idx);
    a.w_ws = at<float>(ws, L.w);
    a.idx_user = idx_user;
    a.w_user = w_user;
    a.err = at<int32_t>(ws, L.status);
    a.din.idx = a.idx_ws;
    a.din.R = R;
    a.din.chunk_tok = chunk_tok;
    a.din.n_experts = a.E;
    a.din.expert_slot = l ? l->expert_slot : nullptr;
    a.din.n_slots = l ? l->experts.n_slots : 0;
    a.dout.sorted_routes = at<int32_t>(ws, L.sorted);
    a.dout.chunks = at<Chunk>(ws, L.chunks);
    a.dout.n_chunks = at<int32_t>(ws, L.nchunks);
    a.dout.counts = at<int32_t>(ws, L.counts);
    a.dout.route_off = at<int32_t>(ws, L.roff);
    a.dout.blk = at<int32_t>(ws, L.dblk);
    const bool small_topk = T <= 64;
    const bool small_disp = l && R <= kDispatchSmallMaxRoutes && a.E + 1 <= kDispatchSmallMaxBuckets;
    a.finish = small_topk ? 1 : 0;
    a.do_dispatch = (small_topk && small_disp) ? 1 : 0;
    if (fused) {
        if (!l || !a.scores || T != 1) return LMOE_EINVAL;
        a.finish = 0;
        a.do_dispatch = 0;
        return cuda_rc(launch_router(a, ksplit, st));
    }
    int rc;
    if (!small_topk && !a.act_f16) {
        // many tokens: logits on the tensor cores; the decode GEMVs' panel
        // (when this layout has one) from the panel kernel
        rc = cuda_rc(launch_router_logits_mma(a, st));
        if (rc) return rc;
        if (a.xpanel) {
            PanelArgs pa;
            std::memset(&pa, 0, sizeof(pa));
            pa.x = a.x;
            pa.rows = T;
            pa.K = H;
            pa.panel = a.xpanel;
            pa.sum16 = a.xsum16;
            pa.bits = a.pbits;
            pa.gs = a.pgs;
            pa.act_f16 = 0;
            rc = cuda_rc(launch_panel(pa, st));
            if (rc) return rc;
        }
    } else {
        rc = cuda_rc(launch_router(a, ksplit, st));
        if (rc) return rc;
    }
    if (!small_topk) {
        TopkArgs tk;
        tk.partial = a.partial;
        tk.scores = a.scores;
        tk.ksplit = ksplit;
        tk.T = T;
        tk.E = a.E;
        tk.top_k = k;
        tk.scoring = a.scoring;
        tk.norm_topk = a.norm_topk;
        tk.scaling = a.scaling;
        tk.bias = a.bias;
        tk.idx_ws = a.idx_ws;
        tk.w_ws = a.w_ws;
        tk.idx_user = idx_user;
        tk.w_user = w_user;
        tk.hash_idx = hash_idx;
        rc = cuda_rc(launch_topk(tk, st));
        if (rc) return rc;
    }
    if (!l || a.do_dispatch) return LMOE_OK;
    return run_dispatch(L, ws, a.idx_ws, R, a.E, l->expert_slot, l->experts.n_slots, chunk_tok, st);
}

int check_router(const lmoe_router *r, int hidden) {
    if (!r || !r->weight || hidden <= 0) return LMOE_EINVAL;
    if (r->n_experts < 1 || r->top_k < 1 || r->top_k > 16 || r->top_k > r->n_experts) return LMOE_EINVAL;
    if (r->n_experts > 32 * kRouterMaxEPL) return LMOE_EUNSUPPORTED;
    if (r->scoring < 0 || r->scoring > 2) return LMOE_EUNSUPPORTED;
    if (!router_hidden_ok(hidden)) return LMOE_EUNSUPPORTED;
    return LMOE_OK;
}

size_t lmoe_workspace_size_route(const lmoe_router *router, int32_t hidden, int32_t max_tokens) {
    if (check_router(router, hidden) || max_tokens < 0) return 0;
    const int T = max_tokens > 0 ? max_tokens : 1;
    // the bf16 split count bounds the f16 one (1)
    return make_layout(T, T * router->top_k, 0, 0, 0, router->n_experts + 1, router->n_experts,
                       router_ksplit(T, router->n_experts, hidden, false), 0).total;
}

static int route_entry(const lmoe_router *router, int32_t hidden, int32_t dtype, const void *x, int32_t tokens,
                       const int32_t *hash_idx, int32_t *idx, float *w, void *workspace, size_t ws_bytes,
                       void *stream) {
    int rc = check_router(router, hidden);
    if (rc) return rc;
    if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_EUNSUPPORTED;
    if (tokens < 0 || (tokens > 0 && (!x || !idx || !w || !workspace))) return LMOE_EINVAL;
    if (tokens == 0) return LMOE_OK;
    const Layout L = make_layout(tokens, tokens * router->top_k, 0, 0, 0, router->n_experts + 1, router->n_experts,
                                 router_ksplit(tokens, router->n_experts, hidden, dtype == LMOE_F16), 0);
    if (ws_bytes < L.total) return LMOE_EWORKSPACE;
    return route_impl(*router, hidden, dtype, nullptr, L, x, tokens, idx, w, workspace,
                      static_cast<cudaStream_t>(stream), hash_idx);
}

int lmoe_route_hashed(const lmoe_router *router, int32_t hidden, int32_t dtype, const void *x, int32_t tokens,
                      const int32_t *hash_idx, int32_t *idx, float *w, void *workspace, size_t ws_bytes,
                      void *stream) {
    if (tokens > 0 && !hash_idx) return LMOE_EINVAL;
    return route_entry(router, hidden, dtype, x, tokens, hash_idx, idx, w, workspace, ws_bytes, stream);
}

int lmoe_route(const lmoe_router *router, int32_t hidden, int32_t dtype, const void *x, int32_t tokens,
               int32_t *idx, float *w, void *workspace, size_t ws_bytes, void *stream) {
    return route_entry(router, hidden, dtype, x, tokens, nullptr, idx, w, workspace, ws_bytes, stream);
}

// shared_slot >= 0: the block's shared expert lives in that arena slot (same
// quantisation as the routed experts) and its row is added to the routed
// sum; residual (may be NULL, may alias out) is added last.
static int layer_entry(const lmoe_layer *layer, const void *x, int32_t tokens, const int32_t *hash_idx, void *out,
                       int32_t *idx, float *w, void *workspace, size_t ws_bytes, void *stream, int32_t path,
                       void *ev_routed, void *ev_gateup, int32_t shared_slot = -1, const void *residual = nullptr,
                       bool events_only = false) {
    int rc = check_layer(layer);
    if (rc) return rc;
    if (tokens < 0 || (tokens > 0 && (!x || !out || !workspace))) return LMOE_EINVAL;
    if (shared_slot >= layer->experts.n_slots) return LMOE_EINVAL;
    if (tokens == 0) return LMOE_OK;
    if (!router_hidden_ok(layer->experts.hidden)) return LMOE_EUNSUPPORTED;
    const int pf = choose_path(layer, tokens, path);
    if (pf < 0) return LMOE_EUNSUPPORTED;
    const bool shared = shared_slot >= 0;
    const Layout L = pf ? prefill_layout(layer, tokens, shared) : layer_layout(layer, tokens, shared);
    if (ws_bytes < L.total) return LMOE_EWORKSPACE;
    if (residual && !aligned16(residual)) return LMOE_EINVAL;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the routing is only complete after gate/up when the top-k is fused:
    // a caller that waits on ev_routed gets the separate finisher (unless the
    // events only mark launch boundaries for timing)
    const bool fused = (!ev_routed || events_only) && topk_fusable(layer, tokens, hash_idx, shared_slot >= 0, pf);
    bool x_pieces = false;
    rc = route_impl(layer->router, layer->experts.hidden, layer->experts.dtype, layer, L, x, tokens, idx, w,
                    workspace, st, hash_idx, fused, shared ? tokens * layer->router.top_k : 0, &x_pieces);
    if (rc) return rc;
    Extra ex;
    ex.residual = static_cast<const uint16_t *>(residual);
    ex.x = static_cast<const uint16_t *>(x);
    ex.x_ready = x_pieces;
    if (fused) {
        ex.tk_scores = router_scores(L, workspace, 1, tokens, layer->router.n_experts);
        ex.idx_user = idx;
        ex.w_user = w;
    }
    if (shared) {
        ex.shared_base = tokens * layer->router.top_k;
        const int ct = pf ? kPfNmax : layer_chunk(layer, tokens);
        rc = cuda_rc(launch_shared_chunks(at<Chunk>(workspace, L.chunks), at<int32_t>(workspace, L.nchunks),
                                          at<int32_t>(workspace, L.sorted), at<float>(workspace, L.w),
                                          ex.shared_base, tokens, ct, shared_slot, st));
        if (rc) return rc;
    }
    if (ev_routed && cudaEventRecord(static_cast<cudaEvent_t>(ev_routed), st) != cudaSuccess) return LMOE_ECUDA;
    const float *rw = at<float>(workspace, L.w);
    if (pf)
        return run_experts_pf(layer, L, workspace, x, tokens, rw, out, st, static_cast<cudaEvent_t>(ev_gateup), 0, ex);
    return run_experts(layer, L, workspace, tokens, rw, out, st, static_cast<cudaEvent_t>(ev_gateup), ex);
}

int lmoe_moe_layer_path(const lmoe_layer *layer, const void *x, int32_t tokens, void *out, int32_t *idx, float *w,
                        void *workspace, size_t ws_bytes, void *stream, int32_t path, void *ev_routed,
                        void *ev_gateup) {
    return layer_entry(layer, x, tokens, nullptr, out, idx, w, workspace, ws_bytes, stream, path, ev_routed,
                       ev_gateup);
}

int lmoe_moe_layer_timed(const lmoe_layer *layer, const void *x, int32_t tokens, void *out, int32_t *idx, float *w,
                         void *workspace, size_t ws_bytes, void *stream, void *ev_router, void *ev_experts) {
    return layer_entry(layer, x, tokens, nullptr, out, idx, w, workspace, ws_bytes, stream, LMOE_PATH_AUTO, ev_router,
                       ev_experts, -1, nullptr, true);
}

int lmoe_moe_layer_host(const lmoe_layer *layer, const void *x_host, int32_t tokens, void *out_host,
                        void *x_stage, void *workspace, size_t ws_bytes, void *stream, int32_t path) {
    int rc = check_layer(layer);
    if (rc) return rc;
    if (tokens < 0 || (tokens > 0 && (!x_host || !out_host || !x_stage))) return LMOE_EINVAL;
    if (tokens == 0) return LMOE_OK;
    void *xd = nullptr, *od = nullptr;
    if (cudaHostGetDevicePointer(&xd, const_cast<void *>(x_host), 0) != cudaSuccess ||
        cudaHostGetDevicePointer(&od, out_host, 0) != cudaSuccess) {
        (void)cudaGetLastError();  // not page-locked, mapped host memory
        return LMOE_EINVAL;
    }
    if ((reinterpret_cast<uintptr_t>(xd) | reinterpret_cast<uintptr_t>(x_stage)) & 15u) return LMOE_EINVAL;
    const size_t bytes = (size_t)tokens * layer->experts.hidden * 2;
    if (bytes & 15u) return LMOE_EUNSUPPORTED;  // the staging kernel moves 16-byte chunks
    rc = cuda_rc(launch_stage_rows(x_stage, xd, bytes, static_cast<cudaStream_t>(stream)));
    if (rc) return rc;
    return layer_entry(layer, x_stage, tokens, nullptr, od, nullptr, nullptr, workspace, ws_bytes, stream, path,
                       nullptr, nullptr);
}

int lmoe_moe_layer_hashed(const lmoe_layer *layer, const void *x, int32_t tokens, const int32_t *hash_idx,
                          void *out, int32_t *idx, float *w, void *workspace, size_t ws_bytes, void *stream,
                          int32_t path) {
    if (tokens > 0 && !hash_idx) return LMOE_EINVAL;
    return layer_entry(layer, x, tokens, hash_idx, out, idx, w, workspace, ws_bytes, stream, path, nullptr,
                       nullptr);
}

int lmoe_moe_block(const lmoe_layer *layer, int32_t shared_slot, const void *x, int32_t tokens,
                   const void *residual, void *out, int32_t *idx, float *w, void *workspace, size_t ws_bytes,
                   void *stream, int32_t path) {
    return layer_entry(layer, x, tokens, nullptr, out, idx, w, workspace, ws_bytes, stream, path, nullptr, nullptr,
                       shared_slot < 0 ? -1 : shared_slot, residual);
}

size_t lmoe_workspace_size_block(const lmoe_layer *layer, int32_t max_tokens, int32_t path) {
    if (check_layer(layer) || max_tokens < 0) return 0;
    const int T = max_tokens > 0 ? max_tokens : 1;
    const int pf = choose_path(layer, T, path);
    if (pf < 0) return 0;
    if (path == LMOE_PATH_PREFILL) return prefill_layout(layer, T, true).total;
    size_t n = layer_layout(layer, T, true).total;
    if (pf) {
        const size_t p = prefill_layout(layer, T, true).total;
        if (p > n) n = p;
    }
    return n;
}

size_t lmoe_workspace_size_path(const lmoe_layer *layer, int32_t max_tokens, int32_t path) {
    if (check_layer(layer) || max_tokens < 0) return 0;
    const int T = max_tokens > 0 ? max_tokens : 1;
    const int pf = choose_path(layer, T, path);
    if (pf < 0) return 0;
    if (path == LMOE_PATH_PREFILL) return prefill_layout(layer, T).total;
    size_t n = layer_layout(layer, T).total;
    // AUTO may take either path at token counts up to T; both layouts grow with T
    if (pf) {
        const size_t p = prefill_layout(layer, T).total;
        if (p > n) n = p;
    }
    return n;
}

int lmoe_moe_layer_staged(const lmoe_layer *layer, const void *x, int32_t tokens, void *out, int32_t *idx,
                          float *w, void *workspace, size_t ws_bytes, void *stream, void *ev_routed,
                          void *ev_gateup) {
    return lmoe_moe_layer_path(layer, x, tokens, out, idx, w, workspace, ws_bytes, stream, LMOE_PATH_AUTO,
                               ev_routed, ev_gateup);
}

int lmoe_moe_layer(const lmoe_layer *layer, const void *x, int32_t tokens, void *out, int32_t *idx,
                   float *w, void *workspace, size_t ws_bytes, void *stream) {
    return lmoe_moe_layer_path(layer, x, tokens, out, idx, w, workspace, ws_bytes, stream, LMOE_PATH_AUTO, nullptr,
                               nullptr);
}

}  // extern "C"

// ------------------------------------------------------------ allocation-free layer
// Some callers cannot allocate device memory for a workspace: a serving loop
// whose device memory is owned by another allocator, a host runtime that
// forbids allocation on its request path, or a foreign-language binding with
// no device allocator at all.  lmoe_moe_layer_static serves them by keeping
// its scratch in this file-scope device array, which every GPU that loads
// the library holds until the process exits.
static __device__ __align__(256) uint8_t g_lmoe_static_ws[LMOE_STATIC_WORKSPACE_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void *g_static_ptr[kMaxDevices] = {};

// Device address of the static scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is looked up
// once per device with that device current.
int static_workspace(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LMOE_ECUDA;
    if (dev < 0 || dev >= kMaxDevices) return LMOE_EUNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_ptr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_lmoe_static_ws) != cudaSuccess || !p) return LMOE_ECUDA;
        g_static_ptr[dev] = p;
    }
    *out = g_static_ptr[dev];
    return LMOE_OK;
}
}  // namespace

extern "C" {

size_t lmoe_static_workspace_bytes(void) { return LMOE_STATIC_WORKSPACE_BYTES; }

int lmoe_moe_layer_static(const lmoe_layer *layer, const void *x, int32_t tokens, void *out, int32_t *idx,
                          float *w, void *stream) {
    // every check that can reject the call runs before anything is enqueued
    int rc = check_layer(layer);
    if (rc) return rc;
    if (tokens < 0 || (tokens > 0 && (!x || !out))) return LMOE_EINVAL;
    if (tokens == 0) return LMOE_OK;
    if (!router_hidden_ok(layer->experts.hidden)) return LMOE_EUNSUPPORTED;
    if (choose_path(layer, tokens, LMOE_PATH_DECODE) < 0) return LMOE_EUNSUPPORTED;
    const Layout L = layer_layout(layer, tokens);
    if (L.total > LMOE_STATIC_WORKSPACE_BYTES) return LMOE_EWORKSPACE;
    void *ws = nullptr;
    rc = static_workspace(&ws);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The array keeps whatever the previous call left in it.  The status
    // word and the router's block counter (the first 256 bytes) must start
    // at zero; the combine counters are zeroed by the router kernel itself.
    if (cudaMemsetAsync(at<uint8_t>(ws, L.status), 0, 256, st) != cudaSuccess) return LMOE_ECUDA;
    return lmoe_moe_layer_path(layer, x, tokens, out, idx, w, ws, LMOE_STATIC_WORKSPACE_BYTES, stream,
                               LMOE_PATH_DECODE, nullptr, nullptr);
}

int lmoe_static_status(void *stream) {
    void *ws = nullptr;
    const int rc = static_workspace(&ws);
    if (rc) return rc;
    return lmoe_workspace_status(ws, stream);
}

// Routing supplied by the caller through the decode GEMVs.  out != nullptr:
// the combined layer output; otherwise the per-route rows go to products
// (routes with a negative id skipped, w == nullptr: unit weights).
static int routed_impl(const lmoe_layer *layer, const void *x, int32_t tokens, const int32_t *idx, const float *w,
                       void *out, void *products, void *workspace, size_t ws_bytes, void *stream) {
    int rc = check_layer(layer);
    if (rc) return rc;
    if (!layer_gemv_ok(layer)) return LMOE_EUNSUPPORTED;  // the decode GEMVs (2/4/8-bit)
    if (tokens < 0 || (tokens > 0 && (!x || !idx || (!w && out) || (!out && !products) || !workspace)))
        return LMOE_EINVAL;
    if (tokens == 0) return LMOE_OK;
    const Layout L = layer_layout(layer, tokens);
    if (ws_bytes < L.total) return LMOE_EWORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const lmoe_experts &ex = layer->experts;
    PanelArgs pa;
    std::memset(&pa, 0, sizeof(pa));
    pa.x = static_cast<const uint16_t *>(x);
    pa.rows = tokens;
    pa.K = ex.hidden;
    pa.zero = at<uint32_t>(workspace, L.cnt);  // this call's combine counters
    pa.zero_words = static_cast<int32_t>((L.zero_end - L.cnt) / 4);
    pa.panel = at<uint16_t>(workspace, L.xpanel);
    pa.sum16 = at<float>(workspace, L.xsum);
    pa.bits = ex.gate.bits;
    pa.gs = ex.gate.group_size;
    pa.act_f16 = ex.dtype == LMOE_F16;
    rc = cuda_rc(launch_panel(pa, st));
    if (rc) return rc;
    const int R = tokens * layer->router.top_k;
    const int ct = layer_chunk(layer, tokens);
    if (ct < 1) return LMOE_EUNSUPPORTED;
    rc = run_dispatch(L, workspace, idx, R, layer->router.n_experts, layer->expert_slot, ex.n_slots, ct, st,
                      /*drop_zero=*/out == nullptr);
    if (rc) return rc;
    Extra e;
    e.yw = static_cast<uint16_t *>(products);
    e.x = static_cast<const uint16_t *>(x);
    return run_experts(layer, L, workspace, tokens, w, out, st, nullptr, e);
}

int lmoe_moe_routed(const lmoe_layer *layer, const void *x, int32_t tokens, const int32_t *idx,
                    const float *w, void *out, void *workspace, size_t ws_bytes, void *stream) {
    if (tokens > 0 && !out) return LMOE_EINVAL;
    return routed_impl(layer, x, tokens, idx, w, out, nullptr, workspace, ws_bytes, stream);
}

int lmoe_moe_products(const lmoe_layer *layer, const void *x, int32_t tokens, const int32_t *idx, const float *w,
                      void *products, void *workspace, size_t ws_bytes, void *stream) {
    if (tokens > 0 && (!products || !aligned16(products))) return LMOE_EINVAL;
    return routed_impl(layer, x, tokens, idx, w, nullptr, products, workspace, ws_bytes, stream);
}

int lmoe_combine_routes(const void *products, const float *w, const int32_t *order, int32_t tokens, int32_t top_k,
                        int32_t hidden, int32_t dtype, void *out, void *stream) {
    if (tokens < 0 || top_k < 1 || top_k > 16 || hidden <= 0 || hidden % 8 != 0) return LMOE_EINVAL;
    if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_EUNSUPPORTED;
    if (tokens == 0) return LMOE_OK;
    if (!products || !out || !aligned16(products) || !aligned16(out)) return LMOE_EINVAL;
    return cuda_rc(launch_combine_routes(dtype == LMOE_F16, static_cast<const uint16_t *>(products), w, order, tokens,
                                         top_k, hidden, static_cast<uint16_t *>(out),
                                         static_cast<cudaStream_t>(stream)));
}

int lmoe_gateup_swiglu(const lmoe_experts *experts, const void *x, int32_t tokens, int32_t top_k,
                       const uint32_t *slots, float limit, int32_t swiglu_mode, void *h,
                       void *workspace, size_t ws_bytes, void *stream) {
    // only gate and up are read here; the down projection is not validated
    if (!experts) return LMOE_EINVAL;
    if (experts->n_slots < 1 || experts->hidden <= 0 || experts->inter <= 0) return LMOE_EINVAL;
    if (experts->dtype != LMOE_BF16 && experts->dtype != LMOE_F16) return LMOE_EUNSUPPORTED;
    int rc = check_proj(experts->gate, experts->inter, experts->hidden);
    if (!rc) rc = check_proj(experts->up, experts->inter, experts->hidden);
    if (rc) return rc;
    if (!gemv_ok(experts->gate.bits, experts->gate.group_size)) return LMOE_EUNSUPPORTED;
    if (experts->gate.bits != experts->up.bits || experts->gate.group_size != experts->up.group_size)
        return LMOE_EUNSUPPORTED;
    if (tokens < 0 || top_k < 1) return LMOE_EINVAL;
    if (tokens > 0 && (!x || !slots || !h || !workspace)) return LMOE_EINVAL;
    if (swiglu_mode != LMOE_SWIGLU_FUSED && swiglu_mode != LMOE_SWIGLU_STOCK) return LMOE_EUNSUPPORTED;
    if (tokens == 0) return LMOE_OK;
    const int R = tokens * top_k;
    const int H = experts->hidden, I = experts->inter;
    const int K = H > I ? H : I;
    const Layout L = make_layout(R, R, K, 0, 0, experts->n_slots + 1, 1, 1, R);
    if (ws_bytes < L.total) return LMOE_EWORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    PanelArgs pa;
    std::memset(&pa, 0, sizeof(pa));
    pa.x = static_cast<const uint16_t *>(x);
    pa.rows = tokens;
    pa.K = H;
    pa.panel = at<uint16_t>(workspace, L.xpanel);
    pa.sum16 = at<float>(workspace, L.xsum);
    pa.bits = experts->gate.bits;
    pa.gs = experts->gate.group_size;
    pa.act_f16 = experts->dtype == LMOE_F16;
    rc = cuda_rc(launch_panel(pa, st));
    if (rc) return rc;
    StreamCfg sc;
    const bool streamed = gateup_streamed(*experts, R < kChunkTok ? R : kChunkTok, tokens, &sc);
    const int ntok_max = streamed ? (R < kChunkTok ? R : kChunkTok)
                                  : chunk_for(MODE_GATEUP, experts->gate.bits, experts->gate.group_size, H, tokens);
    if (ntok_max < 1) return LMOE_EUNSUPPORTED;
    rc = run_dispatch(L, workspace, reinterpret_cast<const int32_t *>(slots), R, experts->n_slots,
                      nullptr, experts->n_slots, ntok_max, st);
    if (rc) return rc;
    GemvArgs gu = gemv_base(L, workspace, experts->n_slots, ntok_max);
    gu.q0 = view(experts->gate, experts->n_slots, I, H);
    gu.q1 = view(experts->up, experts->n_slots, I, H);
    gu.panel = pa.panel;
    gu.sum16 = pa.sum16;
    gu.route_div = top_k;
    gu.out = static_cast<uint16_t *>(h);
    gu.out_panel = 0;
    gu.limit = limit;
    gu.swiglu_mode = swiglu_mode;
    gu.chunks_est = R;
    if (streamed)
        return cuda_rc(launch_stream(SMODE_GATEUP, pa.act_f16, experts->gate.bits, experts->gate.group_size, gu, sc,
                                     L.max_chunks, st));
    if (!experts->gate.weight || !experts->up.weight) return LMOE_EINVAL;
    gu.q0.tiles = gu.q1.tiles = nullptr;
    return cuda_rc(launch_gemv(MODE_GATEUP, pa.act_f16, experts->gate.bits, experts->gate.group_size,
                               gu, L.max_chunks, st));
}

int lmoe_gather_qmm(const lmoe_qproj *proj, int32_t n_slots, int32_t rows, int32_t cols, int32_t dtype,
                    const void *x, int32_t routes, const uint32_t *slots, void *y, void *workspace,
                    size_t ws_bytes, void *stream) {
    if (!proj || n_slots < 1 || rows <= 0 || cols <= 0 || routes < 0) return LMOE_EINVAL;
    if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_EUNSUPPORTED;
    int rc = check_proj(*proj, rows, cols);
    if (!rc && !gemv_ok(proj->bits, proj->group_size)) rc = LMOE_EUNSUPPORTED;
    if (rc) return rc;
    if (routes == 0) return LMOE_OK;
    if (!x || !slots || !y || !workspace) return LMOE_EINVAL;
    const Layout L = make_layout(routes, routes, cols, 0, 0, n_slots + 1, 1, 1, routes);
    if (ws_bytes < L.total) return LMOE_EWORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    PanelArgs pa;
    std::memset(&pa, 0, sizeof(pa));
    pa.x = static_cast<const uint16_t *>(x);
    pa.rows = routes;
    pa.K = cols;
    pa.panel = at<uint16_t>(workspace, L.xpanel);
    pa.sum16 = at<float>(workspace, L.xsum);
    pa.bits = proj->bits;
    pa.gs = proj->group_size;
    pa.act_f16 = dtype == LMOE_F16;
    rc = cuda_rc(launch_panel(pa, st));
    if (rc) return rc;
    const QView qv = view(*proj, n_slots, rows, cols);
    StreamCfg sc;
    const bool streamed = qv.tiles && stream_config(SMODE_PAIR, rows, cols, proj->bits, proj->group_size, false,
                                                    routes < kChunkTok ? routes : kChunkTok, routes, &sc);
    const int ntok_max = streamed ? (routes < kChunkTok ? routes : kChunkTok)
                                  : chunk_for(MODE_QMM, proj->bits, proj->group_size, cols, routes);
    if (ntok_max < 1) return LMOE_EUNSUPPORTED;
    rc = run_dispatch(L, workspace, reinterpret_cast<const int32_t *>(slots), routes, n_slots, nullptr,
                      n_slots, ntok_max, st);
    if (rc) return rc;
    GemvArgs q = gemv_base(L, workspace, n_slots, ntok_max);
    q.q0 = qv;
    q.panel = pa.panel;
    q.sum16 = pa.sum16;
    q.route_div = 1;
    q.out = static_cast<uint16_t *>(y);
    q.chunks_est = routes;
    if (streamed)  // y per route (no weights: the plain gather_qmm output)
        return cuda_rc(launch_stream(SMODE_PAIR, pa.act_f16, proj->bits, proj->group_size, q, sc, L.max_chunks, st));
    if (!proj->weight) return LMOE_EINVAL;
    q.q0.tiles = nullptr;
    return cuda_rc(launch_gemv(MODE_QMM, pa.act_f16, proj->bits, proj->group_size, q, L.max_chunks, st));
}

size_t lmoe_tile_bytes(int32_t rows, int32_t cols, int32_t bits, int32_t group_size) {
    if (rows <= 0 || group_size <= 0 || cols <= 0 || cols % group_size != 0) return 0;
    if (!gemv_ok(bits, group_size)) return 0;
    StreamGeo sg;
    if (!stream_geo(rows, cols, bits, group_size, &sg) || sg.tg.SB != 16) return 0;
    return (size_t)sg.slot;
}

int lmoe_tile_pack(const lmoe_qproj *src, int32_t n_slots, int32_t rows, int32_t cols, int32_t slot_begin,
                   int32_t slot_count, void *tiles, void *stream) {
    if (!src || !tiles || !src->weight || !src->scales || !src->biases) return LMOE_EINVAL;
    if (n_slots < 1 || slot_begin < 0 || slot_count < 0 || slot_begin + slot_count > n_slots) return LMOE_EINVAL;
    if (!aligned16(src->weight) || !aligned16(src->scales) || !aligned16(src->biases) || !aligned16(tiles))
        return LMOE_EINVAL;
    if (lmoe_tile_bytes(rows, cols, src->bits, src->group_size) == 0) return LMOE_EUNSUPPORTED;
    lmoe_qproj p = *src;
    p.tiles = tiles;
    const QView q = view(p, n_slots, rows, cols);
    return cuda_rc(launch_stream_pack(q, src->bits, src->group_size, slot_begin, slot_count,
                                      static_cast<uint8_t *>(tiles), static_cast<cudaStream_t>(stream)));
}

// ------------------------------------------------------------ expert parallel
size_t lmoe_ep_row_bytes(int32_t hidden, int32_t top_k) {
    if (hidden <= 0 || hidden % 8 != 0 || top_k < 1 || top_k > 16) return 0;
    return (size_t)ep_row_bytes(hidden, top_k);
}

int lmoe_ep_dispatch(const int32_t *idx, const float *w, const void *x, int32_t tokens, int32_t hidden,
                     int32_t top_k, int32_t n_experts, int32_t world, void *send, int32_t *slot_of, void *workspace,
                     void *stream) {
    if (tokens < 0 || hidden <= 0 || hidden % 8 != 0 || top_k < 1 || top_k > 16) return LMOE_EINVAL;
    if (world < 1 || world > kEpMaxWorld || n_experts < 1 || n_experts % world != 0) return LMOE_EINVAL;
    if (tokens == 0) return LMOE_OK;
    if (!idx || !w || !x || !send || !slot_of || !aligned16(x) || !aligned16(send)) return LMOE_EINVAL;
    EpDispatchArgs a;
    a.idx = idx;
    a.w = w;
    a.x = static_cast<const uint16_t *>(x);
    a.T = tokens;
    a.k = top_k;
    a.H = hidden;
    a.E = n_experts;
    a.world = world;
    a.send = static_cast<uint8_t *>(send);
    a.slot_of = slot_of;
    a.err = static_cast<int32_t *>(workspace);
    return cuda_rc(launch_ep_dispatch(a, static_cast<cudaStream_t>(stream)));
}

size_t lmoe_ep_workspace_size(const lmoe_layer *local, int32_t rows, int32_t world, int32_t path) {
    if (check_ep_local(local) || rows < 0 || world < 1 || world > kEpMaxWorld) return 0;
    const int n = rows > 0 ? rows : 1;
    const int pf = ep_path(local, n, world, path);
    if (pf < 0) return 0;
    return ep_layout(local, n, pf != 0).total;
}

int lmoe_ep_experts(const lmoe_layer *local, const void *recv, int32_t rows, int32_t world, float *partial,
                    void *workspace, size_t ws_bytes, void *stream, int32_t path) {
    int rc = check_ep_local(local);
    if (rc) return rc;
    if (rows < 0 || world < 1 || world > kEpMaxWorld) return LMOE_EINVAL;
    if (rows == 0) return LMOE_OK;
    if (!recv || !partial || !workspace || !aligned16(recv) || !aligned16(partial)) return LMOE_EINVAL;
    const lmoe_experts &ex = local->experts;
    const int H = ex.hidden, k = local->router.top_k;
    if (H % 8 != 0) return LMOE_EUNSUPPORTED;
    const int pf = ep_path(local, rows, world, path);
    if (pf < 0) return LMOE_EUNSUPPORTED;
    const Layout L = ep_layout(local, rows, pf != 0);
    if (ws_bytes < L.total) return LMOE_EWORKSPACE;
    const int chunk_tok = pf ? kPfNmax : layer_chunk(local, rows);
    if (chunk_tok < 1) return LMOE_EUNSUPPORTED;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int xs = ep_row_bytes(H, k) / 2;  // elements between received rows
    int32_t *ridx = at<int32_t>(workspace, L.idx);
    float *rw = at<float>(workspace, L.w);
    rc = cuda_rc(launch_ep_unpack(static_cast<const uint8_t *>(recv), rows, H, k, ridx, rw, st));
    if (rc) return rc;
    if (!pf) {  // the decode GEMVs read the rows through the activation panel
        PanelArgs pa;
        std::memset(&pa, 0, sizeof(pa));
        pa.x = static_cast<const uint16_t *>(recv);
        pa.rows = rows;
        pa.K = H;
        pa.x_stride = xs;
        pa.panel = at<uint16_t>(workspace, L.xpanel);
        pa.sum16 = at<float>(workspace, L.xsum);
        pa.bits = ex.gate.bits;
        pa.gs = ex.gate.group_size;
        pa.act_f16 = ex.dtype == LMOE_F16;
        rc = cuda_rc(launch_panel(pa, st));
        if (rc) return rc;
    }
    rc = run_dispatch(L, workspace, ridx, rows * k, local->router.n_experts, local->expert_slot, ex.n_slots,
                      chunk_tok, st, /*drop_zero=*/true);
    if (rc) return rc;
    rc = pf ? run_experts_pf(local, L, workspace, recv, rows, rw, nullptr, st, nullptr, xs)
            : run_experts(local, L, workspace, rows, rw, nullptr, st);
    if (rc) return rc;
    return cuda_rc(launch_ep_partial(ex.dtype == LMOE_F16, at<uint16_t>(workspace, L.yw), ridx, rows, H, k,
                                     local->router.n_experts, partial, st));
}

int lmoe_ep_combine(const float *back, int32_t tokens, int32_t world, int32_t hidden, int32_t dtype,
                    const int32_t *slot_of, const void *residual, void *out, void *normed, float eps,
                    void *stream) {
    if (tokens < 0 || world < 1 || world > kEpMaxWorld || hidden <= 0 || hidden % 8 != 0) return LMOE_EINVAL;
    if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_EUNSUPPORTED;
    if (tokens == 0) return LMOE_OK;
    if (!back || !slot_of || !out || !aligned16(back) || !aligned16(out) || (residual && !aligned16(residual)) ||
        (normed && !aligned16(normed)) || !(eps >= 0.0f))
        return LMOE_EINVAL;
    return cuda_rc(launch_ep_combine(dtype == LMOE_F16, back, tokens, world, hidden, slot_of,
                                     static_cast<const uint16_t *>(residual), static_cast<uint16_t *>(out),
                                     static_cast<uint16_t *>(normed), eps, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
