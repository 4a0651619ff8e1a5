// Routing kernels for sm_100a: router logits + top-k, dispatch (routes grouped
// by expert into chunks) and the activation panel producer.
#include <float.h>

#include "lmoe_kernels.cuh"

namespace lmoe {

#define LMOE_FULL 0xffffffffu

// ============================================================ block utilities
// Exclusive scan of one int per thread over a 256-thread block.
__device__ int block_scan_256(int v, int *s_tmp /*[9]*/, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(LMOE_FULL, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) s_tmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = (lane < 8) ? s_tmp[lane] : 0;
        int wi = w;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const int n = __shfl_up_sync(LMOE_FULL, wi, o);
            if (lane >= o) wi += n;
        }
        if (lane < 8) s_tmp[lane] = wi - w;  // exclusive per warp
        if (lane == 7) s_tmp[8] = wi;
    }
    __syncthreads();
    const int out = s_tmp[warp] + incl - v;
    *total = s_tmp[8];
    __syncthreads();
    return out;
}

// ============================================================ dispatch
// Groups routes by expert (stable in route order) and cuts each expert's run
// into chunks of at most 8 routes.  Replaces the host loop of
// arena.py:557-566 and the slot sort of arena.py:650-659.  Runs on one
// 256-thread block; R <= kDispatchSmallMaxRoutes, buckets <= 1024.
__device__ void dispatch_block(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                               int *s_mem) {
    const int tid = threadIdx.x;
    const int R = din.R;
    const int E = din.n_experts;
    const int NBk = E + 1;  // last bucket collects invalid ids (zero slot)
    int *s_b = s_mem;                                  // [512]
    int *s_cnt = s_b + kDispatchSmallMaxRoutes;        // [1025]
    int *s_roff = s_cnt + kDispatchSmallMaxBuckets + 1;
    int *s_coff = s_roff + kDispatchSmallMaxBuckets + 1;
    int *s_tmp = s_coff + kDispatchSmallMaxBuckets + 1;  // [9]
    for (int i = tid; i < NBk; i += blockDim.x) s_cnt[i] = 0;
    __syncthreads();
    for (int r = tid; r < R; r += blockDim.x) {
        const int id = din.idx[r];
        int b = id;
        if (id < 0 || id >= E) {
            b = E;
            if (!(din.drop_zero && id < 0)) set_error(err, -3);
        }
        s_b[r] = b;
        atomicAdd(&s_cnt[b], 1);
    }
    __syncthreads();
    const int per = (NBk + 255) >> 8;
    auto nchunks = [&](int b) { return (din.drop_zero && b == E) ? 0 : (s_cnt[b] + din.chunk_tok - 1) / din.chunk_tok; };
    int lr = 0, lc = 0;
    for (int q = 0; q < per; ++q) {
        const int b = tid * per + q;
        if (b < NBk) {
            lr += s_cnt[b];
            lc += nchunks(b);
        }
    }
    int tr, tc;
    int er = block_scan_256(lr, s_tmp, &tr);
    int ec = block_scan_256(lc, s_tmp, &tc);
    for (int q = 0; q < per; ++q) {
        const int b = tid * per + q;
        if (b < NBk) {
            s_roff[b] = er;
            s_coff[b] = ec;
            er += s_cnt[b];
            ec += nchunks(b);
        }
    }
    __syncthreads();
    for (int r = tid; r < R; r += blockDim.x) {
        const int b = s_b[r];
        int rank = 0;
        for (int r2 = 0; r2 < r; ++r2) rank += (s_b[r2] == b);
        const int pos = s_roff[b] + rank;
        dout.sorted_routes[pos] = r;
        if ((rank % din.chunk_tok) == 0 && !(din.drop_zero && b == E)) {
            int slot = 0;
            if (b < E) {
                slot = din.expert_slot ? din.expert_slot[b] : b;
                if (slot < 0 || slot >= din.n_slots) {
                    set_error(err, -3);
                    slot = 0;
                }
            }
            Chunk ch;
            ch.slot = slot;
            ch.route_start = pos;
            ch.ntok = min(din.chunk_tok, s_cnt[b] - rank);
            ch.expert = b;
            dout.chunks[s_coff[b] + rank / din.chunk_tok] = ch;
        }
    }
    if (tid == 0) *dout.n_chunks = tc;
    __syncthreads();
}

// Dispatch of at most 32 routes by one warp: same output as dispatch_block
// (routes grouped by expert in expert order, stable in route order; chunks
// of at most chunk_tok routes in expert order) without block barriers.
__device__ void dispatch_warp(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                              const int *s_idx = nullptr, const int *s_slot = nullptr) {
    const int lane = threadIdx.x & 31;
    const int R = din.R, E = din.n_experts, ct = din.chunk_tok;
    int b = 0x7fffffff;  // lanes without a route sort after every bucket
    if (lane < R) {
        const int id = s_idx ? s_idx[lane] : din.idx[lane];
        b = id;
        if (id < 0 || id >= E) {
            b = E;
            if (!(din.drop_zero && id < 0)) set_error(err, -3);
        }
    }
    const unsigned same = __match_any_sync(LMOE_FULL, b);
    const int rank = __popc(same & ((1u << lane) - 1u));
    const int cnt = __popc(same);
    const bool dropped = din.drop_zero && b == E;
    // bucket leaders carry the chunk count
    const int nch = (rank == 0 && !dropped) ? (cnt + ct - 1) / ct : 0;
    int before_r = 0, before_c = 0, total_c = 0;
    for (int j = 0; j < R; ++j) {
        const int bj = __shfl_sync(LMOE_FULL, b, j);
        const int cj = __shfl_sync(LMOE_FULL, nch, j);
        before_r += (bj < b);
        before_c += (bj < b) ? cj : 0;
        total_c += cj;
    }
    if (lane < R) {
        const int pos = before_r + rank;
        dout.sorted_routes[pos] = lane;
        if (rank % ct == 0 && !dropped) {
            int slot = 0;
            if (b < E) {
                slot = s_slot ? s_slot[b] : (din.expert_slot ? din.expert_slot[b] : b);
                if (slot < 0 || slot >= din.n_slots) {
                    set_error(err, -3);
                    slot = 0;
                }
            }
            Chunk ch;
            ch.slot = slot;
            ch.route_start = pos;
            ch.ntok = min(ct, cnt - rank);
            ch.expert = b;
            dout.chunks[before_c + rank / ct] = ch;
        }
    }
    if (lane == 0) *dout.n_chunks = total_c;
}

// The shared expert of a block (dsv4_engine.py:259, routed + shared_experts(x)):
// one more route per token, routes R .. R + T - 1 in token order with weight
// 1, in chunks of at most chunk_tok after the dispatched routed chunks.  One
// block, after the dispatch (it appends to the chunk count).
__global__ void __launch_bounds__(256) shared_chunks_kernel(Chunk *chunks, int32_t *n_chunks, int32_t *sorted_routes,
                                                            float *route_w, int R, int T, int ct, int slot) {
    __shared__ int s_n0;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) s_n0 = *n_chunks;
    __syncthreads();
    const int n0 = s_n0;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        sorted_routes[R + t] = R + t;
        route_w[R + t] = 1.0f;
    }
    const int nsc = (T + ct - 1) / ct;
    for (int c = threadIdx.x; c < nsc; c += blockDim.x) {
        Chunk ch;
        ch.slot = slot;
        ch.route_start = R + c * ct;
        ch.ntok = min(ct, T - c * ct);
        ch.expert = -1;
        chunks[n0 + c] = ch;
    }
    __syncthreads();
    if (threadIdx.x == 0) *n_chunks = n0 + nsc;
}

cudaError_t launch_shared_chunks(Chunk *chunks, int32_t *n_chunks, int32_t *sorted_routes, float *route_w, int R,
                                 int T, int chunk_tok, int slot, cudaStream_t st) {
    return launch_pdl(shared_chunks_kernel, dim3(1), dim3(256), 0, st, chunks, n_chunks, sorted_routes, route_w, R, T,
                      chunk_tok, slot);
}

__global__ void __launch_bounds__(256) dispatch_small_kernel(DispatchIn din, DispatchOut dout,
                                                             int32_t *err) {
    __shared__ int s_mem[kDispatchSmallMaxRoutes + 3 * (kDispatchSmallMaxBuckets + 1) + 16];
    pdl_wait();
    pdl_trigger();
    if (din.R <= 32) {
        if (threadIdx.x < 32) dispatch_warp(din, dout, err);
        return;
    }
    dispatch_block(din, dout, err, s_mem);
}

// Large-R dispatch, pass 1: one block per bucket counts its routes and the
// routes of lower buckets, then ranks its own routes in route order.
__global__ void __launch_bounds__(256) dispatch_rank_kernel(DispatchIn din, DispatchOut dout,
                                                            int32_t *err) {
    __shared__ int s_tmp[9];
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x;
    const int E = din.n_experts;
    const int tid = threadIdx.x;
    int lt = 0, eq = 0;
    for (int r = tid; r < din.R; r += blockDim.x) {
        int id = din.idx[r];
        if (id < 0 || id >= E) {
            if (b == 0 && !(din.drop_zero && id < 0)) set_error(err, -3);
            id = E;
        }
        lt += (id < b);
        eq += (id == b);
    }
    int tot_lt, tot_eq;
    block_scan_256(lt, s_tmp, &tot_lt);
    block_scan_256(eq, s_tmp, &tot_eq);
    if (tid == 0) {
        dout.counts[b] = tot_eq;
        dout.route_off[b] = tot_lt;
    }
    if (tot_eq == 0) return;
    int base = 0;
    for (int r0 = 0; r0 < din.R; r0 += blockDim.x) {
        const int r = r0 + tid;
        int id = (r < din.R) ? din.idx[r] : -2;
        if (r < din.R && (id < 0 || id >= E)) id = E;
        const int is = (id == b);
        int tot;
        const int ex = block_scan_256(is, s_tmp, &tot);
        if (is) dout.sorted_routes[tot_lt + base + ex] = r;
        base += tot;
    }
}

// Large-R dispatch, pass 2: chunk table from per-bucket counts (one block).
__global__ void __launch_bounds__(256) dispatch_chunks_kernel(DispatchIn din, DispatchOut dout,
                                                              int32_t *err) {
    __shared__ int s_tmp[9];
    pdl_wait();
    pdl_trigger();
    const int NBk = din.n_experts + 1;
    const int tid = threadIdx.x;
    const int per = (NBk + 255) >> 8;
    // the zero bucket of an expert-parallel receive side gets no chunks
    const int NBc = din.drop_zero ? din.n_experts : NBk;
    int lc = 0;
    for (int q = 0; q < per; ++q) {
        const int b = tid * per + q;
        if (b < NBc) lc += (dout.counts[b] + din.chunk_tok - 1) / din.chunk_tok;
    }
    int tc;
    int ec = block_scan_256(lc, s_tmp, &tc);
    for (int q = 0; q < per; ++q) {
        const int b = tid * per + q;
        if (b >= NBc) continue;
        const int cnt = dout.counts[b];
        int slot = 0;
        if (b < din.n_experts && cnt > 0) {
            slot = din.expert_slot ? din.expert_slot[b] : b;
            if (slot < 0 || slot >= din.n_slots) {
                set_error(err, -3);
                slot = 0;
            }
        }
        for (int c0 = 0; c0 < cnt; c0 += din.chunk_tok) {
            Chunk ch;
            ch.slot = slot;
            ch.route_start = dout.route_off[b] + c0;
            ch.ntok = min(din.chunk_tok, cnt - c0);
            ch.expert = b;
            dout.chunks[ec++] = ch;
        }
    }
    if (tid == 0) *dout.n_chunks = tc;
}

// ============================================================ router
__device__ __forceinline__ float score_fn(float lg, int scoring) {
    if (scoring == 2) {  // sqrt(softplus)
        const float sp = lg > 20.0f ? lg : log1pf(expf(lg));
        return sqrtf(sp);
    }
    return 1.0f / (1.0f + expf(-lg));  // sigmoid
}

// Top-k of one token by one warp (arena.py:501-506): selection on
// score + bias, weights from the raw scores normalised by sum + 1e-20, then
// routed scaling.  Ties go to the lower expert id.  `scores`, when given,
// holds (score, score + bias) already (element-wise scorings, computed by
// the logit blocks); otherwise the logits are scored here.
__device__ void topk_token(const float *partial, const float2 *scores, int ksplit, int T, int E, int tok,
                           const float *bias, int scoring, int top_k, int norm, float scaling,
                           int32_t *idx_ws, float *w_ws, int32_t *idx_user, float *w_user,
                           int *s_idx = nullptr, const int32_t *hash_idx = nullptr) {
    const int lane = threadIdx.x & 31;
    float sc[kRouterMaxEPL], bs[kRouterMaxEPL];
    if (scores) {
#pragma unroll
        for (int i = 0; i < kRouterMaxEPL; ++i) {
            const int e = lane + 32 * i;
            sc[i] = 0.0f;
            bs[i] = -INFINITY;
            if (e < E) {
                const float2 v = __ldcg(scores + (size_t)tok * E + e);
                sc[i] = v.x;
                bs[i] = v.y;
            }
        }
    } else {
        float mx = -FLT_MAX;
#pragma unroll
        for (int i = 0; i < kRouterMaxEPL; ++i) {
            const int e = lane + 32 * i;
            float lg = -FLT_MAX;
            if (e < E) {
                lg = 0.0f;
                for (int ky = 0; ky < ksplit; ++ky) lg += __ldcg(partial + ((size_t)ky * T + tok) * E + e);
                mx = fmaxf(mx, lg);
            }
            sc[i] = lg;
        }
        if (scoring == 1) {  // softmax over all experts
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(LMOE_FULL, mx, o));
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < kRouterMaxEPL; ++i) {
                const int e = lane + 32 * i;
                sc[i] = (e < E) ? expf(sc[i] - mx) : 0.0f;
                sum += sc[i];
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(LMOE_FULL, sum, o);
#pragma unroll
            for (int i = 0; i < kRouterMaxEPL; ++i) sc[i] = sc[i] / sum;
        } else {
#pragma unroll
            for (int i = 0; i < kRouterMaxEPL; ++i) {
                const int e = lane + 32 * i;
                if (e < E) sc[i] = score_fn(sc[i], scoring);
            }
        }
#pragma unroll
        for (int i = 0; i < kRouterMaxEPL; ++i) {
            const int e = lane + 32 * i;
            bs[i] = (e < E) ? sc[i] + (bias ? bias[e] : 0.0f) : -INFINITY;
        }
    }
    int my_e = -1;
    float my_s = 0.0f;
    if (hash_idx) {
        // token-id hash routing: the experts are given (tid2eid[input_ids]);
        // the weights are their scores, normalised and scaled as below.  An
        // id outside [0, E) keeps score 0 (dispatch sends it to the zero slot).
        const int e_l = lane < top_k ? hash_idx[(size_t)tok * top_k + lane] : -1;
#pragma unroll 1
        for (int j = 0; j < top_k; ++j) {
            const int e = __shfl_sync(LMOE_FULL, e_l, j);
            const bool ok = e >= 0 && e < E;
            float v = 0.0f;
#pragma unroll
            for (int i = 0; i < kRouterMaxEPL; ++i)
                if (ok && i == (e >> 5)) v = sc[i];
            const float sv = __shfl_sync(LMOE_FULL, v, ok ? (e & 31) : 0);
            if (lane == j) {
                my_e = e;
                my_s = ok ? sv : 0.0f;
            }
        }
    } else {
    // Each lane keeps its own best candidate; a round takes the warp-wide
    // best and only the winning lane rescans its candidates.  Lane j keeps
    // the j-th winner.
    float lbv = -INFINITY, lbs = 0.0f;
    int lbe = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kRouterMaxEPL; ++i)
        if (bs[i] > lbv) {
            lbv = bs[i];
            lbe = lane + 32 * i;
            lbs = sc[i];
        }
#pragma unroll 1
    for (int j = 0; j < top_k; ++j) {
        float bv = lbv;
        int be = lbe;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(LMOE_FULL, bv, o);
            const int oe = __shfl_xor_sync(LMOE_FULL, be, o);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        const float ws = __shfl_sync(LMOE_FULL, lbs, be & 31);
        if (lane == j) {
            my_e = be;
            my_s = ws;
        }
        if (lbe == be) {  // the winner drops it and rescans
            lbv = -INFINITY;
            lbe = 0x7fffffff;
#pragma unroll
            for (int i = 0; i < kRouterMaxEPL; ++i) {
                if (lane + 32 * i == be) bs[i] = -INFINITY;
                if (bs[i] > lbv) {
                    lbv = bs[i];
                    lbe = lane + 32 * i;
                    lbs = sc[i];
                }
            }
        }
    }
    }
    float ssum = 0.0f;  // fp32, in selection order
#pragma unroll 1
    for (int j = 0; j < top_k; ++j) ssum += __shfl_sync(LMOE_FULL, my_s, j);
    if (lane < top_k) {
        float wv = norm ? my_s / (ssum + 1e-20f) : my_s;
        wv *= scaling;
        const size_t o = (size_t)tok * top_k + lane;
        idx_ws[o] = my_e;
        w_ws[o] = wv;
        if (idx_user) idx_user[o] = my_e;
        if (w_user) w_user[o] = wv;
        if (s_idx) s_idx[o] = my_e;
    }
}

// Routing of a single token by the whole 256-thread block (decode batch 1),
// from precomputed (score, score + bias).  Selection: the top_k-th largest of
// the 8 warp maxima (top_k <= 8; otherwise -inf) is a threshold that at least
// top_k experts reach, so every winner is at or above it.  The experts there
// are gathered in shared memory and each counts the candidates that beat it
// (biased score higher, ties to the lower id): that count is its position in
// topk_token's selection order, so the winners, their order, the fp32 weight
// sum in that order and the weights are topk_token's bit for bit.
// With `disp` the block also writes dispatch_warp's output for these top_k
// distinct experts: routes sorted by expert id, one chunk of one route each.
__device__ void route_one_token(const RouterArgs &a, const int *s_slot, bool disp) {
    constexpr int kMaxE = 512;
    __shared__ float s_wmax[8];
    __shared__ float s_cb[kMaxE], s_cs[kMaxE];
    __shared__ int s_ce[kMaxE];
    __shared__ int s_nc;
    __shared__ float s_ws[16];
    __shared__ int s_we[16];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = a.E, top_k = a.top_k;
    float bs[2], sc[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int e = tid + 256 * q;
        bs[q] = -INFINITY;
        sc[q] = 0.0f;
        if (e < E) {
            const float2 v = __ldcg(a.scores + e);
            sc[q] = v.x;
            bs[q] = v.y;
        }
    }
    if (tid == 0) s_nc = 0;
    if (tid < 16) s_we[tid] = -1;
    float m = fmaxf(bs[0], bs[1]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(LMOE_FULL, m, o));
    if (lane == 0) s_wmax[warp] = m;
    __syncthreads();
    // lane i & 7 tests warp maximum i; a max over each group of 8 lanes
    // gives every lane the threshold (short code: it runs once per layer,
    // with its instructions fetched cold)
    float tau = -INFINITY;
    if (top_k <= 8) {
        const float wi = s_wmax[lane & 7];
        int ge = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) ge += s_wmax[j] >= wi;
        tau = ge >= top_k ? wi : -INFINITY;
        tau = fmaxf(tau, __shfl_xor_sync(LMOE_FULL, tau, 1));
        tau = fmaxf(tau, __shfl_xor_sync(LMOE_FULL, tau, 2));
        tau = fmaxf(tau, __shfl_xor_sync(LMOE_FULL, tau, 4));
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int e = tid + 256 * q;
        const bool cand = e < E && bs[q] >= tau;
        const unsigned bal = __ballot_sync(LMOE_FULL, cand);
        int base = 0;
        if (lane == 0 && bal) base = atomicAdd(&s_nc, __popc(bal));
        base = __shfl_sync(LMOE_FULL, base, 0);
        if (cand) {
            const int pos = base + __popc(bal & ((1u << lane) - 1u));
            s_cb[pos] = bs[q];
            s_cs[pos] = sc[q];
            s_ce[pos] = e;
        }
    }
    __syncthreads();
    const int nc = s_nc;
    for (int c = tid; c < nc; c += blockDim.x) {
        const float mb = s_cb[c];
        const int me = s_ce[c];
        int r = 0;
        for (int i = 0; i < nc; ++i) {
            const float ob = s_cb[i];
            r += (ob > mb) || (ob == mb && s_ce[i] < me);
        }
        if (r < top_k) {
            s_ws[r] = s_cs[c];
            s_we[r] = me;
        }
    }
    __syncthreads();
    if (warp != 0 || lane >= top_k) return;
    float ssum = 0.0f;  // fp32, in selection order
    for (int j = 0; j < top_k; ++j) ssum += s_ws[j];
    const float my_s = s_ws[lane];
    const int my_e = s_we[lane];
    float wv = a.norm_topk ? my_s / (ssum + 1e-20f) : my_s;
    wv *= a.scaling;
    a.idx_ws[lane] = my_e;
    a.w_ws[lane] = wv;
    if (a.idx_user) a.idx_user[lane] = my_e;
    if (a.w_user) a.w_user[lane] = wv;
    if (!disp) return;
    int pos = 0;
    for (int j = 0; j < top_k; ++j) pos += s_we[j] < my_e;
    int slot = 0;
    if (my_e < 0 || my_e >= E) {
        set_error(a.err, -3);
    } else {
        slot = s_slot[my_e];
        if (slot < 0 || slot >= a.din.n_slots) {
            set_error(a.err, -3);
            slot = 0;
        }
    }
    a.dout.sorted_routes[pos] = lane;
    Chunk ch;
    ch.slot = slot;
    ch.route_start = pos;
    ch.ntok = 1;
    ch.expert = my_e;
    a.dout.chunks[pos] = ch;
    if (lane == 0) *a.dout.n_chunks = top_k;
}

// Token rows from host memory the GPU can address (pinned, mapped) into a
// device buffer.  Both the host reads and the device stores follow the wait
// on the preceding kernel: the host rows may be the output of the previous
// layer call (its combine writes straight into pinned host memory), and an
// earlier launch may still read the device buffer.
__global__ void __launch_bounds__(256) stage_rows_kernel(uint4 *dst, const uint4 *src, size_t n16) {
    pdl_trigger();
    pdl_wait();
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) dst[i] = src[i];
}

cudaError_t launch_stage_rows(void *dst, const void *src, size_t bytes, cudaStream_t st) {
    const size_t n16 = bytes / 16;
    size_t blocks = (n16 + 255) / 256;
    if (blocks > 592) blocks = 592;
    if (blocks < 1) blocks = 1;
    return launch_pdl(stage_rows_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st,
                      static_cast<uint4 *>(dst), static_cast<const uint4 *>(src), n16);
}

template <typename TA>
__device__ __forceinline__ float act_to_f(uint16_t v) {
    return Act<TA>::to_f(v);
}

__device__ __forceinline__ float prescale(int p) { return p == 0 ? 1.0f : (p == 1 ? 0.25f : 0.0625f); }

// Router logits x @ Wg^T in fp32 (products of bf16 values are exact).  Block
// (b, z) owns experts [2b, 2b+2) over the full hidden width and tokens
// [64z, 64z+64): each warp reduces its 256-column chunks, warps combine in
// shared memory in a fixed order, so every logit is final when written (no
// split-K partials).  Each block also writes its share of the gate/up
// activation panel (16-column blocks b, b+gridDim.x, ...).  In the decode
// regime (T <= 64) the last block to finish runs top-k and dispatch, so
// routing costs one launch and no host synchronisation (the reference syncs
// here every layer, arena.py:513).
template <typename TA>
__global__ void __launch_bounds__(256) router_kernel(RouterArgs a) {
    constexpr int EPB = 2;
    __shared__ float s_red[8][EPB][8];
    __shared__ int s_last;
    __shared__ int s_disp[kDispatchSmallMaxRoutes + 3 * (kDispatchSmallMaxBuckets + 1) + 16];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int e0 = blockIdx.x * EPB;
    const int tbeg = blockIdx.y * 64;
    const int tend = min(a.T, tbeg + 64);
    // 256-column chunks per warp iteration; the last one may be partial
    // (hidden a multiple of 64): lanes past the width load nothing
    const int nchunk = (a.H + kRouterKS - 1) / kRouterKS;
    __shared__ float s_bias[EPB];
    if (tid < EPB) s_bias[tid] = (a.bias && e0 + tid < a.E) ? a.bias[e0 + tid] : 0.0f;
    // Router weights are read once per layer call: evict-first in L2.
    const uint64_t wpol = evict_first_policy();
    // Decode (one pass of at most 8 tokens): this warp's first two weight
    // chunks are requested before the panel work so their latency overlaps it.
    const bool one_pass = (tend - tbeg) <= 8;
    uint4 wpre[2][EPB];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int ch = warp + 8 * j;
#pragma unroll
        for (int i = 0; i < EPB; ++i) {
            wpre[j][i] = make_uint4(0, 0, 0, 0);
            if (one_pass && ch < nchunk && e0 + i < a.E && ch * kRouterKS + lane * 8 < a.H)
                wpre[j][i] = ldg_u128_hint(
                    reinterpret_cast<const uint4 *>(a.wg + (size_t)(e0 + i) * a.H + ch * kRouterKS + lane * 8), wpol);
        }
    }

    // everything above reads constants only; x and the workspace come from
    // the preceding kernels
    pdl_wait();
    pdl_trigger();
    // the expert -> slot table for the finishing block's small dispatch
    // (every block loads it; one uses it)
    const bool warp_disp = a.finish && a.do_dispatch && a.din.R <= 32 && a.E <= kDispatchSmallMaxRoutes;
    int slot_pre[2] = {0, 0};
    if (warp_disp) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int e = tid + 256 * q;
            if (e < a.E) slot_pre[q] = a.din.expert_slot ? __ldg(a.din.expert_slot + e) : e;
        }
    }
    if (a.zero) {
        const int nb = gridDim.x * gridDim.y;
        for (int i = (blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + tid; i < a.zero_words; i += nb * blockDim.x)
            a.zero[i] = 0u;
    }
    // single token: its first two activation chunks are requested now too
    const bool one_tok = (tend - tbeg) == 1;
    uint4 xpre[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int ch = warp + 8 * j;
        xpre[j] = make_uint4(0, 0, 0, 0);
        if (one_tok && ch < nchunk && ch * kRouterKS + lane * 8 < a.H) xpre[j] = __ldg(reinterpret_cast<const uint4 *>(a.x + (size_t)tbeg * a.H + ch * kRouterKS + lane * 8));
    }

    // ---- gate/up activation panel + 16-column sums for this block's share.
    // Panel positions of group G are G*gs + (position within the group), so a
    // per-block table of one group's positions replaces the index arithmetic.
    if (a.xpanel) {
        __shared__ short s_pos[128];
        __shared__ float s_scale[128];
        if (tid < a.pgs) {
            int p;
            s_pos[tid] = static_cast<short>(panel_pos(tid, a.pbits, a.pgs, &p));
            s_scale[tid] = prescale(p);
        }
        __syncthreads();
        const int nblk = a.H / 16;
        const int ntk = tend - tbeg;
        const int nmy = max(0, (nblk - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x);
        // item = (token, my block, half): lanes 2i / 2i+1 hold the two halves of a block
        const int total = ntk * nmy * 2;
        for (int base = tid - lane; base < total; base += blockDim.x) {
            const int item = base + lane;
            const bool ok = item < total;  // pairs (2i, 2i+1) are valid together
            const int half = item & 1, nb = item >> 1;
            const int n = ok ? nb / nmy : 0, j = ok ? nb - n * nmy : 0;
            const int col0 = (blockIdx.x + j * gridDim.x) * 16 + half * 8;
            const int t = tbeg + n;
            float s = 0.0f, sp = 0.0f;
            if (ok) {
                const uint4 v = *reinterpret_cast<const uint4 *>(a.x + (size_t)t * a.H + col0);
                const uint32_t u[4] = {v.x, v.y, v.z, v.w};
                const int G = col0 / a.pgs, i0 = col0 - G * a.pgs;
                uint16_t *dst = a.xpanel + (size_t)t * a.H + G * a.pgs;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float f =
                        act_to_f<TA>(static_cast<uint16_t>(q & 1 ? u[q >> 1] >> 16 : u[q >> 1] & 0xffffu));
                    const uint16_t pv = Act<TA>::from_f(f * s_scale[i0 + q]);
                    s += f;
                    sp += Act<TA>::to_f(pv);
                    dst[s_pos[i0 + q]] = pv;
                }
            }
            const float other = __shfl_xor_sync(LMOE_FULL, s, 1);
            const float other_p = __shfl_xor_sync(LMOE_FULL, sp, 1);
            if (ok && half == 0)
                *reinterpret_cast<float2 *>(a.xsum16 + ((size_t)t * (a.H / 16) + (col0 >> 4)) * 2) =
                    make_float2(s + other, sp + other_p);
        }
    }

    // ---- single token: int8 pieces of x for the single-token layer kernel,
    // one group per warp over the grid
    if (a.xq && tbeg == 0) {
        const int ngr = a.H / a.pgs, nw = gridDim.x * (blockDim.x >> 5);
        for (int gi = blockIdx.x * (blockDim.x >> 5) + warp; gi < ngr; gi += nw)
            convert_group_rt<TA>(a.pbits, a.pgs, a.x + (size_t)gi * a.pgs, a.xq + (size_t)gi * (2 * a.pgs), a.xs + gi,
                                 false);
    }

    // ---- logits
    for (int ts = tbeg; ts < tend; ts += 8) {
        const int nt = min(8, tend - ts);
        float acc[EPB][8];
#pragma unroll
        for (int i = 0; i < EPB; ++i)
#pragma unroll
            for (int n = 0; n < 8; ++n) acc[i][n] = 0.0f;
#pragma unroll 2
        for (int ch = warp, j = 0; ch < nchunk; ch += 8, ++j) {
            const int col = ch * kRouterKS + lane * 8;
            const bool kin = col < a.H;  // zeros past the width add nothing
            uint4 wv[EPB];
#pragma unroll
            for (int i = 0; i < EPB; ++i) {
                if (one_pass && j == 0) {
                    wv[i] = wpre[0][i];
                } else if (one_pass && j == 1) {
                    wv[i] = wpre[1][i];
                } else {
                    wv[i] = make_uint4(0, 0, 0, 0);
                    if (e0 + i < a.E && kin)
                        wv[i] = ldg_u128_hint(reinterpret_cast<const uint4 *>(a.wg + (size_t)(e0 + i) * a.H + col), wpol);
                }
            }
            uint4 xv[8];
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                xv[n] = make_uint4(0, 0, 0, 0);
                if (n == 0 && one_tok && j == 0) xv[0] = xpre[0];
                else if (n == 0 && one_tok && j == 1) xv[0] = xpre[1];
                else if (n < nt && kin) xv[n] = __ldg(reinterpret_cast<const uint4 *>(a.x + (size_t)(ts + n) * a.H + col));
            }
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                if (n >= nt) continue;
                const uint32_t xu[4] = {xv[n].x, xv[n].y, xv[n].z, xv[n].w};
                float xf[8];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    xf[2 * q] = act_to_f<TA>(static_cast<uint16_t>(xu[q] & 0xffffu));
                    xf[2 * q + 1] = act_to_f<TA>(static_cast<uint16_t>(xu[q] >> 16));
                }
#pragma unroll
                for (int i = 0; i < EPB; ++i) {
                    const uint32_t wu[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
                    float s = acc[i][n];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        s = fmaf(__uint_as_float(wu[q] << 16), xf[2 * q], s);  // router weight is bf16
                        s = fmaf(__uint_as_float(wu[q] & 0xffff0000u), xf[2 * q + 1], s);
                    }
                    acc[i][n] = s;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < EPB; ++i)
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                if (n >= nt) continue;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[i][n] += __shfl_xor_sync(LMOE_FULL, acc[i][n], o);
            }
        if (lane < EPB * 8) {
            float v = 0.0f;
#pragma unroll
            for (int i = 0; i < EPB; ++i)
#pragma unroll
                for (int n = 0; n < 8; ++n)
                    if (lane == i * 8 + n) v = acc[i][n];
            s_red[warp][lane >> 3][lane & 7] = v;
        }
        __syncthreads();
        if (tid < EPB * 8) {
            const int i = tid >> 3, n = tid & 7;
            float v = 0.0f;
            for (int w = 0; w < 8; ++w) v += s_red[w][i][n];
            if (e0 + i < a.E && n < nt) {
                a.partial[(size_t)(ts + n) * a.E + e0 + i] = v;
                if (a.scores) {
                    const float sc = score_fn(v, a.scoring);
                    a.scores[(size_t)(ts + n) * a.E + e0 + i] = make_float2(sc, sc + s_bias[i]);
                }
            }
        }
        __syncthreads();
    }
    if (!a.finish) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned total = gridDim.x * gridDim.y * gridDim.z;
        const unsigned prev = atomicAdd(a.counter, 1u);
        s_last = (prev == total - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid == 0) *a.counter = 0u;
    // small dispatch: the winners and the expert -> slot table (loaded at
    // the kernel start) go through shared memory
    int *s_idx = s_disp;                              // [32]
    int *s_slot = s_disp + 32;                        // [E]
    if (warp_disp) {
        if (tid < a.E) s_slot[tid] = slot_pre[0];
        if (tid + 256 < a.E) s_slot[tid + 256] = slot_pre[1];
        __syncthreads();
    }
    if (a.T == 1 && a.scores && !a.hash_idx && a.E <= 512 && a.top_k <= 16) {
        route_one_token(a, s_slot, warp_disp);
        return;
    }
    for (int tok = warp; tok < a.T; tok += 8)
        topk_token(a.partial, a.scores, 1, a.T, a.E, tok, a.bias, a.scoring, a.top_k, a.norm_topk, a.scaling,
                   a.idx_ws, a.w_ws, a.idx_user, a.w_user, warp_disp ? s_idx : nullptr, a.hash_idx);
    if (!a.do_dispatch) return;
    if (warp_disp) {
        __syncthreads();
        if (warp == 0) dispatch_warp(a.din, a.dout, a.err, s_idx, s_slot);
        return;
    }
    __threadfence();
    __syncthreads();
    dispatch_block(a.din, a.dout, a.err, s_disp);
}

// Router logits for many tokens on the tensor cores (bf16 activations, the
// prefill regime): logits[t][e] = sum_k x[t][k] * Wg[e][k].  bf16 x bf16
// products are exact in fp32 and accumulate in fp32, the arithmetic of the
// per-token path above in another summation order.  Block: 64 tokens x 128
// experts; 8 warps as 2 x 4, each 32 tokens x 32 experts with mma.sync
// m16n8k16; K in stages of 64 columns through a 3-stage cp.async pipeline
// (128-byte rows, 16-byte chunks XOR-swizzled by row for ldmatrix).  Writes
// the logits and, for the element-wise scorings, (score, score + bias); the
// top-k runs in topk_kernel.
constexpr int kRlBM = 64, kRlBN = 128, kRlBK = 64, kRlStages = 3;
constexpr int kRlABytes = kRlBM * 128, kRlStage = (kRlBM + kRlBN) * 128;
constexpr int kRlSmem = kRlStages * kRlStage;

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void cp16_zfill(uint32_t dst, const void *src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0)
                 : "memory");
}

__global__ void __launch_bounds__(256) router_logits_mma_kernel(RouterArgs a) {
    extern __shared__ __align__(128) uint8_t rl_smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * kRlBM, e0 = blockIdx.y * kRlBN;
    const int wm = warp >> 2, wn = warp & 3;
    const uint32_t sb = smem_u32(rl_smem);
    // split z of the hidden dimension: stages [kt0, kt0 + KT)
    const int ks = a.ksplit > 1 ? a.ksplit : 1;
    const int KT = a.H / kRlBK / ks;
    const int kt0 = static_cast<int>(blockIdx.z) * KT;
    pdl_wait();
    pdl_trigger();
    if (a.zero) {
        const int nb = gridDim.x * gridDim.y;
        for (int i = (blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + tid; i < a.zero_words; i += nb * blockDim.x)
            a.zero[i] = 0u;
    }
    auto load_stage = [&](int kt) {
        const int kc = (kt0 + kt) * kRlBK;
        const uint32_t base = sb + (uint32_t)((kt % kRlStages) * kRlStage);
        for (int i = tid; i < (kRlBM + kRlBN) * 8; i += 256) {
            const int row = i >> 3, ch = i & 7;
            if (row < kRlBM) {
                const int t = t0 + row;
                const uint16_t *src = a.x + (size_t)min(t, a.T - 1) * a.H + kc + ch * 8;
                cp16_zfill(base + row * 128 + ((ch ^ (row & 7)) << 4), src, t < a.T);
            } else {
                const int r = row - kRlBM, e = e0 + r;
                const uint16_t *src = a.wg + (size_t)min(e, a.E - 1) * a.H + kc + ch * 8;
                cp16_zfill(base + kRlABytes + r * 128 + ((ch ^ (r & 7)) << 4), src, e < a.E);
            }
        }
    };
    for (int s = 0; s < kRlStages - 1; ++s) {
        if (s < KT) load_stage(s);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    float acc[2][4][4];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mi][ni][e] = 0.0f;
    for (int kt = 0; kt < KT; ++kt) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kRlStages - 2) : "memory");
        __syncthreads();  // stage kt landed for every thread; stage kt-1 is free
        if (kt + kRlStages - 1 < KT) load_stage(kt + kRlStages - 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const uint32_t As = sb + (uint32_t)((kt % kRlStages) * kRlStage), Bs = As + kRlABytes;
#pragma unroll
        for (int kk = 0; kk < kRlBK / 16; ++kk) {
            uint32_t af[2][4], bf[4][2];
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) {
                const int row = wm * 32 + mi * 16 + (lane & 15);
                const int ch = kk * 2 + (lane >> 4);
                ldsm_x4(af[mi], As + row * 128 + ((ch ^ (row & 7)) << 4));
            }
#pragma unroll
            for (int nj = 0; nj < 2; ++nj) {
                const int row = wn * 32 + nj * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int ch = kk * 2 + ((lane >> 3) & 1);
                uint32_t r[4];
                ldsm_x4(r, Bs + row * 128 + ((ch ^ (row & 7)) << 4));
                bf[2 * nj][0] = r[0];
                bf[2 * nj][1] = r[1];
                bf[2 * nj + 1][0] = r[2];
                bf[2 * nj + 1][1] = r[3];
            }
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                for (int ni = 0; ni < 4; ++ni)
                    Act<__nv_bfloat16>::mma(acc[mi][ni], af[mi][0], af[mi][1], af[mi][2], af[mi][3], bf[ni][0],
                                            bf[ni][1]);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int t = t0 + wm * 32 + mi * 16 + g + 8 * (e >> 1);
                const int ex = e0 + wn * 32 + ni * 8 + 2 * tq + (e & 1);
                if (t >= a.T || ex >= a.E) continue;
                const float v = acc[mi][ni][e];
                a.partial[((size_t)blockIdx.z * a.T + t) * a.E + ex] = v;
                if (a.scores && ks == 1) {
                    const float sc = score_fn(v, a.scoring);
                    a.scores[(size_t)t * a.E + ex] = make_float2(sc, sc + (a.bias ? a.bias[ex] : 0.0f));
                }
            }
}

// ------------------------------------------------------------ large dispatch
// Deterministic counting sort for many routes (the prefill regime), stable in
// route order like the single-block dispatch.  Pass 1: each 256-route block
// counts its routes per bucket.  Pass 2 (one block): per bucket, the totals
// and each block's starting position; the bucket offsets (exclusive scan).
// Pass 3: each block scatters its routes (rank inside the block from per-warp
// counts and __match_any_sync).  dispatch_chunks_kernel then cuts the chunks.
__device__ __forceinline__ int dispatch_bucket(const DispatchIn &din, int r, int32_t *err) {
    const int id = din.idx[r];
    if (id < 0 || id >= din.n_experts) {
        if (!(din.drop_zero && id < 0)) set_error(err, -3);
        return din.n_experts;
    }
    return id;
}

__global__ void __launch_bounds__(256) dispatch_count_kernel(DispatchIn din, DispatchOut dout, int32_t *err) {
    __shared__ int s_cnt[kDispatchSmallMaxBuckets + 1];
    pdl_wait();
    pdl_trigger();
    const int NBk = din.n_experts + 1;
    for (int i = threadIdx.x; i < NBk; i += blockDim.x) s_cnt[i] = 0;
    __syncthreads();
    const int r = blockIdx.x * 256 + threadIdx.x;
    if (r < din.R) atomicAdd(&s_cnt[dispatch_bucket(din, r, err)], 1);
    __syncthreads();
    for (int i = threadIdx.x; i < NBk; i += blockDim.x) dout.blk[(size_t)blockIdx.x * NBk + i] = s_cnt[i];
}

// Pass 2, one block of 1024 threads: a warp per bucket turns that bucket's
// per-block counts into exclusive per-block offsets (within the bucket) and
// totals it; then the bucket offsets are an exclusive scan of the totals.
__global__ void __launch_bounds__(1024) dispatch_scan_kernel(DispatchIn din, DispatchOut dout, int nblk) {
    __shared__ int s_tot[kDispatchSmallMaxBuckets + 1];
    __shared__ int s_wsum[32];
    pdl_wait();
    pdl_trigger();
    const int NBk = din.n_experts + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < NBk; b += 32) {
        int run = 0;
        for (int k0 = 0; k0 < nblk; k0 += 32) {
            const int k = k0 + lane;
            int *c = dout.blk + (size_t)k * NBk + b;
            const int v = k < nblk ? *c : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(LMOE_FULL, incl, o);
                if (lane >= o) incl += n;
            }
            if (k < nblk) *c = run + incl - v;
            run += __shfl_sync(LMOE_FULL, incl, 31);
        }
        if (lane == 0) s_tot[b] = run;
    }
    __syncthreads();
    // exclusive scan of the totals: thread t owns buckets 2t, 2t+1
    const int b0 = 2 * threadIdx.x;
    const int t0 = b0 < NBk ? s_tot[b0] : 0, t1 = b0 + 1 < NBk ? s_tot[b0 + 1] : 0;
    int incl = t0 + t1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(LMOE_FULL, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = s_wsum[lane], wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(LMOE_FULL, wi, o);
            if (lane >= o) wi += n;
        }
        s_wsum[lane] = wi - w;
    }
    __syncthreads();
    const int ex = s_wsum[warp] + incl - (t0 + t1);
    if (b0 < NBk) {
        dout.counts[b0] = t0;
        dout.route_off[b0] = ex;
    }
    if (b0 + 1 < NBk) {
        dout.counts[b0 + 1] = t1;
        dout.route_off[b0 + 1] = ex + t0;
    }
}

__global__ void __launch_bounds__(256) dispatch_scatter_kernel(DispatchIn din, DispatchOut dout) {
    __shared__ int s_wcnt[8][kDispatchSmallMaxBuckets + 1];
    pdl_wait();
    pdl_trigger();
    const int NBk = din.n_experts + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = lane; i < NBk; i += 32) s_wcnt[warp][i] = 0;
    __syncwarp();
    const int r = blockIdx.x * 256 + threadIdx.x;
    int b = 0x7fffffff;
    if (r < din.R) {
        const int id = din.idx[r];
        b = (id < 0 || id >= din.n_experts) ? din.n_experts : id;
    }
    const unsigned same = __match_any_sync(LMOE_FULL, b);
    const int rank = __popc(same & ((1u << lane) - 1u));
    if (r < din.R && rank == 0) s_wcnt[warp][b] = __popc(same);
    __syncthreads();
    if (r < din.R) {
        int pos = dout.route_off[b] + dout.blk[(size_t)blockIdx.x * NBk + b] + rank;
        for (int w = 0; w < warp; ++w) pos += s_wcnt[w][b];
        dout.sorted_routes[pos] = r;
    }
}

__global__ void __launch_bounds__(256) topk_kernel(TopkArgs a) {
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int tok = blockIdx.x * 8 + warp;
    if (tok >= a.T) return;
    topk_token(a.partial, a.scores, a.ksplit, a.T, a.E, tok, a.bias, a.scoring, a.top_k, a.norm_topk,
               a.scaling, a.idx_ws, a.w_ws, a.idx_user, a.w_user, nullptr, a.hash_idx);
}

// ============================================================ activation panel
// Natural [rows, K] activations -> consumer panel layout + 16-column sums
// (sums in column order, as the router's panel producer computes them).
template <typename TA>
__global__ void __launch_bounds__(256) panel_kernel(PanelArgs a) {
    pdl_wait();
    pdl_trigger();
    if (a.zero) {
        const int b = blockIdx.y * gridDim.x + blockIdx.x, nb = gridDim.x * gridDim.y;
        for (int i = b * blockDim.x + threadIdx.x; i < a.zero_words; i += nb * blockDim.x) a.zero[i] = 0u;
    }
    const int row = blockIdx.x;
    const int col = blockIdx.y * 256 + threadIdx.x;
    const uint16_t *src = a.x + (size_t)row * (a.x_stride ? a.x_stride : a.K);
    if (col < a.K) {
        int p;
        const int pos = panel_pos(col, a.bits, a.gs, &p);
        a.panel[(size_t)row * a.K + pos] = Act<TA>::from_f(Act<TA>::to_f(src[col]) * prescale(p));
    }
    if (threadIdx.x < 16) {
        const int c0 = blockIdx.y * 256 + threadIdx.x * 16;
        if (c0 < a.K) {
            // two serial 8-column halves, then lo + hi (the router's order);
            // the second sum is over the stored (prescaled) panel values
            float lo = 0.0f, hi = 0.0f, plo = 0.0f, phi = 0.0f;
            for (int q = 0; q < 16; ++q) {
                int p;
                panel_pos(c0 + q, a.bits, a.gs, &p);
                const float f = Act<TA>::to_f(src[c0 + q]);
                const float fp = Act<TA>::to_f(Act<TA>::from_f(f * prescale(p)));
                if (q < 8) {
                    lo += f;
                    plo += fp;
                } else {
                    hi += f;
                    phi += fp;
                }
            }
            *reinterpret_cast<float2 *>(a.sum16 + ((size_t)row * (a.K / 16) + c0 / 16) * 2) =
                make_float2(lo + hi, plo + phi);
        }
    }
}

// ============================================================ launchers
cudaError_t launch_router(const RouterArgs &a, int /*ksplit*/, cudaStream_t st) {
    dim3 grid((a.E + 1) / 2, (a.T + 63) / 64, 1);
    if (a.act_f16) return launch_pdl(router_kernel<__half>, grid, dim3(256), 0, st, a);
    return launch_pdl(router_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, a);
}

cudaError_t launch_topk(const TopkArgs &a, cudaStream_t st) {
    return launch_pdl(topk_kernel, dim3((a.T + 7) / 8), dim3(256), 0, st, a);
}

cudaError_t launch_dispatch_small(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                                  cudaStream_t st) {
    return launch_pdl(dispatch_small_kernel, dim3(1), dim3(256), 0, st, din, dout, err);
}

cudaError_t launch_dispatch_large(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                                  cudaStream_t st) {
    cudaError_t e;
    if (dout.blk && din.n_experts + 1 <= kDispatchSmallMaxBuckets) {
        const int nblk = (din.R + 255) / 256;
        e = launch_pdl(dispatch_count_kernel, dim3(nblk), dim3(256), 0, st, din, dout, err);
        if (e == cudaSuccess) e = launch_pdl(dispatch_scan_kernel, dim3(1), dim3(1024), 0, st, din, dout, nblk);
        if (e == cudaSuccess) e = launch_pdl(dispatch_scatter_kernel, dim3(nblk), dim3(256), 0, st, din, dout);
    } else {
        e = launch_pdl(dispatch_rank_kernel, dim3(din.n_experts + 1), dim3(256), 0, st, din, dout, err);
    }
    if (e != cudaSuccess) return e;
    return launch_pdl(dispatch_chunks_kernel, dim3(1), dim3(256), 0, st, din, dout, err);
}

cudaError_t launch_router_logits_mma(const RouterArgs &a, cudaStream_t st) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(router_logits_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kRlSmem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const int ks = a.ksplit > 1 ? a.ksplit : 1;
    if (a.H % (kRlBK * ks) != 0) return cudaErrorInvalidValue;
    dim3 grid((a.T + kRlBM - 1) / kRlBM, (a.E + kRlBN - 1) / kRlBN, ks);
    return launch_pdl(router_logits_mma_kernel, grid, dim3(256), kRlSmem, st, a);
}

cudaError_t launch_panel(const PanelArgs &a, cudaStream_t st) {
    dim3 grid(a.rows, (a.K + 255) / 256);
    if (a.act_f16)
        return launch_pdl(panel_kernel<__half>, grid, dim3(256), 0, st, a);
    else
        return launch_pdl(panel_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, a);
}

}  // namespace lmoe
