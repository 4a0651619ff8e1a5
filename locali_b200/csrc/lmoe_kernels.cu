// Routed-MoE kernels for sm_100a: router, dispatch, activation panels and the
// fused dequant-GEMV expert products (gate/up + clamped SwiGLU, down + combine).
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
            set_error(err, -3);
        }
        s_b[r] = b;
        atomicAdd(&s_cnt[b], 1);
    }
    __syncthreads();
    const int per = (NBk + 255) >> 8;
    int lr = 0, lc = 0;
    for (int q = 0; q < per; ++q) {
        const int b = tid * per + q;
        if (b < NBk) {
            lr += s_cnt[b];
            lc += (s_cnt[b] + kChunkTok - 1) / kChunkTok;
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
            ec += (s_cnt[b] + kChunkTok - 1) / kChunkTok;
        }
    }
    __syncthreads();
    for (int r = tid; r < R; r += blockDim.x) {
        const int b = s_b[r];
        int rank = 0;
        for (int r2 = 0; r2 < r; ++r2) rank += (s_b[r2] == b);
        const int pos = s_roff[b] + rank;
        dout.sorted_routes[pos] = r;
        if ((rank % kChunkTok) == 0) {
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
            ch.ntok = min(kChunkTok, s_cnt[b] - rank);
            ch.expert = b;
            dout.chunks[s_coff[b] + rank / kChunkTok] = ch;
        }
    }
    if (tid == 0) *dout.n_chunks = tc;
    __syncthreads();
}

__global__ void __launch_bounds__(256) dispatch_small_kernel(DispatchIn din, DispatchOut dout,
                                                             int32_t *err) {
    __shared__ int s_mem[kDispatchSmallMaxRoutes + 3 * (kDispatchSmallMaxBuckets + 1) + 16];
    dispatch_block(din, dout, err, s_mem);
}

// Large-R dispatch, pass 1: one block per bucket counts its routes and the
// routes of lower buckets, then ranks its own routes in route order.
__global__ void __launch_bounds__(256) dispatch_rank_kernel(DispatchIn din, DispatchOut dout,
                                                            int32_t *err) {
    __shared__ int s_tmp[9];
    const int b = blockIdx.x;
    const int E = din.n_experts;
    const int tid = threadIdx.x;
    int lt = 0, eq = 0;
    for (int r = tid; r < din.R; r += blockDim.x) {
        int id = din.idx[r];
        if (id < 0 || id >= E) {
            id = E;
            if (b == 0) set_error(err, -3);
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
    const int NBk = din.n_experts + 1;
    const int tid = threadIdx.x;
    const int per = (NBk + 255) >> 8;
    int lc = 0;
    for (int q = 0; q < per; ++q) {
        const int b = tid * per + q;
        if (b < NBk) lc += (dout.counts[b] + kChunkTok - 1) / kChunkTok;
    }
    int tc;
    int ec = block_scan_256(lc, s_tmp, &tc);
    for (int q = 0; q < per; ++q) {
        const int b = tid * per + q;
        if (b >= NBk) continue;
        const int cnt = dout.counts[b];
        int slot = 0;
        if (b < din.n_experts && cnt > 0) {
            slot = din.expert_slot ? din.expert_slot[b] : b;
            if (slot < 0 || slot >= din.n_slots) {
                set_error(err, -3);
                slot = 0;
            }
        }
        for (int c0 = 0; c0 < cnt; c0 += kChunkTok) {
            Chunk ch;
            ch.slot = slot;
            ch.route_start = dout.route_off[b] + c0;
            ch.ntok = min(kChunkTok, cnt - c0);
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
// routed scaling.  Ties go to the lower expert id.
__device__ void topk_token(const float *partial, int ksplit, int T, int E, int tok,
                           const float *bias, int scoring, int top_k, int norm, float scaling,
                           int32_t *idx_ws, float *w_ws, int32_t *idx_user, float *w_user) {
    const int lane = threadIdx.x & 31;
    float sc[kRouterMaxEPL], bs[kRouterMaxEPL];
    float mx = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < kRouterMaxEPL; ++i) {
        const int e = lane + 32 * i;
        float lg = -FLT_MAX;
        if (e < E) {
            lg = 0.0f;
            for (int ky = 0; ky < ksplit; ++ky)
                lg += __ldcg(partial + ((size_t)ky * T + tok) * E + e);
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
        bs[i] = (e < E) ? sc[i] + (bias ? bias[e] : 0.0f) : -FLT_MAX;
        if (e >= E) bs[i] = -INFINITY;
    }
    float sel_s[16];
    int sel_e[16];
    float ssum = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        if (j >= top_k) break;
        float bv = -INFINITY;
        int be = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kRouterMaxEPL; ++i) {
            if (bs[i] > bv) {
                bv = bs[i];
                be = lane + 32 * i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(LMOE_FULL, bv, o);
            const int oe = __shfl_xor_sync(LMOE_FULL, be, o);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        float ws = 0.0f;
#pragma unroll
        for (int i = 0; i < kRouterMaxEPL; ++i) {
            if (lane + 32 * i == be) {
                ws = sc[i];
                bs[i] = -INFINITY;
            }
        }
        ws = __shfl_sync(LMOE_FULL, ws, be & 31);
        sel_s[j] = ws;
        sel_e[j] = be;
        ssum += ws;
    }
    if (lane == 0) {
        const float den = ssum + 1e-20f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (j >= top_k) break;
            float wv = norm ? sel_s[j] / den : sel_s[j];
            wv *= scaling;
            const size_t o = (size_t)tok * top_k + j;
            idx_ws[o] = sel_e[j];
            w_ws[o] = wv;
            if (idx_user) idx_user[o] = sel_e[j];
            if (w_user) w_user[o] = wv;
        }
    }
}

template <typename TA>
__device__ __forceinline__ float act_to_f(uint16_t v) {
    return Act<TA>::to_f(v);
}

// Router logits x @ Wg^T in fp32 (products of bf16 values are exact) over a
// (32-expert, 256-column, 64-token) tile; partial sums per column slice.
// Block 0 of each column slice also writes the gate/up activation panel.
// In the decode regime the last block to finish runs top-k and dispatch, so
// routing costs a single launch and no host synchronisation (the reference
// syncs here every layer, arena.py:513).
template <typename TA>
__global__ void __launch_bounds__(256) router_kernel(RouterArgs a) {
    __shared__ __align__(16) uint16_t s_x[8][kRouterKS];
    __shared__ int s_last;
    __shared__ int s_disp[kDispatchSmallMaxRoutes + 3 * (kDispatchSmallMaxBuckets + 1) + 16];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int e0 = blockIdx.x * 32 + warp * 4;
    const int k0 = blockIdx.y * kRouterKS;
    const int tbeg = blockIdx.z * 64;
    const int tend = min(a.T, tbeg + 64);

    float wv[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int e = e0 + i;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (e < a.E) v = __ldg(reinterpret_cast<const uint4 *>(a.wg + (size_t)e * a.H + k0 + lane * 8));
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            wv[i][2 * q] = __uint_as_float(u[q] << 16);            // router weight is bf16
            wv[i][2 * q + 1] = __uint_as_float(u[q] & 0xffff0000u);
        }
    }

    for (int ts = tbeg; ts < tend; ts += 8) {
        const int nt = min(8, tend - ts);
        __syncthreads();
        {
            const int n = tid >> 5, c = (tid & 31) * 8;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (n < nt) v = __ldg(reinterpret_cast<const uint4 *>(a.x + (size_t)(ts + n) * a.H + k0 + c));
            *reinterpret_cast<uint4 *>(&s_x[n][c]) = v;
        }
        __syncthreads();
        if (a.xpanel && blockIdx.x == 0) {
            const int n = tid >> 5;
            if (n < nt) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int cl = (tid & 31) * 8 + q;
                    const int col = k0 + cl;
                    int p;
                    const int pos = panel_pos(col, a.pbits, a.pgs, &p);
                    const float v = act_to_f<TA>(s_x[n][cl]) * (p == 0 ? 1.0f : (p == 1 ? 0.25f : 0.0625f));
                    a.xpanel[(size_t)(ts + n) * a.H + pos] = Act<TA>::from_f(v);
                }
            }
            if (tid < 128) {
                const int n2 = tid >> 4, blk = tid & 15;
                if (n2 < nt) {
                    float s = 0.0f;
#pragma unroll
                    for (int q = 0; q < 16; ++q) s += act_to_f<TA>(s_x[n2][blk * 16 + q]);
                    a.xsum16[(size_t)(ts + n2) * (a.H / 16) + k0 / 16 + blk] = s;
                }
            }
        }
        float acc[4][8];
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i][n] = 0.0f;
            if (n < nt) {
                const uint4 v = *reinterpret_cast<const uint4 *>(&s_x[n][lane * 8]);
                const uint32_t u[4] = {v.x, v.y, v.z, v.w};
                float xv[8];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    xv[2 * q] = act_to_f<TA>(static_cast<uint16_t>(u[q] & 0xffffu));
                    xv[2 * q + 1] = act_to_f<TA>(static_cast<uint16_t>(u[q] >> 16));
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float s = 0.0f;
#pragma unroll
                    for (int q = 0; q < 8; ++q) s = fmaf(wv[i][q], xv[q], s);
                    acc[i][n] = s;
                }
            }
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            if (n < nt) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1)
                        acc[i][n] += __shfl_xor_sync(LMOE_FULL, acc[i][n], o);
                }
            }
        }
        {
            const int i = lane >> 3, n = lane & 7;
            float v = 0.0f;
#pragma unroll
            for (int ii = 0; ii < 4; ++ii)
#pragma unroll
                for (int nn = 0; nn < 8; ++nn)
                    if (ii == i && nn == n) v = acc[ii][nn];
            const int e = e0 + i;
            if (e < a.E && n < nt) a.partial[((size_t)blockIdx.y * a.T + ts + n) * a.E + e] = v;
        }
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
    for (int tok = warp; tok < a.T; tok += 8)
        topk_token(a.partial, gridDim.y, a.T, a.E, tok, a.bias, a.scoring, a.top_k, a.norm_topk,
                   a.scaling, a.idx_ws, a.w_ws, a.idx_user, a.w_user);
    if (!a.do_dispatch) return;
    __threadfence();
    __syncthreads();
    dispatch_block(a.din, a.dout, a.err, s_disp);
}

__global__ void __launch_bounds__(256) topk_kernel(TopkArgs a) {
    const int warp = threadIdx.x >> 5;
    const int tok = blockIdx.x * 8 + warp;
    if (tok >= a.T) return;
    topk_token(a.partial, a.ksplit, a.T, a.E, tok, a.bias, a.scoring, a.top_k, a.norm_topk,
               a.scaling, a.idx_ws, a.w_ws, a.idx_user, a.w_user);
}

// ============================================================ activation panel
// Natural [rows, K] activations -> consumer panel layout + 16-column sums.
template <typename TA>
__global__ void __launch_bounds__(256) panel_kernel(PanelArgs a) {
    const int row = blockIdx.x;
    const int col = blockIdx.y * 256 + threadIdx.x;
    const uint16_t *src = a.x + (size_t)row * a.K;
    if (col < a.K) {
        int p;
        const int pos = panel_pos(col, a.bits, a.gs, &p);
        const float v = Act<TA>::to_f(src[col]) * (p == 0 ? 1.0f : (p == 1 ? 0.25f : 0.0625f));
        a.panel[(size_t)row * a.K + pos] = Act<TA>::from_f(v);
    }
    if (threadIdx.x < 16) {
        const int c0 = blockIdx.y * 256 + threadIdx.x * 16;
        if (c0 < a.K) {
            float s = 0.0f;
            for (int q = 0; q < 16; ++q) s += Act<TA>::to_f(src[c0 + q]);
            a.sum16[(size_t)row * (a.K / 16) + c0 / 16] = s;
        }
    }
}

// ============================================================ expert GEMV
// One unit = (chunk of <= 8 routes of one expert, 16-row tile).  The block's
// warps split K; each warp stages its slice of the routes' activation panel
// in shared memory with a bulk copy, streams its codes/scales/biases from HBM
// (software pipelined), and runs the m16n8k16 products per quantisation
// group.  MODE_GATEUP fuses gate and up and applies the clamped SwiGLU
// (dsv4_arena.py:223-235 / dsv4_kernels.py:165-170); MODE_DOWN applies the
// combine weight and finishes each token's weighted sum in route order
// (arena.py:543,619-624) once all its routes are in; MODE_QMM writes the
// plain gather_qmm output.
template <typename TA, int BITS, int GS, int MODE>
__global__ void __launch_bounds__(256) gemv_kernel(const GemvArgs a) {
    using Gm = Geo<BITS, GS>;
    constexpr bool PAIR = (MODE == MODE_GATEUP);
    constexpr int NM = PAIR ? 2 : 1;
    constexpr int NROW = 2 * NM;
    constexpr int WPS = Gm::kWps;
    constexpr int NB = 2;
    constexpr int NP = Gm::kCpw / 2;
    constexpr int SPW = Gm::kStepsPerWord;

    const int nw = blockDim.x >> 5;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int K = a.q0.cols;
    const int GT = K / GS;
    const int Gw = GT / nw;
    const int Gbeg = warp * Gw;
    const int kw = Gw * GS;
    const int rows = a.q0.rows;
    const int RT = rows >> 4;
    const int nch = *a.n_chunks;
    const int units = nch * RT;
    const int pstride = kw * 2 + 32;

    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *s_bar = reinterpret_cast<uint64_t *>(smem);
    int *s_route = reinterpret_cast<int *>(smem + 64);
    int *s_fin = s_route + 8;
    float *s_red = reinterpret_cast<float *>(smem + 128);
    const int red_bytes = nw * 32 * NM * 4 * 4;
    const int wsz = ((Gw * 32 + a.ntok_max * pstride) + 127) & ~127;
    uint8_t *s_wbase = smem + 128 + ((red_bytes + 127) & ~127) + warp * wsz;
    float *s_xs = reinterpret_cast<float *>(s_wbase);
    uint8_t *s_pan = s_wbase + ((Gw * 32 + 15) & ~15);

    if (lane == 0) mbar_init(&s_bar[warp], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    uint32_t phase = 0;

    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int rt = u / nch;
        const int c = u - rt * nch;
        const Chunk ch = a.chunks[c];
        int slot = ch.slot;
        if (slot < 0 || slot >= a.n_slots) {
            if (tid == 0) set_error(a.err, -3);
            slot = 0;
        }
        int ntok = ch.ntok;
        if (ntok > a.ntok_max || ntok < 0) {
            if (tid == 0) set_error(a.err, -3);
            ntok = ntok < 0 ? 0 : a.ntok_max;
        }
        if (tid < 8) s_route[tid] = (tid < ntok) ? a.sorted_routes[ch.route_start + tid] : -1;
        __syncthreads();

        if (lane == 0 && ntok > 0) {
            fence_proxy_async();
            mbar_expect_tx(&s_bar[warp], static_cast<uint32_t>(ntok * kw * 2));
            for (int n = 0; n < ntok; ++n) {
                const int r = s_route[n];
                const uint16_t *src = a.panel + (size_t)(r / a.route_div) * K + (size_t)Gbeg * GS;
                bulk_g2s(s_pan + n * pstride, src, static_cast<uint32_t>(kw * 2), &s_bar[warp]);
            }
        }
        for (int i = lane; i < Gw * 8; i += 32) {
            const int gi = i >> 3, n = i & 7;
            float v = 0.0f;
            if (n < ntok) {
                const int r = s_route[n];
                const float *p = a.sum16 + (size_t)(r / a.route_div) * (K / 16) + (Gbeg + gi) * (GS / 16);
#pragma unroll
                for (int q = 0; q < GS / 16; ++q) v += p[q];
            }
            s_xs[i] = v;
        }

        const uint32_t *wrow[NROW];
        const uint16_t *srow[NROW];
        const uint16_t *brow[NROW];
#pragma unroll
        for (int m = 0; m < NM; ++m) {
            const QView &q = m ? a.q1 : a.q0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = rt * 16 + g + 8 * h;
                wrow[2 * m + h] = q.w + (size_t)slot * q.w_slot_stride + (size_t)row * q.words_per_row +
                                  (size_t)Gbeg * Gm::kWordsPerGroup + t * WPS;
                const size_t so = (size_t)slot * q.sb_slot_stride + (size_t)row * q.groups_per_row + Gbeg;
                srow[2 * m + h] = q.s + so;
                brow[2 * m + h] = q.b + so;
            }
        }

        float acc[NM][4];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[m][e] = 0.0f;

        uint32_t wA[NB][NROW][WPS], wB[NB][NROW][WPS];
        uint16_t sA[NB][NROW], bA[NB][NROW], sB[NB][NROW], bB[NB][NROW];

        auto load = [&](int gi0, uint32_t (&W)[NB][NROW][WPS], uint16_t (&S)[NB][NROW],
                        uint16_t (&Bi)[NB][NROW]) {
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                const int gi = gi0 + i;
                if (gi < Gw) {
#pragma unroll
                    for (int r = 0; r < NROW; ++r) {
                        SliceLoad<WPS>::run(wrow[r] + gi * Gm::kWordsPerGroup, W[i][r]);
                        S[i][r] = ldg_u16(srow[r] + gi);
                        Bi[i][r] = ldg_u16(brow[r] + gi);
                    }
                }
            }
        };
        auto compute = [&](int gi0, uint32_t (&W)[NB][NROW][WPS], uint16_t (&S)[NB][NROW],
                           uint16_t (&Bi)[NB][NROW]) {
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                const int gi = gi0 + i;
                if (gi < Gw) {
                    float d[NM][4];
#pragma unroll
                    for (int m = 0; m < NM; ++m)
#pragma unroll
                        for (int e = 0; e < 4; ++e) d[m][e] = 0.0f;
#pragma unroll
                    for (int wi = 0; wi < WPS; ++wi) {
                        uint32_t P[NROW][NP];
#pragma unroll
                        for (int r = 0; r < NROW; ++r) Unpack<TA, BITS>::run(W[i][r][wi], P[r]);
#pragma unroll
                        for (int s = 0; s < SPW; ++s) {
                            const int kl = gi * Gm::kSteps + wi * SPW + s;
                            uint2 bv = make_uint2(0u, 0u);
                            if (g < ntok)
                                bv = *reinterpret_cast<const uint2 *>(s_pan + g * pstride + (kl * 4 + t) * 8);
#pragma unroll
                            for (int m = 0; m < NM; ++m)
                                Act<TA>::mma(d[m], P[2 * m][2 * s], P[2 * m + 1][2 * s], P[2 * m][2 * s + 1],
                                             P[2 * m + 1][2 * s + 1], bv.x, bv.y);
                        }
                    }
                    const float xs0 = s_xs[gi * 8 + 2 * t];
                    const float xs1 = s_xs[gi * 8 + 2 * t + 1];
#pragma unroll
                    for (int m = 0; m < NM; ++m) {
                        const float s0 = Act<TA>::to_f(S[i][2 * m]), s1 = Act<TA>::to_f(S[i][2 * m + 1]);
                        const float b0 = Act<TA>::to_f(Bi[i][2 * m]), b1 = Act<TA>::to_f(Bi[i][2 * m + 1]);
                        acc[m][0] += fmaf(s0, d[m][0], b0 * xs0);
                        acc[m][1] += fmaf(s0, d[m][1], b0 * xs1);
                        acc[m][2] += fmaf(s1, d[m][2], b1 * xs0);
                        acc[m][3] += fmaf(s1, d[m][3], b1 * xs1);
                    }
                }
            }
        };

        load(0, wA, sA, bA);
        __syncwarp();
        if (ntok > 0) {
            if (!mbar_wait(&s_bar[warp], phase)) set_error(a.err, -4);
            phase ^= 1u;
        }
        for (int gi = 0; gi < Gw; gi += 2 * NB) {
            load(gi + NB, wB, sB, bB);
            compute(gi, wA, sA, bA);
            load(gi + 2 * NB, wA, sA, bA);
            compute(gi + NB, wB, sB, bB);
        }

        // split-K reduction across the block's warps (fixed order)
        {
            float *red = s_red + (warp * 32 + lane) * NM * 4;
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
                for (int e = 0; e < 4; ++e) red[m * 4 + e] = acc[m][e];
        }
        __syncthreads();
        if (warp == 0) {
            float fin[NM][4];
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
                for (int e = 0; e < 4; ++e) fin[m][e] = 0.0f;
            for (int w = 0; w < nw; ++w) {
                const float *red = s_red + (w * 32 + lane) * NM * 4;
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int e = 0; e < 4; ++e) fin[m][e] += red[m * 4 + e];
            }
            if constexpr (MODE == MODE_GATEUP) {
                float hv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float gv = Act<TA>::round(fin[0][e]);
                    float uv = Act<TA>::round(fin[1][e]);
                    if (a.limit > 0.0f) {
                        uv = fminf(fmaxf(uv, -a.limit), a.limit);
                        gv = fminf(gv, a.limit);
                    }
                    float h;
                    if (a.swiglu_mode == 0) {
                        const float silu = gv / (1.0f + expf(-gv));
                        h = Act<TA>::round(silu * uv);
                    } else {
                        const float sig = Act<TA>::round(1.0f / (1.0f + expf(-gv)));
                        const float sg = Act<TA>::round(gv * sig);
                        h = Act<TA>::round(sg * uv);
                    }
                    const int n = 2 * t + (e & 1);
                    const int row = rt * 16 + g + 8 * (e >> 1);
                    hv[e] = 0.0f;
                    if (n < ntok) {
                        const int r = s_route[n];
                        hv[e] = h;
                        if (a.out_panel) {
                            int p;
                            const int pos = panel_pos(row, a.out_bits, a.out_gs, &p);
                            const float sc = (p == 0 ? 1.0f : (p == 1 ? 0.25f : 0.0625f));
                            a.out[(size_t)r * rows + pos] = Act<TA>::from_f(h * sc);
                        } else {
                            a.out[(size_t)r * rows + row] = Act<TA>::from_f(h);
                        }
                    }
                }
                if (a.out_sum16) {
                    float s0 = hv[0] + hv[2];
                    float s1 = hv[1] + hv[3];
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) {
                        s0 += __shfl_xor_sync(LMOE_FULL, s0, o);
                        s1 += __shfl_xor_sync(LMOE_FULL, s1, o);
                    }
                    if (g == 0) {
                        if (2 * t < ntok) a.out_sum16[(size_t)s_route[2 * t] * RT + rt] = s0;
                        if (2 * t + 1 < ntok) a.out_sum16[(size_t)s_route[2 * t + 1] * RT + rt] = s1;
                    }
                }
            } else if constexpr (MODE == MODE_DOWN) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int n = 2 * t + (e & 1);
                    const int row = rt * 16 + g + 8 * (e >> 1);
                    if (n < ntok) {
                        const int r = s_route[n];
                        const float y = Act<TA>::round(fin[0][e]);
                        const float wv = Act<TA>::round(a.route_w[r]);
                        a.out[(size_t)r * rows + row] = Act<TA>::from_f(y * wv);
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int n = 2 * t + (e & 1);
                    const int row = rt * 16 + g + 8 * (e >> 1);
                    if (n < ntok) a.out[(size_t)s_route[n] * rows + row] = Act<TA>::from_f(fin[0][e]);
                }
            }
        }
        if constexpr (MODE == MODE_DOWN) {
            __threadfence();
            __syncthreads();
            if (tid < 8) {
                int fin_tok = -1;
                if (tid < ntok) {
                    const int r = s_route[tid];
                    const int tok = r / a.top_k;
                    const unsigned prev = atomicAdd(a.counters + (size_t)tok * RT + rt, 1u);
                    if (prev == static_cast<unsigned>(a.top_k - 1)) fin_tok = tok;
                }
                s_fin[tid] = fin_tok;
            }
            __syncthreads();
            for (int n = 0; n < ntok; ++n) {
                const int tok = s_fin[n];
                if (tok < 0) continue;
                __threadfence();
                if (tid < 16) {
                    const int row = rt * 16 + tid;
                    float sacc = 0.0f;
                    for (int j = 0; j < a.top_k; ++j) {
                        const uint16_t v = __ldcg(reinterpret_cast<const unsigned short *>(
                            a.out + ((size_t)tok * a.top_k + j) * rows + row));
                        sacc += Act<TA>::to_f(v);
                    }
                    a.combined[(size_t)tok * rows + row] = Act<TA>::from_f(sacc);
                }
                if (tid == 0) a.counters[(size_t)tok * RT + rt] = 0u;
            }
        }
        __syncthreads();
    }
}

// ============================================================ launchers
static int g_num_sms = 0;
static int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

cudaError_t launch_router(const RouterArgs &a, int ksplit, cudaStream_t st) {
    dim3 grid((a.E + 31) / 32, ksplit, (a.T + 63) / 64);
    if (a.act_f16)
        router_kernel<__half><<<grid, 256, 0, st>>>(a);
    else
        router_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_topk(const TopkArgs &a, cudaStream_t st) {
    topk_kernel<<<(a.T + 7) / 8, 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_dispatch_small(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                                  cudaStream_t st) {
    dispatch_small_kernel<<<1, 256, 0, st>>>(din, dout, err);
    return cudaGetLastError();
}

cudaError_t launch_dispatch_large(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                                  cudaStream_t st) {
    dispatch_rank_kernel<<<din.n_experts + 1, 256, 0, st>>>(din, dout, err);
    dispatch_chunks_kernel<<<1, 256, 0, st>>>(din, dout, err);
    return cudaGetLastError();
}

cudaError_t launch_panel(const PanelArgs &a, cudaStream_t st) {
    dim3 grid(a.rows, (a.K + 255) / 256);
    if (a.act_f16)
        panel_kernel<__half><<<grid, 256, 0, st>>>(a);
    else
        panel_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

template <typename TA, int BITS, int GS, int MODE>
static cudaError_t launch_gemv_t(const GemvArgs &a, int max_chunks, cudaStream_t st) {
    constexpr int NM = (MODE == MODE_GATEUP) ? 2 : 1;
    const int K = a.q0.cols;
    const int GT = K / GS;
    // warps per unit: aim for >= 8 groups per warp, divide the groups evenly
    int nw = 8;
    while (nw > 1 && (GT % nw != 0 || GT / nw < 4)) nw >>= 1;
    const int Gw = GT / nw;
    const int kw = Gw * GS;
    const int pstride = kw * 2 + 32;
    const int red_bytes = nw * 32 * NM * 4 * 4;
    const int wsz = ((Gw * 32 + a.ntok_max * pstride) + 127) & ~127;
    const size_t smem = 128 + ((red_bytes + 127) & ~127) + (size_t)nw * wsz;
    auto kern = gemv_kernel<TA, BITS, GS, MODE>;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    // occupancy depends only on (warps, smem); remember the last answer
    static int cached_nw = -1, cached_per_sm = 0;
    static size_t cached_smem = 0;
    int per_sm = 0;
    if (cached_nw == nw && cached_smem == smem) {
        per_sm = cached_per_sm;
    } else {
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, nw * 32, smem);
        if (e != cudaSuccess) return e;
        cached_nw = nw;
        cached_smem = smem;
        cached_per_sm = per_sm;
    }
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const long units_max = (long)max_chunks * (a.q0.rows / 16);
    long grid = (long)per_sm * num_sms();
    if (grid > units_max) grid = units_max;
    if (grid < 1) grid = 1;
    kern<<<static_cast<unsigned>(grid), nw * 32, smem, st>>>(a);
    return cudaGetLastError();
}

template <typename TA, int MODE>
static cudaError_t launch_gemv_bits(int bits, int gs, const GemvArgs &a, int max_chunks,
                                    cudaStream_t st) {
#define LMOE_CASE(B, G) \
    if (bits == B && gs == G) return launch_gemv_t<TA, B, G, MODE>(a, max_chunks, st);
    LMOE_CASE(2, 64)
    LMOE_CASE(2, 128)
    LMOE_CASE(4, 32)
    LMOE_CASE(4, 64)
    LMOE_CASE(4, 128)
    LMOE_CASE(8, 32)
    LMOE_CASE(8, 64)
    LMOE_CASE(8, 128)
#undef LMOE_CASE
    return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(int mode, int act_f16, int bits, int gs, const GemvArgs &a,
                        int max_chunks, cudaStream_t st) {
    if (act_f16) {
        if (mode == MODE_GATEUP) return launch_gemv_bits<__half, MODE_GATEUP>(bits, gs, a, max_chunks, st);
        if (mode == MODE_DOWN) return launch_gemv_bits<__half, MODE_DOWN>(bits, gs, a, max_chunks, st);
        return launch_gemv_bits<__half, MODE_QMM>(bits, gs, a, max_chunks, st);
    }
    if (mode == MODE_GATEUP) return launch_gemv_bits<__nv_bfloat16, MODE_GATEUP>(bits, gs, a, max_chunks, st);
    if (mode == MODE_DOWN) return launch_gemv_bits<__nv_bfloat16, MODE_DOWN>(bits, gs, a, max_chunks, st);
    return launch_gemv_bits<__nv_bfloat16, MODE_QMM>(bits, gs, a, max_chunks, st);
}

bool gemv_supported(int bits, int gs) {
    return (bits == 2 && (gs == 64 || gs == 128)) || ((bits == 4 || bits == 8) && (gs == 32 || gs == 64 || gs == 128));
}

}  // namespace lmoe
