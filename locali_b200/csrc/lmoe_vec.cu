// Single-token decode GEMVs on the integer tensor pipe (sm_100a).
//
// One token per layer call: every chunk of the dispatch holds one route, and
// each weight byte is read once.  The kernels stream the pre-tiled copy of
// the arena (StreamGeo: blocks of two 16-row tiles x 8 quantisation groups)
// and are built around three choices:
//
// * Integer MMA.  A 2-bit code word holds 4 codes in every byte; one AND
//   with 0x03030303 << 2p keeps code class p of all four bytes as exact u8
//   values c * 4^p, so one logic op yields four A operands of
//   mma.sync.m16n8k32.u8.s8.s32 and no shift is needed.  A separate s32
//   accumulator per class is folded afterwards (sum_p D_p * 4^(3-p)).  4-bit
//   codes have two classes, 8-bit codes one.
// * Exact activations as two int8 pieces.  Each 64-column group (the
//   quantisation group) of the activation row gets a power-of-two scale
//   2^S with max |x| * 2^S < 2^14; x * 2^S is then an integer for every
//   element within 2^6 of the group's largest magnitude (all 8 significant
//   bits of bf16), smaller ones round at 2^-14 of that maximum.  The integer
//   splits exactly into hi * 256 + lo with hi, lo in int8, and the two
//   pieces are two columns of the MMA's B operand.  The products and sums
//   over a group are then exact integers; the group result
//   (256 * hi_sum + lo_sum) * 2^-S is scaled and biased in fp32:
//   acc += scale * sum(x * q) + bias * sum(x)  (dsv4_kernels.py:152-154).
// * Column = (group, piece).  The four lanes of an MMA row quad each feed
//   k-values of their own quantisation group; the eight B columns are those
//   four groups times the two pieces, so one MMA covers 16 rows x 32 codes
//   and a lane's accumulators are its own group's (hi, lo) sums.
//
// Work split: gate/up units are (route, 32-row pair of gate and up); the
// down projection's units are 32-row pairs of the output over all routes.
// Units are dealt to blocks round robin (block b: b, b + G, ...), and a
// block's items (unit, K chunk) round robin to its warps.  Each warp streams
// its items -- its gate/up items, then its down items -- through its own
// ring of shared-memory slots filled by bulk copies (cp.async.bulk, plain,
// never multicast) on per-slot mbarriers, so the down weights arrive while
// gate/up still computes.  Partial row sums meet in shared memory and the
// block finishes its units in K order:
//   gate/up: clamped SwiGLU (dsv4_arena.py:223-235) into h, and h's 32 rows
//            as int8 pieces with one scale per 32-row segment (written to
//            global scratch, then counted);
//   down:    per route y = T(sum), T(T(y) * T(w)), summed in route order in
//            fp32, then the shared expert's row and the residual
//            (combine_finish, arena.py:619-624).
// A ninth warp (the finisher) finishes each gate/up unit as soon as its
// items are done and adds one to the count of the unit's h chunk (route,
// down K chunk); a down item waits (bounded) only for the count of the chunk
// it reads, so the first chunks are ready while later units still compute,
// and the next item's chunk is loaded while the current one computes.  The
// kernel needs all its blocks resident (one per SM; the grid is the SM
// count).  Routing: a single token's top-k runs block-wide
// (block_topk) from the router's scores, or the chunk table is read; x's
// int8 pieces come from the router (or are converted here).  The sums run in
// a fixed order, so results repeat bit for bit.
//
// Every wait is bounded (mbar_wait, the unit and h counts); on a timeout the
// kernel flags LMOE_ECUDA, drains the copies it issued (bounded) and stops.
#include <cstdlib>
#include <cstring>

#include "lmoe_kernels.cuh"

namespace lmoe {

namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ void imma_u8s8(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ T lds(const uint8_t *p) {
    return *reinterpret_cast<const T *>(p);
}

// Tile geometry of the stream format for (BITS, GS) (StreamGeo / TileGeo with
// CK = 8 * GS columns per chunk): code bytes per row, scale and bias offsets,
// padded tile bytes, code swizzle mask.
template <int BITS, int GS>
struct VecTile {
    static constexpr int RB = GS * BITS;
    static constexpr int tS = 16 * RB;
    static constexpr int tB = tS + 256;
    static constexpr int TB = (tB + 256 + 127) / 128 * 128;
    static constexpr int FMC = (RB < 128 ? RB : 128) / 16 - 1;
};

// The first MMA of a chain: accumulator from zero.
__device__ __forceinline__ void imma_u8s8_z(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// One item of a phase: the stage's NM tiles (16 rows each) times this
// lane's two groups (2t, 2t + 1) of K chunk cc, accumulated into racc
// (rows g and g + 8 of each tile).  Each group's activations come in NSEG
// segments with their own (sum, factor) (xsr[group * NSEG + seg]).
template <typename TA, int BITS, int GS, int NM, int NSEG>
__device__ __forceinline__ void vec_item(const uint8_t *sb, const uint8_t *xrow, const float2 *xsr,
                                         const uint8_t *zero, int cc, float (&racc)[NM][2]) {
    using VT = VecTile<BITS, GS>;
    constexpr int NC = 8 / BITS;         // code classes per byte
    constexpr int WPG = GS * BITS / 32;  // code words per row of one group
    constexpr int NWP = WPG / 2;         // word pairs (one MMA k-range each)
    constexpr int NJ = NWP * NC;         // MMAs per (tile, group) = GS / 8
    constexpr int NWPS = NWP / NSEG;     // word pairs per segment
    constexpr uint32_t kMask = BITS == 8 ? 0xffffffffu : (BITS == 4 ? 0x0f0f0f0fu : 0x03030303u);
    static_assert(WPG >= 2 && WPG % 2 == 0, "a group row must be whole word pairs");
    static_assert(NWPS >= 1 && NWPS * NSEG == NWP, "segments must be whole word pairs");
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int cfx = g & VT::FMC;       // rows g and g + 8 share the code swizzle
    const bool prov = (g >> 1) == t;   // this lane feeds B column g (group slot g / 2, piece g & 1)
    const uint8_t *rg = sb + g * VT::RB;
    // scales and biases of rows g, g + 8 for this lane's groups 2t, 2t + 1
    uint32_t sw[NM][2], bw[NM][2];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint8_t *tb = sb + m * VT::TB + (g + 8 * h) * 16 + 4 * t;
            sw[m][h] = lds<uint32_t>(tb + VT::tS);
            bw[m][h] = lds<uint32_t>(tb + VT::tB);
        }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const int gi = 2 * t + hf;  // this lane's group in the chunk (A rows and D columns)
        uint2 bf[NJ];
        {
            const uint8_t *bp = prov ? xrow + (size_t)(cc * 8 + 2 * (g >> 1) + hf) * (2 * GS) + (g & 1) * 8 : zero;
#pragma unroll
            for (int jj = 0; jj < NJ; ++jj) bf[jj] = lds<uint2>(bp + (prov ? jj * 16 : 0));
        }
        float X = 0.0f, P[NM][2];
        uint4 qa[NM], qb[NM];  // 16 bytes of rows g and g + 8: word pairs wp, wp + 1
#pragma unroll
        for (int sg = 0; sg < NSEG; ++sg) {
            const float2 xg = xsr[(cc * 8 + gi) * NSEG + sg];
            X += xg.x;
            int32_t D[NM][NC][4];
#pragma unroll
            for (int wl = 0; wl < NWPS; ++wl) {
                const int wp = sg * NWPS + wl;
                const int byte = gi * WPG * 4 + wp * 8;  // word pair's offset in the row
                const int off = (((byte >> 4) ^ cfx) << 4) + (byte & 15);
                uint2 wa[NM], wb[NM];
                if constexpr (WPG >= 4) {  // a group row is whole 16-byte chunks: one load per two word pairs
                    if ((wp & 1) == 0) {
#pragma unroll
                        for (int m = 0; m < NM; ++m) {
                            qa[m] = lds<uint4>(rg + m * VT::TB + off);
                            qb[m] = lds<uint4>(rg + m * VT::TB + 8 * VT::RB + off);
                        }
                    }
#pragma unroll
                    for (int m = 0; m < NM; ++m) {
                        wa[m] = (wp & 1) ? make_uint2(qa[m].z, qa[m].w) : make_uint2(qa[m].x, qa[m].y);
                        wb[m] = (wp & 1) ? make_uint2(qb[m].z, qb[m].w) : make_uint2(qb[m].x, qb[m].y);
                    }
                } else {
#pragma unroll
                    for (int m = 0; m < NM; ++m) {
                        wa[m] = lds<uint2>(rg + m * VT::TB + off);
                        wb[m] = lds<uint2>(rg + m * VT::TB + 8 * VT::RB + off);
                    }
                }
#pragma unroll
                for (int p2 = 0; p2 < NC; ++p2) {
                    const uint32_t mk = kMask << (BITS * p2);
#pragma unroll
                    for (int m = 0; m < NM; ++m) {
                        if (wl == 0)
                            imma_u8s8_z(D[m][p2], wa[m].x & mk, wb[m].x & mk, wa[m].y & mk, wb[m].y & mk,
                                        bf[wp * NC + p2].x, bf[wp * NC + p2].y);
                        else
                            imma_u8s8(D[m][p2], wa[m].x & mk, wb[m].x & mk, wa[m].y & mk, wb[m].y & mk,
                                      bf[wp * NC + p2].x, bf[wp * NC + p2].y);
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < NM; ++m) {
                // classes folded: C = sum_p D_p 2^(BITS (NC - 1 - p)); pieces: V = 256 C_hi + C_lo
                int32_t C[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    int32_t v = D[m][0][e];
#pragma unroll
                    for (int p2 = 1; p2 < NC; ++p2) v = v * (1 << BITS) + D[m][p2][e];
                    C[e] = v;
                }
                const float v0 = static_cast<float>(C[0] * 256 + C[1]) * xg.y;
                const float v1 = static_cast<float>(C[2] * 256 + C[3]) * xg.y;
                P[m][0] = sg == 0 ? v0 : P[m][0] + v0;
                P[m][1] = sg == 0 ? v1 : P[m][1] + v1;
            }
        }
#pragma unroll
        for (int m = 0; m < NM; ++m) {
            const float s0 = Act<TA>::to_f(static_cast<uint16_t>(hf ? sw[m][0] >> 16 : sw[m][0] & 0xffffu));
            const float s1 = Act<TA>::to_f(static_cast<uint16_t>(hf ? sw[m][1] >> 16 : sw[m][1] & 0xffffu));
            const float b0 = Act<TA>::to_f(static_cast<uint16_t>(hf ? bw[m][0] >> 16 : bw[m][0] & 0xffffu));
            const float b1 = Act<TA>::to_f(static_cast<uint16_t>(hf ? bw[m][1] >> 16 : bw[m][1] & 0xffffu));
            racc[m][0] = fmaf(s0, P[m][0], fmaf(b0, X, racc[m][0]));
            racc[m][1] = fmaf(s1, P[m][1], fmaf(b1, X, racc[m][1]));
        }
    }
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Single-token top-k of the block from the router's (score, biased score)
// (arena.py:501-506), with the winners, selection order and weights of the
// router's own finisher (fused_topk).  Experts are ordered by (key desc, id
// asc), a strict order.  Thread tid holds experts tid, tid + NT, ... (NT threads, E <= 512).
//  1. Each warp ranks its own experts among themselves with shuffles.  An
//     expert that k others of its warp beat cannot win, so only local ranks
//     below k go on, into shared memory at [warp][local rank].
//  2. One thread per candidate counts the candidates that beat it; a count
//     below k is its place in the selection order.  Every expert that beats a
//     winner is itself a winner, hence a candidate, so the count is exact for
//     the winners and at least k for the rest.
//  3. Thread j < k takes the j-th winner: weight = score / (fp32 sum of the
//     winners' scores in selection order + 1e-20) * scaling; its chunk in the
//     dispatch is the rank of its id among the winners' ids.  Block 0 writes
//     the routing and the dispatch.
// Lane ch < k of every warp returns chunk ch's (arena slot, route, weight).
struct TkCand {
    uint32_t key;
    int32_t id, slot;
    float score;
};
struct TkChunk {
    int32_t slot, route;
    float w;
    int32_t pad;
};
constexpr int kTkBytes = (kVecBlockWarps * 16 + 16) * 16 + 16 * 16;  // candidates, winners, chunks

template <class A>
__device__ __forceinline__ void block_topk(const A &a, uint8_t *tks, int &cslot, int &croute, float &cw) {
    constexpr int NT = kVecBlockWarps * 32, PER = (512 + NT - 1) / NT;  // experts per thread (E <= 512)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = a.tk_E, k = a.tk_k;
    TkCand *cand = reinterpret_cast<TkCand *>(tks);        // [warps][k]
    TkCand *win = cand + kVecBlockWarps * 16;                   // [k], selection order
    TkChunk *chk = reinterpret_cast<TkChunk *>(win + 16);  // [k], dispatch order
    uint32_t mk[PER];
    float ms[PER];
    int msl[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = tid + NT * i;
        mk[i] = 0u;
        ms[i] = 0.0f;
        msl[i] = e;
        if (e < E) {
            const float2 v = __ldcg(a.tk_scores + e);
            ms[i] = v.x;
            mk[i] = topk_key(v.y);
            if (a.tk_expert_slot) msl[i] = __ldg(a.tk_expert_slot + e);
        }
    }
    // 1. ranks within the warp: set i2 of the warp holds experts warp * 32 + src + NT * i2
    int lr[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) lr[i] = 0;
#pragma unroll
    for (int i2 = 0; i2 < PER; ++i2) {
        if (NT * i2 >= E) break;
#pragma unroll 8
        for (int src = 0; src < 32; ++src) {
            const uint32_t ok = __shfl_sync(kFull, mk[i2], src);
            const int oi = src + NT * i2;
#pragma unroll
            for (int i = 0; i < PER; ++i)
                if (NT * i < E) lr[i] += (ok > mk[i]) || (ok == mk[i] && oi < lane + NT * i);
        }
    }
    if (lane < k) cand[warp * k + lane] = TkCand{0u, 0x7fffffff, 0, 0.0f};
    if (tid < k) {
        win[tid] = TkCand{0u, 0x7fffffff, 0, 0.0f};
        chk[tid] = TkChunk{0, tid, 0.0f, 0};
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < PER; ++i)
        if (mk[i] != 0u && lr[i] < k) cand[warp * k + lr[i]] = TkCand{mk[i], tid + NT * i, msl[i], ms[i]};
    __syncthreads();
    // 2. ranks among the candidates
    const int nc = static_cast<int>(blockDim.x >> 5) * k;
    if (tid < nc) {
        const TkCand me = cand[tid];
        if (me.key != 0u) {
            int rank = 0;
#pragma unroll 4
            for (int o = 0; o < nc; ++o) {
                const TkCand q = cand[o];
                rank += (q.key > me.key) || (q.key == me.key && q.id < me.id);
            }
            if (rank < k) win[rank] = me;
        }
    }
    __syncthreads();
    // 3. weights and the dispatch
    if (tid < k) {
        const TkCand me = win[tid];
        float ssum = 0.0f;  // fp32, in selection order
        int pos = 0;        // rank of this winner's id among the winners' ids
        for (int j = 0; j < k; ++j) {
            const TkCand q = win[j];
            ssum += q.score;
            pos += q.id < me.id;
        }
        float wv = a.tk_norm ? me.score / (ssum + 1e-20f) : me.score;
        wv *= a.tk_scaling;
        int slot = 0;
        if (me.id < 0 || me.id >= E) {
            set_error(a.err, -3);
        } else {
            slot = me.slot;
            if (slot < 0 || slot >= a.n_slots) {
                set_error(a.err, -3);
                slot = 0;
            }
        }
        chk[pos] = TkChunk{slot, tid, wv, 0};
        if (blockIdx.x == 0) {
            a.tk_idx[tid] = me.id;
            a.tk_w[tid] = wv;
            if (a.tk_idx_user) a.tk_idx_user[tid] = me.id;
            if (a.tk_w_user) a.tk_w_user[tid] = wv;
            a.tk_sorted[pos] = tid;
            Chunk ch;
            ch.slot = slot;
            ch.route_start = pos;
            ch.ntok = 1;
            ch.expert = me.id;
            a.tk_chunks[pos] = ch;
            if (tid == 0) *a.tk_nchunks = k;
        }
    }
    __syncthreads();
    if (lane < k) {
        const TkChunk q = chk[lane];
        cslot = q.slot;
        croute = q.route;
        cw = q.w;
    }
}

template <typename TA, int BG, int BD, int GS>
__global__ void __launch_bounds__(kVecBlockWarps * 32, 1) vec_layer_kernel(const VecArgs a, const VecCfg c) {
    constexpr int NSEG_D = GS / 32;  // h segments (32 rows, one gate/up unit each) per down group
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    // warps 0 .. W - 1 stream and compute items; warp W (the finisher)
    // finishes the block's gate/up units as their items complete
    constexpr int W = kVecWarps;
    const int b = static_cast<int>(blockIdx.x), G = static_cast<int>(gridDim.x);
    const bool finisher = warp == W;
    const int nq = c.nq, R = a.routes;
    extern __shared__ __align__(1024) uint8_t smem[];
    volatile int &s_abort = *reinterpret_cast<volatile int *>(smem + c.off_flag);
    uint8_t *ring = smem + c.off_ring + (size_t)warp * c.nq * c.sub;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + c.off_bar) + warp * kVecMaxStages;
    uint64_t *xbar = reinterpret_cast<uint64_t *>(smem + c.off_xbar);  // x pieces
    uint8_t *xq = smem + c.off_xq;                               // x pieces [groups][2 GS]
    float2 *xs = reinterpret_cast<float2 *>(smem + c.off_xs);  // [groups]
    uint8_t *hq = smem + c.off_hq;  // per-warp scratch: one K chunk of h's pieces and factors
    const uint8_t *zero = smem + c.off_zero;                     // 2 GS zero bytes (B of idle lanes)
    float *pa = reinterpret_cast<float *>(smem + c.off_pa);      // [unit j][K chunk][64]
    float *pb = reinterpret_cast<float *>(smem + c.off_pb);      // [pair j][chunk][K chunk][32]
    int *route_ch = reinterpret_cast<int *>(smem + c.off_rch);   // [R]: chunk of each route (-1: none)
    int *ucnt = route_ch + 32;                                   // [unit j]: its items done
    const VecPhase &PA = c.ga, &PB = c.dn;
    const int inter = a.q0.rows, hidden = a.q2.rows;
    const int nseg = inter / 32;  // h segments per route

    if (lane == 0 && !finisher) {
        for (int q = 0; q < nq; ++q) mbar_init(&bar[q], 1);
        if (warp == 0) mbar_init(&xbar[0], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < GS / 8; i += blockDim.x)
        reinterpret_cast<uint4 *>(smem + c.off_zero)[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = threadIdx.x; i < 32; i += blockDim.x) {
        route_ch[i] = -1;
        ucnt[i] = 0;
    }
    if (threadIdx.x == 0) s_abort = 0;
    __syncthreads();

    // ---- this block's units and this warp's items, for nch chunks.  With
    // the top-k fused here the chunk count is k before the routing exists,
    // so the plan is made while the preceding kernel still runs.
    int nch = 0, nuA = 0, npB = 0, perB = 0, myA = 0, myB = 0, total = 0;
    int uch = 0, upr = 0;  // lane j: the block's gate/up unit b + j * G as (chunk, pair)
    auto plan = [&](int n) {
        nch = n;
        const int nunits = nch * PA.pairs;
        nuA = b < nunits ? (nunits - b + G - 1) / G : 0;  // gate/up units b, b + G, ...
        npB = b < PB.pairs ? (PB.pairs - b + G - 1) / G : 0;  // down pairs b, b + G, ...
        perB = nch * PB.nck;
        const int nitA = nuA * PA.nck, nitB = npB * perB;
        myA = !finisher && nitA > warp ? (nitA - warp + W - 1) / W : 0;
        myB = !finisher && nitB > warp ? (nitB - warp + W - 1) / W : 0;
        total = myA + myB;
        if (lane < nuA) {
            const int u = b + lane * G;
            uch = u / PA.pairs;
            upr = u - uch * PA.pairs;
        }
    };
    if (a.tk_scores) plan(a.tk_k);

    // The routing and x's pieces come from the preceding kernel.  Dependent
    // launches are released only after the grid-wide wait below: until then
    // every block of this grid must be able to become resident.
    pdl_wait();
    const uint32_t xq_bytes = static_cast<uint32_t>(PA.ngroups * 2 * GS);
    const uint32_t xs_bytes = static_cast<uint32_t>((PA.ngroups * 8 + 15) & ~15);  // padded on both sides
    if (a.x_ready && threadIdx.x == 0) {
        mbar_expect_tx(&xbar[0], xq_bytes + xs_bytes);
        bulk_g2s(xq, a.xq, xq_bytes, &xbar[0]);
        bulk_g2s(xs, a.xs, xs_bytes, &xbar[0]);
    }
    int cslot = 0, croute = 0;  // lane ch holds chunk ch's (slot, route, weight)
    float cw = 1.0f;
    if (a.tk_scores) {
        block_topk(a, smem + c.off_tk, cslot, croute, cw);
    } else {
        int n = __ldcg(a.n_chunks);
        if (n < 0 || n > a.max_chunks || n > 32 || n > R) {
            set_error(a.err, -3);
            n = n < 0 ? 0 : min(min(a.max_chunks, 32), R);
        }
        plan(n);
        if (lane < nch) {
            const int4 ck = __ldcg(reinterpret_cast<const int4 *>(a.chunks) + lane);  // {slot, start, ntok, expert}
            cslot = ck.x;
            if (cslot < 0 || cslot >= a.n_slots || ck.z != 1 || ck.y < 0 || ck.y >= R) {
                set_error(a.err, -3);
                cslot = 0;
            }
            croute = (ck.y >= 0 && ck.y < R) ? __ldcg(a.sorted_routes + ck.y) : 0;
            if (croute < 0 || croute >= R) {
                set_error(a.err, -3);
                croute = 0;
            }
            if (a.route_w) cw = __ldcg(a.route_w + croute);
        }
    }
    if (warp == 0 && lane < nch) route_ch[croute] = lane;
    // the residual rows of this warp's first combine pair, loaded early
    const uint16_t rv_pre = (a.residual && a.out && warp < npB) ? a.residual[32 * (b + warp * G) + lane] : 0;

    const uint64_t pol = evict_first_policy();
    // Item cursor over this warp's items -- gate/up items warp, warp + W, ...
    // of the block's list (unit j = i / nck, K chunk cc), then its down items
    // (pair j = i / perB, chunk ch, K chunk cc) -- advanced without division.
    struct Cur {
        int n, j, ch, cc;
    };
    auto cur_start = [&](Cur &q) {
        q.n = 0;
        if (myA > 0) {
            q.j = warp / PA.nck;
            q.cc = warp - q.j * PA.nck;
            q.ch = 0;
        } else {
            q.j = warp / perB;
            const int r2 = warp - q.j * perB;
            q.ch = r2 / PB.nck;
            q.cc = r2 - q.ch * PB.nck;
        }
    };
    auto cur_next = [&](Cur &q) {
        ++q.n;
        if (q.n < myA) {
            q.cc += W;
            while (q.cc >= PA.nck) {
                q.cc -= PA.nck;
                ++q.j;
            }
        } else if (q.n == myA) {  // first down item
            q.j = warp / perB;
            const int r2 = warp - q.j * perB;
            q.ch = r2 / PB.nck;
            q.cc = r2 - q.ch * PB.nck;
        } else {
            q.cc += W;
            while (q.cc >= PB.nck) {
                q.cc -= PB.nck;
                if (++q.ch == nch) {
                    q.ch = 0;
                    ++q.j;
                }
            }
        }
    };
    // the item at cursor q into ring sub-slots from pos: c.qa sub-slots for a
    // gate/up item, c.qb for a down item
    auto issue = [&](int pos, const Cur &q, bool reuse) {
        const bool down = q.n >= myA;
        const int ch = down ? q.ch : __shfl_sync(kFull, uch, q.j);
        const int p = down ? b + q.j * G : __shfl_sync(kFull, upr, q.j);
        const int slot = __shfl_sync(kFull, cslot, ch);
        if (lane == 0) {
            uint8_t *dst = ring + (size_t)pos * c.sub;
            if (reuse) fence_proxy_async();  // the ring's earlier contents were read by generic loads
            if (!down) {
                mbar_expect_tx(&bar[pos], static_cast<uint32_t>(2 * PA.blk));
                const size_t off = ((size_t)p * PA.nck + q.cc) * (size_t)PA.blk;
                bulk_g2s_hint(dst, a.q0.tiles + (size_t)slot * a.q0.tile_slot_stride + off,
                              static_cast<uint32_t>(PA.blk), &bar[pos], pol);
                bulk_g2s_hint(dst + PA.blk, a.q1.tiles + (size_t)slot * a.q1.tile_slot_stride + off,
                              static_cast<uint32_t>(PA.blk), &bar[pos], pol);
            } else {
                mbar_expect_tx(&bar[pos], static_cast<uint32_t>(PB.blk));
                const size_t off = ((size_t)p * PB.nck + q.cc) * (size_t)PB.blk;
                bulk_g2s_hint(dst, a.q2.tiles + (size_t)slot * a.q2.tile_slot_stride + off,
                              static_cast<uint32_t>(PB.blk), &bar[pos], pol);
            }
        }
    };
    // ring state: issue / consume positions, sub-slots in use, phase bits
    int issued = 0, consumed = 0, ip = 0, cp = 0, used = 0;
    uint32_t par = 0;
    auto qof = [&](int n) { return n < myA ? c.qa : c.qb; };
    Cur ci;  // issue cursor
    cur_start(ci);
    auto try_issue = [&]() {
        while (issued < total && used + qof(issued) <= nq) {
            const int q = qof(issued);
            issue(ip, ci, consumed > 0);
            cur_next(ci);
            ip += q;
            if (ip == nq) ip = 0;
            used += q;
            ++issued;
        }
    };
    try_issue();

    bool aborted = false;
    // the next item's data (bounded wait); false: gave up
    auto wait_next = [&]() { return mbar_wait(&bar[cp], (par >> cp) & 1u); };
    auto advance = [&]() {
        const int q = qof(consumed);
        par ^= 1u << cp;
        cp += q;
        if (cp == nq) cp = 0;
        used -= q;
        ++consumed;
        __syncwarp();  // every lane is done with the sub-slots
        try_issue();
    };
    // drain the copies this warp still has in flight (bounded) before exiting
    auto drain = [&]() {
        while (consumed < issued) {
            wait_next();
            const int q = qof(consumed);
            par ^= 1u << cp;
            cp += q;
            if (cp == nq) cp = 0;
            ++consumed;
        }
    };
    // ---- x's pieces: from the router (bulk copy above) or converted here
    if (a.x_ready) {
        if (!mbar_wait(&xbar[0], 0)) {
            set_error(a.err, -4);
            aborted = true;
        }
    } else if (!finisher) {
        for (int gi = warp; gi < PA.ngroups; gi += W)
            convert_group<TA, BG, GS>(a.x + (size_t)gi * GS, xq + (size_t)gi * (2 * GS), xs + gi, true);
    }
    __syncthreads();  // x pieces and the route map are complete

    // ============================== gate/up items
    // A unit of this block, once all its items are done (finisher warp): K
    // chunks in order, SwiGLU, and h's int8 pieces (one scale per 32-row
    // segment) into global scratch, then a release increment of the count of
    // finished units of its h chunk.
    const int ml = lane >> 4, rl = lane & 15;  // lane = row of the 32-row pair
    auto finish_unit = [&](int j) {
        const int ch = __shfl_sync(kFull, uch, j), p = __shfl_sync(kFull, upr, j);
        const int route = __shfl_sync(kFull, croute, ch);
        const float *pp = pa + (size_t)j * PA.nck * 64 + ml * 16 + rl;
        float ga = 0.0f, ua = 0.0f;
        for (int cc = 0; cc < PA.nck; ++cc) {
            ga += pp[cc * 64];
            ua += pp[cc * 64 + 32];
        }
        const float hv = swiglu_h<TA>(ga, ua, a.limit, a.swiglu_mode);
        float amax = fabsf(hv), sum = hv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
            sum += __shfl_xor_sync(kFull, sum, o);
        }
        int S = 0;
        if (amax > 0.0f) S = min(13 - (static_cast<int>((__float_as_uint(amax) >> 23) & 0xffu) - 127), 126);
        const int xi = __float2int_rn(hv * __uint_as_float(static_cast<uint32_t>(S + 127) << 23));
        const int hi = (xi + 128) >> 8, lo = xi - (hi << 8);
        const int ngd = PB.ngroups, gd = (32 * p) / GS, e = (32 * p) % GS + lane;
        uint8_t *gq = a.hq + ((size_t)route * ngd + gd) * (2 * GS);
        gq[piece_offset<BD>(e, 0)] = static_cast<uint8_t>(hi & 0xff);
        gq[piece_offset<BD>(e, 1)] = static_cast<uint8_t>(lo & 0xff);
        if (lane == 0) a.hs[(size_t)route * nseg + p] = make_float2(sum, exp2i(-(S + 8 - BD)));
        __syncwarp();
        // cumulative release: the warp's stores above precede the count of
        // finished units of h's K chunk (route, 32 p / CK) of the down GEMV
        if (lane == 0)
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.hready + (size_t)route * PB.nck +
                                                                         (32 * p) / (8 * GS))
                         : "memory");
    };
    Cur cu;  // consume cursor
    cur_start(cu);
    for (int n = 0; n < myA && !aborted; ++n, cur_next(cu)) {
        const int j = cu.j, cc = cu.cc;
        if (!wait_next()) {
            set_error(a.err, -4);
            aborted = true;
            break;
        }
        float racc[4][2];
#pragma unroll
        for (int m = 0; m < 4; ++m) racc[m][0] = racc[m][1] = 0.0f;
        vec_item<TA, BG, GS, 4, 1>(ring + (size_t)cp * c.sub, xq, xs, zero, cc, racc);
        advance();
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                racc[m][h] += __shfl_xor_sync(kFull, racc[m][h], 1);
                racc[m][h] += __shfl_xor_sync(kFull, racc[m][h], 2);
            }
        if (t == 0) {
            float *pp = pa + ((size_t)j * PA.nck + cc) * 64;
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                pp[m * 16 + g] = racc[m][0];
                pp[m * 16 + g + 8] = racc[m][1];
            }
        }
        __syncwarp();
        if (lane == 0) {  // the partial sums above precede the count
            __threadfence_block();
            atomicAdd(&ucnt[j], 1);
        }
    }
    if (aborted) s_abort = 1;
    if (finisher) {
        // units in the order the warps complete them (every warp takes its
        // items unit by unit); each wait is bounded and ends when a compute
        // warp gives up
        for (int j = 0; j < nuA; ++j) {
            bool ok = true;
            if (*reinterpret_cast<volatile int *>(ucnt + j) < PA.nck) {
                const long long t0 = clock64();
                while (*reinterpret_cast<volatile int *>(ucnt + j) < PA.nck) {
                    if (s_abort || clock64() - t0 > kWaitLimitCycles) {
                        ok = false;
                        break;
                    }
                    __nanosleep(20);
                }
            }
            if (!__all_sync(kFull, ok)) {
                if (!s_abort) set_error(a.err, -4);
                s_abort = 1;
                break;
            }
            __threadfence_block();
            finish_unit(j);
        }
    }
    // Every block has passed its launch wait (the routing above follows it):
    // dependents may launch without taking an SM this grid still needs.
    pdl_trigger();

    // ============================== down items
    // Item (pair, chunk ch, K chunk cc) needs h's K chunk cc of its route:
    // the CK / 32 gate/up units of that chunk (count hready[route][cc]).  The
    // warp waits for them (bounded), loads the chunk's int8 pieces and (sum,
    // factor) pairs into registers, and stores them into its own scratch.
    // The next item's chunk is loaded while this item computes when its
    // units are already done.
    const int upc = PB.nck > 0 ? PA.pairs / PB.nck : 1;  // gate/up units per down K chunk
    uint8_t *wq = hq + (size_t)warp * (8 * 2 * GS + 8 * NSEG_D * 8);  // [8 groups][2 GS]
    float2 *wxs = reinterpret_cast<float2 *>(wq + 8 * 2 * GS);         // [8 groups][NSEG_D]
    constexpr int NQ = 8 * 2 * GS / 16, NS = 8 * NSEG_D / 2;  // 16-byte pieces and factor pairs of a chunk
    constexpr int VQ = (NQ + 31) / 32, VS = (NS + 31) / 32;
    uint4 hv[VQ];
    float4 hf[VS];
    auto h_ctr = [&](const Cur &q) {
        return a.hready + (size_t)__shfl_sync(kFull, croute, q.ch) * PB.nck + q.cc;
    };
    auto h_load = [&](const Cur &q) {
        const int route = __shfl_sync(kFull, croute, q.ch);
        const uint4 *sq = reinterpret_cast<const uint4 *>(a.hq + ((size_t)route * PB.ngroups + q.cc * 8) * (2 * GS));
        const float4 *ss = reinterpret_cast<const float4 *>(a.hs + (size_t)route * nseg + q.cc * 8 * NSEG_D);
#pragma unroll
        for (int i = 0; i < VQ; ++i)
            if (lane + 32 * i < NQ) hv[i] = __ldcg(sq + lane + 32 * i);
#pragma unroll
        for (int i = 0; i < VS; ++i)
            if (lane + 32 * i < NS) hf[i] = __ldcg(ss + lane + 32 * i);
    };
    bool have = false;  // hv / hf hold the chunk of the item at cu
    for (int n = 0; n < myB && !aborted; ++n, cur_next(cu)) {
        const int j = cu.j, ch = cu.ch, cc = cu.cc;
        if (!have) {
            const uint32_t *ctr = h_ctr(cu);
            bool ok = true;
            if (ld_acquire_u32(ctr) < static_cast<uint32_t>(upc)) {
                const long long t0 = clock64();
                uint32_t sl = 32;
                while (ld_acquire_u32(ctr) < static_cast<uint32_t>(upc)) {
                    __nanosleep(sl);
                    if (sl < 256) sl <<= 1;
                    if (s_abort || clock64() - t0 > kWaitLimitCycles) {
                        ok = false;
                        break;
                    }
                }
            }
            if (!__all_sync(kFull, ok)) {
                set_error(a.err, -4);
                aborted = true;
                break;
            }
            h_load(cu);
        }
#pragma unroll
        for (int i = 0; i < VQ; ++i)
            if (lane + 32 * i < NQ) reinterpret_cast<uint4 *>(wq)[lane + 32 * i] = hv[i];
#pragma unroll
        for (int i = 0; i < VS; ++i)
            if (lane + 32 * i < NS) reinterpret_cast<float4 *>(wxs)[lane + 32 * i] = hf[i];
        __syncwarp();
        have = false;
        if (n + 1 < myB) {  // every lane acquires the count itself before loading
            Cur cn = cu;
            cur_next(cn);
            if (__all_sync(kFull, ld_acquire_u32(h_ctr(cn)) >= static_cast<uint32_t>(upc))) {
                h_load(cn);
                have = true;
            }
        }
        if (!wait_next()) {
            set_error(a.err, -4);
            aborted = true;
            break;
        }
        float dacc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        vec_item<TA, BD, GS, 2, NSEG_D>(ring + (size_t)cp * c.sub, wq, wxs, zero, 0, dacc);
        advance();
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                dacc[m][h] += __shfl_xor_sync(kFull, dacc[m][h], 1);
                dacc[m][h] += __shfl_xor_sync(kFull, dacc[m][h], 2);
            }
        if (t == 0) {
            float *pp = pb + (((size_t)j * R + ch) * PB.nck + cc) * 32;
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                pp[m * 16 + g] = dacc[m][0];
                pp[m * 16 + g + 8] = dacc[m][1];
            }
        }
    }
    if (aborted) {
        s_abort = 1;
        drain();
    }
    __syncthreads();
    if (s_abort) return;

    // ---- down pairs of this block: per (pair, chunk) y in K order and the
    // route's row T(T(y) * T(w)), spread over the warps; then per pair the
    // combine in route order, the shared expert's row and the residual
    // (combine_finish).  A pair's row of chunk ch replaces its K chunk 0
    // partial in shared memory.
    for (int q = warp; q < npB * nch; q += kVecBlockWarps) {
        const int j = q / nch, ch = q - j * nch;
        const int row = 32 * (b + j * G) + lane;
        float *pp = pb + ((size_t)j * R + ch) * PB.nck * 32 + ml * 16 + rl;
        float y = 0.0f;
        for (int cc = 0; cc < PB.nck; ++cc) y += pp[cc * 32];
        const float v = Act<TA>::round(Act<TA>::round(y) * Act<TA>::round(__shfl_sync(kFull, cw, ch)));
        if (a.yw) a.yw[(size_t)__shfl_sync(kFull, croute, ch) * hidden + row] = Act<TA>::from_f(v);
        pp[0] = v;
    }
    __syncthreads();
    if (a.out)
        for (int j = warp; j < npB; j += kVecBlockWarps) {
            const int row = 32 * (b + j * G) + lane;
            const float *yv = pb + (size_t)j * R * PB.nck * 32 + lane;  // + ch * nck * 32: chunk ch's row
            float sacc = 0.0f;
            for (int r = 0; r < a.top_k && r < R; ++r) {
                const int ch = route_ch[r];
                if (ch >= 0) sacc += yv[(size_t)ch * PB.nck * 32];
            }
            const bool sh = a.shared_base > 0 && a.shared_base < R && route_ch[a.shared_base] >= 0;
            const uint16_t sv = sh ? Act<TA>::from_f(yv[(size_t)route_ch[a.shared_base] * PB.nck * 32]) : 0;
            const uint16_t rv = !a.residual ? 0 : (j == warp ? rv_pre : a.residual[row]);
            a.out[row] = Act<TA>::from_f(combine_finish<TA>(sacc, sh, sv, a.residual != nullptr, rv));
        }
}

int g_vec_sms = 0;
int vec_sm_count() {
    if (g_vec_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_vec_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_vec_sms <= 0) g_vec_sms = 148;
    }
    return g_vec_sms;
}

constexpr int kVecSmem = 227 * 1024;
inline int al128(int v) { return (v + 127) & ~127; }

bool vec_phase(int rows, int K, int bits, int gs, VecPhase *out) {
    if (bits != 2 && bits != 4 && bits != 8) return false;
    if (gs != 32 && gs != 64 && gs != 128) return false;
    StreamGeo sg;
    if (!stream_geo(rows, K, bits, gs, &sg) || sg.tg.SB != 16) return false;
    VecPhase p;
    p.nck = sg.nck;
    p.pairs = sg.pairs;
    p.RB = sg.tg.RB;
    p.fm_c = sg.tg.fm_c;
    p.tS = sg.tg.tS;
    p.tB = sg.tg.tB;
    p.TB = sg.tg.TB;
    p.ngroups = K / gs;
    p.blk = sg.block;
    *out = p;
    return true;
}

template <typename TA, int BG, int BD, int GS>
cudaError_t launch_vec_t(const VecArgs &a, const VecCfg &c, cudaStream_t st) {
    auto kern = vec_layer_kernel<TA, BG, BD, GS>;
    static int configured = 0;
    if (c.smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, c.smem);
        if (e != cudaSuccess) return e;
        configured = c.smem;
    }
    return launch_pdl(kern, dim3(static_cast<unsigned>(c.grid)), dim3(kVecBlockWarps * 32), c.smem, st, a, c);
}

// (gate/up bits, down bits) pairs compiled, for group sizes 32, 64, 128
bool vec_bits_ok(int bg, int bd) { return (bg == 2 && (bd == 2 || bd == 4)) || (bg == 4 && bd == 4) || (bg == 8 && bd == 8); }

template <typename TA>
cudaError_t launch_vec_dt(int bg, int bd, int gs, const VecArgs &a, const VecCfg &c, cudaStream_t st) {
#define LMOE_VCASE(B1, B2, Gs) \
    if (bg == B1 && bd == B2 && gs == Gs) return launch_vec_t<TA, B1, B2, Gs>(a, c, st);
#define LMOE_VGS(B1, B2) LMOE_VCASE(B1, B2, 32) LMOE_VCASE(B1, B2, 64) LMOE_VCASE(B1, B2, 128)
    LMOE_VGS(2, 2)
    LMOE_VGS(2, 4)
    LMOE_VGS(4, 4)
    LMOE_VGS(8, 8)
#undef LMOE_VGS
#undef LMOE_VCASE
    return cudaErrorInvalidValue;
}

}  // namespace

bool vec_layer_config(int hidden, int inter, int bits_g, int gs_g, int bits_d, int gs_d, int routes, VecCfg *out) {
    if (gs_g != gs_d || !vec_bits_ok(bits_g, bits_d)) return false;
    if (routes < 1 || routes > 32) return false;
    VecCfg c;
    std::memset(&c, 0, sizeof(c));
    if (!vec_phase(inter, hidden, bits_g, gs_g, &c.ga) || !vec_phase(hidden, inter, bits_d, gs_d, &c.dn)) return false;
    if (inter % 32 != 0 || c.ga.nck * 8 * gs_g != hidden) return false;
    const int gs = gs_g;
    c.routes = routes;
    c.warps = kVecWarps;
    c.grid = vec_sm_count();
    const int G = c.grid;
    const int u_max = (routes * c.ga.pairs + G - 1) / G, p_max = (c.dn.pairs + G - 1) / G;
    if (u_max > 32) return false;  // a block's gate/up units sit one per lane
    // ring sub-slots: a gate/up item (gate + up block) takes qa of them, a
    // down item qb; both at most 2, so items never straddle the ring's end
    c.sub = al128(static_cast<int>(c.ga.blk < c.dn.blk ? c.ga.blk : c.dn.blk));
    c.qa = static_cast<int>((2 * c.ga.blk + c.sub - 1) / c.sub);
    c.qb = static_cast<int>((c.dn.blk + c.sub - 1) / c.sub);
    if (c.qa > 2 || c.qb > 2) {
        c.sub = al128(static_cast<int>(2 * c.ga.blk > c.dn.blk ? 2 * c.ga.blk : c.dn.blk));
        c.qa = c.qb = 1;
    }
    c.off_bar = 0;
    c.off_flag = kVecWarps * kVecMaxStages * 8;
    c.off_xbar = c.off_flag + 16;
    c.off_zero = al128(c.off_xbar + 16);
    c.off_rch = al128(c.off_zero + 2 * gs);
    c.off_tk = al128(c.off_rch + 64 * 4);  // route -> chunk, unit item counts
    c.off_xs = al128(c.off_tk + kTkBytes);  // top-k candidates, winners and chunks
    c.off_xq = al128(c.off_xs + c.ga.ngroups * 8 + 16);
    // per-warp scratch of one K chunk of h: 8 groups of pieces, 8 * gs / 32 factors
    c.off_hq = al128(c.off_xq + c.ga.ngroups * 2 * gs);
    c.off_pa = al128(c.off_hq + kVecWarps * (8 * 2 * gs + 8 * (gs / 32) * 8));
    c.off_pb = al128(c.off_pa + u_max * c.ga.nck * 64 * 4);
    c.off_ring = al128(c.off_pb + p_max * routes * c.dn.nck * 32 * 4);
    const long room = (long)kVecSmem - c.off_ring;
    int nq = static_cast<int>(room / ((long)kVecWarps * c.sub));
    if (nq > kVecMaxStages) nq = kVecMaxStages;
    if (c.qa == 2 || c.qb == 2) nq &= ~1;
    if (nq < c.qa || nq < c.qb) return false;
    c.nq = nq;
    c.smem = c.off_ring + kVecWarps * nq * c.sub;
    *out = c;
    return true;
}

cudaError_t launch_vec_layer(int act_f16, int bits_g, int bits_d, int gs, const VecArgs &a, const VecCfg &c,
                             cudaStream_t st) {
    if (c.grid < 1 || c.nq < 1 || c.nq > kVecMaxStages || c.warps != kVecWarps) return cudaErrorInvalidValue;
    if (act_f16) return launch_vec_dt<__half>(bits_g, bits_d, gs, a, c, st);
    return launch_vec_dt<__nv_bfloat16>(bits_g, bits_d, gs, a, c, st);
}

}  // namespace lmoe
