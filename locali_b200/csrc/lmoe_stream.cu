// Decode-regime expert GEMVs over the stream format (StreamGeo), sm_100a.
//
// A unit is one chunk (<= 8 routes of one expert) x one pair of 16-row tiles
// over the full K range -- of gate and up together (GATEUP, four matrices:
// gate rows 32p..32p+31 and the same up rows) or of one projection (PAIR:
// down, or a plain gather_qmm).  Units go to groups of kp warps; the warps
// of a group split each unit's K chunks (8 quantisation groups each) into kp
// contiguous parts, and every warp streams its part through its own ring of
// shared-memory stages: each lane cp.async-copies its share of the stage's
// weight blocks and closes them into one cp.async group, so a stage is ready
// when the lanes' groups have landed (no mbarrier, no elected issuing lane).
// With kp > 1 the partial sums meet in a double-buffered shared buffer at a
// named barrier of the group, and one warp of it (rotating) adds them in
// part order and runs the epilogue.  Units are spread over all blocks
// (group g of block b takes units b + G*g, b + G*(g + ng), ...).  The
// activation rows every unit of the launch may read (tokens for gate/up,
// routes for the paired projections) stay resident in shared memory.
//
// Arithmetic per group (dsv4_kernels.py:152-154): acc += scale * sum(x * q)
// + bias * sum(x), fp32; codes become exact small integers with one LOP3 per
// pair (lmoe_common.cuh) and the dot products run on mma.sync m16n8k16 with
// fp32 accumulation.  One token: the MMA's 8 columns are the round's 8
// groups (each lane's B fragment is the token's activations where its group
// equals its column).  Several tokens: the columns are the tokens.
//
// Epilogues: GATEUP rounds gate and up, clamps and applies SwiGLU
// (dsv4_arena.py:223-235) and writes h into the down projection's panel with
// its 16-column sums; PAIR writes T(T(y) * T(w)) per route (w = 1 without
// weights: the plain gather_qmm output), then, when a combined output is
// given, the block sums each token's routes in route order in fp32 over the
// row pairs it owns (its grid divides the pair count), adds the shared
// expert's row and the residual (combine_finish).
//
// The kernel has no spin waits: cp.async groups complete or fault, and the
// named barriers join warps that take the same number of units.
#include <cstdlib>
#include <cstring>

#include "lmoe_kernels.cuh"

namespace lmoe {

#define LMOE_FULL 0xffffffffu

namespace {

template <typename T>
__device__ __forceinline__ T sld(const uint8_t *p) {
    return *reinterpret_cast<const T *>(p);
}

// ------------------------------------------------------------ stream packing
// Row-major slot arrays -> stream blocks: block (tile ti, chunk c) of a slot;
// 16-byte chunks land at their swizzled places, padding zeroed.
__global__ void __launch_bounds__(256) stream_pack_kernel(const QView q, const StreamGeo sg, int32_t slot_begin,
                                                          uint8_t *out) {
    const int tile = blockIdx.x / sg.nck, c = blockIdx.x - tile * sg.nck;
    const int slot = slot_begin + static_cast<int>(blockIdx.y);
    const TileGeo &tg = sg.tg;
    uint8_t *dst = out + (size_t)slot * sg.slot + ((size_t)(tile >> 1) * sg.nck + c) * sg.block +
                   (size_t)(tile & 1) * tg.TB;
    const uint8_t *codes = reinterpret_cast<const uint8_t *>(q.w + (size_t)slot * q.w_slot_stride) +
                           (size_t)tile * 16 * q.words_per_row * 4 + (size_t)c * tg.RB;
    const int cpr = tg.RB / 16;  // 16-byte chunks per row
    for (int i = threadIdx.x; i < 16 * cpr; i += blockDim.x) {
        const int r = i / cpr, j = i - r * cpr;
        *reinterpret_cast<uint4 *>(dst + tile_code_chunk(tg, i)) =
            *reinterpret_cast<const uint4 *>(codes + (size_t)r * q.words_per_row * 4 + j * 16);
    }
    // scales / biases: 8 groups x 2 bytes = 16 bytes per row
    const size_t sb0 = (size_t)slot * q.sb_slot_stride + (size_t)tile * 16 * q.groups_per_row + (size_t)c * 8;
    for (int r = threadIdx.x; r < 16; r += blockDim.x) {
        const int o = tile_sb_chunk(tg, r);
        *reinterpret_cast<uint4 *>(dst + tg.tS + o) =
            *reinterpret_cast<const uint4 *>(q.s + sb0 + (size_t)r * q.groups_per_row);
        *reinterpret_cast<uint4 *>(dst + tg.tB + o) =
            *reinterpret_cast<const uint4 *>(q.b + sb0 + (size_t)r * q.groups_per_row);
    }
    for (int o = tg.tB + 16 * tg.SB + 16 * threadIdx.x; o < tg.TB; o += 16 * blockDim.x)
        *reinterpret_cast<uint4 *>(dst + o) = make_uint4(0u, 0u, 0u, 0u);
}

// Chunk metadata of one unit, held in registers (lane n < ntok: route n)
struct UnitMeta {
    int slot, ntok, p;
    int route, row;
    float w;
};

// Named barrier of one warp group.  The warp reconverges first and the
// barrier is the non-aligned form, so it stays defined even where the
// compiler has not reconverged the warp after a lane-dependent loop.
__device__ __forceinline__ void group_sync(int id, int threads) {
    __syncwarp();
    asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace

cudaError_t launch_stream_pack(const QView &q, int bits, int gs, int slot_begin, int slot_count, uint8_t *out,
                               cudaStream_t st) {
    StreamGeo sg;
    if (!stream_geo(q.rows, q.cols, bits, gs, &sg)) return cudaErrorInvalidValue;
    if (sg.tg.SB != 16) return cudaErrorInvalidValue;  // 8 groups of 2-byte scales per row
    if (slot_count <= 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>((q.rows / 16) * sg.nck), static_cast<unsigned>(slot_count), 1);
    stream_pack_kernel<<<grid, 256, 0, st>>>(q, sg, slot_begin, out);
    return cudaGetLastError();
}

namespace {

// ------------------------------------------------------------ the GEMV
template <typename TA, int BITS, int GS, int SMODE>
__global__ void __launch_bounds__(kStrMaxWarps * 32, 1) stream_kernel(const GemvArgs a, const StreamCfg c) {
    using Gm = Geo<BITS, GS>;
    using PX = PairX<TA, BITS>;
    constexpr int NM = SMODE == SMODE_GATEUP ? 4 : 2;  // matrices per stage
    constexpr int NROW = 2 * NM;                      // (matrix, row half) pairs per lane
    constexpr int WPS = Gm::kWps;                     // words per lane slice of one group
    constexpr int SPW = Gm::kStepsPerWord;            // k16 steps per code word
    constexpr int S = Gm::kSteps;                     // k16 steps per group
    constexpr int WPG = Gm::kWordsPerGroup;
    constexpr int NW = 2 * WPG;                       // words per lane per row in one round (2 groups)
    constexpr bool OFFSET = (BITS != 8) && FoldOffset<TA>::value;
    constexpr float kM = Act<TA>::kMagicVal;
    static_assert(NW % 4 == 0, "a lane's words per round must be whole 16-byte chunks");

    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int kp = c.kp, spp = c.spp;
    const int gi = warp / kp, q = warp - gi * kp;  // warp group, K part
    uint8_t *ring = smem + c.off_stage + (size_t)warp * c.ns * c.stage_bytes;
    float4 *part = reinterpret_cast<float4 *>(smem + c.off_part) + (size_t)gi * 2 * kp * NM * 32;
    const uint8_t *xres = smem + c.off_res;  // panel rows [prow][K]
    const float2 *sres = reinterpret_cast<const float2 *>(smem + c.off_res + c.res_x);  // [prow][K / 16]
    const int K = a.q0.cols;
    const int K16 = K >> 4;
    const int rows = a.q0.rows;
    const int RT = rows >> 4;
    const int nck = c.nck;

    uint16_t *ptab = reinterpret_cast<uint16_t *>(smem + c.off_ptab);
    if (SMODE == SMODE_GATEUP && a.out_panel)
        for (int i = threadIdx.x; i < a.out_gs; i += blockDim.x) {
            int pe;
            const int pos = panel_pos(i, a.out_bits, a.out_gs, &pe);
            ptab[i] = static_cast<uint16_t>(pos | (pe << 8));
        }

    pdl_wait();  // chunk table and activation rows come from the preceding kernels
    pdl_trigger();
    const bool fused = SMODE == SMODE_GATEUP && a.tk_scores != nullptr;
    TopkRegs tk;
    tk.e = -1;
    tk.pos = -1;
    tk.slot = 0;
    tk.w = 0.0f;
    int nch;
    if (fused) {
        // single token: the routing is selected here (see fused_topk)
        tk = fused_topk(a, true);
        nch = a.tk_k;
    } else {
        nch = *a.n_chunks;
    }
    if (nch < 0 || nch > c.max_chunks) {
        set_error(a.err, -3);
        nch = nch < 0 ? 0 : c.max_chunks;
    }
    // this group's units u = first + j * step (unit u: chunk u / own, row
    // pair u % own of the chunk): spread over every block, or, with the
    // block-local combine, the block's own pairs p = blockIdx.x + i * G
    const int G = static_cast<int>(gridDim.x);
    const int own = c.local ? (c.pairs - static_cast<int>(blockIdx.x) + G - 1) / G : c.pairs;
    const int units = nch * own;
    const int first = c.local ? gi : static_cast<int>(blockIdx.x) + G * gi;
    const int step = c.local ? c.ng : G * c.ng;
    const int my_units = first < units ? (units - first + step - 1) / step : 0;
    const int stages = my_units * spp;

    // metadata of unit j (all lanes; lane n < ntok holds route n)
    auto load_meta = [&](int j, UnitMeta &m) {
        m.slot = 0;
        m.p = 0;
        m.ntok = 0;
        m.route = -1;
        m.row = 0;
        m.w = 1.0f;
        if (j >= my_units) return;
        const int u = first + j * step;
        const int ch = u / own;
        const int i = u - ch * own;
        m.p = c.local ? static_cast<int>(blockIdx.x) + i * G : i;
        if (fused) {
            const unsigned bal = __ballot_sync(LMOE_FULL, tk.pos == ch);
            const int src = bal ? __ffs(bal) - 1 : 0;
            m.slot = __shfl_sync(LMOE_FULL, tk.slot, src);
            m.ntok = 1;
            if (lane == 0) {
                m.route = src;
                m.row = route_row(src, a.route_div, a.shared_base);
            }
            return;
        }
        const Chunk chk = a.chunks[ch];
        m.slot = chk.slot;
        if (m.slot < 0 || m.slot >= a.n_slots) {
            set_error(a.err, -3);
            m.slot = 0;
        }
        m.ntok = chk.ntok;
        if (m.ntok < 0 || m.ntok > c.ntok_cap) {
            set_error(a.err, -3);
            m.ntok = m.ntok < 0 ? 0 : c.ntok_cap;
        }
        if (lane < m.ntok) {
            m.route = a.sorted_routes[chk.route_start + lane];
            if (a.route_w) m.w = a.route_w[m.route];
            m.row = SMODE == SMODE_GATEUP ? route_row(m.route, a.route_div, a.shared_base) : m.route;
            if (m.row < 0 || m.row >= c.prow) {
                set_error(a.err, -3);
                m.row = 0;
            }
        }
    };
    const uint64_t pol = evict_first_policy();
    const int n16 = static_cast<int>(c.blk >> 4);  // 16-byte chunks of one weight block
    // stage s (round r of a unit with metadata m) into slot s % ns: every
    // lane copies its share of the stage's weight blocks with cp.async and
    // closes them into one group (the stage's only completion record)
    auto issue = [&](int s, int r, const UnitMeta &m) {
        uint8_t *dst = ring + (size_t)(s % c.ns) * c.stage_bytes;
        const size_t off = ((size_t)m.p * nck + r) * c.blk;
        const uint8_t *s0 = a.q0.tiles + (size_t)m.slot * a.q0.tile_slot_stride + off;
        for (int i = lane; i < n16; i += 32) cp_async16(dst + 16 * i, s0 + 16 * i, pol);
        if (SMODE == SMODE_GATEUP) {
            const uint8_t *s1 = a.q1.tiles + (size_t)m.slot * a.q1.tile_slot_stride + off;
            for (int i = lane; i < n16; i += 32) cp_async16(dst + c.blk + 16 * i, s1 + 16 * i, pol);
        }
        cp_async_commit();
    };

    UnitMeta cur, nxt;
    load_meta(0, cur);
    load_meta(1, nxt);
    // one group per ring slot from the start (empty past the last stage), so
    // before stage s exactly s + ns groups are committed
    for (int i = 0; i < c.ns; ++i) {
        if (i < stages)
            issue(i, q * spp + i, cur);  // ns <= spp: all of unit 0
        else
            cp_async_commit();
    }
    // the activation rows, resident while the first stages stream in: each
    // thread loads up to 8 of its 16-byte pieces before storing any, so their
    // latencies overlap
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(a.panel);
        uint4 *dst = reinterpret_cast<uint4 *>(smem + c.off_res);
        const uint4 *ss = reinterpret_cast<const uint4 *>(a.sum16);
        uint4 *sd = reinterpret_cast<uint4 *>(smem + c.off_res + c.res_x);
        const int nx = c.res_x >> 4, n = nx + (c.res_s >> 4);
        const int T = static_cast<int>(blockDim.x);
        for (int base = threadIdx.x; base < n; base += 8 * T) {
            uint4 v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int i = base + k * T;
                if (i < n) v[k] = i < nx ? __ldcg(src + i) : __ldcg(ss + (i - nx));
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int i = base + k * T;
                if (i < n) {
                    if (i < nx)
                        dst[i] = v[k];
                    else
                        sd[i - nx] = v[k];
                }
            }
        }
    }
    __syncthreads();

    // per-lane row bases of the swizzled tiles: matrix m, row half h
    int crow[NROW], srow[NROW], sfx[NROW];
#pragma unroll
    for (int r = 0; r < NROW; ++r) {
        const int rr = g + 8 * (r & 1);
        crow[r] = (r >> 1) * c.TB + rr * c.RB;
        srow[r] = (r >> 1) * c.TB + rr * c.SB;
        sfx[r] = (c.sb_l2 >= 0 ? (rr & c.fm_s) : 0) << 4;
    }
    const int cfx = (g & c.fm_c) << 4;  // code rows g and g + 8 share the swizzle
    const int tS = 16 * c.RB;  // scale block of a tile (TileGeo)
    const int tB = tS + 16 * c.SB;

    int s = 0;  // stage counter of this warp
    for (int j = 0; j < my_units; ++j) {
        if (j > 0) {
            cur = nxt;
            load_meta(j + 1, nxt);  // needed ns stages before its first round
        }
        const int ntok = cur.ntok, p = cur.p;
        const bool gpath = ntok == 1;
        // resident panel rows of the unit's tokens
        const int row0 = __shfl_sync(LMOE_FULL, cur.row, 0);
        const int rowg = __shfl_sync(LMOE_FULL, cur.row, g < ntok ? g : 0);
        const int rown0 = __shfl_sync(LMOE_FULL, cur.row, 2 * t < ntok ? 2 * t : 0);
        const int rown1 = __shfl_sync(LMOE_FULL, cur.row, 2 * t + 1 < ntok ? 2 * t + 1 : 0);
        float racc[NM][4];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int e = 0; e < 4; ++e) racc[m][e] = 0.0f;

        for (int ii = 0; ii < spp; ++ii, ++s) {
            const int r = q * spp + ii;  // round of this stage
            cp_async_wait_pending(c.ns - 1);
            __syncwarp();  // every lane's copies of the stage have landed
            const uint8_t *sb = ring + (size_t)(s % c.ns) * c.stage_bytes;
            if (gpath) {
                // ---- one token: columns = the round's 8 groups; lane t
                // covers words [t * NW, (t + 1) * NW) = groups 2t, 2t + 1
                const uint8_t *xs8 = xres + ((size_t)row0 * K + (size_t)r * c.CK) * 2;
                const float2 *xsum = sres + (size_t)row0 * K16 + (size_t)r * (c.CK / 16);
                float2 gx = make_float2(0.0f, 0.0f);
                {
                    const int n = lane >> 2, sub = lane & 3;  // 4 lanes per group
                    for (int qq = sub; qq < S; qq += 4) {
                        const float2 v = xsum[n * S + qq];
                        gx.x += v.x;
                        gx.y += v.y;
                    }
                }
                // scales / biases of groups 2t and 2t + 1 (adjacent: one word)
                uint32_t sw[NM][2], bw[NM][2];
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int rr = 2 * m + h;
                        const int os = srow[rr] + ((4 * t) ^ sfx[rr]);
                        sw[m][h] = sld<uint32_t>(sb + tS + os);
                        bw[m][h] = sld<uint32_t>(sb + tB + os);
                    }
                float d[NM][4];
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int e = 0; e < 4; ++e) d[m][e] = 0.0f;
#pragma unroll 1
                for (int qc = 0; qc < NW / 4; ++qc) {
                    const int w0 = t * NW + 4 * qc;  // first code word of this chunk in the row
                    const bool act = (g == w0 / WPG);
                    uint32_t raw[NROW][4];
#pragma unroll
                    for (int rr = 0; rr < NROW; ++rr) {
                        const uint4 v = sld<uint4>(sb + crow[rr] + ((w0 * 4) ^ cfx));
                        raw[rr][0] = v.x;
                        raw[rr][1] = v.y;
                        raw[rr][2] = v.z;
                        raw[rr][3] = v.w;
                    }
                    const uint8_t *bp = xs8 + w0 * SPW * 8;
                    uint4 bq = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        typename PX::W pw[NROW];
#pragma unroll
                        for (int rr = 0; rr < NROW; ++rr) pw[rr] = PX::prep(raw[rr][i]);
#pragma unroll
                        for (int s2 = 0; s2 < SPW; ++s2) {
                            const int js = i * SPW + s2;
                            if ((js & 1) == 0 && act) bq = sld<uint4>(bp + js * 8);
                            const uint32_t b0 = (js & 1) ? bq.z : bq.x;
                            const uint32_t b1 = (js & 1) ? bq.w : bq.y;
#pragma unroll
                            for (int m = 0; m < NM; ++m)
                                Act<TA>::mma(d[m], PX::get(pw[2 * m], 2 * s2), PX::get(pw[2 * m + 1], 2 * s2),
                                             PX::get(pw[2 * m], 2 * s2 + 1), PX::get(pw[2 * m + 1], 2 * s2 + 1), b0,
                                             b1);
                        }
                    }
                }
                gx.x += __shfl_xor_sync(LMOE_FULL, gx.x, 1);
                gx.y += __shfl_xor_sync(LMOE_FULL, gx.y, 1);
                gx.x += __shfl_xor_sync(LMOE_FULL, gx.x, 2);
                gx.y += __shfl_xor_sync(LMOE_FULL, gx.y, 2);
                const float X0 = __shfl_sync(LMOE_FULL, gx.x, 8 * t), P0 = __shfl_sync(LMOE_FULL, gx.y, 8 * t);
                const float X1 = __shfl_sync(LMOE_FULL, gx.x, 8 * t + 4), P1 = __shfl_sync(LMOE_FULL, gx.y, 8 * t + 4);
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const float s0 = Act<TA>::to_f(static_cast<uint16_t>(sw[m][h] & 0xffffu));
                        const float s1 = Act<TA>::to_f(static_cast<uint16_t>(sw[m][h] >> 16));
                        const float b0 = Act<TA>::to_f(static_cast<uint16_t>(bw[m][h] & 0xffffu));
                        const float b1 = Act<TA>::to_f(static_cast<uint16_t>(bw[m][h] >> 16));
                        float e0 = d[m][2 * h], e1 = d[m][2 * h + 1];
                        if constexpr (OFFSET) {
                            e0 = fmaf(-kM, P0, e0);
                            e1 = fmaf(-kM, P1, e1);
                        }
                        float tot = fmaf(s0, e0, b0 * X0);
                        tot = fmaf(s1, e1, tot);
                        tot = fmaf(b1, X1, tot);
                        tot += __shfl_xor_sync(LMOE_FULL, tot, 1);
                        tot += __shfl_xor_sync(LMOE_FULL, tot, 2);
                        racc[m][2 * h] += tot;  // column 0: the unit's single token
                    }
            } else {
                // ---- several tokens: columns = tokens (lane column g);
                // per group, lane t's slice of WPS words per row
                const bool has_b = g < ntok;
                const uint8_t *xrow = xres + ((size_t)rowg * K + (size_t)r * c.CK) * 2;
#pragma unroll 1
                for (int G8 = 0; G8 < 8; ++G8) {
                    typename PX::W pw[NROW][WPS];
                    uint16_t sv[NROW], bv[NROW];
                    const int goff = G8 * WPG * 4 + t * WPS * 4;
#pragma unroll
                    for (int rr = 0; rr < NROW; ++rr) {
                        uint32_t wd[WPS];
                        if constexpr (WPS == 1) {
                            wd[0] = sld<uint32_t>(sb + crow[rr] + (goff ^ cfx));
                        } else if constexpr (WPS == 2) {
                            const uint2 v = sld<uint2>(sb + crow[rr] + (goff ^ cfx));
                            wd[0] = v.x;
                            wd[1] = v.y;
                        } else {
#pragma unroll
                            for (int qq = 0; qq < WPS / 4; ++qq) {
                                const uint4 v = sld<uint4>(sb + crow[rr] + ((goff + 16 * qq) ^ cfx));
                                wd[4 * qq] = v.x;
                                wd[4 * qq + 1] = v.y;
                                wd[4 * qq + 2] = v.z;
                                wd[4 * qq + 3] = v.w;
                            }
                        }
#pragma unroll
                        for (int qq = 0; qq < WPS; ++qq) pw[rr][qq] = PX::prep(wd[qq]);
                        const int os = srow[rr] + ((2 * G8) ^ sfx[rr]);
                        sv[rr] = sld<uint16_t>(sb + tS + os);
                        bv[rr] = sld<uint16_t>(sb + tB + os);
                    }
                    // (sum x, sum of stored panel values) of the lane's two token columns
                    float2 xt[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int n = 2 * t + h;
                        if (n < ntok) {
                            const float2 *p2 =
                                sres + (size_t)(h ? rown1 : rown0) * K16 + (size_t)r * (c.CK / 16) + G8 * S;
#pragma unroll
                            for (int qq = 0; qq < S; ++qq) {
                                const float2 v = p2[qq];
                                xt[h].x += v.x;
                                xt[h].y += v.y;
                            }
                        }
                    }
                    float d[NM][4];
#pragma unroll
                    for (int m = 0; m < NM; ++m)
#pragma unroll
                        for (int e = 0; e < 4; ++e) d[m][e] = 0.0f;
                    uint4 bq = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                    for (int k = 0; k < S; ++k) {
                        const int wi = k / SPW, s2 = k % SPW;
                        if ((k & 1) == 0 && has_b) bq = sld<uint4>(xrow + ((G8 * 4 + t) * S + k) * 8);
                        const uint32_t b0 = (k & 1) ? bq.z : bq.x;
                        const uint32_t b1 = (k & 1) ? bq.w : bq.y;
#pragma unroll
                        for (int m = 0; m < NM; ++m)
                            Act<TA>::mma(d[m], PX::get(pw[2 * m][wi], 2 * s2), PX::get(pw[2 * m + 1][wi], 2 * s2),
                                         PX::get(pw[2 * m][wi], 2 * s2 + 1), PX::get(pw[2 * m + 1][wi], 2 * s2 + 1),
                                         b0, b1);
                    }
#pragma unroll
                    for (int m = 0; m < NM; ++m) {
                        float e[4] = {d[m][0], d[m][1], d[m][2], d[m][3]};
                        if constexpr (OFFSET) {
                            e[0] = fmaf(-kM, xt[0].y, e[0]);
                            e[1] = fmaf(-kM, xt[1].y, e[1]);
                            e[2] = fmaf(-kM, xt[0].y, e[2]);
                            e[3] = fmaf(-kM, xt[1].y, e[3]);
                        }
                        const float s0 = Act<TA>::to_f(sv[2 * m]), s1 = Act<TA>::to_f(sv[2 * m + 1]);
                        const float b0 = Act<TA>::to_f(bv[2 * m]), b1 = Act<TA>::to_f(bv[2 * m + 1]);
                        racc[m][0] = fmaf(e[0], s0, fmaf(xt[0].x, b0, racc[m][0]));
                        racc[m][1] = fmaf(e[1], s0, fmaf(xt[1].x, b0, racc[m][1]));
                        racc[m][2] = fmaf(e[2], s1, fmaf(xt[0].x, b1, racc[m][2]));
                        racc[m][3] = fmaf(e[3], s1, fmaf(xt[1].x, b1, racc[m][3]));
                    }
                }
            }
            // release the slot (every lane is done reading it), then queue
            // stage s + ns into it
            __syncwarp();
            const int sn = s + c.ns;
            if (sn < stages) {
                const int jn = sn / spp;  // j or j + 1 (ns <= spp)
                issue(sn, q * spp + (sn - jn * spp), jn == j ? cur : nxt);
            } else {
                cp_async_commit();
            }
        }

        // ---- K parts: each warp leaves its partial sums in the group's
        // buffer for this unit; one warp (rotating) adds them in part order
        if (kp > 1) {
            float4 *pb = part + (size_t)((j & 1) * kp + q) * NM * 32;
#pragma unroll
            for (int m = 0; m < NM; ++m) pb[m * 32 + lane] = make_float4(racc[m][0], racc[m][1], racc[m][2], racc[m][3]);
            group_sync(1 + gi, kp * 32);
            if (q != j % kp) continue;
            const float4 *p0 = part + (size_t)(j & 1) * kp * NM * 32;
#pragma unroll
            for (int m = 0; m < NM; ++m) {
                float4 v = p0[m * 32 + lane];
                for (int qq = 1; qq < kp; ++qq) {
                    const float4 w = p0[(qq * NM + m) * 32 + lane];
                    v.x += w.x;
                    v.y += w.y;
                    v.z += w.z;
                    v.w += w.w;
                }
                racc[m][0] = v.x;
                racc[m][1] = v.y;
                racc[m][2] = v.z;
                racc[m][3] = v.w;
            }
        }

        // ---- epilogue of the unit (racc: rows g / g + 8 x token columns 2t, 2t + 1)
        if constexpr (SMODE == SMODE_GATEUP) {
            // matrices: 0 / 1 = gate tiles 2p / 2p + 1, 2 / 3 = the same up tiles
#pragma unroll
            for (int ti = 0; ti < 2; ++ti) {
                const int rt = 2 * p + ti;
                float hv[4], hp[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float h = swiglu_h<TA>(racc[ti][e], racc[2 + ti][e], a.limit, a.swiglu_mode);
                    const int n = 2 * t + (e & 1);
                    const int row = rt * 16 + g + 8 * (e >> 1);
                    const int route = __shfl_sync(LMOE_FULL, cur.route, n < ntok ? n : 0);
                    hv[e] = 0.0f;
                    hp[e] = 0.0f;
                    if (n < ntok) {
                        hv[e] = h;
                        if (a.out_panel) {
                            const int tv = ptab[row & (a.out_gs - 1)];
                            const int out_lg = __ffs(a.out_gs) - 1;
                            const int pos = ((row >> out_lg) << out_lg) + (tv & 0xff);
                            const int pe = tv >> 8;
                            const uint16_t pv =
                                Act<TA>::from_f(h * (pe == 0 ? 1.0f : (pe == 1 ? 0.25f : 0.0625f)));
                            hp[e] = Act<TA>::to_f(pv);
                            a.out[(size_t)route * rows + pos] = pv;
                        } else {
                            a.out[(size_t)route * rows + row] = Act<TA>::from_f(h);
                        }
                    }
                }
                if (a.out_sum16) {
                    float s0 = hv[0] + hv[2], s1 = hv[1] + hv[3];
                    float p0 = hp[0] + hp[2], p1 = hp[1] + hp[3];
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) {
                        s0 += __shfl_xor_sync(LMOE_FULL, s0, o);
                        s1 += __shfl_xor_sync(LMOE_FULL, s1, o);
                        p0 += __shfl_xor_sync(LMOE_FULL, p0, o);
                        p1 += __shfl_xor_sync(LMOE_FULL, p1, o);
                    }
                    const int r0 = __shfl_sync(LMOE_FULL, cur.route, 2 * t < ntok ? 2 * t : 0);
                    const int r1 = __shfl_sync(LMOE_FULL, cur.route, 2 * t + 1 < ntok ? 2 * t + 1 : 0);
                    if (g == 0) {
                        if (2 * t < ntok)
                            *reinterpret_cast<float2 *>(a.out_sum16 + ((size_t)r0 * RT + rt) * 2) = make_float2(s0, p0);
                        if (2 * t + 1 < ntok)
                            *reinterpret_cast<float2 *>(a.out_sum16 + ((size_t)r1 * RT + rt) * 2) = make_float2(s1, p1);
                    }
                }
            }
        } else {
            // y * w per route row of both tiles (w = 1 without weights)
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int n = 2 * t + (e & 1);
                    const int row = (2 * p + m) * 16 + g + 8 * (e >> 1);
                    const int route = __shfl_sync(LMOE_FULL, cur.route, n < ntok ? n : 0);
                    const float wr = __shfl_sync(LMOE_FULL, cur.w, n < ntok ? n : 0);
                    if (n < ntok) {
                        const float y = Act<TA>::round(racc[m][e]);
                        const float wv = a.route_w ? Act<TA>::round(wr) : 1.0f;
                        a.out[(size_t)route * rows + row] = Act<TA>::from_f(y * wv);
                    }
                }
        }
    }
    cp_async_wait_pending(0);  // only empty groups remain
    if constexpr (SMODE == SMODE_PAIR) {
        if (!c.local || !a.combined) return;
        // block-local combine over the pairs this block owns: each token's
        // k route rows summed in route order in fp32 (read back from L2),
        // then the shared expert's row and the residual (combine_finish)
        __threadfence_block();
        __syncthreads();
        const int items = own * 32 * a.n_tok;
        for (int i = threadIdx.x; i < items; i += blockDim.x) {
            const int ri = i & 31, rest = i >> 5;
            const int tok = rest % a.n_tok, jp = rest / a.n_tok;
            const int row = (static_cast<int>(blockIdx.x) + jp * G) * 32 + ri;
            float sacc = 0.0f;
            for (int r = 0; r < a.top_k; ++r)
                sacc += Act<TA>::to_f(__ldcg(reinterpret_cast<const unsigned short *>(
                    a.out + ((size_t)tok * a.top_k + r) * rows + row)));
            const bool sh = a.shared_base > 0;
            const uint16_t sv = sh ? __ldcg(reinterpret_cast<const unsigned short *>(
                                         a.out + ((size_t)a.shared_base + tok) * rows + row))
                                   : 0;
            const uint16_t rv = a.residual ? a.residual[(size_t)tok * rows + row] : 0;
            a.combined[(size_t)tok * rows + row] =
                Act<TA>::from_f(combine_finish<TA>(sacc, sh, sv, a.residual != nullptr, rv));
        }
    }
}

int g_sms = 0;
int sm_count() {
    if (g_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_sms <= 0) g_sms = 148;
    }
    return g_sms;
}

constexpr int kStrSmem = 227 * 1024;

inline int align128(int v) { return (v + 127) & ~127; }

// Shared-memory plan for kp warps per unit and ns stages per warp: the
// panel-position table (256 B), each group's double-buffered partials, the
// resident activation rows, then the warps' rings; as many warps (a multiple
// of kp, <= 8) as fit.
bool plan_fit(StreamCfg &c, int kp, int ns) {
    const int part_w = kp > 1 ? 2 * c.nm * 32 * 16 : 0;
    for (int nc = kStrMaxWarps - kStrMaxWarps % kp; nc >= kp; nc -= kp) {
        const int off_part = 256;
        const int off_res = align128(off_part + nc * part_w);
        const long off_stage = align128(off_res + c.res_x + c.res_s);
        const long smem = off_stage + (long)nc * ns * c.stage_bytes;
        if (smem > kStrSmem) continue;
        c.kp = kp;
        c.ng = nc / kp;
        c.nc = nc;
        c.ns = ns;
        c.spp = c.nck / kp;
        c.off_ptab = 0;
        c.off_part = off_part;
        c.off_res = off_res;
        c.off_stage = static_cast<int>(off_stage);
        c.smem = static_cast<int>(smem);
        return true;
    }
    return false;
}

// Work split for a launch of at most `units` units (local: per block): the
// K-part count whose slowest warp streams the fewest stages (a one-stage
// ring counts half again: nothing overlaps its waits), ties to fewer parts.
// LMOE_STREAM_KP (1, 2, 4 or 8) forces the part count when it fits.
bool stream_plan(StreamCfg &c, long units, int sms) {
    static int forced = -1;
    if (forced < 0) {
        const char *e = getenv("LMOE_STREAM_KP");
        forced = e ? atoi(e) : 0;
    }
    StreamCfg best = c;
    double best_cost = 0.0;
    bool have = false;
    for (int kp = 1; kp <= 8; kp <<= 1) {
        if (c.nck % kp) continue;
        if (forced > 0 && kp != forced) continue;
        const int spp = c.nck / kp;
        StreamCfg x = c;
        int ns = spp < (kp == 1 ? 3 : 2) ? spp : (kp == 1 ? 3 : 2);
        while (ns >= 1 && !plan_fit(x, kp, ns)) --ns;
        if (ns < 1) continue;
        long grid, rounds;
        if (x.local) {
            grid = x.grid;
            rounds = (units + x.ng - 1) / x.ng;
        } else {
            grid = (units + x.ng - 1) / x.ng;
            if (grid > sms) grid = sms;
            if (grid < 1) grid = 1;
            rounds = (units + grid * x.ng - 1) / (grid * x.ng);
        }
        x.grid = static_cast<int>(grid);
        double cost = (double)rounds * spp * (x.ns == 1 && spp > 1 ? 1.5 : 1.0);
        if (kp > 1) cost += 0.5 * rounds;  // the partials' reduction
        if (!have || cost < best_cost) {
            best = x;
            best_cost = cost;
            have = true;
        }
    }
    if (!have) return false;
    c = best;
    return true;
}

template <typename TA, int BITS, int GS, int SMODE>
cudaError_t launch_stream_t(const GemvArgs &a, const StreamCfg &c0, int max_chunks, cudaStream_t st) {
    auto kern = stream_kernel<TA, BITS, GS, SMODE>;
    if (a.ntok_max > c0.ntok_cap || max_chunks < 1) return cudaErrorInvalidValue;
    StreamCfg c = c0;
    c.max_chunks = max_chunks;
    // chunks to plan for: each holds at least one route, so the caller's
    // route count bounds them as well as the table's capacity
    const long est = a.chunks_est > 0 && a.chunks_est < max_chunks ? a.chunks_est : max_chunks;
    const long units = c.local ? est * ((c.pairs + c.grid - 1) / (c.grid > 0 ? c.grid : 1)) : est * c.pairs;
    if (c.local && c.grid < 1) return cudaErrorInvalidValue;
    if (!stream_plan(c, units, sm_count())) return cudaErrorInvalidValue;
    static int configured = 0;
    if (c.smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, c.smem);
        if (e != cudaSuccess) return e;
        configured = c.smem;
    }
    return launch_pdl(kern, dim3(static_cast<unsigned>(c.grid)), dim3(c.nc * 32), c.smem, st, a, c);
}

template <typename TA, int SMODE>
cudaError_t launch_stream_bits(int bits, int gs, const GemvArgs &a, const StreamCfg &c, int max_chunks,
                               cudaStream_t st) {
#define LMOE_SCASE(B, Gs) \
    if (bits == B && gs == Gs) return launch_stream_t<TA, B, Gs, SMODE>(a, c, max_chunks, st);
    LMOE_SCASE(2, 64)
    LMOE_SCASE(2, 128)
    LMOE_SCASE(4, 32)
    LMOE_SCASE(4, 64)
    LMOE_SCASE(4, 128)
    LMOE_SCASE(8, 32)
    LMOE_SCASE(8, 64)
    LMOE_SCASE(8, 128)
#undef LMOE_SCASE
    return cudaErrorInvalidValue;
}

}  // namespace

// Geometry and the shared-memory footprint: a stage holds the round's weight
// blocks (gate and up, or one projection); the activation rows the launch
// may read stay resident.  The work split is chosen at launch (stream_plan).
bool stream_config(int smode, int rows, int K, int bits, int gs, bool local, int ntok_cap, int prow,
                   StreamCfg *out) {
    StreamGeo sg;
    if (!stream_geo(rows, K, bits, gs, &sg) || sg.tg.SB != 16) return false;
    if (ntok_cap < 1 || ntok_cap > kChunkTok || prow < 1) return false;
    StreamCfg c;
    std::memset(&c, 0, sizeof(c));
    c.nm = smode == SMODE_GATEUP ? 4 : 2;
    c.TB = sg.tg.TB;
    c.RB = sg.tg.RB;
    c.SB = sg.tg.SB;
    c.sb_l2 = sg.tg.sb_l2;
    c.fm_c = sg.tg.fm_c;
    c.fm_s = sg.tg.fm_s;
    c.CK = sg.CK;
    c.nck = sg.nck;
    c.pairs = sg.pairs;
    c.blk = sg.block;
    c.ntok_cap = ntok_cap;
    c.prow = prow;
    const long rx = (long)prow * K * 2, rs = (long)prow * (K / 16) * 8;
    if (rx + rs > kStrSmem) return false;
    c.res_x = static_cast<int>(rx);
    c.res_s = static_cast<int>(rs);
    c.stage_bytes = align128(static_cast<int>(c.nm / 2 * c.blk));
    c.local = local ? 1 : 0;
    c.grid = 0;
    StreamCfg probe = c;
    if (!plan_fit(probe, 1, 1)) return false;  // at least one warp with one stage
    *out = c;
    return true;
}

cudaError_t launch_stream(int smode, int act_f16, int bits, int gs, const GemvArgs &a, const StreamCfg &c,
                          int max_chunks, cudaStream_t st) {
    if (act_f16) {
        if (smode == SMODE_GATEUP) return launch_stream_bits<__half, SMODE_GATEUP>(bits, gs, a, c, max_chunks, st);
        return launch_stream_bits<__half, SMODE_PAIR>(bits, gs, a, c, max_chunks, st);
    }
    if (smode == SMODE_GATEUP) return launch_stream_bits<__nv_bfloat16, SMODE_GATEUP>(bits, gs, a, c, max_chunks, st);
    return launch_stream_bits<__nv_bfloat16, SMODE_PAIR>(bits, gs, a, c, max_chunks, st);
}

}  // namespace lmoe
