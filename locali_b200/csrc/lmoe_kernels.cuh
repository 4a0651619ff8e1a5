// Kernel argument structs and launch helpers shared by lmoe_kernels.cu and
// lmoe_api.cu.
#pragma once

#include <cuda.h>

#include "lmoe_common.cuh"

namespace lmoe {

// MODE_DOWN2: down + weighted combine over pairs of row tiles, each block
// owning whole pairs for every chunk (block-local combine, decode layers)
enum GemvMode { MODE_GATEUP = 0, MODE_DOWN = 1, MODE_QMM = 2, MODE_DOWN2 = 3 };

// Geometry of one 16-row weight tile as the GEMV consumers read it from
// shared memory: [codes 16 x RB][scales 16 x SB][biases 16 x SB], padded to
// 128 bytes.  Rows are contiguous; inside each 128-byte line the 16-byte
// chunks of row r are XOR-swizzled (codes by r & 7, scale/bias rows by r) so
// the rows a warp reads at once fall in distinct bank groups.  The same
// layout is the pre-tiled HBM format, so one bulk copy moves a tile.
struct TileGeo {
    int32_t RB, SB;        // code / scale bytes per row
    int32_t rb_l2, sb_l2;  // log2(16-byte chunks per row); sb_l2 < 0: rows < 16 B
    int32_t fm_c, fm_s;    // swizzle masks
    int32_t tS, tB, TB;    // scale and bias offsets, padded tile bytes
};

__host__ __device__ inline int tile_log2_exact(int v) {
    int l = 0;
    while ((1 << l) < v) ++l;
    return (1 << l) == v ? l : -1;
}

// false when (K, bits, gs) has no tile layout (rows must be a power-of-two
// number of 16-byte chunks)
__host__ __device__ inline bool tile_geo(int K, int bits, int gs, TileGeo *g) {
    TileGeo t;
    t.RB = K * bits / 8;
    t.SB = (K / gs) * 2;
    if (t.RB < 16 || t.RB % 16) return false;
    t.rb_l2 = tile_log2_exact(t.RB / 16);
    if (t.rb_l2 < 0) return false;
    t.fm_c = (t.RB < 128 ? t.RB : 128) / 16 - 1;
    if (t.SB >= 16) {
        t.sb_l2 = tile_log2_exact(t.SB / 16);
        if (t.sb_l2 < 0) return false;
        t.fm_s = (t.SB < 128 ? t.SB : 128) / 16 - 1;
    } else {
        t.sb_l2 = -1;  // rows shorter than a chunk: the 16-row block is stored unswizzled
        t.fm_s = 0;
    }
    t.tS = 16 * t.RB;
    t.tB = t.tS + 16 * t.SB;
    t.TB = (t.tB + 16 * t.SB + 127) / 128 * 128;
    *g = t;
    return true;
}

// Byte offset inside a tile of 16-byte chunk i of the code block (chunks in
// row-major order, 2^rb_l2 per row).
__host__ __device__ inline int tile_code_chunk(const TileGeo &t, int i) {
    const int row = i >> t.rb_l2;
    return (i << 4) ^ (((row & 7) & t.fm_c) << 4);
}
// Byte offset, relative to the scale (or bias) block, of its 16-byte chunk i.
__host__ __device__ inline int tile_sb_chunk(const TileGeo &t, int i) {
    if (t.sb_l2 < 0) return i << 4;
    return (i << 4) ^ ((((i >> t.sb_l2)) & t.fm_s) << 4);
}

// ------------------------------------------------------------ stream format
// The pre-tiled HBM copy the decode GEMVs stream (lmoe_tile_pack).  The K
// dimension is cut into chunks of 8 quantisation groups (CK = 8 * gs, one
// round of the GEMV's 8 group columns); 16-row tiles are paired (2p, 2p+1).
// Block (pair p, chunk c) = two TileGeo(CK) tiles, rows 32p..32p+15 then
// 32p+16..32p+31, each [codes 16 x RB][scales 16 x SB][biases 16 x SB]
// swizzled and padded as TileGeo lays them out.  Per slot: pairs x chunks
// blocks in (pair, chunk) order, so a GEMV unit's rounds are consecutive.
struct StreamGeo {
    TileGeo tg;     // one 16-row tile of a CK-column chunk
    int32_t CK;     // columns per chunk
    int32_t nck;    // chunks per row
    int32_t pairs;  // 32-row pairs
    int64_t block;  // bytes of one (pair, chunk) block = 2 * tg.TB
    int64_t slot;   // bytes per slot
};
__host__ __device__ inline bool stream_geo(int rows, int K, int bits, int gs, StreamGeo *g) {
    StreamGeo s;
    s.CK = 8 * gs;
    if (rows <= 0 || rows % 32 != 0 || K <= 0 || K % s.CK != 0) return false;
    if (!tile_geo(s.CK, bits, gs, &s.tg)) return false;
    s.nck = K / s.CK;
    s.pairs = rows / 32;
    s.block = 2 * (int64_t)s.tg.TB;
    s.slot = s.block * s.nck * s.pairs;
    *g = s;
    return true;
}

struct DispatchOut {
    int32_t *sorted_routes;  // [R]
    Chunk *chunks;           // [max_chunks]
    int32_t *n_chunks;       // [1]
    int32_t *counts;         // [buckets] (large path)
    int32_t *route_off;      // [buckets] (large path)
    int32_t *blk;            // [ceil(R / 256)][buckets] scratch of the large path, or nullptr
};

struct DispatchIn {
    const int32_t *idx;          // [R] expert id (or slot) per route
    int32_t R;
    int32_t chunk_tok;           // routes per chunk (1..8)
    int32_t n_experts;           // valid ids are [0, n_experts); others -> zero bucket
    const int32_t *expert_slot;  // [n_experts] or nullptr (identity: id is the slot)
    int32_t n_slots;
    // expert-parallel receive side: negative ids are routes owned by another
    // rank (dropped without an error) and the zero bucket gets no chunks
    int32_t drop_zero = 0;
};

struct RouterArgs {
    const uint16_t *x;  // [T, H]
    int32_t T, H;
    const uint16_t *wg;  // [E, H] bf16
    const float *bias;   // [E] or nullptr
    int32_t E, top_k, scoring, norm_topk;
    float scaling;
    float *partial;  // [ksplit][T][E] logits
    float2 *scores;  // [T][E] (score, score + bias) for the element-wise scorings, or nullptr
    // single token: int8 pieces of x for the single-token layer kernel
    // (pbits / pgs of its gate/up), or nullptr
    uint8_t *xq;
    float2 *xs;
    // panel producer for the gate/up consumer (optional)
    uint16_t *xpanel;
    float *xsum16;  // [T, H/16, 2]: per 16 columns, sum of x and sum of the stored panel values
    int32_t pbits, pgs;
    int32_t act_f16;
    // finisher (decode regime): last CTA runs top-k + dispatch
    int32_t finish;
    int32_t do_dispatch;
    uint32_t *counter;
    int32_t *idx_ws;  // [T*k]
    float *w_ws;      // [T*k]
    int32_t *idx_user;
    float *w_user;
    DispatchIn din;
    DispatchOut dout;
    int32_t *err;
    // combine counters of this call, zeroed by the router blocks
    uint32_t *zero;
    int32_t zero_words;
    // token-id hash routing: [T, top_k] expert ids replacing the top-k search, or nullptr
    const int32_t *hash_idx;
    // tensor-core logits split over the hidden dimension (router_ksplit):
    // block z writes partial[z][T][E]; the top-k sums the splits in order
    int32_t ksplit;
};

// Splits of the hidden dimension for the tensor-core router logits: with few
// tokens the 64-token x 128-expert tiles leave most SMs idle, so each tile's
// K range is divided over up to KT/4 blocks (at least four 64-column stages
// each) until about one block per SM.  The partial logits are summed in
// split order by the top-k (fixed order: deterministic).
__host__ __device__ inline int router_ksplit(int T, int E, int H, bool act_f16) {
    if (T <= 64 || act_f16 || T > 1024 || H % 64 != 0) return 1;
    const int blocks = ((T + 63) / 64) * ((E + 127) / 128);
    const int KT = H / 64;
    const int want = (148 + blocks - 1) / blocks;
    int ks = 1;
    for (int c = 1; c <= KT / 4 && c <= want; ++c)
        if (KT % c == 0) ks = c;
    return ks;
}

struct TopkArgs {
    const float *partial;
    const float2 *scores;  // precomputed (score, biased score) or nullptr
    int32_t ksplit, T, E, top_k, scoring, norm_topk;
    float scaling;
    const float *bias;
    int32_t *idx_ws;
    float *w_ws;
    int32_t *idx_user;
    float *w_user;
    const int32_t *hash_idx;  // as RouterArgs::hash_idx
};

struct PanelArgs {
    const uint16_t *x;  // natural [rows, K]
    int32_t rows, K;
    int32_t x_stride;   // elements between rows of x (0: K)
    uint16_t *panel;    // [rows, K]
    float *sum16;       // [rows, K/16, 2] (sum of x, sum of panel values)
    int32_t bits, gs;
    int32_t act_f16;
    uint32_t *zero;  // combine counters of this call, zeroed here (or nullptr)
    int32_t zero_words;
};

struct GemvArgs {
    QView q0, q1;
    const uint16_t *panel;
    const float *sum16;  // [routes or tokens, K/16, 2]
    int32_t route_div;
    const Chunk *chunks;
    const int32_t *n_chunks;
    const int32_t *sorted_routes;
    int32_t n_slots;
    int32_t ntok_max;
    int32_t chunks_est;  // host-side planning hint: chunks this launch expects (0: the table's capacity)
    uint16_t *out;
    float *out_sum16;  // [routes, rows/16, 2]
    int32_t out_panel, out_bits, out_gs;
    float limit;
    int32_t swiglu_mode;
    const float *route_w;
    int32_t top_k;
    int32_t n_tok;  // tokens of the layer (MODE_DOWN2 combine)
    uint32_t *counters;
    uint16_t *combined;
    int32_t *err;
    // shared expert: routes >= shared_base (> 0 when present) are the shared
    // expert's, one per token (route shared_base + t reads activation row t);
    // the combine adds its row after rounding the routed sum, then residual
    int32_t shared_base;
    const uint16_t *residual;  // [tokens, rows] or nullptr
    // single-token layers (stream gate/up): every block selects the top-k
    // from the router's (score, biased score) itself instead of the router's
    // last block; block 0 writes the routing and the dispatch for the down
    // kernel and the caller.  tk_scores == nullptr: chunks come from memory.
    const float2 *tk_scores;
    int32_t tk_E, tk_k, tk_norm;
    float tk_scaling;
    const int32_t *tk_expert_slot;
    int32_t *tk_idx, *tk_idx_user, *tk_sorted, *tk_nchunks;
    float *tk_w, *tk_w_user;
    Chunk *tk_chunks;
#ifdef LMOE_PROFILE_TRACE
    // per-unit timeline (nanoseconds, %globaltimer) of a profiling build:
    // [block][unit slot][8]
    uint64_t *trace;
    int32_t trace_units;
#endif
};

// Shared-memory plan of one gemv launch (computed on the host, passed by value).
struct GemvCfg {
    int32_t ncw, nst, gw;                       // consumer warps, stages, groups per consumer
    int32_t RB, SB, TBp;                        // code / scale bytes per row, tile stride (TileGeo)
    int32_t rb_l2, sb_l2;                       // log2(16-byte chunks per row); sb_l2 < 0: rows < 16 B
    int32_t fm_c, fm_s;                         // swizzle masks of code / scale tiles
    int32_t PB, PBp, S16B;                      // panel row bytes, padded stride, sum16 row bytes
    int32_t off_codes, off_s, off_b;            // matrix m's tile at off_codes + m * TBp
    int32_t off_panel, off_sum, stage_bytes;
    int32_t off_bars, off_shdr, off_rhdr, off_red, off_xs, off_list, off_ptab, off_stage, smem, list_cap;
};
// Consumer warps per block: two per SM sub-partition.  Sixteen (four per
// sub-partition, register cap 80) made the C1 gate/up GEMV slower on B200
// (30.5 against 26.7 us): a unit's consumers start together and each warp's
// mma.sync stream with its code extraction is latency-bound.
constexpr int kGemvMaxConsumers = 8;
constexpr int kGemvEpi = 4;  // epilogue warps
constexpr int kGemvMaxThreads = (kGemvMaxConsumers + 2 + kGemvEpi) * 32;  // + 2 producer warps
constexpr int kGemvMaxStages = 4;
// per-stage header (ints): [0] ntok, [1] row tile, [2] slot, then the
// routes, their combine weights and the activation rows held by the stage
constexpr int kHdrBytes = 128;
constexpr int kHdrRoute = 4;
constexpr int kHdrWeight = 12;
constexpr int kHdrPanel = 20;
constexpr int kHdrPanelN = 28;
bool gemv_config(int mode, int bits, int gs, int K, int ntok_max, GemvCfg *out);

// Single-token routing held in registers (lane j < k: the j-th winner's
// expert id, weight, arena slot, and its rank among the winners' ids, which
// is its chunk in the dispatch; other lanes hold pos = -1).
struct TopkRegs {
    int e, pos, slot;
    float w;
};

// Order-preserving 32-bit key of a biased score for the warp max: larger
// key = larger score; -0 folds into +0 (float compares treat them as equal)
// and -inf / NaN map to 0, which is never selected.
__device__ __forceinline__ uint32_t topk_key(float v) {
    v = v + 0.0f;
    if (!(v > -INFINITY)) return 0u;
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Top-k of a single token by one warp from the router's (score, biased
// score) (arena.py:501-506): selection on the biased score, ties to the
// lower id.  Each lane keeps its best candidate (first of equals in id
// order); a round is a warp max of the keys and a warp min of the ids that
// reach it (redux.sync), and only the winner's lane rescans.  Weights: raw
// scores normalised by their fp32 sum in selection order + 1e-20, times the
// routed scaling.  The dispatch of the k distinct experts: chunk i = the
// route of the i-th smallest expert id.  The same winners, order and weights
// as the router's own finisher.  Every warp of the launch computes it; warp
// 0 of block 0 also writes the routing and the dispatch to memory for the
// down kernel and the caller (write = true; a kernel that only needs the
// winners passes false).
template <class A>
__device__ __forceinline__ TopkRegs fused_topk(const A &a, bool write) {
    const int lane = threadIdx.x & 31;
    const int E = a.tk_E, k = a.tk_k;
    uint32_t key[16];
    float sc[16];
    int sl[16];  // arena slots of the candidates, loaded with the scores
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int e = lane + 32 * i;
        key[i] = 0u;
        sc[i] = 0.0f;
        sl[i] = e;
        if (32 * i < E && e < E) {
            const float2 v = __ldcg(a.tk_scores + e);
            sc[i] = v.x;
            key[i] = topk_key(v.y);
            if (a.tk_expert_slot) sl[i] = __ldg(a.tk_expert_slot + e);
        }
    }
    uint32_t lk = 0u;
    int lbe = 0x7fffffff, lbsl = 0;
    float lbs = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i)
        if (key[i] > lk) {
            lk = key[i];
            lbe = lane + 32 * i;
            lbs = sc[i];
            lbsl = sl[i];
        }
    int my_e = -1, my_slot = 0;
    float my_s = 0.0f;
#pragma unroll 1
    for (int j = 0; j < k; ++j) {
        const uint32_t mk = __reduce_max_sync(0xffffffffu, lk);
        const int be = static_cast<int>(__reduce_min_sync(0xffffffffu, lk == mk ? static_cast<uint32_t>(lbe) : 0xffffffffu));
        const float ws = __shfl_sync(0xffffffffu, lbs, be & 31);
        const int wsl = __shfl_sync(0xffffffffu, lbsl, be & 31);
        if (lane == j) {
            my_e = be;
            my_s = ws;
            my_slot = wsl;
        }
        if (lbe == be) {  // the winner drops it and rescans
            lk = 0u;
            lbe = 0x7fffffff;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (lane + 32 * i == be) key[i] = 0u;
                if (key[i] > lk) {
                    lk = key[i];
                    lbe = lane + 32 * i;
                    lbs = sc[i];
                    lbsl = sl[i];
                }
            }
        }
    }
    float ssum = 0.0f;  // fp32, in selection order
    int pos = 0;        // rank of this lane's expert id among the winners
#pragma unroll 1
    for (int j = 0; j < k; ++j) {
        ssum += __shfl_sync(0xffffffffu, my_s, j);
        pos += __shfl_sync(0xffffffffu, my_e, j) < my_e;
    }
    TopkRegs r;
    r.e = my_e;
    r.pos = -1;
    r.slot = 0;
    r.w = 0.0f;
    if (lane >= k) return r;
    float wv = a.tk_norm ? my_s / (ssum + 1e-20f) : my_s;
    wv *= a.tk_scaling;
    int slot = 0;
    if (my_e < 0 || my_e >= E) {
        set_error(a.err, -3);
    } else {
        slot = my_slot;
        if (slot < 0 || slot >= a.n_slots) {
            set_error(a.err, -3);
            slot = 0;
        }
    }
    r.pos = pos;
    r.slot = slot;
    r.w = wv;
    if (write && blockIdx.x == 0 && threadIdx.x < 32) {
        a.tk_idx[lane] = my_e;
        a.tk_w[lane] = wv;
        if (a.tk_idx_user) a.tk_idx_user[lane] = my_e;
        if (a.tk_w_user) a.tk_w_user[lane] = wv;
        a.tk_sorted[pos] = lane;
        Chunk ch;
        ch.slot = slot;
        ch.route_start = pos;
        ch.ntok = 1;
        ch.expert = my_e;
        a.tk_chunks[pos] = ch;
        if (lane == 0) *a.tk_nchunks = k;
    }
    return r;
}

// ------------------------------------------------------------ stream GEMV (lmoe_stream.cu)
// SMODE_GATEUP: units of gate + up tile pairs, clamped SwiGLU into the down
// panel.  SMODE_PAIR: units of one projection's tile pair, y * w per route,
// optional block-local combine.
enum StreamMode { SMODE_GATEUP = 0, SMODE_PAIR = 1 };
constexpr int kStrMaxWarps = 8;  // consumer warps per block (each feeds itself)
constexpr int kStrStages = 4;    // ring stages per warp
struct StreamCfg {
    int32_t nm, nc, ns, stage_bytes;
    int32_t TB, RB, SB, sb_l2, fm_c, fm_s;
    int32_t CK, nck, pairs;
    int64_t blk;
    int32_t ntok_cap;
    // activation rows resident in shared memory for the whole launch: the
    // first prow panel rows (res_x bytes) and their 16-column sums (res_s)
    int32_t prow, res_x, res_s;
    // work split: the kp warps of a group share each unit's K range (spp
    // rounds each, partial sums reduced through shared memory); ng groups
    // per block (nc = kp * ng warps)
    int32_t kp, ng, spp, max_chunks;
    int32_t off_ptab, off_part, off_res, off_stage, smem;
    int32_t local;  // 1: the block owns pairs blockIdx.x + i * gridDim.x (block-local combine)
    int32_t grid;   // grid of a local launch
};
// prow: panel rows the launch may read (tokens for gate/up, routes for the
// paired projections); false when the geometry or the resident rows do not fit
bool stream_config(int smode, int rows, int K, int bits, int gs, bool local, int ntok_cap, int prow,
                   StreamCfg *out);
cudaError_t launch_stream(int smode, int act_f16, int bits, int gs, const GemvArgs &a, const StreamCfg &c,
                          int max_chunks, cudaStream_t st);
cudaError_t launch_stream_pack(const QView &q, int bits, int gs, int slot_begin, int slot_count, uint8_t *out,
                               cudaStream_t st);

// Launch with programmatic stream serialisation (see pdl_wait).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ------------------------------------------------------------ int8 activation pieces
// A group of gs activations as two int8 pieces for the integer MMA of the
// single-token layer (lmoe_vec.cu): with a power-of-two scale 2^S such that
// max |x| * 2^S < 2^14, x * 2^S is an integer for every element within 2^6 of
// the group's largest magnitude, and it splits exactly into hi * 256 + lo
// (hi in [-64, 64], lo in [-128, 127]).  Stored in the B-operand order of
// the consumer's code bit width, with the group's fp32 sum and the factor
// 2^-(S + 8 - bits) that turns the MMA's integer sum back into sum(x * q).
// Byte offset, inside one group's 2 * GS piece bytes, of element e's piece
// pc for a consumer with BITS-bit codes.  MMA j of the group (word pair
// j / NC, code class j % NC) reads 16 bytes: [piece 0: word 2wp, word 2wp+1]
// [piece 1: ...], four int8 per word in byte order (byte i of a code word
// holds codes i * NC .. i * NC + NC - 1 of it, class p being code i * NC + p).
template <int BITS>
__device__ __forceinline__ int piece_offset(int e, int pc) {
    constexpr int nc = 8 / BITS, cpw = 32 / BITS;
    const int w = e / cpw, rem = e % cpw;
    const int i = rem / nc, p = rem % nc;
    const int j = (w >> 1) * nc + p;
    return ((j * 2 + pc) * 2 + (w & 1)) * 4 + i;
}

// 2^e as a float, e in [-149, 127]
__device__ __forceinline__ float exp2i(int e) {
    if (e >= -126) return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
    return __uint_as_float(1u << (e + 149));
}

// One warp converts one group of GS activations (16-bit, src) into its int8
// pieces (dst, 2 * GS bytes) and (sum of x in fp32, 2^-(S + 8 - BITS)) -> xs
// (the factor also undoes the class fold).  Fixed-order sums: the result
// repeats bit for bit.
template <typename TA, int BITS, int GS>
__device__ __forceinline__ void convert_group(const uint16_t *src, uint8_t *dst, float2 *xs, bool from_global) {
    constexpr int PER = GS / 32;  // elements per lane
    const int lane = threadIdx.x & 31;
    float v[PER];
    float amax = 0.0f, sum = 0.0f;
#pragma unroll
    for (int q = 0; q < PER; ++q) {
        const int e = lane + 32 * q;
        const uint16_t raw = from_global ? __ldcg(reinterpret_cast<const unsigned short *>(src + e)) : src[e];
        v[q] = Act<TA>::to_f(raw);
        amax = fmaxf(amax, fabsf(v[q]));
        sum += v[q];
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    int S = 0;
    if (amax > 0.0f) {
        const int E = static_cast<int>((__float_as_uint(amax) >> 23) & 0xffu) - 127;  // amax in [2^E, 2^(E+1))
        S = min(13 - E, 126);
    }
    const float scale = __uint_as_float(static_cast<uint32_t>(S + 127) << 23);
#pragma unroll
    for (int q = 0; q < PER; ++q) {
        const int e = lane + 32 * q;
        const int xi = __float2int_rn(v[q] * scale);  // |xi| <= 2^14
        const int hi = (xi + 128) >> 8;                // [-64, 64]
        const int lo = xi - (hi << 8);                 // [-128, 127]
        dst[piece_offset<BITS>(e, 0)] = static_cast<uint8_t>(hi & 0xff);
        dst[piece_offset<BITS>(e, 1)] = static_cast<uint8_t>(lo & 0xff);
    }
    if (lane == 0) *xs = make_float2(sum, exp2i(-(S + 8 - BITS)));
}

// The same for a consumer whose bit width and group size are known at run time.
template <typename TA>
__device__ __forceinline__ void convert_group_rt(int bits, int gs, const uint16_t *src, uint8_t *dst, float2 *xs,
                                                 bool from_global) {
#define LMOE_CG(B, Gs) \
    if (bits == B && gs == Gs) return convert_group<TA, B, Gs>(src, dst, xs, from_global);
    LMOE_CG(2, 32)
    LMOE_CG(2, 64)
    LMOE_CG(2, 128)
    LMOE_CG(4, 32)
    LMOE_CG(4, 64)
    LMOE_CG(4, 128)
    LMOE_CG(8, 32)
    LMOE_CG(8, 64)
    LMOE_CG(8, 128)
#undef LMOE_CG
}

// ------------------------------------------------------------ single-token layer (lmoe_vec.cu)
// Decode of one token over the stream format on the integer tensor pipe, in
// one persistent launch: gate/up + SwiGLU, then down + combine.  Every chunk
// of the dispatch holds one route.  Work items are (sub-unit, K chunk) pairs
// dealt out in contiguous ranges to all warps of the grid; a sub-unit's
// partial sums meet in global scratch and the last share to arrive runs its
// epilogue.  The down projection's weights stream in while gate/up still
// computes; a grid-wide counter of converted h groups (bounded wait) starts
// the down products.
constexpr int kVecWarps = 8;      // warps per block, each with its own copy ring
constexpr int kVecBlockWarps = kVecWarps + 1;  // and one warp that finishes the gate/up units
constexpr int kVecMaxStages = 8;  // ring sub-slots per warp
struct VecPhase {                  // geometry of one projection's stream format
    int32_t nck, pairs, RB, fm_c, tS, tB, TB, ngroups;
    int64_t blk;
};
struct VecArgs {
    QView q0, q1, q2;  // stream-format tiles of gate, up and down
    // the natural activation row [K] (the layer's single token), and its int8
    // pieces [groups][2 gs] and (sum, factor) per group: written by the
    // router (x_ready) or converted here from x
    const uint16_t *x;
    const uint8_t *xq;
    const float2 *xs;
    int32_t x_ready;
    // dispatch of one token: chunk i holds the single route sorted_routes[i]
    const Chunk *chunks;
    const int32_t *n_chunks;
    const int32_t *sorted_routes;
    int32_t n_slots, max_chunks;
    int32_t routes;       // route rows R (top_k, + 1 with the shared expert)
    int32_t shared_base;  // > 0: route shared_base is the shared expert's (reads x)
    // single token: routing selected from the router's (score, biased score)
    // inside the kernel (block_topk); tk_scores == nullptr: chunks from memory
    const float2 *tk_scores;
    int32_t tk_E, tk_k, tk_norm;
    float tk_scaling;
    const int32_t *tk_expert_slot;
    int32_t *tk_idx, *tk_idx_user, *tk_sorted, *tk_nchunks;
    float *tk_w, *tk_w_user;
    Chunk *tk_chunks;
    // h's int8 pieces [R][groups][2 gs] and (sum, factor) per 32-row
    // segment [R][inter / 32]
    uint8_t *hq;
    float2 *hs;
    float limit;
    int32_t swiglu_mode;
    // route weights (nullptr: unit weights), residual (or nullptr), combined
    // output row (or nullptr) and per-route rows T(T(y) * T(w)) [R][hidden]
    // of the computed routes (or nullptr)
    const float *route_w;
    int32_t top_k;
    const uint16_t *residual;
    uint16_t *out;
    uint16_t *yw;
    uint32_t *hready;  // [R][down K chunks]: gate/up units finished (zero at the start of the call)
    int32_t *err;
};
struct VecCfg {
    VecPhase ga, dn;  // gate/up (two tiles of gate, two of up per stage) and down
    int32_t routes;   // h rows resident in the down phase
    int32_t sub, nq, qa, qb, warps;  // ring: nq sub-slots of sub bytes per warp; qa / qb per item
    int32_t off_bar, off_flag, off_xbar, off_zero, off_rch, off_tk, off_xq, off_xs, off_hq, off_pa, off_pb, off_ring,
        smem;
    int32_t grid;
};
// geometry check and shared-memory plan; false when the kernel cannot run it
bool vec_layer_config(int hidden, int inter, int bits_g, int gs_g, int bits_d, int gs_d, int routes, VecCfg *out);
cudaError_t launch_vec_layer(int act_f16, int bits_g, int bits_d, int gs, const VecArgs &a, const VecCfg &c,
                             cudaStream_t st);


// host-side launchers (lmoe_route.cu, lmoe_gemv.cu)
cudaError_t launch_router(const RouterArgs &a, int ksplit, cudaStream_t st);
cudaError_t launch_topk(const TopkArgs &a, cudaStream_t st);
// logits (+ element-wise scores) of many bf16 tokens on the tensor cores; the
// top-k then runs in launch_topk
cudaError_t launch_router_logits_mma(const RouterArgs &a, cudaStream_t st);
cudaError_t launch_dispatch_small(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                                  cudaStream_t st);
cudaError_t launch_dispatch_large(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                                  cudaStream_t st);
cudaError_t launch_panel(const PanelArgs &a, cudaStream_t st);
// returns cudaErrorInvalidValue for an unsupported (bits, gs)
cudaError_t launch_gemv(int mode, int act_f16, int bits, int gs, const GemvArgs &a,
                        int max_chunks, cudaStream_t st);
// host rows (device-mapped pointer) -> device buffer; bytes a multiple of 16
cudaError_t launch_stage_rows(void *dst, const void *src, size_t bytes, cudaStream_t st);
// blocks of a MODE_DOWN2 launch over `pairs` row pairs (0: use MODE_DOWN)
int down2_grid(int pairs);
// MODE_DOWN2 serves layers of at most this many tokens (the decode path's
// range under AUTO at 256 experts, top-6)
constexpr int kDown2MaxTokens = 64;
// row-major slots [slot_begin, slot_begin + slot_count) of q -> tiles
cudaError_t launch_tile_pack(const QView &q, int bits, int gs, int slot_begin, int slot_count, uint8_t *tiles,
                             cudaStream_t st);

// ------------------------------------------------------------ prefill grouped GEMM
// (lmoe_prefill.cu).  Routes are grouped by expert into chunks of at most
// kPfNmax (the MMA N); each chunk owns a block of panel rows starting at
// pf_row_base, 16-aligned and at least round_up(ntok, 16) long.
constexpr int kPfNmax = 128;
enum PfMode { PF_GATEUP = 0, PF_DOWN = 1 };

__host__ __device__ inline int pf_row_base(int route_start, int chunk) {
    return ((route_start + 15) & ~15) + 16 * chunk;
}
// panel rows needed for R routes in at most n_chunks chunks
inline int pf_panel_rows(int R, int n_chunks) { return ((R + 15) & ~15) + 16 * n_chunks + 16; }
// chunks of at most kPfNmax routes over `buckets` experts (+ zero bucket)
inline int pf_max_chunks(int buckets, int R) {
    const int distinct = buckets < R ? buckets : R;
    return distinct + R / kPfNmax + 1;
}

// Activation panel of the prefill kernels: [K/64][rows/8][1024 bytes].  Each
// 1024-byte block holds 8 rows x 64 columns in the 128-byte-swizzled K-major
// layout of the tensor core's shared-memory operands (16-byte chunk j of row
// r at chunk position j ^ (r & 7)), with the in-word pair permutation of the
// consuming projection's bit width (pf_perm_pos).
struct PfPanelArgs {
    const uint16_t *x;  // [rows of x, K]
    int32_t K;
    int32_t x_stride;   // elements between rows of x (0: K)
    int32_t shared_base;  // routes >= shared_base (> 0) read row route - shared_base
    int32_t route_div;  // route r reads x row r / route_div
    const Chunk *chunks;
    const int32_t *n_chunks;
    const int32_t *sorted_routes;
    uint8_t *panel;
    int32_t prow;  // panel rows
    int32_t bits;  // bit width of the projection that consumes the panel
};

struct PfArgs {
    // 2-D TMA maps over the arena arrays of the item's two 128-row blocks
    // (gate and up for PF_GATEUP; the down array twice for PF_DOWN): codes
    // [n_slots * rows][row bytes] (uint8), scales and biases
    // [n_slots * rows][groups] (16-bit)
    CUtensorMap tm_code[2];
    CUtensorMap tm_scale[2];
    CUtensorMap tm_bias[2];
    int32_t wrows;          // rows of the projection array (per slot)
    const uint8_t *panel;   // activation panel of this kernel
    int32_t prow;
    int32_t K;
    const Chunk *chunks;
    const int32_t *n_chunks;
    const int32_t *sorted_routes;
    int32_t rbn;            // work items per chunk (row-block pairs)
    // PF_GATEUP: h into the down kernel's panel
    uint8_t *hpanel;
    int32_t hprow;
    int32_t hbits;
    float limit;
    int32_t swiglu_mode;
    // PF_DOWN: bf16(y) * bf16(w) rows [R, H]
    uint16_t *yw;
    int32_t H;
    const float *route_w;
    int32_t *err;
};

// Fills a.tm_* for the projection(s) of `mode` (q1 = up for PF_GATEUP).
cudaError_t pf_prepare(PfArgs &a, int mode, const QView &q0, const QView &q1, int bits, int gs, int n_slots);
bool pf_supported(int K, int rows, int bits, int gs, int mode);
cudaError_t launch_pf_panel(const PfPanelArgs &a, int max_chunks, cudaStream_t st);
cudaError_t launch_pf_gemm(int mode, int act_f16, int bits, int gs, const PfArgs &a, cudaStream_t st);
cudaError_t launch_pf_combine(int act_f16, const uint16_t *yw, int T, int H, int top_k, uint16_t *out,
                              cudaStream_t st, int shared_base = 0, const uint16_t *residual = nullptr);
// appends the shared expert's chunks (routes R .. R + T - 1, weight 1, arena
// slot `slot`) after the dispatched chunks (lmoe_route.cu)
cudaError_t launch_shared_chunks(Chunk *chunks, int32_t *n_chunks, int32_t *sorted_routes, float *route_w, int R,
                                 int T, int chunk_tok, int slot, cudaStream_t st);

// Activation row of a route: routed routes r read row r / route_div; the
// shared expert's routes (r >= shared_base > 0) read row r - shared_base.
__host__ __device__ inline int route_row(int r, int route_div, int shared_base) {
    return (shared_base > 0 && r >= shared_base) ? r - shared_base : r / route_div;
}
// Final value of one output element: routed fp32 sum rounded once; with the
// shared expert's row the sum is rounded again after adding it; with a
// residual, once more after adding that (dsv4_engine.py:259, routed +
// shared_experts(x), then the decoder layer's residual add).
template <typename TA>
__device__ __forceinline__ float combine_finish(float routed, bool has_shared, uint16_t shared_v, bool has_res,
                                                uint16_t res_v) {
    float o = Act<TA>::round(routed);
    if (has_shared) o = Act<TA>::round(o + Act<TA>::to_f(shared_v));
    if (has_res) o = Act<TA>::round(Act<TA>::to_f(res_v) + o);
    return o;
}

// ------------------------------------------------------------ expert parallel (lmoe_ep.cu)
constexpr int kEpMaxWorld = 32;
// trailer of one exchanged row: int32 ids[k], fp32 w[k], int32 token, zero
// padding to a multiple of 16 bytes
__host__ __device__ inline int ep_trailer_bytes(int k) { return (8 * k + 4 + 15) / 16 * 16; }
__host__ __device__ inline int ep_row_bytes(int H, int k) { return 2 * H + ep_trailer_bytes(k); }

struct EpDispatchArgs {
    const int32_t *idx;  // [T, k] global expert ids
    const float *w;      // [T, k] combine weights
    const uint16_t *x;   // [T, H] activations
    int32_t T, k, H, E, world;
    uint8_t *send;     // [world][T][ep_row_bytes]
    int32_t *slot_of;  // [T][world]: slot of token t in destination d's rows, -1 if none
    int32_t *err;
};
cudaError_t launch_ep_dispatch(const EpDispatchArgs &a, cudaStream_t st);
// out[t] = T(sum_i y[t*k + order_i] * w[...]) in fp32 (lmoe_combine_routes)
cudaError_t launch_combine_routes(int act_f16, const uint16_t *y, const float *w, const int32_t *order, int T, int k,
                                  int H, uint16_t *out, cudaStream_t st);
cudaError_t launch_ep_unpack(const uint8_t *recv, int rows, int H, int k, int32_t *idx, float *w, cudaStream_t st);
cudaError_t launch_ep_partial(int act_f16, const uint16_t *yw, const int32_t *idx, int rows, int H, int k,
                              int n_local, float *partial, cudaStream_t st);
cudaError_t launch_ep_combine(int act_f16, const float *back, int T, int world, int H, const int32_t *slot_of,
                              const uint16_t *residual, uint16_t *out, uint16_t *normed, float eps,
                              cudaStream_t st);

constexpr int kDispatchSmallMaxRoutes = 512;
constexpr int kDispatchSmallMaxBuckets = 1024;
constexpr int kRouterKS = 256;      // K columns per router CTA
constexpr int kRouterMaxEPL = 16;   // experts per lane in top-k (E <= 512)

}  // namespace lmoe
