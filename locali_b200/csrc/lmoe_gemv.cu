// Expert products for sm_100a: a warp-specialised, TMA-fed dequant GEMV.
//
// One unit = (chunk of <= chunk_tok routes of one expert, 16-row tile of a
// projection; gate and up together for MODE_GATEUP).  Per block:
//   * a producer warp streams each unit's codes, scales, biases and the
//     routes' activation panel + 16-column sums from HBM/L2 into a ring of
//     shared-memory stages with plain (non-multicast) cp.async.bulk copies
//     completing on mbarriers -- every code byte crosses HBM once and several
//     units are in flight per SM without holding registers;
//   * consumer warps split each unit's K range, unpack codes to exact small
//     integers in registers, run mma.m16n8k16 (fp32 accumulate) per
//     quantisation group and apply acc += scale*dot + bias*sum(x)
//     (dsv4_kernels.py:152-154), then hand their partial sums over;
//   * an epilogue warp reduces the partials in a fixed order and finishes the
//     unit: clamped SwiGLU into the down projection's panel (dsv4_arena.py:
//     223-235), or y*w for the weighted combine (arena.py:543,619-624), or the
//     plain gather_qmm output.  The combine of a token's k routes is done by
//     whichever block completes the token's last route, after one batched
//     memory fence per block (deterministic route-order fp32 sum).
// All waits are bounded in time; a wait that gives up records an error and the
// block stops instead of hanging.
#include <cstring>

#include "lmoe_kernels.cuh"

namespace lmoe {

#define LMOE_FULL 0xffffffffu

__device__ __forceinline__ uint32_t lds_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
    return v;
}
__device__ __forceinline__ uint2 lds_u64(const void *p) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
    return v;
}
__device__ __forceinline__ uint4 lds_u128(const void *p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}
// predicated 16-byte shared load: v keeps its value where pred is false
__device__ __forceinline__ void lds_u128_if(uint4 &v, const void *p, bool pred) {
    asm volatile(
        "{ .reg .pred q; setp.ne.b32 q, %5, 0; @q ld.shared.v4.u32 {%0,%1,%2,%3}, [%4]; }"
        : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w)
        : "r"(smem_u32(p)), "r"(static_cast<int>(pred)));
}
__device__ __forceinline__ uint16_t lds_u16(const void *p) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(smem_u32(p)));
    return v;
}

template <int WPS>
__device__ __forceinline__ void lds_slice(const uint8_t *p, uint32_t (&w)[WPS]) {
    if constexpr (WPS == 1) {
        w[0] = lds_u32(p);
    } else if constexpr (WPS == 2) {
        const uint2 v = lds_u64(p);
        w[0] = v.x;
        w[1] = v.y;
    } else {
#pragma unroll
        for (int q = 0; q < WPS / 4; ++q) {
            const uint4 v = lds_u128(p + 16 * q);
            w[4 * q] = v.x;
            w[4 * q + 1] = v.y;
            w[4 * q + 2] = v.z;
            w[4 * q + 3] = v.w;
        }
    }
}

__device__ __forceinline__ bool aborted(volatile int *flag) { return *flag != 0; }

// Swizzle factor of a code row: the 16-byte chunks of row r are XOR-ed with
// r & 7, so the 8 rows a warp reads at once (both consumer access patterns,
// every lane-slice width) land in distinct 16-byte bank groups.
template <int WPS>
__device__ __forceinline__ int code_xor(int row) {
    return row & 7;
}

// Profiling builds (-DLMOE_PROFILE_TRACE) record one globaltimer stamp per
// (block, unit, point); the default build compiles these calls away.
__device__ __forceinline__ void trace_point(const GemvArgs &a, int it, int point) {
#ifdef LMOE_PROFILE_TRACE
    if (a.trace && it < a.trace_units && (threadIdx.x & 31) == 0)
        a.trace[((size_t)blockIdx.x * a.trace_units + it) * 8 + point] = globaltimer_ns();
#else
    (void)a, (void)it, (void)point;
#endif
}

template <typename TA, int BITS, int GS, int MODE>
__global__ void __launch_bounds__(kGemvMaxThreads, 1) gemv_kernel(const GemvArgs a, const GemvCfg c) {
    using Gm = Geo<BITS, GS>;
    // MODE_DOWN2: a unit is two adjacent row tiles of one projection, held
    // as the two matrices of the paired layout
    constexpr bool PAIRT = (MODE == MODE_DOWN2);
    constexpr bool PAIR = (MODE == MODE_GATEUP) || PAIRT;
    constexpr int NM = PAIR ? 2 : 1;
    constexpr int NROW = 2 * NM;
    constexpr int WPS = Gm::kWps;
    constexpr int NP = Gm::kCpw / 2;
    constexpr int SPW = Gm::kStepsPerWord;
    constexpr int S = Gm::kSteps;
    constexpr int WPG = Gm::kWordsPerGroup;

    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + c.off_bars);
    uint64_t *empty = full + c.nst;
    uint64_t *rfull = empty + c.nst;
    uint64_t *rempty = rfull + kGemvEpi;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(rempty + kGemvEpi);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int K = a.q0.cols;
    const int rows = a.q0.rows;
    const int RT = rows >> 4;
    const int UT = PAIRT ? RT / 2 : RT;  // row positions of a chunk's units
    const int GT = K / GS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < c.nst; ++s) {
            // 64 cp.async arrivals (one per producer lane) + the bulk-copy arrive
            mbar_init(&full[s], 65);
            mbar_init(&empty[s], c.ncw);
            // no activation rows staged yet
            reinterpret_cast<int *>(smem + c.off_shdr + s * kHdrBytes)[kHdrPanelN] = -1;
        }
        for (int b = 0; b < kGemvEpi; ++b) {
            mbar_init(&rfull[b], c.ncw);
            mbar_init(&rempty[b], 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // panel position (low 8 bits) and 2-bit prescale exponent (bits 8-9) of
    // each row offset inside one output group (gate/up epilogue)
    uint16_t *ptab = reinterpret_cast<uint16_t *>(smem + c.off_ptab);
    if (MODE == MODE_GATEUP && a.out_panel) {
        for (int i = threadIdx.x; i < a.out_gs; i += blockDim.x) {
            int p;
            const int pos = panel_pos(i, a.out_bits, a.out_gs, &p);
            ptab[i] = static_cast<uint16_t>(pos | (p << 8));
        }
    }
    __syncthreads();
    // MODE_DOWN2 with pre-tiled weights: the chunk table was written by the
    // router, two launches back (the gate/up kernel, which precedes this one,
    // allowed this launch only after its own wait on the router), and the
    // weight tiles are static.  So the producer requests the weight tiles of
    // its first stages before waiting on the gate/up kernel, whose output
    // (the activation rows) is copied only after the wait.
    int npre = 0;
    if constexpr (MODE == MODE_DOWN2) {
        if (warp == c.ncw && a.q0.tiles) {
            const int u = static_cast<int>(blockIdx.x) + lane * static_cast<int>(gridDim.x);
            const bool pre = lane < c.nst && u < *a.n_chunks * UT;
            if (pre) {
                int slot = a.chunks[u / UT].slot;
                if (slot < 0 || slot >= a.n_slots) {
                    set_error(a.err, -3);
                    slot = 0;
                }
                const int rt = u % UT;
                uint8_t *sb = smem + c.off_stage + (size_t)lane * c.stage_bytes;
                const uint8_t *src = a.q0.tiles + (size_t)slot * a.q0.tile_slot_stride + (size_t)(2 * rt) * c.TBp;
                mbar_add_tx(&full[lane], static_cast<uint32_t>(2 * c.TBp));
                const uint64_t pol = evict_first_policy();
                bulk_g2s_hint(sb + c.off_codes, src, static_cast<uint32_t>(c.TBp), &full[lane], pol);
                bulk_g2s_hint(sb + c.off_codes + c.TBp, src + c.TBp, static_cast<uint32_t>(c.TBp), &full[lane], pol);
            }
            npre = __popc(__ballot_sync(LMOE_FULL, pre));
        }
    }
    // the chunk table and activations come from the preceding kernels
    pdl_wait();
    pdl_trigger();
    const int nch = *a.n_chunks;
    const int units = nch * UT;

    if (warp == c.ncw || warp == c.ncw + 1) {
        // ===================================================== producers
        // Two warps (on different schedulers) share each stage's copies:
        // warp 0 of the pair also issues the header and the bulk activation
        // copies; code chunks alternate between the warps, warp 0 copies the
        // scales and warp 1 the biases.
        const int pw = warp - c.ncw;
        const uint64_t pol = evict_first_policy();
        // unit metadata is fetched 32 units ahead: lane j holds the chunk and
        // routes of unit it + j, so the per-unit issue path has no dependent
        // global loads
        int m_slot = 0, m_ntok = 0;
        int m_route[8];
        float m_w[8];
        int it = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
            if ((it & 31) == 0) {
                const int uj = u + lane * static_cast<int>(gridDim.x);
                m_slot = 0;
                m_ntok = 0;
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    m_route[n] = -1;
                    m_w[n] = 0.0f;
                }
                if (uj < units) {
                    const Chunk chj = a.chunks[uj / UT];
                    m_slot = chj.slot;
                    if (m_slot < 0 || m_slot >= a.n_slots) {
                        set_error(a.err, -3);
                        m_slot = 0;
                    }
                    m_ntok = chj.ntok;
                    if (m_ntok < 0 || m_ntok > a.ntok_max) {
                        set_error(a.err, -3);
                        m_ntok = m_ntok < 0 ? 0 : a.ntok_max;
                    }
#pragma unroll
                    for (int n = 0; n < 8; ++n)
                        if (n < m_ntok) m_route[n] = a.sorted_routes[chj.route_start + n];
                    if (a.route_w) {
#pragma unroll
                        for (int n = 0; n < 8; ++n)
                            if (n < m_ntok) m_w[n] = a.route_w[m_route[n]];
                    }
                }
            }
            const int st = it % c.nst;
            const uint32_t ph = (it / c.nst) & 1;
            if (!mbar_wait(&empty[st], ph ^ 1u) || aborted(abort_flag)) {
                if (lane == 0) {
                    *abort_flag = 1;
                    set_error(a.err, -4);
                }
                break;
            }
            const int rt = u % UT;  // units run row-tile fastest: a block's consecutive units share a chunk
            if (pw == 0) trace_point(a, it, 0);
            const int src = it & 31;
            const int slot = __shfl_sync(LMOE_FULL, m_slot, src);
            uint8_t *sb = smem + c.off_stage + (size_t)st * c.stage_bytes;
            const bool tiled0 = a.q0.tiles != nullptr;
            const bool tiled1 = NM > 1 && a.q1.tiles != nullptr;
            // Pre-tiled weight tiles go first: they need only the slot, and
            // they are most of the stage's bytes.  Their bytes are added to
            // the stage's transaction count without an arrival, so the stage
            // cannot complete before the header and activation rows below.
            // The proxy fence orders the consumers' reads of this slot's last
            // unit (observed through the empty barrier) before the copies.
            const uint32_t tile_bytes = static_cast<uint32_t>(((tiled0 ? 1 : 0) + (tiled1 ? 1 : 0)) * c.TBp);
            if (pw == 0 && tile_bytes && it >= npre) {  // stages below npre: requested before the wait
                if (lane == 0) {
                    fence_proxy_async();
                    mbar_add_tx(&full[st], tile_bytes);
                }
                __syncwarp();
                if (lane == 8 && tiled0)
                    bulk_g2s_hint(sb + c.off_codes,
                                  a.q0.tiles + (size_t)slot * a.q0.tile_slot_stride +
                                      (size_t)(PAIRT ? 2 * rt : rt) * c.TBp,
                                  static_cast<uint32_t>(c.TBp), &full[st], pol);
                if (lane == 9 && tiled1)
                    bulk_g2s_hint(sb + c.off_codes + c.TBp,
                                  a.q1.tiles + (size_t)slot * a.q1.tile_slot_stride +
                                      (size_t)(PAIRT ? 2 * rt + 1 : rt) * c.TBp,
                                  static_cast<uint32_t>(c.TBp), &full[st], pol);
            }
            const int ntok = __shfl_sync(LMOE_FULL, m_ntok, src);
            int rr[8];
            float ww[8];
            int route = -1;
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                rr[n] = __shfl_sync(LMOE_FULL, m_route[n], src);
                ww[n] = __shfl_sync(LMOE_FULL, m_w[n], src);
                if (lane == n) route = rr[n];
            }
            int *hdr = reinterpret_cast<int *>(smem + c.off_shdr + st * kHdrBytes);
            // Bulk (TMA) copies for the per-route activation rows (two per
            // route); projections in the plain row-major layout go through
            // 16-byte cp.async, swizzled into the tile layout on the way.
            // The activation rows already in this stage (from its previous
            // unit) are reused when the new unit needs the same rows in the
            // same order: in decode every unit of a chunk reads one row.
            // gate/up reads token rows (the shared expert's routes map to their
            // token); down reads the h row of each route
            const int prow = route < 0 ? -1
                             : (MODE == MODE_GATEUP ? route_row(route, a.route_div, a.shared_base)
                                                    : route / a.route_div);
            bool reuse = false;
            if (pw == 0) {
                const bool same = lane >= ntok || lane >= 8 || hdr[kHdrPanel + lane] == prow;
                reuse = __all_sync(LMOE_FULL, same) && hdr[kHdrPanelN] == ntok;
            }
            const uint32_t bulk_bytes = static_cast<uint32_t>(reuse ? 0 : ntok * (c.PB + K / 2));
            if (pw == 0 && lane == 0) {
                hdr[0] = ntok;
                hdr[1] = rt;
                hdr[2] = slot;
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    hdr[kHdrRoute + n] = rr[n];
                    hdr[kHdrWeight + n] = __float_as_int(ww[n]);
                }
                hdr[kHdrPanelN] = ntok;
                fence_proxy_async();
                mbar_expect_tx(&full[st], bulk_bytes);
            }
            if (pw == 0 && lane < 8) hdr[kHdrPanel + lane] = lane < ntok ? prow : -1;
            __syncwarp();
            if (pw == 0 && lane < ntok && !reuse) {
                bulk_g2s(sb + c.off_panel + lane * c.PBp, a.panel + (size_t)prow * K, static_cast<uint32_t>(c.PB),
                         &full[st]);
                bulk_g2s(sb + c.off_sum + lane * c.S16B, a.sum16 + (size_t)prow * (K / 8), static_cast<uint32_t>(K / 2),
                         &full[st]);
            }
            if (pw == 0) trace_point(a, it, 5);
            // codes: a matrix's 16 rows are one contiguous block of the slot;
            // consecutive lanes copy consecutive 16-byte chunks (coalesced),
            // each landing at its swizzled position in the same 128-byte line
            const int n16c = 16 << c.rb_l2;
#pragma unroll 1
            for (int m = 0; m < NM; ++m) {
                const QView &q = m ? a.q1 : a.q0;
                if (q.tiles) continue;
                const uint8_t *src = reinterpret_cast<const uint8_t *>(
                    q.w + (size_t)slot * q.w_slot_stride + (size_t)((PAIRT ? 2 * rt + m : rt) * 16) * q.words_per_row);
                uint8_t *dst = sb + c.off_codes + m * c.TBp;
#pragma unroll 4
                for (int i = lane + 32 * pw; i < n16c; i += 64) {
                    const int o = i << 4, row = i >> c.rb_l2;
                    cp_async16(dst + swz(o, code_xor<WPS>(row) & c.fm_c), src + o, pol);
                }
            }
            if (pw == 0) trace_point(a, it, 7);
            // scales (warp 0) or biases (warp 1): 16 contiguous rows per matrix
            const int n16s = c.SB;  // 16 rows * SB bytes / 16
            const int kind = pw;
#pragma unroll 1
            for (int m = 0; m < NM; ++m) {
                const QView &q = m ? a.q1 : a.q0;
                if (q.tiles) continue;
                const uint8_t *src = reinterpret_cast<const uint8_t *>(
                    (kind ? q.b : q.s) + (size_t)slot * q.sb_slot_stride +
                    (size_t)((PAIRT ? 2 * rt + m : rt) * 16) * q.groups_per_row);
                uint8_t *dst = sb + (kind ? c.off_b : c.off_s) + m * c.TBp;
                for (int i = lane; i < n16s; i += 32) {
                    const int o = i << 4;
                    const int f = c.sb_l2 >= 0 ? ((i >> c.sb_l2) & c.fm_s) : 0;
                    cp_async16(dst + swz(o, f), src + o, pol);
                }
            }
            cp_async_arrive_noinc(&full[st]);
            if (pw == 0) trace_point(a, it, 1);
        }
        if (aborted(abort_flag)) {
            // drain: let copies already issued (in the loop, or before the
            // wait on the preceding kernel) land before the block exits
            const int issued = it > npre ? it : npre;
            for (int j = (issued > c.nst ? issued - c.nst : 0); j < issued; ++j)
                mbar_wait(&full[j % c.nst], (j / c.nst) & 1);
        }
        return;
    }

    if (warp >= c.ncw + 2) {
        // ===================================================== epilogue
        // kGemvEpi warps take the units round robin (unit it -> warp it %
        // kGemvEpi, reduction buffer it % kGemvEpi): one warp alone cannot
        // keep up with the consumers on its chain of dependent steps.
        const int ew = warp - (c.ncw + 2);
        int *list = reinterpret_cast<int *>(smem + c.off_list) + ew * c.list_cap;
        int list_n = 0;
        const int out_lg = (MODE == MODE_GATEUP && a.out_panel) ? __ffs(a.out_gs) - 1 : 0;
        auto flush = [&]() {
            // one fence covers every y*w row this block wrote since the last flush
            __threadfence();
            for (int base = 0; base < list_n; base += 32) {
                const int i = base + lane;
                int done_key = -1;
                if (i < list_n) {
                    const int key = list[i];
                    const unsigned prev = atomicAdd(a.counters + key, 1u);
                    // the token's routed rows, plus its shared-expert row when present
                    if (prev == static_cast<unsigned>(a.top_k - (a.shared_base > 0 ? 0 : 1))) done_key = key;
                }
                unsigned m = __ballot_sync(LMOE_FULL, done_key >= 0);
                while (m) {
                    const int src = __ffs(m) - 1;
                    m &= m - 1;
                    const int key = __shfl_sync(LMOE_FULL, done_key, src);
                    const int tok = key / RT, rt = key - tok * RT;
                    __threadfence();
                    if (lane < 16) {
                        const int row = rt * 16 + lane;
                        float sacc = 0.0f;
                        for (int j = 0; j < a.top_k; ++j) {
                            const uint16_t v = __ldcg(reinterpret_cast<const unsigned short *>(
                                a.out + ((size_t)tok * a.top_k + j) * rows + row));
                            sacc += Act<TA>::to_f(v);
                        }
                        const bool sh = a.shared_base > 0;
                        const uint16_t sv = sh ? __ldcg(reinterpret_cast<const unsigned short *>(
                                                     a.out + ((size_t)a.shared_base + tok) * rows + row))
                                               : 0;
                        const uint16_t rv = a.residual ? a.residual[(size_t)tok * rows + row] : 0;
                        a.combined[(size_t)tok * rows + row] =
                            Act<TA>::from_f(combine_finish<TA>(sacc, sh, sv, a.residual != nullptr, rv));
                    }
                    if (lane == 0) a.counters[key] = 0u;
                }
            }
            list_n = 0;
            __syncwarp();
        };
        for (int u = blockIdx.x + ew * gridDim.x, it = ew; u < units; u += kGemvEpi * gridDim.x, it += kGemvEpi) {
            const int rb = ew;
            const uint32_t rph = (it / kGemvEpi) & 1;
            const bool got = mbar_wait(&rfull[rb], rph);
            trace_point(a, it, 4);
            if (!got || aborted(abort_flag)) {
                if (lane == 0) {
                    *abort_flag = 1;
                    set_error(a.err, -4);
                }
                break;
            }
            const int *rh = reinterpret_cast<const int *>(smem + c.off_rhdr + rb * kHdrBytes);
            const int ntok = rh[0], rt = rh[1];
            int rr[8];
            float rw[8];
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                rr[n] = rh[kHdrRoute + n];
                rw[n] = __int_as_float(rh[kHdrWeight + n]);
            }
            float fin[NM][4];
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
                for (int e = 0; e < 4; ++e) fin[m][e] = 0.0f;
            const float *red = reinterpret_cast<const float *>(smem + c.off_red) + (size_t)rb * c.ncw * 32 * NM * 4;
            for (int w = 0; w < c.ncw; ++w) {
                const float *p = red + (w * 32 + lane) * NM * 4;
#pragma unroll
                for (int m = 0; m < NM; ++m) {
                    const float4 v = *reinterpret_cast<const float4 *>(p + m * 4);
                    fin[m][0] += v.x;
                    fin[m][1] += v.y;
                    fin[m][2] += v.z;
                    fin[m][3] += v.w;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rempty[rb]);
            if constexpr (MODE == MODE_GATEUP) {
                float hv[4], hp[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float h = swiglu_h<TA>(fin[0][e], fin[1][e], a.limit, a.swiglu_mode);
                    const int n = 2 * t + (e & 1);
                    const int row = rt * 16 + g + 8 * (e >> 1);
                    hv[e] = 0.0f;
                    hp[e] = 0.0f;
                    if (n < ntok) {
                        int route = rr[0];
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            if (q == n) route = rr[q];
                        hv[e] = h;
                        if (a.out_panel) {
                            const int tv = ptab[row & (a.out_gs - 1)];
                            const int pos = ((row >> out_lg) << out_lg) + (tv & 0xff);
                            const int p = tv >> 8;
                            const uint16_t pv = Act<TA>::from_f(h * (p == 0 ? 1.0f : (p == 1 ? 0.25f : 0.0625f)));
                            hp[e] = Act<TA>::to_f(pv);
                            a.out[(size_t)route * rows + pos] = pv;
                        } else {
                            a.out[(size_t)route * rows + row] = Act<TA>::from_f(h);
                        }
                    }
                }
                if (a.out_sum16) {
                    float s0 = hv[0] + hv[2];
                    float s1 = hv[1] + hv[3];
                    float p0 = hp[0] + hp[2];
                    float p1 = hp[1] + hp[3];
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) {
                        s0 += __shfl_xor_sync(LMOE_FULL, s0, o);
                        s1 += __shfl_xor_sync(LMOE_FULL, s1, o);
                        p0 += __shfl_xor_sync(LMOE_FULL, p0, o);
                        p1 += __shfl_xor_sync(LMOE_FULL, p1, o);
                    }
                    if (g == 0) {
                        int r0 = rr[0], r1 = rr[0];
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            if (q == 2 * t) r0 = rr[q];
                            if (q == 2 * t + 1) r1 = rr[q];
                        }
                        if (2 * t < ntok)
                            *reinterpret_cast<float2 *>(a.out_sum16 + ((size_t)r0 * RT + rt) * 2) = make_float2(s0, p0);
                        if (2 * t + 1 < ntok)
                            *reinterpret_cast<float2 *>(a.out_sum16 + ((size_t)r1 * RT + rt) * 2) = make_float2(s1, p1);
                    }
                }
            } else if constexpr (MODE == MODE_DOWN2) {
                // y*w of both row tiles; the block sums each token's k rows
                // after its last unit (it owns every chunk of these rows)
#pragma unroll
                for (int m = 0; m < 2; ++m)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int n = 2 * t + (e & 1);
                        const int row = (2 * rt + m) * 16 + g + 8 * (e >> 1);
                        if (n < ntok) {
                            int route = rr[0];
                            float wr = rw[0];
#pragma unroll
                            for (int q = 0; q < 8; ++q)
                                if (q == n) {
                                    route = rr[q];
                                    wr = rw[q];
                                }
                            const float y = Act<TA>::round(fin[m][e]);
                            const float wv = a.route_w ? Act<TA>::round(wr) : 1.0f;  // no weights: y itself
                            a.out[(size_t)route * rows + row] = Act<TA>::from_f(y * wv);
                        }
                    }
            } else if constexpr (MODE == MODE_DOWN) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int n = 2 * t + (e & 1);
                    const int row = rt * 16 + g + 8 * (e >> 1);
                    if (n < ntok) {
                        int route = rr[0];
                        float wr = rw[0];
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            if (q == n) {
                                route = rr[q];
                                wr = rw[q];
                            }
                        const float y = Act<TA>::round(fin[0][e]);
                        const float wv = a.route_w ? Act<TA>::round(wr) : 1.0f;  // no weights: y itself
                        a.out[(size_t)route * rows + row] = Act<TA>::from_f(y * wv);
                    }
                }
                if (a.counters) {  // without counters the caller combines the y*w rows
                    if (lane < ntok) {
                        int route = rr[0];
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            if (q == lane) route = rr[q];
                        list[list_n + lane] = route_row(route, a.top_k, a.shared_base) * RT + rt;
                    }
                    list_n += ntok;
                    __syncwarp();
                    if (list_n + 8 > c.list_cap) flush();
                }
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int n = 2 * t + (e & 1);
                    const int row = rt * 16 + g + 8 * (e >> 1);
                    if (n < ntok) {
                        int route = rr[0];
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            if (q == n) route = rr[q];
                        a.out[(size_t)route * rows + row] = Act<TA>::from_f(fin[0][e]);
                    }
                }
            }
        }
        if constexpr (MODE == MODE_DOWN) {
            if (list_n > 0) flush();
        }
        if constexpr (MODE == MODE_DOWN2) {
            if (!a.combined) return;  // the caller combines the y*w rows
            // Weighted combine of the row pairs this block owns (u = chunk *
            // UT + pair with gridDim.x dividing UT, so the block ran every
            // chunk of pairs blockIdx.x + j * gridDim.x): each token's k y*w
            // rows summed in route order in fp32 and rounded once, the
            // arithmetic of the MODE_DOWN combine.  Rows written by the other
            // epilogue warps are read back from L2 after the named barrier.
            __threadfence_block();
            asm volatile("bar.sync 1, %0;" ::"r"(kGemvEpi * 32) : "memory");
            if (!aborted(abort_flag)) {
                const int own = (UT - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                                static_cast<int>(gridDim.x);
                const int items = own * 32 * a.n_tok;
                for (int i = ew * 32 + lane; i < items; i += kGemvEpi * 32) {
                    const int ri = i & 31, rest = i >> 5;
                    const int tok = rest % a.n_tok, j = rest / a.n_tok;
                    const int row = (static_cast<int>(blockIdx.x) + j * static_cast<int>(gridDim.x)) * 32 + ri;
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
        return;
    }

    // ========================================================= consumers
    using PX = PairX<TA, BITS>;
    constexpr bool OFFSET = (BITS != 8) && FoldOffset<TA>::value;  // magic offset removed after the MMA
    constexpr float kM = Act<TA>::kMagicVal;
    const int Gw = c.gw;
    const int Gbeg = warp * Gw;
    const int Gend = min(GT, Gbeg + Gw);
    const int ng = max(0, Gend - Gbeg);
    float *xs = reinterpret_cast<float *>(smem + c.off_xs) + warp * Gw * 16;  // [gi][token][sum, prescaled sum]
    // per-lane row bases of the swizzled code and scale tiles
    int crow[NROW], cfx[NROW], srow[NROW], sfx[NROW];
#pragma unroll
    for (int r = 0; r < NROW; ++r) {
        const int rr = g + 8 * (r & 1);
        crow[r] = c.off_codes + (r >> 1) * c.TBp + rr * c.RB;
        cfx[r] = (code_xor<WPS>(rr) & c.fm_c) << 4;
        srow[r] = (r >> 1) * c.TBp + rr * c.SB;
        sfx[r] = (c.sb_l2 >= 0 ? (rr & c.fm_s) : 0) << 4;
    }
    const int tw = t * WPS * 4;
    // single-token units use the group-column path when the warp's code words
    // split into whole 16-byte chunks per lane
    const bool gn_ok = ng > 0 && ng <= 8 && (ng * WPS) % 4 == 0;
    int it = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
        const int st = it % c.nst;
        const uint32_t ph = (it / c.nst) & 1;
        if (warp == 0) trace_point(a, it, 6);
        const bool got = mbar_wait(&full[st], ph);
        if (warp == 0) trace_point(a, it, 2);
        if (!got || aborted(abort_flag)) {
            if (lane == 0) {
                *abort_flag = 1;
                set_error(a.err, -4);
            }
            break;
        }
        const int *hdr = reinterpret_cast<const int *>(smem + c.off_shdr + st * kHdrBytes);
        const int ntok = hdr[0], rt = hdr[1];
        const int my_route = (lane < 8) ? hdr[kHdrRoute + lane] : -1;
        const int my_w = (lane < 8) ? hdr[kHdrWeight + lane] : 0;
        const uint8_t *sb = smem + c.off_stage + (size_t)st * c.stage_bytes;
        const float2 *s16 = reinterpret_cast<const float2 *>(sb + c.off_sum);
        const bool gpath = gn_ok && ntok == 1;

        float acc[NM][4];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[m][e] = 0.0f;
        if (gpath) {
            // ---- single-token unit: the MMA's 8 columns carry the warp's
            // groups instead of tokens.  Lane t covers a contiguous run of
            // NW code words per row (whole groups when NW >= WPG); its B
            // fragment is the token's activations where the lane's group
            // equals its column (g), zero elsewhere, so D[row][n] collects
            // group n's dot product over all k-steps in one accumulator.
            const int NW = ng * WPS;
            // per-group sum(x) and sum(panel) of token 0, 4 lanes per group
            float2 gx = make_float2(0.0f, 0.0f);
            {
                const int n = lane >> 2, sub = lane & 3;
                if (n < ng) {
                    const float2 *p = s16 + (Gbeg + n) * S;
                    for (int q = sub; q < S; q += 4) {
                        const float2 w = p[q];
                        gx.x += w.x;
                        gx.y += w.y;
                    }
                }
            }
            float d[NM][4];
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
                for (int e = 0; e < 4; ++e) d[m][e] = 0.0f;
            const uint8_t *panel0 = sb + c.off_panel;
            // scales and biases of the lane's two group columns (2t, 2t + 1),
            // read before the MMA loop so their latency hides behind it
            uint16_t sbr[NM][2][4];
            {
                const bool v0 = 2 * t < ng, v1 = 2 * t + 1 < ng;
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int r = 2 * m + h;
                        const int os0 = srow[r] + ((2 * (Gbeg + 2 * t)) ^ sfx[r]);
                        const int os1 = srow[r] + ((2 * (Gbeg + 2 * t + 1)) ^ sfx[r]);
                        sbr[m][h][0] = v0 ? *reinterpret_cast<const uint16_t *>(sb + c.off_s + os0) : 0;
                        sbr[m][h][1] = v0 ? *reinterpret_cast<const uint16_t *>(sb + c.off_b + os0) : 0;
                        sbr[m][h][2] = v1 ? *reinterpret_cast<const uint16_t *>(sb + c.off_s + os1) : 0;
                        sbr[m][h][3] = v1 ? *reinterpret_cast<const uint16_t *>(sb + c.off_b + os1) : 0;
                    }
            }
            // straight-line over the (at most 2 * WPS) 16-byte chunks of a
            // lane: as a rolled loop the compiler keeps too few values live
            // and the MMA issue rate drops several-fold
            constexpr int kMaxChunks = 2 * WPS;
#pragma unroll
            for (int qc = 0; qc < kMaxChunks; ++qc) {
                const int q = 4 * qc;
                if (q >= NW) break;
                const int w0 = Gbeg * WPG + t * NW + q;  // first code word of this chunk in the row
                const bool act = (g == w0 / WPG - Gbeg);
                uint32_t raw[NROW][4];
#pragma unroll
                for (int r = 0; r < NROW; ++r) {
                    const uint4 v = lds_u128(sb + crow[r] + ((w0 * 4) ^ cfx[r]));
                    raw[r][0] = v.x;
                    raw[r][1] = v.y;
                    raw[r][2] = v.z;
                    raw[r][3] = v.w;
                }
                const uint8_t *bp = panel0 + w0 * SPW * 8;
                uint4 bq = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    typename PX::W pw[NROW];
#pragma unroll
                    for (int r = 0; r < NROW; ++r) pw[r] = PX::prep(raw[r][i]);
#pragma unroll
                    for (int s2 = 0; s2 < SPW; ++s2) {
                        const int js = i * SPW + s2;
                        if ((js & 1) == 0) lds_u128_if(bq, bp + js * 8, act);
                        const uint32_t b0 = (js & 1) ? bq.z : bq.x;
                        const uint32_t b1 = (js & 1) ? bq.w : bq.y;
#pragma unroll
                        for (int m = 0; m < NM; ++m)
                            Act<TA>::mma(d[m], PX::get(pw[2 * m], 2 * s2), PX::get(pw[2 * m + 1], 2 * s2),
                                         PX::get(pw[2 * m], 2 * s2 + 1), PX::get(pw[2 * m + 1], 2 * s2 + 1), b0, b1);
                    }
                }
            }
            // the group sums (loaded before the MMA loop) reduced over each
            // group's 4 lanes; this lane's D columns are n0 = 2t and n1 = 2t + 1
            gx.x += __shfl_xor_sync(LMOE_FULL, gx.x, 1);
            gx.y += __shfl_xor_sync(LMOE_FULL, gx.y, 1);
            gx.x += __shfl_xor_sync(LMOE_FULL, gx.x, 2);
            gx.y += __shfl_xor_sync(LMOE_FULL, gx.y, 2);
            const float X0 = __shfl_sync(LMOE_FULL, gx.x, 8 * t), P0 = __shfl_sync(LMOE_FULL, gx.y, 8 * t);
            const float X1 = __shfl_sync(LMOE_FULL, gx.x, 8 * t + 4), P1 = __shfl_sync(LMOE_FULL, gx.y, 8 * t + 4);
            // epilogue: scale, bias and offset correction per group column,
            // then the row sums over the quad's columns
#pragma unroll
            for (int m = 0; m < NM; ++m) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float s0 = Act<TA>::to_f(sbr[m][h][0]), b0 = Act<TA>::to_f(sbr[m][h][1]);
                    const float s1 = Act<TA>::to_f(sbr[m][h][2]), b1 = Act<TA>::to_f(sbr[m][h][3]);
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
                    acc[m][2 * h] = tot;  // column 0: the unit's single token
                }
            }
        } else {
            // per (group, token): sum(x) for the bias term and the sum of the
            // stored panel values for the magic-offset correction, from the
            // staged 16-column sums (one lane per item, column order)
            for (int i = lane; i < ng * 8; i += 32) {
                const int gi = i >> 3, n = i & 7;
                float2 v = make_float2(0.0f, 0.0f);
                if (n < ntok) {
                    const float2 *p = s16 + n * (c.S16B / 8) + (Gbeg + gi) * S;
    #pragma unroll
                    for (int q = 0; q < S; ++q) {
                        const float2 w = p[q];
                        v.x += w.x;
                        v.y += w.y;
                    }
                }
                *reinterpret_cast<float2 *>(xs + i * 2) = v;
            }
            __syncwarp();

            const uint8_t *panel_g = sb + c.off_panel + g * c.PBp;
            const bool has_b = g < ntok;
    #pragma unroll 2
            for (int gi = 0; gi < ng; ++gi) {
                const int G = Gbeg + gi;
                const int goff = G * WPG * 4 + tw;
                typename PX::W pw[NROW][WPS];
                uint16_t sv[NROW], bv[NROW];
    #pragma unroll
                for (int r = 0; r < NROW; ++r) {
                    uint32_t wd[WPS];
                    if constexpr (WPS <= 4) {
                        lds_slice<WPS>(sb + crow[r] + (goff ^ cfx[r]), wd);
                    } else {
    #pragma unroll
                        for (int q = 0; q < WPS / 4; ++q) {
                            const uint4 v = lds_u128(sb + crow[r] + ((goff + 16 * q) ^ cfx[r]));
                            wd[4 * q] = v.x;
                            wd[4 * q + 1] = v.y;
                            wd[4 * q + 2] = v.z;
                            wd[4 * q + 3] = v.w;
                        }
                    }
    #pragma unroll
                    for (int q = 0; q < WPS; ++q) pw[r][q] = PX::prep(wd[q]);
                    const int os = srow[r] + ((2 * G) ^ sfx[r]);
                    sv[r] = lds_u16(sb + c.off_s + os);
                    bv[r] = lds_u16(sb + c.off_b + os);
                }
                float d[NM][4];
    #pragma unroll
                for (int m = 0; m < NM; ++m)
    #pragma unroll
                    for (int e = 0; e < 4; ++e) d[m][e] = 0.0f;
                uint4 bq = make_uint4(0u, 0u, 0u, 0u);
    #pragma unroll
                for (int k = 0; k < S; ++k) {
                    const int wi = k / SPW, s = k % SPW;
                    if ((k & 1) == 0 && has_b) bq = lds_u128(panel_g + ((G * 4 + t) * S + k) * 8);
                    const uint32_t b0 = (k & 1) ? bq.z : bq.x;
                    const uint32_t b1 = (k & 1) ? bq.w : bq.y;
    #pragma unroll
                    for (int m = 0; m < NM; ++m)
                        Act<TA>::mma(d[m], PX::get(pw[2 * m][wi], 2 * s), PX::get(pw[2 * m + 1][wi], 2 * s),
                                     PX::get(pw[2 * m][wi], 2 * s + 1), PX::get(pw[2 * m + 1][wi], 2 * s + 1), b0, b1);
                }
                const float4 xv = *reinterpret_cast<const float4 *>(xs + (gi * 8 + 2 * t) * 2);
                const float2 xsum = make_float2(xv.x, xv.z);
                const float2 xoff = make_float2(-kM * xv.y, -kM * xv.w);
    #pragma unroll
                for (int m = 0; m < NM; ++m) {
                    float2 d01 = make_float2(d[m][0], d[m][1]);
                    float2 d23 = make_float2(d[m][2], d[m][3]);
                    if constexpr (OFFSET) {
                        d01 = __fadd2_rn(d01, xoff);
                        d23 = __fadd2_rn(d23, xoff);
                    }
                    const float s0 = Act<TA>::to_f(sv[2 * m]), s1 = Act<TA>::to_f(sv[2 * m + 1]);
                    const float b0 = Act<TA>::to_f(bv[2 * m]), b1 = Act<TA>::to_f(bv[2 * m + 1]);
                    float2 a01 = make_float2(acc[m][0], acc[m][1]);
                    float2 a23 = make_float2(acc[m][2], acc[m][3]);
                    a01 = __ffma2_rn(d01, make_float2(s0, s0), a01);
                    a23 = __ffma2_rn(d23, make_float2(s1, s1), a23);
                    a01 = __ffma2_rn(xsum, make_float2(b0, b0), a01);
                    a23 = __ffma2_rn(xsum, make_float2(b1, b1), a23);
                    acc[m][0] = a01.x;
                    acc[m][1] = a01.y;
                    acc[m][2] = a23.x;
                    acc[m][3] = a23.y;
                }
            }
        }
        __syncwarp();
        if (warp == 0) trace_point(a, it, 3);
        if (lane == 0) mbar_arrive(&empty[st]);

        const int rb = it % kGemvEpi;
        const uint32_t rph = (it / kGemvEpi) & 1;
        if (!mbar_wait(&rempty[rb], rph ^ 1u) || aborted(abort_flag)) {
            if (lane == 0) {
                *abort_flag = 1;
                set_error(a.err, -4);
            }
            break;
        }
        float *red = reinterpret_cast<float *>(smem + c.off_red) + ((size_t)(rb * c.ncw + warp) * 32 + lane) * NM * 4;
#pragma unroll
        for (int m = 0; m < NM; ++m)
            *reinterpret_cast<float4 *>(red + m * 4) = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
        if (warp == 0) {
            int *rh = reinterpret_cast<int *>(smem + c.off_rhdr + rb * kHdrBytes);
            if (lane == 0) {
                rh[0] = ntok;
                rh[1] = rt;
            }
            if (lane < 8) {
                rh[kHdrRoute + lane] = my_route;
                rh[kHdrWeight + lane] = my_w;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rfull[rb]);
    }
}

// ============================================================ launch
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

bool gemv_config(int mode, int bits, int gs, int K, int ntok_max, GemvCfg *out) {
    const int NM = (mode == MODE_GATEUP || mode == MODE_DOWN2) ? 2 : 1;
    GemvCfg c;
    std::memset(&c, 0, sizeof(c));
    const int GT = K / gs;
    // groups per consumer warp: at least one 16-byte chunk of code words per
    // lane (the single-token path's unit of work), at most 16 warps
    const int wps = gs * bits / 128;
    const int gmin = wps >= 4 ? 1 : 4 / wps;
    int gw = (GT + kGemvMaxConsumers - 1) / kGemvMaxConsumers;
    gw = (gw + gmin - 1) / gmin * gmin;
    c.gw = gw;
    c.ncw = (GT + gw - 1) / gw;
    TileGeo tg;
    if (!tile_geo(K, bits, gs, &tg)) return false;
    c.RB = tg.RB;
    c.SB = tg.SB;
    c.rb_l2 = tg.rb_l2;
    c.sb_l2 = tg.sb_l2;
    c.fm_c = tg.fm_c;
    c.fm_s = tg.fm_s;
    c.TBp = tg.TB;
    c.PB = K * 2;
    c.PBp = c.PB + 16;
    c.S16B = (K / 16) * 8;
    int off = 0;
    auto al = [](int v, int a) { return (v + a - 1) / a * a; };
    // NM weight tiles (the HBM tile layout), then the activation rows
    c.off_codes = off;
    c.off_s = off + tg.tS;
    c.off_b = off + tg.tB;
    off += NM * tg.TB;
    c.off_panel = off;
    off = al(off + ntok_max * c.PBp, 16);
    c.off_sum = off;
    off = al(off + ntok_max * c.S16B, 16);
    c.stage_bytes = al(off, 128);
    int h = 0;
    c.off_bars = h;
    h += 256;
    c.off_shdr = h;
    h += kHdrBytes * kGemvMaxStages;
    c.off_rhdr = h;
    h += kGemvEpi * kHdrBytes;
    c.off_red = h;
    h = al(h + kGemvEpi * c.ncw * 32 * NM * 4 * 4, 128);
    c.off_xs = h;
    h = al(h + c.ncw * c.gw * 16 * 4, 128);
    c.off_list = h;
    // per epilogue warp; 8 = every unit is combined as soon as it is written
    // (four epilogue warps have the slack), so no burst is left for the tail
    c.list_cap = 8;
    h = al(h + kGemvEpi * c.list_cap * 4, 128);
    c.off_ptab = h;
    h = al(h + 128 * 2, 128);
    c.off_stage = h;
    const int budget = 227 * 1024;
    int nst = (budget - h) / c.stage_bytes;
    if (nst > kGemvMaxStages) nst = kGemvMaxStages;
    if (nst < 2) return false;
    c.nst = nst;
    c.smem = h + nst * c.stage_bytes;
    *out = c;
    return true;
}

// ============================================================ tile packing
// Row-major projection slots -> pre-tiled HBM layout (TileGeo): one block per
// (16-row tile, slot); 16-byte chunks are copied to their swizzled places and
// the tile's padding is zeroed.
__global__ void __launch_bounds__(256) tile_pack_kernel(const QView q, const TileGeo tg, int32_t slot_begin,
                                                        uint8_t *tiles) {
    const int rt = blockIdx.x;
    const int slot = slot_begin + static_cast<int>(blockIdx.y);
    uint8_t *dst = tiles + (size_t)slot * q.tile_slot_stride + (size_t)rt * tg.TB;
    const uint4 *csrc = reinterpret_cast<const uint4 *>(q.w + (size_t)slot * q.w_slot_stride +
                                                        (size_t)rt * 16 * q.words_per_row);
    const int n16c = 16 << tg.rb_l2;
    for (int i = threadIdx.x; i < n16c; i += blockDim.x)
        *reinterpret_cast<uint4 *>(dst + tile_code_chunk(tg, i)) = csrc[i];
    const size_t sb_off = (size_t)slot * q.sb_slot_stride + (size_t)rt * 16 * q.groups_per_row;
    const uint4 *ssrc = reinterpret_cast<const uint4 *>(q.s + sb_off);
    const uint4 *bsrc = reinterpret_cast<const uint4 *>(q.b + sb_off);
    const int n16s = tg.SB;  // 16 rows * SB bytes / 16
    for (int i = threadIdx.x; i < n16s; i += blockDim.x) {
        const int o = tile_sb_chunk(tg, i);
        *reinterpret_cast<uint4 *>(dst + tg.tS + o) = ssrc[i];
        *reinterpret_cast<uint4 *>(dst + tg.tB + o) = bsrc[i];
    }
    for (int o = tg.tB + 16 * tg.SB + 16 * threadIdx.x; o < tg.TB; o += 16 * blockDim.x)
        *reinterpret_cast<uint4 *>(dst + o) = make_uint4(0u, 0u, 0u, 0u);
}

cudaError_t launch_tile_pack(const QView &q, int bits, int gs, int slot_begin, int slot_count, uint8_t *tiles,
                             cudaStream_t st) {
    TileGeo tg;
    if (!tile_geo(q.cols, bits, gs, &tg)) return cudaErrorInvalidValue;
    if (slot_count <= 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>(q.rows / 16), static_cast<unsigned>(slot_count), 1);
    tile_pack_kernel<<<grid, 256, 0, st>>>(q, tg, slot_begin, tiles);
    return cudaGetLastError();
}

// Blocks of a MODE_DOWN2 launch for `pairs` row pairs: the largest divisor of
// pairs not above the SM count, or 0 when that leaves more than half the SMs
// idle (the caller then uses MODE_DOWN).
int down2_grid(int pairs) {
    const int sms = num_sms();
    if (pairs < 1) return 0;
    int g = pairs < sms ? pairs : sms;
    while (g > 1 && pairs % g != 0) --g;
    const int want = pairs < sms ? pairs : sms;
    return 2 * g >= want ? g : 0;
}

template <typename TA, int BITS, int GS, int MODE>
static cudaError_t launch_gemv_t(const GemvArgs &a, int max_chunks, cudaStream_t st) {
    GemvCfg c;
    if (!gemv_config(MODE, BITS, GS, a.q0.cols, a.ntok_max, &c)) return cudaErrorInvalidValue;
    auto kern = gemv_kernel<TA, BITS, GS, MODE>;
    static int configured = 0;
    if (c.smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, c.smem);
        if (e != cudaSuccess) return e;
        configured = c.smem;
    }
    long grid = num_sms();
    if (MODE == MODE_DOWN2) {
        // every block owns whole row pairs: the grid divides their number
        const int pairs = a.q0.rows / 32;
        grid = down2_grid(pairs);
        if (grid < 1 || (a.q0.rows & 31) != 0) return cudaErrorInvalidValue;
    } else {
        const long units_max = (long)max_chunks * (a.q0.rows / 16);
        if (grid > units_max) grid = units_max;
        if (grid < 1) grid = 1;
    }
    return launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3((c.ncw + 2 + kGemvEpi) * 32), c.smem, st, a, c);
}

template <typename TA, int MODE>
static cudaError_t launch_gemv_bits(int bits, int gs, const GemvArgs &a, int max_chunks, cudaStream_t st) {
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

cudaError_t launch_gemv(int mode, int act_f16, int bits, int gs, const GemvArgs &a, int max_chunks,
                        cudaStream_t st) {
    if (act_f16) {
        if (mode == MODE_GATEUP) return launch_gemv_bits<__half, MODE_GATEUP>(bits, gs, a, max_chunks, st);
        if (mode == MODE_DOWN) return launch_gemv_bits<__half, MODE_DOWN>(bits, gs, a, max_chunks, st);
        if (mode == MODE_DOWN2) return launch_gemv_bits<__half, MODE_DOWN2>(bits, gs, a, max_chunks, st);
        return launch_gemv_bits<__half, MODE_QMM>(bits, gs, a, max_chunks, st);
    }
    if (mode == MODE_GATEUP) return launch_gemv_bits<__nv_bfloat16, MODE_GATEUP>(bits, gs, a, max_chunks, st);
    if (mode == MODE_DOWN) return launch_gemv_bits<__nv_bfloat16, MODE_DOWN>(bits, gs, a, max_chunks, st);
    if (mode == MODE_DOWN2) return launch_gemv_bits<__nv_bfloat16, MODE_DOWN2>(bits, gs, a, max_chunks, st);
    return launch_gemv_bits<__nv_bfloat16, MODE_QMM>(bits, gs, a, max_chunks, st);
}

}  // namespace lmoe
