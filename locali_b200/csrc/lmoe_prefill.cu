// Prefill grouped GEMM of the routed experts on the 5th-generation tensor
// cores (tcgen05, sm_100a).
//
// Used where per-expert token counts make the expert products dense
// contractions (prefill).  The dispatch kernels group routes by expert into
// chunks of at most kPfNmax = 128 routes.  One work item is a chunk times a
// pair of 128-row weight blocks: (gate rows, up rows) for the gate/up kernel,
// two consecutive 128-row blocks of the down projection for the down kernel.
// For each 64-column K stage:
//   * 8 dequantisation warps turn the packed codes of one weight row each
//     into operand A in shared memory, in the activation dtype (one rounding
//     of scale * q + bias per weight: fma.rn on the packed pair), laid out in
//     the 128-byte-swizzled K-major form the tensor core reads.  Their code,
//     scale and bias bytes stream through a per-thread cp.async ring several
//     stages ahead;
//   * a producer warp moves operand B (N routes x 64 columns) with one bulk
//     copy (no multicast) from a panel kept in the same swizzled form;
//   * one thread issues tcgen05.mma (M 128, N = routes rounded up to 16,
//     K 16) into fp32 accumulators in tensor memory (TMEM): two accumulators
//     per item, double-buffered across items (all 512 TMEM columns);
//   * 4 epilogue warps read the accumulators back (tcgen05.ld), apply the
//     clamped SwiGLU (gate/up; h goes straight into the down kernel's panel)
//     or the combine weight (down; bf16(y) * bf16(w) rows, summed per token
//     in route order by pf_combine_kernel).
//
// K order.  Inside the span of n = 32/bits columns covered by one code word,
// both operands are stored as pairs (c_m, c_{m+n/2}) at positions (2m, 2m+1):
// one mask-and-or of the word then yields both codes of a packed 16-bit pair.
// The activation panels use the same permutation, so the contraction is
// unchanged.
//
// Every wait is bounded (mbar_wait); a wait that gives up latches LMOE_ECUDA,
// raises the block's abort flag, and the block drains its tensor-core work
// and frees its TMEM before returning.
#include "lmoe_kernels.cuh"

namespace lmoe {

namespace {

constexpr int kPfM = 128;       // weight rows per accumulator (MMA M)
constexpr int kPfKS = 64;       // K columns per stage: one 128-byte swizzle row of 16-bit values
constexpr int kPfStages = 3;
constexpr int kPfDeqWarps = 8;  // 256 threads: one (accumulator, row) each
constexpr int kPfEpiWarps = 4;
constexpr int kPfThreads = (2 + kPfDeqWarps + kPfEpiWarps) * 32;
constexpr int kPfATile = kPfM * kPfKS * 2;           // 16 KB
constexpr int kPfBTile = kPfNmax * kPfKS * 2;        // 16 KB
constexpr int kPfStageBytes = 2 * kPfATile + kPfBTile;
constexpr int kPfTmemCols = 512;                     // 2 buffers x 2 accumulators x 128 columns
constexpr int kPfPanelAtoms = 8;                     // 64-column blocks per panel-builder block

// ------------------------------------------------------------ tcgen05 primitives
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] = A * B^T (+ D when `accumulate`), A and B K-major in shared memory
__device__ __forceinline__ void umma_f16(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive once on `bar` when every MMA issued so far by this thread has completed
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns (lane = accumulator row)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// waits for this thread's tcgen05.ld; the registers pass through the asm so
// no use of them is scheduled above the wait
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                   "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                   "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes (stride byte offset 1024), Blackwell descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// Instruction descriptor of kind::f16: fp32 accumulator, A and B of the same
// 16-bit type (bf16 or f16), both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_f16(int n, bool f16) {
    const uint32_t fmt = f16 ? 0u : 1u;
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kPfM >> 4) << 24);
}

__device__ __forceinline__ void cp16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// ------------------------------------------------------------ packed 16-bit pair math
template <typename TA>
struct Pf2;
template <>
struct Pf2<__nv_bfloat16> {
    static constexpr uint32_t kOne = 0x3F803F80u, kNegMagic = 0xC300C300u, kMagic = 0x43004300u;
    static constexpr uint32_t kNegZero = 0x80008000u, kQuarter = 0x3E803E80u, kSixteenth = 0x3D803D80u;
    static constexpr uint32_t kSixteen = 0x41804180u;
    __device__ __forceinline__ static uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
        uint32_t d;
        asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        return d;
    }
};
template <>
struct Pf2<__half> {
    static constexpr uint32_t kOne = 0x3C003C00u, kNegMagic = 0xE400E400u, kMagic = 0x64006400u;
    static constexpr uint32_t kNegZero = 0x80008000u, kQuarter = 0x34003400u, kSixteenth = 0x2C002C00u;
    static constexpr uint32_t kSixteen = 0x4C004C00u;
    __device__ __forceinline__ static uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
        uint32_t d;
        asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        return d;
    }
};

// Exact codes of pair m of a word, as a packed 16-bit pair scaled by 4^p.
// Only bf16 2-bit codes are taken in place (p = m mod 3, from w, w >> 6,
// w >> 12; the scale is then divided by 4^p, exactly, a power of two); all
// other widths shift each pair down first (p = 0).
template <typename TA, int BITS>
struct PfCodes {
    static constexpr int kPairs = 16 / BITS;
    static constexpr bool kPrescale = (BITS == 2) && std::is_same<TA, __nv_bfloat16>::value;
    struct W {
        uint32_t w0, w6, w12;
    };
    __device__ __forceinline__ static W prep(uint32_t w) {
        W r;
        r.w0 = w;
        r.w6 = kPrescale ? (w >> 6) : 0u;
        r.w12 = kPrescale ? (w >> 12) : 0u;
        return r;
    }
    __host__ __device__ static constexpr int pexp(int m) { return kPrescale ? (m < 6 ? m % 3 : m - 6) : 0; }
    __device__ __forceinline__ static uint32_t q(const W &w, int m) {
        using P = Pf2<TA>;
        if constexpr (kPrescale) {
            const uint32_t src = m < 3 ? w.w0 : (m < 6 ? w.w6 : w.w12);
            const uint32_t v = (src & (0x00030003u << (2 * pexp(m)))) | P::kMagic;
            return P::fma2(v, P::kOne, P::kNegMagic);
        } else if constexpr (BITS == 8 && std::is_same<TA, __nv_bfloat16>::value) {
            // 8-bit codes exceed the bf16 magic's mantissa: two exact nibbles
            const uint32_t s = w.w0 >> (8 * m);
            const uint32_t lo = P::fma2((s & 0x000F000Fu) | P::kMagic, P::kOne, P::kNegMagic);
            const uint32_t hi = P::fma2(((s >> 4) & 0x000F000Fu) | P::kMagic, P::kOne, P::kNegMagic);
            return P::fma2(hi, P::kSixteen, lo);
        } else {
            constexpr uint32_t mask = BITS == 2 ? 0x00030003u : (BITS == 4 ? 0x000F000Fu : 0x00FF00FFu);
            const uint32_t v = ((w.w0 >> (BITS * m)) & mask) | P::kMagic;
            return P::fma2(v, P::kOne, P::kNegMagic);
        }
    }
};

// Per-thread cp.async ring of the dequantisation threads: the code bytes of
// RS stages and two 8-group blocks of scales and biases.  The ring stride is
// an odd number of 16-byte chunks so the 16-byte accesses of consecutive
// threads hit distinct bank groups.
template <int BITS, int GS>
struct PfRing {
    static constexpr int CB = 8 * BITS;   // code bytes of one row per stage
    static constexpr int SPB = GS / 8;    // stages per block of 8 groups
    static constexpr int RS0 = 128 / CB;
    static constexpr int RS = RS0 < SPB ? RS0 : SPB;  // stages in flight (lookahead RS - 1 < SPB)
    static constexpr int RAW = RS * CB + 64;
    static constexpr int BYTES = ((RAW / 16) | 1) * 16;
    static_assert(RS >= 2, "ring");
};

template <int BITS, int GS>
constexpr int pf_smem_bytes() {
    return 1024 + kPfStages * kPfStageBytes + 256 * PfRing<BITS, GS>::BYTES + 256;
}

// Panel position of column f for a projection quantised with `bits`.
__host__ __device__ __forceinline__ int pf_perm_pos(int f, int bits) {
    const int n = 32 / bits, h = n >> 1;
    const int base = f - f % n, c = f % n;
    return c < h ? base + 2 * c : base + 2 * (c - h) + 1;
}
// Byte offset of (panel row pr, panel position kp) in a [K/64][prow/8][1024] panel.
__host__ __device__ __forceinline__ size_t pf_panel_off(int pr, int kp, int prow) {
    return ((size_t)(kp >> 6) * (size_t)(prow >> 3) + (size_t)(pr >> 3)) * 1024u + (size_t)(pr & 7) * 128u +
           (size_t)((((kp & 63) >> 3) ^ (pr & 7)) << 4) + (size_t)((kp & 7) << 1);
}

// ------------------------------------------------------------ panel builder
// Permuted chunk h (positions 8h..8h+7) of one 64-column block of a row.
template <int BITS>
__device__ __forceinline__ uint4 pf_perm_chunk(const uint16_t *row64, int h) {
    uint4 o;
    if constexpr (BITS == 2) {
        // span of 16 columns: positions (2m, 2m+1) <- columns (m, m + 8)
        const uint4 lo = *reinterpret_cast<const uint4 *>(row64 + (h >> 1) * 16);
        const uint4 hi = *reinterpret_cast<const uint4 *>(row64 + (h >> 1) * 16 + 8);
        const uint32_t l0 = (h & 1) ? lo.z : lo.x, l1 = (h & 1) ? lo.w : lo.y;
        const uint32_t h0 = (h & 1) ? hi.z : hi.x, h1 = (h & 1) ? hi.w : hi.y;
        o.x = __byte_perm(l0, h0, 0x5410);
        o.y = __byte_perm(l0, h0, 0x7632);
        o.z = __byte_perm(l1, h1, 0x5410);
        o.w = __byte_perm(l1, h1, 0x7632);
    } else if constexpr (BITS == 4) {
        // span of 8: (2m, 2m+1) <- (m, m + 4)
        const uint4 v = *reinterpret_cast<const uint4 *>(row64 + h * 8);
        o.x = __byte_perm(v.x, v.z, 0x5410);
        o.y = __byte_perm(v.x, v.z, 0x7632);
        o.z = __byte_perm(v.y, v.w, 0x5410);
        o.w = __byte_perm(v.y, v.w, 0x7632);
    } else {
        // two spans of 4: (2m, 2m+1) <- (m, m + 2)
        const uint4 v = *reinterpret_cast<const uint4 *>(row64 + h * 8);
        o.x = __byte_perm(v.x, v.y, 0x5410);
        o.y = __byte_perm(v.x, v.y, 0x7632);
        o.z = __byte_perm(v.z, v.w, 0x5410);
        o.w = __byte_perm(v.z, v.w, 0x7632);
    }
    return o;
}

// x rows of every chunk's routes -> the gate/up kernel's panel (rows past a
// chunk's routes up to its 16-row boundary are zero).  Grid: (chunks,
// K / (64 * kPfPanelAtoms)); 8 threads per row and 64-column block.
template <int BITS>
__global__ void __launch_bounds__(256) pf_panel_kernel(const PfPanelArgs a) {
    pdl_wait();
    pdl_trigger();
    const int c = blockIdx.x;
    if (c >= *a.n_chunks) return;
    const Chunk ch = a.chunks[c];
    const int N = (ch.ntok + 15) & ~15;
    const int pbase = pf_row_base(ch.route_start, c);
    const int h = threadIdx.x & 7;
    const int atoms = a.K >> 6;
    const int a0 = blockIdx.y * kPfPanelAtoms;
    const int a1 = min(atoms, a0 + kPfPanelAtoms);
    for (int j = threadIdx.x >> 3; j < N; j += 32) {
        const int pr = pbase + j;
        const uint16_t *src = nullptr;
        if (j < ch.ntok) src = a.x + (size_t)(a.sorted_routes[ch.route_start + j] / a.route_div) * a.K;
        for (int at = a0; at < a1; ++at) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (src) v = pf_perm_chunk<BITS>(src + at * 64, h);
            *reinterpret_cast<uint4 *>(a.panel + pf_panel_off(pr, at * 64 + h * 8, a.prow)) = v;
        }
    }
}

// out[t] = sum over j < k, in route order, of the fp32 values of yw[t*k + j],
// rounded once (the combine of arena.py:619-624 as the decode kernels do it).
template <typename TA>
__global__ void __launch_bounds__(256) pf_combine_kernel(const uint16_t *yw, int T, int H, int k, uint16_t *out) {
    pdl_wait();
    pdl_trigger();
    const int per = H >> 3;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)T * per) return;
    const long t = i / per;
    const int cc = (int)(i - t * per);
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    for (int j = 0; j < k; ++j) {
        const uint4 v = *reinterpret_cast<const uint4 *>(yw + ((size_t)(t * k + j) * H + (size_t)cc * 8));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            acc[2 * e] += Act<TA>::to_f(static_cast<uint16_t>(w[e] & 0xFFFFu));
            acc[2 * e + 1] += Act<TA>::to_f(static_cast<uint16_t>(w[e] >> 16));
        }
    }
    uint4 o;
    o.x = Act<TA>::pack2(acc[0], acc[1]);
    o.y = Act<TA>::pack2(acc[2], acc[3]);
    o.z = Act<TA>::pack2(acc[4], acc[5]);
    o.w = Act<TA>::pack2(acc[6], acc[7]);
    *reinterpret_cast<uint4 *>(out + (size_t)t * H + (size_t)cc * 8) = o;
}

// ------------------------------------------------------------ the grouped GEMM
template <typename TA, int BITS, int GS, int MODE>
__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_kernel(const PfArgs a) {
    using RG = PfRing<BITS, GS>;
    using C = PfCodes<TA, BITS>;
    using P = Pf2<TA>;
    constexpr int NW = RG::CB / 4;           // code words of one row per stage
    constexpr int CPW = 32 / BITS;           // codes per word
    constexpr int NPAIR = NW * C::kPairs;    // 32 packed pairs = 64 weights
    static_assert(NPAIR == 32, "a stage row is 64 weights");
    constexpr bool kF16 = std::is_same<TA, __half>::value;

    extern __shared__ __align__(1024) uint8_t pf_raw[];
    uint8_t *smem = pf_raw + ((1024u - (smem_u32(pf_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    uint8_t *ring = smem + kPfStages * kPfStageBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + 256 * RG::BYTES);
    uint64_t *full_a = bars;
    uint64_t *full_b = bars + kPfStages;
    uint64_t *empty = bars + 2 * kPfStages;
    uint64_t *acc_full = bars + 3 * kPfStages;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kPfStages; ++s) {
            mbar_init(&full_a[s], kPfDeqWarps);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kPfEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kPfTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the chunk table and the panel come from the preceding kernels
    pdl_wait();
    pdl_trigger();
    const int items = *a.n_chunks * a.rbn;
    const int KS = a.K / kPfKS;

    if (warp == 0) {
        // ---------------------------------------------------- operand B producer
        if (lane == 0) {
            const size_t kstride = (size_t)(a.prow >> 3) * 1024u;
            int g = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
                if (*abort_flag) break;
                const int c = item / a.rbn;
                const Chunk ch = a.chunks[c];
                const uint32_t bytes = (uint32_t)((ch.ntok + 15) & ~15) * 128u;
                const uint8_t *src = a.panel + (size_t)(pf_row_base(ch.route_start, c) >> 3) * 1024u;
                for (int ks = 0; ks < KS; ++ks, ++g) {
                    const int s = g % kPfStages;
                    if (!mbar_wait(&empty[s], ((g / kPfStages) & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full_b[s], bytes);
                    bulk_g2s(smem + s * kPfStageBytes + 2 * kPfATile, src + (size_t)ks * kstride, bytes,
                             &full_b[s]);
                }
            }
            if (!ok) {
                *abort_flag = 1;
                set_error(a.err, -4);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        if (lane == 0) {
            int g = 0, it = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x, ++it) {
                if (*abort_flag) break;
                const Chunk ch = a.chunks[item / a.rbn];
                const uint32_t idesc = idesc_f16((ch.ntok + 15) & ~15, kF16);
                const int b = it & 1;
                if (!mbar_wait(&acc_empty[b], ((it >> 1) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d0 = tmem + (uint32_t)(b * 256), d1 = d0 + 128u;
                for (int ks = 0; ks < KS; ++ks, ++g) {
                    const int s = g % kPfStages;
                    const uint32_t ph = (g / kPfStages) & 1;
                    if (!mbar_wait(&full_b[s], ph) || !mbar_wait(&full_a[s], ph)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = sbase + (uint32_t)(s * kPfStageBytes);
                    const uint64_t da0 = sw128_desc(st), da1 = sw128_desc(st + kPfATile);
                    const uint64_t db = sw128_desc(st + 2 * kPfATile);
#pragma unroll
                    for (int kk = 0; kk < kPfKS / 16; ++kk) {
                        // K step of 16 = 32 bytes along the swizzled row
                        const uint32_t acc = (ks | kk) ? 1u : 0u;
                        umma_f16(d0, da0 + 2u * kk, db + 2u * kk, idesc, acc);
                        umma_f16(d1, da1 + 2u * kk, db + 2u * kk, idesc, acc);
                    }
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&acc_full[b]);
            }
            if (!ok) {
                *abort_flag = 1;
                set_error(a.err, -4);
            }
            // nothing may still write TMEM when it is freed
            umma_commit(drain);
            if (!mbar_wait(drain, 0)) set_error(a.err, -4);
        }
    } else if (warp < 2 + kPfDeqWarps) {
        // ---------------------------------------------------- dequantisation (operand A)
        const int td = threadIdx.x - 64;
        const int p = td >> 7, r = td & (kPfM - 1);
        const QView &q = (MODE == PF_GATEUP && p == 1) ? a.q1 : a.q0;
        const uint32_t ring_t = smem_u32(ring) + (uint32_t)(td * RG::BYTES);
        const uint32_t sring_t = ring_t + RG::RS * RG::CB;  // 2 x (16 B scales, 16 B biases)
        const uint32_t arow = sbase + (uint32_t)(p * kPfATile + (r >> 3) * 1024 + (r & 7) * 128);
        const int r7 = r & 7;
        // issue cursor: the cp.async stream runs RS - 1 stages ahead, across items
        int iss_item = blockIdx.x, iss_ks = 0, iss_nb = 0;
        const uint8_t *iss_codes = nullptr;
        const uint16_t *iss_s = nullptr, *iss_b = nullptr;
        auto locate = [&](int item) {
            const int c = item / a.rbn, rb = item - c * a.rbn;
            const long slot = a.chunks[c].slot;
            const long row = MODE == PF_GATEUP ? (long)rb * kPfM + r : (long)rb * 2 * kPfM + p * kPfM + r;
            iss_codes = reinterpret_cast<const uint8_t *>(q.w + slot * q.w_slot_stride + row * q.words_per_row);
            iss_s = q.s + slot * q.sb_slot_stride + row * q.groups_per_row;
            iss_b = q.b + slot * q.sb_slot_stride + row * q.groups_per_row;
        };
        auto issue = [&](int n) {
            if (iss_item < items) {
                const uint32_t dst = ring_t + (uint32_t)((n % RG::RS) * RG::CB);
#pragma unroll
                for (int i = 0; i < RG::CB / 16; ++i) cp16(dst + 16 * i, iss_codes + iss_ks * RG::CB + 16 * i);
                if (iss_ks % RG::SPB == 0) {
                    const int blk = iss_ks / RG::SPB;
                    const uint32_t sd = sring_t + (uint32_t)((iss_nb & 1) * 32);
                    cp16(sd, iss_s + blk * 8);
                    cp16(sd + 16, iss_b + blk * 8);
                    ++iss_nb;
                }
                if (++iss_ks == KS) {
                    iss_ks = 0;
                    iss_item += gridDim.x;
                    if (iss_item < items) locate(iss_item);
                }
            }
            cp_commit();
        };
        if (iss_item < items) locate(iss_item);
        for (int n = 0; n < RG::RS - 1; ++n) issue(n);
        int g = 0, nb = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
            if (*abort_flag) break;
            for (int ks = 0; ks < KS; ++ks, ++g) {
                issue(g + RG::RS - 1);
                cp_wait<RG::RS - 1>();
                const int s = g % kPfStages;
                if (!mbar_wait(&empty[s], ((g / kPfStages) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                if (ks % RG::SPB == 0) ++nb;
                const uint32_t sslot = sring_t + (uint32_t)(((nb - 1) & 1) * 32);
                const int gi = ((ks % RG::SPB) * kPfKS) / GS;  // first group of this stage in the block
                // scale variants per group of this stage (GS = 32: two groups)
                uint32_t sp[2][3], b2[2];
#pragma unroll
                for (int gg = 0; gg < (GS < kPfKS ? 2 : 1); ++gg) {
                    const uint32_t s16 = lds16(sslot + 2 * (gi + gg));
                    const uint32_t bb16 = lds16(sslot + 16 + 2 * (gi + gg));
                    sp[gg][0] = s16 | (s16 << 16);
                    b2[gg] = bb16 | (bb16 << 16);
                    if constexpr (C::kPrescale) {
                        sp[gg][1] = P::fma2(sp[gg][0], P::kQuarter, P::kNegZero);
                        sp[gg][2] = P::fma2(sp[gg][0], P::kSixteenth, P::kNegZero);
                    } else {
                        sp[gg][1] = sp[gg][2] = sp[gg][0];
                    }
                }
                uint32_t words[NW];
                const uint32_t csrc = ring_t + (uint32_t)((g % RG::RS) * RG::CB);
#pragma unroll
                for (int i = 0; i < NW / 4; ++i) {
                    const uint4 v = lds128(csrc + 16 * i);
                    words[4 * i] = v.x;
                    words[4 * i + 1] = v.y;
                    words[4 * i + 2] = v.z;
                    words[4 * i + 3] = v.w;
                }
                uint32_t pr[NPAIR];
#pragma unroll
                for (int u = 0; u < NW; ++u) {
                    const int gg = (GS < kPfKS) ? (u * CPW) / GS : 0;
                    const typename C::W w = C::prep(words[u]);
#pragma unroll
                    for (int m = 0; m < C::kPairs; ++m)
                        pr[u * C::kPairs + m] = P::fma2(C::q(w, m), sp[gg][C::pexp(m)], b2[gg]);
                }
                const uint32_t adst = arow + (uint32_t)(s * kPfStageBytes);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    sts128(adst + (uint32_t)((j ^ r7) << 4), pr[4 * j], pr[4 * j + 1], pr[4 * j + 2], pr[4 * j + 3]);
                // generic-proxy writes -> visible to the tensor core (async proxy)
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full_a[s]);
            }
        }
        if (!ok) {
            *abort_flag = 1;
            set_error(a.err, -4);
        }
        cp_wait<0>();
    } else {
        // ---------------------------------------------------- epilogue
        const int q4 = warp & 3;  // TMEM lanes 32*q4 .. 32*q4+31 (a warp reaches its own quarter)
        const int r = q4 * 32 + lane;
        int it = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < items; item += gridDim.x, ++it) {
            if (*abort_flag) break;
            const int c = item / a.rbn, rb = item - c * a.rbn;
            const Chunk ch = a.chunks[c];
            const int N = (ch.ntok + 15) & ~15;
            const int b = it & 1;
            if (!mbar_wait(&acc_full[b], (it >> 1) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t t0 = tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(b * 256);
            if constexpr (MODE == PF_GATEUP) {
                const int f = rb * kPfM + r;
                const int kp = pf_perm_pos(f, a.hbits);
                const int pbase = pf_row_base(ch.route_start, c);
                for (int j0 = 0; j0 < N; j0 += 16) {
                    uint32_t gv[16], uv[16];
                    tmem_ld16(t0 + (uint32_t)j0, gv);
                    tmem_ld16(t0 + 128u + (uint32_t)j0, uv);
                    tmem_wait_ld(gv);
                    tmem_wait_ld(uv);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int j = j0 + i;
                        float h = 0.0f;
                        if (j < ch.ntok)
                            h = swiglu_h<TA>(__uint_as_float(gv[i]), __uint_as_float(uv[i]), a.limit, a.swiglu_mode);
                        *reinterpret_cast<uint16_t *>(a.hpanel + pf_panel_off(pbase + j, kp, a.hprow)) =
                            Act<TA>::from_f(h);
                    }
                }
            } else {
#pragma unroll 1
                for (int pp = 0; pp < 2; ++pp) {
                    const int f = rb * 2 * kPfM + pp * kPfM + r;
                    for (int j0 = 0; j0 < N; j0 += 16) {
                        uint32_t yv[16];
                        tmem_ld16(t0 + (uint32_t)(pp * 128 + j0), yv);
                        // route and combine weight of column j0 + (lane & 15)
                        const int jl = j0 + (lane & 15);
                        int my_route = 0;
                        float my_w = 0.0f;
                        if (jl < ch.ntok) {
                            my_route = a.sorted_routes[ch.route_start + jl];
                            my_w = a.route_w[my_route];
                        }
                        tmem_wait_ld(yv);
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int route = __shfl_sync(0xffffffffu, my_route, i);
                            const float wv = __shfl_sync(0xffffffffu, my_w, i);
                            if (j0 + i < ch.ntok) {
                                const float y = Act<TA>::round(__uint_as_float(yv[i]));
                                a.yw[(size_t)route * a.H + f] = Act<TA>::from_f(y * Act<TA>::round(wv));
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (!ok) {
            *abort_flag = 1;
            set_error(a.err, -4);
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kPfTmemCols);
    }
}

int g_pf_sms = 0;
int pf_num_sms() {
    if (g_pf_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_pf_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_pf_sms <= 0) g_pf_sms = 148;
    }
    return g_pf_sms;
}

template <typename TA, int BITS, int GS, int MODE>
cudaError_t launch_pf_t(const PfArgs &a, cudaStream_t st) {
    auto kern = pf_gemm_kernel<TA, BITS, GS, MODE>;
    constexpr int smem = pf_smem_bytes<BITS, GS>();
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    return launch_pdl(kern, dim3(static_cast<unsigned>(pf_num_sms())), dim3(kPfThreads), smem, st, a);
}

template <typename TA, int MODE>
cudaError_t launch_pf_bits(int bits, int gs, const PfArgs &a, cudaStream_t st) {
#define LMOE_PF_CASE(B, G) \
    if (bits == B && gs == G) return launch_pf_t<TA, B, G, MODE>(a, st);
    LMOE_PF_CASE(2, 64)
    LMOE_PF_CASE(2, 128)
    LMOE_PF_CASE(4, 32)
    LMOE_PF_CASE(4, 64)
    LMOE_PF_CASE(4, 128)
    LMOE_PF_CASE(8, 32)
    LMOE_PF_CASE(8, 64)
    LMOE_PF_CASE(8, 128)
#undef LMOE_PF_CASE
    return cudaErrorInvalidValue;
}

}  // namespace

// K a multiple of 64 and of 8 groups (16-byte scale blocks), rows a multiple
// of 128 (gate/up) or 256 (down), and a compiled (bits, group) pair.
bool pf_supported(int K, int rows, int bits, int gs, int mode) {
    const bool bg = (bits == 2 && (gs == 64 || gs == 128)) ||
                    ((bits == 4 || bits == 8) && (gs == 32 || gs == 64 || gs == 128));
    if (!bg) return false;
    if (K <= 0 || K % kPfKS != 0 || K % (8 * gs) != 0) return false;
    return rows > 0 && rows % (mode == PF_GATEUP ? kPfM : 2 * kPfM) == 0;
}

cudaError_t launch_pf_panel(const PfPanelArgs &a, int max_chunks, cudaStream_t st) {
    if (max_chunks < 1) return cudaSuccess;
    const int atoms = a.K / 64;
    dim3 grid(static_cast<unsigned>(max_chunks), static_cast<unsigned>((atoms + kPfPanelAtoms - 1) / kPfPanelAtoms));
    if (a.bits == 2) return launch_pdl(pf_panel_kernel<2>, grid, dim3(256), 0, st, a);
    if (a.bits == 4) return launch_pdl(pf_panel_kernel<4>, grid, dim3(256), 0, st, a);
    if (a.bits == 8) return launch_pdl(pf_panel_kernel<8>, grid, dim3(256), 0, st, a);
    return cudaErrorInvalidValue;
}

cudaError_t launch_pf_gemm(int mode, int act_f16, int bits, int gs, const PfArgs &a, cudaStream_t st) {
    if (act_f16) {
        if (mode == PF_GATEUP) return launch_pf_bits<__half, PF_GATEUP>(bits, gs, a, st);
        return launch_pf_bits<__half, PF_DOWN>(bits, gs, a, st);
    }
    if (mode == PF_GATEUP) return launch_pf_bits<__nv_bfloat16, PF_GATEUP>(bits, gs, a, st);
    return launch_pf_bits<__nv_bfloat16, PF_DOWN>(bits, gs, a, st);
}

cudaError_t launch_pf_combine(int act_f16, const uint16_t *yw, int T, int H, int top_k, uint16_t *out,
                              cudaStream_t st) {
    const long n = (long)T * (H / 8);
    if (n <= 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>((n + 255) / 256));
    if (act_f16) return launch_pdl(pf_combine_kernel<__half>, grid, dim3(256), 0, st, yw, T, H, top_k, out);
    return launch_pdl(pf_combine_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, yw, T, H, top_k, out);
}

}  // namespace lmoe
