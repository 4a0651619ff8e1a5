// Prefill grouped GEMM of the routed experts on the 5th-generation tensor
// cores (tcgen05, sm_100a).
//
// Used where per-expert token counts make the expert products dense
// contractions (prefill).  The dispatch kernels group routes by expert into
// chunks of at most kPfNmax = 128 routes.  One work item is a chunk times a
// pair of 128-row weight blocks: (gate rows, up rows) for the gate/up kernel,
// two consecutive 128-row blocks of the down projection for the down kernel.
// For each 64-column K stage:
//   * a weight-stream warp moves the packed codes of both 128-row blocks
//     (2-D TMA tiles of 128 rows x one stage, into a ring of stages) and
//     their scales and biases (8 groups at a time);
//   * 8 dequantisation warps turn the codes of one weight row each into
//     operand A in shared memory, in the activation dtype (one rounding of
//     scale * q + bias per weight: fma.rn on the packed pair), laid out in
//     the 128-byte-swizzled K-major form the tensor core reads;
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
#include <cudaTypedefs.h>

#include "lmoe_kernels.cuh"

namespace lmoe {

namespace {

constexpr int kPfM = 128;        // weight rows per accumulator (MMA M)
constexpr int kPfKS = 128;       // K columns per stage: two 128-byte swizzle atoms of 16-bit values
constexpr int kPfSS = 2;         // stages in flight: operand A in tensor memory, operand B in shared memory
constexpr int kPfDeqWarps = 16;  // 512 threads: one (accumulator, row, K half) each
constexpr int kPfEpiWarps = 8;   // two per TMEM lane quarter, alternate 16-column chunks
constexpr int kPfDeq0 = 3;       // warps: 0 operand B, 1 MMA, 2 weights, 3..18 dequantisation, 19..26 epilogue
constexpr int kPfThreads = (kPfDeq0 + kPfDeqWarps + kPfEpiWarps) * 32;
constexpr int kPfBAtom = kPfNmax * 128;              // one 64-column atom of B: 16 KB
constexpr int kPfBTile = 2 * kPfBAtom;               // B slot: 2 atoms, 32 KB
constexpr int kPfOpBytes = kPfSS * kPfBTile;
constexpr int kPfStgBytes = kPfM * 512;              // epilogue staging: 128 rows x 256 16-bit values
// TMEM columns: accumulators [0, 256) (two of 128 columns); operand A stages
// [256, 512): stage s, accumulator p, K half hf at 256 + 128 s + 64 p + 32 hf
// (a row's 16-bit K values packed two per 32-bit column)
constexpr int kPfTmemA = 256;
constexpr int kPfTmemCols = 512;
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
// same with operand A in tensor memory (M = 128 lanes, 8 columns per K step of 16)
__device__ __forceinline__ void umma_f16_ts(uint32_t d, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Four K steps for two accumulators (A from TMEM): d0 += A0[k] B[k], d1 +=
// A1[k] B[k] for k = 0..3, in one asm block so nothing is scheduled between
// the MMAs (an MMA blocks its issuing thread while it runs).  `acc` = 0
// overwrites the accumulators at the first K step.
__device__ __forceinline__ void umma4x2_ts(uint32_t d0, uint32_t d1, uint32_t a0, uint32_t a1, uint64_t b0,
                                          uint64_t b1, uint64_t b2, uint64_t b3, uint32_t idesc, uint32_t acc) {
    // operands: %0 a0, %1 a1 (advanced by 8 columns per K step), %2 d0, %3 d1,
    // %4..%7 B descriptors, %8 instruction descriptor, %9 accumulate flag
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.b32 p, %9, 0;\n\t"
        "setp.eq.b32 q, %9, %9;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%2], [%0], %4, %8, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%3], [%1], %4, %8, p;\n\t"
        "add.u32 %0, %0, 8;\n\t"
        "add.u32 %1, %1, 8;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%2], [%0], %5, %8, q;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%3], [%1], %5, %8, q;\n\t"
        "add.u32 %0, %0, 8;\n\t"
        "add.u32 %1, %1, 8;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%2], [%0], %6, %8, q;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%3], [%1], %6, %8, q;\n\t"
        "add.u32 %0, %0, 8;\n\t"
        "add.u32 %1, %1, 8;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%2], [%0], %7, %8, q;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%3], [%1], %7, %8, q;\n\t"
        "}\n"
        : "+r"(a0), "+r"(a1)
        : "r"(d0), "r"(d1), "l"(b0), "l"(b1), "l"(b2), "l"(b3), "r"(idesc), "r"(acc)
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
// 32 lanes x 16 consecutive 32-bit columns, from registers (lane = row)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
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

// Non-blocking test of an mbarrier phase (try_wait may suspend the thread for
// hundreds of cycles when the phase is not complete yet).
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Pipeline wait of the prefill roles: mbarrier.try_wait suspends the thread
// in hardware until the phase completes (or a short time limit passes), so a
// plain loop keeps hand-off latency low; bounded like mbar_wait.
__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_try(bar, parity)) return true;
        if (clock64() - t0 > kWaitLimitCycles) return false;
    }
}

// 2-D tiled TMA load (no multicast): box at (x, y) of `map` -> shared memory,
// completion counted in bytes on `bar`
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128v(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
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
    static constexpr int kPairs = BITS == 3 ? 16 : 16 / BITS;  // pairs per word (3-bit: per 3-word span)
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

// Exact codes of packed pair pi of a half stage row (64 codes in `words`).
// Positions (2 pi, 2 pi + 1) hold (c_m, c_{m + n/2}) of the pi-th span of n
// columns: one word of 32/bits codes, or for 3-bit (a continuous LSB-first
// bit stream, 8 codes per 3 bytes) a 3-word span of 32 codes, whose codes
// are cut out with funnel shifts.
template <typename TA, int BITS, int HW>
__device__ __forceinline__ uint32_t pf_pair(const uint32_t (&words)[HW], int pi) {
    using C = PfCodes<TA, BITS>;
    using P = Pf2<TA>;
    if constexpr (BITS == 3) {
        const int sp = pi >> 4, m = pi & 15;
        const uint32_t w0 = words[3 * sp], w1 = words[3 * sp + 1], w2 = words[3 * sp + 2];
        const int bl = 3 * m, bh = 3 * m + 48;
        const uint32_t lo = bl < 32 ? __funnelshift_r(w0, w1, bl) : __funnelshift_r(w1, w2, bl - 32);
        const uint32_t hi = bh < 64 ? __funnelshift_r(w1, w2, bh - 32) : (w2 >> (bh - 64));
        const uint32_t v = (lo & 7u) | ((hi & 7u) << 16) | P::kMagic;
        return P::fma2(v, P::kOne, P::kNegMagic);
    } else {
        return C::q(C::prep(words[pi / C::kPairs]), pi % C::kPairs);
    }
}

// Weight stream of one block: the producer warp moves the codes of both
// 128-row blocks, stage by stage, into a ring of CR stages, and their scales
// and biases, 8 groups at a time, into a ring of 2 blocks (2-D TMA copies,
// never multicast).  The dequantisation threads read their row from there.
constexpr int kPfScaleSlotBytes = 2 * 2 * kPfM * 16;  // [block][scale|bias][row][8 groups]
template <int BITS, int GS>
struct PfRing {
    static constexpr int CB = 16 * BITS;  // code bytes of one row per stage
    static constexpr int SPB = GS / 16;   // stages per block of 8 groups
    static constexpr int RING = BITS == 2 ? 32 * 1024 : (BITS == 8 ? 64 * 1024 : 48 * 1024);
    static constexpr int CR = RING / (2 * kPfM * CB);
    static_assert(CR >= 2 && SPB >= 2, "rings");
};

template <int BITS, int GS>
constexpr int pf_smem_bytes() {
    return 1024 + kPfOpBytes + kPfStgBytes + PfRing<BITS, GS>::RING + 2 * kPfScaleSlotBytes + 512;
}

// Panel position of column f for a projection quantised with `bits`.
__host__ __device__ __forceinline__ int pf_perm_pos(int f, int bits) {
    const int n = bits == 3 ? 32 : 32 / bits, h = n >> 1;
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
    } else if constexpr (BITS == 3) {
        // span of 32: (2m, 2m+1) <- (m, m + 16); chunk h holds m = 4 (h % 4) .. + 3
        const uint16_t *sp = row64 + (h >> 2) * 32 + (h & 3) * 4;
        const uint2 lo = *reinterpret_cast<const uint2 *>(sp);
        const uint2 hi = *reinterpret_cast<const uint2 *>(sp + 16);
        o.x = __byte_perm(lo.x, hi.x, 0x5410);
        o.y = __byte_perm(lo.x, hi.x, 0x7632);
        o.z = __byte_perm(lo.y, hi.y, 0x5410);
        o.w = __byte_perm(lo.y, hi.y, 0x7632);
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
        if (j < ch.ntok)
            src = a.x + (size_t)route_row(a.sorted_routes[ch.route_start + j], a.route_div, a.shared_base) *
                            (a.x_stride ? a.x_stride : a.K);
        for (int at = a0; at < a1; ++at) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (src) v = pf_perm_chunk<BITS>(src + at * 64, h);
            *reinterpret_cast<uint4 *>(a.panel + pf_panel_off(pr, at * 64 + h * 8, a.prow)) = v;
        }
    }
}

// out[t] = sum over j < k, in route order, of the fp32 values of yw[t*k + j],
// rounded once (the combine of arena.py:619-624 as the decode kernels do it);
// then the shared expert's row yw[shared_base + t] and the residual, each
// followed by a rounding (combine_finish).
template <typename TA>
__global__ void __launch_bounds__(256) pf_combine_kernel(const uint16_t *yw, int T, int H, int k, uint16_t *out,
                                                         int shared_base, const uint16_t *residual) {
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
    if (shared_base > 0 || residual) {
        uint4 s4 = make_uint4(0u, 0u, 0u, 0u), r4 = make_uint4(0u, 0u, 0u, 0u);
        if (shared_base > 0)
            s4 = *reinterpret_cast<const uint4 *>(yw + ((size_t)(shared_base + t) * H + (size_t)cc * 8));
        if (residual) r4 = *reinterpret_cast<const uint4 *>(residual + (size_t)t * H + (size_t)cc * 8);
        const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w}, rw[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint16_t sv = static_cast<uint16_t>(e & 1 ? sw[e >> 1] >> 16 : sw[e >> 1] & 0xFFFFu);
            const uint16_t rv = static_cast<uint16_t>(e & 1 ? rw[e >> 1] >> 16 : rw[e >> 1] & 0xFFFFu);
            acc[e] = combine_finish<TA>(acc[e], shared_base > 0, sv, residual != nullptr, rv);
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
__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_kernel(const __grid_constant__ PfArgs a) {
    using RG = PfRing<BITS, GS>;
    using C = PfCodes<TA, BITS>;
    using P = Pf2<TA>;
    constexpr int HW = RG::CB / 8;           // code words of half a row per stage (64 weights)
    constexpr int CPW = 32 / BITS;           // codes per word
    static_assert(HW * 32 / BITS == 64, "half a stage row is 64 weights");
    constexpr bool kF16 = std::is_same<TA, __half>::value;
    constexpr int CSTAGE = 2 * kPfM * RG::CB;  // code bytes of one ring stage

    extern __shared__ __align__(1024) uint8_t pf_raw[];
    uint8_t *smem = pf_raw + ((1024u - (smem_u32(pf_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t stg = sbase + kPfOpBytes;
    const uint32_t cring = stg + kPfStgBytes;
    const uint32_t sring = cring + RG::RING;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kPfOpBytes + kPfStgBytes + RG::RING + 2 * kPfScaleSlotBytes);
    // stage s: operand A written (dequantisation warps), operand B landed
    // (bulk copies), stage free again (one tcgen05.commit after its MMAs)
    uint64_t *full_a = bars;
    uint64_t *full_b = full_a + kPfSS;
    uint64_t *empty = full_b + kPfSS;
    uint64_t *acc_full = empty + kPfSS;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *drain = acc_empty + 1;
    uint64_t *code_full = drain + 1;
    uint64_t *code_empty = code_full + RG::CR;
    uint64_t *sc_full = code_empty + RG::CR;
    uint64_t *sc_empty = sc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kPfSS; ++s) {
            mbar_init(&full_a[s], kPfDeqWarps);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kPfEpiWarps);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sc_full[b], 1);
            mbar_init(&sc_empty[b], kPfDeqWarps);
        }
        for (int c = 0; c < RG::CR; ++c) {
            mbar_init(&code_full[c], 1);
            mbar_init(&code_empty[c], kPfDeqWarps);
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
            const size_t kstride = (size_t)(a.prow >> 3) * 1024u;  // one 64-column atom of the panel
            int sb = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
                if (*abort_flag) break;
                const int c = item / a.rbn;
                const Chunk ch = a.chunks[c];
                const uint32_t bytes = (uint32_t)((ch.ntok + 15) & ~15) * 128u;
                const uint8_t *src = a.panel + (size_t)(pf_row_base(ch.route_start, c) >> 3) * 1024u;
                for (int ks = 0; ks < KS; ++ks) {
                    if (!pf_wait(&empty[sb], ph ^ 1u)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full_b[sb], 2u * bytes);
                    uint8_t *dst = smem + sb * kPfBTile;
                    bulk_g2s(dst, src + (size_t)(2 * ks) * kstride, bytes, &full_b[sb]);
                    bulk_g2s(dst + kPfBAtom, src + (size_t)(2 * ks + 1) * kstride, bytes, &full_b[sb]);
                    if (++sb == kPfSS) {
                        sb = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok) {
                *abort_flag = 1;
                set_error(a.err, -4);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        // An MMA blocks its issuing thread for its whole duration (52 cycles
        // below N = 104, N / 2 above), a tcgen05.commit for about 256 and an
        // mbarrier.try_wait on an incomplete phase for several hundred
        // (measured on B200).  So one commit per stage, and the next stage's
        // barriers are polled between this stage's MMAs with the non-blocking
        // test_wait.
        if (lane == 0) {
            int it = 0, s = 0;
            uint32_t ph = 0;
            bool ok = true;
            const uint64_t db_base = sw128_desc(sbase);
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x, ++it) {
                if (*abort_flag) break;
                const Chunk ch = a.chunks[item / a.rbn];
                const uint32_t idesc = idesc_f16((ch.ntok + 15) & ~15, kF16);
                // the accumulators are free once the epilogue has copied out the previous item
                if (!pf_wait(acc_empty, (it & 1) ^ 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                bool ready = false;  // this stage's operands known to be in place
                for (int ks = 0; ks < KS; ++ks) {
                    if (!ready && (!pf_wait(&full_b[s], ph) || !pf_wait(&full_a[s], ph))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = tmem + (uint32_t)(kPfTmemA + s * 128), a1 = a0 + 64u;
                    const uint64_t db = db_base + (uint64_t)(s * (kPfBTile >> 4));
                    // B: 32 bytes per K step along the swizzled row; K 64..127 in the second atom
                    const uint64_t dbh = db + (uint64_t)(kPfBAtom >> 4);
                    umma4x2_ts(tmem, tmem + 128u, a0, a1, db, db + 2u, db + 4u, db + 6u, idesc, ks ? 1u : 0u);
                    umma4x2_ts(tmem, tmem + 128u, a0 + 32u, a1 + 32u, dbh, dbh + 2u, dbh + 4u, dbh + 6u, idesc, 1u);
                    const int ns = s + 1 == kPfSS ? 0 : s + 1;
                    const uint32_t nph = ns == 0 ? ph ^ 1u : ph;
                    ready = ks + 1 < KS && mbar_test(&full_b[ns], nph) && mbar_test(&full_a[ns], nph);
                    umma_commit(&empty[s]);
                    s = ns;
                    ph = nph;
                }
                if (!ok) break;
                umma_commit(acc_full);
            }
            if (!ok) {
                *abort_flag = 1;
                set_error(a.err, -4);
            }
            // nothing may still write TMEM when it is freed
            umma_commit(drain);
            if (!mbar_wait(drain, 0)) set_error(a.err, -4);
        }
    } else if (warp == 2) {
        // ---------------------------------------------------- weight stream producer
        if (lane == 0) {
            int g = 0, nb = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
                if (*abort_flag) break;
                const int c = item / a.rbn, rb = item - c * a.rbn;
                const int y0 = a.chunks[c].slot * a.wrows;
                const int y[2] = {MODE == PF_GATEUP ? y0 + rb * kPfM : y0 + rb * 2 * kPfM,
                                  MODE == PF_GATEUP ? y0 + rb * kPfM : y0 + rb * 2 * kPfM + kPfM};
                for (int ks = 0; ks < KS; ++ks, ++g) {
                    if (ks % RG::SPB == 0) {
                        const int j = nb & 1;
                        if (!pf_wait(&sc_empty[j], ((nb >> 1) & 1) ^ 1)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(&sc_full[j], kPfScaleSlotBytes);
                        const uint32_t sd = sring + (uint32_t)(j * kPfScaleSlotBytes);
#pragma unroll
                        for (int p = 0; p < 2; ++p) {
                            tma_load_2d(sd + p * 4096, &a.tm_scale[p], (ks / RG::SPB) * 8, y[p], &sc_full[j]);
                            tma_load_2d(sd + p * 4096 + 2048, &a.tm_bias[p], (ks / RG::SPB) * 8, y[p], &sc_full[j]);
                        }
                        ++nb;
                    }
                    const int cs = g % RG::CR;
                    if (!pf_wait(&code_empty[cs], ((g / RG::CR) & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&code_full[cs], CSTAGE);
#pragma unroll
                    for (int p = 0; p < 2; ++p)
                        tma_load_2d(cring + (uint32_t)(cs * CSTAGE + p * kPfM * RG::CB), &a.tm_code[p], ks * RG::CB,
                                    y[p], &code_full[cs]);
                }
            }
            if (!ok) {
                *abort_flag = 1;
                set_error(a.err, -4);
            }
        }
    } else if (warp < kPfDeq0 + kPfDeqWarps) {
        // ---------------------------------------------------- dequantisation (operand A)
        // thread = (accumulator p, K half hf, row r): 64 weights of one row
        // per stage.  A warp reaches only its quarter of the TMEM lanes
        // (warp % 4): rows 32 * (warp % 4) + lane; the 16 warps cover
        // (p, hf) x 4 quarters.
        const int wi = (warp - kPfDeq0) >> 2;
        const int p = wi >> 1, hf = wi & 1, r = (warp & 3) * 32 + lane;
        const uint32_t arow = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(kPfTmemA + p * 64 + hf * 32);
        const uint32_t crow = cring + (uint32_t)(p * kPfM * RG::CB + r * RG::CB + hf * (RG::CB / 2));
        const uint32_t srow = sring + (uint32_t)(p * 4096 + r * 16);
        int g = 0, nb = 0;
        uint4 sreg = make_uint4(0u, 0u, 0u, 0u), breg = make_uint4(0u, 0u, 0u, 0u);
        bool ok = true;
        for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
            if (*abort_flag) break;
            for (int ks = 0; ks < KS; ++ks, ++g) {
                if (ks % RG::SPB == 0) {
                    // scales and biases of this row for the next 8 groups
                    const int j = nb & 1;
                    if (!pf_wait(&sc_full[j], (nb >> 1) & 1)) {
                        ok = false;
                        break;
                    }
                    sreg = lds128(srow + (uint32_t)(j * kPfScaleSlotBytes));
                    breg = lds128(srow + (uint32_t)(j * kPfScaleSlotBytes + 2048));
                    ++nb;
                }
                const int cs = g % RG::CR;
                if (!pf_wait(&code_full[cs], (g / RG::CR) & 1)) {
                    ok = false;
                    break;
                }
                uint32_t words[HW];
                if constexpr (HW % 4 == 0) {
#pragma unroll
                    for (int i = 0; i < HW / 4; ++i) {
                        const uint4 v = lds128(crow + (uint32_t)(cs * CSTAGE + 16 * i));
                        words[4 * i] = v.x;
                        words[4 * i + 1] = v.y;
                        words[4 * i + 2] = v.z;
                        words[4 * i + 3] = v.w;
                    }
                } else {  // 3-bit: 24 bytes
#pragma unroll
                    for (int i = 0; i < HW / 2; ++i) {
                        const uint2 v = lds64(crow + (uint32_t)(cs * CSTAGE + 8 * i));
                        words[2 * i] = v.x;
                        words[2 * i + 1] = v.y;
                    }
                }
                const int s = g % kPfSS;
                if (!pf_wait(&empty[s], ((g / kPfSS) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // scale and bias variants of the groups this half row covers
                // (64 columns: one group, two for GS = 32, half of one for 128)
                constexpr int NG = GS < 64 ? 2 : 1;
                const int gi = ((ks % RG::SPB) * kPfKS + hf * (kPfKS / 2)) / GS;
                uint32_t sp[NG][3], b2[NG];
#pragma unroll
                for (int gg = 0; gg < NG; ++gg) {
                    const int q = gi + gg;
                    const uint32_t sw = (q & 4) ? ((q & 2) ? sreg.w : sreg.z) : ((q & 2) ? sreg.y : sreg.x);
                    const uint32_t bw = (q & 4) ? ((q & 2) ? breg.w : breg.z) : ((q & 2) ? breg.y : breg.x);
                    const int sh = (q & 1) * 16;
                    const uint32_t s16 = (sw >> sh) & 0xFFFFu, bb16 = (bw >> sh) & 0xFFFFu;
                    b2[gg] = bb16 | (bb16 << 16);
                    sp[gg][0] = s16 | (s16 << 16);
                    if constexpr (C::kPrescale) {
                        sp[gg][1] = P::fma2(sp[gg][0], P::kQuarter, P::kNegZero);
                        sp[gg][2] = P::fma2(sp[gg][0], P::kSixteenth, P::kNegZero);
                    } else {
                        sp[gg][1] = sp[gg][2] = sp[gg][0];
                    }
                }
                // 32 packed pairs in 4 stores of 8 TMEM columns
                const uint32_t adst = arow + (uint32_t)(s * 128);
#pragma unroll
                for (int blk = 0; blk < 4; ++blk) {
                    uint32_t pr[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        // span of the pair: one word (3-bit: 3 words of 32 codes)
                        constexpr int SC = BITS == 3 ? 32 : CPW;
                        const int pi = blk * 8 + i;
                        const int gg = NG == 2 ? ((pi / (SC / 2)) * SC) / GS : 0;
                        pr[i] = P::fma2(pf_pair<TA, BITS, HW>(words, pi), sp[gg][C::pexp(pi % C::kPairs)], b2[gg]);
                    }
                    tmem_st8(adst + (uint32_t)(8 * blk), pr);
                }
                tmem_wait_st();
                // the generic-proxy reads of the code and scale slots must be
                // ordered before their TMA refills (without this fence a refill
                // could land before those reads, measured on B200)
                fence_proxy_async();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&full_a[s]);
                    mbar_arrive(&code_empty[cs]);
                    if (ks % RG::SPB == 0) mbar_arrive(&sc_empty[(nb - 1) & 1]);
                }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            set_error(a.err, -4);
        }
    } else {
        // ---------------------------------------------------- epilogue
        // Copies the item's accumulators out of TMEM into shared memory,
        // rounded to the activation dtype (the first operation of both
        // epilogues), frees TMEM for the next item, then finishes the item
        // from shared memory while the next item's MMAs run.  Thread = row r
        // (TMEM lane; a warp reaches its own quarter): staging row r holds
        // 32 chunks of 8 values (accumulator 0 in chunks 0-15, 1 in 16-31),
        // chunk c at position c ^ (r & 31).
        const int q4 = warp & 3;
        const int hc = (warp - kPfDeq0 - kPfDeqWarps) >> 2;  // this warp's 16-column chunks: (j0 / 16) % 2 == hc
        const int r = q4 * 32 + lane;
        const uint32_t srow_e = stg + (uint32_t)(r * 512);
        const int rx = r & 31;
        int it = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < items; item += gridDim.x, ++it) {
            if (*abort_flag) break;
            const int c = item / a.rbn, rb = item - c * a.rbn;
            const Chunk ch = a.chunks[c];
            const int N = (ch.ntok + 15) & ~15;
            if (!pf_wait(acc_full, it & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t t0 = tmem + ((uint32_t)(q4 * 32) << 16);
            for (int j0 = 16 * hc; j0 < N; j0 += 32) {
                uint32_t v0[16], v1[16];
                tmem_ld16(t0 + (uint32_t)j0, v0);
                tmem_ld16(t0 + 128u + (uint32_t)j0, v1);
                tmem_wait_ld(v0);
                tmem_wait_ld(v1);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int cc = (j0 >> 3) + h;
                    const uint32_t *u0 = v0 + 8 * h, *u1 = v1 + 8 * h;
                    sts128v(srow_e + (uint32_t)(((cc) ^ rx) << 4),
                            Act<TA>::pack2(__uint_as_float(u0[0]), __uint_as_float(u0[1])),
                            Act<TA>::pack2(__uint_as_float(u0[2]), __uint_as_float(u0[3])),
                            Act<TA>::pack2(__uint_as_float(u0[4]), __uint_as_float(u0[5])),
                            Act<TA>::pack2(__uint_as_float(u0[6]), __uint_as_float(u0[7])));
                    sts128v(srow_e + (uint32_t)(((16 + cc) ^ rx) << 4),
                            Act<TA>::pack2(__uint_as_float(u1[0]), __uint_as_float(u1[1])),
                            Act<TA>::pack2(__uint_as_float(u1[2]), __uint_as_float(u1[3])),
                            Act<TA>::pack2(__uint_as_float(u1[4]), __uint_as_float(u1[5])),
                            Act<TA>::pack2(__uint_as_float(u1[6]), __uint_as_float(u1[7])));
                }
            }
            // TMEM is free for the next item's MMAs
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
            if constexpr (MODE == PF_GATEUP) {
                const int f = rb * kPfM + r;
                const int kp = pf_perm_pos(f, a.hbits);
                const int pbase = pf_row_base(ch.route_start, c);
                for (int j0 = 16 * hc; j0 < N; j0 += (j0 & 8) ? 24 : 8) {
                    const uint4 gq = lds128(srow_e + (uint32_t)(((j0 >> 3) ^ rx) << 4));
                    const uint4 uq = lds128(srow_e + (uint32_t)(((16 + (j0 >> 3)) ^ rx) << 4));
                    const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w}, uw[4] = {uq.x, uq.y, uq.z, uq.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int j = j0 + i;
                        float h = 0.0f;
                        if (j < ch.ntok) {
                            const float gv = Act<TA>::to_f((uint16_t)(i & 1 ? gw[i >> 1] >> 16 : gw[i >> 1] & 0xFFFFu));
                            const float uv = Act<TA>::to_f((uint16_t)(i & 1 ? uw[i >> 1] >> 16 : uw[i >> 1] & 0xFFFFu));
                            h = swiglu_h<TA>(gv, uv, a.limit, a.swiglu_mode);
                        }
                        *reinterpret_cast<uint16_t *>(a.hpanel + pf_panel_off(pbase + j, kp, a.hprow)) =
                            Act<TA>::from_f(h);
                    }
                }
            } else {
#pragma unroll 1
                for (int pp = 0; pp < 2; ++pp) {
                    const int f = rb * 2 * kPfM + pp * kPfM + r;
                    for (int j0 = 16 * hc; j0 < N; j0 += (j0 & 8) ? 24 : 8) {
                        // route and combine weight of column j0 + (lane & 7)
                        const int jl = j0 + (lane & 7);
                        int my_route = 0;
                        float my_w = 0.0f;
                        if (jl < ch.ntok) {
                            my_route = a.sorted_routes[ch.route_start + jl];
                            my_w = a.route_w[my_route];
                        }
                        const uint4 yq = lds128(srow_e + (uint32_t)(((pp * 16 + (j0 >> 3)) ^ rx) << 4));
                        const uint32_t yw4[4] = {yq.x, yq.y, yq.z, yq.w};
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int route = __shfl_sync(0xffffffffu, my_route, i);
                            const float wv = __shfl_sync(0xffffffffu, my_w, i);
                            if (j0 + i < ch.ntok) {
                                const float y = Act<TA>::to_f((uint16_t)(i & 1 ? yw4[i >> 1] >> 16 : yw4[i >> 1] & 0xFFFFu));
                                a.yw[(size_t)route * a.H + f] = Act<TA>::from_f(y * Act<TA>::round(wv));
                            }
                        }
                    }
                }
            }
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
    LMOE_PF_CASE(3, 32)
    LMOE_PF_CASE(3, 64)
    LMOE_PF_CASE(3, 128)
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

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

cudaError_t map2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t dim0, uint64_t dim1,
                  uint64_t stride1, uint32_t box0, uint32_t box1) {
    if (!g_encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess) return e;
        if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dims[2] = {dim0, dim1};
    const cuuint64_t strides[1] = {stride1};
    const cuuint32_t box[2] = {box0, box1};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = g_encode(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}
}  // namespace

cudaError_t pf_prepare(PfArgs &a, int mode, const QView &q0, const QView &q1, int bits, int gs, int n_slots) {
    (void)gs;
    const QView *qs[2] = {&q0, mode == PF_GATEUP ? &q1 : &q0};
    for (int p = 0; p < 2; ++p) {
        const QView &q = *qs[p];
        const uint64_t rows = (uint64_t)n_slots * (uint64_t)q.rows;
        const uint64_t row_bytes = (uint64_t)q.words_per_row * 4u, G = (uint64_t)q.groups_per_row;
        cudaError_t e = map2d(&a.tm_code[p], CU_TENSOR_MAP_DATA_TYPE_UINT8, q.w, row_bytes, rows, row_bytes,
                              (uint32_t)(kPfKS * bits / 8), (uint32_t)kPfM);
        if (e == cudaSuccess)
            e = map2d(&a.tm_scale[p], CU_TENSOR_MAP_DATA_TYPE_UINT16, q.s, G, rows, G * 2u, 8u, (uint32_t)kPfM);
        if (e == cudaSuccess)
            e = map2d(&a.tm_bias[p], CU_TENSOR_MAP_DATA_TYPE_UINT16, q.b, G, rows, G * 2u, 8u, (uint32_t)kPfM);
        if (e != cudaSuccess) return e;
    }
    a.wrows = q0.rows;
    return cudaSuccess;
}

// K a multiple of 64 and of 8 groups (16-byte scale blocks), rows a multiple
// of 128 (gate/up) or 256 (down), and a compiled (bits, group) pair.
bool pf_supported(int K, int rows, int bits, int gs, int mode) {
    const bool bg = (bits == 2 && (gs == 64 || gs == 128)) || (bits == 3 && (gs == 32 || gs == 64 || gs == 128)) ||
                    ((bits == 4 || bits == 8) && (gs == 32 || gs == 64 || gs == 128));
    if (!bg) return false;
    if (K <= 0 || K % kPfKS != 0 || K % (8 * gs) != 0) return false;  // (kPfKS = 128)
    return rows > 0 && rows % (mode == PF_GATEUP ? kPfM : 2 * kPfM) == 0;
}

cudaError_t launch_pf_panel(const PfPanelArgs &a, int max_chunks, cudaStream_t st) {
    if (max_chunks < 1) return cudaSuccess;
    const int atoms = a.K / 64;
    dim3 grid(static_cast<unsigned>(max_chunks), static_cast<unsigned>((atoms + kPfPanelAtoms - 1) / kPfPanelAtoms));
    if (a.bits == 2) return launch_pdl(pf_panel_kernel<2>, grid, dim3(256), 0, st, a);
    if (a.bits == 3) return launch_pdl(pf_panel_kernel<3>, grid, dim3(256), 0, st, a);
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
                              cudaStream_t st, int shared_base, const uint16_t *residual) {
    const long n = (long)T * (H / 8);
    if (n <= 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>((n + 255) / 256));
    if (act_f16)
        return launch_pdl(pf_combine_kernel<__half>, grid, dim3(256), 0, st, yw, T, H, top_k, out, shared_base,
                          residual);
    return launch_pdl(pf_combine_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, yw, T, H, top_k, out, shared_base,
                      residual);
}

}  // namespace lmoe
