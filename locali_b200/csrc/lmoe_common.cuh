// Device helpers shared by the routed-MoE kernels (sm_100a).
//
// Decode GEMV design: weights stay in the reference's MLX layout
// (uint32 codes LSB-first, dsv4_kernels.py:135-150).  Each warp owns a
// 16-row tile of a projection and feeds register operands to the tensor
// pipe: codes are unpacked with LOP3 magic-number tricks into exact
// small integers (bf16/f16), multiplied against activations by
// mma.m16n8k16 with fp32 accumulation, and every quantisation group's fp32
// dot product is then scaled: acc += scale*dot + bias*sum(x), exactly the
// arithmetic of dsv4_kernels.py:152-154 (no bf16 rounding of dequantised
// weights).
//
// The activation operand is pre-permuted ("panel" layout) so that the column
// order the code unpacker produces is matched by one 8-byte load per lane per
// k-step, and 2-bit activations are pre-scaled by 4^-p so that codes can be
// extracted in place (value c*4^p) without a shift.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lmoe {

constexpr int kChunkTok = 8;  // tokens per chunk = the n-dimension of one MMA

// Dispatch output: one chunk = up to 8 routes of the same expert.
struct Chunk {
    int32_t slot;         // arena slot of the expert
    int32_t route_start;  // first index into sorted_routes
    int32_t ntok;         // routes in this chunk (1..8)
    int32_t expert;       // expert id (bucket)
};

// Device view of one projection of all slots.
struct QView {
    const uint32_t *w;
    const uint16_t *s;
    const uint16_t *b;
    int64_t w_slot_stride;   // words per slot
    int64_t sb_slot_stride;  // scale elements per slot
    int32_t words_per_row;
    int32_t groups_per_row;
    int32_t rows;
    int32_t cols;
    // optional pre-tiled copy ([slot][rows/16][tile_bytes], see TileGeo):
    // when set, the GEMV streams whole tiles with bulk copies
    const uint8_t *tiles;
    int64_t tile_slot_stride;  // bytes per slot
};

// ------------------------------------------------------------ dtype traits
template <typename TA>
struct Act;

template <>
struct Act<__nv_bfloat16> {
    static constexpr uint32_t kMagic = 0x43004300u;  // (128, 128)
    static constexpr float kMagicVal = 128.0f;
    __device__ __forceinline__ static float to_f(uint16_t v) {
        return __uint_as_float(static_cast<uint32_t>(v) << 16);
    }
    __device__ __forceinline__ static uint16_t from_f(float v) {
        __nv_bfloat16 h = __float2bfloat16_rn(v);
        return *reinterpret_cast<uint16_t *>(&h);
    }
    __device__ __forceinline__ static float round(float v) { return to_f(from_f(v)); }
    __device__ __forceinline__ static uint32_t sub_magic(uint32_t v) {
        __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162 *>(&v);
        __nv_bfloat162 r = __hsub2(a, __floats2bfloat162_rn(kMagicVal, kMagicVal));
        return *reinterpret_cast<uint32_t *>(&r);
    }
    __device__ __forceinline__ static uint32_t pack2(float lo, float hi) {
        __nv_bfloat162 r = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&r);
    }
    __device__ __forceinline__ static void mma(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
};

template <>
struct Act<__half> {
    static constexpr uint32_t kMagic = 0x64006400u;  // (1024, 1024)
    static constexpr float kMagicVal = 1024.0f;
    __device__ __forceinline__ static float to_f(uint16_t v) {
        return __half2float(*reinterpret_cast<__half *>(&v));
    }
    __device__ __forceinline__ static uint16_t from_f(float v) {
        __half h = __float2half_rn(v);
        return *reinterpret_cast<uint16_t *>(&h);
    }
    __device__ __forceinline__ static float round(float v) { return to_f(from_f(v)); }
    __device__ __forceinline__ static uint32_t sub_magic(uint32_t v) {
        __half2 a = *reinterpret_cast<__half2 *>(&v);
        __half2 r = __hsub2(a, __floats2half2_rn(kMagicVal, kMagicVal));
        return *reinterpret_cast<uint32_t *>(&r);
    }
    __device__ __forceinline__ static uint32_t pack2(float lo, float hi) {
        __half2 r = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&r);
    }
    __device__ __forceinline__ static void mma(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
};

// Clamped SwiGLU of one (gate, up) pair of fp32 accumulators
// (dsv4_arena.py:223-235): both rounded to the activation dtype first, then
// up clamped to [-L, L] and gate to min(gate, L) when L > 0.  Mode 0 takes
// silu in fp32 with one rounding of silu * up (dsv4_kernels.py:165-170);
// mode 1 rounds op by op in the activation dtype (nn.silu(gate) * up).
template <typename TA>
__device__ __forceinline__ float swiglu_h(float gacc, float uacc, float limit, int mode) {
    float gv = Act<TA>::round(gacc);
    float uv = Act<TA>::round(uacc);
    if (limit > 0.0f) {
        uv = fminf(fmaxf(uv, -limit), limit);
        gv = fminf(gv, limit);
    }
    if (mode == 0) return Act<TA>::round((gv / (1.0f + expf(-gv))) * uv);
    const float sig = Act<TA>::round(1.0f / (1.0f + expf(-gv)));
    return Act<TA>::round(Act<TA>::round(gv * sig) * uv);
}

// ------------------------------------------------------------ code geometry
template <int BITS, int GS>
struct Geo {
    static_assert(BITS == 2 || BITS == 4 || BITS == 8, "bits");
    static constexpr int kCpw = 32 / BITS;           // codes per 32-bit word
    static constexpr int kSlice = GS / 4;            // columns per lane slice
    static constexpr int kWps = kSlice / kCpw;       // words per lane slice
    static constexpr int kStepsPerWord = kCpw / 4;   // k16 steps per word
    static constexpr int kSteps = GS / 16;           // k16 steps per group
    static constexpr int kWordsPerGroup = GS * BITS / 32;
    static_assert(kWps >= 1 && kSlice % kCpw == 0, "lane slice must be whole words");
};

// 2-bit prescale exponents of the eight in-word pairs (value c*4^p).
__host__ __device__ __forceinline__ int pmap2(int m) {
    return m % 3;  // 0,1,2,0,1,2,0,1
}

// Panel position and 4^-p prescale exponent of column `col` for a consumer
// quantised with (bits, gs).  Runtime version (used by producers).
__host__ __device__ __forceinline__ int panel_pos(int col, int bits, int gs, int *p_out) {
    const int G = col / gs, i = col - G * gs;
    const int slice = gs >> 2;
    const int t = i / slice, ii = i - t * slice;
    const int cpw = 32 / bits;
    const int wi = ii / cpw, j = ii - wi * cpw;
    const int half_n = cpw >> 1;
    const int m = j % half_n, half = j / half_n;
    const int s = wi * (cpw >> 2) + (m >> 1);
    const int reg = m & 1;
    *p_out = (bits == 2) ? pmap2(m) : 0;
    // [group][lane slot t][k-step s][4 values]: one lane's steps are contiguous
    return (((G * 4 + t) * (gs >> 4) + s) * 4) + reg * 2 + half;
}

// Unpack one 32-bit word of codes into kCpw/2 pairs of exact small integers
// (as packed 16-bit activation values).  Pair m holds (c_m, c_{m+kCpw/2}).
template <typename TA, int BITS>
struct Unpack;

template <typename TA>
struct Unpack<TA, 2> {
    __device__ __forceinline__ static void run(uint32_t w, uint32_t (&P)[8]) {
        constexpr uint32_t M = Act<TA>::kMagic;
        const uint32_t v1 = w >> 6, v2 = w >> 12;
        P[0] = (w & 0x00030003u) | M;
        P[1] = (w & 0x000C000Cu) | M;
        P[2] = (w & 0x00300030u) | M;
        P[3] = (v1 & 0x00030003u) | M;
        P[4] = (v1 & 0x000C000Cu) | M;
        P[5] = (v1 & 0x00300030u) | M;
        P[6] = (v2 & 0x00030003u) | M;
        P[7] = (v2 & 0x000C000Cu) | M;
#pragma unroll
        for (int m = 0; m < 8; ++m) P[m] = Act<TA>::sub_magic(P[m]);
    }
};

template <typename TA>
struct Unpack<TA, 4> {
    __device__ __forceinline__ static void run(uint32_t w, uint32_t (&P)[4]) {
        constexpr uint32_t M = Act<TA>::kMagic;
        P[0] = (w & 0x000F000Fu) | M;
        P[1] = ((w >> 4) & 0x000F000Fu) | M;
        P[2] = ((w >> 8) & 0x000F000Fu) | M;
        P[3] = ((w >> 12) & 0x000F000Fu) | M;
#pragma unroll
        for (int m = 0; m < 4; ++m) P[m] = Act<TA>::sub_magic(P[m]);
    }
};

template <typename TA>
struct Unpack<TA, 8> {
    __device__ __forceinline__ static void run(uint32_t w, uint32_t (&P)[2]) {
        const float c0 = __uint_as_float(0x4B000000u | (w & 0xFFu)) - 8388608.0f;
        const float c1 = __uint_as_float(0x4B000000u | ((w >> 8) & 0xFFu)) - 8388608.0f;
        const float c2 = __uint_as_float(0x4B000000u | ((w >> 16) & 0xFFu)) - 8388608.0f;
        const float c3 = __uint_as_float(0x4B000000u | (w >> 24)) - 8388608.0f;
        P[0] = Act<TA>::pack2(c0, c2);
        P[1] = Act<TA>::pack2(c1, c3);
    }
};

// On-demand pair extraction for the MMA A operand.  prep() runs once per code
// word, get(w, m) yields pair m (c_m, c_{m+kCpw/2}) as packed 16-bit values.
// bf16, 2- and 4-bit codes: the pair keeps the magic offset (value 128 +
// c*4^p resp. 128 + c) and the consumer removes 128 * sum(panel) per group
// after the MMA (kFoldOffset); the cancellation costs about 7 of fp32's 24
// bits, far below bf16 output precision.  f16: the offset is 1024 and the
// 10 lost bits would show in f16 outputs, so the magic is subtracted from
// every pair (exact small integers) instead.
template <typename TA>
struct FoldOffset {
    static constexpr bool value = false;
};
template <>
struct FoldOffset<__nv_bfloat16> {
    static constexpr bool value = true;
};

template <typename TA, int BITS>
struct PairX;

// (v & mask) | magic as one three-input logic operation (LUT 0xEA = a & b | c).
__device__ __forceinline__ uint32_t and_or(uint32_t v, uint32_t mask, uint32_t magic) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "r"(mask), "r"(magic));
    return r;
}

template <typename TA>
struct PairX<TA, 2> {
    struct W {
        uint32_t v0, v1, v2;
    };
    __device__ __forceinline__ static W prep(uint32_t w) { return W{w, w >> 6, w >> 12}; }
    __device__ __forceinline__ static uint32_t get(const W &w, int m) {
        const uint32_t v = m < 3 ? w.v0 : (m < 6 ? w.v1 : w.v2);
        const uint32_t r = and_or(v, 0x00030003u << (2 * (m % 3)), Act<TA>::kMagic);
        return FoldOffset<TA>::value ? r : Act<TA>::sub_magic(r);
    }
};

template <typename TA>
struct PairX<TA, 4> {
    using W = uint32_t;
    __device__ __forceinline__ static W prep(uint32_t w) { return w; }
    __device__ __forceinline__ static uint32_t get(W w, int m) {
        const uint32_t r = and_or(w >> (4 * m), 0x000F000Fu, Act<TA>::kMagic);
        return FoldOffset<TA>::value ? r : Act<TA>::sub_magic(r);
    }
};

template <typename TA>
struct PairX<TA, 8> {
    using W = uint32_t;
    __device__ __forceinline__ static W prep(uint32_t w) { return w; }
    __device__ __forceinline__ static uint32_t get(W w, int m) {
        // exact small integers through the fp32 magic 2^23
        const float lo = __uint_as_float(0x4B000000u | ((w >> (8 * m)) & 0xFFu)) - 8388608.0f;
        const float hi = __uint_as_float(0x4B000000u | ((w >> (8 * m + 16)) & 0xFFu)) - 8388608.0f;
        return Act<TA>::pack2(lo, hi);
    }
};

// ------------------------------------------------------------ memory helpers
__device__ __forceinline__ uint32_t ldg_nc_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldg_nc_u64(const uint32_t *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ldg_nc_u128(const uint32_t *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ldg_u16(const uint16_t *p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// Loads the lane's slice words (WPS of them) of one row for one group.
template <int WPS>
struct SliceLoad {
    __device__ __forceinline__ static void run(const uint32_t *p, uint32_t (&w)[WPS]) {
        if constexpr (WPS == 1) {
            w[0] = ldg_nc_u32(p);
        } else if constexpr (WPS == 2) {
            uint2 v = ldg_nc_u64(p);
            w[0] = v.x;
            w[1] = v.y;
        } else {
#pragma unroll
            for (int q = 0; q < WPS / 4; ++q) {
                uint4 v = ldg_nc_u128(p + 4 * q);
                w[4 * q + 0] = v.x;
                w[4 * q + 1] = v.y;
                w[4 * q + 2] = v.z;
                w[4 * q + 3] = v.w;
            }
        }
    }
};

// ------------------------------------------------------------ mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
// Adds expected transaction bytes to the current phase without an arrival.
__device__ __forceinline__ void mbar_add_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Wait on an mbarrier phase, bounded (kWaitLimitCycles of the SM clock,
// about 2 s).  Returns false if the wait gave up; the caller records an error
// and stops instead of hanging the GPU.  Between polls the warp sleeps (32 ns
// doubling to 256 ns): a warp polling flat out takes issue slots from the
// warps of its sub-partition that do the math.  The bound is kept on clock64,
// which is cheap to read, rather than on the global timer.
constexpr long long kWaitLimitCycles = 4000000000ll;
__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    uint32_t ns = 32;
    for (;;) {
        __nanosleep(ns);
        if (mbar_try(bar, parity)) return true;
        if (ns < 256) ns <<= 1;
        if (clock64() - t0 > kWaitLimitCycles) return false;
    }
}

// Bulk copy global -> shared with an L2 cache policy (streamed weights use
// evict-first, so the layer's small hot data keeps its L2 lines).
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// 16-byte read-only global load with an L2 cache policy.
__device__ __forceinline__ uint4 ldg_u128_hint(const void *p, uint64_t policy) {
    uint4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(policy));
    return v;
}

// XOR swizzle of 16-byte chunks inside each 128-byte line of a shared-memory
// tile: rows stay contiguous (so 16-byte cp.async of a row writes whole lines)
// while the consumers' per-row reads land in distinct bank groups.
__device__ __forceinline__ int swz(int o, int f) { return o ^ (f << 4); }
// Plain (non-multicast) bulk copy global -> shared, completion on mbarrier.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// 16-byte asynchronous global->shared copy (L2 only, evict-first policy for
// streamed weights) and the arrive that fires when this thread's copies land.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "l"(policy)
                 : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// cp.async groups: close this thread's copies issued since the last commit
// into a group; wait until at most n (0..3) of its groups are still pending.
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_pending(int n) {
    switch (n) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    }
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Programmatic dependent launch.  The routing and expert kernels are launched
// with programmatic stream serialisation: a kernel may start while its
// predecessor in the stream is still running.  pdl_wait() blocks until the
// predecessor has completed and its memory is visible; every kernel calls it
// before touching data another kernel produces or consumes (constant inputs
// such as weights may be read earlier).  pdl_trigger() lets the successor
// launch.  Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void set_error(int32_t *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

}  // namespace lmoe
