// Expert-parallel exchange kernels for sm_100a.
//
// Rank r owns experts [r * E/N, (r+1) * E/N) and routes its own tokens.  One
// layer step moves token rows to the ranks that own their experts and the
// per-row partial outputs back, with two NCCL all-to-alls of equal splits (a
// fixed capacity of T rows per rank pair, so no host-side counts and no host
// wait: the whole step can be captured in a CUDA graph).
//
// Exchanged row (ep_row_bytes): the token's hidden activations (2 bytes
// each), then a trailer of int32 local expert ids [k] (-1: the route is
// owned by another rank), fp32 combine weights [k], the int32 source token
// (-1: padding row), zero padding to a multiple of 16 bytes.
//
//   ep_dispatch_kernel  (source)   rows for each owning rank at a slot given
//                                  by token order, trailers, padding marks,
//                                  and the slot table [T][N] for the combine
//   ep_unpack_kernel    (expert)   trailers -> route ids and weights
//   ep_partial_kernel   (expert)   per received row, the y*w rows of its
//                                  local routes summed in route order (fp32)
//   ep_combine_kernel   (source)   per token, the partials of its owning
//                                  ranks added in rank order (fp32), rounded
//                                  once, plus an optional residual
//
// The reference runs every expert on one device (arena.py:508-672); this is
// the expert-parallel deployment of the same layer arithmetic.
#include "lmoe_kernels.cuh"

namespace lmoe {

__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EpDispatchArgs a) {
    __shared__ int s_before[kEpMaxWorld], s_total[kEpMaxWorld];
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x, tid = threadIdx.x;
    const int per = a.E / a.world;
    if (tid < a.world) {
        s_before[tid] = 0;
        s_total[tid] = 0;
    }
    __syncthreads();
    // rows each destination receives from tokens before t, and in total
    for (int base = 0; base < a.T; base += blockDim.x) {
        const int tp = base + tid;
        uint32_t m = 0;
        if (tp < a.T)
            for (int j = 0; j < a.k; ++j) {
                const int e = a.idx[(size_t)tp * a.k + j];
                if (e >= 0 && e < a.E) m |= 1u << (e / per);
            }
        for (int d = 0; d < a.world; ++d) {
            const bool h = (m >> d) & 1u;
            const int nb = __syncthreads_count(h && tp < t);
            const int nt = __syncthreads_count(h);
            if (tid == 0) {
                s_before[d] += nb;
                s_total[d] += nt;
            }
        }
    }
    __syncthreads();
    uint32_t mine = 0;
    for (int j = 0; j < a.k; ++j) {
        const int e = a.idx[(size_t)t * a.k + j];
        if (e >= 0 && e < a.E) {
            mine |= 1u << (e / per);
        } else if (tid == 0) {
            set_error(a.err, -3);  // contributes zero, as the single-device zero slot does
        }
    }
    const int RB = ep_row_bytes(a.H, a.k);
    const int TW = ep_trailer_bytes(a.k) / 4;
    // the token's row to every owning rank (one 16-byte load, up to N stores)
    const uint4 *src = reinterpret_cast<const uint4 *>(a.x + (size_t)t * a.H);
    for (int i = tid; i < a.H / 8; i += blockDim.x) {
        const uint4 v = src[i];
        for (int d = 0; d < a.world; ++d)
            if ((mine >> d) & 1u)
                reinterpret_cast<uint4 *>(a.send + ((size_t)d * a.T + s_before[d]) * RB)[i] = v;
    }
    // trailers: one thread per 32-bit word
    if (tid < TW) {
        for (int d = 0; d < a.world; ++d) {
            const bool hit = (mine >> d) & 1u;
            if (hit) {
                int32_t v = 0;
                if (tid < a.k) {
                    const int e = a.idx[(size_t)t * a.k + tid];
                    v = (e >= 0 && e < a.E && e / per == d) ? e - d * per : -1;
                } else if (tid < 2 * a.k) {
                    const int e = a.idx[(size_t)t * a.k + tid - a.k];
                    v = (e >= 0 && e < a.E && e / per == d) ? __float_as_int(a.w[(size_t)t * a.k + tid - a.k]) : 0;
                } else if (tid == 2 * a.k) {
                    v = t;
                }
                reinterpret_cast<int32_t *>(a.send + ((size_t)d * a.T + s_before[d]) * RB + 2 * (size_t)a.H)[tid] = v;
            }
            // slot t of destination d holds no row: mark it as padding
            if (t >= s_total[d]) {
                const int32_t v = (tid < a.k || tid == 2 * a.k) ? -1 : 0;
                reinterpret_cast<int32_t *>(a.send + ((size_t)d * a.T + t) * RB + 2 * (size_t)a.H)[tid] = v;
            }
        }
    }
    if (tid < a.world) a.slot_of[(size_t)t * a.world + tid] = ((mine >> tid) & 1u) ? s_before[tid] : -1;
}

// Trailers of the received rows -> route ids (local expert, -1 = not here)
// and weights, route r = row * k + j.
__global__ void __launch_bounds__(256) ep_unpack_kernel(const uint8_t *recv, int rows, int H, int k,
                                                        int32_t *idx, float *w) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * k) return;
    const int r = i / k, j = i - r * k;
    const int32_t *tr = reinterpret_cast<const int32_t *>(recv + (size_t)r * ep_row_bytes(H, k) + 2 * (size_t)H);
    const bool row_ok = tr[2 * k] >= 0;
    idx[i] = row_ok ? tr[j] : -1;
    w[i] = row_ok ? __int_as_float(tr[k + j]) : 0.0f;
}

// partial[r] = sum over the local routes j of row r, in route order, of the
// fp32 values of yw[r * k + j] (the rounded y*w rows of the down kernels);
// padding rows are left unwritten (the source rank never reads them).
template <typename TA>
__global__ void __launch_bounds__(256) ep_partial_kernel(const uint16_t *yw, const int32_t *idx, int rows, int H,
                                                         int k, int n_local, float *partial) {
    pdl_wait();
    pdl_trigger();
    const int per = H >> 3;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)rows * per) return;
    const long r = i / per;
    const int cc = (int)(i - r * per);
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    bool any = false;
    for (int j = 0; j < k; ++j) {
        const int id = idx[r * k + j];
        if (id < 0 || id >= n_local) continue;
        any = true;
        const uint4 v = *reinterpret_cast<const uint4 *>(yw + ((size_t)(r * k + j) * H + (size_t)cc * 8));
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            acc[2 * e] += Act<TA>::to_f(static_cast<uint16_t>(u[e] & 0xFFFFu));
            acc[2 * e + 1] += Act<TA>::to_f(static_cast<uint16_t>(u[e] >> 16));
        }
    }
    if (!any && idx[r * k] < 0) {
        // a row with no local route is a padding row (a real row always
        // carries at least one route of this rank): nothing to send back
        bool pad = true;
        for (int j = 1; j < k; ++j) pad &= idx[r * k + j] < 0;
        if (pad) return;
    }
    float4 *dst = reinterpret_cast<float4 *>(partial + (size_t)r * H + (size_t)cc * 8);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// One block per token t:
//   out[t] = T(sum over ranks d, in rank order, of back[d][slot_of[t][d]]);
//   with a residual, out[t] = T(residual[t] + that);
//   with normed, normed[t] = T((out[t] - mean) * rsqrt(var + eps)), fp32
//   statistics of the rounded out values (a weightless LayerNorm: the next
//   layer's MoE input when out is the residual stream; centring removes
//   the common-mode component that expert outputs carry when the
//   dequantised weights are not zero-mean, which would otherwise steer
//   every token to the same experts).
template <typename TA>
__global__ void __launch_bounds__(256) ep_combine_kernel(const float *back, int T, int world, int H,
                                                         const int32_t *slot_of, const uint16_t *residual,
                                                         uint16_t *out, uint16_t *normed, float eps) {
    __shared__ int s_slot[kEpMaxWorld];
    __shared__ float s_red[2][8];
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x, tid = threadIdx.x;
    if (tid < world) s_slot[tid] = slot_of[(size_t)t * world + tid];
    __syncthreads();
    const int per = H >> 3;
    float s1 = 0.0f, ss = 0.0f;
    for (int cc = tid; cc < per; cc += blockDim.x) {
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
        for (int d = 0; d < world; ++d) {
            const int s = s_slot[d];
            if (s < 0) continue;
            const float4 *p = reinterpret_cast<const float4 *>(back + ((size_t)d * T + s) * H + (size_t)cc * 8);
            const float4 v0 = p[0], v1 = p[1];
            acc[0] += v0.x;
            acc[1] += v0.y;
            acc[2] += v0.z;
            acc[3] += v0.w;
            acc[4] += v1.x;
            acc[5] += v1.y;
            acc[6] += v1.z;
            acc[7] += v1.w;
        }
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = Act<TA>::round(acc[e]);
        if (residual) {
            const uint4 v = *reinterpret_cast<const uint4 *>(residual + (size_t)t * H + (size_t)cc * 8);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                o[2 * e] = Act<TA>::round(o[2 * e] + Act<TA>::to_f(static_cast<uint16_t>(u[e] & 0xFFFFu)));
                o[2 * e + 1] = Act<TA>::round(o[2 * e + 1] + Act<TA>::to_f(static_cast<uint16_t>(u[e] >> 16)));
            }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            s1 += o[e];
            ss = fmaf(o[e], o[e], ss);
        }
        uint4 r;
        r.x = Act<TA>::pack2(o[0], o[1]);
        r.y = Act<TA>::pack2(o[2], o[3]);
        r.z = Act<TA>::pack2(o[4], o[5]);
        r.w = Act<TA>::pack2(o[6], o[7]);
        *reinterpret_cast<uint4 *>(out + (size_t)t * H + (size_t)cc * 8) = r;
    }
    if (!normed) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
    }
    if ((tid & 31) == 0) {
        s_red[0][tid >> 5] = s1;
        s_red[1][tid >> 5] = ss;
    }
    __syncthreads();
    float t1 = 0.0f, t2 = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {  // fixed order
        t1 += s_red[0][w];
        t2 += s_red[1][w];
    }
    const float mean = t1 / static_cast<float>(H);
    const float var = fmaxf(t2 / static_cast<float>(H) - mean * mean, 0.0f);
    const float inv = rsqrtf(var + eps);
    // each thread re-reads only the chunks it wrote above
    for (int cc = tid; cc < per; cc += blockDim.x) {
        const uint4 v = *reinterpret_cast<const uint4 *>(out + (size_t)t * H + (size_t)cc * 8);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        uint32_t q[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
            q[e] = Act<TA>::pack2((Act<TA>::to_f(static_cast<uint16_t>(u[e] & 0xFFFFu)) - mean) * inv,
                                  (Act<TA>::to_f(static_cast<uint16_t>(u[e] >> 16)) - mean) * inv);
        *reinterpret_cast<uint4 *>(normed + (size_t)t * H + (size_t)cc * 8) = make_uint4(q[0], q[1], q[2], q[3]);
    }
}

// out[t] = T(sum over i < k of y[t*k + o_i] (* w[t*k + o_i]) in fp32), o_i =
// order[t*k + i] (route order without an order).  Without weights the rows
// are already the rounded y*w products (the single-tier combine of
// arena.py:619-624); with fp32 weights the sum is the mixed-tier path's fp32
// scatter-add of y * g in tier order (arena.py:632-672).
template <typename TA>
__global__ void __launch_bounds__(256) combine_routes_kernel(const uint16_t *y, const float *w, const int32_t *order,
                                                             int T, int k, int H, uint16_t *out) {
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
        const int r = (int)(t * k) + (order ? order[t * k + j] : j);
        const float wr = w ? w[r] : 1.0f;
        const uint4 v = *reinterpret_cast<const uint4 *>(y + (size_t)r * H + (size_t)cc * 8);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            acc[2 * e] = fmaf(Act<TA>::to_f(static_cast<uint16_t>(u[e] & 0xFFFFu)), wr, acc[2 * e]);
            acc[2 * e + 1] = fmaf(Act<TA>::to_f(static_cast<uint16_t>(u[e] >> 16)), wr, acc[2 * e + 1]);
        }
    }
    uint4 o;
    o.x = Act<TA>::pack2(acc[0], acc[1]);
    o.y = Act<TA>::pack2(acc[2], acc[3]);
    o.z = Act<TA>::pack2(acc[4], acc[5]);
    o.w = Act<TA>::pack2(acc[6], acc[7]);
    *reinterpret_cast<uint4 *>(out + (size_t)t * H + (size_t)cc * 8) = o;
}

cudaError_t launch_combine_routes(int act_f16, const uint16_t *y, const float *w, const int32_t *order, int T, int k,
                                  int H, uint16_t *out, cudaStream_t st) {
    const long n = (long)T * (H / 8);
    if (n <= 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>((n + 255) / 256));
    if (act_f16)
        return launch_pdl(combine_routes_kernel<__half>, grid, dim3(256), 0, st, y, w, order, T, k, H, out);
    return launch_pdl(combine_routes_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, y, w, order, T, k, H, out);
}

cudaError_t launch_ep_dispatch(const EpDispatchArgs &a, cudaStream_t st) {
    if (a.T <= 0) return cudaSuccess;
    return launch_pdl(ep_dispatch_kernel, dim3(static_cast<unsigned>(a.T)), dim3(256), 0, st, a);
}

cudaError_t launch_ep_unpack(const uint8_t *recv, int rows, int H, int k, int32_t *idx, float *w, cudaStream_t st) {
    const long n = (long)rows * k;
    if (n <= 0) return cudaSuccess;
    return launch_pdl(ep_unpack_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st, recv, rows,
                      H, k, idx, w);
}

cudaError_t launch_ep_partial(int act_f16, const uint16_t *yw, const int32_t *idx, int rows, int H, int k,
                              int n_local, float *partial, cudaStream_t st) {
    const long n = (long)rows * (H / 8);
    if (n <= 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>((n + 255) / 256));
    if (act_f16)
        return launch_pdl(ep_partial_kernel<__half>, grid, dim3(256), 0, st, yw, idx, rows, H, k, n_local, partial);
    return launch_pdl(ep_partial_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, yw, idx, rows, H, k, n_local,
                      partial);
}

cudaError_t launch_ep_combine(int act_f16, const float *back, int T, int world, int H, const int32_t *slot_of,
                              const uint16_t *residual, uint16_t *out, uint16_t *normed, float eps,
                              cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    dim3 grid(static_cast<unsigned>(T));
    if (act_f16)
        return launch_pdl(ep_combine_kernel<__half>, grid, dim3(256), 0, st, back, T, world, H, slot_of, residual, out,
                          normed, eps);
    return launch_pdl(ep_combine_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, back, T, world, H, slot_of, residual,
                      out, normed, eps);
}

}  // namespace lmoe
