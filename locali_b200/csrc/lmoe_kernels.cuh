// Kernel argument structs and launch helpers shared by lmoe_kernels.cu and
// lmoe_api.cu.
#pragma once

#include "lmoe_common.cuh"

namespace lmoe {

enum GemvMode { MODE_GATEUP = 0, MODE_DOWN = 1, MODE_QMM = 2 };

struct DispatchOut {
    int32_t *sorted_routes;  // [R]
    Chunk *chunks;           // [max_chunks]
    int32_t *n_chunks;       // [1]
    int32_t *counts;         // [buckets] (large path)
    int32_t *route_off;      // [buckets] (large path)
};

struct DispatchIn {
    const int32_t *idx;          // [R] expert id (or slot) per route
    int32_t R;
    int32_t n_experts;           // valid ids are [0, n_experts); others -> zero bucket
    const int32_t *expert_slot;  // [n_experts] or nullptr (identity: id is the slot)
    int32_t n_slots;
};

struct RouterArgs {
    const uint16_t *x;  // [T, H]
    int32_t T, H;
    const uint16_t *wg;  // [E, H] bf16
    const float *bias;   // [E] or nullptr
    int32_t E, top_k, scoring, norm_topk;
    float scaling;
    float *partial;  // [ksplit][T][E]
    // panel producer for the gate/up consumer (optional)
    uint16_t *xpanel;
    float *xsum16;
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
};

struct TopkArgs {
    const float *partial;
    int32_t ksplit, T, E, top_k, scoring, norm_topk;
    float scaling;
    const float *bias;
    int32_t *idx_ws;
    float *w_ws;
    int32_t *idx_user;
    float *w_user;
};

struct PanelArgs {
    const uint16_t *x;  // natural [rows, K]
    int32_t rows, K;
    uint16_t *panel;    // [rows, K]
    float *sum16;       // [rows, K/16]
    int32_t bits, gs;
    int32_t act_f16;
};

struct GemvArgs {
    QView q0, q1;
    const uint16_t *panel;
    const float *sum16;
    int32_t route_div;
    const Chunk *chunks;
    const int32_t *n_chunks;
    const int32_t *sorted_routes;
    int32_t n_slots;
    int32_t ntok_max;
    uint16_t *out;
    float *out_sum16;
    int32_t out_panel, out_bits, out_gs;
    float limit;
    int32_t swiglu_mode;
    const float *route_w;
    int32_t top_k;
    uint32_t *counters;
    uint16_t *combined;
    int32_t *err;
};

// host-side launchers (lmoe_kernels.cu)
cudaError_t launch_router(const RouterArgs &a, int ksplit, cudaStream_t st);
cudaError_t launch_topk(const TopkArgs &a, cudaStream_t st);
cudaError_t launch_dispatch_small(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                                  cudaStream_t st);
cudaError_t launch_dispatch_large(const DispatchIn &din, const DispatchOut &dout, int32_t *err,
                                  cudaStream_t st);
cudaError_t launch_panel(const PanelArgs &a, cudaStream_t st);
// returns cudaErrorInvalidValue for an unsupported (bits, gs)
cudaError_t launch_gemv(int mode, int act_f16, int bits, int gs, const GemvArgs &a,
                        int max_chunks, cudaStream_t st);

constexpr int kDispatchSmallMaxRoutes = 512;
constexpr int kDispatchSmallMaxBuckets = 1024;
constexpr int kRouterKS = 256;      // K columns per router CTA
constexpr int kRouterMaxEPL = 16;   // experts per lane in top-k (E <= 512)

}  // namespace lmoe
