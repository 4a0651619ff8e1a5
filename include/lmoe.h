/*
 * lmoe.h - C ABI of liblmoe.so, the sm_100a routed-MoE kernels that replace
 * Locali's kernel module and MLX gather_qmm on the expert hot path.
 *
 * Every entry point takes raw device pointers, plain sizes, a caller-owned
 * workspace and a cudaStream_t (passed as void*), enqueues its kernels on that
 * stream and returns an int status (LMOE_OK = 0, negative on error).  None of
 * them allocates device memory or synchronises the host; all of them are safe
 * to enqueue while a stream is being captured into a CUDA graph, once the
 * workspace has been initialised by lmoe_workspace_init().
 *
 * Arena layout (unchanged from the reference, arena.py:150-160 and
 * dsv4_index.py:111-124): per projection, three stacked arrays indexed by
 * arena slot -- weight uint32 [n_slots, rows, cols*bits/32] (codes LSB-first,
 * dsv4_kernels.py:135-150), scales and biases [n_slots, rows, cols/group] in
 * the activation dtype.  Slot 0 is reserved as all zeros (arena.py:123-126).
 *
 * Error convention follows native/locali_core.c (-1 bad argument, -3 bad
 * key): see the LMOE_E* codes below.
 */
#ifndef LMOE_H
#define LMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LMOE_ABI_VERSION 2

/* status codes */
#define LMOE_OK 0
#define LMOE_EINVAL (-1)        /* null pointer or inconsistent sizes            */
#define LMOE_EUNSUPPORTED (-2)  /* geometry / bits / group size not compiled     */
#define LMOE_EINDEX (-3)        /* expert id or arena slot out of range (device) */
#define LMOE_ECUDA (-4)         /* CUDA launch or runtime error                  */
#define LMOE_EWORKSPACE (-5)    /* workspace too small                           */

/* activation / scale dtype */
#define LMOE_BF16 0
#define LMOE_F16 1

/* router scoring functions (arena.py:502 is sigmoid; the V4 gate also uses
 * sqrtsoftplus, tests/test_dsv4_engine_small.py:59) */
#define LMOE_SCORE_SIGMOID 0
#define LMOE_SCORE_SOFTMAX 1
#define LMOE_SCORE_SQRTSOFTPLUS 2

/* SwiGLU rounding: FUSED = one rounding of silu_f32(gate)*up
 * (dsv4_kernels.py:165-170, dsv4_arena.py:228-232); STOCK = MLX
 * nn.silu(gate)*up op by op in the activation dtype (dsv4_arena.py:234). */
#define LMOE_SWIGLU_FUSED 0
#define LMOE_SWIGLU_STOCK 1

/* One quantized projection for all arena slots. */
typedef struct lmoe_qproj {
    const uint32_t *weight; /* [n_slots, rows, cols*bits/32] */
    const void *scales;     /* [n_slots, rows, cols/group_size] */
    const void *biases;     /* [n_slots, rows, cols/group_size] */
    int32_t bits;           /* 2, 4 or 8 */
    int32_t group_size;     /* 64 or 128 (32 for 4- and 8-bit) */
    /* Optional pre-tiled copy of all slots (lmoe_tile_pack), 16-byte aligned,
     * lmoe_tile_bytes() per slot; NULL = stream the row-major arrays above.
     * When set, the expert GEMVs read only this copy (weight/scales/biases
     * may then be NULL).  No counterpart in the reference: its arena keeps the
     * row-major MLX arrays only. */
    const void *tiles;
} lmoe_qproj;

/* The routed experts of one tier: SwitchGLU gate/up [inter, hidden] and
 * down [hidden, inter] (dsv4_arena.py:168-235). */
typedef struct lmoe_experts {
    int32_t n_slots;
    int32_t hidden;
    int32_t inter;
    int32_t dtype; /* LMOE_BF16 or LMOE_F16 */
    lmoe_qproj gate;
    lmoe_qproj up;
    lmoe_qproj down;
} lmoe_experts;

/* V4 router (arena.py:501-506 + routed scaling). weight bf16 [E, hidden]. */
typedef struct lmoe_router {
    const void *weight;
    const float *bias; /* [E] selection-only bias, or NULL */
    int32_t n_experts;
    int32_t top_k;
    int32_t scoring;
    int32_t norm_topk;
    float routed_scaling;
} lmoe_router;

typedef struct lmoe_layer {
    lmoe_router router;
    lmoe_experts experts;
    const int32_t *expert_slot; /* [E] device: arena slot of each expert */
    float swiglu_limit;         /* <= 0 disables the clamp */
    int32_t swiglu_mode;        /* LMOE_SWIGLU_* */
} lmoe_layer;

/* ABI version and error text. */
int lmoe_version(void);
const char *lmoe_strerror(int status);

/* Bytes of workspace needed for up to max_tokens tokens of this layer. */
size_t lmoe_workspace_size(const lmoe_layer *layer, int32_t max_tokens);

/* Zero a fresh workspace (once; kernels leave it reusable afterwards). */
int lmoe_workspace_init(void *workspace, size_t bytes, void *stream);

/* Device error flag raised by kernels (bad expert id / slot); reading it
 * synchronises the stream, then clears the flag.  Returns LMOE_OK or
 * LMOE_EINDEX. */
int lmoe_workspace_status(void *workspace, void *stream);

/* Router only: replaces the V4 MoEGate call at dsv4_arena.py:165-166
 * (arena.py:501-506).  x [T, hidden] activations of `dtype`; idx [T, top_k]
 * int32 (ordered by biased score, ties to the lower id); w [T, top_k] fp32
 * combine weights (already multiplied by routed_scaling).  hidden must be a
 * multiple of 64 (LMOE_EUNSUPPORTED otherwise); the layer entry points below
 * share this rule. */
int lmoe_route(const lmoe_router *router, int32_t hidden, int32_t dtype,
               const void *x, int32_t tokens, int32_t *idx, float *w,
               void *workspace, size_t ws_bytes, void *stream);

/* lmoe_route for a layer with token-id hash routing (the first layers of the
 * V4 gate, dsv4_arena.py:149-152): the experts of token t are given,
 * hash_idx[t * top_k + j] (the checkpoint's token-id -> expert table gathered
 * at the token ids, on the device); w receives their scores normalised and
 * routed-scaled as for a scored layer.  The V4 MoEGate that defines the
 * reference arithmetic is not part of the reference repository; this follows
 * the scored layers' weight computation. */
int lmoe_route_hashed(const lmoe_router *router, int32_t hidden, int32_t dtype,
                      const void *x, int32_t tokens, const int32_t *hash_idx,
                      int32_t *idx, float *w, void *workspace, size_t ws_bytes,
                      void *stream);

/* Workspace bytes for lmoe_route with up to max_tokens tokens. */
size_t lmoe_workspace_size_route(const lmoe_router *router, int32_t hidden,
                                 int32_t max_tokens);

/* Whole routed-MoE layer: ArenaMoE.__call__ single-tier path
 * (arena.py:508-547, _apply :569-624, V4 _gather dsv4_arena.py:168-235):
 * router -> dispatch -> fused gate/up + clamped SwiGLU -> down + weighted
 * combine.  out [T, hidden] in the activation dtype.  idx/w may be NULL;
 * when given they receive the routing. */
int lmoe_moe_layer(const lmoe_layer *layer, const void *x, int32_t tokens,
                   void *out, int32_t *idx, float *w, void *workspace,
                   size_t ws_bytes, void *stream);

/* lmoe_moe_layer that also records two caller-owned CUDA events
 * (cudaEvent_t, either may be NULL) on the stream: ev_routed after the
 * routing/dispatch kernel, ev_gateup after the gate/up kernel.  Lets a
 * caller time each kernel of the layer with events on its launching stream. */
int lmoe_moe_layer_staged(const lmoe_layer *layer, const void *x, int32_t tokens,
                          void *out, int32_t *idx, float *w, void *workspace,
                          size_t ws_bytes, void *stream, void *ev_routed,
                          void *ev_gateup);

/* Expert-product path of a layer call.  The decode path runs the fused
 * dequant GEMVs (legacy tensor-core MMA on exact codes, fp32 scale and bias
 * per group).  The prefill path runs the tcgen05 grouped GEMM: each 128-row
 * weight block is dequantised once per chunk of up to 128 routes of one
 * expert into the activation dtype (one rounding of scale * q + bias per
 * weight, as a tensor-core operand) and contracted on the 5th-generation
 * tensor cores; it needs hidden % 256 == 0, inter % 128 == 0, both a multiple
 * of 8 quantisation groups, and row-major arena arrays.  AUTO takes the
 * prefill path when the geometry allows it and the routes (tokens * top_k)
 * reach both LMOE_PREFILL_MIN_ROUTES and LMOE_PREFILL_ROUTES_PER_4_EXPERTS /
 * 4 * n_experts (measured crossover on B200 at 256 experts, top-6: the
 * decode path leads at 64 tokens, the prefill path at 96).  No
 * counterpart in the reference's own code; MLX's gather_qmm
 * (dsv4_arena.py:198-221) also changes kernels with the batch size. */
#define LMOE_PATH_AUTO 0
#define LMOE_PATH_DECODE 1
#define LMOE_PATH_PREFILL 2
#define LMOE_PREFILL_MIN_ROUTES 256
#define LMOE_PREFILL_ROUTES_PER_4_EXPERTS 7

/* lmoe_moe_layer with two caller-owned CUDA events (either may be NULL)
 * recorded at kernel boundaries only, for timing the kernels of exactly the
 * launches lmoe_moe_layer makes: ev_router after the routing kernel,
 * ev_experts after the first expert kernel (for one token over the pre-tiled
 * copy, the single-token layer kernel, which also selects the top-k).  Unlike
 * lmoe_moe_layer_staged, ev_router does not mark the routing as complete:
 * idx/w are written by the layer's later kernels.  No counterpart in the
 * reference (a timing hook). */
int lmoe_moe_layer_timed(const lmoe_layer *layer, const void *x, int32_t tokens,
                         void *out, int32_t *idx, float *w, void *workspace,
                         size_t ws_bytes, void *stream, void *ev_router,
                         void *ev_experts);

/* lmoe_moe_layer_staged on an explicit path (LMOE_PATH_*); LMOE_EUNSUPPORTED
 * when the layer's geometry does not allow the requested path. */
int lmoe_moe_layer_path(const lmoe_layer *layer, const void *x, int32_t tokens,
                        void *out, int32_t *idx, float *w, void *workspace,
                        size_t ws_bytes, void *stream, int32_t path,
                        void *ev_routed, void *ev_gateup);

/* The layer with its input and output in page-locked, mapped host memory
 * (e.g. torch pin_memory(); cudaHostGetDevicePointer must accept both):
 * a kernel reads the token rows from host memory into x_stage (device,
 * tokens * hidden elements, 16-byte aligned, no allocation here) and the
 * combine writes the result straight into out_host, so the host<->device
 * transfers are part of the launch chain instead of copy-engine calls
 * between layers.  Both host buffers are in use until the stream reaches
 * the end of this call.  LMOE_EINVAL for host memory the device cannot
 * address.  Same workspace as lmoe_moe_layer_path.  No counterpart in the
 * reference, whose arrays live in unified memory (MLX on Apple silicon). */
int lmoe_moe_layer_host(const lmoe_layer *layer, const void *x_host, int32_t tokens,
                        void *out_host, void *x_stage, void *workspace, size_t ws_bytes,
                        void *stream, int32_t path);

/* lmoe_moe_layer_path with token-id hash routing (see lmoe_route_hashed);
 * same workspace as lmoe_moe_layer_path. */
int lmoe_moe_layer_hashed(const lmoe_layer *layer, const void *x, int32_t tokens,
                          const int32_t *hash_idx, void *out, int32_t *idx,
                          float *w, void *workspace, size_t ws_bytes,
                          void *stream, int32_t path);

/* The patched DeepSeek-V4 MoE block (dsv4_engine.py:255-261: routed +
 * shared_experts(x)) with the decoder layer's residual add, fused into the
 * routed layer's combine:
 *   out = T(residual + T(T(sum_j y_j * w_j) + T(shared(x))))
 * (T = rounding to the activation dtype; each term as lmoe_moe_layer_path
 * computes it).  The shared expert is an ordinary SwitchGLU expert stored
 * in arena slot shared_slot of the same arrays (so with the routed experts'
 * quantisation), taken by every token with weight 1; shared_slot < 0 leaves
 * it out.  residual [tokens, hidden] may be NULL and may alias out (an
 * in-place residual stream); x may alias both.  Workspace:
 * lmoe_workspace_size_block. */
int lmoe_moe_block(const lmoe_layer *layer, int32_t shared_slot, const void *x,
                   int32_t tokens, const void *residual, void *out,
                   int32_t *idx, float *w, void *workspace, size_t ws_bytes,
                   void *stream, int32_t path);
size_t lmoe_workspace_size_block(const lmoe_layer *layer, int32_t max_tokens,
                                 int32_t path);

/* Workspace bytes for lmoe_moe_layer_path calls of up to max_tokens tokens
 * on `path` (0 when the path is unavailable).  lmoe_workspace_size equals
 * this with LMOE_PATH_AUTO. */
size_t lmoe_workspace_size_path(const lmoe_layer *layer, int32_t max_tokens,
                                int32_t path);

/* Allocation-free lmoe_moe_layer.  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory for a workspace (a serving
 * loop whose device memory belongs to another allocator, a runtime that
 * forbids allocation on its request path, a binding without a device
 * allocator).  Scratch lives in a static device array of
 * LMOE_STATIC_WORKSPACE_BYTES (8 MiB), held by every GPU that loads the
 * library until the process exits.  The call always runs the decode path
 * (lmoe_moe_layer_path with LMOE_PATH_DECODE), so:
 *   - layers that path cannot run (3-bit projections, or widths without a
 *     decode tile plan such as hidden 7168 at 2 bits) return
 *     LMOE_EUNSUPPORTED;
 *   - calls with lmoe_workspace_size_path(layer, tokens, LMOE_PATH_DECODE)
 *     > LMOE_STATIC_WORKSPACE_BYTES (about 80 tokens at DeepSeek-V4-Flash
 *     shapes) return LMOE_EWORKSPACE;
 * both before anything is enqueued.  Where AUTO would take the tcgen05 path
 * (LMOE_PREFILL_MIN_ROUTES and more), the results follow the decode path's
 * arithmetic, not lmoe_moe_layer's.  The first call on a device looks up the
 * array's device address with that device current; make that first call
 * before any stream capture.  The call allocates nothing (no
 * cudaMalloc/cudaFree), clears the array's status word and router counter on
 * the stream, then runs the kernels.  All calls on a device share the one
 * array and it keeps the last call's contents, so calls that overlap on the
 * GPU (different streams, or concurrent host threads without ordering) race
 * and corrupt each other's results. */
#define LMOE_STATIC_WORKSPACE_BYTES (8u << 20)
int lmoe_moe_layer_static(const lmoe_layer *layer, const void *x,
                          int32_t tokens, void *out, int32_t *idx, float *w,
                          void *stream);
size_t lmoe_static_workspace_bytes(void);

/* Device error flag of the most recent lmoe_moe_layer_static call on the
 * current device (each call clears it when it starts): synchronises the
 * stream, reads the flag, clears it.  Returns LMOE_OK, LMOE_EINDEX (a bad
 * expert id or arena slot was met and contributed zeros) or LMOE_ECUDA.  The
 * lmoe_workspace_status of the static scratch, whose address callers never
 * see. */
int lmoe_static_status(void *stream);

/* Same layer with routing supplied by the caller (an external gate, as
 * V4ArenaMoE.route returns it): idx [T, top_k] expert ids, w [T, top_k]
 * fp32 weights (arena.py:512-546). */
int lmoe_moe_routed(const lmoe_layer *layer, const void *x, int32_t tokens,
                    const int32_t *idx, const float *w, void *out,
                    void *workspace, size_t ws_bytes, void *stream);

/* The expert products of lmoe_moe_routed without its combine, for the
 * layer calls the reference splits (ArenaMoE._apply, arena.py:549-672):
 * for every route r = t * top_k + j with idx[r] >= 0, products[r] =
 * T(T(y_r) * T(w[r])), or T(y_r) when w is NULL; routes with idx[r] < 0
 * (another tier's, or not ready yet) are skipped and their rows left as they
 * were.  products [tokens * top_k, hidden], 16-byte aligned.  Decode GEMVs;
 * same workspace as lmoe_moe_routed. */
int lmoe_moe_products(const lmoe_layer *layer, const void *x, int32_t tokens,
                      const int32_t *idx, const float *w, void *products,
                      void *workspace, size_t ws_bytes, void *stream);

/* out[t] = T(sum over i < top_k of products[t * top_k + o_i] * w[...] in
 * fp32), o_i = order[t * top_k + i] (route order when order is NULL; w NULL
 * = 1).  Without weights: the single-tier combine of rows that lmoe_moe_products
 * already weighted (arena.py:619-624; lmoe_moe_layer's arithmetic bit for
 * bit).  With fp32 weights (the routing weights rounded to the activation
 * dtype) over unweighted rows and a tier-major order: the mixed-tier fp32
 * scatter-add of y * g (arena.py:632-672). */
int lmoe_combine_routes(const void *products, const float *w, const int32_t *order,
                        int32_t tokens, int32_t top_k, int32_t hidden,
                        int32_t dtype, void *out, void *stream);

/* Fused gate/up products + clamped SwiGLU over arena slots: replaces
 * fused_affine2_swiglu (dsv4_kernels.py:246-300) for 2/4/8-bit and any batch.
 * x [T, hidden]; slots [T, top_k] uint32 arena slots (gather_qmm
 * rhs_indices); h [T*top_k, inter] activations (route r = t*top_k + j). */
int lmoe_gateup_swiglu(const lmoe_experts *experts, const void *x,
                       int32_t tokens, int32_t top_k, const uint32_t *slots,
                       float limit, int32_t swiglu_mode, void *h,
                       void *workspace, size_t ws_bytes, void *stream);

/* mx.gather_qmm(x, w, s, b, rhs_indices=slots, transpose=True) for one
 * projection (dsv4_arena.py:198-221, arena.py:676-681).  x [routes, cols]
 * (one input row per route); slots [routes]; y [routes, rows]. */
int lmoe_gather_qmm(const lmoe_qproj *proj, int32_t n_slots, int32_t rows,
                    int32_t cols, int32_t dtype, const void *x,
                    int32_t routes, const uint32_t *slots, void *y,
                    void *workspace, size_t ws_bytes, void *stream);

/* Workspace bytes for lmoe_gateup_swiglu / lmoe_gather_qmm calls. */
size_t lmoe_workspace_size_routes(int32_t max_routes, int32_t hidden,
                                  int32_t inter, int32_t n_slots);

/* Pre-tiled weight format (no counterpart in the reference, whose arena
 * holds row-major MLX arrays, arena.py:96-150).  A projection [rows, cols]
 * of one slot becomes rows/16 tiles of lmoe_tile_bytes()/(rows/16) bytes:
 * the 16 rows' codes, scales and biases contiguous and pre-swizzled, so the
 * decode GEMV moves each tile with one bulk copy.  Returns bytes per slot,
 * 0 when the geometry has no tile layout. */
size_t lmoe_tile_bytes(int32_t rows, int32_t cols, int32_t bits,
                       int32_t group_size);

/* Pack slots [slot_begin, slot_begin + slot_count) of the row-major
 * projection src (weight/scales/biases, 16-byte aligned) into tiles (slot 0
 * at tiles, lmoe_tile_bytes() per slot).  Asynchronous on stream. */
int lmoe_tile_pack(const lmoe_qproj *src, int32_t n_slots, int32_t rows,
                   int32_t cols, int32_t slot_begin, int32_t slot_count,
                   void *tiles, void *stream);

/* ---- Expert parallel (no counterpart in the reference, which runs every
 * expert of a layer on one device, arena.py:508-672; the arithmetic is that
 * layer's, split by expert owner).  world ranks; rank r owns experts
 * [r * E/world, (r+1) * E/world) and routes its own tokens.  One layer step:
 *   lmoe_route (replicated router) -> lmoe_ep_dispatch -> all-to-all of the
 *   send rows (equal splits of tokens rows per rank pair) -> lmoe_ep_experts
 *   -> all-to-all of the fp32 partial rows back -> lmoe_ep_combine.
 * Every buffer has a fixed size, so the step needs no host-side counts and
 * no host wait.  An exchanged row is lmoe_ep_row_bytes(hidden, top_k)
 * bytes: the hidden activations, then int32 local expert ids [top_k] (-1:
 * owned by another rank), fp32 weights [top_k], the int32 source token (-1:
 * padding row) and zero padding to 16 bytes. */
size_t lmoe_ep_row_bytes(int32_t hidden, int32_t top_k);

/* Source side.  idx/w [tokens, top_k] (lmoe_route output), x [tokens,
 * hidden]; send [world][tokens][row_bytes] receives, for every destination
 * rank d, the rows of the tokens with an expert on d in token order (then
 * padding rows); slot_of [tokens][world] the row of token t in d's block
 * (-1: none).  workspace: any lmoe workspace (its status word receives
 * LMOE_EINDEX for an expert id outside [0, n_experts), which then
 * contributes zero) or NULL.  n_experts % world == 0, world <= 32,
 * hidden % 8 == 0. */
int lmoe_ep_dispatch(const int32_t *idx, const float *w, const void *x,
                     int32_t tokens, int32_t hidden, int32_t top_k,
                     int32_t n_experts, int32_t world, void *send,
                     int32_t *slot_of, void *workspace, void *stream);

/* Expert side.  local: the rank's experts as a layer (router.n_experts =
 * experts per rank, router.top_k = the route width, expert_slot = local
 * expert -> arena slot; the router weights are not read).  recv [rows]
 * exchanged rows (rows = world * tokens per rank).  partial [rows, hidden]
 * fp32: for each real row, the rounded y*w rows of its local routes summed
 * in route order (padding rows are left unwritten).  path as in
 * lmoe_moe_layer_path; AUTO applies its rule to rows * top_k / world
 * routes. */
size_t lmoe_ep_workspace_size(const lmoe_layer *local, int32_t rows,
                              int32_t world, int32_t path);
int lmoe_ep_experts(const lmoe_layer *local, const void *recv, int32_t rows,
                    int32_t world, float *partial, void *workspace,
                    size_t ws_bytes, void *stream, int32_t path);

/* Source side, after the return exchange.  back [world][tokens][hidden] fp32
 * (rank d's partials in the order of d's received rows); out[t] = the
 * partials of the ranks that own t's experts added in rank order in fp32,
 * rounded once to dtype; with residual [tokens, hidden] (may be NULL),
 * out[t] = dtype(residual[t] + that).  out may alias residual.  With normed
 * (may be NULL), normed[t] = dtype((out[t] - mean) * rsqrt(var + eps)) with
 * fp32 statistics over the row: a weightless LayerNorm of the updated
 * residual stream, the next layer's MoE input (the decoder's ffn_norm
 * without its weight; centred so that a common-mode component in the expert
 * outputs does not steer every token to the same experts). */
int lmoe_ep_combine(const float *back, int32_t tokens, int32_t world,
                    int32_t hidden, int32_t dtype, const int32_t *slot_of,
                    const void *residual, void *out, void *normed, float eps,
                    void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LMOE_H */
