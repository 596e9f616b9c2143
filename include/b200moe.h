/*
 * b200moe.h -- C ABI of the B200 (sm_100a) Qwen3-MoE expert-execution path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as `void *`.  Nothing here allocates device memory: the caller owns
 * every buffer (the Python host layer allocates them through the PyTorch
 * caching allocator so the calls can be captured in CUDA graphs).  Work is
 * enqueued on `stream` and the call returns without synchronising.
 *
 * Return value: B200MOE_OK (0) or an error code; b200moe_last_error() gives a
 * thread-local message for the last failing call on the calling thread.
 *
 * Reference interfaces are cited as file:line inside kagami4243/extend-nano-vLLM
 * (package `nanovllm`, version 0.3.0).  The reference implements this path in
 * Python + Triton inside class ExpertParallelMoE (nanovllm/layers/moe.py:237);
 * these functions replace its router, packing, grouped GEMM, SwiGLU, combine
 * and expert-parallel exchange steps.
 */
#ifndef B200MOE_H_
#define B200MOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200MOE_API __attribute__((visibility("default")))
#else
#define B200MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define B200MOE_OK 0
#define B200MOE_EINVAL 1      /* bad argument (shape, dtype, null pointer) */
#define B200MOE_ECUDA 2       /* CUDA runtime / driver error */
#define B200MOE_EUNSUPPORTED 3 /* valid but unsupported configuration */

/* ---- element type codes -------------------------------------------------- */
#define B200MOE_BF16 0
#define B200MOE_F16 1
#define B200MOE_F32 2
#define B200MOE_F64 3

/* ---- expert GEMM engines ---------------------------------------------------- */
#define B200MOE_ENGINE_STREAM 0 /* CUDA-core weight streaming (small decode buckets) */
#define B200MOE_ENGINE_TCGEN05 1 /* tcgen05/TMEM grouped GEMM fed by TMA; the variant is
                                   chosen per call: SWAP for <= 4096 routes, else WIDE */
#define B200MOE_ENGINE_TCGEN05_WIDE 2 /* routed rows as the MMA M operand (128-row tiles),
                                        128/256-wide weight tiles as N */
#define B200MOE_ENGINE_TCGEN05_SWAP 3 /* weight rows as the MMA M operand (128 features),
                                        routed rows as N (rounded to 16) */
#define B200MOE_ENGINE_TCGEN05_TALL 5 /* 256 routed rows of one expert per work item: two
                                        M=128 MMAs share each staged 256-wide weight tile
                                        (needs x_packed; otherwise runs WIDE) */
#define B200MOE_ENGINE_TCGEN05_PAIR 4 /* two-SM (cta_group::2) swap-AB: 256 weight rows as M,
                                        row chunks of <= 256 routed rows as N; needs the
                                        `chunks` list of b200moe_pack_routes */

/* Size of the 128-row work-tile records written by b200moe_pack_routes:
 * {local expert, first packed row, end packed row (exclusive)}. */
#define B200MOE_MTILE_WORDS 3
#define B200MOE_MTILE_ROWS 128
/* Largest row chunk (same record layout): an expert's kept rows split into
 * ceil(rows / 256) chunks of equal 16-row multiples (the last one shorter). */
#define B200MOE_CHUNK_ROWS 256
/* Packing alignment of every expert's row group (reference _MOE_BLOCK_M,
 * nanovllm/layers/moe.py:36). */
#define B200MOE_BLOCK_ROWS 16

/* counters[] written by b200moe_pack_routes */
#define B200MOE_CNT_PADDED_ROWS 0 /* reference num_tokens_post_padded, moe.py:807 */
#define B200MOE_CNT_MTILES 1      /* number of 128-row work tiles */
#define B200MOE_CNT_LOCAL_KEPT 2  /* local assignments, moe.py:864-867 */
#define B200MOE_CNT_DROPPED 3     /* capacity drops, moe.py:913-917 */
#define B200MOE_CNT_CHUNKS 4      /* number of row chunks (0 when `chunks` is NULL) */
#define B200MOE_NUM_COUNTERS 5

B200MOE_API const char *b200moe_last_error(void);
B200MOE_API int b200moe_abi_version(void);

/* Sticky device-side status word: non-zero after a kernel gave up a bounded
 * wait (bit 0) or saw an out-of-range index (bit 1).  Copies the word of the
 * current device to *status (synchronises) and, if clear != 0, resets it. */
B200MOE_API int b200moe_device_status(int *status, int clear);

/*
 * Router: softmax (fp32) over `num_experts` logits per token, top-k selection,
 * optional renormalisation over the selected k, bf16 weights.
 * Replaces ExpertParallelMoE._route softmax/topk/renorm/cast,
 * nanovllm/layers/moe.py:872-878 (the gate projection moe.py:871 stays a
 * library GEMM in the caller).
 * The result equals, bit for bit, what the reference's torch calls return on
 * a CUDA device: the same fp32 softmax arithmetic (per-lane then butterfly
 * sum), the same top-k order for equal probabilities (torch's gather order
 * followed by its 32-wide bitonic sort), and the same renormalisation sum
 * order, so ids and bf16 weights match even when bf16 logits tie.
 *   logits     [num_tokens, num_experts] of logits_dtype (BF16/F16/F32), row-major
 *   weights    [num_tokens, top_k] bf16 out
 *   expert_ids [num_tokens, top_k] int64 out
 * Limits: num_experts <= 1024, top_k <= min(32, num_experts).
 */
B200MOE_API int b200moe_route_topk(const void *logits, int logits_dtype, int64_t num_tokens,
                       int num_experts, int top_k, int renormalize,
                       void *weights, int64_t *expert_ids, void *stream);

/*
 * b200moe_route_topk plus one shared-expert slot per token, for layers with a
 * shared expert (moe.py:195-234, added at moe.py:1259-1262 as
 * output + sigmoid(shared_expert_gate(x)) * shared_expert(x)).  Each output
 * row holds top_k + 1 slots: the routed experts exactly as
 * b200moe_route_topk writes them, then id num_experts with weight
 * bf16(sigmoid(shared_logits[t])) (fp32 sigmoid of the bf16 gate logit, as
 * torch.sigmoid on a bf16 tensor).  The shared expert then runs as expert
 * num_experts of the grouped GEMMs (b200moe_pack_routes_shared), and the
 * route-order combine adds it after the routed slots.
 *   shared_logits [num_tokens] bf16 (the shared-expert gate's output)
 *   weights       [num_tokens, top_k + 1] bf16 out
 *   expert_ids    [num_tokens, top_k + 1] int64 out
 * Limits: num_experts <= 1024, top_k <= min(31, num_experts).
 */
B200MOE_API int b200moe_route_topk_shared(const void *logits, int logits_dtype,
                                          int64_t num_tokens, int num_experts, int top_k,
                                          int renormalize, const void *shared_logits,
                                          void *weights, int64_t *expert_ids, void *stream);

/*
 * The router projection fused with b200moe_route_topk, for small batches
 * (num_tokens <= B200MOE_ROUTE_GATE_MAX_TOKENS).  Replaces the bf16 gate
 * F.linear of moe.py:871 (linear.py:51) plus the routing of moe.py:872-878.
 * logits[t, e] = bf16(sum_h x[t, h] * gate_w[e, h]) accumulated in fp32 in a
 * fixed order (16-byte vectors l, l + 32, ... per lane, then a butterfly over
 * the warp); cuBLAS accumulates in its own order, so a logit can differ from
 * the reference's by one bf16 unit where the fp32 sums straddle a rounding
 * boundary -- the routing of such tokens can then differ.  The routing of the
 * written logits is exactly b200moe_route_topk's.
 *   x        [num_tokens, hidden] bf16 (hidden % 8 == 0, <= 4096)
 *   gate_w   [num_experts, hidden] bf16
 *   logits   [num_tokens, num_experts] bf16 out
 *   weights  [num_tokens, top_k] bf16 out;  expert_ids [num_tokens, top_k] int64 out
 *   sync     int32 [ceil(num_tokens / 8)], zero before the first call; the
 *            kernel leaves it zero (one buffer serves calls in stream order)
 */
#define B200MOE_ROUTE_GATE_MAX_TOKENS 64
B200MOE_API int b200moe_route_gate_topk(const void *x, int hidden, const void *gate_w,
                                        int64_t num_tokens, int num_experts, int top_k,
                                        int renormalize, void *logits, void *weights,
                                        int64_t *expert_ids, int32_t *sync, void *stream);

/* Scratch bytes b200moe_pack_routes needs for `num_routes` routes. */
B200MOE_API size_t b200moe_pack_scratch_bytes(int64_t num_routes, int num_experts);

/* Rows the packed layout can occupy: num_routes + min(num_routes, E_loc) * 15,
 * rounded up to 16 (reference max_padded_rows, moe.py:793-797). */
B200MOE_API int64_t b200moe_pack_row_capacity(int64_t num_routes, int num_local_experts);

/* Upper bound of 128-row work tiles: ceil(num_routes/128) + min(num_routes, E_loc). */
B200MOE_API int64_t b200moe_pack_max_mtiles(int64_t num_routes, int num_local_experts);

/*
 * Capacity + expert-major packing, graph-safe (no host synchronisation).
 * Replaces: capacity keep-mask, moe.py:879-919; _local_routes and the Triton
 * _map_expert_routes_kernel, moe.py:491-517 and :142-161; compact expert-task
 * construction of _forward_static_decode, moe.py:790-847; the dynamic packing
 * of _forward_triton, moe.py:698-740 and :763-767.
 *
 * Routes are the flat [num_routes] array `expert_ids` in token-major, slot-
 * minor order.  A route's capacity position is expert_base[e] (0 when NULL)
 * plus the number of earlier routes to the same expert; it is kept when the
 * position is < capacity (capacity < 0: no limit).  Dropped routes are
 * rewritten in place to id = num_experts and weight 0 (moe.py:918-919).
 * Local experts are [expert_start, expert_start + num_local_experts) when
 * local_index is NULL, else local_index[e] (>= 0 local id, -1 remote).
 * Ids outside [0, num_experts) are never local (moe.py:512-517).
 *
 * Outputs (all int32, caller-allocated):
 *   row_route      [row_capacity]   packed row -> route id, unused rows = num_routes
 *                                   (reference row_ids in route layout, moe.py:828-832)
 *   route_row      [num_routes]     route -> packed row, else row_capacity
 *                                   (reference route_rows, moe.py:763-767)
 *   combine_rows   [num_routes]     route -> route id if computed here, else num_routes
 *                                   (may be NULL)
 *   tile_expert    [row_capacity/16] local expert of each 16-row tile, unused 0
 *                                   (reference expert_ids, moe.py:833-844)
 *   expert_offsets [E_loc + 1]      first packed row of each local expert; [E_loc] = total
 *   expert_counts  [E_loc]          kept local routes per expert
 *   mtiles         [max_mtiles * 3] 128-row work tiles {expert, row_begin, row_end}
 *   chunks         [max_mtiles * 3] row chunks of <= 256 rows, same records (may be
 *                                   NULL; the TCGEN05_PAIR engine reads them)
 *   counters       [5]              see B200MOE_CNT_*
 *   stats          [2] int64 or NULL: += local kept, += dropped (device accumulators)
 */
B200MOE_API int b200moe_pack_routes(int64_t *expert_ids, void *route_weights, int64_t num_routes,
                        int num_experts, const int64_t *local_index, int expert_start,
                        int num_local_experts, const int32_t *expert_base,
                        int64_t capacity, int64_t row_capacity, int32_t *row_route,
                        int32_t *route_row, int32_t *combine_rows, int32_t *tile_expert,
                        int32_t *expert_offsets, int32_t *expert_counts, int32_t *mtiles,
                        int64_t max_mtiles, int32_t *chunks, int32_t *counters,
                        int64_t *stats, void *scratch, size_t scratch_bytes, void *stream);

/*
 * b200moe_pack_routes with device-side bounds, for callers whose route count
 * or capacity exists only on the GPU (the expert-parallel receiver below,
 * inside a CUDA graph).  Same arguments and results as b200moe_pack_routes
 * plus:
 *   route_count  device int32 or NULL: only routes [0, *route_count) are
 *                packed (clamped to num_routes); the per-route outputs of
 *                the others (route_row, combine_rows) are left unwritten and
 *                their ids are never read.  num_routes still sizes the layout
 *                (row_capacity, max_mtiles, scratch) and is the row_route
 *                sentinel.
 *   capacity_dev device int64 or NULL: overrides `capacity` (< 0: no limit).
 * Same reference lines as b200moe_pack_routes (moe.py:879-919, :491-517,
 * :783-868, :680-771).
 */
B200MOE_API int b200moe_pack_routes_device_bounds(
    int64_t *expert_ids, void *route_weights, int64_t num_routes, const int32_t *route_count,
    int num_experts, const int64_t *local_index, int expert_start, int num_local_experts,
    const int32_t *expert_base, int64_t capacity, const int64_t *capacity_dev,
    int64_t row_capacity, int32_t *row_route, int32_t *route_row, int32_t *combine_rows,
    int32_t *tile_expert, int32_t *expert_offsets, int32_t *expert_counts, int32_t *mtiles,
    int64_t max_mtiles, int32_t *chunks, int32_t *counters, int64_t *stats, void *scratch,
    size_t scratch_bytes, void *stream);

/*
 * b200moe_route_topk followed by b200moe_pack_routes in one launch, for small
 * batches (num_tokens * top_k <= B200MOE_ROUTE_PACK_MAX_ROUTES: one route
 * block).  Writes the same weights/expert_ids as b200moe_route_topk (the same
 * warp routine; capacity drops then applied in place as b200moe_pack_routes
 * does) and the same layout as b200moe_pack_routes over them.  Replaces
 * moe.py:870-919 plus the packing lines of b200moe_pack_routes.
 *   weights    [num_tokens, top_k] bf16 out;  expert_ids [num_tokens, top_k] int64 out
 * Other arguments as b200moe_pack_routes (num_routes = num_tokens * top_k,
 * no expert_base).
 */
#define B200MOE_ROUTE_PACK_MAX_ROUTES 1024
B200MOE_API int b200moe_route_pack(
    const void *logits, int logits_dtype, int64_t num_tokens, int num_experts, int top_k,
    int renormalize, void *weights, int64_t *expert_ids, const int64_t *local_index,
    int expert_start, int num_local_experts, int64_t capacity, int64_t row_capacity,
    int32_t *row_route, int32_t *route_row, int32_t *combine_rows, int32_t *tile_expert,
    int32_t *expert_offsets, int32_t *expert_counts, int32_t *mtiles, int64_t max_mtiles,
    int32_t *chunks, int32_t *counters, int64_t *stats, void *scratch, size_t scratch_bytes,
    void *stream);

/*
 * b200moe_pack_routes over routed plus shared experts: experts
 * [num_experts - num_shared_experts, num_experts) are shared experts (routes
 * written by b200moe_route_topk_shared); they have no capacity limit (the
 * reference applies capacity to routed experts only, moe.py:879-919) and are
 * left out of counters[B200MOE_CNT_LOCAL_KEPT] and `stats`.  Capacity
 * positions and drops of the routed experts are those of b200moe_pack_routes
 * over the routed slots alone (the shared slots form their own expert group).
 * Dropped routes are rewritten to id = num_experts (routed + shared).
 * Other arguments as b200moe_pack_routes without expert_base.
 */
B200MOE_API int b200moe_pack_routes_shared(
    int64_t *expert_ids, void *route_weights, int64_t num_routes, int num_experts,
    int num_shared_experts, const int64_t *local_index, int expert_start, int num_local_experts,
    int64_t capacity, int64_t row_capacity, int32_t *row_route, int32_t *route_row,
    int32_t *combine_rows, int32_t *tile_expert, int32_t *expert_offsets, int32_t *expert_counts,
    int32_t *mtiles, int64_t max_mtiles, int32_t *chunks, int32_t *counters, int64_t *stats,
    void *scratch, size_t scratch_bytes, void *stream);

/*
 * b200moe_pack_routes for callers that cannot provide scratch memory.  No
 * counterpart in the reference: it exists for hosts that have committed
 * (nearly) all device memory to their own fixed pools, or that drive this
 * library from plain C / FFI without a device allocator, so the histogram
 * scratch of the packing kernels comes from a static device array inside the
 * library instead of a caller buffer.
 *  - Same arguments and results as b200moe_pack_routes, minus scratch and
 *    the row-chunk list (counters[B200MOE_CNT_CHUNKS] = 0).
 *  - Limit: a call is accepted exactly when
 *    b200moe_pack_scratch_bytes(num_routes, num_experts) <=
 *    b200moe_pack_static_scratch_capacity() (256 KiB); check that before
 *    calling.  Other calls fail with B200MOE_EINVAL and a message.  The
 *    need is not monotone in num_routes (the packing kernels widen their
 *    route chunks once more than 512 blocks would be needed): at 128
 *    experts, 520,193 to 524,288 routes are rejected while 600,000 fit.
 *    Every call with up to 65,536 routes and up to 1,023 experts fits.
 *    Each GPU that loads the library holds the array until the process
 *    exits.
 *  - Allocates nothing: no cudaMalloc/cudaFree.  The first call on each
 *    device (and the first call after that device's context was re-created,
 *    e.g. after cudaDeviceReset) looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that call before
 *    any stream capture.
 *  - All calls on a device share the one array and every call overwrites the
 *    part it uses (nothing needs to start at zero); calls whose kernels
 *    overlap on the GPU (different streams without ordering) race and must be
 *    serialised by the caller.
 */
B200MOE_API size_t b200moe_pack_static_scratch_capacity(void);
B200MOE_API int b200moe_pack_routes_static_scratch(
    int64_t *expert_ids, void *route_weights, int64_t num_routes, int num_experts,
    const int64_t *local_index, int expert_start, int num_local_experts,
    const int32_t *expert_base, int64_t capacity, int64_t row_capacity, int32_t *row_route,
    int32_t *route_row, int32_t *combine_rows, int32_t *tile_expert, int32_t *expert_offsets,
    int32_t *expert_counts, int32_t *mtiles, int64_t max_mtiles, int32_t *counters,
    int64_t *stats, void *stream);

/*
 * Per-expert route counts of a flat route array: counts[e] for e < num_experts
 * (ids outside the range are ignored).  Used by the expert-parallel exchange to
 * agree on global capacity positions (the reference routes the gathered global
 * batch, moe.py:979).
 */
B200MOE_API int b200moe_expert_histogram(const int64_t *expert_ids, int64_t num_routes, int num_experts,
                             int32_t *counts, void *stream);

/*
 * Gather the hidden rows of packed routes into expert-major order:
 * x_packed[p] = x[token(row_route[p])] for p < counters[PADDED_ROWS] and
 * row_route[p] < num_routes, where token(r) = token_of_route[r] when given,
 * else r / top_k.  Feeds the tcgen05 gate/up GEMM (reference A-row gather of
 * _grouped_moe_gemm_kernel, moe.py:103-118).
 */
B200MOE_API int b200moe_gather_rows(const void *x, int64_t x_rows, int hidden, const int32_t *row_route,
                        const int32_t *token_of_route, int top_k, int64_t num_routes,
                        int64_t row_capacity, const int32_t *counters, void *x_packed,
                        void *stream);

/*
 * Grouped gate/up projection fused with SwiGLU:
 *   act[p, j] = bf16( bf16(silu(bf16(g))) * bf16(u) ),  g = x_p . W13[e, j],
 *   u = x_p . W13[e, I + j], fp32 accumulation, for every packed row p of
 *   local expert e.  Rounding points follow the reference, which stores
 *   gate/up in bf16 and applies F.silu and the product in bf16
 *   (moe.py:848-854 and :742-746, kernel moe.py:63-139).
 *   w13   [E_loc, 2I, H] bf16 (gate rows first, moe.py:532-539)
 *   act   [row_capacity, I] bf16 out, packed order
 * engine STREAM reads x ([x_rows, H], token-major) through row_route; the
 * TCGEN05 engines read x_packed ([row_capacity, H], from b200moe_gather_rows)
 * when it is not NULL, else (WIDE, SWAP and the per-call choice TCGEN05) the
 * rows of x directly: the GEMM's TMA loads gather token rows through
 * row_route and token_of_route (tile::gather4), so no packed copy is
 * written.  PAIR requires x_packed.  Work lists: the 128-row `mtiles`
 * (STREAM, WIDE, SWAP) or the row `chunks` (PAIR; may be NULL otherwise).
 */
B200MOE_API int b200moe_expert_gate_up(int engine, const void *x, int64_t x_rows, const void *x_packed,
                           int hidden, int inter, const void *w13, int num_local_experts,
                           const int32_t *row_route, const int32_t *token_of_route, int top_k,
                           int64_t num_routes, int64_t row_capacity, const int32_t *mtiles,
                           int64_t max_mtiles, const int32_t *chunks, const int32_t *counters,
                           void *act, void *stream);

/*
 * Grouped down projection with the route-weight scale applied to the fp32
 * accumulator before the bf16 store (moe.py:129-139; pinned by the reference
 * xfail test tests/test_moe_graph_capture.py:151-174):
 *   y[r, h] = bf16( (act_p . W2[e, h]) * float(w_r) ),  r = row_route[p]
 *   w2  [E_loc, H, I] bf16;  route_weights [num_routes] bf16;
 *   y   [num_routes, H] bf16 out in route order (rows of routes not computed
 *       here are not written; combine masks them through combine_rows).
 *   max_expert_rows: upper bound on the rows of one expert (the token rows of
 *       the call: a token has at most one route per expert), or 0 if unknown;
 *       lets the streaming engine pick a register-lean variant.
 */
B200MOE_API int b200moe_expert_down(int engine, const void *act, int hidden, int inter, const void *w2,
                        int num_local_experts, const int32_t *row_route,
                        const void *route_weights, int64_t num_routes, int64_t max_expert_rows,
                        int64_t row_capacity,
                        const int32_t *mtiles, int64_t max_mtiles, const int32_t *chunks,
                        const int32_t *counters, void *y, void *stream);

/*
 * b200moe_expert_down writing each route's row into another buffer instead of
 * y: route r's bf16 row goes to dst_bases[dst_rank[r]] + dst_offset bytes,
 * row dst_row[r] (rows of H values, dst_row < dst_rows).  The expert-parallel
 * exchange passes the ranks' exchange buffers (peer memory mapped with CUDA
 * IPC) at their return region and the received routes' source rank / source
 * route, so the rows land at their sources from the GEMM epilogue while
 * later tiles compute, replacing the copy of b200moe_nvl_return (then
 * b200moe_nvl_return_signal publishes the phase).  Same arithmetic as
 * b200moe_expert_down.  Engines: TCGEN05 (the library picks), TCGEN05_WIDE,
 * TCGEN05_SWAP.  Limits: dst_ranks <= 16, dst_rows < 2^24, dst_offset and
 * the bases 16-byte aligned; an out-of-range rank or row sets the index
 * status bit and the row is not written.
 */
B200MOE_API int b200moe_expert_down_scatter(
    int engine, const void *act, int hidden, int inter, const void *w2, int num_local_experts,
    const int32_t *row_route, const void *route_weights, int64_t num_routes,
    int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles, const int32_t *counters,
    const uint64_t *dst_bases, int dst_ranks, int64_t dst_offset, const int32_t *dst_rank,
    const int32_t *dst_row, int64_t dst_rows, void *stream);

/*
 * Fused expert path for tiny decode batches (num_tokens * top_k <= 16, no
 * capacity limit): router + gate/up + SwiGLU + down + route-order combine in
 * two launches.  Every CTA routes its token itself (same routine as
 * b200moe_route_topk), so no packing step is needed; the arithmetic equals the
 * streaming engine followed by b200moe_combine (bf16 act, bf16 route rows,
 * fp32 slot-order sum), so results are identical to that path.  Replaces the
 * reference's whole _forward_static_decode for such buckets
 * (nanovllm/layers/moe.py:783-868 with _route, :870-878).
 *   logits [T, E] (BF16/F32), x [T, H] bf16, w13/w2 as above,
 *   act    [T*top_k, I] bf16 caller scratch,
 *   out    [T, H] bf16 (routes to non-local experts contribute zero),
 *   stats  [2] int64 or NULL: stats[0] += local routes.
 */
B200MOE_API int b200moe_decode_tiny(const void *logits, int logits_dtype, const void *x,
                                    int64_t num_tokens, int hidden, int inter, int num_experts,
                                    int top_k, int renormalize, const void *w13, const void *w2,
                                    int num_local_experts, const int64_t *local_index,
                                    int expert_start, void *act, void *out, int64_t *stats,
                                    void *stream);

/*
 * Route-order combine: out[t, :] = sum_{s < top_k} Y[route_rows[t*top_k+s], :]
 * accumulated in fp32 (accum_f64 != 0: fp64) in slot order, rows >= num_rows
 * read as zero, stored as out_dtype (BF16/F32/F64).  route_rows NULL means the
 * identity.  Replaces _combine_expert_routes and the Triton
 * _combine_expert_routes_kernel, moe.py:642-678 and :164-192.
 */
B200MOE_API int b200moe_combine(const void *y, int64_t num_rows, const int32_t *route_rows,
                    int64_t num_tokens, int top_k, int hidden, int accum_f64, void *out,
                    int out_dtype, void *stream);

/*
 * Expert-parallel dispatch plan for the NCCL all-to-all backend
 * "all_to_all_nvlink" (replaces the token all-gather and global re-routing of
 * _forward_global_dp, nanovllm/layers/moe.py:964-982).  For this rank's flat
 * routes (after capacity) and owner[e], the EP rank that holds expert e:
 *   send_token_slot [num_tokens * ep_size]  slot of token t in destination d's
 *                    token list, or -1 (t has no kept route to d)
 *   route_dest_slot [num_tokens * top_k]    slot of route r in its destination's
 *                    route list, or -1 (dropped / invalid id)
 *   counts [2 * ep_size] int32: tokens per destination, then routes per destination
 * Lists are in ascending token / route order.  ep_size <= 16.
 */
B200MOE_API int b200moe_ep_plan(const int64_t *expert_ids, int64_t num_tokens, int top_k, int num_experts,
                    const int32_t *owner, int ep_size, int32_t *send_token_slot,
                    int32_t *route_dest_slot, int32_t *counts, void *stream);

/*
 * Pack the dispatch payload.  token_offsets_host / route_offsets_host are HOST
 * arrays [ep_size]: exclusive prefix sums of the plan counts.
 *   send_x     [sum tokens, H] bf16 rows, grouped by destination
 *   send_meta  [sum routes, 4] int32 records {global expert id, token row in the
 *              destination's token list, bf16 weight bits, source route id}
 */
B200MOE_API int b200moe_ep_pack(const void *x, int hidden, const int64_t *expert_ids,
                    const void *route_weights, int64_t num_tokens, int top_k, int num_experts,
                    const int32_t *owner, int ep_size, const int32_t *send_token_slot,
                    const int32_t *route_dest_slot, const int32_t *token_offsets_host,
                    const int32_t *route_offsets_host, void *send_x, int32_t *send_meta,
                    void *stream);

/*
 * Receiver: expand received route records into the flat arrays the local
 * pipeline consumes.  recv_route_offsets_host [ep_size + 1] and
 * recv_token_offsets_host [ep_size] are HOST prefix sums of what each source
 * sent (records; token rows).  recv_meta_starts_host [ep_size] (HOST, may be
 * NULL = recv_route_offsets_host) is the 16-byte record index in recv_meta
 * where each source's records start, so records may sit inside a combined
 * payload buffer.  Outputs: expert_ids (global ids), token_of_route (row in
 * the received token buffer), route_weights (bf16).
 */
B200MOE_API int b200moe_ep_unpack_routes(const int32_t *recv_meta, int64_t num_recv_routes, int ep_size,
                             const int32_t *recv_route_offsets_host,
                             const int32_t *recv_token_offsets_host,
                             const int32_t *recv_meta_starts_host, int64_t *expert_ids,
                             int32_t *token_of_route, void *route_weights, void *stream);

/*
 * Source, after the return all-to-all: route r's result is row
 * route_offsets_host[dest(r)] + route_dest_slot[r] of the returned buffer;
 * combine_rows[r] gets that row or num_rows_returned (dropped routes).  The
 * combine then runs in slot order as with EP=1 (moe.py:642-678).
 */
B200MOE_API int b200moe_ep_return_rows(const int64_t *expert_ids, const int32_t *owner, int64_t num_routes,
                           int num_experts, int ep_size, const int32_t *route_dest_slot,
                           const int32_t *route_offsets_host, int64_t num_rows_returned,
                           int32_t *combine_rows, void *stream);

/* ---- expert-parallel exchange over NVLink peer memory ---------------------
 * Graph-safe replacement of the reference's cross-DP exchange (all-gather of
 * every replica's tokens, global routing on every rank, reduction of
 * [N*T, H] partial outputs: nanovllm/layers/moe.py:942-1018, and the
 * rank-0 all-to-all experiment :1020-1216).  Each EP rank owns one exchange
 * buffer (b200moe_nvl_buffer_bytes) and maps every peer's buffer into its
 * address space (b200moe_ipc_handle / b200moe_ipc_open); `peer_bases` is a
 * HOST array of ep_size device pointers (256-byte aligned), entry r being
 * rank r's buffer as mapped in the calling process (own buffer included).
 * All sizes that vary per step stay on the device, so every call can be
 * captured in a CUDA graph.  One exchange is:
 *   [capacity] b200moe_nvl_histogram_send, _wait -> expert_base, capacity
 *   b200moe_pack_routes(_device_bounds) over own routes with capacity
 *   b200moe_ep_plan                    -> slots and counts
 *   b200moe_nvl_dispatch               (bump_epoch = 1 unless the histogram ran)
 *   b200moe_nvl_receive                -> received routes (device count)
 *   local packing / expert GEMMs over the received routes
 *   b200moe_nvl_return                 -> rows into the sources' return buffers
 *   b200moe_nvl_wait_return            -> then b200moe_combine over the
 *                                         return buffer with combine_rows
 * Every rank must make the same sequence of calls (an exchange is a
 * collective).  Waits on peers are bounded (2 s); on expiry the device
 * status word gets bit 0 and the kernels return.  ep_size <= 16.
 */
#define B200MOE_NVL_LAYOUT_WORDS 10

/* Bytes of one rank's exchange buffer for batches of up to max_tokens
 * tokens per rank (or -1 on bad arguments); fills layout[10] (byte offsets
 * of its sections, used by the calls below). */
B200MOE_API int64_t b200moe_nvl_buffer_bytes(int ep_size, int64_t max_tokens, int top_k,
                                             int num_experts, int num_local_experts, int hidden,
                                             int64_t *layout);

/* CUDA IPC of device memory: a 64-byte handle of the allocation holding
 * `ptr` and ptr's offset inside it; open maps a peer's allocation (peer
 * access enabled lazily) and returns the peer's pointer; close unmaps. */
B200MOE_API int b200moe_ipc_handle(const void *ptr, void *handle, int64_t *offset);
B200MOE_API int b200moe_ipc_open(const void *handle, int64_t offset, void **ptr);
B200MOE_API int b200moe_ipc_close(void *ptr, int64_t offset);

/* Capacity agreement, in two halves so that one device can drive several
 * ranks in turn.  Send: this rank's per-expert route counts and token count
 * go to every peer (advances the exchange epoch).  Wait: once every peer's
 * counts are in, (device) expert_base[e] = routes to e of lower ranks,
 * *global_tokens = tokens of all ranks, and (capacity_factor > 0)
 * *capacity = max(1, ceil(factor * global_tokens * top_k / num_experts)),
 * the reference's formula (moe.py:882-885). */
B200MOE_API int b200moe_nvl_histogram_send(const int64_t *expert_ids, int64_t num_tokens,
                                           int top_k, int num_experts, int rank, int ep_size,
                                           const uint64_t *peer_bases, const int64_t *layout,
                                           void *stream);
B200MOE_API int b200moe_nvl_histogram_wait(int top_k, int num_experts, int rank, int ep_size,
                                           const uint64_t *peer_bases, const int64_t *layout,
                                           double capacity_factor, int32_t *expert_base,
                                           int64_t *global_tokens, int64_t *capacity,
                                           void *stream);

/* Dispatch (after capacity and b200moe_ep_plan): each token row once per
 * destination owning one of its kept routes, the route records
 * {expert, token slot, bf16 weight bits, route id} and the counts, written
 * into the destinations' regions for this rank.  combine_rows[r] (device,
 * [num_tokens * top_k]) = r for routes sent anywhere, else
 * num_tokens * top_k. */
B200MOE_API int b200moe_nvl_dispatch(const void *x, int hidden, const int64_t *expert_ids,
                                     const void *route_weights, int64_t num_tokens, int top_k,
                                     int num_experts, const int32_t *owner, int rank,
                                     int ep_size, const int32_t *send_token_slot,
                                     const int32_t *route_dest_slot, const int32_t *counts,
                                     const uint64_t *peer_bases, const int64_t *layout,
                                     int64_t max_tokens, int bump_epoch, int32_t *combine_rows,
                                     void *stream);

/* Receiver: waits for every source, then flat arrays of the received routes
 * in (source, slot) order, [ep_size * route_cap] each (route_cap = layout[8]):
 * global expert ids, token_of_route (row of the exchange buffer's token
 * section viewed as [ep_size * max_tokens, hidden]), bf16 weights, source
 * rank, source route id; *route_count (device) = number received. */
B200MOE_API int b200moe_nvl_receive(int rank, int ep_size, const uint64_t *peer_bases,
                                    const int64_t *layout, int64_t max_tokens,
                                    int64_t *expert_ids, int32_t *token_of_route,
                                    void *route_weights, int32_t *src_rank, int32_t *src_route,
                                    int32_t *route_count, void *stream);

/* Return: y [max_routes, hidden] bf16 (received-route order); rows
 * j < *route_count go to rank src_rank[j]'s return buffer at row
 * src_route[j] (< max_source_routes). */
B200MOE_API int b200moe_nvl_return(const void *y, int hidden, const int32_t *src_rank,
                                   const int32_t *src_route, const int32_t *route_count,
                                   int64_t max_routes, int64_t max_source_routes, int rank,
                                   int ep_size, const uint64_t *peer_bases, const int64_t *layout,
                                   void *stream);

/*
 * The return phase without the copy: the received routes' rows were already
 * written into the sources' return buffers by b200moe_expert_down_scatter
 * (earlier in this stream, destinations = every rank's exchange buffer at the
 * layout's `returned` offset, dst_rank/dst_row = the src_rank/src_route of
 * b200moe_nvl_receive).  Publishes the phase to every source like
 * b200moe_nvl_return does after its copies.
 */
B200MOE_API int b200moe_nvl_return_signal(int rank, int ep_size, const uint64_t *peer_bases,
                                          const int64_t *layout, void *stream);

/* Source: waits until every destination returned its rows. */
B200MOE_API int b200moe_nvl_wait_return(int rank, int ep_size, const uint64_t *peer_bases,
                                        const int64_t *layout, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* B200MOE_H_ */
