// C entry points of the grouped expert projections: argument checks and the
// choice between the weight-streaming engine (small decode buckets) and the
// tcgen05 grouped GEMM (prefill and larger buckets).
#include "common.cuh"

namespace b200moe {
int stream_gate_up(const void *x, int64_t x_rows, int hidden, int inter, const void *w13,
                   const int32_t *row_route, const int32_t *token_of_route, int top_k,
                   int64_t num_routes, const int32_t *mtiles, int64_t max_mtiles,
                   const int32_t *counters, void *act, cudaStream_t s);
int stream_down(const void *act, int hidden, int inter, const void *w2, const int32_t *row_route,
                const void *route_weights, int64_t num_routes, int64_t max_expert_rows,
                const int32_t *mtiles, int64_t max_mtiles, const int32_t *counters, void *y,
                cudaStream_t s);
int tc_gate_up(const RowSource &src, int hidden, int inter, const void *w13, int num_local,
               int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
               const int32_t *counters, void *act, cudaStream_t s);
int tc_down(const void *act, int hidden, int inter, const void *w2, int num_local,
            const int32_t *row_route, const void *route_weights, int64_t num_routes,
            int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
            const int32_t *counters, void *y, const RowScatter *scatter, cudaStream_t s);
int tcs_gate_up(const RowSource &src, int hidden, int inter, const void *w13, int num_local,
                int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
                const int32_t *counters, void *act, cudaStream_t s);
int tcs_down(const void *act, int hidden, int inter, const void *w2, int num_local,
             const int32_t *row_route, const void *route_weights, int64_t num_routes,
             int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
             const int32_t *counters, void *y, const RowScatter *scatter, cudaStream_t s);
int tct_gate_up(const void *x_packed, int hidden, int inter, const void *w13, int num_local,
                int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
                const int32_t *counters, void *act, cudaStream_t s);
int tct_down(const void *act, int hidden, int inter, const void *w2, int num_local,
             const int32_t *row_route, const void *route_weights, int64_t num_routes,
             int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
             const int32_t *counters, void *y, cudaStream_t s);
bool tall_fits(int64_t max_mtiles);
int tcp_gate_up(const void *x_packed, int hidden, int inter, const void *w13, int num_local,
                int64_t row_capacity, const int32_t *chunks, int64_t max_chunks,
                const int32_t *counters, void *act, cudaStream_t s);
int tcp_down(const void *act, int hidden, int inter, const void *w2, int num_local,
             const int32_t *row_route, const void *route_weights, int64_t num_routes,
             int64_t row_capacity, const int32_t *chunks, int64_t max_chunks,
             const int32_t *counters, void *y, cudaStream_t s);

namespace {
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ENGINE_TCGEN05 picks the tcgen05 variant per call: decode-sized calls
// (<= 4096 routes) put the weight rows on the MMA M side so each stage carries
// almost only weight bytes; prefill-sized calls use 128-row x 256-column tiles,
// whose N=256 MMAs need a third less shared-memory bandwidth per FLOP.
int resolve_engine(int engine, int64_t num_routes) {
  if (engine != B200MOE_ENGINE_TCGEN05) return engine;
  return num_routes <= 4096 ? B200MOE_ENGINE_TCGEN05_SWAP : B200MOE_ENGINE_TCGEN05_WIDE;
}
}  // namespace
}  // namespace b200moe

extern "C" {

int b200moe_expert_gate_up(int engine, const void *x, int64_t x_rows, const void *x_packed,
                           int hidden, int inter, const void *w13, int num_local_experts,
                           const int32_t *row_route, const int32_t *token_of_route, int top_k,
                           int64_t num_routes, int64_t row_capacity, const int32_t *mtiles,
                           int64_t max_mtiles, const int32_t *chunks, const int32_t *counters,
                           void *act, void *stream) {
  using namespace b200moe;
  B200_ARG(hidden > 0 && inter > 0 && num_local_experts > 0 && top_k > 0, "bad shape");
  B200_UNSUPPORTED(hidden % 16 == 0 && inter % 16 == 0,
                   "hidden (%d) and intermediate (%d) sizes must be multiples of 16", hidden, inter);
  if (num_routes == 0 || max_mtiles == 0) return B200MOE_OK;
  B200_ARG(w13 && row_route && mtiles && counters && act, "null pointer argument");
  B200_ARG(aligned16(w13) && aligned16(act), "w13 and act must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  engine = resolve_engine(engine, num_routes);
  if (engine == B200MOE_ENGINE_TCGEN05_TALL) {
    // 256-row tiles read a packed copy of the rows; without one, or beyond
    // the work list it holds, the wide tiles run instead (same results).
    if (x_packed != nullptr && aligned16(x_packed) && tall_fits(max_mtiles))
      return tct_gate_up(x_packed, hidden, inter, w13, num_local_experts, row_capacity, mtiles,
                         max_mtiles, counters, act, s);
    engine = B200MOE_ENGINE_TCGEN05_WIDE;
  }
  if (engine == B200MOE_ENGINE_STREAM) {
    B200_ARG(x != nullptr && aligned16(x), "x must be a 16-byte aligned device pointer");
    return stream_gate_up(x, x_rows, hidden, inter, w13, row_route, token_of_route, top_k,
                          num_routes, mtiles, max_mtiles, counters, act, s);
  }
  if (engine == B200MOE_ENGINE_TCGEN05_SWAP || engine == B200MOE_ENGINE_TCGEN05_WIDE) {
    // Rows come from x_packed when given, else straight from x (gathered by
    // the GEMM's loads through row_route).
    RowSource src;
    src.x = x;
    src.x_rows = x_rows;
    src.x_packed = x_packed;
    src.row_route = row_route;
    src.token_of_route = token_of_route;
    src.top_k = top_k;
    src.num_routes = num_routes;
    if (x_packed != nullptr) {
      B200_ARG(aligned16(x_packed), "x_packed must be 16-byte aligned");
    } else {
      B200_ARG(x != nullptr && aligned16(x) && x_rows > 0,
               "x must be a 16-byte aligned device pointer with x_rows > 0");
    }
    if (engine == B200MOE_ENGINE_TCGEN05_SWAP)
      return tcs_gate_up(src, hidden, inter, w13, num_local_experts, row_capacity, mtiles,
                         max_mtiles, counters, act, s);
    return tc_gate_up(src, hidden, inter, w13, num_local_experts, row_capacity, mtiles,
                      max_mtiles, counters, act, s);
  }
  if (engine == B200MOE_ENGINE_TCGEN05_PAIR) {
    B200_ARG(x_packed != nullptr && aligned16(x_packed), "x_packed must be 16-byte aligned");
    B200_ARG(chunks != nullptr, "the two-SM engine needs the row-chunk list of pack_routes");
    return tcp_gate_up(x_packed, hidden, inter, w13, num_local_experts, row_capacity, chunks,
                       max_mtiles, counters, act, s);
  }
  set_error("unknown engine %d", engine);
  return B200MOE_EINVAL;
}

int b200moe_expert_down(int engine, const void *act, int hidden, int inter, const void *w2,
                        int num_local_experts, const int32_t *row_route,
                        const void *route_weights, int64_t num_routes, int64_t max_expert_rows,
                        int64_t row_capacity,
                        const int32_t *mtiles, int64_t max_mtiles, const int32_t *chunks,
                        const int32_t *counters, void *y, void *stream) {
  using namespace b200moe;
  B200_ARG(hidden > 0 && inter > 0 && num_local_experts > 0, "bad shape");
  B200_UNSUPPORTED(hidden % 16 == 0 && inter % 16 == 0,
                   "hidden (%d) and intermediate (%d) sizes must be multiples of 16", hidden, inter);
  if (num_routes == 0 || max_mtiles == 0) return B200MOE_OK;
  B200_ARG(act && w2 && row_route && route_weights && mtiles && counters && y,
           "null pointer argument");
  B200_ARG(aligned16(act) && aligned16(w2) && aligned16(y), "act, w2, y must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  engine = resolve_engine(engine, num_routes);
  if (engine == B200MOE_ENGINE_TCGEN05_TALL) {
    if (tall_fits(max_mtiles))
      return tct_down(act, hidden, inter, w2, num_local_experts, row_route, route_weights,
                      num_routes, row_capacity, mtiles, max_mtiles, counters, y, s);
    engine = B200MOE_ENGINE_TCGEN05_WIDE;
  }
  if (engine == B200MOE_ENGINE_STREAM)
    return stream_down(act, hidden, inter, w2, row_route, route_weights, num_routes,
                       max_expert_rows, mtiles, max_mtiles, counters, y, s);
  if (engine == B200MOE_ENGINE_TCGEN05_SWAP)
    return tcs_down(act, hidden, inter, w2, num_local_experts, row_route, route_weights,
                    num_routes, row_capacity, mtiles, max_mtiles, counters, y, nullptr, s);
  if (engine == B200MOE_ENGINE_TCGEN05_WIDE)
    return tc_down(act, hidden, inter, w2, num_local_experts, row_route, route_weights,
                   num_routes, row_capacity, mtiles, max_mtiles, counters, y, nullptr, s);
  if (engine == B200MOE_ENGINE_TCGEN05_PAIR) {
    B200_ARG(chunks != nullptr, "the two-SM engine needs the row-chunk list of pack_routes");
    return tcp_down(act, hidden, inter, w2, num_local_experts, row_route, route_weights,
                    num_routes, row_capacity, chunks, max_mtiles, counters, y, s);
  }
  set_error("unknown engine %d", engine);
  return B200MOE_EINVAL;
}

int b200moe_expert_down_scatter(int engine, const void *act, int hidden, int inter,
                                const void *w2, int num_local_experts, const int32_t *row_route,
                                const void *route_weights, int64_t num_routes,
                                int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
                                const int32_t *counters, const uint64_t *dst_bases,
                                int dst_ranks, int64_t dst_offset, const int32_t *dst_rank,
                                const int32_t *dst_row, int64_t dst_rows, void *stream) {
  using namespace b200moe;
  B200_ARG(hidden > 0 && inter > 0 && num_local_experts > 0, "bad shape");
  B200_UNSUPPORTED(hidden % 16 == 0 && inter % 16 == 0,
                   "hidden (%d) and intermediate (%d) sizes must be multiples of 16", hidden, inter);
  B200_ARG(dst_ranks >= 1 && dst_ranks <= kMaxScatterRanks, "dst_ranks must be in [1, %d]",
           kMaxScatterRanks);
  B200_ARG(dst_rows >= 0 && dst_rows <= 0xffffff, "dst_rows must be < 2^24");
  B200_ARG(dst_offset >= 0 && dst_offset % 16 == 0, "dst_offset must be a multiple of 16");
  if (num_routes == 0 || max_mtiles == 0) return B200MOE_OK;
  B200_ARG(act && w2 && row_route && route_weights && mtiles && counters && dst_bases &&
               dst_rank && dst_row,
           "null pointer argument");
  B200_ARG(aligned16(act) && aligned16(w2), "act, w2 must be 16-byte aligned");
  RowScatter sc;
  for (int i = 0; i < kMaxScatterRanks; ++i) sc.base[i] = 0;
  for (int i = 0; i < dst_ranks; ++i) {
    B200_ARG(dst_bases[i] != 0 && dst_bases[i] % 16 == 0,
             "destination buffer %d is null or not 16-byte aligned", i);
    sc.base[i] = dst_bases[i];
  }
  sc.rank = dst_rank;
  sc.row = dst_row;
  sc.offset = dst_offset;
  sc.rows = dst_rows;
  sc.ranks = dst_ranks;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  engine = resolve_engine(engine, num_routes);
  if (engine == B200MOE_ENGINE_TCGEN05_SWAP)
    return tcs_down(act, hidden, inter, w2, num_local_experts, row_route, route_weights,
                    num_routes, row_capacity, mtiles, max_mtiles, counters, nullptr, &sc, s);
  if (engine == B200MOE_ENGINE_TCGEN05_WIDE)
    return tc_down(act, hidden, inter, w2, num_local_experts, row_route, route_weights,
                   num_routes, row_capacity, mtiles, max_mtiles, counters, nullptr, &sc, s);
  set_error("scattered down rows need the tcgen05 wide or swap-AB engine (got %d)", engine);
  return B200MOE_EUNSUPPORTED;
}

}  // extern "C"
