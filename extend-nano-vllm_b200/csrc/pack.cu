// Capacity keep-mask + expert-major packing (compact expert tasks), graph-safe.
//
// Reference behaviour reproduced bit-exactly:
//  * capacity positions: stable order of the flat (token-major, slot-minor)
//    routes within each expert; keep = position < capacity; dropped routes get
//    id = num_experts and weight 0 (nanovllm/layers/moe.py:879-919);
//  * local-route mapping for contiguous or explicit placements
//    (moe.py:491-517, Triton _map_expert_routes_kernel moe.py:142-161);
//  * expert-major packing with each expert's group padded to 16 rows, packed
//    starts in local-expert order, route ids per packed row, one expert id per
//    16-row tile, the device-side padded length (moe.py:790-847), and the
//    route -> packed-row map of the dynamic path (moe.py:698-740, :763-767).
//
// Two kernels, no host synchronisation:
//  1. pack_hist:    per-block expert histograms of contiguous route chunks
//                   (scratch), plus sentinel fills of the outputs;
//  2. pack_scatter: every block prefixes the histograms of the blocks before
//                   it, recomputes the local-expert layout, then ranks its own
//                   routes in order (warp match + per-warp counts) and scatters.
// With a single route block (up to 1024 routes: decode buckets) pack_scatter
// does pack_hist's work itself and pack_hist is not launched.
#include "common.cuh"
#include "route_warp.cuh"

namespace b200moe {
namespace {

constexpr int kPackThreads = 256;
constexpr int kPackWarps = kPackThreads / 32;

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

struct PackGeometry {
  int64_t chunk;
  int nblk;
};

PackGeometry pack_geometry(int64_t num_routes) {
  PackGeometry g;
  g.chunk = 1024;
  int64_t nblk = (num_routes + g.chunk - 1) / g.chunk;
  if (nblk > 512) {
    g.chunk = ((num_routes + 511) / 512 + kPackThreads - 1) / kPackThreads * kPackThreads;
    nblk = (num_routes + g.chunk - 1) / g.chunk;
  }
  g.nblk = static_cast<int>(nblk < 1 ? 1 : nblk);
  return g;
}

__device__ __forceinline__ int route_key(int64_t id, int num_experts) {
  return (id >= 0 && id < num_experts) ? static_cast<int>(id) : num_experts;
}

// Routes the packing kernels process: num_routes, or fewer when the caller
// gives a device-side count (routes at or above it are left untouched).
__device__ __forceinline__ int64_t routes_in_use(int64_t num_routes, const int32_t *route_count) {
  return route_count ? min64(num_routes, max64(0, *route_count)) : num_routes;
}

__global__ void __launch_bounds__(kPackThreads) pack_hist_kernel(
    const int64_t *ids, int64_t num_routes, const int32_t *route_count, int num_experts,
    int64_t chunk, int32_t *__restrict__ hist, int32_t *__restrict__ row_route,
    int64_t row_capacity, int32_t *__restrict__ tile_expert, int32_t *__restrict__ counters) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int32_t sh_hist[];
  const int E1 = num_experts + 1;
  for (int e = threadIdx.x; e < E1; e += blockDim.x) sh_hist[e] = 0;
  __syncthreads();
  const int64_t begin = blockIdx.x * chunk;
  const int64_t end = min(routes_in_use(num_routes, route_count), begin + chunk);
  for (int64_t r = begin + threadIdx.x; r < end; r += blockDim.x)
    atomicAdd(&sh_hist[route_key(ids[r], num_experts)], 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E1; e += blockDim.x)
    hist[static_cast<int64_t>(blockIdx.x) * E1 + e] = sh_hist[e];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int32_t sentinel = static_cast<int32_t>(num_routes);
  for (int64_t i = first; i < row_capacity; i += stride) row_route[i] = sentinel;
  for (int64_t i = first; i < row_capacity / B200MOE_BLOCK_ROWS; i += stride) tile_expert[i] = 0;
  if (first < B200MOE_NUM_COUNTERS) counters[first] = 0;
}

struct ScatterArgs {
  int64_t *ids;
  __nv_bfloat16 *weights;
  int64_t num_routes;
  int num_experts;
  const int64_t *local_index;
  int expert_start;
  int num_local;
  const int32_t *expert_base;
  int64_t capacity;  // < 0: unlimited
  // Experts [capped_experts, num_experts) have no capacity limit and are left
  // out of the kept/dropped counts (shared experts appended to the routed
  // ones); capped_experts == num_experts otherwise.
  int capped_experts;
  const int64_t *capacity_dev;  // device-side capacity (overrides capacity) or null
  const int32_t *route_count;   // device-side number of routes in use, or null
  int64_t row_capacity;
  int32_t *row_route;
  int32_t *route_row;
  int32_t *combine_rows;
  int32_t *tile_expert;
  int32_t *expert_offsets;
  int32_t *expert_counts;
  int32_t *mtiles;
  int64_t max_mtiles;
  int32_t *chunks;  // may be null
  int32_t *counters;
  int64_t *stats;
  const int32_t *hist;
  int64_t chunk;
  int nblk;
  // One route block (nblk == 1): the scatter kernel also does the pack_hist
  // work (its histogram, the sentinel fills, zeroed counters), one launch
  // instead of two.
  int single;
};

// Shared memory (int32 words): base[E1] tot[E1] run[E1] loc[E1]
// warp_cnt[8][E1] lstart[L] lkept[L] gof[L] mstart[L] cstart[L] + 5 reduction
// words.
__device__ __forceinline__ void pack_scatter_body(const ScatterArgs &a);

__global__ void __launch_bounds__(kPackThreads) pack_scatter_kernel(ScatterArgs a) {
  pdl_trigger();
  pdl_wait();
  pack_scatter_body(a);
}

// Small batches (one route block): the router and the packing in one launch.
// Warp w routes tokens w, w + 8, ... exactly as route_topk_kernel does (same
// warp routine), writes ids and bf16 weights, and after a block barrier the
// block packs them (the single-block pack_scatter work).
template <typename T, int VPL>
__global__ void __launch_bounds__(kPackThreads) route_pack_kernel(
    const T *logits, int64_t num_tokens, int top_k, int renormalize, ScatterArgs a) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int64_t t = warp; t < num_tokens; t += kPackWarps) {
    float w;
    int id;
    warp_route_token<T, VPL>(logits + t * a.num_experts, a.num_experts, top_k, renormalize,
                             lane, &w, &id);
    if (lane < top_k) {
      a.weights[t * top_k + lane] = __float2bfloat16_rn(w);
      a.ids[t * top_k + lane] = id;
    }
  }
  __syncthreads();
  pack_scatter_body(a);
}

__device__ __forceinline__ void pack_scatter_body(const ScatterArgs &a) {
  extern __shared__ int32_t sm[];
  const int E = a.num_experts;
  const int E1 = E + 1;
  const int L = a.num_local;
  int32_t *base = sm;
  int32_t *tot = base + E1;
  int32_t *run = tot + E1;
  int32_t *loc = run + E1;
  int32_t *warp_cnt = loc + E1;
  int32_t *lstart = warp_cnt + kPackWarps * E1;
  int32_t *lkept = lstart + L;
  int32_t *gof = lkept + L;
  int32_t *mstart = gof + L;
  int32_t *cstart = mstart + L;
  // [0] kept, [1] dropped, [2] total padded, [3] total mtiles, [4] total chunks
  int32_t *red = cstart + L;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int b = blockIdx.x;
  const int64_t cap_value = a.capacity_dev ? *a.capacity_dev : a.capacity;
  const int64_t cap = cap_value < 0 ? (int64_t)0x3fffffffffffffffLL : cap_value;
  const int64_t n_routes = routes_in_use(a.num_routes, a.route_count);
  if (b == 0 && threadIdx.x == 0 && a.route_count && *a.route_count > a.num_routes)
    atomicOr(&g_status, kStatusIndex);  // more routes than the layout was sized for

  for (int i = tid; i < L; i += blockDim.x) gof[i] = -1;
  if (tid < 5) red[tid] = 0;
  for (int i = tid; i < kPackWarps * E1; i += blockDim.x) warp_cnt[i] = 0;
  if (a.single) {
    // pack_hist's work for the only block: histogram into tot, sentinels.
    for (int e = tid; e < E1; e += blockDim.x) tot[e] = 0;
    const int32_t sentinel = static_cast<int32_t>(a.num_routes);
    for (int64_t i = tid; i < a.row_capacity; i += blockDim.x) a.row_route[i] = sentinel;
    for (int64_t i = tid; i < a.row_capacity / B200MOE_BLOCK_ROWS; i += blockDim.x)
      a.tile_expert[i] = 0;
    if (tid < B200MOE_NUM_COUNTERS) a.counters[tid] = 0;
    __syncthreads();
    for (int64_t r = tid; r < n_routes; r += blockDim.x)
      atomicAdd(&tot[route_key(a.ids[r], E)], 1);
  }
  __syncthreads();
  for (int e = tid; e < E1; e += blockDim.x) {
    int32_t before = 0, all = 0;
    if (a.single) {
      all = tot[e];
    } else {
      // Independent loads: unrolled so several are in flight (this prefix
      // over the blocks' histograms is the scatter kernel's critical path).
#pragma unroll 8
      for (int bb = 0; bb < a.nblk; ++bb) {
        const int32_t h = a.hist[static_cast<int64_t>(bb) * E1 + e];
        if (bb < b) before += h;
        all += h;
      }
    }
    base[e] = before;
    tot[e] = all;
    run[e] = 0;
    int l = -1;
    if (e < E) {
      if (a.local_index) {
        const int64_t li = a.local_index[e];
        if (li >= 0 && li < L) l = static_cast<int>(li);
        else if (li >= L) atomicOr(&g_status, kStatusIndex);
      } else if (e >= a.expert_start && e < a.expert_start + L) {
        l = e - a.expert_start;
      }
    }
    loc[e] = l;
    if (l >= 0) gof[l] = e;
  }
  __syncthreads();

  // Local layout: kept rows per local expert, 16-row padded starts, 128-row
  // work-tile starts, row-chunk starts.  Warp 0 scans; each lane owns a
  // contiguous range.
  if (warp == 0) {
    const int per = (L + 31) / 32;
    const int l0 = min(L, lane * per);
    const int l1 = min(L, l0 + per);
    int64_t rows = 0, tiles = 0, chunks = 0;
    for (int l = l0; l < l1; ++l) {
      const int g = gof[l];
      int64_t kept = 0;
      if (g >= 0) {
        const int64_t eb = a.expert_base ? a.expert_base[g] : 0;
        kept = g < a.capped_experts ? min64(tot[g], max64(0, cap - eb)) : tot[g];
      }
      lkept[l] = static_cast<int32_t>(kept);
      rows += (kept + B200MOE_BLOCK_ROWS - 1) / B200MOE_BLOCK_ROWS * B200MOE_BLOCK_ROWS;
      tiles += (kept + B200MOE_MTILE_ROWS - 1) / B200MOE_MTILE_ROWS;
      chunks += (kept + B200MOE_CHUNK_ROWS - 1) / B200MOE_CHUNK_ROWS;
    }
    int64_t rows_incl = rows, tiles_incl = tiles, chunks_incl = chunks;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t r = __shfl_up_sync(0xffffffffu, rows_incl, off);
      const int64_t t = __shfl_up_sync(0xffffffffu, tiles_incl, off);
      const int64_t c = __shfl_up_sync(0xffffffffu, chunks_incl, off);
      if (lane >= off) {
        rows_incl += r;
        tiles_incl += t;
        chunks_incl += c;
      }
    }
    int64_t row_off = rows_incl - rows, tile_off = tiles_incl - tiles;
    int64_t chunk_off = chunks_incl - chunks;
    for (int l = l0; l < l1; ++l) {
      lstart[l] = static_cast<int32_t>(row_off);
      mstart[l] = static_cast<int32_t>(tile_off);
      cstart[l] = static_cast<int32_t>(chunk_off);
      const int64_t kept = lkept[l];
      row_off += (kept + B200MOE_BLOCK_ROWS - 1) / B200MOE_BLOCK_ROWS * B200MOE_BLOCK_ROWS;
      tile_off += (kept + B200MOE_MTILE_ROWS - 1) / B200MOE_MTILE_ROWS;
      chunk_off += (kept + B200MOE_CHUNK_ROWS - 1) / B200MOE_CHUNK_ROWS;
    }
    if (lane == 31) {
      red[2] = static_cast<int32_t>(rows_incl);
      red[3] = static_cast<int32_t>(tiles_incl);
      red[4] = static_cast<int32_t>(chunks_incl);
    }
  }
  __syncthreads();

  if (b == 0) {
    const int32_t total_rows = red[2];
    int32_t total_tiles = red[3];
    int32_t total_chunks = a.chunks ? red[4] : 0;
    if (total_rows > a.row_capacity || total_tiles > a.max_mtiles) {
      atomicOr(&g_status, kStatusIndex);
      total_tiles = static_cast<int32_t>(min64(total_tiles, a.max_mtiles));
      total_chunks = static_cast<int32_t>(min64(total_chunks, a.max_mtiles));
    }
    for (int l = tid; l < L; l += blockDim.x) {
      a.expert_offsets[l] = lstart[l];
      a.expert_counts[l] = lkept[l];
      const int32_t kept = lkept[l];
      const int32_t start = lstart[l];
      const int32_t padded = (kept + B200MOE_BLOCK_ROWS - 1) / B200MOE_BLOCK_ROWS * B200MOE_BLOCK_ROWS;
      for (int32_t t = start / B200MOE_BLOCK_ROWS; t < (start + padded) / B200MOE_BLOCK_ROWS; ++t)
        if (t < a.row_capacity / B200MOE_BLOCK_ROWS) a.tile_expert[t] = l;
      const int32_t nm = (kept + B200MOE_MTILE_ROWS - 1) / B200MOE_MTILE_ROWS;
      for (int32_t i = 0; i < nm; ++i) {
        const int64_t m = static_cast<int64_t>(mstart[l]) + i;
        if (m >= a.max_mtiles) break;
        a.mtiles[m * B200MOE_MTILE_WORDS + 0] = l;
        a.mtiles[m * B200MOE_MTILE_WORDS + 1] = start + i * B200MOE_MTILE_ROWS;
        a.mtiles[m * B200MOE_MTILE_WORDS + 2] = min(start + (i + 1) * B200MOE_MTILE_ROWS, start + kept);
      }
      if (a.chunks && kept > 0) {
        // ceil(kept / 256) chunks of equal 16-row multiples; the last one is
        // shorter.  Every chunk is non-empty because kept > 256 * (nc - 1).
        const int32_t nc = (kept + B200MOE_CHUNK_ROWS - 1) / B200MOE_CHUNK_ROWS;
        const int32_t q = ((kept + nc - 1) / nc + B200MOE_BLOCK_ROWS - 1) / B200MOE_BLOCK_ROWS *
                          B200MOE_BLOCK_ROWS;
        for (int32_t i = 0; i < nc; ++i) {
          const int64_t c = static_cast<int64_t>(cstart[l]) + i;
          if (c >= a.max_mtiles) break;
          a.chunks[c * B200MOE_MTILE_WORDS + 0] = l;
          a.chunks[c * B200MOE_MTILE_WORDS + 1] = start + i * q;
          a.chunks[c * B200MOE_MTILE_WORDS + 2] = min(start + (i + 1) * q, start + kept);
        }
      }
    }
    if (tid == 0) {
      a.expert_offsets[L] = total_rows;
      a.counters[B200MOE_CNT_PADDED_ROWS] = total_rows;
      a.counters[B200MOE_CNT_MTILES] = total_tiles;
      a.counters[B200MOE_CNT_CHUNKS] = total_chunks;
    }
  }

  // Rank this block's routes in order and scatter.
  const int64_t begin = static_cast<int64_t>(b) * a.chunk;
  const int64_t end = min(n_routes, begin + a.chunk);
  int my_kept = 0, my_dropped = 0;
  const int32_t route_sentinel = static_cast<int32_t>(a.num_routes);
  const int32_t row_sentinel = static_cast<int32_t>(a.row_capacity);
  for (int64_t sub = begin; sub < end; sub += kPackThreads) {
    const int64_t r = sub + tid;
    const bool active = r < end;
    const int key = active ? route_key(a.ids[r], E) : -1 - lane;  // inactive lanes stay alone
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(peers & lanemask_lt());
    if (active && rank == 0) warp_cnt[warp * E1 + key] = __popc(peers);
    __syncthreads();
    int64_t pos = 0;
    if (active) {
      int32_t before = run[key];
      for (int w = 0; w < warp; ++w) before += warp_cnt[w * E1 + key];
      pos = static_cast<int64_t>(base[key]) + before + rank;
    }
    __syncthreads();
    if (active && rank == 0) {
      // Leaders of different warps may share a key.
      atomicAdd(&run[key], __popc(peers));
      warp_cnt[warp * E1 + key] = 0;
    }
    __syncwarp();
    if (active) {
      int32_t rr = row_sentinel, cr = route_sentinel;
      if (key < E) {
        const int64_t eb = a.expert_base ? a.expert_base[key] : 0;
        const bool capped = key < a.capped_experts;
        if (capped && eb + pos >= cap) {
          a.ids[r] = E;
          if (a.weights) a.weights[r] = __float2bfloat16_rn(0.f);
          ++my_dropped;
        } else {
          const int l = loc[key];
          if (l >= 0) {
            const int64_t p = static_cast<int64_t>(lstart[l]) + pos;
            if (p < a.row_capacity) {
              a.row_route[p] = static_cast<int32_t>(r);
              rr = static_cast<int32_t>(p);
              cr = static_cast<int32_t>(r);
              my_kept += capped;
            } else {
              atomicOr(&g_status, kStatusIndex);
            }
          }
        }
      }
      a.route_row[r] = rr;
      if (a.combine_rows) a.combine_rows[r] = cr;
    }
  }
  // Block totals -> global counters.
  for (int off = 16; off > 0; off >>= 1) {
    my_kept += __shfl_xor_sync(0xffffffffu, my_kept, off);
    my_dropped += __shfl_xor_sync(0xffffffffu, my_dropped, off);
  }
  if (lane == 0) {
    atomicAdd(&red[0], my_kept);
    atomicAdd(&red[1], my_dropped);
  }
  __syncthreads();
  if (tid == 0) {
    atomicAdd(&a.counters[B200MOE_CNT_LOCAL_KEPT], red[0]);
    atomicAdd(&a.counters[B200MOE_CNT_DROPPED], red[1]);
    if (a.stats) {
      atomicAdd(reinterpret_cast<unsigned long long *>(&a.stats[0]),
                static_cast<unsigned long long>(red[0]));
      atomicAdd(reinterpret_cast<unsigned long long *>(&a.stats[1]),
                static_cast<unsigned long long>(red[1]));
    }
  }
}

__global__ void histogram_kernel(const int64_t *__restrict__ ids, int64_t num_routes,
                                 int num_experts, int32_t *__restrict__ counts) {
  extern __shared__ int32_t sh[];
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < num_routes;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = ids[r];
    if (e >= 0 && e < num_experts) atomicAdd(&sh[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x)
    if (sh[e]) atomicAdd(&counts[e], sh[e]);
}

// Routing done inside the packing launch (b200moe_route_pack).
struct RouteSpec {
  const void *logits;
  int dtype;
  int64_t tokens;
  int top_k;
  int renormalize;
};

template <typename T>
int launch_route_pack(const RouteSpec &r, const ScatterArgs &a, size_t smem, cudaStream_t s) {
  const int vpl = (a.num_experts + 31) / 32;
  const T *lg = static_cast<const T *>(r.logits);
#define B200_ROUTE_PACK_CASE(V)                                                             \
  if (vpl <= V) {                                                                           \
    if (smem > 48 * 1024)                                                                   \
      B200_CUDA(cudaFuncSetAttribute(route_pack_kernel<T, V>,                               \
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,           \
                                     static_cast<int>(smem)));                              \
    B200_LAUNCH_PDL(kPdlPack, route_pack_kernel<T, V>, dim3(1), dim3(kPackThreads), smem, s, \
                    lg, r.tokens, r.top_k, r.renormalize, a);                               \
    B200_LAUNCHED();                                                                        \
    return B200MOE_OK;                                                                      \
  }
  B200_ROUTE_PACK_CASE(1)
  B200_ROUTE_PACK_CASE(2)
  B200_ROUTE_PACK_CASE(4)
  B200_ROUTE_PACK_CASE(8)
  B200_ROUTE_PACK_CASE(16)
  B200_ROUTE_PACK_CASE(32)
#undef B200_ROUTE_PACK_CASE
  set_error("num_experts %d exceeds 1024", a.num_experts);
  return B200MOE_EUNSUPPORTED;
}

size_t scatter_smem_bytes(int num_experts, int num_local) {
  const size_t E1 = static_cast<size_t>(num_experts) + 1;
  return sizeof(int32_t) * (E1 * (4 + kPackWarps) + 5 * static_cast<size_t>(num_local) + 5);
}

}  // namespace
}  // namespace b200moe

static int pack_routes_impl(int64_t *expert_ids, void *route_weights, int64_t num_routes,
                            int num_experts, int num_shared_experts,
                            const int64_t *local_index, int expert_start,
                            int num_local_experts, const int32_t *expert_base, int64_t capacity,
                            const int64_t *capacity_dev, const int32_t *route_count,
                            int64_t row_capacity, int32_t *row_route, int32_t *route_row,
                            int32_t *combine_rows, int32_t *tile_expert, int32_t *expert_offsets,
                            int32_t *expert_counts, int32_t *mtiles, int64_t max_mtiles,
                            int32_t *chunks, int32_t *counters, int64_t *stats, void *scratch,
                            size_t scratch_bytes, void *stream,
                            const b200moe::RouteSpec *route = nullptr) {
  using namespace b200moe;
  B200_ARG(num_routes >= 0 && num_routes < (int64_t)0x7fffffff, "num_routes out of range");
  B200_ARG(num_experts >= 1 && num_experts <= 4096, "num_experts must be in [1, 4096]");
  B200_ARG(num_local_experts >= 1 && num_local_experts <= num_experts,
           "num_local_experts must be in [1, num_experts]");
  B200_ARG(counters != nullptr && expert_offsets && expert_counts, "null output pointer");
  B200_ARG(num_shared_experts >= 0 && num_shared_experts < num_experts,
           "num_shared_experts must be in [0, num_experts)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (num_routes == 0) {
    B200_CUDA(cudaMemsetAsync(counters, 0, sizeof(int32_t) * B200MOE_NUM_COUNTERS, s));
    B200_CUDA(cudaMemsetAsync(expert_offsets, 0, sizeof(int32_t) * (num_local_experts + 1), s));
    B200_CUDA(cudaMemsetAsync(expert_counts, 0, sizeof(int32_t) * num_local_experts, s));
    return B200MOE_OK;
  }
  B200_ARG(expert_ids && row_route && route_row && tile_expert && mtiles, "null pointer argument");
  B200_ARG(row_capacity >= b200moe_pack_row_capacity(num_routes, num_local_experts) &&
               row_capacity % B200MOE_BLOCK_ROWS == 0 && row_capacity < (int64_t)0x7fffffff,
           "row_capacity %lld too small or not a multiple of 16", (long long)row_capacity);
  B200_ARG(max_mtiles >= b200moe_pack_max_mtiles(num_routes, num_local_experts),
           "max_mtiles too small");
  const auto g = pack_geometry(num_routes);
  const size_t need = static_cast<size_t>(g.nblk) * (num_experts + 1) * sizeof(int32_t);
  B200_ARG(scratch != nullptr && scratch_bytes >= need, "scratch needs %zu bytes", need);
  int32_t *hist = static_cast<int32_t *>(scratch);

  const bool single = g.nblk == 1;
  if (!single) {
    const size_t hist_smem = sizeof(int32_t) * (num_experts + 1);
    B200_LAUNCH_PDL(kPdlPack, pack_hist_kernel, dim3(g.nblk), dim3(kPackThreads), hist_smem, s,
        expert_ids, num_routes, route_count, num_experts, g.chunk, hist, row_route, row_capacity,
        tile_expert, counters);
    B200_LAUNCHED();
  }

  ScatterArgs a;
  a.ids = expert_ids;
  a.weights = static_cast<__nv_bfloat16 *>(route_weights);
  a.num_routes = num_routes;
  a.num_experts = num_experts;
  a.local_index = local_index;
  a.expert_start = expert_start;
  a.num_local = num_local_experts;
  a.expert_base = expert_base;
  a.capacity = capacity;
  a.capped_experts = num_experts - num_shared_experts;
  a.capacity_dev = capacity_dev;
  a.route_count = route_count;
  a.row_capacity = row_capacity;
  a.row_route = row_route;
  a.route_row = route_row;
  a.combine_rows = combine_rows;
  a.tile_expert = tile_expert;
  a.expert_offsets = expert_offsets;
  a.expert_counts = expert_counts;
  a.mtiles = mtiles;
  a.max_mtiles = max_mtiles;
  a.chunks = chunks;
  a.counters = counters;
  a.stats = stats;
  a.hist = hist;
  a.chunk = g.chunk;
  a.nblk = g.nblk;
  a.single = single ? 1 : 0;
  const size_t smem = scatter_smem_bytes(num_experts, num_local_experts);
  if (route != nullptr) {
    B200_ARG(single && route->tokens * route->top_k == num_routes,
             "routing inside the packing launch needs num_tokens * top_k = num_routes <= %d",
             B200MOE_ROUTE_PACK_MAX_ROUTES);
    B200_ARG(route_weights != nullptr && route->logits != nullptr, "null pointer argument");
    switch (route->dtype) {
      case B200MOE_F32: return launch_route_pack<float>(*route, a, smem, s);
      case B200MOE_BF16: return launch_route_pack<__nv_bfloat16>(*route, a, smem, s);
      case B200MOE_F16: return launch_route_pack<__half>(*route, a, smem, s);
      default:
        set_error("unsupported logits dtype code %d", route->dtype);
        return B200MOE_EINVAL;
    }
  }
  if (smem > 48 * 1024) {
    B200_CUDA(cudaFuncSetAttribute(pack_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem)));
  }
  B200_LAUNCH_PDL(kPdlPack, pack_scatter_kernel, dim3(g.nblk), dim3(kPackThreads), smem, s, a);
  B200_LAUNCHED();
  return B200MOE_OK;
}

extern "C" {

int64_t b200moe_pack_row_capacity(int64_t num_routes, int num_local_experts) {
  const int64_t active = num_routes < num_local_experts ? num_routes : num_local_experts;
  const int64_t rows = num_routes + active * (B200MOE_BLOCK_ROWS - 1);
  return (rows + B200MOE_BLOCK_ROWS - 1) / B200MOE_BLOCK_ROWS * B200MOE_BLOCK_ROWS;
}

int64_t b200moe_pack_max_mtiles(int64_t num_routes, int num_local_experts) {
  const int64_t active = num_routes < num_local_experts ? num_routes : num_local_experts;
  return (num_routes + B200MOE_MTILE_ROWS - 1) / B200MOE_MTILE_ROWS + active;
}

size_t b200moe_pack_scratch_bytes(int64_t num_routes, int num_experts) {
  const auto g = b200moe::pack_geometry(num_routes);
  return static_cast<size_t>(g.nblk) * (static_cast<size_t>(num_experts) + 1) * sizeof(int32_t);
}

int b200moe_pack_routes(int64_t *expert_ids, void *route_weights, int64_t num_routes,
                        int num_experts, const int64_t *local_index, int expert_start,
                        int num_local_experts, const int32_t *expert_base, int64_t capacity,
                        int64_t row_capacity, int32_t *row_route, int32_t *route_row,
                        int32_t *combine_rows, int32_t *tile_expert, int32_t *expert_offsets,
                        int32_t *expert_counts, int32_t *mtiles, int64_t max_mtiles,
                        int32_t *chunks, int32_t *counters, int64_t *stats, void *scratch,
                        size_t scratch_bytes, void *stream) {
  return pack_routes_impl(expert_ids, route_weights, num_routes, num_experts, 0, local_index,
                          expert_start, num_local_experts, expert_base, capacity, nullptr,
                          nullptr, row_capacity, row_route, route_row, combine_rows,
                          tile_expert, expert_offsets, expert_counts, mtiles, max_mtiles, chunks,
                          counters, stats, scratch, scratch_bytes, stream);
}

int b200moe_pack_routes_device_bounds(
    int64_t *expert_ids, void *route_weights, int64_t num_routes, const int32_t *route_count,
    int num_experts, const int64_t *local_index, int expert_start, int num_local_experts,
    const int32_t *expert_base, int64_t capacity, const int64_t *capacity_dev,
    int64_t row_capacity, int32_t *row_route, int32_t *route_row, int32_t *combine_rows,
    int32_t *tile_expert, int32_t *expert_offsets, int32_t *expert_counts, int32_t *mtiles,
    int64_t max_mtiles, int32_t *chunks, int32_t *counters, int64_t *stats, void *scratch,
    size_t scratch_bytes, void *stream) {
  return pack_routes_impl(expert_ids, route_weights, num_routes, num_experts, 0, local_index,
                          expert_start, num_local_experts, expert_base, capacity, capacity_dev,
                          route_count, row_capacity, row_route, route_row, combine_rows,
                          tile_expert, expert_offsets, expert_counts, mtiles, max_mtiles, chunks,
                          counters, stats, scratch, scratch_bytes, stream);
}

int b200moe_pack_routes_shared(int64_t *expert_ids, void *route_weights, int64_t num_routes,
                               int num_experts, int num_shared_experts,
                               const int64_t *local_index, int expert_start,
                               int num_local_experts, int64_t capacity, int64_t row_capacity,
                               int32_t *row_route, int32_t *route_row, int32_t *combine_rows,
                               int32_t *tile_expert, int32_t *expert_offsets,
                               int32_t *expert_counts, int32_t *mtiles, int64_t max_mtiles,
                               int32_t *chunks, int32_t *counters, int64_t *stats,
                               void *scratch, size_t scratch_bytes, void *stream) {
  return pack_routes_impl(expert_ids, route_weights, num_routes, num_experts,
                          num_shared_experts, local_index, expert_start, num_local_experts,
                          nullptr, capacity, nullptr, nullptr, row_capacity, row_route,
                          route_row, combine_rows, tile_expert, expert_offsets, expert_counts,
                          mtiles, max_mtiles, chunks, counters, stats, scratch, scratch_bytes,
                          stream);
}

int b200moe_route_pack(const void *logits, int logits_dtype, int64_t num_tokens,
                       int num_experts, int top_k, int renormalize, void *weights,
                       int64_t *expert_ids, const int64_t *local_index, int expert_start,
                       int num_local_experts, int64_t capacity, int64_t row_capacity,
                       int32_t *row_route, int32_t *route_row, int32_t *combine_rows,
                       int32_t *tile_expert, int32_t *expert_offsets, int32_t *expert_counts,
                       int32_t *mtiles, int64_t max_mtiles, int32_t *chunks, int32_t *counters,
                       int64_t *stats, void *scratch, size_t scratch_bytes, void *stream) {
  B200_ARG(num_tokens >= 1, "num_tokens must be >= 1");
  B200_ARG(top_k >= 1 && top_k <= num_experts, "top_k must be between 1 and num_experts");
  B200_UNSUPPORTED(top_k <= 32, "top_k %d > 32 is not supported", top_k);
  B200_UNSUPPORTED(num_experts <= 1024, "num_experts %d > 1024 is not supported", num_experts);
  B200_ARG(num_tokens * top_k <= B200MOE_ROUTE_PACK_MAX_ROUTES,
           "num_tokens * top_k must be <= %d", B200MOE_ROUTE_PACK_MAX_ROUTES);
  const b200moe::RouteSpec route{logits, logits_dtype, num_tokens, top_k, renormalize};
  return pack_routes_impl(expert_ids, weights, num_tokens * top_k, num_experts, 0, local_index,
                          expert_start, num_local_experts, nullptr, capacity, nullptr, nullptr,
                          row_capacity, row_route, route_row, combine_rows, tile_expert,
                          expert_offsets, expert_counts, mtiles, max_mtiles, chunks, counters,
                          stats, scratch, scratch_bytes, stream, &route);
}

int b200moe_expert_histogram(const int64_t *expert_ids, int64_t num_routes, int num_experts,
                             int32_t *counts, void *stream) {
  using namespace b200moe;
  B200_ARG(num_experts >= 1 && num_experts <= 4096, "num_experts must be in [1, 4096]");
  B200_ARG(counts != nullptr, "counts must not be NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  B200_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * num_experts, s));
  if (num_routes <= 0) return B200MOE_OK;
  B200_ARG(expert_ids != nullptr, "expert_ids must not be NULL");
  int64_t blocks = (num_routes + 1023) / 1024;
  if (blocks > 4 * sm_count()) blocks = 4 * sm_count();
  histogram_kernel<<<static_cast<int>(blocks), 256, sizeof(int32_t) * num_experts, s>>>(
      expert_ids, num_routes, num_experts, counts);
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Packing without caller-provided scratch.
//
// Some callers cannot hand this library a scratch buffer: embedders that have
// already given almost all device memory to their own fixed-size pools (for
// example a KV-cache arena that reserves the remaining HBM at start-up), and
// plain C / FFI hosts with no device allocator of their own.  For them the
// per-block histograms of b200moe_pack_routes live in one file-scope device
// array instead.  That array is part of the library image: every GPU that
// loads the library holds it (kPackStaticScratchBytes) until the process
// exits, and nothing is allocated at call time.
// ---------------------------------------------------------------------------
#include <mutex>

namespace b200moe {
namespace {

constexpr size_t kPackStaticScratchBytes = 256 * 1024;
static __device__ __align__(256) int32_t g_pack_static_scratch[kPackStaticScratchBytes / 4];

std::mutex g_static_scratch_mutex;
void *g_static_scratch_addr[64] = {nullptr};
unsigned long long g_static_scratch_ctx[64] = {0};

// Unique id of the calling thread's current CUDA context (cuCtxGetId, fetched
// from the driver at run time); false when there is no current context or
// the driver cannot say.
bool current_context_id(unsigned long long *id) {
  using GetCurrent = CUresult (*)(CUcontext *);
  using GetId = CUresult (*)(CUcontext, unsigned long long *);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static bool resolved = false;
  if (!resolved) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
    resolved = true;
  }
  if (get_current == nullptr || get_id == nullptr) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

// Device address of the static array in the current device's context.  The
// first call on a device (and the first call after that device's context was
// destroyed and re-created, e.g. by cudaDeviceReset) looks it up with
// cudaGetSymbolAddress, that device current; later calls in the same context
// reuse the address.
int static_scratch_address(void **out) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) {
    set_error("device ordinal %d out of range for the static scratch table", dev);
    return B200MOE_EUNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  unsigned long long ctx = 0;
  const bool known = current_context_id(&ctx);
  if (g_static_scratch_addr[dev] == nullptr || !known || ctx != g_static_scratch_ctx[dev]) {
    void *p = nullptr;
    B200_CUDA(cudaGetSymbolAddress(&p, g_pack_static_scratch));
    unsigned long long now = 0;
    // Without a context id the address is looked up on every call.
    g_static_scratch_addr[dev] = current_context_id(&now) ? p : nullptr;
    g_static_scratch_ctx[dev] = now;
    *out = p;
    return B200MOE_OK;
  }
  *out = g_static_scratch_addr[dev];
  return B200MOE_OK;
}

}  // namespace
}  // namespace b200moe

extern "C" {

size_t b200moe_pack_static_scratch_capacity(void) { return b200moe::kPackStaticScratchBytes; }

int b200moe_pack_routes_static_scratch(
    int64_t *expert_ids, void *route_weights, int64_t num_routes, int num_experts,
    const int64_t *local_index, int expert_start, int num_local_experts,
    const int32_t *expert_base, int64_t capacity, int64_t row_capacity, int32_t *row_route,
    int32_t *route_row, int32_t *combine_rows, int32_t *tile_expert, int32_t *expert_offsets,
    int32_t *expert_counts, int32_t *mtiles, int64_t max_mtiles, int32_t *counters,
    int64_t *stats, void *stream) {
  const size_t need = b200moe_pack_scratch_bytes(num_routes, num_experts);
  B200_ARG(need <= b200moe::kPackStaticScratchBytes,
           "%lld routes over %d experts need %zu scratch bytes; the static scratch holds %zu "
           "(use b200moe_pack_routes with a caller buffer)",
           (long long)num_routes, num_experts, need, b200moe::kPackStaticScratchBytes);
  void *scratch = nullptr;
  const int rc = b200moe::static_scratch_address(&scratch);
  if (rc != B200MOE_OK) return rc;
  // The histogram kernel writes every word the scatter kernel reads, so the
  // array needs no clearing between calls.
  return b200moe_pack_routes(expert_ids, route_weights, num_routes, num_experts, local_index,
                             expert_start, num_local_experts, expert_base, capacity,
                             row_capacity, row_route, route_row, combine_rows, tile_expert,
                             expert_offsets, expert_counts, mtiles, max_mtiles, nullptr,
                             counters, stats, scratch, b200moe::kPackStaticScratchBytes, stream);
}

}  // extern "C"
