// Expert-parallel exchange over NVLink peer memory.
//
// The reference's cross-DP backends all-gather every replica's tokens and
// reduce partial outputs (nanovllm/layers/moe.py:942-1018).  Here each EP rank
// routes its own tokens and moves only what the routes need, with plain peer
// loads/stores into buffers that every rank maps from every other rank
// (CUDA IPC), so no size has to reach the host:
//   histogram (capacity only): every rank's per-expert counts and token count
//             go to every peer; each rank derives the capacity positions of
//             the global (rank-major, token-major, slot-minor) route order;
//   dispatch: each token row once per destination that owns one of its kept
//             routes, into the destination's region for this source, plus one
//             16-byte record per route {expert, token slot, weight, route id}
//             and the two counts in the destination's mailbox;
//   return:   the destination writes each route's bf16 result row into the
//             source's return buffer at the route's own index, so the source
//             combines in slot order exactly as with one rank.
// Regions are sized for the largest batch (max_tokens per rank), so the
// addresses are fixed and every step can be captured in a CUDA graph.
//
// Synchronisation: each phase ends with a release store of the phase's epoch
// into every peer's flag for this source (by the last CTA of the producing
// kernel, after every CTA fenced its stores at system scope); consumers wait
// with acquire loads until all sources' flags reach the epoch.  Waits are
// bounded (2 s): on expiry the status word gets the timeout bit and the
// kernel returns.  Epochs live in device memory and advance once per
// exchange, identically on every rank, so captured graphs replay correctly.
// Buffer reuse is safe without extra handshakes: a source writes a peer's
// region again only after it received that peer's return rows of the
// previous exchange, which the peer sends after its last read of the region.
#include <string.h>

#include "common.cuh"

namespace b200moe {
namespace {

constexpr int kNvlMaxRanks = 16;
constexpr int kPhaseHist = 0;
constexpr int kPhaseDispatch = 1;
constexpr int kPhaseReturn = 2;
constexpr int kNvlPhases = 3;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Byte offsets of one rank's exchange buffer (B200MOE_NVL_* word order).
struct NvlLayout {
  int64_t flags;     // uint64 [kNvlPhases][kNvlMaxRanks]: epoch each source reached
  int64_t control;   // uint64 epoch; uint32 done[kNvlPhases] (CTA retirement counters)
  int64_t mailbox;   // int32 [kNvlMaxRanks][4]: {tokens, routes, 0, 0} from each source
  int64_t hist;      // int32 [kNvlMaxRanks][num_experts + 1]: counts + token count
  int64_t meta;      // int32 [kNvlMaxRanks + 1]: received route prefix, then total
  int64_t records;   // int4 [kNvlMaxRanks][route_cap]
  int64_t tokens;    // bf16 [kNvlMaxRanks][max_tokens][hidden]
  int64_t returned;  // bf16 [max_tokens * top_k][hidden]
  int64_t route_cap; // records per source region
  int64_t total;     // bytes
};
static_assert(sizeof(NvlLayout) == B200MOE_NVL_LAYOUT_WORDS * sizeof(int64_t),
              "layout words");

struct Peers {
  char *base[kNvlMaxRanks];
};

__host__ __device__ __forceinline__ int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

NvlLayout make_layout(int ep_size, int64_t max_tokens, int top_k, int num_experts,
                      int num_local_experts, int hidden) {
  NvlLayout l;
  const int64_t per_token = top_k < num_local_experts ? top_k : num_local_experts;
  l.route_cap = max_tokens * per_token;
  int64_t off = 0;
  l.flags = off;
  off = align256(off + int64_t(kNvlPhases) * kNvlMaxRanks * 8);
  l.control = off;
  off = align256(off + 8 + 4 * kNvlPhases);
  l.mailbox = off;
  off = align256(off + int64_t(kNvlMaxRanks) * 16);
  l.hist = off;
  off = align256(off + int64_t(kNvlMaxRanks) * (num_experts + 1) * 4);
  l.meta = off;
  off = align256(off + int64_t(kNvlMaxRanks + 1) * 4);
  l.records = off;
  off = align256(off + int64_t(ep_size) * l.route_cap * 16);
  l.tokens = off;
  off = align256(off + int64_t(ep_size) * max_tokens * hidden * 2);
  l.returned = off;
  off = align256(off + max_tokens * top_k * hidden * 2);
  l.total = off;
  return l;
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t *p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t *flag_ptr(char *base, const NvlLayout &l, int phase,
                                              int src) {
  return reinterpret_cast<uint64_t *>(base + l.flags) + phase * kNvlMaxRanks + src;
}

__device__ __forceinline__ uint64_t *epoch_ptr(char *base, const NvlLayout &l) {
  return reinterpret_cast<uint64_t *>(base + l.control);
}

__device__ __forceinline__ uint32_t *done_ptr(char *base, const NvlLayout &l, int phase) {
  return reinterpret_cast<uint32_t *>(base + l.control + 8) + phase;
}

// Wait until every source's flag of `phase` reached this rank's epoch.
// Called by threads 0..ep_size-1 (one source each).  Bounded.
__device__ void wait_sources(char *own, const NvlLayout &l, int phase, int ep_size) {
  const int s = threadIdx.x;
  if (s >= ep_size) return;
  const uint64_t e = *epoch_ptr(own, l);
  const uint64_t *f = flag_ptr(own, l, phase, s);
  if (ld_acquire_sys(f) >= e) return;
  const uint64_t start = global_timer_ns();
  while (ld_acquire_sys(f) < e) {
    __nanosleep(64);
    if (global_timer_ns() - start > kWaitLimitNs) {
      atomicOr(&g_status, kStatusTimeout);
      return;
    }
  }
}

// End of a producing kernel: every thread fences its stores at system scope,
// the last CTA to retire (optionally) advances the epoch and publishes it to
// every peer's flag for this source.
__device__ void retire_and_signal(const Peers &peers, const NvlLayout &l, int phase, int rank,
                                  int ep_size, bool bump_epoch) {
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  char *own = peers.base[rank];
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(done_ptr(own, l, phase), 1u);
    last = prev == gridDim.x - 1;
    if (last) *done_ptr(own, l, phase) = 0u;
  }
  __syncthreads();
  if (!last) return;
  if (threadIdx.x == 0 && bump_epoch) {
    uint64_t *ep = epoch_ptr(own, l);
    *ep = *ep + 1;
  }
  __syncthreads();
  const uint64_t e = *reinterpret_cast<volatile uint64_t *>(epoch_ptr(own, l));
  __threadfence_system();
  if (threadIdx.x < ep_size) st_release_sys(flag_ptr(peers.base[threadIdx.x], l, phase, rank), e);
}

__device__ __forceinline__ int owner_of(int64_t id, int num_experts, const int32_t *owner,
                                        int ep_size) {
  if (id < 0 || id >= num_experts) return -1;
  const int d = owner[id];
  return (d >= 0 && d < ep_size) ? d : -1;
}

__device__ __forceinline__ void copy_row(uint4 *dst, const uint4 *src, int vecs, int lane) {
  int v = lane;
  for (; v + 96 < vecs; v += 128) {
    const uint4 a = src[v], b = src[v + 32], c = src[v + 64], d = src[v + 96];
    dst[v] = a;
    dst[v + 32] = b;
    dst[v + 64] = c;
    dst[v + 96] = d;
  }
  for (; v < vecs; v += 32) dst[v] = src[v];
}

// Capacity agreement, send half (one CTA per rank): this rank's per-expert
// counts and token count go to every peer.  Advances the epoch: it is the
// first phase of an exchange with a capacity limit.
__global__ void __launch_bounds__(1024) nvl_hist_send_kernel(
    const int64_t *__restrict__ ids, int64_t num_tokens, int top_k, int num_experts, int rank,
    int ep_size, const __grid_constant__ Peers peers, NvlLayout l) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int32_t sh[];
  const int E1 = num_experts + 1;
  for (int e = threadIdx.x; e < E1; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int64_t n = num_tokens * top_k;
  for (int64_t r = threadIdx.x; r < n; r += blockDim.x) {
    const int64_t e = ids[r];
    if (e >= 0 && e < num_experts) atomicAdd(&sh[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) sh[num_experts] = static_cast<int32_t>(num_tokens);
  __syncthreads();
  for (int d = 0; d < ep_size; ++d) {
    int32_t *dst = reinterpret_cast<int32_t *>(peers.base[d] + l.hist) + int64_t(rank) * E1;
    for (int e = threadIdx.x; e < E1; e += blockDim.x) dst[e] = sh[e];
  }
  retire_and_signal(peers, l, kPhaseHist, rank, ep_size, true);
}

// Capacity agreement, wait half (one CTA): with every peer's counts in, the
// capacity base of each expert (routes of lower ranks), the global token
// count and, for a capacity factor, the capacity itself.
__global__ void __launch_bounds__(1024) nvl_hist_wait_kernel(
    int top_k, int num_experts, int rank, int ep_size, const __grid_constant__ Peers peers,
    NvlLayout l, double capacity_factor, int32_t *__restrict__ expert_base,
    int64_t *__restrict__ global_tokens, int64_t *__restrict__ capacity) {
  pdl_trigger();
  pdl_wait();
  wait_sources(peers.base[rank], l, kPhaseHist, ep_size);
  __syncthreads();
  const int E1 = num_experts + 1;
  const int32_t *hist = reinterpret_cast<const int32_t *>(peers.base[rank] + l.hist);
  for (int e = threadIdx.x; e < E1; e += blockDim.x) {
    int64_t below = 0, all = 0;
    for (int s = 0; s < ep_size; ++s) {
      const int32_t h = hist[int64_t(s) * E1 + e];
      if (s < rank) below += h;
      all += h;
    }
    if (e < num_experts) {
      expert_base[e] = static_cast<int32_t>(below);
    } else {
      if (global_tokens) *global_tokens = all;
      if (capacity && capacity_factor > 0.0) {
        // max(1, ceil(factor * tokens * top_k / num_experts)), the reference's
        // expression (moe.py:882-885) in its evaluation order, in double.
        const double v = __ddiv_rn(__dmul_rn(__dmul_rn(capacity_factor, double(all)),
                                             double(top_k)),
                                   double(num_experts));
        const double c = ceil(v);
        *capacity = c < 1.0 ? 1 : static_cast<int64_t>(c);
      }
    }
  }
}

// Dispatch: one warp per token (grid-stride): its row to every destination
// that owns one of its kept routes, then its route records; the CTA 0 writes
// the counts into every destination's mailbox.  combine_rows[r] = r for
// routes that leave for some rank, else the sentinel num_tokens * top_k.
__global__ void __launch_bounds__(256) nvl_dispatch_kernel(
    const __nv_bfloat16 *__restrict__ x, int hidden, const int64_t *__restrict__ ids,
    const __nv_bfloat16 *__restrict__ rw, int64_t num_tokens, int top_k, int num_experts,
    const int32_t *__restrict__ owner, int rank, int ep_size,
    const int32_t *__restrict__ send_token_slot, const int32_t *__restrict__ route_dest_slot,
    const int32_t *__restrict__ counts, const __grid_constant__ Peers peers, NvlLayout l, int64_t max_tokens,
    int bump_epoch, int32_t *__restrict__ combine_rows) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int vecs = hidden / 8;
  const int64_t routes = num_tokens * top_k;
  for (int64_t t = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); t < num_tokens;
       t += int64_t(gridDim.x) * warps) {
    const uint4 *src = reinterpret_cast<const uint4 *>(x + t * hidden);
    for (int d = 0; d < ep_size; ++d) {
      const int32_t slot = send_token_slot[t * ep_size + d];
      if (slot < 0 || slot >= max_tokens) continue;
      uint4 *dst = reinterpret_cast<uint4 *>(peers.base[d] + l.tokens) +
                   ((int64_t(rank) * max_tokens + slot) * vecs);
      copy_row(dst, src, vecs, lane);
    }
    if (lane < top_k) {
      const int64_t r = t * top_k + lane;
      const int64_t id = ids[r];
      const int d = owner_of(id, num_experts, owner, ep_size);
      const int32_t slot = route_dest_slot[r];
      const bool sent = d >= 0 && slot >= 0 && slot < l.route_cap;
      if (sent) {
        int4 *rec = reinterpret_cast<int4 *>(peers.base[d] + l.records) +
                    (int64_t(rank) * l.route_cap + slot);
        *rec = make_int4(static_cast<int>(id), send_token_slot[t * ep_size + d],
                         static_cast<int>(__bfloat16_as_ushort(rw[r])), static_cast<int>(r));
      }
      combine_rows[r] = sent ? static_cast<int32_t>(r) : static_cast<int32_t>(routes);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < ep_size) {
    const int d = threadIdx.x;
    int32_t *mb = reinterpret_cast<int32_t *>(peers.base[d] + l.mailbox) + rank * 4;
    const int32_t nt = num_tokens ? counts[d] : 0;
    const int32_t nr = num_tokens ? counts[ep_size + d] : 0;
    mb[0] = nt;
    mb[1] = nr;
    if (nt > max_tokens || nr > l.route_cap) atomicOr(&g_status, kStatusIndex);
  }
  retire_and_signal(peers, l, kPhaseDispatch, rank, ep_size, bump_epoch != 0);
}

// Receiver, one CTA: wait for every source's dispatch, then the prefix of the
// received route counts (meta[s] = first flat route of source s,
// meta[ep_size] = total) and the device route count.
__global__ void nvl_receive_wait_kernel(int rank, int ep_size, const __grid_constant__ Peers peers, NvlLayout l,
                                        int32_t *__restrict__ route_count) {
  pdl_trigger();
  pdl_wait();
  char *own = peers.base[rank];
  wait_sources(own, l, kPhaseDispatch, ep_size);
  __syncthreads();
  if (threadIdx.x == 0) {
    const int32_t *mb = reinterpret_cast<const int32_t *>(own + l.mailbox);
    int32_t *meta = reinterpret_cast<int32_t *>(own + l.meta);
    int32_t acc = 0;
    for (int s = 0; s < ep_size; ++s) {
      meta[s] = acc;
      acc += min(static_cast<int64_t>(mb[s * 4 + 1]), l.route_cap);
    }
    meta[ep_size] = acc;
    *route_count = acc;
  }
}

// Received records -> flat route arrays in (source, slot) order.
__global__ void __launch_bounds__(256) nvl_unpack_kernel(
    int rank, int ep_size, const __grid_constant__ Peers peers, NvlLayout l, int64_t max_tokens,
    int64_t *__restrict__ ids, int32_t *__restrict__ token_of_route,
    __nv_bfloat16 *__restrict__ rw, int32_t *__restrict__ src_rank,
    int32_t *__restrict__ src_route) {
  pdl_trigger();
  pdl_wait();
  char *own = peers.base[rank];
  const int32_t *meta = reinterpret_cast<const int32_t *>(own + l.meta);
  const int32_t total = meta[ep_size];
  const int4 *rec = reinterpret_cast<const int4 *>(own + l.records);
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < total;
       j += int64_t(gridDim.x) * blockDim.x) {
    int s = 0;
    while (s + 1 < ep_size && j >= meta[s + 1]) ++s;
    const int4 m = rec[int64_t(s) * l.route_cap + (j - meta[s])];
    ids[j] = m.x;
    const int32_t slot = m.y;
    if (slot < 0 || slot >= max_tokens) atomicOr(&g_status, kStatusIndex);
    token_of_route[j] = static_cast<int32_t>(int64_t(s) * max_tokens + min64(max64(slot, 0), max_tokens - 1));
    rw[j] = __ushort_as_bfloat16(static_cast<unsigned short>(m.z & 0xffff));
    src_rank[j] = s;
    src_route[j] = m.w;
  }
}

// Return: one warp per received route (grid-stride over the device count):
// its result row into the source rank's return buffer at the route's index.
__global__ void __launch_bounds__(256) nvl_return_kernel(
    const __nv_bfloat16 *__restrict__ y, int hidden, const int32_t *__restrict__ src_rank,
    const int32_t *__restrict__ src_route, const int32_t *__restrict__ route_count,
    int64_t max_routes, int64_t max_source_routes, int rank, int ep_size,
    const __grid_constant__ Peers peers, NvlLayout l) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int vecs = hidden / 8;
  // More routes than y has rows (a host bound below what the peers sent):
  // flag it and return only the rows that exist.
  const int64_t n = min64(max64(*route_count, 0), max_routes);
  if (blockIdx.x == 0 && threadIdx.x == 0 && *route_count > max_routes)
    atomicOr(&g_status, kStatusIndex);
  for (int64_t j = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); j < n;
       j += int64_t(gridDim.x) * warps) {
    const int s = src_rank[j];
    const int64_t r = src_route[j];
    if (s < 0 || s >= ep_size || r < 0 || r >= max_source_routes) {
      if (lane == 0) atomicOr(&g_status, kStatusIndex);
      continue;
    }
    uint4 *dst = reinterpret_cast<uint4 *>(peers.base[s] + l.returned) + r * vecs;
    copy_row(dst, reinterpret_cast<const uint4 *>(y + j * hidden), vecs, lane);
  }
  retire_and_signal(peers, l, kPhaseReturn, rank, ep_size, false);
}

// Destination, one CTA: the received routes' rows were written into the
// sources' return buffers by the down GEMM's epilogue (b200moe_expert_down_scatter,
// earlier in this stream); publish the return phase.
__global__ void nvl_signal_return_kernel(int rank, int ep_size,
                                         const __grid_constant__ Peers peers, NvlLayout l) {
  pdl_trigger();
  pdl_wait();
  retire_and_signal(peers, l, kPhaseReturn, rank, ep_size, false);
}

// Source, one CTA: wait until every destination returned its rows.
__global__ void nvl_return_wait_kernel(int rank, int ep_size, const __grid_constant__ Peers peers, NvlLayout l) {
  pdl_trigger();
  pdl_wait();
  wait_sources(peers.base[rank], l, kPhaseReturn, ep_size);
}

int load_peers(Peers &p, const NvlLayout *&l, const uint64_t *peer_bases, const int64_t *layout,
               int ep_size) {
  for (int i = 0; i < kNvlMaxRanks; ++i) p.base[i] = nullptr;
  for (int i = 0; i < ep_size; ++i) {
    if (peer_bases[i] == 0 || (peer_bases[i] & 255u) != 0) {
      set_error("peer buffer %d is null or not 256-byte aligned", i);
      return B200MOE_EINVAL;
    }
    p.base[i] = reinterpret_cast<char *>(peer_bases[i]);
  }
  l = reinterpret_cast<const NvlLayout *>(layout);
  return B200MOE_OK;
}

int grid_for(int64_t items, int per_cta) {
  const int64_t want = (items + per_cta - 1) / per_cta;
  const int64_t cap = int64_t(sm_count()) * 8;
  return static_cast<int>(want < 1 ? 1 : want > cap ? cap : want);
}

// Driver API entry points for IPC base lookups, fetched at run time.
using GetRange = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
GetRange get_range_fn() {
  static GetRange fn = nullptr;
  static bool resolved = false;
  if (!resolved) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRange>(p);
    resolved = true;
  }
  return fn;
}

}  // namespace
}  // namespace b200moe

#define B200_NVL_CHECK(ep_size, rank)                                                     \
  B200_ARG((ep_size) >= 1 && (ep_size) <= b200moe::kNvlMaxRanks,                          \
           "ep_size must be in [1, %d]", b200moe::kNvlMaxRanks);                          \
  B200_ARG((rank) >= 0 && (rank) < (ep_size), "rank %d out of range", (rank))

extern "C" {

int64_t b200moe_nvl_buffer_bytes(int ep_size, int64_t max_tokens, int top_k, int num_experts,
                                 int num_local_experts, int hidden, int64_t *layout) {
  if (ep_size < 1 || ep_size > b200moe::kNvlMaxRanks || max_tokens < 1 || top_k < 1 ||
      num_experts < 1 || num_local_experts < 1 || hidden < 8 || hidden % 8) {
    b200moe::set_error("bad exchange geometry");
    return -1;
  }
  const b200moe::NvlLayout l =
      b200moe::make_layout(ep_size, max_tokens, top_k, num_experts, num_local_experts, hidden);
  if (layout) *reinterpret_cast<b200moe::NvlLayout *>(layout) = l;
  return l.total;
}

int b200moe_ipc_handle(const void *ptr, void *handle, int64_t *offset) {
  using namespace b200moe;
  B200_ARG(ptr && handle && offset, "null pointer argument");
  GetRange range = get_range_fn();
  B200_UNSUPPORTED(range != nullptr, "cuMemGetAddressRange is unavailable from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) {
    set_error("cuMemGetAddressRange failed with CUresult %d", static_cast<int>(r));
    return B200MOE_ECUDA;
  }
  cudaIpcMemHandle_t h;
  B200_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)));
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return B200MOE_OK;
}

int b200moe_ipc_open(const void *handle, int64_t offset, void **ptr) {
  using namespace b200moe;
  B200_ARG(handle && ptr && offset >= 0, "bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  B200_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = static_cast<char *>(base) + offset;
  return B200MOE_OK;
}

int b200moe_ipc_close(void *ptr, int64_t offset) {
  using namespace b200moe;
  B200_ARG(ptr && offset >= 0, "bad argument");
  B200_CUDA(cudaIpcCloseMemHandle(static_cast<char *>(ptr) - offset));
  return B200MOE_OK;
}

int b200moe_nvl_histogram_send(const int64_t *expert_ids, int64_t num_tokens, int top_k,
                               int num_experts, int rank, int ep_size,
                               const uint64_t *peer_bases, const int64_t *layout, void *stream) {
  using namespace b200moe;
  B200_NVL_CHECK(ep_size, rank);
  B200_ARG(num_tokens >= 0 && top_k >= 1 && num_experts >= 1 && num_experts <= 8192,
           "bad shape");
  B200_ARG(peer_bases && layout && (expert_ids || num_tokens == 0), "null pointer argument");
  Peers p;
  const NvlLayout *l = nullptr;
  const int rc = load_peers(p, l, peer_bases, layout, ep_size);
  if (rc != B200MOE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  B200_LAUNCH_PDL(kPdlExchange, nvl_hist_send_kernel, dim3(1), dim3(1024),
                  sizeof(int32_t) * (num_experts + 1), s, expert_ids, num_tokens, top_k,
                  num_experts, rank, ep_size, p, *l);
  B200_LAUNCHED();
  return B200MOE_OK;
}

int b200moe_nvl_histogram_wait(int top_k, int num_experts, int rank, int ep_size,
                               const uint64_t *peer_bases, const int64_t *layout,
                               double capacity_factor, int32_t *expert_base,
                               int64_t *global_tokens, int64_t *capacity, void *stream) {
  using namespace b200moe;
  B200_NVL_CHECK(ep_size, rank);
  B200_ARG(top_k >= 1 && num_experts >= 1 && num_experts <= 8192, "bad shape");
  B200_ARG(peer_bases && layout && expert_base, "null pointer argument");
  Peers p;
  const NvlLayout *l = nullptr;
  const int rc = load_peers(p, l, peer_bases, layout, ep_size);
  if (rc != B200MOE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  B200_LAUNCH_PDL(kPdlExchange, nvl_hist_wait_kernel, dim3(1), dim3(1024), 0, s, top_k,
                  num_experts, rank, ep_size, p, *l, capacity_factor, expert_base,
                  global_tokens, capacity);
  B200_LAUNCHED();
  return B200MOE_OK;
}

int b200moe_nvl_dispatch(const void *x, int hidden, const int64_t *expert_ids,
                         const void *route_weights, int64_t num_tokens, int top_k,
                         int num_experts, const int32_t *owner, int rank, int ep_size,
                         const int32_t *send_token_slot, const int32_t *route_dest_slot,
                         const int32_t *counts, const uint64_t *peer_bases,
                         const int64_t *layout, int64_t max_tokens, int bump_epoch,
                         int32_t *combine_rows, void *stream) {
  using namespace b200moe;
  B200_NVL_CHECK(ep_size, rank);
  B200_UNSUPPORTED(hidden % 8 == 0, "hidden must be a multiple of 8");
  B200_ARG(top_k >= 1 && top_k <= 32 && num_experts >= 1, "bad shape");
  B200_ARG(num_tokens >= 0 && num_tokens <= max_tokens, "num_tokens %lld exceeds the exchange's "
           "max_tokens %lld", (long long)num_tokens, (long long)max_tokens);
  B200_ARG(peer_bases && layout && owner, "null pointer argument");
  B200_ARG(num_tokens == 0 || (x && expert_ids && route_weights && send_token_slot &&
                               route_dest_slot && counts && combine_rows),
           "null pointer argument");
  Peers p;
  const NvlLayout *l = nullptr;
  const int rc = load_peers(p, l, peer_bases, layout, ep_size);
  if (rc != B200MOE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  B200_LAUNCH_PDL(kPdlExchange, nvl_dispatch_kernel, dim3(grid_for(num_tokens, 8)), dim3(256), 0,
                  s, static_cast<const __nv_bfloat16 *>(x), hidden, expert_ids,
                  static_cast<const __nv_bfloat16 *>(route_weights), num_tokens, top_k,
                  num_experts, owner, rank, ep_size, send_token_slot, route_dest_slot, counts, p,
                  *l, max_tokens, bump_epoch, combine_rows);
  B200_LAUNCHED();
  return B200MOE_OK;
}

int b200moe_nvl_receive(int rank, int ep_size, const uint64_t *peer_bases,
                        const int64_t *layout, int64_t max_tokens, int64_t *expert_ids,
                        int32_t *token_of_route, void *route_weights, int32_t *src_rank,
                        int32_t *src_route, int32_t *route_count, void *stream) {
  using namespace b200moe;
  B200_NVL_CHECK(ep_size, rank);
  B200_ARG(peer_bases && layout && expert_ids && token_of_route && route_weights && src_rank &&
               src_route && route_count && max_tokens >= 1,
           "null pointer argument");
  Peers p;
  const NvlLayout *l = nullptr;
  const int rc = load_peers(p, l, peer_bases, layout, ep_size);
  if (rc != B200MOE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  B200_LAUNCH_PDL(kPdlExchange, nvl_receive_wait_kernel, dim3(1), dim3(32), 0, s, rank, ep_size,
                  p, *l, route_count);
  B200_LAUNCHED();
  B200_LAUNCH_PDL(kPdlExchange, nvl_unpack_kernel,
                  dim3(grid_for(int64_t(ep_size) * l->route_cap, 256)), dim3(256), 0, s, rank,
                  ep_size, p, *l, max_tokens, expert_ids, token_of_route,
                  static_cast<__nv_bfloat16 *>(route_weights), src_rank, src_route);
  B200_LAUNCHED();
  return B200MOE_OK;
}

int b200moe_nvl_return(const void *y, int hidden, const int32_t *src_rank,
                       const int32_t *src_route, const int32_t *route_count, int64_t max_routes,
                       int64_t max_source_routes, int rank, int ep_size,
                       const uint64_t *peer_bases, const int64_t *layout, void *stream) {
  using namespace b200moe;
  B200_NVL_CHECK(ep_size, rank);
  B200_UNSUPPORTED(hidden % 8 == 0, "hidden must be a multiple of 8");
  B200_ARG(peer_bases && layout && route_count && max_routes >= 0 && max_source_routes >= 0,
           "bad argument");
  B200_ARG(max_routes == 0 || (y && src_rank && src_route), "null pointer argument");
  Peers p;
  const NvlLayout *l = nullptr;
  const int rc = load_peers(p, l, peer_bases, layout, ep_size);
  if (rc != B200MOE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  B200_LAUNCH_PDL(kPdlExchange, nvl_return_kernel, dim3(grid_for(max_routes, 8)), dim3(256), 0, s,
                  static_cast<const __nv_bfloat16 *>(y), hidden, src_rank, src_route,
                  route_count, max_routes, max_source_routes, rank, ep_size, p, *l);
  B200_LAUNCHED();
  return B200MOE_OK;
}

int b200moe_nvl_return_signal(int rank, int ep_size, const uint64_t *peer_bases,
                              const int64_t *layout, void *stream) {
  using namespace b200moe;
  B200_NVL_CHECK(ep_size, rank);
  B200_ARG(peer_bases && layout, "null pointer argument");
  Peers p;
  const NvlLayout *l = nullptr;
  const int rc = load_peers(p, l, peer_bases, layout, ep_size);
  if (rc != B200MOE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  B200_LAUNCH_PDL(kPdlExchange, nvl_signal_return_kernel, dim3(1), dim3(32), 0, s, rank, ep_size,
                  p, *l);
  B200_LAUNCHED();
  return B200MOE_OK;
}

int b200moe_nvl_wait_return(int rank, int ep_size, const uint64_t *peer_bases,
                            const int64_t *layout, void *stream) {
  using namespace b200moe;
  B200_NVL_CHECK(ep_size, rank);
  B200_ARG(peer_bases && layout, "null pointer argument");
  Peers p;
  const NvlLayout *l = nullptr;
  const int rc = load_peers(p, l, peer_bases, layout, ep_size);
  if (rc != B200MOE_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  B200_LAUNCH_PDL(kPdlExchange, nvl_return_wait_kernel, dim3(1), dim3(32), 0, s, rank, ep_size, p,
                  *l);
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // extern "C"
