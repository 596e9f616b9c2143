// Expert-parallel dispatch / combine around NCCL all-to-all.
//
// The reference's cross-DP backends all-gather every replica's tokens, route
// the global batch on every rank and reduce the [N*T, H] partial outputs
// (nanovllm/layers/moe.py:942-1018).  Here each rank routes only its own
// tokens and exchanges:
//   dispatch: every token once per destination rank that owns at least one
//             of its kept routes, plus 16-byte route records
//             {expert, token row at the destination, weight, source route};
//   return:   one bf16 row per kept route, in the order it was received, so
//             the source combines its routes in slot order exactly as with
//             EP=1 (moe.py:642-678).
// These kernels build the plan (per-destination slots), pack the payload and
// translate received records; the all-to-all itself is NCCL.
#include "common.cuh"

namespace b200moe {
namespace {

constexpr int kMaxEp = 16;
constexpr int kPlanThreads = 512;

struct Offsets {
  int32_t v[kMaxEp + 1];
};

__device__ __forceinline__ int dest_of(int64_t id, int num_experts, const int32_t *owner,
                                       int ep_size) {
  if (id < 0 || id >= num_experts) return -1;
  const int d = owner[id];
  return (d >= 0 && d < ep_size) ? d : -1;
}

// Ordered slots per destination for tokens and routes, one CTA per
// kPlanThreads tokens (thread = token).  A CTA first counts, per destination,
// the tokens and routes of every token before its range (each CTA reads that
// prefix of the route array itself, so the CTAs need not communicate), then
// stages its own routes' destinations in shared memory with coalesced loads;
// each thread counts its routes per destination, and one block-wide exclusive
// scan of all destinations at once (token sends in the high 16 bits, routes
// in the low 16) gives the token's slot and its first route slot per
// destination, in token order (routes: token-major, then slot, i.e. route
// order) -- the slots of a single pass over the whole batch.  The last CTA
// writes the totals.
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(
    const int64_t *__restrict__ ids, int64_t num_tokens, int top_k, int num_experts,
    const int32_t *__restrict__ owner, int ep_size, int32_t *__restrict__ send_token_slot,
    int32_t *__restrict__ route_dest_slot, int32_t *__restrict__ counts) {
  constexpr int kWarps = kPlanThreads / 32;
  static_assert(kWarps >= kMaxEp, "one warp per destination in the cross-warp scan");
  __shared__ int32_t warp_tot[kWarps][kMaxEp];  // per-warp sums, then warp offsets
  __shared__ int32_t batch_tot[kMaxEp];
  __shared__ int32_t run_tok[kMaxEp];
  __shared__ int32_t run_rt[kMaxEp];
  __shared__ int8_t s_dest[kPlanThreads * 32];  // destinations of the batch's routes
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int N = ep_size;
  if (tid < kMaxEp) {
    run_tok[tid] = 0;
    run_rt[tid] = 0;
  }
  __syncthreads();
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kPlanThreads;

  // Tokens and routes per destination before this CTA's range.
  {
    int32_t tok_c[kMaxEp], rt_c[kMaxEp];
#pragma unroll
    for (int d = 0; d < kMaxEp; ++d) tok_c[d] = rt_c[d] = 0;
    for (int64_t t = tid; t < t0; t += kPlanThreads) {
      int32_t v[kMaxEp];
#pragma unroll
      for (int d = 0; d < kMaxEp; ++d) v[d] = 0;
      for (int s2 = 0; s2 < top_k; ++s2) {
        const int ds = dest_of(ids[t * top_k + s2], num_experts, owner, N);
#pragma unroll
        for (int d = 0; d < kMaxEp; ++d) v[d] += ds == d ? 1 : 0;
      }
#pragma unroll
      for (int d = 0; d < kMaxEp; ++d) {
        tok_c[d] += v[d] > 0 ? 1 : 0;
        rt_c[d] += v[d];
      }
    }
#pragma unroll
    for (int d = 0; d < kMaxEp; ++d) {
      const int32_t tk = __reduce_add_sync(0xffffffffu, tok_c[d]);
      const int32_t rt = __reduce_add_sync(0xffffffffu, rt_c[d]);
      if (lane == 0 && d < N && (tk | rt)) {
        atomicAdd(&run_tok[d], tk);
        atomicAdd(&run_rt[d], rt);
      }
    }
  }

  const int64_t t = t0 + tid;
  const bool valid = t < num_tokens;
  const int64_t r0 = t0 * top_k;
  const int64_t nr = min64(num_tokens - t0, kPlanThreads) * top_k;
  for (int64_t i = tid; i < nr; i += kPlanThreads)
    s_dest[i] = static_cast<int8_t>(dest_of(ids[r0 + i], num_experts, owner, N));
  __syncthreads();
  const int8_t *my_dest = s_dest + static_cast<int64_t>(tid) * top_k;
  // Per destination: routes (low 16 bits, <= kPlanThreads * 32 in a batch)
  // and the token itself (high bits).
  int32_t v[kMaxEp];
#pragma unroll
  for (int d = 0; d < kMaxEp; ++d) v[d] = 0;
  if (valid)
    for (int s2 = 0; s2 < top_k; ++s2) {
      const int ds = my_dest[s2];
#pragma unroll
      for (int d = 0; d < kMaxEp; ++d) v[d] += ds == d ? 1 : 0;
    }
#pragma unroll
  for (int d = 0; d < kMaxEp; ++d) v[d] |= (v[d] > 0 ? 1 : 0) << 16;
  int32_t incl[kMaxEp];
#pragma unroll
  for (int d = 0; d < kMaxEp; ++d) {
    int32_t x = v[d];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += u;
    }
    incl[d] = x;
  }
  if (lane == 31) {
#pragma unroll
    for (int d = 0; d < kMaxEp; ++d) warp_tot[warp][d] = incl[d];
  }
  __syncthreads();
  if (warp < N) {  // warp d scans destination d across the kWarps warps
    const int32_t w = lane < kWarps ? warp_tot[lane][warp] : 0;
    int32_t wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += u;
    }
    if (lane < kWarps) warp_tot[lane][warp] = wi - w;
    if (lane == 31) batch_tot[warp] = wi;
  }
  __syncthreads();
  if (valid) {
#pragma unroll
    for (int d = 0; d < kMaxEp; ++d) {
      if (d >= N) break;
      const int32_t before = warp_tot[warp][d] + incl[d] - v[d];
      const int32_t c = v[d] & 0xffff;
      send_token_slot[t * N + d] = c > 0 ? run_tok[d] + (before >> 16) : -1;
      int32_t slot = run_rt[d] + (before & 0xffff);
      if (c > 0)
        for (int s2 = 0; s2 < top_k; ++s2)
          if (my_dest[s2] == d) route_dest_slot[t * top_k + s2] = slot++;
    }
    // Routes to no rank (dropped or invalid ids).
    for (int s2 = 0; s2 < top_k; ++s2)
      if (my_dest[s2] < 0) route_dest_slot[t * top_k + s2] = -1;
  }
  if (blockIdx.x == gridDim.x - 1 && tid < N) {
    counts[tid] = run_tok[tid] + (batch_tot[tid] >> 16);
    counts[N + tid] = run_rt[tid] + (batch_tot[tid] & 0xffff);
  }
}

// One warp per token: copy its row to every destination slot, then write the
// records of its routes.
__global__ void __launch_bounds__(256) ep_pack_kernel(
    const __nv_bfloat16 *__restrict__ x, int hidden, const int64_t *__restrict__ ids,
    const __nv_bfloat16 *__restrict__ rw, int64_t num_tokens, int top_k, int num_experts,
    const int32_t *__restrict__ owner, int ep_size, const int32_t *__restrict__ send_token_slot,
    const int32_t *__restrict__ route_dest_slot, Offsets tok_off, Offsets route_off,
    __nv_bfloat16 *__restrict__ send_x, int4 *__restrict__ send_meta) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (t >= num_tokens) return;
  const int vecs = hidden / 8;
  const uint4 *src = reinterpret_cast<const uint4 *>(x + t * hidden);
  for (int d = 0; d < ep_size; ++d) {
    const int32_t slot = send_token_slot[t * ep_size + d];
    if (slot < 0) continue;
    uint4 *dst = reinterpret_cast<uint4 *>(send_x + static_cast<int64_t>(tok_off.v[d] + slot) * hidden);
    for (int v = lane; v < vecs; v += 32) dst[v] = src[v];
  }
  if (lane < top_k) {
    const int64_t r = t * top_k + lane;
    const int64_t id = ids[r];
    const int d = dest_of(id, num_experts, owner, ep_size);
    const int32_t slot = route_dest_slot[r];
    if (d >= 0 && slot >= 0) {
      const uint16_t wbits = __bfloat16_as_ushort(rw[r]);
      send_meta[route_off.v[d] + slot] =
          make_int4(static_cast<int>(id), send_token_slot[t * ep_size + d], static_cast<int>(wbits),
                    static_cast<int>(r));
    }
  }
}

__global__ void ep_unpack_kernel(const int4 *__restrict__ meta, int64_t n, int ep_size,
                                 Offsets recv_route_off, Offsets recv_tok_off,
                                 Offsets meta_start, int64_t *__restrict__ ids,
                                 int32_t *__restrict__ token_of_route,
                                 __nv_bfloat16 *__restrict__ rw) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int src = 0;
  while (src + 1 < ep_size && i >= recv_route_off.v[src + 1]) ++src;
  const int4 m = meta[meta_start.v[src] + (i - recv_route_off.v[src])];
  ids[i] = m.x;
  token_of_route[i] = recv_tok_off.v[src] + m.y;
  rw[i] = __ushort_as_bfloat16(static_cast<unsigned short>(m.z & 0xffff));
}

__global__ void ep_return_rows_kernel(const int64_t *__restrict__ ids,
                                      const int32_t *__restrict__ owner, int64_t num_routes,
                                      int num_experts, int ep_size,
                                      const int32_t *__restrict__ route_dest_slot, Offsets route_off,
                                      int64_t num_rows_returned, int32_t *__restrict__ combine_rows) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= num_routes) return;
  const int d = dest_of(ids[r], num_experts, owner, ep_size);
  const int32_t slot = route_dest_slot[r];
  combine_rows[r] = (d >= 0 && slot >= 0) ? route_off.v[d] + slot
                                          : static_cast<int32_t>(num_rows_returned);
}

int load_offsets(Offsets &o, const int32_t *host, int n) {
  for (int i = 0; i <= kMaxEp; ++i) o.v[i] = 0;
  for (int i = 0; i < n; ++i) o.v[i] = host[i];
  return B200MOE_OK;
}

}  // namespace
}  // namespace b200moe

extern "C" {

int b200moe_ep_plan(const int64_t *expert_ids, int64_t num_tokens, int top_k, int num_experts,
                    const int32_t *owner, int ep_size, int32_t *send_token_slot,
                    int32_t *route_dest_slot, int32_t *counts, void *stream) {
  using namespace b200moe;
  B200_ARG(ep_size >= 1 && ep_size <= kMaxEp, "ep_size must be in [1, %d]", kMaxEp);
  B200_ARG(num_tokens >= 0 && top_k >= 1 && top_k <= 32 && num_experts >= 1, "bad shape");
  B200_ARG(owner && counts, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (num_tokens == 0) {
    B200_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * 2 * ep_size, s));
    return B200MOE_OK;
  }
  B200_ARG(expert_ids && send_token_slot && route_dest_slot, "null pointer argument");
  const int64_t blocks = (num_tokens + kPlanThreads - 1) / kPlanThreads;
  B200_ARG(blocks < (int64_t)0x7fffffff, "num_tokens out of range");
  ep_plan_kernel<<<static_cast<unsigned>(blocks), kPlanThreads, 0, s>>>(
      expert_ids, num_tokens, top_k, num_experts, owner, ep_size, send_token_slot,
      route_dest_slot, counts);
  B200_LAUNCHED();
  return B200MOE_OK;
}

int b200moe_ep_pack(const void *x, int hidden, const int64_t *expert_ids,
                    const void *route_weights, int64_t num_tokens, int top_k, int num_experts,
                    const int32_t *owner, int ep_size, const int32_t *send_token_slot,
                    const int32_t *route_dest_slot, const int32_t *token_offsets_host,
                    const int32_t *route_offsets_host, void *send_x, int32_t *send_meta,
                    void *stream) {
  using namespace b200moe;
  B200_ARG(ep_size >= 1 && ep_size <= kMaxEp, "ep_size must be in [1, %d]", kMaxEp);
  B200_UNSUPPORTED(hidden % 8 == 0, "hidden must be a multiple of 8");
  B200_ARG(top_k >= 1 && top_k <= 32, "top_k must be in [1, 32]");
  if (num_tokens == 0) return B200MOE_OK;
  B200_ARG(x && expert_ids && route_weights && owner && send_token_slot && route_dest_slot &&
               token_offsets_host && route_offsets_host,
           "null pointer argument");
  Offsets to, ro;
  load_offsets(to, token_offsets_host, ep_size);
  load_offsets(ro, route_offsets_host, ep_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t blocks = (num_tokens * 32 + 255) / 256;
  ep_pack_kernel<<<blocks, 256, 0, s>>>(
      static_cast<const __nv_bfloat16 *>(x), hidden, expert_ids,
      static_cast<const __nv_bfloat16 *>(route_weights), num_tokens, top_k, num_experts, owner,
      ep_size, send_token_slot, route_dest_slot, to, ro, static_cast<__nv_bfloat16 *>(send_x),
      reinterpret_cast<int4 *>(send_meta));
  B200_LAUNCHED();
  return B200MOE_OK;
}

int b200moe_ep_unpack_routes(const int32_t *recv_meta, int64_t num_recv_routes, int ep_size,
                             const int32_t *recv_route_offsets_host,
                             const int32_t *recv_token_offsets_host,
                             const int32_t *recv_meta_starts_host, int64_t *expert_ids,
                             int32_t *token_of_route, void *route_weights, void *stream) {
  using namespace b200moe;
  B200_ARG(ep_size >= 1 && ep_size <= kMaxEp, "ep_size must be in [1, %d]", kMaxEp);
  if (num_recv_routes == 0) return B200MOE_OK;
  B200_ARG(recv_meta && recv_route_offsets_host && recv_token_offsets_host && expert_ids &&
               token_of_route && route_weights,
           "null pointer argument");
  Offsets ro, to, ms;
  load_offsets(ro, recv_route_offsets_host, ep_size + 1);
  load_offsets(to, recv_token_offsets_host, ep_size);
  // Records of each source are contiguous at recv_meta + start[s] (default:
  // all sources back to back).
  load_offsets(ms, recv_meta_starts_host ? recv_meta_starts_host : recv_route_offsets_host,
               ep_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t blocks = (num_recv_routes + 255) / 256;
  ep_unpack_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const int4 *>(recv_meta),
                                          num_recv_routes, ep_size, ro, to, ms, expert_ids,
                                          token_of_route,
                                          static_cast<__nv_bfloat16 *>(route_weights));
  B200_LAUNCHED();
  return B200MOE_OK;
}

int b200moe_ep_return_rows(const int64_t *expert_ids, const int32_t *owner, int64_t num_routes,
                           int num_experts, int ep_size, const int32_t *route_dest_slot,
                           const int32_t *route_offsets_host, int64_t num_rows_returned,
                           int32_t *combine_rows, void *stream) {
  using namespace b200moe;
  B200_ARG(ep_size >= 1 && ep_size <= kMaxEp, "ep_size must be in [1, %d]", kMaxEp);
  if (num_routes == 0) return B200MOE_OK;
  B200_ARG(expert_ids && owner && route_dest_slot && route_offsets_host && combine_rows,
           "null pointer argument");
  Offsets ro;
  load_offsets(ro, route_offsets_host, ep_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t blocks = (num_routes + 255) / 256;
  ep_return_rows_kernel<<<blocks, 256, 0, s>>>(expert_ids, owner, num_routes, num_experts,
                                               ep_size, route_dest_slot, ro, num_rows_returned,
                                               combine_rows);
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // extern "C"
