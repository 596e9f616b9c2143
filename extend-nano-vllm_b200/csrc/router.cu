// Router: fp32 softmax + top-k + optional renormalisation, one warp per token.
//
// Reference: ExpertParallelMoE._route, nanovllm/layers/moe.py:870-878
//   probs = F.softmax(logits, dim=-1, dtype=float32)
//   w, ids = torch.topk(probs, k);  if norm_topk_prob: w /= w.sum(-1)
//   w = w.to(bf16)
// The warp routine (route_warp.cuh) reproduces torch's CUDA softmax, top-k
// order for equal probabilities and renormalisation sum, so ids and weights
// equal the reference's GPU routing bit for bit.
#include "route_warp.cuh"

namespace b200moe {
namespace {

// With `shared_logits` (bf16 [num_tokens], the shared-expert gate of
// moe.py:1259-1261) each output row holds top_k + 1 slots: the routed
// experts, then the shared expert (id num_experts) weighted by
// sigmoid(shared logit) in fp32, rounded to bf16 like torch.sigmoid on a bf16
// tensor.
template <typename T, int VPT>
__global__ void __launch_bounds__(256) route_topk_kernel(const T *logits,
                                                         int64_t num_tokens, int num_experts,
                                                         int top_k, int renormalize,
                                                         const __nv_bfloat16 *shared_logits,
                                                         __nv_bfloat16 *__restrict__ weights,
                                                         int64_t *__restrict__ ids) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t token = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (token >= num_tokens) return;
  float my_w;
  int my_id;
  warp_route_token<T, VPT>(logits + token * num_experts, num_experts, top_k, renormalize, lane,
                           &my_w, &my_id);
  const int slots = shared_logits ? top_k + 1 : top_k;
  if (lane < top_k) {
    weights[token * slots + lane] = __float2bfloat16_rn(my_w);
    ids[token * slots + lane] = my_id;
  } else if (shared_logits && lane == top_k) {
    const float g = __bfloat162float(shared_logits[token]);
    weights[token * slots + lane] = __float2bfloat16_rn(1.f / (1.f + expf(-g)));
    ids[token * slots + lane] = num_experts;
  }
}

template <typename T>
int launch_route(const void *logits, int64_t num_tokens, int num_experts, int top_k,
                 int renormalize, const void *shared_logits, void *weights, int64_t *ids,
                 cudaStream_t stream) {
  const int threads = 256;
  const int64_t blocks = (num_tokens * 32 + threads - 1) / threads;
  const T *lg = static_cast<const T *>(logits);
  auto *w = static_cast<__nv_bfloat16 *>(weights);
  const auto *sl = static_cast<const __nv_bfloat16 *>(shared_logits);
  const int vpt = (num_experts + 31) / 32;
#define B200_ROUTE_CASE(V)                                                                  \
  if (vpt <= V) {                                                                           \
    B200_LAUNCH_PDL(kPdlRoute, route_topk_kernel<T, V>, dim3(blocks), dim3(threads), 0, stream, lg, num_tokens, num_experts,    \
                                                           top_k, renormalize, sl, w, ids); \
    B200_LAUNCHED();                                                                        \
    return B200MOE_OK;                                                                      \
  }
  B200_ROUTE_CASE(1)
  B200_ROUTE_CASE(2)
  B200_ROUTE_CASE(4)
  B200_ROUTE_CASE(8)
  B200_ROUTE_CASE(16)
  B200_ROUTE_CASE(32)
#undef B200_ROUTE_CASE
  set_error("num_experts %d exceeds 1024", num_experts);
  return B200MOE_EUNSUPPORTED;
}

// ---------------------------------------------------------------------------
// Router projection fused with routing (small batches): logits = x Wg^T in
// fp32, rounded to bf16 (the dtype of the reference's bf16 F.linear, moe.py:871
// via linear.py:51), then the same warp routine as route_topk_kernel.
// grid = (ceil(T / 8), ceil(E / 8)); block = 256.  CTA (g, c) stages token
// group g's x rows in shared memory, warp w computes expert c * 8 + w's logits
// for those tokens (lane l reads the 16-byte vectors l, l + 32, ... of the
// gate row and multiplies them in order; a butterfly sum over the warp), and
// the last CTA of a token group to finish (device-scope counter, reset by it
// for the next call) routes the group's tokens from the logits in L2.
// ---------------------------------------------------------------------------
constexpr int kGateTokens = 8;
constexpr int kGateMaxVpl = 16;  // hidden <= 4096

template <int VPT>
__global__ void __launch_bounds__(256) route_gate_kernel(
    const __nv_bfloat16 *x, int hidden, const __nv_bfloat16 *gate_w, int64_t num_tokens,
    int num_experts, int top_k, int renormalize, __nv_bfloat16 *logits,
    __nv_bfloat16 *__restrict__ weights, int64_t *__restrict__ ids, int32_t *sync) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ uint4 gate_smem[];  // [kGateTokens][V] x rows, then [8][E] bf16 logits
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int V = hidden / 8;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kGateTokens;
  const int nt = static_cast<int>(min64(kGateTokens, num_tokens - t0));
  const uint4 *xg = reinterpret_cast<const uint4 *>(x + t0 * hidden);
  for (int v = threadIdx.x; v < nt * V; v += blockDim.x) gate_smem[v] = xg[v];
  __syncthreads();
  const int e = blockIdx.y * 8 + warp;
  if (e < num_experts) {
    const uint4 *wrow = reinterpret_cast<const uint4 *>(gate_w + static_cast<int64_t>(e) * hidden);
    uint4 w[kGateMaxVpl];
#pragma unroll
    for (int i = 0; i < kGateMaxVpl; ++i) {
      const int v = lane + 32 * i;
      w[i] = v < V ? wrow[v] : make_uint4(0, 0, 0, 0);
    }
    for (int t = 0; t < nt; ++t) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < kGateMaxVpl; ++i) {
        const int v = lane + 32 * i;
        if (v < V) dot8_bf16(w[i], gate_smem[t * V + v], acc);
      }
      acc = warp_sum(acc);
      if (lane == 0) logits[(t0 + t) * num_experts + e] = __float2bfloat16_rn(acc);
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int done = atomicAdd(&sync[blockIdx.x], 1);
    s_last = done == static_cast<int>(gridDim.y) - 1;
    if (s_last) sync[blockIdx.x] = 0;  // ready for the next call
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Route the group's tokens: one warp per token, logits read from L2.
  auto *rows = reinterpret_cast<__nv_bfloat16 *>(gate_smem + kGateTokens * V);
  if (warp < nt) {
    __nv_bfloat16 *row = rows + warp * num_experts;
    const __nv_bfloat16 *src = logits + (t0 + warp) * num_experts;
    for (int i = lane; i < num_experts; i += 32) {
      const unsigned short bits = __ldcg(reinterpret_cast<const unsigned short *>(src + i));
      row[i] = __ushort_as_bfloat16(bits);
    }
    __syncwarp();
    float wgt;
    int id;
    warp_route_token<__nv_bfloat16, VPT>(row, num_experts, top_k, renormalize, lane, &wgt, &id);
    if (lane < top_k) {
      weights[(t0 + warp) * top_k + lane] = __float2bfloat16_rn(wgt);
      ids[(t0 + warp) * top_k + lane] = id;
    }
  }
}

template <int VPT>
int launch_route_gate(const void *x, int hidden, const void *gate_w, int64_t num_tokens,
                      int num_experts, int top_k, int renormalize, void *logits, void *weights,
                      int64_t *ids, int32_t *sync, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>((num_tokens + kGateTokens - 1) / kGateTokens),
                  static_cast<unsigned>((num_experts + 7) / 8));
  const size_t smem = static_cast<size_t>(kGateTokens) * hidden * 2 +
                      static_cast<size_t>(kGateTokens) * num_experts * 2;
  if (smem > 48 * 1024)
    B200_CUDA(cudaFuncSetAttribute(route_gate_kernel<VPT>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  B200_LAUNCH_PDL(kPdlRoute, route_gate_kernel<VPT>, grid, dim3(256), smem, s,
                  static_cast<const __nv_bfloat16 *>(x), hidden,
                  static_cast<const __nv_bfloat16 *>(gate_w), num_tokens, num_experts, top_k,
                  renormalize, static_cast<__nv_bfloat16 *>(logits),
                  static_cast<__nv_bfloat16 *>(weights), ids, sync);
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // namespace
}  // namespace b200moe

extern "C" int b200moe_route_gate_topk(const void *x, int hidden, const void *gate_w,
                                       int64_t num_tokens, int num_experts, int top_k,
                                       int renormalize, void *logits, void *weights,
                                       int64_t *expert_ids, int32_t *sync, void *stream) {
  B200_ARG(num_tokens >= 0, "num_tokens must be >= 0");
  B200_ARG(num_experts >= 1, "num_experts must be >= 1");
  B200_ARG(top_k >= 1 && top_k <= num_experts, "top_k must be between 1 and num_experts");
  B200_UNSUPPORTED(top_k <= 32, "top_k %d > 32 is not supported", top_k);
  B200_UNSUPPORTED(num_experts <= 1024, "num_experts %d > 1024 is not supported", num_experts);
  B200_UNSUPPORTED(hidden % 8 == 0 && hidden <= 4096,
                   "hidden must be a multiple of 8 and at most 4096");
  B200_UNSUPPORTED(num_tokens <= B200MOE_ROUTE_GATE_MAX_TOKENS,
                   "the fused router projection takes at most %d tokens",
                   B200MOE_ROUTE_GATE_MAX_TOKENS);
  if (num_tokens == 0) return B200MOE_OK;
  B200_ARG(x && gate_w && logits && weights && expert_ids && sync, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int vpt = (num_experts + 31) / 32;
#define B200_GATE_CASE(V)                                                                   \
  if (vpt <= V)                                                                             \
    return b200moe::launch_route_gate<V>(x, hidden, gate_w, num_tokens, num_experts, top_k, \
                                         renormalize, logits, weights, expert_ids, sync, s);
  B200_GATE_CASE(1)
  B200_GATE_CASE(4)
  B200_GATE_CASE(8)
  B200_GATE_CASE(32)
#undef B200_GATE_CASE
  return B200MOE_EUNSUPPORTED;
}

static int route_entry(const void *logits, int logits_dtype, int64_t num_tokens,
                       int num_experts, int top_k, int renormalize, const void *shared_logits,
                       void *weights, int64_t *expert_ids, void *stream) {
  B200_ARG(num_tokens >= 0, "num_tokens must be >= 0");
  B200_ARG(num_experts >= 1, "num_experts must be >= 1");
  B200_ARG(top_k >= 1 && top_k <= num_experts, "top_k must be between 1 and num_experts");
  B200_UNSUPPORTED(top_k <= (shared_logits ? 31 : 32), "top_k %d > %d is not supported", top_k,
                   shared_logits ? 31 : 32);
  B200_UNSUPPORTED(num_experts <= 1024, "num_experts %d > 1024 is not supported", num_experts);
  if (num_tokens == 0) return B200MOE_OK;
  B200_ARG(logits && weights && expert_ids, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (logits_dtype) {
    case B200MOE_F32:
      return b200moe::launch_route<float>(logits, num_tokens, num_experts, top_k, renormalize,
                                          shared_logits, weights, expert_ids, s);
    case B200MOE_BF16:
      return b200moe::launch_route<__nv_bfloat16>(logits, num_tokens, num_experts, top_k,
                                                  renormalize, shared_logits, weights,
                                                  expert_ids, s);
    case B200MOE_F16:
      return b200moe::launch_route<__half>(logits, num_tokens, num_experts, top_k, renormalize,
                                           shared_logits, weights, expert_ids, s);
    default:
      b200moe::set_error("unsupported logits dtype code %d", logits_dtype);
      return B200MOE_EINVAL;
  }
}

extern "C" int b200moe_route_topk(const void *logits, int logits_dtype, int64_t num_tokens,
                                  int num_experts, int top_k, int renormalize, void *weights,
                                  int64_t *expert_ids, void *stream) {
  return route_entry(logits, logits_dtype, num_tokens, num_experts, top_k, renormalize, nullptr,
                     weights, expert_ids, stream);
}

extern "C" int b200moe_route_topk_shared(const void *logits, int logits_dtype,
                                         int64_t num_tokens, int num_experts, int top_k,
                                         int renormalize, const void *shared_logits,
                                         void *weights, int64_t *expert_ids, void *stream) {
  B200_ARG(num_tokens == 0 || shared_logits, "shared_logits is null");
  return route_entry(logits, logits_dtype, num_tokens, num_experts, top_k, renormalize,
                     shared_logits, weights, expert_ids, stream);
}
