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

}  // namespace
}  // namespace b200moe

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
