// Router: fp32 softmax + top-k + optional renormalisation, one warp per token.
//
// Reference: ExpertParallelMoE._route, nanovllm/layers/moe.py:870-878
//   probs = F.softmax(logits, dim=-1, dtype=float32)
//   w, ids = torch.topk(probs, k);  if norm_topk_prob: w /= w.sum(-1)
//   w = w.to(bf16)
// Selection ranks experts by descending logit with ties going to the lower
// index; softmax is monotone so this is the same set and order as top-k over
// the probabilities wherever the probabilities are distinct.
#include <float.h>

#include "common.cuh"

namespace b200moe {
namespace {

template <typename T, int VPT>
__global__ void __launch_bounds__(256) route_topk_kernel(const T *__restrict__ logits,
                                                         int64_t num_tokens, int num_experts,
                                                         int top_k, int renormalize,
                                                         __nv_bfloat16 *__restrict__ weights,
                                                         int64_t *__restrict__ ids) {
  const int lane = threadIdx.x & 31;
  const int64_t token = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (token >= num_tokens) return;
  const T *row = logits + token * num_experts;

  // Element i of this lane is expert lane + 32 * i (coalesced loads).
  float v[VPT];
  bool live[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int e = lane + 32 * i;
    live[i] = e < num_experts;
    v[i] = live[i] ? to_f32(row[e]) : -FLT_MAX;
  }
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPT; ++i)
    if (live[i]) m = fmaxf(m, v[i]);
  m = warp_max(m);
  float p[VPT];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    p[i] = live[i] ? expf(v[i] - m) : 0.f;
    s += p[i];
  }
  s = warp_sum(s);
#pragma unroll
  for (int i = 0; i < VPT; ++i) p[i] = p[i] / s;

  // k rounds of warp arg-max over (logit desc, index asc).
  float my_w = 0.f;
  int my_id = 0;
  for (int slot = 0; slot < top_k; ++slot) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    float bp = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = lane + 32 * i;
      if (live[i] && (v[i] > bv || (v[i] == bv && e < bi))) {
        bv = v[i];
        bi = e;
        bp = p[i];
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const float op = __shfl_xor_sync(0xffffffffu, bp, off);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
        bp = op;
      }
    }
    // The owning lane retires the winner.
#pragma unroll
    for (int i = 0; i < VPT; ++i)
      if (lane + 32 * i == bi) live[i] = false;
    if (lane == slot) {
      my_w = bp;
      my_id = bi;
    }
  }
  if (renormalize) {
    // Sequential sum over the slots, identical on every lane.
    float total = 0.f;
    for (int slot = 0; slot < top_k; ++slot) total += __shfl_sync(0xffffffffu, my_w, slot);
    my_w = my_w / total;
  }
  if (lane < top_k) {
    weights[token * top_k + lane] = __float2bfloat16_rn(my_w);
    ids[token * top_k + lane] = my_id;
  }
}

template <typename T>
int launch_route(const void *logits, int64_t num_tokens, int num_experts, int top_k,
                 int renormalize, void *weights, int64_t *ids, cudaStream_t stream) {
  const int threads = 256;
  const int64_t blocks = (num_tokens * 32 + threads - 1) / threads;
  const T *lg = static_cast<const T *>(logits);
  auto *w = static_cast<__nv_bfloat16 *>(weights);
  const int vpt = (num_experts + 31) / 32;
#define B200_ROUTE_CASE(V)                                                                  \
  if (vpt <= V) {                                                                           \
    route_topk_kernel<T, V><<<blocks, threads, 0, stream>>>(lg, num_tokens, num_experts,    \
                                                           top_k, renormalize, w, ids);    \
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

extern "C" int b200moe_route_topk(const void *logits, int logits_dtype, int64_t num_tokens,
                                  int num_experts, int top_k, int renormalize, void *weights,
                                  int64_t *expert_ids, void *stream) {
  B200_ARG(num_tokens >= 0, "num_tokens must be >= 0");
  B200_ARG(num_experts >= 1, "num_experts must be >= 1");
  B200_ARG(top_k >= 1 && top_k <= num_experts, "top_k must be between 1 and num_experts");
  B200_UNSUPPORTED(top_k <= 32, "top_k %d > 32 is not supported", top_k);
  B200_UNSUPPORTED(num_experts <= 1024, "num_experts %d > 1024 is not supported", num_experts);
  if (num_tokens == 0) return B200MOE_OK;
  B200_ARG(logits && weights && expert_ids, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (logits_dtype) {
    case B200MOE_F32:
      return b200moe::launch_route<float>(logits, num_tokens, num_experts, top_k, renormalize,
                                          weights, expert_ids, s);
    case B200MOE_BF16:
      return b200moe::launch_route<__nv_bfloat16>(logits, num_tokens, num_experts, top_k,
                                                  renormalize, weights, expert_ids, s);
    case B200MOE_F16:
      return b200moe::launch_route<__half>(logits, num_tokens, num_experts, top_k, renormalize,
                                           weights, expert_ids, s);
    default:
      b200moe::set_error("unsupported logits dtype code %d", logits_dtype);
      return B200MOE_EINVAL;
  }
}
