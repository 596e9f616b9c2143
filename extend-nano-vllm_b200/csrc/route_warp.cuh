// One warp routes one token: fp32 softmax over the logits, top-k of the
// probabilities, optional renormalisation over the selected k.  Shared by the
// router kernel and the fused tiny-batch decode kernels so both select and
// weight experts identically.
// Reference: ExpertParallelMoE._route, nanovllm/layers/moe.py:872-878:
//   probs = F.softmax(logits, dim=-1, dtype=float32)
//   w, ids = torch.topk(probs, k)
//   if norm_topk_prob: w /= w.sum(-1, keepdim=True)
//   w = w.to(bf16)
//
// Every step reproduces the arithmetic and the selection order of those torch
// calls on a CUDA device, so ids (ties included) and weights are the same bits:
//  * softmax: lane l holds experts l + 32 i; max, then p = expf(v - max),
//    a per-lane sum over i in ascending order, a butterfly sum over the warp
//    (xor 16, 8, 4, 2, 1), and p / sum -- the persistent warp softmax torch
//    uses for rows of <= 1024 elements;
//  * top-k: torch selects the k-th largest probability, then writes the
//    elements strictly above it in ascending index order followed by the
//    first elements equal to it (ascending index), and sorts those k
//    (key, index) pairs with a 32-wide bitonic network (k <= 32) whose
//    compare-exchange is not stable.  The same network runs here, one element
//    per lane, so equal probabilities come out in torch's order;
//  * renormalisation: torch's sum over the k slots reduces slot t and slot
//    t + W (W = largest power of two <= k) per thread, then a shuffle-down
//    tree with offsets W/2 ... 1.
#pragma once

#include <float.h>

#include "common.cuh"

namespace b200moe {

// One compare-exchange of the bitonic network between this lane and
// lane ^ stride.  The lower lane holds element A, the upper lane element B.
// A and B are exchanged when ((A > B and A valid) or B invalid) == dir; equal
// valid keys therefore exchange when dir is false.
__device__ __forceinline__ void bitonic_step(float &key, int &id, int lane, int stride,
                                             bool dir) {
  const float other_key = __shfl_xor_sync(0xffffffffu, key, stride);
  const int other_id = __shfl_xor_sync(0xffffffffu, id, stride);
  const bool lower = (lane & stride) == 0;
  const float ka = lower ? key : other_key;
  const float kb = lower ? other_key : key;
  const bool va = (lower ? id : other_id) >= 0;
  const bool vb = (lower ? other_id : id) >= 0;
  const bool swap = (ka > kb && va) || !vb;
  if (swap == dir) {
    key = other_key;
    id = other_id;
  }
}

// On return, lane s < top_k holds slot s: its probability weight (renormalised
// if requested, fp32, not yet rounded) in *w and its expert id in *id.
// VPL = ceil(num_experts / 32) logits per lane (expert lane + 32 * i).
template <typename T, int VPL>
__device__ __forceinline__ void warp_route_token(const T *row, int num_experts,
                                                 int top_k, int renormalize, int lane,
                                                 float *w, int *id) {
  float v[VPL];
  bool live[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    live[i] = e < num_experts;
    v[i] = live[i] ? to_f32(row[e]) : -FLT_MAX;
  }
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    if (live[i]) m = fmaxf(m, v[i]);
  m = warp_max(m);
  float p[VPL];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    p[i] = live[i] ? expf(v[i] - m) : 0.f;
    s += p[i];
  }
  s = warp_sum(s);
#pragma unroll
  for (int i = 0; i < VPL; ++i) p[i] = p[i] / s;

  // Selection keys: probabilities are >= 0, so their bit patterns (+1) order
  // like the values; 0 marks a taken or absent expert.  Each round takes the
  // largest key, lowest expert id among equal keys.
  uint32_t key[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) key[i] = live[i] ? __float_as_uint(p[i]) + 1u : 0u;
  float sel_p = 0.f;
  int sel_id = -1;
  for (int slot = 0; slot < top_k; ++slot) {
    uint32_t bk = 0u;
    int bi = 0;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (key[i] > bk) {
        bk = key[i];
        bi = i;
      }
    }
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, bk);
    const uint32_t mine = (bk == kmax && kmax != 0u) ? static_cast<uint32_t>(lane + 32 * bi)
                                                     : 0xffffffffu;
    const uint32_t win = __reduce_min_sync(0xffffffffu, mine);
    const int owner = static_cast<int>(win & 31u);
    // Selects instead of p[win >> 5]: an index computed at run time would
    // move p and key to local memory.
    const int wi = static_cast<int>(win >> 5);
    float bp = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const bool hit = lane == owner && i == wi;
      bp = hit ? p[i] : bp;
      key[i] = hit ? 0u : key[i];
    }
    bp = __shfl_sync(0xffffffffu, bp, owner);
    if (lane == slot) {
      sel_p = bp;
      sel_id = static_cast<int>(win);
    }
  }

  // Lanes 0..k-1 now hold the top k by (probability desc, id asc).  Without
  // equal probabilities among them the bitonic network below returns exactly
  // this descending list, so only tokens with such ties run it.
  const float prev_p = __shfl_up_sync(0xffffffffu, sel_p, 1);
  const bool tie = lane > 0 && lane < top_k && sel_p == prev_p;
  float sk = sel_p;
  int sid = lane < top_k ? sel_id : -1;
  if (__any_sync(0xffffffffu, tie)) {
    // torch's pre-sort order: ids strictly above the k-th probability by
    // ascending id, then the ids equal to it (already ascending, at the tail
    // of this list).
    const float kth = __shfl_sync(0xffffffffu, sel_p, top_k - 1);
    const bool above = lane < top_k && sel_p > kth;
    const unsigned above_mask = __ballot_sync(0xffffffffu, above);
    int rank_above = 0;
    for (int s2 = 0; s2 < top_k; ++s2) {
      const int other = __shfl_sync(0xffffffffu, sel_id, s2);
      rank_above += ((above_mask >> s2) & 1u) && other < sel_id;
    }
    const int pos = above ? rank_above : lane;
    int src = lane;
    for (int t = 0; t < top_k; ++t) {
      const unsigned hit = __ballot_sync(0xffffffffu, lane < top_k && pos == t);
      if (lane == t) src = __ffs(hit) - 1;
    }
    sk = __shfl_sync(0xffffffffu, sel_p, src);
    sid = __shfl_sync(0xffffffffu, sel_id, src);
    if (lane >= top_k) {
      // Padding entries of the 32-wide network: key 0, invalid.
      sk = 0.f;
      sid = -1;
    }
    // Bitonic network over 32 positions: merge phases of size 2..16 with the
    // direction taken from bit `size` of the position, then the final merge
    // with direction false (descending keys, invalid entries last).
#pragma unroll
    for (int size = 2; size < 32; size <<= 1) {
      const bool dir = (lane & size) != 0;
#pragma unroll
      for (int stride = size >> 1; stride > 0; stride >>= 1) bitonic_step(sk, sid, lane, stride, dir);
    }
#pragma unroll
    for (int stride = 16; stride > 0; stride >>= 1) bitonic_step(sk, sid, lane, stride, false);
  }

  float my_w = sk;
  if (renormalize) {
    // torch's sum over k values: thread t < W adds slots t and t + W, then a
    // shuffle-down tree over W threads.  Lane 0's chain reads lanes < W only.
    int width = 1;
    while (width * 2 <= top_k) width *= 2;
    const float upper = __shfl_down_sync(0xffffffffu, sk, width);
    float acc = (lane + width < top_k) ? sk + upper : sk;
    for (int off = width >> 1; off > 0; off >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, off);
    const float total = __shfl_sync(0xffffffffu, acc, 0);
    my_w = sk / total;
  }
  *w = my_w;
  *id = sid;
}

}  // namespace b200moe
