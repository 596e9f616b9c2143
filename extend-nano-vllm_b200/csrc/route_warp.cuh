// One warp routes one token: fp32 softmax over the logits, top-k by
// descending logit (ties to the lower expert index), optional renormalisation
// over the selected k.  Shared by the router kernel and the fused tiny-batch
// decode kernels so both select and weight experts identically.
// Reference: ExpertParallelMoE._route, nanovllm/layers/moe.py:872-878.
#pragma once

#include <float.h>

#include "common.cuh"

namespace b200moe {

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

  // Selection keys: logits mapped to order-preserving unsigned integers
  // (0 = already taken or not an expert), so each round is one warp max over
  // the keys and one warp min over the expert ids that hold it.
  uint32_t key[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    uint32_t b = __float_as_uint(v[i]);
    if (b == 0x80000000u) b = 0u;  // -0 ties with +0, as in a float compare
    key[i] = live[i] ? ((b & 0x80000000u) ? ~b : (b | 0x80000000u)) : 0u;
  }
  float my_w = 0.f;
  int my_id = 0;
  for (int slot = 0; slot < top_k; ++slot) {
    // This lane's best remaining (largest key, lowest expert id on ties).
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
      my_w = bp;
      my_id = static_cast<int>(win);
    }
  }
  if (renormalize) {
    // Sequential sum over the slots, identical on every lane.
    float total = 0.f;
    for (int slot = 0; slot < top_k; ++slot) total += __shfl_sync(0xffffffffu, my_w, slot);
    my_w = my_w / total;
  }
  *w = my_w;
  *id = my_id;
}

}  // namespace b200moe
