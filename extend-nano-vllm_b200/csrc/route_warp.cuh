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

  float my_w = 0.f;
  int my_id = 0;
  for (int slot = 0; slot < top_k; ++slot) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    float bp = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
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
#pragma unroll
    for (int i = 0; i < VPL; ++i)
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
  *w = my_w;
  *id = my_id;
}

}  // namespace b200moe
