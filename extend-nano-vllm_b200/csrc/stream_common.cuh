// Helpers of the weight-streaming kernels: 16-byte non-allocating loads of
// weight rows (lane l reads vectors l, l+32, ...), dot products against
// activation rows held in shared memory, 8-wide bf16 stores.
#pragma once

#include "common.cuh"

namespace b200moe {

__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void store8_bf16(__nv_bfloat16 *dst, const float *v) {
  uint4 o;
  __nv_bfloat162 *op = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) op[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4 *>(dst) = o;
}

template <int VPL>
__device__ __forceinline__ void load_row(const uint4 *row, int V, int lane, uint4 (&w)[VPL]) {
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int v = lane + 32 * i;
    w[i] = v < V ? ld_stream(row + v) : make_uint4(0, 0, 0, 0);
  }
}

// Dot products of one weight row with NR activation rows held in shared memory.
template <int VPL, int NR>
__device__ __forceinline__ void dot_rows(const uint4 (&w)[VPL], const uint4 *xs, int V, int lane,
                                         float (&acc)[NR]) {
#pragma unroll
  for (int n = 0; n < NR; ++n) acc[n] = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int v = lane + 32 * i;
    if (v < V) {
#pragma unroll
      for (int n = 0; n < NR; ++n) dot8_bf16(w[i], xs[n * V + v], acc[n]);
    }
  }
}

}  // namespace b200moe
