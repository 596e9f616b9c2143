// Weight-streaming expert kernels for small decode buckets (engine STREAM).
//
// In a decode bucket each active expert owns only a handful of routes, so the
// grouped GEMMs of the reference (Triton _grouped_moe_gemm_kernel,
// nanovllm/layers/moe.py:63-139, launched per 16-row tile) are bound by
// reading every active expert's weights once from HBM.  These kernels stream
// each weight row exactly once per chunk of up to kRows routes with 16-byte
// non-allocating loads, keep the routes' activations in shared memory, and
// reduce the dot products with warp shuffles.  Every warp owns 8 consecutive
// output features so the results leave as one 16-byte store per route.
#include "common.cuh"

namespace b200moe {
namespace {

constexpr int kStreamThreads = 128;            // 4 warps
constexpr int kStreamWarps = kStreamThreads / 32;
constexpr int kFeatPerWarp = 8;                // outputs per warp (one 16B store)
constexpr int kRows = 8;                       // routes per shared-memory chunk

__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void store8_bf16(__nv_bfloat16 *dst, const float (&v)[8]) {
  uint4 o;
  __nv_bfloat162 *op = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) op[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4 *>(dst) = o;
}

// grid = (max m-tiles, ceil(I / 32)); VPL = ceil(H / 256) vectors per lane.
template <int VPL>
__global__ void __launch_bounds__(kStreamThreads) gate_up_stream_kernel(
    const __nv_bfloat16 *__restrict__ x, int64_t x_rows, int hidden, int inter,
    const __nv_bfloat16 *__restrict__ w13, const int32_t *__restrict__ row_route,
    const int32_t *__restrict__ token_of_route, int top_k, int64_t num_routes,
    const int32_t *__restrict__ mtiles, const int32_t *__restrict__ counters,
    __nv_bfloat16 *__restrict__ act) {
  const int tile = blockIdx.x;
  if (tile >= counters[B200MOE_CNT_MTILES]) return;
  const int e = mtiles[tile * B200MOE_MTILE_WORDS + 0];
  const int rb = mtiles[tile * B200MOE_MTILE_WORDS + 1];
  const int re = mtiles[tile * B200MOE_MTILE_WORDS + 2];
  extern __shared__ uint4 xs[];  // [kRows][V]
  const int V = hidden / 8;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int j0 = (blockIdx.y * kStreamWarps + warp) * kFeatPerWarp;
  const __nv_bfloat16 *w_exp = w13 + static_cast<int64_t>(e) * 2 * inter * hidden;

  for (int c = rb; c < re; c += kRows) {
    const int nr = min(kRows, re - c);
    for (int i = threadIdx.x; i < nr * V; i += blockDim.x) {
      const int n = i / V;
      const int v = i - n * V;
      const int32_t r = row_route[c + n];
      int64_t t = token_of_route ? static_cast<int64_t>(token_of_route[r]) : r / top_k;
      if (r < 0 || r >= num_routes || t < 0 || t >= x_rows) {
        atomicOr(&g_status, kStatusIndex);
        t = 0;
      }
      xs[i] = reinterpret_cast<const uint4 *>(x + t * hidden)[v];
    }
    __syncthreads();
    if (j0 < inter) {
      float out[kFeatPerWarp][kRows];
#pragma unroll
      for (int f = 0; f < kFeatPerWarp; ++f) {
        const int j = j0 + f;
        float ag[kRows], au[kRows];
#pragma unroll
        for (int n = 0; n < kRows; ++n) ag[n] = au[n] = 0.f;
        if (j < inter) {
          const uint4 *gp = reinterpret_cast<const uint4 *>(w_exp + static_cast<int64_t>(j) * hidden);
          const uint4 *up =
              reinterpret_cast<const uint4 *>(w_exp + static_cast<int64_t>(inter + j) * hidden);
          uint4 wg[VPL], wu[VPL];
#pragma unroll
          for (int i = 0; i < VPL; ++i) {
            const int v = lane + 32 * i;
            if (v < V) {
              wg[i] = ld_stream(gp + v);
              wu[i] = ld_stream(up + v);
            }
          }
#pragma unroll
          for (int i = 0; i < VPL; ++i) {
            const int v = lane + 32 * i;
            if (v < V) {
#pragma unroll
              for (int n = 0; n < kRows; ++n) {
                if (n < nr) {
                  const uint4 xv = xs[n * V + v];
                  dot8_bf16(wg[i], xv, ag[n]);
                  dot8_bf16(wu[i], xv, au[n]);
                }
              }
            }
          }
        }
#pragma unroll
        for (int n = 0; n < kRows; ++n) {
          if (n < nr) {
            const float g = warp_sum(ag[n]);
            const float u = warp_sum(au[n]);
            out[f][n] = swiglu_bf16(g, u);
          }
        }
      }
      // Lane n stores route n's 8 features.
#pragma unroll
      for (int n = 0; n < kRows; ++n) {
        if (lane == n && n < nr) {
          float v8[8];
#pragma unroll
          for (int f = 0; f < 8; ++f) v8[f] = out[f][n];
          if (j0 + 8 <= inter) {
            store8_bf16(act + static_cast<int64_t>(c + n) * inter + j0, v8);
          } else {
            for (int f = 0; f < 8 && j0 + f < inter; ++f)
              act[static_cast<int64_t>(c + n) * inter + j0 + f] = __float2bfloat16_rn(v8[f]);
          }
        }
      }
    }
    __syncthreads();
  }
}

// grid = (max m-tiles, ceil(H / 32)); VPL = ceil(I / 256).
template <int VPL>
__global__ void __launch_bounds__(kStreamThreads) down_stream_kernel(
    const __nv_bfloat16 *__restrict__ act, int hidden, int inter,
    const __nv_bfloat16 *__restrict__ w2, const int32_t *__restrict__ row_route,
    const __nv_bfloat16 *__restrict__ route_weights, int64_t num_routes,
    const int32_t *__restrict__ mtiles, const int32_t *__restrict__ counters,
    __nv_bfloat16 *__restrict__ y) {
  const int tile = blockIdx.x;
  if (tile >= counters[B200MOE_CNT_MTILES]) return;
  const int e = mtiles[tile * B200MOE_MTILE_WORDS + 0];
  const int rb = mtiles[tile * B200MOE_MTILE_WORDS + 1];
  const int re = mtiles[tile * B200MOE_MTILE_WORDS + 2];
  extern __shared__ uint4 as[];  // [kRows][V]
  __shared__ int32_t s_route[kRows];
  __shared__ float s_w[kRows];
  const int V = inter / 8;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int h0 = (blockIdx.y * kStreamWarps + warp) * kFeatPerWarp;
  const __nv_bfloat16 *w_exp = w2 + static_cast<int64_t>(e) * hidden * inter;

  for (int c = rb; c < re; c += kRows) {
    const int nr = min(kRows, re - c);
    const uint4 *src = reinterpret_cast<const uint4 *>(act + static_cast<int64_t>(c) * inter);
    for (int i = threadIdx.x; i < nr * V; i += blockDim.x) as[i] = src[i];
    if (threadIdx.x < nr) {
      int32_t r = row_route[c + threadIdx.x];
      if (r < 0 || r >= num_routes) {
        atomicOr(&g_status, kStatusIndex);
        r = -1;
      }
      s_route[threadIdx.x] = r;
      s_w[threadIdx.x] = r >= 0 ? __bfloat162float(route_weights[r]) : 0.f;
    }
    __syncthreads();
    if (h0 < hidden) {
      float out[kFeatPerWarp][kRows];
#pragma unroll
      for (int f = 0; f < kFeatPerWarp; ++f) {
        const int h = h0 + f;
        float acc[kRows];
#pragma unroll
        for (int n = 0; n < kRows; ++n) acc[n] = 0.f;
        if (h < hidden) {
          const uint4 *wp = reinterpret_cast<const uint4 *>(w_exp + static_cast<int64_t>(h) * inter);
          uint4 wv[VPL];
#pragma unroll
          for (int i = 0; i < VPL; ++i) {
            const int v = lane + 32 * i;
            if (v < V) wv[i] = ld_stream(wp + v);
          }
#pragma unroll
          for (int i = 0; i < VPL; ++i) {
            const int v = lane + 32 * i;
            if (v < V) {
#pragma unroll
              for (int n = 0; n < kRows; ++n)
                if (n < nr) dot8_bf16(wv[i], as[n * V + v], acc[n]);
            }
          }
        }
#pragma unroll
        for (int n = 0; n < kRows; ++n)
          if (n < nr) out[f][n] = warp_sum(acc[n]) * s_w[n];
      }
#pragma unroll
      for (int n = 0; n < kRows; ++n) {
        if (lane == n && n < nr && s_route[n] >= 0) {
          float v8[8];
#pragma unroll
          for (int f = 0; f < 8; ++f) v8[f] = out[f][n];
          __nv_bfloat16 *dst = y + static_cast<int64_t>(s_route[n]) * hidden + h0;
          if (h0 + 8 <= hidden) {
            store8_bf16(dst, v8);
          } else {
            for (int f = 0; f < 8 && h0 + f < hidden; ++f) dst[f] = __float2bfloat16_rn(v8[f]);
          }
        }
      }
    }
    __syncthreads();
  }
}

template <int VPL>
int launch_gate_up_stream(dim3 grid, size_t smem, cudaStream_t s, const __nv_bfloat16 *x,
                          int64_t x_rows, int hidden, int inter, const __nv_bfloat16 *w13,
                          const int32_t *row_route, const int32_t *tor, int top_k, int64_t R,
                          const int32_t *mtiles, const int32_t *counters, __nv_bfloat16 *act) {
  if (smem > 48 * 1024)
    B200_CUDA(cudaFuncSetAttribute(gate_up_stream_kernel<VPL>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  gate_up_stream_kernel<VPL><<<grid, kStreamThreads, smem, s>>>(
      x, x_rows, hidden, inter, w13, row_route, tor, top_k, R, mtiles, counters, act);
  B200_LAUNCHED();
  return B200MOE_OK;
}

template <int VPL>
int launch_down_stream(dim3 grid, size_t smem, cudaStream_t s, const __nv_bfloat16 *act,
                       int hidden, int inter, const __nv_bfloat16 *w2, const int32_t *row_route,
                       const __nv_bfloat16 *rw, int64_t R, const int32_t *mtiles,
                       const int32_t *counters, __nv_bfloat16 *y) {
  if (smem > 48 * 1024)
    B200_CUDA(cudaFuncSetAttribute(down_stream_kernel<VPL>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  down_stream_kernel<VPL><<<grid, kStreamThreads, smem, s>>>(act, hidden, inter, w2, row_route,
                                                             rw, R, mtiles, counters, y);
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // namespace

int stream_gate_up(const void *x, int64_t x_rows, int hidden, int inter, const void *w13,
                   const int32_t *row_route, const int32_t *token_of_route, int top_k,
                   int64_t num_routes, const int32_t *mtiles, int64_t max_mtiles,
                   const int32_t *counters, void *act, cudaStream_t s) {
  const int V = hidden / 8;
  const int vpl = (V + 31) / 32;
  const dim3 grid(static_cast<unsigned>(max_mtiles),
                  static_cast<unsigned>((inter + kStreamWarps * kFeatPerWarp - 1) /
                                        (kStreamWarps * kFeatPerWarp)));
  const size_t smem = static_cast<size_t>(kRows) * V * sizeof(uint4);
  const auto *xp = static_cast<const __nv_bfloat16 *>(x);
  const auto *wp = static_cast<const __nv_bfloat16 *>(w13);
  auto *ap = static_cast<__nv_bfloat16 *>(act);
#define B200_GU(VV)                                                                          \
  if (vpl <= VV)                                                                             \
    return launch_gate_up_stream<VV>(grid, smem, s, xp, x_rows, hidden, inter, wp, row_route, \
                                     token_of_route, top_k, num_routes, mtiles, counters, ap);
  B200_GU(1)
  B200_GU(2)
  B200_GU(4)
  B200_GU(8)
  B200_GU(16)
#undef B200_GU
  set_error("hidden %d too large for the streaming engine (max 4096)", hidden);
  return B200MOE_EUNSUPPORTED;
}

int stream_down(const void *act, int hidden, int inter, const void *w2, const int32_t *row_route,
                const void *route_weights, int64_t num_routes, const int32_t *mtiles,
                int64_t max_mtiles, const int32_t *counters, void *y, cudaStream_t s) {
  const int V = inter / 8;
  const int vpl = (V + 31) / 32;
  const dim3 grid(static_cast<unsigned>(max_mtiles),
                  static_cast<unsigned>((hidden + kStreamWarps * kFeatPerWarp - 1) /
                                        (kStreamWarps * kFeatPerWarp)));
  const size_t smem = static_cast<size_t>(kRows) * V * sizeof(uint4);
  const auto *ap = static_cast<const __nv_bfloat16 *>(act);
  const auto *wp = static_cast<const __nv_bfloat16 *>(w2);
  const auto *rw = static_cast<const __nv_bfloat16 *>(route_weights);
  auto *yp = static_cast<__nv_bfloat16 *>(y);
#define B200_DN(VV)                                                                       \
  if (vpl <= VV)                                                                          \
    return launch_down_stream<VV>(grid, smem, s, ap, hidden, inter, wp, row_route, rw,    \
                                  num_routes, mtiles, counters, yp);
  B200_DN(1)
  B200_DN(2)
  B200_DN(3)
  B200_DN(4)
  B200_DN(6)
  B200_DN(8)
#undef B200_DN
  set_error("intermediate %d too large for the streaming engine (max 2048)", inter);
  return B200MOE_EUNSUPPORTED;
}

}  // namespace b200moe
