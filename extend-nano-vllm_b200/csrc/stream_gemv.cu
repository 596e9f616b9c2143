// Weight-streaming expert kernels for small decode buckets (engine STREAM).
//
// In a decode bucket each active expert owns only a handful of routes, so the
// grouped GEMMs of the reference (Triton _grouped_moe_gemm_kernel,
// nanovllm/layers/moe.py:63-139, launched per 16-row tile) are bound by
// reading every active expert's weights once from HBM.  These kernels stream
// each weight row once per chunk of routes with 16-byte non-allocating loads
// (lane l reads vectors l, l+32, ... of a row: fully coalesced), keep the
// chunk's activations in shared memory and reduce the dot products with warp
// shuffles.
//  * The inner loops are specialised on the chunk's route count (1, 2, 4 or
//    8) so no instruction is issued for absent routes.
//  * gate/up: a warp owns 8 consecutive features; the gate and up rows of the
//    next feature are loaded while the current one is reduced (register
//    double buffering), so every warp always has a full row pair in flight.
//  * down: a warp owns 8 consecutive output rows and loads all of them (or
//    half, for long rows) before reducing.
//  * Results go through shared memory and leave as one 16-byte store per
//    route and warp.
#include "common.cuh"

namespace b200moe {
namespace {

constexpr int kStreamThreads = 128;  // 4 warps
constexpr int kStreamWarps = kStreamThreads / 32;
constexpr int kFeatPerWarp = 8;      // outputs per warp (one 16B store per route)
constexpr int kRows = 8;             // routes per shared-memory chunk

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

// One chunk of NR routes for the warp's 8 features; results to res[f][n].
template <int VPL, int NR>
__device__ __forceinline__ void gate_up_chunk(const __nv_bfloat16 *w_exp, int inter, int V,
                                              int j0, int lane, const uint4 *xs,
                                              float (*res)[kRows]) {
  // Row sequence gate(j0), up(j0), gate(j0+1), up(j0+1), ...: the next row is
  // in flight while the current one is reduced.
  const int hidden = V * 8;
  const int nfeat = min(kFeatPerWarp, inter - j0);
  auto row_ptr = [&](int s) {
    const int j = j0 + (s >> 1);
    const int row = (s & 1) ? inter + j : j;
    return reinterpret_cast<const uint4 *>(w_exp + static_cast<int64_t>(row) * hidden);
  };
  uint4 cur[VPL];
  load_row<VPL>(row_ptr(0), V, lane, cur);
  float gsum[NR];
#pragma unroll
  for (int s = 0; s < 2 * kFeatPerWarp; ++s) {
    if ((s >> 1) >= nfeat) break;
    uint4 nxt[VPL];
    const bool more = s + 1 < 2 * nfeat;
    if (more) load_row<VPL>(row_ptr(s + 1), V, lane, nxt);
    float acc[NR];
    dot_rows<VPL, NR>(cur, xs, V, lane, acc);
#pragma unroll
    for (int n = 0; n < NR; ++n) {
      const float sum = warp_sum(acc[n]);
      if ((s & 1) == 0) {
        gsum[n] = sum;
      } else if (lane == 0) {
        res[s >> 1][n] = swiglu_bf16(gsum[n], sum);
      }
    }
    if (more) {
#pragma unroll
      for (int i = 0; i < VPL; ++i) cur[i] = nxt[i];
    }
  }
}

// grid = (max m-tiles, ceil(I / 32)); VPL >= ceil(H / 256) vectors per lane;
// NRMAX (1, 2, 4 or 8) bounds the routes handled per chunk.
template <int VPL, int NRMAX>
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
  extern __shared__ uint4 xs[];  // [NRMAX][V]
  __shared__ float s_res[kStreamWarps][kFeatPerWarp][kRows];
  const int V = hidden / 8;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int j0 = (blockIdx.y * kStreamWarps + warp) * kFeatPerWarp;
  const __nv_bfloat16 *w_exp = w13 + static_cast<int64_t>(e) * 2 * inter * hidden;

  for (int c = rb; c < re; c += NRMAX) {
    const int nr = min(NRMAX, re - c);
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
      float(*res)[kRows] = s_res[warp];
      if (nr == 1) {
        gate_up_chunk<VPL, 1>(w_exp, inter, V, j0, lane, xs, res);
      } else if constexpr (NRMAX >= 2) {
        if (nr == 2)
          gate_up_chunk<VPL, 2>(w_exp, inter, V, j0, lane, xs, res);
        else if constexpr (NRMAX >= 4) {
          if (nr <= 4)
            gate_up_chunk<VPL, 4>(w_exp, inter, V, j0, lane, xs, res);
          else if constexpr (NRMAX >= 8)
            gate_up_chunk<VPL, 8>(w_exp, inter, V, j0, lane, xs, res);
        }
      }
      __syncwarp();
      if (lane < nr) {
        float v8[8];
#pragma unroll
        for (int f = 0; f < 8; ++f) v8[f] = res[f][lane];
        __nv_bfloat16 *dst = act + static_cast<int64_t>(c + lane) * inter + j0;
        if (j0 + 8 <= inter) {
          store8_bf16(dst, v8);
        } else {
          for (int f = 0; f < 8 && j0 + f < inter; ++f) dst[f] = __float2bfloat16_rn(v8[f]);
        }
      }
    }
    __syncthreads();
  }
}

// One chunk of NR routes for the warp's 8 output rows; rows are loaded RB at
// a time.
template <int VPL, int NR, int RB>
__device__ __forceinline__ void down_chunk(const __nv_bfloat16 *w_exp, int hidden, int V, int h0,
                                           int lane, const uint4 *as, const float *s_w,
                                           float (*res)[kRows]) {
  const int inter = V * 8;
#pragma unroll
  for (int f0 = 0; f0 < kFeatPerWarp; f0 += RB) {
    uint4 w[RB][VPL];
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const int h = h0 + f0 + r;
      if (h < hidden)
        load_row<VPL>(reinterpret_cast<const uint4 *>(w_exp + static_cast<int64_t>(h) * inter), V,
                      lane, w[r]);
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      if (h0 + f0 + r < hidden) {
        float acc[NR];
        dot_rows<VPL, NR>(w[r], as, V, lane, acc);
#pragma unroll
        for (int n = 0; n < NR; ++n) {
          const float s = warp_sum(acc[n]);
          if (lane == 0) res[f0 + r][n] = s * s_w[n];
        }
      }
    }
  }
}

// grid = (max m-tiles, ceil(H / 32)); VPL >= ceil(I / 256); NRMAX as above.
template <int VPL, int NRMAX>
__global__ void __launch_bounds__(kStreamThreads) down_stream_kernel(
    const __nv_bfloat16 *__restrict__ act, int hidden, int inter,
    const __nv_bfloat16 *__restrict__ w2, const int32_t *__restrict__ row_route,
    const __nv_bfloat16 *__restrict__ route_weights, int64_t num_routes,
    const int32_t *__restrict__ mtiles, const int32_t *__restrict__ counters,
    __nv_bfloat16 *__restrict__ y) {
  constexpr int RB = VPL == 1 ? 8 : (VPL <= 3 ? 4 : 2);  // rows in flight per warp
  const int tile = blockIdx.x;
  if (tile >= counters[B200MOE_CNT_MTILES]) return;
  const int e = mtiles[tile * B200MOE_MTILE_WORDS + 0];
  const int rb = mtiles[tile * B200MOE_MTILE_WORDS + 1];
  const int re = mtiles[tile * B200MOE_MTILE_WORDS + 2];
  extern __shared__ uint4 as[];  // [NRMAX][V]
  __shared__ int32_t s_route[kRows];
  __shared__ float s_w[kRows];
  __shared__ float s_res[kStreamWarps][kFeatPerWarp][kRows];
  const int V = inter / 8;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int h0 = (blockIdx.y * kStreamWarps + warp) * kFeatPerWarp;
  const __nv_bfloat16 *w_exp = w2 + static_cast<int64_t>(e) * hidden * inter;

  for (int c = rb; c < re; c += NRMAX) {
    const int nr = min(NRMAX, re - c);
    const uint4 *src = reinterpret_cast<const uint4 *>(act + static_cast<int64_t>(c) * inter);
    for (int i = threadIdx.x; i < nr * V; i += blockDim.x) as[i] = src[i];
    if (threadIdx.x < kRows) {
      int32_t r = -1;
      if (static_cast<int>(threadIdx.x) < nr) {
        r = row_route[c + threadIdx.x];
        if (r < 0 || r >= num_routes) {
          atomicOr(&g_status, kStatusIndex);
          r = -1;
        }
      }
      s_route[threadIdx.x] = r;
      s_w[threadIdx.x] = r >= 0 ? __bfloat162float(route_weights[r]) : 0.f;
    }
    __syncthreads();
    if (h0 < hidden) {
      float(*res)[kRows] = s_res[warp];
      if (nr == 1) {
        down_chunk<VPL, 1, RB>(w_exp, hidden, V, h0, lane, as, s_w, res);
      } else if constexpr (NRMAX >= 2) {
        if (nr == 2)
          down_chunk<VPL, 2, RB>(w_exp, hidden, V, h0, lane, as, s_w, res);
        else if constexpr (NRMAX >= 4) {
          if (nr <= 4)
            down_chunk<VPL, 4, RB>(w_exp, hidden, V, h0, lane, as, s_w, res);
          else if constexpr (NRMAX >= 8)
            down_chunk<VPL, 8, RB>(w_exp, hidden, V, h0, lane, as, s_w, res);
        }
      }
      __syncwarp();
      if (lane < nr && s_route[lane] >= 0) {
        float v8[8];
#pragma unroll
        for (int f = 0; f < 8; ++f) v8[f] = res[f][lane];
        __nv_bfloat16 *dst = y + static_cast<int64_t>(s_route[lane]) * hidden + h0;
        if (h0 + 8 <= hidden) {
          store8_bf16(dst, v8);
        } else {
          for (int f = 0; f < 8 && h0 + f < hidden; ++f) dst[f] = __float2bfloat16_rn(v8[f]);
        }
      }
    }
    __syncthreads();
  }
}

template <int VPL, int NRMAX>
int launch_gate_up_stream(dim3 grid, size_t smem, cudaStream_t s, const __nv_bfloat16 *x,
                          int64_t x_rows, int hidden, int inter, const __nv_bfloat16 *w13,
                          const int32_t *row_route, const int32_t *tor, int top_k, int64_t R,
                          const int32_t *mtiles, const int32_t *counters, __nv_bfloat16 *act) {
  if (smem > 48 * 1024)
    B200_CUDA(cudaFuncSetAttribute(gate_up_stream_kernel<VPL, NRMAX>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  gate_up_stream_kernel<VPL, NRMAX><<<grid, kStreamThreads, smem, s>>>(
      x, x_rows, hidden, inter, w13, row_route, tor, top_k, R, mtiles, counters, act);
  B200_LAUNCHED();
  return B200MOE_OK;
}

template <int VPL, int NRMAX>
int launch_down_stream(dim3 grid, size_t smem, cudaStream_t s, const __nv_bfloat16 *act,
                       int hidden, int inter, const __nv_bfloat16 *w2, const int32_t *row_route,
                       const __nv_bfloat16 *rw, int64_t R, const int32_t *mtiles,
                       const int32_t *counters, __nv_bfloat16 *y) {
  if (smem > 48 * 1024)
    B200_CUDA(cudaFuncSetAttribute(down_stream_kernel<VPL, NRMAX>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  down_stream_kernel<VPL, NRMAX><<<grid, kStreamThreads, smem, s>>>(act, hidden, inter, w2, row_route,
                                                             rw, R, mtiles, counters, y);
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // namespace

int nr_bound(int64_t max_expert_rows) {
  if (max_expert_rows == 1) return 1;
  if (max_expert_rows == 2) return 2;
  if (max_expert_rows >= 3 && max_expert_rows <= 4) return 4;
  return 8;
}

int stream_gate_up(const void *x, int64_t x_rows, int hidden, int inter, const void *w13,
                   const int32_t *row_route, const int32_t *token_of_route, int top_k,
                   int64_t num_routes, const int32_t *mtiles, int64_t max_mtiles,
                   const int32_t *counters, void *act, cudaStream_t s) {
  const int V = hidden / 8;
  const int vpl = (V + 31) / 32;
  const dim3 grid(static_cast<unsigned>(max_mtiles),
                  static_cast<unsigned>((inter + kStreamWarps * kFeatPerWarp - 1) /
                                        (kStreamWarps * kFeatPerWarp)));
  // A token contributes at most one route per expert, so an expert never has
  // more rows than there are token rows.
  const int nrmax = nr_bound(x_rows);
  const size_t smem = static_cast<size_t>(nrmax) * V * sizeof(uint4);
  const auto *xp = static_cast<const __nv_bfloat16 *>(x);
  const auto *wp = static_cast<const __nv_bfloat16 *>(w13);
  auto *ap = static_cast<__nv_bfloat16 *>(act);
#define B200_GU(VV, NN)                                                                      \
  if (vpl <= VV && nrmax == NN)                                                              \
    return launch_gate_up_stream<VV, NN>(grid, smem, s, xp, x_rows, hidden, inter, wp,       \
                                         row_route, token_of_route, top_k, num_routes,       \
                                         mtiles, counters, ap);
#define B200_GU_ALL(VV) B200_GU(VV, 1) B200_GU(VV, 2) B200_GU(VV, 4) B200_GU(VV, 8)
  B200_GU_ALL(1)
  B200_GU_ALL(2)
  B200_GU_ALL(4)
  B200_GU_ALL(8)
  B200_GU_ALL(16)
#undef B200_GU_ALL
#undef B200_GU
  set_error("hidden %d too large for the streaming engine (max 4096)", hidden);
  return B200MOE_EUNSUPPORTED;
}

int stream_down(const void *act, int hidden, int inter, const void *w2, const int32_t *row_route,
                const void *route_weights, int64_t num_routes, int64_t max_expert_rows,
                const int32_t *mtiles, int64_t max_mtiles, const int32_t *counters, void *y,
                cudaStream_t s) {
  const int V = inter / 8;
  const int vpl = (V + 31) / 32;
  const dim3 grid(static_cast<unsigned>(max_mtiles),
                  static_cast<unsigned>((hidden + kStreamWarps * kFeatPerWarp - 1) /
                                        (kStreamWarps * kFeatPerWarp)));
  const int nrmax = nr_bound(max_expert_rows);
  const size_t smem = static_cast<size_t>(nrmax) * V * sizeof(uint4);
  const auto *ap = static_cast<const __nv_bfloat16 *>(act);
  const auto *wp = static_cast<const __nv_bfloat16 *>(w2);
  const auto *rw = static_cast<const __nv_bfloat16 *>(route_weights);
  auto *yp = static_cast<__nv_bfloat16 *>(y);
#define B200_DN(VV, NN)                                                                      \
  if (vpl <= VV && nrmax == NN)                                                              \
    return launch_down_stream<VV, NN>(grid, smem, s, ap, hidden, inter, wp, row_route, rw,   \
                                      num_routes, mtiles, counters, yp);
#define B200_DN_ALL(VV) B200_DN(VV, 1) B200_DN(VV, 2) B200_DN(VV, 4) B200_DN(VV, 8)
  B200_DN_ALL(1)
  B200_DN_ALL(2)
  B200_DN_ALL(3)
  B200_DN_ALL(6)
  B200_DN_ALL(8)
#undef B200_DN_ALL
#undef B200_DN
  set_error("intermediate %d too large for the streaming engine (max 2048)", inter);
  return B200MOE_EUNSUPPORTED;
}

}  // namespace b200moe
