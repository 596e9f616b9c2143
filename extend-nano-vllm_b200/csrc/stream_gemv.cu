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
#include "route_warp.cuh"
#include "stream_common.cuh"

namespace b200moe {
namespace {

constexpr int kStreamThreads = 128;  // 4 warps
constexpr int kStreamWarps = kStreamThreads / 32;
constexpr int kFeatPerWarp = 8;      // outputs per warp (one 16B store per route)
constexpr int kRows = 8;             // routes per shared-memory chunk

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
    const __nv_bfloat16 *x, int64_t x_rows, int hidden, int inter,
    const __nv_bfloat16 *__restrict__ w13, const int32_t *row_route, const int32_t *token_of_route,
    int top_k, int64_t num_routes, const int32_t *mtiles, const int32_t *counters,
    __nv_bfloat16 *__restrict__ act) {
  pdl_trigger();
  pdl_wait();
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
    const __nv_bfloat16 *act, int hidden, int inter, const __nv_bfloat16 *__restrict__ w2,
    const int32_t *row_route, const __nv_bfloat16 *route_weights, int64_t num_routes,
    const int32_t *mtiles, const int32_t *counters,
    __nv_bfloat16 *__restrict__ y) {
  pdl_trigger();
  pdl_wait();
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
  B200_LAUNCH_PDL(kPdlStream, gate_up_stream_kernel<VPL, NRMAX>, dim3(grid), dim3(kStreamThreads), smem, s,
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
  B200_LAUNCH_PDL(kPdlStream, down_stream_kernel<VPL, NRMAX>, dim3(grid), dim3(kStreamThreads), smem, s, act, hidden, inter, w2, row_route,
                                                             rw, R, mtiles, counters, y);
  B200_LAUNCHED();
  return B200MOE_OK;
}

// ---------------------------------------------------------------------------
// Fused tiny-batch decode (at most 16 routes, no capacity): two launches
// replace router + packing + two projections + combine.  Every CTA routes its
// own token with the router's warp routine, so no packing is needed; the
// arithmetic (routing, gate/up rows, down rows, bf16 rounding points, fp32
// slot-order sum) is the same as the unfused streaming path, so the results
// are identical to it.
// ---------------------------------------------------------------------------
constexpr int kTinyWarps = 8;       // gate/up: 8 warps x 4 features per CTA
constexpr int kTinyFeat = 4;
constexpr int kTinyDownRows = 8;    // down: 8 output rows per CTA, one warp per route slot

// Asks the TMA unit to pull [p, p + bytes) into L2; p and bytes are multiples
// of 16.  Nothing waits on it: it only warms L2 for the loads that follow.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ int local_expert(int e, int num_experts, const int64_t *local_index,
                                            int expert_start, int num_local) {
  if (e < 0 || e >= num_experts) return -1;
  if (local_index) {
    const int64_t l = local_index[e];
    return (l >= 0 && l < num_local) ? static_cast<int>(l) : -1;
  }
  return (e >= expert_start && e < expert_start + num_local) ? e - expert_start : -1;
}

// grid = (num_tokens * top_k, ceil(I / 32)); block = 256.  act: [T*k, I].
// Warp w owns features j0..j0+3 and streams their gate/up rows with one row
// in flight ahead; the dot products and SwiGLU are those of gate_up_chunk.
template <typename TL, int VPT, int VPL>
__global__ void __launch_bounds__(32 * kTinyWarps) tiny_gate_up_kernel(
    const TL *logits, const __nv_bfloat16 *x, int hidden, int inter, int num_experts,
    int top_k, int renormalize, const __nv_bfloat16 *__restrict__ w13, int num_local,
    const int64_t *local_index, int expert_start,
    __nv_bfloat16 *__restrict__ act, int64_t *__restrict__ stats) {
  // Trigger only once the logits are complete, so the down kernel may read
  // them before its own wait.
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint4 xs[];  // [V]
  __shared__ int s_expert;
  const int route = blockIdx.x;
  const int token = route / top_k;
  const int slot = route - token * top_k;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int V = hidden / 8;
  if (warp == 0) {
    float w;
    int id;
    warp_route_token<TL, VPT>(logits + static_cast<int64_t>(token) * num_experts, num_experts,
                              top_k, renormalize, lane, &w, &id);
    if (lane == slot) s_expert = id;
  }
  const uint4 *xrow = reinterpret_cast<const uint4 *>(x + static_cast<int64_t>(token) * hidden);
  for (int v = threadIdx.x; v < V; v += blockDim.x) xs[v] = xrow[v];
  __syncthreads();
  const int le = local_expert(s_expert, num_experts, local_index, expert_start, num_local);
  if (le < 0) return;
  if (stats && blockIdx.y == 0 && threadIdx.x == 0)
    atomicAdd(reinterpret_cast<unsigned long long *>(&stats[0]), 1ull);
  const int j0 = (blockIdx.y * kTinyWarps + warp) * kTinyFeat;
  if (j0 >= inter) return;
  const int nfeat = min(kTinyFeat, inter - j0);
  const __nv_bfloat16 *w_exp = w13 + static_cast<int64_t>(le) * 2 * inter * hidden;
  auto row_ptr = [&](int s) {
    const int j = j0 + (s >> 1);
    const int row = (s & 1) ? inter + j : j;
    return reinterpret_cast<const uint4 *>(w_exp + static_cast<int64_t>(row) * hidden);
  };
  float res[kTinyFeat] = {0.f, 0.f, 0.f, 0.f};
  uint4 cur[VPL];
  load_row<VPL>(row_ptr(0), V, lane, cur);
  float gsum = 0.f;
#pragma unroll
  for (int s = 0; s < 2 * kTinyFeat; ++s) {
    if ((s >> 1) >= nfeat) break;
    uint4 nxt[VPL];
    const bool more = s + 1 < 2 * nfeat;
    if (more) load_row<VPL>(row_ptr(s + 1), V, lane, nxt);
    float acc[1];
    dot_rows<VPL, 1>(cur, xs, V, lane, acc);
    const float sum = warp_sum(acc[0]);
    if ((s & 1) == 0)
      gsum = sum;
    else
      res[s >> 1] = swiglu_bf16(gsum, sum);
    if (more) {
#pragma unroll
      for (int i = 0; i < VPL; ++i) cur[i] = nxt[i];
    }
  }
  if (lane == 0) {
    __nv_bfloat16 *dst = act + static_cast<int64_t>(route) * inter + j0;
#pragma unroll
    for (int f = 0; f < kTinyFeat; ++f)
      if (f < nfeat) dst[f] = __float2bfloat16_rn(res[f]);
  }
}

// grid = (num_tokens, ceil(H / 8)); block = 32 * top_k.  Warp s computes the
// bf16 down-projection rows of route slot s for the CTA's 8 outputs; the
// routes are then summed in fp32 in slot order and stored as bf16.
template <typename TL, int VPT, int VPL>
__global__ void __launch_bounds__(512) tiny_down_combine_kernel(
    const TL *logits, const __nv_bfloat16 *act, int hidden, int inter, int num_experts,
    int top_k, int renormalize, const __nv_bfloat16 *__restrict__ w2, int num_local,
    const int64_t *local_index, int expert_start,
    __nv_bfloat16 *__restrict__ out) {
  pdl_trigger();
  // Rows in flight per warp, sized so the row buffers (RB * VPL 16-byte
  // registers) stay within the 128 registers a 512-thread block allows.
  constexpr int RB = VPL <= 2 ? 8 : (VPL <= 4 ? 4 : 2);
  extern __shared__ uint4 as[];  // [top_k][V]
  __shared__ int s_le[16];
  __shared__ float s_w[16];
  __shared__ float s_y[16][kTinyDownRows];
  const int token = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int V = inter / 8;
  if (warp == 0) {
    float w;
    int id;
    warp_route_token<TL, VPT>(logits + static_cast<int64_t>(token) * num_experts, num_experts,
                              top_k, renormalize, lane, &w, &id);
    if (lane < top_k) {
      s_le[lane] = local_expert(id, num_experts, local_index, expert_start, num_local);
      s_w[lane] = bf16_round(w);  // the router stores bf16 weights
    }
  }
  __syncthreads();
  const int le = s_le[warp];
  const int h0 = blockIdx.y * kTinyDownRows;
  // Routing reads only the logits, which were complete before the gate/up
  // kernel triggered this launch: warm L2 with this CTA's weight rows while
  // the gate/up kernel still runs, then wait for its activations.
  if (le >= 0 && lane == 0 && kTinyDownRows > RB) {
    const int nrows = min(kTinyDownRows - RB, hidden - h0 - RB);
    if (nrows > 0)
      prefetch_l2_bulk(w2 + (static_cast<int64_t>(le) * hidden + h0 + RB) * inter,
                       static_cast<uint32_t>(nrows) * inter * 2);
  }
  // The first RB weight rows go to registers before the wait (the weights are
  // not written by the gate/up kernel); the rest were prefetched into L2.
  const __nv_bfloat16 *w_exp = w2 + static_cast<int64_t>(le < 0 ? 0 : le) * hidden * inter;
  uint4 w_first[RB][VPL];
  if (le >= 0) {
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const int h = h0 + r;
      if (h < hidden)
        load_row<VPL>(reinterpret_cast<const uint4 *>(w_exp + static_cast<int64_t>(h) * inter), V,
                      lane, w_first[r]);
    }
  }
  pdl_wait();
  if (le >= 0) {
    const uint4 *src = reinterpret_cast<const uint4 *>(
        act + (static_cast<int64_t>(token) * top_k + warp) * inter);
    for (int v = lane; v < V; v += 32) as[warp * V + v] = src[v];
  }
  __syncwarp();
  if (le >= 0) {
#pragma unroll
    for (int f0 = 0; f0 < kTinyDownRows; f0 += RB) {
      uint4 w[RB][VPL];
      if (f0 == 0) {
#pragma unroll
        for (int r = 0; r < RB; ++r)
#pragma unroll
          for (int i = 0; i < VPL; ++i) w[r][i] = w_first[r][i];
      } else {
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          const int h = h0 + f0 + r;
          if (h < hidden)
            load_row<VPL>(reinterpret_cast<const uint4 *>(w_exp + static_cast<int64_t>(h) * inter),
                          V, lane, w[r]);
        }
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        if (h0 + f0 + r < hidden) {
          float acc[1];
          dot_rows<VPL, 1>(w[r], as + warp * V, V, lane, acc);
          const float y = bf16_round(warp_sum(acc[0]) * s_w[warp]);
          if (lane == 0) s_y[warp][f0 + r] = y;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < kTinyDownRows && h0 + static_cast<int>(threadIdx.x) < hidden) {
    float total = 0.f;
    for (int s = 0; s < top_k; ++s)
      if (s_le[s] >= 0) total += s_y[s][threadIdx.x];
    out[static_cast<int64_t>(token) * hidden + h0 + threadIdx.x] = __float2bfloat16_rn(total);
  }
}

template <typename TL, int VPT, int VPLG, int VPLD>
int launch_tiny(const void *logits, const void *x, int64_t num_tokens, int hidden, int inter,
                int num_experts, int top_k, int renormalize, const void *w13, const void *w2,
                int num_local, const int64_t *local_index, int expert_start, void *act, void *out,
                int64_t *stats, cudaStream_t s) {
  const auto *lg = static_cast<const TL *>(logits);
  const dim3 g1(static_cast<unsigned>(num_tokens * top_k),
                static_cast<unsigned>((inter + kTinyWarps * kTinyFeat - 1) /
                                      (kTinyWarps * kTinyFeat)));
  const size_t smem1 = static_cast<size_t>(hidden / 8) * sizeof(uint4);
  if (smem1 > 48 * 1024)
    B200_CUDA(cudaFuncSetAttribute(tiny_gate_up_kernel<TL, VPT, VPLG>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1));
  B200_LAUNCH_PDL(kPdlTiny, tiny_gate_up_kernel<TL, VPT, VPLG>, dim3(g1), dim3(32 * kTinyWarps), smem1, s,
      lg, static_cast<const __nv_bfloat16 *>(x), hidden, inter, num_experts, top_k, renormalize,
      static_cast<const __nv_bfloat16 *>(w13), num_local, local_index, expert_start,
      static_cast<__nv_bfloat16 *>(act), stats);
  B200_LAUNCHED();
  const dim3 g2(static_cast<unsigned>(num_tokens),
                static_cast<unsigned>((hidden + kTinyDownRows - 1) / kTinyDownRows));
  const size_t smem2 = static_cast<size_t>(top_k) * (inter / 8) * sizeof(uint4);
  if (smem2 > 48 * 1024)
    B200_CUDA(cudaFuncSetAttribute(tiny_down_combine_kernel<TL, VPT, VPLD>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2));
  B200_LAUNCH_PDL(kPdlTiny, tiny_down_combine_kernel<TL, VPT, VPLD>, dim3(g2), dim3(32 * top_k), smem2, s,
      lg, static_cast<const __nv_bfloat16 *>(act), hidden, inter, num_experts, top_k,
      renormalize, static_cast<const __nv_bfloat16 *>(w2), num_local, local_index, expert_start,
      static_cast<__nv_bfloat16 *>(out));
  B200_LAUNCHED();
  return B200MOE_OK;
}

template <typename TL, int VPT>
int dispatch_tiny(const void *logits, const void *x, int64_t num_tokens, int hidden, int inter,
                  int num_experts, int top_k, int renormalize, const void *w13, const void *w2,
                  int num_local, const int64_t *local_index, int expert_start, void *act,
                  void *out, int64_t *stats, cudaStream_t s) {
  const int vg = (hidden / 8 + 31) / 32;
  const int vd = (inter / 8 + 31) / 32;
#define B200_TINY(G, D)                                                                         \
  if (vg <= G && vd <= D)                                                                       \
    return launch_tiny<TL, VPT, G, D>(logits, x, num_tokens, hidden, inter, num_experts, top_k, \
                                      renormalize, w13, w2, num_local, local_index,             \
                                      expert_start, act, out, stats, s);
  B200_TINY(1, 1)
  B200_TINY(8, 3)
  B200_TINY(16, 6)
  B200_TINY(16, 8)
#undef B200_TINY
  set_error("tiny decode path: hidden %d / intermediate %d unsupported", hidden, inter);
  return B200MOE_EUNSUPPORTED;
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

extern "C" int b200moe_decode_tiny(const void *logits, int logits_dtype, const void *x,
                                   int64_t num_tokens, int hidden, int inter, int num_experts,
                                   int top_k, int renormalize, const void *w13, const void *w2,
                                   int num_local_experts, const int64_t *local_index,
                                   int expert_start, void *act, void *out, int64_t *stats,
                                   void *stream) {
  using namespace b200moe;
  B200_ARG(num_tokens >= 0 && hidden > 0 && inter > 0 && num_local_experts > 0, "bad shape");
  B200_ARG(top_k >= 1 && top_k <= num_experts, "top_k must be between 1 and num_experts");
  B200_UNSUPPORTED(num_tokens * top_k <= 16, "the tiny decode path takes at most 16 routes");
  B200_UNSUPPORTED(num_experts <= 1024, "num_experts %d > 1024 is not supported", num_experts);
  B200_UNSUPPORTED(hidden % 16 == 0 && inter % 16 == 0 && hidden <= 4096 && inter <= 2048,
                   "hidden/intermediate sizes must be multiples of 16 (max 4096/2048)");
  if (num_tokens == 0) return B200MOE_OK;
  B200_ARG(logits && x && w13 && w2 && act && out, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int vpt = (num_experts + 31) / 32;
#define B200_TINY_L(TL, V)                                                                       \
  if (vpt <= V)                                                                                  \
    return dispatch_tiny<TL, V>(logits, x, num_tokens, hidden, inter, num_experts, top_k,       \
                                renormalize, w13, w2, num_local_experts, local_index,           \
                                expert_start, act, out, stats, s);
  if (logits_dtype == B200MOE_F32) {
    B200_TINY_L(float, 1)
    B200_TINY_L(float, 4)
    B200_TINY_L(float, 32)
  } else if (logits_dtype == B200MOE_BF16) {
    B200_TINY_L(__nv_bfloat16, 1)
    B200_TINY_L(__nv_bfloat16, 4)
    B200_TINY_L(__nv_bfloat16, 32)
  }
#undef B200_TINY_L
  set_error("tiny decode path: unsupported logits dtype %d", logits_dtype);
  return B200MOE_EINVAL;
}
