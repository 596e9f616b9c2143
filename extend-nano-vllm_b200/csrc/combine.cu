// Route-order combine and the A-row gather of the tcgen05 gate/up GEMM.
//
// combine: out[t, :] = sum_{s < k} Y[route_rows[t*k + s], :] in fp32 (or
// fp64) in slot order; rows >= num_rows contribute zero.  Same arithmetic as
// the reference Triton _combine_expert_routes_kernel
// (nanovllm/layers/moe.py:164-192), so its results are bit-identical.
#include "common.cuh"

namespace b200moe {
namespace {

template <typename Acc, typename Out>
__device__ __forceinline__ void store8(Out *dst, const Acc (&v)[8]);

template <>
__device__ __forceinline__ void store8<float, __nv_bfloat16>(__nv_bfloat16 *dst,
                                                           const float (&v)[8]) {
  uint4 o;
  __nv_bfloat162 *op = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) op[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4 *>(dst) = o;
}
template <>
__device__ __forceinline__ void store8<double, __nv_bfloat16>(__nv_bfloat16 *dst,
                                                            const double (&v)[8]) {
  uint4 o;
  __nv_bfloat16 *op = reinterpret_cast<__nv_bfloat16 *>(&o);
#pragma unroll
  for (int i = 0; i < 8; ++i) op[i] = __double2bfloat16(v[i]);
  *reinterpret_cast<uint4 *>(dst) = o;
}
template <>
__device__ __forceinline__ void store8<float, float>(float *dst, const float (&v)[8]) {
  reinterpret_cast<float4 *>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4 *>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
__device__ __forceinline__ void store8<double, float>(float *dst, const double (&v)[8]) {
  reinterpret_cast<float4 *>(dst)[0] = make_float4((float)v[0], (float)v[1], (float)v[2], (float)v[3]);
  reinterpret_cast<float4 *>(dst)[1] = make_float4((float)v[4], (float)v[5], (float)v[6], (float)v[7]);
}
template <>
__device__ __forceinline__ void store8<float, double>(double *dst, const float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) dst[i] = v[i];
}
template <>
__device__ __forceinline__ void store8<double, double>(double *dst, const double (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) dst[i] = v[i];
}

// One thread per 8 columns of one token.  hidden % 8 == 0.
// kBatch (small batches, latency-bound): the slot rows of eight routes are
// requested together before any is summed; otherwise four at a time (fewer
// registers, so bandwidth-bound batches keep more threads resident).  The sum
// is in slot order either way.
template <typename Acc, typename Out, bool kBatch>
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16 *y,
                                                      int64_t num_rows,
                                                      const int32_t *route_rows,
                                                      int64_t num_tokens, int top_k, int hidden,
                                                      Out *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int vec_per_row = hidden / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t token = idx / vec_per_row;
  const int col = static_cast<int>(idx % vec_per_row) * 8;
  if (token >= num_tokens) return;
  Acc acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = Acc(0);
  auto add = [&](const uint4 &v) {
    const __nv_bfloat162 *vp = reinterpret_cast<const __nv_bfloat162 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(vp[i]);
      acc[2 * i] += Acc(f.x);
      acc[2 * i + 1] += Acc(f.y);
    }
  };
  if constexpr (kBatch) {
    for (int s0 = 0; s0 < top_k; s0 += 8) {
      int64_t row[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t route = token * top_k + s0 + j;
        row[j] = s0 + j >= top_k ? -1
                 : (route_rows ? static_cast<int64_t>(route_rows[route]) : route);
      }
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (row[j] >= 0 && row[j] < num_rows)
          v[j] = *reinterpret_cast<const uint4 *>(y + row[j] * hidden + col);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (row[j] >= 0 && row[j] < num_rows) add(v[j]);
    }
  } else {
    // Four slots per step: their row indices, then their rows, are requested
    // together (two round trips per four slots instead of eight).
    for (int s0 = 0; s0 < top_k; s0 += 4) {
      int64_t row[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t route = token * top_k + s0 + j;
        row[j] = s0 + j >= top_k ? -1
                 : (route_rows ? static_cast<int64_t>(route_rows[route]) : route);
      }
      uint4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (row[j] >= 0 && row[j] < num_rows)
          v[j] = *reinterpret_cast<const uint4 *>(y + row[j] * hidden + col);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (row[j] >= 0 && row[j] < num_rows) add(v[j]);
    }
  }
  store8<Acc, Out>(out + token * hidden + col, acc);
}

// Token counts up to which the combine requests all slot rows at once.
constexpr int64_t kCombineBatchTokens = 256;

template <typename Acc>
int launch_combine(const void *y, int64_t num_rows, const int32_t *route_rows,
                   int64_t num_tokens, int top_k, int hidden, void *out, int out_dtype,
                   cudaStream_t s) {
  const int64_t threads_total = num_tokens * (hidden / 8);
  const int threads = 256;
  const int64_t blocks = (threads_total + threads - 1) / threads;
  const auto *yp = static_cast<const __nv_bfloat16 *>(y);
  const bool batch = num_tokens <= kCombineBatchTokens;
#define B200_COMBINE(OUT)                                                                      \
  if (batch)                                                                                   \
    B200_LAUNCH_PDL(kPdlCombine, combine_kernel<Acc, OUT, true>, dim3(blocks), dim3(threads),  \
                    0, s, yp, num_rows, route_rows, num_tokens, top_k, hidden,                 \
                    static_cast<OUT *>(out));                                                  \
  else                                                                                         \
    B200_LAUNCH_PDL(kPdlCombine, combine_kernel<Acc, OUT, false>, dim3(blocks), dim3(threads), \
                    0, s, yp, num_rows, route_rows, num_tokens, top_k, hidden,                 \
                    static_cast<OUT *>(out));
  switch (out_dtype) {
    case B200MOE_BF16:
      B200_COMBINE(__nv_bfloat16)
      break;
    case B200MOE_F32:
      B200_COMBINE(float)
      break;
    case B200MOE_F64:
      B200_COMBINE(double)
      break;
    default:
      set_error("unsupported combine output dtype %d", out_dtype);
      return B200MOE_EINVAL;
  }
#undef B200_COMBINE
  B200_LAUNCHED();
  return B200MOE_OK;
}

// One warp per packed row; copies hidden bf16 values with 16-byte vectors.
__global__ void __launch_bounds__(256) gather_rows_kernel(
    const __nv_bfloat16 *x, int64_t x_rows, int hidden, const int32_t *row_route,
    const int32_t *token_of_route, int top_k, int64_t num_routes, int64_t row_capacity,
    const int32_t *counters,
    __nv_bfloat16 *__restrict__ x_packed) {
  pdl_trigger();
  pdl_wait();
  const int64_t total = counters[B200MOE_CNT_PADDED_ROWS];
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int vecs = hidden / 8;
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       p < total && p < row_capacity; p += warps) {
    const int32_t r = row_route[p];
    if (r < 0 || r >= num_routes) continue;
    const int64_t t = token_of_route ? static_cast<int64_t>(token_of_route[r]) : r / top_k;
    if (t < 0 || t >= x_rows) {
      if (lane == 0) atomicOr(&g_status, kStatusIndex);
      continue;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(x + t * hidden);
    uint4 *dst = reinterpret_cast<uint4 *>(x_packed + p * hidden);
    // Four 16-byte loads in flight per lane before the stores.
    int v = lane;
    for (; v + 96 < vecs; v += 128) {
      const uint4 a = src[v], b = src[v + 32], c = src[v + 64], d = src[v + 96];
      dst[v] = a;
      dst[v + 32] = b;
      dst[v + 64] = c;
      dst[v + 96] = d;
    }
    for (; v < vecs; v += 32) dst[v] = src[v];
  }
}

}  // namespace
}  // namespace b200moe

extern "C" {

int b200moe_combine(const void *y, int64_t num_rows, const int32_t *route_rows,
                    int64_t num_tokens, int top_k, int hidden, int accum_f64, void *out,
                    int out_dtype, void *stream) {
  B200_ARG(num_tokens >= 0 && top_k >= 1 && hidden >= 1, "bad combine shape");
  B200_UNSUPPORTED(hidden % 8 == 0, "hidden %d must be a multiple of 8", hidden);
  if (num_tokens == 0) return B200MOE_OK;
  B200_ARG(out != nullptr, "out must not be NULL");
  B200_ARG(num_rows == 0 || y != nullptr, "y must not be NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (accum_f64)
    return b200moe::launch_combine<double>(y, num_rows, route_rows, num_tokens, top_k, hidden,
                                           out, out_dtype, s);
  return b200moe::launch_combine<float>(y, num_rows, route_rows, num_tokens, top_k, hidden, out,
                                        out_dtype, s);
}

int b200moe_gather_rows(const void *x, int64_t x_rows, int hidden, const int32_t *row_route,
                        const int32_t *token_of_route, int top_k, int64_t num_routes,
                        int64_t row_capacity, const int32_t *counters, void *x_packed,
                        void *stream) {
  B200_ARG(hidden > 0 && top_k >= 1, "bad gather shape");
  B200_UNSUPPORTED(hidden % 8 == 0, "hidden %d must be a multiple of 8", hidden);
  if (row_capacity == 0 || num_routes == 0) return B200MOE_OK;
  B200_ARG(x && row_route && counters && x_packed, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t blocks = (row_capacity + 7) / 8;
  const int64_t cap = 8LL * b200moe::sm_count();
  if (blocks > cap) blocks = cap;
  B200_LAUNCH_PDL(b200moe::kPdlGather, b200moe::gather_rows_kernel, dim3(static_cast<int>(blocks)), dim3(256), 0, s,
      static_cast<const __nv_bfloat16 *>(x), x_rows, hidden, row_route, token_of_route, top_k,
      num_routes, row_capacity, counters, static_cast<__nv_bfloat16 *>(x_packed));
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // extern "C"
