// Shared helpers for the b200moe kernels: argument checking, the thread-local
// error message, bf16 conversion, warp reductions, and the PTX wrappers for
// mbarriers, TMA and tcgen05 used by the sm_100a grouped GEMM.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b200moe.h"

namespace b200moe {

void set_error(const char *fmt, ...);
int sm_count();                    // SMs of the current device
int current_device();
// Kernel families whose launches use programmatic dependent launch; the
// B200MOE_PDL environment variable (read once) holds the enabled mask,
// default all.  "0" turns programmatic launch off everywhere.
enum PdlFamily : unsigned {
  kPdlRoute = 1u,
  kPdlPack = 2u,
  kPdlGather = 4u,
  kPdlCombine = 8u,
  kPdlStream = 16u,
  kPdlTiny = 32u,
  kPdlTcgen05 = 64u,
  kPdlExchange = 128u,
};
bool pdl_enabled(unsigned family);
// Device-side sticky status word (bit 0: bounded wait gave up, bit 1: index
// out of range).  Kernels OR bits into it; the host reads it through
// b200moe_device_status.
extern __device__ int g_status;
constexpr int kStatusTimeout = 1;
constexpr int kStatusIndex = 2;

}  // namespace b200moe

#define B200_ARG(cond, ...)                  \
  do {                                       \
    if (!(cond)) {                           \
      b200moe::set_error(__VA_ARGS__);       \
      return B200MOE_EINVAL;                 \
    }                                        \
  } while (0)

#define B200_UNSUPPORTED(cond, ...)          \
  do {                                       \
    if (!(cond)) {                           \
      b200moe::set_error(__VA_ARGS__);       \
      return B200MOE_EUNSUPPORTED;           \
    }                                        \
  } while (0)

#define B200_CUDA(call)                                                        \
  do {                                                                         \
    cudaError_t err_ = (call);                                                 \
    if (err_ != cudaSuccess) {                                                 \
      b200moe::set_error("%s failed: %s", #call, cudaGetErrorString(err_));   \
      return B200MOE_ECUDA;                                                    \
    }                                                                          \
  } while (0)

#define B200_LAUNCHED() B200_CUDA(cudaGetLastError())
#define B200_LAUNCH_PDL(...) B200_CUDA(b200moe::launch_pdl(__VA_ARGS__))

namespace b200moe {

// Programmatic dependent launch: every hot-path kernel lets the next kernel in
// its stream start launching at once (pdl_trigger) and waits for the previous
// kernel's results (pdl_wait) before reading them, so launches and prologues
// overlap the tail of the predecessor.  Both are no-ops when the kernel was
// launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(unsigned family, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                       size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled(family) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// silu as torch computes it for a bf16 input: x / (1 + exp(-x)) in fp32.
__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + expf(-x)); }

// SwiGLU with the reference's bf16 rounding points:
// gate and up are stored in bf16, F.silu(gate) rounds to bf16, and the
// product of two bf16 tensors rounds to bf16.
__device__ __forceinline__ float swiglu_bf16(float g_acc, float u_acc) {
  const float g = bf16_round(g_acc);
  const float u = bf16_round(u_acc);
  const float s = bf16_round(silu_f32(g));
  return s * u;  // rounded by the caller's bf16 store
}

__device__ __forceinline__ void dot8_bf16(const uint4 &w, const uint4 &x, float &acc) {
  const __nv_bfloat162 *wp = reinterpret_cast<const __nv_bfloat162 *>(&w);
  const __nv_bfloat162 *xp = reinterpret_cast<const __nv_bfloat162 *>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 wf = __bfloat1622float2(wp[i]);
    const float2 xf = __bfloat1622float2(xp[i]);
    acc = fmaf(wf.x, xf.x, acc);
    acc = fmaf(wf.y, xf.y, acc);
  }
}

// ----------------------------------------------------------------------------
// Shared-memory address helpers and mbarriers.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit_ns` of global time, records the timeout
// in the sticky status word and sets *abort so every role of the CTA leaves
// its loop.  Returns false when it gave up (or another role already did).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile int *abort,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (*abort) return false;
      if (global_timer_ns() - start > limit_ns) {
        *abort = 1;
        atomicOr(&g_status, kStatusTimeout);
        return false;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) loads into shared memory, completing on an
// mbarrier.  No multicast: every CTA loads its own tiles.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Where a gate/up GEMM reads its routed rows: a packed copy (x_packed, row p
// of the packed layout) or, when x_packed is null, the token matrix x through
// row_route and token_of_route (or route / top_k).
struct RowSource {
  const void *x;
  int64_t x_rows;
  const void *x_packed;
  const int32_t *row_route;
  const int32_t *token_of_route;
  int top_k;
  int64_t num_routes;
};

// Where a down projection writes its route rows when they do not go to y in
// route order: route r's row (n_out bf16 values) goes to buffer base[rank[r]]
// at byte offset `offset`, row row[r] (row < rows).  The expert-parallel
// exchange uses it to write each received route's result straight into its
// source's return buffer (peer memory) from the GEMM epilogue.  ranks == 0:
// rows go to y.
constexpr int kMaxScatterRanks = 16;
struct RowScatter {
  uint64_t base[kMaxScatterRanks];
  const int32_t *rank = nullptr;
  const int32_t *row = nullptr;
  int64_t offset = 0;
  int64_t rows = 0;
  int ranks = 0;
};

// The destination row of route r under `sc` (null when out of range, which
// sets the status word), or y's row r when scattering is off.
__device__ __forceinline__ __nv_bfloat16 *scatter_row(const RowScatter &sc, __nv_bfloat16 *y,
                                                      int64_t r, int n_out) {
  if (sc.ranks == 0) return y + r * n_out;
  const int d = sc.rank[r];
  const int64_t row = sc.row[r];
  if (d < 0 || d >= sc.ranks || row < 0 || row >= sc.rows) {
    atomicOr(&g_status, kStatusIndex);
    return nullptr;
  }
  return reinterpret_cast<__nv_bfloat16 *>(sc.base[d] + sc.offset) + row * n_out;
}

// Four rows r0..r3 (64 columns from c0) of a 2-D tensor whose map has a
// one-row box, written as consecutive 128-byte rows at dst (swizzled like a
// tile load).  Used to read routed rows of the token matrix directly.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int c0, int r0, int r1, int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(r0), "r"(r1), "r"(r2),
      "r"(r3)
      : "memory");
}

// Token row of packed row p for a gathering producer: row_route maps p to a
// route, the route to its token (token_of_route, else route / top_k).  Rows
// without a route (padding, past the tile) read token 0; their results are
// never stored.
__device__ __forceinline__ int gather_token(int64_t p, int64_t row_end, const int32_t *row_route,
                                            const int32_t *token_of_route, int top_k,
                                            int64_t num_routes, int64_t x_rows) {
  if (p >= row_end) return 0;
  const int32_t r = row_route[p];
  if (r < 0 || r >= num_routes) return 0;
  const int64_t t = token_of_route ? static_cast<int64_t>(token_of_route[r]) : r / top_k;
  if (t < 0 || t >= x_rows) {
    atomicOr(&g_status, kStatusIndex);
    return 0;
  }
  return static_cast<int>(t);
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------------------------
// tcgen05 (5th generation tensor core) wrappers.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t holder_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   holder_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05 op of this
// thread has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand written by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row core groups 1024 bytes apart.
// Fields: start address >> 4 (bits 0-13), leading byte offset >> 4 (16-29,
// unused for swizzled K-major, set to 1), stride byte offset >> 4 (32-45),
// descriptor version 1 (46-47), layout type 2 = 128B swizzle (61-63).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), bf16 A
// and B (bits 7-9 and 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at
// bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

}  // namespace b200moe
