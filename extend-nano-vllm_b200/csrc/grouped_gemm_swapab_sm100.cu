// Grouped expert GEMMs on tcgen05 with the expert's weight rows as the MMA M
// operand ("swap AB"): D^T[feature, row] = W[feature, :] . X[row, :].
//
// Why: an expert owns an arbitrary number of packed rows.  With rows as the
// 128-row M operand, an expert with 320 rows runs 3 full 128-row tiles (83%
// useful) and decode-sized experts (1-32 rows) drag a 16 KB activation tile
// through every pipeline stage.  Here the rows are the N operand: N is a
// runtime field of the instruction descriptor, rounded up to 16, and the rows
// arrive as 16-row TMA boxes, so each stage carries the weight tile(s) plus
// only the rows that exist.
//
// Work item = (128-row tile of one expert, 128-feature block).  The tile list
// comes from b200moe_pack_routes on the device.  Warp 0: TMA producer (W tile
// 128 x 64 per projection, row boxes 16 x 64, 128-byte swizzle) into an
// mbarrier ring.  Warp 1: tcgen05.mma M=128, N=round16(rows), K=16 into one of
// two TMEM accumulators.  Warps 2-5: epilogue (TMEM lane = feature, column =
// row), gate/up -> SwiGLU with the reference's bf16 rounding points (moe.py:
// 742-746, 853-854), down -> fp32 accumulator x route weight -> bf16 in route
// order (moe.py:129-139).  Reference kernel replaced: the Triton
// _grouped_moe_gemm_kernel, nanovllm/layers/moe.py:63-139.
// Every wait is bounded; on expiry the CTA records a status bit, leaves its
// loops and frees TMEM.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace b200moe {
namespace tcg {
int make_map(CUtensorMap *map, const void *base, int rank, const uint64_t *dims,
             const uint64_t *strides_bytes, const uint32_t *box);
}  // namespace tcg

namespace tcs {

constexpr int FM = 128;    // features per work item (MMA M)
constexpr int NMAX = 128;  // rows per work item (largest MMA N)
constexpr int BK = 64;
constexpr int BOX_ROWS = 16;
constexpr int W_BYTES = FM * BK * 2;
constexpr int X_BYTES = NMAX * BK * 2;
constexpr int BOX_BYTES = BOX_ROWS * BK * 2;
constexpr int EPI_GROUPS = 2;                 // epilogue warp groups (4 warps each)
constexpr int THREADS = 64 + 128 * EPI_GROUPS;  // producer, MMA, epilogue

template <bool kGateUp>
struct Cfg {
  static constexpr int NW = kGateUp ? 2 : 1;  // weight tiles per stage (gate + up)
  static constexpr int STAGE_BYTES = NW * W_BYTES + X_BYTES;
  static constexpr int STAGES = (200 * 1024 / STAGE_BYTES) < 8 ? (200 * 1024 / STAGE_BYTES) : 8;
  static constexpr int ACC_COLS = kGateUp ? 2 * NMAX : NMAX;  // one accumulator buffer
  static constexpr int TMEM_COLS = 2 * ACC_COLS;
  static constexpr size_t SMEM_BYTES = 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + 2048;
};

struct Args {
  const int32_t *mtiles;
  const int32_t *counters;
  int64_t max_mtiles;
  int n_blocks;  // 128-feature blocks: ceil(I / 128) or ceil(H / 128)
  int num_kb;    // K blocks of 64
  int n_out;     // output features: I (gate/up) or H (down)
  __nv_bfloat16 *out;
  const int32_t *row_route;
  const __nv_bfloat16 *route_w;
  int64_t num_routes;
  // gate/up only: gather the routed rows from the token matrix (map with a
  // one-row box) instead of 16-row boxes of a packed copy.
  int gather;
  const int32_t *token_of_route;
  int top_k;
  int64_t x_rows;
  // down only: rows to other buffers instead of out (ranks == 0: out).
  RowScatter scatter;
};

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(128 * EPI_GROUPS) : "memory");
}

template <bool kGateUp>
__global__ void __launch_bounds__(THREADS, 1)
    swapab_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ Args args) {
  using C = Cfg<kGateUp>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  // Stage s: [W gate (or W) 16 KB][W up 16 KB, gate/up only][rows 16 KB].
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * C::STAGE_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *acc_full = bars + 2 * STAGES;
  uint64_t *acc_empty = bars + 2 * STAGES + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  int32_t *s_route = reinterpret_cast<int32_t *>(tmem_holder + 4);  // [NMAX]
  float *s_w = reinterpret_cast<float *>(s_route + NMAX);           // [NMAX]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), 4 * EPI_GROUPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // The prologue above overlaps the previous kernel; the m-tile list and the
  // operands are its outputs.
  pdl_wait();
  const int num_mtiles =
      static_cast<int>(min64(args.counters[B200MOE_CNT_MTILES], args.max_mtiles));
  const int num_work = num_mtiles * args.n_blocks;

  if (warp == 0) {
    // ---------------- TMA producer (warp 0) ----------------
    // Lane 0 waits, arms the stage and loads the weight tile(s) (and the rows
    // of a packed copy); when gathering, lane l loads routed rows 4l..4l+3.
    const bool gather = kGateUp && args.gather != 0;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < num_work && ok; w += gridDim.x) {
      const int m = w / args.n_blocks;
      const int fb = w - m * args.n_blocks;
      const int e = args.mtiles[m * B200MOE_MTILE_WORDS + 0];
      const int rb = args.mtiles[m * B200MOE_MTILE_WORDS + 1];
      const int re = args.mtiles[m * B200MOE_MTILE_WORDS + 2];
      const int nbox = (re - rb + BOX_ROWS - 1) / BOX_ROWS;
      const uint32_t bytes = C::NW * W_BYTES + nbox * BOX_BYTES;
      const bool my_rows = gather && lane < nbox * (BOX_ROWS / 4);
      int tok[4] = {0, 0, 0, 0};
      if (my_rows) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tok[j] = gather_token(rb + 4 * lane + j, re, args.row_route, args.token_of_route,
                                args.top_k, args.num_routes, args.x_rows);
      }
      for (int kb = 0; kb < args.num_kb; ++kb) {
        bool got = true;
        if (lane == 0) got = mbar_wait_bounded(smem_u32(&empty[stage]), phase ^ 1, abort_flag);
        if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) {
          ok = false;
          break;
        }
        uint8_t *st = smem + stage * C::STAGE_BYTES;
        const uint32_t fbar = smem_u32(&full[stage]);
        uint8_t *sx = st + C::NW * W_BYTES;
        if (my_rows)
          tma_gather4(smem_u32(sx + lane * 4 * BK * 2), &tmX, fbar, kb * BK, tok[0], tok[1],
                      tok[2], tok[3]);
        if (lane == 0) {
          mbar_arrive_expect_tx(fbar, bytes);
          if (kGateUp) {
            tma_load_3d(smem_u32(st), &tmW, fbar, kb * BK, fb * FM, 2 * e);
            tma_load_3d(smem_u32(st + W_BYTES), &tmW, fbar, kb * BK, fb * FM, 2 * e + 1);
          } else {
            tma_load_3d(smem_u32(st), &tmW, fbar, kb * BK, fb * FM, e);
          }
          if (!gather)
            for (int b = 0; b < nbox; ++b)
              tma_load_2d(smem_u32(sx + b * BOX_BYTES), &tmX, fbar, kb * BK, rb + b * BOX_ROWS);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_work && ok; w += gridDim.x) {
        const int m = w / args.n_blocks;
        const int rb = args.mtiles[m * B200MOE_MTILE_WORDS + 1];
        const int re = args.mtiles[m * B200MOE_MTILE_WORDS + 2];
        const int n_mma = (re - rb + BOX_ROWS - 1) / BOX_ROWS * BOX_ROWS;
        const uint32_t idesc = idesc_bf16_f32(FM, n_mma);
        if (!mbar_wait_bounded(smem_u32(&acc_empty[acc]), acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d0 = tmem_base + static_cast<uint32_t>(acc * C::ACC_COLS);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&full[stage]), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sx = st + C::NW * W_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t accum = (kb | kk) != 0 ? 1u : 0u;
            const uint64_t xd = sw128_kmajor_desc(sx + kk * 32);
            tc_mma_f16(d0, sw128_kmajor_desc(st + kk * 32), xd, idesc, accum);
            if (kGateUp)
              tc_mma_f16(d0 + NMAX, sw128_kmajor_desc(st + W_BYTES + kk * 32), xd, idesc, accum);
          }
          tc_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(&acc_full[acc]));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..) ----------------
    const int q = warp & 3;  // TMEM lane quarter = 32 features
    const int et = threadIdx.x - 64;  // index among the epilogue threads
    const int grp = (warp - 2) >> 2;  // group g takes column chunks g, g + G, ...
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int w = blockIdx.x; w < num_work; w += gridDim.x) {
      const int m = w / args.n_blocks;
      const int fb = w - m * args.n_blocks;
      const int rb = args.mtiles[m * B200MOE_MTILE_WORDS + 1];
      const int re = args.mtiles[m * B200MOE_MTILE_WORDS + 2];
      const int rows = re - rb;
      const int n_mma = (rows + BOX_ROWS - 1) / BOX_ROWS * BOX_ROWS;
      if (!kGateUp) {
        // Route id and weight of every row of this tile.
        epi_bar();
        if (et < rows) {
          int32_t r = args.row_route[rb + et];
          if (r < 0 || r >= args.num_routes) {
            atomicOr(&g_status, kStatusIndex);
            r = -1;
          }
          s_w[et] = r >= 0 ? __bfloat162float(args.route_w[r]) : 0.f;
          if (r >= 0 && args.scatter.ranks != 0) {
            const int d = args.scatter.rank[r];
            const int64_t row = args.scatter.row[r];
            if (d < 0 || d >= args.scatter.ranks || row < 0 || row >= args.scatter.rows ||
                row > 0xffffff) {
              atomicOr(&g_status, kStatusIndex);
              r = -1;
            } else {
              r = (d << 24) | static_cast<int32_t>(row);
            }
          }
          s_route[et] = r;
        }
        epi_bar();
      }
      if (!mbar_wait_bounded(smem_u32(&acc_full[acc]), acc_phase, abort_flag)) break;
      tc_fence_after();
      const int f = fb * FM + q * 32 + lane;  // this thread's output feature
      const bool fvalid = f < args.n_out;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(acc * C::ACC_COLS);
#pragma unroll 1
      for (int c = 16 * grp; c < n_mma; c += 16 * EPI_GROUPS) {
        if (kGateUp) {
          float g[16], u[16];
          tmem_ld16(taddr + c, g);
          tmem_ld16(taddr + NMAX + c, u);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c + i;
            if (fvalid && n < rows)
              args.out[static_cast<int64_t>(rb + n) * args.n_out + f] =
                  __float2bfloat16_rn(swiglu_bf16(g[i], u[i]));
          }
        } else {
          float v[16];
          tmem_ld16(taddr + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c + i;
            if (fvalid && n < rows) {
              const int32_t r = s_route[n];
              if (r >= 0) {
                // Scattering: s_route holds rank << 24 | row (checked when
                // the tile's routes were read).
                __nv_bfloat16 *dst =
                    args.scatter.ranks == 0
                        ? args.out + static_cast<int64_t>(r) * args.n_out
                        : reinterpret_cast<__nv_bfloat16 *>(args.scatter.base[r >> 24] +
                                                            args.scatter.offset) +
                              static_cast<int64_t>(r & 0xffffff) * args.n_out;
                dst[f] = __float2bfloat16_rn(v[i] * s_w[n]);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc]));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <bool kGateUp>
int launch(const CUtensorMap &mw, const CUtensorMap &mx, const Args &args, cudaStream_t s) {
  static bool done[64] = {false};
  const int dev = current_device();
  if (!(dev >= 0 && dev < 64 && done[dev])) {
    B200_CUDA(cudaFuncSetAttribute(swapab_kernel<kGateUp>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(Cfg<kGateUp>::SMEM_BYTES)));
    if (dev >= 0 && dev < 64) done[dev] = true;
  }
  const int64_t work = args.max_mtiles * args.n_blocks;
  int grid = sm_count();
  if (work < grid) grid = static_cast<int>(work);
  if (grid < 1) grid = 1;
  B200_LAUNCH_PDL(kPdlTcgen05, swapab_kernel<kGateUp>, dim3(grid), dim3(THREADS), Cfg<kGateUp>::SMEM_BYTES, s,
                  mw, mx, args);
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // namespace tcs

int tcs_gate_up(const RowSource &src, int hidden, int inter, const void *w13, int num_local,
                int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
                const int32_t *counters, void *act, cudaStream_t s) {
  using namespace tcs;
  CUtensorMap mw, mx;
  // W13 [E, 2I, H] as [2E][I][H]: gate rows of expert e are slab 2e, up rows 2e+1.
  const uint64_t dw[3] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(inter),
                          static_cast<uint64_t>(2) * num_local};
  const uint64_t sw[2] = {static_cast<uint64_t>(hidden) * 2,
                          static_cast<uint64_t>(inter) * hidden * 2};
  const uint32_t bw[3] = {BK, FM, 1};
  int rc = tcg::make_map(&mw, w13, 3, dw, sw, bw);
  if (rc) return rc;
  // Packed copy: 16-row boxes.  Token matrix: one-row boxes for gather4.
  const bool gather = src.x_packed == nullptr;
  const uint64_t dx[2] = {static_cast<uint64_t>(hidden),
                          static_cast<uint64_t>(gather ? src.x_rows : row_capacity)};
  const uint64_t sx[1] = {static_cast<uint64_t>(hidden) * 2};
  const uint32_t bx[2] = {BK, gather ? 1u : static_cast<uint32_t>(BOX_ROWS)};
  rc = tcg::make_map(&mx, gather ? src.x : src.x_packed, 2, dx, sx, bx);
  if (rc) return rc;
  Args a;
  a.mtiles = mtiles;
  a.counters = counters;
  a.max_mtiles = max_mtiles;
  a.n_blocks = (inter + FM - 1) / FM;
  a.num_kb = (hidden + BK - 1) / BK;
  a.n_out = inter;
  a.out = static_cast<__nv_bfloat16 *>(act);
  a.row_route = src.row_route;
  a.route_w = nullptr;
  a.num_routes = src.num_routes;
  a.gather = gather ? 1 : 0;
  a.token_of_route = src.token_of_route;
  a.top_k = src.top_k;
  a.x_rows = src.x_rows;
  return launch<true>(mw, mx, a, s);
}

int tcs_down(const void *act, int hidden, int inter, const void *w2, int num_local,
             const int32_t *row_route, const void *route_weights, int64_t num_routes,
             int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
             const int32_t *counters, void *y, const RowScatter *scatter, cudaStream_t s) {
  using namespace tcs;
  CUtensorMap mw, mx;
  const uint64_t dw[3] = {static_cast<uint64_t>(inter), static_cast<uint64_t>(hidden),
                          static_cast<uint64_t>(num_local)};
  const uint64_t sw[2] = {static_cast<uint64_t>(inter) * 2,
                          static_cast<uint64_t>(hidden) * inter * 2};
  const uint32_t bw[3] = {BK, FM, 1};
  int rc = tcg::make_map(&mw, w2, 3, dw, sw, bw);
  if (rc) return rc;
  const uint64_t dx[2] = {static_cast<uint64_t>(inter), static_cast<uint64_t>(row_capacity)};
  const uint64_t sx[1] = {static_cast<uint64_t>(inter) * 2};
  const uint32_t bx[2] = {BK, BOX_ROWS};
  rc = tcg::make_map(&mx, act, 2, dx, sx, bx);
  if (rc) return rc;
  Args a;
  a.mtiles = mtiles;
  a.counters = counters;
  a.max_mtiles = max_mtiles;
  a.n_blocks = (hidden + FM - 1) / FM;
  a.num_kb = (inter + BK - 1) / BK;
  a.n_out = hidden;
  a.out = static_cast<__nv_bfloat16 *>(y);
  a.row_route = row_route;
  a.route_w = static_cast<const __nv_bfloat16 *>(route_weights);
  a.num_routes = num_routes;
  a.gather = 0;
  a.token_of_route = nullptr;
  a.top_k = 1;
  a.x_rows = 0;
  if (scatter) a.scatter = *scatter;
  return launch<false>(mw, mx, a, s);
}

}  // namespace b200moe
