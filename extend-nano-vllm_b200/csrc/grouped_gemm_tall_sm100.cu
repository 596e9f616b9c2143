// Grouped expert GEMMs on tcgen05 with 256-row work tiles (engine TCGEN05_TALL).
//
// Replaces the reference Triton _grouped_moe_gemm_kernel (nanovllm/layers/
// moe.py:63-139) and the separate SwiGLU (moe.py:853-854) for prefill-sized
// calls, like the wide engine (grouped_gemm_sm100.cu), with one change in the
// tile shape.  A tcgen05 tile of 128 routed rows x 256 weight columns stages
// 48 KB of operands per 64-deep K block for 2.1 M multiply-adds, and the rate
// at which an SM fills its shared memory, not the MMA, sets the pace.  Here a
// work item is 256 routed rows of one expert (two consecutive 128-row tiles of
// the packing call's list) x 256 weight columns: every K stage loads both row
// halves (2 x 16 KB) and ONE weight tile (32 KB) that two M=128 MMAs share,
// 64 KB for 4.2 M multiply-adds -- a third fewer bytes per MAC.  An expert's
// last tile without a second half skips that half's load and MMA, so no more
// rows are computed than with 128-row tiles.
//
// Roles: warp 0 issues the TMA loads into a 3-stage mbarrier ring; warp 1
// issues tcgen05.mma M=128 N=256 K=16 into two TMEM accumulators (the two
// row halves, 256 fp32 columns each); epilogue group g (4 warps) drains half g
// with tcgen05.ld: SwiGLU with the reference's bf16 rounding points (gate/up,
// act in packed order) or the route-weight scale before the bf16 store (down,
// route-order rows, staged through shared memory so each store writes whole
// 64-byte row segments).  The accumulators are single-buffered: the next
// tile's MMAs start once both groups drained theirs.
// The 256-row work list is built by every CTA in shared memory from the
// 128-row tiles: a tile starts a work item when its number inside its expert
// is even.
// Every mbarrier wait is bounded (2 s); on expiry the CTA records the timeout
// in the status word, all roles leave their loops and TMEM is released.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace b200moe {
namespace tcg {
int make_map(CUtensorMap *map, const void *base, int rank, const uint64_t *dims,
             const uint64_t *strides_bytes, const uint32_t *box);
}  // namespace tcg

namespace tct {

constexpr int BM = 128;                 // rows per half
constexpr int BN = 256;                 // weight columns per tile
constexpr int BK = 64;                  // K per stage (one 128-byte swizzled row)
constexpr int A_BYTES = BM * BK * 2;    // 16 KB per half
constexpr int B_BYTES = BN * BK * 2;    // 32 KB
constexpr int STAGE_BYTES = 2 * A_BYTES + B_BYTES;  // 64 KB
constexpr int STAGES = 3;
constexpr int TMEM_COLS = 2 * BN;       // two halves
constexpr int EPI_GROUPS = 2;
constexpr int THREADS = 64 + 128 * EPI_GROUPS;
constexpr int EPI_STAGE_WARP_BYTES = 32 * 32 * 2;  // down: 32 rows x 32 columns per warp
// Largest 128-row tile list the in-shared-memory work list holds (the down
// kernel's shared memory then totals 230,656 bytes).
constexpr int MAX_MTILES = 4096;

__host__ __device__ constexpr size_t smem_bytes(bool gate_up, int64_t max_mtiles) {
  return 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + 256 +
         (gate_up ? 0 : static_cast<size_t>(4 * EPI_GROUPS) * EPI_STAGE_WARP_BYTES) +
         static_cast<size_t>(max_mtiles < 1 ? 1 : max_mtiles) * 4;
}

struct Args {
  const int32_t *mtiles;
  const int32_t *counters;
  int64_t max_mtiles;
  int n_tiles;  // 256-column tiles of the output
  int num_kb;   // K blocks of 64
  int n_out;    // output columns: I (gate/up) or H (down)
  __nv_bfloat16 *out;
  const int32_t *row_route;
  const __nv_bfloat16 *route_w;
  int64_t num_routes;
};

__device__ __forceinline__ void store16(__nv_bfloat16 *dst, const float (&v)[16], int valid) {
  if (valid >= 16) {
    uint4 o[2];
    __nv_bfloat162 *op = reinterpret_cast<__nv_bfloat162 *>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i) op[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    reinterpret_cast<uint4 *>(dst)[0] = o[0];
    reinterpret_cast<uint4 *>(dst)[1] = o[1];
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < valid) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

// Waits for this thread's TMEM loads; the destination registers are tied to
// the wait so no use of them is scheduled before it.
__device__ __forceinline__ void wait_into(float (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]),
                 "+f"(v[6]), "+f"(v[7]), "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]),
                 "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15])
               :
               : "memory");
}
__device__ __forceinline__ void tie(float (&v)[16]) {
  asm volatile(""
               : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]),
                 "+f"(v[6]), "+f"(v[7]), "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]),
                 "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15])
               :
               : "memory");
}

// Block-wide exclusive scan (sum or max) of one value per thread; `scratch`
// holds a word per warp plus the total.  All threads call it.
template <bool kMax>
__device__ int block_exclusive_scan(int v, int identity, int32_t *scratch, int *total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl = kMax ? max(incl, u) : incl + u;
  }
  int excl = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) excl = identity;
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = identity;
    for (int w = 0; w < nw; ++w) {
      const int c = scratch[w];
      scratch[w] = acc;
      acc = kMax ? max(acc, c) : acc + c;
    }
    scratch[nw] = acc;
  }
  __syncthreads();
  const int base = scratch[warp];
  *total = scratch[nw];
  __syncthreads();
  return kMax ? max(base, excl) : base + excl;
}

// Work list: indices of the 128-row tiles that start a 256-row item -- the
// even-numbered tiles of each expert (tiles of an expert are consecutive in
// the list) -- compacted in tile order.  A tile's number inside its expert is
// its index minus the index of the expert's first tile, found with a
// block-wide max-scan.  All threads of the CTA call it; returns the number
// of items.
__device__ int build_work_list(const Args &a, int num_mtiles, int32_t *list, int32_t *scratch) {
  const int per = (num_mtiles + blockDim.x - 1) / blockDim.x;
  const int m0 = threadIdx.x * per;
  const int m1 = min(num_mtiles, m0 + per);
  auto expert_of = [&](int m) { return a.mtiles[m * B200MOE_MTILE_WORDS + 0]; };
  // Index of the latest expert start within this thread's range (or -1).
  int last_start = -1;
  for (int m = m0; m < m1; ++m)
    if (m == 0 || expert_of(m - 1) != expert_of(m)) last_start = m;
  int total = 0;
  const int carry = block_exclusive_scan<true>(last_start, -1, scratch, &total);
  int first = carry;
  int count = 0;
  for (int m = m0; m < m1; ++m) {
    if (m == 0 || expert_of(m - 1) != expert_of(m)) first = m;
    count += ((m - first) & 1) == 0;
  }
  int pos = block_exclusive_scan<false>(count, 0, scratch, &total);
  first = carry;
  for (int m = m0; m < m1; ++m) {
    if (m == 0 || expert_of(m - 1) != expert_of(m)) first = m;
    if (((m - first) & 1) == 0) list[pos++] = m;
  }
  __syncthreads();
  return total;
}

template <bool kGateUp>
__global__ void __launch_bounds__(THREADS, 1)
    tall_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  // Stage s: [A half 0][A half 1][B], 1 KB aligned.
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *acc_full = bars + 2 * STAGES;
  uint64_t *acc_empty = bars + 2 * STAGES + 1;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  int32_t *scan_scratch = reinterpret_cast<int32_t *>(tmem_holder + 2);  // 16 words
  uint8_t *epi_stage = smem + STAGES * STAGE_BYTES + 256;
  int32_t *work = reinterpret_cast<int32_t *>(
      epi_stage + (kGateUp ? 0 : 4 * EPI_GROUPS * EPI_STAGE_WARP_BYTES));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(acc_full), 1);
    mbar_init(smem_u32(acc_empty), 4 * EPI_GROUPS);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // The tile list and the operands are outputs of the previous kernels.
  pdl_wait();
  const int num_mtiles = static_cast<int>(
      min64(min64(args.counters[B200MOE_CNT_MTILES], args.max_mtiles), MAX_MTILES));
  const int num_items = build_work_list(args, num_mtiles, work, scan_scratch);
  const int num_work = num_items * args.n_tiles;

  // Rows [rb, rb + 128) of half 0 and [rb + 128, re1) of half 1 (if any).
  auto item = [&](int s, int &e, int &rb, int &re0, int &re1) {
    const int m = work[s];
    e = args.mtiles[m * B200MOE_MTILE_WORDS + 0];
    rb = args.mtiles[m * B200MOE_MTILE_WORDS + 1];
    re0 = args.mtiles[m * B200MOE_MTILE_WORDS + 2];
    re1 = rb + BM;  // empty second half
    if (m + 1 < num_mtiles && args.mtiles[(m + 1) * B200MOE_MTILE_WORDS + 0] == e &&
        args.mtiles[(m + 1) * B200MOE_MTILE_WORDS + 1] == rb + BM)
      re1 = args.mtiles[(m + 1) * B200MOE_MTILE_WORDS + 2];
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_work && ok; w += gridDim.x) {
        const int s = w / args.n_tiles;
        const int n = w - s * args.n_tiles;
        int e, rb, re0, re1;
        item(s, e, rb, re0, re1);
        const bool two = re1 > rb + BM;
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&empty[stage]), phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *st = smem + stage * STAGE_BYTES;
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, two ? STAGE_BYTES : STAGE_BYTES - A_BYTES);
          tma_load_2d(smem_u32(st), &tmA, fb, kb * BK, rb);
          if (two) tma_load_2d(smem_u32(st + A_BYTES), &tmA, fb, kb * BK, rb + BM);
          uint8_t *sb = st + 2 * A_BYTES;
          if (kGateUp) {
            tma_load_3d(smem_u32(sb), &tmB, fb, kb * BK, n * (BN / 2), 2 * e);
            tma_load_3d(smem_u32(sb + B_BYTES / 2), &tmB, fb, kb * BK, n * (BN / 2), 2 * e + 1);
          } else {
            tma_load_3d(smem_u32(sb), &tmB, fb, kb * BK, n * BN, e);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_work && ok; w += gridDim.x) {
        const int s = w / args.n_tiles;
        int e, rb, re0, re1;
        item(s, e, rb, re0, re1);
        const bool two = re1 > rb + BM;
        if (!mbar_wait_bounded(smem_u32(acc_empty), acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&full[stage]), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b0 = a0 + 2 * A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bd = sw128_kmajor_desc(b0 + kk * 32);
            const uint32_t acc = (kb | kk) != 0 ? 1u : 0u;
            tc_mma_f16(tmem_base, sw128_kmajor_desc(a0 + kk * 32), bd, idesc, acc);
            if (two)
              tc_mma_f16(tmem_base + BN, sw128_kmajor_desc(a0 + A_BYTES + kk * 32), bd, idesc,
                         acc);
          }
          tc_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(acc_full));
        acc_phase ^= 1;
      }
    }
  } else {
    // ---------------- epilogue: group g drains row half g ----------------
    const int q = warp & 3;               // TMEM lane quarter this warp may access
    const int grp = (warp - 2) >> 2;
    uint32_t acc_phase = 0;
    for (int w = blockIdx.x; w < num_work; w += gridDim.x) {
      const int s = w / args.n_tiles;
      const int n = w - s * args.n_tiles;
      int e, rb, re0, re1;
      item(s, e, rb, re0, re1);
      const int row_end = grp == 0 ? re0 : re1;
      if (!mbar_wait_bounded(smem_u32(acc_full), acc_phase, abort_flag)) break;
      tc_fence_after();
      const int row = rb + grp * BM + q * 32 + lane;
      const bool valid = row < row_end;
      const bool any_row = rb + grp * BM + q * 32 < row_end;  // warp-uniform
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(grp * BN);
      if (any_row && kGateUp) {
        const int col0 = n * (BN / 2);
        __nv_bfloat16 *dst_row = args.out + static_cast<int64_t>(row) * args.n_out;
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 16) {
          float g[16], u[16];
          tmem_ld16(taddr + c, g);
          tmem_ld16(taddr + BN / 2 + c, u);
          wait_into(g);
          tie(u);
          const int cols = args.n_out - (col0 + c);
          if (valid && cols > 0) {
            float a[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) a[i] = swiglu_bf16(g[i], u[i]);
            store16(dst_row + col0 + c, a, cols);
          }
        }
      } else if (any_row) {
        int32_t route = -1;
        float rw = 0.f;
        if (valid) {
          route = args.row_route[row];
          if (route < 0 || route >= args.num_routes) {
            atomicOr(&g_status, kStatusIndex);
            route = -1;
          } else {
            rw = __bfloat162float(args.route_w[route]);
          }
        }
        const int col0 = n * BN;
        // 32 columns at a time: scaled, rounded to bf16 and written to this
        // warp's staging rows (16-byte slot j of row l at j ^ (l & 3)), then
        // stored eight rows per instruction, four lanes per 64-byte segment.
        uint4 *stage_w = reinterpret_cast<uint4 *>(epi_stage + (warp - 2) * EPI_STAGE_WARP_BYTES);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v0[16], v1[16];
          tmem_ld16(taddr + c, v0);
          tmem_ld16(taddr + c + 16, v1);
          wait_into(v0);
          tie(v1);
#define B200_TALL_STAGE(V, J)                                                            \
  do {                                                                                   \
    uint4 o[2];                                                                          \
    __nv_bfloat162 *op = reinterpret_cast<__nv_bfloat162 *>(o);                          \
    _Pragma("unroll") for (int i = 0; i < 8; ++i)                                        \
        op[i] = __floats2bfloat162_rn(V[2 * i] * rw, V[2 * i + 1] * rw);                 \
    stage_w[lane * 4 + ((J) ^ (lane & 3))] = o[0];                                       \
    stage_w[lane * 4 + (((J) + 1) ^ (lane & 3))] = o[1];                                 \
  } while (0)
          B200_TALL_STAGE(v0, 0);
          B200_TALL_STAGE(v1, 2);
#undef B200_TALL_STAGE
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int r = it * 8 + (lane >> 2);
            const int sl = lane & 3;
            const int r_route = __shfl_sync(0xffffffffu, route, r);
            const uint4 o = stage_w[r * 4 + (sl ^ (r & 3))];
            const int col = col0 + c + sl * 8;
            if (r_route >= 0 && col < args.n_out)
              *reinterpret_cast<uint4 *>(args.out + static_cast<int64_t>(r_route) * args.n_out +
                                         col) = o;
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(acc_empty));
      acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <bool kGateUp>
int launch(const CUtensorMap &ma, const CUtensorMap &mb, const Args &args, cudaStream_t s) {
  static bool prepared[64] = {false};
  const int dev = current_device();
  if (dev < 0 || dev >= 64 || !prepared[dev]) {
    B200_CUDA(cudaFuncSetAttribute(tall_kernel<kGateUp>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem_bytes(kGateUp, MAX_MTILES))));
    if (dev >= 0 && dev < 64) prepared[dev] = true;
  }
  const size_t smem = smem_bytes(kGateUp, args.max_mtiles);
  int64_t work = (args.max_mtiles + 1) / 2 * args.n_tiles;
  int grid = sm_count();
  if (work < grid) grid = static_cast<int>(work);
  if (grid < 1) grid = 1;
  B200_LAUNCH_PDL(kPdlTcgen05, tall_kernel<kGateUp>, dim3(grid), dim3(THREADS), smem, s, ma, mb,
                  args);
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // namespace tct

bool tall_fits(int64_t max_mtiles) { return max_mtiles <= tct::MAX_MTILES; }

int tct_gate_up(const void *x_packed, int hidden, int inter, const void *w13, int num_local,
                int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
                const int32_t *counters, void *act, cudaStream_t s) {
  using namespace tct;
  CUtensorMap ma, mb;
  const uint64_t da[2] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(row_capacity)};
  const uint64_t sa[1] = {static_cast<uint64_t>(hidden) * 2};
  const uint32_t ba[2] = {BK, BM};
  int rc = tcg::make_map(&ma, x_packed, 2, da, sa, ba);
  if (rc) return rc;
  // W13 [E, 2I, H] viewed as [2E][I][H]: gate rows of expert e are slab 2e, up rows 2e+1.
  const uint64_t db[3] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(inter),
                          static_cast<uint64_t>(2) * num_local};
  const uint64_t sb[2] = {static_cast<uint64_t>(hidden) * 2,
                          static_cast<uint64_t>(inter) * hidden * 2};
  const uint32_t bb[3] = {BK, BN / 2, 1};
  rc = tcg::make_map(&mb, w13, 3, db, sb, bb);
  if (rc) return rc;
  Args a;
  a.mtiles = mtiles;
  a.counters = counters;
  a.max_mtiles = max_mtiles;
  a.n_tiles = (inter + BN / 2 - 1) / (BN / 2);
  a.num_kb = (hidden + BK - 1) / BK;
  a.n_out = inter;
  a.out = static_cast<__nv_bfloat16 *>(act);
  a.row_route = nullptr;
  a.route_w = nullptr;
  a.num_routes = 0;
  return launch<true>(ma, mb, a, s);
}

int tct_down(const void *act, int hidden, int inter, const void *w2, int num_local,
             const int32_t *row_route, const void *route_weights, int64_t num_routes,
             int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
             const int32_t *counters, void *y, cudaStream_t s) {
  using namespace tct;
  CUtensorMap ma, mb;
  const uint64_t da[2] = {static_cast<uint64_t>(inter), static_cast<uint64_t>(row_capacity)};
  const uint64_t sa[1] = {static_cast<uint64_t>(inter) * 2};
  const uint32_t ba[2] = {BK, BM};
  int rc = tcg::make_map(&ma, act, 2, da, sa, ba);
  if (rc) return rc;
  const uint64_t db[3] = {static_cast<uint64_t>(inter), static_cast<uint64_t>(hidden),
                          static_cast<uint64_t>(num_local)};
  const uint64_t sb[2] = {static_cast<uint64_t>(inter) * 2,
                          static_cast<uint64_t>(hidden) * inter * 2};
  const uint32_t bb[3] = {BK, BN, 1};
  rc = tcg::make_map(&mb, w2, 3, db, sb, bb);
  if (rc) return rc;
  Args a;
  a.mtiles = mtiles;
  a.counters = counters;
  a.max_mtiles = max_mtiles;
  a.n_tiles = (hidden + BN - 1) / BN;
  a.num_kb = (inter + BK - 1) / BK;
  a.n_out = hidden;
  a.out = static_cast<__nv_bfloat16 *>(y);
  a.row_route = row_route;
  a.route_w = static_cast<const __nv_bfloat16 *>(route_weights);
  a.num_routes = num_routes;
  return launch<false>(ma, mb, a, s);
}

}  // namespace b200moe
