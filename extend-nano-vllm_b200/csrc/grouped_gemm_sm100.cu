// Grouped expert GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM),
// fed by TMA, for prefill and the larger decode buckets (engine TCGEN05).
//
// Replaces the reference Triton _grouped_moe_gemm_kernel
// (nanovllm/layers/moe.py:63-139: one program per 16-row tile x 64 columns,
// K step 32) and the separate SwiGLU (moe.py:853-854).  Design:
//  * Work = (128-row tile of one expert's packed rows) x (256-column tile of
//    its weights).  The tile list comes from b200moe_pack_routes on the device,
//    so inactive experts cost nothing and no host sync is needed; the grid is
//    persistent (one CTA per SM) and walks the list with a static stride.
//  * Warp 0 issues TMA loads (A: 128 x 64 activation rows, B: 256 x 64 weight
//    rows, 128-byte swizzle) into a 4-stage mbarrier ring; warp 1 issues
//    tcgen05.mma (M=128, N=256, K=16) into one of two TMEM accumulators
//    (2 x 256 fp32 columns); warps 2-5 drain the other accumulator with
//    tcgen05.ld and run the epilogue, so the epilogue of tile i overlaps the
//    MMAs of tile i+1.
//  * gate/up: the 256 B rows are 128 gate rows and the matching 128 up rows
//    (two TMA boxes of a [2E, I, H] view of W13), so each thread holds gate
//    and up of the same feature and applies SwiGLU in registers with the
//    reference's bf16 rounding points, writing act in packed order.
//  * down: the epilogue scales the fp32 accumulator by the route weight before
//    the bf16 store (moe.py:129-139) and writes rows in route order.
// Every mbarrier wait is bounded (2 s of global time); on expiry the CTA
// records the timeout in the status word, all roles leave their loops and
// TMEM is released before the kernel returns.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace b200moe {
namespace tcg {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int A_BYTES = BM * BK * 2;
constexpr int EPI_GROUPS = 2;                 // epilogue warp groups (4 warps each)
constexpr int THREADS = 64 + 128 * EPI_GROUPS;  // producer, MMA, epilogue

// Tile configuration for an N tile of BN columns (BN in {128, 256}).
template <int BN>
struct Cfg {
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // As many pipeline stages as fit in ~200 KB of shared memory (at most 8).
  static constexpr int STAGES = (200 * 1024 / STAGE_BYTES) < 8 ? (200 * 1024 / STAGE_BYTES) : 8;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators
  static constexpr size_t SMEM_BYTES = 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + 256;
};

// Down epilogue staging: per epilogue warp, 32 rows x 64 bf16 columns (4 KB),
// so that each global store instruction writes four whole 128-byte row
// segments instead of 32 scattered 16-byte pieces.
constexpr int EPI_STAGE_WARP_BYTES = 32 * 64 * 2;
template <bool kGateUp, int BN>
constexpr size_t kernel_smem_bytes() {
  return Cfg<BN>::SMEM_BYTES +
         (kGateUp ? 0 : static_cast<size_t>(4 * EPI_GROUPS) * EPI_STAGE_WARP_BYTES);
}

struct Args {
  const int32_t *mtiles;
  const int32_t *counters;
  int64_t max_mtiles;
  int n_tiles;  // column tiles per row tile
  int num_kb;   // K blocks of 64
  int n_out;    // output columns: I (gate/up) or H (down)
  __nv_bfloat16 *out;
  const int32_t *row_route;
  const __nv_bfloat16 *route_w;
  int64_t num_routes;
  // gate/up only: gather the A rows from the token matrix (map with a
  // one-row box) instead of loading 128-row boxes of a packed copy.
  int gather;
  const int32_t *token_of_route;
  int top_k;
  int64_t x_rows;
  // down only: rows to other buffers instead of out (ranks == 0: out).
  RowScatter scatter;
};

__device__ __forceinline__ void store16_bf16(__nv_bfloat16 *dst, const float (&v)[16], int valid) {
  if (valid >= 16) {
    uint4 o[2];
    __nv_bfloat162 *op = reinterpret_cast<__nv_bfloat162 *>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i) op[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    reinterpret_cast<uint4 *>(dst)[0] = o[0];
    reinterpret_cast<uint4 *>(dst)[1] = o[1];
  } else {
    // Fully unrolled with a predicate: a loop bounded by `valid` would index
    // v dynamically and move the array to local memory.
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < valid) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

// Waits for this thread's TMEM loads.  The 16 destination registers are tied
// to the wait so that no use of them can be scheduled before it; tie16 does
// the same for a second array after the same wait.
__device__ __forceinline__ void tmem_wait_into(float (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]),
                 "+f"(v[6]), "+f"(v[7]), "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]),
                 "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15])
               :
               : "memory");
}
__device__ __forceinline__ void tie16(float (&v)[16]) {
  asm volatile(""
               : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]),
                 "+f"(v[6]), "+f"(v[7]), "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]),
                 "+f"(v[12]), "+f"(v[13]), "+f"(v[14]), "+f"(v[15])
               :
               : "memory");
}

template <bool kGateUp, int BN>
__global__ void __launch_bounds__(THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ Args args) {
  constexpr int STAGES = Cfg<BN>::STAGES;
  constexpr int B_BYTES = Cfg<BN>::B_BYTES;
  constexpr int STAGE_BYTES = Cfg<BN>::STAGE_BYTES;
  constexpr int TMEM_COLS = Cfg<BN>::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + STAGES * A_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sB + STAGES * B_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *acc_full = bars + 2 * STAGES;
  uint64_t *acc_empty = bars + 2 * STAGES + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  // Down epilogue staging (kernel_smem_bytes reserves it for the down kernel).
  uint8_t *epi_stage = smem + STAGES * STAGE_BYTES + 256;

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
  // The prologue above overlaps the previous kernel; the m-tile list and the
  // operands are its outputs.
  pdl_wait();
  const int num_mtiles =
      static_cast<int>(min64(args.counters[B200MOE_CNT_MTILES], args.max_mtiles));
  const int num_work = num_mtiles * args.n_tiles;

  if (warp == 0) {
    // ---------------- TMA producer (warp 0) ----------------
    // Lane 0 waits, arms the stage and loads B (and A from a packed copy);
    // when gathering, lane l loads A rows 4l..4l+3 of the tile.
    const bool gather = kGateUp && args.gather != 0;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < num_work && ok; w += gridDim.x) {
      const int m = w / args.n_tiles;
      const int n = w - m * args.n_tiles;
      const int e = args.mtiles[m * B200MOE_MTILE_WORDS + 0];
      const int rb = args.mtiles[m * B200MOE_MTILE_WORDS + 1];
      int tok[4] = {0, 0, 0, 0};
      if (gather) {
        const int re = args.mtiles[m * B200MOE_MTILE_WORDS + 2];
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
        const uint32_t fb = smem_u32(&full[stage]);
        if (gather)
          tma_gather4(smem_u32(sA + stage * A_BYTES + lane * 4 * BK * 2), &tmA, fb, kb * BK,
                      tok[0], tok[1], tok[2], tok[3]);
        if (lane == 0) {
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          if (!gather) tma_load_2d(smem_u32(sA + stage * A_BYTES), &tmA, fb, kb * BK, rb);
          if (kGateUp) {
            tma_load_3d(smem_u32(sB + stage * B_BYTES), &tmB, fb, kb * BK, n * (BN / 2), 2 * e);
            tma_load_3d(smem_u32(sB + stage * B_BYTES + B_BYTES / 2), &tmB, fb, kb * BK,
                        n * (BN / 2), 2 * e + 1);
          } else {
            tma_load_3d(smem_u32(sB + stage * B_BYTES), &tmB, fb, kb * BK, n * BN, e);
          }
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
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_work && ok; w += gridDim.x) {
        if (!mbar_wait_bounded(smem_u32(&acc_empty[acc]), acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&full[stage]), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            tc_mma_f16(d_tmem, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32),
                       idesc, (kb | kk) != 0 ? 1u : 0u);
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
    // Each TMEM lane quarter is read by one warp of every group; group g
    // takes the g-th share of the accumulator's columns.
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int grp = (warp - 2) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int w = blockIdx.x; w < num_work; w += gridDim.x) {
      const int m = w / args.n_tiles;
      const int n = w - m * args.n_tiles;
      const int rb = args.mtiles[m * B200MOE_MTILE_WORDS + 1];
      const int re = args.mtiles[m * B200MOE_MTILE_WORDS + 2];
      if (!mbar_wait_bounded(smem_u32(&acc_full[acc]), acc_phase, abort_flag)) break;
      tc_fence_after();
      const int row = rb + q * 32 + lane;
      const bool valid = row < re;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (kGateUp) {
        const int col0 = n * (BN / 2);
        __nv_bfloat16 *dst_row = args.out + static_cast<int64_t>(row) * args.n_out;
        constexpr int kGuCols = BN / 2 / EPI_GROUPS;
#pragma unroll 1
        for (int c = grp * kGuCols; c < (grp + 1) * kGuCols; c += 16) {
          float g[16], u[16];
          tmem_ld16(taddr + c, g);
          tmem_ld16(taddr + BN / 2 + c, u);
          tmem_wait_into(g);
          tie16(u);
          const int cols = args.n_out - (col0 + c);
          if (valid && cols > 0) {
            float a[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) a[i] = swiglu_bf16(g[i], u[i]);
            store16_bf16(dst_row + col0 + c, a, cols);
          }
        }
      } else {
        int32_t route = -1;
        float rw = 0.f;
        __nv_bfloat16 *row_dst = nullptr;
        if (valid) {
          route = args.row_route[row];
          if (route < 0 || route >= args.num_routes) {
            atomicOr(&g_status, kStatusIndex);
            route = -1;
          } else {
            rw = __bfloat162float(args.route_w[route]);
            row_dst = scatter_row(args.scatter, args.out, route, args.n_out);
          }
        }
        const int col0 = n * BN;
        // 64 columns at a time: scaled, rounded to bf16 and written to this
        // warp's staging rows (16-byte slot j of row l at j ^ (l & 7), so
        // neither the writes nor the reads conflict on banks), then stored
        // four rows per instruction, eight lanes per 128-byte row segment.
        uint4 *stage_w = reinterpret_cast<uint4 *>(epi_stage + (warp - 2) * EPI_STAGE_WARP_BYTES);
        constexpr int kDnCols = BN / EPI_GROUPS;  // a multiple of 64
        static_assert(kDnCols % 64 == 0, "down epilogue works on 64-column chunks");
        const int c_begin = grp * kDnCols, c_end = c_begin + kDnCols;
#pragma unroll 1
        for (int c = c_begin; c < c_end; c += 64) {
          float v0[16], v1[16], v2[16], v3[16];
          tmem_ld16(taddr + c, v0);
          tmem_ld16(taddr + c + 16, v1);
          tmem_ld16(taddr + c + 32, v2);
          tmem_ld16(taddr + c + 48, v3);
          tmem_wait_into(v0);
          tie16(v1);
          tie16(v2);
          tie16(v3);
#define B200_STAGE_DOWN(V, J)                                                             \
  do {                                                                                    \
    uint4 o[2];                                                                           \
    __nv_bfloat162 *op = reinterpret_cast<__nv_bfloat162 *>(o);                           \
    _Pragma("unroll") for (int i = 0; i < 8; ++i)                                         \
        op[i] = __floats2bfloat162_rn(V[2 * i] * rw, V[2 * i + 1] * rw);                  \
    stage_w[lane * 8 + ((J) ^ (lane & 7))] = o[0];                                        \
    stage_w[lane * 8 + (((J) + 1) ^ (lane & 7))] = o[1];                                  \
  } while (0)
          B200_STAGE_DOWN(v0, 0);
          B200_STAGE_DOWN(v1, 2);
          B200_STAGE_DOWN(v2, 4);
          B200_STAGE_DOWN(v3, 6);
#undef B200_STAGE_DOWN
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int r = it * 4 + (lane >> 3);
            const int sl = lane & 7;
            auto *r_dst = reinterpret_cast<__nv_bfloat16 *>(__shfl_sync(
                0xffffffffu, reinterpret_cast<unsigned long long>(row_dst), r));
            const uint4 o = stage_w[r * 8 + (sl ^ (r & 7))];
            const int col = col0 + c + sl * 8;
            if (r_dst != nullptr && col < args.n_out)
              *reinterpret_cast<uint4 *>(r_dst + col) = o;
          }
          __syncwarp();
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
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ----------------------------------------------------------------------------
// Host side: tensor maps and launch.
// ----------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_map(CUtensorMap *map, const void *base, int rank, const uint64_t *dims,
             const uint64_t *strides_bytes, const uint32_t *box) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    return B200MOE_ECUDA;
  }
  if (rank < 1 || rank > 5) {
    set_error("tensor map rank %d out of range", rank);
    return B200MOE_EINVAL;
  }
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5];
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
  }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides_bytes[i];
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                        const_cast<void *>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult %d", static_cast<int>(r));
    return B200MOE_ECUDA;
  }
  return B200MOE_OK;
}

template <bool kGateUp, int BN>
int prepare_kernel() {
  static bool done[64] = {false};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && done[dev]) return B200MOE_OK;
  B200_CUDA(cudaFuncSetAttribute(grouped_gemm_kernel<kGateUp, BN>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kernel_smem_bytes<kGateUp, BN>())));
  if (dev >= 0 && dev < 64) done[dev] = true;
  return B200MOE_OK;
}

template <bool kGateUp, int BN>
int launch(const CUtensorMap &ma, const CUtensorMap &mb, const Args &args, cudaStream_t s) {
  int rc = prepare_kernel<kGateUp, BN>();
  if (rc != B200MOE_OK) return rc;
  int64_t work = args.max_mtiles * args.n_tiles;
  int grid = sm_count();
  if (work < grid) grid = static_cast<int>(work);
  if (grid < 1) grid = 1;
  B200_LAUNCH_PDL(kPdlTcgen05, grouped_gemm_kernel<kGateUp, BN>, dim3(grid), dim3(THREADS),
                  kernel_smem_bytes<kGateUp, BN>(), s,
                  ma, mb, args);
  B200_LAUNCHED();
  return B200MOE_OK;
}

}  // namespace tcg

// N tile for a call: wide tiles for prefill-sized route counts, 128 for
// decode buckets so the few active experts still cover every SM.  (64-wide
// tiles measured slower: the 128-row A tile then dominates each stage.)
int pick_bn(int64_t num_routes) {
  if (num_routes > 4096) return 256;
  return 128;
}

template <int BN>
int tc_gate_up_bn(const RowSource &src, int hidden, int inter, const void *w13, int num_local,
                  int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
                  const int32_t *counters, void *act, cudaStream_t s) {
  using namespace tcg;
  CUtensorMap ma, mb;
  const bool gather = src.x_packed == nullptr;
  // Packed copy: 128-row boxes.  Token matrix: one-row boxes for gather4.
  const uint64_t da[2] = {static_cast<uint64_t>(hidden),
                          static_cast<uint64_t>(gather ? src.x_rows : row_capacity)};
  const uint64_t sa[1] = {static_cast<uint64_t>(hidden) * 2};
  const uint32_t ba[2] = {BK, gather ? 1u : static_cast<uint32_t>(BM)};
  int rc = make_map(&ma, gather ? src.x : src.x_packed, 2, da, sa, ba);
  if (rc) return rc;
  // W13 [E, 2I, H] viewed as [2E][I][H]: gate rows of expert e are slab 2e, up rows 2e+1.
  const uint64_t db[3] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(inter),
                          static_cast<uint64_t>(2) * num_local};
  const uint64_t sb[2] = {static_cast<uint64_t>(hidden) * 2,
                          static_cast<uint64_t>(inter) * hidden * 2};
  const uint32_t bb[3] = {BK, BN / 2, 1};
  rc = make_map(&mb, w13, 3, db, sb, bb);
  if (rc) return rc;
  Args a;
  a.mtiles = mtiles;
  a.counters = counters;
  a.max_mtiles = max_mtiles;
  a.n_tiles = (inter + BN / 2 - 1) / (BN / 2);
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
  return launch<true, BN>(ma, mb, a, s);
}

template <int BN>
int tc_down_bn(const void *act, int hidden, int inter, const void *w2, int num_local,
               const int32_t *row_route, const void *route_weights, int64_t num_routes,
               int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
               const int32_t *counters, void *y, const RowScatter *scatter, cudaStream_t s) {
  using namespace tcg;
  CUtensorMap ma, mb;
  const uint64_t da[2] = {static_cast<uint64_t>(inter), static_cast<uint64_t>(row_capacity)};
  const uint64_t sa[1] = {static_cast<uint64_t>(inter) * 2};
  const uint32_t ba[2] = {BK, BM};
  int rc = make_map(&ma, act, 2, da, sa, ba);
  if (rc) return rc;
  const uint64_t db[3] = {static_cast<uint64_t>(inter), static_cast<uint64_t>(hidden),
                          static_cast<uint64_t>(num_local)};
  const uint64_t sb[2] = {static_cast<uint64_t>(inter) * 2,
                          static_cast<uint64_t>(hidden) * inter * 2};
  const uint32_t bb[3] = {BK, BN, 1};
  rc = make_map(&mb, w2, 3, db, sb, bb);
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
  a.gather = 0;
  a.token_of_route = nullptr;
  a.top_k = 1;
  a.x_rows = 0;
  if (scatter) a.scatter = *scatter;
  return launch<false, BN>(ma, mb, a, s);
}

int tc_gate_up(const RowSource &src, int hidden, int inter, const void *w13, int num_local,
               int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
               const int32_t *counters, void *act, cudaStream_t s) {
  switch (pick_bn(src.num_routes)) {
    case 256:
      return tc_gate_up_bn<256>(src, hidden, inter, w13, num_local, row_capacity, mtiles,
                                max_mtiles, counters, act, s);
    case 128:
    default:
      return tc_gate_up_bn<128>(src, hidden, inter, w13, num_local, row_capacity, mtiles,
                                max_mtiles, counters, act, s);
  }
}

int tc_down(const void *act, int hidden, int inter, const void *w2, int num_local,
            const int32_t *row_route, const void *route_weights, int64_t num_routes,
            int64_t row_capacity, const int32_t *mtiles, int64_t max_mtiles,
            const int32_t *counters, void *y, const RowScatter *scatter, cudaStream_t s) {
  switch (pick_bn(num_routes)) {
    case 256:
      return tc_down_bn<256>(act, hidden, inter, w2, num_local, row_route, route_weights,
                             num_routes, row_capacity, mtiles, max_mtiles, counters, y, scatter,
                             s);
    case 128:
    default:
      return tc_down_bn<128>(act, hidden, inter, w2, num_local, row_route, route_weights,
                             num_routes, row_capacity, mtiles, max_mtiles, counters, y, scatter,
                             s);
  }
}

}  // namespace b200moe
