// Grouped expert GEMMs on tcgen05 across an SM pair (cta_group::2) with the
// expert's weight rows as the MMA M operand and its routed rows as N:
//   D^T[w, n] = W[w, :] . X[rb + n, :]
//
// Why: with routed rows as a 128-row M tile, an expert that owns 265 rows
// computes 384 (69% useful).  Here a work item is a row chunk of <= 256 rows
// (b200moe_pack_routes splits every expert into ceil(rows/256) chunks of
// equal 16-row multiples), which becomes the runtime N of the instruction
// descriptor, so padding stays below 16 rows per chunk.  The two CTAs of a
// cluster form one M=256 MMA: each loads 128 weight rows (A) and half of the
// chunk's rows (B) into its own shared memory (the MMA reads the other half
// from the peer), so each CTA stages at most 32 KB per K step for 128 x N x 64
// MACs -- a third less L2-to-SM traffic per MAC than a one-SM 128 x 256 tile.
//
// Work item = (chunk, weight block).  gate/up: 128 features per pair, each CTA
// 64, its A tile interleaving 16 gate and 16 up rows per 32-lane TMEM quarter
// (one 5-D TMA box), so SwiGLU pairs lanes l and l+16 of one warp.  down: 256
// output features per pair, 128 per CTA.
//
// Roles per CTA: warp 0 lane 0 issues the TMA loads of its CTA (both signal
// the leader CTA's full barrier, the leader arms it with the pair's bytes);
// warp 1 lane 0 of the leader issues tcgen05.mma M=256, N=round16(rows), K=16
// into one of two TMEM accumulators (256 fp32 columns each, 512 allocated per
// SM) and commits to the barriers of both CTAs; warps 2-5 of each CTA read their
// 128 TMEM lanes, apply SwiGLU (gate/up, reference rounding points moe.py:
// 742-746, 853-854) or the route-weight scale (down, moe.py:129-139) and store
// bf16, then arrive on the leader's accumulator-empty barrier.
// Reference kernel replaced: _grouped_moe_gemm_kernel, moe.py:63-139.
//
// Every mbarrier wait is bounded; on expiry the CTA records a status bit and
// its roles leave their loops.  Both CTAs meet at a final cluster barrier
// before TMEM is freed, so no CTA exits while its peer may still signal it.
// Every TMA load writes only the issuing CTA's shared memory; the MMA
// completion is signalled to each CTA of the pair by its own commit.
#include <cudaTypedefs.h>

#include "common.cuh"

namespace b200moe {
namespace tcg {
int make_map(CUtensorMap *map, const void *base, int rank, const uint64_t *dims,
             const uint64_t *strides_bytes, const uint32_t *box);
}  // namespace tcg

namespace tcp {

constexpr int BK = 64;                     // K per stage: one 128-byte swizzled row
constexpr int MW = 128;                    // weight rows per CTA (pair M = 256)
constexpr int NMAX = B200MOE_CHUNK_ROWS;   // routed rows per chunk (pair N)
constexpr int HALF_MAX = NMAX / 2;         // routed rows per CTA
constexpr int BIG_ROWS = 64;               // routed rows per large TMA box
constexpr int SMALL_ROWS = 8;              // ... and per small box (8-row swizzle atom)
constexpr int ROW_BYTES = BK * 2;
constexpr int A_BYTES = MW * ROW_BYTES;          // 16 KB
constexpr int B_BYTES = HALF_MAX * ROW_BYTES;    // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;   // 32 KB
constexpr int STAGES = 6;
constexpr int ACC_COLS = NMAX;
constexpr int TMEM_COLS = 2 * ACC_COLS;
constexpr int THREADS = 192;
constexpr int EPI_WARPS = 4;
constexpr size_t SMEM_BYTES = 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + 4096;

struct Args {
  const int32_t *chunks;
  const int32_t *counters;
  int64_t max_chunks;
  int n_blocks;  // weight blocks per chunk: ceil(I / 128) (gate/up) or ceil(H / 256) (down)
  int num_kb;    // K blocks of 64
  int n_out;     // output features: I (gate/up) or H (down)
  __nv_bfloat16 *out;
  const int32_t *row_route;
  const __nv_bfloat16 *route_w;
  int64_t num_routes;
};

// ---- cluster / pair primitives ---------------------------------------------
__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

// TMA tile loads into this CTA's shared memory whose completion is counted on
// `bar`, an mbarrier of either CTA of the pair (cluster address).
__device__ __forceinline__ void tma2_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                          int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma3_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                          int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma5_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                          int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(c4)
      : "memory");
}

// TMEM allocation shared by the pair: one warp of each CTA (same warp id).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t holder_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   holder_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the mbarrier at cluster address `bar` (this CTA's or the
// peer's) when all MMAs issued so far by this thread have completed.
__device__ __forceinline__ void commit_to(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// The same completion signalled to the barrier at local offset `bar` in both
// CTAs of the pair.
__device__ __forceinline__ void commit_pair(uint32_t bar) {
  commit_to(cluster_addr(bar, 0));
  commit_to(cluster_addr(bar, 1));
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// ---- the kernel ----------------------------------------------------------------
template <bool kGateUp>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    pair_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXb,
                const __grid_constant__ CUtensorMap tmXs, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  // Stage s: [A: 128 weight rows x 64][B: up to 128 routed rows x 64].
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *full = bars;                    // leader only: both CTAs' bytes
  uint64_t *empty = bars + STAGES;          // each CTA: MMA done with the stage
  uint64_t *acc_full = bars + 2 * STAGES;   // each CTA: accumulator ready
  uint64_t *acc_empty = bars + 2 * STAGES + 2;  // leader only: both epilogues drained
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  int32_t *s_route = reinterpret_cast<int32_t *>(tmem_holder + 4);  // [NMAX]
  float *s_w = reinterpret_cast<float *>(s_route + NMAX);           // [NMAX]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank_in_cluster();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), 2 * EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmXb);
    prefetch_tmap(&tmXs);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Both CTAs' barriers are initialised before either CTA signals the other.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // The prologue above overlaps the previous kernel; the chunk list and the
  // operands are its outputs.
  pdl_wait();
  const int num_chunks =
      static_cast<int>(min64(args.counters[B200MOE_CNT_CHUNKS], args.max_chunks));
  const int num_work = num_chunks * args.n_blocks;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = pair; w < num_work && ok; w += npairs) {
        const int c = w / args.n_blocks;
        const int wb = w - c * args.n_blocks;
        const int e = args.chunks[c * B200MOE_MTILE_WORDS + 0];
        const int rb = args.chunks[c * B200MOE_MTILE_WORDS + 1];
        const int re = args.chunks[c * B200MOE_MTILE_WORDS + 2];
        const int n = (re - rb + 15) / 16 * 16;
        const int half = n / 2;  // multiple of 8
        const int nbig = half / BIG_ROWS;
        const int nsmall = (half - nbig * BIG_ROWS) / SMALL_ROWS;
        const int my_rb = rb + static_cast<int>(rank) * half;
        const uint32_t cta_bytes = A_BYTES + static_cast<uint32_t>(half) * ROW_BYTES;
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&empty[stage]), phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *st = smem + stage * STAGE_BYTES;
          const uint32_t fbar_local = smem_u32(&full[stage]);
          if (leader) mbar_arrive_expect_tx(fbar_local, 2 * cta_bytes);
          const uint32_t fbar = cluster_addr(fbar_local, 0);
          if (kGateUp) {
            // View [E][gate|up][I/16][16][H]: box (64, 16 rows, gate+up, 4 groups)
            // -> rows ordered (group, gate/up, 16 rows).
            const int g0 = (wb * 128 + static_cast<int>(rank) * 64) / 16;
            tma5_pair(smem_u32(st), &tmW, fbar, kb * BK, 0, 0, g0, e);
          } else {
            tma3_pair(smem_u32(st), &tmW, fbar, kb * BK, wb * 256 + static_cast<int>(rank) * MW,
                      e);
          }
          uint8_t *sb = st + A_BYTES;
          for (int b = 0; b < nbig; ++b)
            tma2_pair(smem_u32(sb + b * BIG_ROWS * ROW_BYTES), &tmXb, fbar, kb * BK,
                      my_rb + b * BIG_ROWS);
          for (int b = 0; b < nsmall; ++b)
            tma2_pair(smem_u32(sb + (nbig * BIG_ROWS + b * SMALL_ROWS) * ROW_BYTES), &tmXs, fbar,
                      kb * BK, my_rb + nbig * BIG_ROWS + b * SMALL_ROWS);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // ---------------- MMA issuer (leader CTA) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int w = pair; w < num_work && ok; w += npairs) {
        const int c = w / args.n_blocks;
        const int rb = args.chunks[c * B200MOE_MTILE_WORDS + 1];
        const int re = args.chunks[c * B200MOE_MTILE_WORDS + 2];
        const int n = (re - rb + 15) / 16 * 16;
        const uint32_t idesc = idesc_bf16_f32(2 * MW, n);
        if (!mbar_wait_bounded(smem_u32(&acc_empty[acc]), acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d0 = tmem_base + static_cast<uint32_t>(acc * ACC_COLS);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&full[stage]), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_pair(d0, sw128_kmajor_desc(sa + kk * 32), sw128_kmajor_desc(sb + kk * 32), idesc,
                     (kb | kk) != 0 ? 1u : 0u);
          commit_pair(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        commit_pair(smem_u32(&acc_full[acc]));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    const int q = warp & 3;           // TMEM lane quarter
    const int et = threadIdx.x - 64;  // 0..127 among epilogue threads
    const uint32_t acc_empty_leader0 = cluster_addr(smem_u32(&acc_empty[0]), 0);
    const uint32_t acc_empty_leader1 = cluster_addr(smem_u32(&acc_empty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int w = pair; w < num_work; w += npairs) {
      const int c = w / args.n_blocks;
      const int wb = w - c * args.n_blocks;
      const int rb = args.chunks[c * B200MOE_MTILE_WORDS + 1];
      const int re = args.chunks[c * B200MOE_MTILE_WORDS + 2];
      const int rows = re - rb;
      const int n = (rows + 15) / 16 * 16;
      if (!kGateUp) {
        // Route id and weight of every row of this chunk.
        epi_bar();
        for (int i = et; i < rows; i += 32 * EPI_WARPS) {
          int32_t r = args.row_route[rb + i];
          if (r < 0 || r >= args.num_routes) {
            atomicOr(&g_status, kStatusIndex);
            r = -1;
          }
          s_route[i] = r;
          s_w[i] = r >= 0 ? __bfloat162float(args.route_w[r]) : 0.f;
        }
        epi_bar();
      }
      if (!mbar_wait_bounded(smem_u32(&acc_full[acc]), acc_phase, abort_flag)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(acc * ACC_COLS);
      if (kGateUp) {
        // Lane l < 16: gate of feature f, lane l + 16: up of the same feature.
        const int f = wb * 128 + static_cast<int>(rank) * 64 + q * 16 + (lane & 15);
        const bool fvalid = f < args.n_out;
        const bool low = lane < 16;
#pragma unroll 1
        for (int c0 = 0; c0 < n; c0 += 16) {
          float v[16];
          tmem_ld16(taddr + c0, v);
          tmem_ld_wait();
          // Low lanes finish columns c0..c0+7, high lanes c0+8..c0+15.
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float mine = low ? v[i] : v[8 + i];
            const float other = __shfl_xor_sync(0xffffffffu, low ? v[8 + i] : v[i], 16);
            const float g = low ? mine : other;
            const float u = low ? other : mine;
            const int col = c0 + (low ? i : 8 + i);
            if (fvalid && col < rows)
              args.out[static_cast<int64_t>(rb + col) * args.n_out + f] =
                  __float2bfloat16_rn(swiglu_bf16(g, u));
          }
        }
      } else {
        const int h = wb * 256 + static_cast<int>(rank) * MW + q * 32 + lane;
        const bool hvalid = h < args.n_out;
#pragma unroll 1
        for (int c0 = 0; c0 < n; c0 += 16) {
          float v[16];
          tmem_ld16(taddr + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = c0 + i;
            if (hvalid && col < rows) {
              const int32_t r = s_route[col];
              if (r >= 0)
                args.out[static_cast<int64_t>(r) * args.n_out + h] =
                    __float2bfloat16_rn(v[i] * s_w[col]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? acc_empty_leader1 : acc_empty_leader0);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  tc_fence_before();
  // No CTA leaves (or frees TMEM) while its peer may still write its barriers
  // or its accumulator.
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// Pairs that can be resident at once (cluster placement is per GPC).
template <bool kGateUp>
int max_pairs(int *out) {
  static int cached[64] = {0};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && cached[dev] > 0) {
    *out = cached[dev];
    return B200MOE_OK;
  }
  B200_CUDA(cudaFuncSetAttribute(pair_kernel<kGateUp>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(SMEM_BYTES)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  B200_CUDA(cudaOccupancyMaxActiveClusters(&n, pair_kernel<kGateUp>, &cfg));
  if (n < 1) {
    set_error("no SM pair can host the two-SM expert GEMM");
    return B200MOE_EUNSUPPORTED;
  }
  if (dev >= 0 && dev < 64) cached[dev] = n;
  *out = n;
  return B200MOE_OK;
}

template <bool kGateUp>
int launch(const CUtensorMap &mw, const CUtensorMap &mxb, const CUtensorMap &mxs,
           const Args &args, cudaStream_t s) {
  int pairs = 0;
  int rc = max_pairs<kGateUp>(&pairs);
  if (rc != B200MOE_OK) return rc;
  const int64_t work = args.max_chunks * args.n_blocks;
  if (work < pairs) pairs = static_cast<int>(work);
  if (pairs < 1) pairs = 1;
  B200_LAUNCH_PDL(kPdlTcgen05, pair_kernel<kGateUp>, dim3(2 * pairs), dim3(THREADS), SMEM_BYTES,
                  s, mw, mxb, mxs, args);
  B200_LAUNCHED();
  return B200MOE_OK;
}

// Row maps of a [rows, k] bf16 matrix: 64-row and 8-row boxes of 64 columns.
int row_maps(CUtensorMap *big, CUtensorMap *small, const void *base, int k, int64_t rows) {
  const uint64_t d[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(rows)};
  const uint64_t st[1] = {static_cast<uint64_t>(k) * 2};
  const uint32_t bb[2] = {BK, BIG_ROWS};
  const uint32_t bs[2] = {BK, SMALL_ROWS};
  int rc = tcg::make_map(big, base, 2, d, st, bb);
  if (rc) return rc;
  return tcg::make_map(small, base, 2, d, st, bs);
}

}  // namespace tcp

int tcp_gate_up(const void *x_packed, int hidden, int inter, const void *w13, int num_local,
                int64_t row_capacity, const int32_t *chunks, int64_t max_chunks,
                const int32_t *counters, void *act, cudaStream_t s) {
  using namespace tcp;
  CUtensorMap mw, mxb, mxs;
  // W13 [E, 2I, H] as [E][gate|up][I/16][16][H] (innermost first below); the
  // box takes 4 consecutive 16-feature groups of both halves.
  const uint64_t dw[5] = {static_cast<uint64_t>(hidden), 16, 2, static_cast<uint64_t>(inter) / 16,
                          static_cast<uint64_t>(num_local)};
  const uint64_t sw[4] = {static_cast<uint64_t>(hidden) * 2,
                          static_cast<uint64_t>(inter) * hidden * 2,
                          static_cast<uint64_t>(16) * hidden * 2,
                          static_cast<uint64_t>(2) * inter * hidden * 2};
  const uint32_t bw[5] = {BK, 16, 2, 4, 1};
  int rc = tcg::make_map(&mw, w13, 5, dw, sw, bw);
  if (rc) return rc;
  rc = row_maps(&mxb, &mxs, x_packed, hidden, row_capacity);
  if (rc) return rc;
  Args a;
  a.chunks = chunks;
  a.counters = counters;
  a.max_chunks = max_chunks;
  a.n_blocks = (inter + 127) / 128;
  a.num_kb = (hidden + BK - 1) / BK;
  a.n_out = inter;
  a.out = static_cast<__nv_bfloat16 *>(act);
  a.row_route = nullptr;
  a.route_w = nullptr;
  a.num_routes = 0;
  return launch<true>(mw, mxb, mxs, a, s);
}

int tcp_down(const void *act, int hidden, int inter, const void *w2, int num_local,
             const int32_t *row_route, const void *route_weights, int64_t num_routes,
             int64_t row_capacity, const int32_t *chunks, int64_t max_chunks,
             const int32_t *counters, void *y, cudaStream_t s) {
  using namespace tcp;
  CUtensorMap mw, mxb, mxs;
  const uint64_t dw[3] = {static_cast<uint64_t>(inter), static_cast<uint64_t>(hidden),
                          static_cast<uint64_t>(num_local)};
  const uint64_t sw[2] = {static_cast<uint64_t>(inter) * 2,
                          static_cast<uint64_t>(hidden) * inter * 2};
  const uint32_t bw[3] = {BK, MW, 1};
  int rc = tcg::make_map(&mw, w2, 3, dw, sw, bw);
  if (rc) return rc;
  rc = row_maps(&mxb, &mxs, act, inter, row_capacity);
  if (rc) return rc;
  Args a;
  a.chunks = chunks;
  a.counters = counters;
  a.max_chunks = max_chunks;
  a.n_blocks = (hidden + 255) / 256;
  a.num_kb = (inter + BK - 1) / BK;
  a.n_out = hidden;
  a.out = static_cast<__nv_bfloat16 *>(y);
  a.row_route = row_route;
  a.route_w = static_cast<const __nv_bfloat16 *>(route_weights);
  a.num_routes = num_routes;
  return launch<false>(mw, mxb, mxs, a, s);
}

}  // namespace b200moe
