// Dense GEMM on CTA pairs (cluster of 2, tcgen05 cta_group::2), sm_100a.
//
// Same contract as the dense path of gemm_tc.cuh (kernels/gemm.py:7-40 of the
// reference: C = A * B, row-major, GROUP_M raster, masked edges), with
// 256 x BN tiles computed by a pair of CTAs on two SMs:
//   * CTA r of the pair stages rows [m0 + 128 r, +128) of A and columns
//     [n0 + r BN/2, +BN/2) of B, each with its own TMA loads (no cross-CTA
//     copies); both CTAs' loads complete on the leader's (r = 0) barrier;
//   * the leader issues tcgen05.mma.cta_group::2 (M = 256, N = BN, K = 16),
//     which reads both CTAs' shared memory and accumulates 128 rows x BN
//     columns in each CTA's TMEM;
//   * the leader's commits free both CTAs' stages and hand both CTAs'
//     accumulators to their epilogues; each epilogue warp arrives on the
//     leader's accumulator-empty barrier.
// Per SM the MMA reads 8 KB of operands per 128 x 256 x 16 step instead of
// 12 KB, and a stage is 32 KB (BN = 256), so the ring is 6 deep.
#pragma once

#include "bokt_device.cuh"
#include "gemm_tc.cuh"

namespace bokt {

template <int BN>
struct GemmTc2Shape {
  static constexpr int kBHalf = BN / 2;
  static constexpr int kBBytes = kBHalf * kGemmBK * 2;
  static constexpr int kStageBytes = kGemmABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static_assert(BN == 128 || BN == 256, "pair tiles need BN of 128 or 256");
};

__host__ __device__ inline int gemm_tc2_smem_bytes(int bn, int stages, int experts = 0) {
  return 1024 + stages * (kGemmABytes + (bn / 2) * kGemmBK * 2) + kEpiBytes +
         (2 * stages + 4) * 8 + 16 + (experts > 0 ? (4 * experts + 4) * 4 : 0);
}

// ROWSCALE: the epilogue scales C row m by args.row_scale[m] (fp32) before
// rounding (fused RMSNorm -> GEMM with the norm weight folded into B).
// GROUPED: the MoE grouped GEMM on pair tiles inside each expert
// (kernels/moe_grouped_gemm.py:11-58; schedule built per CTA from the device
// offsets, W read through a 3-D tensor map [E][K][N]).  An expert's rows are
// cut into 256-row tiles (M = 256, 128 rows per CTA); a last block of at most
// 128 rows is a half-height tile (tcgen05 M = 128, 64 rows per CTA, A box of
// 64 rows from tmA64), so padding stays that of 128-row tiles and the weight
// column block of a short tail is read alongside the expert's other tiles.
// Half-tile accumulator (per CTA, per-SM M = 64): TMEM lanes 0-63 hold the
// CTA's 64 rows for output columns [0, BN/2), lanes 64-127 the same rows for
// columns [BN/2, BN), both in TMEM columns [0, BN/2) of the accumulator.
// SCATTER (grouped only): the expert-parallel epilogue of gemm_tc_kernel —
// packed row l goes to its token owner's buffer (possibly a peer GPU's).
template <int BN, typename OutT, bool ROWSCALE = false, bool GROUPED = false, bool SCATTER = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmA64, GemmTcArgs args) {
  using Shape = GemmTc2Shape<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int stages = args.stages;
  uint8_t* sA = smem;
  uint8_t* sB = smem + stages * kGemmABytes;
  uint8_t* sEpi = sB + stages * Shape::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + kEpiBytes);
  uint64_t* empty = full + stages;
  uint64_t* tfull = empty + stages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  GroupedSchedule sched;  // GROUPED only: [E+1] + 3 x [E] + [3] ints
  sched.pre = reinterpret_cast<int*>(tmem_holder + 4);
  sched.pstart = sched.pre + (args.E + 1);
  sched.pcount = sched.pstart + args.E;
  sched.pexp = sched.pcount + args.E;
  sched.totals = sched.pexp + args.E;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int M = args.M, N = args.N;
  const int nm = (M + 2 * kGemmBM - 1) / (2 * kGemmBM);
  const int nn = (N + BN - 1) / BN;
  const int nkb = (args.K + kGemmBK - 1) / kGemmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * 4);  // one arrival per epilogue warp of both CTAs
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (GROUPED) tma_prefetch_desc(&tmA64);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, Shape::kTmemCols);
    tmem_relinquish_pair();
  }
  pdl_allow_next();
  pdl_wait();
  if constexpr (GROUPED) {
    // Every CTA builds the same schedule (cluster_sync publishes it).
    build_grouped_schedule(args, nn, sched, 2 * kGemmBM);
  }
  // Split-K (dense pairs only): workers are CTA pairs; CTA r of pair p uses
  // workspace slot 2 p + r for the 128 accumulator rows it holds.
  const int split = args.split_k > 1 ? args.split_k : 1;
  SplitKView sk = {};
  const bool fixup = split > 1 && !args.splitk_reduce;  // owner fix-up with flags
  if (split > 1) {
    sk = splitk_view(args.splitk_ws, args.splitk_slots, BN);
    if (fixup && threadIdx.x == 0) tmem_holder[2] = ld_acquire_gpu(sk.header) + 1u;
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised, TMEM allocated, schedule built
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t expected = tmem_holder[2];
  const int ntiles = GROUPED ? sched.totals[0] : nm * nn;
  const int workers = splitk_workers(npairs, ntiles, split);

  // 256-row tiles: dense in the GROUP_M raster of kernels/gemm.py:20-26;
  // grouped inside each expert (rows_valid = rows of the expert in the tile).
  auto tile_at = [&](int t) -> TileCoord {
    if constexpr (GROUPED) {
      return grouped_tile(t, sched, args.E, nn, BN, args.raster, 2 * kGemmBM);
    } else {
      const int per_group = args.group_m * nn;
      const int group = t / per_group;
      const int first_m = group * args.group_m;
      const int gm = min(nm - first_m, args.group_m);
      const int local = t - group * per_group;
      TileCoord c;
      c.a_row = (first_m + local % gm) * 2 * kGemmBM;
      c.n0 = (local / gm) * BN;
      c.expert = 0;
      c.c_row = c.a_row;
      c.rows_valid = min(2 * kGemmBM, M - c.a_row);
      return c;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producers (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      SegmentCursor cur = segment_cursor(pair, workers, ntiles, split);
      Segment sg;
      for (int i = 0; ok && segment_next(cur, split, nkb, sg); ++i) {
        const TileCoord tc = tile_at(sg.tile);
        const bool rev = k_reversed_for<GROUPED>(i, split, tc.n0, BN);
        for (int kk = sg.kb0; kk < sg.kb1; ++kk) {
          const int kb = rev ? sg.kb1 - 1 - (kk - sg.kb0) : kk;
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, abort_flag, 11)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = map_shared(smem_addr(&full[stage]), 0);
          const bool half = GROUPED && tc.rows_valid <= kGemmBM;
          if (leader)
            mbar_arrive_expect_tx(&full[stage], 2 * (half ? kGemmABytes / 2 + Shape::kBBytes
                                                          : Shape::kStageBytes));
          if (half) {
            tma_load_2d_pair(sA + stage * kGemmABytes, &tmA64, full_leader, kb * kGemmBK,
                             tc.a_row + static_cast<int>(rank) * (kGemmBM / 2));
          } else {
            tma_load_2d_pair(sA + stage * kGemmABytes, &tmA, full_leader, kb * kGemmBK,
                             tc.a_row + static_cast<int>(rank) * kGemmBM);
          }
#pragma unroll
          for (int c = 0; c < Shape::kBHalf / 64; ++c) {
            const int col = tc.n0 + static_cast<int>(rank) * Shape::kBHalf + c * 64;
            if constexpr (GROUPED) {
              tma_load_3d_pair(sB + stage * Shape::kBBytes + c * 8192, &tmB, full_leader, col,
                               kb * kGemmBK, tc.expert);
            } else {
              tma_load_2d_pair(sB + stage * Shape::kBBytes + c * 8192, &tmB, full_leader, col,
                               kb * kGemmBK);
            }
          }
          if (++stage == stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int i = 0;
      bool ok = true;
      SegmentCursor cur = segment_cursor(pair, workers, ntiles, split);
      Segment sg;
      for (; ok && segment_next(cur, split, nkb, sg); ++i) {
        uint32_t idesc = args.idesc;
        if constexpr (GROUPED) {
          if (tile_at(sg.tile).rows_valid <= kGemmBM) idesc = args.idesc_half;
        }
        const int acc = i & 1;
        const uint32_t acc_phase = (static_cast<uint32_t>(i) >> 1) & 1u;
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, abort_flag, 12)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
          if (!mbar_wait_cluster(&full[stage], phase, abort_flag, 13)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(sA + stage * kGemmABytes);
          const uint32_t b_addr = smem_addr(sB + stage * Shape::kBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t a_desc = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t b_desc = smem_desc_sw128(b_addr + k * 2048, 64 * 128, 1024);
            umma_f16_ss_pair(d_tmem, a_desc, b_desc, idesc, (kb != sg.kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit_both(&empty[stage]);
          if (++stage == stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_both(&tfull[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int r = q * 32 + lane;
    OutT* C = reinterpret_cast<OutT*>(args.C);
    uint8_t* stage = sEpi + (warp - 2) * kEpiStageBytes;
    OutT** rowptr = reinterpret_cast<OutT**>(sEpi + kEpiWarps * kEpiStageBytes) + (warp - 2) * 32;
    const int64_t slot_floats = static_cast<int64_t>(kGemmBM) * BN;
    const int my_slot = 2 * pair + static_cast<int>(rank);
    int i = 0;
    SegmentCursor cur = segment_cursor(pair, workers, ntiles, split);
    Segment sg;
    for (; segment_next(cur, split, nkb, sg); ++i) {
      const TileCoord tc = tile_at(sg.tile);
      const int acc = i & 1;
      const uint32_t acc_phase = (static_cast<uint32_t>(i) >> 1) & 1u;
      const bool ok = mbar_wait_cluster(&tfull[acc], acc_phase, abort_flag, 14);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (args.splitk_reduce && (sg.kb0 > 0 || sg.kb1 < nkb)) {
        // Separate reduction: only the partial (slot 2 c for the pair's first
        // segment, 2 c + 1 for its last; c = 2 pair + rank).
        epilogue_store_partial<BN>(taddr, sk.partials + slot_floats * (2 * my_slot + (i > 0)),
                                   q * 32, 0, lane);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(map_shared(smem_addr(&tempty[acc]), 0));
        continue;
      }
      if (sg.kb0 > 0) {
        // Split-K non-owner (this pair's first segment): publish this warp's
        // fp32 partial rows into the CTA's slot.
        epilogue_store_partial<BN>(taddr, sk.partials + slot_floats * my_slot, q * 32, 0, lane);
        splitk_publish(sk.flags, my_slot, q, expected, lane);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(map_shared(smem_addr(&tempty[acc]), 0));
        continue;
      }
      int first = 0, count = 0;
      if (sg.kb1 < nkb) {
        count = splitk_contributors(pair, workers, ntiles, split, sg.tile, &first);
        count = splitk_acquire(sk.flags, 2 * first + static_cast<int>(rank), 2, count, q,
                               expected, lane, 22);
      }
      const float* pfirst = sk.partials + slot_floats * (2 * first + static_cast<int>(rank));
      // Full tile: this CTA's accumulator rows are tile rows [128 rank, +128),
      // warp quadrant q holds rows 32 q .. 32 q + 31, all BN columns.
      // Half tile (grouped): this CTA's rows are [64 rank, +64); quadrant q holds
      // rows 32 (q & 1) .. +31 of column half q >> 1 (BN / 2 columns each).
      const bool half = GROUPED && tc.rows_valid <= kGemmBM;
      const int local = half ? static_cast<int>(rank) * (kGemmBM / 2) + (q & 1) * 32 + lane
                             : static_cast<int>(rank) * kGemmBM + r;
      const int col0 = tc.n0 + (half ? (q >> 1) * (BN / 2) : 0);
      bool row_ok = local < tc.rows_valid;
      const int row = tc.c_row + local;
      OutT* crow = row_ok ? C + static_cast<size_t>(row) * N + col0 : nullptr;
      if constexpr (SCATTER) {
        if (row_ok) {
          const int a = args.rowmap[row];
          const int o = a / args.rows_per_owner;
          if (a < 0 || o >= args.owners) {
            report_status(kStatusBadExpertId, row);
            crow = nullptr;
          } else {
            crow = reinterpret_cast<OutT*>(args.out_ptrs[o]) +
                   static_cast<size_t>(a - o * args.rows_per_owner) * N + col0;
          }
        }
      }
      rowptr[lane] = crow;
      float scale = 1.f;
      if constexpr (ROWSCALE) scale = row_ok ? args.row_scale[row] : 1.f;
      __syncwarp();
      if (half) {
        epilogue_store_tile<BN / 2, OutT, ROWSCALE>(taddr, stage, rowptr, col0, N, lane, scale);
      } else {
        epilogue_store_tile<BN, OutT, ROWSCALE>(taddr, stage, rowptr, col0, N, lane, scale,
                                                pfirst, 2 * slot_floats, count, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(map_shared(smem_addr(&tempty[acc]), 0));
    }
    if constexpr (SCATTER) __threadfence_system();  // peer stores visible before the barrier
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (fixup && threadIdx.x == 0) splitk_finish(sk.header, expected);
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Shape::kTmemCols);
  }
}

}  // namespace bokt
