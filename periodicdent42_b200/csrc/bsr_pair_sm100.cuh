// BSR x dense SpMM on a CTA pair, computed transposed: C^T[cols, rows] = B^T A_bsr^T, so the operand two CTAs can
// share is the sparse block.
//
// A cluster of two CTAs takes one work unit = (block-row r, 512 output columns n0 .. n0 + 511). For every
// nonzero block (r, kb) of A and K slice s of it:
//   * M side (rows of the MMA) = output columns. CTA `rank` loads, for h = 0, 1, the dense B rows
//     [kb*128 + s*BK, +BK) x columns [n0 + 256h + 128 rank, +128): MN-major operand, two 64-column slabs each;
//   * N side = the block-row's 128 rows. CTA `rank` loads rows [64 rank, +64) of the A block, K-major;
//   * the leader issues, per K step, two tcgen05.mma.cta_group::2 of M = 256, N = 128 (h = 0, 1), both reading the
//     same A-block halves: each CTA's shared-memory traffic per K block is 64 KB of B + 16 KB of A for 8.4 MFLOP,
//     against 64 + 32 KB in the 1-CTA 128 x 256 tile (where the A block is re-read for every 256 columns).
// TMEM per CTA: lane = output column (128 per accumulator), column = output row; accumulator h of tile buffer t at
// columns [256 t + 128 h, +128); two tile buffers, so the epilogue of one unit overlaps the MMAs of the next. The
// epilogue thread owning column c writes 32 rows per tcgen05.ld; a warp's 32 lanes are 32 adjacent columns, so each
// store instruction writes 128 contiguous bytes of a row.
#pragma once

#include "gemm_pair_sm100.cuh"

namespace bsk {

constexpr int kBsrPairTileN = 512;                 // output columns per unit
constexpr int kBsrPairBK = 64;                     // K elements per stage (128 B of fp16)
constexpr int kBsrPairSlab = kBsrPairBK * 128;     // one 64-column x BK slab of B, 8 KB
constexpr int kBsrPairStageB = 4 * kBsrPairSlab;   // 2 accumulators x 2 slabs = 32 KB
constexpr int kBsrPairStageA = 64 * 128;           // 64 rows of the A block x 128 B = 8 KB
constexpr int kBsrPairStage = kBsrPairStageB + kBsrPairStageA;
constexpr int kBsrPairStages = 5;
constexpr int kBsrPairSmemBytes = 1024 + kBsrPairStages * kBsrPairStage + 256;
// L2 policies: bit 0 streams the output stores (evict-first: C is written once and must not push the operands out
// of L2), bit 1 loads the sparse blocks evict-last (each is read again for every 512 output columns), bit 2 loads
// the dense B rows evict-last.
#ifndef BSK_BSR_PAIR_HINTS
#define BSK_BSR_PAIR_HINTS 3
#endif

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    spmm_bsr_pair_sm100_kernel(const __grid_constant__ CUtensorMap tmVals, const __grid_constant__ CUtensorMap tmB,
                               const GemmArgs a) {
  constexpr int BK = kBsrPairBK;
  constexpr int K_STEPS = BK / 16;
  constexpr int STEPS = 128 / BK;  // stages per nonzero block
  // M = 256 output columns (MN-major dense B), N = 128 block rows (K-major A block)
  constexpr uint32_t IDESC = ptx::instr_desc(256, 128, 0, 0, 1, 0);
  constexpr uint32_t PAIR_TX = 2 * kBsrPairStage;
  constexpr uint32_t KID = kKidSpmmBsr;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBsrPairStages * kBsrPairStage);
  uint64_t* full = bars;
  uint64_t* empty = bars + kBsrPairStages;
  uint64_t* tfull = bars + 2 * kBsrPairStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();  // 0: leader (issues the MMAs)
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBsrPairStages; ++s) {
      ptx::mbar_init(ptx::smem_u32(&full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(ptx::smem_u32(&tfull[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&tempty[s]), 8);  // 4 epilogue warps x 2 CTAs
    }
    ptx::mbar_init(ptx::smem_u32(drain), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmVals);
    ptx::prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(ptx::smem_u32(tmem_holder), kPairTmemCols);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();  // barriers of both CTAs initialised, TMEM of both allocated
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  WaitCtl ctl{abort_flag, a.err, a.timeout_ns, KID};
  const int num_units = a.num_m_tiles * a.num_n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    // The warp walks the block-row index: per 32 nonzeros of the row, one coalesced load of their column indices
    // (lane l holds col_idx[jb + l]), handed to lane 0 by shuffle; lane 0 alone waits on the ring and issues the
    // TMA loads, so no per-stage warp collective sits on the issue path.
    uint32_t stage = 0, phase = 0, issued = 0;
    bool ok = true;
    const uint32_t s0 = ptx::smem_u32(smem);
    const uint32_t full0 = ptx::smem_u32(full), empty0 = ptx::smem_u32(empty);
    const uint32_t full0_leader = ptx::mapa_shared(full0, 0);
    const uint64_t pol_a = (BSK_BSR_PAIR_HINTS & 2) ? ptx::policy_evict_last() : 0;
    const uint64_t pol_b = (BSK_BSR_PAIR_HINTS & 4) ? ptx::policy_evict_last() : 0;
    for (int unit = pair; unit < num_units && ok; unit += npairs) {
      int mt, nt;
      gemm_tile_coords(unit, a, mt, nt);
      const int r = a.row_begin + mt;
      int j0, j1;
      if (!bsr_row_range(a, r, j0, j1) && rank == 0 && lane == 0)
        atomicCAS(a.err, 0u, kErrBounds | (KID << 8) | (7u << 16));
      const int col0 = nt * kBsrPairTileN + static_cast<int>(rank) * 128;
      for (int jb = j0; jb < j1 && ok; jb += 32) {
        const int cidx = (jb + lane < j1) ? __ldg(&a.col_idx[jb + lane]) : 0;
        const int cnt = min(32, j1 - jb);
        for (int jj = 0; jj < cnt && ok; ++jj) {
          int kb = __shfl_sync(0xFFFFFFFFu, cidx, jj);
          if (lane == 0) {
            const int j = jb + jj;
            if (kb < 0 || kb >= a.kb_count) {  // out-of-range column: flag it; the B rows read zero fill
              if (rank == 0) atomicCAS(a.err, 0u, kErrBounds | (KID << 8) | (8u << 16));
              kb = a.kb_count;
            }
            for (int s = 0; s < STEPS; ++s) {
              ok = wait_bounded<true, BSK_PROD_SLEEP_NS>(empty0 + stage * 8, phase ^ 1, ctl, 1);
              if (!ok) break;
              if (rank == 0) ptx::mbar_arrive_expect_tx(full0 + stage * 8, PAIR_TX);
              const uint32_t st = s0 + stage * kBsrPairStage;
              const uint32_t fb = full0_leader + stage * 8;
              // A block j, this CTA's 64 rows, K slice s (K-major)
              if constexpr ((BSK_BSR_PAIR_HINTS & 2) != 0)
                ptx::tma_load_2d_pair_hint(st + kBsrPairStageB, &tmVals, fb, s * BK,
                                           j * 128 + 64 * static_cast<int>(rank), pol_a);
              else
                ptx::tma_load_2d_pair(st + kBsrPairStageB, &tmVals, fb, s * BK, j * 128 + 64 * static_cast<int>(rank));
              // dense B rows of K slice s of block column kb, columns col0 + 256 h + 64 q (MN-major slabs)
#pragma unroll
              for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                  if constexpr ((BSK_BSR_PAIR_HINTS & 4) != 0)
                    ptx::tma_load_2d_pair_hint(st + (2 * h + q) * kBsrPairSlab, &tmB, fb, col0 + 256 * h + 64 * q,
                                               kb * 128 + s * BK, pol_b);
                  else
                    ptx::tma_load_2d_pair(st + (2 * h + q) * kBsrPairSlab, &tmB, fb, col0 + 256 * h + 64 * q,
                                          kb * 128 + s * BK);
                }
              ++issued;
              if (++stage == kBsrPairStages) { stage = 0; phase ^= 1; }
            }
          }
          ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        }
      }
    }
    if (rank == 0 && lane == 0) {  // every load of the pair has landed (the leader's full barriers count both CTAs')
      const uint32_t first = issued > kBsrPairStages ? issued - kBsrPairStages : 0;
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      for (uint32_t i = first; i < issued; ++i)
        wait_bounded<true>(full0 + (i % kBsrPairStages) * 8, (i / kBsrPairStages) & 1, dctl, 2);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      // ---------------------------------------------------------------- MMA issuer (leader, one thread)
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t full0 = ptx::smem_u32(full), empty0 = ptx::smem_u32(empty);
      const uint32_t empty0_peer = ptx::mapa_shared(empty0, 1);
      const uint32_t tfull0 = ptx::smem_u32(tfull), tempty0 = ptx::smem_u32(tempty);
      const uint32_t tfull0_peer = ptx::mapa_shared(tfull0, 1);
      // MN-major B slabs: 64-column slabs BK rows deep (LBO = slab stride), K step = 16 rows of 128 B.
      const uint64_t bdesc0 = ptx::smem_desc(ptx::smem_u32(smem), kBsrPairSlab, 1024);
      // K-major A-block half: 128-B rows, K step = 32 B.
      const uint64_t adesc0 = ptx::smem_desc(ptx::smem_u32(smem) + kBsrPairStageB, 16, 1024);
      for (int unit = pair; unit < num_units && ok; unit += npairs) {
        int mt, nt;
        gemm_tile_coords(unit, a, mt, nt);
        int j0, j1;
        bsr_row_range(a, a.row_begin + mt, j0, j1);
        const int nk = (j1 - j0) * STEPS;
        ok = wait_bounded<true, BSK_MMA_SLEEP_NS>(tempty0 + acc * 8, acc_phase ^ 1, ctl, 3);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        for (int kk = 0; kk < nk; ++kk) {
          ok = wait_bounded<true, BSK_MMA_SLEEP_NS>(full0 + stage * 8, phase, ctl, 4);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint64_t st = (stage * kBsrPairStage) >> 4;
#pragma unroll
          for (int k = 0; k < K_STEPS; ++k) {
#pragma unroll
            for (int h = 0; h < 2; ++h)  // output columns 256 h + [0, 256) of the unit -> TMEM columns 128 h + ...
              ptx::mma_f16_pair(d_tmem + 128 * h, bdesc0 + st + ((2 * h * kBsrPairSlab) >> 4) + k * ((16 * 128) >> 4),
                                adesc0 + st + k * 2, IDESC, (kk != 0 || k != 0) ? 1u : 0u);
          }
          ptx::mma_commit_pair(empty0 + stage * 8);
          ptx::mma_commit_pair(empty0_peer + stage * 8);
          if (++stage == kBsrPairStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        ptx::mma_commit_pair(tfull0 + acc * 8);
        ptx::mma_commit_pair(tfull0_peer + acc * 8);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      ptx::mma_commit_pair(ptx::smem_u32(drain));
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      wait_bounded<true>(ptx::smem_u32(drain), 0, dctl, 5);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int q = warp & 3;
    uint32_t acc = 0, acc_phase = 0;
    float* out = reinterpret_cast<float*>(a.out);
    for (int unit = pair; unit < num_units; unit += npairs) {
      int mt, nt;
      gemm_tile_coords(unit, a, mt, nt);
      const int r = a.row_begin + mt;
      int j0, j1;
      bsr_row_range(a, r, j0, j1);
      if (!warp_wait_bounded<true, BSK_EPI_SLEEP_NS>(ptx::smem_u32(&tfull[acc]), acc_phase, ctl, 6)) break;
      ptx::tc_fence_after();
      const int64_t row0 = static_cast<int64_t>(r) * 128;
      const uint32_t t_lane = tmem_base + acc * 256 + (static_cast<uint32_t>(32 * q) << 16);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int col = nt * kBsrPairTileN + 256 * h + 128 * static_cast<int>(rank) + 32 * q + lane;
        const bool col_ok = col < a.N;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {  // output rows 32 cc .. 32 cc + 31
          uint32_t u[32];
          __syncwarp();
          if (j1 > j0) {
            ptx::tmem_ld_32x32b_x32(t_lane + 128 * h + 32 * cc, u);
            ptx::tmem_wait_ld();
          } else {  // an empty block-row: zeros
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = 0u;
          }
          if (col_ok) {
            float* dst = out + (row0 + 32 * cc) * a.ldo + col;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if constexpr ((BSK_BSR_PAIR_HINTS & 1) != 0)
                __stcs(dst + static_cast<int64_t>(i) * a.ldo, __uint_as_float(u[i]));
              else
                dst[static_cast<int64_t>(i) * a.ldo] = __uint_as_float(u[i]);
            }
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_u32(&tempty[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  ptx::tc_fence_before();
  ptx::cluster_sync();  // no CTA leaves while its peer may still read its shared memory or signal its barriers
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc_pair(tmem_base, kPairTmemCols);
}

}  // namespace bsk
