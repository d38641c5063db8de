// CTA-pair (cta_group::2) tcgen05 GEMM for the dense fp16 -> fp32 and e4m3 -> bf16 operators.
//
// A cluster of two CTAs on two SMs computes one 256 x 256 output tile per step of its persistent loop:
//   * each CTA's producer warp loads ITS half of A (128 rows) and ITS half of B^T (128 rows) into its own
//     shared memory (6-stage ring, 32 KB per stage), completing on the even (leader) CTA's "full" barrier;
//   * one thread of the leader issues tcgen05.mma.cta_group::2 256x256xK, which reads A and B from both
//     CTAs' shared memory at the same offsets and accumulates rows 0-127 in the leader's TMEM and rows
//     128-255 in the peer's (2 x 256 fp32 columns each, double-buffered);
//   * stage releases and "accumulator ready" are committed to both CTAs' barriers (two plain commits,
//     own address and the peer's mapa address); each CTA's 4 epilogue warps drain their own TMEM and arrive
//     on the leader's "accumulator free" barrier.
// Per SM and K step this moves 32 KB through shared memory instead of the 48 KB of a 1-CTA 128 x 256 tile.
#pragma once

#include "gemm_sm100.cuh"

namespace bsk {

constexpr int kPairBM = 256;
#ifndef BSK_PAIR_STAGES
#define BSK_PAIR_STAGES 6
#endif
// Back-off ceilings of the waiting roles (ns): the epilogue waits a whole tile, the producer waits on a
// full ring; the MMA issuer polls tightly.
#ifndef BSK_EPI_SLEEP_NS
#define BSK_EPI_SLEEP_NS 4096
#endif
#ifndef BSK_PROD_SLEEP_NS
#define BSK_PROD_SLEEP_NS 512
#endif
#ifndef BSK_MMA_SLEEP_NS
#define BSK_MMA_SLEEP_NS 0
#endif
constexpr int kPairThreads = 192;
constexpr int kPairTmemCols = 512;

// Shape of the pair tile: kNHalves = 1 -> 256 x 256 with two 256-column TMEM accumulators (the epilogue of
// one tile overlaps the MMAs of the next); kNHalves = 2 -> 256 x 512 with one 512-column accumulator: two
// N=256 MMAs per K step share the A operand, so each byte brought into shared memory feeds more FLOPs.
template <int kNHalves>
struct PairTile {
  static constexpr int BN = 256 * kNHalves;
  static constexpr int kStageA = 128 * 128;             // this CTA's 128 rows of A, 128 B of K
  static constexpr int kStageB = kNHalves * 128 * 128;  // this CTA's 128 rows of each B^T half
  static constexpr int kStages = kNHalves == 1 ? BSK_PAIR_STAGES : 4;
  static constexpr int kAccBufs = 2 / kNHalves;
  static constexpr int kSmemBytes = 1024 + kStages * (kStageA + kStageB) + 256;
};
constexpr int kPairBN = 256;  // narrow variant
constexpr int kPairSmemBytes = PairTile<1>::kSmemBytes;
constexpr int kPairWideSmemBytes = PairTile<2>::kSmemBytes;

template <int kElemBytes, Epi kEpi, int kNHalves>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_pair_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const GemmArgs a) {
  using T = PairTile<kNHalves>;
  constexpr int kPairStages = T::kStages;
  constexpr int kPairStageA = T::kStageA;
  constexpr int kPairStageB = T::kStageB;
  constexpr int kTileN = T::BN;
  constexpr int BK = kGemmRowBytes / kElemBytes;
  constexpr int MMA_K = 32 / kElemBytes;
  constexpr int K_STEPS = BK / MMA_K;
  constexpr uint32_t IDESC = ptx::instr_desc(kPairBM, 256, 0, 0, 0, 0);
  constexpr uint32_t PAIR_TX = 2 * (kPairStageA + kPairStageB);
  constexpr uint32_t KID = kElemBytes == 1 ? kKidGemmE4m3 : kKidGemmF16;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kPairStages * kPairStageA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kPairStages * kPairStageB);
  uint64_t* full = bars;
  uint64_t* empty = bars + kPairStages;
  uint64_t* tfull = bars + 2 * kPairStages;
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
    for (int s = 0; s < kPairStages; ++s) {
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
    ptx::prefetch_tmap(&tmA);
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
  // Work unit = (output tile, K split), the split outer: units running at the same time cover the same K range of
  // different tiles, so their A and B panels are shared in L2 as in an unsplit GEMM.
  const int num_tiles = a.num_m_tiles * a.num_n_tiles;
  const int num_units = num_tiles * a.k_splits;
  auto unit_coords = [&](int unit, int& mt, int& nt, int& kb0, int& kb1) {
    gemm_tile_coords(unit % num_tiles, a, mt, nt);
    kb0 = (unit / num_tiles) * a.kb_per_split;
    kb1 = min(a.num_k_blocks, kb0 + a.kb_per_split);
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs, one thread)
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      const uint32_t sA0 = ptx::smem_u32(sA), sB0 = ptx::smem_u32(sB);
      const uint32_t full0 = ptx::smem_u32(full), empty0 = ptx::smem_u32(empty);
      const uint32_t full0_leader = ptx::mapa_shared(full0, 0);
      for (int unit = pair; unit < num_units && ok; unit += npairs) {
        int mt, nt, kb0, kb1;
        unit_coords(unit, mt, nt, kb0, kb1);
        const int m_row = mt * kPairBM + static_cast<int>(rank) * 128;
        const int n_row = nt * kTileN + static_cast<int>(rank) * 128;
        for (int kb = kb0; kb < kb1; ++kb) {
          ok = wait_bounded<true, BSK_PROD_SLEEP_NS>(empty0 + stage * 8, phase ^ 1, ctl, 1);
          if (!ok) break;
          if (rank == 0) ptx::mbar_arrive_expect_tx(full0 + stage * 8, PAIR_TX);
          ptx::tma_load_2d_pair(sA0 + stage * kPairStageA, &tmA, full0_leader + stage * 8, kb * BK, m_row);
#pragma unroll
          for (int h = 0; h < kNHalves; ++h)  // B^T rows of N half h: n0 + 256 h + 128 rank
            ptx::tma_load_2d_pair(sB0 + stage * kPairStageB + h * 128 * 128, &tmB, full0_leader + stage * 8, kb * BK,
                                  n_row + 256 * h);
          ++issued;
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
      }
      // Drain (leader): the full barriers count both CTAs' bytes, so once they complete every load of the
      // pair has landed. The peer's loads are covered by the cluster barrier that follows.
      if (rank == 0) {
        const uint32_t first = issued > kPairStages ? issued - kPairStages : 0;
        WaitCtl dctl = ctl;
        volatile int never = 0;
        dctl.abort = &never;
        for (uint32_t i = first; i < issued; ++i)
          wait_bounded<true>(full0 + (i % kPairStages) * 8, (i / kPairStages) & 1, dctl, 2);
      }
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
      // Descriptors differ only in the start-address field: build them once and add the offset (>> 4).
      const uint64_t adesc0 = ptx::smem_desc(ptx::smem_u32(sA), 16, 1024);
      const uint64_t bdesc0 = ptx::smem_desc(ptx::smem_u32(sB), 16, 1024);
      for (int unit = pair; unit < num_units && ok; unit += npairs) {
        int mt, nt, kb0, kb1;
        unit_coords(unit, mt, nt, kb0, kb1);
        ok = wait_bounded<true, BSK_MMA_SLEEP_NS>(tempty0 + acc * 8, acc_phase ^ 1, ctl, 3);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        for (int kb = kb0; kb < kb1; ++kb) {
          ok = wait_bounded<true, BSK_MMA_SLEEP_NS>(full0 + stage * 8, phase, ctl, 4);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint64_t ad = adesc0 + ((stage * kPairStageA) >> 4);
          const uint64_t bd = bdesc0 + ((stage * kPairStageB) >> 4);
#pragma unroll
          for (int k = 0; k < K_STEPS; ++k) {
#pragma unroll
            for (int h = 0; h < kNHalves; ++h) {  // N half h accumulates in TMEM columns [256 h, 256 h + 256)
              const uint64_t bdh = bd + ((h * 128 * 128) >> 4) + k * 2;
              const uint32_t accum = (kb != kb0 || k != 0) ? 1u : 0u;
              if constexpr (kElemBytes == 1)
                ptx::mma_f8_pair(d_tmem + 256 * h, ad + k * 2, bdh, IDESC, accum);
              else
                ptx::mma_f16_pair(d_tmem + 256 * h, ad + k * 2, bdh, IDESC, accum);
            }
          }
          ptx::mma_commit_pair(empty0 + stage * 8);
          ptx::mma_commit_pair(empty0_peer + stage * 8);
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        ptx::mma_commit_pair(tfull0 + acc * 8);
        ptx::mma_commit_pair(tfull0_peer + acc * 8);
        if (++acc == T::kAccBufs) { acc = 0; acc_phase ^= 1; }
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
    float scale = 1.0f;
    if constexpr (kEpi == Epi::BF16Scaled) scale = __ldg(a.scale_a) * __ldg(a.scale_b);
    for (int unit = pair; unit < num_units; unit += npairs) {
      int mt, nt, kb0, kb1;
      unit_coords(unit, mt, nt, kb0, kb1);
      const int split = unit / num_tiles;
      const int n0 = nt * kTileN;
      if (!warp_wait_bounded<true, BSK_EPI_SLEEP_NS>(ptx::smem_u32(&tfull[acc]), acc_phase, ctl, 6)) break;
      ptx::tc_fence_after();
      const int row = mt * kPairBM + static_cast<int>(rank) * 128 + 32 * q + lane;
      const bool row_ok = row < a.M;
      const uint32_t t_row = tmem_base + acc * 256 + (static_cast<uint32_t>(32 * q) << 16);
#pragma unroll 1
      for (int c = 0; c < kTileN; c += 32) {
        uint32_t r[32];
        __syncwarp();
        ptx::tmem_ld_32x32b_x32(t_row + c, r);
        ptx::tmem_wait_ld();
        const int col0 = n0 + c;
        if (row_ok) {
          if constexpr (kEpi == Epi::F32 || kEpi == Epi::F32PeerRows) {
            float* dst;
            if constexpr (kEpi == Epi::F32PeerRows) {  // row -> its owner's slot `my_rank` (NVLink store)
              const int owner = row / a.rows_per_rank;
              const int local = row - owner * a.rows_per_rank;
              dst = a.peer_out[owner] + (static_cast<int64_t>(a.my_rank) * a.rows_per_rank + local) * a.ldo + col0;
            } else {
              dst = reinterpret_cast<float*>(a.out) + split * a.split_stride + static_cast<int64_t>(row) * a.ldo +
                    col0;
            }
            store_row32_f32(dst, r, a.vec_ok && col0 + 32 <= a.N, a.N - col0,
                            kEpi == Epi::F32 ? a.accumulate : 0);
          } else {
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) + static_cast<int64_t>(row) * a.ldo + col0;
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * i]) * scale,
                                                       __uint_as_float(r[2 * i + 1]) * scale);
              pk[i] = *reinterpret_cast<uint32_t*>(&h);
            }
            if (a.vec_ok && col0 + 32 <= a.N && (reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
              st_global_v8(dst, pk);
              st_global_v8(dst + 16, pk + 8);
            } else if (a.vec_ok && col0 + 32 <= a.N) {
#pragma unroll
              for (int v = 0; v < 4; ++v)
                st_global_v4(reinterpret_cast<float*>(dst + 8 * v), pk[4 * v], pk[4 * v + 1], pk[4 * v + 2],
                             pk[4 * v + 3]);
            } else {
              for (int i = 0; i < 32; ++i)
                if (col0 + i < a.N) {
                  const uint32_t w = pk[i >> 1];
                  reinterpret_cast<unsigned short*>(dst)[i] =
                      (i & 1) ? static_cast<unsigned short>(w >> 16) : static_cast<unsigned short>(w & 0xFFFF);
                }
            }
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_u32(&tempty[acc]), 0));
      if (++acc == T::kAccBufs) { acc = 0; acc_phase ^= 1; }
    }
  }

  if constexpr (kEpi == Epi::F32PeerRows) __threadfence_system();  // peer-slot stores visible system-wide
  ptx::tc_fence_before();
  ptx::cluster_sync();  // no CTA leaves while its peer may still read its shared memory or signal its barriers
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc_pair(tmem_base, kPairTmemCols);
}

// Split-K reduction: C[row, col] = sum over s of ws[s][row][col], added in split order (deterministic).
// ws slabs are [M, ld_ws] fp32 with ld_ws a multiple of 4 and 16-byte aligned rows.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws, int splits,
                                                            int64_t split_stride, int64_t ld_ws,
                                                            float* __restrict__ C, int64_t ldc, int M, int N,
                                                            int vec_ok) {
  const int groups = (N + 3) / 4;
  const int64_t total = static_cast<int64_t>(M) * groups;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(g / groups);
    const int c4 = static_cast<int>(g % groups) * 4;
    const float* src = ws + static_cast<int64_t>(row) * ld_ws + c4;
    float4 acc = *reinterpret_cast<const float4*>(src);
    for (int sidx = 1; sidx < splits; ++sidx) {
      const float4 v = *reinterpret_cast<const float4*>(src + sidx * split_stride);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    float* dst = C + static_cast<int64_t>(row) * ldc + c4;
    if (vec_ok && c4 + 4 <= N) {
      *reinterpret_cast<float4*>(dst) = acc;
    } else {
      const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
      for (int i = 0; i < 4 && c4 + i < N; ++i) dst[i] = vals[i];
    }
  }
}

}  // namespace bsk
