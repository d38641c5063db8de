// Persistent, warp-specialised tcgen05 GEMM for sm_100a, shared by three operators:
//   * dense fp16 x fp16 -> fp32       (A [M,K] row-major, B given as B^T [N,K] row-major, i.e. column-major B)
//   * dense e4m3 x e4m3 -> bf16       (same layouts, per-tensor scales applied in the epilogue)
//   * BSR fp16 x dense fp16 -> fp32   (A = 128x128 nonzero blocks, B [K,N] row-major, gathered by column index)
//
// One CTA per SM; 6 warps:
//   warp 0     TMA producer: fills a 4-stage shared-memory ring (A 128 x 128 B, B 256 x 128 B per stage)
//   warp 1     TMEM owner + MMA issuer: tcgen05.mma 128x256xK into one of two TMEM accumulators
//   warps 2-5  epilogue: tcgen05.ld the finished accumulator (warp w reads TMEM lanes 32*(w%4)..+31)
//              and stores it, while the MMA warp fills the other accumulator.
// Output tile 128 x 256, 2 x 256 fp32 TMEM columns (all 512). Each wait is bounded: a wait that runs
// out records an error word, raises the CTA abort flag and every role drains and returns.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx_sm100.cuh"

namespace bsk {

constexpr int kGemmBM = 128;
constexpr int kGemmBN = 256;
constexpr int kGemmRowBytes = 128;  // K extent of one stage, in bytes (one 128-B swizzle span)
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 192;
constexpr int kGemmAStage = kGemmBM * kGemmRowBytes;  // 16 KB
constexpr int kGemmBStage = kGemmBN * kGemmRowBytes;  // 32 KB
constexpr int kGemmTmemCols = 512;
constexpr int kGemmSmemBytes = 1024 /*align slack*/ + kGemmStages * (kGemmAStage + kGemmBStage) + 256;
// BSR x BSR: B's block map (block-row x block-column -> stored block, -1 absent) staged in shared memory after the
// barriers, up to this many entries; larger maps fall back to a binary search per lookup.
constexpr int kBsrTableMax = 8192;
constexpr int kGemmBsrBsrSmemBytes = kGemmSmemBytes + kBsrTableMax * 4 + 1024;  // + staged row pointers

enum class Mainloop : int { Dense = 0, Bsr = 1, BsrBsr = 2 };
// F32PeerRows: fp32 partial rows stored into their owner rank's receive slot (split-K reduce-scatter).
enum class Epi : int { F32 = 0, BF16Scaled = 1, F32PeerRows = 2 };
constexpr int kMaxPeers = 8;

// Kernel ids recorded in the device error word.
enum : uint32_t { kKidGemmF16 = 1, kKidGemmE4m3 = 2, kKidSpmmBsr = 3, kKidBsAttn = 4, kKidWaitProbe = 5,
                  kKidSpmmBsrBsr = 6 };

struct GemmArgs {
  int M, N;                  // output extent (rows / cols of C that exist)
  int num_m_tiles, num_n_tiles;
  int num_k_blocks;          // dense: stages per tile
  int group_m;               // tile rasterisation group (M tiles per group)
  void* out;                 // C (fp32) or D (bf16)
  int64_t ldo;               // elements
  int vec_ok;                // 16-byte aligned rows: vector stores allowed
  const float* scale_a;      // e4m3 only
  const float* scale_b;
  const int* row_ptr;        // BSR only: block-row pointer (int32)
  const int* col_idx;        // BSR only: block-column index per nonzero block
  int row_begin;             // BSR only: first block-row of this launch
  int nnzb;                  // BSR only: number of nonzero blocks (clamp for row_ptr)
  int kb_count;              // BSR only: number of block-columns (K / 128)
  int k_splits;              // CTA-pair kernels: K splits per output tile (1 = none)
  int kb_per_split;          // K stages per split (every split non-empty)
  int64_t split_stride;      // elements between the partial-output slabs of consecutive splits
  float* peer_out[kMaxPeers];  // F32PeerRows: receive-slot buffer of each rank ([world][rows_per_rank][ldo])
  int rows_per_rank;           // F32PeerRows: output rows owned by each rank
  int my_rank;                 // F32PeerRows: slot this rank writes in every owner's buffer
  int accumulate;              // F32 only: C += result (C read before the store) instead of C = result
  const int* b_row_ptr;        // BSR x BSR only: B's block-row pointer (K/128 + 1 entries, int32)
  const int* b_col_idx;        // BSR x BSR only: B's block columns, ascending within each block-row
  int b_nnzb;                  // BSR x BSR only: B's stored blocks (a load at block b_nnzb reads zero fill)
  int b_nbc;                   // BSR x BSR only: B's block columns when its block map is staged in shared
                               // memory (kb_count * b_nbc <= kBsrTableMax), else 0 (binary search in global)
  uint32_t* err;
  uint64_t timeout_ns;
};

__device__ __forceinline__ void gemm_tile_coords(int tile, const GemmArgs& a, int& mt, int& nt) {
#if BSK_RASTER_NMAJOR
  if (a.row_ptr == nullptr) {
    const int gn_ = a.group_m < a.num_n_tiles ? a.group_m : a.num_n_tiles;
    const int per = gn_ * a.num_m_tiles;
    const int gg = tile / per;
    const int fn = gg * gn_;
    const int gnn = min(a.num_n_tiles - fn, gn_);
    const int tt = tile - gg * per;
    nt = fn + tt % gnn;
    mt = tt / gnn;
    return;
  }
#endif
  const int per_group = a.group_m * a.num_n_tiles;
  const int g = tile / per_group;
  const int first_m = g * a.group_m;
  const int gm = min(a.num_m_tiles - first_m, a.group_m);
  const int t = tile - g * per_group;
  mt = first_m + t % gm;
  nt = t / gm;
}

// Nonzero-block range of block-row r, clamped to [0, nnzb] so a corrupt row_ptr can neither loop long
// nor read outside the value array. Returns true when clamping changed nothing.
__device__ __forceinline__ bool bsr_row_range(const GemmArgs& a, int r, int& j0, int& j1) {
  const int p0 = __ldg(&a.row_ptr[r]);
  const int p1 = __ldg(&a.row_ptr[r + 1]);
  j0 = min(max(p0, 0), a.nnzb);
  j1 = min(max(p1, j0), a.nnzb);
  return j0 == p0 && j1 == p1;
}

// Position of B block (kb, jc) in B's BSR arrays, or -1: from the shared-memory block map when it is staged,
// else a binary search of the ascending block-row kb (row pointers clamped to [0, b_nnzb]).
__device__ __forceinline__ int bsr_b_find(const GemmArgs& a, const int* tab, int kb, int jc) {
  if (tab) return jc < a.b_nbc ? tab[kb * a.b_nbc + jc] : -1;
  int lo = min(max(__ldg(&a.b_row_ptr[kb]), 0), a.b_nnzb);
  int hi = min(max(__ldg(&a.b_row_ptr[kb + 1]), lo), a.b_nnzb);
  const int end = hi;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(&a.b_col_idx[mid]) < jc) lo = mid + 1; else hi = mid;
  }
  return (lo < end && __ldg(&a.b_col_idx[lo]) == jc) ? lo : -1;
}

// BSR x BSR: for A's stored block j (block column kb = col_idx[j]) and the output tile whose first block column
// is jc, the B blocks (kb, jc) and (kb, jc + 1). Returns false when neither exists or kb is out of range (the
// A block then contributes nothing to the tile).
__device__ __forceinline__ bool bsrbsr_pair(const GemmArgs& a, const int* tab, int j, int jc, int& p0, int& p1) {
  const int kb = __ldg(&a.col_idx[j]);
  p0 = p1 = -1;
  if (kb < 0 || kb >= a.kb_count) return false;
  p0 = bsr_b_find(a, tab, kb, jc);
  p1 = bsr_b_find(a, tab, kb, jc + 1);
  return p0 >= 0 || p1 >= 0;
}

// Warp-collective: how many of A's blocks [j0, j1) meet B block (kb, jc) (*c0) and (kb, jc + 1) (*c1), i.e. how
// many MMAs each 128-column half of the tile receives. Same answer on every lane and in every role of the CTA.
__device__ __forceinline__ void bsrbsr_half_counts(const GemmArgs& a, const int* tab, int j0, int j1, int jc, int* c0,
                                                   int* c1) {
  const int lane = threadIdx.x & 31;
  int n0 = 0, n1 = 0;
  for (int jb = j0; jb < j1; jb += 32) {
    int p0 = -1, p1 = -1;
    if (jb + lane < j1) bsrbsr_pair(a, tab, jb + lane, jc, p0, p1);
    n0 += __popc(__ballot_sync(0xFFFFFFFFu, p0 >= 0));
    n1 += __popc(__ballot_sync(0xFFFFFFFFu, p1 >= 0));
  }
  *c0 = n0;
  *c1 = n1;
}

__device__ __forceinline__ void st_global_v4(float* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Stores 32 fp32 accumulator values of one output row at dst (columns col0 .. col0+31, `valid` of them inside
// the matrix). vec: 16-byte aligned full chunk. accumulate: dst[i] = dst[i] + r[i] (the previous value first).
__device__ __forceinline__ void store_row32_f32(float* dst, uint32_t (&r)[32], bool vec, int valid, int accumulate) {
  if (vec) {
    if (accumulate) {
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const float4 c = *reinterpret_cast<const float4*>(dst + 4 * v);
        r[4 * v + 0] = __float_as_uint(c.x + __uint_as_float(r[4 * v + 0]));
        r[4 * v + 1] = __float_as_uint(c.y + __uint_as_float(r[4 * v + 1]));
        r[4 * v + 2] = __float_as_uint(c.z + __uint_as_float(r[4 * v + 2]));
        r[4 * v + 3] = __float_as_uint(c.w + __uint_as_float(r[4 * v + 3]));
      }
    }
    if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {  // 32-byte stores: one sector each
#pragma unroll
      for (int v = 0; v < 4; ++v) st_global_v8(dst + 8 * v, &r[8 * v]);
    } else {
#pragma unroll
      for (int v = 0; v < 8; ++v) st_global_v4(dst + 4 * v, r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
    }
  } else {
    for (int i = 0; i < 32; ++i)
      if (i < valid) dst[i] = accumulate ? dst[i] + __uint_as_float(r[i]) : __uint_as_float(r[i]);
  }
}

template <int kElemBytes, Mainloop kML, Epi kEpi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs a) {
  constexpr int BK = kGemmRowBytes / kElemBytes;  // elements of K per stage (64 fp16 / 128 e4m3)
  constexpr int MMA_K = 32 / kElemBytes;          // K per tcgen05.mma (16 fp16 / 32 e4m3)
  constexpr int K_STEPS = BK / MMA_K;             // 4
  constexpr bool kMNB = (kML != Mainloop::Dense);  // B operand MN-major (row-major [K,N] source or blocks)
  constexpr uint32_t IDESC = ptx::instr_desc(kGemmBM, kGemmBN, 0, 0, 0, kMNB ? 1 : 0);
  constexpr uint32_t STAGE_TX = kGemmAStage + kGemmBStage;
  constexpr int BSR_STEPS = 128 / BK;             // stages per 128-wide nonzero block
  constexpr uint32_t KID = kML == Mainloop::Bsr      ? kKidSpmmBsr
                           : kML == Mainloop::BsrBsr ? kKidSpmmBsrBsr
                                                     : (kElemBytes == 1 ? kKidGemmE4m3 : kKidGemmF16);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kGemmStages * kGemmAStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kGemmStages * kGemmBStage);
  uint64_t* full = bars;
  uint64_t* empty = bars + kGemmStages;
  uint64_t* tfull = bars + 2 * kGemmStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      ptx::mbar_init(ptx::smem_u32(&full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(ptx::smem_u32(&tfull[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&tempty[s]), 4);
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
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), kGemmTmemCols);
    ptx::tmem_relinquish();
  }
  // BSR x BSR: stage B's block map in shared memory (all threads; one global read per stored block).
  const int* btab = nullptr;
  if constexpr (kML == Mainloop::BsrBsr) {
    if (a.b_nbc > 0) {
      int* tab = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bars) + 256);
      int* rp = tab + kBsrTableMax;  // B row pointers, clamped to [0, b_nnzb]
      const int entries = a.kb_count * a.b_nbc;
      for (int i = threadIdx.x; i < entries; i += blockDim.x) tab[i] = -1;
      for (int i = threadIdx.x; i <= a.kb_count; i += blockDim.x) rp[i] = min(max(__ldg(&a.b_row_ptr[i]), 0), a.b_nnzb);
      __syncthreads();
      for (int p = threadIdx.x; p < a.b_nnzb; p += blockDim.x) {
        int lo = 0, hi = a.kb_count;  // block-row of stored block p: the last kb with rp[kb] <= p
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (rp[mid] <= p) lo = mid; else hi = mid - 1;
        }
        const int col = __ldg(&a.b_col_idx[p]);
        if (lo < a.kb_count && p < rp[lo + 1] && col >= 0 && col < a.b_nbc) tab[lo * a.b_nbc + col] = p;
      }
      btab = tab;
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  WaitCtl ctl{abort_flag, a.err, a.timeout_ns, KID};
  const int num_tiles = a.num_m_tiles * a.num_n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    uint32_t stage = 0, phase = 0;
    uint32_t issued = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int mt, nt;
      gemm_tile_coords(tile, a, mt, nt);
      const int n0 = nt * kGemmBN;
      if constexpr (kML == Mainloop::Dense) {
        const int m0 = mt * kGemmBM;
        for (int kb = 0; kb < a.num_k_blocks; ++kb) {
          ok = warp_wait_bounded(ptx::smem_u32(&empty[stage]), phase ^ 1, ctl, 1);
          if (!ok) break;
          if (lane == 0) {
            const uint32_t fb = ptx::smem_u32(&full[stage]);
            ptx::mbar_arrive_expect_tx(fb, STAGE_TX);
            ptx::tma_load_2d(ptx::smem_u32(sA + stage * kGemmAStage), &tmA, fb, kb * BK, m0);
            ptx::tma_load_2d(ptx::smem_u32(sB + stage * kGemmBStage), &tmB, fb, kb * BK, n0);
          }
          ++issued;
          if (++stage == kGemmStages) { stage = 0; phase ^= 1; }
        }
      } else if constexpr (kML == Mainloop::BsrBsr) {
        const int r = a.row_begin + mt;
        const int jc = n0 / 128;
        int j0, j1;
        if (!bsr_row_range(a, r, j0, j1) && lane == 0) atomicCAS(a.err, 0u, kErrBounds | (KID << 8) | (7u << 16));
        for (int jb = j0; jb < j1 && ok; jb += 32) {
          // each lane resolves the B pair of one of the next 32 A blocks; then the warp walks them in order
          int p0 = -1, p1 = -1;
          bool on = false;
          if (jb + lane < j1) {
            on = bsrbsr_pair(a, btab, jb + lane, jc, p0, p1);
            const int kb = __ldg(&a.col_idx[jb + lane]);
            if (kb < 0 || kb >= a.kb_count) atomicCAS(a.err, 0u, kErrBounds | (KID << 8) | (8u << 16));
          }
          unsigned live = __ballot_sync(0xFFFFFFFFu, on);
          while (live && ok) {
            const int jj = __ffs(live) - 1;
            live &= live - 1;
            const int q0 = __shfl_sync(0xFFFFFFFFu, p0, jj);
            const int q1 = __shfl_sync(0xFFFFFFFFu, p1, jj);
            const int r0 = (q0 >= 0 ? q0 : a.b_nnzb) * 128, r1 = (q1 >= 0 ? q1 : a.b_nnzb) * 128;
            for (int s = 0; s < BSR_STEPS; ++s) {
              ok = warp_wait_bounded(ptx::smem_u32(&empty[stage]), phase ^ 1, ctl, 1);
              if (!ok) break;
              if (lane == 0) {
                const uint32_t fb = ptx::smem_u32(&full[stage]);
                ptx::mbar_arrive_expect_tx(fb, kGemmAStage + (q0 >= 0 ? kGemmBStage / 2 : 0) +
                                                   (q1 >= 0 ? kGemmBStage / 2 : 0));
                ptx::tma_load_2d(ptx::smem_u32(sA + stage * kGemmAStage), &tmA, fb, s * BK, (jb + jj) * 128);
                // B: K rows [s*BK, +BK) of block (kb, jc) -> columns [0,128) and of (kb, jc+1) -> [128,256) of the
                // tile; only the blocks that exist are loaded (the MMA warp skips the other half)
                const uint32_t bdst = ptx::smem_u32(sB + stage * kGemmBStage);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  if ((q < 2 ? q0 : q1) >= 0)
                    ptx::tma_load_2d(bdst + q * (BK * 128), &tmB, fb, (q & 1) * 64, (q < 2 ? r0 : r1) + s * BK);
              }
              ++issued;
              if (++stage == kGemmStages) { stage = 0; phase ^= 1; }
            }
          }
        }
      } else {
        const int r = a.row_begin + mt;
        int j0, j1;
        if (!bsr_row_range(a, r, j0, j1) && lane == 0) atomicCAS(a.err, 0u, kErrBounds | (KID << 8) | (7u << 16));
        for (int jb = j0; jb < j1 && ok; jb += 32) {
          // warp-level prefetch of the next 32 column indices of this block-row
          const int cidx = (jb + lane < j1) ? __ldg(&a.col_idx[jb + lane]) : 0;
          const int cnt = min(32, j1 - jb);
          for (int jj = 0; jj < cnt && ok; ++jj) {
            int kblk = __shfl_sync(0xffffffffu, cidx, jj);
            if (kblk < 0 || kblk >= a.kb_count) {  // out-of-range column: flag it; the load reads zero fill
              if (lane == 0) atomicCAS(a.err, 0u, kErrBounds | (KID << 8) | (8u << 16));
              kblk = a.kb_count;
            }
            for (int s = 0; s < BSR_STEPS; ++s) {
              ok = warp_wait_bounded(ptx::smem_u32(&empty[stage]), phase ^ 1, ctl, 1);
              if (!ok) break;
              if (lane == 0) {
                const uint32_t fb = ptx::smem_u32(&full[stage]);
                ptx::mbar_arrive_expect_tx(fb, STAGE_TX);
                // A: nonzero block (jb+jj), K slice s -> 128 rows x 128 B, K-major
                ptx::tma_load_2d(ptx::smem_u32(sA + stage * kGemmAStage), &tmA, fb, s * BK, (jb + jj) * 128);
                // B: rows [kblk*128 + s*BK, +BK) of B[K,N], 4 slabs of 64 columns (MN-major atoms)
                const uint32_t bdst = ptx::smem_u32(sB + stage * kGemmBStage);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  ptx::tma_load_2d(bdst + q * (BK * 128), &tmB, fb, n0 + q * 64, kblk * 128 + s * BK);
              }
              ++issued;
              if (++stage == kGemmStages) { stage = 0; phase ^= 1; }
            }
          }
        }
      }
    }
    // Drain: every load this warp issued must have landed before the CTA may exit.
    if (lane == 0) {
      const uint32_t first = issued > kGemmStages ? issued - kGemmStages : 0;
      for (uint32_t i = first; i < issued; ++i) {
        WaitCtl dctl = ctl;
        volatile int never = 0;
        dctl.abort = &never;
        wait_bounded(ptx::smem_u32(&full[i % kGemmStages]), (i / kGemmStages) & 1, dctl, 2);
      }
    }
    __syncwarp();
  } else if (warp == 1 && kML == Mainloop::BsrBsr) {
    // ------------------------------------------------------------------ MMA issuer, BSR x BSR
    // The warp counts each tile's contributing A blocks together (lookups of B); lane 0 issues the MMAs.
    uint32_t stage = 0, phase = 0;
    uint32_t acc = 0, acc_phase = 0;
    bool ok = true;
    const uint32_t full0 = ptx::smem_u32(full), empty0 = ptx::smem_u32(empty);
    const uint32_t tfull0 = ptx::smem_u32(tfull), tempty0 = ptx::smem_u32(tempty);
    const uint64_t adesc0 = ptx::smem_desc(ptx::smem_u32(sA), 16, 1024);
    const uint64_t bdesc0 = ptx::smem_desc(ptx::smem_u32(sB), BK * 128, 1024);
    constexpr uint32_t B_KSTEP = (MMA_K * 128) >> 4;
    constexpr uint32_t IDESC_HALF = ptx::instr_desc(kGemmBM, 128, 0, 0, 0, 1);  // one B block: N = 128
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mt, nt;
      gemm_tile_coords(tile, a, mt, nt);
      int j0, j1;
      bsr_row_range(a, a.row_begin + mt, j0, j1);
      const int jc = nt * kGemmBN / 128;
      if (lane == 0) {
        ok = wait_bounded(tempty0 + acc * 8, acc_phase ^ 1, ctl, 3);
        if (ok) ptx::tc_fence_after();
      }
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      const uint32_t d_tmem = tmem_base + acc * kGemmBN;
      bool init0 = false, init1 = false;  // lane 0: the tile's half has received its first (overwriting) MMA
      // Blocks in the producer's order: ascending within each group of 32; per block, an N = 128 MMA for each
      // B block that exists (column half 0 <- (kb, jc), half 1 <- (kb, jc + 1)).
      for (int jb = j0; jb < j1 && ok; jb += 32) {
        int p0 = -1, p1 = -1;
        if (jb + lane < j1) bsrbsr_pair(a, btab, jb + lane, jc, p0, p1);
        const unsigned h0 = __ballot_sync(0xFFFFFFFFu, p0 >= 0), h1 = __ballot_sync(0xFFFFFFFFu, p1 >= 0);
        if (lane == 0) {
          unsigned live = h0 | h1;
          while (live && ok) {
            const int jj = __ffs(live) - 1;
            live &= live - 1;
            const bool has0 = (h0 >> jj) & 1u, has1 = (h1 >> jj) & 1u;
            for (int s = 0; s < BSR_STEPS && ok; ++s) {
              ok = wait_bounded(full0 + stage * 8, phase, ctl, 4);
              if (!ok) break;
              ptx::tc_fence_after();
              const uint64_t ad = adesc0 + ((stage * kGemmAStage) >> 4);
              const uint64_t bd = bdesc0 + ((stage * kGemmBStage) >> 4);
#pragma unroll
              for (int k = 0; k < K_STEPS; ++k) {
                if (has0) ptx::mma_f16_ss(d_tmem, ad + k * 2, bd + k * B_KSTEP, IDESC_HALF, (init0 || k) ? 1u : 0u);
                if (has1)
                  ptx::mma_f16_ss(d_tmem + 128, ad + k * 2, bd + ((2 * BK * 128) >> 4) + k * B_KSTEP, IDESC_HALF,
                                  (init1 || k) ? 1u : 0u);
              }
              init0 = init0 || has0;
              init1 = init1 || has1;
              ptx::mma_commit(empty0 + stage * 8);
              if (++stage == kGemmStages) { stage = 0; phase ^= 1; }
            }
          }
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      }
      if (!ok) break;
      if (lane == 0) {
        ptx::mma_commit(tfull0 + acc * 8);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      __syncwarp();
    }
    if (lane == 0) {  // all MMAs this thread issued complete before TMEM is released
      ptx::mma_commit(ptx::smem_u32(drain));
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      wait_bounded(ptx::smem_u32(drain), 0, dctl, 5);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t acc = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t full0 = ptx::smem_u32(full), empty0 = ptx::smem_u32(empty);
      const uint32_t tfull0 = ptx::smem_u32(tfull), tempty0 = ptx::smem_u32(tempty);
      // Descriptors differ only in the start-address field: build once, add the offset (>> 4).
      const uint64_t adesc0 = ptx::smem_desc(ptx::smem_u32(sA), 16, 1024);
      const uint64_t bdesc0 = kMNB ? ptx::smem_desc(ptx::smem_u32(sB), BK * 128, 1024)
                                   : ptx::smem_desc(ptx::smem_u32(sB), 16, 1024);
      constexpr uint32_t B_KSTEP = kMNB ? (MMA_K * 128) >> 4 : 2;  // +16 rows (MN-major) or +32 B (K-major)
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mt, nt;
        gemm_tile_coords(tile, a, mt, nt);
        int nk;
        if constexpr (kML == Mainloop::Dense) {
          nk = a.num_k_blocks;
        } else {
          int j0, j1;
          bsr_row_range(a, a.row_begin + mt, j0, j1);
          nk = (j1 - j0) * BSR_STEPS;
        }
        ok = wait_bounded(tempty0 + acc * 8, acc_phase ^ 1, ctl, 3);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kGemmBN;
        for (int kb = 0; kb < nk; ++kb) {
          ok = wait_bounded(full0 + stage * 8, phase, ctl, 4);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint64_t ad = adesc0 + ((stage * kGemmAStage) >> 4);
          const uint64_t bd = bdesc0 + ((stage * kGemmBStage) >> 4);
#pragma unroll
          for (int k = 0; k < K_STEPS; ++k) {
            if constexpr (kElemBytes == 1)
              ptx::mma_f8_ss(d_tmem, ad + k * 2, bd + k * B_KSTEP, IDESC, (kb | k) != 0);
            else
              ptx::mma_f16_ss(d_tmem, ad + k * 2, bd + k * B_KSTEP, IDESC, (kb | k) != 0);
          }
          ptx::mma_commit(empty0 + stage * 8);
          if (++stage == kGemmStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        ptx::mma_commit(tfull0 + acc * 8);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // Drain: all MMAs this thread issued complete before TMEM is released.
      ptx::mma_commit(ptx::smem_u32(drain));
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      wait_bounded(ptx::smem_u32(drain), 0, dctl, 5);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;
    uint32_t acc = 0, acc_phase = 0;
    float scale = 1.0f;
    if constexpr (kEpi == Epi::BF16Scaled) scale = __ldg(a.scale_a) * __ldg(a.scale_b);
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mt, nt;
      gemm_tile_coords(tile, a, mt, nt);
      int m0, nk = 1, nk1 = 1;  // nk1: MMAs into the second 128-column half (BSR x BSR), else unused
      if constexpr (kML == Mainloop::Dense) {
        m0 = mt * kGemmBM;
      } else {
        const int r = a.row_begin + mt;
        m0 = r * kGemmBM;
        int j0, j1;
        bsr_row_range(a, r, j0, j1);
        if constexpr (kML == Mainloop::BsrBsr)
          bsrbsr_half_counts(a, btab, j0, j1, nt * kGemmBN / 128, &nk, &nk1);
        else
          nk = nk1 = j1 - j0;
      }
      const int n0 = nt * kGemmBN;
      if (!warp_wait_bounded(ptx::smem_u32(&tfull[acc]), acc_phase, ctl, 6)) break;
      ptx::tc_fence_after();
      const int row = m0 + 32 * q + lane;
      const bool row_ok = row < a.M;
      const uint32_t t_row = tmem_base + acc * kGemmBN + (static_cast<uint32_t>(32 * q) << 16);
#pragma unroll 1
      for (int c = 0; c < kGemmBN; c += 32) {
        uint32_t r[32];
        __syncwarp();
        if ((c < 128 ? nk : nk1) > 0) {  // a half no MMA wrote holds stale values: it is zero
          ptx::tmem_ld_32x32b_x32(t_row + c, r);
          ptx::tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
        const int col0 = n0 + c;
        if (row_ok) {
        if constexpr (kEpi == Epi::F32) {
          float* dst = reinterpret_cast<float*>(a.out) + static_cast<int64_t>(row) * a.ldo + col0;
          store_row32_f32(dst, r, a.vec_ok && col0 + 32 <= a.N, a.N - col0, a.accumulate);
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
                const unsigned short hb = (i & 1) ? static_cast<unsigned short>(w >> 16)
                                                  : static_cast<unsigned short>(w & 0xFFFF);
                reinterpret_cast<unsigned short*>(dst)[i] = hb;
              }
          }
        }
        }  // row_ok
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&tempty[acc]));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem_base, kGemmTmemCols);
}

}  // namespace bsk
