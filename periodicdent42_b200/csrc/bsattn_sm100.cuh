// Block-sparse attention forward for sm_100a (fp16 / bf16 in and out, fp32 online softmax), 128x128 blocks,
// head dim 64 or 128.
//
// Work item = one query block-row of one (b, h) pair (head-major; the longest rows of a causal pattern first). For
// every nonzero key block j of the row's mask the CTA computes
//     S_j = Q K_j^T                 tcgen05.mma 128x128x16 x (D/16) into TMEM S buffer j % 2
//     P_j = exp2(S_j * c - m)       online softmax, one query row per thread pair; P (16-bit) is written back into
//                                   the S buffer (tcgen05.st): keys 0-63 in columns [0, 32), 64-127 in [64, 96)
//     O  += P_j V_j                 tcgen05.mma with A = P from TMEM, V an MN-major shared-memory operand
// and writes O / l. Only nonzero blocks are loaded (TMA through a 5-slot K/V ring).
//
// Why this shape: one thread issues a 128x128x16 tcgen05.mma only every ~115-160 SM cycles while the tensor pipe
// finishes it in 64, and two to four issuing warps bring the aggregate back to 68-84 cycles (measured on B200). So
// the S MMAs and the PV MMAs have an issuing thread each (warps 1 and 2), and S is double-buffered in TMEM, so
// S_{j+1} is computed while the softmax of block j runs. The softmax itself is split across two warps per row: warps
// 4-7 take keys 0-63, warps 8-11 keys 64-127 of the rows of their TMEM lane quarter, and exchange each row's partial
// max through the last S column of their key range (63, 127: already loaded, not overwritten by P). A cycle trace of
// this kernel on the attention workload puts a block at ~2000-2250 SM cycles, set by the softmax (TMEM load ~250, max
// ~200, exchange ~300-550, exponentials ~950 -- the MUFU of a sub-partition shared by the two halves -- and ~200 per
// barrier wait), against 1024 cycles of tensor work; the first two blocks of a row take ~2500 cycles more (a per-row
// cost of ~3300 cycles in total from a sweep of blocks per row, while the output warps write the previous row).
// Variants measured slower on B200: speculative exponentials before the exchange (735 vs 890 TFLOPS), P in its own
// TMEM buffers with the exchange in shared memory and one Q buffer (832 vs 887), independent halves with one O
// accumulator each (no exchange; P aliased onto S, so S_{j+2} waits for PV_j: 850 vs 876), and both halves loading
// the whole S row to take the max without an exchange, P in its own TMEM buffers so S_{j+2} only waits for S_j to be
// loaded (790 vs 917: the S row is read from TMEM twice, and the longer load costs more than the exchange it
// removes), and suspend-hint waits (try_wait with a time hint) for the MMA issuers (872 vs 884) or for the issuers
// and the softmax warps (867 vs 884): the re-polling waits stay. Two blocks per softmax step (warps 4-7 take block
// 2t, warps 8-11 block 2t+1, each thread a whole 128-column row, the two blocks' maxima exchanged once per pair, P in
// its own TMEM columns) ran at 744 vs 888: 128 live scores per thread spill under the 176-register cap and the two
// warps of a sub-partition still run their exponentials in lockstep. The MUFU computes 16 exp2 per clock per SM in
// the f32, f16x2 and bf16x2 forms alike (measured), so packed exponentials do not raise that ceiling. Output warps
// reading O 64 columns per TMEM round trip (903 vs 920), a non-blocking test of the next block's S before the P store
// (914 vs 920), pacing the output warps' stores (within 0.5 %), loading the next row's column indices during a row's
// first block (901 vs 923) and exchanging bf16 maxima through the 1 KB of shared memory that the alignment pad would
// take (920 vs 928) were no better.
//
// Roles (16 warps): warp 0 TMA producer, warp 1 TMEM owner + S issuer, warp 2 PV issuer, warp 3 idle, warps 4-11
// softmax, warps 12-15 output (O / l from TMEM to global once a row's last PV completed, so the softmax warps go
// straight on to the next row). TMEM: S buffers [0,128) and [128,256), O of alternate rows [256, 256 + D) and
// [384, 384 + D), so the first PV of a row never waits for the output warps to read the previous row's O (+1.3 %
// on the attention workload). Each output thread writes its row of O with 32-byte stores (one sector each): its
// stores run beside the softmax warps' shared-memory barrier traffic, and with 16-byte stores the output of a row
// cost ~5 % of the kernel time (measured by leaving the stores out), with 32-byte stores ~2.5 % (staging the tile
// in the row's freed Q buffer for a TMA store measured the same). Shared memory: Q x 2, the K/V ring, barriers,
// and the row sums / maxima handed to the output warps.
//
// Softmax: the reference max moves only when a block raises it by more than 8 (log2 units), so P <= 2^8 and O is
// rescaled in TMEM only on those moves. Scale, sums and the polynomial use packed fp32x2 FMA/ADD; row max uses
// three-input max. exp2 runs on the MUFU for 3/4 of the elements and on the FMA pipe for 1/4 (ex2_poly2 below),
// balancing the MUFU against instruction issue.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx_sm100.cuh"

namespace bsk {

constexpr int kAttnBlk = 128;
constexpr int kAttnThreads = 512;
constexpr int kAttnChunk = kAttnBlk * 64 * 2;  // 16 KB: 128 rows x 64 columns (one 128-B swizzle atom wide)
constexpr int kAttnKVSlots = 5;
// Eighths of the exponentials computed on the FMA pipe (ex2_poly2) instead of the MUFU.
#ifndef BSK_ATTN_POLY_EIGHTHS
#define BSK_ATTN_POLY_EIGHTHS 2
#endif
constexpr int kAttnPolyEighths = BSK_ATTN_POLY_EIGHTHS;

// Head dimension D (64 or 128) and element type (fp16 or bf16) of one instantiation.
template <bool kF16, int kD>
struct AttnShape {
  static_assert(kD == 64 || kD == 128, "head dim 64 or 128");
  static constexpr int kTile = kAttnBlk * kD * 2;  // one 128 x D tile: kD / 64 chunks of 16 KB
  static constexpr int kChunks = kD / 64;
  static constexpr int kSmemBytes = 1024 + kTile * (2 /*Q*/ + kAttnKVSlots) + 512 + 3 * 128 * 4;
  static constexpr uint32_t kFmt = kF16 ? 0u : 1u;  // tcgen05 kind::f16 A/B format: 0 f16, 1 bf16
};
constexpr int kAttnSmemBytes = AttnShape<false, 128>::kSmemBytes;  // largest instantiation
constexpr int kAttnTmemCols = 512;
constexpr uint32_t kAttnTmemO = 256;  // O accumulators of alternate rows: columns [256 + 128 o, +D), o = 0, 1
constexpr uint32_t kAttnRegsLaunch = 128;  // 65536 / 512
constexpr uint32_t kAttnRegsLow = 80;      // producer and MMA issuers
constexpr uint32_t kAttnRegsHigh = 168;    // softmax warpgroups
constexpr uint32_t kAttnRegsOut = 96;      // output warpgroup
static_assert(128 * (kAttnRegsLow + 2 * kAttnRegsHigh + kAttnRegsOut) <= kAttnThreads * kAttnRegsLaunch,
              "setmaxnreg split exceeds the launch allocation");
static_assert(AttnShape<false, 128>::kSmemBytes <= 232448, "shared memory above the 227 KB per-CTA limit");

struct AttnArgs {
  void* O;            // fp16 or bf16 [B*H*S, D]
  float* lse;         // optional [B*H*S]: natural-log log-sum-exp of each row's scaled scores (-inf: empty row)
  const int* row_ptr;
  const int* col_idx;
  int S;              // sequence length
  int nqb;            // S / 128
  int bh_begin;       // first (b,h) pair of this launch
  int num_items;      // (#pairs) * nqb
  float scale_log2;   // softmax scale * log2(e)
  int causal_diag;
  uint32_t* err;
  uint64_t timeout_ns;
};

// Work item -> (bh, query block-row qb, first nonzero j0, nonzero count n). Head-major, so concurrent CTAs share a
// head's K/V in L2; within a head the last rows (the longest of a causal pattern) come first.
__device__ __forceinline__ void attn_row(const AttnArgs& a, int item, int& bh, int& qb, int& j0, int& n) {
  bh = a.bh_begin + item / a.nqb;
  qb = a.nqb - 1 - item % a.nqb;
  const int p = bh * a.nqb + qb;
  j0 = __ldg(&a.row_ptr[p]);
  n = max(__ldg(&a.row_ptr[p + 1]) - j0, 0);
}

// Position of a row's tiles in the K/V ring sequence (t = 0 .. 2n-1 within the row): K_0, then K_j, V_{j-1} for
// j = 1 .. n-1, then V_{n-1}. The producer pushes in this order; each issuer counts through it and takes its own.
__device__ __forceinline__ int attn_k_pos(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int attn_v_pos(int j, int n) { return j == n - 1 ? 2 * n - 1 : 2 * j + 2; }

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32x2 helpers (sm_100 FMA pipe processes both halves in one instruction).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair on the FMA pipe (Cody-Waite split, published FlashAttention-4 approach): x = n + f with
// n = round(x) from the 1.5*2^23 magic addition, f in [-1/2, 1/2], 2^f by a cubic fitted here (constrained
// minimax: 1 + 0.693282906 f + 0.242210542 f^2 + 0.055008705 f^3, max relative error 1.01e-4), and 2^n added
// to the exponent field. Inputs below -125 are clamped (result ~2^-125; only masked elements get there).
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& y0, float& y1) {
  const uint64_t kMagic = f2_pack(12582912.0f, 12582912.0f);
  const uint64_t kNegMagic = f2_pack(-12582912.0f, -12582912.0f);
  const uint64_t xc = f2_pack(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t xr = f2_add(xc, kMagic);        // n in the low mantissa bits
  const uint64_t fl = f2_add(xr, kNegMagic);     // n as a float
  const uint64_t f = f2_fma(fl, f2_pack(-1.0f, -1.0f), xc);
  uint64_t p = f2_fma(f2_pack(0.055008705f, 0.055008705f), f, f2_pack(0.242210542f, 0.242210542f));
  p = f2_fma(p, f, f2_pack(0.693282906f, 0.693282906f));
  p = f2_fma(p, f, f2_pack(1.0f, 1.0f));
  float p0, p1, r0, r1;
  f2_unpack(p, p0, p1);
  f2_unpack(xr, r0, r1);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(r0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(r1) << 23));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <bool kF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return kF16 ? pack_f16(lo, hi) : pack_bf16(lo, hi);
}

template <bool kF16, int kD>
__global__ void __launch_bounds__(kAttnThreads, 1)
    bsattn_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  using Sh = AttnShape<kF16, kD>;
  constexpr int kAttnTile = Sh::kTile;
  constexpr int kHalfD = kD / 2;  // O columns a softmax warp writes
  constexpr uint32_t IDESC_S = ptx::instr_desc(128, 128, Sh::kFmt, Sh::kFmt, 0, 0);  // K = D, both K-major
  constexpr uint32_t IDESC_PV = ptx::instr_desc(128, kD, Sh::kFmt, Sh::kFmt, 0, 1);  // N = D, V MN-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                       // [2] Q of alternate rows
  uint8_t* sKV = sQ + 2 * kAttnTile;        // [kAttnKVSlots]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kAttnKVSlots * kAttnTile);
  uint64_t* q_full = bars + 0;                       // [2]
  uint64_t* q_empty = bars + 2;                      // [2] the row's last S MMAs completed
  uint64_t* kv_full = bars + 4;                      // [kAttnKVSlots]
  uint64_t* kv_empty = kv_full + kAttnKVSlots;       // [kAttnKVSlots]
  uint64_t* s_full = kv_empty + kAttnKVSlots;        // [2] S_j in TMEM buffer j % 2
  uint64_t* s_free = s_full + 2;                     // [2] PV_j completed: buffer j % 2 free, O holds block j
  uint64_t* p_full = s_free + 2;                     // [2] P_j written (8 softmax warps)
  uint64_t* o_done = p_full + 2;                     // [2] last PV of a row into O buffer o completed
  uint64_t* xbar = o_done + 2;                       // [4 quarters][2 slots]: both halves stored their value
  uint64_t* drain = xbar + 8;                        // [2] issuers' final commits
  uint64_t* l_ready = drain + 2;                     // a row's sums and max are in shared memory (8 warps)
  uint64_t* o_free = l_ready + 1;                    // [2] the output warps read O buffer o (4 warps)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(o_free + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  static_assert(4 + 2 * kAttnKVSlots + 2 + 2 + 2 + 2 + 8 + 2 + 1 + 2 <= 63, "barrier area exceeds its 512 bytes");
  float* l_part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 512);  // [2 halves][128 rows]
  float* m_row = l_part + 256;                                                         // [128 rows]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(ptx::smem_u32(&q_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&q_empty[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&s_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&s_free[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&p_full[s]), 8);
      ptx::mbar_init(ptx::smem_u32(&drain[s]), 1);
    }
    for (int s = 0; s < kAttnKVSlots; ++s) {
      ptx::mbar_init(ptx::smem_u32(&kv_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&kv_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(ptx::smem_u32(&o_done[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&o_free[s]), 4);
    }
    ptx::mbar_init(ptx::smem_u32(l_ready), 8);
    for (int s = 0; s < 8; ++s) ptx::mbar_init(ptx::smem_u32(&xbar[s]), 2);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), kAttnTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  WaitCtl ctl{abort_flag, a.err, a.timeout_ns, kKidBsAttn};

  // Launch allocation 512 x 128 registers; warpgroup 0 (producer, issuers, 1 idle warp) drops to kAttnRegsLow per
  // thread and the output warpgroup to kAttnRegsOut, the two softmax warpgroups rise to kAttnRegsHigh (sum checked
  // at compile time).
  static_assert(kAttnThreads == 512, "register split assumes 16 warps");
  if (warp < 4) ptx::setmaxnreg_dec<kAttnRegsLow>();
  if (warp >= 12) ptx::setmaxnreg_dec<kAttnRegsOut>();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (one thread)
    if (lane == 0) {
      uint32_t slot = 0, slot_phase = 0, q_issued = 0, kv_issued = 0;
      bool ok = true;
      const uint32_t kv0 = ptx::smem_u32(sKV);
      auto push = [&](const CUtensorMap* m, int row) -> bool {
        if (!wait_bounded<false, 512>(ptx::smem_u32(&kv_empty[slot]), slot_phase ^ 1, ctl, 2)) return false;
        const uint32_t fb = ptx::smem_u32(&kv_full[slot]);
        const uint32_t dst = kv0 + slot * kAttnTile;
        ptx::mbar_arrive_expect_tx(fb, kAttnTile);
#pragma unroll
        for (int c = 0; c < Sh::kChunks; ++c) ptx::tma_load_2d(dst + c * kAttnChunk, m, fb, 64 * c, row);
        ++kv_issued;
        if (++slot == kAttnKVSlots) { slot = 0; slot_phase ^= 1; }
        return true;
      };
      for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
        int bh, qb, j0, n;
        attn_row(a, item, bh, qb, j0, n);
        if (n == 0) continue;
        const uint32_t qbuf = q_issued & 1;
        ok = wait_bounded<false, 512>(ptx::smem_u32(&q_empty[qbuf]), ((q_issued >> 1) & 1) ^ 1, ctl, 1);
        if (!ok) break;
        const uint32_t qf = ptx::smem_u32(&q_full[qbuf]);
        ptx::mbar_arrive_expect_tx(qf, kAttnTile);
        const int row0 = bh * a.S;
#pragma unroll
        for (int c = 0; c < Sh::kChunks; ++c)
          ptx::tma_load_2d(ptx::smem_u32(sQ) + qbuf * kAttnTile + c * kAttnChunk, &tmQ, qf, 64 * c,
                           row0 + qb * kAttnBlk);
        ++q_issued;
        // key block j of the row -> first row of its K/V tile in the [B*H*S, D] view
        auto kvrow = [&](int j) -> int {
          int kb = __ldg(&a.col_idx[j0 + j]);
          if (kb < 0 || kb >= a.nqb) {  // out-of-range index: flag it; the load reads zero fill
            atomicCAS(a.err, 0u, kErrBounds | (kKidBsAttn << 8) | (7u << 16));
            kb = a.nqb;
          }
          return row0 + kb * kAttnBlk;
        };
        ok = push(&tmK, kvrow(0));
        for (int j = 1; j < n && ok; ++j) {
          ok = push(&tmK, kvrow(j));
          if (ok) ok = push(&tmV, kvrow(j - 1));
        }
        if (ok) ok = push(&tmV, kvrow(n - 1));
      }
      // Drain loads still in flight.
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      for (uint32_t i = q_issued > 2 ? q_issued - 2 : 0; i < q_issued; ++i)
        wait_bounded(ptx::smem_u32(&q_full[i & 1]), (i >> 1) & 1, dctl, 8);
      const uint32_t first = kv_issued > kAttnKVSlots ? kv_issued - kAttnKVSlots : 0;
      for (uint32_t i = first; i < kv_issued; ++i)
        wait_bounded(ptx::smem_u32(&kv_full[i % kAttnKVSlots]), (i / kAttnKVSlots) & 1, dctl, 8);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------------ MMA issuers (one thread each)
    // warp 1: S_j = Q K_j^T into buffer j % 2, once PV_{j-2} has released it; warp 2: O += P_j V_j, once the
    // softmax has written P_j. The two threads' MMAs interleave on the tensor pipe.
    if (lane == 0) {
      const bool s_role = warp == 1;
      uint32_t g = 0, rows = 0, seq = 0;  // blocks, non-empty rows and ring positions passed
      bool ok = true;
      const uint32_t kv0 = ptx::smem_u32(sKV);
      const uint64_t qdesc0 = ptx::smem_desc(ptx::smem_u32(sQ), 16, 1024);  // Q, K: K-major
      const uint64_t kdesc0 = ptx::smem_desc(kv0, 16, 1024);
      const uint64_t vdesc0 = ptx::smem_desc(kv0, kAttnChunk, 1024);       // V: MN-major, 64-column slabs
      for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
        int bh, qb, j0, n;
        attn_row(a, item, bh, qb, j0, n);
        if (n == 0) continue;
        const uint32_t qbuf = rows & 1;
        if (s_role) {
          ok = wait_bounded(ptx::smem_u32(&q_full[qbuf]), (rows >> 1) & 1, ctl, 14);
          if (!ok) break;
        }
        for (int j = 0; j < n && ok; ++j, ++g) {
          const uint32_t b = g & 1;
          if (s_role) {
            if (g >= 2) {  // PV_{g-2} read P from this buffer
              ok = wait_bounded(ptx::smem_u32(&s_free[b]), ((g - 2) >> 1) & 1, ctl, 11);
              if (!ok) break;
            }
            const uint32_t pos = seq + attn_k_pos(j);
            const uint32_t sl = pos % kAttnKVSlots;
            ok = wait_bounded(ptx::smem_u32(&kv_full[sl]), (pos / kAttnKVSlots) & 1, ctl, 12);
            if (!ok) break;
            ptx::tc_fence_after();
            const uint64_t qd = qdesc0 + ((qbuf * kAttnTile) >> 4), kd = kdesc0 + ((sl * kAttnTile) >> 4);
#pragma unroll
            for (int k = 0; k < kD / 16; ++k) {  // K = D in steps of 16: 4 steps per 64-column chunk
              const uint32_t off = ((k >> 2) * kAttnChunk + (k & 3) * 32) >> 4;
              ptx::mma_f16_ss(tmem_base + 128 * b, qd + off, kd + off, IDESC_S, k != 0);
            }
            ptx::mma_commit(ptx::smem_u32(&kv_empty[sl]));
            ptx::mma_commit(ptx::smem_u32(&s_full[b]));
            if (j == n - 1) ptx::mma_commit(ptx::smem_u32(&q_empty[qbuf]));
          } else {
            if (j == 0 && rows > 1) {  // the first PV of a row overwrites O buffer rows % 2: row rows-2's O is read
              ok = wait_bounded(ptx::smem_u32(&o_free[rows & 1]), ((rows >> 1) - 1) & 1, ctl, 17);
              if (!ok) break;
            }
            ok = wait_bounded(ptx::smem_u32(&p_full[b]), (g >> 1) & 1, ctl, 13);
            if (!ok) break;
            const uint32_t pos = seq + attn_v_pos(j, n);
            const uint32_t sl = pos % kAttnKVSlots;
            ok = wait_bounded(ptx::smem_u32(&kv_full[sl]), (pos / kAttnKVSlots) & 1, ctl, 15);
            if (!ok) break;
            ptx::tc_fence_after();
            const uint64_t vd = vdesc0 + ((sl * kAttnTile) >> 4);
            const uint32_t t_o = tmem_base + kAttnTmemO + 128 * (rows & 1), t_p = tmem_base + 128 * b;
#pragma unroll
            for (int k = 0; k < 8; ++k)  // K step k: keys [16k, 16k+16) in P columns 8k (+32 for the second half)
              ptx::mma_f16_ts(t_o, t_p + 8 * k + (k >= 4 ? 32 : 0), vd + ((k * 2048) >> 4), IDESC_PV,
                              (j == 0 && k == 0) ? 0u : 1u);
            ptx::mma_commit(ptx::smem_u32(&kv_empty[sl]));
            ptx::mma_commit(ptx::smem_u32(&s_free[b]));
            if (j == n - 1) ptx::mma_commit(ptx::smem_u32(&o_done[rows & 1]));
          }
        }
        seq += 2 * n;
        ++rows;
      }
      const uint32_t dr = ptx::smem_u32(&drain[s_role ? 0 : 1]);
      ptx::mma_commit(dr);
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      wait_bounded(dr, 0, dctl, 16);
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------------ softmax (warps 4..11)
    ptx::setmaxnreg_inc<kAttnRegsHigh>();
    const int h = (warp - 4) >> 2;  // key half: S columns [64 h, 64 h + 64)
    const int q = warp & 3;         // TMEM lane quarter
    const int r = 32 * q + lane;    // query row within the block == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    const uint32_t tO0 = tmem_base + kAttnTmemO + lane_off + h * kHalfD;  // this warp's O columns (buffer 0)
    const float c = a.scale_log2;
    uint32_t g = 0, rows = 0, x_cnt = 0;
    bool ok = true;
    // Row-wise exchange with the warp of the other key half (same rows): store this half's value in the last column
    // of its own key range of the S buffer (63 or 127: already loaded, and P lands in columns [0, 32) and [64, 96)),
    // meet on the quarter's barrier, read the other half's column. The buffer is rewritten only after PV of this
    // block, which follows both halves' P and so both reads.
    auto exchange = [&](uint32_t tSb, float v, float& other) -> bool {
      const uint32_t slot = x_cnt & 1;
      ptx::tmem_st_32x32b_x1(tSb + 64 * h + 63, __float_as_uint(v));
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      __syncwarp();
      const uint32_t xb = ptx::smem_u32(&xbar[q * 2 + slot]);
      if (lane == 0) ptx::mbar_arrive(xb);
      if (!warp_wait_bounded(xb, (x_cnt >> 1) & 1, ctl, 23)) return false;
      ++x_cnt;
      ptx::tc_fence_after();
      other = __uint_as_float(ptx::tmem_ld_32x32b_x1(tSb + 64 * (h ^ 1) + 63));
      ptx::tmem_wait_ld();
      return true;
    };
    // The next row's bounds are looked up one row ahead (their loads overlap this row's blocks).
    int item = blockIdx.x;
    int bh = 0, qb = 0, j0 = 0, n = 0;
    if (item < a.num_items) attn_row(a, item, bh, qb, j0, n);
    for (; item < a.num_items && ok; item += gridDim.x) {
      const int rbh = bh, rqb = qb, rj0 = j0, rn = n;  // this row; (bh, qb, j0, n) become the next row's
      if (item + static_cast<int>(gridDim.x) < a.num_items) attn_row(a, item + gridDim.x, bh, qb, j0, n);
      const int64_t grow = static_cast<int64_t>(rbh) * a.S + rqb * kAttnBlk + r;
      uint16_t* orow = static_cast<uint16_t*>(a.O) + grow * kD + h * kHalfD;
      if (rn == 0) {
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int cc = 0; cc < kHalfD / 8; ++cc) reinterpret_cast<uint4*>(orow)[cc] = z;
        if (a.lse && h == 0) a.lse[grow] = -INFINITY;
        continue;
      }
      float m_run = -INFINITY, l_run = 0.0f;  // m_run in scaled log2 units; l_run sums this half's keys
      const uint32_t tO = tO0 + 128 * (rows & 1);  // this row's O buffer
      int cidx = 0;  // lane l: column index of nonzero (j & ~31) + l of the row (warp-level prefetch)
      for (int j = 0; j < rn; ++j, ++g) {
        if ((j & 31) == 0) cidx = (j + lane < rn) ? __ldg(&a.col_idx[rj0 + j + lane]) : 0;
        const int kb = __shfl_sync(0xffffffffu, cidx, j & 31);
        const bool diag = a.causal_diag && kb == rqb;
        const uint32_t b = g & 1;
        const uint32_t tS = tmem_base + 128 * b + lane_off;
        ok = warp_wait_bounded(ptx::smem_u32(&s_full[b]), (g >> 1) & 1, ctl, 20);
        if (!ok) break;
        ptx::tc_fence_after();
        uint32_t sv[64];  // this half of the S row, loaded straight into the registers the softmax works in
        ptx::tmem_ld_32x32b_x32(tS + 64 * h, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        ptx::tmem_ld_32x32b_x32(tS + 64 * h + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        ptx::tmem_wait_ld();
        float* v = reinterpret_cast<float*>(sv);
        if (diag) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (64 * h + i > r) v[i] = -INFINITY;
        }
        // Row max as 8 independent partial chains, then the other half's partial max.
        float pm[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) pm[k] = v[k];
#pragma unroll
        for (int i = 8; i < 64; i += 16)
#pragma unroll
          for (int k = 0; k < 8; ++k) pm[k] = max3f(pm[k], v[i + k], v[i + 8 + k]);
        const float mh = max3f(max3f(pm[0], pm[1], pm[2]), max3f(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7]));
        float mo;
        ok = exchange(tS, mh, mo);
        if (!ok) break;
        const float mbs = fmaxf(mh, mo) * c;
        const bool move = mbs > m_run + 8.0f;
        float alpha = 1.0f;
        if (move) alpha = (m_run == -INFINITY) ? 0.0f : ex2_approx(m_run - mbs);
        if (move) m_run = mbs;
        const bool need_rescale = __any_sync(0xffffffffu, move && j > 0);
        const float m_sub = (m_run == -INFINITY) ? 0.0f : m_run;  // fully masked so far: P = 0, no NaN
        // exp2 on pairs: t = s * c - m by fma.f32x2; 3 of every 4 pairs on the MUFU, 1 on the FMA pipe.
        // P is packed to 16-bit pairs in place: pair k lands in sv[k], whose S value (element k <= i) is used.
        const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-m_sub, -m_sub);
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          float t0, t1, e0, e1;
          f2_unpack(f2_fma(f2_pack(v[i], v[i + 1]), c2, nm2), t0, t1);
          if (((i >> 1) & 7) >= 8 - kAttnPolyEighths) {
            ex2_poly2(t0, t1, e0, e1);
          } else {
            e0 = ex2_approx(t0);
            e1 = ex2_approx(t1);
          }
          acc[(i >> 1) & 3] = f2_add(acc[(i >> 1) & 3], f2_pack(e0, e1));
          sv[i >> 1] = pack2<kF16>(e0, e1);
        }
        float rs;
        {
          const uint64_t a01 = f2_add(acc[0], acc[1]), a23 = f2_add(acc[2], acc[3]);
          float lo, hi;
          f2_unpack(f2_add(a01, a23), lo, hi);
          rs = lo + hi;
        }
        l_run = l_run * alpha + rs;
        if (need_rescale) {  // O *= alpha once it holds block j-1 (PV_{g-1} completed), this half's columns
          ok = warp_wait_bounded(ptx::smem_u32(&s_free[(g - 1) & 1]), ((g - 1) >> 1) & 1, ctl, 21);
          if (!ok) break;
          ptx::tc_fence_after();
          const float al = move ? alpha : 1.0f;
#pragma unroll 1
          for (int cc = 0; cc < kHalfD / 32; ++cc) {
            uint32_t u[32];
            ptx::tmem_ld_32x32b_x32(tO + cc * 32, u);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * al);
            ptx::tmem_st_32x32b_x32(tO + cc * 32, u);
          }
        }
        // P of this half (32 packed columns) -> TMEM columns [32 h, 32 h + 32) of the S buffer.
        ptx::tmem_st_32x32b_x32(tS + 64 * h, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&p_full[b]));
      }
      if (!ok) break;
      // Hand this half's row sum (and half 0's max, for the LSE) to the output warps. The previous row's values
      // must have been read first (its O read completes after them).
      if (rows > 0) {
        ok = warp_wait_bounded(ptx::smem_u32(&o_free[(rows - 1) & 1]), ((rows - 1) >> 1) & 1, ctl, 24);
        if (!ok) break;
      }
      l_part[h * 128 + r] = l_run;
      if (h == 0) m_row[r] = m_run;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(l_ready));
      ++rows;
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------------ output (warps 12..15)
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t tO0 = tmem_base + kAttnTmemO + (static_cast<uint32_t>(32 * q) << 16);
    const bool o_v8 = (reinterpret_cast<uintptr_t>(a.O) & 31) == 0;  // rows are multiples of 32 bytes apart
    uint32_t rows = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
      int bh, qb, j0, n;
      attn_row(a, item, bh, qb, j0, n);
      if (n == 0) continue;  // written by the softmax warps
      ok = warp_wait_bounded<false, 256>(ptx::smem_u32(l_ready), rows & 1, ctl, 25);
      if (ok) ok = warp_wait_bounded<false, 256>(ptx::smem_u32(&o_done[rows & 1]), (rows >> 1) & 1, ctl, 22);
      if (!ok) break;
      const uint32_t tO = tO0 + 128 * (rows & 1);
      const uint32_t ob = rows & 1;
      ++rows;
      ptx::tc_fence_after();
      const float l_tot = l_part[r] + l_part[128 + r];  // half 0 + half 1, a fixed order
      const float m_run = m_row[r];
      const int64_t grow = static_cast<int64_t>(bh) * a.S + qb * kAttnBlk + r;
      const float inv_l = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
      // l sums 2^(s*c - m_run) whatever m_run lagged behind, so m_run + log2(l) is exact
      if (a.lse) a.lse[grow] = l_tot > 0.0f ? (m_run + log2f(l_tot)) * 0.6931471805599453f : -INFINITY;
      // O / l in 16 bits, 32-byte stores (one sector each): 32 columns of the row per TMEM load.
      uint16_t* orow = static_cast<uint16_t*>(a.O) + grow * kD;
#pragma unroll 1
      for (int cc = 0; cc < kD / 32; ++cc) {
        uint32_t u[32];
        ptx::tmem_ld_32x32b_x32(tO + cc * 32, u);
        ptx::tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack2<kF16>(__uint_as_float(u[2 * i]) * inv_l, __uint_as_float(u[2 * i + 1]) * inv_l);
        if (o_v8) {
          st_global_v8(orow + cc * 32, pk);
          st_global_v8(orow + cc * 32 + 16, pk + 8);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
          for (int gg = 0; gg < 4; ++gg)
            dst[gg] = make_uint4(pk[4 * gg], pk[4 * gg + 1], pk[4 * gg + 2], pk[4 * gg + 3]);
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&o_free[ob]));
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem_base, kAttnTmemCols);
}

// One warp waits on an mbarrier that nothing completes; the bounded wait runs out, records
// kErrWaitTimeout in the error word and the kernel returns. Used by the failure-detection self-test.
__global__ void wait_probe_kernel(uint32_t* err, uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(&bar), 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncwarp();
  WaitCtl c{&abort_flag, err, timeout_ns, kKidWaitProbe};
  warp_wait_bounded(ptx::smem_u32(&bar), 0, c, 1);
}

// y[i] = 2^x[i] by the softmax's exponential routes, for the accuracy self-test: fma_pipe = 1 takes the
// FMA-pipe polynomial (ex2_poly2, on the pairs (x[2j], x[2j+1]) exactly as the softmax feeds it), 0 the
// MUFU instruction (ex2.approx.ftz). Grid-stride over pairs; an odd tail element is paired with itself.
__global__ void exp2_probe_kernel(const float* __restrict__ x, float* __restrict__ y, int n, int fma_pipe) {
  const int pairs = (n + 1) / 2;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < pairs; j += gridDim.x * blockDim.x) {
    const int i0 = 2 * j, i1 = (2 * j + 1 < n) ? 2 * j + 1 : 2 * j;
    float y0, y1;
    if (fma_pipe) {
      ex2_poly2(x[i0], x[i1], y0, y1);
    } else {
      y0 = ex2_approx(x[i0]);
      y1 = ex2_approx(x[i1]);
    }
    y[i0] = y0;
    if (i1 != i0) y[i1] = y1;
  }
}

}  // namespace bsk
