// Block-sparse attention forward for sm_100a (bf16 in/out, fp32 online softmax), 128x128 blocks, D = 128.
//
// Work item = (b, h) pair and TWO query block-rows of it ("streams" A and B, rows 2t+1 and 2t counted from
// the end, so the longest rows of a causal pattern come first). For every nonzero key block j of a stream's
// mask row the CTA computes
//     S_j = Q K_j^T                 tcgen05.mma 128x128x16 x 8 into the stream's TMEM S buffer
//     P_j = exp2(S_j * c - m)       online softmax, one query row per thread; P (bf16) is written back into
//                                   the first 64 columns of the stream's S buffer in TMEM (tcgen05.st)
//     O  += P_j V_j                 tcgen05.mma with A = P from TMEM, V an MN-major shared-memory operand
// and writes O / l as bf16. Only nonzero blocks are loaded (TMA through a 5-slot K/V ring).
//
// Roles (12 warps): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 4-7 softmax of stream A,
// warps 8-11 softmax of stream B (warp w reads TMEM lanes 32*(w%4)..+31). Per block j the MMA warp issues
// PV_A(j), S_A(j+1), PV_B(j), S_B(j+1): tcgen05.mma ops of one thread execute in issue order, so S_A(j+1) may
// overwrite the TMEM columns PV_A(j) reads, and the two streams interleave so that one stream's softmax
// overlaps the other stream's tensor work. TMEM: S/P_A [0,128), S/P_B [128,256), O_A [256,384), O_B [384,512).
//
// Softmax: the reference max moves only when a block raises it by more than 8 (log2 units), so P <= 2^8 and
// O is rescaled in TMEM only on those moves. Scale, sums and the polynomial use packed fp32x2 FMA/ADD; row
// max uses three-input max. exp2 runs on the MUFU for 3/4 of the elements and on the FMA pipe for 1/4
// (ex2_poly2 below), balancing the MUFU against instruction issue.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx_sm100.cuh"

namespace bsk {

constexpr int kAttnBlk = 128;
constexpr int kAttnThreads = 384;
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
  static constexpr int kSmemBytes = 1024 + kTile * (2 /*Q*/ + kAttnKVSlots) + 256;
  static constexpr uint32_t kFmt = kF16 ? 0u : 1u;  // tcgen05 kind::f16 A/B format: 0 f16, 1 bf16
};
constexpr int kAttnSmemBytes = AttnShape<false, 128>::kSmemBytes;  // largest instantiation
constexpr int kAttnTmemCols = 512;
constexpr uint32_t kAttnRegsLaunch = 168;  // 65536 / 384, rounded down to a multiple of 8
constexpr uint32_t kAttnRegsLow = 112;
constexpr uint32_t kAttnRegsHigh = 184;
static_assert(128 * kAttnRegsLow + 256 * kAttnRegsHigh <= kAttnThreads * kAttnRegsLaunch,
              "setmaxnreg split exceeds the launch allocation");

struct AttnArgs {
  void* O;            // fp16 or bf16 [B*H*S, D]
  float* lse;         // optional [B*H*S]: natural-log log-sum-exp of each row's scaled scores (-inf: empty row)
  const int* row_ptr;
  const int* col_idx;
  int S;              // sequence length
  int nqb;            // S / 128
  int items_per_pair; // ceil(nqb / 2)
  int bh_begin;       // first (b,h) pair of this launch
  int num_items;      // (#pairs) * items_per_pair
  float scale_log2;   // softmax scale * log2(e)
  int causal_diag;
  uint32_t* err;
  uint64_t timeout_ns;
};

struct AttnStream {
  int qb;  // query block-row (-1: no row)
  int j0;  // first nonzero of the row
  int n;   // nonzero blocks of the row
};

// Work item -> (bh, two query block-rows). Head-major, so concurrent CTAs share a head's K/V in L2.
__device__ __forceinline__ void attn_item(const AttnArgs& a, int item, int& bh, AttnStream& sa, AttnStream& sb) {
  bh = a.bh_begin + item / a.items_per_pair;
  const int t = item % a.items_per_pair;
  sa.qb = a.nqb - 1 - 2 * t;
  sb.qb = a.nqb - 2 - 2 * t;
  const int pa = bh * a.nqb + sa.qb;
  sa.j0 = __ldg(&a.row_ptr[pa]);
  sa.n = __ldg(&a.row_ptr[pa + 1]) - sa.j0;
  if (sb.qb >= 0) {
    sb.j0 = __ldg(&a.row_ptr[pa - 1]);
    sb.n = sa.j0 - sb.j0;
  } else {
    sb.j0 = 0;
    sb.n = 0;
  }
  sa.n = max(sa.n, 0);
  sb.n = max(sb.n, 0);
}

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

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <bool kF16, int kD>
__global__ void __launch_bounds__(kAttnThreads, 1)
    bsattn_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  using Sh = AttnShape<kF16, kD>;
  constexpr int kAttnTile = Sh::kTile;
  constexpr uint32_t IDESC_S = ptx::instr_desc(128, 128, Sh::kFmt, Sh::kFmt, 0, 0);  // K = D, both K-major
  constexpr uint32_t IDESC_PV = ptx::instr_desc(128, kD, Sh::kFmt, Sh::kFmt, 0, 1);  // N = D, V MN-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                       // [2] Q_A, Q_B
  uint8_t* sKV = sQ + 2 * kAttnTile;        // [kAttnKVSlots]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kAttnKVSlots * kAttnTile);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;                 // [3]
  uint64_t* kv_empty = bars + 2 + kAttnKVSlots;  // [3]
  uint64_t* s_full = bars + 2 + 2 * kAttnKVSlots;  // [2] per stream: S_j in TMEM
  uint64_t* p_full = s_full + 2;                   // [2] P_j written to TMEM (4 warp arrivals)
  uint64_t* o_done = p_full + 2;                   // [2] last PV of the stream's row completed
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(q_full), 1);
    ptx::mbar_init(ptx::smem_u32(q_empty), 1);
    for (int s = 0; s < kAttnKVSlots; ++s) {
      ptx::mbar_init(ptx::smem_u32(&kv_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&kv_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(ptx::smem_u32(&s_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&p_full[s]), 4);
      ptx::mbar_init(ptx::smem_u32(&o_done[s]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(drain), 1);
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

  // Launch allocation 384 x 168 = 64512 registers; warpgroup 0 (producer, MMA, 2 idle warps) drops to
  // kAttnRegsLow per thread, the two softmax warpgroups rise to kAttnRegsHigh (sum checked at compile time).
  static_assert(kAttnThreads == 384, "register split assumes 12 warps");
  if (warp < 4) ptx::setmaxnreg_dec<kAttnRegsLow>();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (one thread)
    if (lane == 0) {
      uint32_t q_phase = 0, slot = 0, slot_phase = 0, q_issued = 0, kv_issued = 0;
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
      // key block j of a stream -> first row of its K/V tile in the [B*H*S, D] view
      auto kvrow = [&](int bh, const AttnStream& st, int j) -> int {
        int kb = __ldg(&a.col_idx[st.j0 + j]);
        if (kb < 0 || kb >= a.nqb) {  // out-of-range index: flag it; the load reads zero fill
          atomicCAS(a.err, 0u, kErrBounds | (kKidBsAttn << 8) | (7u << 16));
          kb = a.nqb;
        }
        return bh * a.S + kb * kAttnBlk;
      };
      for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
        int bh;
        AttnStream A, B;
        attn_item(a, item, bh, A, B);
        if (A.n + B.n == 0) continue;
        ok = wait_bounded<false, 512>(ptx::smem_u32(q_empty), q_phase ^ 1, ctl, 1);
        if (!ok) break;
        const uint32_t qf = ptx::smem_u32(q_full);
        ptx::mbar_arrive_expect_tx(qf, (A.n > 0 ? kAttnTile : 0) + (B.n > 0 ? kAttnTile : 0));
        const int row0 = bh * a.S;
#pragma unroll
        for (int c = 0; c < Sh::kChunks; ++c) {
          if (A.n > 0)
            ptx::tma_load_2d(ptx::smem_u32(sQ) + c * kAttnChunk, &tmQ, qf, 64 * c, row0 + A.qb * kAttnBlk);
          if (B.n > 0)
            ptx::tma_load_2d(ptx::smem_u32(sQ) + kAttnTile + c * kAttnChunk, &tmQ, qf, 64 * c,
                             row0 + B.qb * kAttnBlk);
        }
        ++q_issued;
        q_phase ^= 1;
        // Same order as the MMA warp consumes: K_A0, K_B0, then per j: V_A(j), K_A(j+1), V_B(j), K_B(j+1).
        if (A.n > 0) ok = ok && push(&tmK, kvrow(bh, A, 0));
        if (B.n > 0) ok = ok && push(&tmK, kvrow(bh, B, 0));
        const int n = max(A.n, B.n);
        for (int j = 0; j < n && ok; ++j) {
          if (j < A.n) ok = ok && push(&tmV, kvrow(bh, A, j));
          if (j + 1 < A.n) ok = ok && push(&tmK, kvrow(bh, A, j + 1));
          if (j < B.n) ok = ok && push(&tmV, kvrow(bh, B, j));
          if (j + 1 < B.n) ok = ok && push(&tmK, kvrow(bh, B, j + 1));
        }
      }
      // Drain loads still in flight.
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      if (q_issued) wait_bounded(ptx::smem_u32(q_full), (q_issued - 1) & 1, dctl, 8);
      const uint32_t first = kv_issued > kAttnKVSlots ? kv_issued - kAttnKVSlots : 0;
      for (uint32_t i = first; i < kv_issued; ++i)
        wait_bounded(ptx::smem_u32(&kv_full[i % kAttnKVSlots]), (i / kAttnKVSlots) & 1, dctl, 8);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      uint32_t q_phase = 0, slot = 0, slot_phase = 0;
      uint32_t p_uses[2] = {0, 0};
      bool ok = true;
      const uint32_t sQa = ptx::smem_u32(sQ), kv0 = ptx::smem_u32(sKV);
      const uint64_t qdesc0 = ptx::smem_desc(sQa, 16, 1024);              // Q, K: K-major
      const uint64_t kvdesc_k0 = ptx::smem_desc(kv0, 16, 1024);
      const uint64_t kvdesc_v0 = ptx::smem_desc(kv0, kAttnChunk, 1024);   // V: MN-major, 64-column slabs
      auto advance = [&]() {
        if (++slot == kAttnKVSlots) { slot = 0; slot_phase ^= 1; }
      };
      // A shared-memory access (an mbarrier poll included) issued after tcgen05.mma waits until the queued MMAs
      // have been handed to the tensor pipe, so the pipe runs dry during every poll that follows an MMA group.
      // The barrier waits of a block are therefore made back to back, before its MMAs: PV_x(j) and S_x(j+1)
      // go out as one group of 16 behind one burst of waits (P_x(j), V_x(j), K_x(j+1)).
      auto s_mmas = [&](int x, uint32_t sl) {  // S_x = Q_x K^T from ring slot sl
        const uint64_t qd = qdesc0 + ((x * kAttnTile) >> 4), kd = kvdesc_k0 + ((sl * kAttnTile) >> 4);
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {  // K = D in steps of 16: 4 steps per 64-column chunk
          const uint32_t off = ((k >> 2) * kAttnChunk + (k & 3) * 32) >> 4;
          ptx::mma_f16_ss(tmem_base + x * 128, qd + off, kd + off, IDESC_S, k != 0);
        }
      };
      auto issue_s = [&](int x) -> bool {  // S_x(0) of a row
        const uint32_t sk = slot;
        if (!wait_bounded(ptx::smem_u32(&kv_full[sk]), slot_phase, ctl, 11)) return false;
        advance();
        ptx::tc_fence_after();
        s_mmas(x, sk);
        ptx::mma_commit(ptx::smem_u32(&kv_empty[sk]));
        ptx::mma_commit(ptx::smem_u32(&s_full[x]));
        return true;
      };
      // O_x += P_x(j) V_x(j) (P from TMEM), then (next) S_x(j+1), which may overwrite the P columns: in issue order.
      auto issue_pv_s = [&](int x, bool first, bool last, bool next) -> bool {
        if (!wait_bounded(ptx::smem_u32(&p_full[x]), p_uses[x] & 1, ctl, 12)) return false;
        ++p_uses[x];
        const uint32_t sv = slot;
        if (!wait_bounded(ptx::smem_u32(&kv_full[sv]), slot_phase, ctl, 13)) return false;
        advance();
        uint32_t sk = 0;
        if (next) {
          sk = slot;
          if (!wait_bounded(ptx::smem_u32(&kv_full[sk]), slot_phase, ctl, 11)) return false;
          advance();
        }
        ptx::tc_fence_after();
        const uint64_t vd = kvdesc_v0 + ((sv * kAttnTile) >> 4);
#pragma unroll
        for (int k = 0; k < 8; ++k)  // K step k: P columns [8k, 8k+8) hold kv positions [16k, 16k+16)
          ptx::mma_f16_ts(tmem_base + 256 + x * 128, tmem_base + x * 128 + 8 * k, vd + ((k * 2048) >> 4), IDESC_PV,
                          (first && k == 0) ? 0u : 1u);
        ptx::mma_commit(ptx::smem_u32(&kv_empty[sv]));
        if (last) ptx::mma_commit(ptx::smem_u32(&o_done[x]));
        if (next) {
          s_mmas(x, sk);
          ptx::mma_commit(ptx::smem_u32(&kv_empty[sk]));
          ptx::mma_commit(ptx::smem_u32(&s_full[x]));
        }
        return true;
      };
      for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
        int bh;
        AttnStream A, B;
        attn_item(a, item, bh, A, B);
        if (A.n + B.n == 0) continue;
        ok = wait_bounded(ptx::smem_u32(q_full), q_phase, ctl, 14);
        if (!ok) break;
        q_phase ^= 1;
        // Ring order (the producer's): K_A(0), K_B(0), then per j: V_A(j), K_A(j+1), V_B(j), K_B(j+1).
        if (A.n > 0) ok = ok && issue_s(0);
        if (B.n > 0) ok = ok && issue_s(1);
        const int n = max(A.n, B.n);
        for (int j = 0; j < n && ok; ++j) {
          if (j < A.n) ok = ok && issue_pv_s(0, j == 0, j + 1 == A.n, j + 1 < A.n);
          if (j < B.n) ok = ok && issue_pv_s(1, j == 0, j + 1 == B.n, j + 1 < B.n);
        }
        if (ok) ptx::mma_commit(ptx::smem_u32(q_empty));
      }
      ptx::mma_commit(ptx::smem_u32(drain));
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      wait_bounded(ptx::smem_u32(drain), 0, dctl, 15);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax + output (warps 4..11)
    ptx::setmaxnreg_inc<kAttnRegsHigh>();
    const int x = (warp - 4) >> 2;  // stream of this warp group
    const int q = warp & 3;
    const int r = 32 * q + lane;  // query row within the block == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    const uint32_t tS = tmem_base + x * 128 + lane_off;
    const uint32_t tO = tmem_base + 256 + x * 128 + lane_off;
    const float c = a.scale_log2;
    uint32_t s_cnt = 0, o_cnt = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
      int bh;
      AttnStream A, B;
      attn_item(a, item, bh, A, B);
      const AttnStream st = x == 0 ? A : B;
      if (st.qb < 0) continue;
      const int64_t grow = static_cast<int64_t>(bh) * a.S + st.qb * kAttnBlk + r;
      uint16_t* orow = static_cast<uint16_t*>(a.O) + grow * kD;
      if (st.n <= 0) {
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int cc = 0; cc < kD / 8; ++cc) reinterpret_cast<uint4*>(orow)[cc] = z;
        if (a.lse) a.lse[grow] = -INFINITY;
        continue;
      }
      float m_run = -INFINITY, l_run = 0.0f;  // m_run in scaled log2 units
      for (int j = 0; j < st.n; ++j) {
        const int kb = __ldg(&a.col_idx[st.j0 + j]);
        const bool diag = a.causal_diag && kb == st.qb;
        // S_j complete; it was issued after PV_{j-1}, so O already holds block j-1's contribution.
        ok = warp_wait_bounded(ptx::smem_u32(&s_full[x]), s_cnt & 1, ctl, 20);
        if (!ok) break;
        ++s_cnt;
        ptx::tc_fence_after();
        uint32_t sv[128];  // S row, loaded straight into the registers the softmax works in
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          ptx::tmem_ld_32x32b_x32(tS + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[cc * 32]));
        ptx::tmem_wait_ld();
        float* v = reinterpret_cast<float*>(sv);
        if (diag) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i > r) v[i] = -INFINITY;
        }
        // Row max and row sum as 8 independent partial chains (a single chain is 127 dependent ops deep).
        float pm[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) pm[k] = v[k];
#pragma unroll
        for (int i = 8; i < 128; i += 16)
#pragma unroll
          for (int k = 0; k < 8; ++k) pm[k] = max3f(pm[k], v[i + k], v[i + 8 + k]);
        const float mb = max3f(max3f(pm[0], pm[1], pm[2]), max3f(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7]));
        const float mbs = mb * c;
        const bool move = mbs > m_run + 8.0f;
        float alpha = 1.0f;
        if (move) alpha = (m_run == -INFINITY) ? 0.0f : ex2_approx(m_run - mbs);
        if (move) m_run = mbs;
        const bool need_rescale = __any_sync(0xffffffffu, move && j > 0);
        const float m_sub = (m_run == -INFINITY) ? 0.0f : m_run;  // fully masked so far: P = 0, no NaN
        // exp2 on pairs: t = s * c - m by fma.f32x2; 3 of every 4 pairs on the MUFU, 1 on the FMA pipe.
        // P is packed to bf16 pairs in place: pair k lands in sv[k], whose S value (element k <= i) is used.
        const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-m_sub, -m_sub);
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int i = 0; i < 128; i += 2) {
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
        if (need_rescale) {  // O (complete through block j-1) *= alpha, in TMEM
          const float al = move ? alpha : 1.0f;
#pragma unroll 1
          for (int cc = 0; cc < kD / 32; ++cc) {
            uint32_t u[32];
            ptx::tmem_ld_32x32b_x32(tO + cc * 32, u);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * al);
            ptx::tmem_st_32x32b_x32(tO + cc * 32, u);
          }
        }
        // P row r (bf16 pairs) -> TMEM columns [0, 64) of this stream's S buffer.
        ptx::tmem_st_32x32b_x32(tS, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        ptx::tmem_st_32x32b_x32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&p_full[x]));
      }
      if (!ok) break;
      // Output: wait for the last PV of this row, then O / l -> bf16.
      ok = warp_wait_bounded<false, 256>(ptx::smem_u32(&o_done[x]), o_cnt & 1, ctl, 22);
      if (!ok) break;
      ++o_cnt;
      ptx::tc_fence_after();
      const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      // l_run sums 2^(s*c - m_run) whatever m_run lagged behind, so m_run + log2(l_run) is exact
      if (a.lse) a.lse[grow] = l_run > 0.0f ? (m_run + log2f(l_run)) * 0.6931471805599453f : -INFINITY;
#pragma unroll 1
      for (int cc = 0; cc < kD / 32; ++cc) {
        uint32_t u[32];
        ptx::tmem_ld_32x32b_x32(tO + cc * 32, u);
        ptx::tmem_wait_ld();
        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          dst[g] = make_uint4(pack2<kF16>(__uint_as_float(u[8 * g + 0]) * inv_l, __uint_as_float(u[8 * g + 1]) * inv_l),
                              pack2<kF16>(__uint_as_float(u[8 * g + 2]) * inv_l, __uint_as_float(u[8 * g + 3]) * inv_l),
                              pack2<kF16>(__uint_as_float(u[8 * g + 4]) * inv_l, __uint_as_float(u[8 * g + 5]) * inv_l),
                              pack2<kF16>(__uint_as_float(u[8 * g + 6]) * inv_l, __uint_as_float(u[8 * g + 7]) * inv_l));
        }
      }
      ptx::tc_fence_before();
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
