// Block-sparse attention forward for sm_100a (bf16 in/out, fp32 online softmax), 128x128 blocks, D = 128.
//
// Work item = (b, h, query block-row i). For the nonzero key blocks j of that row (BSR index of the
// per-(b,h) block mask) the CTA computes
//     S_j = Q_i K_j^T          tcgen05.mma 128x128x16 x 8, K-major operands, fp32 into TMEM (2 S buffers)
//     P_j = exp2(S_j*scale*log2e - m)  online softmax by 4 warps, one query row per thread, P -> smem bf16
//     O  += P_j V_j            tcgen05.mma with V as an MN-major operand (row-major [kv, d] tile)
// and writes O / l as bf16. Only nonzero blocks are ever loaded (TMA, 2-stage K and V rings).
// Roles: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 2-5 softmax + output.
// The running max is only moved when a block raises it by more than 8 (log2 units); P then stays
// below 2^8 and O is rescaled in TMEM (tcgen05.ld / st) only on those moves.
#pragma once

#include <cuda_bf16.h>

#include "ptx_sm100.cuh"

namespace bsk {

constexpr int kAttnBlk = 128;
constexpr int kAttnD = 128;
constexpr int kAttnThreads = 192;
constexpr int kAttnTile = kAttnBlk * kAttnD * 2;  // 32 KB: one 128 x 128 bf16 tile (two 64-col SW128 chunks)
constexpr int kAttnChunk = kAttnTile / 2;          // 16 KB
constexpr int kAttnKVStages = 2;
constexpr int kAttnSmemBytes = 1024 + kAttnTile * (1 /*Q*/ + 2 * kAttnKVStages /*K,V*/ + 1 /*P*/) + 256;
constexpr int kAttnTmemCols = 512;  // S0 [0,128), S1 [128,256), O [256,384)

struct AttnArgs {
  __nv_bfloat16* O;
  const int* row_ptr;
  const int* col_idx;
  int S;          // sequence length
  int nqb;        // S / 128
  int bh_begin;   // first (b,h) pair of this launch
  int num_items;  // (#pairs) * nqb
  float scale_log2;
  int causal_diag;
  uint32_t* err;
  uint64_t timeout_ns;
};

// Work item -> (bh, qb): head-major, so the CTAs running at the same time share one or two heads' K and V
// blocks in L2; within a head the longest rows (highest query block under a causal pattern) come first.
__device__ __forceinline__ void attn_item(const AttnArgs& a, int item, int& bh, int& qb) {
  qb = a.nqb - 1 - item % a.nqb;
  bh = a.bh_begin + item / a.nqb;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    bsattn_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  constexpr uint32_t IDESC_S = ptx::instr_desc(128, 128, 1, 1, 0, 0);   // bf16, both K-major
  constexpr uint32_t IDESC_PV = ptx::instr_desc(128, 128, 1, 1, 0, 1);  // V MN-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kAttnTile;
  uint8_t* sV = sK + kAttnKVStages * kAttnTile;
  uint8_t* sP = sV + kAttnKVStages * kAttnTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kAttnTile);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;   // [2]
  uint64_t* k_empty = bars + 4;  // [2]
  uint64_t* v_full = bars + 6;   // [2]
  uint64_t* v_empty = bars + 8;  // [2]
  uint64_t* s_full = bars + 10;  // [2]
  uint64_t* s_empty = bars + 12; // [2]
  uint64_t* p_full = bars + 14;
  uint64_t* pv_done = bars + 15;
  uint64_t* drain = bars + 16;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(q_full), 1);
    ptx::mbar_init(ptx::smem_u32(q_empty), 1);
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(ptx::smem_u32(&k_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&k_empty[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&v_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&v_empty[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&s_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&s_empty[s]), 4);
    }
    ptx::mbar_init(ptx::smem_u32(p_full), 4);
    ptx::mbar_init(ptx::smem_u32(pv_done), 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    uint32_t q_phase = 0, kv_stage = 0, kv_phase = 0;
    uint32_t q_issued = 0, kv_issued = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
      int bh, qb;
      attn_item(a, item, bh, qb);
      const int p = bh * a.nqb + qb;
      const int j0 = __ldg(&a.row_ptr[p]);
      const int j1 = __ldg(&a.row_ptr[p + 1]);
      if (j1 <= j0) continue;
      ok = warp_wait_bounded(ptx::smem_u32(q_empty), q_phase ^ 1, ctl, 1);
      if (!ok) break;
      const int row0 = bh * a.S;
      if (lane == 0) {
        const uint32_t fb = ptx::smem_u32(q_full);
        ptx::mbar_arrive_expect_tx(fb, kAttnTile);
        ptx::tma_load_2d(ptx::smem_u32(sQ), &tmQ, fb, 0, row0 + qb * kAttnBlk);
        ptx::tma_load_2d(ptx::smem_u32(sQ + kAttnChunk), &tmQ, fb, 64, row0 + qb * kAttnBlk);
      }
      ++q_issued;
      q_phase ^= 1;
      for (int jb = j0; jb < j1 && ok; jb += 32) {
        const int cidx = (jb + lane < j1) ? __ldg(&a.col_idx[jb + lane]) : 0;
        const int cnt = min(32, j1 - jb);
        for (int jj = 0; jj < cnt; ++jj) {
          int kb = __shfl_sync(0xffffffffu, cidx, jj);
          if (kb < 0 || kb >= a.nqb) {  // out-of-range index: flag it, load nothing real (zero fill)
            if (lane == 0) atomicCAS(a.err, 0u, kErrBounds | (kKidBsAttn << 8) | (7u << 16));
            kb = a.nqb;
          }
          const int kvrow = row0 + kb * kAttnBlk;
          ok = warp_wait_bounded(ptx::smem_u32(&k_empty[kv_stage]), kv_phase ^ 1, ctl, 2);
          if (!ok) break;
          if (lane == 0) {
            const uint32_t fb = ptx::smem_u32(&k_full[kv_stage]);
            const uint32_t dst = ptx::smem_u32(sK + kv_stage * kAttnTile);
            ptx::mbar_arrive_expect_tx(fb, kAttnTile);
            ptx::tma_load_2d(dst, &tmK, fb, 0, kvrow);
            ptx::tma_load_2d(dst + kAttnChunk, &tmK, fb, 64, kvrow);
          }
          ok = warp_wait_bounded(ptx::smem_u32(&v_empty[kv_stage]), kv_phase ^ 1, ctl, 3);
          if (!ok) break;
          if (lane == 0) {
            const uint32_t fb = ptx::smem_u32(&v_full[kv_stage]);
            const uint32_t dst = ptx::smem_u32(sV + kv_stage * kAttnTile);
            ptx::mbar_arrive_expect_tx(fb, kAttnTile);
            ptx::tma_load_2d(dst, &tmV, fb, 0, kvrow);
            ptx::tma_load_2d(dst + kAttnChunk, &tmV, fb, 64, kvrow);
          }
          ++kv_issued;
          if (++kv_stage == kAttnKVStages) { kv_stage = 0; kv_phase ^= 1; }
        }
      }
    }
    // Drain loads still in flight.
    if (lane == 0) {
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      if (q_issued) wait_bounded(ptx::smem_u32(q_full), (q_issued - 1) & 1, dctl, 8);
      const uint32_t first = kv_issued > kAttnKVStages ? kv_issued - kAttnKVStages : 0;
      for (uint32_t i = first; i < kv_issued; ++i) {
        wait_bounded(ptx::smem_u32(&k_full[i % kAttnKVStages]), (i / kAttnKVStages) & 1, dctl, 8);
        wait_bounded(ptx::smem_u32(&v_full[i % kAttnKVStages]), (i / kAttnKVStages) & 1, dctl, 8);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    uint32_t q_phase = 0;
    uint32_t k_stage = 0, k_phase = 0, v_stage = 0, v_phase = 0;
    uint32_t s_cnt = 0;   // S computations issued (buffer = s_cnt & 1)
    uint32_t p_cnt = 0;   // P tiles consumed
    bool ok = true;
    const uint32_t sQa = ptx::smem_u32(sQ);
    const uint32_t sPa = ptx::smem_u32(sP);
    const uint32_t tO = tmem_base + 256;

    auto issue_s = [&](bool last_of_item) -> bool {
      const uint32_t sb = s_cnt & 1;
      // S buffer sb is free once the softmax warps have read its previous use.
      if (!warp_wait_bounded(ptx::smem_u32(&s_empty[sb]), ((s_cnt >> 1) & 1) ^ 1, ctl, 10)) return false;
      if (!warp_wait_bounded(ptx::smem_u32(&k_full[k_stage]), k_phase, ctl, 11)) return false;
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint32_t kA = ptx::smem_u32(sK + k_stage * kAttnTile);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kAttnChunk + (k & 3) * 32;
          ptx::mma_f16_ss(tmem_base + sb * 128, ptx::smem_desc(sQa + off, 16, 1024), ptx::smem_desc(kA + off, 16, 1024),
                          IDESC_S, k != 0);
        }
        ptx::mma_commit(ptx::smem_u32(&k_empty[k_stage]));
        ptx::mma_commit(ptx::smem_u32(&s_full[sb]));
        if (last_of_item) ptx::mma_commit(ptx::smem_u32(q_empty));
      }
      __syncwarp();
      ++s_cnt;
      if (++k_stage == kAttnKVStages) { k_stage = 0; k_phase ^= 1; }
      return true;
    };
    auto issue_pv = [&](bool first_of_item) -> bool {
      if (!warp_wait_bounded(ptx::smem_u32(p_full), p_cnt & 1, ctl, 12)) return false;
      if (!warp_wait_bounded(ptx::smem_u32(&v_full[v_stage]), v_phase, ctl, 13)) return false;
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint32_t vA = ptx::smem_u32(sV + v_stage * kAttnTile);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t aoff = (k >> 2) * kAttnChunk + (k & 3) * 32;
          ptx::mma_f16_ss(tO, ptx::smem_desc(sPa + aoff, 16, 1024), ptx::smem_desc(vA + k * 2048, kAttnChunk, 1024),
                          IDESC_PV, (first_of_item && k == 0) ? 0u : 1u);
        }
        ptx::mma_commit(ptx::smem_u32(&v_empty[v_stage]));
        ptx::mma_commit(ptx::smem_u32(pv_done));
      }
      __syncwarp();
      ++p_cnt;
      if (++v_stage == kAttnKVStages) { v_stage = 0; v_phase ^= 1; }
      return true;
    };

    for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
      int bh, qb;
      attn_item(a, item, bh, qb);
      const int p = bh * a.nqb + qb;
      const int n = __ldg(&a.row_ptr[p + 1]) - __ldg(&a.row_ptr[p]);
      if (n <= 0) continue;
      ok = warp_wait_bounded(ptx::smem_u32(q_full), q_phase, ctl, 14);
      if (!ok) break;
      q_phase ^= 1;
      ok = issue_s(n == 1);
      for (int jj = 0; jj < n && ok; ++jj) {
        if (jj + 1 < n) {
          ok = issue_s(jj + 2 == n);
          if (!ok) break;
        }
        ok = issue_pv(jj == 0);
      }
    }
    if (lane == 0) {
      ptx::mma_commit(ptx::smem_u32(drain));
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      wait_bounded(ptx::smem_u32(drain), 0, dctl, 15);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax + output (warps 2..5)
    const int q = warp & 3;
    const int r = 32 * q + lane;  // query row within the block == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    const uint32_t tO = tmem_base + 256 + lane_off;
    uint32_t s_cnt = 0, pv_cnt = 0;
    const uint32_t sPa = ptx::smem_u32(sP);
    bool ok = true;
    for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
      int bh, qb;
      attn_item(a, item, bh, qb);
      const int p = bh * a.nqb + qb;
      const int j0 = __ldg(&a.row_ptr[p]);
      const int n = __ldg(&a.row_ptr[p + 1]) - j0;
      __nv_bfloat16* orow = a.O + (static_cast<int64_t>(bh) * a.S + qb * kAttnBlk + r) * kAttnD;
      if (n <= 0) {
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int c = 0; c < 16; ++c) reinterpret_cast<uint4*>(orow)[c] = z;
        continue;
      }
      float m_run = -INFINITY, l_run = 0.0f;
      for (int jj = 0; jj < n; ++jj) {
        const int kb = __ldg(&a.col_idx[j0 + jj]);
        const bool diag = a.causal_diag && kb == qb;
        const uint32_t sb = s_cnt & 1;
        ok = warp_wait_bounded(ptx::smem_u32(&s_full[sb]), (s_cnt >> 1) & 1, ctl, 20);
        if (!ok) break;
        ptx::tc_fence_after();
        float x[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          ptx::tmem_ld_32x32b_x32(tmem_base + sb * 128 + lane_off + c * 32, v);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(v[i]) * a.scale_log2;
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&s_empty[sb]));
        ++s_cnt;
        float mb = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          if (diag && i > r) x[i] = -INFINITY;
          mb = fmaxf(mb, x[i]);
        }
        // Move the reference max only when this block raises it by more than 8.
        const bool move = mb > m_run + 8.0f;
        const float m_new = move ? mb : m_run;
        float alpha = 1.0f;
        if (move) alpha = (m_run == -INFINITY) ? 0.0f : ex2_approx(m_run - m_new);
        const bool need_rescale = __any_sync(0xffffffffu, move && jj > 0);
        const float m_sub = (m_new == -INFINITY) ? 0.0f : m_new;  // fully masked so far: P = 0, no NaN
        float rs = 0.0f;
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          x[i] = ex2_approx(x[i] - m_sub);
          rs += x[i];
        }
        l_run = l_run * alpha + rs;
        m_run = m_new;
        // P shared memory and O are free once the previous PV has completed.
        if (jj > 0) {
          ok = warp_wait_bounded(ptx::smem_u32(pv_done), pv_cnt & 1, ctl, 21);
          if (!ok) break;
          ++pv_cnt;
          ptx::tc_fence_after();
          if (need_rescale) {
            const float al = move ? alpha : 1.0f;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t v[32];
              ptx::tmem_ld_32x32b_x32(tO + c * 32, v);
              ptx::tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * al);
              ptx::tmem_st_32x32b_x32(tO + c * 32, v);
            }
            ptx::tmem_wait_st();
          }
        }
        // P row r -> shared memory, K-major, 128-B swizzle: 16-B chunk ch of a 128-B row lands at ch ^ (r & 7).
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t rowbase = sPa + half * kAttnChunk + r * 128;
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const float* xs = &x[half * 64 + ch * 8];
            st_shared_v4(rowbase + ((ch ^ (r & 7)) << 4), pack_bf16(xs[0], xs[1]), pack_bf16(xs[2], xs[3]),
                         pack_bf16(xs[4], xs[5]), pack_bf16(xs[6], xs[7]));
          }
        }
        ptx::fence_proxy_async_smem();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(p_full));
      }
      if (!ok) break;
      // Output: wait for the last PV of this row, then O / l -> bf16.
      ok = warp_wait_bounded(ptx::smem_u32(pv_done), pv_cnt & 1, ctl, 22);
      if (!ok) break;
      ++pv_cnt;
      ptx::tc_fence_after();
      const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        ptx::tmem_ld_32x32b_x32(tO + c * 32, v);
        ptx::tmem_wait_ld();
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          dst[g] = make_uint4(pack_bf16(__uint_as_float(v[8 * g + 0]) * inv_l, __uint_as_float(v[8 * g + 1]) * inv_l),
                              pack_bf16(__uint_as_float(v[8 * g + 2]) * inv_l, __uint_as_float(v[8 * g + 3]) * inv_l),
                              pack_bf16(__uint_as_float(v[8 * g + 4]) * inv_l, __uint_as_float(v[8 * g + 5]) * inv_l),
                              pack_bf16(__uint_as_float(v[8 * g + 6]) * inv_l, __uint_as_float(v[8 * g + 7]) * inv_l));
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

}  // namespace bsk
