// Block-sparse attention backward for sm_100a (tcgen05 + TMA), deterministic (no atomics).
//
// Given Q, K, V, O, dO [B*H*S, D] (fp16 or bf16), the forward's natural-log LSE per query row, and the block mask
// (row lists: query block -> key blocks; column lists: key block -> query blocks), computes
//   Delta_i = sum_d dO[i,d] O[i,d]                                      (bsattn_bwd_delta_kernel)
//   P = exp(scale * Q K^T - LSE), dP = dO V^T, dS = P * (dP - Delta)    (recomputed per block pair)
//   dV = P^T dO, dK = scale * dS^T Q                                    (bsattn_bwd_dkdv_kernel, per key block)
//   dQ = scale * dS K                                                   (bsattn_bwd_dq_kernel, per query block)
// The causal diagonal block masks key position > query position, as the forward does. The dK/dV and dQ passes
// each recompute the scores they need, so every output element is written by one CTA in a fixed order.
//
// The reference has no backward kernel (its launch_attention_backward in
// .archive/src_experiments/blackwell_sparsek/kernels/attention_fmha.cu:436-453 is a stub and its autograd
// function falls back to torch, kernels/sparsek.py:100-142).
//
// CTA layout (both passes, 384 threads): warp 0 producer (one thread, TMA), warp 1 MMA issuer (one thread),
// warps 2-3 idle, warps 4-11 two warpgroups of elementwise work; warpgroup x takes columns [64x, 64x + 64) of
// the 128 x 128 score tiles (each warp its 32-lane quarter of TMEM), and half of D for the output. P is kept in
// fp32 registers between the P step and the dS step; the tensor-core operands P^T / dS^T are rounded to the
// input type.
#pragma once

#include "bsattn_sm100.cuh"

namespace bsk {

// 12 warps per CTA in both backward passes: producer, MMA issuer, 2 idle, two compute warpgroups; the launch
// allocation of 384 x 168 registers is split 112 (warpgroup 0) / 184 (compute warpgroups).
constexpr int kBwdThreads = 384;
constexpr uint32_t kBwdRegsLow = 112;
constexpr uint32_t kBwdRegsHigh = 184;
static_assert(128 * kBwdRegsLow + 256 * kBwdRegsHigh <= kBwdThreads * 168, "setmaxnreg split exceeds the launch allocation");

constexpr uint32_t kKidBsAttnBwd = 7;
constexpr uint32_t kBwdSuspendNs = 2000;  // suspend hint of the compute and MMA waits (woken at completion)
// Eighths of the exponentials of P computed on the FMA pipe (ex2_poly2) instead of the MUFU, in both passes.
#ifndef BSK_BWD_POLY_EIGHTHS
#define BSK_BWD_POLY_EIGHTHS 2
#endif
constexpr int kBwdPolyEighths = BSK_BWD_POLY_EIGHTHS;

// exp2 of a packed pair on the MUFU, or on the FMA pipe when `poly` (a compile-time choice after unrolling).
__device__ __forceinline__ uint64_t f2_ex2_split(uint64_t t, bool poly) {
  float a, b;
  f2_unpack(t, a, b);
  if (poly) {
    float ya, yb;
    ex2_poly2(a, b, ya, yb);
    return f2_pack(ya, yb);
  }
  return f2_pack(ex2_approx(a), ex2_approx(b));
}

struct AttnBwdArgs {
  const void* dO;        // [B*H*S, D]
  const void* O;         // [B*H*S, D]   (delta pass)
  const float* lse;      // [B*H*S] natural log
  float* delta;          // [B*H*S] written by the delta pass, read by the others
  float* nlse2;          // [B*H*S] -LSE * log2(e), written by the delta pass (exponent offset in log2 units)
  void* dQ;              // [B*H*S, D]
  void* dK;
  void* dV;
  const int* row_ptr;    // [BH*nqb + 1] -> col_idx (key blocks of each query block-row)
  const int* col_idx;
  const int* col_ptr;    // [BH*nqb + 1] -> row_idx (query blocks of each key block-column), ascending
  const int* row_idx;
  int S, nqb, bh_begin, num_items;
  float scale;           // softmax scale
  float scale_log2;      // scale * log2(e)
  int causal_diag;
  uint32_t* err;
  uint64_t timeout_ns;
};

// Delta_i = dO_i . O_i in fp32 (8 elements, 16 bytes, per thread; D / 8 threads per row; grid-stride), and the
// row's exponent offset -LSE_i * log2(e) that the passes below add to scale * log2(e) * S.
template <bool kF16, int kD>
__global__ void __launch_bounds__(256) bsattn_bwd_delta_kernel(const uint16_t* __restrict__ dO,
                                                               const uint16_t* __restrict__ O,
                                                               const float* __restrict__ lse,
                                                               float* __restrict__ delta,
                                                               float* __restrict__ nlse2, int64_t rows) {
  constexpr int kTpr = kD / 8;  // threads per row: 16 (D = 128) or 8 (D = 64), a power of two
  const int64_t total = rows * kTpr;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i - (threadIdx.x & 31) < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc = 0.0f;
    if (i < total) {
      const uint4 a = reinterpret_cast<const uint4*>(dO)[i];
      const uint4 b = reinterpret_cast<const uint4*>(O)[i];
      const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float a0, a1, b0, b1;
        if (kF16) {
          const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&wa[k]));
          const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&wb[k]));
          a0 = fa.x; a1 = fa.y; b0 = fb.x; b1 = fb.y;
        } else {
          const float2 fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wa[k]));
          const float2 fb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wb[k]));
          a0 = fa.x; a1 = fa.y; b0 = fb.x; b1 = fb.y;
        }
        acc = fmaf(a0, b0, acc);
        acc = fmaf(a1, b1, acc);
      }
    }
#pragma unroll
    for (int o = kTpr / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (i < total && (i % kTpr) == 0) {
      delta[i / kTpr] = acc;
      nlse2[i / kTpr] = -lse[i / kTpr] * 1.4426950408889634f;
    }
  }
}

// Column lists of the block mask: for every (b,h) pair, the query blocks of each key block-column in ascending
// order (a counting sort of the row lists, one thread per pair). col_ptr shares row_ptr's numbering: pair p's
// entries occupy [row_ptr[p*nqb], row_ptr[(p+1)*nqb]) in both. Out-of-range key blocks are dropped and flagged.
__global__ void bsattn_mask_transpose_kernel(const int* __restrict__ row_ptr, const int* __restrict__ col_idx,
                                             int pairs, int nqb, int* __restrict__ col_ptr,
                                             int* __restrict__ row_idx, int* __restrict__ cursor,
                                             int* __restrict__ bad) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += gridDim.x * blockDim.x) {
    const int base = row_ptr[p * nqb];
    int* cnt = cursor + static_cast<int64_t>(p) * nqb;
    for (int j = 0; j < nqb; ++j) cnt[j] = 0;
    for (int i = 0; i < nqb; ++i)
      for (int e = row_ptr[p * nqb + i]; e < row_ptr[p * nqb + i + 1]; ++e) {
        const int kb = col_idx[e];
        if (kb < 0 || kb >= nqb) {
          *bad = 1;
          continue;
        }
        ++cnt[kb];
      }
    int run = base;
    for (int j = 0; j < nqb; ++j) {
      const int c = cnt[j];
      col_ptr[p * nqb + j] = run;
      cnt[j] = run;
      run += c;
    }
    if (p == pairs - 1) col_ptr[pairs * nqb] = run;
    for (int i = 0; i < nqb; ++i)
      for (int e = row_ptr[p * nqb + i]; e < row_ptr[p * nqb + i + 1]; ++e) {
        const int kb = col_idx[e];
        if (kb >= 0 && kb < nqb) row_idx[cnt[kb]++] = i;
      }
  }
}

// Column lists, one CTA per (b,h) pair (nqb <= kTransposeSmemMaxBlocks): the pair's block mask as an nqb x nqb bit
// map in shared memory (set from the row lists by the threads of each row), per-column counts, a CTA scan into
// col_ptr, and each column's thread writes its query blocks in ascending order. Same output as the kernel above.
constexpr int kTransposeSmemMaxBlocks = 512;  // bit map of 512 x 512 bits = 32 KB

__global__ void __launch_bounds__(256) bsattn_mask_transpose_smem_kernel(const int* __restrict__ row_ptr,
                                                                         const int* __restrict__ col_idx, int pairs,
                                                                         int nqb, int* __restrict__ col_ptr,
                                                                         int* __restrict__ row_idx,
                                                                         int* __restrict__ bad) {
  extern __shared__ uint32_t bits[];  // [nqb][words per row]
  __shared__ int warp_sum[8];
  const int wpr = (nqb + 31) / 32;
  for (int p = blockIdx.x; p < pairs; p += gridDim.x) {
    for (int w = threadIdx.x; w < nqb * wpr; w += blockDim.x) bits[w] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < nqb; i += blockDim.x)
      for (int e = row_ptr[p * nqb + i]; e < row_ptr[p * nqb + i + 1]; ++e) {
        const int kb = col_idx[e];
        if (kb < 0 || kb >= nqb) {
          *bad = 1;
          continue;
        }
        atomicOr(&bits[i * wpr + (kb >> 5)], 1u << (kb & 31));
      }
    __syncthreads();
    // scan of the column counts, nqb columns in chunks of blockDim, running carry in `base`
    int base = row_ptr[p * nqb];
    for (int j0 = 0; j0 < nqb; j0 += blockDim.x) {
      const int j = j0 + threadIdx.x;
      int cnt = 0;
      if (j < nqb)
        for (int i = 0; i < nqb; ++i) cnt += (bits[i * wpr + (j >> 5)] >> (j & 31)) & 1u;
      int incl = cnt;
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if ((threadIdx.x & 31) >= o) incl += v;
      }
      if ((threadIdx.x & 31) == 31) warp_sum[threadIdx.x >> 5] = incl;
      __syncthreads();
      int before = base;
      for (int w = 0; w < (threadIdx.x >> 5); ++w) before += warp_sum[w];
      int pos = before + incl - cnt;
      if (j < nqb) {
        col_ptr[p * nqb + j] = pos;
        for (int i = 0; i < nqb; ++i)
          if ((bits[i * wpr + (j >> 5)] >> (j & 31)) & 1u) row_idx[pos++] = i;
      }
      int total = 0;
      for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total += warp_sum[w];
      __syncthreads();
      base += total;
    }
    if (p == pairs - 1 && threadIdx.x == 0) col_ptr[pairs * nqb] = base;
    __syncthreads();
  }
}

// Block mask of dense (every key block) or causal// Block mask of dense (every key block) or causal (key blocks 0..i of query block i) attention for `pairs`
// (b,h) pairs: one thread per block-row writes its row pointer and column list.
__global__ void attn_full_mask_kernel(int pairs, int nqb, int causal, int* __restrict__ row_ptr,
                                      int* __restrict__ col_idx) {
  const int rows = pairs * nqb;
  const int64_t per_pair = causal ? static_cast<int64_t>(nqb) * (nqb + 1) / 2 : static_cast<int64_t>(nqb) * nqb;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < rows; t += gridDim.x * blockDim.x) {
    const int p = t / nqb, i = t % nqb;
    const int64_t start = p * per_pair + (causal ? static_cast<int64_t>(i) * (i + 1) / 2 : static_cast<int64_t>(i) * nqb);
    const int n = causal ? i + 1 : nqb;
    row_ptr[t] = static_cast<int>(start);
    for (int j = 0; j < n; ++j) col_idx[start + j] = j;
    if (t == rows - 1) row_ptr[rows] = static_cast<int>(start + n);
  }
}

// 32 scaled columns of this thread's row -> 16-bit values at dst (64 bytes): two 32-byte stores (one sector each)
// when dst is 32-byte aligned (every row is, when the tensor is: rows are multiples of 32 bytes apart), else four
// 16-byte stores. Each thread writes its own row, so fewer, wider stores mean fewer memory transactions per warp.
template <bool kF16>
__device__ __forceinline__ void store_row_half(uint16_t* dst, const uint32_t (&u)[32], float mul) {
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    pk[i] = pack2<kF16>(__uint_as_float(u[2 * i]) * mul, __uint_as_float(u[2 * i + 1]) * mul);
  if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
    st_global_v8(dst, pk);
    st_global_v8(dst + 16, pk + 8);
  } else {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int g = 0; g < 4; ++g) d[g] = make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
  }
}

// TMEM columns [t0 + 32 * (D/64) * x, ...) of this thread's row (kD/2 columns: warpgroup x's half of an
// accumulator) -> scaled fp16/bf16 row segment.
template <bool kF16, int kD>
__device__ __forceinline__ void write_acc_half(uint32_t t_row, int x, uint16_t* row_out, float mul) {
#pragma unroll 1
  for (int cc = 0; cc < kD / 64; ++cc) {
    const int col = x * (kD / 2) + cc * 32;
    uint32_t u[32];
    ptx::tmem_ld_32x32b_x32(t_row + col, u);
    ptx::tmem_wait_ld();
    store_row_half<kF16>(row_out + col, u, mul);
  }
}

template <int kD>
__device__ __forceinline__ void zero_row_half(int x, uint16_t* row_out) {
  const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int cc = 0; cc < kD / 16; ++cc) reinterpret_cast<uint4*>(row_out + x * (kD / 2))[cc] = z;
}

// Packed fp32x2 multiply (FMA pipe, both halves in one instruction) and 2^x of a pair.
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

template <int kD>
__device__ __forceinline__ void mma_kmajor(uint32_t d, uint32_t A, uint32_t B, uint32_t idesc) {
#pragma unroll
  for (int k = 0; k < kD / 16; ++k) {
    const uint32_t off = (k >> 2) * kAttnChunk + (k & 3) * 32;
    ptx::mma_f16_ss(d, ptx::smem_desc(A + off, 16, 1024), ptx::smem_desc(B + off, 16, 1024), idesc, k != 0);
  }
}

// ------------------------------------------------------------------------------------------------ dQ pass
// Item = (b,h) pair and query block i; streams the K_j / V_j tiles of row i's key blocks through a ring.
// TMEM: S [0,128), dP [128,256), dQ accumulator [256, 256 + D), dS (packed pairs) [384, 448). Warpgroup x takes
// key positions [64x, 64x + 64). Order per block j: S(j), dP(j); once S(j) sits in registers the next block's S is
// issued; once dS(j) is in TMEM, dQ += dS(j) K_j and the next block's dP -- so the warps compute P while dP runs
// and the scores of block j + 1 while they finish block j.
template <bool kF16, int kD>
struct BwdDqShape {
  static constexpr int kTile = kAttnBlk * kD * 2;
  static constexpr int kChunks = kD / 64;
  static constexpr int kSlots = kD == 128 ? 4 : 8;
  static constexpr int kSmemBytes = 1024 + kTile * (2 + kSlots) + 512;
};

template <bool kF16, int kD>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bsattn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                         const AttnBwdArgs a) {
  using Sh = BwdDqShape<kF16, kD>;
  constexpr int kTile = Sh::kTile;
  constexpr int kSlots = Sh::kSlots;
  constexpr uint32_t kFmt = kF16 ? 0u : 1u;
  constexpr uint32_t IDESC_S = ptx::instr_desc(128, 128, kFmt, kFmt, 0, 0);  // S, dP: K = D, both K-major
  constexpr uint32_t IDESC_DQ = ptx::instr_desc(128, kD, kFmt, kFmt, 0, 1);  // dQ += dS K: K MN-major
  constexpr uint32_t T_S = 0, T_DP = 128, T_DQ = 256, T_DS = 384;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sdO = sQ + kTile;
  uint8_t* sKV = sdO + kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kSlots * kTile);
  uint64_t* qd_full = bars + 0;
  uint64_t* qd_empty = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = kv_full + kSlots;
  uint64_t* s_full = kv_empty + kSlots;   // S of the current block in TMEM
  uint64_t* dp_full = s_full + 1;         // dP of the current block in TMEM
  uint64_t* s_free = dp_full + 1;         // 8 warp arrivals: S has been read into registers
  uint64_t* ds_full = s_free + 1;         // 8 warp arrivals: dS written (packed) to TMEM
  uint64_t* dq_done = ds_full + 1;
  uint64_t* dq_empty = dq_done + 1;        // 8 warp arrivals: the accumulator has been read out
  uint64_t* drain = dq_empty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(qd_full), 1);
    ptx::mbar_init(ptx::smem_u32(qd_empty), 1);
    for (int s = 0; s < kSlots; ++s) {
      ptx::mbar_init(ptx::smem_u32(&kv_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&kv_empty[s]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(s_full), 1);
    ptx::mbar_init(ptx::smem_u32(dp_full), 1);
    ptx::mbar_init(ptx::smem_u32(s_free), 8);
    ptx::mbar_init(ptx::smem_u32(ds_full), 8);
    ptx::mbar_init(ptx::smem_u32(dq_done), 1);
    ptx::mbar_init(ptx::smem_u32(dq_empty), 8);
    ptx::mbar_init(ptx::smem_u32(drain), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
    ptx::prefetch_tmap(&tmdO);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), kAttnTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  WaitCtl ctl{abort_flag, a.err, a.timeout_ns, kKidBsAttnBwd};
  if (warp < 4) ptx::setmaxnreg_dec<kBwdRegsLow>();

  // item -> (bh, query block), longest rows (last blocks under a causal mask) first
  auto item_of = [&](int item, int& bh, int& qb, int& j0, int& n) {
    bh = a.bh_begin + item / a.nqb;
    qb = a.nqb - 1 - item % a.nqb;
    const int p = bh * a.nqb + qb;
    j0 = __ldg(&a.row_ptr[p]);
    n = max(__ldg(&a.row_ptr[p + 1]) - j0, 0);
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (one thread)
    if (lane == 0) {
      uint32_t qd_phase = 0, slot = 0, slot_phase = 0, qd_issued = 0, kv_issued = 0;
      bool ok = true;
      const uint32_t kv0 = ptx::smem_u32(sKV);
      auto push = [&](const CUtensorMap* m, int row) -> bool {
        if (!wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(&kv_empty[slot]), slot_phase ^ 1, ctl, 2)) return false;
        const uint32_t fb = ptx::smem_u32(&kv_full[slot]);
        ptx::mbar_arrive_expect_tx(fb, kTile);
#pragma unroll
        for (int c = 0; c < Sh::kChunks; ++c) ptx::tma_load_2d(kv0 + slot * kTile + c * kAttnChunk, m, fb, 64 * c, row);
        ++kv_issued;
        if (++slot == kSlots) { slot = 0; slot_phase ^= 1; }
        return true;
      };
      for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
        int bh, qb, j0, n;
        item_of(item, bh, qb, j0, n);
        if (n == 0) continue;
        ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(qd_empty), qd_phase ^ 1, ctl, 1);
        if (!ok) break;
        const uint32_t qf = ptx::smem_u32(qd_full);
        ptx::mbar_arrive_expect_tx(qf, 2 * kTile);
        const int qrow = bh * a.S + qb * kAttnBlk;
#pragma unroll
        for (int c = 0; c < Sh::kChunks; ++c) {
          ptx::tma_load_2d(ptx::smem_u32(sQ) + c * kAttnChunk, &tmQ, qf, 64 * c, qrow);
          ptx::tma_load_2d(ptx::smem_u32(sdO) + c * kAttnChunk, &tmdO, qf, 64 * c, qrow);
        }
        ++qd_issued;
        qd_phase ^= 1;
        for (int j = 0; j < n && ok; ++j) {
          int kb = __ldg(&a.col_idx[j0 + j]);
          if (kb < 0 || kb >= a.nqb) {  // out-of-range index: flag it; the loads read zero fill
            atomicCAS(a.err, 0u, kErrBounds | (kKidBsAttnBwd << 8) | (7u << 16));
            kb = a.nqb;
          }
          const int krow = bh * a.S + kb * kAttnBlk;
          ok = push(&tmK, krow) && push(&tmV, krow);
        }
      }
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      if (qd_issued) wait_bounded(ptx::smem_u32(qd_full), (qd_issued - 1) & 1, dctl, 8);
      const uint32_t first = kv_issued > kSlots ? kv_issued - kSlots : 0;
      for (uint32_t i = first; i < kv_issued; ++i)
        wait_bounded(ptx::smem_u32(&kv_full[i % kSlots]), (i / kSlots) & 1, dctl, 8);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      uint32_t qd_phase = 0, slot = 0, slot_phase = 0, items_done = 0, sf_cnt = 0, ds_cnt = 0;
      bool ok = true;
      const uint32_t kv0 = ptx::smem_u32(sKV), q0 = ptx::smem_u32(sQ), do0 = ptx::smem_u32(sdO);
      auto take = [&](uint32_t site) -> uint32_t {
        if (!wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(&kv_full[slot]), slot_phase, ctl, site)) return 0xFFFFFFFFu;
        const uint32_t s = slot;
        if (++slot == kSlots) { slot = 0; slot_phase ^= 1; }
        return s;
      };
      auto issue_s = [&](uint32_t sk) {  // S = Q K^T
        mma_kmajor<kD>(tmem_base + T_S, q0, kv0 + sk * kTile, IDESC_S);
        ptx::mma_commit(ptx::smem_u32(s_full));
      };
      auto issue_dp = [&](uint32_t sv) {  // dP = dO V^T
        mma_kmajor<kD>(tmem_base + T_DP, do0, kv0 + sv * kTile, IDESC_S);
        ptx::mma_commit(ptx::smem_u32(dp_full));
      };
      auto issue_dq = [&](uint32_t sk, bool first) {  // dQ += dS K: K step k = keys [16k, 16k + 16), dS columns 8k
        const uint32_t kA = kv0 + sk * kTile;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          ptx::mma_f16_ts(tmem_base + T_DQ, tmem_base + T_DS + 8 * k,
                          ptx::smem_desc(kA + k * 2048, kAttnChunk, 1024), IDESC_DQ, (first && k == 0) ? 0u : 1u);
      };
      // Per block j: S(j), dP(j) | S read -> S(j+1) | dS(j) written -> dQ(j), dP(j+1): the scores of the next block
      // are computed while the warps work on this one.
      for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
        int bh, qb, j0, n;
        item_of(item, bh, qb, j0, n);
        if (n == 0) continue;
        ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(qd_full), qd_phase, ctl, 10);
        if (!ok) break;
        qd_phase ^= 1;
        uint32_t sk = take(11), sv = 0xFFFFFFFFu;
        if (sk != 0xFFFFFFFFu) sv = take(12);
        if (sv == 0xFFFFFFFFu) { ok = false; break; }
        ptx::tc_fence_after();
        issue_s(sk);
        issue_dp(sv);
        if (items_done > 0) {  // the previous item's dQ has been read out of TMEM
          ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(dq_empty), (items_done - 1) & 1, ctl, 16);
          if (!ok) break;
        }
        for (int j = 0; j < n && ok; ++j) {
          ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(s_free), sf_cnt & 1, ctl, 13);
          if (!ok) break;
          ++sf_cnt;
          uint32_t nk = 0xFFFFFFFFu, nv = 0xFFFFFFFFu;
          if (j + 1 < n) {
            nk = take(11);
            if (nk != 0xFFFFFFFFu) nv = take(12);
            if (nv == 0xFFFFFFFFu) { ok = false; break; }
            ptx::tc_fence_after();
            issue_s(nk);
          }
          ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(ds_full), ds_cnt & 1, ctl, 14);
          if (!ok) break;
          ++ds_cnt;
          ptx::tc_fence_after();
          issue_dq(sk, j == 0);
          ptx::mma_commit(ptx::smem_u32(&kv_empty[sk]));
          ptx::mma_commit(ptx::smem_u32(&kv_empty[sv]));
          if (j + 1 < n) issue_dp(nv);
          sk = nk;
          sv = nv;
        }
        if (!ok) break;
        ptx::mma_commit(ptx::smem_u32(dq_done));
        ptx::mma_commit(ptx::smem_u32(qd_empty));
        ++items_done;
      }
      ptx::mma_commit(ptx::smem_u32(drain));
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      wait_bounded(ptx::smem_u32(drain), 0, dctl, 15);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ dS = P (dP - Delta), dQ out
    ptx::setmaxnreg_inc<kBwdRegsHigh>();
    const int x = (warp - 4) >> 2;  // key half: positions [64x, 64x + 64)
    const int q = warp & 3;
    const int r = 32 * q + lane;    // query row within the block == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    const uint64_t c2 = f2_pack(a.scale_log2, a.scale_log2);
    uint32_t s_cnt = 0, dp_cnt = 0, dq_cnt = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
      int bh, qb, j0, n;
      item_of(item, bh, qb, j0, n);
      const int64_t grow = static_cast<int64_t>(bh) * a.S + qb * kAttnBlk + r;
      uint16_t* dq_row = static_cast<uint16_t*>(a.dQ) + grow * kD;
      if (n == 0) {
        zero_row_half<kD>(x, dq_row);
        continue;
      }
      const float off = __ldg(&a.nlse2[grow]);
      const float ndlt = -__ldg(&a.delta[grow]);
      const uint64_t off2 = f2_pack(off, off), ndlt2 = f2_pack(ndlt, ndlt);
      for (int j = 0; j < n; ++j) {
        const int kb = __ldg(&a.col_idx[j0 + j]);
        ok = warp_wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(s_full), s_cnt & 1, ctl, 20);
        if (!ok) break;
        ++s_cnt;
        ptx::tc_fence_after();
        uint32_t pv[64];  // S, then P (fp32) of this warp's 64 keys
        const uint32_t ts = tmem_base + lane_off + T_S + 64 * x, tp = tmem_base + lane_off + T_DP + 64 * x;
        ptx::tmem_ld_32x32b_x32(ts, *reinterpret_cast<uint32_t(*)[32]>(&pv[0]));
        ptx::tmem_ld_32x32b_x32(ts + 32, *reinterpret_cast<uint32_t(*)[32]>(&pv[32]));
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(s_free));  // the next block's S may overwrite it
        const bool diag = a.causal_diag && kb == qb;
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          float p0, p1;
          f2_unpack(f2_ex2_split(f2_fma(f2_pack(__uint_as_float(pv[i]), __uint_as_float(pv[i + 1])), c2, off2),
                                 ((i >> 1) & 7) >= 8 - kBwdPolyEighths),
                    p0, p1);
          if (diag && 64 * x + i > r) p0 = 0.0f;      // key position above the query row
          if (diag && 64 * x + i + 1 > r) p1 = 0.0f;
          pv[i] = __float_as_uint(p0);
          pv[i + 1] = __float_as_uint(p1);
        }
        ok = warp_wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(dp_full), dp_cnt & 1, ctl, 21);
        if (!ok) break;
        ++dp_cnt;
        ptx::tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t dv[32];
          ptx::tmem_ld_32x32b_x32(tp + 32 * cc, dv);
          ptx::tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float g0, g1;
            f2_unpack(f2_mul(f2_pack(__uint_as_float(pv[32 * cc + i]), __uint_as_float(pv[32 * cc + i + 1])),
                             f2_add(f2_pack(__uint_as_float(dv[i]), __uint_as_float(dv[i + 1])), ndlt2)),
                      g0, g1);
            pk[i >> 1] = pack2<kF16>(g0, g1);
          }
          ptx::tmem_st_32x32b_x16(tmem_base + lane_off + T_DS + 32 * x + 16 * cc, pk);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(ds_full));
      }
      if (!ok) break;
      ok = warp_wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(dq_done), dq_cnt & 1, ctl, 22);
      if (!ok) break;
      ++dq_cnt;
      ptx::tc_fence_after();
      write_acc_half<kF16, kD>(tmem_base + lane_off + T_DQ, x, dq_row, a.scale);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(dq_empty));
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem_base, kAttnTmemCols);
}

// ------------------------------------------------------------------------------------------------ dK/dV pass
// Item = (b,h) pair and key block j; streams Q_i, dO_i (+ -LSE_i log2(e), Delta_i) of column j's query blocks.
// TMEM: S^T [0,128) -> packed P^T of warpgroup x's query positions [64x, 64x + 64) at [64x, 64x + 32); dP^T
// [128,256) -> packed dS^T likewise at [128 + 64x, ...); dV accumulator [256, 256 + D), dK [256 + D, 256 + 2D).
// Order per block t: S^T(t), dP^T(t); P^T written -> dV(t), S^T(t+1); dS^T written -> dK(t), dP^T(t+1).
template <bool kF16, int kD>
struct BwdDkdvShape {
  static constexpr int kTile = kAttnBlk * kD * 2;
  static constexpr int kChunks = kD / 64;
  static constexpr int kSlotBytes = 2 * kTile + 1024;  // Q, dO, -LSE*log2(e) [128], Delta [128]
  static constexpr int kSlots = kD == 128 ? 2 : 4;
  static constexpr int kSmemBytes = 1024 + 2 * kTile + kSlots * kSlotBytes + 512;
};

template <bool kF16, int kD>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bsattn_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                           const AttnBwdArgs a) {
  using Sh = BwdDkdvShape<kF16, kD>;
  constexpr int kTile = Sh::kTile;
  constexpr int kSlots = Sh::kSlots;
  constexpr int kSlotBytes = Sh::kSlotBytes;
  constexpr uint32_t kFmt = kF16 ? 0u : 1u;
  constexpr uint32_t IDESC_S = ptx::instr_desc(128, 128, kFmt, kFmt, 0, 0);   // S^T, dP^T: K = D, both K-major
  constexpr uint32_t IDESC_ACC = ptx::instr_desc(128, kD, kFmt, kFmt, 0, 1);  // dV, dK: B (dO, Q) MN-major
  constexpr uint32_t T_S = 0, T_DP = 128, T_DV = 256, T_DK = 256 + kD;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kTile;
  uint8_t* sQD = sV + kTile;  // [kSlots] x (Q tile, dO tile, -LSE*log2(e), Delta)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sQD + kSlots * kSlotBytes);
  uint64_t* kv_full = bars + 0;
  uint64_t* kv_empty = bars + 1;
  uint64_t* qd_full = bars + 2;
  uint64_t* qd_empty = qd_full + kSlots;
  uint64_t* s_full = qd_empty + kSlots;   // S^T of the current block in TMEM
  uint64_t* dp_full = s_full + 1;         // dP^T of the current block in TMEM
  uint64_t* p_full = dp_full + 1;         // 8 warp arrivals: P^T written (packed) to TMEM
  uint64_t* ds_full = p_full + 1;         // 8 warp arrivals: dS^T written (packed) to TMEM
  uint64_t* acc_done = ds_full + 1;
  uint64_t* acc_empty = acc_done + 1;      // 8 warp arrivals: dK / dV read out of TMEM
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(kv_full), 1);
    ptx::mbar_init(ptx::smem_u32(kv_empty), 1);
    for (int s = 0; s < kSlots; ++s) {
      ptx::mbar_init(ptx::smem_u32(&qd_full[s]), 1);
      ptx::mbar_init(ptx::smem_u32(&qd_empty[s]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(s_full), 1);
    ptx::mbar_init(ptx::smem_u32(dp_full), 1);
    ptx::mbar_init(ptx::smem_u32(p_full), 8);
    ptx::mbar_init(ptx::smem_u32(ds_full), 8);
    ptx::mbar_init(ptx::smem_u32(acc_done), 1);
    ptx::mbar_init(ptx::smem_u32(acc_empty), 8);
    ptx::mbar_init(ptx::smem_u32(drain), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
    ptx::prefetch_tmap(&tmdO);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), kAttnTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  WaitCtl ctl{abort_flag, a.err, a.timeout_ns, kKidBsAttnBwd};
  if (warp < 4) ptx::setmaxnreg_dec<kBwdRegsLow>();

  // item -> (bh, key block), column list [i0, i0 + n) of query blocks
  auto item_of = [&](int item, int& bh, int& kb, int& i0, int& n) {
    bh = a.bh_begin + item / a.nqb;
    kb = item % a.nqb;
    const int p = bh * a.nqb + kb;
    i0 = __ldg(&a.col_ptr[p]);
    n = max(__ldg(&a.col_ptr[p + 1]) - i0, 0);
  };
  auto qblock = [&](int e) -> int {  // query block of column entry e, clamped (flagged) when out of range
    int qb = __ldg(&a.row_idx[e]);
    if (qb < 0 || qb >= a.nqb) {
      atomicCAS(a.err, 0u, kErrBounds | (kKidBsAttnBwd << 8) | (9u << 16));
      qb = a.nqb;
    }
    return qb;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (one thread)
    if (lane == 0) {
      uint32_t kv_phase = 0, slot = 0, slot_phase = 0, kv_issued = 0, qd_issued = 0;
      bool ok = true;
      const uint32_t qd0 = ptx::smem_u32(sQD);
      for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
        int bh, kb, i0, n;
        item_of(item, bh, kb, i0, n);
        if (n == 0) continue;
        ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(kv_empty), kv_phase ^ 1, ctl, 1);
        if (!ok) break;
        const uint32_t kf = ptx::smem_u32(kv_full);
        ptx::mbar_arrive_expect_tx(kf, 2 * kTile);
        const int krow = bh * a.S + kb * kAttnBlk;
#pragma unroll
        for (int c = 0; c < Sh::kChunks; ++c) {
          ptx::tma_load_2d(ptx::smem_u32(sK) + c * kAttnChunk, &tmK, kf, 64 * c, krow);
          ptx::tma_load_2d(ptx::smem_u32(sV) + c * kAttnChunk, &tmV, kf, 64 * c, krow);
        }
        ++kv_issued;
        kv_phase ^= 1;
        for (int t = 0; t < n && ok; ++t) {
          const int qb = qblock(i0 + t);
          ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(&qd_empty[slot]), slot_phase ^ 1, ctl, 2);
          if (!ok) break;
          const uint32_t fb = ptx::smem_u32(&qd_full[slot]);
          const uint32_t dst = qd0 + slot * kSlotBytes;
          const int qrow = bh * a.S + qb * kAttnBlk;
          if (qb < a.nqb) {
            ptx::mbar_arrive_expect_tx(fb, 2 * kTile + 1024);
            ptx::bulk_load_1d(dst + 2 * kTile, a.nlse2 + qrow, 512, fb);
            ptx::bulk_load_1d(dst + 2 * kTile + 512, a.delta + qrow, 512, fb);
          } else {
            ptx::mbar_arrive_expect_tx(fb, 2 * kTile);  // zero-filled tiles; offsets left unread (P = 0)
          }
#pragma unroll
          for (int c = 0; c < Sh::kChunks; ++c) {
            ptx::tma_load_2d(dst + c * kAttnChunk, &tmQ, fb, 64 * c, qrow);
            ptx::tma_load_2d(dst + kTile + c * kAttnChunk, &tmdO, fb, 64 * c, qrow);
          }
          ++qd_issued;
          if (++slot == kSlots) { slot = 0; slot_phase ^= 1; }
        }
      }
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      if (kv_issued) wait_bounded(ptx::smem_u32(kv_full), (kv_issued - 1) & 1, dctl, 8);
      const uint32_t first = qd_issued > kSlots ? qd_issued - kSlots : 0;
      for (uint32_t i = first; i < qd_issued; ++i)
        wait_bounded(ptx::smem_u32(&qd_full[i % kSlots]), (i / kSlots) & 1, dctl, 8);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      uint32_t kv_phase = 0, slot = 0, slot_phase = 0, items_done = 0, p_cnt = 0, ds_cnt = 0;
      bool ok = true;
      const uint32_t qd0 = ptx::smem_u32(sQD), k0 = ptx::smem_u32(sK), v0 = ptx::smem_u32(sV);
      auto take = [&](uint32_t site) -> uint32_t {
        if (!wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(&qd_full[slot]), slot_phase, ctl, site)) return 0xFFFFFFFFu;
        const uint32_t s = slot;
        if (++slot == kSlots) { slot = 0; slot_phase ^= 1; }
        return s;
      };
      auto issue_s = [&](uint32_t sl) {  // S^T = K Q^T
        mma_kmajor<kD>(tmem_base + T_S, k0, qd0 + sl * kSlotBytes, IDESC_S);
        ptx::mma_commit(ptx::smem_u32(s_full));
      };
      auto issue_dp = [&](uint32_t sl) {  // dP^T = V dO^T
        mma_kmajor<kD>(tmem_base + T_DP, v0, qd0 + sl * kSlotBytes + kTile, IDESC_S);
        ptx::mma_commit(ptx::smem_u32(dp_full));
      };
      // K step k = query rows [16k, 16k + 16): packed columns 8k of half 0, 64 + 8(k - 4) of half 1
      auto pcol = [](int k) -> uint32_t { return 8 * k + (k >= 4 ? 32 : 0); };
      auto issue_dv = [&](uint32_t sl, bool first) {  // dV += P^T dO
        const uint32_t dA = qd0 + sl * kSlotBytes + kTile;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          ptx::mma_f16_ts(tmem_base + T_DV, tmem_base + T_S + pcol(k), ptx::smem_desc(dA + k * 2048, kAttnChunk, 1024),
                          IDESC_ACC, (first && k == 0) ? 0u : 1u);
      };
      auto issue_dk = [&](uint32_t sl, bool first) {  // dK += dS^T Q
        const uint32_t qA = qd0 + sl * kSlotBytes;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          ptx::mma_f16_ts(tmem_base + T_DK, tmem_base + T_DP + pcol(k), ptx::smem_desc(qA + k * 2048, kAttnChunk, 1024),
                          IDESC_ACC, (first && k == 0) ? 0u : 1u);
      };
      // Per block t: S^T(t), dP^T(t) | P^T written -> dV(t), S^T(t+1) | dS^T written -> dK(t), dP^T(t+1): the
      // warps compute P^T while dP^T runs and dS^T while dV and the next S^T run.
      for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
        int bh, kb, i0, n;
        item_of(item, bh, kb, i0, n);
        if (n == 0) continue;
        ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(kv_full), kv_phase, ctl, 10);
        if (!ok) break;
        kv_phase ^= 1;
        uint32_t cur = take(11);
        if (cur == 0xFFFFFFFFu) { ok = false; break; }
        ptx::tc_fence_after();
        issue_s(cur);
        issue_dp(cur);
        if (items_done > 0) {  // the previous item's dK / dV have been read out of TMEM
          ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(acc_empty), (items_done - 1) & 1, ctl, 16);
          if (!ok) break;
        }
        for (int t = 0; t < n && ok; ++t) {
          // The next slot is taken in the same burst of waits as P^T (a poll after queued MMAs drains the pipe).
          ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(p_full), p_cnt & 1, ctl, 12);
          if (!ok) break;
          ++p_cnt;
          uint32_t nxt = 0xFFFFFFFFu;
          if (t + 1 < n) {
            nxt = take(11);
            if (nxt == 0xFFFFFFFFu) { ok = false; break; }
          }
          ptx::tc_fence_after();
          issue_dv(cur, t == 0);
          if (t + 1 < n) issue_s(nxt);
          ok = wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(ds_full), ds_cnt & 1, ctl, 13);
          if (!ok) break;
          ++ds_cnt;
          ptx::tc_fence_after();
          issue_dk(cur, t == 0);
          ptx::mma_commit(ptx::smem_u32(&qd_empty[cur]));
          if (t + 1 < n) issue_dp(nxt);
          cur = nxt;
        }
        if (!ok) break;
        ptx::mma_commit(ptx::smem_u32(acc_done));
        ptx::mma_commit(ptx::smem_u32(kv_empty));
        ++items_done;
      }
      ptx::mma_commit(ptx::smem_u32(drain));
      WaitCtl dctl = ctl;
      volatile int never = 0;
      dctl.abort = &never;
      wait_bounded(ptx::smem_u32(drain), 0, dctl, 15);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ P^T, dS^T, dK / dV out
    ptx::setmaxnreg_inc<kBwdRegsHigh>();
    const int x = (warp - 4) >> 2;  // query half (positions [64x, 64x + 64))
    const int q = warp & 3;
    const int r = 32 * q + lane;    // key row within the block == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    const uint64_t c2 = f2_pack(a.scale_log2, a.scale_log2);
    uint32_t s_cnt = 0, dp_cnt = 0, acc_cnt = 0, slot = 0, slot_phase = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.num_items && ok; item += gridDim.x) {
      int bh, kb, i0, n;
      item_of(item, bh, kb, i0, n);
      const int64_t grow = static_cast<int64_t>(bh) * a.S + kb * kAttnBlk + r;
      uint16_t* dk_row = static_cast<uint16_t*>(a.dK) + grow * kD;
      uint16_t* dv_row = static_cast<uint16_t*>(a.dV) + grow * kD;
      if (n == 0) {
        zero_row_half<kD>(x, dk_row);
        zero_row_half<kD>(x, dv_row);
        continue;
      }
      for (int t = 0; t < n; ++t) {
        const int qb = __ldg(&a.row_idx[i0 + t]);
        const bool valid = qb >= 0 && qb < a.nqb;
        ok = warp_wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(&qd_full[slot]), slot_phase, ctl, 19);  // offsets
        if (ok) ok = warp_wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(s_full), s_cnt & 1, ctl, 20);
        if (!ok) break;
        ++s_cnt;
        ptx::tc_fence_after();
        const float* off_s = reinterpret_cast<const float*>(sQD + slot * kSlotBytes + 2 * kTile) + 64 * x;
        const float* dlt_s = off_s + 128;
        const uint32_t ts = tmem_base + lane_off + T_S + 64 * x, tp = tmem_base + lane_off + T_DP + 64 * x;
        const bool diag = a.causal_diag && qb == kb;
        float pf[64];  // P^T (fp32) of this warp's 64 query positions, kept for dS^T
        // Two chunks of 32 positions; chunk cc's packed values (16 columns) land at ts + 16cc, inside the columns
        // [0, 32) this warp has already read, never over chunk 1's unread scores.
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t sv[32];
          ptx::tmem_ld_32x32b_x32(ts + 32 * cc, sv);
          ptx::tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 o = *reinterpret_cast<const float4*>(off_s + 32 * cc + i);
            float p0, p1, p2, p3;
            f2_unpack(f2_ex2_split(f2_fma(f2_pack(__uint_as_float(sv[i]), __uint_as_float(sv[i + 1])), c2,
                                          f2_pack(o.x, o.y)),
                                   ((i >> 1) & 7) >= 8 - kBwdPolyEighths),
                      p0, p1);
            f2_unpack(f2_ex2_split(f2_fma(f2_pack(__uint_as_float(sv[i + 2]), __uint_as_float(sv[i + 3])), c2,
                                          f2_pack(o.z, o.w)),
                                   (((i >> 1) + 1) & 7) >= 8 - kBwdPolyEighths),
                      p2, p3);
            const int col = 64 * x + 32 * cc + i;  // query position
            if (!valid) p0 = p1 = p2 = p3 = 0.0f;
            if (diag) {  // key row r above the query position
              if (r > col) p0 = 0.0f;
              if (r > col + 1) p1 = 0.0f;
              if (r > col + 2) p2 = 0.0f;
              if (r > col + 3) p3 = 0.0f;
            }
            pf[32 * cc + i] = p0;
            pf[32 * cc + i + 1] = p1;
            pf[32 * cc + i + 2] = p2;
            pf[32 * cc + i + 3] = p3;
            pk[i >> 1] = pack2<kF16>(p0, p1);
            pk[(i >> 1) + 1] = pack2<kF16>(p2, p3);
          }
          ptx::tmem_st_32x32b_x16(ts + 16 * cc, pk);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(p_full));
        ok = warp_wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(dp_full), dp_cnt & 1, ctl, 21);
        if (!ok) break;
        ++dp_cnt;
        ptx::tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t dv[32];
          ptx::tmem_ld_32x32b_x32(tp + 32 * cc, dv);
          ptx::tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 d = *reinterpret_cast<const float4*>(dlt_s + 32 * cc + i);
            float g0, g1, g2, g3;
            f2_unpack(f2_mul(f2_pack(pf[32 * cc + i], pf[32 * cc + i + 1]),
                             f2_add(f2_pack(__uint_as_float(dv[i]), __uint_as_float(dv[i + 1])), f2_pack(-d.x, -d.y))),
                      g0, g1);
            f2_unpack(f2_mul(f2_pack(pf[32 * cc + i + 2], pf[32 * cc + i + 3]),
                             f2_add(f2_pack(__uint_as_float(dv[i + 2]), __uint_as_float(dv[i + 3])),
                                    f2_pack(-d.z, -d.w))),
                      g2, g3);
            pk[i >> 1] = pack2<kF16>(g0, g1);
            pk[(i >> 1) + 1] = pack2<kF16>(g2, g3);
          }
          ptx::tmem_st_32x32b_x16(tp + 16 * cc, pk);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(ds_full));
        if (++slot == kSlots) { slot = 0; slot_phase ^= 1; }
      }
      if (!ok) break;
      ok = warp_wait_bounded_hint<kBwdSuspendNs>(ptx::smem_u32(acc_done), acc_cnt & 1, ctl, 22);
      if (!ok) break;
      ++acc_cnt;
      ptx::tc_fence_after();
      write_acc_half<kF16, kD>(tmem_base + lane_off + T_DV, x, dv_row, 1.0f);
      write_acc_half<kF16, kD>(tmem_base + lane_off + T_DK, x, dk_row, a.scale);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(acc_empty));
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem_base, kAttnTmemCols);
}

}  // namespace bsk
