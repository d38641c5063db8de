// Device-side conversion of dense and CSR matrices to BSR with square bs x bs blocks.
//
// Semantics are those of torch's `dense.to_sparse_bsr((bs, bs))`, which the reference's convert_to_bsr calls
// (BlackwellSparseK/python/utils.py:51-52) and which its CSR path would reach through `to_dense()`
// (utils.py:32-35; ops.py:193-197 left CSR -> BSR unimplemented):
//   * a block is stored iff one of its elements is nonzero; "nonzero" compares the value with zero, so -0.0
//     counts as zero and NaN as nonzero (tested on the bits with the sign cleared);
//   * block columns of a block-row are stored in ascending order; values are the dense block, bit for bit.
// Two phases, so the caller can size the outputs: pattern (flags, per-row counts, row_ptr, nnzb and the
// element nonzero count) and fill (col_idx, the block-index map and the values).
//
// HBM-bound byte work: the dense pattern pass reads the matrix once with 16-byte loads, the fill pass reads the
// stored blocks once more and writes them. Workspace: int32 flags [Mb * Kb] (later the block-index map, -1 for
// absent blocks), int32 block_row [Mb * Kb] (block-row of each stored block), int32 counts [Mb] and a small tail
// (element count, bad-index flag, nnzb).
#pragma once

#include <cstdint>

#include "ptx_sm100.cuh"

namespace bsk {

constexpr int kConvThreads = 256;

template <int kElemBytes>
__device__ __forceinline__ bool elem_nonzero(uint32_t bits) {
  return kElemBytes == 2 ? (bits & 0x7FFFu) != 0u : (bits & 0x7FFFFFFFu) != 0u;
}

// Pattern of a dense row-major matrix, vector path: bs % (16 / elem) == 0, lda % (16 / elem) == 0, A 16-B
// aligned. A warp task is kConvU x 32 consecutive 16-byte chunks of one row (kConvU loads in flight per lane);
// a chunk never straddles a block boundary. Lanes that find a nonzero store 1 to the block's flag (lanes of one
// store instruction that hit the same flag merge into one write; no atomics needed for a constant).
constexpr int kConvU = 4;

template <int kElemBytes>
__device__ __forceinline__ int chunk_nonzeros(const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  int c = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (kElemBytes == 2)
      c += ((w[j] & 0x7FFFu) != 0u) + ((w[j] & 0x7FFF0000u) != 0u);
    else
      c += (w[j] & 0x7FFFFFFFu) != 0u;
  }
  return c;
}

template <int kElemBytes>
__global__ void __launch_bounds__(kConvThreads) dense_flags_vec_kernel(const uint8_t* __restrict__ A, int64_t lda,
                                                                      int M, int K, int bs, int Kb,
                                                                      int* __restrict__ flags,
                                                                      unsigned long long* __restrict__ nnz_out) {
  constexpr int kPer = 16 / kElemBytes;
  const int cpr = K / kPer;   // chunks per row
  const int cpb = bs / kPer;  // chunks per block width
  const int tpr = (cpr + 32 * kConvU - 1) / (32 * kConvU);  // warp tasks per row
  const int64_t tasks = static_cast<int64_t>(M) * tpr;
  const int lane = threadIdx.x & 31;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  unsigned long long count = 0;
  // Software pipeline: the loads of the warp's next task are issued before the current task is examined, so
  // each lane keeps 2 x kConvU 16-byte loads in flight.
  auto load = [&](int64_t task, uint4 (&v)[kConvU], int& row, int& c0) {
    row = static_cast<int>(task / tpr);
    c0 = static_cast<int>(task - static_cast<int64_t>(row) * tpr) * (32 * kConvU) + lane;
    const uint4* rp = reinterpret_cast<const uint4*>(A + static_cast<int64_t>(row) * lda * kElemBytes);
#pragma unroll
    for (int u = 0; u < kConvU; ++u) {
      const int c = c0 + 32 * u;
      v[u] = c < cpr ? ptx::ldg_stream_16(rp + c) : make_uint4(0, 0, 0, 0);
    }
  };
  int64_t task = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  uint4 v[kConvU];
  int row = 0, c0 = 0;
  if (task < tasks) load(task, v, row, c0);
  for (; task < tasks; task += nw) {
    uint4 vn[kConvU];
    int row_n = 0, c0_n = 0;
    if (task + nw < tasks) load(task + nw, vn, row_n, c0_n);
    int* frow = flags + static_cast<int64_t>(row / bs) * Kb;
#pragma unroll
    for (int u = 0; u < kConvU; ++u) {
      const int n = chunk_nonzeros<kElemBytes>(v[u]);
      count += n;
      if (n) frow[(c0 + 32 * u) / cpb] = 1;
    }
#pragma unroll
    for (int u = 0; u < kConvU; ++u) v[u] = vn[u];
    row = row_n;
    c0 = c0_n;
  }
  for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xFFFFFFFFu, count, o);
  if (lane == 0 && count) atomicAdd(nnz_out, count);
}

// Pattern of a dense matrix, element path for any bs / alignment (one thread per element, grid-stride).
template <int kElemBytes>
__global__ void __launch_bounds__(kConvThreads) dense_flags_scalar_kernel(const uint8_t* __restrict__ A,
                                                                         int64_t lda, int M, int K, int bs, int Kb,
                                                                         int* __restrict__ flags,
                                                                         unsigned long long* __restrict__ nnz_out) {
  const int64_t total = static_cast<int64_t>(M) * K;
  unsigned long long count = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / K, col = i - row * K;
    const uint8_t* p = A + (row * lda + col) * kElemBytes;
    const uint32_t bits = kElemBytes == 2 ? *reinterpret_cast<const uint16_t*>(p) : *reinterpret_cast<const uint32_t*>(p);
    if (elem_nonzero<kElemBytes>(bits)) {
      ++count;
      flags[(row / bs) * Kb + col / bs] = 1;
    }
  }
  for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xFFFFFFFFu, count, o);
  if ((threadIdx.x & 31) == 0 && count) atomicAdd(nnz_out, count);
}

template <int kElemBytes>
__device__ __forceinline__ uint32_t load_bits(const uint8_t* p) {
  return kElemBytes == 2 ? static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(p))
                         : *reinterpret_cast<const uint32_t*>(p);
}

// CSR entries are processed entry-parallel: warp w owns one contiguous slice of the entries
// [crow[0], crow[M]) (about nnz / warps entries, a multiple of 32), walked in trips of 32 x kConvCsrU
// lane-contiguous entries (coalesced loads). The slice's first row comes from one binary search of crow; each lane
// then advances its row past empty rows and row ends as its entries move on. Entry indices are 32-bit when nnz
// fits (E = int), and block arithmetic uses shifts when bs is a power of two (kPow2, shift `lg`).
constexpr int kConvCsrU = 8;

template <typename IdxIn, typename E>
__device__ __forceinline__ E crow_at(const IdxIn* crow, int r, E nnz) {
  const int64_t v = static_cast<int64_t>(crow[r]);
  return static_cast<E>(v < 0 ? 0 : (v > static_cast<int64_t>(nnz) ? static_cast<int64_t>(nnz) : v));
}

template <typename IdxIn, typename E>
__device__ __forceinline__ int csr_row_of(const IdxIn* crow, int M, E e, E nnz) {
  int lo = 0, hi = M;  // answer in [0, M): last r with crow[r] <= e
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (crow_at(crow, mid, nnz) <= e) lo = mid; else hi = mid;
  }
  return lo;
}

template <bool kPow2>
__device__ __forceinline__ int div_bs(int x, int bs, int lg) { return kPow2 ? (x >> lg) : x / bs; }
template <bool kPow2>
__device__ __forceinline__ int mod_bs(int x, int bs, int lg) { return kPow2 ? (x & (bs - 1)) : x % bs; }

// The slice [E0, E1) of warp `w` among `nw` warps over entries [eb, ee).
template <typename E>
__device__ __forceinline__ void warp_slice(E eb, E ee, int64_t w, int64_t nw, E& E0, E& E1) {
  const int64_t n = static_cast<int64_t>(ee - eb);
  const int64_t per = ((n + nw - 1) / nw + 31) / 32 * 32;
  const int64_t a = w * per, b = a + per;
  E0 = static_cast<E>(eb + (a < n ? a : n));
  E1 = static_cast<E>(eb + (b < n ? b : n));
}

// Pattern of a CSR matrix: entries whose value is nonzero flag their block. Column indices outside [0, K) are
// skipped and reported through `bad` (no out-of-range write).
template <int kElemBytes, typename IdxIn, typename E, bool kPow2>
__global__ void __launch_bounds__(kConvThreads) csr_flags_kernel(const IdxIn* __restrict__ crow,
                                                                const IdxIn* __restrict__ col,
                                                                const uint8_t* __restrict__ vals, E nnz, int M, int K,
                                                                int bs, int lg, int Kb, int* __restrict__ flags,
                                                                unsigned long long* __restrict__ nnz_out,
                                                                int* __restrict__ bad) {
  const int lane = threadIdx.x & 31;
  const E eb = crow_at(crow, 0, nnz), ee = crow_at(crow, M, nnz);
  E E0, E1;
  warp_slice(eb, ee, (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5,
             (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5, E0, E1);
  unsigned long long count = 0;
  if (E0 < E1) {
    int row = csr_row_of(crow, M, E0, nnz);
    E row_end = crow_at(crow, row + 1, nnz);
    int* frow = flags + static_cast<int64_t>(div_bs<kPow2>(row, bs, lg)) * Kb;
    int* last = nullptr;
    for (E base = E0 + lane; base < E1 + lane; base += 32 * kConvCsrU) {
      int c[kConvCsrU];
      uint32_t bits[kConvCsrU];
#pragma unroll
      for (int u = 0; u < kConvCsrU; ++u) {
        const E p = base + 32 * u;
        c[u] = p < E1 ? static_cast<int>(max(min(static_cast<int64_t>(col[p]), static_cast<int64_t>(INT32_MAX)),
                                             static_cast<int64_t>(-1)))
                      : -1;
        bits[u] = p < E1 ? load_bits<kElemBytes>(vals + static_cast<int64_t>(p) * kElemBytes) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kConvCsrU; ++u) {
        const E p = base + 32 * u;
        if (p >= E1) break;
        if (p >= row_end) {
          while (p >= row_end && row + 1 < M) row_end = crow_at(crow, ++row + 1, nnz);
          frow = flags + static_cast<int64_t>(div_bs<kPow2>(row, bs, lg)) * Kb;
        }
        if (c[u] < 0 || c[u] >= K) {
          *bad = 1;
        } else if (elem_nonzero<kElemBytes>(bits[u])) {
          ++count;
          int* f = frow + div_bs<kPow2>(c[u], bs, lg);
          if (f != last) {  // a lane's entries 32 apart usually share a block: store each flag once per run
            *f = 1;
            last = f;
          }
        }
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xFFFFFFFFu, count, o);
  if (lane == 0 && count) atomicAdd(nnz_out, count);
}

// counts[br] = number of flagged blocks in block-row br (one CTA per block-row, grid-stride over rows).
__global__ void __launch_bounds__(kConvThreads) bsr_row_counts_kernel(const int* __restrict__ flags, int Mb, int Kb,
                                                                     int* __restrict__ counts) {
  __shared__ int warp_sums[kConvThreads / 32];
  for (int br = blockIdx.x; br < Mb; br += gridDim.x) {
    int c = 0;
    for (int j = threadIdx.x; j < Kb; j += blockDim.x) c += flags[static_cast<int64_t>(br) * Kb + j] != 0;
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
      int t = 0;
      for (int w = 0; w < kConvThreads / 32; ++w) t += warp_sums[w];
      counts[br] = t;
    }
    __syncthreads();
  }
}

// Exclusive scan of counts into row_ptr[0..Mb] (one CTA; chunks of kConvThreads with a running carry).
template <typename IdxOut>
__global__ void __launch_bounds__(kConvThreads) bsr_row_ptr_kernel(const int* __restrict__ counts, int Mb,
                                                                  IdxOut* __restrict__ row_ptr,
                                                                  long long* __restrict__ nnzb_out) {
  __shared__ long long warp_tot[kConvThreads / 32];
  __shared__ long long carry_s;
  if (threadIdx.x == 0) carry_s = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < Mb; base += kConvThreads) {
    const int i = base + threadIdx.x;
    const long long v = i < Mb ? counts[i] : 0;
    long long incl = v;
    for (int o = 1; o < 32; o <<= 1) {
      const long long n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    long long before = carry_s;
    for (int w = 0; w < warp; ++w) before += warp_tot[w];
    if (i < Mb) row_ptr[i] = static_cast<IdxOut>(before + incl - v);
    __syncthreads();
    if (threadIdx.x == kConvThreads - 1) carry_s = before + incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    row_ptr[Mb] = static_cast<IdxOut>(carry_s);
    *nnzb_out = carry_s;
  }
}

// Fill, step 1: per block-row, the ascending ranks of its flagged blocks. Writes col_idx[row_ptr[br] + rank] =
// block column and block_row[...] = br for positions below `cap`, and turns flags into the block-index map
// (position, or -1). One CTA per block-row.
template <typename IdxOut>
__global__ void __launch_bounds__(kConvThreads) bsr_compact_kernel(int* __restrict__ flags, int Mb, int Kb,
                                                                  const IdxOut* __restrict__ row_ptr,
                                                                  IdxOut* __restrict__ col_idx,
                                                                  int* __restrict__ block_row, int64_t cap) {
  __shared__ int warp_tot[kConvThreads / 32];
  __shared__ int carry_s;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int br = blockIdx.x; br < Mb; br += gridDim.x) {
    if (threadIdx.x == 0) carry_s = 0;
    __syncthreads();
    const int64_t start = static_cast<int64_t>(row_ptr[br]);
    for (int base = 0; base < Kb; base += kConvThreads) {
      const int j = base + threadIdx.x;
      int* f = flags + static_cast<int64_t>(br) * Kb + j;
      const bool on = j < Kb && *f != 0;
      const unsigned bal = __ballot_sync(0xFFFFFFFFu, on);
      if (lane == 0) warp_tot[warp] = __popc(bal);
      __syncthreads();
      int before = carry_s;
      for (int w = 0; w < warp; ++w) before += warp_tot[w];
      const int rank = before + __popc(bal & ((1u << lane) - 1u));
      if (j < Kb) {
        if (on) {
          if (start + rank < cap) {  // positions past the caller's capacity are mapped but not written
            col_idx[start + rank] = static_cast<IdxOut>(j);
            block_row[start + rank] = br;
          }
          *f = static_cast<int>(start + rank);
        } else {
          *f = -1;
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int t = 0;
        for (int w = 0; w < kConvThreads / 32; ++w) t += warp_tot[w];
        carry_s += t;
      }
      __syncthreads();
    }
  }
}

// The whole index pass of a small block grid (Mb <= kIndexSmallMaxRows, Mb * Kb <= kIndexSmallMaxFlags) in one
// CTA: per-block-row counts of the flags, their exclusive scan into row_ptr[0..Mb] and nnzb, then per block-row
// the ascending ranks of the flagged blocks (col_idx / block_row below `cap`, flags turned into the block-index
// map) -- what bsr_row_counts_kernel, bsr_row_ptr_kernel and bsr_compact_kernel do in three launches.
constexpr int kIndexSmallThreads = 1024;
constexpr int kIndexSmallMaxRows = 4096;
constexpr int64_t kIndexSmallMaxFlags = int64_t(1) << 18;

template <typename IdxOut>
__global__ void __launch_bounds__(kIndexSmallThreads) bsr_index_small_kernel(int* __restrict__ flags, int Mb, int Kb,
                                                                           IdxOut* __restrict__ row_ptr,
                                                                           IdxOut* __restrict__ col_idx,
                                                                           int* __restrict__ block_row, int64_t cap,
                                                                           long long* __restrict__ nnzb_out) {
  constexpr int kWarps = kIndexSmallThreads / 32;
  constexpr int kPerThread = kIndexSmallMaxRows / kIndexSmallThreads;  // rows whose counts a thread scans
  __shared__ int off[kIndexSmallMaxRows];
  __shared__ int warp_tot[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1. flagged blocks per block-row (a warp per row)
  for (int br = warp; br < Mb; br += kWarps) {
    const int* f = flags + static_cast<int64_t>(br) * Kb;
    int c = 0;
    for (int j = lane; j < Kb; j += 32) c += f[j] != 0;
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
    if (lane == 0) off[br] = c;
  }
  __syncthreads();
  // 2. exclusive scan: thread t owns rows [kPerThread t, kPerThread t + kPerThread)
  int local[kPerThread];
  int sum = 0;
#pragma unroll
  for (int u = 0; u < kPerThread; ++u) {
    const int br = kPerThread * threadIdx.x + u;
    local[u] = br < Mb ? off[br] : 0;
    sum += local[u];
  }
  int incl = sum;
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int before = incl - sum;
  for (int w = 0; w < warp; ++w) before += warp_tot[w];
#pragma unroll
  for (int u = 0; u < kPerThread; ++u) {
    const int br = kPerThread * threadIdx.x + u;
    if (br < Mb) {
      off[br] = before;
      row_ptr[br] = static_cast<IdxOut>(before);
    }
    before += local[u];
  }
  if (threadIdx.x == kIndexSmallThreads - 1) {  // the last thread's running sum is the total
    row_ptr[Mb] = static_cast<IdxOut>(before);
    *nnzb_out = before;
  }
  __syncthreads();
  // 3. ranks within each block-row (a warp per row, 32 flags per step)
  for (int br = warp; br < Mb; br += kWarps) {
    int* f = flags + static_cast<int64_t>(br) * Kb;
    const int64_t start = off[br];
    int carry = 0;
    for (int base = 0; base < Kb; base += 32) {
      const int j = base + lane;
      const bool on = j < Kb && f[j] != 0;
      const unsigned bal = __ballot_sync(0xFFFFFFFFu, on);
      const int64_t pos = start + carry + __popc(bal & ((1u << lane) - 1u));
      if (j < Kb) {
        if (on) {
          if (pos < cap) {  // positions past the caller's capacity are mapped but not written
            col_idx[pos] = static_cast<IdxOut>(j);
            block_row[pos] = br;
          }
          f[j] = static_cast<int>(pos);
        } else {
          f[j] = -1;
        }
      }
      carry += __popc(bal);
    }
  }
}

// Fill, step 2 (dense): values[p] = the dense block of stored block p, reading only the stored blocks, for
// p < min(nnzb, cap) (nnzb read from device memory). A warp task is kConvU x 32 units (16-byte chunks when kVec,
// else elements) of one block; block p sits at block-row block_row[p] and block column col_idx[p].
template <int kElemBytes, bool kVec, typename IdxOut>
__global__ void __launch_bounds__(kConvThreads) dense_block_copy_kernel(const uint8_t* __restrict__ A, int64_t lda,
                                                                       int bs, const int* __restrict__ block_row,
                                                                       const IdxOut* __restrict__ col_idx,
                                                                       const long long* __restrict__ nnzb_dev,
                                                                       int64_t cap, uint8_t* __restrict__ values) {
  const int64_t nnzb = min(static_cast<int64_t>(*nnzb_dev), cap);
  constexpr int kUnit = kVec ? 16 : kElemBytes;  // bytes per unit
  const int upr = bs * kElemBytes / kUnit;       // units per block row
  const int upb = upr * bs;                      // units per block
  const int tpb = (upb + 32 * kConvU - 1) / (32 * kConvU);
  const int64_t tasks = nnzb * tpb;
  const int lane = threadIdx.x & 31;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t task = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; task < tasks; task += nw) {
    const int64_t p = task / tpb;
    const int q0 = static_cast<int>(task - p * tpb) * (32 * kConvU) + lane;
    const int64_t br = block_row[p];
    const int64_t bj = static_cast<int64_t>(col_idx[p]);
    const uint8_t* src0 = A + (br * bs * lda + bj * bs) * kElemBytes;
    uint8_t* dst0 = values + p * static_cast<int64_t>(upb) * kUnit;
    if (kVec) {
      uint4 v[kConvU];
#pragma unroll
      for (int u = 0; u < kConvU; ++u) {
        const int q = q0 + 32 * u;
        if (q < upb) {
          const int r = q / upr, cc = q - r * upr;
          v[u] = *reinterpret_cast<const uint4*>(src0 + static_cast<int64_t>(r) * lda * kElemBytes + cc * 16);
        }
      }
#pragma unroll
      for (int u = 0; u < kConvU; ++u) {
        const int q = q0 + 32 * u;
        if (q < upb) reinterpret_cast<uint4*>(dst0)[q] = v[u];
      }
    } else {
#pragma unroll
      for (int u = 0; u < kConvU; ++u) {
        const int q = q0 + 32 * u;
        if (q < upb) {
          const int r = q / upr, cc = q - r * upr;
          const uint8_t* sp = src0 + (static_cast<int64_t>(r) * lda + cc) * kElemBytes;
          if (kElemBytes == 2)
            reinterpret_cast<uint16_t*>(dst0)[q] = *reinterpret_cast<const uint16_t*>(sp);
          else
            reinterpret_cast<uint32_t*>(dst0)[q] = *reinterpret_cast<const uint32_t*>(sp);
        }
      }
    }
  }
}

// Fill, step 2 (CSR): values (zeroed beforehand) receive every in-range entry at its block position, with the
// pattern pass's slicing. A (row, col) pair stored twice ends with one of its values (torch's to_dense would add
// them).
template <int kElemBytes, typename IdxIn, typename E, bool kPow2>
__global__ void __launch_bounds__(kConvThreads) csr_scatter_kernel(const IdxIn* __restrict__ crow,
                                                                  const IdxIn* __restrict__ col,
                                                                  const uint8_t* __restrict__ vals, E nnz, int M, int K,
                                                                  int bs, int lg, int Kb, const int* __restrict__ map,
                                                                  int64_t cap, uint8_t* __restrict__ values) {
  const int lane = threadIdx.x & 31;
  const E eb = crow_at(crow, 0, nnz), ee = crow_at(crow, M, nnz);
  E E0, E1;
  warp_slice(eb, ee, (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5,
             (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5, E0, E1);
  if (E0 >= E1) return;
  int row = csr_row_of(crow, M, E0, nnz);
  E row_end = crow_at(crow, row + 1, nnz);
  const int* mrow = map + static_cast<int64_t>(div_bs<kPow2>(row, bs, lg)) * Kb;
  int r_in = mod_bs<kPow2>(row, bs, lg);
  for (E base = E0 + lane; base < E1 + lane; base += 32 * kConvCsrU) {
    int c[kConvCsrU];
    uint32_t bits[kConvCsrU];
#pragma unroll
    for (int u = 0; u < kConvCsrU; ++u) {
      const E p = base + 32 * u;
      c[u] = p < E1 ? static_cast<int>(max(min(static_cast<int64_t>(col[p]), static_cast<int64_t>(INT32_MAX)),
                                           static_cast<int64_t>(-1)))
                    : -1;
      bits[u] = p < E1 ? load_bits<kElemBytes>(vals + static_cast<int64_t>(p) * kElemBytes) : 0u;
    }
#pragma unroll
    for (int u = 0; u < kConvCsrU; ++u) {
      const E p = base + 32 * u;
      if (p >= E1) break;
      if (p >= row_end) {
        while (p >= row_end && row + 1 < M) row_end = crow_at(crow, ++row + 1, nnz);
        mrow = map + static_cast<int64_t>(div_bs<kPow2>(row, bs, lg)) * Kb;
        r_in = mod_bs<kPow2>(row, bs, lg);
      }
      if (c[u] < 0 || c[u] >= K) continue;
      const int pos = mrow[div_bs<kPow2>(c[u], bs, lg)];
      if (pos < 0 || pos >= cap) continue;  // block of explicit zeros only (not stored), or past capacity
      uint8_t* dst = values +
                     ((static_cast<int64_t>(pos) * bs + r_in) * bs + mod_bs<kPow2>(c[u], bs, lg)) * kElemBytes;
      if (kElemBytes == 2)
        *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(bits[u]);
      else
        *reinterpret_cast<uint32_t*>(dst) = bits[u];
    }
  }
}

// Quad path of the two CSR passes, taken when col is 16-byte aligned and vals is aligned to 4 elements: a lane
// handles whole quads (4 consecutive entries, quad q = entries [4q, 4q + 4)) with one vector load of 4 columns and
// one of 4 values, a warp owns a contiguous run of quads and walks it in trips of 32 x kConvQuadU lane-contiguous
// quads. Entries outside [crow[0], crow[M]) that share a quad with entries inside are loaded and skipped; a quad
// that runs past the end of the arrays (nnz) is loaded entry by entry.
constexpr int kConvQuadU = 4;
constexpr int kConvQuadCtas = 4;  // resident CTAs per SM at the kernels' register budget (<= 64 per thread)

template <typename E>
__device__ __forceinline__ void warp_quads(E eb, E ee, int64_t w, int64_t nw, E& Q0, E& Q1) {
  const int64_t qa = static_cast<int64_t>(eb) >> 2, qb = (static_cast<int64_t>(ee) + 3) >> 2;
  const int64_t n = qb - qa;
  const int64_t per = ((n + nw - 1) / nw + 31) / 32 * 32;
  const int64_t a = w * per, b = a + per;
  Q0 = static_cast<E>(qa + (a < n ? a : n));
  Q1 = static_cast<E>(qa + (b < n ? b : n));
}

// Last r in [0, M) with crow[r] <= e, by a 32-way search over the warp (three rounds for M <= 32768). All lanes
// pass the same e.
template <typename IdxIn, typename E>
__device__ __forceinline__ int csr_row_of_warp(const IdxIn* crow, int M, E e, E nnz, int lane) {
  int lo = 0, hi = M;
  while (hi - lo > 1) {
    const int64_t span = hi - lo;
    const bool le = crow_at(crow, lo + static_cast<int>(span * lane / 32), nnz) <= e;
    const int L = 31 - __clz(__ballot_sync(0xFFFFFFFFu, le) | 1u);
    const int nlo = lo + static_cast<int>(span * L / 32);
    hi = L == 31 ? hi : lo + static_cast<int>(span * (L + 1) / 32);
    lo = nlo;
  }
  return lo;
}

template <typename IdxIn>
__device__ __forceinline__ int clamp_col(IdxIn v) {
  return static_cast<int>(max(min(static_cast<int64_t>(v), static_cast<int64_t>(INT32_MAX)), static_cast<int64_t>(-1)));
}

// Columns (clamped to [-1, INT32_MAX]) and value bits of quad q; entries at or past nnz read as (-1, 0).
template <int kElemBytes, typename IdxIn, typename E>
__device__ __forceinline__ void load_quad(const IdxIn* __restrict__ col, const uint8_t* __restrict__ vals, E q, E nnz,
                                          int (&c)[4], uint32_t (&bits)[4], uint4& raw) {
  const int64_t p0 = static_cast<int64_t>(q) * 4;
  if (p0 + 4 <= static_cast<int64_t>(nnz)) {
    if (sizeof(IdxIn) == 4) {
      const uint4 v = ptx::ldg_stream_16(col + p0);
      c[0] = clamp_col(static_cast<int>(v.x)); c[1] = clamp_col(static_cast<int>(v.y));
      c[2] = clamp_col(static_cast<int>(v.z)); c[3] = clamp_col(static_cast<int>(v.w));
    } else {
      const uint4 v0 = ptx::ldg_stream_16(col + p0), v1 = ptx::ldg_stream_16(col + p0 + 2);
      c[0] = clamp_col(static_cast<long long>((static_cast<uint64_t>(v0.y) << 32) | v0.x));
      c[1] = clamp_col(static_cast<long long>((static_cast<uint64_t>(v0.w) << 32) | v0.z));
      c[2] = clamp_col(static_cast<long long>((static_cast<uint64_t>(v1.y) << 32) | v1.x));
      c[3] = clamp_col(static_cast<long long>((static_cast<uint64_t>(v1.w) << 32) | v1.z));
    }
    if (kElemBytes == 2) {
      const uint2 v = ptx::ldg_stream_8(vals + p0 * 2);
      raw = make_uint4(v.x, v.y, 0u, 0u);
      bits[0] = v.x & 0xFFFFu; bits[1] = v.x >> 16; bits[2] = v.y & 0xFFFFu; bits[3] = v.y >> 16;
    } else {
      raw = ptx::ldg_stream_16(vals + p0 * 4);
      bits[0] = raw.x; bits[1] = raw.y; bits[2] = raw.z; bits[3] = raw.w;
    }
  } else {
    raw = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool in = p0 + j < static_cast<int64_t>(nnz);
      c[j] = in ? clamp_col(col[p0 + j]) : -1;
      bits[j] = in ? load_bits<kElemBytes>(vals + (p0 + j) * kElemBytes) : 0u;
    }
  }
}

// Pattern pass, quad path (same results as csr_flags_kernel).
template <int kElemBytes, typename IdxIn, typename E, bool kPow2>
__global__ void __launch_bounds__(kConvThreads, kConvQuadCtas)
    csr_flags_quad_kernel(const IdxIn* __restrict__ crow, const IdxIn* __restrict__ col,
                          const uint8_t* __restrict__ vals, E nnz, int M, int K, int bs, int lg, int Kb,
                          int* __restrict__ flags, unsigned long long* __restrict__ nnz_out, int* __restrict__ bad) {
  const int lane = threadIdx.x & 31;
  const E eb = crow_at(crow, 0, nnz), ee = crow_at(crow, M, nnz);
  E Q0, Q1;
  warp_quads(eb, ee, (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5,
             (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5, Q0, Q1);
  unsigned long long count = 0;
  if (Q0 < Q1) {
    const E E0 = max(eb, static_cast<E>(4 * Q0)), E1 = min(ee, static_cast<E>(4 * Q1));
    int row = csr_row_of_warp(crow, M, E0, nnz, lane);
    E row_end = crow_at(crow, row + 1, nnz);
    int* frow = flags + static_cast<int64_t>(div_bs<kPow2>(row, bs, lg)) * Kb;
    int* last = nullptr;
    bool any_bad = false;
    auto visit = [&](E p, int c, uint32_t b) {
      if (p >= row_end) {
        while (p >= row_end && row + 1 < M) row_end = crow_at(crow, ++row + 1, nnz);
        frow = flags + static_cast<int64_t>(div_bs<kPow2>(row, bs, lg)) * Kb;
      }
      if (static_cast<unsigned>(c) >= static_cast<unsigned>(K)) {
        any_bad = true;
      } else if (elem_nonzero<kElemBytes>(b)) {
        ++count;
        int* f = frow + div_bs<kPow2>(c, bs, lg);
        if (f != last) {  // a lane's consecutive entries usually share a block: store each flag once per run
          *f = 1;
          last = f;
        }
      }
    };
    for (E qb = Q0 + lane; qb < Q1 + lane; qb += 32 * kConvQuadU) {
      int c[kConvQuadU][4];
      uint32_t bits[kConvQuadU][4];
      uint4 raw[kConvQuadU];
#pragma unroll
      for (int u = 0; u < kConvQuadU; ++u) {
        const E q = qb + 32 * u;
        if (q < Q1) {
          load_quad<kElemBytes>(col, vals, q, nnz, c[u], bits[u], raw[u]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) { c[u][j] = -1; bits[u][j] = 0u; }
        }
      }
#pragma unroll
      for (int u = 0; u < kConvQuadU; ++u) {
        const E q = qb + 32 * u;
        if (q >= Q1) break;
        const E p0 = 4 * q;
        if (p0 >= E0 && p0 + 4 <= E1) {
#pragma unroll
          for (int j = 0; j < 4; ++j) visit(p0 + j, c[u][j], bits[u][j]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (p0 + j >= E0 && p0 + j < E1) visit(p0 + j, c[u][j], bits[u][j]);
        }
      }
    }
    if (any_bad) *bad = 1;
  }
  for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xFFFFFFFFu, count, o);
  if (lane == 0 && count) atomicAdd(nnz_out, count);
}

// Fill step 2, quad path (same results as csr_scatter_kernel). A warp walks its quads last trip first and each
// lane its entries in descending order, so that the entries the pattern pass read last, the ones most likely
// still in L2, are read first. A quad of 4 consecutive in-range columns starting at a multiple of 4 (one block,
// one row) is written with one 4-element store when `values` is aligned to 4 elements and bs % 4 == 0 (kStore4).
template <int kElemBytes, typename IdxIn, typename E, bool kPow2, bool kStore4>
__global__ void __launch_bounds__(kConvThreads, kConvQuadCtas)
    csr_scatter_quad_kernel(const IdxIn* __restrict__ crow, const IdxIn* __restrict__ col,
                            const uint8_t* __restrict__ vals, E nnz, int M, int K, int bs, int lg, int Kb,
                            const int* __restrict__ map, int64_t cap, uint8_t* __restrict__ values) {
  const int lane = threadIdx.x & 31;
  const E eb = crow_at(crow, 0, nnz), ee = crow_at(crow, M, nnz);
  E Q0, Q1;
  warp_quads(eb, ee, (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5,
             (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5, Q0, Q1);
  if (Q0 >= Q1) return;
  const E E0 = max(eb, static_cast<E>(4 * Q0)), E1 = min(ee, static_cast<E>(4 * Q1));
  // rows move backwards only: every entry a lane visits lies below the previous one (row_end stays above it)
  int row = csr_row_of_warp(crow, M, static_cast<E>(E1 - 1), nnz, lane);
  E row_start = crow_at(crow, row, nnz);
  const int* mrow = map + static_cast<int64_t>(div_bs<kPow2>(row, bs, lg)) * Kb;
  int r_in = mod_bs<kPow2>(row, bs, lg);
  auto seek = [&](E p) {
    if (p < row_start) {
      while (p < row_start && row > 0) row_start = crow_at(crow, --row, nnz);
      mrow = map + static_cast<int64_t>(div_bs<kPow2>(row, bs, lg)) * Kb;
      r_in = mod_bs<kPow2>(row, bs, lg);
    }
  };
  auto put = [&](int c, uint32_t b) {
    if (static_cast<unsigned>(c) >= static_cast<unsigned>(K)) return;
    const int pos = mrow[div_bs<kPow2>(c, bs, lg)];
    if (pos < 0 || pos >= cap) return;  // block of explicit zeros only (not stored), or past capacity
    uint8_t* dst = values + ((static_cast<int64_t>(pos) * bs + r_in) * bs + mod_bs<kPow2>(c, bs, lg)) * kElemBytes;
    if (kElemBytes == 2)
      *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(b);
    else
      *reinterpret_cast<uint32_t*>(dst) = b;
  };
  const int64_t trips = (static_cast<int64_t>(Q1 - Q0) + 32 * kConvQuadU - 1) / (32 * kConvQuadU);
  for (int64_t t = trips - 1; t >= 0; --t) {
    const E qb = Q0 + static_cast<E>(t * 32 * kConvQuadU) + lane;
    int c[kConvQuadU][4];
    uint32_t bits[kConvQuadU][4];
    uint4 raw[kConvQuadU];
#pragma unroll
    for (int u = 0; u < kConvQuadU; ++u) {
      const E q = qb + 32 * u;
      if (q < Q1) {
        load_quad<kElemBytes>(col, vals, q, nnz, c[u], bits[u], raw[u]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) { c[u][j] = -1; bits[u][j] = 0u; }
        raw[u] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int u = kConvQuadU - 1; u >= 0; --u) {
      const E q = qb + 32 * u;
      if (q >= Q1) continue;
      const E p0 = 4 * q;
      if (p0 >= E0 && p0 + 4 <= E1) {
        seek(p0 + 3);
        if (kStore4 && p0 >= row_start && (c[u][0] & 3) == 0 && c[u][1] == c[u][0] + 1 &&
            c[u][2] == c[u][0] + 2 && c[u][3] == c[u][0] + 3 && c[u][0] >= 0 && c[u][3] < K) {
          const int pos = mrow[div_bs<kPow2>(c[u][0], bs, lg)];
          if (pos >= 0 && pos < cap) {
            uint8_t* dst = values +
                           ((static_cast<int64_t>(pos) * bs + r_in) * bs + mod_bs<kPow2>(c[u][0], bs, lg)) * kElemBytes;
            if (kElemBytes == 2)
              *reinterpret_cast<uint2*>(dst) = make_uint2(raw[u].x, raw[u].y);
            else
              *reinterpret_cast<uint4*>(dst) = raw[u];
          }
          continue;
        }
#pragma unroll
        for (int j = 3; j >= 0; --j) {
          seek(p0 + j);
          put(c[u][j], bits[u][j]);
        }
      } else {
#pragma unroll
        for (int j = 3; j >= 0; --j) {
          if (p0 + j < E0 || p0 + j >= E1) continue;
          seek(p0 + j);
          put(c[u][j], bits[u][j]);
        }
      }
    }
  }
}

// values[0 .. min(nnzb, cap) blocks) = 0 (nnzb read from device memory): 16-byte stores when the span allows.
__global__ void __launch_bounds__(kConvThreads) zero_blocks_kernel(uint8_t* __restrict__ values,
                                                                  const long long* __restrict__ nnzb_dev, int64_t cap,
                                                                  int64_t block_bytes) {
  const int64_t bytes = min(static_cast<int64_t>(*nnzb_dev), cap) * block_bytes;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool vec = (reinterpret_cast<uintptr_t>(values) & 15u) == 0;
  const int64_t nvec = vec ? bytes / 16 : 0;
  for (int64_t i = t0; i < nvec; i += stride) reinterpret_cast<uint4*>(values)[i] = make_uint4(0, 0, 0, 0);
  for (int64_t i = nvec * 16 + t0; i < bytes; i += stride) values[i] = 0;
}

// Host-side launchers of the CSR kernels for one input index type: 32-bit entry indices when nnz < 2^31,
// shifts when bs is a power of two.
inline int log2_exact(int bs) {
  int lg = 0;
  while ((1 << lg) < bs) ++lg;
  return (1 << lg) == bs ? lg : -1;
}

inline bool csr_quad_ok(const void* col, const void* vals, int elem_bytes) {
  return reinterpret_cast<uintptr_t>(col) % 16 == 0 && reinterpret_cast<uintptr_t>(vals) % (4 * elem_bytes) == 0;
}

template <typename IdxIn>
void launch_csr_flags(int elem_bytes, const void* crow, const void* col, const void* vals, int64_t nnz, int M, int K,
                      int bs, int Kb, int* flags, unsigned long long* counter, int* bad, int sm_count,
                      cudaStream_t s) {
  const IdxIn* c = static_cast<const IdxIn*>(crow);
  const IdxIn* ci = static_cast<const IdxIn*>(col);
  const uint8_t* v = static_cast<const uint8_t*>(vals);
  const int lg = log2_exact(bs);
  const bool small = nnz < (int64_t(1) << 31) - 32 * kConvCsrU * 2;
  const bool quad = csr_quad_ok(col, vals, elem_bytes);
#define BSK_CF(EB, E, P)                                                                                              \
  do {                                                                                                                \
    if (quad)                                                                                                         \
      csr_flags_quad_kernel<EB, IdxIn, E, P><<<sm_count * kConvQuadCtas, kConvThreads, 0, s>>>(                      \
          c, ci, v, static_cast<E>(nnz), M, K, bs, lg, Kb, flags, counter, bad);                                      \
    else                                                                                                              \
      csr_flags_kernel<EB, IdxIn, E, P><<<sm_count * 8, kConvThreads, 0, s>>>(c, ci, v, static_cast<E>(nnz), M, K,   \
                                                                              bs, lg, Kb, flags, counter, bad);       \
  } while (0)
  if (elem_bytes == 2) {
    if (small) { if (lg >= 0) BSK_CF(2, int, true); else BSK_CF(2, int, false); }
    else { if (lg >= 0) BSK_CF(2, int64_t, true); else BSK_CF(2, int64_t, false); }
  } else {
    if (small) { if (lg >= 0) BSK_CF(4, int, true); else BSK_CF(4, int, false); }
    else { if (lg >= 0) BSK_CF(4, int64_t, true); else BSK_CF(4, int64_t, false); }
  }
#undef BSK_CF
}

template <typename IdxIn>
void launch_csr_scatter(int elem_bytes, const void* crow, const void* col, const void* vals, int64_t nnz, int M,
                        int K, int bs, int Kb, const int* map, int64_t cap, void* values, int sm_count,
                        cudaStream_t s) {
  const IdxIn* c = static_cast<const IdxIn*>(crow);
  const IdxIn* ci = static_cast<const IdxIn*>(col);
  const uint8_t* v = static_cast<const uint8_t*>(vals);
  uint8_t* out = static_cast<uint8_t*>(values);
  const int lg = log2_exact(bs);
  const bool small = nnz < (int64_t(1) << 31) - 32 * kConvCsrU * 2;
  const bool quad = csr_quad_ok(col, vals, elem_bytes);
  const bool store4 = reinterpret_cast<uintptr_t>(values) % (4 * elem_bytes) == 0 && bs % 4 == 0;
#define BSK_CS(EB, E, P)                                                                                              \
  do {                                                                                                                \
    const int g = sm_count * kConvQuadCtas;                                                                           \
    if (quad && store4)                                                                                               \
      csr_scatter_quad_kernel<EB, IdxIn, E, P, true><<<g, kConvThreads, 0, s>>>(c, ci, v, static_cast<E>(nnz), M, K, \
                                                                                bs, lg, Kb, map, cap, out);           \
    else if (quad)                                                                                                    \
      csr_scatter_quad_kernel<EB, IdxIn, E, P, false><<<g, kConvThreads, 0, s>>>(c, ci, v, static_cast<E>(nnz), M,   \
                                                                                 K, bs, lg, Kb, map, cap, out);       \
    else                                                                                                              \
      csr_scatter_kernel<EB, IdxIn, E, P><<<sm_count * 8, kConvThreads, 0, s>>>(c, ci, v, static_cast<E>(nnz), M, K, \
                                                                                bs, lg, Kb, map, cap, out);           \
  } while (0)
  if (elem_bytes == 2) {
    if (small) { if (lg >= 0) BSK_CS(2, int, true); else BSK_CS(2, int, false); }
    else { if (lg >= 0) BSK_CS(2, int64_t, true); else BSK_CS(2, int64_t, false); }
  } else {
    if (small) { if (lg >= 0) BSK_CS(4, int, true); else BSK_CS(4, int, false); }
    else { if (lg >= 0) BSK_CS(4, int64_t, true); else BSK_CS(4, int64_t, false); }
  }
#undef BSK_CS
}

}  // namespace bsk
