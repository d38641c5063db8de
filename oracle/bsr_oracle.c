/*
 * Plain-C restatement of the reference's CPU BSR checker -- TEST INFRASTRUCTURE ONLY.
 *
 * Follows cpu_bsr (BlackwellSparseK/src/bsr_reference.cu:72-93): C is cleared, then for every output
 * block (bm, bn) and every nonzero block idx of block-row bm, each C element receives one fp32 partial
 * sum over the block's k range (products of fp16 values converted exactly to fp32, accumulated in k
 * order), added to C in nonzero order. Blocks are BM x BK, row-major; B is row-major [K, N]; edges are
 * clipped exactly as the reference clips them (i < M, j < N, k < K).
 *
 * Built with -ffp-contract=off (as is the reference's host code by oracle/build_ref.sh) so that both
 * evaluate a*b then +, and the two agree bit for bit.
 */
#include <stdint.h>
#include <string.h>

/* IEEE-754 binary16 -> binary32, exact (every half is representable as a float). */
static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while ((man & 0x400u) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 0x1Fu) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

void oracle_half_to_float(const uint16_t* h, float* f, int64_t n) {
  for (int64_t i = 0; i < n; ++i) f[i] = half_to_float(h[i]);
}

void oracle_cpu_bsr(const uint16_t* A_blocks, const int32_t* row_ptr, const int32_t* col_idx, const uint16_t* B,
                    float* C, int M, int N, int K, int BM, int BN, int BK) {
  const int Mb = (M + BM - 1) / BM;
  const int Nb = (N + BN - 1) / BN;
  for (int64_t t = 0; t < (int64_t)M * N; ++t) C[t] = 0.0f;
  for (int bm = 0; bm < Mb; ++bm) {
    for (int bn = 0; bn < Nb; ++bn) {
      for (int idx = row_ptr[bm]; idx < row_ptr[bm + 1]; ++idx) {
        const int kb = col_idx[idx];
        for (int i = 0; i < BM && bm * BM + i < M; ++i) {
          for (int j = 0; j < BN && bn * BN + j < N; ++j) {
            float sum = 0.0f;
            for (int k = 0; k < BK && kb * BK + k < K; ++k) {
              const float a = half_to_float(A_blocks[(int64_t)idx * BM * BK + i * BK + k]);
              const float b = half_to_float(B[(int64_t)(kb * BK + k) * N + (bn * BN + j)]);
              sum += a * b;
            }
            C[(int64_t)(bm * BM + i) * N + (bn * BN + j)] += sum;
          }
        }
      }
    }
  }
}
