// Wrapper that exposes the reference's own CPU BSR checker cpu_bsr (BlackwellSparseK/src/bsr_reference.cu:72-93)
// through a C signature -- TEST INFRASTRUCTURE ONLY. The reference source is included from its location in the
// reference checkout at build time (path in BSK_REF_SRC); nothing of it is copied. Its main() is renamed so the
// translation unit links as a shared library. The reference fixes BM=128, BN=128, BK=64.
#include <cstring>
#include <vector>
#define main bsk_reference_bsr_main
#include BSK_REF_SRC
#undef main

extern "C" int ref_block_dims(int* bm, int* bn, int* bk) {
  *bm = BM;
  *bn = BN;
  *bk = BK;
  return 0;
}

extern "C" void ref_cpu_bsr(const unsigned short* A_blocks, long long nA, const int* row_ptr, int Mb,
                            const int* col_idx, int nnz, const unsigned short* B, long long nB, float* C, int M, int N,
                            int K) {
  std::vector<half> a(nA), b(nB);
  std::memcpy(a.data(), A_blocks, nA * sizeof(unsigned short));
  std::memcpy(b.data(), B, nB * sizeof(unsigned short));
  std::vector<int> rp(row_ptr, row_ptr + Mb + 1), ci(col_idx, col_idx + nnz);
  std::vector<float> c((size_t)M * N);
  cpu_bsr(a, rp, ci, b, c, M, N, K, Mb, (N + BN - 1) / BN);
  std::memcpy(C, c.data(), c.size() * sizeof(float));
}
