// Host side of the C ABI (include/bsk_capi.h): argument validation, per-device set-up, TMA tensor-map
// encoding and kernel launches. One translation unit holds every kernel of the library so that the
// device error word below is a single symbol.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "bsk_capi.h"
#include "gemm_sm100.cuh"
#include "gemm_pair_sm100.cuh"
#include "bsr_pair_sm100.cuh"
#include "bsattn_sm100.cuh"
#include "bsr_convert.cuh"
#include "bsattn_bwd_sm100.cuh"

namespace {

// Per-device error word written by bounded waits and device-side index checks.
__device__ uint32_t g_bsk_err_word;

thread_local std::string t_last_error;
thread_local uint64_t t_timeout_ns = 2000000000ull;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return set_error(BSK_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;

struct DeviceState {
  std::once_flag once;
  int status = BSK_OK;
  std::string init_error;
  int sm_count = 0;
  int pair_clusters = 0;       // co-resident 2-CTA clusters of the pair GEMM kernels (all share one footprint)
  int bsr_pair_clusters = 0;   // co-resident 2-CTA clusters of the pair BSR SpMM kernel (0: not used)
  uint32_t* err_word = nullptr;
};
DeviceState g_devices[kMaxDevices];

std::once_flag g_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

template <class K>
cudaError_t allow_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// How many 2-CTA clusters of `kernel` can be resident at once (persistent grids are sized to this).
template <class K>
int max_clusters(K kernel, int threads, int smem) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(kernel), &cfg) != cudaSuccess) return -1;
  return n;
}

// Per-shape launch configurations registered by the caller (an autotuner and its persisted cache): for an
// operator and an exact (M, N, K), the tile kind (-1 = the built-in policy) and the rasterisation group (<= 0 =
// the built-in choice). Process-wide, guarded by a mutex; looked up once per launch.
struct ShapeConfig {
  int op, M, N, K, tile, group;
};
std::mutex g_cfg_mu;
std::vector<ShapeConfig> g_cfg;

bool find_config(int op, int M, int N, int K, int* tile, int* group) {
  std::lock_guard<std::mutex> lk(g_cfg_mu);
  for (const ShapeConfig& c : g_cfg)
    if (c.op == op && c.M == M && c.N == N && c.K == K) {
      *tile = c.tile;
      *group = c.group;
      return true;
    }
  return false;
}

// Tile policy of the dense GEMMs (0 = single-CTA 128x256, 1 = CTA pair 256x256, 2 = CTA pair 256x512):
// single when M fits one 128-row tile; the wide pair tile when N and K are large enough that its exposed
// per-tile epilogue (one 512-column accumulator) is amortised; otherwise the double-buffered 256x256 tile.
// BSK_GEMM_TILE=single|pair|wide overrides (diagnostics and tests).
int gemm_tile_kind(int M, int N, int K) {
  const char* v = getenv("BSK_GEMM_TILE");
  if (v && strcmp(v, "single") == 0) return 0;
  if (v && strcmp(v, "pair") == 0) return 1;
  if (v && strcmp(v, "wide") == 0) return 2;
  if (M <= 128) return 0;
  return (N >= 512 && K >= 8192) ? 2 : 1;
}

void init_device(DeviceState& st, int dev) {
  int major = 0, minor = 0;
  cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (e != cudaSuccess) {
    st.status = BSK_ERR_NO_DEVICE;
    st.init_error = std::string("device query failed: ") + cudaGetErrorString(e);
    return;
  }
  if (major != 10 || minor != 0) {
    st.status = BSK_ERR_UNSUPPORTED;
    char b[128];
    snprintf(b, sizeof(b), "device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev, major,
             minor);
    st.init_error = b;
    return;
  }
  cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev);
  using namespace bsk;
  const cudaError_t errs[] = {
      allow_smem(gemm_sm100_kernel<2, Mainloop::Dense, Epi::F32>, kGemmSmemBytes),
      allow_smem(gemm_sm100_kernel<1, Mainloop::Dense, Epi::BF16Scaled>, kGemmSmemBytes),
      allow_smem(gemm_sm100_kernel<2, Mainloop::Bsr, Epi::F32>, kGemmSmemBytes),
      allow_smem(gemm_sm100_kernel<2, Mainloop::BsrBsr, Epi::F32>, kGemmBsrBsrSmemBytes),
      allow_smem(bsattn_sm100_kernel<false, 128>, AttnShape<false, 128>::kSmemBytes),
      allow_smem(bsattn_sm100_kernel<false, 64>, AttnShape<false, 64>::kSmemBytes),
      allow_smem(bsattn_sm100_kernel<true, 128>, AttnShape<true, 128>::kSmemBytes),
      allow_smem(bsattn_sm100_kernel<true, 64>, AttnShape<true, 64>::kSmemBytes),
      allow_smem(bsattn_bwd_dq_kernel<false, 128>, BwdDqShape<false, 128>::kSmemBytes),
      allow_smem(bsattn_bwd_dq_kernel<false, 64>, BwdDqShape<false, 64>::kSmemBytes),
      allow_smem(bsattn_bwd_dq_kernel<true, 128>, BwdDqShape<true, 128>::kSmemBytes),
      allow_smem(bsattn_bwd_dq_kernel<true, 64>, BwdDqShape<true, 64>::kSmemBytes),
      allow_smem(bsattn_bwd_dkdv_kernel<false, 128>, BwdDkdvShape<false, 128>::kSmemBytes),
      allow_smem(bsattn_bwd_dkdv_kernel<false, 64>, BwdDkdvShape<false, 64>::kSmemBytes),
      allow_smem(bsattn_bwd_dkdv_kernel<true, 128>, BwdDkdvShape<true, 128>::kSmemBytes),
      allow_smem(bsattn_bwd_dkdv_kernel<true, 64>, BwdDkdvShape<true, 64>::kSmemBytes),
      allow_smem(gemm_pair_sm100_kernel<2, Epi::F32, 1>, kPairSmemBytes),
      allow_smem(gemm_pair_sm100_kernel<1, Epi::BF16Scaled, 1>, kPairSmemBytes),
      allow_smem(gemm_pair_sm100_kernel<2, Epi::F32, 2>, kPairWideSmemBytes),
      allow_smem(gemm_pair_sm100_kernel<2, Epi::F32PeerRows, 1>, kPairSmemBytes),
      allow_smem(gemm_pair_sm100_kernel<2, Epi::F32PeerRows, 2>, kPairWideSmemBytes),
      allow_smem(gemm_pair_sm100_kernel<1, Epi::BF16Scaled, 2>, kPairWideSmemBytes),
      allow_smem(spmm_bsr_pair_sm100_kernel, kBsrPairSmemBytes),
  };
  for (cudaError_t x : errs) {
    if (x != cudaSuccess) {
      st.status = BSK_ERR_CUDA;
      st.init_error = std::string("cudaFuncSetAttribute failed: ") + cudaGetErrorString(x);
      return;
    }
  }
  {
    const int c[4] = {max_clusters(gemm_pair_sm100_kernel<2, Epi::F32, 1>, kPairThreads, kPairSmemBytes),
                      max_clusters(gemm_pair_sm100_kernel<1, Epi::BF16Scaled, 1>, kPairThreads, kPairSmemBytes),
                      max_clusters(gemm_pair_sm100_kernel<2, Epi::F32, 2>, kPairThreads, kPairWideSmemBytes),
                      max_clusters(gemm_pair_sm100_kernel<1, Epi::BF16Scaled, 2>, kPairThreads, kPairWideSmemBytes)};
    st.pair_clusters = c[0];
    for (int i = 1; i < 4; ++i) st.pair_clusters = c[i] < st.pair_clusters ? c[i] : st.pair_clusters;
  }
  st.bsr_pair_clusters = max_clusters(spmm_bsr_pair_sm100_kernel, kPairThreads, kBsrPairSmemBytes);
  if (st.pair_clusters <= 0) {
    st.status = BSK_ERR_CUDA;
    st.init_error = "cudaOccupancyMaxActiveClusters reports no co-resident CTA pair";
    return;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_bsk_err_word);
  if (e != cudaSuccess) {
    st.status = BSK_ERR_CUDA;
    st.init_error = std::string("cudaGetSymbolAddress(error word) failed: ") + cudaGetErrorString(e);
    return;
  }
  st.err_word = static_cast<uint32_t*>(p);
  e = cudaMemset(st.err_word, 0, sizeof(uint32_t));
  if (e != cudaSuccess) {
    st.status = BSK_ERR_CUDA;
    st.init_error = std::string("clearing the error word failed: ") + cudaGetErrorString(e);
  }
}

int device_state(DeviceState** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(BSK_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
  int count = 0;
  e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) return set_error(BSK_ERR_NO_DEVICE, "no CUDA device available");
  if (dev < 0 || dev >= kMaxDevices) return set_error(BSK_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
  DeviceState& st = g_devices[dev];
  std::call_once(st.once, [&] { init_device(st, dev); });
  if (st.status != BSK_OK) return set_error(st.status, "%s", st.init_error.c_str());
  *out = &st;
  return BSK_OK;
}

int encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  std::call_once(g_encode_once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  if (!g_encode) return set_error(BSK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  *fn = g_encode;
  return BSK_OK;
}

// Row-major 2-D (or, with `planes`, 3-D) tensor map with 128-B swizzle.
int make_map(CUtensorMap* m, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t inner,
             uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, const char* what) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (int rc = encoder(&enc)) return rc;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(BSK_ERR_INVALID_ARG, "%s: base address must be 16-byte aligned", what);
  if (row_stride_bytes % 16 != 0)
    return set_error(BSK_ERR_INVALID_ARG, "%s: row stride (%llu bytes) must be a multiple of 16", what,
                     (unsigned long long)row_stride_bytes);
  if (inner == 0 || outer == 0) return set_error(BSK_ERR_INVALID_ARG, "%s: empty tensor map", what);
  if (box_inner * elem_bytes > 128)
    return set_error(BSK_ERR_INVALID_ARG, "%s: box inner extent exceeds the 128-B swizzle span", what);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(BSK_ERR_INVALID_ARG, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return BSK_OK;
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return BSK_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// M tiles per rasterisation group: concurrent tiles then span ~2048 rows of A and a few B column panels.
// Measured on B200 (same-box A/B): with long K the 256x512 tile runs fastest when a wave's tiles walk the whole
// M extent of a couple of column panels (group 32: 8192x8192x237568 +3.5 % over group 12); with K = 16384 the
// smaller group is as good or better; the 1-CTA BSR tiles prefer 64 block-rows per group (+4 %).
#ifndef BSK_WIDE_GROUP_M
#define BSK_WIDE_GROUP_M 12
#endif
#ifndef BSK_WIDE_LONGK_GROUP_M
#define BSK_WIDE_LONGK_GROUP_M 32
#endif
#ifndef BSK_PAIR_GROUP_M
#define BSK_PAIR_GROUP_M 8
#endif
#ifndef BSK_SINGLE_GROUP_M
#define BSK_SINGLE_GROUP_M 64
#endif
int pick_group_m(int num_m_tiles, int kind = 0, int k_extent = 0) {
  const int g = kind == 2 ? (k_extent >= 65536 ? BSK_WIDE_LONGK_GROUP_M : BSK_WIDE_GROUP_M)
                          : (kind == 1 ? BSK_PAIR_GROUP_M : BSK_SINGLE_GROUP_M);
  return num_m_tiles < g ? num_m_tiles : g;
}

// Tile kind and rasterisation group for one launch: the registered configuration of (op, M, N, K) where one
// exists (tile kinds the operator lacks fall back to the policy), else the built-in policy.
void launch_config(int op, int M, int N, int K, bool has_tiles, int* kind, int* group_for_tiles) {
  int tile = -1, group = 0;
  find_config(op, M, N, K, &tile, &group);
  *kind = has_tiles ? ((tile >= 0 && tile <= 2) ? tile : gemm_tile_kind(M, N, K)) : 0;
  *group_for_tiles = group;
}

int resolve_group(int group, int num_m_tiles, int kind, int k_extent) {
  if (group > 0) return group < num_m_tiles ? group : num_m_tiles;
  return pick_group_m(num_m_tiles, kind, k_extent);
}

}  // namespace

extern "C" {

int bsk_version(void) { return (0 << 16) | (1 << 8) | 0; }

const char* bsk_last_error(void) { return t_last_error.c_str(); }

int bsk_device_sm_count(void) {
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  return st->sm_count;
}

int bsk_config_set(int op, int M, int N, int K, int tile, int group_m) {
  if (op < BSK_OP_GEMM_F16F32 || op > BSK_OP_SPMM_BSR_BSR)
    return set_error(BSK_ERR_INVALID_ARG, "config_set: unknown operator %d", op);
  if (M < 0 || N < 0 || K < 0) return set_error(BSK_ERR_INVALID_ARG, "config_set: negative extent");
  if (tile < -1 || tile > 2) return set_error(BSK_ERR_INVALID_ARG, "config_set: tile %d not in {-1, 0, 1, 2}", tile);
  if (group_m < 0 || group_m > 4096) return set_error(BSK_ERR_INVALID_ARG, "config_set: group_m %d outside [0, 4096]", group_m);
  std::lock_guard<std::mutex> lk(g_cfg_mu);
  for (ShapeConfig& c : g_cfg)
    if (c.op == op && c.M == M && c.N == N && c.K == K) {
      c.tile = tile;
      c.group = group_m;
      return BSK_OK;
    }
  g_cfg.push_back({op, M, N, K, tile, group_m});
  return BSK_OK;
}

int bsk_config_get(int op, int M, int N, int K, int* tile, int* group_m) {
  if (!tile || !group_m) return set_error(BSK_ERR_INVALID_ARG, "config_get: null output");
  *tile = -1;
  *group_m = 0;
  return find_config(op, M, N, K, tile, group_m) ? 1 : 0;
}

int bsk_config_clear(void) {
  std::lock_guard<std::mutex> lk(g_cfg_mu);
  g_cfg.clear();
  return BSK_OK;
}

int bsk_set_wait_timeout_ns(uint64_t ns) {
  if (ns < 1000ull || ns > 60000000000ull)
    return set_error(BSK_ERR_INVALID_ARG, "wait timeout %llu ns outside [1e3, 6e10]", (unsigned long long)ns);
  t_timeout_ns = ns;
  return BSK_OK;
}

namespace {

// Dense fp16 GEMM over K range [k_begin, k_end): C = A B (accumulate = 0) or C += A B (accumulate = 1).
int gemm_f16_launch(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M, int N,
                    int K, int k_begin, int k_end, int accumulate, void* stream) {
  using namespace bsk;
  if (M < 0 || N < 0 || K < 0) return set_error(BSK_ERR_INVALID_ARG, "gemm_f16f32: negative extent");
  if (k_begin < 0 || k_end > K || k_begin > k_end)
    return set_error(BSK_ERR_INVALID_ARG, "gemm_f16f32: bad K range [%d, %d) for K=%d", k_begin, k_end, K);
  if (k_begin % 8 != 0) return set_error(BSK_ERR_INVALID_ARG, "gemm_f16f32: k_begin must be a multiple of 8");
  if (lda < K || ldb < K || ldc < N)
    return set_error(BSK_ERR_INVALID_ARG, "gemm_f16f32: leading dimensions smaller than the extents");
  if (lda % 8 || ldb % 8) return set_error(BSK_ERR_INVALID_ARG, "gemm_f16f32: lda and ldb must be multiples of 8");
  if (!A || !B || !C) return set_error(BSK_ERR_INVALID_ARG, "gemm_f16f32: null pointer");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (M == 0 || N == 0) return BSK_OK;
  const int kr = k_end - k_begin;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (kr == 0) {
    if (accumulate) return BSK_OK;  // C += 0
    cudaError_t e = cudaMemset2DAsync(C, ldc * sizeof(float), 0, (size_t)N * sizeof(float), M, s);
    return e == cudaSuccess ? BSK_OK : cuda_fail(e, "gemm_f16f32: zero fill");
  }
  const __half* Ah = static_cast<const __half*>(A) + k_begin;
  const __half* Bh = static_cast<const __half*>(B) + k_begin;
  int kind, group;
  launch_config(BSK_OP_GEMM_F16F32, M, N, kr, true, &kind, &group);
  const uint32_t a_rows = kind ? 128 : kGemmBM;  // rows per CTA of the A tile
  const uint32_t b_rows = kind ? 128 : kGemmBN;  // rows of B^T per TMA box
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Ah, kr, M, lda * 2, 64, a_rows, "A")) return rc;
  if (int rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Bh, kr, N, ldb * 2, 64, b_rows, "B")) return rc;
  GemmArgs a{};
  const int tm = kind ? kPairBM : kGemmBM, tn = kind == 2 ? 512 : kGemmBN;
  a.M = M;
  a.N = N;
  a.num_m_tiles = (M + tm - 1) / tm;
  a.num_n_tiles = (N + tn - 1) / tn;
  a.num_k_blocks = (kr + 63) / 64;
  a.group_m = resolve_group(group, a.num_m_tiles, kind, kr);
  a.k_splits = 1;
  a.kb_per_split = a.num_k_blocks;
  a.out = C;
  a.ldo = ldc;
  a.vec_ok = aligned16(C) && (ldc % 4 == 0);
  a.accumulate = accumulate;
  a.err = st->err_word;
  a.timeout_ns = t_timeout_ns;
  const int tiles = a.num_m_tiles * a.num_n_tiles;
  const int clusters = tiles < st->pair_clusters ? tiles : st->pair_clusters;
  if (kind == 2) {
    gemm_pair_sm100_kernel<2, Epi::F32, 2><<<2 * clusters, kPairThreads, kPairWideSmemBytes, s>>>(ta, tb, a);
  } else if (kind == 1) {
    gemm_pair_sm100_kernel<2, Epi::F32, 1><<<2 * clusters, kPairThreads, kPairSmemBytes, s>>>(ta, tb, a);
  } else {
    const int grid = tiles < st->sm_count ? tiles : st->sm_count;
    gemm_sm100_kernel<2, Mainloop::Dense, Epi::F32><<<grid, kGemmThreads, kGemmSmemBytes, s>>>(ta, tb, a);
  }
  return launch_status("gemm_f16f32 launch");
}

}  // namespace

int bsk_gemm_f16f32(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M, int N,
                    int K, int k_begin, int k_end, void* stream) {
  return gemm_f16_launch(A, lda, B, ldb, C, ldc, M, N, K, k_begin, k_end, 0, stream);
}

int bsk_gemm_f16f32_acc(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M, int N,
                        int K, int k_begin, int k_end, void* stream) {
  return gemm_f16_launch(A, lda, B, ldb, C, ldc, M, N, K, k_begin, k_end, 1, stream);
}

namespace {

// K-chunk plan of the host-streaming GEMM: chunk width (multiple of 64), device workspace layout.
struct HostPlan {
  int kc = 0;             // K elements per chunk (pitch of the chunk buffers)
  int64_t a_bytes = 0;    // one A chunk buffer [M, kc] fp16
  int64_t b_bytes = 0;    // one B^T chunk buffer [N, kc] fp16
  int64_t ldc_dev = 0;    // row stride of the device C
  int64_t total = 0;      // A0, A1, B0, B1, C, each rounded up to 256 bytes
};

int64_t round256(int64_t x) { return (x + 255) / 256 * 256; }

// Row panel of the host-streaming GEMM's last chunk: about 8 panels, whole 256-row tiles, at least one tile.
int host_panel_rows(int M) {
  int r = (M + 7) / 8;
  r = (r + 255) / 256 * 256;
  return r > 0 ? r : 256;
}

HostPlan plan_host(int M, int N, int K, int k_chunk) {
  HostPlan p;
  int kc = k_chunk;
  if (kc <= 0) {  // ~16 chunks of >= 4096 (enough K per launch to keep the tiles busy), never above K
    kc = (K + 15) / 16;
    if (kc < 4096) kc = 4096;
  }
  kc = (kc + 63) / 64 * 64;
  const int k_pad = (K + 63) / 64 * 64;
  if (kc > k_pad) kc = k_pad > 0 ? k_pad : 64;
  p.kc = kc;
  p.a_bytes = round256((int64_t)M * kc * 2);
  p.b_bytes = round256((int64_t)N * kc * 2);
  p.ldc_dev = (N + 3) / 4 * 4;
  p.total = 2 * p.a_bytes + 2 * p.b_bytes + round256((int64_t)M * p.ldc_dev * 4);
  return p;
}

}  // namespace

int bsk_gemm_host_chunk(int K, int k_chunk) {
  if (K < 0) return set_error(BSK_ERR_INVALID_ARG, "gemm_host: negative K");
  if (k_chunk > 0 && k_chunk % 64) return set_error(BSK_ERR_INVALID_ARG, "gemm_host: k_chunk must be a multiple of 64");
  return plan_host(1, 1, K, k_chunk).kc;
}

int bsk_copy_2d_async(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width_bytes, int64_t rows,
                      void* stream) {
  if (width_bytes < 0 || rows < 0 || dpitch < width_bytes || spitch < width_bytes)
    return set_error(BSK_ERR_INVALID_ARG, "copy_2d: bad extents");
  if (width_bytes == 0 || rows == 0) return BSK_OK;
  if (!dst || !src) return set_error(BSK_ERR_INVALID_ARG, "copy_2d: null pointer");
  cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)dpitch, src, (size_t)spitch, (size_t)width_bytes, (size_t)rows,
                                    cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BSK_OK : cuda_fail(e, "copy_2d");
}

int64_t bsk_gemm_host_workspace_bytes(int M, int N, int K, int k_chunk) {
  if (M < 0 || N < 0 || K < 0) return set_error(BSK_ERR_INVALID_ARG, "gemm_host: negative extent");
  if (k_chunk > 0 && k_chunk % 64) return set_error(BSK_ERR_INVALID_ARG, "gemm_host: k_chunk must be a multiple of 64");
  return plan_host(M, N, K, k_chunk).total;
}

int bsk_gemm_f16f32_host(const void* A_host, int64_t lda, const void* B_host, int64_t ldb, float* C_host,
                         int64_t ldc, int M, int N, int K, int k_chunk, void* workspace, int64_t workspace_bytes,
                         void* stream) {
  using namespace bsk;
  if (M < 0 || N < 0 || K < 0) return set_error(BSK_ERR_INVALID_ARG, "gemm_host: negative extent");
  if (lda < K || ldb < K || ldc < N) return set_error(BSK_ERR_INVALID_ARG, "gemm_host: leading dimensions smaller than the extents");
  if (k_chunk > 0 && k_chunk % 64) return set_error(BSK_ERR_INVALID_ARG, "gemm_host: k_chunk must be a multiple of 64");
  if (!A_host || !B_host || !C_host) return set_error(BSK_ERR_INVALID_ARG, "gemm_host: null host pointer");
  const HostPlan p = plan_host(M, N, K, k_chunk);
  if (!workspace || workspace_bytes < p.total)
    return set_error(BSK_ERR_INVALID_ARG, "gemm_host: workspace of %lld bytes needed, %lld given", (long long)p.total,
                     (long long)workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return set_error(BSK_ERR_INVALID_ARG, "gemm_host: workspace must be 256-byte aligned");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (M == 0 || N == 0) return BSK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  __half* abuf[2] = {reinterpret_cast<__half*>(ws), reinterpret_cast<__half*>(ws + p.a_bytes)};
  __half* bbuf[2] = {reinterpret_cast<__half*>(ws + 2 * p.a_bytes),
                     reinterpret_cast<__half*>(ws + 2 * p.a_bytes + p.b_bytes)};
  float* Cd = reinterpret_cast<float*>(ws + 2 * p.a_bytes + 2 * p.b_bytes);
  const int nchunks = K == 0 ? 0 : (K + p.kc - 1) / p.kc;

  // Copies run on their own stream so chunk i+1 crosses PCIe while chunk i is on the tensor cores; events order
  // them: ready[b] (chunk in buffer b has landed) before its GEMM, freed[b] (that GEMM has finished reading
  // buffer b) before the copy two chunks later overwrites it. The LAST chunk goes by row panels: its B part
  // first, then A's rows panel by panel, each panel's GEMM as soon as it lands, and that panel's C rows (now
  // final) back to the host on a third stream while the next panel's rows still cross the link (the two copy
  // directions run concurrently), so only one panel's GEMM and copy back remain after the last upload. Streams
  // and events are released at the end of this call; CUDA keeps them alive until the enqueued work that uses
  // them has completed (a wait captures the event's most recent record, so one event serves every panel).
  cudaStream_t cs = nullptr, ds = nullptr;
  cudaEvent_t start = nullptr, ready[2] = {nullptr, nullptr}, freed[2] = {nullptr, nullptr}, panel = nullptr;
  int rc = BSK_OK;
  cudaError_t e = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ds, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&start, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&panel, cudaEventDisableTiming);
  for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
    e = cudaEventCreateWithFlags(&ready[b], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&freed[b], cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaEventRecord(start, s);  // earlier work on `stream` (e.g. a previous user of the
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, start, 0);  // workspace or of C_host) comes first
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ds, start, 0);
  if (e != cudaSuccess) rc = cuda_fail(e, "gemm_host: stream/event setup");
  const int rows_per_panel = host_panel_rows(M);
  for (int i = 0; i < nchunks && rc == BSK_OK; ++i) {
    const int b = i & 1;
    const int k0 = i * p.kc;
    const int kw = K - k0 < p.kc ? K - k0 : p.kc;
    const bool last = i == nchunks - 1;
    if (i >= 2) e = cudaStreamWaitEvent(cs, freed[b], 0);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(bbuf[b], (size_t)p.kc * 2, static_cast<const __half*>(B_host) + k0, (size_t)ldb * 2,
                            (size_t)kw * 2, N, cudaMemcpyHostToDevice, cs);
    if (!last) {
      if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(abuf[b], (size_t)p.kc * 2, static_cast<const __half*>(A_host) + k0, (size_t)lda * 2,
                              (size_t)kw * 2, M, cudaMemcpyHostToDevice, cs);
      if (e == cudaSuccess) e = cudaEventRecord(ready[b], cs);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ready[b], 0);
      if (e != cudaSuccess) {
        rc = cuda_fail(e, "gemm_host: chunk copy");
        break;
      }
      rc = gemm_f16_launch(abuf[b], p.kc, bbuf[b], p.kc, Cd, p.ldc_dev, M, N, kw, 0, kw, i > 0 ? 1 : 0, stream);
      if (rc == BSK_OK && (e = cudaEventRecord(freed[b], s)) != cudaSuccess) rc = cuda_fail(e, "gemm_host: event");
      continue;
    }
    for (int m0 = 0; m0 < M && rc == BSK_OK; m0 += rows_per_panel) {
      const int mr = M - m0 < rows_per_panel ? M - m0 : rows_per_panel;
      __half* ap = abuf[b] + (int64_t)m0 * p.kc;
      float* cp = Cd + (int64_t)m0 * p.ldc_dev;
      if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(ap, (size_t)p.kc * 2, static_cast<const __half*>(A_host) + (int64_t)m0 * lda + k0,
                              (size_t)lda * 2, (size_t)kw * 2, mr, cudaMemcpyHostToDevice, cs);
      if (e == cudaSuccess) e = cudaEventRecord(ready[b], cs);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ready[b], 0);
      if (e != cudaSuccess) {
        rc = cuda_fail(e, "gemm_host: panel copy");
        break;
      }
      rc = gemm_f16_launch(ap, p.kc, bbuf[b], p.kc, cp, p.ldc_dev, mr, N, kw, 0, kw, i > 0 ? 1 : 0, stream);
      if (rc != BSK_OK) break;
      e = cudaEventRecord(panel, s);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(ds, panel, 0);
      if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(C_host + (int64_t)m0 * ldc, (size_t)ldc * 4, cp, (size_t)p.ldc_dev * 4,
                              (size_t)N * 4, mr, cudaMemcpyDeviceToHost, ds);
      if (e != cudaSuccess) rc = cuda_fail(e, "gemm_host: result copy");
    }
  }
  if (rc == BSK_OK && nchunks == 0) {
    e = cudaMemset2DAsync(Cd, p.ldc_dev * 4, 0, (size_t)N * 4, M, s);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(C_host, (size_t)ldc * 4, Cd, (size_t)p.ldc_dev * 4, (size_t)N * 4, M,
                            cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) rc = cuda_fail(e, "gemm_host: zero fill");
  }
  // `stream` must not run ahead of copies already queued on cs and ds (also when a step failed part-way).
  if (cs && start) {
    if (cudaEventRecord(start, cs) == cudaSuccess) cudaStreamWaitEvent(s, start, 0);
  }
  if (ds && panel) {
    if (cudaEventRecord(panel, ds) == cudaSuccess) cudaStreamWaitEvent(s, panel, 0);
  }
  for (int b = 0; b < 2; ++b) {
    if (ready[b]) cudaEventDestroy(ready[b]);
    if (freed[b]) cudaEventDestroy(freed[b]);
  }
  if (start) cudaEventDestroy(start);
  if (panel) cudaEventDestroy(panel);
  if (cs) cudaStreamDestroy(cs);
  if (ds) cudaStreamDestroy(ds);
  return rc;
}

int bsk_gemm_e4m3_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, const float* scale_a,
                       const float* scale_b, void* D, int64_t ldd, int M, int N, int K, void* stream) {
  using namespace bsk;
  if (M < 0 || N < 0 || K < 0) return set_error(BSK_ERR_INVALID_ARG, "gemm_e4m3: negative extent");
  if (lda < K || ldb < K || ldd < N)
    return set_error(BSK_ERR_INVALID_ARG, "gemm_e4m3: leading dimensions smaller than the extents");
  if (lda % 16 || ldb % 16) return set_error(BSK_ERR_INVALID_ARG, "gemm_e4m3: lda and ldb must be multiples of 16");
  if (!A || !B || !D || !scale_a || !scale_b) return set_error(BSK_ERR_INVALID_ARG, "gemm_e4m3: null pointer");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (M == 0 || N == 0) return BSK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    cudaError_t e = cudaMemset2DAsync(D, ldd * 2, 0, (size_t)N * 2, M, s);
    return e == cudaSuccess ? BSK_OK : cuda_fail(e, "gemm_e4m3: zero fill");
  }
  int kind, group;
  launch_config(BSK_OP_GEMM_E4M3_BF16, M, N, K, true, &kind, &group);
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, K, M, lda, 128, kind ? 128 : kGemmBM, "A")) return rc;
  if (int rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, B, K, N, ldb, 128, kind ? 128 : kGemmBN, "B")) return rc;
  GemmArgs a{};
  const int tm = kind ? kPairBM : kGemmBM, tn = kind == 2 ? 512 : kGemmBN;
  a.M = M;
  a.N = N;
  a.num_m_tiles = (M + tm - 1) / tm;
  a.num_n_tiles = (N + tn - 1) / tn;
  a.num_k_blocks = (K + 127) / 128;
  a.group_m = resolve_group(group, a.num_m_tiles, kind, 0);
  a.k_splits = 1;
  a.kb_per_split = a.num_k_blocks;
  a.out = D;
  a.ldo = ldd;
  a.vec_ok = aligned16(D) && (ldd % 8 == 0);
  a.scale_a = scale_a;
  a.scale_b = scale_b;
  a.err = st->err_word;
  a.timeout_ns = t_timeout_ns;
  const int tiles = a.num_m_tiles * a.num_n_tiles;
  const int clusters = tiles < st->pair_clusters ? tiles : st->pair_clusters;
  if (kind == 2) {
    gemm_pair_sm100_kernel<1, Epi::BF16Scaled, 2><<<2 * clusters, kPairThreads, kPairWideSmemBytes, s>>>(ta, tb, a);
  } else if (kind == 1) {
    gemm_pair_sm100_kernel<1, Epi::BF16Scaled, 1><<<2 * clusters, kPairThreads, kPairSmemBytes, s>>>(ta, tb, a);
  } else {
    const int grid = tiles < st->sm_count ? tiles : st->sm_count;
    gemm_sm100_kernel<1, Mainloop::Dense, Epi::BF16Scaled><<<grid, kGemmThreads, kGemmSmemBytes, s>>>(ta, tb, a);
  }
  return launch_status("gemm_e4m3 launch");
}

}  // extern "C"

namespace {

struct SplitPlan {
  int kind;          // 1: pair 256x256, 2: pair 256x512
  int splits;        // K splits per tile (1 = no split)
  int kb_per_split;  // 64-element K stages per split
  int64_t ld_ws;     // row stride of a partial slab (elements)
};

// K splits for an fp16 GEMM of the given shape: enough (tile, split) units to occupy every co-resident CTA
// pair, each split at least 4 K stages, at most 32 splits.
SplitPlan plan_splitk(const DeviceState& st, int M, int N, int kr, int splits_req) {
  SplitPlan p{};
  const int nkb = (kr + 63) / 64;
  const int tiles = ((M + 255) / 256) * ((N + 255) / 256);
  int s = splits_req;
  if (s <= 0) {
    s = tiles >= st.pair_clusters ? 1 : st.pair_clusters / tiles;
    const int cap = nkb / 4 > 1 ? nkb / 4 : 1;
    s = s < cap ? s : cap;
    s = s < 32 ? s : 32;
  }
  s = s < 1 ? 1 : (s > nkb ? nkb : s);
  p.kb_per_split = (nkb + s - 1) / s;
  p.splits = (nkb + p.kb_per_split - 1) / p.kb_per_split;  // every split non-empty
  p.kind = (N >= 512 && p.kb_per_split * 64 >= 8192) ? 2 : 1;
  p.ld_ws = (static_cast<int64_t>(N) + 3) / 4 * 4;
  return p;
}

// One CTA-pair launch over (tile, split) units writing fp32 partial slabs (or C when splits == 1).
int launch_pair_f16(const DeviceState& st, const SplitPlan& p, const __half* Ah, int64_t lda, const __half* Bh,
                    int64_t ldb, int M, int N, int kr, float* out, int64_t ldo, int64_t split_stride,
                    cudaStream_t s) {
  using namespace bsk;
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Ah, kr, M, lda * 2, 64, 128, "A")) return rc;
  if (int rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Bh, kr, N, ldb * 2, 64, 128, "B")) return rc;
  GemmArgs a{};
  const int tn = p.kind == 2 ? 512 : 256;
  a.M = M;
  a.N = N;
  a.num_m_tiles = (M + kPairBM - 1) / kPairBM;
  a.num_n_tiles = (N + tn - 1) / tn;
  a.num_k_blocks = (kr + 63) / 64;
  a.group_m = pick_group_m(a.num_m_tiles, p.kind, p.kb_per_split * 64);
  a.k_splits = p.splits;
  a.kb_per_split = p.kb_per_split;
  a.split_stride = split_stride;
  a.out = out;
  a.ldo = ldo;
  a.vec_ok = aligned16(out) && (ldo % 4 == 0);
  a.err = st.err_word;
  a.timeout_ns = t_timeout_ns;
  const int units = a.num_m_tiles * a.num_n_tiles * a.k_splits;
  const int clusters = units < st.pair_clusters ? units : st.pair_clusters;
  if (p.kind == 2)
    gemm_pair_sm100_kernel<2, Epi::F32, 2><<<2 * clusters, kPairThreads, kPairWideSmemBytes, s>>>(ta, tb, a);
  else
    gemm_pair_sm100_kernel<2, Epi::F32, 1><<<2 * clusters, kPairThreads, kPairSmemBytes, s>>>(ta, tb, a);
  return launch_status("gemm split-K launch");
}

int splitk_reduce(const DeviceState& st, const float* ws, const SplitPlan& p, float* C, int64_t ldc, int M, int N,
                  cudaStream_t s) {
  const int64_t groups = static_cast<int64_t>(M) * ((N + 3) / 4);
  int64_t blocks = (groups + 255) / 256;
  const int64_t cap = static_cast<int64_t>(st.sm_count) * 8;
  blocks = blocks < cap ? blocks : cap;
  bsk::splitk_reduce_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(
      ws, p.splits, static_cast<int64_t>(M) * p.ld_ws, p.ld_ws, C, ldc, M, N, aligned16(C) && (ldc % 4 == 0));
  return launch_status("split-K reduce launch");
}

}  // namespace

extern "C" {

int64_t bsk_gemm_splitk_workspace_bytes(int M, int N, int K, int splits) {
  if (M < 0 || N < 0 || K < 0) return set_error(BSK_ERR_INVALID_ARG, "splitk workspace: negative extent");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (M == 0 || N == 0 || K == 0) return 0;
  const SplitPlan p = plan_splitk(*st, M, N, K, splits);
  return p.splits <= 1 ? 0 : static_cast<int64_t>(p.splits) * M * p.ld_ws * static_cast<int64_t>(sizeof(float));
}

int bsk_gemm_f16f32_splitk(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M,
                           int N, int K, int splits, void* workspace, int64_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || K < 0) return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk: negative extent");
  if (lda < K || ldb < K || ldc < N)
    return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk: leading dimensions smaller than the extents");
  if (lda % 8 || ldb % 8) return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk: lda and ldb must be multiples of 8");
  if (!A || !B || !C) return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk: null pointer");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (M == 0 || N == 0) return BSK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    cudaError_t e = cudaMemset2DAsync(C, ldc * sizeof(float), 0, (size_t)N * sizeof(float), M, s);
    return e == cudaSuccess ? BSK_OK : cuda_fail(e, "gemm_splitk: zero fill");
  }
  const SplitPlan p = plan_splitk(*st, M, N, K, splits);
  const __half* Ah = static_cast<const __half*>(A);
  const __half* Bh = static_cast<const __half*>(B);
  if (p.splits <= 1) return launch_pair_f16(*st, p, Ah, lda, Bh, ldb, M, N, K, C, ldc, 0, s);
  const int64_t need = static_cast<int64_t>(p.splits) * M * p.ld_ws * static_cast<int64_t>(sizeof(float));
  if (!workspace || workspace_bytes < need)
    return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk: workspace of %lld bytes needed (%d splits), %lld given",
                     (long long)need, p.splits, (long long)workspace_bytes);
  if (!aligned16(workspace)) return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk: workspace must be 16-byte aligned");
  float* ws = static_cast<float*>(workspace);
  if (int rc = launch_pair_f16(*st, p, Ah, lda, Bh, ldb, M, N, K, ws, p.ld_ws, static_cast<int64_t>(M) * p.ld_ws, s))
    return rc;
  return splitk_reduce(*st, ws, p, C, ldc, M, N, s);
}

}  // extern "C"

namespace {

// Scratch of bsk_gemm_f16f32_splitk_static: the split-K partial slabs, for callers that cannot allocate device
// memory. A fixed 32 MiB that every GPU which loads this library holds until the process exits. All calls
// share it and it keeps the last call's contents; nothing in it has to start at zero (each call overwrites
// every partial element it later reads).
constexpr int64_t kStaticScratchBytes = 32ll << 20;
static __device__ __align__(256) unsigned char g_bsk_static_scratch[kStaticScratchBytes];

// Device address of g_bsk_static_scratch, looked up once per device (with that device current) on the first
// call of bsk_gemm_f16f32_splitk_static there: in host code the array's name is only a host-side stand-in.
struct StaticScratch {
  std::once_flag once;
  cudaError_t status = cudaSuccess;
  void* ptr = nullptr;
};
StaticScratch g_static_scratch[kMaxDevices];

}  // namespace

extern "C" {

int bsk_gemm_f16f32_splitk_static(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc,
                                  int M, int N, int K, int splits, void* stream) {
  if (M < 0 || N < 0 || K < 0) return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk_static: negative extent");
  if (lda < K || ldb < K || ldc < N)
    return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk_static: leading dimensions smaller than the extents");
  if (lda % 8 || ldb % 8)
    return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk_static: lda and ldb must be multiples of 8");
  if (!A || !B || !C) return set_error(BSK_ERR_INVALID_ARG, "gemm_splitk_static: null pointer");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_splitk_static: current device");
  StaticScratch& sc = g_static_scratch[dev];
  std::call_once(sc.once, [&] { sc.status = cudaGetSymbolAddress(&sc.ptr, g_bsk_static_scratch); });
  if (sc.status != cudaSuccess) return cuda_fail(sc.status, "gemm_splitk_static: cudaGetSymbolAddress(scratch)");
  if (M == 0 || N == 0) return BSK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    e = cudaMemset2DAsync(C, ldc * sizeof(float), 0, (size_t)N * sizeof(float), M, s);
    return e == cudaSuccess ? BSK_OK : cuda_fail(e, "gemm_splitk_static: zero fill");
  }
  const SplitPlan p = plan_splitk(*st, M, N, K, splits);
  const __half* Ah = static_cast<const __half*>(A);
  const __half* Bh = static_cast<const __half*>(B);
  if (p.splits <= 1) return launch_pair_f16(*st, p, Ah, lda, Bh, ldb, M, N, K, C, ldc, 0, s);
  const int64_t need = static_cast<int64_t>(p.splits) * M * p.ld_ws * static_cast<int64_t>(sizeof(float));
  if (need > kStaticScratchBytes)
    return set_error(BSK_ERR_INVALID_ARG,
                     "gemm_splitk_static: %d splits of a %dx%d fp32 output need %lld bytes of scratch; the static "
                     "scratch holds %lld (use fewer splits, or bsk_gemm_f16f32_splitk with a workspace)",
                     p.splits, M, N, (long long)need, (long long)kStaticScratchBytes);
  float* ws = static_cast<float*>(sc.ptr);
  if (int rc = launch_pair_f16(*st, p, Ah, lda, Bh, ldb, M, N, K, ws, p.ld_ws, static_cast<int64_t>(M) * p.ld_ws, s))
    return rc;
  return splitk_reduce(*st, ws, p, C, ldc, M, N, s);
}

int bsk_peer_buffer_alloc(int64_t bytes, void** dev_ptr, void* ipc_handle) {
  if (bytes <= 0 || !dev_ptr || !ipc_handle) return set_error(BSK_ERR_INVALID_ARG, "peer_buffer_alloc: bad arguments");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "peer_buffer_alloc: cudaMalloc");
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "peer_buffer_alloc: cudaIpcGetMemHandle");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
  memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return BSK_OK;
}

int bsk_peer_buffer_open(const void* ipc_handle, void** dev_ptr) {
  if (!ipc_handle || !dev_ptr) return set_error(BSK_ERR_INVALID_ARG, "peer_buffer_open: null argument");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "peer_buffer_open: cudaIpcOpenMemHandle");
  *dev_ptr = p;
  return BSK_OK;
}

int bsk_peer_buffer_close(void* dev_ptr) {
  if (!dev_ptr) return BSK_OK;
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? BSK_OK : cuda_fail(e, "peer_buffer_close");
}

int bsk_peer_buffer_free(void* dev_ptr) {
  if (!dev_ptr) return BSK_OK;
  cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? BSK_OK : cuda_fail(e, "peer_buffer_free");
}

int bsk_gemm_f16f32_splitk_scatter(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K,
                                   int k_begin, int k_end, int world, int rank, void* const* slot_bufs,
                                   int64_t ld_slot, void* stream) {
  using namespace bsk;
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return set_error(BSK_ERR_INVALID_ARG, "splitk_scatter: world %d / rank %d outside [1, %d]", world, rank, kMaxPeers);
  if (M <= 0 || N <= 0 || K <= 0 || M % world)
    return set_error(BSK_ERR_INVALID_ARG, "splitk_scatter: M (%d) must be a positive multiple of world (%d)", M, world);
  if (k_begin < 0 || k_end > K || k_begin >= k_end || k_begin % 8)
    return set_error(BSK_ERR_INVALID_ARG, "splitk_scatter: bad K range [%d, %d)", k_begin, k_end);
  if (lda < K || ldb < K || lda % 8 || ldb % 8)
    return set_error(BSK_ERR_INVALID_ARG, "splitk_scatter: lda/ldb must cover K and be multiples of 8");
  if (ld_slot < N || ld_slot % 4) return set_error(BSK_ERR_INVALID_ARG, "splitk_scatter: ld_slot must be >= N, %4");
  if (!A || !B || !slot_bufs) return set_error(BSK_ERR_INVALID_ARG, "splitk_scatter: null pointer");
  for (int r = 0; r < world; ++r)
    if (!slot_bufs[r] || !aligned16(slot_bufs[r]))
      return set_error(BSK_ERR_INVALID_ARG, "splitk_scatter: slot buffer of rank %d missing or misaligned", r);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  const int kr = k_end - k_begin;
  const __half* Ah = static_cast<const __half*>(A) + k_begin;
  const __half* Bh = static_cast<const __half*>(B) + k_begin;
  const int kind = gemm_tile_kind(M, N, kr) == 2 ? 2 : 1;
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Ah, kr, M, lda * 2, 64, 128, "A")) return rc;
  if (int rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Bh, kr, N, ldb * 2, 64, 128, "B")) return rc;
  GemmArgs a{};
  const int tn = kind == 2 ? 512 : 256;
  a.M = M;
  a.N = N;
  a.num_m_tiles = (M + kPairBM - 1) / kPairBM;
  a.num_n_tiles = (N + tn - 1) / tn;
  a.num_k_blocks = (kr + 63) / 64;
  a.group_m = pick_group_m(a.num_m_tiles, kind, kr);
  a.k_splits = 1;
  a.kb_per_split = a.num_k_blocks;
  a.ldo = ld_slot;
  a.vec_ok = 1;
  for (int r = 0; r < world; ++r) a.peer_out[r] = static_cast<float*>(slot_bufs[r]);
  a.rows_per_rank = M / world;
  a.my_rank = rank;
  a.err = st->err_word;
  a.timeout_ns = t_timeout_ns;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int tiles = a.num_m_tiles * a.num_n_tiles;
  const int clusters = tiles < st->pair_clusters ? tiles : st->pair_clusters;
  if (kind == 2)
    gemm_pair_sm100_kernel<2, Epi::F32PeerRows, 2><<<2 * clusters, kPairThreads, kPairWideSmemBytes, s>>>(ta, tb, a);
  else
    gemm_pair_sm100_kernel<2, Epi::F32PeerRows, 1><<<2 * clusters, kPairThreads, kPairSmemBytes, s>>>(ta, tb, a);
  return launch_status("splitk_scatter launch");
}

int bsk_splitk_slots_reduce(const float* slots, int world, int rows, int N, int64_t ld_slot, float* C, int64_t ldc,
                            void* stream) {
  if (world < 1 || rows < 0 || N < 0 || ld_slot < N || ld_slot % 4 || ldc < N)
    return set_error(BSK_ERR_INVALID_ARG, "slots_reduce: bad extents");
  if (!slots || !C || !aligned16(slots)) return set_error(BSK_ERR_INVALID_ARG, "slots_reduce: null or misaligned");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (rows == 0 || N == 0) return BSK_OK;
  SplitPlan p{};
  p.splits = world;
  p.ld_ws = ld_slot;
  return splitk_reduce(*st, slots, p, C, ldc, rows, N, static_cast<cudaStream_t>(stream));
}

int bsk_bsr_validate_host(const int32_t* row_ptr, const int32_t* col_idx, int Mb, int Kb, int nnzb) {
  if (Mb < 0 || Kb < 0 || nnzb < 0) return set_error(BSK_ERR_INVALID_ARG, "bsr: negative extent");
  if (!row_ptr) return set_error(BSK_ERR_INVALID_ARG, "bsr: null row_ptr");
  if (nnzb > 0 && !col_idx) return set_error(BSK_ERR_INVALID_ARG, "bsr: null col_idx");
  if (row_ptr[0] != 0) return set_error(BSK_ERR_INVALID_ARG, "bsr: row_ptr[0] = %d, expected 0", row_ptr[0]);
  for (int r = 0; r < Mb; ++r)
    if (row_ptr[r + 1] < row_ptr[r])
      return set_error(BSK_ERR_INVALID_ARG, "bsr: row_ptr decreases at block-row %d", r);
  if (row_ptr[Mb] != nnzb)
    return set_error(BSK_ERR_INVALID_ARG, "bsr: row_ptr[Mb] = %d but nnzb = %d", row_ptr[Mb], nnzb);
  for (int j = 0; j < nnzb; ++j)
    if (col_idx[j] < 0 || col_idx[j] >= Kb)
      return set_error(BSK_ERR_INVALID_ARG, "bsr: col_idx[%d] = %d outside [0, %d)", j, col_idx[j], Kb);
  return BSK_OK;
}

int bsk_spmm_bsr_f16f32(const int32_t* row_ptr, const int32_t* col_idx, const void* vals, int bs_r, int bs_c,
                        int Mb, int nnzb, const void* B, int64_t ldb, float* C, int64_t ldc, int M, int N, int K,
                        int row_begin, int row_end, void* stream) {
  using namespace bsk;
  if (bs_r != 128 || bs_c != 128)
    return set_error(BSK_ERR_UNSUPPORTED, "spmm_bsr: block shape %dx%d unsupported (the sm_100 kernel needs 128x128)",
                     bs_r, bs_c);
  if (M < 0 || N < 0 || K < 0 || Mb < 0 || nnzb < 0) return set_error(BSK_ERR_INVALID_ARG, "spmm_bsr: negative extent");
  if (M != Mb * bs_r) return set_error(BSK_ERR_INVALID_ARG, "spmm_bsr: M=%d != Mb*bs_r=%d", M, Mb * bs_r);
  if (K % bs_c) return set_error(BSK_ERR_INVALID_ARG, "spmm_bsr: K=%d not a multiple of the block width", K);
  if (row_begin < 0 || row_end > Mb || row_begin > row_end)
    return set_error(BSK_ERR_INVALID_ARG, "spmm_bsr: bad block-row range [%d, %d) for Mb=%d", row_begin, row_end, Mb);
  if (ldb < N || ldc < N) return set_error(BSK_ERR_INVALID_ARG, "spmm_bsr: leading dimensions smaller than N");
  if (ldb % 8) return set_error(BSK_ERR_INVALID_ARG, "spmm_bsr: ldb must be a multiple of 8");
  if (!row_ptr || !C || (N > 0 && K > 0 && !B) || (nnzb > 0 && (!col_idx || !vals)))
    return set_error(BSK_ERR_INVALID_ARG, "spmm_bsr: null pointer");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (row_end == row_begin || N == 0) return BSK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0 || nnzb == 0) {
    float* c0 = C + static_cast<int64_t>(row_begin) * bs_r * ldc;
    cudaError_t e = cudaMemset2DAsync(c0, ldc * sizeof(float), 0, (size_t)N * sizeof(float),
                                      (size_t)(row_end - row_begin) * bs_r, s);
    return e == cudaSuccess ? BSK_OK : cuda_fail(e, "spmm_bsr: zero fill");
  }
  // Tile kind: 0 = one CTA per 128 x 256 output tile; 1 = a CTA pair per 128 x 512 tile computed transposed
  // (the sparse block is the shared operand). BSK_SPMM_TILE=single|pair overrides, then a registered shape
  // configuration, then the built-in choice: the pair kernel from 512 output columns up.
  int kind = -1, group = 0;
  find_config(BSK_OP_SPMM_BSR, M, N, K, &kind, &group);
  if (const char* v = getenv("BSK_SPMM_TILE")) {
    if (strcmp(v, "single") == 0) kind = 0;
    if (strcmp(v, "pair") == 0) kind = 1;
  }
  if (kind < 0 || kind > 1) kind = N >= kBsrPairTileN ? 1 : 0;
  if (st->bsr_pair_clusters <= 0) kind = 0;
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, vals, 128, (uint64_t)nnzb * 128, 256, 64,
                        kind ? 64 : 128, "A values"))
    return rc;
  if (int rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, N, K, ldb * 2, 64, 64, "B")) return rc;
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.num_m_tiles = row_end - row_begin;
  a.num_n_tiles = (N + (kind ? kBsrPairTileN : kGemmBN) - 1) / (kind ? kBsrPairTileN : kGemmBN);
  a.num_k_blocks = 0;
  a.group_m = resolve_group(group, a.num_m_tiles, 0, 0);
  a.k_splits = 1;
  a.kb_per_split = a.num_k_blocks;
  a.out = C;
  a.ldo = ldc;
  a.vec_ok = aligned16(C) && (ldc % 4 == 0);
  a.row_ptr = row_ptr;
  a.col_idx = col_idx;
  a.row_begin = row_begin;
  a.nnzb = nnzb;
  a.kb_count = K / bs_c;
  a.err = st->err_word;
  a.timeout_ns = t_timeout_ns;
  const int tiles = a.num_m_tiles * a.num_n_tiles;
  if (kind == 1) {
    const int clusters = tiles < st->bsr_pair_clusters ? tiles : st->bsr_pair_clusters;
    spmm_bsr_pair_sm100_kernel<<<2 * clusters, kPairThreads, kBsrPairSmemBytes, s>>>(ta, tb, a);
    return launch_status("spmm_bsr pair launch");
  }
  const int grid = tiles < st->sm_count ? tiles : st->sm_count;
  gemm_sm100_kernel<2, Mainloop::Bsr, Epi::F32><<<grid, kGemmThreads, kGemmSmemBytes, s>>>(ta, tb, a);
  return launch_status("spmm_bsr launch");
}

int bsk_spmm_bsr_bsr_f16f32(const int32_t* a_row_ptr, const int32_t* a_col_idx, const void* a_vals, int Mb,
                            int a_nnzb, const int32_t* b_row_ptr, const int32_t* b_col_idx, const void* b_vals,
                            int b_nnzb, float* C, int64_t ldc, int M, int N, int K, int row_begin, int row_end,
                            void* stream) {
  using namespace bsk;
  const char* what = "spmm_bsr_bsr";
  if (M < 0 || N < 0 || K < 0 || Mb < 0 || a_nnzb < 0 || b_nnzb < 0)
    return set_error(BSK_ERR_INVALID_ARG, "%s: negative extent", what);
  if (M != Mb * 128 || K % 128 || N % 128)
    return set_error(BSK_ERR_INVALID_ARG, "%s: M=%d, K=%d, N=%d must be multiples of the 128 block size (Mb=%d)", what,
                     M, K, N, Mb);
  if ((int64_t)b_nnzb * 128 + 128 >= ((int64_t)1 << 31))
    return set_error(BSK_ERR_UNSUPPORTED, "%s: %d stored B blocks exceed the tensor-map row range", what, b_nnzb);
  if (row_begin < 0 || row_end > Mb || row_begin > row_end)
    return set_error(BSK_ERR_INVALID_ARG, "%s: bad block-row range [%d, %d) for Mb=%d", what, row_begin, row_end, Mb);
  if (ldc < N) return set_error(BSK_ERR_INVALID_ARG, "%s: ldc < N", what);
  if (!a_row_ptr || !C || (K > 0 && !b_row_ptr) || (a_nnzb > 0 && (!a_col_idx || !a_vals)) ||
      (b_nnzb > 0 && (!b_col_idx || !b_vals)))
    return set_error(BSK_ERR_INVALID_ARG, "%s: null pointer", what);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (row_end == row_begin || N == 0) return BSK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0 || a_nnzb == 0 || b_nnzb == 0) {
    float* c0 = C + static_cast<int64_t>(row_begin) * 128 * ldc;
    cudaError_t e = cudaMemset2DAsync(c0, ldc * sizeof(float), 0, (size_t)N * sizeof(float),
                                      (size_t)(row_end - row_begin) * 128, s);
    return e == cudaSuccess ? BSK_OK : cuda_fail(e, what);
  }
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a_vals, 128, (uint64_t)a_nnzb * 128, 256, 64, 128,
                        "A values"))
    return rc;
  // B's blocks stacked as rows: block p, K row r -> row p*128 + r; 64 x 64 boxes (one MN-major slab of a stage)
  if (int rc = make_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b_vals, 128, (uint64_t)b_nnzb * 128, 256, 64, 64,
                        "B values"))
    return rc;
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.num_m_tiles = row_end - row_begin;
  a.num_n_tiles = (N + kGemmBN - 1) / kGemmBN;
  {
    int kind_unused, group;
    launch_config(BSK_OP_SPMM_BSR_BSR, M, N, K, false, &kind_unused, &group);
    a.group_m = resolve_group(group, a.num_m_tiles, 0, 0);
  }
  a.k_splits = 1;
  a.out = C;
  a.ldo = ldc;
  a.vec_ok = aligned16(C) && (ldc % 4 == 0);
  a.row_ptr = a_row_ptr;
  a.col_idx = a_col_idx;
  a.row_begin = row_begin;
  a.nnzb = a_nnzb;
  a.kb_count = K / 128;
  a.b_row_ptr = b_row_ptr;
  a.b_col_idx = b_col_idx;
  a.b_nnzb = b_nnzb;
  // B's block map staged in shared memory when it fits (map entries and kb_count + 1 row pointers); the
  // environment variable BSK_BSRBSR_TABLE=0 keeps the binary searches in global memory.
  {
    const int nbc = N / 128;
    const char* v = getenv("BSK_BSRBSR_TABLE");
    const bool off = v && strcmp(v, "0") == 0;
    a.b_nbc = (!off && a.kb_count + 1 <= 256 && (int64_t)a.kb_count * nbc <= kBsrTableMax) ? nbc : 0;
  }
  a.err = st->err_word;
  a.timeout_ns = t_timeout_ns;
  const int tiles = a.num_m_tiles * a.num_n_tiles;
  const int grid = tiles < st->sm_count ? tiles : st->sm_count;
  gemm_sm100_kernel<2, Mainloop::BsrBsr, Epi::F32><<<grid, kGemmThreads, kGemmBsrBsrSmemBytes, s>>>(ta, tb, a);
  return launch_status("spmm_bsr_bsr launch");
}

void launch_bsr_spmm_async(const int* A_row_ptr, const int* A_col_idx, const void* A_vals, int A_M_blocks,
                           int A_K_blocks, int A_nnzb, const int* B_row_ptr, const int* B_col_idx, const void* B_vals,
                           int B_K_blocks, int B_N_blocks, int B_nnzb, float* C, int M, int N, int K, int ldc, int BM,
                           int BN, int BK, void* stream) {
  (void)B_row_ptr;
  (void)B_col_idx;
  (void)BM;
  (void)BN;
  (void)BK;
  if (A_M_blocks <= 0 || A_K_blocks <= 0 || M % A_M_blocks || K % A_K_blocks) {
    set_error(BSK_ERR_INVALID_ARG, "launch_bsr_spmm_async: M/K not divisible by the block counts");
    return;
  }
  if (B_nnzb != B_K_blocks * B_N_blocks) {  // a sparse B: its values are blocks, found by B's row_ptr / col_idx
    if (B_K_blocks != A_K_blocks || B_K_blocks <= 0 || B_N_blocks <= 0 || K / B_K_blocks != 128 ||
        N / B_N_blocks != 128) {
      set_error(BSK_ERR_UNSUPPORTED, "launch_bsr_spmm_async: a sparse B needs 128x128 blocks matching A's K blocking");
      return;
    }
    const int rc = bsk_spmm_bsr_bsr_f16f32(A_row_ptr, A_col_idx, A_vals, A_M_blocks, A_nnzb, B_row_ptr, B_col_idx,
                                           B_vals, B_nnzb, C, ldc, M, N, K, 0, A_M_blocks, stream);
    if (rc == BSK_OK) t_last_error.clear();
    return;
  }
  const int rc = bsk_spmm_bsr_f16f32(A_row_ptr, A_col_idx, A_vals, M / A_M_blocks, K / A_K_blocks, A_M_blocks,
                                     A_nnzb, B_vals, N, C, ldc, M, N, K, 0, A_M_blocks, stream);
  if (rc == BSK_OK) t_last_error.clear();
}

namespace {

// Shared launcher of the fp16 and bf16 entry points: same argument checks, element type picks the
// instantiation and the tensor-map data type.
int bsattn_launch(bool f16, const void* Q, const void* K, const void* V, void* O, float* lse, const int32_t* row_ptr,
                  const int32_t* col_idx, int B, int H, int S, int D, int blk, float scale, int causal_diag,
                  int bh_begin, int bh_end, void* stream) {
  using namespace bsk;
  if (D != 64 && D != 128) return set_error(BSK_ERR_UNSUPPORTED, "bsattn: head_dim %d unsupported (64 or 128)", D);
  if (blk != kAttnBlk) return set_error(BSK_ERR_UNSUPPORTED, "bsattn: block size %d unsupported (needs %d)", blk, kAttnBlk);
  if (B < 0 || H < 0 || S < 0) return set_error(BSK_ERR_INVALID_ARG, "bsattn: negative extent");
  if (S % blk) return set_error(BSK_ERR_INVALID_ARG, "bsattn: S=%d not a multiple of the block size %d", S, blk);
  if (bh_begin < 0 || bh_end > B * H || bh_begin > bh_end)
    return set_error(BSK_ERR_INVALID_ARG, "bsattn: bad (b,h) range [%d, %d)", bh_begin, bh_end);
  if (!(scale > 0.0f) || !(scale < 1e30f)) return set_error(BSK_ERR_INVALID_ARG, "bsattn: scale must be positive and finite");
  if (!Q || !K || !V || !O || !row_ptr || !col_idx) return set_error(BSK_ERR_INVALID_ARG, "bsattn: null pointer");
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O))
    return set_error(BSK_ERR_INVALID_ARG, "bsattn: Q/K/V/O must be 16-byte aligned");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (bh_end == bh_begin || S == 0) return BSK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t rows = (uint64_t)B * H * S;
  const CUtensorMapDataType dt = f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq, tk, tv;
  if (int rc = make_map(&tq, dt, 2, Q, D, rows, D * 2, 64, kAttnBlk, "Q")) return rc;
  if (int rc = make_map(&tk, dt, 2, K, D, rows, D * 2, 64, kAttnBlk, "K")) return rc;
  if (int rc = make_map(&tv, dt, 2, V, D, rows, D * 2, 64, kAttnBlk, "V")) return rc;
  AttnArgs a{};
  a.O = O;
  a.lse = lse;
  a.row_ptr = row_ptr;
  a.col_idx = col_idx;
  a.S = S;
  a.nqb = S / blk;
  a.bh_begin = bh_begin;
  a.num_items = (bh_end - bh_begin) * a.nqb;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal_diag = causal_diag;
  a.err = st->err_word;
  a.timeout_ns = t_timeout_ns;
  const int grid = a.num_items < st->sm_count ? a.num_items : st->sm_count;
  if (f16 && D == 128)
    bsattn_sm100_kernel<true, 128><<<grid, kAttnThreads, AttnShape<true, 128>::kSmemBytes, s>>>(tq, tk, tv, a);
  else if (f16)
    bsattn_sm100_kernel<true, 64><<<grid, kAttnThreads, AttnShape<true, 64>::kSmemBytes, s>>>(tq, tk, tv, a);
  else if (D == 128)
    bsattn_sm100_kernel<false, 128><<<grid, kAttnThreads, AttnShape<false, 128>::kSmemBytes, s>>>(tq, tk, tv, a);
  else
    bsattn_sm100_kernel<false, 64><<<grid, kAttnThreads, AttnShape<false, 64>::kSmemBytes, s>>>(tq, tk, tv, a);
  return launch_status("bsattn launch");
}

}  // namespace

int bsk_bsattn_fwd_bf16(const void* Q, const void* K, const void* V, void* O, const int32_t* row_ptr,
                        const int32_t* col_idx, int B, int H, int S, int D, int blk, float scale, int causal_diag,
                        int bh_begin, int bh_end, void* stream) {
  return bsattn_launch(false, Q, K, V, O, nullptr, row_ptr, col_idx, B, H, S, D, blk, scale, causal_diag, bh_begin,
                       bh_end, stream);
}

int bsk_bsattn_fwd_f16(const void* Q, const void* K, const void* V, void* O, const int32_t* row_ptr,
                       const int32_t* col_idx, int B, int H, int S, int D, int blk, float scale, int causal_diag,
                       int bh_begin, int bh_end, void* stream) {
  return bsattn_launch(true, Q, K, V, O, nullptr, row_ptr, col_idx, B, H, S, D, blk, scale, causal_diag, bh_begin,
                       bh_end, stream);
}

namespace {

// Workspace of the BSR converters: int32 flags / block-index map [Mb * Kb], int32 block_row [Mb * Kb], int32
// counts [Mb], then a 256-byte tail: ConvTail (element nonzero counter, bad-index flag, nnzb).
struct ConvTail {
  unsigned long long nnz_elems;
  int bad;
  int pad;
  long long nnzb;
};

struct ConvPlan {
  int Mb = 0, Kb = 0;
  int64_t flags_bytes = 0, counts_bytes = 0, total = 0;
};

int conv_plan(int M, int K, int bs, ConvPlan* p, const char* what) {
  if (M < 0 || K < 0) return set_error(BSK_ERR_INVALID_ARG, "%s: negative extent", what);
  if (bs <= 0) return set_error(BSK_ERR_INVALID_ARG, "%s: block size must be positive", what);
  if (M % bs || K % bs)
    return set_error(BSK_ERR_INVALID_ARG, "%s: shape %dx%d is not divisible by the block size %d", what, M, K, bs);
  p->Mb = M / bs;
  p->Kb = K / bs;
  if ((int64_t)p->Mb * p->Kb >= (int64_t)1 << 31)
    return set_error(BSK_ERR_UNSUPPORTED, "%s: %d x %d blocks exceed the int32 block map", what, p->Mb, p->Kb);
  p->flags_bytes = round256((int64_t)p->Mb * p->Kb * 4);
  p->counts_bytes = round256((int64_t)p->Mb * 4);
  p->total = 2 * p->flags_bytes + p->counts_bytes + 256;
  return BSK_OK;
}

struct ConvWs {
  int* flags;
  int* block_row;
  int* counts;
  ConvTail* tail;
};

ConvWs conv_ws(const ConvPlan& p, void* workspace) {
  char* ws = static_cast<char*>(workspace);
  return {reinterpret_cast<int*>(ws), reinterpret_cast<int*>(ws + p.flags_bytes),
          reinterpret_cast<int*>(ws + 2 * p.flags_bytes),
          reinterpret_cast<ConvTail*>(ws + 2 * p.flags_bytes + p.counts_bytes)};
}

int conv_common_checks(int elem_bytes, int index_bytes, const ConvPlan& p, const void* workspace,
                       int64_t workspace_bytes, const char* what) {
  if (elem_bytes != 2 && elem_bytes != 4)
    return set_error(BSK_ERR_UNSUPPORTED, "%s: element size %d unsupported (2 or 4 bytes)", what, elem_bytes);
  if (index_bytes != 4 && index_bytes != 8)
    return set_error(BSK_ERR_INVALID_ARG, "%s: index size must be 4 or 8 bytes", what);
  if (!workspace || workspace_bytes < p.total)
    return set_error(BSK_ERR_INVALID_ARG, "%s: workspace of %lld bytes needed, %lld given", what, (long long)p.total,
                     (long long)workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return set_error(BSK_ERR_INVALID_ARG, "%s: workspace must be 256-byte aligned", what);
  return BSK_OK;
}

int conv_grid(const DeviceState* st) { return st->sm_count * 8; }

int conv_clear(const ConvPlan& p, void* ws, cudaStream_t s, const char* what) {
  cudaError_t e = cudaMemsetAsync(ws, 0, p.total, s);  // flags, block_row, counts and the tail in one fill
  return e == cudaSuccess ? BSK_OK : cuda_fail(e, what);
}

int conv_compact(const ConvPlan& p, const ConvWs& w, const void* row_ptr, void* col_idx, int index_bytes,
                 int64_t cap, const DeviceState* st, cudaStream_t s) {
  using namespace bsk;
  if (p.Mb == 0) return BSK_OK;
  const int g = p.Mb < conv_grid(st) ? p.Mb : conv_grid(st);
  if (index_bytes == 4)
    bsr_compact_kernel<int32_t><<<g, kConvThreads, 0, s>>>(w.flags, p.Mb, p.Kb, static_cast<const int32_t*>(row_ptr),
                                                           static_cast<int32_t*>(col_idx), w.block_row, cap);
  else
    bsr_compact_kernel<int64_t><<<g, kConvThreads, 0, s>>>(w.flags, p.Mb, p.Kb, static_cast<const int64_t*>(row_ptr),
                                                           static_cast<int64_t*>(col_idx), w.block_row, cap);
  return launch_status("bsr compact");
}

// Single-call converters on a small block grid: the index pass (counts, row_ptr, ranks) in one CTA.
bool conv_small(const ConvPlan& p) {
  return p.Mb > 0 && p.Mb <= bsk::kIndexSmallMaxRows && (int64_t)p.Mb * p.Kb <= bsk::kIndexSmallMaxFlags;
}

int conv_index_small(const ConvPlan& p, const ConvWs& w, void* row_ptr, void* col_idx, int index_bytes, int64_t cap,
                     cudaStream_t s) {
  using namespace bsk;
  if (index_bytes == 4)
    bsr_index_small_kernel<int32_t><<<1, kIndexSmallThreads, 0, s>>>(w.flags, p.Mb, p.Kb, static_cast<int32_t*>(row_ptr),
                                                                     static_cast<int32_t*>(col_idx), w.block_row, cap,
                                                                     &w.tail->nnzb);
  else
    bsr_index_small_kernel<int64_t><<<1, kIndexSmallThreads, 0, s>>>(w.flags, p.Mb, p.Kb, static_cast<int64_t*>(row_ptr),
                                                                     static_cast<int64_t*>(col_idx), w.block_row, cap,
                                                                     &w.tail->nnzb);
  return launch_status("bsr index");
}

bool dense_vec_ok(const void* A, int64_t lda, int elem_bytes, int bs) {
  const int per = 16 / elem_bytes;
  return aligned16(A) && lda % per == 0 && bs % per == 0;
}

}  // namespace

namespace {

// Pattern pass (no host synchronisation): workspace cleared, flags (+ element count, bad flag), counts, row_ptr
// and nnzb in the workspace tail.
int dense_pattern_enqueue(const void* A, int64_t lda, int elem_bytes, int M, int K, int bs, void* row_ptr,
                          int index_bytes, const ConvPlan& p, void* workspace, const DeviceState* st, cudaStream_t s,
                          const char* what, bool index = true) {
  using namespace bsk;
  if (int rc = conv_clear(p, workspace, s, what)) return rc;
  const ConvWs w = conv_ws(p, workspace);
  if ((int64_t)M * K > 0) {
    const uint8_t* a = static_cast<const uint8_t*>(A);
    const int g = conv_grid(st);
    unsigned long long* counter = &w.tail->nnz_elems;
    if (dense_vec_ok(A, lda, elem_bytes, bs)) {
      if (elem_bytes == 2) dense_flags_vec_kernel<2><<<g, kConvThreads, 0, s>>>(a, lda, M, K, bs, p.Kb, w.flags, counter);
      else dense_flags_vec_kernel<4><<<g, kConvThreads, 0, s>>>(a, lda, M, K, bs, p.Kb, w.flags, counter);
    } else {
      if (elem_bytes == 2) dense_flags_scalar_kernel<2><<<g, kConvThreads, 0, s>>>(a, lda, M, K, bs, p.Kb, w.flags, counter);
      else dense_flags_scalar_kernel<4><<<g, kConvThreads, 0, s>>>(a, lda, M, K, bs, p.Kb, w.flags, counter);
    }
  }
  if (!index) return launch_status(what);
  if (p.Mb > 0) {
    const int g = p.Mb < conv_grid(st) ? p.Mb : conv_grid(st);
    bsr_row_counts_kernel<<<g, kConvThreads, 0, s>>>(w.flags, p.Mb, p.Kb, w.counts);
  }
  if (index_bytes == 4)
    bsr_row_ptr_kernel<int32_t><<<1, kConvThreads, 0, s>>>(w.counts, p.Mb, static_cast<int32_t*>(row_ptr), &w.tail->nnzb);
  else
    bsr_row_ptr_kernel<int64_t><<<1, kConvThreads, 0, s>>>(w.counts, p.Mb, static_cast<int64_t*>(row_ptr), &w.tail->nnzb);
  return launch_status(what);
}

int csr_pattern_enqueue(const void* crow, const void* col, int index_bytes_in, const void* vals, int elem_bytes,
                        int64_t nnz, int M, int K, int bs, void* row_ptr, int index_bytes, const ConvPlan& p,
                        void* workspace, const DeviceState* st, cudaStream_t s, const char* what, bool index = true) {
  using namespace bsk;
  if (int rc = conv_clear(p, workspace, s, what)) return rc;
  const ConvWs w = conv_ws(p, workspace);
  if (M > 0 && nnz > 0) {
    if (index_bytes_in == 4)
      launch_csr_flags<int32_t>(elem_bytes, crow, col, vals, nnz, M, K, bs, p.Kb, w.flags, &w.tail->nnz_elems,
                                &w.tail->bad, st->sm_count, s);
    else
      launch_csr_flags<int64_t>(elem_bytes, crow, col, vals, nnz, M, K, bs, p.Kb, w.flags, &w.tail->nnz_elems,
                                &w.tail->bad, st->sm_count, s);
  }
  if (!index) return launch_status(what);
  if (p.Mb > 0) {
    const int g = p.Mb < conv_grid(st) ? p.Mb : conv_grid(st);
    bsr_row_counts_kernel<<<g, kConvThreads, 0, s>>>(w.flags, p.Mb, p.Kb, w.counts);
  }
  if (index_bytes == 4)
    bsr_row_ptr_kernel<int32_t><<<1, kConvThreads, 0, s>>>(w.counts, p.Mb, static_cast<int32_t*>(row_ptr), &w.tail->nnzb);
  else
    bsr_row_ptr_kernel<int64_t><<<1, kConvThreads, 0, s>>>(w.counts, p.Mb, static_cast<int64_t*>(row_ptr), &w.tail->nnzb);
  return launch_status(what);
}

// Reads the workspace tail back (one copy, synchronising the stream).
int conv_read_tail(const ConvPlan& p, void* workspace, int index_bytes, int64_t* nnzb, int64_t* nnz_elems,
                   cudaStream_t s, const char* what) {
  const ConvWs w = conv_ws(p, workspace);
  ConvTail t{};
  cudaError_t e = cudaMemcpyAsync(&t, w.tail, sizeof(t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, what);
  if (t.bad) return set_error(BSK_ERR_INVALID_ARG, "%s: CSR column index outside [0, K)", what);
  if (index_bytes == 4 && t.nnzb > INT32_MAX)
    return set_error(BSK_ERR_UNSUPPORTED, "%s: %lld blocks overflow int32 indices", what, (long long)t.nnzb);
  if (nnzb) *nnzb = t.nnzb;
  if (nnz_elems) *nnz_elems = static_cast<int64_t>(t.nnz_elems);
  return BSK_OK;
}

// Fill pass: col_idx, block_row and the map, then the values of the first min(nnzb, cap) blocks.
int dense_fill_enqueue(const void* A, int64_t lda, int elem_bytes, int bs, const void* row_ptr, void* col_idx,
                       int index_bytes, void* values, int64_t cap, const ConvPlan& p, void* workspace,
                       const DeviceState* st, cudaStream_t s, const char* what, bool compact = true) {
  using namespace bsk;
  const ConvWs w = conv_ws(p, workspace);
  if (compact)
    if (int rc = conv_compact(p, w, row_ptr, col_idx, index_bytes, cap, st, s)) return rc;
  const uint8_t* a = static_cast<const uint8_t*>(A);
  uint8_t* v = static_cast<uint8_t*>(values);
  const bool vec = dense_vec_ok(A, lda, elem_bytes, bs) && aligned16(values);
  const int g = conv_grid(st);
  const int* br = w.block_row;
  const long long* nz = &w.tail->nnzb;
#define BSK_COPY(E, V, I) \
  dense_block_copy_kernel<E, V, I><<<g, kConvThreads, 0, s>>>(a, lda, bs, br, static_cast<const I*>(col_idx), nz, cap, v)
  if (index_bytes == 4) {
    if (elem_bytes == 2) { if (vec) BSK_COPY(2, true, int32_t); else BSK_COPY(2, false, int32_t); }
    else { if (vec) BSK_COPY(4, true, int32_t); else BSK_COPY(4, false, int32_t); }
  } else {
    if (elem_bytes == 2) { if (vec) BSK_COPY(2, true, int64_t); else BSK_COPY(2, false, int64_t); }
    else { if (vec) BSK_COPY(4, true, int64_t); else BSK_COPY(4, false, int64_t); }
  }
#undef BSK_COPY
  return launch_status(what);
}

int csr_fill_enqueue(const void* crow, const void* col, int index_bytes_in, const void* vals, int elem_bytes,
                     int64_t nnz, int M, int K, int bs, const void* row_ptr, void* col_idx, int index_bytes,
                     void* values, int64_t cap, const ConvPlan& p, void* workspace, const DeviceState* st,
                     cudaStream_t s, const char* what, bool compact = true) {
  using namespace bsk;
  const ConvWs w = conv_ws(p, workspace);
  if (compact)
    if (int rc = conv_compact(p, w, row_ptr, col_idx, index_bytes, cap, st, s)) return rc;
  const int g = conv_grid(st);
  zero_blocks_kernel<<<g, kConvThreads, 0, s>>>(static_cast<uint8_t*>(values), &w.tail->nnzb, cap,
                                                (int64_t)bs * bs * elem_bytes);
  if (M > 0 && nnz > 0) {
    if (index_bytes_in == 4)
      launch_csr_scatter<int32_t>(elem_bytes, crow, col, vals, nnz, M, K, bs, p.Kb, w.flags, cap, values, st->sm_count,
                                  s);
    else
      launch_csr_scatter<int64_t>(elem_bytes, crow, col, vals, nnz, M, K, bs, p.Kb, w.flags, cap, values, st->sm_count,
                                  s);
  }
  return launch_status(what);
}

int csr_checks(const void* crow, const void* col, int index_bytes_in, const void* vals, int64_t nnz, int M,
               const char* what) {
  if (index_bytes_in != 4 && index_bytes_in != 8)
    return set_error(BSK_ERR_INVALID_ARG, "%s: CSR index size must be 4 or 8 bytes", what);
  if (nnz < 0) return set_error(BSK_ERR_INVALID_ARG, "%s: negative nnz", what);
  if (!crow && M > 0) return set_error(BSK_ERR_INVALID_ARG, "%s: null crow_indices", what);
  if (nnz > 0 && (!col || !vals)) return set_error(BSK_ERR_INVALID_ARG, "%s: null col_indices/values", what);
  return BSK_OK;
}

int dense_checks(const void* A, int64_t lda, int elem_bytes, int index_bytes, int M, int K, int bs, ConvPlan* p,
                 const void* workspace, int64_t workspace_bytes, const char* what) {
  if (int rc = conv_plan(M, K, bs, p, what)) return rc;
  if (int rc = conv_common_checks(elem_bytes, index_bytes, *p, workspace, workspace_bytes, what)) return rc;
  if (lda < K) return set_error(BSK_ERR_INVALID_ARG, "%s: lda < K", what);
  if (!A && M > 0 && K > 0) return set_error(BSK_ERR_INVALID_ARG, "%s: null A", what);
  return BSK_OK;
}

}  // namespace

int64_t bsk_bsr_convert_workspace_bytes(int M, int K, int bs) {
  ConvPlan p;
  if (int rc = conv_plan(M, K, bs, &p, "bsr_convert")) return rc;
  return p.total;
}

int bsk_dense_to_bsr_pattern(const void* A, int64_t lda, int elem_bytes, int M, int K, int bs, void* row_ptr,
                             int index_bytes, void* workspace, int64_t workspace_bytes, int64_t* nnzb,
                             int64_t* nnz_elems, void* stream) {
  const char* what = "dense_to_bsr_pattern";
  ConvPlan p;
  if (int rc = dense_checks(A, lda, elem_bytes, index_bytes, M, K, bs, &p, workspace, workspace_bytes, what)) return rc;
  if (!row_ptr) return set_error(BSK_ERR_INVALID_ARG, "%s: null row_ptr", what);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int rc = dense_pattern_enqueue(A, lda, elem_bytes, M, K, bs, row_ptr, index_bytes, p, workspace, st, s, what))
    return rc;
  return conv_read_tail(p, workspace, index_bytes, nnzb, nnz_elems, s, what);
}

int bsk_dense_to_bsr_fill(const void* A, int64_t lda, int elem_bytes, int M, int K, int bs, const void* row_ptr,
                          void* col_idx, int index_bytes, void* values, int64_t nnzb, void* workspace,
                          int64_t workspace_bytes, void* stream) {
  const char* what = "dense_to_bsr_fill";
  ConvPlan p;
  if (int rc = dense_checks(A, lda, elem_bytes, index_bytes, M, K, bs, &p, workspace, workspace_bytes, what)) return rc;
  if (nnzb < 0) return set_error(BSK_ERR_INVALID_ARG, "%s: negative nnzb", what);
  if ((int64_t)M * K == 0 || nnzb == 0) return BSK_OK;
  if (!row_ptr || !col_idx || !values) return set_error(BSK_ERR_INVALID_ARG, "%s: null pointer", what);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  return dense_fill_enqueue(A, lda, elem_bytes, bs, row_ptr, col_idx, index_bytes, values, nnzb, p, workspace, st,
                            static_cast<cudaStream_t>(stream), what);
}

int bsk_dense_to_bsr_bounded(const void* A, int64_t lda, int elem_bytes, int M, int K, int bs, void* row_ptr,
                             void* col_idx, int index_bytes, void* values, int64_t max_nnzb, void* workspace,
                             int64_t workspace_bytes, void* stream) {
  const char* what = "dense_to_bsr_bounded";
  ConvPlan p;
  if (int rc = dense_checks(A, lda, elem_bytes, index_bytes, M, K, bs, &p, workspace, workspace_bytes, what)) return rc;
  if (max_nnzb < 0) return set_error(BSK_ERR_INVALID_ARG, "%s: negative max_nnzb", what);
  if (!row_ptr || (max_nnzb > 0 && (!col_idx || !values)))
    return set_error(BSK_ERR_INVALID_ARG, "%s: null output pointer", what);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool small = conv_small(p);
  if (int rc = dense_pattern_enqueue(A, lda, elem_bytes, M, K, bs, row_ptr, index_bytes, p, workspace, st, s, what,
                                     !small))
    return rc;
  if (small)
    if (int rc = conv_index_small(p, conv_ws(p, workspace), row_ptr, col_idx, index_bytes, max_nnzb, s)) return rc;
  if (max_nnzb == 0 || (int64_t)M * K == 0) return BSK_OK;
  return dense_fill_enqueue(A, lda, elem_bytes, bs, row_ptr, col_idx, index_bytes, values, max_nnzb, p, workspace,
                            st, s, what, !small);
}

int bsk_csr_to_bsr_pattern(const void* crow, const void* col, int index_bytes_in, const void* vals, int elem_bytes,
                           int64_t nnz, int M, int K, int bs, void* row_ptr, int index_bytes, void* workspace,
                           int64_t workspace_bytes, int64_t* nnzb, int64_t* nnz_elems, void* stream) {
  const char* what = "csr_to_bsr_pattern";
  ConvPlan p;
  if (int rc = conv_plan(M, K, bs, &p, what)) return rc;
  if (int rc = conv_common_checks(elem_bytes, index_bytes, p, workspace, workspace_bytes, what)) return rc;
  if (int rc = csr_checks(crow, col, index_bytes_in, vals, nnz, M, what)) return rc;
  if (!row_ptr) return set_error(BSK_ERR_INVALID_ARG, "%s: null row_ptr", what);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int rc = csr_pattern_enqueue(crow, col, index_bytes_in, vals, elem_bytes, nnz, M, K, bs, row_ptr, index_bytes, p,
                                   workspace, st, s, what))
    return rc;
  return conv_read_tail(p, workspace, index_bytes, nnzb, nnz_elems, s, what);
}

int bsk_csr_to_bsr_fill(const void* crow, const void* col, int index_bytes_in, const void* vals, int elem_bytes,
                        int64_t nnz, int M, int K, int bs, const void* row_ptr, void* col_idx, int index_bytes,
                        void* values, int64_t nnzb, void* workspace, int64_t workspace_bytes, void* stream) {
  const char* what = "csr_to_bsr_fill";
  ConvPlan p;
  if (int rc = conv_plan(M, K, bs, &p, what)) return rc;
  if (int rc = conv_common_checks(elem_bytes, index_bytes, p, workspace, workspace_bytes, what)) return rc;
  if (int rc = csr_checks(crow, col, index_bytes_in, vals, nnz, M, what)) return rc;
  if (nnzb < 0) return set_error(BSK_ERR_INVALID_ARG, "%s: negative nnzb", what);
  if (nnzb == 0) return BSK_OK;
  if (!row_ptr || !col_idx || !values) return set_error(BSK_ERR_INVALID_ARG, "%s: null output pointer", what);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  return csr_fill_enqueue(crow, col, index_bytes_in, vals, elem_bytes, nnz, M, K, bs, row_ptr, col_idx, index_bytes,
                          values, nnzb, p, workspace, st, static_cast<cudaStream_t>(stream), what);
}

int bsk_csr_to_bsr_bounded(const void* crow, const void* col, int index_bytes_in, const void* vals, int elem_bytes,
                           int64_t nnz, int M, int K, int bs, void* row_ptr, void* col_idx, int index_bytes,
                           void* values, int64_t max_nnzb, void* workspace, int64_t workspace_bytes, void* stream) {
  const char* what = "csr_to_bsr_bounded";
  ConvPlan p;
  if (int rc = conv_plan(M, K, bs, &p, what)) return rc;
  if (int rc = conv_common_checks(elem_bytes, index_bytes, p, workspace, workspace_bytes, what)) return rc;
  if (int rc = csr_checks(crow, col, index_bytes_in, vals, nnz, M, what)) return rc;
  if (max_nnzb < 0) return set_error(BSK_ERR_INVALID_ARG, "%s: negative max_nnzb", what);
  if (!row_ptr || (max_nnzb > 0 && (!col_idx || !values)))
    return set_error(BSK_ERR_INVALID_ARG, "%s: null output pointer", what);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool small = conv_small(p);
  if (int rc = csr_pattern_enqueue(crow, col, index_bytes_in, vals, elem_bytes, nnz, M, K, bs, row_ptr, index_bytes, p,
                                   workspace, st, s, what, !small))
    return rc;
  if (small)
    if (int rc = conv_index_small(p, conv_ws(p, workspace), row_ptr, col_idx, index_bytes, max_nnzb, s)) return rc;
  if (max_nnzb == 0) return BSK_OK;
  return csr_fill_enqueue(crow, col, index_bytes_in, vals, elem_bytes, nnz, M, K, bs, row_ptr, col_idx, index_bytes,
                          values, max_nnzb, p, workspace, st, s, what, !small);
}

int bsk_bsattn_fwd_ex(int dtype, const void* Q, const void* K, const void* V, void* O, float* lse,
                      const int32_t* row_ptr, const int32_t* col_idx, int B, int H, int S, int D, int blk, float scale,
                      int causal_diag, int bh_begin, int bh_end, void* stream) {
  if (dtype != 0 && dtype != 1) return set_error(BSK_ERR_INVALID_ARG, "bsattn_fwd_ex: dtype must be 0 (bf16) or 1 (f16)");
  if (lse && reinterpret_cast<uintptr_t>(lse) % 4) return set_error(BSK_ERR_INVALID_ARG, "bsattn_fwd_ex: lse misaligned");
  return bsattn_launch(dtype == 1, Q, K, V, O, lse, row_ptr, col_idx, B, H, S, D, blk, scale, causal_diag, bh_begin,
                       bh_end, stream);
}

int bsk_bsattn_mask_transpose(const int32_t* row_ptr, const int32_t* col_idx, int pairs, int nqb, int32_t* col_ptr,
                              int32_t* row_idx, void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace bsk;
  if (pairs < 0 || nqb < 0) return set_error(BSK_ERR_INVALID_ARG, "bsattn_mask_transpose: negative extent");
  if (!row_ptr || !col_ptr || (pairs > 0 && nqb > 0 && (!col_idx || !row_idx)))
    return set_error(BSK_ERR_INVALID_ARG, "bsattn_mask_transpose: null pointer");
  const int64_t need = (int64_t)pairs * nqb * 4 + 16;
  if (!workspace || workspace_bytes < need)
    return set_error(BSK_ERR_INVALID_ARG, "bsattn_mask_transpose: workspace of %lld bytes needed", (long long)need);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (pairs == 0 || nqb == 0) {
    cudaError_t e = cudaMemcpyAsync(col_ptr, row_ptr, sizeof(int32_t), cudaMemcpyDeviceToDevice, s);
    return e == cudaSuccess ? BSK_OK : cuda_fail(e, "bsattn_mask_transpose");
  }
  int* cursor = static_cast<int*>(workspace);
  int* bad = reinterpret_cast<int*>(static_cast<char*>(workspace) + (int64_t)pairs * nqb * 4);
  cudaError_t e = cudaMemsetAsync(bad, 0, sizeof(int), s);
  if (e != cudaSuccess) return cuda_fail(e, "bsattn_mask_transpose");
  if (nqb <= kTransposeSmemMaxBlocks) {
    const int smem = nqb * ((nqb + 31) / 32) * 4;
    const int grid = pairs < st->sm_count * 4 ? pairs : st->sm_count * 4;
    bsattn_mask_transpose_smem_kernel<<<grid, 256, smem, s>>>(row_ptr, col_idx, pairs, nqb, col_ptr, row_idx, bad);
  } else {
    const int threads = 128, grid = (pairs + threads - 1) / threads;
    bsattn_mask_transpose_kernel<<<grid, threads, 0, s>>>(row_ptr, col_idx, pairs, nqb, col_ptr, row_idx, cursor, bad);
  }
  return launch_status("bsattn_mask_transpose");
}

int bsk_bsattn_bwd(int dtype, const void* dO, const void* Q, const void* K, const void* V, const void* O,
                   const float* lse, void* dQ, void* dK, void* dV, const int32_t* row_ptr, const int32_t* col_idx,
                   const int32_t* col_ptr, const int32_t* row_idx, int B, int H, int S, int D, int blk, float scale,
                   int causal_diag, float* delta, void* stream) {
  using namespace bsk;
  const char* what = "bsattn_bwd";
  if (dtype != 0 && dtype != 1) return set_error(BSK_ERR_INVALID_ARG, "%s: dtype must be 0 (bf16) or 1 (f16)", what);
  if (D != 64 && D != 128) return set_error(BSK_ERR_UNSUPPORTED, "%s: head_dim %d unsupported (64 or 128)", what, D);
  if (blk != kAttnBlk) return set_error(BSK_ERR_UNSUPPORTED, "%s: block size %d unsupported (needs %d)", what, blk, kAttnBlk);
  if (B < 0 || H < 0 || S < 0) return set_error(BSK_ERR_INVALID_ARG, "%s: negative extent", what);
  if (S % blk) return set_error(BSK_ERR_INVALID_ARG, "%s: S=%d not a multiple of the block size %d", what, S, blk);
  if (!(scale > 0.0f) || !(scale < 1e30f)) return set_error(BSK_ERR_INVALID_ARG, "%s: scale must be positive and finite", what);
  const int pairs = B * H;
  if (pairs == 0 || S == 0) return BSK_OK;
  if (!dO || !Q || !K || !V || !O || !lse || !dQ || !dK || !dV || !row_ptr || !col_idx || !col_ptr || !row_idx || !delta)
    return set_error(BSK_ERR_INVALID_ARG, "%s: null pointer", what);
  if (!aligned16(dO) || !aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) || !aligned16(dQ) ||
      !aligned16(dK) || !aligned16(dV) || !aligned16(lse) || !aligned16(delta))
    return set_error(BSK_ERR_INVALID_ARG, "%s: tensors must be 16-byte aligned", what);
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t rows = (uint64_t)pairs * S;
  const CUtensorMapDataType dt = dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq, tk, tv, tdo;
  if (int rc = make_map(&tq, dt, 2, Q, D, rows, D * 2, 64, kAttnBlk, "Q")) return rc;
  if (int rc = make_map(&tk, dt, 2, K, D, rows, D * 2, 64, kAttnBlk, "K")) return rc;
  if (int rc = make_map(&tv, dt, 2, V, D, rows, D * 2, 64, kAttnBlk, "V")) return rc;
  if (int rc = make_map(&tdo, dt, 2, dO, D, rows, D * 2, 64, kAttnBlk, "dO")) return rc;
  AttnBwdArgs a{};
  a.dO = dO;
  a.O = O;
  a.lse = lse;
  a.delta = delta;
  a.nlse2 = delta + rows;
  a.dQ = dQ;
  a.dK = dK;
  a.dV = dV;
  a.row_ptr = row_ptr;
  a.col_idx = col_idx;
  a.col_ptr = col_ptr;
  a.row_idx = row_idx;
  a.S = S;
  a.nqb = S / blk;
  a.bh_begin = 0;
  a.num_items = pairs * a.nqb;
  a.scale = scale;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal_diag = causal_diag;
  a.err = st->err_word;
  a.timeout_ns = t_timeout_ns;
  const int grid = a.num_items < st->sm_count ? a.num_items : st->sm_count;
  const uint16_t* dO16 = static_cast<const uint16_t*>(dO);
  const uint16_t* O16 = static_cast<const uint16_t*>(O);
  const int dgrid = st->sm_count * 8;
#define BSK_BWD(F16, DD)                                                                                            \
  do {                                                                                                              \
    bsattn_bwd_delta_kernel<F16, DD><<<dgrid, 256, 0, s>>>(dO16, O16, lse, delta, delta + rows, (int64_t)rows);     \
    bsattn_bwd_dkdv_kernel<F16, DD><<<grid, kBwdThreads, BwdDkdvShape<F16, DD>::kSmemBytes, s>>>(tq, tk, tv, tdo, a); \
    bsattn_bwd_dq_kernel<F16, DD><<<grid, kBwdThreads, BwdDqShape<F16, DD>::kSmemBytes, s>>>(tq, tk, tv, tdo, a);     \
  } while (0)
  if (dtype == 1 && D == 128) BSK_BWD(true, 128);
  else if (dtype == 1) BSK_BWD(true, 64);
  else if (D == 128) BSK_BWD(false, 128);
  else BSK_BWD(false, 64);
#undef BSK_BWD
  return launch_status(what);
}

namespace {

// Stream-ordered scratch for the reference-signature attention launchers (freed on the same stream).
struct StreamScratch {
  cudaStream_t s;
  std::vector<void*> ptrs;
  explicit StreamScratch(cudaStream_t st) : s(st) {}
  void* get(size_t bytes, cudaError_t* e) {
    void* p = nullptr;
    if (*e == cudaSuccess) *e = cudaMallocAsync(&p, bytes < 16 ? 16 : bytes, s);
    if (*e == cudaSuccess) ptrs.push_back(p);
    return p;
  }
  ~StreamScratch() {
    for (void* p : ptrs) cudaFreeAsync(p, s);
  }
};

// Dense or causal block mask of `pairs` (b,h) pairs in stream-ordered scratch.
int full_mask(StreamScratch& ss, int pairs, int nqb, bool causal, int** row_ptr, int** col_idx, int64_t* nnz,
              const char* what) {
  const int64_t per = causal ? (int64_t)nqb * (nqb + 1) / 2 : (int64_t)nqb * nqb;
  *nnz = per * pairs;
  if (*nnz >= INT32_MAX) return set_error(BSK_ERR_UNSUPPORTED, "%s: %lld mask blocks exceed int32", what, (long long)*nnz);
  cudaError_t e = cudaSuccess;
  *row_ptr = static_cast<int*>(ss.get(((size_t)pairs * nqb + 1) * 4, &e));
  *col_idx = static_cast<int*>(ss.get((size_t)*nnz * 4, &e));
  if (e != cudaSuccess) return cuda_fail(e, what);
  const int rows = pairs * nqb;
  bsk::attn_full_mask_kernel<<<(rows + 255) / 256, 256, 0, ss.s>>>(pairs, nqb, causal ? 1 : 0, *row_ptr, *col_idx);
  return launch_status(what);
}

int ref_attention_checks(int B, int H, int S, int D, const char* what) {
  if (B < 0 || H < 0 || S < 0) return set_error(BSK_ERR_INVALID_ARG, "%s: negative extent", what);
  if (D != 64 && D != 128) return set_error(BSK_ERR_UNSUPPORTED, "%s: head_dim %d unsupported (64 or 128)", what, D);
  if (S % 128) return set_error(BSK_ERR_UNSUPPORTED, "%s: S=%d must be a multiple of 128", what, S);
  return BSK_OK;
}

}  // namespace

void launch_attention_forward(const void* Q, const void* K, const void* V, void* O, int B, int H, int S, int D,
                              float scale, bool causal, void* stream) {
  const char* what = "launch_attention_forward";
  if (ref_attention_checks(B, H, S, D, what)) return;
  if (B * H == 0 || S == 0) return;
  DeviceState* st;
  if (device_state(&st)) return;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  StreamScratch ss(s);
  int *rp = nullptr, *ci = nullptr;
  int64_t nnz = 0;
  if (full_mask(ss, B * H, S / 128, causal, &rp, &ci, &nnz, what)) return;
  if (bsattn_launch(true, Q, K, V, O, nullptr, rp, ci, B, H, S, D, 128, scale, causal ? 1 : 0, 0, B * H, stream) ==
      BSK_OK)
    t_last_error.clear();
}

void launch_attention_backward(const void* grad_out, const void* Q, const void* K, const void* V, const void* O,
                               void* grad_Q, void* grad_K, void* grad_V, int B, int H, int S, int D, float scale,
                               bool causal, void* stream) {
  const char* what = "launch_attention_backward";
  if (ref_attention_checks(B, H, S, D, what)) return;
  if (B * H == 0 || S == 0) return;
  DeviceState* st;
  if (device_state(&st)) return;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  StreamScratch ss(s);
  const int pairs = B * H, nqb = S / 128;
  int *rp = nullptr, *ci = nullptr;
  int64_t nnz = 0;
  if (full_mask(ss, pairs, nqb, causal, &rp, &ci, &nnz, what)) return;
  // The signature carries no log-sum-exp: a forward pass recomputes it (its output goes to scratch).
  cudaError_t e = cudaSuccess;
  const size_t rows = (size_t)pairs * S;
  float* lse = static_cast<float*>(ss.get(rows * 4, &e));
  float* delta = static_cast<float*>(ss.get(rows * 8, &e));  // Delta and -LSE log2(e)
  void* o_tmp = ss.get(rows * D * 2, &e);
  int* col_ptr = static_cast<int*>(ss.get(((size_t)pairs * nqb + 1) * 4, &e));
  int* row_idx = static_cast<int*>(ss.get((size_t)nnz * 4, &e));
  void* tws = ss.get((size_t)pairs * nqb * 4 + 16, &e);
  if (e != cudaSuccess) {
    cuda_fail(e, what);
    return;
  }
  if (bsattn_launch(true, Q, K, V, o_tmp, lse, rp, ci, B, H, S, D, 128, scale, causal ? 1 : 0, 0, pairs, stream))
    return;
  if (bsk_bsattn_mask_transpose(rp, ci, pairs, nqb, col_ptr, row_idx, tws, (int64_t)pairs * nqb * 4 + 16, stream))
    return;
  if (bsk_bsattn_bwd(1, grad_out, Q, K, V, O, lse, grad_Q, grad_K, grad_V, rp, ci, col_ptr, row_idx, B, H, S, D, 128,
                     scale, causal ? 1 : 0, delta, stream) == BSK_OK)
    t_last_error.clear();
}

int bsk_device_error(uint32_t* out) {
  if (!out) return set_error(BSK_ERR_INVALID_ARG, "device_error: null output");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "device_error: synchronize");
  e = cudaMemcpy(out, st->err_word, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "device_error: read");
  e = cudaMemset(st->err_word, 0, sizeof(uint32_t));
  if (e != cudaSuccess) return cuda_fail(e, "device_error: clear");
  return BSK_OK;
}

int bsk_selftest_wait_timeout(uint64_t timeout_ns, void* stream) {
  if (timeout_ns < 1000ull || timeout_ns > 10000000000ull)
    return set_error(BSK_ERR_INVALID_ARG, "selftest: timeout outside [1e3, 1e10] ns");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "selftest: pre-sync");
  e = cudaMemsetAsync(st->err_word, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "selftest: clear");
  bsk::wait_probe_kernel<<<1, 32, 0, s>>>(st->err_word, timeout_ns);
  if (int rc = launch_status("selftest launch")) return rc;
  uint32_t word = 0;
  e = cudaMemcpyAsync(&word, st->err_word, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "selftest: read back");
  cudaMemsetAsync(st->err_word, 0, sizeof(uint32_t), s);
  cudaStreamSynchronize(s);
  if ((word & 0xFF) == bsk::kErrWaitTimeout && ((word >> 8) & 0xFF) == bsk::kKidWaitProbe)
    return set_error(BSK_ERR_DEVICE_TIMEOUT, "bounded wait ran out after %llu ns (expected)",
                     (unsigned long long)timeout_ns);
  return set_error(BSK_ERR_CUDA, "selftest: the probe kernel did not report a timeout (word=0x%08x)", word);
}

int bsk_selftest_exp2(const float* x, float* y, int n, int fma_pipe, void* stream) {
  if (n < 0) return set_error(BSK_ERR_INVALID_ARG, "selftest_exp2: negative length");
  if (fma_pipe != 0 && fma_pipe != 1) return set_error(BSK_ERR_INVALID_ARG, "selftest_exp2: fma_pipe must be 0 or 1");
  if (n > 0 && (!x || !y)) return set_error(BSK_ERR_INVALID_ARG, "selftest_exp2: null pointer");
  DeviceState* st;
  if (int rc = device_state(&st)) return rc;
  if (n == 0) return BSK_OK;
  const int pairs = (n + 1) / 2;
  const int blocks_needed = (pairs + 255) / 256;
  const int grid = blocks_needed < 4 * st->sm_count ? blocks_needed : 4 * st->sm_count;
  bsk::exp2_probe_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n, fma_pipe);
  return launch_status("selftest_exp2 launch");
}

}  // extern "C"
