/*
 * bsk_capi.h — C ABI of the B200 (sm_100a) BlackwellSparseK operator family.
 *
 * Library: libbsk_sm100.so (periodicdent42_b200/libbsk_sm100.so). Plain pointers and sizes only.
 *
 * Conventions shared by every entry point:
 *  - Return 0 (BSK_OK) on success, a negative BSK_ERR_* code otherwise; bsk_last_error() returns a
 *    thread-local message for the last failure on the calling thread.
 *  - Device pointers are borrowed; outputs are preallocated by the caller. Nothing is synchronised:
 *    work is enqueued on `stream` (a cudaStream_t, NULL = legacy default stream) of the current device.
 *  - Arguments are validated on the host before any launch (shapes, strides, the 16-byte alignment TMA
 *    needs); BSR index structures in host memory can be checked with bsk_bsr_validate_host, and the kernels
 *    clamp and flag out-of-range indices on the device.
 *  - Every device-side wait is bounded. A wait that runs out records a code in a per-device error word
 *    (read and cleared by bsk_device_error) and the kernel returns early with its output incomplete.
 *  - There is no CPU fallback: without a usable sm_100 device every compute entry point fails with
 *    BSK_ERR_NO_DEVICE.
 */
#ifndef BSK_CAPI_H_
#define BSK_CAPI_H_

#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BSK_OK 0
#define BSK_ERR_INVALID_ARG (-1)
#define BSK_ERR_UNSUPPORTED (-2)
#define BSK_ERR_CUDA (-3)
#define BSK_ERR_DEVICE_TIMEOUT (-4)
#define BSK_ERR_NO_DEVICE (-5)

/* Library version, (major << 16) | (minor << 8) | patch. */
int bsk_version(void);

/* Message for the last failing call on this thread ("" if none). */
const char* bsk_last_error(void);

/* Number of SMs of the current device, or a negative error code. */
int bsk_device_sm_count(void);

/*
 * Per-shape launch configurations (what an autotuner found best, e.g. restored from its JSON cache). For an
 * operator and an exact (M, N, K) -- K being the K extent of the launch -- the later launches use:
 *   tile    : -1 the built-in policy, 0 single-CTA 128x256, 1 CTA pair 256x256, 2 CTA pair 256x512
 *             (dense GEMMs only; ignored by the SpMMs)
 *   group_m : tile-rasterisation group (M tiles walked together), 0 = the built-in choice
 * Process-wide; bsk_config_get returns 1 and the entry when one is registered, 0 (tile -1, group 0) otherwise.
 * Replaces the reference's size-bucketed _autotune_config (BlackwellSparseK/python/ops.py:209-217) and its
 * variant cache (optim_local/src/sparse/autotune_sparse.h).
 */
#define BSK_OP_GEMM_F16F32 1
#define BSK_OP_GEMM_E4M3_BF16 2
#define BSK_OP_SPMM_BSR 3
#define BSK_OP_SPMM_BSR_BSR 4
int bsk_config_set(int op, int M, int N, int K, int tile, int group_m);
int bsk_config_get(int op, int M, int N, int K, int* tile, int* group_m);
int bsk_config_clear(void);

/*
 * Dense GEMM, fp16 x fp16 -> fp32:  C[M,N] = A[M, k_begin:k_end] * B[k_begin:k_end, N].
 *   A   : fp16, row-major [M, K], row stride lda (elements, multiple of 8, 16-B aligned base)
 *   B   : fp16, column-major [K, N] (equivalently B^T row-major [N, K]), column stride ldb
 *   C   : fp32, row-major [M, N], row stride ldc; overwritten (not accumulated)
 *   k_begin/k_end select the K range (split-K shards); k_begin must be a multiple of 8.
 * Replaces the reference's standalone CUTLASS Sm90 program
 * (BlackwellSparseK/src/gemm_h100_599tflops_final.cu:38-67, run at :144-151), which had no callable
 * entry point.
 */
int bsk_gemm_f16f32(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M, int N,
                    int K, int k_begin, int k_end, void* stream);

/*
 * bsk_gemm_f16f32 that accumulates: C[M,N] += A[M, k_begin:k_end] * B[k_begin:k_end, N] (each C element read
 * once, the product added to it, stored). For callers that sweep K in pieces (K-chunked streaming, K shards
 * summed on one GPU). No reference counterpart.
 */
int bsk_gemm_f16f32_acc(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M, int N,
                        int K, int k_begin, int k_end, void* stream);

/*
 * Dense GEMM from HOST memory: C_host[M,N] = A_host[M,K] * B_host[K,N] (same layouts as bsk_gemm_f16f32), streamed
 * through the GPU in K chunks: the host-to-device copies of chunk i+1 (on a stream of this call's own) overlap
 * the tensor-core work on chunk i and C accumulates in device memory. The last chunk goes by row panels (about
 * M/8 rows, whole 256-row tiles): each panel's C rows are final after its GEMM and are copied back while the
 * next panel's rows are still being uploaded.
 *   A_host, B_host, C_host : host memory; page-locked (cudaHostAlloc / cudaHostRegister) for the copies to be
 *                            asynchronous and overlap; pageable memory works but serialises.
 *   k_chunk   : K elements per chunk, a multiple of 64; <= 0 chooses (about 16 chunks of at least 4096).
 *   workspace : device memory, 256-byte aligned, of bsk_gemm_host_workspace_bytes(M, N, K, k_chunk) bytes
 *               (two A chunks, two B chunks, the fp32 C); used by this call until `stream` reaches its end.
 * Everything is ordered on `stream`: the call returns once the work is enqueued and C_host is complete when
 * the stream has synchronised. No reference counterpart (the reference's GEMM programs time device-resident
 * operands only).
 */
int bsk_gemm_f16f32_host(const void* A_host, int64_t lda, const void* B_host, int64_t ldb, float* C_host,
                         int64_t ldc, int M, int N, int K, int k_chunk, void* workspace, int64_t workspace_bytes,
                         void* stream);

/* K elements per chunk that bsk_gemm_f16f32_host uses for this K and k_chunk request (k_chunk <= 0: automatic),
 * or a negative error code; lets a caller that stages chunks itself use the same plan. */
int bsk_gemm_host_chunk(int K, int k_chunk);

/* Asynchronous 2-D copy on `stream`: `rows` rows of `width_bytes` bytes from src (row pitch spitch bytes) to dst
 * (row pitch dpitch bytes), either side host or device (unified addressing decides the direction). A helper for
 * callers that stage row ranges of host matrices into device chunk buffers. */
int bsk_copy_2d_async(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width_bytes, int64_t rows,
                      void* stream);

/* Workspace bytes of bsk_gemm_f16f32_host for this shape and chunk (k_chunk <= 0: the automatic chunk), or a
 * negative error code. */
int64_t bsk_gemm_host_workspace_bytes(int M, int N, int K, int k_chunk);

/*
 * Dense GEMM as bsk_gemm_f16f32 (k range = all of K) with the K dimension split across CTA pairs, for shapes
 * whose output has too few 256 x 256 tiles to occupy the GPU (e.g. 1024 x 1024 with long K). Each split writes
 * an fp32 partial slab into `workspace`; a second kernel sums the slabs in split order (deterministic) into C.
 *   splits <= 0 : automatic (enough (tile, split) units for every CTA pair, >= 4 K stages per split, <= 32)
 *   workspace   : device memory of at least bsk_gemm_splitk_workspace_bytes(M, N, K, splits) bytes, 16-byte
 *                 aligned; may be NULL when that size is 0 (no split chosen). Used as scratch by this call only.
 * No reference counterpart (the reference's GEMM programs, BlackwellSparseK/src/gemm_h100_*.cu, had no split-K).
 */
int bsk_gemm_f16f32_splitk(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M,
                           int N, int K, int splits, void* workspace, int64_t workspace_bytes, void* stream);

/* Workspace bytes bsk_gemm_f16f32_splitk needs on the current device (0 if it would not split K), or a negative
 * error code. */
int64_t bsk_gemm_splitk_workspace_bytes(int M, int N, int K, int splits);

/*
 * bsk_gemm_f16f32_splitk for callers that cannot allocate device memory -- code bound to a fixed C signature
 * with no workspace argument (an FFI stub or plugin interface), or running where device allocation is not
 * permitted or is owned by another allocator. It allocates nothing: the split partials go to a static device
 * array of 32 MiB built into this library (every GPU that loads the library holds it until exit).
 *   - splits * M * round_up(N, 4) * 4 bytes must fit in 32 MiB, else BSK_ERR_INVALID_ARG with a message
 *     (e.g. 1024 x 1024 with up to 8 splits). Automatic splits (splits <= 0) always fit: the plan keeps
 *     (256 x 256 tiles) x splits at or below the co-resident CTA pairs (74 on a B200), i.e. at most
 *     74 x 256 KiB = 18.5 MiB of partials; only an explicit `splits` can exceed the array.
 *   - The first call on each device looks up the array's device address (cudaGetSymbolAddress); make that
 *     first call on a device before any stream capture.
 *   - All calls share the array: calls that overlap on the GPU (other streams, other threads) race on it.
 * No counterpart in the reference.
 */
int bsk_gemm_f16f32_splitk_static(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc,
                                  int M, int N, int K, int splits, void* stream);

/*
 * Split-K across ranks with the reduce-scatter fused into the GEMM (one process per GPU, NVLink peers).
 * Each rank r computes C_r = A[:, k_begin:k_end] * B[k_begin:k_end, :] for its K range and its epilogue stores
 * every output row i straight into the receive buffer of the row's owner (i / (M/world)), slot r:
 *   slot_bufs[o] -> owner o's buffer [world][M/world][ld_slot] fp32 (its own buffer for o == rank, the others
 *                   opened with bsk_peer_buffer_open); the stores cross NVLink while later tiles compute.
 * After every rank's call has completed (a stream-ordered barrier such as a one-element all-reduce),
 * bsk_splitk_slots_reduce on each rank sums its world slots in rank order (deterministic) into its M/world rows.
 * Replaces the split-K + NCCL reduce-scatter plan of the operator family's multi-GPU dense GEMM; no reference
 * counterpart (the reference has no multi-GPU code).
 */
int bsk_gemm_f16f32_splitk_scatter(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K,
                                   int k_begin, int k_end, int world, int rank, void* const* slot_bufs,
                                   int64_t ld_slot, void* stream);

/* C[rows, N] = sum over s < world of slots[s][rows][ld_slot], in slot order. */
int bsk_splitk_slots_reduce(const float* slots, int world, int rows, int N, int64_t ld_slot, float* C, int64_t ldc,
                            void* stream);

/* Receive buffers shared between processes: cudaMalloc + a 64-byte CUDA IPC handle; open a peer's handle
 * (peer access enabled lazily), close it, free an own buffer. */
int bsk_peer_buffer_alloc(int64_t bytes, void** dev_ptr, void* ipc_handle);
int bsk_peer_buffer_open(const void* ipc_handle, void** dev_ptr);
int bsk_peer_buffer_close(void* dev_ptr);
int bsk_peer_buffer_free(void* dev_ptr);

/*
 * FP8 GEMM, e4m3 x e4m3 -> bf16:  D[M,N] = bf16( (A_q[M,K] * B_q[K,N]) * scale_a * scale_b ).
 *   A   : e4m3 bytes, row-major [M, K] (lda multiple of 16)
 *   B   : e4m3 bytes, column-major [K, N] (B^T row-major [N, K], ldb multiple of 16)
 *   scale_a, scale_b : device pointers to one fp32 each (per-tensor dequantisation scales)
 *   D   : bf16, row-major [M, N], row stride ldd
 * No reference counterpart exists (the reference only declares e4m3 typedefs,
 * BlackwellSparseK/.archive/src_experiments/blackwell_sparsek/kernels/attention_fmha.cu:32-42); the
 * semantics follow torch._scaled_mm(A_q, B_q, scale_a, scale_b, out_dtype=bfloat16).
 */
int bsk_gemm_e4m3_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, const float* scale_a,
                       const float* scale_b, void* D, int64_t ldd, int M, int N, int K, void* stream);

/*
 * BSR block-sparse x dense SpMM, fp16 x fp16 -> fp32:  C[M,N] = A_bsr[M,K] * B[K,N].
 *   row_ptr : int32 [Mb+1] block-row pointer (torch crow_indices() narrowed to int32)
 *   col_idx : int32 [nnzb] block-column indices (torch col_indices()), any order within a row
 *   vals    : fp16 [nnzb, bs_r, bs_c] row-major blocks (torch values())
 *   B       : fp16 row-major [K, N], row stride ldb (multiple of 8)
 *   C       : fp32 row-major [M, N], row stride ldc; block-rows [row_begin, row_end) are overwritten
 *             (rows without nonzero blocks are written as zeros), other rows are untouched.
 *   Supported block shape: bs_r = bs_c = 128.
 * Replaces extern "C" launch_bsr_spmm_async (BlackwellSparseK/src/kernel_launch.cu:33-61), bound by
 * BlackwellSparseK/python/bsk_bindings.cpp:13-43 and called at :122-129; dense B replaces the
 * "dense B as BSR" arguments built in BlackwellSparseK/python/ops.py:104-107.
 */
int bsk_spmm_bsr_f16f32(const int32_t* row_ptr, const int32_t* col_idx, const void* vals, int bs_r, int bs_c,
                        int Mb, int nnzb, const void* B, int64_t ldb, float* C, int64_t ldc, int M, int N, int K,
                        int row_begin, int row_end, void* stream);

/*
 * BSR x BSR SpMM, fp16 -> fp32:  C[M,N] = A_bsr[M,K] * B_bsr[K,N], both with 128 x 128 blocks, C dense.
 *   A: a_row_ptr [Mb + 1], a_col_idx [a_nnzb], a_vals [a_nnzb, 128, 128] (as bsk_spmm_bsr_f16f32).
 *   B: b_row_ptr [K/128 + 1], b_col_idx [b_nnzb] ascending within each block-row (the kernel binary-searches
 *      them), b_vals [b_nnzb, 128, 128] row-major blocks. Missing blocks are zero.
 *   M, K, N multiples of 128; block-rows [row_begin, row_end) of C are written.
 * Replaces the sparse-B case of launch_bsr_spmm_async (BlackwellSparseK/src/kernel_launch.cu:33-61, whose
 * kernel looks B blocks up by binary search, src/sparse_h100_async.cu:105-119); launch_bsr_spmm_async
 * routes a B with fewer than (K/128) x (N/128) stored blocks here.
 */
int bsk_spmm_bsr_bsr_f16f32(const int32_t* a_row_ptr, const int32_t* a_col_idx, const void* a_vals, int Mb,
                            int a_nnzb, const int32_t* b_row_ptr, const int32_t* b_col_idx, const void* b_vals,
                            int b_nnzb, float* C, int64_t ldc, int M, int N, int K, int row_begin, int row_end,
                            void* stream);

/*
 * Host-side check of a BSR index structure held in HOST memory (row_ptr[0] == 0, non-decreasing,
 * row_ptr[Mb] == nnzb, 0 <= col_idx < Kb). Returns BSK_OK or BSK_ERR_INVALID_ARG with a message.
 * The reference performs no such check (BlackwellSparseK/python/ops.py:56-69 validates shapes only).
 */
int bsk_bsr_validate_host(const int32_t* row_ptr, const int32_t* col_idx, int Mb, int Kb, int nnzb);

/*
 * Block-sparse attention forward, bf16:  O = softmax(scale * Q K^T, restricted to the block mask) V
 *   Q, K, V, O : bf16 contiguous [B, H, S, D], D = 64 or 128 (fp32 accumulation, fp32 softmax statistics)
 *   row_ptr    : int32 [B*H*(S/blk) + 1], col_idx int32 [nnz]: for (b,h) pair p and query block-row i
 *                the nonzero key blocks are col_idx[row_ptr[p*(S/blk)+i] .. row_ptr[p*(S/blk)+i+1]).
 *                col_idx values are within-sequence block indices (0 .. S/blk-1).
 *   blk        : 128. A key block with index equal to the query block index is masked elementwise-causally
 *                (key position > query position excluded) when `causal_diag` is non-zero.
 *   bh_begin/bh_end : the (b,h) pairs to compute (sharding); other pairs of O are untouched.
 *   Query rows whose mask row is empty are written as zeros.
 * Replaces extern "C" launch_attention_forward
 * (BlackwellSparseK/.archive/src_experiments/blackwell_sparsek/kernels/attention_fmha.cu:386-426), which
 * had no block mask, and its binding attention_forward_cuda (.../kernels/kernel_bindings.cpp:66-102).
 */
int bsk_bsattn_fwd_bf16(const void* Q, const void* K, const void* V, void* O, const int32_t* row_ptr,
                        const int32_t* col_idx, int B, int H, int S, int D, int blk, float scale, int causal_diag,
                        int bh_begin, int bh_end, void* stream);

/*
 * The same forward for fp16 Q, K, V, O (the element type of the reference's launch_attention_forward,
 * .archive/src_experiments/blackwell_sparsek/kernels/attention_fmha.cu:386-426, whose binding accepts
 * head dims 64 and 128, kernel_bindings.cpp:53-54). Arguments as bsk_bsattn_fwd_bf16; P is rounded to
 * fp16 before the P V product.
 */
int bsk_bsattn_fwd_f16(const void* Q, const void* K, const void* V, void* O, const int32_t* row_ptr,
                       const int32_t* col_idx, int B, int H, int S, int D, int blk, float scale, int causal_diag,
                       int bh_begin, int bh_end, void* stream);

/*
 * Dense / CSR -> BSR conversion on the device, square bs x bs blocks, in two phases (the caller sizes the outputs
 * from the first): the result equals torch's dense.to_sparse_bsr((bs, bs)) -- the conversion the reference's
 * convert_to_bsr performs (BlackwellSparseK/python/utils.py:10-57; its CSR path goes through to_dense(),
 * utils.py:32-35, and ops.py:193-197 left CSR -> BSR unimplemented):
 *   - a block is stored iff one of its elements is nonzero (-0.0 counts as zero, NaN as nonzero);
 *   - block columns ascend within a block-row; values [nnzb, bs, bs] hold the blocks bit for bit.
 * elem_bytes: 2 (fp16 / bf16) or 4 (fp32); index_bytes: 4 (int32) or 8 (int64, torch's default) for the outputs
 * row_ptr [M/bs + 1] and col_idx [nnzb]. M and K must be multiples of bs.
 * workspace: device memory of bsk_bsr_convert_workspace_bytes(M, K, bs) bytes, 256-byte aligned; the fill call
 * must get the workspace, row_ptr and nnzb its pattern call produced, unchanged (col_idx and values may be NULL
 * when nnzb is 0).
 * The pattern call synchronises `stream` to return *nnzb (stored blocks) and *nnz_elems (nonzero elements).
 * CSR input: crow [M + 1], col [nnz] (index_bytes_in 4 or 8), vals [nnz]; row r holds entries [crow[r], crow[r+1])
 * and entries outside [crow[0], crow[M]) are ignored; a column index outside [0, K) fails the pattern call with
 * BSK_ERR_INVALID_ARG. Entries stored twice for one (row, col) are not summed (one value wins).
 */
int64_t bsk_bsr_convert_workspace_bytes(int M, int K, int bs);
int bsk_dense_to_bsr_pattern(const void* A, int64_t lda, int elem_bytes, int M, int K, int bs, void* row_ptr,
                             int index_bytes, void* workspace, int64_t workspace_bytes, int64_t* nnzb,
                             int64_t* nnz_elems, void* stream);
int bsk_dense_to_bsr_fill(const void* A, int64_t lda, int elem_bytes, int M, int K, int bs, const void* row_ptr,
                          void* col_idx, int index_bytes, void* values, int64_t nnzb, void* workspace,
                          int64_t workspace_bytes, void* stream);
int bsk_csr_to_bsr_pattern(const void* crow, const void* col, int index_bytes_in, const void* vals, int elem_bytes,
                           int64_t nnz, int M, int K, int bs, void* row_ptr, int index_bytes, void* workspace,
                           int64_t workspace_bytes, int64_t* nnzb, int64_t* nnz_elems, void* stream);
int bsk_csr_to_bsr_fill(const void* crow, const void* col, int index_bytes_in, const void* vals, int elem_bytes,
                        int64_t nnz, int M, int K, int bs, const void* row_ptr, void* col_idx, int index_bytes,
                        void* values, int64_t nnzb, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Single-call forms of the two conversions for callers that can bound the number of stored blocks: pattern and
 * fill in one call, all on `stream`, with no host synchronisation (so they can be captured in a CUDA graph).
 * col_idx and values have room for max_nnzb blocks. When the stream has reached the end of the call,
 * row_ptr[M/bs] holds the true nnzb; if it exceeds max_nnzb, only the first max_nnzb blocks (in BSR order) were
 * written. A CSR column index outside [0, K) is skipped (the two-phase pattern call reports it instead).
 * No reference counterpart.
 */
int bsk_dense_to_bsr_bounded(const void* A, int64_t lda, int elem_bytes, int M, int K, int bs, void* row_ptr,
                             void* col_idx, int index_bytes, void* values, int64_t max_nnzb, void* workspace,
                             int64_t workspace_bytes, void* stream);
int bsk_csr_to_bsr_bounded(const void* crow, const void* col, int index_bytes_in, const void* vals, int elem_bytes,
                           int64_t nnz, int M, int K, int bs, void* row_ptr, void* col_idx, int index_bytes,
                           void* values, int64_t max_nnzb, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Block-sparse attention forward with the row log-sum-exp: as bsk_bsattn_fwd_bf16 / _f16 (dtype 0 = bf16,
 * 1 = fp16), and when lse is not NULL, lse[b*H*S + h*S + s] = natural-log log-sum-exp of query row s's scaled
 * scores over its unmasked keys (-inf for a row with no key blocks) -- what the backward needs.
 */
int bsk_bsattn_fwd_ex(int dtype, const void* Q, const void* K, const void* V, void* O, float* lse,
                      const int32_t* row_ptr, const int32_t* col_idx, int B, int H, int S, int D, int blk, float scale,
                      int causal_diag, int bh_begin, int bh_end, void* stream);

/*
 * Column lists of a block mask: for pair p (of `pairs`) and key block-column j, the query blocks whose row lists
 * contain j, ascending: row_idx[col_ptr[p*nqb + j] .. col_ptr[p*nqb + j + 1]). col_ptr [pairs*nqb + 1] uses the
 * numbering of row_ptr (pair p's entries start at row_ptr[p*nqb] in both); row_idx has row_ptr[pairs*nqb]
 * entries. workspace: pairs*nqb*4 + 16 bytes of device scratch.
 */
int bsk_bsattn_mask_transpose(const int32_t* row_ptr, const int32_t* col_idx, int pairs, int nqb, int32_t* col_ptr,
                              int32_t* row_idx, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Block-sparse attention backward (dtype 0 = bf16, 1 = fp16; D = 64 or 128; blk = 128):
 *   dV = P^T dO,  dK = scale * dS^T Q,  dQ = scale * dS K,  dS = P * (dO V^T - rowsum(dO * O)),
 *   P = exp(scale * Q K^T - lse) on the mask (the forward's; causal_diag as there).
 * dO, Q, K, V, O, dQ, dK, dV: [B, H, S, D] contiguous; lse [B*H*S] from bsk_bsattn_fwd_ex; row_ptr/col_idx the
 * forward's mask and col_ptr/row_idx its column lists (bsk_bsattn_mask_transpose); delta: device scratch of
 * 2*B*H*S floats (each row's rowsum(dO * O) and its exponent offset -lse * log2(e)). Deterministic: each output row is produced by one CTA in a fixed order (two passes recompute
 * the scores: one per key block for dK/dV, one per query block for dQ). Rows of dK/dV whose key block no query
 * block attends, and rows of dQ with no key blocks, are zero.
 * The reference declares launch_attention_backward
 * (.archive/src_experiments/blackwell_sparsek/kernels/attention_fmha.cu:436-453) but leaves it unimplemented.
 */
int bsk_bsattn_bwd(int dtype, const void* dO, const void* Q, const void* K, const void* V, const void* O,
                   const float* lse, void* dQ, void* dK, void* dV, const int32_t* row_ptr, const int32_t* col_idx,
                   const int32_t* col_ptr, const int32_t* row_idx, int B, int H, int S, int D, int blk, float scale,
                   int causal_diag, float* delta, void* stream);

/*
 * The reference's attention launchers, same signatures (.archive/src_experiments/blackwell_sparsek/kernels/
 * attention_fmha.cu:386-426 and :436-453): fp16 [B, H, S, D] tensors, dense attention (causal: key position <=
 * query position), D = 64 or 128, S a multiple of 128. Implemented with the block-sparse kernels on the full (or
 * lower-triangular) block mask, built in stream-ordered scratch (cudaMallocAsync / cudaFreeAsync on `stream`).
 * The backward takes no log-sum-exp, so it first runs the forward into scratch to recompute it. They return
 * nothing, like the reference; failures are reported through bsk_last_error().
 */
void launch_attention_forward(const void* Q, const void* K, const void* V, void* O, int B, int H, int S, int D,
                              float scale, bool causal, void* stream);
void launch_attention_backward(const void* grad_out, const void* Q, const void* K, const void* V, const void* O,
                               void* grad_Q, void* grad_K, void* grad_V, int B, int H, int S, int D, float scale,
                               bool causal, void* stream);

/*
 * Drop-in for the reference's launcher signature (BlackwellSparseK/src/kernel_launch.cu:33-61).
 * A is BSR with blocks of (M/A_M_blocks) x (K/A_K_blocks). A B with every block present is read as the dense
 * row-major [K, N] matrix the reference Python layer passes (BlackwellSparseK/python/ops.py:104-107); a B with
 * fewer blocks is a true BSR operand (128 x 128 blocks) and goes to bsk_spmm_bsr_bsr_f16f32. BM/BN/BK are accepted and ignored (the sm_100 kernel picks its own tiles). Returns
 * nothing, like the reference; failures are reported through bsk_last_error().
 */
void launch_bsr_spmm_async(const int* A_row_ptr, const int* A_col_idx, const void* A_vals, int A_M_blocks,
                           int A_K_blocks, int A_nnzb, const int* B_row_ptr, const int* B_col_idx, const void* B_vals,
                           int B_K_blocks, int B_N_blocks, int B_nnzb, float* C, int M, int N, int K, int ldc, int BM,
                           int BN, int BK, void* stream);

/*
 * Reads and clears the per-device error word of the current device. *out = 0 when no kernel reported
 * anything; otherwise bits [0,8) kind (1 wait timeout, 2 bounds), [8,16) kernel id, [16,32) site.
 * Synchronises the device.
 */
int bsk_device_error(uint32_t* out);

/* Per-wait limit in nanoseconds used by subsequent launches on this thread (default 2e9). */
int bsk_set_wait_timeout_ns(uint64_t ns);

/*
 * Failure-detection self-test: launches one CTA that waits on an mbarrier nothing will complete, with
 * the given limit (1e3 .. 1e10 ns). Returns BSK_ERR_DEVICE_TIMEOUT when the bounded wait ran out and the
 * kernel returned, which is the expected outcome. No reference counterpart (the reference has no
 * device-side failure detection).
 */
int bsk_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

/*
 * Accuracy self-test of the attention softmax's two exponential routes: y[i] = 2^x[i] for n device floats,
 * by the FMA-pipe polynomial (fma_pipe = 1; a quarter of the softmax's exponentials take it) or by the MUFU
 * instruction (fma_pipe = 0). Asynchronous on `stream`. No reference counterpart.
 */
int bsk_selftest_exp2(const float* x, float* y, int n, int fma_pipe, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BSK_CAPI_H_ */
