/*
 * forgeml_b200.h -- C ABI of the sm_100a (B200) kernels behind the ForgeML
 * compiled-forward dispatch and the Nebula decode step.
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers unless the comment says "host".
 *   - Strides are in ELEMENTS, not bytes.
 *   - `stream` is a cudaStream_t passed as void* (0 = legacy default stream).
 *   - The return value is 0 on success.  A nonzero value is an FML_E* code and
 *     fml_last_error() returns a message for the calling thread.  Nothing is
 *     launched when validation fails.  No entry point falls back to another
 *     implementation: an unsupported layout is an error.
 *   - Kernels never allocate.  Entry points that need scratch take a
 *     caller-owned workspace and have a *_workspace_size() query; the one
 *     exception is neb_ar_create, which allocates the all-reduce context's
 *     symmetric buffer once (freed by neb_ar_destroy).
 *   - dtype codes: FML_F32, FML_F16, FML_BF16.
 */
#ifndef FORGEML_B200_H
#define FORGEML_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FML_API __attribute__((visibility("default")))
#else
#define FML_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FML_OK = 0,
  FML_EINVAL = 1,        /* invalid argument (shape, stride, dtype, null pointer) */
  FML_EUNSUPPORTED = 2,  /* layout/size this kernel family does not handle */
  FML_ECUDA = 3,         /* CUDA runtime / driver error at launch */
  FML_EWORKSPACE = 4,    /* workspace missing or too small */
  FML_EDEVICE = 5        /* a kernel reported a device-side error (bounded wait expired) */
};

enum { FML_F32 = 0, FML_F16 = 1, FML_BF16 = 2 };
enum { FML_ACT_NONE = 0, FML_ACT_GELU_ERF = 1, FML_ACT_GELU_TANH = 2 };

/* Tile hints; mirrors forgeml.kernels.KernelConfig(block_m, block_n, block_k,
 * num_warps, num_stages) (src/forgeml/kernels.py:12-18).  block_n selects the
 * UMMA N tile (16..256), num_stages the shared-memory pipeline depth, and
 * block_k the K elements carried per pipeline stage (one, two or four 128-byte
 * slabs; 16-bit inputs only).  NULL
 * means "choose by heuristic".  block_m, block_k and num_warps are fixed by the
 * tcgen05 design (128-row UMMA tiles, 128-byte K slabs, 9 warps) and are only
 * range-checked. */
typedef struct fml_tile_cfg {
  int32_t block_m, block_n, block_k, num_warps, num_stages;
} fml_tile_cfg;

/* ---------------------------------------------------------------------------
 * GEMM with fused epilogue.
 * Replaces src/forgeml/_triton.py:6-62 (_matmul_kernel) and :65-93 (launch);
 * reached from src/forgeml/kernels.py:52-116 (matmul) and, for Nebula's
 * F.linear calls, src/nebula/runtime.py:131-133,145,152-153,186.
 *
 *   C[m,n] = act( r( r( sum_k A[m,k] B[k,n] ) + bias[n] ) )     (+ residual)
 *
 * r() rounds to the output dtype (bf16/fp16; identity for fp32), the same
 * double rounding as the Triton template (_triton.py:43,46).  When
 * `residual` is non-null the epilogue instead computes
 *   C = r( r(act(...)) + residual[m,n] )
 * which is Nebula's `x + F.linear(...)` in the reference dtype.
 * A[m,k] lives at a[m*lda_m + k*lda_k]; B[k,n] at b[k*ldb_k + n*ldb_n];
 * C is row-major with row stride ldc; residual has row stride ldr.
 * fp32 inputs run as 3xTF32 (split hi/lo, three tf32 products) to keep
 * IEEE-level accuracy; they need workspace.  16-bit operands whose layout a
 * TMA descriptor cannot address (unaligned strides, neither stride 1) are
 * packed into workspace first.
 * ------------------------------------------------------------------------- */
FML_API size_t fml_gemm_workspace_size(int64_t m, int64_t n, int64_t k, int dtype,
                               int64_t lda_m, int64_t lda_k, int64_t ldb_k,
                               int64_t ldb_n, const void* a, const void* b,
                               const fml_tile_cfg* cfg);

FML_API int fml_gemm(const void* a, int64_t lda_m, int64_t lda_k,
             const void* b, int64_t ldb_k, int64_t ldb_n,
             const void* bias, int64_t bias_stride,
             const void* residual, int64_t ldr,
             void* c, int64_t ldc,
             int64_t m, int64_t n, int64_t k,
             int dtype, int act, const fml_tile_cfg* cfg,
             void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * fp32 GEMM with a constant B split once.  fml_gemm splits both fp32
 * operands into their 3xTF32 images on every call; a compiled graph's
 * weights never change, so fml_gemm_pack_b writes B's image once
 * (fml_gemm_packed_b_bytes bytes at a 256-byte aligned dst; B[k,n] at
 * b[k*ldb_k + n*ldb_n] as in fml_gemm) and fml_gemm_packed_b then runs the
 * same product as fml_gemm on it, splitting only A (its workspace:
 * fml_gemm_packed_b_workspace_size).  Same results as fml_gemm.  fp32 only
 * (FML_EUNSUPPORTED otherwise).  An extension of the fml_gemm entry point
 * (the reference's launch, src/forgeml/_triton.py:65-93) for the compiled
 * dispatch of src/forgeml/compiler.py:93-126.
 * ------------------------------------------------------------------------- */
FML_API size_t fml_gemm_packed_b_bytes(int64_t n, int64_t k, int dtype);
FML_API int fml_gemm_pack_b(const void* b, int64_t ldb_k, int64_t ldb_n, int64_t k, int64_t n, int dtype,
                    void* dst, size_t dst_bytes, void* stream);
FML_API size_t fml_gemm_packed_b_workspace_size(int64_t m, int64_t n, int64_t k, int dtype, int64_t lda_m,
                                        int64_t lda_k, const void* a, const fml_tile_cfg* cfg);
FML_API int fml_gemm_packed_b(const void* a, int64_t lda_m, int64_t lda_k, const void* b_packed,
                      const void* bias, int64_t bias_stride, const void* residual, int64_t ldr,
                      void* c, int64_t ldc, int64_t m, int64_t n, int64_t k,
                      int dtype, int act, const fml_tile_cfg* cfg,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Allocation-free GEMM.  This entry point has no counterpart in the
 * reference; it exists for callers that cannot allocate device memory at the
 * call site -- for example a host runtime that reserves the GPU's memory up
 * front through its own allocator and forbids any further cudaMalloc, or a
 * latency-critical caller that must not go through cudaMalloc/cudaFree,
 * which can synchronise the device.  Same arguments and results as fml_gemm,
 * minus the workspace: the operand packing that fml_gemm stages in a caller
 * workspace (the fp32 3xTF32 split, 16-bit operands TMA cannot address) goes
 * to a scratch array of FML_GEMM_NOALLOC_SCRATCH_BYTES that the library
 * keeps in device memory (every GPU that loads the library holds it until
 * the process exits).  Problems whose packing needs more than that return
 * FML_EWORKSPACE without launching.  The first call on a device looks up the
 * scratch address (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture.  The address is kept for the life of
 * the process: after cudaDeviceReset on a device, do not call this entry point
 * on that device again in the same process.  All calls share the one array:
 * calls whose executions overlap on the GPU (different streams, or other
 * host threads) race on it, so serialise them.  Everything the kernels read
 * from the scratch is written earlier in the same call, so the contents left
 * by a previous call never matter.  Nothing is allocated: no cudaMalloc,
 * cudaFree or allocating library routine is called.
 * ------------------------------------------------------------------------- */
#define FML_GEMM_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
FML_API int fml_gemm_noalloc(const void* a, int64_t lda_m, int64_t lda_k,
                             const void* b, int64_t ldb_k, int64_t ldb_n,
                             const void* bias, int64_t bias_stride,
                             const void* residual, int64_t ldr,
                             void* c, int64_t ldc,
                             int64_t m, int64_t n, int64_t k,
                             int dtype, int act, const fml_tile_cfg* cfg, void* stream);

/* ---------------------------------------------------------------------------
 * Constant-weight linear layer, y = x W^T (+ bias) (-> GELU) (+ residual),
 * with the same epilogue contract as fml_gemm.  Replaces Nebula's
 * F.linear(h, W) for the per-layer weights (src/nebula/runtime.py:131-133,
 * 145,152-153,186), whose W is fixed for the engine's lifetime.
 * fml_pack_weight rewrites W [N, K] (row stride ldw, K contiguous, 16-bit)
 * once into 16 KB tiles of 128 rows x 128 bytes of K, each already in the
 * swizzled shared-memory layout the tensor cores read, so a decode-step GEMM
 * streams the weight as sequential bulk copies.  The packed buffer
 * (fml_packed_weight_bytes bytes) must be 1024-byte aligned.  x is row-major
 * [M, K] with row stride ldx (16-byte aligned rows).
 * ------------------------------------------------------------------------- */
FML_API size_t fml_packed_weight_bytes(int64_t n, int64_t k, int dtype);
FML_API int fml_pack_weight(const void* w, int64_t ldw, int64_t n, int64_t k, int dtype,
                            void* packed, void* stream);
FML_API int fml_linear_packed(const void* x, int64_t ldx, const void* packed, int64_t n,
                              int64_t k, const void* bias, int64_t bias_stride,
                              const void* residual, int64_t ldr, void* out, int64_t ldo,
                              int64_t m, int dtype, int act, const fml_tile_cfg* cfg,
                              void* stream);

/* ---------------------------------------------------------------------------
 * LayerNorm over the trailing `cols` elements of each of `rows` rows.
 * Replaces the F.layer_norm evaluation of src/forgeml/ops.py:54-60 and
 * src/nebula/runtime.py:130,151,185.  gamma/beta may both be null (no affine).
 * Statistics in fp32; y rounded once to dtype.
 * ------------------------------------------------------------------------- */
FML_API int fml_layernorm(const void* x, int64_t x_row_stride, const void* gamma,
                  const void* beta, float eps, void* y, int64_t y_row_stride,
                  int64_t rows, int64_t cols, int dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Rank-4 scaled dot-product attention, out = softmax(q k^T * scale + mask) v.
 * Replaces F.scaled_dot_product_attention in src/forgeml/ops.py:61-70.
 * q is [B,H,Sq,D], k/v are [B,H,Sk,D], out is [B,H,Sq,D]; each has its own
 * 4 element strides (innermost stride must be 1).  `mask` (optional) is
 * broadcast to [B,H,Sq,Sk] through mask_strides (0 for broadcast dims);
 * mask_kind 0 = none, 1 = bool (nonzero keeps), 2 = additive in dtype.
 * is_causal keeps key j for query i when j <= i (top-left aligned, as torch).
 * D <= 256.  Softmax in fp32.
 * ------------------------------------------------------------------------- */
FML_API int fml_sdpa(const void* q, const int64_t q_strides[4],
             const void* k, const int64_t k_strides[4],
             const void* v, const int64_t v_strides[4],
             const void* mask, const int64_t mask_strides[4], int mask_kind,
             int is_causal, float scale,
             void* out, const int64_t out_strides[4],
             int64_t batch, int64_t heads, int64_t sq, int64_t sk, int64_t d,
             int dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Nebula attention over the contiguous per-request KV cache.
 * Replaces src/nebula/runtime.py:139-144 together with the prefix
 * torch.stack in src/nebula/cache.py:163-165 (no copy of the cache is made).
 * The cache of one layer is a pool [slots, H, max_seq, D]; request b uses pool
 * slot slot_of[b] (int32, device).  Query b,t sits at absolute position
 * start_pos[b] + t (int32, device) and attends keys 0..start_pos[b]+t.
 * q is [B,T,H,D] with element strides q_strides (innermost 1); out is
 * [B,T,H,D] contiguous rows of H*D.  Scores and softmax in fp32.  The pools
 * hold pool_slots slots.  Steps of more than one token per request (prefill)
 * with 16-bit data and head dim 64 or 128 run on the tensor cores (scores
 * and P V by tcgen05, P rounded to the model dtype as in the reference's
 * attn.to(x.dtype)); single-token steps stream the keys on CUDA cores.
 * ------------------------------------------------------------------------- */
FML_API int neb_attention(const void* q, const int64_t q_strides[4],
                  const void* k_pool, const void* v_pool,
                  const int32_t* slot_of, const int32_t* start_pos,
                  void* out, int64_t batch, int64_t t, int64_t heads,
                  int64_t head_dim, int64_t max_seq, int64_t pool_slots, float scale,
                  int dtype, void* stream);

/* ---------------------------------------------------------------------------
 * KV-cache append: pool[slot_of[b], h, start_pos[b]+t, :] = kv[b,t,h,:] for
 * both K and V.  Replaces the copy_ in src/nebula/cache.py:158-162.  k/v are
 * [B,T,H,D] with element strides (innermost 1), e.g. column views of the QKV
 * GEMM output.  Bit-exact copy.
 * ------------------------------------------------------------------------- */
FML_API int neb_kv_append(const void* k, const int64_t k_strides[4],
                  const void* v, const int64_t v_strides[4],
                  void* k_pool, void* v_pool,
                  const int32_t* slot_of, const int32_t* start_pos,
                  int64_t batch, int64_t t, int64_t heads, int64_t head_dim,
                  int64_t max_seq, int dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Token + learned position embedding:
 *   x[b,t,:] = r( tok_emb[tokens[b,t],:] + pos_emb[start_pos[b]+t,:] )
 * Replaces src/nebula/runtime.py:166-169.  tokens int64 [B,T] contiguous,
 * start_pos int32 [B] (device).  Ids outside [0,vocab) raise the device error
 * flag and write zeros.
 * ------------------------------------------------------------------------- */
FML_API int neb_embed(const int64_t* tokens, const int32_t* start_pos,
              const void* tok_emb, const void* pos_emb, void* x,
              int64_t batch, int64_t t, int64_t hidden, int64_t vocab,
              int64_t max_seq, int dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Greedy sampling: out[b] = argmax_j logits[b*row_stride + j], first index
 * on ties (torch.argmax semantics, src/nebula/runtime.py:477,485).
 * ------------------------------------------------------------------------- */
FML_API int neb_argmax(const void* logits, int64_t row_stride, int64_t rows,
               int64_t cols, int64_t* out, int dtype, void* stream);

/* Elementwise y = r(a + b) on contiguous buffers (Nebula residual add after
 * a tensor-parallel all-reduce, src/nebula/runtime.py:177,179). */
FML_API int neb_add(const void* a, const void* b, void* y, int64_t n, int dtype,
            void* stream);

/* ---------------------------------------------------------------------------
 * Tensor-parallel SUM all-reduce over NVLink peer memory, fused with the
 * residual add.  Replaces ParallelContext.all_reduce
 * (src/nebula/parallel.py:112-116) followed by `x = x + part`
 * (src/nebula/runtime.py:146,154):  out = round(round(sum_r part_r) + residual)
 * with the sum taken in rank order (bit-identical on every rank).  Each rank
 * creates a context (a symmetric buffer of 2 x world slots of max_bytes),
 * exchanges the IPC handles with its TP group, opens the peers' buffers, then
 * every rank calls neb_ar_all_reduce with the same sizes in the same order
 * (stream-ordered, CUDA-graph capturable).  A wait that exceeds timeout_ms
 * raises bit 32 of fml_device_status() instead of hanging.  Protocol: each
 * 4-byte word travels with the call's epoch in one 8-byte store and readers
 * poll the words (low latency), either one-shot (every rank pushes its whole
 * partial to every peer) or two-shot (reduce-scatter to sub-shard owners,
 * then all-gather of the sums); see neb_ar_set_protocol.
 * ------------------------------------------------------------------------- */
/* Bytes of one IPC handle (cudaIpcMemHandle_t). */
FML_API int64_t neb_ar_handle_bytes(void);
FML_API int neb_ar_create(int64_t max_bytes, int world, int rank, double timeout_ms, void** ctx_out,
                          void* handle_out);
/* handles: world consecutive handles in rank order (this rank's is ignored). */
FML_API int neb_ar_open(void* ctx, const void* handles);
/* Single-process alternative to neb_ar_open: device pointers of every rank's
 * buffer (neb_ar_buffer of the other contexts); this rank's entry ignored. */
FML_API int neb_ar_set_peers(void* ctx, void* const* bases);
FML_API void* neb_ar_buffer(void* ctx);
/* Protocol of this context's standalone all-reduce: 0 = the library's
 * choice (one-shot), 1 = one-shot LL, 2 = two-shot LL.  Every rank of a
 * group must use the same protocol.  No reference counterpart (NCCL chose
 * its own algorithm there). */
FML_API int neb_ar_set_protocol(void* ctx, int protocol);
/* n elements of dtype; residual may be NULL (then out = round(sum)); 16-byte
 * aligned pointers, n * sizeof(dtype) a multiple of 16 and <= max_bytes. */
FML_API int neb_ar_all_reduce(void* ctx, const void* part, const void* residual, void* out, int64_t n,
                              int dtype, void* stream);
FML_API int neb_ar_destroy(void* ctx);

/* ---------------------------------------------------------------------------
 * Fused decode linear: one launch for each of the decode step's chains
 *   LN -> QKV linear -> KV append        (src/nebula/runtime.py:130-138, cache.py:161-165)
 *   o linear -> SUM all-reduce -> + x    (runtime.py:145-146, parallel.py:112-116)
 *   LN -> up linear -> GELU              (runtime.py:151-152)
 *   down linear -> SUM all-reduce -> + x (runtime.py:153-154)
 * on a packed weight (fml_pack_weight), for M <= 32 tokens.  Same results as
 * the unfused chain (fml_layernorm, fml_linear_packed, neb_kv_append,
 * neb_ar_all_reduce) up to the LayerNorm statistics, which are summed in a
 * different order.
 *   LayerNorm prologue (ln_gamma != NULL): the GEMM reads LN(x) over x's k
 *     columns (eps ln_eps, ln_beta required); k a multiple of 64.
 *   LayerNorm fold (ln_wsum != NULL, ln_gamma NULL): the packed weight is
 *     W diag(gamma); the GEMM reads x itself and returns
 *     rstd * (x W'^T - mean * ln_wsum[n]) + ln_wbias[n]  (= LN(x) W^T with
 *     ln_wsum[n] = sum_k W'[n][k], ln_wbias[n] = sum_k W[n][k] beta[k], fp32
 *     vectors of n; ln_wbias may be NULL), the row statistics computed while
 *     the product runs; k a multiple of 64.
 *   KV epilogue (k_pool != NULL): output features [0, q_cols) go to out (row
 *     stride ldo >= q_cols); features q_cols + [0, kv_heads*head_dim) go to
 *     K and the next kv_heads*head_dim to V, at pool[slot_of[b], head,
 *     start_pos[b] + t, d] for token m = b*tq + t (pools [slots, kv_heads,
 *     max_seq, head_dim]); an out-of-range position raises bit 4 of
 *     fml_device_status() like neb_kv_append.  n = q_cols + 2*kv_heads*head_dim.
 *   All-reduce epilogue (ar_ctx != NULL, a neb_ar context opened on every TP
 *     rank): out = round(round(sum over ranks in rank order) + residual),
 *     exchanged in 16-feature sub-blocks over NVLink from the GEMM epilogue;
 *     every rank calls with the same n and m in the same order; n a multiple
 *     of 16 with n * 64 <= the context's max_bytes; act must be 0; not
 *     combined with the KV epilogue.  A peer wait beyond the context's timeout
 *     raises bit 32 of fml_device_status().
 * ------------------------------------------------------------------------- */
typedef struct neb_fusion {
  const void* ln_gamma;
  const void* ln_beta;
  float ln_eps;
  const float* ln_wsum;
  const float* ln_wbias;
  void* k_pool;
  void* v_pool;
  const int32_t* slot_of;
  const int32_t* start_pos;
  int32_t q_cols, kv_heads, head_dim, max_seq, tq;
  void* ar_ctx;
} neb_fusion;

FML_API int neb_linear_fused(const void* x, int64_t ldx, const void* packed, int64_t n, int64_t k,
                             const void* residual, int64_t ldr, void* out, int64_t ldo, int64_t m,
                             int dtype, int act, const neb_fusion* fusion, void* stream);
/* 1 if neb_linear_fused covers an [m x k] x [n x k]^T product on this device
 * (16-bit, m <= 32, every output tile resident at once), else 0. */
FML_API int neb_linear_fused_ok(int64_t n, int64_t k, int64_t m, int dtype);

/* ---------------------------------------------------------------------------
 * Diagnostics.
 * ------------------------------------------------------------------------- */
/* Message for the last nonzero return on this thread ("" if none). */
FML_API const char* fml_last_error(void);
/* Reads and clears the device-side error word of the current device
 * (bounded waits that expired, out-of-range token ids).  0 = clean.
 * Bits: 1 GEMM pipeline wait expired, 2 token id out of range, 4 attention
 * position/slot out of range, 8 split-K cluster reduce wait expired,
 * 16 attention copy-pipeline wait expired, 32 all-reduce peer wait expired.
 * Synchronizes the current device. */
FML_API int fml_device_status(void);
/* Stream-ordered copy of the device error word (same bits) into host memory
 * `host_dst` (4 bytes; pinned for the copy to stay asynchronous) once the
 * work queued on `stream` before it has run.  Does not clear the word and
 * does not synchronise: the caller reads *host_dst after the stream (or an
 * event recorded after this call) has completed.  A serving engine checks
 * every step this way without a host wait (Nebula's poisoning contract,
 * src/nebula/runtime.py:299-301,361-363: an engine whose step failed on the
 * device raises EngineFailed and drops its cache). */
FML_API int fml_device_status_async(int32_t* host_dst, void* stream);
/* Number of kernel launches issued by this library in this process. */
FML_API int64_t fml_launch_count(void);
/* Library version string. */
FML_API const char* fml_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FORGEML_B200_H */
