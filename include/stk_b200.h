/*
 * stk_b200.h -- C ABI of the B200 (sm_100a) streaming top-k SAE encoder.
 *
 *   scores = X @ W_enc^T + b_enc        (B, F), never written to memory
 *   V, I   = top_k(scores, k)           V fp32 (B, k) descending, I int32 (B, k)
 *
 * Plain pointers and sizes only; every pointer argument is device memory on
 * the current CUDA device unless stated otherwise; `stream` is a cudaStream_t
 * (NULL = legacy default stream).  All calls are asynchronous on `stream` and
 * allocate nothing: scratch memory is caller-provided (`workspace`, sized by
 * stk_workspace_bytes).
 *
 * Return value: STK_OK (0) or an STK_E* code; stk_last_error() gives the
 * message of the last failing call on the calling thread.  Argument messages
 * repeat the reference's TORCH_CHECK texts.
 *
 * Ties: among equal scores the smaller feature index ranks first, so results
 * do not depend on how F is tiled, on the number of CTAs or on the number of
 * GPUs.
 */
#ifndef STK_B200_H
#define STK_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define STK_API __attribute__((visibility("default")))
#else
#define STK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum stk_status {
  STK_OK = 0,
  STK_EINVAL = 1,   /* bad argument (message in stk_last_error) */
  STK_ECUDA = 2,    /* CUDA runtime / driver error */
  STK_EDEVICE = 3,  /* a kernel reported a device-side error (bounded wait ran out) */
  STK_ENOSPACE = 4  /* workspace too small */
};

/* Element types.  STK_E4M3 (one byte: FP8 E4M3, bias 7, max 448) is only
 * W_enc's type in the stk_*_fp8 calls; X is then fp32, fp16 or bf16. */
enum stk_dtype { STK_F32 = 0, STK_F16 = 1, STK_BF16 = 2, STK_E4M3 = 3 };

/* Flags for the *_forward calls. */
enum stk_flags {
  STK_FLAG_ANY_K = 1, /* accept any 1 <= k <= 128, not only {1,2,4,8,16,32,64,128}; and any
                         k <= F when F <= 4096 (whole-row sort, no workspace) */
  STK_FLAG_ANY_D = 2, /* lift the reference's d <= 4096 limit */
  STK_FLAG_SIMT = 4,    /* force the fp32-FMA SIMT kernel (testing / comparison, or bit-faithful fp32) */
  STK_FLAG_NO_PILOT = 8, /* skip the sampled threshold floor (testing / comparison) */
  STK_FLAG_TF32 = 16,    /* fp32 inputs on tensor cores (3-pass TF32) also for d > 2048 (the default up to
                            d = 2048, d % 4 == 0); otherwise fp32 uses the SIMT kernel */
  STK_FLAG_SEPARATE_FINISH = 32, /* finish the rows in a second kernel even where the score kernel
                                    could do it in its tail (testing / comparison) */
  STK_FLAG_NO_PAIR = 64 /* no CTA pairs (tcgen05 cta_group::2, used for k > 64 with several 128-row
                           M tiles per call) (testing / comparison) */
};

/* Library version (major * 10000 + minor * 100 + patch). */
STK_API int stk_version(void);

/* Message of the last failing call on this thread ("" if none). */
STK_API const char* stk_last_error(void);

/* Length L of the per-row key lists used for a given k (32, 64 or 128; 0 if k > 128). */
STK_API int stk_list_len(int64_t k);

/*
 * Bytes of device workspace stk_exact_forward / stk_approx_forward /
 * stk_shard_forward need for this shape on the current device.
 */
STK_API int stk_workspace_bytes(int64_t B, int64_t d, int64_t F, int64_t k, int dtype, size_t* bytes);

/*
 * Exact streaming top-k encode.
 * Replaces streamtopk_cuda_exact_forward(X, W_enc, b_enc, k)
 *   (reference: streamtopk_sae/csrc/cuda/streamtopk_exact.cu:788-833, bound in
 *    streamtopk_sae/csrc/bindings.cpp:33-34 and called from
 *    streamtopk_sae/ops.py:43-57).
 * X (B, d) and W (F, d) row-major in `dtype`; b (F,) fp32; V (B, k) fp32 and
 * I (B, k) int32 outputs, each row descending.
 */
STK_API int stk_exact_forward(const void* X, const void* W, const float* b, float* V, int32_t* I, int64_t B, int64_t d,
                      int64_t F, int64_t k, int dtype, int flags, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * Pipelined exact encode for loops that encode batch after batch of one shape
 * (serving, activation sweeps): each batch gets exactly stk_exact_forward's
 * result for its inputs (same op, reference streamtopk_exact.cu:788-833; the
 * pipelining has no counterpart there).  One launch per batch: the score
 * kernel of batch s also finishes batch s - 1 (while its first W_enc tile
 * streams in), so a batch's V / I are complete, in stream order, once the next
 * batch has been submitted or after stk_pipeline_flush.  Read a batch's
 * results only after that point.
 * The pipeline keeps its per-batch lists in a workspace of
 * stk_pipeline_workspace_bytes (two halves, used by alternate batches); the
 * caller allocates it and keeps it for the pipeline's lifetime.  Submit and
 * flush on one stream (or order the streams), from one host thread at a time
 * (a pipeline holds host state: the pending batch).  stk_pipeline_destroy
 * does not finish a pending batch: flush first, or its V / I stay unwritten.  Shapes that do not pipeline
 * (k > 64, several rounds of units per CTA, unaligned operands:
 * stk_pipeline_pipelined() == 0) run each batch as stk_exact_forward
 * (complete at once).  X, W, b, V, I per batch as in stk_exact_forward;
 * k <= 128; B >= 1.
 */
typedef struct stk_pipeline stk_pipeline;
STK_API int stk_pipeline_workspace_bytes(int64_t B, int64_t d, int64_t F, int64_t k, int dtype, int flags,
                                         size_t* bytes);
STK_API int stk_pipeline_create(stk_pipeline** out, int64_t B, int64_t d, int64_t F, int64_t k, int dtype, int flags,
                                void* workspace, size_t workspace_bytes);
STK_API int stk_pipeline_submit(stk_pipeline* p, const void* X, const void* W, const float* b, float* V, int32_t* I,
                                void* stream);
STK_API int stk_pipeline_flush(stk_pipeline* p, void* stream);
STK_API int stk_pipeline_pipelined(const stk_pipeline* p);
STK_API int stk_pipeline_destroy(stk_pipeline* p);

/*
 * Approximate (per-128-feature-tile top-c candidates) encode, final top-k
 * included.  Replaces streamtopk_cuda_approx_forward + the torch.topk/gather
 * that follows it (reference: streamtopk_sae/csrc/cuda/streamtopk_approx.cu:
 * 234-291 and streamtopk_sae/ops.py:60-83).  c must be in {16,32,64,128} and
 * k <= c, as in the reference.  For k <= c the tile filter keeps every
 * feature of the global top-k (a top-k feature ranks <= k <= c inside its
 * tile), so the result equals stk_exact_forward's.
 */
STK_API int stk_approx_forward(const void* X, const void* W, const float* b, float* V, int32_t* I, int64_t B, int64_t d,
                       int64_t F, int64_t k, int64_t c, int dtype, int flags, void* workspace,
                       size_t workspace_bytes, void* stream);

/*
 * Per-tile candidates of the approximate path: for every row and every
 * 128-feature tile t, the tile's best c scores, descending, padded with
 * (-FLT_MAX, -1) where the tile holds fewer than c features.
 * cand_vals / cand_idxs: (B, ceil(F/128), c).  Replaces the candidate buffer
 * written by streamtopk_approx_kernel (streamtopk_approx.cu:42-167, returned
 * by streamtopk_cuda_approx_forward at :286-290).  c in {16,32,64,128}.
 * Workspace sized by stk_candidates_workspace_bytes.
 */
STK_API int stk_approx_candidates(const void* X, const void* W, const float* b, float* cand_vals, int32_t* cand_idxs,
                                  int64_t B, int64_t d, int64_t F, int64_t c, int dtype, void* workspace,
                                  size_t workspace_bytes, void* stream);
STK_API int stk_candidates_workspace_bytes(int64_t B, int64_t d, int64_t F, int64_t c, int dtype, size_t* bytes);

/*
 * The approximate op with its candidate buffer (reference: ops.py:60-83 with
 * candidate_buffer, streamtopk_approx.cu:234-291): the final (B, k) result V/I
 * and each 128-feature tile's top c per row, cand_vals / cand_idxs (B,
 * ceil(F/128), c) descending, (-FLT_MAX, -1) past a tile's last feature.  For
 * fp16 / bf16 inputs with c <= 32 one W_enc pass computes both (the fused
 * kernel's candidate variant); otherwise the candidates pass and the exact
 * top-k run one after the other.  Buffers 16-byte aligned; workspace from
 * stk_approx_cand_workspace_bytes (enough for either way).
 */
STK_API int stk_approx_cand_workspace_bytes(int64_t B, int64_t d, int64_t F, int64_t k, int64_t c, int dtype,
                                            size_t* bytes);
STK_API int stk_approx_forward_cand(const void* X, const void* W, const float* b, float* V, int32_t* I,
                                    float* cand_vals, int32_t* cand_idxs, int64_t B, int64_t d, int64_t F, int64_t k,
                                    int64_t c, int dtype, int flags, void* workspace, size_t workspace_bytes,
                                    void* stream);

/*
 * One F-shard of a multi-GPU encode: per row of this shard, with feature
 * indices offset by `index_offset`, sorted 64-bit keys in keys_out (B, L),
 * L = stk_list_len(k): the shard's exact top k, then further keys of the
 * shard in descending order (not necessarily the next best), then empty keys
 * (0).  Key = (order-preserving bits of the fp32 score << 32) | ~feature.
 * keys_out must be 16-byte aligned.  Keys from several shards are
 * combined by stk_merge_keys.  (No reference counterpart: the reference has no
 * multi-GPU path.)
 */
STK_API int stk_shard_forward(const void* X, const void* W_shard, const float* b_shard, uint64_t* keys_out, int64_t B,
                      int64_t d, int64_t F_shard, int64_t k, int64_t index_offset, int dtype, int flags,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * Final merge of n key lists per row: lists (n, B, L) as written by
 * stk_shard_forward (e.g. after an all-gather), L = stk_list_len(k).
 * Writes V (B, k) fp32 and I (B, k) int32.  lists must be 16-byte aligned.
 * Replaces the reference's merge pass (streamtopk_exact.cu:429-499) for the
 * cross-GPU step.
 */
STK_API int stk_merge_keys(const uint64_t* lists, int64_t nlists, int64_t B, int64_t k, float* V, int32_t* I,
                   void* stream);

/*
 * Synchronise `stream`, then read and clear the device error word of the
 * current device.  *code = 0 if no kernel reported an error.
 */
STK_API int stk_device_error(void* stream, unsigned* code);

/*
 * Exact encode that allocates nothing and takes no workspace (no counterpart in
 * the reference).  For callers that cannot allocate device memory (allocator
 * hooks, plugins whose host owns all allocations, fixed-memory embedded or
 * real-time code).  Same arguments and results as stk_exact_forward, minus the
 * workspace: scratch comes from a 24 MiB array built into the library, which
 * every GPU that loads the library holds until the process exits.  Shapes that
 * need more scratch (more than one 128-row M tile, or k > 64 at large F) return
 * STK_ENOSPACE.  The first call on a device looks up the array's device address
 * (make it before any stream capture).  All calls share the array: calls that
 * overlap on the GPU race and must be serialised by the caller.
 */
STK_API int stk_exact_forward_noalloc(const void* X, const void* W, const float* b, float* V, int32_t* I, int64_t B,
                                      int64_t d, int64_t F, int64_t k, int dtype, int flags, void* stream);

/*
 * FP8 W_enc streaming (no counterpart in the reference, whose dtype set is
 * fp32 / fp16 / bf16, streamtopk_exact.cu:803-804): W_enc is (F, d) E4M3 with
 * one fp32 dequantization scale per feature (w[f][j] ~= w_scale[f] * W8[f][j],
 * e.g. from stk_quantize_rows_fp8), half the HBM bytes of bf16.  X (B, d) in
 * x_dtype (fp32 / fp16 / bf16) is quantized per row to E4M3 by the library
 * into the workspace (x_scale[r] = max_j |x[r][j]| / 448), and the tensor cores
 * run kind::f8f6f4 with fp32 accumulation:
 *     score[r][f] = x_scale[r] * w_scale[f] * sum_j X8[r][j] * W8[f][j] + b[f]
 * and V / I are the exact top-k of these scores (keys as in stk_exact_forward).
 * Lossy against the unquantized scores: a different operator, not a drop-in
 * for the reference's.  Needs d % 16 == 0 and 16-byte aligned X and W8; k as
 * in stk_exact_forward up to 128.
 */
STK_API int stk_workspace_bytes_fp8(int64_t B, int64_t d, int64_t F, int64_t k, size_t* bytes);
STK_API int stk_exact_forward_fp8(const void* X, int x_dtype, const void* W8, const float* w_scale, const float* b,
                                  float* V, int32_t* I, int64_t B, int64_t d, int64_t F, int64_t k, int flags,
                                  void* workspace, size_t workspace_bytes, void* stream);
/* Per-row E4M3 quantization of a (rows, d) matrix in x_dtype (d % 16 == 0):
 * scale[r] = max_j |x[r][j]| / 448 (1 for an all-zero row), Q[r][j] =
 * E4M3(x[r][j] * 448 / max_j |x[r][j]|), round to nearest even, saturating.
 * The quantization the fp8 encode applies to X; also makes W8 / w_scale. */
STK_API int stk_quantize_rows_fp8(const void* X, int x_dtype, void* Q, float* scale, int64_t rows, int64_t d,
                                  void* stream);

/*
 * SAE decoder over the encoder's output (no counterpart in the reference,
 * which stops at the encoder, README.md:9-14; the next step of an SAE forward):
 *     out[b][:] = b_dec[:] + sum_j V[b][j] * W_dec[I[b][j]][:]
 * V (B, k) fp32 and I (B, k) int32 as stk_exact_forward returns them (entries
 * with I < 0 or I >= F are skipped), W_dec (F, d) in dtype, b_dec (d,) fp32 or
 * NULL, out (B, d) fp32.  A gather-GEMM: B * k rows of W_dec read once each
 * (fp32 accumulation), never the dense (B, F) codes.  1 <= k <= 1024; d % 8 == 0
 * for fp16 / bf16 W_dec (d % 4 for fp32); W_dec, b_dec, out 16-byte aligned.
 */
STK_API int stk_decode_forward(const float* V, const int32_t* I, const void* W_dec, const float* b_dec, float* out,
                               int64_t B, int64_t k, int64_t F, int64_t d, int dtype, void* stream);

/*
 * Direct GPU-to-GPU exchange for the F-sharded encode (no counterpart in the
 * reference, which is single-GPU; the F-sharding follows the multi-GPU scheme
 * of the hot path: shard W_enc / b_enc along F, exchange each rank's per-row
 * top-L key lists, merge).  One process per GPU, all GPUs on one node with
 * peer access (NVLink); at most 8 ranks.  Replaces the all-gather + merge of
 * stk_shard_forward / stk_merge_keys with peer stores: each rank writes its
 * rows' best keys straight into every rank's receive buffer and sets a per-row
 * flag there to the step number; each rank waits for all ranks' rows (bounded
 * by wait_seconds) and finishes them.  All of this runs in the tail of the
 * score kernel when its units are all resident at once (one launch per step),
 * else in one finish kernel after it.  A wait that runs out reports device
 * error 3 through stk_device_error; that step's rows are then finished over
 * the ranks whose rows had arrived.  Steps are tagged with their absolute
 * number, so rows that arrive late are never taken for a later step's rows
 * (a rank that skipped a step entirely leaves the ranks one step apart, and
 * every later step times out until the exchange is re-created).
 *
 * Setup (collective: every rank, same world / max_rows / k):
 *   stk_exchange_bytes -> allocate a 256-byte aligned device buffer of that size
 *     (plain cudaMalloc-backed memory: cudaIpcGetMemHandle must accept it)
 *   stk_exchange_create (clears its flags, synchronously)
 *   stk_exchange_ipc_handle -> share the STK_IPC_HANDLE_BYTES handle + offset
 *     with every rank (any host transport)
 *   stk_exchange_connect with all ranks' handles / offsets (rank order)
 * Each encode (collective, same B on every rank, calls in the same order):
 *   stk_exchange_forward -> V (B, k) fp32, I (B, k) int32 over the global F.
 * The step counter lives on the device, so forwards can be captured in a CUDA
 * graph and replayed.  Teardown: make sure no rank has a forward in flight
 * (synchronise + a host barrier), stk_exchange_destroy on every rank, a host
 * barrier, then free the buffers.  The handle object is a small host struct.
 */
#define STK_IPC_HANDLE_BYTES 64
typedef struct stk_exchange stk_exchange;
STK_API int stk_exchange_bytes(int world, int64_t max_rows, int64_t k, size_t* bytes);
STK_API int stk_exchange_create(int rank, int world, int64_t max_rows, int64_t k, void* buffer, size_t bytes,
                                double wait_seconds, stk_exchange** out);
STK_API int stk_exchange_ipc_handle(const stk_exchange* ex, void* handle /* STK_IPC_HANDLE_BYTES */,
                                    int64_t* offset);
STK_API int stk_exchange_connect(stk_exchange* ex, const void* handles /* world x STK_IPC_HANDLE_BYTES */,
                                 const int64_t* offsets /* world */);
STK_API int stk_exchange_forward(stk_exchange* ex, const void* X, const void* W_shard, const float* b_shard, float* V,
                                 int32_t* I, int64_t B, int64_t d, int64_t F_shard, int64_t k, int64_t index_offset,
                                 int dtype, int flags, void* workspace, size_t workspace_bytes, void* stream);
STK_API int stk_exchange_destroy(stk_exchange* ex);

/*
 * The pipelined encode (stk_pipeline_*, above) for one rank of the F-sharded encode over a connected
 * peer exchange (stk_exchange_*): W / b are this rank's rows [index_offset,
 * index_offset + F_shard) and each batch's V / I are the global top-k,
 * identical on every rank (as stk_exchange_forward).  Every rank submits and
 * flushes the same batches in the same order; the cross-GPU publish, wait and
 * merge of batch s run in the score kernel of batch s + 1 (or the flush).
 * The exchange must outlive the pipeline.
 */
STK_API int stk_pipeline_create_sharded(stk_pipeline** out, stk_exchange* ex, int64_t B, int64_t d, int64_t F_shard,
                                        int64_t k, int64_t index_offset, int dtype, int flags, void* workspace,
                                        size_t workspace_bytes);

/*
 * Profiling hook (no reference counterpart).  stk_profile_begin arms CUDA
 * events around each kernel launched by the calls that follow (up to
 * max_launches launches, any thread); stk_profile_end synchronises them and
 * returns, per kernel kind (0 fused tcgen05 score kernel, its finish step
 * included when it runs in the kernel's tail; 1 SIMT score kernel; 2 standalone
 * finish kernel; 3 standalone finish kernel with the exchange), the summed
 * device time in ms and the number of launches.  No work is skipped or reordered.
 */
STK_API int stk_profile_begin(int64_t max_launches);
STK_API int stk_profile_end(double* ms_by_kind /* [4] */, int64_t* launches_by_kind /* [4] */);

#ifdef __cplusplus
}
#endif

#endif /* STK_B200_H */
