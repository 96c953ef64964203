// Shared declarations of the encoder kernels: tile configurations, shared-
// memory layouts, launch parameters and the launch helpers defined in
// stk_kernels.cu.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "stk_device.cuh"

namespace stk {

constexpr int kEpilogueWarps = 4;
constexpr int kFusedThreads = 64 + 32 * kEpilogueWarps;  // producer, MMA, 4 epilogue warps
constexpr int kSimtThreads = 256;

// Units of work (see stk_kernels.cu header comment).
struct UnitGrid {
  int m_tiles;      // ceil(B / 128)
  int segs;         // feature ranges
  int units;        // m_tiles * segs
  int64_t nchunks;  // ceil(F / 32)
  int fixed_chunks; // > 0: range s is chunks [s*fixed_chunks, (s+1)*fixed_chunks); 0: balanced split
  int quantum;      // balanced split: range bounds are multiples of quantum chunks (1, or 4 = 128 features)
};

// Per-CTA global append buffers (configurations whose append slots do not fit
// in shared memory): [gridDim.x][kAppendMax][kRows] keys in the workspace.
constexpr size_t kAppendBytesPerCta = (size_t)kAppendMax * kRows * 8;

// Pilot threshold: every CTA takes the scores of its first kPilotChunks * 32
// features per row, histograms the maximum of each group of kPilotGroup of
// them (bins = top kPilotBits of the order-preserving key), the CTAs meet at
// a bounded grid barrier, and each row starts with the lower edge of the bin
// that holds its k-th largest histogrammed score as filter floor.
constexpr int kPilotBits = 12;
constexpr int kPilotChunks = 2;  // default sampled 32-feature chunks per CTA
constexpr int kPilotGroup = 16;  // scores per histogrammed group maximum (8: 2-4 % slower at cfg2 / one N = 8
                                 // shard -- twice the global atomics for about the same bound)
constexpr int kPilotBins = 1 << kPilotBits;
constexpr uint32_t kPilotTopSlack = 8;  // bins (one octave) the bound's window reaches above a CTA's own top
constexpr unsigned long long kPilotWaitNs = 200000;  // give up (no floor) after 200 us

// Direct GPU-to-GPU exchange of per-rank key lists (F-sharded encode, one
// process per GPU on one node).  Each rank owns one exchange buffer:
//   recv  [2][world][max_rows][L] keys   (slot = step & 1)
//   flag  [2][world][max_rows] u64        (step + 1 once rank p's row arrived)
//   state [2] u64: step counter, CTAs done with the current step
// peer_recv / peer_flag[p] are rank p's recv / flag mapped into this process
// (CUDA IPC); entry `rank` is the local buffer.
constexpr int kMaxWorld = 8;
struct ExchangeDev {
  uint64_t* peer_recv[kMaxWorld];
  unsigned long long* peer_flag[kMaxWorld];
  uint64_t* recv;
  unsigned long long* flag;
  unsigned long long* state;
  int rank, world;
  int64_t max_rows;
  unsigned long long wait_ns;
};
constexpr unsigned kErrExchangeTimeout = 3;
constexpr unsigned kErrFinishBarrier = 4;  // the fused kernel's CTAs did not all reach the finish step in time

// Finish step (stk_finish.cuh): per-row top-k over the units' sorted lists
// (list s of row b at lists[(s * stride + b) * L]), results to V/I and/or
// keys_out, optionally through the exchange.
struct FinishArgs {
  const uint64_t* lists;  // list s of row b at lists[(s * stride + b) * pitch]: L sorted keys, then
  int nlists;             // `tail` more sorted keys (a second run; 0 or kAppendMax)
  int64_t stride;
  int pitch;
  int tail;
  int64_t rows;
  int k;
  float* V;            // (rows, k) or null
  int32_t* I;          // (rows, k) or null
  uint64_t* keys_out;  // (rows, L) or null: the row's top k, then further real keys descending, then empty keys
  int use_ex;
  ExchangeDev ex;
  uint32_t* zero;      // pipelined encode: the finished batch's sync region (counters, pilot histogram), cleared
  int64_t zero_words;  // after its rows for the batch after next (a multiple of 4 words); or null
};

struct FusedParams {
  UnitGrid grid;
  const float* bias;
  uint64_t* partials;  // [units][128][L] keys
  uint64_t* app;       // [gridDim.x][kAppendMax][128] keys (global append slots)
  uint32_t* pilot_hist;    // [m_tiles][128][kPilotBins] counts, zeroed by the host; null = no pilot
  uint32_t* pilot_count;   // CTAs that finished their sample
  uint32_t* tail_count;    // CTAs whose lists are stored (finish barrier); zeroed by the host
  uint32_t* row_floor;     // [m_tiles][128] shared lower bound of each row's k-th score (float_order; 0 =
                           // none), raised by every unit as its threshold rises; zeroed by the host; null = off
  int finish;              // 1: the kernel finishes the rows itself (fin), after a grid barrier
  int list_pitch;          // keys per row list in partials: L, or L + kAppendMax with a sorted tail run
  FinishArgs fin;
  int64_t B, F;
  int k;
  int num_kb;          // ceil(d / 64) (16-bit inputs; the kernel groups kSub per stage), ceil(d / 16) for TF32
  int ab_format;       // 0 fp16, 1 bf16
  int w_evict_first;   // W is read once (single M tile): stream it past L2
  uint32_t index_offset;
  int pilot_chunks;    // sampled 32-feature chunks per CTA (<= the first tile's chunks)
  float* cand_vals;      // kModeCand: (B, cand_tiles, cand_c) per-tile top-c values (-FLT_MAX padding)
  int32_t* cand_idxs;    // kModeCand: their feature indices (-1 padding)
  int64_t cand_tiles;    // ceil(F / 128)
  int cand_c;            // 16 or 32
  const float* x_scale;  // FP8: [B] per-row dequantization scale of X
  const float* w_scale;  // FP8: [F] per-feature dequantization scale of W (scores = x_s * w_s * acc + b)
  int prev_finish;       // pipelined encode: the epilogue warps first finish the previous step's rows (pfin)
  FinishArgs pfin;
};

struct SimtParams {
  UnitGrid grid;
  const float* bias;
  uint64_t* partials;
  uint64_t* app;
  int64_t B, F, d;
  int k;
  uint32_t index_offset;
};

// Shared-memory plan of the fused kernel: STAGES x (X tile 128x64, W tile
// NTx64, both K-major 128-byte swizzled), the per-row top lists unless they
// live in tensor memory (TOPT), the per-row append slots when they live in
// shared memory (APP_SMEM), then the mbarriers.
template <int L, int NT, int STAGES, int A, bool APP_SMEM, bool TOPT, bool PAIR = false>
struct FusedCfg {
  static constexpr int kXBytes = kRows * 64 * 2;
  static constexpr int kWBytes = (PAIR ? NT / 2 : NT) * 64 * 2;  // CTA pairs: each CTA holds half the W tile
  // 64-element K boxes per pipeline stage.  Two (K = 128 per stage: the X
  // boxes, then the W boxes) for the TMEM-list configurations with 128-feature
  // tiles: each stage's handoff (TMA barrier, MMA issue, commit) then carries
  // eight MMAs, which keeps the tensor pipe busier (cfg5: 10.9 -> 10.3 ms).
  static constexpr int kSub = (TOPT && NT == 128) ? 2 : 1;
  static constexpr int kStageBytes = kSub * (kXBytes + kWBytes);
  static constexpr int kTopOff = STAGES * kStageBytes;
  static constexpr int kAppOff = kTopOff + (TOPT ? 0 : L * kRows * 8);
  static constexpr int kBarOff = kAppOff + (APP_SMEM ? A * kRows * 8 : 0);
  static constexpr int kSmemBytes = 1024 + kBarOff + 256;
  static constexpr int kTmemCols = (2 * NT <= 32) ? 32 : (2 * NT <= 64) ? 64 : (2 * NT <= 128) ? 128 : (2 * NT <= 256) ? 256 : 512;
  static_assert(NT % 32 == 0 && NT >= 32 && NT <= 256, "tile width");
  static_assert(kStageBytes % 1024 == 0, "stage alignment");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// Shared-memory plan of the SIMT kernel: score tile (aliased by the GEMM
// staging buffers), top lists.
template <int L>
struct SimtCfg {
  static constexpr int kNT = 128;
  static constexpr int kKc = 32;
  static constexpr int kXsOff = 0;
  static constexpr int kWsOff = kKc * (kRows + 1) * 4;
  static constexpr int kScOff = 0;
  static constexpr int kScBytes = kRows * (kRows + 1) * 4;
  static constexpr int kTopOff = (kScBytes + 15) & ~15;
  static constexpr int kSmemBytes = 16 + kTopOff + L * kRows * 8;
  static_assert(kWsOff + kKc * (kRows + 1) * 4 <= kScBytes, "staging must fit in the score tile");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// (L, NT, STAGES, A, APP_SMEM, TOPT) instantiated for the fused kernel (the
// defaults are chosen in stk_capi.cu).  TOPT: the per-row top lists live in
// tensor memory beside the accumulators (two NT-column buffers, or one when
// 2 x NT + 2 x L > 512 columns), which leaves the shared memory to the TMA ring.
#define STK_FUSED_CONFIGS(X)      \
  X(32, 256, 3, 32, true, false)  \
  X(64, 256, 3, 16, true, false)  \
  X(64, 128, 4, 16, true, false)  \
  X(32, 128, 5, 32, true, false)  \
  X(128, 256, 2, 32, false, false) \
  X(128, 128, 3, 32, false, false) \
  X(128, 128, 3, 32, true, true)  \
  X(128, 256, 4, 32, true, true)

// Configurations of the fp32 (3-pass TF32) variant: same shared-memory plan
// (X and its residual take the bytes of the 16-bit X tile, W and its residual
// those of the 16-bit W tile, K = 16 per stage with 64-byte swizzle); NT <= 128
// because each accumulator buffer holds two NT-column accumulators.
#define STK_FUSED_TF32_CONFIGS(X)   \
  X(32, 128, 5, 32, true, false)    \
  X(64, 128, 4, 16, true, false)    \
  X(128, 128, 3, 32, false, false)

// Configurations of the FP8 variant (E4M3 X and W_enc, K = 128 per 128-byte
// box): the 16-bit shared-memory plan, half the bytes per K element.
#define STK_FUSED_FP8_CONFIGS(X)      \
  X(32, 256, 3, 32, true, false)     \
  X(64, 256, 3, 16, true, false)     \
  X(64, 128, 4, 16, true, false)     \
  X(32, 128, 5, 32, true, false)     \
  X(128, 128, 3, 32, true, true)

// Operand modes of the fused kernel.
constexpr int kModeF16 = 0;   // fp16 / bf16 X and W, kind::f16
constexpr int kModeTF32 = 1;  // fp32 X and W, 3-pass kind::tf32
constexpr int kModeFP8 = 2;   // E4M3 X (quantized per row by the library) and W (per-feature scale), kind::f8f6f4
constexpr int kModePair = 4;  // flag: 2-CTA clusters, tcgen05.mma.cta_group::2 with M = 256 (16-bit or FP8)
constexpr int kModeCand = 8;  // flag: also write each 128-feature tile's top c (c <= 32) per row (approx op)

// Configurations of the candidate variant (16-bit inputs, k <= c <= 32).
#define STK_FUSED_CAND_CONFIGS(X)    \
  X(32, 256, 3, 32, true, false)    \
  X(32, 128, 5, 32, true, false)

// Configurations of the CTA-pair variant (B >= 256 with an even number of
// 128-row M tiles, several units per CTA): each CTA's stage holds its X boxes
// and half the W rows, so four 48 KB stages (K = 128) fit beside the append slots.
#define STK_FUSED_PAIR_CONFIGS(X) \
  X(128, 128, 4, 32, true, true)

// Launches a pair-variant kernel (MODE includes kModePair) as 2-CTA clusters;
// grid is even.
template <int L, int NT, int STAGES, int A, bool APP_SMEM, bool TOPT, int MODE>
cudaError_t launch_fused_pair(const CUtensorMap& tx, const CUtensorMap& tw, const FusedParams& p, int grid,
                              cudaStream_t stream);
// Largest number of 2-CTA clusters of a pair-variant kernel that fit on the
// device at once (0 if none).
template <int L, int NT, int STAGES, int A, bool APP_SMEM, bool TOPT, int MODE>
int pair_clusters_max();

// TF32: X is read through two maps (tx: X itself, txl: its residual
// X - trunc13(X)); otherwise txl is unused.
template <int L, int NT, int STAGES, int A, bool APP_SMEM, bool TOPT, int MODE>
cudaError_t launch_fused(const CUtensorMap& tx, const CUtensorMap& txl, const CUtensorMap& tw, const CUtensorMap& tw32,
                         const FusedParams& p, int grid, cudaStream_t stream);

// Xl = X - trunc13(X) (exact in fp32), n elements.
cudaError_t launch_residual_tf32(const float* X, float* Xl, int64_t n, cudaStream_t stream);

// Per-row E4M3 quantization of a (rows, d) matrix of T (float, __half or
// __nv_bfloat16): scale[r] = max_j |x[r][j]| / 448 (1 for an all-zero row),
// Q[r][j] = E4M3(x[r][j] * (448 / max_j |x[r][j]|)), round to nearest even,
// saturating.  x[r][j] ~= scale[r] * Q[r][j].
template <typename T>
cudaError_t launch_quantize_rows_e4m3(const T* X, uint8_t* Q, float* scale, int64_t rows, int64_t d,
                                      cudaStream_t stream);

template <typename T, int L>
cudaError_t launch_simt(const void* X, const void* W, const SimtParams& p, int grid, cudaStream_t stream);

// Standalone finish (after a score kernel that does not finish its rows
// itself, or over lists all-gathered from other GPUs): a programmatic
// dependent launch of `grid` CTAs of kFinishThreads.
constexpr int kFinishThreads = 256;
template <int L>
cudaError_t launch_finish(const FinishArgs& fa, int grid, cudaStream_t stream);


// SAE decoder over the encoder's sparse codes (no reference counterpart):
// out[b][:] = b_dec[:] + sum_j V[b][j] * W_dec[I[b][j]][:], W_dec (F, d) in T
// (float, __half or __nv_bfloat16), fp32 accumulation and output; b_dec may be
// null; indices < 0 (padding) or >= F are skipped.  d % 8 == 0 for 16-bit W_dec
// (d % 4 for fp32) and 16-byte aligned W_dec / out / b_dec.
template <typename T>
cudaError_t launch_decode(const float* V, const int32_t* I, const T* W_dec, const float* b_dec, float* out, int64_t B,
                          int k, int64_t F, int64_t d, cudaStream_t stream);

// Exact top-k of rows over F <= kFullSortMaxF features by a whole-row sort,
// any 1 <= k <= F (dtype: 0 fp32, 1 fp16, 2 bf16; grid.x = B must fit).
constexpr int kFullSortMaxF = 4096;
cudaError_t launch_fullsort(const void* X, const void* W, const float* bias, float* V, int32_t* I, int64_t B,
                            int64_t d, int F, int k, int dtype, cudaStream_t stream);

// Per-tile candidates of the approximate path: partials[(tile * m_tiles + m) *
// 128 + r][0..L) -> cand_vals / cand_idxs [(row) * tiles + tile][0..c),
// empty keys as (-FLT_MAX, -1).
cudaError_t launch_candidates_out(const uint64_t* partials, int L, int m_tiles, int64_t tiles, int64_t rows, int c,
                                  float* vals, int32_t* idxs, cudaStream_t stream);

cudaError_t read_and_clear_device_error(unsigned* out, cudaStream_t stream);

}  // namespace stk
