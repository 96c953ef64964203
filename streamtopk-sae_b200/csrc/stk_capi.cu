// C ABI of the encoder (include/stk_b200.h): argument checks with the
// reference's messages, path and tile selection, TMA descriptor encoding,
// work decomposition and launches.  No allocation happens here: the caller
// passes the workspace.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <numeric>
#include <string>
#include <vector>

#include "../../include/stk_b200.h"
#include "stk_kernels.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  g_err = std::string(where) + ": " + cudaGetErrorName(e) + ": " + cudaGetErrorString(e);
  return STK_ECUDA;
}

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  int sms = 0;
  int pair_grid = -1;  // CTAs of the CTA-pair kernel (even; 0: unavailable); -1 not queried yet
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_sms(int* sms);

// CTAs to launch the CTA-pair kernel with: two per 2-CTA cluster, as many
// clusters as fit on the device at once (at most one CTA per SM).
int pair_grid(int* grid) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(STK_EINVAL, "device ordinal out of range");
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (g_dev[dev].pair_grid >= 0) {
      *grid = g_dev[dev].pair_grid;
      return STK_OK;
    }
  }
  int sms = 0;
  int rc = device_sms(&sms);
  if (rc) return rc;
  int clusters = 0;
#define STK_PAIR_MAX(Lc, NTc, Sc, Ac, SMc, TTc) \
  clusters = stk::pair_clusters_max<Lc, NTc, Sc, Ac, SMc, TTc, stk::kModeF16 | stk::kModePair>();
  STK_FUSED_PAIR_CONFIGS(STK_PAIR_MAX)
#undef STK_PAIR_MAX
  cudaGetLastError();  // an occupancy query that failed leaves no sticky error
  if (clusters > sms / 2) clusters = sms / 2;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  g_dev[dev].pair_grid = clusters > 0 ? 2 * clusters : 0;
  *grid = g_dev[dev].pair_grid;
  return STK_OK;
}

int device_sms(int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(STK_EINVAL, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_dev[dev].sms == 0) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    g_dev[dev].sms = n;
  }
  *sms = g_dev[dev].sms;
  return STK_OK;
}

// Optional per-launch CUDA-event timing (stk_profile_begin/end): events are
// recorded on the launching stream around each kernel, nothing is skipped.
enum ProfKind { kProfFused = 0, kProfSimt = 1, kProfMerge = 2, kProfExchange = 3, kProfKinds = 4 };
struct ProfState {
  std::mutex mu;
  std::atomic<bool> on{false};
  std::vector<cudaEvent_t> ev;
  std::vector<int> kind;
  size_t used = 0;
};
ProfState g_prof;

// Inside a stream capture the records become event-record nodes of the graph
// (cudaEventRecordExternal), re-recorded at every replay.
void prof_record(cudaEvent_t e, cudaStream_t s) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &st) == cudaSuccess && st == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
  else
    cudaEventRecord(e, s);
}

struct ProfScope {
  cudaStream_t s;
  cudaEvent_t e1 = nullptr;
  ProfScope(int kind, cudaStream_t stream) : s(stream) {
    if (!g_prof.on) return;
    std::lock_guard<std::mutex> lk(g_prof.mu);
    if (!g_prof.on || g_prof.used + 2 > g_prof.ev.size()) return;
    cudaEvent_t e0 = g_prof.ev[g_prof.used];
    e1 = g_prof.ev[g_prof.used + 1];
    g_prof.kind[g_prof.used / 2] = kind;
    g_prof.used += 2;
    prof_record(e0, s);
  }
  ~ProfScope() {
    if (e1) prof_record(e1, s);
  }
};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}

// 2-D K-major tensor map over a (rows, d) row-major 16-bit matrix with a
// (64 x box_rows) box and 128-byte swizzle; out-of-range elements read as 0.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t d, int box_rows, bool bf16) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(STK_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)d * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return fail(STK_ECUDA, buf);
  }
  return STK_OK;
}

// 2-D K-major tensor map over a (rows, d) row-major fp32 matrix with a
// (16 x box_rows) box (64 bytes of K per row) and 64-byte swizzle.
int make_map_f32(CUtensorMap* map, const void* base, int64_t rows, int64_t d, int box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(STK_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)d * 4};
  const cuuint32_t box[2] = {16, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled (fp32) failed (CUresult %d)", (int)r);
    return fail(STK_ECUDA, buf);
  }
  return STK_OK;
}

// 2-D K-major tensor map over a (rows, d) row-major byte matrix (E4M3) with a
// (128 x box_rows) box (128 bytes of K per row) and 128-byte swizzle.
int make_map_u8(CUtensorMap* map, const void* base, int64_t rows, int64_t d, int box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(STK_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)d};
  const cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled (e4m3) failed (CUresult %d)", (int)r);
    return fail(STK_ECUDA, buf);
  }
  return STK_OK;
}

int list_len(int64_t k) { return k <= 32 ? 32 : k <= 64 ? 64 : k <= 128 ? 128 : 0; }

bool ref_k(int64_t k) {
  return k == 1 || k == 2 || k == 4 || k == 8 || k == 16 || k == 32 || k == 64 || k == 128;
}

// Work decomposition: units = M tiles x feature ranges, sized so the
// persistent grid (one CTA per SM) gets a whole number of units each.
stk::UnitGrid make_grid(int64_t B, int64_t F, int sms) {
  stk::UnitGrid g;
  g.m_tiles = (int)((B + stk::kRows - 1) / stk::kRows);
  g.nchunks = (F + 31) / 32;
  int segs = sms / std::gcd(g.m_tiles, sms);
  if (segs < 1) segs = 1;
  if ((int64_t)segs > g.nchunks) segs = (int)g.nchunks;
  g.segs = segs;
  g.units = g.m_tiles * segs;
  g.fixed_chunks = 0;
  g.quantum = 1;
  return g;
}

// One unit per 128-feature tile (the approximate path's candidate tiles).
stk::UnitGrid make_tile_grid(int64_t B, int64_t F) {
  stk::UnitGrid g;
  g.m_tiles = (int)((B + stk::kRows - 1) / stk::kRows);
  g.nchunks = (F + 31) / 32;
  g.fixed_chunks = 4;
  g.segs = (int)((F + 127) / 128);
  g.units = g.m_tiles * g.segs;
  g.quantum = 1;
  return g;
}

size_t partial_bytes(const stk::UnitGrid& g, int pitch) {
  return (size_t)g.units * stk::kRows * pitch * sizeof(uint64_t);
}

struct Plan {
  bool tc;    // tcgen05 path
  bool tf32;  // tcgen05 path for fp32 inputs (3-pass TF32), opt-in
  bool fp8;   // E4M3 W_enc, X quantized per row into the workspace (kind::f8f6f4)
  int x_dtype;              // fp8: X's element type
  const float* w_scale;     // fp8: per-feature scale of W_enc (call data)
  int L;
  stk::UnitGrid grid;
  int ctas;
  bool pilot;
  bool fin_fused;  // the fused kernel finishes the rows itself (all units resident at once)
  bool shared_floor;  // units publish their thresholds per row (several units per CTA, no pilot)
  bool pair;          // CTA pairs (tcgen05 cta_group::2, M = 256): k > 64, an even number of M tiles
  bool cand;          // approximate op with candidates in one pass (each 128-feature tile's top c)
  float* cand_vals;   // cand: (B, ceil(F / 128), cand_c) outputs (call data)
  int32_t* cand_idxs;
  int cand_c;
  int pitch;       // keys per row list in the partials: L, or L + kAppendMax (sorted tail run, fused finish)
  size_t ws_partials;
  size_t ws_app;
  size_t ws_sync;   // zeroed per call: barrier counters, then the pilot histogram or the shared row floor
  size_t ws_split;  // TF32: X's residual X - trunc13(X), 256-byte aligned
  size_t ws_q;      // fp8: X quantized (B x d bytes, 256-aligned), then its row scales
  size_t ws;
  bool presync;     // pipelined encode: the sync region is already zero (cleared by an earlier batch's finish)
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

constexpr int64_t kTf32DefaultMaxD = 2048;

// Counters at the start of the zeroed sync region: [0] pilot arrivals,
// [1] finish-barrier arrivals; the pilot histogram follows at kSyncBytes.
constexpr size_t kSyncBytes = 256;

int plan(const void* X, const void* W, int64_t B, int64_t d, int64_t F, int64_t k, int dtype, int flags, Plan* pl) {
  int sms = 0;
  int rc = device_sms(&sms);
  if (rc) return rc;
  pl->L = list_len(k);
  pl->presync = false;
  const bool aligned = (X == nullptr || aligned16(X)) && (W == nullptr || aligned16(W));
  // fp32 inputs run on tensor cores (3-pass TF32) by default up to d =
  // kTf32DefaultMaxD, where its accuracy is shown against float64 to hold the
  // fp32 tolerance; beyond that only on request (STK_FLAG_TF32).  STK_FLAG_SIMT
  // forces fp32 FMA.
  pl->tf32 = dtype == STK_F32 && ((flags & STK_FLAG_TF32) || d <= kTf32DefaultMaxD) && (d % 4 == 0) &&
             !(flags & STK_FLAG_SIMT) && aligned;
  pl->fp8 = dtype == STK_E4M3;
  pl->x_dtype = dtype;
  pl->w_scale = nullptr;
  pl->cand = false;
  pl->cand_vals = nullptr;
  pl->cand_idxs = nullptr;
  pl->cand_c = 0;
  pl->tc = ((dtype == STK_BF16 || dtype == STK_F16) && (d % 8 == 0) && !(flags & STK_FLAG_SIMT) && aligned) ||
           pl->tf32 || (pl->fp8 && d % 16 == 0 && aligned);
  pl->grid = make_grid(B, F, sms);
  pl->ctas = pl->grid.units < sms ? pl->grid.units : sms;
  // CTA pairs for k > 64 with several rounds of units per CTA and an even
  // number of M tiles: the pair's MMA covers two M tiles (M = 256) and each
  // CTA loads half the W tile, which cuts the L2-to-SM bytes per MMA by a
  // quarter (the TMEM-list kernel at B = 4096 is bound by them).
  pl->pair = false;
  if (pl->tc && !pl->tf32 && pl->L == 128 && pl->grid.m_tiles >= 2 && pl->grid.m_tiles % 2 == 0 &&
      !(flags & STK_FLAG_NO_PAIR)) {
    int pg = 0;
    rc = pair_grid(&pg);
    if (rc) return rc;
    if (pg >= 2 && pl->grid.units > pg) {
      pl->pair = true;
      pl->ctas = pg;
    }
  }
  // partial lists, then one append buffer per CTA, then (optionally) the
  // pilot histogram and arrival counters (256-byte aligned parts)
  pl->ws_app = ((size_t)pl->ctas * stk::kAppendBytesPerCta + 255) & ~size_t(255);
  // The sample step needs one unit per CTA (all CTAs resident together) and
  // pays off when each CTA streams several chunks after its sample.
  pl->pilot = pl->tc && pl->grid.units <= pl->ctas && pl->grid.m_tiles <= 2 &&
              pl->grid.nchunks >= 4 * (int64_t)pl->grid.segs && !(flags & STK_FLAG_NO_PILOT);
  // One unit per CTA and every CTA resident (one per SM): the fused kernel
  // meets at a grid barrier and finishes the rows itself, no second launch.
  pl->fin_fused = pl->tc && pl->grid.units <= pl->ctas && !(flags & STK_FLAG_SEPARATE_FINISH);
  // With one unit per CTA (the fused finish, or a pipelined step's separate
  // finish) each row list carries its last survivors as a sorted second run
  // (no final merge in the score kernel).
  pl->pitch = (pl->tc && pl->grid.units <= pl->ctas && !std::getenv("STK_FULL_FLUSH")) ? pl->L + stk::kAppendMax
                                                                                        : pl->L;
  pl->ws_partials = (partial_bytes(pl->grid, pl->pitch) + 255) & ~size_t(255);
  // Without the pilot (several units per CTA, e.g. B > 256), the units of an
  // M tile share their rising thresholds as a floor instead.  Not for the
  // approximate path's per-tile candidate units (fixed_chunks), whose lists
  // must hold each tile's own top c.
  pl->shared_floor = pl->tc && !pl->pilot && pl->grid.units > pl->ctas && pl->grid.fixed_chunks == 0 &&
                     !(flags & STK_FLAG_NO_PILOT);
  const size_t pilot_bytes = pl->pilot ? (size_t)pl->grid.m_tiles * stk::kRows * stk::kPilotBins * 4 : 0;
  const size_t floor_bytes = pl->shared_floor ? (size_t)pl->grid.m_tiles * stk::kRows * 4 : 0;
  pl->ws_sync = (pl->pilot || pl->fin_fused || pl->shared_floor)
                    ? ((kSyncBytes + pilot_bytes + floor_bytes + 255) & ~size_t(255))
                    : 0;
  pl->ws_split = pl->tf32 ? (((size_t)B * d * 4 + 255) & ~size_t(255)) : 0;
  pl->ws_q = pl->fp8 ? (((size_t)B * d + 255) & ~size_t(255)) + (((size_t)B * 4 + 255) & ~size_t(255)) : 0;
  pl->ws = pl->ws_partials + pl->ws_app + pl->ws_sync + pl->ws_split + pl->ws_q;
  return STK_OK;
}

// Optional override of the fused tile configuration,
// "L,NT,STAGES,A,APP_SMEM[,TOPT]", for tuning.
bool fused_override(int L, int* nt, int* stages, int* app, int* app_smem, int* topt) {
  const char* s = std::getenv("STK_FUSED_CFG");
  if (!s) return false;
  int l = 0, n = 0, st = 0, a = 0, sm = 0, tt = 0;
  const int got = std::sscanf(s, "%d,%d,%d,%d,%d,%d", &l, &n, &st, &a, &sm, &tt);
  if (got < 5 || l != L) return false;
  *nt = n;
  *stages = st;
  *app = a;
  *app_smem = sm;
  *topt = got == 6 ? tt : 0;
  return true;
}

int run_fused(const Plan& pl, const void* X, const void* W, const float* b, uint64_t* partials, uint64_t* app,
              int64_t B, int64_t d, int64_t F, int64_t k, int dtype, uint32_t index_offset,
              const stk::FinishArgs* fin, cudaStream_t stream, const stk::FinishArgs* prev_fin = nullptr) {
  // Defaults: 256-feature tiles, append slots in shared memory where 3
  // pipeline stages still fit.  When a CTA's unit fits in one such tile (F
  // small per CTA, e.g. one shard of a multi-GPU encode) 128-feature tiles
  // are used instead: the epilogue of the first tile then overlaps the loads
  // of the second, and the pilot barrier comes after half the loads.
  const int64_t unit_feats =
      32 * (pl.grid.fixed_chunks > 0 ? (int64_t)pl.grid.fixed_chunks
                                     : (pl.grid.nchunks + pl.grid.segs - 1) / pl.grid.segs);
  const bool narrow = unit_feats <= 256;
  // TF32 (two accumulators per buffer): always 128-feature tiles.
  const bool nt128 = narrow || pl.tf32;
  int nt = nt128 ? 128 : 256;
  int stages = nt128 ? (pl.L == 128 ? 3 : pl.L == 64 ? 4 : 5) : (pl.L == 128 ? 2 : 3);
  int nslots = pl.L == 64 ? 16 : 32;
  int app_smem = pl.L == 128 ? 0 : 1;
  int topt = 0;
  if (pl.L == 128 && !pl.tf32) {
    // k > 64: the per-row top-128 lists (128 KB) go to tensor memory beside
    // 128-column accumulators, and the shared memory holds a three-stage TMA
    // ring of 64 KB stages (K = 128 each; two 48 KB stages fit beside the
    // lists in shared memory).
    nt = 128;
    stages = 3;
    app_smem = 1;
    topt = 1;
  }
  if (pl.pair) {
    // The pair configuration: 128-feature tiles, four 48 KB stages (each CTA's
    // X boxes and half the W rows, K = 128), lists in TMEM.
    nt = 128;
    stages = 4;
    nslots = 32;
    app_smem = 1;
    topt = 1;
  } else if (!pl.cand) {
    fused_override(pl.L, &nt, &stages, &nslots, &app_smem, &topt);
  }
  const int w_box = pl.pair ? nt / 2 : nt;  // pairs: each CTA loads half the tile's W rows
  CUtensorMap tx, txl, tw, tw32;
  const bool bf16 = dtype == STK_BF16;
  int rc = STK_OK;
  const float* x_scale = nullptr;
  if (pl.fp8) {
    // X is quantized per row (E4M3 + one scale per row) into the workspace;
    // W_enc is E4M3 already.  Both through byte maps, 128 K elements per box.
    uint8_t* xq = reinterpret_cast<uint8_t*>(partials) + pl.ws_partials + pl.ws_app + pl.ws_sync + pl.ws_split;
    float* xs = reinterpret_cast<float*>(xq + (((size_t)B * d + 255) & ~size_t(255)));
    cudaError_t qe = cudaErrorInvalidValue;
    if (pl.x_dtype == STK_F32) qe = stk::launch_quantize_rows_e4m3(static_cast<const float*>(X), xq, xs, B, d, stream);
    if (pl.x_dtype == STK_F16) qe = stk::launch_quantize_rows_e4m3(static_cast<const __half*>(X), xq, xs, B, d, stream);
    if (pl.x_dtype == STK_BF16)
      qe = stk::launch_quantize_rows_e4m3(static_cast<const __nv_bfloat16*>(X), xq, xs, B, d, stream);
    if (qe != cudaSuccess) return cuda_fail(qe, "quantize_rows_e4m3_kernel launch");
    x_scale = xs;
    rc = make_map_u8(&tx, xq, B, d, stk::kRows);
    if (!rc) rc = make_map_u8(&tw, W, F, d, w_box);
    if (!rc) rc = make_map_u8(&tw32, W, F, d, 32);
    txl = tx;
  } else if (pl.tf32) {
    // X's residual X - trunc13(X) is computed once per call (L2-resident,
    // re-read by every tile); W's residual tile by tile inside the kernel.  The
    // raw X and W are the hi operands (the tensor core reads them as TF32).
    float* xl = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(partials) + pl.ws_partials + pl.ws_app + pl.ws_sync);
    cudaError_t se = stk::launch_residual_tf32(static_cast<const float*>(X), xl, B * d, stream);
    if (se != cudaSuccess) return cuda_fail(se, "residual_tf32_kernel launch");
    rc = make_map_f32(&tx, X, B, d, stk::kRows);
    if (!rc) rc = make_map_f32(&txl, xl, B, d, stk::kRows);
    if (!rc) rc = make_map_f32(&tw, W, F, d, nt);
    if (!rc) rc = make_map_f32(&tw32, W, F, d, 32);
  } else {
    rc = make_map(&tx, X, B, d, stk::kRows, bf16);
    if (!rc) rc = make_map(&tw, W, F, d, w_box, bf16);
    if (!rc) rc = make_map(&tw32, W, F, d, 32, bf16);
    txl = tx;
  }
  if (rc) return rc;
  stk::FusedParams p;
  p.grid = pl.grid;
  p.bias = b;
  p.partials = partials;
  p.app = app;
  p.B = B;
  p.F = F;
  p.k = (int)k;
  p.num_kb = pl.tf32 ? (int)((d + 15) / 16) : pl.fp8 ? (int)((d + 127) / 128) : (int)((d + 63) / 64);
  p.x_scale = x_scale;
  p.w_scale = pl.w_scale;
  p.cand_vals = pl.cand_vals;
  p.cand_idxs = pl.cand_idxs;
  p.cand_tiles = (F + 127) / 128;
  p.cand_c = pl.cand_c;
  p.ab_format = bf16 ? 1 : 0;
  p.w_evict_first = pl.grid.m_tiles == 1 ? 1 : 0;
  p.index_offset = index_offset;
  p.pilot_chunks = stk::kPilotChunks;
  if (const char* e = std::getenv("STK_PILOT_CHUNKS")) {  // tuning sweeps
    const int v = std::atoi(e);
    if (v >= 1 && v <= 8) p.pilot_chunks = v;
  }
  p.pilot_hist = nullptr;
  p.pilot_count = nullptr;
  p.tail_count = nullptr;
  p.row_floor = nullptr;
  p.finish = 0;
  p.list_pitch = pl.pitch;
  std::memset(&p.fin, 0, sizeof p.fin);
  if (pl.ws_sync) {
    uint8_t* base = reinterpret_cast<uint8_t*>(partials) + pl.ws_partials + pl.ws_app;
    p.pilot_count = reinterpret_cast<uint32_t*>(base);
    p.tail_count = p.pilot_count + 1;
    if (pl.pilot) {
      p.pilot_hist = reinterpret_cast<uint32_t*>(base + kSyncBytes);
    }
    if (pl.shared_floor) p.row_floor = reinterpret_cast<uint32_t*>(base + kSyncBytes);
    if (!pl.presync) {
      cudaError_t me = cudaMemsetAsync(base, 0, pl.ws_sync, stream);
      if (me != cudaSuccess) return cuda_fail(me, "cudaMemsetAsync(sync)");
    }
  }
  p.prev_finish = 0;
  std::memset(&p.pfin, 0, sizeof p.pfin);
  if (prev_fin) {
    p.prev_finish = 1;
    p.pfin = *prev_fin;
  }
  if (fin) {
    p.finish = 1;
    p.fin = *fin;
  }
  cudaError_t e = cudaErrorInvalidValue;
  ProfScope prof(kProfFused, stream);
#define STK_TRY_FUSED_PAIR(Lc, NTc, Sc, Ac, SMc, TTc)                                                      \
  if (pl.pair && pl.L == Lc && nt == NTc && stages == Sc && nslots == Ac && (app_smem != 0) == SMc &&           \
      (topt != 0) == TTc) {                                                                                    \
    if (pl.fp8)                                                                                                \
      e = stk::launch_fused_pair<Lc, NTc, Sc, Ac, SMc, TTc, stk::kModeFP8 | stk::kModePair>(tx, tw, p, pl.ctas, \
                                                                                             stream);          \
    else                                                                                                       \
      e = stk::launch_fused_pair<Lc, NTc, Sc, Ac, SMc, TTc, stk::kModeF16 | stk::kModePair>(tx, tw, p, pl.ctas, \
                                                                                             stream);          \
  }
  STK_FUSED_PAIR_CONFIGS(STK_TRY_FUSED_PAIR)
#undef STK_TRY_FUSED_PAIR
#define STK_TRY_FUSED_CAND(Lc, NTc, Sc, Ac, SMc, TTc)                                                 \
  if (pl.cand && pl.L == Lc && nt == NTc && stages == Sc && nslots == Ac && (app_smem != 0) == SMc &&   \
      (topt != 0) == TTc)                                                                               \
    e = stk::launch_fused<Lc, NTc, Sc, Ac, SMc, TTc, stk::kModeF16 | stk::kModeCand>(tx, txl, tw, tw32, p, pl.ctas, \
                                                                                     stream);
  STK_FUSED_CAND_CONFIGS(STK_TRY_FUSED_CAND)
#undef STK_TRY_FUSED_CAND
#define STK_TRY_FUSED(Lc, NTc, Sc, Ac, SMc, TTc)                                                      \
  if (!pl.cand && !pl.pair && !pl.tf32 && !pl.fp8 && pl.L == Lc && nt == NTc && stages == Sc && nslots == Ac && (app_smem != 0) == SMc &&  \
      (topt != 0) == TTc)                                                                               \
    e = stk::launch_fused<Lc, NTc, Sc, Ac, SMc, TTc, stk::kModeF16>(tx, txl, tw, tw32, p, pl.ctas, stream);
  STK_FUSED_CONFIGS(STK_TRY_FUSED)
#undef STK_TRY_FUSED
#define STK_TRY_FUSED_TF32(Lc, NTc, Sc, Ac, SMc, TTc)                                                 \
  if (pl.tf32 && pl.L == Lc && nt == NTc && stages == Sc && nslots == Ac && (app_smem != 0) == SMc &&   \
      (topt != 0) == TTc)                                                                               \
    e = stk::launch_fused<Lc, NTc, Sc, Ac, SMc, TTc, stk::kModeTF32>(tx, txl, tw, tw32, p, pl.ctas, stream);
  STK_FUSED_TF32_CONFIGS(STK_TRY_FUSED_TF32)
#undef STK_TRY_FUSED_TF32
#define STK_TRY_FUSED_FP8(Lc, NTc, Sc, Ac, SMc, TTc)                                                  \
  if (!pl.pair && pl.fp8 && pl.L == Lc && nt == NTc && stages == Sc && nslots == Ac && (app_smem != 0) == SMc &&    \
      (topt != 0) == TTc)                                                                               \
    e = stk::launch_fused<Lc, NTc, Sc, Ac, SMc, TTc, stk::kModeFP8>(tx, txl, tw, tw32, p, pl.ctas, stream);
  STK_FUSED_FP8_CONFIGS(STK_TRY_FUSED_FP8)
#undef STK_TRY_FUSED_FP8
  if (e != cudaSuccess) return cuda_fail(e, "fused_topk_kernel launch");
  return STK_OK;
}

int run_simt(const Plan& pl, const void* X, const void* W, const float* b, uint64_t* partials, uint64_t* app,
             int64_t B, int64_t d, int64_t F, int64_t k, int dtype, uint32_t index_offset, cudaStream_t stream) {
  stk::SimtParams p;
  p.grid = pl.grid;
  p.bias = b;
  p.partials = partials;
  p.app = app;
  p.B = B;
  p.F = F;
  p.d = d;
  p.k = (int)k;
  p.index_offset = index_offset;
  cudaError_t e = cudaErrorInvalidValue;
  ProfScope prof(kProfSimt, stream);
#define STK_SIMT_L(Lc)                                                                                     \
  if (pl.L == Lc) {                                                                                        \
    if (dtype == STK_F32) e = stk::launch_simt<float, Lc>(X, W, p, pl.ctas, stream);                      \
    if (dtype == STK_F16) e = stk::launch_simt<__half, Lc>(X, W, p, pl.ctas, stream);                     \
    if (dtype == STK_BF16) e = stk::launch_simt<__nv_bfloat16, Lc>(X, W, p, pl.ctas, stream);             \
  }
  STK_SIMT_L(32)
  STK_SIMT_L(64)
  STK_SIMT_L(128)
#undef STK_SIMT_L
  if (e != cudaSuccess) return cuda_fail(e, "simt_topk_kernel launch");
  return STK_OK;
}

// Standalone finish kernel (kind: kProfMerge, or kProfExchange with the
// exchange).  With the exchange every CTA must be resident at once (each
// publishes all of its rows before it waits), so the grid is capped.
int run_finish(int L, const stk::FinishArgs& fa, cudaStream_t stream) {
  int sms = 0;
  int rc = device_sms(&sms);
  if (rc) return rc;
  int64_t grid = fa.rows;
  if (fa.use_ex && grid > 4 * (int64_t)sms) grid = 4 * (int64_t)sms;
  if (grid > 0x7fffffff) grid = 0x7fffffff;
  cudaError_t e = cudaErrorInvalidValue;
  ProfScope prof(fa.use_ex ? kProfExchange : kProfMerge, stream);
  if (L == 32) e = stk::launch_finish<32>(fa, (int)grid, stream);
  if (L == 64) e = stk::launch_finish<64>(fa, (int)grid, stream);
  if (L == 128) e = stk::launch_finish<128>(fa, (int)grid, stream);
  if (e != cudaSuccess) return cuda_fail(e, "finish_kernel launch");
  return STK_OK;
}

stk::FinishArgs finish_args(const uint64_t* lists, int nlists, int64_t stride, int pitch, int tail, int64_t rows,
                            int64_t k, float* V, int32_t* I, uint64_t* keys_out, const stk::ExchangeDev* ex) {
  stk::FinishArgs fa;
  std::memset(&fa, 0, sizeof fa);
  fa.lists = lists;
  fa.nlists = nlists;
  fa.stride = stride;
  fa.pitch = pitch;
  fa.tail = tail;
  fa.rows = rows;
  fa.k = (int)k;
  fa.V = V;
  fa.I = I;
  fa.keys_out = keys_out;
  fa.use_ex = ex != nullptr;
  if (ex) fa.ex = *ex;
  return fa;
}

// Scores + per-unit lists, then the finish step: in the fused kernel's tail
// when its units are all resident at once, else as a second kernel.
int score_and_finish(const Plan& pl, const void* X, const void* W, const float* b, float* V, int32_t* I,
                     uint64_t* keys_out, int64_t B, int64_t d, int64_t F, int64_t k, int dtype, uint32_t index_offset,
                     const stk::ExchangeDev* ex, void* workspace, cudaStream_t stream) {
  uint64_t* partials = static_cast<uint64_t*>(workspace);
  uint64_t* app = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + pl.ws_partials);
  const stk::FinishArgs fa = finish_args(partials, pl.grid.segs, (int64_t)pl.grid.m_tiles * stk::kRows, pl.pitch,
                                         pl.pitch - pl.L, B, k, V, I, keys_out, ex);
  int rc = pl.tc ? run_fused(pl, X, W, b, partials, app, B, d, F, k, dtype, index_offset,
                             pl.fin_fused ? &fa : nullptr, stream)
                 : run_simt(pl, X, W, b, partials, app, B, d, F, k, dtype, index_offset, stream);
  if (rc) return rc;
  if (pl.tc && pl.fin_fused) return STK_OK;
  return run_finish(pl.L, fa, stream);
}

int check_common(const char* op, int64_t B, int64_t d, int64_t F, int dtype) {
  if (dtype != STK_F32 && dtype != STK_F16 && dtype != STK_BF16)
    return fail(STK_EINVAL, "X dtype must be fp32, fp16, or bf16");
  if (B < 0 || d < 1 || F < 1) return fail(STK_EINVAL, std::string(op) + ": empty or negative shape");
  if (F > 0x7fffffffLL) return fail(STK_EINVAL, std::string(op) + ": F must fit int32 indices");
  return STK_OK;
}

// Scores + per-unit partial lists, then the merge of the units of each row.
int encode(const void* X, const void* W, const float* b, float* V, int32_t* I, uint64_t* keys_out, int64_t B,
           int64_t d, int64_t F, int64_t k, int dtype, int flags, uint32_t index_offset, void* workspace,
           size_t workspace_bytes, cudaStream_t stream) {
  Plan pl;
  int rc = plan(X, W, B, d, F, k, dtype, flags, &pl);
  if (rc) return rc;
  if (B == 0) return STK_OK;
  if (workspace_bytes < pl.ws || (pl.ws && workspace == nullptr))
    return fail(STK_ENOSPACE, "workspace too small (need " + std::to_string(pl.ws) + " bytes)");
  return score_and_finish(pl, X, W, b, V, I, keys_out, B, d, F, k, dtype, index_offset, nullptr, workspace, stream);
}

}  // namespace

extern "C" {

int stk_version(void) { return 100; }

const char* stk_last_error(void) { return g_err.c_str(); }

int stk_list_len(int64_t k) { return k >= 1 ? list_len(k) : 0; }

int stk_workspace_bytes(int64_t B, int64_t d, int64_t F, int64_t k, int dtype, size_t* bytes) {
  if (!bytes) return fail(STK_EINVAL, "bytes is NULL");
  int rc = check_common("stk_workspace_bytes", B, d, F, dtype);
  if (rc) return rc;
  if (k < 1 || (list_len(k) == 0 && !(k <= F && F <= stk::kFullSortMaxF))) return fail(STK_EINVAL, "k out of range");
  if (list_len(k) == 0) {  // whole-row sort: no workspace
    *bytes = 0;
    return STK_OK;
  }
  // Sized for every path a call with these shapes may take: fp32 inputs
  // include the split X of the TF32 path (STK_FLAG_TF32 is a call flag).
  Plan pl;
  rc = plan(nullptr, nullptr, B, d, F, k, dtype, dtype == STK_F32 ? STK_FLAG_TF32 : 0, &pl);
  if (rc) return rc;
  *bytes = pl.ws;
  return STK_OK;
}

int stk_exact_forward(const void* X, const void* W, const float* b, float* V, int32_t* I, int64_t B, int64_t d,
                      int64_t F, int64_t k, int dtype, int flags, void* workspace, size_t workspace_bytes,
                      void* stream) {
  int rc = check_common("streamtopk_cuda_exact", B, d, F, dtype);
  if (rc) return rc;
  // streamtopk_exact.cu:812-813,818-830
  if (!(k >= 1 && k <= F)) return fail(STK_EINVAL, "k out of range");
  if (d > 4096 && !(flags & STK_FLAG_ANY_D)) return fail(STK_EINVAL, "d exceeds D_MAX=4096");
  if (!(flags & STK_FLAG_ANY_K) && !ref_k(k))
    return fail(STK_EINVAL, "streamtopk_cuda_exact: unsupported k=" + std::to_string(k) +
                                ". Supported: 1,2,4,8,16,32,64,128.");
  if (k > 128) {
    // Extension (STK_FLAG_ANY_K): k beyond the streaming lists for small F, by
    // sorting whole rows (no workspace).
    if (F > stk::kFullSortMaxF)
      return fail(STK_EINVAL, "streamtopk_cuda_exact: unsupported k=" + std::to_string(k) +
                                  " (k <= 128, or any k <= F when F <= " + std::to_string(stk::kFullSortMaxF) + ")");
    if (B == 0) return STK_OK;
    if (B > 0x7fffffffLL) return fail(STK_EINVAL, "B too large for the whole-row sort");
    cudaError_t e = stk::launch_fullsort(X, W, b, V, I, B, d, (int)F, (int)k,
                                         dtype == STK_F32 ? 0 : dtype == STK_F16 ? 1 : 2,
                                         static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "fullsort_kernel launch");
    return STK_OK;
  }
  return encode(X, W, b, V, I, nullptr, B, d, F, k, dtype, flags, 0u, workspace, workspace_bytes,
                static_cast<cudaStream_t>(stream));
}

int stk_quantize_rows_fp8(const void* X, int x_dtype, void* Q, float* scale, int64_t rows, int64_t d, void* stream) {
  if (x_dtype != STK_F32 && x_dtype != STK_F16 && x_dtype != STK_BF16)
    return fail(STK_EINVAL, "stk_quantize_rows_fp8: X dtype must be fp32, fp16, or bf16");
  if (rows < 0 || d < 1) return fail(STK_EINVAL, "stk_quantize_rows_fp8: empty or negative shape");
  if (d % 16 != 0) return fail(STK_EINVAL, "stk_quantize_rows_fp8: d must be a multiple of 16");
  if (rows == 0) return STK_OK;
  if (!X || !Q || !scale || !aligned16(Q)) return fail(STK_EINVAL, "stk_quantize_rows_fp8: null or unaligned pointer");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaErrorInvalidValue;
  uint8_t* q = static_cast<uint8_t*>(Q);
  if (x_dtype == STK_F32) e = stk::launch_quantize_rows_e4m3(static_cast<const float*>(X), q, scale, rows, d, s);
  if (x_dtype == STK_F16) e = stk::launch_quantize_rows_e4m3(static_cast<const __half*>(X), q, scale, rows, d, s);
  if (x_dtype == STK_BF16)
    e = stk::launch_quantize_rows_e4m3(static_cast<const __nv_bfloat16*>(X), q, scale, rows, d, s);
  if (e != cudaSuccess) return cuda_fail(e, "quantize_rows_e4m3_kernel launch");
  return STK_OK;
}

int stk_workspace_bytes_fp8(int64_t B, int64_t d, int64_t F, int64_t k, size_t* bytes) {
  if (!bytes) return fail(STK_EINVAL, "bytes is NULL");
  int rc = check_common("stk_workspace_bytes_fp8", B, d, F, STK_BF16);
  if (rc) return rc;
  if (k < 1 || list_len(k) == 0) return fail(STK_EINVAL, "k out of range");
  Plan pl;
  rc = plan(nullptr, nullptr, B, d, F, k, STK_E4M3, 0, &pl);
  if (rc) return rc;
  *bytes = pl.ws;
  return STK_OK;
}

int stk_exact_forward_fp8(const void* X, int x_dtype, const void* W8, const float* w_scale, const float* b, float* V,
                          int32_t* I, int64_t B, int64_t d, int64_t F, int64_t k, int flags, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = check_common("streamtopk_cuda_exact_fp8", B, d, F, x_dtype);
  if (rc) return rc;
  if (!(k >= 1 && k <= F)) return fail(STK_EINVAL, "k out of range");
  if (d > 4096 && !(flags & STK_FLAG_ANY_D)) return fail(STK_EINVAL, "d exceeds D_MAX=4096");
  if (!(flags & STK_FLAG_ANY_K) && !ref_k(k))
    return fail(STK_EINVAL, "streamtopk_cuda_exact_fp8: unsupported k=" + std::to_string(k) +
                                ". Supported: 1,2,4,8,16,32,64,128.");
  if (k > 128) return fail(STK_EINVAL, "streamtopk_cuda_exact_fp8: k must be <= 128");
  if (d % 16 != 0) return fail(STK_EINVAL, "streamtopk_cuda_exact_fp8: d must be a multiple of 16");
  if (B > 0 && (!X || !W8 || !w_scale || !b || !aligned16(X) || !aligned16(W8)))
    return fail(STK_EINVAL, "streamtopk_cuda_exact_fp8: null or unaligned (16-byte) input");
  if (flags & STK_FLAG_SIMT) return fail(STK_EINVAL, "streamtopk_cuda_exact_fp8: no SIMT path for FP8");
  Plan pl;
  rc = plan(X, W8, B, d, F, k, STK_E4M3, flags, &pl);
  if (rc) return rc;
  pl.x_dtype = x_dtype;
  pl.w_scale = w_scale;
  if (B == 0) return STK_OK;
  if (workspace_bytes < pl.ws || (pl.ws && workspace == nullptr))
    return fail(STK_ENOSPACE, "workspace too small (need " + std::to_string(pl.ws) + " bytes)");
  return score_and_finish(pl, X, W8, b, V, I, nullptr, B, d, F, k, STK_E4M3, 0u, nullptr, workspace,
                          static_cast<cudaStream_t>(stream));
}

int stk_approx_forward(const void* X, const void* W, const float* b, float* V, int32_t* I, int64_t B, int64_t d,
                       int64_t F, int64_t k, int64_t c, int dtype, int flags, void* workspace,
                       size_t workspace_bytes, void* stream) {
  int rc = check_common("streamtopk_cuda_approx", B, d, F, dtype);
  if (rc) return rc;
  // streamtopk_approx.cu:253,276-284
  if (!(k >= 1 && k <= c)) return fail(STK_EINVAL, "k must be <= c");
  if (!(c == 16 || c == 32 || c == 64 || c == 128))
    return fail(STK_EINVAL,
                "streamtopk_cuda_approx: unsupported c=" + std::to_string(c) + ". Supported: 16,32,64,128.");
  return encode(X, W, b, V, I, nullptr, B, d, F, k, dtype, flags | STK_FLAG_ANY_D, 0u, workspace, workspace_bytes,
                static_cast<cudaStream_t>(stream));
}

}  // extern "C"

extern "C" int candidates_plan(const void* X, const void* W, int64_t B, int64_t d, int64_t F, int64_t c, int dtype,
                               Plan* pl);

namespace {
// Plan of the approximate op with candidates: the exact encode's plan with
// feature ranges aligned to the reference's 128-feature tiles, and the fused
// kernel's candidate variant when it applies (16-bit inputs, c <= 32);
// *single = false means the two-pass fallback (candidates pass, then the
// exact top-k).
int cand_plan(const void* X, const void* W, int64_t B, int64_t d, int64_t F, int64_t k, int64_t c, int dtype,
              int flags, Plan* pl, bool* single) {
  int rc = plan(X, W, B, d, F, k, dtype, flags | STK_FLAG_ANY_D, pl);
  if (rc) return rc;
  const int64_t nq = (pl->grid.nchunks + 3) / 4;
  *single = pl->tc && !pl->tf32 && !pl->fp8 && !pl->pair && (dtype == STK_BF16 || dtype == STK_F16) && c <= 32 &&
            pl->L == 32 && pl->grid.fixed_chunks == 0 && nq >= pl->grid.segs;
  if (*single) {
    pl->grid.quantum = 4;
    pl->cand = true;
    pl->cand_c = (int)c;
  }
  return STK_OK;
}
}  // namespace

extern "C" {

int stk_approx_cand_workspace_bytes(int64_t B, int64_t d, int64_t F, int64_t k, int64_t c, int dtype, size_t* bytes) {
  if (!bytes) return fail(STK_EINVAL, "bytes is NULL");
  int rc = check_common("stk_approx_cand_workspace_bytes", B, d, F, dtype);
  if (rc) return rc;
  if (!(k >= 1 && k <= c) || !(c == 16 || c == 32 || c == 64 || c == 128))
    return fail(STK_EINVAL, "streamtopk_cuda_approx: need 1 <= k <= c, c in {16,32,64,128}");
  // Enough for either path (one pass, or candidates then the exact top-k).
  Plan pl;
  bool single = false;
  rc = cand_plan(nullptr, nullptr, B, d, F, k, c, dtype, 0, &pl, &single);
  if (rc) return rc;
  Plan pc;
  rc = candidates_plan(nullptr, nullptr, B, d, F, c, dtype, &pc);
  if (rc) return rc;
  Plan pe;
  rc = plan(nullptr, nullptr, B, d, F, k, dtype, dtype == STK_F32 ? STK_FLAG_TF32 : 0, &pe);
  if (rc) return rc;
  *bytes = pl.ws > pc.ws ? pl.ws : pc.ws;
  if (pe.ws > *bytes) *bytes = pe.ws;
  return STK_OK;
}

int stk_approx_forward_cand(const void* X, const void* W, const float* b, float* V, int32_t* I, float* cand_vals,
                            int32_t* cand_idxs, int64_t B, int64_t d, int64_t F, int64_t k, int64_t c, int dtype,
                            int flags, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common("streamtopk_cuda_approx", B, d, F, dtype);
  if (rc) return rc;
  if (!(k >= 1 && k <= c)) return fail(STK_EINVAL, "k must be <= c");
  if (!(c == 16 || c == 32 || c == 64 || c == 128))
    return fail(STK_EINVAL,
                "streamtopk_cuda_approx: unsupported c=" + std::to_string(c) + ". Supported: 16,32,64,128.");
  if (B == 0) return STK_OK;
  if (!cand_vals || !cand_idxs || !aligned16(cand_vals) || !aligned16(cand_idxs))
    return fail(STK_EINVAL, "candidate buffers must be non-null and 16-byte aligned");
  Plan pl;
  bool single = false;
  rc = cand_plan(X, W, B, d, F, k, c, dtype, flags, &pl, &single);
  if (rc) return rc;
  if (!single) {
    // Two passes: the per-tile candidates, then the exact top-k (equal to the
    // approximate result for k <= c).
    rc = stk_approx_candidates(X, W, b, cand_vals, cand_idxs, B, d, F, c, dtype, workspace, workspace_bytes, stream);
    if (rc) return rc;
    return stk_approx_forward(X, W, b, V, I, B, d, F, k, c, dtype, flags, workspace, workspace_bytes, stream);
  }
  pl.cand_vals = cand_vals;
  pl.cand_idxs = cand_idxs;
  if (workspace_bytes < pl.ws || (pl.ws && workspace == nullptr))
    return fail(STK_ENOSPACE, "workspace too small (need " + std::to_string(pl.ws) + " bytes)");
  return score_and_finish(pl, X, W, b, V, I, nullptr, B, d, F, k, dtype, 0u, nullptr, workspace,
                          static_cast<cudaStream_t>(stream));
}

int stk_shard_forward(const void* X, const void* W_shard, const float* b_shard, uint64_t* keys_out, int64_t B,
                      int64_t d, int64_t F_shard, int64_t k, int64_t index_offset, int dtype, int flags,
                      void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common("stk_shard_forward", B, d, F_shard, dtype);
  if (rc) return rc;
  if (k < 1 || k > 128) return fail(STK_EINVAL, "k out of range");
  if (index_offset < 0 || index_offset + F_shard > 0x7fffffffLL)
    return fail(STK_EINVAL, "index_offset + F_shard must fit int32 indices");
  if (!keys_out) return fail(STK_EINVAL, "keys_out is NULL");
  if (reinterpret_cast<uintptr_t>(keys_out) & 15) return fail(STK_EINVAL, "keys_out must be 16-byte aligned");
  // Only the sorted keys leave this call (no V/I).
  return encode(X, W_shard, b_shard, nullptr, nullptr, keys_out, B, d, F_shard, k, dtype, flags,
                (uint32_t)index_offset, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int stk_merge_keys(const uint64_t* lists, int64_t nlists, int64_t B, int64_t k, float* V, int32_t* I,
                   void* stream) {
  if (k < 1 || k > 128) return fail(STK_EINVAL, "k out of range");
  if (nlists < 1) return fail(STK_EINVAL, "nlists must be >= 1");
  if (B < 0) return fail(STK_EINVAL, "B must be >= 0");
  if (nlists > 0x7fffffff) return fail(STK_EINVAL, "nlists out of range");
  if (reinterpret_cast<uintptr_t>(lists) & 15) return fail(STK_EINVAL, "lists must be 16-byte aligned");
  return run_finish(list_len(k), finish_args(lists, (int)nlists, B, list_len(k), 0, B, k, V, I, nullptr, nullptr),
                    static_cast<cudaStream_t>(stream));
}

// Plan of the candidates path: one unit per 128-feature tile, list length L >= c.
int candidates_plan(const void* X, const void* W, int64_t B, int64_t d, int64_t F, int64_t c, int dtype, Plan* pl) {
  int sms = 0;
  int rc = device_sms(&sms);
  if (rc) return rc;
  pl->L = list_len(c);
  pl->tc = (dtype == STK_BF16 || dtype == STK_F16) && (d % 8 == 0) && (X == nullptr || aligned16(X)) &&
           (W == nullptr || aligned16(W));
  pl->grid = make_tile_grid(B, F);
  if (pl->grid.units > 0x7fffffff / 2) return fail(STK_EINVAL, "too many candidate tiles");
  pl->ctas = pl->grid.units < sms ? pl->grid.units : sms;
  pl->pilot = false;
  pl->shared_floor = false;  // each tile's own top c, not the row's top k
  pl->pair = false;
  pl->cand = false;
  pl->cand_vals = nullptr;
  pl->cand_idxs = nullptr;
  pl->cand_c = 0;
  pl->fp8 = false;
  pl->x_dtype = dtype;
  pl->w_scale = nullptr;
  pl->ws_q = 0;
  pl->pitch = pl->L;
  pl->ws_partials = (partial_bytes(pl->grid, pl->pitch) + 255) & ~size_t(255);
  pl->ws_app = ((size_t)pl->ctas * stk::kAppendBytesPerCta + 255) & ~size_t(255);
  pl->ws_sync = 0;
  pl->fin_fused = false;
  pl->tf32 = false;
  pl->ws_split = 0;
  pl->ws = pl->ws_partials + pl->ws_app;
  return STK_OK;
}

int stk_candidates_workspace_bytes(int64_t B, int64_t d, int64_t F, int64_t c, int dtype, size_t* bytes) {
  if (!bytes) return fail(STK_EINVAL, "bytes is NULL");
  int rc = check_common("stk_candidates_workspace_bytes", B, d, F, dtype);
  if (rc) return rc;
  if (!(c == 16 || c == 32 || c == 64 || c == 128))
    return fail(STK_EINVAL, "streamtopk_cuda_approx: unsupported c=" + std::to_string(c) + ". Supported: 16,32,64,128.");
  Plan pl;
  rc = candidates_plan(nullptr, nullptr, B, d, F, c, dtype, &pl);
  if (rc) return rc;
  *bytes = pl.ws;
  return STK_OK;
}

int stk_approx_candidates(const void* X, const void* W, const float* b, float* cand_vals, int32_t* cand_idxs,
                          int64_t B, int64_t d, int64_t F, int64_t c, int dtype, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = check_common("streamtopk_cuda_approx", B, d, F, dtype);
  if (rc) return rc;
  if (!(c == 16 || c == 32 || c == 64 || c == 128))
    return fail(STK_EINVAL, "streamtopk_cuda_approx: unsupported c=" + std::to_string(c) + ". Supported: 16,32,64,128.");
  Plan pl;
  rc = candidates_plan(X, W, B, d, F, c, dtype, &pl);
  if (rc) return rc;
  if (B == 0) return STK_OK;
  if (workspace_bytes < pl.ws || workspace == nullptr)
    return fail(STK_ENOSPACE, "workspace too small (need " + std::to_string(pl.ws) + " bytes)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint64_t* partials = static_cast<uint64_t*>(workspace);
  uint64_t* app = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + pl.ws_partials);
  // Every tile keeps its best L >= c scores per row (k = c); no threshold floor.
  rc = pl.tc ? run_fused(pl, X, W, b, partials, app, B, d, F, c, dtype, 0u, nullptr, s)
             : run_simt(pl, X, W, b, partials, app, B, d, F, c, dtype, 0u, s);
  if (rc) return rc;
  cudaError_t e = stk::launch_candidates_out(partials, pl.L, pl.grid.m_tiles, pl.grid.segs, B, (int)c, cand_vals,
                                             cand_idxs, s);
  if (e != cudaSuccess) return cuda_fail(e, "candidates_out_kernel launch");
  return STK_OK;
}

int stk_decode_forward(const float* V, const int32_t* I, const void* W_dec, const float* b_dec, float* out, int64_t B,
                       int64_t k, int64_t F, int64_t d, int dtype, void* stream) {
  if (dtype != STK_F32 && dtype != STK_F16 && dtype != STK_BF16)
    return fail(STK_EINVAL, "stk_decode_forward: W_dec dtype must be fp32, fp16, or bf16");
  if (B < 0 || d < 1 || F < 1 || k < 1 || k > 1024)
    return fail(STK_EINVAL, "stk_decode_forward: need B >= 0, d >= 1, F >= 1 and 1 <= k <= 1024");
  if (F > 0x7fffffffLL) return fail(STK_EINVAL, "stk_decode_forward: F must fit int32 indices");
  if (d % (dtype == STK_F32 ? 4 : 8) != 0)
    return fail(STK_EINVAL, "stk_decode_forward: d must be a multiple of 8 (fp16/bf16) or 4 (fp32)");
  if (B == 0) return STK_OK;
  if (!V || !I || !W_dec || !out || !aligned16(W_dec) || !aligned16(out) || (b_dec && !aligned16(b_dec)))
    return fail(STK_EINVAL, "stk_decode_forward: null or unaligned (16-byte) pointer");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaErrorInvalidValue;
  if (dtype == STK_F32) e = stk::launch_decode(V, I, static_cast<const float*>(W_dec), b_dec, out, B, (int)k, F, d, s);
  if (dtype == STK_F16) e = stk::launch_decode(V, I, static_cast<const __half*>(W_dec), b_dec, out, B, (int)k, F, d, s);
  if (dtype == STK_BF16)
    e = stk::launch_decode(V, I, static_cast<const __nv_bfloat16*>(W_dec), b_dec, out, B, (int)k, F, d, s);
  if (e != cudaSuccess) return cuda_fail(e, "decode_kernel launch");
  return STK_OK;
}

int stk_profile_begin(int64_t max_launches) {
  if (max_launches < 1) return fail(STK_EINVAL, "max_launches must be >= 1");
  std::lock_guard<std::mutex> lk(g_prof.mu);
  for (cudaEvent_t e : g_prof.ev) cudaEventDestroy(e);
  g_prof.ev.assign((size_t)max_launches * 2, nullptr);
  g_prof.kind.assign((size_t)max_launches, 0);
  for (auto& e : g_prof.ev) {
    cudaError_t r = cudaEventCreate(&e);
    if (r != cudaSuccess) return cuda_fail(r, "cudaEventCreate");
  }
  g_prof.used = 0;
  g_prof.on = true;
  return STK_OK;
}

int stk_profile_end(double* ms_by_kind, int64_t* launches_by_kind) {
  if (!ms_by_kind || !launches_by_kind) return fail(STK_EINVAL, "null output");
  std::lock_guard<std::mutex> lk(g_prof.mu);
  for (int i = 0; i < kProfKinds; ++i) {
    ms_by_kind[i] = 0.0;
    launches_by_kind[i] = 0;
  }
  int rc = STK_OK;
  for (size_t j = 0; j < g_prof.used; j += 2) {
    cudaError_t r = cudaEventSynchronize(g_prof.ev[j + 1]);
    float ms = 0.f;
    if (r == cudaSuccess) r = cudaEventElapsedTime(&ms, g_prof.ev[j], g_prof.ev[j + 1]);
    if (r != cudaSuccess) {
      rc = cuda_fail(r, "stk_profile_end");
      break;
    }
    const int k = g_prof.kind[j / 2];
    ms_by_kind[k] += ms;
    launches_by_kind[k] += 1;
  }
  for (cudaEvent_t e : g_prof.ev) cudaEventDestroy(e);
  g_prof.ev.clear();
  g_prof.kind.clear();
  g_prof.used = 0;
  g_prof.on = false;
  return rc;
}

int stk_device_error(void* stream, unsigned* code) {
  if (!code) return fail(STK_EINVAL, "code is NULL");
  cudaError_t e = stk::read_and_clear_device_error(code, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "stk_device_error");
  if (*code) {
    char buf[96];
    std::snprintf(buf, sizeof buf, "device error code %u (a bounded wait in a kernel ran out)", *code);
    g_err = buf;
    return STK_EDEVICE;
  }
  return STK_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Direct GPU-to-GPU exchange for the F-sharded encode.
// ---------------------------------------------------------------------------
struct stk_exchange {
  stk::ExchangeDev dev;
  int device;
  int L;
  void* mapped[stk::kMaxWorld];  // IPC mapping bases of the peers' allocations
};

namespace {

// recv [2][world][max_rows][L] keys, flag [2][world][max_rows] u64, state (256 B).
struct ExchangeLayout {
  size_t recv, flag, state, total;
};

ExchangeLayout exchange_layout(int world, int64_t max_rows, int L) {
  ExchangeLayout x;
  x.recv = 0;
  x.flag = (size_t(2) * world * max_rows * L * 8 + 255) & ~size_t(255);
  x.state = x.flag + ((size_t(2) * world * max_rows * 8 + 255) & ~size_t(255));
  x.total = x.state + 256;
  return x;
}

int exchange_check(int world, int64_t max_rows, int64_t k) {
  if (world < 1 || world > stk::kMaxWorld)
    return fail(STK_EINVAL, "world must be in [1, " + std::to_string(stk::kMaxWorld) + "]");
  if (max_rows < 1 || max_rows > (int64_t(1) << 24)) return fail(STK_EINVAL, "max_rows out of range");
  if (k < 1 || k > 128) return fail(STK_EINVAL, "k out of range");
  return STK_OK;
}

}  // namespace

extern "C" {

int stk_exchange_bytes(int world, int64_t max_rows, int64_t k, size_t* bytes) {
  if (!bytes) return fail(STK_EINVAL, "bytes is NULL");
  int rc = exchange_check(world, max_rows, k);
  if (rc) return rc;
  *bytes = exchange_layout(world, max_rows, list_len(k)).total;
  return STK_OK;
}

int stk_exchange_create(int rank, int world, int64_t max_rows, int64_t k, void* buffer, size_t bytes,
                        double wait_seconds, stk_exchange** out) {
  if (!out) return fail(STK_EINVAL, "out is NULL");
  *out = nullptr;
  int rc = exchange_check(world, max_rows, k);
  if (rc) return rc;
  if (rank < 0 || rank >= world) return fail(STK_EINVAL, "rank out of range");
  if (!(wait_seconds > 0.0 && wait_seconds <= 600.0)) return fail(STK_EINVAL, "wait_seconds must be in (0, 600]");
  const int L = list_len(k);
  const ExchangeLayout lay = exchange_layout(world, max_rows, L);
  if (!buffer || bytes < lay.total)
    return fail(STK_ENOSPACE, "exchange buffer too small (need " + std::to_string(lay.total) + " bytes)");
  if (reinterpret_cast<uintptr_t>(buffer) % 256) return fail(STK_EINVAL, "exchange buffer must be 256-byte aligned");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  char* base = static_cast<char*>(buffer);
  // Flags and the step start at zero; synchronous, so that no peer can
  // store into the buffer before it is cleared.
  e = cudaMemset(base + lay.flag, 0, lay.total - lay.flag);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "exchange buffer clear");
  stk_exchange* x = new (std::nothrow) stk_exchange();
  if (!x) return fail(STK_ENOSPACE, "out of host memory");
  x->device = device;
  x->L = L;
  x->dev.recv = reinterpret_cast<uint64_t*>(base + lay.recv);
  x->dev.flag = reinterpret_cast<unsigned long long*>(base + lay.flag);
  x->dev.state = reinterpret_cast<unsigned long long*>(base + lay.state);
  x->dev.rank = rank;
  x->dev.world = world;
  x->dev.max_rows = max_rows;
  x->dev.wait_ns = (unsigned long long)(wait_seconds * 1e9);
  x->dev.peer_recv[rank] = x->dev.recv;
  x->dev.peer_flag[rank] = x->dev.flag;
  *out = x;
  return STK_OK;
}

int stk_exchange_ipc_handle(const stk_exchange* x, void* handle, int64_t* offset) {
  if (!x || !handle || !offset) return fail(STK_EINVAL, "null argument");
  AddressRangeFn range = address_range();
  if (!range) return fail(STK_ECUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr alloc_base = 0;
  size_t alloc_size = 0;
  CUresult r = range(&alloc_base, &alloc_size, reinterpret_cast<CUdeviceptr>(x->dev.recv));
  if (r != CUDA_SUCCESS) return fail(STK_ECUDA, "cuMemGetAddressRange failed (CUresult " + std::to_string(r) + ")");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(alloc_base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof h);
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(x->dev.recv) - alloc_base);
  return STK_OK;
}

int stk_exchange_connect(stk_exchange* x, const void* handles, const int64_t* offsets) {
  if (!x || !handles || !offsets) return fail(STK_EINVAL, "null argument");
  const ExchangeLayout lay = exchange_layout(x->dev.world, x->dev.max_rows, x->L);
  for (int p = 0; p < x->dev.world; ++p) {
    if (p == x->dev.rank || x->mapped[p]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + (size_t)p * STK_IPC_HANDLE_BYTES, sizeof h);
    void* m = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&m, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, ("cudaIpcOpenMemHandle (rank " + std::to_string(p) + ")").c_str());
    x->mapped[p] = m;
    char* peer = static_cast<char*>(m) + offsets[p];
    x->dev.peer_recv[p] = reinterpret_cast<uint64_t*>(peer + lay.recv);
    x->dev.peer_flag[p] = reinterpret_cast<unsigned long long*>(peer + lay.flag);
  }
  return STK_OK;
}

int stk_exchange_forward(stk_exchange* x, const void* X, const void* W_shard, const float* b_shard, float* V,
                         int32_t* I, int64_t B, int64_t d, int64_t F_shard, int64_t k, int64_t index_offset,
                         int dtype, int flags, void* workspace, size_t workspace_bytes, void* stream) {
  if (!x) return fail(STK_EINVAL, "exchange is NULL");
  for (int p = 0; p < x->dev.world; ++p)
    if (!x->dev.peer_recv[p]) return fail(STK_EINVAL, "exchange is not connected");
  // An empty shard (F_shard == 0) still publishes (empty lists): every rank's
  // final merge waits for the rows of all ranks.
  int rc = check_common("stk_exchange_forward", B, d, F_shard > 0 ? F_shard : 1, dtype);
  if (rc) return rc;
  if (k < 1 || k > 128 || list_len(k) != x->L) return fail(STK_EINVAL, "k does not match the exchange");
  if (B > x->dev.max_rows) return fail(STK_EINVAL, "B exceeds the exchange's max_rows");
  if (index_offset < 0 || index_offset + F_shard > 0x7fffffffLL)
    return fail(STK_EINVAL, "index_offset + F_shard must fit int32 indices");
  Plan pl;
  if (F_shard > 0) {
    rc = plan(X, W_shard, B, d, F_shard, k, dtype, flags, &pl);
    if (rc) return rc;
  }
  if (B == 0) return STK_OK;
  if (F_shard > 0 && (workspace_bytes < pl.ws || (pl.ws && workspace == nullptr)))
    return fail(STK_ENOSPACE, "workspace too small (need " + std::to_string(pl.ws) + " bytes)");
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (device != x->device) return fail(STK_EINVAL, "current device is not the exchange's device");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (F_shard > 0)
    return score_and_finish(pl, X, W_shard, b_shard, V, I, nullptr, B, d, F_shard, k, dtype, (uint32_t)index_offset,
                            &x->dev, workspace, s);
  // Empty shard: publish empty lists (every rank's finish waits for all ranks).
  return run_finish(x->L, finish_args(nullptr, 0, 0, x->L, 0, B, k, V, I, nullptr, &x->dev), s);
}

int stk_exchange_destroy(stk_exchange* x) {
  if (!x) return STK_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(x->device);
  int rc = STK_OK;
  for (int p = 0; p < stk::kMaxWorld; ++p) {
    if (!x->mapped[p]) continue;
    cudaError_t e = cudaIpcCloseMemHandle(x->mapped[p]);
    if (e != cudaSuccess && rc == STK_OK) rc = cuda_fail(e, "cudaIpcCloseMemHandle");
  }
  cudaSetDevice(prev);
  delete x;
  return rc;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Pipelined exact encode: batch after batch of one shape, one launch per batch.
// The score kernel of batch s also finishes batch s - 1: its four epilogue
// warps select and write the previous batch's rows from the lists that batch
// left, while the CTA's producer streams the first W_enc tile (they would wait
// for it anyway).  The finish step (grid barrier, row selection) then costs
// nothing on the critical path, and the lists of consecutive batches live in
// the two halves of the pipeline's workspace.  A batch's V / I are complete
// once the next batch has been submitted, or after stk_pipeline_flush (a
// standalone finish kernel for the last batch).  Shapes whose units are not
// all resident at once (several rounds of units per CTA, CTA pairs), or
// unaligned operands, or k > 64, run as stk_exact_forward does (complete at once).
// ---------------------------------------------------------------------------
struct stk_pipeline {
  int64_t B, d, F, k;
  int dtype, flags, device;
  char* ws;
  size_t half;                 // bytes of one half of the workspace
  unsigned long long step;     // batches submitted so far
  bool piped;                  // the shape pipelines (one unit per CTA on the tcgen05 path)
  bool pending;                // a batch waits for its finish
  stk::FinishArgs pending_fin; // its finish (lists in its half, its V / I)
  int pending_L;
  int pending_half;
  bool clean[2];               // the half's sync region is zero (its last batch's finish cleared it)
  stk_exchange* ex;            // F-sharded encode: the peer exchange of the finish (else null)
  int64_t index_offset;        // F-sharded encode: this rank's first feature
};

namespace {
int pipeline_plan(const void* X, const void* W, const stk_pipeline* pp, Plan* pl) {
  return plan(X, W, pp->B, pp->d, pp->F, pp->k, pp->dtype, pp->flags | STK_FLAG_SEPARATE_FINISH, pl);
}
// L = 128 (k > 64) is left out: its finish takes longer than the first tile's
// loads and would delay the score kernel.
bool pipelines(const Plan& pl) {
  return pl.tc && !pl.pair && !pl.cand && !pl.fp8 && pl.L <= 64 && pl.grid.units <= pl.ctas;
}

int pipeline_check(int64_t B, int64_t d, int64_t F, int64_t k, int dtype, int flags) {
  int rc = check_common("stk_pipeline", B, d, F, dtype);
  if (rc) return rc;
  if (!(k >= 1 && k <= F)) return fail(STK_EINVAL, "k out of range");
  if (d > 4096 && !(flags & STK_FLAG_ANY_D)) return fail(STK_EINVAL, "d exceeds D_MAX=4096");
  if (!(flags & STK_FLAG_ANY_K) && !ref_k(k))
    return fail(STK_EINVAL, "streamtopk_cuda_exact: unsupported k=" + std::to_string(k) +
                                ". Supported: 1,2,4,8,16,32,64,128.");
  if (k > 128) return fail(STK_EINVAL, "stk_pipeline: k must be <= 128");
  if (B < 1) return fail(STK_EINVAL, "stk_pipeline: B must be >= 1");
  return STK_OK;
}

// Bytes of one half: the larger of the pipelined plan's and the one-call
// plan's workspace (a batch that cannot pipeline runs as one call in a half).
int pipeline_half(int64_t B, int64_t d, int64_t F, int64_t k, int dtype, int flags, size_t* half) {
  Plan a, b;
  const int f = flags | (dtype == STK_F32 ? STK_FLAG_TF32 : 0);
  int rc = plan(nullptr, nullptr, B, d, F, k, dtype, f | STK_FLAG_SEPARATE_FINISH, &a);
  if (rc) return rc;
  rc = plan(nullptr, nullptr, B, d, F, k, dtype, f, &b);
  if (rc) return rc;
  *half = ((a.ws > b.ws ? a.ws : b.ws) + 255) & ~size_t(255);
  if (*half == 0) *half = 256;
  return STK_OK;
}

int pipeline_device(const stk_pipeline* pp) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != pp->device) return fail(STK_EINVAL, "current device is not the pipeline's device");
  return STK_OK;
}

int pipeline_flush(stk_pipeline* pp, cudaStream_t s) {
  if (!pp->pending) return STK_OK;
  pp->pending = false;
  int rc = run_finish(pp->pending_L, pp->pending_fin, s);
  if (rc) return rc;
  if (pp->pending_fin.zero) pp->clean[pp->pending_half] = true;
  return STK_OK;
}
}  // namespace

extern "C" {

int stk_pipeline_workspace_bytes(int64_t B, int64_t d, int64_t F, int64_t k, int dtype, int flags, size_t* bytes) {
  if (!bytes) return fail(STK_EINVAL, "bytes is NULL");
  int rc = pipeline_check(B, d, F, k, dtype, flags);
  if (rc) return rc;
  size_t half = 0;
  rc = pipeline_half(B, d, F, k, dtype, flags, &half);
  if (rc) return rc;
  *bytes = 2 * half;
  return STK_OK;
}

int stk_pipeline_create(stk_pipeline** out, int64_t B, int64_t d, int64_t F, int64_t k, int dtype, int flags,
                        void* workspace, size_t workspace_bytes) {
  if (!out) return fail(STK_EINVAL, "out is NULL");
  *out = nullptr;
  int rc = pipeline_check(B, d, F, k, dtype, flags);
  if (rc) return rc;
  size_t half = 0;
  rc = pipeline_half(B, d, F, k, dtype, flags, &half);
  if (rc) return rc;
  if (workspace == nullptr || workspace_bytes < 2 * half || !aligned16(workspace))
    return fail(STK_ENOSPACE, "stk_pipeline_create: workspace too small or unaligned (need " +
                                  std::to_string(2 * half) + " bytes, 16-byte aligned)");
  Plan pl;
  stk_pipeline* pp = new stk_pipeline();
  pp->B = B;
  pp->d = d;
  pp->F = F;
  pp->k = k;
  pp->dtype = dtype;
  pp->flags = flags;
  cudaGetDevice(&pp->device);
  pp->ws = static_cast<char*>(workspace);
  pp->half = half;
  pp->step = 0;
  pp->pending = false;
  pp->pending_half = 0;
  pp->clean[0] = pp->clean[1] = false;
  pp->ex = nullptr;
  pp->index_offset = 0;
  rc = pipeline_plan(nullptr, nullptr, pp, &pl);
  if (rc) {
    delete pp;
    return rc;
  }
  pp->piped = pipelines(pl);
  *out = pp;
  return STK_OK;
}

int stk_pipeline_create_sharded(stk_pipeline** out, stk_exchange* x, int64_t B, int64_t d, int64_t F_shard,
                                int64_t k, int64_t index_offset, int dtype, int flags, void* workspace,
                                size_t workspace_bytes) {
  if (!out) return fail(STK_EINVAL, "out is NULL");
  *out = nullptr;
  if (!x) return fail(STK_EINVAL, "exchange is NULL");
  for (int p = 0; p < x->dev.world; ++p)
    if (!x->dev.peer_recv[p]) return fail(STK_EINVAL, "exchange is not connected");
  if (k < 1 || k > 128 || list_len(k) != x->L) return fail(STK_EINVAL, "k does not match the exchange");
  if (B > x->dev.max_rows) return fail(STK_EINVAL, "B exceeds the exchange's max_rows");
  if (F_shard < 1) return fail(STK_EINVAL, "stk_pipeline_create_sharded: F_shard must be >= 1");
  if (index_offset < 0 || index_offset + F_shard > 0x7fffffffLL)
    return fail(STK_EINVAL, "index_offset + F_shard must fit int32 indices");
  int device = 0;
  cudaGetDevice(&device);
  if (device != x->device) return fail(STK_EINVAL, "current device is not the exchange's device");
  int rc = stk_pipeline_create(out, B, d, F_shard, k, dtype, flags | STK_FLAG_ANY_K | STK_FLAG_ANY_D, workspace,
                               workspace_bytes);
  if (rc) return rc;
  (*out)->ex = x;
  (*out)->index_offset = index_offset;
  return STK_OK;
}

int stk_pipeline_submit(stk_pipeline* pp, const void* X, const void* W, const float* b, float* V, int32_t* I,
                        void* stream) {
  if (!pp) return fail(STK_EINVAL, "pipeline is NULL");
  int rc = pipeline_device(pp);
  if (rc) return rc;
  if (!X || !W || !b || !V || !I) return fail(STK_EINVAL, "stk_pipeline_submit: null pointer");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  Plan pl;
  rc = pipeline_plan(X, W, pp, &pl);
  if (rc) return rc;
  const int h = (int)(pp->step & 1ull);
  char* half = pp->ws + (size_t)h * pp->half;
  if (!pipelines(pl) || pl.ws > pp->half) {
    // Not pipelined: the pending batch first, then this one as one call.
    rc = pipeline_flush(pp, s);
    if (rc) return rc;
    if (pp->ex) {
      Plan one;
      rc = plan(X, W, pp->B, pp->d, pp->F, pp->k, pp->dtype, pp->flags, &one);
      if (rc) return rc;
      if (one.ws > pp->half) return fail(STK_ENOSPACE, "stk_pipeline_submit: workspace too small");
      rc = score_and_finish(one, X, W, b, V, I, nullptr, pp->B, pp->d, pp->F, pp->k, pp->dtype,
                            (uint32_t)pp->index_offset, &pp->ex->dev, half, s);
    } else {
      rc = encode(X, W, b, V, I, nullptr, pp->B, pp->d, pp->F, pp->k, pp->dtype, pp->flags, 0u, half, pp->half, s);
    }
    if (rc) return rc;
    pp->clean[h] = false;
    ++pp->step;
    return STK_OK;
  }
  uint64_t* partials = reinterpret_cast<uint64_t*>(half);
  uint64_t* app = reinterpret_cast<uint64_t*>(half + pl.ws_partials);
  const stk::FinishArgs fa = finish_args(partials, pl.grid.segs, (int64_t)pl.grid.m_tiles * stk::kRows, pl.pitch,
                                         pl.pitch - pl.L, pp->B, pp->k, V, I, nullptr,
                                         pp->ex ? &pp->ex->dev : nullptr);
  stk::FinishArgs fz = fa;  // this batch's finish also clears its sync region
  if (pl.ws_sync) {
    fz.zero = reinterpret_cast<uint32_t*>(half + pl.ws_partials + pl.ws_app);
    fz.zero_words = (int64_t)(pl.ws_sync / 4);
  }
  const bool merge_prev = pp->pending && pp->pending_L == pl.L;
  if (pp->pending && !merge_prev) {
    rc = pipeline_flush(pp, s);
    if (rc) return rc;
  }
  pl.presync = pp->clean[h];
  rc = run_fused(pl, X, W, b, partials, app, pp->B, pp->d, pp->F, pp->k, pp->dtype, (uint32_t)pp->index_offset,
                 nullptr, s, merge_prev ? &pp->pending_fin : nullptr);
  if (rc) return rc;
  if (merge_prev && pp->pending_fin.zero) pp->clean[pp->pending_half] = true;
  pp->clean[h] = false;
  pp->pending = true;
  pp->pending_fin = fz;
  pp->pending_half = h;
  pp->pending_L = pl.L;
  ++pp->step;
  return STK_OK;
}

int stk_pipeline_flush(stk_pipeline* pp, void* stream) {
  if (!pp) return fail(STK_EINVAL, "pipeline is NULL");
  int rc = pipeline_device(pp);
  if (rc) return rc;
  return pipeline_flush(pp, static_cast<cudaStream_t>(stream));
}

int stk_pipeline_pipelined(const stk_pipeline* pp) { return pp && pp->piped ? 1 : 0; }

int stk_pipeline_destroy(stk_pipeline* pp) {
  delete pp;
  return STK_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Exact encode without any allocation, for callers that cannot allocate device
// memory at all: code that runs inside another allocator's hooks, plugins whose
// host process owns every allocation, and embedded / real-time callers whose
// memory is fixed up front.  Instead of a caller-provided workspace it uses the
// built-in scratch array below.
//
//  * Size: kNoAllocScratchBytes (24 MiB).  That covers one M tile (B <= 128)
//    with k <= 64 at any F and d on a 148-SM B200; larger shapes are rejected
//    with STK_ENOSPACE and a message giving both sizes.
//  * The array is a file-scope __device__ variable, so every GPU on which this
//    library's module is loaded holds its 24 MiB until the process exits.
//  * Host code cannot use the array's name as a device address; its address is
//    looked up with cudaGetSymbolAddress once per device, with that device
//    current, on the first call made on that device (so make that first call
//    before any stream capture).
//  * All calls share the one array, which keeps the last call's contents: the
//    parts that must start at zero are cleared by the call itself (a
//    cudaMemsetAsync on the caller's stream), everything else is written before
//    it is read.  Calls whose kernels overlap on the GPU (two streams, or two
//    threads) race on the array; serialise them.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(24) << 20;
}  // namespace

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
void* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of g_noalloc_scratch on the current device (set up once).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(STK_EINVAL, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return STK_OK;
}
}  // namespace

extern "C" int stk_exact_forward_noalloc(const void* X, const void* W, const float* b, float* V, int32_t* I,
                                         int64_t B, int64_t d, int64_t F, int64_t k, int dtype, int flags,
                                         void* stream) {
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // Argument errors are reported by stk_exact_forward with the usual messages;
  // it also checks this call's own plan (flags included) against the array.
  rc = stk_exact_forward(X, W, b, V, I, B, d, F, k, dtype, flags, scratch, kNoAllocScratchBytes, stream);
  if (rc == STK_ENOSPACE) {
    Plan pl;
    if (plan(X, W, B, d, F, k, dtype, flags, &pl) == STK_OK)
      return fail(STK_ENOSPACE, "stk_exact_forward_noalloc: this shape needs " + std::to_string(pl.ws) +
                                    " bytes of scratch; the built-in scratch holds " +
                                    std::to_string(kNoAllocScratchBytes) +
                                    " bytes (use stk_exact_forward with a caller-allocated workspace)");
  }
  return rc;
}
