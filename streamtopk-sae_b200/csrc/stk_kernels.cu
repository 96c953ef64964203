// Kernels of the B200 streaming top-k SAE encoder.
//
//   fused_topk_kernel  scores = X @ W^T + b on tcgen05 (TMEM accumulators, TMA
//                      + mbarrier pipeline), bias add and running per-row top-k
//                      in the epilogue; the (B, F) score matrix never leaves
//                      the SM.  Replaces the reference's pass-1 tile kernels
//                      (streamtopk_sae/csrc/cuda/streamtopk_exact.cu:58-187,
//                      208-411) and single-pass kernel (:506-638).
//   simt_topk_kernel   the same contract with fp32 SIMT FMA: fp32 inputs and
//                      shapes TMA cannot describe (d not a multiple of 8,
//                      unaligned bases).
//   finish_kernel      per-row top-k of several sorted key lists (the units'
//                      lists of a score kernel that did not finish its rows
//                      itself, or lists all-gathered from other GPUs), with the
//                      optional cross-GPU exchange (stk_finish.cuh).  The fused
//                      kernel runs the same finish in its tail when all of its
//                      units are resident at once.  Replaces the reference's
//                      pass-2 merge (streamtopk_exact.cu:429-499).
//
// Work decomposition shared by the two score kernels: the batch is cut into
// M tiles of 128 rows; F is cut into `segs` contiguous feature ranges whose
// bounds are multiples of 32.  A unit is (range, M tile); persistent CTAs walk
// units u = blockIdx.x, blockIdx.x + gridDim.x, ... with
// range = u / m_tiles, M tile = u % m_tiles, so CTAs running at the same time
// read the same W rows (L2 reuse across M tiles).  Each unit writes its best
// L keys per row to partials[u][row][0..L).
#include "stk_kernels.cuh"

namespace stk {
__device__ unsigned int g_device_error = 0;
}  // namespace stk

#include "stk_finish.cuh"

namespace stk {

__device__ __forceinline__ void unit_range(const UnitGrid& g, int u, int& m, int64_t& f_begin, int64_t& f_end) {
  const int seg = u / g.m_tiles;
  m = u - seg * g.m_tiles;
  const int64_t q = g.quantum > 1 ? g.quantum : 1;  // balanced bounds in multiples of q chunks
  const int64_t nq = (g.nchunks + q - 1) / q;
  const int64_t c0 = g.fixed_chunks > 0 ? (int64_t)seg * g.fixed_chunks : q * ((int64_t)seg * nq / g.segs);
  const int64_t c1 = g.fixed_chunks > 0 ? min(c0 + g.fixed_chunks, g.nchunks)
                                        : min(q * ((int64_t)(seg + 1) * nq / g.segs), g.nchunks);
  f_begin = c0 * 32;
  f_end = c1 * 32;  // may pass F by < 32 on the last range; masked in the epilogue
}

// Loads the bias for 32 consecutive features starting at f (zero past F).
__device__ __forceinline__ void load_bias32(const float* __restrict__ bias, int64_t f, int64_t F, bool vec_ok,
                                            float (&bv)[32]) {
  if (vec_ok && f + 32 <= F) {
    const float4* p = reinterpret_cast<const float4*>(bias + f);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 t = __ldg(p + q);
      bv[4 * q + 0] = t.x;
      bv[4 * q + 1] = t.y;
      bv[4 * q + 2] = t.z;
      bv[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) bv[j] = (f + j < F) ? __ldg(bias + f + j) : 0.f;
  }
}

__device__ __forceinline__ uint32_t feature_mask(int64_t f, int64_t F) {
  const int64_t n = F - f;
  return n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
}

// Writes the top lists of the 32 rows of this warp (warp-cooperative,
// coalesced); row r's list starts at out_unit[r * pitch].
template <int L>
__device__ __forceinline__ void store_partials(uint32_t top, uint64_t* __restrict__ out_unit, int pitch,
                                               int warp_row0, int lane) {
  __syncwarp();
#pragma unroll 1
  for (int rr = 0; rr < 32; ++rr) {
    const int r = warp_row0 + rr;
#pragma unroll
    for (int e = 0; e < L / 32; ++e)
      out_unit[(int64_t)r * pitch + e * 32 + lane] = top_slot(top, e * 32 + lane, r);
  }
  __syncwarp();
}

// Copies this thread's row list from tensor memory (TOPT) to row_out
// (16-byte aligned), 16 keys per warp-wide TMEM load.
template <int L>
__device__ __forceinline__ void store_list_tmem(uint32_t tlist, uint64_t* __restrict__ row_out) {
#pragma unroll 1
  for (int c = 0; c < 2 * L; c += 32) {
    uint32_t v[32];
    tmem_ld32(tlist + c, v);
    tmem_wait_ld(v);
    ulonglong2* d = reinterpret_cast<ulonglong2*>(row_out + c / 2);
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] = make_ulonglong2(col_key(v, 2 * j), col_key(v, 2 * j + 1));
  }
}

// Width of the tile starting at ft in the unit range [fb, fe).  (A schedule
// that ended long units with a narrow tile, to shorten the exposed epilogue of
// the last tile, measured slower at cfg3: its extra tile re-reads all of X.)
template <int NT>
__device__ __forceinline__ int tile_width(int64_t ft, int64_t fb, int64_t fe) {
  (void)fb;
  return (int)min((int64_t)NT, fe - ft);
}

// The j-th unit of this CTA.  One CTA per unit: u = blockIdx.x + j * gridDim.x.
// CTA pairs (PAIR, a 2-CTA cluster sharing the MMA): pair-unit pu = cluster +
// j * clusters covers one feature range of two adjacent M tiles, the CTA of
// rank r taking M tile 2 * (pu % (m_tiles / 2)) + r (m_tiles is even), so a
// CTA's units are still units u = range * m_tiles + m of the plain grid.
template <bool PAIR>
__device__ __forceinline__ bool unit_at(const UnitGrid& g, int j, uint32_t rank, int& u, int& m, int64_t& fb,
                                        int64_t& fe) {
  if constexpr (PAIR) {
    const int mp_tiles = g.m_tiles / 2;
    const int pu = (int)(blockIdx.x / 2) + j * (int)(gridDim.x / 2);
    if (pu >= g.segs * mp_tiles) return false;
    u = (pu / mp_tiles) * g.m_tiles + 2 * (pu % mp_tiles) + (int)rank;
  } else {
    u = (int)blockIdx.x + j * (int)gridDim.x;
    if (u >= g.units) return false;
  }
  unit_range(g, u, m, fb, fe);
  return true;
}

// Walks the tiles of this CTA: its units (unit_at), tiles of tile_width<NT>
// features within each unit's range.
template <int NT, bool PAIR>
struct TileWalk {
  int j, u, m;
  int64_t fb, fe, ft;
  bool ok;
  __device__ __forceinline__ void start(const UnitGrid& g, uint32_t rank) {
    j = 0;
    ok = unit_at<PAIR>(g, 0, rank, u, m, fb, fe);
    ft = fb;
  }
  __device__ __forceinline__ bool valid(const UnitGrid&) const { return ok; }
  __device__ __forceinline__ bool first_of_unit() const { return ft == fb; }
  __device__ __forceinline__ int width() const { return tile_width<NT>(ft, fb, fe); }
  __device__ __forceinline__ bool last_of_unit() const { return ft + width() >= fe; }
  __device__ __forceinline__ void next(const UnitGrid& g, uint32_t rank) {
    ft += width();
    if (ft >= fe) {
      ++j;
      ok = unit_at<PAIR>(g, j, rank, u, m, fb, fe);
      ft = fb;
    }
  }
};

__device__ __forceinline__ void epilogue_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpilogueWarps * 32) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Lower bound of a row's k-th largest sampled score from its histogram:
// the lower edge of the highest bin at which the count from the top reaches
// k.  Returns false when fewer than k samples lie within 256 bins of the top.
__device__ __forceinline__ bool pilot_bound(const uint32_t* __restrict__ hist, uint32_t top_bin, int k, float& lb) {
  // First look: the 64 bins ending at the 4-aligned group that holds top_bin,
  // fetched as 16 independent 16-byte loads (one memory round trip), scanned
  // from top_bin down with predicated adds.
  const int hi = (int)(top_bin | 3u);
  const int base = hi - 63;
  uint32_t c[64];
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    uint4 t = make_uint4(0u, 0u, 0u, 0u);
    if (base + 4 * q >= 0) t = __ldcg(reinterpret_cast<const uint4*>(hist + base + 4 * q));
    c[4 * q + 0] = t.x;
    c[4 * q + 1] = t.y;
    c[4 * q + 2] = t.z;
    c[4 * q + 3] = t.w;
  }
  uint32_t total = 0;
  int found = -1;
#pragma unroll
  for (int q = 63; q >= 0; --q) {
    const bool in = base + q <= (int)top_bin;
    total += in ? c[q] : 0u;
    if (found < 0 && total >= (uint32_t)k) found = base + q;
  }
  if (found >= 0) {
    lb = order_float((uint32_t)found << (32 - kPilotBits));
    return true;
  }
  // Rare: the k-th sampled score lies deeper; continue 32 bins at a time.
#pragma unroll 1
  for (int round = 0; round < 6 && base - 32 * round > 0; ++round) {
    const int b0 = base - 1 - 32 * round;  // scan b0, b0 - 1, ...
#pragma unroll
    for (int q = 0; q < 32; ++q) c[q] = b0 - q >= 0 ? __ldcg(hist + b0 - q) : 0u;
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      total += c[q];
      if (total >= (uint32_t)k) {
        lb = order_float((uint32_t)(b0 - q) << (32 - kPilotBits));
        return true;
      }
    }
  }
  return false;
}

// One 32-column chunk of scores of an accumulator buffer (this warp's 32
// lanes): the accumulator itself, or for TF32 the sum of the Xh*Wh accumulator
// and the cross-term accumulator NT columns after it.
template <bool TF32, int NT>
__device__ __forceinline__ void load_chunk(uint32_t tcol, int c, uint32_t (&v)[32]) {
  tmem_ld32(tcol + (uint32_t)(c * 32), v);
  if constexpr (TF32) {
    uint32_t u[32];
    tmem_ld32(tcol + (uint32_t)(NT + c * 32), u);
    tmem_wait_ld(v);
    tmem_wait_ld(u);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(u[j]));
  } else {
    tmem_wait_ld(v);
  }
}

// b[i] for a runtime i < N without dynamic register indexing.
template <int N>
__device__ __forceinline__ float pick(const float (&b)[N], int i) {
  float v = b[0];
#pragma unroll
  for (int c = 1; c < N; ++c) v = (i == c) ? b[c] : v;
  return v;
}

// Score of column j of a chunk (lane j's bias bl and, for FP8, scale sl):
// the accumulator plus the bias, or for FP8 the dequantized product
// x_scale * w_scale * acc plus the bias.
template <bool FP8>
__device__ __forceinline__ float chunk_score(uint32_t acc_bits, float bl, float sl, float sxr, int j) {
  const float b = __shfl_sync(0xffffffffu, bl, j);
  if constexpr (FP8)
    return fmaf(__uint_as_float(acc_bits), sxr * __shfl_sync(0xffffffffu, sl, j), b);
  else
    return __uint_as_float(acc_bits) + b;
}

// Bias of one tile: lane l holds bias[ft + 32 c + l] for chunk c (0 past F).
template <int NT>
__device__ __forceinline__ void load_bias_tile(const float* __restrict__ bias, int64_t ft, int w, int64_t F, int lane,
                                               float (&b)[NT / 32]) {
#pragma unroll
  for (int c = 0; c < NT / 32; ++c) {
    const int64_t f = ft + 32 * c + lane;
    b[c] = (32 * c < w && f < F) ? __ldg(bias + f) : 0.f;
  }
}

// ---------------------------------------------------------------------------
// Fused tcgen05 kernel.
//   warp 0: TMA producer        warp 1: TMEM owner + MMA issuer
//   warps 2..5: epilogue, warp w reads TMEM lanes 32*(w%4)..+31 (= batch rows)
// ---------------------------------------------------------------------------
// TF32 = false: 16-bit X / W, K = 64 per stage, 128-byte swizzle, warps 0 TMA,
// 1 MMA, 2-5 epilogue.  TF32 = true (fp32 inputs, 3-pass TF32): K = 16 per
// stage, 64-byte swizzle.  The tensor core reads an fp32 operand as TF32 by
// ignoring its low 13 mantissa bits, so the raw X and W tiles serve as the
// "hi" parts h = trunc13(v) as they are; a stage also holds X's residual
// X - trunc13(X) (precomputed once per call, second map) and W's residual,
// written next to the W tile by warps 2-3.  The MMA issuer accumulates Xh*Wh
// into one TMEM accumulator and Xh*Wl + Xl*Wh into a second one (kept apart so
// that the small terms do not add to the rounding of the large accumulator);
// the epilogue (warps 4-7) adds the two.  The dropped Xl*Wl term is below
// 2^-20 of |x||w|.
//
// MODE = kModeFP8: E4M3 X and W, kind::f8f6f4, K = 128 per 128-byte box (the
// 16-bit plan with one byte per element); the epilogue scales each score by
// its row's and feature's dequantization factors before the bias.
//
// MODE | kModePair: CTA pairs (2-CTA clusters).  The pair's first CTA issues
// tcgen05.mma.cta_group::2 with M = 256 (each CTA's 128 X rows, its own M
// tile) and N = NT (each CTA holds NT / 2 of the W tile's rows): every CTA
// loads half the W bytes per tile, and the accumulator of each CTA's rows
// lands in its own TMEM, read by its own epilogue as in the one-CTA kernel.
// Both CTAs' TMA loads count on the first CTA's full barrier (it alone waits
// on it and expects both CTAs' bytes); its commits arrive on both CTAs' empty
// and acc_full barriers; the second CTA's epilogue arrives remotely on the
// first CTA's acc_empty barrier (8 arrivals per phase).
template <int L, int NT, int STAGES, int A, bool APP_SMEM, bool TOPT, int MODE>
__global__ void __launch_bounds__((MODE & 3) == kModeTF32 ? kFusedThreads + 64 : kFusedThreads, 1)
    fused_topk_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_xl,
                      const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_w32,
                      const FusedParams p) {
  constexpr bool PAIR = (MODE & kModePair) != 0;
  using Cfg = FusedCfg<L, NT, STAGES, A, APP_SMEM, TOPT, PAIR>;
  constexpr bool TF32 = (MODE & 3) == kModeTF32;
  constexpr bool FP8 = (MODE & 3) == kModeFP8;
  constexpr bool CAND = (MODE & kModeCand) != 0;
  static_assert(!CAND || (!PAIR && !TF32 && !FP8 && !TOPT && L == 32), "candidate variant: 16-bit, k <= c <= 32");
  static_assert(!PAIR || (!TF32 && NT % 32 == 0), "CTA pairs: 16-bit or FP8 operands");
  constexpr int kSplitThreads = 64;                 // warps 2-3 (TF32)
  constexpr int kFirstEpiWarp = TF32 ? 4 : 2;
  constexpr uint32_t kWRowBytes = TF32 ? 64u : 128u;  // bytes of one W row in a stage
  constexpr int kKPerStage = TF32 ? 16 : FP8 ? 128 : 64;  // elements of K per 128-byte box
  // TMEM: two accumulator buffers (tile parity), each NT columns, or for TF32
  // each 2 x NT (Xh*Wh, then the cross terms).
  constexpr uint32_t kAccCols = TF32 ? 2 * NT : NT;
  constexpr uint32_t kTmemCols = (TF32 || TOPT) ? 512u : (uint32_t)Cfg::kTmemCols;
  static_assert(!TF32 || NT <= 128, "TF32 needs 4 x NT TMEM columns");
  static_assert(!TOPT || (!TF32 && NT + 2 * L <= 512), "TMEM lists need 2 x L columns beside the accumulators");
  // Accumulator buffers: two (the MMA of tile t + 1 overlaps the epilogue of
  // tile t) unless TMEM-resident lists leave room for one only (NT = 256 with
  // L = 128); then the TMA ring keeps filling during the epilogue and only the
  // MMA waits.
  constexpr int kAccBufs = (TOPT && 2 * kAccCols + 2 * L > 512) ? 1 : 2;
  static_assert(!TOPT || kAccBufs * kAccCols + 2 * L <= 512, "TMEM columns");
  constexpr uint32_t kListCol = kAccBufs * kAccCols;  // TOPT: the row lists' first column
  uint8_t* smem = stk_smem + ((1024u - (smem_u32(stk_smem) & 1023u)) & 1023u);
  uint64_t* top = reinterpret_cast<uint64_t*>(smem + Cfg::kTopOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint64_t* split_done = mma_done + 1;  // [STAGES], TF32 only
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(split_done + (TF32 ? STAGES : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* pilot_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // The merge kernel that follows waits for this grid's completion itself
  // (griddepcontrol.wait), so it may be scheduled right away.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], PAIR ? 2 * kEpilogueWarps : kEpilogueWarps);
    }
    mbar_init(mma_done, 1);
    if constexpr (TF32)
      for (int s = 0; s < STAGES; ++s) mbar_init(&split_done[s], kSplitThreads);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_x);
    if constexpr (TF32) tma_prefetch_desc(&tmap_xl);
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_w32);
  }
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // 0: the pair's MMA-issuing CTA
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers are initialised before any remote arrival
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const UnitGrid& g = p.grid;
  // Pipeline stages per tile: K blocks of kKPerStage elements, kSub per stage.
  const int num_kb = TF32 ? p.num_kb : (p.num_kb + Cfg::kSub - 1) / Cfg::kSub;
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_x = l2_policy_evict_last();
      const uint64_t pol_w = p.w_evict_first ? l2_policy_evict_first() : l2_policy_evict_normal();
      uint32_t it = 0;
      bool ok = true;
      int u, m;
      int64_t fb, fe;
      for (int j = 0; ok && unit_at<PAIR>(g, j, rank, u, m, fb, fe); ++j) {
        for (int64_t ft = fb, w = 0; ft < fe && ok; ft += w) {
          w = tile_width<NT>(ft, fb, fe);
          // Pairs: each CTA loads its X tile and NT / 2 W rows (the whole half
          // even for a narrow tile: columns past w are never read).
          const uint32_t bytes = PAIR ? 2u * Cfg::kStageBytes
                                      : Cfg::kSub * (Cfg::kXBytes + (uint32_t)w * kWRowBytes);
          for (int kb = 0; kb < num_kb; ++kb, ++it) {
            const int s = it % STAGES;
            if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            if (!PAIR || rank == 0) mbar_arrive_expect_tx(&full[s], bytes);
            // kSub K boxes: X boxes first, then the W boxes (a box past d
            // reads zeros and adds nothing).
            for (int h = 0; h < Cfg::kSub; ++h) {
              uint8_t* sx = smem + s * Cfg::kStageBytes + h * Cfg::kXBytes;
              uint8_t* sw = smem + s * Cfg::kStageBytes + Cfg::kSub * Cfg::kXBytes + h * Cfg::kWBytes;
              const int kx = (kb * Cfg::kSub + h) * kKPerStage;
              if constexpr (PAIR) {
                const uint32_t full0 = mapa_shared(smem_u32(&full[s]), 0u);
                tma_load_2d_pair(&tmap_x, full0, sx, kx, m * kRows, pol_x);
                tma_load_2d_pair(&tmap_w, full0, sw, kx, (int)ft + (int)rank * (NT / 2), pol_w);
              } else {
                tma_load_2d(&tmap_x, &full[s], sx, kx, m * kRows, pol_x);
                if constexpr (TF32) tma_load_2d(&tmap_xl, &full[s], sx + Cfg::kXBytes / 2, kx, m * kRows, pol_x);
                if (w == NT) {
                  tma_load_2d(&tmap_w, &full[s], sw, kx, (int)ft, pol_w);
                } else {
                  for (int q = 0; q < w / 32; ++q)
                    tma_load_2d(&tmap_w32, &full[s], sw + q * 32 * kWRowBytes, kx, (int)ft + 32 * q, pol_w);
                }
              }
            }
          }
        }
      }
      const uint32_t n = it < (uint32_t)STAGES ? it : (uint32_t)STAGES;
      if (!ok) {
        raise_device_error(kErrWaitTimeout);
        *abort_flag = 1;
        // Let the copies already issued land before the CTA can exit.  (A
        // pair's copies count on the first CTA's barrier: its MMA issuer
        // waits for them, or gives up too, and the pair meets at the final
        // cluster barrier.)
        if (!PAIR)
          for (uint32_t i0 = 0; i0 < n; ++i0) {
            const uint32_t i = it - 1 - i0;
            mbar_wait(&full[i % STAGES], (i / STAGES) & 1, nullptr);
          }
      }
      if constexpr (PAIR) {
        // The first CTA's last commits arrive on this CTA's empty barriers:
        // wait for them (bounded) so that none is still in flight at exit.
        for (uint32_t i0 = 0; i0 < n; ++i0) {
          const uint32_t i = it - 1 - i0;
          mbar_wait(&empty[i % STAGES], (i / STAGES) & 1, nullptr);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && (!PAIR || rank == 0)) {
      uint32_t it = 0, tile = 0;
      bool ok = true;
      int u, m;
      int64_t fb, fe;
      for (int j = 0; ok && unit_at<PAIR>(g, j, rank, u, m, fb, fe); ++j) {
        for (int64_t ft = fb, w = 0; ft < fe && ok; ft += w, ++tile) {
          w = tile_width<NT>(ft, fb, fe);
          const int a = (int)(tile % kAccBufs);
          if (!mbar_wait(&acc_empty[a], ((tile / kAccBufs) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)a * kAccCols;
          const uint32_t mma_m = PAIR ? 256u : 128u;
          const uint32_t mma_n = PAIR ? (uint32_t)NT : (uint32_t)w;
          const uint32_t idesc = TF32 ? make_idesc_tf32(128u, (uint32_t)w)
                                 : FP8  ? make_idesc_f16(0u, mma_m, mma_n)  // E4M3 x E4M3
                                        : make_idesc_f16((uint32_t)p.ab_format, mma_m, mma_n);
          for (int kb = 0; kb < num_kb; ++kb, ++it) {
            const int s = it % STAGES;
            // TF32: the W tile must also have been split by warps 2-3.
            if (!mbar_wait(TF32 ? &split_done[s] : &full[s], (it / STAGES) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sx = smem_u32(smem + s * Cfg::kStageBytes);
            if constexpr (TF32) {
              const uint64_t dxh = smem_desc_sw64(sx);
              const uint64_t dxl = smem_desc_sw64(sx + Cfg::kXBytes / 2);
              const uint64_t dwh = smem_desc_sw64(sx + Cfg::kXBytes);
              const uint64_t dwl = smem_desc_sw64(sx + Cfg::kXBytes + NT * kWRowBytes);
#pragma unroll
              for (int kk = 0; kk < 2; ++kk) {
                const uint32_t acc = (kb | kk) != 0 ? 1u : 0u;
                umma_tf32(d_tmem, dxh + 2 * kk, dwh + 2 * kk, idesc, acc);
                umma_tf32(d_tmem + NT, dxh + 2 * kk, dwl + 2 * kk, idesc, acc);
                umma_tf32(d_tmem + NT, dxl + 2 * kk, dwh + 2 * kk, idesc, 1u);
              }
            } else {
#pragma unroll
              for (int h = 0; h < Cfg::kSub; ++h) {
                const uint64_t dx = smem_desc_sw128(sx + h * Cfg::kXBytes);
                const uint64_t dw = smem_desc_sw128(sx + Cfg::kSub * Cfg::kXBytes + h * Cfg::kWBytes);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                  const uint32_t acc = (kb | h | kk) != 0 ? 1u : 0u;
                  if constexpr (PAIR && FP8)
                    umma_f8_pair(d_tmem, dx + 2 * kk, dw + 2 * kk, idesc, acc);
                  else if constexpr (PAIR)
                    umma_f16_pair(d_tmem, dx + 2 * kk, dw + 2 * kk, idesc, acc);
                  else if constexpr (FP8)
                    umma_f8(d_tmem, dx + 2 * kk, dw + 2 * kk, idesc, acc);
                  else
                    umma_f16(d_tmem, dx + 2 * kk, dw + 2 * kk, idesc, acc);
                }
              }
            }
            if constexpr (PAIR) {
              umma_commit_pair(smem_u32(&empty[s]));
              umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1u));
            } else {
              umma_commit(&empty[s]);
            }
          }
          if (ok) {
            if constexpr (PAIR) {
              umma_commit_pair(smem_u32(&acc_full[a]));
              umma_commit_pair(mapa_shared(smem_u32(&acc_full[a]), 1u));
            } else {
              umma_commit(&acc_full[a]);
            }
          }
        }
      }
      if (!ok) {
        raise_device_error(kErrWaitTimeout);
        *abort_flag = 1;
      }
      // Every MMA issued above has completed once this barrier flips.
      if constexpr (PAIR)
        umma_commit_pair(smem_u32(mma_done));
      else
        umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr);
    }
    __syncwarp();
  } else if (TF32 && warp < kFirstEpiWarp) {
    // ------------------------------------------------------------ W splitter (TF32)
    // Walks the producer's stage sequence; every thread waits for the stage's
    // TMA itself (so that the loaded bytes are visible to its own reads),
    // writes the residual W - trunc13(W) of its share of the W tile to the
    // tile's second half (the raw tile is the hi operand as it is), then makes
    // the writes visible to the tensor core and arrives on split_done.
    const int st = (warp - 2) * 32 + lane;
    uint32_t it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < g.units && ok; u += gridDim.x) {
      int m;
      int64_t fb, fe;
      unit_range(g, u, m, fb, fe);
      for (int64_t ft = fb, w = 0; ft < fe && ok; ft += w) {
        w = tile_width<NT>(ft, fb, fe);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const bool got = mbar_wait(&full[s], (it / STAGES) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          const float4* wh = reinterpret_cast<const float4*>(smem + s * Cfg::kStageBytes + Cfg::kXBytes);
          float4* wl = reinterpret_cast<float4*>(smem + s * Cfg::kStageBytes + Cfg::kXBytes) + NT * (kWRowBytes / 16);
#pragma unroll 4
          for (int i = st; i < NT * (int)(kWRowBytes / 16); i += kSplitThreads) {
            const float4 v = wh[i];
            float4 l;
            l.x = v.x - trunc_tf32(v.x);
            l.y = v.y - trunc_tf32(v.y);
            l.z = v.z - trunc_tf32(v.z);
            l.w = v.w - trunc_tf32(v.w);
            wl[i] = l;
          }
          fence_proxy_async_smem();
          mbar_arrive(&split_done[s]);
        }
      }
    }
    if (!ok && lane == 0) {
      raise_device_error(kErrWaitTimeout);
      *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Pipelined encode: the previous step's rows, from the lists that step's
    // score kernel left (complete: it ran before this grid in the stream),
    // while this CTA's first tile streams in.  CTA c takes rows c,
    // c + gridDim.x, ...; the shared memory of the top lists / append slots is
    // not in use before the first tile's epilogue.  Over the peer exchange this
    // includes the publication, the wait for the other ranks' rows and the
    // world select.  (Moving the wait and the world select after the last tile
    // measured no faster on 2 GPUs.)
    static_assert(PAIR || CAND || Cfg::kBarOff - Cfg::kTopOff >= (int)sizeof(FinishSmem), "finish scratch");
    if constexpr (!PAIR && !CAND) {
      if (p.prev_finish) {
        const int etid = threadIdx.x - kFirstEpiWarp * 32;
        finish_rows<L, SyncEpilogue>(p.pfin, *reinterpret_cast<FinishSmem*>(smem + Cfg::kTopOff), blockIdx.x,
                                     gridDim.x, etid, kEpilogueWarps * 32);
        clear_sync_region(p.pfin, blockIdx.x, gridDim.x, etid, kEpilogueWarps * 32);
      }
    }
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)(q * 32) << 16);
    const uint32_t top_s = (uint32_t)(reinterpret_cast<uint8_t*>(top) - stk_smem);
    const uint32_t app_s = (uint32_t)(reinterpret_cast<uint8_t*>(smem + Cfg::kAppOff) - stk_smem);
    uint64_t* app_cta = p.app + (size_t)blockIdx.x * (kAppendMax * kRows);
    RowTopK<L, A, APP_SMEM, TOPT> acc;
    const uint32_t list_s = TOPT ? t_lane + kListCol : top_s;  // where this thread's row list lives
    uint32_t tile = 0;
    bool ok = true;
    TileWalk<NT, PAIR> cur;
    cur.start(g, rank);
    float published = -__int_as_float(0x7f800000);  // this unit's last published threshold
    float bcur[NT / 32], bnext[NT / 32];
    float scur[NT / 32], snext[NT / 32];  // FP8: per-feature scales, like the bias
    if (cur.valid(g)) {
      load_bias_tile<NT>(p.bias, cur.ft, cur.width(), p.F, lane, bcur);
      if constexpr (FP8) load_bias_tile<NT>(p.w_scale, cur.ft, cur.width(), p.F, lane, scur);
    }
    while (cur.valid(g)) {
      {  // the next tile's bias, prefetched (its walker is not kept: registers)
        TileWalk<NT, PAIR> nxt = cur;
        nxt.next(g, rank);
        if (nxt.valid(g)) {
          load_bias_tile<NT>(p.bias, nxt.ft, nxt.width(), p.F, lane, bnext);
          if constexpr (FP8) load_bias_tile<NT>(p.w_scale, nxt.ft, nxt.width(), p.F, lane, snext);
        }
      }
      if (cur.first_of_unit()) {
        acc.init(list_s, app_s, app_cta, r, p.k);
        published = -__int_as_float(0x7f800000);
      }
      const bool row_ok = (int64_t)cur.m * kRows + r < p.B;
      float sxr = 1.f;  // FP8: this row's dequantization scale
      if constexpr (FP8) sxr = row_ok ? __ldg(p.x_scale + (size_t)cur.m * kRows + r) : 0.f;
      const int w = cur.width();
      const int a = (int)(tile % kAccBufs);
      // Warp-uniform wait: lane 0 polls, the others follow its verdict.
      int got = 1;
      if (lane == 0) got = mbar_wait(&acc_full[a], (tile / kAccBufs) & 1, abort_flag) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) {
        if (p.pilot_hist != nullptr && cur.first_of_unit()) {
          // Match the two epilogue barriers of the sample step so the other
          // epilogue warps cannot wait on this one forever.
          epilogue_bar();
          if (warp == kFirstEpiWarp && lane == 0) *pilot_flag = 0;
          epilogue_bar();
        }
        ok = false;
        break;
      }
      tc_fence_after();
      const int nchunk = w / 32;
      const uint32_t tcol = t_lane + (uint32_t)a * kAccCols;
      uint64_t run[CAND ? 32 : 1];  // kModeCand: the current 128-feature tile's best 32 keys
      (void)run;
      // Shared floor: the best lower bound of this row's k-th score that the
      // other units of this M tile published so far (read now, applied after
      // the tile, so the load's latency hides behind the chunks).
      uint32_t shared_floor = 0u;
      if (p.row_floor != nullptr && row_ok) shared_floor = __ldcg(p.row_floor + (size_t)cur.m * kRows + r);
      if (p.pilot_hist != nullptr && cur.first_of_unit()) {
        // Sample: histogram the first chunks of this tile (they stay in TMEM
        // and are offered below), meet the other CTAs, read back a floor.
        uint32_t* h = p.pilot_hist + ((size_t)cur.m * kRows + r) * kPilotBins;
        uint32_t bmax = 0;
        bool any = false;
#pragma unroll 1
        for (int c = 0; c < p.pilot_chunks && c < nchunk; ++c) {
          uint32_t v[32];
          load_chunk<TF32, NT>(tcol, c, v);
          const int64_t f = cur.ft + 32 * c;
          const float bl = pick<NT / 32>(bcur, c);
          const float sl = FP8 ? pick<NT / 32>(scur, c) : 0.f;
          const uint32_t valid = row_ok ? feature_mask(f, p.F) : 0u;
          // Histogram the maximum of each group of kPilotGroup scores: they
          // are real scores of distinct features, so the k-th largest of them
          // still bounds the row's k-th score from below, at 1/kPilotGroup of
          // the global atomics of histogramming every sample.
#pragma unroll
          for (int g0 = 0; g0 < 32; g0 += kPilotGroup) {
            float gm = -__int_as_float(0x7f800000);
#pragma unroll
            for (int j = g0; j < g0 + kPilotGroup; ++j) {
              const float vj = chunk_score<FP8>(v[j], bl, sl, sxr, j);
              if (valid & (1u << j)) gm = fmaxf(gm, vj);
            }
            if ((valid >> g0) & ((1u << kPilotGroup) - 1u)) {
              const uint32_t bin = float_order(gm) >> (32 - kPilotBits);
              atomicAdd(h + bin, 1u);
              bmax = max(bmax, bin);
            }
          }
          any |= valid != 0u;
        }
        __threadfence();
        epilogue_bar();
        if (warp == kFirstEpiWarp && lane == 0) {
          atomicAdd(p.pilot_count, 1u);
          const unsigned long long t0 = global_timer_ns();
          int ok_all = 1;
          while (ld_acquire_u32(p.pilot_count) < gridDim.x) {
            if (global_timer_ns() - t0 > kPilotWaitNs) {
              ok_all = 0;
              break;
            }
            __nanosleep(256);
          }
          *pilot_flag = ok_all;
        }
        epilogue_bar();
        if (*pilot_flag && row_ok && any) {
          // The histogram window is anchored kPilotTopSlack bins (one octave)
          // above this CTA's own highest sampled bin instead of at the row's
          // global one (which would cost another memory round trip after the
          // barrier).  Counts above the window, if any, are only left out of
          // the count from the top, which makes the bound lower: still valid.
          const uint32_t tb = min(bmax + kPilotTopSlack, (uint32_t)(kPilotBins - 1));
          float lb;
          if (pilot_bound(h, tb, p.k, lb)) acc.set_floor(lb);
        }
      }
#pragma unroll 1
      for (int c = 0; c < nchunk; ++c) {
        uint32_t v[32];
        load_chunk<TF32, NT>(tcol, c, v);
        if (c == nchunk - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (PAIR && rank != 0)
              mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[a]), 0u));  // the pair's MMA issuer waits on it
            else
              mbar_arrive(&acc_empty[a]);
          }
        }
        const int64_t f = cur.ft + 32 * c;
        const float bl = pick<NT / 32>(bcur, c);
        const float sl = FP8 ? pick<NT / 32>(scur, c) : 0.f;
        float vals[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) vals[j] = chunk_score<FP8>(v[j], bl, sl, sxr, j);
        const uint32_t valid = row_ok ? feature_mask(f, p.F) : 0u;
        if constexpr (CAND) {
          // The 128-feature tile's top c (the reference's per-tile candidates,
          // streamtopk_approx.cu:42-167): this chunk's 32 keys sorted, merged
          // into the tile's running best 32 (bitonic merge of two descending
          // runs); at the tile's end written out, and its best min(c, k)
          // offered to the row's top-k (which only they can enter: k <= c).
          uint64_t kc[32];
#pragma unroll
          for (int j = 0; j < 32; ++j)
            kc[j] = ((valid >> j) & 1u) ? make_key(vals[j], p.index_offset + (uint32_t)f + (uint32_t)j) : kEmptyKey;
          sort_desc<32>(kc);
          if ((c & 3) == 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j) run[j] = kc[j];
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) run[j] = kmax(run[j], kc[31 - j]);
            merge_desc<32>(run);
          }
          if ((c & 3) == 3 || c == nchunk - 1) {
            if (row_ok) {
              const int64_t t = (cur.ft + 32 * (c & ~3)) / 128;
              const int64_t o = (((int64_t)cur.m * kRows + r) * p.cand_tiles + t) * p.cand_c;
              float4* vo = reinterpret_cast<float4*>(p.cand_vals + o);
              int4* io = reinterpret_cast<int4*>(p.cand_idxs + o);
#pragma unroll
              for (int q4 = 0; q4 < 8; ++q4) {
                if (4 * q4 < p.cand_c) {
                  float vv[4];
                  int ii[4];
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const uint64_t kk = run[4 * q4 + e];
                    vv[e] = kk ? key_value(kk) : -3.402823466e+38f;
                    ii[e] = kk ? key_index(kk) : -1;
                  }
                  vo[q4] = make_float4(vv[0], vv[1], vv[2], vv[3]);
                  io[q4] = make_int4(ii[0], ii[1], ii[2], ii[3]);
                }
              }
            }
            acc.offer_sorted(run, min(p.cand_c, p.k));
          }
        } else {
          acc.offer(vals, p.index_offset + (uint32_t)f, valid);
        }
      }
      if (p.row_floor != nullptr && row_ok) {
        // A unit's threshold is the k-th best of k real scores of the row (or
        // a floor already known), so it bounds the row's k-th score from
        // below for every unit: publish it, and take the others' bound.
        if (shared_floor != 0u) acc.set_floor(order_float(shared_floor));
        if (acc.thr > published) {
          atomicMax(p.row_floor + (size_t)cur.m * kRows + r, float_order(acc.thr));
          published = acc.thr;
        }
      }
      if (cur.last_of_unit()) {
        uint64_t* out_unit = p.partials + (int64_t)cur.u * kRows * p.list_pitch;
        if (p.list_pitch > L)
          acc.store_tail(out_unit + (int64_t)r * p.list_pitch + L);  // no final merge: a sorted second run
        else
          acc.finish();
        if constexpr (TOPT)
          store_list_tmem<L>(list_s, out_unit + (int64_t)r * p.list_pitch);
        else
          store_partials<L>(top_s, out_unit, p.list_pitch, q * 32, lane);
        __threadfence();  // the lists are read by other CTAs in the finish step
      }
#pragma unroll
      for (int c = 0; c < NT / 32; ++c) {
        bcur[c] = bnext[c];
        if constexpr (FP8) scur[c] = snext[c];
      }
      cur.next(g, rank);
      ++tile;
    }
    if (!ok && lane == 0) {
      raise_device_error(kErrWaitTimeout);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) {
    // Neither CTA of a pair frees its TMEM or exits while the other may still
    // touch its barriers (remote arrivals) or the pair's tensor memory.
    cluster_sync();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc_pair(tmem_base, kTmemCols);
    }
    return;  // (the host never asks a pair kernel for the in-kernel finish)
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (p.finish) {
    // Finish step in this kernel: once every CTA's lists are stored (bounded
    // grid barrier; the grid is one CTA per SM), CTA c finishes rows c,
    // c + gridDim.x, ...  The pipeline's shared memory is free by now.
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
      __threadfence();
      atomicAdd(p.tail_count, 1u);
      const unsigned long long t0 = global_timer_ns();
      while (ld_acquire_u32(p.tail_count) < gridDim.x) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          raise_device_error(kErrFinishBarrier);
          break;
        }
        __nanosleep(64);
      }
    }
    __syncthreads();
    finish_rows<L>(p.fin, *reinterpret_cast<FinishSmem*>(smem), blockIdx.x, gridDim.x, threadIdx.x, blockDim.x);
  }
}

// ---------------------------------------------------------------------------
// SIMT kernel: 256 threads compute a 128 x 128 score tile with fp32 FMA
// (8 x 8 per thread), stage it in shared memory, then threads 0..127 (one per
// batch row) feed it to the same top-k accumulator.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T, int L>
__global__ void __launch_bounds__(kSimtThreads, 1) simt_topk_kernel(const T* __restrict__ X, const T* __restrict__ W,
                                                                    const SimtParams p) {
  using Cfg = SimtCfg<L>;
  uint8_t* smem = stk_smem;
  float* xs = reinterpret_cast<float*>(smem + Cfg::kXsOff);        // [kKc][129] rows
  float* ws = reinterpret_cast<float*>(smem + Cfg::kWsOff);        // [kKc][129] features
  float* sc = reinterpret_cast<float*>(smem + Cfg::kScOff);        // [128 rows][129]
  const uint32_t top_s = (uint32_t)Cfg::kTopOff;
  uint64_t* app_cta = p.app + (size_t)blockIdx.x * (kAppendMax * kRows);

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int lane = tid & 31;
  const UnitGrid& g = p.grid;
  RowTopK<L, 32, false> acc;
  const bool vec_bias = (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0;

  for (int u = blockIdx.x; u < g.units; u += gridDim.x) {
    int m;
    int64_t fb, fe;
    unit_range(g, u, m, fb, fe);
    const int64_t row0 = (int64_t)m * kRows;
    if (tid < kRows) acc.init(top_s, 0u, app_cta, tid, p.k);
    for (int64_t ft = fb; ft < fe; ft += Cfg::kNT) {
      const int w = (int)min((int64_t)Cfg::kNT, fe - ft);
      float c[8][8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) c[i][j] = 0.f;
      for (int64_t k0 = 0; k0 < p.d; k0 += Cfg::kKc) {
        __syncthreads();
        // Stage X[row0 + i][k0 + kk] -> xs[kk][i], W[ft + n][k0 + kk] -> ws[kk][n].
        for (int e = tid; e < Cfg::kKc * kRows; e += kSimtThreads) {
          const int i = e / Cfg::kKc, kk = e % Cfg::kKc;
          const int64_t row = row0 + i, col = k0 + kk;
          xs[kk * (kRows + 1) + i] = (row < p.B && col < p.d) ? to_f32(X[row * p.d + col]) : 0.f;
          const int64_t fr = ft + i;
          ws[kk * (kRows + 1) + i] = (i < w && fr < p.F && col < p.d) ? to_f32(W[fr * p.d + col]) : 0.f;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < Cfg::kKc; ++kk) {
          float xa[8], wb[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) xa[i] = xs[kk * (kRows + 1) + ty + 16 * i];
#pragma unroll
          for (int j = 0; j < 8; ++j) wb[j] = ws[kk * (kRows + 1) + tx + 16 * j];
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) c[i][j] = fmaf(xa[i], wb[j], c[i][j]);
        }
      }
      __syncthreads();  // the score tile aliases the staging buffers
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) sc[(ty + 16 * i) * (kRows + 1) + tx + 16 * j] = c[i][j];
      __syncthreads();
      if (tid < kRows) {
        const bool row_ok = row0 + tid < p.B;
        for (int cc = 0; cc < w / 32; ++cc) {
          const int64_t f = ft + cc * 32;
          float bv[32];
          load_bias32(p.bias, f, p.F, vec_bias, bv);
          float vals[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) vals[j] = sc[tid * (kRows + 1) + cc * 32 + j] + bv[j];
          const uint32_t valid = row_ok ? feature_mask(f, p.F) : 0u;
          acc.offer(vals, p.index_offset + (uint32_t)f, valid);
        }
      }
    }
    if (tid < kRows) {
      acc.finish();
      store_partials<L>(top_s, p.partials + (int64_t)u * kRows * L, L, tid & ~31, lane);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Standalone finish kernel (stk_finish.cuh).  Launched with programmatic
// dependent launch after the score kernel: griddepcontrol.wait blocks until
// that grid has completed and its writes are visible (a no-op otherwise).
// ---------------------------------------------------------------------------
template <int L>
__global__ void __launch_bounds__(kFinishThreads, 2) finish_kernel(const FinishArgs fa) {
  __shared__ FinishSmem sm;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  finish_rows<L>(fa, sm, blockIdx.x, gridDim.x, threadIdx.x, blockDim.x);
  clear_sync_region(fa, blockIdx.x, gridDim.x, threadIdx.x, blockDim.x);
}

// ---------------------------------------------------------------------------
// Explicit instantiations and launch helpers (host side of this TU).
// ---------------------------------------------------------------------------
template <int L, int NT, int STAGES, int A, bool APP_SMEM, bool TOPT, int MODE>
cudaError_t launch_fused(const CUtensorMap& tx, const CUtensorMap& txl, const CUtensorMap& tw, const CUtensorMap& tw32,
                         const FusedParams& p, int grid, cudaStream_t stream) {
  using Cfg = FusedCfg<L, NT, STAGES, A, APP_SMEM, TOPT>;
  auto kern = fused_topk_kernel<L, NT, STAGES, A, APP_SMEM, TOPT, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return e;
  kern<<<grid, MODE == kModeTF32 ? kFusedThreads + 64 : kFusedThreads, Cfg::kSmemBytes, stream>>>(tx, txl, tw, tw32,
                                                                                                  p);
  return cudaGetLastError();
}

template <int L, int NT, int STAGES, int A, bool APP_SMEM, bool TOPT, int MODE>
cudaError_t launch_fused_pair(const CUtensorMap& tx, const CUtensorMap& tw, const FusedParams& p, int grid,
                              cudaStream_t stream) {
  static_assert((MODE & kModePair) != 0, "pair variant");
  using Cfg = FusedCfg<L, NT, STAGES, A, APP_SMEM, TOPT, true>;
  auto kern = fused_topk_kernel<L, NT, STAGES, A, APP_SMEM, TOPT, MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tx, tx, tw, tw, p);
}

template <int L, int NT, int STAGES, int A, bool APP_SMEM, bool TOPT, int MODE>
int pair_clusters_max() {
  using Cfg = FusedCfg<L, NT, STAGES, A, APP_SMEM, TOPT, true>;
  auto kern = fused_topk_kernel<L, NT, STAGES, A, APP_SMEM, TOPT, MODE>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) return 0;
  return n;
}

__global__ void residual_tf32_kernel(const float* __restrict__ X, float* __restrict__ Xl, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = X[i];
    Xl[i] = x - trunc_tf32(x);
  }
}

cudaError_t launch_residual_tf32(const float* X, float* Xl, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = (n + 255) / 256;
  residual_tf32_kernel<<<(unsigned)(blocks < 1184 ? blocks : 1184), 256, 0, stream>>>(X, Xl, n);
  return cudaGetLastError();
}

template <typename T, int L>
cudaError_t launch_simt(const void* X, const void* W, const SimtParams& p, int grid, cudaStream_t stream) {
  using Cfg = SimtCfg<L>;
  auto kern = simt_topk_kernel<T, L>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return e;
  kern<<<grid, kSimtThreads, Cfg::kSmemBytes, stream>>>(static_cast<const T*>(X), static_cast<const T*>(W), p);
  return cudaGetLastError();
}

template <int L>
cudaError_t launch_finish(const FinishArgs& fa, int grid, cudaStream_t stream) {
  if (fa.rows <= 0 || grid <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kFinishThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, finish_kernel<L>, fa);
}

#define STK_INST_FUSED(L, NT, S, A, SM, TT)                                                                  \
  template cudaError_t launch_fused<L, NT, S, A, SM, TT, kModeF16>(const CUtensorMap&, const CUtensorMap&,     \
                                                                   const CUtensorMap&, const CUtensorMap&,     \
                                                                   const FusedParams&, int, cudaStream_t);
STK_FUSED_CONFIGS(STK_INST_FUSED)
#define STK_INST_FUSED_TF32(L, NT, S, A, SM, TT)                                                             \
  template cudaError_t launch_fused<L, NT, S, A, SM, TT, kModeTF32>(const CUtensorMap&, const CUtensorMap&,    \
                                                                    const CUtensorMap&, const CUtensorMap&,    \
                                                                    const FusedParams&, int, cudaStream_t);
STK_FUSED_TF32_CONFIGS(STK_INST_FUSED_TF32)
#define STK_INST_FUSED_FP8(L, NT, S, A, SM, TT)                                                              \
  template cudaError_t launch_fused<L, NT, S, A, SM, TT, kModeFP8>(const CUtensorMap&, const CUtensorMap&,     \
                                                                   const CUtensorMap&, const CUtensorMap&,     \
                                                                   const FusedParams&, int, cudaStream_t);
STK_FUSED_FP8_CONFIGS(STK_INST_FUSED_FP8)
#define STK_INST_FUSED_CAND(L, NT, S, A, SM, TT)                                                             \
  template cudaError_t launch_fused<L, NT, S, A, SM, TT, kModeF16 | kModeCand>(                               \
      const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const FusedParams&, int,  \
      cudaStream_t);
STK_FUSED_CAND_CONFIGS(STK_INST_FUSED_CAND)
#define STK_INST_FUSED_PAIR(L, NT, S, A, SM, TT)                                                             \
  template cudaError_t launch_fused_pair<L, NT, S, A, SM, TT, kModeF16 | kModePair>(                          \
      const CUtensorMap&, const CUtensorMap&, const FusedParams&, int, cudaStream_t);                         \
  template cudaError_t launch_fused_pair<L, NT, S, A, SM, TT, kModeFP8 | kModePair>(                          \
      const CUtensorMap&, const CUtensorMap&, const FusedParams&, int, cudaStream_t);                         \
  template int pair_clusters_max<L, NT, S, A, SM, TT, kModeF16 | kModePair>();                                \
  template int pair_clusters_max<L, NT, S, A, SM, TT, kModeFP8 | kModePair>();
STK_FUSED_PAIR_CONFIGS(STK_INST_FUSED_PAIR)

#define STK_INST_SIMT(L)                                                                                         \
  template cudaError_t launch_simt<float, L>(const void*, const void*, const SimtParams&, int, cudaStream_t);   \
  template cudaError_t launch_simt<__half, L>(const void*, const void*, const SimtParams&, int, cudaStream_t);  \
  template cudaError_t launch_simt<__nv_bfloat16, L>(const void*, const void*, const SimtParams&, int,          \
                                                     cudaStream_t);                                             \
  template cudaError_t launch_finish<L>(const FinishArgs&, int, cudaStream_t);
STK_INST_SIMT(32)
STK_INST_SIMT(64)
STK_INST_SIMT(128)

// ---------------------------------------------------------------------------
// Per-row E4M3 quantization (the FP8 path's X, or W_enc once ahead of use):
// one warp per row, the row's absolute maximum by a warp reduction, then 4
// elements per lane and step converted with the hardware's round-to-nearest-
// even, saturating E4M3 conversion and stored as one 32-bit word.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void quantize_rows_e4m3_kernel(const T* __restrict__ X, uint8_t* __restrict__ Q,
                                          float* __restrict__ scale, int64_t rows, int64_t d) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* x = X + row * d;
  float m = 0.f;
  for (int64_t j = lane; j < d; j += 32) m = fmaxf(m, fabsf(to_f32(x[j])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float inv = m > 0.f ? 448.f / m : 1.f;
  if (lane == 0) scale[row] = m > 0.f ? m / 448.f : 1.f;
  uint32_t* q = reinterpret_cast<uint32_t*>(Q + row * d);  // d % 16 == 0: 16-byte aligned rows
  for (int64_t j = 4 * lane; j < d; j += 128) {
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_fp8_storage_t b = __nv_cvt_float_to_fp8(to_f32(x[j + e]) * inv, __NV_SATFINITE, __NV_E4M3);
      word |= (uint32_t)b << (8 * e);
    }
    q[j / 4] = word;
  }
}

template <typename T>
cudaError_t launch_quantize_rows_e4m3(const T* X, uint8_t* Q, float* scale, int64_t rows, int64_t d,
                                      cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  constexpr int kWarps = 8;
  const int64_t blocks = (rows + kWarps - 1) / kWarps;
  quantize_rows_e4m3_kernel<T><<<(unsigned)blocks, 32 * kWarps, 0, stream>>>(X, Q, scale, rows, d);
  return cudaGetLastError();
}
template cudaError_t launch_quantize_rows_e4m3<float>(const float*, uint8_t*, float*, int64_t, int64_t, cudaStream_t);
template cudaError_t launch_quantize_rows_e4m3<__half>(const __half*, uint8_t*, float*, int64_t, int64_t,
                                                       cudaStream_t);
template cudaError_t launch_quantize_rows_e4m3<__nv_bfloat16>(const __nv_bfloat16*, uint8_t*, float*, int64_t,
                                                              int64_t, cudaStream_t);

// ---------------------------------------------------------------------------
// Whole-row sort for small F (k up to F <= kFullSortMaxF, beyond the list
// lengths of the streaming kernels): one CTA per row computes all F scores
// (one warp per feature, lanes across d, fp32 accumulation) as 64-bit keys in
// shared memory, sorts them with a block-wide bitonic network and writes the
// first k.  Same key order as every other path (score, then smaller index).
// ---------------------------------------------------------------------------
constexpr int kFullSortThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kFullSortThreads) fullsort_kernel(const T* __restrict__ X, const T* __restrict__ W,
                                                                     const float* __restrict__ bias, float* __restrict__ V,
                                                                     int32_t* __restrict__ I, int64_t d, int F, int k) {
  __shared__ uint64_t keys[kFullSortMaxF];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int n = 1;
  while (n < F) n <<= 1;
  const T* x = X + row * d;
  for (int f = warp; f < n; f += kFullSortThreads / 32) {
    float acc = 0.f;
    if (f < F) {
      const T* w = W + (int64_t)f * d;
      for (int64_t j = lane; j < d; j += 32) acc = fmaf(to_f32(x[j]), to_f32(w[j]), acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    }
    if (lane == 0) keys[f] = f < F ? make_key(acc + bias[f], (uint32_t)f) : kEmptyKey;
  }
  __syncthreads();
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n; i += kFullSortThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const uint64_t a = keys[i], c = keys[j];
          const bool desc = (i & size) == 0;
          if (desc ? (a < c) : (a > c)) {
            keys[i] = c;
            keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < k; i += kFullSortThreads) {
    V[row * k + i] = key_value(keys[i]);
    I[row * k + i] = key_index(keys[i]);
  }
}

cudaError_t launch_fullsort(const void* X, const void* W, const float* bias, float* V, int32_t* I, int64_t B,
                            int64_t d, int F, int k, int dtype, cudaStream_t stream) {
  if (B <= 0) return cudaSuccess;
  const unsigned grid = (unsigned)B;
  if (dtype == 0)
    fullsort_kernel<float><<<grid, kFullSortThreads, 0, stream>>>(static_cast<const float*>(X),
                                                                  static_cast<const float*>(W), bias, V, I, d, F, k);
  else if (dtype == 1)
    fullsort_kernel<__half><<<grid, kFullSortThreads, 0, stream>>>(static_cast<const __half*>(X),
                                                                   static_cast<const __half*>(W), bias, V, I, d, F, k);
  else
    fullsort_kernel<__nv_bfloat16><<<grid, kFullSortThreads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(X), static_cast<const __nv_bfloat16*>(W), bias, V, I, d, F, k);
  return cudaGetLastError();
}

__global__ void candidates_out_kernel(const uint64_t* __restrict__ partials, int L, int m_tiles, int64_t tiles,
                                      int64_t rows, int c, float* __restrict__ vals, int32_t* __restrict__ idxs) {
  const int64_t total = rows * tiles * c;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int s = (int)(i % c);
    const int64_t t = (i / c) % tiles;
    const int64_t b = i / ((int64_t)c * tiles);
    const int64_t m = b / kRows, r = b % kRows;
    const uint64_t key = partials[((t * m_tiles + m) * kRows + r) * L + s];
    vals[i] = key ? key_value(key) : -3.402823466e+38f;
    idxs[i] = key ? key_index(key) : -1;
  }
}

cudaError_t launch_candidates_out(const uint64_t* partials, int L, int m_tiles, int64_t tiles, int64_t rows, int c,
                                  float* vals, int32_t* idxs, cudaStream_t stream) {
  const int64_t total = rows * tiles * c;
  if (total <= 0) return cudaSuccess;
  const int64_t blocks = min((total + 255) / 256, (int64_t)148 * 16);
  candidates_out_kernel<<<(unsigned)blocks, 256, 0, stream>>>(partials, L, m_tiles, tiles, rows, c, vals, idxs);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Decoder gather-GEMM (the consumer of (V, I)): one CTA per (row, slice of
// 8 x kDecThreads features of d); each thread owns 8 consecutive outputs and
// walks the row's k codes, loading 16 bytes of the selected W_dec row per
// code -- coalesced across the CTA -- with four codes in flight at a time.
// The row's codes are staged in shared memory.  HBM-bound: B * k * d *
// sizeof(T) gathered bytes (rows repeated across the batch hit in L2).
// (Splitting a row's codes over four thread groups with a shared-memory sum
// measured slower at B = 4096.)
// ---------------------------------------------------------------------------
constexpr int kDecThreads = 128;
constexpr int kDecMaxK = 1024;

template <typename T>
__device__ __forceinline__ void dec_load8(const T* __restrict__ p, float (&w)[8]);
template <>
__device__ __forceinline__ void dec_load8<__nv_bfloat16>(const __nv_bfloat16* __restrict__ p, float (&w)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w[2 * i] = __uint_as_float(q[i] << 16);
    w[2 * i + 1] = __uint_as_float(q[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void dec_load8<__half>(const __half* __restrict__ p, float (&w)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    w[2 * i] = f.x;
    w[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void dec_load8<float>(const float* __restrict__ p, float (&w)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 c = __ldg(reinterpret_cast<const float4*>(p) + 1);
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  w[4] = c.x; w[5] = c.y; w[6] = c.z; w[7] = c.w;
}

template <typename T>
__global__ void __launch_bounds__(kDecThreads) decode_kernel(const float* __restrict__ V, const int32_t* __restrict__ I,
                                                             const T* __restrict__ W, const float* __restrict__ bias,
                                                             float* __restrict__ out, int64_t B, int k, int64_t F,
                                                             int64_t d) {
  __shared__ float sv[kDecMaxK];
  __shared__ int32_t si[kDecMaxK];
  const int64_t col = ((int64_t)blockIdx.x * kDecThreads + threadIdx.x) * 8;
  const bool active = col < d;
  const bool full = col + 8 <= d;
  for (int64_t b = blockIdx.y; b < B; b += gridDim.y) {
    __syncthreads();  // the previous row's codes are no longer read
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
      const int32_t ix = I[b * k + j];
      const bool ok = ix >= 0 && (int64_t)ix < F;
      sv[j] = ok ? V[b * k + j] : 0.f;
      si[j] = ok ? ix : -1;
    }
    __syncthreads();
    if (!active) continue;
    float acc[8];
    if (bias != nullptr && full) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(bias + col));
      const float4 c = __ldg(reinterpret_cast<const float4*>(bias + col) + 1);
      acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w;
      acc[4] = c.x; acc[5] = c.y; acc[6] = c.z; acc[7] = c.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = (bias != nullptr && col + e < d) ? bias[col + e] : 0.f;
    }
    int j = 0;
    if (full) {
      for (; j + 4 <= k; j += 4) {
        float w[4][8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int32_t ix = si[j + q];
          if (ix >= 0) {
            dec_load8<T>(W + (int64_t)ix * d + col, w[q]);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) w[q][e] = 0.f;
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = fmaf(sv[j + q], w[q][e], acc[e]);
      }
      for (; j < k; ++j) {
        const int32_t ix = si[j];
        if (ix < 0) continue;
        float w[8];
        dec_load8<T>(W + (int64_t)ix * d + col, w);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(sv[j], w[e], acc[e]);
      }
      float4* o = reinterpret_cast<float4*>(out + b * d + col);
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      for (; j < k; ++j) {
        const int32_t ix = si[j];
        if (ix < 0) continue;
        for (int e = 0; e < 8 && col + e < d; ++e) acc[e] = fmaf(sv[j], to_f32(W[(int64_t)ix * d + col + e]), acc[e]);
      }
      for (int e = 0; e < 8 && col + e < d; ++e) out[b * d + col + e] = acc[e];
    }
  }
}

template <typename T>
cudaError_t launch_decode(const float* V, const int32_t* I, const T* W_dec, const float* b_dec, float* out, int64_t B,
                          int k, int64_t F, int64_t d, cudaStream_t stream) {
  if (B <= 0 || d <= 0) return cudaSuccess;
  if (k < 0 || k > kDecMaxK) return cudaErrorInvalidValue;
  const int64_t slices = (d + 8 * kDecThreads - 1) / (8 * kDecThreads);
  if (slices > 65535) return cudaErrorInvalidValue;
  const unsigned rows = (unsigned)(B < 65535 ? B : 65535);
  decode_kernel<T><<<dim3((unsigned)slices, rows), kDecThreads, 0, stream>>>(V, I, W_dec, b_dec, out, B, k, F, d);
  return cudaGetLastError();
}
template cudaError_t launch_decode<float>(const float*, const int32_t*, const float*, const float*, float*, int64_t,
                                          int, int64_t, int64_t, cudaStream_t);
template cudaError_t launch_decode<__half>(const float*, const int32_t*, const __half*, const float*, float*, int64_t,
                                           int, int64_t, int64_t, cudaStream_t);
template cudaError_t launch_decode<__nv_bfloat16>(const float*, const int32_t*, const __nv_bfloat16*, const float*,
                                                  float*, int64_t, int, int64_t, int64_t, cudaStream_t);

cudaError_t read_and_clear_device_error(unsigned* out, cudaStream_t stream) {
  unsigned zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_device_error, sizeof(unsigned), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return e;
  if (*out) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(unsigned));
  return e;
}

}  // namespace stk
