// Finish step of an encode: the top-k of each row over the sorted key lists the
// score kernel left per work unit (pass 2 of the reference,
// streamtopk_sae/csrc/cuda/streamtopk_exact.cu:429-499), optionally followed by
// the cross-GPU exchange of the F-sharded encode.
//
// Runs either in the tail of the fused score kernel (all CTAs meet at a bounded
// grid barrier once every unit's lists are stored, then each CTA finishes rows
// blockIdx.x, blockIdx.x + gridDim.x, ...) or as the standalone finish_kernel
// after a score kernel whose units cannot all be resident at once.  Both give
// bit-identical results: keys are unique, so a row's top-k is unique.
//
// Per row:
//   1. tau = a lower bound of the row's k-th key from k distinct real keys:
//      the k-th largest list head (many lists), or, when there are fewer than
//      2k lists (but more than 2k / L), the k-th largest of the first
//      ceil(2k / nlists) keys of every list; and at least the largest k-th key
//      of any one list (a list holds k keys >= its own k-th).  tau = 1 (every key) when no bound exists.  The
//      heads bound suits the score kernel's many sparse lists, the prefix bound
//      the few full lists of the exchange (one per GPU) or of a large batch.
//   2. Every key >= tau is gathered into shared memory.  Many lists: one
//      thread per list, 4 keys at a time until a key below tau (lists are
//      sorted).  The score kernel's lists are sparse -- each key passed the
//      row's threshold floor -- so this is ~1.3 k keys per row on Gaussian
//      data.  Few or full lists (at most kFinishFewLists lists, e.g. one per
//      GPU, or at most 8 chunks per thread, e.g. the full per-unit lists of a
//      large batch): one thread per 4-key chunk, all chunks at once, so a list
//      costs one memory round trip whatever its depth.
//   3. Each candidate's position in the row's sorted result is the number of
//      larger candidates (keys are distinct): one thread per candidate.
//   More candidates than kFinishCap (adversarial inputs): the lists are folded
//   instead, warp by warp, with a warp-cooperative bitonic merge.
//
// Exchange (ExchangeDev, one process per GPU): a row's best L keys are stored
// into slot [step & 1][rank] of every rank's receive buffer (plain stores into
// the peers' memory over NVLink, CUDA IPC mappings), and after a system-scope
// fence a per-row flag in the peer's memory is set to step + 1.  Each rank then
// waits (bounded) until the flags of all ranks' copies of its rows read
// step + 1, and finishes the rows over the world lists.  The step tag is
// absolute, so rows that arrive after a wait gave up can never be taken for a
// later step's rows; double buffering by step parity is race-free because a
// rank starts step s + 2 only after its step s + 1, which needed every rank's
// step s + 1 rows, which each rank stores only after finishing its step s.
#pragma once
#include "stk_kernels.cuh"

namespace stk {

constexpr int kFinishCap = 1024;      // candidates ranked by counting
constexpr int kFinishMaxLists = 256;  // lists whose heads are held in shared memory
constexpr int kFoldBatch = 8;         // lists loaded per warp and memory round trip (fold)
constexpr int kFinishMaxWarps = 8;    // fold tree buffer: kFinishMaxWarps * L <= kFinishCap
constexpr int kFinishFewLists = 32;   // at most this many lists: gather chunk-parallel

struct __align__(16) FinishSmem {
  uint64_t heads[kFinishMaxLists];
  uint64_t cand[kFinishCap];
  uint64_t best[128];
  uint64_t tau;
  int cnt;
  uint32_t valid;
};

// g_device_error: the device error word, defined by the translation unit
// that includes this header (stk_kernels.cu), ahead of the include.
__device__ __forceinline__ void raise_device_error(unsigned code) { atomicCAS(&g_device_error, 0u, code); }

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ bool list_on(uint32_t mask, int s) { return s >= 32 || ((mask >> s) & 1u); }

// Barrier over the threads that run a finish: the whole CTA, or (pipelined
// encode) the score kernel's four epilogue warps, which finish the previous
// step's rows while the CTA's producer streams the first tile (named barrier 1).
struct SyncCta {
  __device__ static __forceinline__ void sync() { __syncthreads(); }
};
struct SyncEpilogue {
  __device__ static __forceinline__ void sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
};

// Best L keys of row b over nlists lists, written to sm.best[0..L) descending
// with empty keys after the last one.  List s of row b starts at
// lists[(s * stride + b) * pitch]: L keys descending (empty keys 0 at the end),
// then, if tail > 0, a second descending run of `tail` keys (the score kernel's
// last survivors, stored without a final merge).  Lists s < 32 whose bit is
// clear in list_mask count as empty.  Every thread of the CTA calls it
// (nthreads = the threads that S synchronises, at most kFinishMaxWarps warps);
// it ends with S::sync().  Lists must be 16-byte aligned.
template <int L, class S = SyncCta>
__device__ void select_row(const uint64_t* __restrict__ lists, int nlists, int64_t stride, int pitch, int tail,
                           int64_t b, int k, uint32_t list_mask, FinishSmem& sm, int tid, int nthreads) {
  const bool use_heads = nlists <= kFinishMaxLists;
  if (tid == 0) {
    sm.tau = 1ull;
    sm.cnt = 0;
  }
  uint64_t kth = 0ull;  // largest k-th key of one list among this thread's lists
  // One list per thread (the common case): its first 4 keys of each run come
  // with the head in the same memory round trip and are gathered from registers.
  const bool chunk_parallel =
      use_heads && (nlists <= kFinishFewLists || (int64_t)nlists * ((L + tail) / 4) <= 8 * (int64_t)nthreads);
  const bool one_each = use_heads && nlists <= nthreads && !chunk_parallel;
  uint64_t first[4] = {0ull, 0ull, 0ull, 0ull}, tfirst[4] = {0ull, 0ull, 0ull, 0ull};
  if (use_heads)
    for (int s = tid; s < nlists; s += nthreads) {
      const uint64_t* ps = lists + ((int64_t)s * stride + b) * pitch;
      const bool on = list_on(list_mask, s);
      uint64_t h = 0ull;
      if (on) {
        const ulonglong2 u0 = __ldcg(reinterpret_cast<const ulonglong2*>(ps));
        const ulonglong2 u1 = __ldcg(reinterpret_cast<const ulonglong2*>(ps + 2));
        first[0] = u0.x;
        first[1] = u0.y;
        first[2] = u1.x;
        first[3] = u1.y;
        h = first[0];
        if (tail > 0) {
          const ulonglong2 t0 = __ldcg(reinterpret_cast<const ulonglong2*>(ps + L));
          const ulonglong2 t1 = __ldcg(reinterpret_cast<const ulonglong2*>(ps + L + 2));
          tfirst[0] = t0.x;
          tfirst[1] = t0.y;
          tfirst[2] = t1.x;
          tfirst[3] = t1.y;
          h = kmax(h, tfirst[0]);
        }
        if (k <= L) kth = kmax(kth, (uint64_t)__ldcg(reinterpret_cast<const unsigned long long*>(ps + k - 1)));
      }
      sm.heads[s] = h;
    }
  // Few lists for this k (nlists < 2k): the bound comes from the first
  // m = ceil(2k / nlists) keys of every list instead of the heads alone -- the
  // k-th largest of these nlists * m >= 2k real keys (k distinct keys >= it).
  // Not when m would cover whole lists (one or two lists): the largest k-th
  // key of one list is then as good, and the gather reads the lists anyway.
  const int m2k = (use_heads && nlists > 0) ? max(1, (2 * k + nlists - 1) / nlists) : 0;
  const int m = m2k < L ? m2k : 0;
  const int P = nlists * m;  // <= 2k + nlists <= kFinishCap when m > 1
  if (m > 1)
    for (int t = tid; t < P; t += nthreads) {
      const int s = t / m, j = t - (t / m) * m;
      sm.cand[t] = list_on(list_mask, s) ? (uint64_t)__ldcg(reinterpret_cast<const unsigned long long*>(
                                               lists + ((int64_t)s * stride + b) * pitch + j))
                                         : 0ull;
    }
  S::sync();
  if (m > 1) {
    for (int t = tid; t < P; t += nthreads) {
      const uint64_t key = sm.cand[t];
      if (key == 0ull) continue;
      int r = 0;
      for (int j = 0; j < P; ++j) r += sm.cand[j] > key ? 1 : 0;
      if (r == k - 1) atomicMax(reinterpret_cast<unsigned long long*>(&sm.tau), (unsigned long long)key);
    }
  } else if (use_heads) {
    for (int s = tid; s < nlists; s += nthreads) {
      const uint64_t h = sm.heads[s];
      if (h == 0ull) continue;
      int r = 0;
      for (int j = 0; j < nlists; ++j) r += sm.heads[j] > h ? 1 : 0;
      if (r == k - 1) atomicMax(reinterpret_cast<unsigned long long*>(&sm.tau), (unsigned long long)h);
    }
  }
  if (kth != 0ull) atomicMax(reinterpret_cast<unsigned long long*>(&sm.tau), (unsigned long long)kth);
  S::sync();
  const uint64_t tau = sm.tau;
  auto keep4 = [&](const uint64_t (&kk)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (kk[j] >= tau) {
        const int pos = atomicAdd(&sm.cnt, 1);
        if (pos < kFinishCap) sm.cand[pos] = kk[j];
      }
    }
    return kk[3] >= tau;  // the run may continue past these 4 keys
  };
  auto take4 = [&](const uint64_t* p4) {
    const ulonglong2 u0 = __ldcg(reinterpret_cast<const ulonglong2*>(p4));
    const ulonglong2 u1 = __ldcg(reinterpret_cast<const ulonglong2*>(p4 + 2));
    const uint64_t kk[4] = {u0.x, u0.y, u1.x, u1.y};
    return keep4(kk);
  };
  if (chunk_parallel) {
    const int chunks = (L + tail) / 4;
    for (int t = tid; t < nlists * chunks; t += nthreads) {
      const int s = t / chunks, q = (t % chunks) * 4;
      if (sm.heads[s] < tau) continue;
      take4(lists + ((int64_t)s * stride + b) * pitch + q);
    }
  } else if (one_each) {
    if (tid < nlists && sm.heads[tid] >= tau) {
      const uint64_t* ps = lists + ((int64_t)tid * stride + b) * pitch;
      if (keep4(first))
        for (int q = 4; q < L; q += 4)
          if (!take4(ps + q)) break;  // sorted: the rest is smaller
      if (tail > 0 && keep4(tfirst))
        for (int q = 4; q < tail; q += 4)
          if (!take4(ps + L + q)) break;
    }
  } else if (use_heads) {
    for (int s = tid; s < nlists; s += nthreads) {
      if (sm.heads[s] < tau) continue;  // empty lists too (tau >= 1)
      const uint64_t* ps = lists + ((int64_t)s * stride + b) * pitch;
      for (int q = 0; q < L; q += 4)
        if (!take4(ps + q)) break;  // sorted: the rest is smaller
      for (int q = 0; q < tail; q += 4)
        if (!take4(ps + L + q)) break;
    }
  }
  S::sync();
  const int C = use_heads ? sm.cnt : kFinishCap + 1;
  if (C <= kFinishCap) {
    for (int i = tid; i < C; i += nthreads) {
      const uint64_t key = sm.cand[i];
      int r = 0;
      for (int j = 0; j < C; ++j) r += sm.cand[j] > key ? 1 : 0;
      if (r < L) sm.best[r] = key;
    }
    for (int i = C + tid; i < L; i += nthreads) sm.best[i] = 0ull;
    S::sync();
    return;
  }
  // Fold: warp w merges runs w, w + nw, ... (every list's L-key run, then
  // every list's tail run, each as a sorted list of up to L keys) into its best
  // L (a run whose best key does not beat the warp's current L-th is skipped),
  // then warp 0 merges the warps' results.
  constexpr int E = L / 32;
  const int warp = tid >> 5, lane = tid & 31, nw = nthreads >> 5;
  const int nruns = tail > 0 ? 2 * nlists : nlists;
  uint64_t acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0ull;
  for (int v0 = warp; v0 < nruns; v0 += nw * kFoldBatch) {
    uint64_t buf[kFoldBatch][E];
#pragma unroll
    for (int q = 0; q < kFoldBatch; ++q) {
      const int v = v0 + q * nw;
      const bool is_tail = v >= nlists;
      const int s = is_tail ? v - nlists : v;
      const bool on = v < nruns && list_on(list_mask, s) && (!use_heads || sm.heads[s] >= tau);
      const uint64_t* ps = lists + ((int64_t)s * stride + b) * pitch + (is_tail ? L : 0);
      const int len = is_tail ? tail : L;
#pragma unroll
      for (int e = 0; e < E; ++e)
        buf[q][e] = (on && e * 32 + lane < len)
                        ? (uint64_t)__ldcg(reinterpret_cast<const unsigned long long*>(ps + e * 32 + lane))
                        : 0ull;
    }
#pragma unroll
    for (int q = 0; q < kFoldBatch; ++q) {
      const uint64_t hi = __shfl_sync(0xffffffffu, buf[q][0], 0);
      const uint64_t lo = __shfl_sync(0xffffffffu, acc[E - 1], 31);
      if (hi > lo) warp_merge_lists<E>(acc, buf[q], lane);
    }
  }
  uint64_t* red = sm.cand;  // [nw][L]
#pragma unroll
  for (int e = 0; e < E; ++e) red[warp * L + e * 32 + lane] = acc[e];
  S::sync();
  if (warp == 0) {
    for (int w = 1; w < nw; ++w) {
      uint64_t u[E];
#pragma unroll
      for (int e = 0; e < E; ++e) u[e] = red[w * L + e * 32 + lane];
      warp_merge_lists<E>(acc, u, lane);
    }
#pragma unroll
    for (int e = 0; e < E; ++e) sm.best[e * 32 + lane] = acc[e];
  }
  S::sync();
}

// Writes the row's result from sm.best: V/I (first k; empty keys as
// (-FLT_MAX, -1)) and/or its L keys.
template <int L>
__device__ __forceinline__ void write_row(const FinishArgs& fa, const FinishSmem& sm, int64_t b, int tid,
                                          int nthreads) {
  for (int i = tid; i < L; i += nthreads) {
    const uint64_t key = sm.best[i];
    if (fa.V != nullptr && i < fa.k) {
      fa.V[b * fa.k + i] = key ? key_value(key) : -3.402823466e+38f;
      fa.I[b * fa.k + i] = key ? key_index(key) : -1;
    }
    if (fa.keys_out != nullptr) fa.keys_out[b * L + i] = key;
  }
}

// Stores sm.best (row b) into slot [slot][rank] of every rank's receive
// buffer and sets the row's flag there to `tag`: thread p (of the first
// warp) writes rank p's copy with 16-byte stores and then the flag with a
// system-scope release store, so the row is visible to rank p before its flag
// by program order alone.
template <int L>
__device__ __forceinline__ void publish_row(const ExchangeDev& ex, const FinishSmem& sm, int slot,
                                            unsigned long long tag, int64_t b, int tid) {
  if (tid >= ex.world) return;
  const int p = tid;
  const int64_t at = ((int64_t)slot * ex.world + ex.rank) * ex.max_rows + b;
  ulonglong2* dst = reinterpret_cast<ulonglong2*>(ex.peer_recv[p] + at * L);
  const ulonglong2* src = reinterpret_cast<const ulonglong2*>(sm.best);
#pragma unroll 8
  for (int i = 0; i < L / 2; ++i) __stcg(dst + i, src[i]);
  st_release_sys_u64(ex.peer_flag[p] + at, tag);
}

// Clears fa.zero (pipelined encode): part of CTA `cta` of `ctas`, `nthreads`
// threads, 16-byte stores.
__device__ __forceinline__ void clear_sync_region(const FinishArgs& fa, int cta, int ctas, int tid, int nthreads) {
  if (fa.zero == nullptr) return;
  uint4* z = reinterpret_cast<uint4*>(fa.zero);
  const int64_t n = fa.zero_words / 4;
  for (int64_t i = (int64_t)cta * nthreads + tid; i < n; i += (int64_t)ctas * nthreads) z[i] = make_uint4(0u, 0u, 0u, 0u);
}

// Finishes rows row0, row0 + row_step, ... < fa.rows.  Every thread of the
// CTA (or of the group S synchronises) calls it.  Two phases, which the
// pipelined encode runs apart (the first while the next batch's first tile
// streams, the second after that batch's last tile):
//   finish_rows_local: each row's select over this GPU's lists, then its V / I
//     (or keys) -- or, with the exchange, its publication to every rank;
//   finish_rows_world (exchange only): the bounded wait for the other ranks'
//     copies of these rows, the select over the world's lists, V / I.
// With the exchange, all of a CTA's rows are published before any wait, so
// CTAs that run at the same time on different GPUs never wait on each other
// in a cycle.  finish_rows_local returns the exchange's step (0 without it).
template <int L, class S = SyncCta>
__device__ unsigned long long finish_rows_local(const FinishArgs& fa, FinishSmem& sm, int64_t row0, int64_t row_step,
                                                int tid, int nthreads) {
  unsigned long long step = 0;
  int slot = 0;
  if (fa.use_ex) {
    step = *reinterpret_cast<volatile unsigned long long*>(fa.ex.state);
    slot = (int)(step & 1ull);
  }
  for (int64_t b = row0; b < fa.rows; b += row_step) {
    select_row<L, S>(fa.lists, fa.nlists, fa.stride, fa.pitch, fa.tail, b, fa.k, 0xffffffffu, sm, tid, nthreads);
    if (fa.use_ex)
      publish_row<L>(fa.ex, sm, slot, step + 1ull, b, tid);
    else
      write_row<L>(fa, sm, b, tid, nthreads);
    S::sync();
  }
  return step;
}

template <int L, class S = SyncCta>
__device__ void finish_rows_world(const FinishArgs& fa, FinishSmem& sm, int64_t row0, int64_t row_step, int tid,
                                  int nthreads, unsigned long long step) {
  if (!fa.use_ex) return;
  const int slot = (int)(step & 1ull);
  const ExchangeDev& ex = fa.ex;
  const unsigned long long t0 = global_timer_ns();
  for (int64_t b = row0; b < fa.rows; b += row_step) {
    if (tid == 0) sm.valid = 0u;
    S::sync();
    if (tid < ex.world) {
      const unsigned long long* f = ex.flag + ((int64_t)slot * ex.world + tid) * ex.max_rows + b;
      bool ok = true;
      while (ld_acquire_sys_u64(f) != step + 1ull) {
        if (global_timer_ns() - t0 > ex.wait_ns) {
          ok = false;
          break;
        }
        __nanosleep(64);
      }
      if (ok)
        atomicOr(&sm.valid, 1u << tid);
      else
        raise_device_error(kErrExchangeTimeout);
    }
    S::sync();
    select_row<L, S>(ex.recv + (int64_t)slot * ex.world * ex.max_rows * L, ex.world, ex.max_rows, L, 0, b, fa.k,
                     sm.valid, sm, tid, nthreads);
    write_row<L>(fa, sm, b, tid, nthreads);
    S::sync();
  }
  // Every CTA of this step has passed its waits: the last one advances the step.
  if (tid == 0) {
    __threadfence();
    const unsigned long long done = atomicAdd(ex.state + 1, 1ull);
    if (done == (unsigned long long)gridDim.x - 1ull) {
      ex.state[1] = 0ull;
      __threadfence();
      ex.state[0] = step + 1ull;
    }
  }
}

template <int L, class S = SyncCta>
__device__ void finish_rows(const FinishArgs& fa, FinishSmem& sm, int64_t row0, int64_t row_step, int tid,
                            int nthreads) {
  const unsigned long long step = finish_rows_local<L, S>(fa, sm, row0, row_step, tid, nthreads);
  finish_rows_world<L, S>(fa, sm, row0, row_step, tid, nthreads, step);
}

}  // namespace stk
