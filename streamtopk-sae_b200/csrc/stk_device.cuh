// Device-side building blocks for the B200 streaming top-k SAE encoder.
//
//   * 64-bit selection keys: (order-preserving float bits << 32) | ~feature.
//     Larger key == larger score, and among equal scores the smaller feature
//     index.  Keys are unique, so every selection below is deterministic and
//     independent of tile order, CTA count and GPU count.  Key 0 means
//     "empty" and sorts below every real score.
//   * Per-thread bitonic networks over register arrays (one thread owns one
//     batch row), used by the top-k accumulator.
//   * Warp-cooperative bitonic merge over lists spread across a warp (merge
//     kernel).
//   * Thin inline-PTX wrappers for mbarrier, TMA, tcgen05 and TMEM.
//
// Semantics kept from the reference (streamtopk_sae/csrc/cuda/topk_buffer.cuh:
// 9-81, streamtopk_exact.cu:137-148): a score enters the running top-k only
// if it is strictly greater than the current k-th value; NaN never enters.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace stk {

constexpr int kRows = 128;          // batch rows per M tile (tcgen05 M)
constexpr int kAppendMax = 32;      // most per-row append slots between merges
constexpr uint64_t kEmptyKey = 0ull;
// Upper bound for any single spin-wait on an mbarrier (nanoseconds).  A wait
// that runs out sets the device error word and makes every role drain out.
constexpr unsigned long long kWaitLimitNs = 4000000000ull;

// Error codes written to the device error word (first one wins).
constexpr unsigned kErrWaitTimeout = 1;
constexpr unsigned kErrTmemAlloc = 2;

__device__ __forceinline__ uint32_t float_order(float v) {
  uint32_t u = __float_as_uint(v);
  if ((u << 1) == 0) u = 0;  // -0.0 and +0.0 are the same score
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float order_float(uint32_t o) {
  uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t make_key(float v, uint32_t feature) {
  return (uint64_t(float_order(v)) << 32) | uint64_t(~feature);
}

__device__ __forceinline__ float key_value(uint64_t key) {
  return order_float(uint32_t(key >> 32));
}

__device__ __forceinline__ int32_t key_index(uint64_t key) {
  return int32_t(~uint32_t(key));
}

__device__ __forceinline__ uint64_t kmax(uint64_t a, uint64_t b) { return a > b ? a : b; }
__device__ __forceinline__ uint64_t kmin(uint64_t a, uint64_t b) { return a > b ? b : a; }

// Compare-exchange of two keys: a <- max, b <- min.  Written as one 64-bit
// setp and two selp so the compiler emits predicated selects (no branches).
__device__ __forceinline__ void cx(uint64_t& a, uint64_t& b) {
  uint64_t mx, mn;
  asm("{\n\t.reg .pred p;\n\t"
      "setp.gt.u64 p, %2, %3;\n\t"
      "selp.b64 %0, %2, %3, p;\n\t"
      "selp.b64 %1, %3, %2, p;\n\t}\n"
      : "=l"(mx), "=l"(mn)
      : "l"(a), "l"(b));
  a = mx;
  b = mn;
}

// ---------------------------------------------------------------------------
// PTX wrappers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// One try_wait that may suspend the thread for up to kSuspendNs (the thread
// is woken early when the phase completes), so waiting warps do not spin and
// steal issue slots from the epilogue warps sharing their scheduler.
constexpr uint32_t kSuspendNs = 200000;
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false if the
// wait ran out, or if abort is given and another role already gave up
// (*abort != 0).  Drain waits pass abort = nullptr and end on time only.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(a, parity)) return true;
    if (abort != nullptr && *abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tma_prefetch_desc(const void* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 2-D tiled TMA load (no multicast) into this CTA's shared memory; completion
// is signalled as transaction bytes on the mbarrier.
__device__ __forceinline__ void tma_load_2d(const void* map, uint64_t* bar, void* dst, int x, int y,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Warp-wide TMEM allocation; the base address is written to *dst (shared).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 or fp16 in, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier once all previously issued tcgen05.mma of this thread complete.
// Same with operands in TF32 (fp32 bit patterns; the tensor core reads the top
// 19 bits), K = 8 per instruction.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with FP8 operands, kind::f8f6f4 (the instruction descriptor's A/B
// format code 0 = E4M3), K = 32 per instruction: 32 bytes of a 128-byte row,
// so the descriptor advances exactly as for 16-bit operands.
__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Makes this thread's generic-proxy writes to shared memory visible to the
// async proxy (tensor-core operand reads) after the next synchronisation.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// The TF32 value the tensor core reads from an fp32 operand: the low 13
// mantissa bits cleared (truncation toward zero).  x - trunc_tf32(x) is exact
// in fp32 and carries the 13 bits the hi part drops.
__device__ __forceinline__ float trunc_tf32(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane
// (base lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
        "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
        "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
        "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Wait for outstanding TMEM loads and tie the destination registers of the
// last load to the wait, so no use of them is scheduled before it.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
        "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
        "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]),
        "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
      :
      : "memory");
}

// Thread t of the warp stores v[j] to lane (base lane + t), column col + j,
// j < 32 (the store counterpart of tmem_ld32).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32"
      " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Two consecutive 32-bit columns of this thread's lane (one 64-bit key).
__device__ __forceinline__ uint64_t tmem_ld_key(uint32_t taddr) {
  uint32_t lo, hi;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(lo), "=r"(hi) : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(lo), "+r"(hi)::"memory");
  return (uint64_t(hi) << 32) | lo;
}

// ---- CTA pairs (a 2-CTA cluster sharing one MMA: cta_group::2) ----------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier of another CTA of the cluster (cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory whose completion is counted
// on an mbarrier of either CTA of the pair (cluster address; no multicast).
__device__ __forceinline__ void tma_load_2d_pair(const void* map, uint32_t cluster_bar, void* dst, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(cluster_bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D (both CTAs' TMEM, M/2 rows each) (+)= A * B^T across the pair, issued by
// the pair's first CTA: A's rows and B's rows are split between the two CTAs'
// shared memory at the same offsets.  No output lanes disabled.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  const uint32_t z = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}

// The pair form of umma_f8 (E4M3 operands, kind::f8f6f4).
__device__ __forceinline__ void umma_f8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  const uint32_t z = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}

// Arrive on the mbarrier (cluster address, either CTA of the pair) once the
// pair MMAs issued so far by this thread complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: rows of 128 B, 8-row atoms of 1024 B (stride byte offset),
// version 1 (sm_100), layout type 2 (SWIZZLE_128B).  The tile base must be
// 1024-byte aligned; advancing K by 16 elements adds 32 B to the start address.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr & 0x3ffffu) >> 4);         // start address
  d |= uint64_t(1) << 16;                          // leading byte offset (ignored for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;                  // stride byte offset
  d |= uint64_t(1) << 46;                          // descriptor version
  d |= uint64_t(2) << 61;                          // SWIZZLE_128B
  return d;
}

// Shared-memory matrix descriptor, K-major, 64-byte swizzle (8-row groups
// 512 bytes apart); K advances by 32 bytes = +2 in the address field.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr & 0x3ffffu) >> 4);         // start address
  d |= uint64_t(1) << 16;                          // leading byte offset (ignored for swizzled K-major)
  d |= uint64_t(512 >> 4) << 32;                   // stride byte offset
  d |= uint64_t(1) << 46;                          // descriptor version
  d |= uint64_t(4) << 61;                          // SWIZZLE_64B
  return d;
}

// Instruction descriptor, kind::f16, fp32 accumulate, A and B K-major.
// ab_format: 0 = fp16, 1 = bf16.
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t ab_format, uint32_t m, uint32_t n) {
  return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Instruction descriptor, kind::tf32 (A and B format 2), fp32 accumulate, K-major.
__host__ __device__ constexpr uint32_t make_idesc_tf32(uint32_t m, uint32_t n) { return make_idesc_f16(2u, m, n); }

// ---------------------------------------------------------------------------
// Per-thread networks (N is a compile-time power of two; fully unrolled so the
// arrays stay in registers).
// ---------------------------------------------------------------------------
template <int N>
__device__ __forceinline__ void sort_desc(uint64_t (&a)[N]) {
#pragma unroll
  for (int size = 2; size <= N; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          if ((i & size) == 0)
            cx(a[i], a[j]);  // descending block
          else
            cx(a[j], a[i]);  // ascending block
        }
      }
    }
  }
}

// Turns a bitonic sequence into a descending one.
template <int N>
__device__ __forceinline__ void merge_desc(uint64_t (&a)[N]) {
#pragma unroll
  for (int stride = N >> 1; stride > 0; stride >>= 1) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const int j = i ^ stride;
      if (j > i) cx(a[i], a[j]);
    }
  }
}

// ---------------------------------------------------------------------------
// Per-row top-L accumulator, one thread per batch row.
//
// Layout (slot-major, row-minor, so the 32 threads of a warp touch 32
// consecutive 8-byte words):
//   top[s * kRows + (r ^ (s & 31))], s < L : row r's best L keys, descending
//                               (0 = empty), shared memory.  The XOR swizzle
//                               keeps per-thread access conflict-free and lets
//                               a warp read one row's 32 consecutive slots in
//                               2 wavefronts instead of 32 (store_partials).
//   app[s * kRows + r], s < A : row r's unsorted survivors since the last
//                               merge, in shared memory or (when shared
//                               memory is short) in an L2-resident workspace
//                               slice of this CTA, written and read back by
//                               the same thread only
// ---------------------------------------------------------------------------
// Dynamic shared memory of every kernel in this library.  Per-row lists are
// addressed by byte offset from this symbol so that code outside the kernel
// body still compiles to shared-memory instructions.
extern __shared__ __align__(16) uint8_t stk_smem[];

__device__ __forceinline__ uint64_t* smem_keys(uint32_t off) { return reinterpret_cast<uint64_t*>(stk_smem + off); }

// Slot s of row r in a swizzled top list at byte offset `top`.
__device__ __forceinline__ uint64_t& top_slot(uint32_t top, int s, int r) {
  return smem_keys(top)[s * kRows + (r ^ (s & 31))];
}

// Merge row r's n waiting survivors (A append slots, unsorted) into its sorted
// top list and return the new threshold: the value of the (kth+1)-th best key,
// never below floor_thr (a lower bound known from elsewhere, -inf if none).
// The append slots are in shared memory (APP_SMEM, app_off = byte offset from
// stk_smem) or in global memory (app_g).  Kept out of line: it runs rarely and
// is large.
template <int L, int A, bool APP_SMEM>
__device__ __forceinline__ float merge_survivors_impl(uint32_t top_off, uint32_t app_off,
                                                      const uint64_t* __restrict__ app_g, int r, int n, int kth,
                                                      float floor_thr) {
  static_assert(A == 16 || A == 32, "append slots");
#define TOP(s) top_slot(top_off, (s), r)
  uint64_t a[A];
#pragma unroll
  for (int s = 0; s < A; ++s) {
    if constexpr (APP_SMEM)
      a[s] = (s < n) ? smem_keys(app_off)[s * kRows + r] : kEmptyKey;
    else
      a[s] = (s < n) ? (uint64_t)__ldcg(reinterpret_cast<const unsigned long long*>(app_g + s * kRows + r))
                     : kEmptyKey;
  }
  sort_desc<A>(a);
  if constexpr (L == 32) {
    // top-32 of two sorted lists: c[i] = max(top[i], a'[31 - i]) is bitonic
    // (a' = a padded with empty keys; only the last A positions change).
    uint64_t c[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) c[i] = TOP(i);
#pragma unroll
    for (int q = 0; q < A; ++q) c[32 - A + q] = kmax(c[32 - A + q], a[A - 1 - q]);
    merge_desc<32>(c);
#pragma unroll
    for (int i = 0; i < 32; ++i) TOP(i) = c[i];
  } else {
    // Only the last A positions can change in c[i] = max(top[i], a'[L-1-i]).
#pragma unroll
    for (int q = 0; q < A; ++q) TOP(L - A + q) = kmax(TOP(L - A + q), a[A - 1 - q]);
    // Bitonic merge: strides >= 32 in shared memory, then 32-blocks in registers.
#pragma unroll
    for (int stride = L >> 1; stride >= 32; stride >>= 1) {
#pragma unroll 16
      for (int i = 0; i < L; ++i) {
        if ((i & stride) == 0) {
          uint64_t x = TOP(i), y = TOP(i + stride);
          cx(x, y);
          TOP(i) = x;
          TOP(i + stride) = y;
        }
      }
    }
#pragma unroll 1
    for (int blk = 0; blk < L / 32; ++blk) {
      uint64_t c[32];
#pragma unroll
      for (int q = 0; q < 32; ++q) c[q] = TOP(blk * 32 + q);
      merge_desc<32>(c);
#pragma unroll
      for (int q = 0; q < 32; ++q) TOP(blk * 32 + q) = c[q];
    }
  }
  const uint64_t kk = TOP(kth);
#undef TOP
  return kk ? fmaxf(key_value(kk), floor_thr) : floor_thr;
}

// Out of line (the hot loop stays small: the instruction cache matters).
template <int L, int A, bool APP_SMEM>
__device__ __noinline__ float merge_survivors(uint32_t top_off, uint32_t app_off, const uint64_t* __restrict__ app_g,
                                              int r, int n, int kth, float floor_thr) {
  return merge_survivors_impl<L, A, APP_SMEM>(top_off, app_off, app_g, r, n, kth, floor_thr);
}

// Key i of a list held in tensor memory occupies 32-bit columns 2i (low half)
// and 2i + 1 (high half) of the owning thread's lane.
__device__ __forceinline__ uint64_t col_key(const uint32_t (&v)[32], int j) {
  return (uint64_t(v[2 * j + 1]) << 32) | v[2 * j];
}
__device__ __forceinline__ void set_col_key(uint32_t (&v)[32], int j, uint64_t key) {
  v[2 * j] = uint32_t(key);
  v[2 * j + 1] = uint32_t(key >> 32);
}

// merge_survivors for a top list in tensor memory (tlist: the TMEM address of
// key 0 of this thread's row; L keys at columns [0, 2L)).  Same steps and
// result: the A sorted survivors enter through the last A positions, then a
// bitonic merge -- strides >= 32 on pairs of 16-key groups, then 32-key blocks
// in registers.  Every lane of the warp calls it together (warp-wide TMEM
// loads and stores).
template <int L, int A, bool APP_SMEM>
__device__ __noinline__ float merge_survivors_tmem(uint32_t tlist, uint32_t app_off,
                                                   const uint64_t* __restrict__ app_g, int r, int n, int kth,
                                                   float floor_thr) {
  static_assert(A == 16 || A == 32, "append slots");
  static_assert(L >= 64 && L % 32 == 0, "list length");
  uint64_t a[A];
#pragma unroll
  for (int s = 0; s < A; ++s) {
    if constexpr (APP_SMEM)
      a[s] = (s < n) ? smem_keys(app_off)[s * kRows + r] : kEmptyKey;
    else
      a[s] = (s < n) ? (uint64_t)__ldcg(reinterpret_cast<const unsigned long long*>(app_g + s * kRows + r))
                     : kEmptyKey;
  }
  sort_desc<A>(a);
#pragma unroll
  for (int h = 0; h < A / 16; ++h) {
    uint32_t v[32];
    const int i0 = L - A + 16 * h;
    tmem_ld32(tlist + 2 * i0, v);
    tmem_wait_ld(v);
#pragma unroll
    for (int q = 0; q < 16; ++q) set_col_key(v, q, kmax(col_key(v, q), a[A - 1 - (16 * h + q)]));
    tmem_st32(tlist + 2 * i0, v);
  }
  tmem_wait_st();
#pragma unroll 1
  for (int stride = L >> 1; stride >= 32; stride >>= 1) {
#pragma unroll 1
    for (int i0 = 0; i0 < L; i0 += 16) {
      if (i0 & stride) continue;
      uint32_t p[32], q[32];
      tmem_ld32(tlist + 2 * i0, p);
      tmem_ld32(tlist + 2 * (i0 + stride), q);
      tmem_wait_ld(p);
      tmem_wait_ld(q);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        uint64_t x = col_key(p, j), y = col_key(q, j);
        cx(x, y);
        set_col_key(p, j, x);
        set_col_key(q, j, y);
      }
      tmem_st32(tlist + 2 * i0, p);
      tmem_st32(tlist + 2 * (i0 + stride), q);
    }
    tmem_wait_st();
  }
#pragma unroll 1
  for (int blk = 0; blk < L / 32; ++blk) {
    uint32_t p[32], q[32];
    tmem_ld32(tlist + 64 * blk, p);
    tmem_ld32(tlist + 64 * blk + 32, q);
    tmem_wait_ld(p);
    tmem_wait_ld(q);
    uint64_t c[32];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      c[j] = col_key(p, j);
      c[16 + j] = col_key(q, j);
    }
    merge_desc<32>(c);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      set_col_key(p, j, c[j]);
      set_col_key(q, j, c[16 + j]);
    }
    tmem_st32(tlist + 64 * blk, p);
    tmem_st32(tlist + 64 * blk + 32, q);
  }
  tmem_wait_st();
  const uint64_t kk = tmem_ld_key(tlist + 2 * kth);
  return kk ? fmaxf(key_value(kk), floor_thr) : floor_thr;
}

// vals[j & 31] for a per-lane (divergent) j, by a 5-level select tree.
__device__ __forceinline__ float pick32(const float (&vals)[32], int j) {
  float t16[16], t8[8], t4[4], t2[2];
#pragma unroll
  for (int i = 0; i < 16; ++i) t16[i] = (j & 16) ? vals[i + 16] : vals[i];
#pragma unroll
  for (int i = 0; i < 8; ++i) t8[i] = (j & 8) ? t16[i + 8] : t16[i];
#pragma unroll
  for (int i = 0; i < 4; ++i) t4[i] = (j & 4) ? t8[i + 4] : t8[i];
#pragma unroll
  for (int i = 0; i < 2; ++i) t2[i] = (j & 2) ? t4[i + 2] : t4[i];
  return (j & 1) ? t2[1] : t2[0];
}

// The n (<= A) unsorted append slots of row r, sorted descending and padded
// with empty keys to kAppendMax keys, stored at dst (16-byte aligned).  Out of
// line like merge_survivors: it runs once per unit.
// The first S slots sorted (S >= n), the rest of the run empty.
template <int S, int A, bool APP_SMEM>
__device__ __forceinline__ void sort_tail_run(uint32_t app_off, const uint64_t* __restrict__ app_g, int r, int n,
                                              ulonglong2* __restrict__ d) {
  uint64_t a[S];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    if constexpr (APP_SMEM)
      a[s] = (s < n) ? smem_keys(app_off)[s * kRows + r] : kEmptyKey;
    else
      a[s] = (s < n) ? (uint64_t)__ldcg(reinterpret_cast<const unsigned long long*>(app_g + s * kRows + r))
                     : kEmptyKey;
  }
  sort_desc<S>(a);
#pragma unroll
  for (int i = 0; i < S / 2; ++i) d[i] = make_ulonglong2(a[2 * i], a[2 * i + 1]);
#pragma unroll
  for (int i = S / 2; i < kAppendMax / 2; ++i) d[i] = make_ulonglong2(0ull, 0ull);
}

template <int A, bool APP_SMEM>
__device__ __noinline__ void store_sorted_tail(uint32_t app_off, const uint64_t* __restrict__ app_g, int r, int n,
                                               uint64_t* __restrict__ dst) {
  ulonglong2* d = reinterpret_cast<ulonglong2*>(dst);
  // The network's size follows the warp's largest count (usually a few keys
  // are pending at a unit's end): 8 keys cost 24 compare-exchanges, A = 32
  // cost 240.  Warp-uniform, so no lane diverges.
  int nmax = n;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) nmax = max(nmax, __shfl_xor_sync(0xffffffffu, nmax, o));
  if (nmax <= 8) {
    sort_tail_run<8, A, APP_SMEM>(app_off, app_g, r, n, d);
  } else if (A > 16 && nmax > 16) {
    sort_tail_run<(A > 16 ? A : 16), A, APP_SMEM>(app_off, app_g, r, n, d);
  } else {
    sort_tail_run<16, A, APP_SMEM>(app_off, app_g, r, n, d);
  }
}

template <int L, int A, bool APP_SMEM, bool TOPT = false>
struct RowTopK {
  uint32_t top;     // byte offset of top[0] from stk_smem, or (TOPT) the TMEM address of this row's list
  uint32_t app_s;   // byte offset of the shared append slots (APP_SMEM)
  uint64_t* app_g;  // global append slots (!APP_SMEM)
  int r;            // row within the M tile
  int cnt;          // survivors waiting in the append slots
  float thr;        // value of the k-th best key so far (-inf until k are held)
  float floor_thr;  // known lower bound of the row's k-th score (-inf if none)
  int kth;          // k - 1

  __device__ __forceinline__ void init(uint32_t top_, uint32_t app_s_, uint64_t* app_g_, int row, int k) {
    top = top_;
    app_s = app_s_;
    app_g = app_g_;
    r = row;
    cnt = 0;
    thr = -__int_as_float(0x7f800000);
    floor_thr = thr;
    kth = k - 1;
    if constexpr (TOPT) {
      uint32_t z[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) z[j] = 0u;
#pragma unroll
      for (int c = 0; c < 2 * L; c += 32) tmem_st32(top + c, z);
      tmem_wait_st();
    } else {
#pragma unroll 4
      for (int s = 0; s < L; ++s) top_slot(top, s, r) = kEmptyKey;
    }
  }

  __device__ __forceinline__ void flush() {
    if constexpr (TOPT)
      thr = merge_survivors_tmem<L, A, APP_SMEM>(top, app_s, app_g, r, cnt, kth, floor_thr);
    else
      thr = merge_survivors<L, A, APP_SMEM>(top, app_s, app_g, r, cnt, kth, floor_thr);
    cnt = 0;
  }

  // flush() without the call: for callers that hold many keys in registers
  // across it (a call would make them spill around the loop).
  __device__ __forceinline__ void flush_inline() {
    if constexpr (TOPT) {
      flush();
    } else {
      thr = merge_survivors_impl<L, A, APP_SMEM>(top, app_s, app_g, r, cnt, kth, floor_thr);
      cnt = 0;
    }
  }

  __device__ __forceinline__ void push(uint64_t key) {
    if constexpr (APP_SMEM)
      smem_keys(app_s)[cnt * kRows + r] = key;
    else
      __stcg(reinterpret_cast<unsigned long long*>(app_g + cnt * kRows + r), (unsigned long long)key);
    ++cnt;
  }

  // Offer one chunk of 32 scores (vals[j] is feature f0 + j).  valid_mask
  // marks real features (tail of F, rows beyond B).  All 32 lanes of the warp
  // must call this together: a merge runs for every lane as soon as one lane
  // would overflow its append slots.  A chunk may bring more survivors than
  // A, so the chunk is taken in (at most 32 / A) passes of A candidates.
  // Survivors are rare once a threshold is known, so the warp loops once per
  // survivor of its busiest lane; each lane takes its lowest pending survivor
  // (value picked from registers by a select tree, no divergent branches).
  __device__ __forceinline__ void offer(const float (&vals)[32], uint32_t f0, uint32_t valid_mask) {
    uint32_t mask = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) mask |= (vals[j] > thr) ? (1u << j) : 0u;
    mask &= valid_mask;
#pragma unroll
    for (int part = 0; part < 32 / A; ++part) {
      const uint32_t pm = A == 32 ? 0xffffffffu : (0xffffu << (16 * part));
      if (__any_sync(0xffffffffu, cnt + __popc(mask & pm) > A)) {
        flush();
        mask = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) mask |= (vals[j] > thr) ? (1u << j) : 0u;
        mask &= valid_mask;
      }
      uint32_t m = mask & pm;
      while (__any_sync(0xffffffffu, m != 0u)) {
        const bool has = m != 0u;
        const int j = __ffs(m) - 1;  // -1 (ignored) when this lane has none
        m &= m - 1u;
        const float v = pick32(vals, j);
        if (has) push(make_key(v, f0 + uint32_t(j)));
      }
    }
  }

  // Offer keys[0..n) of a descending array (n <= N, n <= A): the ones above
  // the threshold form a prefix.  Warp-wide like offer().
  template <int N>
  __device__ __forceinline__ void offer_sorted(const uint64_t (&keys)[N], int n) {
    int s = 0;
#pragma unroll
    for (int j = 0; j < N; ++j) s += (j < n && keys[j] != kEmptyKey && key_value(keys[j]) > thr) ? 1 : 0;
    if (__any_sync(0xffffffffu, cnt + s > A)) {
      flush_inline();
      s = 0;
#pragma unroll
      for (int j = 0; j < N; ++j) s += (j < n && keys[j] != kEmptyKey && key_value(keys[j]) > thr) ? 1 : 0;
    }
#pragma unroll
    for (int j = 0; j < N; ++j) {
      if (!__any_sync(0xffffffffu, j < s)) break;
      if (j < s) push(keys[j]);
    }
  }

  // Raise the filter to a lower bound of the row's k-th score obtained from a
  // sample (scores strictly below `lb` can never be in the row's top-k).
  __device__ __forceinline__ void set_floor(float lb) {
    const float t = nextafterf(lb, -__int_as_float(0x7f800000));  // keep scores == lb
    floor_thr = fmaxf(floor_thr, t);
    thr = fmaxf(thr, floor_thr);
  }

  __device__ __forceinline__ void finish() {
    if (__any_sync(0xffffffffu, cnt > 0)) flush();
  }

  // Instead of a final flush: writes the pending survivors, sorted descending
  // and padded with empty keys to kAppendMax, at dst (16-byte aligned) -- a
  // second sorted run beside the row's list, which the finish step reads too.
  __device__ __forceinline__ void store_tail(uint64_t* dst) {
    store_sorted_tail<A, APP_SMEM>(app_s, app_g, r, cnt, dst);
    cnt = 0;
  }
};

// ---------------------------------------------------------------------------
// Warp-cooperative lists: element i = e * 32 + lane, E = L / 32 per lane.
// ---------------------------------------------------------------------------
template <int E>
__device__ __forceinline__ void warp_merge_desc(uint64_t (&a)[E], int lane) {
#pragma unroll
  for (int stride = E * 16; stride > 0; stride >>= 1) {
    if (stride >= 32) {
      const int s = stride >> 5;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if ((e & s) == 0) {
          const uint64_t x = a[e], y = a[e | s];
          a[e] = kmax(x, y);
          a[e | s] = kmin(x, y);
        }
      }
    } else {
      const bool lower = (lane & stride) == 0;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const uint64_t y = __shfl_xor_sync(0xffffffffu, a[e], stride);
        a[e] = lower ? kmax(a[e], y) : kmin(a[e], y);
      }
    }
  }
}

// t <- best L of (t u u), both descending lists of L = 32 * E keys.
template <int E>
__device__ __forceinline__ void warp_merge_lists(uint64_t (&t)[E], const uint64_t (&u)[E], int lane) {
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const uint64_t y = __shfl_sync(0xffffffffu, u[E - 1 - e], 31 - lane);
    t[e] = kmax(t[e], y);
  }
  warp_merge_desc<E>(t, lane);
}

}  // namespace stk
