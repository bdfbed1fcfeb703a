// sm100.cuh — thin inline-PTX wrappers for the Blackwell (sm_100a) features the
// GEMM kernels use: mbarriers, TMA tiled loads, tcgen05 (TMEM alloc, MMA,
// commit, loads) and the shared-memory matrix descriptors.
//
// Every spin wait in this file is bounded: it gives up after `budget` SM clock
// cycles (or as soon as another warp of the CTA has given up), records
// OJX_DEVERR_TIMEOUT in the device error word and reports failure to the
// caller, which then drains its in-flight work and returns.  No wait here can
// hang a GPU.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace ojx {

// Device error word of the library (all kernels are built as one translation
// unit, ojx_kernels.cu).  Bit 0: a bounded wait expired.
__device__ unsigned int g_dev_error = 0;
constexpr unsigned int OJX_DEVERR_TIMEOUT = 1u;
// Bit 1: a device-side bounds check failed (only the OJX_DEBUG_BOUNDS build checks).
constexpr unsigned int OJX_DEVERR_BOUNDS = 2u;

// ── debug bounds checks (build with -DOJX_DEBUG_BOUNDS) ─────────────────────
// Every TMA tile origin and every epilogue store of the GEMM kernels passes through
// these checks in the debug build (libojx_debug.so); in the normal build they are
// constant true and vanish.  A failed check sets OJX_DEVERR_BOUNDS, records the
// first failure in g_bounds_info (site, two coordinates, the extent they broke)
// and the caller skips the access: nothing traps, a skipped TMA load leaves its
// consumer to a bounded wait, and the host reads the record through
// ojx_poll_device_error.
#ifdef OJX_DEBUG_BOUNDS
constexpr bool kDebugBounds = true;
#else
constexpr bool kDebugBounds = false;
#endif
__device__ long long g_bounds_info[4] = {0, 0, 0, 0};

enum BoundsSite : int {
  SITE_TC_LOAD_A = 1, SITE_TC_LOAD_B = 2, SITE_TC_STORE_TMA = 3, SITE_TC_STORE_REG = 4,
  SITE_SK_LOAD_W = 5, SITE_SK_LOAD_X = 6, SITE_SK_STORE = 7, SITE_SK_SLOT = 8,
  SITE_SIMT_STORE = 9, SITE_FA_LOAD = 10, SITE_FA_STORE = 11
};

__device__ __forceinline__ bool bounds_check(bool ok, int site, long long a, long long b,
                                             long long ext) {
  if (!kDebugBounds || ok) return true;
  if ((atomicOr(&g_dev_error, OJX_DEVERR_BOUNDS) & OJX_DEVERR_BOUNDS) == 0) {
    g_bounds_info[0] = site;
    g_bounds_info[1] = a;
    g_bounds_info[2] = b;
    g_bounds_info[3] = ext;
  }
  return false;
}

// Origin (c0, c1) of a tiled TMA copy over a tensor with extents (e0, e1) of esz-byte
// elements: inside the tensor, and c0 * esz on a 16-byte boundary (an unaligned
// innermost coordinate is an illegal instruction on this GPU).
__device__ __forceinline__ bool tma_origin_ok(int site, long long c0, long long c1, long long e0,
                                              long long e1, int esz) {
  if (!kDebugBounds) return true;
  const bool ok = c0 >= 0 && c1 >= 0 && c0 < e0 && c1 < e1 && (c0 * esz) % 16 == 0;
  return bounds_check(ok, site, c0, c1, c0 < e0 ? e1 : e0);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Explicit shared-space accesses (32-bit shared addresses).
__device__ __forceinline__ float ld_shared_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// ── mbarrier ────────────────────────────────────────────────────────────────
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  `abort_flag` lives in the
// CTA's shared memory; any warp that times out sets it so the others stop too.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t budget,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (static_cast<uint64_t>(clock64() - t0) > budget) {
      *abort_flag = 1;
      atomicOr(&g_dev_error, OJX_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// Bounded wait used while draining in-flight work before a CTA exits: it ignores
// the abort flag (the point is to let already-issued copies/MMAs land) but still
// gives up after `budget` cycles.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, uint64_t budget) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (static_cast<uint64_t>(clock64() - t0) > budget) {
      atomicOr(&g_dev_error, OJX_DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// ── TMA ─────────────────────────────────────────────────────────────────────
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Fetch a 2-D tile into L2 only (no shared memory, no completion signal).  A
// prefetch is a hint: reads issued later still observe every write to the tile.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

// Load with acquire semantics at GPU scope: later reads of this thread (and of
// threads that synchronise with it afterwards) see what the releasing writer saw.
__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Strong (relaxed, GPU scope) 64-bit accesses.  An aligned 64-bit strong access is
// single-copy atomic: a reader sees either the whole old or the whole new word,
// which is what lets a value and the tag written beside it validate each other.
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Release/acquire fence at GPU scope (lighter than __threadfence's sequentially
// consistent fence): before a signalling atomic it releases the writes that this
// thread observed, after an observing atomic it acquires the writes it announced.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned)
// from global memory into this CTA's shared memory, completing on `bar` through
// complete_tx.  No multicast.
__device__ __forceinline__ void bulk_load_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}
// Orders this thread's earlier generic-proxy accesses (and what it acquired)
// before its later async-proxy (TMA) accesses, in every state space.
__device__ __forceinline__ void fence_proxy_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }

// ── programmatic dependent launch ───────────────────────────────────────────
// Block until the grids this one depends on (the previous kernel on the stream,
// when it was launched with programmatic stream serialization) have completed and
// their memory writes are visible.  Returns at once without such a dependency.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel on the stream to begin launching before this grid ends.
__device__ __forceinline__ void grid_dep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// 2-D tiled load into this CTA's shared memory; completion is signalled on `bar`
// through complete_tx.  c0 is the innermost coordinate (elements).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// 3-D tiled load (c2: batch index of a batched operand).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 2-D tiled store from this CTA's shared memory (bulk-group completion).
// Elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t c0,
                                             int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int32_t c0,
                                             int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until every committed bulk store has finished READING shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until every committed bulk store has completed (writes performed).
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ── tcgen05 ─────────────────────────────────────────────────────────────────
// TMEM allocation: executed by one full warp; the address lands in shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (bf16 or fp16 inputs, fp32 accumulate).
// The same MMA with its A operand (M rows = TMEM lanes, K packed two 16-bit
// elements per 32-bit column) read from tensor memory at column address a_tmem.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same for tf32 inputs (32-bit containers, the MMA reads the tf32 bits).
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on `bar` when every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (tcgen05 "version 1" format):
// start address, leading-dimension byte offset and stride byte offset, all >>4.
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 / kind::tf32 with fp32 accumulation.
// fmt: 0 = f16, 1 = bf16, 2 = tf32.  a_mn/b_mn: operand is MN-major in smem.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t fmt, uint32_t a_mn, uint32_t b_mn,
                                                  uint32_t m, uint32_t n) {
  return (1u << 4)            // D format: f32
         | (fmt << 7)         // A format
         | (fmt << 10)        // B format
         | (a_mn << 15)       // A major
         | (b_mn << 16)       // B major
         | ((n >> 3) << 17)   // N / 8
         | ((m >> 4) << 24);  // M / 16
}

// ── CTA pairs (thread-block clusters of 2) for cta_group::2 MMAs ─────────────
// Rank of this CTA in its cluster.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address, in the shared::cluster window, of the variable at shared::cta address
// `addr` of the CTA with cluster rank `rank` (the same offset in its shared memory).
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive (release, cluster scope) on an mbarrier of any CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// Every thread of both CTAs of the pair arrives, then waits for all of them.
// Used twice: after barrier initialisation (before any CTA signals the other's
// barriers) and before the pair frees its tensor memory and exits (so that no CTA
// leaves while the other's MMAs may still read its shared memory).  Both CTAs of a
// cluster are resident together and every path of the kernel reaches both calls.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory (dst) whose completion is counted
// on an mbarrier that may belong to the peer CTA of the pair (bar: shared::cluster
// address).  No multicast: each CTA loads its own tile.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                 int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
// Tensor memory of a CTA pair: one warp of EACH CTA (the same warp index) runs these;
// both receive the same column address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D (M = 256 rows over the pair's TMEM, 128 per CTA) (+)= A (each CTA supplies its
// 128 rows) * B (each CTA supplies half of the N columns); issued by one thread of
// the pair's rank-0 CTA; descriptors address the same offsets in both CTAs.
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at shared::cta offset `bar` in every CTA of `cta_mask`
// when the pair MMAs this thread issued so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// Named barrier among a subset of warps (id 1..15).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate over the participating threads.
__device__ __forceinline__ bool named_bar_red_or(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

}  // namespace ojx
