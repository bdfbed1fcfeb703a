// gemm_skinny.cuh — decode-shaped GEMM (M <= 16 rows of X) that streams W from HBM.
//
// The reference sends M < 32 to matmul_naive_f32 / matmul_bias_f32
// (torchcl/kernels/matmul.cl:346-385 via engine.py:166-179): one work-item per
// output element reading a whole column of B.  Here the GEMM is transposed so
// the weight is the 128-row tcgen05 operand:
//     C^T[n, m] = sum_k W^T[n, k] * X^T[k, m]      (MMA M = 128 columns of C,
//                                                   MMA N = 16 padded rows of X)
// Work is cut into units of (column group g = SK_TPU tiles of 128 columns, one
// 64-deep k block): 32 KB of W and 8 MMAs per unit, so the per-unit
// synchronisation (barrier wait, fence, commit) stays small next to the data.
// The U = groups * k_blocks units are divided evenly ("stream-K") over a
// persistent grid of one CTA per SM, so every SM streams the same number of W
// bytes.  A CTA's units form at most a few segments (consecutive k blocks of one
// group).  A segment that covers its whole group is finished directly; otherwise
// each contributor writes its fp32 partial into a scratch slot and bumps the
// group's arrival counter, and the CTA that arrives last sums the partials in
// contributor order (deterministic) and runs the fused epilogue; no CTA waits on
// another.  Eager launches in which no CTA covers more than one group's k blocks
// use a faster hand-off instead: the group's last contributor, which reaches the
// group at the end of its own stream, polls the others' epoch-tagged partials
// (SkinnyParams::tagged) and waits only for lower-indexed CTAs, which wait on
// nothing.  Both hand-offs add the same partials in the same order.
//
// Scratch per call: partial slots  groups * max_contributors * SK_TPU*16*128 fp32,
// and one 64-bit arrival counter per group holding (launch epoch << 32 | count),
// so stale counts from an earlier (or aborted) launch never need resetting.  The
// last arriver also stores 0 into its counter, so a completed launch leaves the
// counters as it found them: a launch replayed from a CUDA graph (same epoch
// every time) then starts from zero as well.
//
// Back-to-back decode launches (one per layer) overlap through programmatic
// dependent launch.  The kernel is sized for two CTAs per SM (3-stage ring,
// 8-row epilogue staging: ~111 KB of shared memory), and each CTA lets the next
// launch in once it has issued its last W load.  The next grid's CTAs then take
// the second slot on every SM, set up, and (when the host has established that
// the previous launch does not write W) load the W tiles of their first units
// into their ring while this grid drains and runs its split-K tail; only then do
// they pass griddepcontrol.wait.  Every other global access (X, the epilogue
// operand, C, the scratch) comes after that wait, so it sees all of the previous
// kernel's writes.
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <unordered_map>
#include "sm100.cuh"
#include "epilogue.cuh"
#include "internal.h"
#include "tmap.h"

namespace ojx {

constexpr int SK_BN = 128;   // columns of C per tile (MMA M)
constexpr int SK_TPU = 2;    // tiles per unit
constexpr int SK_MN = 16;    // padded rows of X (MMA N)
constexpr int SK_BK = 64;    // k per unit (one 128-byte swizzle row of bf16)
constexpr int SK_STAGES = 3;
constexpr int SK_THREADS = 192;
constexpr int SK_W_BYTES = SK_TPU * SK_BN * 128;
constexpr int SK_X_BYTES = SK_MN * 128;
constexpr int SK_STAGE_BYTES = SK_W_BYTES + SK_X_BYTES;
constexpr int SK_NBUF = 4;  // TMEM accumulator buffers (segments in flight)
constexpr uint32_t SK_TMEM_COLS = SK_NBUF * SK_TPU * SK_MN;
constexpr int SK_SLOT = SK_TPU * SK_MN * SK_BN;  // floats per partial slot
constexpr int SK_EPI_ROWS = 8;  // rows of a finished group staged at a time
constexpr int SK_EPI_BYTES = SK_TPU * SK_EPI_ROWS * SK_BN * 4;  // staging, fp32
constexpr int SK_SMEM = SK_STAGES * SK_STAGE_BYTES + SK_EPI_BYTES + 512 + 1024;
// Two CTAs per SM (228 KB of shared memory, 1 KB reserved per CTA): the next
// launch's CTAs become resident beside this launch's while it drains.
static_assert(2 * (SK_SMEM + 1024) <= 228 * 1024, "two skinny CTAs must fit on one SM");
static_assert(SK_MN == 2 * SK_EPI_ROWS, "the finish stages the rows in two passes");
static_assert(SK_TPU * SK_BN == 256, "the finish maps 32 threads x 8 columns onto one row of a group");
static_assert(SK_STAGE_BYTES % 1024 == 0, "stage alignment");
static_assert(SK_TMEM_COLS >= 32 && (SK_TMEM_COLS & (SK_TMEM_COLS - 1)) == 0, "TMEM alloc size");

struct SkinnyParams {
  int M, N, K;
  int n_groups, KB;
  long long U;  // total units
  int G;        // CTAs
  int maxc;     // partial slots per group
  float* partials;
  unsigned long long* counters;
  unsigned int epoch;
  uint64_t budget;
  int silence_producer;
  int trigger_early;  // let the next launch in after the last W load is issued
  int early_w;        // W of the first SK_STAGES units may be loaded before the dependency wait
  // Tagged hand-off (see the epilogue): each split group is finished by its last
  // contributor, which reads the others' partials from `tagged_parts` (one 64-bit
  // word per value: epoch << 32 | fp32 bits) as soon as they carry this launch's
  // epoch.  Only used when every CTA covers at most KB units, so that a group's
  // last contributor reaches that group at the very end of its own stream.
  int tagged;
  unsigned long long* tagged_parts;
  int silence_contributors;  // test hook: contributors publish nothing (the finishers' polls expire)
};

__device__ __forceinline__ long long unit_begin(int c, const SkinnyParams& p) {
  return static_cast<long long>(c) * p.U / p.G;
}
// CTA whose unit range contains unit u.
__device__ __forceinline__ int cta_of_unit(long long u, const SkinnyParams& p) {
  int c = static_cast<int>((u * p.G) / p.U);
  while (c + 1 < p.G && unit_begin(c + 1, p) <= u) ++c;
  while (c > 0 && unit_begin(c, p) > u) --c;
  return c;
}

// A CTA visits its units [ub, ue) starting with the head of the last group it
// touches, when that head is only part of the group (its other k blocks belong
// to later CTAs), then wraps around to ub.  Its partial for that group is then
// written early, and the one segment this CTA ends its stream with is the tail
// of its first group, which the CTAs before it began early: at the end of the
// stream each CTA has at most one split-K arrival (and one finish) left to do.
__device__ __forceinline__ long long first_unit(long long ub, long long ue, int KB) {
  const long long hs = (ue - 1) / KB * KB;
  return (hs > ub && ue % KB != 0) ? hs : ub;
}

template <int FMT, int W_MN>
__global__ void __launch_bounds__(SK_THREADS, 2)
    skinny_gemm_kernel(const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmX, const EpiParams ep,
                       const SkinnyParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t epi_u32 = smem_u32(smem + SK_STAGES * SK_STAGE_BYTES);  // finished block
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SK_STAGES * SK_STAGE_BYTES + SK_EPI_BYTES);
  constexpr int NB = 2 * SK_STAGES + 2 * SK_NBUF + 2;  // full, empty, tfull, tempty, done, red
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + NB);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + NB + 1);
  volatile int* s_last = reinterpret_cast<volatile int*>(bars + NB + 2);
  static_assert((NB + 3) * 8 <= 512, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (SK_STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * SK_STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * SK_STAGES + SK_NBUF + a); };
  const uint32_t done_bar = bar0 + 8u * (2 * SK_STAGES + 2 * SK_NBUF);
  const uint32_t red_bar = done_bar + 8u;  // partial slots copied in for the last finish

  if (threadIdx.x == 0) {
    for (int s = 0; s < SK_STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < SK_NBUF; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(done_bar, 1);
    mbar_init(red_bar, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), SK_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  const long long ub = unit_begin(blockIdx.x, p);
  const long long ue = unit_begin(blockIdx.x + 1, p);
  const int g_begin = static_cast<int>(ub / p.KB);
  const int kb_begin = static_cast<int>(ub - static_cast<long long>(g_begin) * p.KB);
  const int n_units = static_cast<int>(ue - ub);
  const long long u_first = first_unit(ub, ue, p.KB);
  const int g_first = static_cast<int>(u_first / p.KB);
  const int kb_first = static_cast<int>(u_first - static_cast<long long>(g_first) * p.KB);
  // Step (u, g, kb) by n units in the visiting order (n never crosses ue).
  auto advance = [&](long long& u, int& g, int& kb, int n) {
    u += n;
    if (u == ue) {
      u = ub;
      g = g_begin;
      kb = kb_begin;
    } else {
      kb += n;
      if (kb == p.KB) {
        kb = 0;
        ++g;
      }
    }
  };

  if (warp == 0) {
    // ── TMA producer ────────────────────────────────────────────────────
    if (lane == 0 && !p.silence_producer) {
      auto load_w = [&](uint32_t sW, uint32_t fb, int g, int kb) {
        const int n0 = g * (SK_TPU * SK_BN), k0 = kb * SK_BK;
        // (the unit's first box must start inside W; the others of a ragged last group
        // may start past N and read the zero fill)
        if (W_MN ? !tma_origin_ok(SITE_SK_LOAD_W, n0, k0, p.N, p.K, 2)
                 : !tma_origin_ok(SITE_SK_LOAD_W, k0, n0, p.K, p.N, 2))
          return;
#pragma unroll
        for (int j = 0; j < SK_TPU; ++j) {
          if (W_MN) {
            tma_load_2d(sW + j * (SK_BN * 128), &tmW, fb, n0 + j * SK_BN, k0);
            tma_load_2d(sW + j * (SK_BN * 128) + 64 * 128, &tmW, fb, n0 + j * SK_BN + 64, k0);
          } else {
            tma_load_2d(sW + j * (SK_BN * 128), &tmW, fb, k0, n0 + j * SK_BN);
          }
        }
      };
      // Before the dependency wait, while the previous grid drains: the W tiles
      // of the first n_early units go straight into the (empty) ring when the
      // host has established that the previous launch on this stream does not
      // write W (p.early_w).  X, which that launch usually wrote, is loaded after
      // the wait.
      const int n_early = p.early_w ? min(n_units, SK_STAGES) : 0;
      {
        long long u = u_first;
        int g = g_first, kb = kb_first;
        for (int i = 0; i < n_early; ++i) {
          mbar_arrive_expect_tx(full_bar(i), SK_STAGE_BYTES);
          load_w(sbase + i * SK_STAGE_BYTES, full_bar(i), g, kb);
          advance(u, g, kb, 1);
        }
      }
      grid_dep_wait();
      int stage = 0, g = g_first, kb = kb_first;
      long long u = u_first;
      uint32_t phase = 0, issued = 0, issued_parity = 0;
      for (int i = 0; i < n_early; ++i) {  // X of the units whose W is already on its way
        if (tma_origin_ok(SITE_SK_LOAD_X, kb * SK_BK, 0, p.K, p.M, 2))
          tma_load_2d(sbase + i * SK_STAGE_BYTES + SK_W_BYTES, &tmX, full_bar(i), kb * SK_BK, 0);
        issued |= 1u << i;
        advance(u, g, kb, 1);
      }
      stage = n_early % SK_STAGES;
      phase = n_early == SK_STAGES ? 1u : 0u;
      for (int i = n_early; i < n_units; ++i) {
        if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.budget, s_abort)) break;
        const uint32_t fb = full_bar(stage);
        mbar_arrive_expect_tx(fb, SK_STAGE_BYTES);
        const uint32_t sW = sbase + stage * SK_STAGE_BYTES;
        load_w(sW, fb, g, kb);
        if (tma_origin_ok(SITE_SK_LOAD_X, kb * SK_BK, 0, p.K, p.M, 2))
          tma_load_2d(sW + SK_W_BYTES, &tmX, fb, kb * SK_BK, 0);
        issued |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == SK_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
        advance(u, g, kb, 1);
      }
      // Every W load of this CTA is issued: the next launch may begin.  Its CTAs
      // take the second slot on each SM and start on their first units while this
      // grid drains its ring and runs its split-K tail.  (The first execution in a
      // CTA counts; a CTA that exits without it counts too.)
      if (p.trigger_early) grid_dep_launch_dependents();
      for (int s = 0; s < SK_STAGES; ++s)
        if ((issued >> s) & 1u) mbar_wait_drain(full_bar(s), (issued_parity >> s) & 1u, p.budget);
    }
  } else if (warp == 1) {
    // ── MMA issuer ──────────────────────────────────────────────────────
    if (lane == 0) {
      grid_dep_wait();  // the bounded waits below start once the inputs are final
      constexpr uint32_t IDESC = make_idesc(FMT, W_MN, 0, SK_BN, SK_MN);
      int stage = 0, acc = 0, g = g_first, kb = kb_first;
      long long u = u_first;
      uint32_t phase = 0, acc_phase = 0;
      bool seg_start = true;
      for (int i = 0; i < n_units; ++i) {
        const bool seg_end = (i + 1 == n_units) || (kb + 1 == p.KB) || (u + 1 == ue);
        if (seg_start) {
          if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.budget, s_abort)) break;
          tc_fence_after();
        }
        if (!mbar_wait(full_bar(stage), phase, p.budget, s_abort)) break;
        tc_fence_after();
        const uint32_t sW = sbase + stage * SK_STAGE_BYTES;
        const uint64_t bd0 = make_sw128_desc(sW + SK_W_BYTES, 16, 1024);
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * SK_TPU * SK_MN);
#pragma unroll
        for (int j = 0; j < SK_TPU; ++j) {
          const uint32_t sWj = sW + j * (SK_BN * 128);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t ad = W_MN ? make_sw128_desc(sWj + ks * 2048, 64 * 128, 1024)
                                     : make_sw128_desc(sWj + ks * 32, 16, 1024);
            mma_f16(d + j * SK_MN, ad, bd0 + static_cast<uint64_t>((ks * 32) >> 4), IDESC,
                    (seg_start && ks == 0) ? 0u : 1u);
          }
        }
        mma_commit(empty_bar(stage));
        if (++stage == SK_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
        seg_start = false;
        if (seg_end) {
          mma_commit(tfull_bar(acc));
          seg_start = true;
          if (++acc == SK_NBUF) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
        advance(u, g, kb, 1);
      }
      mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0, p.budget);
    }
    __syncwarp();
  } else {
    // ── epilogue: 128 threads, thread <-> one column of each tile of the group
    const int q = warp & 3;
    const int etid = threadIdx.x - 64;  // 0..127
    grid_dep_wait();  // the operand, C and the scratch may belong to the previous kernel
    int acc = 0;
    uint32_t acc_phase = 0;
    int g = g_first, kb = kb_first, left = n_units;
    long long u = u_first;
    // Pass 0 runs the finishing code once on zeros with its stores disabled, while
    // the accumulators are still far from ready: the tail's first real finish then
    // finds that code in the instruction caches instead of fetching it from memory
    // behind the last contributor's reduction.  `warm` goes through an empty asm so
    // the compiler cannot specialise (and duplicate) the loop body for pass 0.
    int warm = 1;
    while (true) {
      asm volatile("" : "+r"(warm));
      if (!warm && left <= 0) break;
      float v[SK_TPU][SK_MN];
      bool finish = true;
      int seg_units = 0;
      // In the finish below, thread etid owns the 8 columns fc .. fc+7 of the
      // group (fc = 8 * (etid % 32)) in rows etid / 32, + 4, + 8, + 12.  Their
      // row operand (bias) is loaded here, before the accumulator is ready, so
      // its latency is off the tail.
      const int fc = 8 * (etid & 31);
      const int fn = g * (SK_TPU * SK_BN) + fc;
      const int fvalid = min(8, p.N - fn);
      float row_op[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) row_op[k] = 0.0f;
      if (ep.operand_kind == OJX_OPERAND_ROW && fvalid > 0)
        load8(ep.operand, ep.dtype_operand, fn, fvalid, row_op);
      if (warm) {
#pragma unroll
        for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
          for (int m = 0; m < SK_MN; ++m) v[j][m] = 0.0f;
      } else {
        seg_units = static_cast<int>(min(static_cast<long long>(min(left, p.KB - kb)), ue - u));
        const bool whole = kb == 0 && seg_units == p.KB;
        left -= seg_units;
        // The group's contributors (64-bit divisions) are worked out while the
        // accumulator is still being computed.
        int c_first = blockIdx.x, ncontrib = 1;
        if (!whole) {
          c_first = cta_of_unit(static_cast<long long>(g) * p.KB, p);
          const int c_last = cta_of_unit(min(static_cast<long long>(g + 1) * p.KB, p.U) - 1, p);
          ncontrib = c_last - c_first + 1;
        }
        const int jc = blockIdx.x - c_first;
        // Tagged hand-off: the group's last contributor (highest CTA index) finishes it.
        const bool tag_finisher = p.tagged && !whole && jc == ncontrib - 1;
        // With more than 4 rows, the last finish of the CTA (its ring is idle by
        // then: every MMA has completed) bulk-copies the other contributors' slots
        // into the ring, one round trip instead of one per 4 rows; with up to 4
        // rows, loads into registers are already a single round trip and faster.
        const bool staged = left <= 0 && p.M > 4 && ncontrib * p.M * 1024 <= SK_STAGES * SK_STAGE_BYTES;
        // The four epilogue warps meet at named barriers below, so they must agree
        // on whether to go on: any warp that failed its wait stops all four.
        const bool waited = mbar_wait(tfull_bar(acc), acc_phase, p.budget, s_abort);
        if (named_bar_red_or(1, 128, !waited)) break;
        tc_fence_after();
        uint32_t r[SK_TPU][16];
        const uint32_t tq = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(acc * SK_TPU * SK_MN);
#pragma unroll
        for (int j = 0; j < SK_TPU; ++j) tmem_ld16(tq + j * SK_MN, r[j]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar(acc));
        if (++acc == SK_NBUF) {
          acc = 0;
          acc_phase ^= 1u;
        }
#pragma unroll
        for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
          for (int m = 0; m < SK_MN; ++m) v[j][m] = __uint_as_float(r[j][m]);
        if (!whole && p.tagged && !tag_finisher) {
          // Tagged hand-off, contributor side: publish each value beside this
          // launch's epoch in one 64-bit word and move on (no barrier, fence or
          // counter: every word validates itself, and this CTA finishes nothing).
          unsigned long long* slot = p.tagged_parts +
                                     (static_cast<long long>(g) * p.maxc + jc) * SK_SLOT + q * 32 + lane;
          const unsigned long long tag = static_cast<unsigned long long>(p.epoch) << 32;
#pragma unroll
          for (int j = 0; j < SK_TPU && !p.silence_contributors; ++j)
#pragma unroll
            for (int m = 0; m < SK_MN; ++m)
              if (m < p.M) st_relaxed_gpu_u64(slot + (j * SK_MN + m) * SK_BN, tag | __float_as_uint(v[j][m]));
          finish = false;
        } else if (tag_finisher) {
          // Tagged hand-off, finisher side: this CTA reached the group at the end of
          // its stream; the other contributors (lower CTA indices, none of which
          // waits on anything) publish their words at about the same time or
          // earlier.  Poll them until every word carries this launch's epoch
          // (bounded), and sum in contributor order with this CTA's own partial
          // last, which is its place in that order: the same sums as the counter
          // hand-off below.
          const unsigned long long* tb =
              p.tagged_parts + static_cast<long long>(g) * p.maxc * SK_SLOT + q * 32 + lane;
          const unsigned int want = p.epoch;
          const unsigned long long valid = static_cast<unsigned long long>(want) << 32;
          const long long t0 = clock64();
          bool ok = true;
#pragma unroll
          for (int mc = 0; mc < SK_MN / 4; ++mc) {
            if (4 * mc >= p.M || !ok) break;
            float sum[SK_TPU][4];
#pragma unroll
            for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
              for (int mm = 0; mm < 4; ++mm) sum[j][mm] = 0.0f;
            for (int jj0 = 0; jj0 < jc && ok; jj0 += 2) {
              unsigned long long t[2][SK_TPU][4];
#pragma unroll
              for (int bb = 0; bb < 2; ++bb)
#pragma unroll
                for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
                  for (int mm = 0; mm < 4; ++mm)
                    t[bb][j][mm] = (jj0 + bb < jc && 4 * mc + mm < p.M)
                                       ? ld_relaxed_gpu_u64(tb + static_cast<long long>(jj0 + bb) * SK_SLOT +
                                                            (j * SK_MN + 4 * mc + mm) * SK_BN)
                                       : valid;
              while (true) {
                bool all = true;
#pragma unroll
                for (int bb = 0; bb < 2; ++bb)
#pragma unroll
                  for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
                    for (int mm = 0; mm < 4; ++mm) all &= static_cast<unsigned int>(t[bb][j][mm] >> 32) == want;
                if (all) break;
                if (*s_abort) {
                  ok = false;
                  break;
                }
                if (static_cast<uint64_t>(clock64() - t0) > p.budget) {
                  *s_abort = 1;
                  atomicOr(&g_dev_error, OJX_DEVERR_TIMEOUT);
                  ok = false;
                  break;
                }
#pragma unroll
                for (int bb = 0; bb < 2; ++bb)
#pragma unroll
                  for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
                    for (int mm = 0; mm < 4; ++mm)
                      if (static_cast<unsigned int>(t[bb][j][mm] >> 32) != want)
                        t[bb][j][mm] = ld_relaxed_gpu_u64(tb + static_cast<long long>(jj0 + bb) * SK_SLOT +
                                                          (j * SK_MN + 4 * mc + mm) * SK_BN);
              }
#pragma unroll
              for (int bb = 0; bb < 2; ++bb)
                if (jj0 + bb < jc)
#pragma unroll
                  for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
                    for (int mm = 0; mm < 4; ++mm)
                      sum[j][mm] += __uint_as_float(static_cast<unsigned int>(t[bb][j][mm]));
            }
#pragma unroll
            for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
              for (int mm = 0; mm < 4; ++mm) v[j][4 * mc + mm] = sum[j][mm] + v[j][4 * mc + mm];
          }
          // The four epilogue warps meet at named barriers below: any thread that
          // gave up stops all four.
          if (named_bar_red_or(1, 128, !ok)) break;
        } else if (!whole) {
          float* slot = p.partials + (static_cast<long long>(g) * p.maxc + jc) * SK_SLOT +
                        q * 32 + lane;
#pragma unroll
          for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
            for (int m = 0; m < SK_MN; ++m)
              if (m < p.M) slot[(j * SK_MN + m) * SK_BN] = v[j][m];
          named_bar_sync(1, 128);
          if (etid == 0) {
            fence_acq_rel_gpu();  // with the barrier above: releases every thread's slot
            unsigned long long* ctr = p.counters + g;
            // First guess: this CTA is the last to arrive (the case on the tail's
            // critical path), so the last arriver needs a single atomic.
            unsigned long long old =
                (static_cast<unsigned long long>(p.epoch) << 32) | static_cast<unsigned int>(ncontrib - 1);
            unsigned int count;
            while (true) {  // ends as soon as the CAS succeeds
              const unsigned int e = static_cast<unsigned int>(old >> 32);
              count = (e == p.epoch) ? static_cast<unsigned int>(old & 0xffffffffu) + 1u : 1u;
              const unsigned long long nv = (static_cast<unsigned long long>(p.epoch) << 32) | count;
              const unsigned long long seen = atomicCAS(ctr, old, nv);
              if (seen == old) break;
              old = seen;
            }
            *s_last = (count == static_cast<unsigned int>(ncontrib)) ? 1 : 0;
            if (*s_last) {
              fence_acq_rel_gpu();  // acquire: the other slots are read after this
              *ctr = 0ull;          // every contributor of this group has arrived
              if (staged) {
                fence_proxy_async_all();  // the slots are read through the async proxy
                mbar_arrive_expect_tx(red_bar, static_cast<uint32_t>((ncontrib - 1) * SK_TPU * p.M * 512));
                const float* gb = p.partials + static_cast<long long>(g) * p.maxc * SK_SLOT;
                for (int jj = 0; jj < ncontrib; ++jj) {
                  if (jj == jc || !bounds_check(jj < p.maxc, SITE_SK_SLOT, g, jj, p.maxc)) continue;
#pragma unroll
                  for (int j = 0; j < SK_TPU; ++j)
                    bulk_load_g2s(sbase + static_cast<uint32_t>(((jj * SK_TPU + j) * p.M) * 512),
                                  gb + static_cast<long long>(jj) * SK_SLOT + j * SK_MN * SK_BN,
                                  static_cast<uint32_t>(p.M * 512), red_bar);
                }
              }
            }
          }
          named_bar_sync(1, 128);
          finish = *s_last != 0;
          if (finish && staged) {
            // Part (jj, j) = rows 0..M-1 of tile j of contributor jj's slot lands at
            // (jj * 2 + j) * M * 512 in the ring (bulk copies issued above by the
            // thread that took the last arrival); this thread's own values go to
            // their place too, then it sums its column over the contributors in
            // contributor order (the same order, and so the same result, as below).
            const uint32_t col4 = 4u * static_cast<uint32_t>(q * 32 + lane);
#pragma unroll
            for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
              for (int m = 0; m < SK_MN; ++m)
                if (m < p.M)
                  st_shared_f32(sbase + static_cast<uint32_t>(((jc * SK_TPU + j) * p.M + m) * 512) + col4,
                                v[j][m]);
            const bool ok = mbar_wait(red_bar, 0, p.budget, s_abort);
            if (named_bar_red_or(1, 128, !ok)) {
              if (etid == 0) mbar_wait_drain(red_bar, 0, p.budget);  // copies still in flight
              break;
            }
#pragma unroll
            for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
              for (int m = 0; m < SK_MN; ++m) v[j][m] = 0.0f;
            for (int jj = 0; jj < ncontrib; ++jj)
#pragma unroll
              for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
                for (int m = 0; m < SK_MN; ++m)
                  if (m < p.M)
                    v[j][m] += ld_shared_f32(sbase + static_cast<uint32_t>(((jj * SK_TPU + j) * p.M + m) * 512) + col4);
          } else if (finish) {
            // Sum the partials in contributor order (this CTA's own from its
            // registers, the same values its slot holds), four rows and four
            // contributors at a time: every load of a batch is issued before its
            // first add, so M <= 4 with up to four contributors costs one L2
            // round trip.
            const float* base = p.partials + static_cast<long long>(g) * p.maxc * SK_SLOT + q * 32 + lane;
#pragma unroll
            for (int mc = 0; mc < SK_MN / 4; ++mc) {
              if (4 * mc >= p.M) break;
              float sum[SK_TPU][4];
#pragma unroll
              for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
                for (int mm = 0; mm < 4; ++mm) sum[j][mm] = 0.0f;
              for (int jj0 = 0; jj0 < ncontrib; jj0 += 4) {
                float t[4][SK_TPU][4];
#pragma unroll
                for (int bb = 0; bb < 4; ++bb) {
                  const int jj = jj0 + bb;
                  const float* sl = base + static_cast<long long>(jj) * SK_SLOT;
#pragma unroll
                  for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
                    for (int mm = 0; mm < 4; ++mm) {
                      const int m = 4 * mc + mm;
                      t[bb][j][mm] = (jj < ncontrib && jj != jc && m < p.M)
                                         ? __ldcg(sl + (j * SK_MN + m) * SK_BN)
                                         : v[j][m];
                    }
                }
#pragma unroll
                for (int bb = 0; bb < 4; ++bb)
                  if (jj0 + bb < ncontrib)
#pragma unroll
                    for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
                      for (int mm = 0; mm < 4; ++mm) sum[j][mm] += t[bb][j][mm];
              }
#pragma unroll
              for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
                for (int mm = 0; mm < 4; ++mm) v[j][4 * mc + mm] = sum[j][mm];
            }
          }
          named_bar_sync(1, 128);  // s_last may be rewritten by the next segment
        }
      }
      if (finish) {
        // Stage SK_EPI_ROWS rows of the finished M x 256 block at a time in shared
        // memory, then each thread runs the 8-wide epilogue on its 8 columns of
        // every fourth staged row and writes them with one 16-byte store per
        // destination (a warp covers a whole 256-column row: 512 contiguous
        // bytes).  The second pass (rows 8..15) selects its registers with
        // compile-time indices, so v stays in registers.
#pragma unroll 1
        for (int r0 = 0; r0 < p.M; r0 += SK_EPI_ROWS) {
#pragma unroll
          for (int j = 0; j < SK_TPU; ++j)
#pragma unroll
            for (int mm = 0; mm < SK_EPI_ROWS; ++mm)
              if (r0 + mm < p.M)
                st_shared_f32(epi_u32 + 4u * ((j * SK_EPI_ROWS + mm) * SK_BN + q * 32 + lane),
                              r0 ? v[j][SK_EPI_ROWS + mm] : v[j][mm]);
          named_bar_sync(1, 128);
          if (fvalid > 0) {
            const int r1 = min(p.M, r0 + SK_EPI_ROWS);
#pragma unroll 1
            for (int m = r0 + (etid >> 5); m < r1; m += 4) {
              float y[8], x[8];
              const uint32_t sa =
                  epi_u32 + 4u * (((fc >> 7) * SK_EPI_ROWS + (m - r0)) * SK_BN + (fc & 127));
#pragma unroll
              for (int k = 0; k < 8; ++k) y[k] = ld_shared_f32(sa + 4u * k);
              if (ep.operand_kind == OJX_OPERAND_FULL)
                load8(ep.operand, ep.dtype_operand, static_cast<int64_t>(m) * ep.ld_operand + fn,
                      fvalid, x);
              else
#pragma unroll
                for (int k = 0; k < 8; ++k) x[k] = row_op[k];
              if (ep.operand_kind != OJX_OPERAND_NONE)
                binary_n<8>(ep.binary_op, ep.operand_is_lhs != 0, y, x);
              for (int i = 0; i < ep.n_unary; ++i) unary_n_half<8>(unary_at(ep.unary_packed, i), y);
              if (!warm && epi_store_ok(ep, SITE_SK_STORE, m, fn, fvalid)) {
#pragma unroll
                for (int di = 0; di < OJX_MAX_PEERS; ++di) {
                  if (di >= ep.n_dst) break;
                  store8(ep.dst[di], ep.dtype_c,
                         static_cast<int64_t>(m) * ep.ldc + ep.col_offset + fn, fvalid, y);
                }
              }
            }
          }
          named_bar_sync(1, 128);  // the staging block is rewritten by the next pass
        }
      }
      if (warm) {
        warm = 0;
        continue;
      }
      advance(u, g, kb, seg_units);
    }
    if (ep.n_dst > 1) __threadfence_system();  // peer stores visible before completion
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, SK_TMEM_COLS);
  }
}

bool skinny_supported(const ojx_gemm_desc& d) {
  if (d.dtype_a != d.dtype_b || (d.dtype_a != OJX_BF16 && d.dtype_a != OJX_F16)) return false;
  if (d.M < 1 || d.M > SK_MN || d.K <= 0 || d.trans_a) return false;
  if (d.N > INT32_MAX || d.K > INT32_MAX) return false;
  if (reinterpret_cast<uintptr_t>(d.a) % 16 || reinterpret_cast<uintptr_t>(d.b) % 16) return false;
  if ((d.lda * 2) % 16 || (d.ldb * 2) % 16) return false;
  return true;
}

static std::atomic<unsigned int> g_skinny_epoch{1};


// Host-side partition bookkeeping; mirrors unit_begin / cta_of_unit.
static int skinny_max_contrib(int n_groups, int KB, long long U, int G) {
  auto ub = [&](long long c) { return c * U / G; };
  auto cta_of = [&](long long u) {
    long long c = (u * G) / U;
    while (c + 1 < G && ub(c + 1) <= u) ++c;
    while (c > 0 && ub(c) > u) --c;
    return c;
  };
  int mx = 1;
  for (int g = 0; g < n_groups; ++g) {
    const long long a = cta_of(static_cast<long long>(g) * KB);
    const long long b = cta_of(std::min<long long>(static_cast<long long>(g + 1) * KB, U) - 1);
    mx = std::max<int>(mx, static_cast<int>(b - a + 1));
  }
  return mx;
}

// CTAs of a skinny launch.  The group whose split-K contributors finish last sets the
// tail: its last arriver waits for, and reads, every other contributor's partial
// slot.  Among grids within 8 % of the SM count, take the largest one whose busiest
// group has the fewest contributors.  Measured at cfg4's shape (56 groups of 64
// k-blocks): 140 CTAs give every group 3 contributors and 23.8 / 24.1 / 27.5 us per
// launch at M = 1 / 4 / 16, while every grid of 132-148 CTAs with 4-contributor
// groups took 24.7-25.8 / 25.2-25.8 / 28.6-29.9 us; 112 CTAs (2 per group) lost the
// gain again in streaming bandwidth.  Cached per (groups, k blocks, SMs).
static int skinny_grid(int n_groups, int KB, long long U, int sm_count) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, int>* cache = new std::map<std::tuple<int, int, int>, int>();
  const long long gmax = std::min<long long>(U, sm_count);
  if (gmax <= 1) return static_cast<int>(std::max<long long>(gmax, 1));
  const auto key = std::make_tuple(n_groups, KB, sm_count);
  std::lock_guard<std::mutex> g(mu);
  auto it = cache->find(key);
  if (it != cache->end()) return it->second;
  const int gmin = static_cast<int>(std::max<long long>(1, (gmax * 92 + 99) / 100));
  int best = static_cast<int>(gmax), best_c = skinny_max_contrib(n_groups, KB, U, best);
  for (int G = best - 1; G >= gmin; --G) {
    const int c = skinny_max_contrib(n_groups, KB, U, G);
    if (c < best_c) {
      best = G;
      best_c = c;
    }
  }
  (*cache)[key] = best;
  return best;
}

// Byte ranges written by the last eager skinny launch on each stream.  The next
// eager launch on that stream may start before it completes (programmatic
// dependent launch); it loads W ahead of its dependency wait only when W lies
// outside these ranges.  (A kernel of any other kind in between completes before
// the next launch starts, so only the last skinny launch can still be writing.)
struct SkinnyOut {
  int n = 0;
  uintptr_t lo[OJX_MAX_PEERS], hi[OJX_MAX_PEERS];
};
static std::mutex g_skinny_out_mu;
static std::unordered_map<cudaStream_t, SkinnyOut>* g_skinny_out =
    new std::unordered_map<cudaStream_t, SkinnyOut>();

int launch_skinny_gemm(const ojx_gemm_desc& d, cudaStream_t s, const Dests* dests) {
  SkinnyParams p{};
  p.M = static_cast<int>(d.M);
  p.N = static_cast<int>(d.N);
  p.K = static_cast<int>(d.K);
  p.n_groups = (p.N + SK_TPU * SK_BN - 1) / (SK_TPU * SK_BN);
  p.KB = (p.K + SK_BK - 1) / SK_BK;
  p.U = static_cast<long long>(p.n_groups) * p.KB;
  const DeviceProps& dp = current_props();
  p.G = skinny_grid(p.n_groups, p.KB, p.U, dp.sm_count);
  p.maxc = skinny_max_contrib(p.n_groups, p.KB, p.U, p.G);
  // Capture status first: the tagged hand-off needs a fresh epoch per execution,
  // which a replayed graph (fixed kernel parameters) does not give.
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (s && cudaStreamIsCapturing(s, &cs) != cudaSuccess) cs = cudaStreamCaptureStatusActive;
  const bool eager = cs == cudaStreamCaptureStatusNone;
  p.tagged = eager && !(d.flags & OJX_GEMM_FLAG_SKINNY_COUNTER) && (p.U + p.G - 1) / p.G <= p.KB ? 1 : 0;
  if (p.tagged) {
    p.silence_contributors = g_silence_contributors_once.exchange(0);
    // Its own zero-initialised slot: the words there only ever carry the epochs of
    // earlier skinny launches (or 0), never this launch's.
    p.tagged_parts = static_cast<unsigned long long*>(
        stream_workspace(s, static_cast<size_t>(p.n_groups) * p.maxc * SK_SLOT * 8, 6, /*zero=*/true));
    if (!p.tagged_parts) return workspace_error();
  } else {
    const size_t part_bytes = static_cast<size_t>(p.n_groups) * p.maxc * SK_SLOT * 4;
    p.partials = static_cast<float*>(stream_workspace(s, part_bytes, 1, false));
    if (!p.partials) return workspace_error();
    p.counters = static_cast<unsigned long long*>(
        stream_workspace(s, static_cast<size_t>(p.n_groups) * 8, 2, /*zero=*/true));
    if (!p.counters) return workspace_error();
  }
  p.epoch = g_skinny_epoch.fetch_add(1);
  if (p.epoch == 0) p.epoch = g_skinny_epoch.fetch_add(1);
  p.budget = g_wait_budget.load();
  p.silence_producer = g_silence_producer_once.exchange(0);

  const CUtensorMapDataType tdt =
      d.dtype_a == OJX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tw, tx;
  int st;
  const bool w_mn = !d.trans_b;  // W stored [K,N] row-major: n contiguous
  if (w_mn)
    st = make_tmap_2d_sw128(&tw, tdt, 2, d.b, p.N, p.K, d.ldb * 2, 64, 64);
  else
    st = make_tmap_2d_sw128(&tw, tdt, 2, d.b, p.K, p.N, d.ldb * 2, 64, SK_BN);
  if (st) return st;
  if ((st = make_tmap_2d_sw128(&tx, tdt, 2, d.a, p.K, p.M, d.lda * 2, 64, SK_MN))) return st;
  const EpiParams ep = make_epi(d, dests);
  const bool bf = d.dtype_a == OJX_BF16;
  // Programmatic stream serialization on eager launches (captured launches keep
  // plain stream order and never let the next kernel in early): the grid may
  // start while the previous kernel on the stream finishes, and holds every
  // dependent access until griddepcontrol.wait.
  p.trigger_early = eager ? 1 : 0;
  {
    const uintptr_t w_lo = reinterpret_cast<uintptr_t>(d.b);
    const uintptr_t w_hi =
        w_lo + 2u * static_cast<uintptr_t>(w_mn ? (d.K - 1) * d.ldb + d.N : (d.N - 1) * d.ldb + d.K);
    const int esz_c = d.dtype_c == OJX_F32 ? 4 : 2;
    const uintptr_t c_len =
        static_cast<uintptr_t>(esz_c) * static_cast<uintptr_t>((d.M - 1) * ep.ldc + ep.col_offset + d.N);
    std::lock_guard<std::mutex> lk(g_skinny_out_mu);
    SkinnyOut& last = (*g_skinny_out)[s];
    bool overlap = false;
    for (int i = 0; i < last.n; ++i) overlap |= w_lo < last.hi[i] && last.lo[i] < w_hi;
    p.early_w = eager && !overlap ? 1 : 0;
    if (eager) {
      last.n = ep.n_dst;
      for (int i = 0; i < ep.n_dst; ++i) {
        last.lo[i] = reinterpret_cast<uintptr_t>(ep.dst[i]);
        last.hi[i] = last.lo[i] + c_len;
      }
    }
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = cs == cudaStreamCaptureStatusNone ? 1 : 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.G);
  cfg.blockDim = dim3(SK_THREADS);
  cfg.dynamicSmemBytes = SK_SMEM;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto launch = [&](auto kern) {
    int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), SK_SMEM);
    if (r) return r;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, ep, p);
    g_launches.fetch_add(1);
    if (e != cudaSuccess) return cuda_status(e, "skinny_gemm launch");
    return cuda_status(cudaGetLastError(), "skinny_gemm launch");
  };
  if (bf) return w_mn ? launch(skinny_gemm_kernel<1, 1>) : launch(skinny_gemm_kernel<1, 0>);
  return w_mn ? launch(skinny_gemm_kernel<0, 1>) : launch(skinny_gemm_kernel<0, 0>);
}

}  // namespace ojx
