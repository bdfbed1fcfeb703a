// flash_attn.cuh — fused attention forward for bf16/fp16 on tcgen05 (head dim 64
// or 128).  One CTA per (problem, 128-query tile); the scores never leave the SM.
//
//   warp 0       TMA producers (lane 0: Q once, then K_j; lane 1: V_j; 128 keys
//                per tile) into 2-stage rings (rank-3 maps: d, row, problem).
//                K and V slots are released separately: K_j's as soon as S_j is
//                computed, V_j's after PV_j, so K_{j+2} loads while PV_j runs.
//   warp 1       MMA issuer: S_j = Q K_j^T into one of two TMEM score buffers
//                (S_{j+1} is issued before PV_j so it overlaps the softmax of S_j),
//                then O += P_j V_j into the TMEM output accumulator, with P_j read
//                from TMEM (it overwrites the first half of S_j's buffer).  One
//                thread issues every MMA, in order, so S_{j+2} cannot overwrite
//                P_j before PV_j has read it.
//   warps 2-9    softmax: warp w owns TMEM lane quarter w%4 (one query row per
//                thread) and key half (w-2)/4 of each tile (two warps per scheduler
//                hide each other's latency).  The two threads of a row exchange
//                their tile maxima through shared memory; each keeps its half of
//                the scores in registers, stores its half of P_j as packed 16-bit
//                pairs into TMEM, rescales its half of the row's O in TMEM when the
//                max grows by more than 2^8, and stores its half of the final
//                O / (sum + 1e-6) (the reference's denominator) to HBM
//
// Semantics are flash_attention.cl:8-187's: scores = scale * q.k, causal keeps
// key j <= query i (top-left aligned), keys >= nk are ignored.
#include <cuda_runtime.h>
#include "sm100.cuh"
#include "internal.h"
#include "tmap.h"

namespace ojx {

constexpr int FA_BM = 128;       // query rows per CTA (MMA M)
constexpr int FA_BN = 128;       // keys per tile
constexpr int FA_ST = 2;         // K/V ring stages
constexpr int FA_THREADS = 320;  // producer, MMA, 8 softmax warps
constexpr int FA_SMX = 256;      // softmax threads

template <int D>
struct FaLayout {
  static constexpr int DB = D / 64;                    // 64-wide d blocks (128-byte rows)
  static constexpr int Q_BYTES = FA_BM * D * 2;        // DB sub-tiles of 128 rows x 128 B
  static constexpr int K_BYTES = FA_BN * D * 2;
  static constexpr int V_BYTES = FA_BN * D * 2;        // 2 key blocks x DB d blocks of 64 x 64
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int XCH_BYTES = 6 * FA_BM * 4;     // row maxima (2 buffers x 2 halves), row sums
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = Q_BYTES + FA_ST * STAGE_BYTES + XCH_BYTES + BAR_BYTES + 1024;
  // S0 [0,128), S1 [128,256) (P_j packed into the first 64 columns of S_j's), O [256,256+D)
  static constexpr uint32_t TMEM_COLS = 512;
};

// 2^x on the special-function unit (flush-to-zero: P is rounded to 16 bits, and a
// denormal probability is 0 there anyway).
__device__ __forceinline__ float fa_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct FaParams {
  int M, nk, BH, q_tiles;
  float scale_log2;  // scale * log2(e)
  int causal;
  void* out;         // [BH][M][D]
  uint64_t budget;
};

template <int FMT, int D>
__global__ void __launch_bounds__(FA_THREADS, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const FaParams p) {
  using L = FaLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase;
  const uint32_t sKV = sQ + L::Q_BYTES;
  float* xch = reinterpret_cast<float*>(smem + L::Q_BYTES + FA_ST * L::STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::Q_BYTES + FA_ST * L::STAGE_BYTES + L::XCH_BYTES);
  const uint32_t bar0 = smem_u32(bars);
  // barrier slots
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (1 + FA_ST + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (1 + 2 * FA_ST + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (1 + 3 * FA_ST + s); };
  auto s_full = [&](int b) { return bar0 + 8u * (1 + 4 * FA_ST + b); };
  const uint32_t p_full = bar0 + 8u * (5 + 4 * FA_ST);
  const uint32_t pv_done = bar0 + 8u * (6 + 4 * FA_ST);
  const uint32_t done_bar = bar0 + 8u * (7 + 4 * FA_ST);
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + 8 + 4 * FA_ST);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 9 + 4 * FA_ST);
  static_assert((10 + 4 * FA_ST) * 8 <= L::BAR_BYTES, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heaviest (last, for causal) query tiles first
  const int bh = blockIdx.x % p.BH;
  const int qt = p.q_tiles - 1 - static_cast<int>(blockIdx.x / p.BH);
  const int q0 = qt * FA_BM;
  int kv_tiles = (p.nk + FA_BN - 1) / FA_BN;
  if (p.causal) kv_tiles = min(kv_tiles, (min(q0 + FA_BM, p.M) - 1) / FA_BN + 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < FA_ST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) mbar_init(s_full(b), 1);
    mbar_init(p_full, 8);
    mbar_init(pv_done, 1);
    mbar_init(done_bar, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ── TMA producers: lane 0 loads Q and the K tiles, lane 1 the V tiles ──────
    if (lane < 2 && kv_tiles > 0) {
      const bool is_k = lane == 0;
      uint32_t issued = 0, issued_parity = 0;
      if (is_k) {
        mbar_arrive_expect_tx(q_full, L::Q_BYTES);
#pragma unroll
        for (int db = 0; db < L::DB; ++db)
          if (tma_origin_ok(SITE_FA_LOAD, db * 64, q0, D, p.M, 2) &&
              bounds_check(bh < p.BH, SITE_FA_LOAD, bh, q0, p.BH))
            tma_load_3d(sQ + db * 16384, &tmQ, q_full, db * 64, q0, bh);
      }
      for (int j = 0; j < kv_tiles; ++j) {
        const int st = j % FA_ST;
        const uint32_t ph = static_cast<uint32_t>(j / FA_ST) & 1u;
        const uint32_t sK = sKV + st * L::STAGE_BYTES, sV = sK + L::K_BYTES;
        if (is_k) {
          if (!mbar_wait(k_empty(st), ph ^ 1u, p.budget, s_abort)) break;
          mbar_arrive_expect_tx(k_full(st), L::K_BYTES);
#pragma unroll
          for (int db = 0; db < L::DB; ++db)
            if (tma_origin_ok(SITE_FA_LOAD, db * 64, j * FA_BN, D, p.nk, 2))
              tma_load_3d(sK + db * 16384, &tmK, k_full(st), db * 64, j * FA_BN, bh);
        } else {
          if (!mbar_wait(v_empty(st), ph ^ 1u, p.budget, s_abort)) break;
          mbar_arrive_expect_tx(v_full(st), L::V_BYTES);
          // (the second 64-key box of a ragged last tile may start past the keys)
          const int v_boxes = tma_origin_ok(SITE_FA_LOAD, 0, j * FA_BN, D, p.nk, 2) ? 2 : 0;
#pragma unroll
          for (int kb = 0; kb < v_boxes; ++kb)
#pragma unroll
            for (int db = 0; db < L::DB; ++db)
              tma_load_3d(sV + (kb * L::DB + db) * 8192, &tmV, v_full(st), db * 64,
                          j * FA_BN + kb * 64, bh);
        }
        issued |= 1u << st;
        issued_parity = (issued_parity & ~(1u << st)) | (ph << st);
      }
      // Let every copy this thread issued land before the CTA may exit.
      if (is_k) mbar_wait_drain(q_full, 0, p.budget);
      for (int s = 0; s < FA_ST; ++s)
        if ((issued >> s) & 1u)
          mbar_wait_drain(is_k ? k_full(s) : v_full(s), (issued_parity >> s) & 1u, p.budget);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ── MMA issuer ───────────────────────────────────────────────────────
    if (lane == 0 && kv_tiles > 0) {
      constexpr uint32_t IDESC_S = make_idesc(FMT, 0, 0, FA_BM, FA_BN);
      constexpr uint32_t IDESC_PV = make_idesc(FMT, 0, 1, FA_BM, D);
      bool ok = mbar_wait(q_full, 0, p.budget, s_abort);
      auto issue_s = [&](int j) {
        const int st = j % FA_ST, buf = j & 1;
        // S_j reuses the buffer of P_{j-2}: PV_{j-2} was issued before, by this thread
        if (!mbar_wait(k_full(st), static_cast<uint32_t>(j / FA_ST) & 1u, p.budget, s_abort)) return false;
        tc_fence_after();
        const uint32_t sK = sKV + st * L::STAGE_BYTES;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
          mma_f16(tmem + buf * FA_BN, make_sw128_desc(sQ + off, 16, 1024),
                  make_sw128_desc(sK + off, 16, 1024), IDESC_S, ks > 0 ? 1u : 0u);
        }
        mma_commit(s_full(buf));
        mma_commit(k_empty(st));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < kv_tiles && ok; ++j) {
        if (j + 1 < kv_tiles && !(ok = issue_s(j + 1))) break;
        const int st = j % FA_ST;
        if (!mbar_wait(v_full(st), static_cast<uint32_t>(j / FA_ST) & 1u, p.budget, s_abort)) break;
        if (!mbar_wait(p_full, static_cast<uint32_t>(j) & 1u, p.budget, s_abort)) break;
        tc_fence_after();
        const uint32_t sV = sKV + st * L::STAGE_BYTES + L::K_BYTES;
        const uint32_t p_tmem = tmem + (j & 1) * FA_BN;  // P_j: 16 keys per 8 columns
#pragma unroll
        for (int ks = 0; ks < FA_BN / 16; ++ks) {
          const uint64_t b =
              make_sw128_desc(sV + (ks >> 2) * (L::DB * 8192) + (ks & 3) * 2048, 8192, 1024);
          mma_f16_ts(tmem + 2 * FA_BN, p_tmem + ks * 8, b, IDESC_PV, (j > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(pv_done);
        mma_commit(v_empty(st));
      }
      // Every MMA issued above must complete before TMEM is released.
      mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0, p.budget);
    }
    __syncwarp();
  } else {
    // ── softmax warps: thread = query row q0 + 32*(warp%4) + lane, key half ──
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // keys [64 half, 64 half + 64) of each tile
    const int row = quarter * 32 + lane;
    const int qi = q0 + row;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t o_col = 2 * FA_BN;
    constexpr int HK = FA_BN / 2;  // keys per thread
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    bool failed = false;  // a bounded wait of this thread gave up; agreed at the next barrier
    for (int j = 0; j < kv_tiles; ++j) {
      const int buf = j & 1;
      failed |= !mbar_wait(s_full(buf), static_cast<uint32_t>(j >> 1) & 1u, p.budget, s_abort);
      tc_fence_after();
      const int key0 = j * FA_BN;
      // keys of this row in this thread's half: [key0 + 64 half, key0 + 64 half + n_vis)
      int n_vis = min(FA_BN, p.nk - key0);
      if (p.causal) n_vis = min(n_vis, qi - key0 + 1);
      n_vis -= 64 * half;
      // this thread's half of the score row: 4 loads, one wait
      uint32_t r[HK];
#pragma unroll
      for (int c = 0; c < HK; c += 16)
        tmem_ld16(trow + buf * FA_BN + 64 * half + c, *reinterpret_cast<uint32_t(*)[16]>(&r[c]));
      tmem_wait_ld();
      // Row maximum (log2 domain).  The running maximum is only raised when the
      // tile's exceeds it by more than 8 (a factor 256): terms stay below 2^8, and
      // the output accumulator is rescaled only on those rare steps.  Maxima and
      // sums use 8 independent accumulators (short dependency chains).
      float mx8[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) mx8[t] = -INFINITY;
      if (n_vis >= HK) {
#pragma unroll
        for (int i = 0; i < HK; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(r[i]));
      } else {
#pragma unroll
        for (int i = 0; i < HK; ++i)
          if (i < n_vis) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(r[i]));
      }
      float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // the row's maximum over both halves (double-buffered exchange slot); after
      // this barrier both halves have read their scores, so P may overwrite them.
      // The same barrier makes every softmax warp agree on stopping when any wait
      // gave up (the loop's only other barrier use is the next tile's).
      {
        float* slot = xch + ((j & 1) * 2) * FA_BM;
        slot[half * FA_BM + row] = mx;
        if (named_bar_red_or(1, FA_SMX, failed)) {
          ok = false;
          break;
        }
        mx = fmaxf(mx, slot[(1 - half) * FA_BM + row]);
      }
      mx *= p.scale_log2;  // scale > 0: the maximum of the scaled scores
      const bool raise = mx > m_run + 8.0f;
      const float m_new = raise ? mx : m_run;
      const float m_use = m_new == -INFINITY ? 0.0f : m_new;
      const float alpha = raise ? fa_exp2(m_run - m_use) : 1.0f;  // 0 on the first tile
      // P = 2^(s * scale - m) as 16-bit pairs, and the row sum
      uint32_t pk[HK / 2];
      float sum8[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) sum8[t] = 0.0f;
      const bool full = n_vis >= HK;
#pragma unroll
      for (int i = 0; i < HK; i += 2) {
        float e0 = fa_exp2(fmaf(__uint_as_float(r[i]), p.scale_log2, -m_use));
        float e1 = fa_exp2(fmaf(__uint_as_float(r[i + 1]), p.scale_log2, -m_use));
        if (!full) {
          e0 = i < n_vis ? e0 : 0.0f;
          e1 = i + 1 < n_vis ? e1 : 0.0f;
        }
        sum8[(i >> 1) & 7] += e0 + e1;
        if (FMT == 1) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(e0, e1);
          pk[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
        } else {
          const __half2 h = __floats2half2_rn(e0, e1);
          pk[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
        }
      }
      const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) +
                        ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      l_run = l_run * alpha + sum;
      m_run = m_new;
      // P_j into the first 64 columns of S_j's buffer: this half's 64 keys are
      // 32 packed columns at 32 * half
#pragma unroll
      for (int c = 0; c < HK / 2; c += 16)
        tmem_st16(trow + buf * FA_BN + 32 * half + c, *reinterpret_cast<const uint32_t(*)[16]>(&pk[c]));
      // PV_{j-1} must be done before O is rescaled (and PV_j waits for this tile's
      // arrival below); usually it finished while the exponentials were computed
      bool o_ready = true;
      if (j > 0) {
        o_ready = mbar_wait(pv_done, static_cast<uint32_t>(j - 1) & 1u, p.budget, s_abort);
        failed |= !o_ready;
        tc_fence_after();
      }
      // rescale this half of the rows whose maximum was raised (warp-wide collective access)
      if (j > 0 && __all_sync(0xffffffffu, o_ready) && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
        for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 16) {
          uint32_t o[16];
          tmem_ld16(trow + o_col + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16(trow + o_col + c, o);
        }
      }
      tmem_wait_st();  // P_j (and a rescaled O) written before PV_j may read them
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // final: O / (sum + 1e-6) -> HBM
    bool have_o = ok && kv_tiles > 0;
    if (have_o) {
      const bool w3 =
          mbar_wait(pv_done, static_cast<uint32_t>(kv_tiles - 1) & 1u, p.budget, s_abort);
      have_o = !named_bar_red_or(1, FA_SMX, !w3 || failed);
      if (have_o) tc_fence_after();
    }
    // the row's sum over both halves (its own slots: a partner may still read the
    // last maxima)
    float* lslot = xch + 4 * FA_BM;
    lslot[half * FA_BM + row] = l_run;
    named_bar_sync(1, FA_SMX);
    const float inv = 1.0f / (l_run + lslot[(1 - half) * FA_BM + row] + 1e-6f);
    char* dst = static_cast<char*>(p.out) + (static_cast<int64_t>(bh) * p.M + qi) * D * 2;
    if (have_o || (ok && kv_tiles == 0)) {
#pragma unroll 1
      for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 16) {
        uint32_t r[16];
        if (kv_tiles > 0) {
          tmem_ld16(trow + o_col + c, r);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) r[i] = 0u;
        }
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float a = __uint_as_float(r[i]) * inv, b = __uint_as_float(r[i + 1]) * inv;
          if (FMT == 1) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
            pk[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
          } else {
            const __half2 h = __floats2half2_rn(a, b);
            pk[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
        if (qi < p.M && bounds_check(c + 16 <= D && bh < p.BH, SITE_FA_STORE, qi, c, D)) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 2);
          d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

bool flash_attn_supported(int dtype, int64_t D) {
  return (dtype == OJX_BF16 || dtype == OJX_F16) && (D == 64 || D == 128);
}

int launch_flash_attn(const void* q, const void* k, const void* v, void* out, int dtype, int64_t BH,
                      int64_t M, int64_t N, int64_t nk, int64_t D, float scale, int causal,
                      cudaStream_t s) {
  const CUtensorMapDataType tdt =
      dtype == OJX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  int st;
  if ((st = make_tmap_3d_sw128(&tq, tdt, 2, q, D, M, BH, D * 2, M * D * 2, 64, FA_BM))) return st;
  if ((st = make_tmap_3d_sw128(&tk, tdt, 2, k, D, N, BH, D * 2, N * D * 2, 64, FA_BN))) return st;
  if ((st = make_tmap_3d_sw128(&tv, tdt, 2, v, D, N, BH, D * 2, N * D * 2, 64, 64))) return st;
  FaParams prm{};
  prm.M = static_cast<int>(M);
  prm.nk = static_cast<int>(nk);
  prm.BH = static_cast<int>(BH);
  prm.q_tiles = static_cast<int>((M + FA_BM - 1) / FA_BM);
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.causal = causal;
  prm.out = out;
  prm.budget = g_wait_budget.load();
  const long grid = static_cast<long>(prm.q_tiles) * BH;
  if (grid > 2147483647L) return set_error(OJX_ERR_INVALID, "attention: too many query tiles");
  auto launch = [&](auto kern, int smem) {
    int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
    if (r) return r;
    kern<<<static_cast<unsigned>(grid), FA_THREADS, smem, s>>>(tq, tk, tv, prm);
    g_launches.fetch_add(1);
    return cuda_status(cudaGetLastError(), "flash_attn launch");
  };
  const bool bf = dtype == OJX_BF16;
  if (D == 64)
    return bf ? launch(flash_attn_kernel<1, 64>, FaLayout<64>::SMEM)
              : launch(flash_attn_kernel<0, 64>, FaLayout<64>::SMEM);
  return bf ? launch(flash_attn_kernel<1, 128>, FaLayout<128>::SMEM)
            : launch(flash_attn_kernel<0, 128>, FaLayout<128>::SMEM);
}

}  // namespace ojx
