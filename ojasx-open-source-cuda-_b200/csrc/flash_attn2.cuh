// flash_attn2.cuh — fused attention forward for bf16/fp16 on tcgen05 (head dim 64
// or 128), two query tiles per CTA in ping-pong.  One CTA per (problem, 256
// queries); the scores never leave the SM.
//
//   warp 0       TMA producers (lane 0: both Q tiles once, then K_j; lane 1: V_j;
//                128 keys per tile) into rings of 2 K stages and 1 (D=128) or 2 V
//                stages (rank-3 maps: d, row, problem).
//   warp 1       MMA issuer.  S_t(j+1) = Q_t K_{j+1}^T is issued into S_t's buffer as
//                soon as softmax t has copied S_t(j) into registers (s_free), so it
//                runs under the rest of that softmax; O_t += P_t(j) V_j once softmax
//                t has written P_t(j) (p_full).  One thread issues every MMA, in order.
//   warps 2-5    softmax of query tile 0, warps 6-9 of tile 1: one query row per
//                thread (TMEM lane quarter w%4), the whole 128-key score row in
//                registers, so no exchange between threads.  Each writes its row of
//                P_t(j) to shared memory (K-major, 128-byte swizzle: the PV MMA's A
//                operand), rescales its row of O_t when the running maximum grows by
//                more than 2^8, and finally stores O_t / (sum + 1e-6) (the
//                reference's denominator) to HBM.
//
// Tensor memory (512 columns): S_0 [0,128), S_1 [128,256), O_0 [256, 256+D),
// O_1 [256+D, 256+2D).
// Semantics are flash_attention.cl:8-187's: scores = scale * q.k, causal keeps
// key j <= query i (top-left aligned), keys >= nk are ignored.
#include <cuda_runtime.h>
#include "sm100.cuh"
#include "internal.h"
#include "tmap.h"

namespace ojx {

constexpr int F2_BM = 128;       // query rows per tile (MMA M)
constexpr int F2_QT = 2;         // query tiles per CTA
constexpr int F2_BN = 128;       // keys per tile
constexpr int F2_KST = 2;        // K ring stages
constexpr int F2_THREADS = 320;  // producer, MMA, 2 x 4 softmax warps

template <int D>
struct F2Layout {
  static constexpr int DB = D / 64;                       // 64-wide d blocks (128-byte rows)
  static constexpr int VST = D == 128 ? 1 : 2;            // V ring stages (shared memory is full at D=128)
  static constexpr int QT_BYTES = F2_BM * D * 2;          // one query tile: DB sub-tiles of 128 x 128 B
  static constexpr int P_BYTES = F2_BM * F2_BN * 2;       // one P tile: 2 key blocks of 128 rows x 128 B
  static constexpr int K_BYTES = F2_BN * D * 2;
  static constexpr int V_BYTES = F2_BN * D * 2;           // 2 key blocks x DB d blocks of 64 x 64
  static constexpr int BAR_BYTES = 256;
  static constexpr int OFF_P = F2_QT * QT_BYTES;
  static constexpr int OFF_K = OFF_P + F2_QT * P_BYTES;
  static constexpr int OFF_V = OFF_K + F2_KST * K_BYTES;
  static constexpr int OFF_BAR = OFF_V + VST * V_BYTES;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(2 * F2_BN + 2 * D <= 512, "tensor memory layout");
};

__device__ __forceinline__ float f2_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct F2Params {
  int M, nk, BH, q_tiles;  // q_tiles: 256-query blocks per problem
  float scale_log2;        // scale * log2(e)
  int causal;
  void* out;               // [BH][M][D]
  uint64_t budget;
};

template <int FMT, int D>
__global__ void __launch_bounds__(F2_THREADS, 1)
    flash_attn2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const F2Params p) {
  using L = F2Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase;
  const uint32_t sP = sbase + L::OFF_P;
  const uint32_t sK0 = sbase + L::OFF_K;
  const uint32_t sV0 = sbase + L::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  const uint32_t bar0 = smem_u32(bars);
  constexpr int VST = L::VST;
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (1 + F2_KST + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (1 + 2 * F2_KST + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (1 + 2 * F2_KST + VST + s); };
  constexpr int B1 = 1 + 2 * F2_KST + 2 * VST;  // per-tile barriers from here
  auto s_full = [&](int t) { return bar0 + 8u * (B1 + t); };
  auto s_free = [&](int t) { return bar0 + 8u * (B1 + 2 + t); };
  auto p_full = [&](int t) { return bar0 + 8u * (B1 + 4 + t); };
  auto pv_done = [&](int t) { return bar0 + 8u * (B1 + 6 + t); };
  const uint32_t done_bar = bar0 + 8u * (B1 + 8);
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + B1 + 9);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + B1 + 10);
  static_assert((B1 + 11) * 8 <= L::BAR_BYTES, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heaviest (last, for causal) query blocks first
  const int bh = blockIdx.x % p.BH;
  const int qb = p.q_tiles - 1 - static_cast<int>(blockIdx.x / p.BH);
  const int q0 = qb * (F2_QT * F2_BM);
  int kv_tiles = (p.nk + F2_BN - 1) / F2_BN;
  if (p.causal) kv_tiles = min(kv_tiles, (min(q0 + F2_QT * F2_BM, p.M) - 1) / F2_BN + 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < F2_KST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int t = 0; t < F2_QT; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(s_free(t), 4);
      mbar_init(p_full(t), 4);
      mbar_init(pv_done(t), 1);
    }
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
    // ── TMA producers: lane 0 loads both Q tiles and the K tiles, lane 1 the V tiles
    if (lane < 2 && kv_tiles > 0) {
      const bool is_k = lane == 0;
      uint32_t issued = 0, issued_parity = 0;
      if (is_k) {
        mbar_arrive_expect_tx(q_full, F2_QT * L::QT_BYTES);
        // (tile 0 must start inside Q; tile 1 of a ragged last block may start past M)
        const int q_loads = tma_origin_ok(SITE_FA_LOAD, 0, q0, D, p.M, 2) &&
                                    bounds_check(bh < p.BH, SITE_FA_LOAD, bh, q0, p.BH)
                                ? F2_QT
                                : 0;
#pragma unroll
        for (int t = 0; t < q_loads; ++t)
#pragma unroll
          for (int db = 0; db < L::DB; ++db)
            tma_load_3d(sQ + t * L::QT_BYTES + db * 16384, &tmQ, q_full, db * 64, q0 + t * F2_BM, bh);
      }
      const int nst = is_k ? F2_KST : VST;
      for (int j = 0; j < kv_tiles; ++j) {
        const int st = j % nst;
        const uint32_t ph = static_cast<uint32_t>(j / nst) & 1u;
        if (is_k) {
          const uint32_t sK = sK0 + st * L::K_BYTES;
          if (!mbar_wait(k_empty(st), ph ^ 1u, p.budget, s_abort)) break;
          mbar_arrive_expect_tx(k_full(st), L::K_BYTES);
#pragma unroll
          for (int db = 0; db < L::DB; ++db)
            if (tma_origin_ok(SITE_FA_LOAD, db * 64, j * F2_BN, D, p.nk, 2))
              tma_load_3d(sK + db * 16384, &tmK, k_full(st), db * 64, j * F2_BN, bh);
        } else {
          const uint32_t sV = sV0 + st * L::V_BYTES;
          if (!mbar_wait(v_empty(st), ph ^ 1u, p.budget, s_abort)) break;
          mbar_arrive_expect_tx(v_full(st), L::V_BYTES);
          // (the second 64-key box of a ragged last tile may start past the keys)
          const int v_boxes = tma_origin_ok(SITE_FA_LOAD, 0, j * F2_BN, D, p.nk, 2) ? 2 : 0;
#pragma unroll
          for (int kb = 0; kb < v_boxes; ++kb)
#pragma unroll
            for (int db = 0; db < L::DB; ++db)
              tma_load_3d(sV + (kb * L::DB + db) * 8192, &tmV, v_full(st), db * 64,
                          j * F2_BN + kb * 64, bh);
        }
        issued |= 1u << st;
        issued_parity = (issued_parity & ~(1u << st)) | (ph << st);
      }
      // Let every copy this thread issued land before the CTA may exit.
      if (is_k) mbar_wait_drain(q_full, 0, p.budget);
      for (int s = 0; s < nst; ++s)
        if ((issued >> s) & 1u)
          mbar_wait_drain(is_k ? k_full(s) : v_full(s), (issued_parity >> s) & 1u, p.budget);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ── MMA issuer ───────────────────────────────────────────────────────
    if (lane == 0 && kv_tiles > 0) {
      constexpr uint32_t IDESC_S = make_idesc(FMT, 0, 0, F2_BM, F2_BN);
      constexpr uint32_t IDESC_PV = make_idesc(FMT, 0, 1, F2_BM, D);
      bool ok = mbar_wait(q_full, 0, p.budget, s_abort);
      // S_t(j) = Q_t K_j^T into S_t's buffer (K_j's stage must be full)
      auto issue_s = [&](int t, int j) {
        const uint32_t sK = sK0 + (j % F2_KST) * L::K_BYTES;
        const uint32_t sQt = sQ + t * L::QT_BYTES;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
          mma_f16(tmem + t * F2_BN, make_sw128_desc(sQt + off, 16, 1024),
                  make_sw128_desc(sK + off, 16, 1024), IDESC_S, ks > 0 ? 1u : 0u);
        }
        mma_commit(s_full(t));
      };
      // O_t += P_t(j) V_j (P_t K-major in shared memory)
      auto issue_pv = [&](int t, int j) {
        const uint32_t sV = sV0 + (j % VST) * L::V_BYTES;
        const uint32_t sPt = sP + t * L::P_BYTES;
#pragma unroll
        for (int ks = 0; ks < F2_BN / 16; ++ks) {
          const uint64_t a = make_sw128_desc(sPt + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
          const uint64_t b =
              make_sw128_desc(sV + (ks >> 2) * (L::DB * 8192) + (ks & 3) * 2048, 8192, 1024);
          mma_f16(tmem + 2 * F2_BN + t * D, a, b, IDESC_PV, (j > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(pv_done(t));
      };
      if (ok) ok = mbar_wait(k_full(0), 0, p.budget, s_abort);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        mma_commit(k_empty(0));
      }
      for (int j = 0; j < kv_tiles && ok; ++j) {
        const bool more = j + 1 < kv_tiles;
        if (more && !(ok = mbar_wait(k_full((j + 1) % F2_KST), static_cast<uint32_t>((j + 1) / F2_KST) & 1u,
                                     p.budget, s_abort)))
          break;
#pragma unroll
        for (int t = 0; t < F2_QT; ++t) {
          if (more) {  // S_t(j) is in registers: compute S_t(j+1) under the rest of softmax t
            if (!(ok = mbar_wait(s_free(t), static_cast<uint32_t>(j) & 1u, p.budget, s_abort))) break;
            tc_fence_after();
            issue_s(t, j + 1);
          }
          // V_j (with one V stage, loaded once PV_1(j-1) finished) only gates the PVs
          if (t == 0 && !(ok = mbar_wait(v_full(j % VST), static_cast<uint32_t>(j / VST) & 1u, p.budget, s_abort)))
            break;
          if (!(ok = mbar_wait(p_full(t), static_cast<uint32_t>(j) & 1u, p.budget, s_abort))) break;
          tc_fence_after();
          issue_pv(t, j);
        }
        if (!ok) break;
        if (more) mma_commit(k_empty((j + 1) % F2_KST));
        mma_commit(v_empty(j % VST));
      }
      // Every MMA issued above must complete before TMEM is released.
      mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0, p.budget);
    }
    __syncwarp();
  } else {
    // ── softmax: query tile t = (warp - 2) / 4, one row per thread ──────────────
    const int t = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qi = q0 + t * F2_BM + row;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t s_col = t * F2_BN;
    const uint32_t o_col = 2 * F2_BN + t * D;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < kv_tiles; ++j) {
      const bool got = mbar_wait(s_full(t), static_cast<uint32_t>(j) & 1u, p.budget, s_abort);
      if (__any_sync(0xffffffffu, !got)) {  // the warp's TMEM accesses are collective
        ok = false;
        break;
      }
      tc_fence_after();
      const int key0 = j * F2_BN;
      int n_vis = min(F2_BN, p.nk - key0);
      if (p.causal) n_vis = min(n_vis, qi - key0 + 1);
      uint32_t r[F2_BN];
#pragma unroll
      for (int c = 0; c < F2_BN; c += 16)
        tmem_ld16(trow + s_col + c, *reinterpret_cast<uint32_t(*)[16]>(&r[c]));
      tmem_wait_ld();
      // S_t(j) is in registers: the MMA warp may compute S_t(j+1) into the buffer.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free(t));
      // Row maximum (log2 domain), 8 independent accumulators.  The running
      // maximum is only raised when the tile's exceeds it by more than 8 (a
      // factor 256): terms stay below 2^8, and O is rescaled only on those steps.
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
      const bool full = n_vis >= F2_BN;
      if (full) {
#pragma unroll
        for (int i = 0; i < F2_BN; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(r[i]));
      } else {
#pragma unroll
        for (int i = 0; i < F2_BN; ++i)
          if (i < n_vis) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(r[i]));
      }
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) *
                       p.scale_log2;  // scale > 0: the maximum of the scaled scores
      const bool raise = mx > m_run + 8.0f;
      const float m_new = raise ? mx : m_run;
      const float m_use = m_new == -INFINITY ? 0.0f : m_new;
      const float alpha = raise ? f2_exp2(m_run - m_use) : 1.0f;  // 0 on the first tile
      // PV_t(j-1) must be done: it reads P_t's buffer, and O_t is rescaled below
      // (PV_t(j) waits for this tile's arrival); usually it finished long before.
      bool o_ready = true;
      if (j > 0) {
        o_ready = mbar_wait(pv_done(t), static_cast<uint32_t>(j - 1) & 1u, p.budget, s_abort);
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, !o_ready)) {
        ok = false;
        break;
      }
      // P = 2^(s * scale - m) as 16-bit pairs into P_t's row: keys 8c .. 8c+7 are
      // 16-byte chunk c%8 of key block c/8 (128-byte swizzle, the MMA's K-major A)
      float sum8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum8[i] = 0.0f;
      const uint32_t prow = sP + t * L::P_BYTES + row * 128;
#pragma unroll
      for (int c = 0; c < F2_BN / 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const int kk = 8 * c + i;
          float e0 = f2_exp2(fmaf(__uint_as_float(r[kk]), p.scale_log2, -m_use));
          float e1 = f2_exp2(fmaf(__uint_as_float(r[kk + 1]), p.scale_log2, -m_use));
          if (!full) {
            e0 = kk < n_vis ? e0 : 0.0f;
            e1 = kk + 1 < n_vis ? e1 : 0.0f;
          }
          sum8[(kk >> 1) & 7] += e0 + e1;
          if (FMT == 1) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(e0, e1);
            pk[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
          } else {
            const __half2 h = __floats2half2_rn(e0, e1);
            pk[i / 2] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
        const uint32_t a = prow + (c >> 3) * 16384 + (((c & 7) ^ (row & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(pk[0]), "r"(pk[1]),
                     "r"(pk[2]), "r"(pk[3])
                     : "memory");
      }
      const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) +
                        ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      l_run = l_run * alpha + sum;
      m_run = m_new;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
        for (int c = 0; c < D; c += 16) {
          uint32_t o[16];
          tmem_ld16(trow + o_col + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16(trow + o_col + c, o);
        }
      }
      tmem_wait_st();            // a rescaled O_t written before PV_t(j) adds to it
      fence_proxy_async_smem();  // P_t(j) (generic-proxy stores) -> visible to the MMA
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(t));
    }
    // final: O_t / (sum + 1e-6) -> HBM
    bool have_o = ok && kv_tiles > 0;
    if (have_o) {
      const bool w3 = mbar_wait(pv_done(t), static_cast<uint32_t>(kv_tiles - 1) & 1u, p.budget, s_abort);
      have_o = !__any_sync(0xffffffffu, !w3);
      if (have_o) tc_fence_after();
    }
    const float inv = 1.0f / (l_run + 1e-6f);
    char* dst = static_cast<char*>(p.out) + (static_cast<int64_t>(bh) * p.M + qi) * D * 2;
    if (have_o || (ok && kv_tiles == 0)) {
#pragma unroll 1
      for (int c = 0; c < D; c += 16) {
        uint32_t o[16];
        if (kv_tiles > 0) {
          tmem_ld16(trow + o_col + c, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = 0u;
        }
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float a = __uint_as_float(o[i]) * inv, b = __uint_as_float(o[i + 1]) * inv;
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

int launch_flash_attn2(const void* q, const void* k, const void* v, void* out, int dtype, int64_t BH,
                       int64_t M, int64_t N, int64_t nk, int64_t D, float scale, int causal,
                       cudaStream_t s) {
  const CUtensorMapDataType tdt =
      dtype == OJX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  int st;
  if ((st = make_tmap_3d_sw128(&tq, tdt, 2, q, D, M, BH, D * 2, M * D * 2, 64, F2_BM))) return st;
  if ((st = make_tmap_3d_sw128(&tk, tdt, 2, k, D, N, BH, D * 2, N * D * 2, 64, F2_BN))) return st;
  if ((st = make_tmap_3d_sw128(&tv, tdt, 2, v, D, N, BH, D * 2, N * D * 2, 64, 64))) return st;
  F2Params prm{};
  prm.M = static_cast<int>(M);
  prm.nk = static_cast<int>(nk);
  prm.BH = static_cast<int>(BH);
  prm.q_tiles = static_cast<int>((M + F2_QT * F2_BM - 1) / (F2_QT * F2_BM));
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.causal = causal;
  prm.out = out;
  prm.budget = g_wait_budget.load();
  const long grid = static_cast<long>(prm.q_tiles) * BH;
  if (grid > 2147483647L) return set_error(OJX_ERR_INVALID, "attention: too many query tiles");
  auto launch = [&](auto kern, int smem) {
    int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
    if (r) return r;
    kern<<<static_cast<unsigned>(grid), F2_THREADS, smem, s>>>(tq, tk, tv, prm);
    g_launches.fetch_add(1);
    return cuda_status(cudaGetLastError(), "flash_attn launch");
  };
  const bool bf = dtype == OJX_BF16;
  if (D == 64)
    return bf ? launch(flash_attn2_kernel<1, 64>, F2Layout<64>::SMEM)
              : launch(flash_attn2_kernel<0, 64>, F2Layout<64>::SMEM);
  return bf ? launch(flash_attn2_kernel<1, 128>, F2Layout<128>::SMEM)
            : launch(flash_attn2_kernel<0, 128>, F2Layout<128>::SMEM);
}

}  // namespace ojx
