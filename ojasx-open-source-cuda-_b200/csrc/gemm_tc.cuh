// gemm_tc.cuh — persistent, warp-specialised tcgen05 GEMM with the fused epilogue.
//
// Replaces the reference's matmul_reg_tiled_f32 / matmul_reg_tiled_bias_f32 /
// linear_forward_tiled_f32 / matmul_tiled_fp16 (torchcl/kernels/matmul.cl:19-224,
// 297-343, 422-463) and the JIT's second elementwise launch
// (torchcl/jit/compiler.py:99-133): C = epilogue(A·B) in one launch, one store.
//
// CTA = 320 threads, one CTA per SM, grid = min(#tiles, #SMs), tiles walked with a
// stride of gridDim.x in a grouped raster (16 M-blocks per N sweep) for L2 reuse.
//   warp 0      TMA producer: STAGES-deep ring of 128B-swizzled A/B tiles
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue: TMEM -> registers -> bias/binary/unary chain -> store;
//               warp w reads TMEM lane quarter w%4, half (w-2)/4 of the columns
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns), so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// KIND 0: bf16/fp16 operands, tcgen05 kind::f16, either operand K- or MN-major
//         (transposes are expressed in the TMA/UMMA descriptors, never copied).
// KIND 1: fp32 via 3xTF32: A = Ah + Al, B = Bh + Bl (tf32 parts produced by
//         split_tf32_kernel), acc += Al·Bh + Ah·Bl + Ah·Bh per k-step, kind::tf32.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <algorithm>
#include <map>
#include <mutex>
#include "sm100.cuh"
#include "epilogue.cuh"
#include "internal.h"
#include "tmap.h"

namespace ojx {

constexpr int TC_BM = 128;
constexpr int TC_THREADS = 320;  // 2 control warps + 8 epilogue warps
constexpr int TC_EPI_WARPS = 8;
// 3xTF32 accumulates each run of TC_TF32_CHUNK_KB k-blocks (256 k) into a fresh
// TMEM accumulator; the epilogue warps add the runs' sums in registers.  The
// tensor cores' fp32 accumulation does not round to nearest (it truncates), so
// one accumulator carried over the whole K collects an error that grows in
// proportion to K (three MMAs add into it per k-step): measured against the
// ascending-k fp32 oracle with U(-1,1) operands, rel-L2 1.4e-5 at K = 2048 and
// 5.7e-5 at K = 8192.  Runs of 256 k bound that part to one run, and the runs
// are added with IEEE round-to-nearest.
constexpr int TC_TF32_CHUNK_KB = 8;

// Output tensor maps of the TMA-store epilogue: one per destination buffer.
struct StoreMaps {
  CUtensorMap m[OJX_MAX_PEERS];
};

// Batched GEMM (kernel instances with BATCH = 1): `batch` independent problems.
// A and B come from rank-3 tensor maps whose third coordinate is the batch index
// (a_bc / b_bc = 0: one matrix shared by every problem); C and the epilogue
// operand of problem b start stride_c / stride_op elements after problem b-1's.
struct BatchParams {
  int batch;
  int a_bc, b_bc;
  int64_t stride_c, stride_op;
};

// CG = 2: a CTA pair (cluster of 2) computes a 256 x BN tile with cta_group::2 MMAs;
// each CTA holds 128 rows of A and BN/2 columns of B per stage, and 128 rows x BN
// columns of the accumulator in its tensor memory.
template <int KIND, int BN, int STAGES, int STORE_TMA = 0, int CG = 1>
struct TcLayout {
  static constexpr int ELEM = KIND == 0 ? 2 : 4;
  static constexpr int BK = 128 / ELEM;  // elements in one 128-byte swizzle row
  static constexpr int B_ROWS = BN / CG;  // columns of B this CTA loads per stage
  static constexpr int A_BYTES = TC_BM * 128;
  static constexpr int B_BYTES = B_ROWS * 128;
  static constexpr int NPART = KIND == 0 ? 1 : 2;  // tf32: hi and lo copies
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * NPART;
  // 3xTF32 keeps two accumulators per tile (the Ah*Bh term and the two small terms),
  // so each of the two TMEM buffers is 2*BN columns wide.
  static constexpr uint32_t TMEM_COLS = (KIND == 1 ? 4 : 2) * BN;
  static constexpr int BAR_BYTES = 256;
  // TMA-store epilogue: one 32-row x 128-byte (swizzled) staging box per epilogue warp.
  static constexpr int STAGE_OUT_BYTES = 32 * 128;
  static constexpr int OUT_BYTES = STORE_TMA ? 8 * STAGE_OUT_BYTES : 0;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + OUT_BYTES + BAR_BYTES + 1024;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert((2 * STAGES + 6) * 8 + 8 <= BAR_BYTES, "barrier area too small");
};

// Grouped raster: GROUP consecutive M-blocks share each N-block sweep.  GROUP is 16
// blocks of 128 rows, or 8 of 256 rows for CTA pairs: either way one wave of tiles
// spans 2048 rows of A (a wave's A and B panels read least when it is about square).
template <int GROUP = 16>
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& mb, int& nb) {
  const int span = GROUP * tiles_n;
  const int g = tile / span;
  const int first_m = g * GROUP;
  const int gsize = min(tiles_m - first_m, GROUP);
  const int r = tile - g * span;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

// Descriptor of one 32-byte k-step of an operand tile.
//  K-major : rows of 128 B along k, 8-row groups 1024 B apart; a k-step moves 32 B.
//  MN-major: rows of 128 B (64 elements) along M/N, one row per k; 64-wide MN
//            blocks are `BK*128` bytes apart (LBO), 8-k groups 1024 B apart (SBO);
//            a k-step of 16 (f16) rows moves 2048 B.
template <int MN, int BK>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int ks) {
  if (MN) return make_sw128_desc(base + ks * 2048, BK * 128, 1024);
  return make_sw128_desc(base + ks * 32, 16, 1024);
}

// Loads of one operand tile (rows = 128 for A, BN for B) at (mn0, k0) of matrix bc.
// ext_mn / ext_k: the operand's extents (debug bounds checks only; the tile origin
// must lie inside, further 64-wide MN boxes of a partial tile may start past the
// edge and read the zero fill).
// CG = 2: `bar` is the shared::cluster address of the pair leader's barrier.
template <int MN, int BK, int ROWS, int BATCH, int CG = 1>
__device__ __forceinline__ void load_operand(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                             int mn0, int k0, int bc, int site, int ext_mn,
                                             int ext_k) {
  constexpr int ESZ = 128 / BK;
  static_assert(CG == 1 || BATCH == 0, "pair loads are 2-D");
  if (MN ? !tma_origin_ok(site, mn0, k0, ext_mn, ext_k, ESZ)
         : !tma_origin_ok(site, k0, mn0, ext_k, ext_mn, ESZ))
    return;
  if (MN) {
#pragma unroll
    for (int j = 0; j < ROWS / 64; ++j) {
      if (CG == 2)
        tma_load_2d_pair(dst + j * (BK * 128), map, bar, mn0 + 64 * j, k0);
      else if (BATCH)
        tma_load_3d(dst + j * (BK * 128), map, bar, mn0 + 64 * j, k0, bc);
      else
        tma_load_2d(dst + j * (BK * 128), map, bar, mn0 + 64 * j, k0);
    }
  } else {
    if (CG == 2)
      tma_load_2d_pair(dst, map, bar, k0, mn0);
    else if (BATCH)
      tma_load_3d(dst, map, bar, k0, mn0, bc);
    else
      tma_load_2d(dst, map, bar, k0, mn0);
  }
}

// Epilogue for 16 consecutive columns of one output row (accumulator values in v).
__device__ __forceinline__ void store_row16f(const EpiParams& ep, float (&v)[16], int64_t row,
                                             int col0, int N) {
  const int valid = min(16, N - col0);
  if (!epi_store_ok(ep, SITE_TC_STORE_REG, row, col0, valid)) return;
  epilogue16(ep, v, row, col0, valid);
  const int esz = ep.dtype_c == OJX_F32 ? 4 : 2;
  const int64_t off = (row * ep.ldc + ep.col_offset + col0) * esz;
  uint32_t p[8];
  if (ep.dtype_c != OJX_F32) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (ep.dtype_c == OJX_BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        p[j] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        p[j] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
  }
  // Static loop over the destination slots (no dynamic indexing of the
  // parameter array); slot i is used when i < n_dst.
#pragma unroll
  for (int di = 0; di < OJX_MAX_PEERS; ++di) {
    if (di >= ep.n_dst) break;
    char* dst = static_cast<char*>(ep.dst[di]) + off;
    if (valid == 16 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
      if (ep.dtype_c == OJX_F32) {
        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int j = 0; j < 4; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      } else {
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        d4[0] = make_uint4(p[0], p[1], p[2], p[3]);
        d4[1] = make_uint4(p[4], p[5], p[6], p[7]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < valid) store_elem(ep.dst[di], row * ep.ldc + ep.col_offset + col0 + j, ep.dtype_c, v[j]);
    }
  }
}
__device__ __forceinline__ void store_row16(const EpiParams& ep, const uint32_t (&r)[16],
                                            int64_t row, int col0, int N) {
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
  store_row16f(ep, v, row, col0, N);
}

// TMA-store epilogue of one 128-byte-wide chunk of a warp's 32 rows: accumulator
// values -> epilogue -> packed values in the warp's swizzled staging box -> one
// tensor store per destination.  ESZ = output element bytes (chunk = 128/ESZ
// columns); `col0` is the chunk's first output column (relative to the
// destination maps), `row0` the box's first row.  epi_chunk_tma_regs takes the
// values in registers, epi_chunk_tma reads them from TMEM columns tcol...
template <int ESZ, int BATCH>
__device__ __forceinline__ void epi_chunk_tma_regs(const EpiParams& ep, const StoreMaps& maps,
                                                   float (&v)[128 / ESZ], int64_t row, int M,
                                                   int col0, int N, uint32_t stage, int lane,
                                                   int row0, int bidx) {
  constexpr int V = 128 / ESZ;
#pragma unroll
  for (int i = 0; i < V / 16; ++i) {
    float w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j] = v[i * 16 + j];
    const int c = col0 + i * 16;
    // rows past M are computed but never stored (the tensor store clips them);
    // valid = 0 keeps their operand loads in bounds
    epilogue16(ep, w, row, c, row < M ? max(0, min(16, N - c)) : 0);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[i * 16 + j] = w[j];
  }
  uint32_t packed[32];  // 128 bytes of this row
  if (ESZ == 4) {
#pragma unroll
    for (int j = 0; j < 32; ++j) packed[j] = __float_as_uint(v[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (ep.dtype_c == OJX_BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        packed[j] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        packed[j] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
  }
  // The previous chunk's stores must have finished reading the staging box.
  if (lane == 0) bulk_wait_read_all();
  __syncwarp();
  const uint32_t rowaddr = stage + lane * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t a = rowaddr + ((j ^ (lane & 7)) << 4);  // 128-byte swizzle
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(packed[4 * j]),
                 "r"(packed[4 * j + 1]), "r"(packed[4 * j + 2]), "r"(packed[4 * j + 3])
                 : "memory");
  }
  fence_proxy_async_smem();  // generic-proxy writes -> visible to the TMA engine
  __syncwarp();
  // A box whose rows all lie past M (the last M-block of a ragged M) has nothing
  // to write: the tensor store would clip it whole.
  if (lane == 0 && row0 < M && tma_origin_ok(SITE_TC_STORE_TMA, col0, row0, N, M, ESZ)) {
#pragma unroll
    for (int d = 0; d < OJX_MAX_PEERS; ++d) {
      if (d >= ep.n_dst) break;
      if (BATCH)
        tma_store_3d(&maps.m[d], stage, col0, row0, bidx);
      else
        tma_store_2d(&maps.m[d], stage, col0, row0);
    }
    bulk_commit_group();
  }
}
template <int ESZ, int BATCH>
__device__ __forceinline__ void epi_chunk_tma(const EpiParams& ep, const StoreMaps& maps,
                                              uint32_t tcol, int64_t row, int M, int col0, int N,
                                              uint32_t stage, int lane, int row0, int bidx) {
  constexpr int V = 128 / ESZ;
  float v[V];
#pragma unroll
  for (int i = 0; i < V / 16; ++i) {
    uint32_t r[16];
    tmem_ld16(tcol + i * 16, r);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 16; ++j) v[i * 16 + j] = __uint_as_float(r[j]);
  }
  epi_chunk_tma_regs<ESZ, BATCH>(ep, maps, v, row, M, col0, N, stage, lane, row0, bidx);
}

// CG = 2 (bf16/fp16, unbatched): launched as clusters of 2 CTAs.  Each pair walks the
// 256-row tiles; rank 0 (the leader) owns the barriers the pair shares: its `full`
// barriers count both CTAs' TMA bytes, its `tempty` barriers both CTAs' epilogue
// warps, and its MMA thread issues the cta_group::2 MMAs and commits them to the
// `empty` and `tfull` barriers of both CTAs.  The other CTA's MMA thread is idle.
template <int KIND, int FMT, int A_MN, int B_MN, int BN, int STAGES, int STORE_TMA, int BATCH = 0,
          int CG = 1>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB2, const EpiParams ep,
                   const __grid_constant__ StoreMaps smaps, const int M, const int N, const int K,
                   const uint64_t budget, const int silence_producer, const BatchParams bp) {
  static_assert(CG == 1 || (CG == 2 && KIND == 0 && BATCH == 0), "CTA pairs: bf16/fp16, unbatched");
  using L = TcLayout<KIND, BN, STAGES, STORE_TMA, CG>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * L::STAGE_BYTES + L::OUT_BYTES);
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 5);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 6);
  const uint32_t sout = smem_u32(smem + STAGES * L::STAGE_BYTES);  // staging boxes

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = smem_u32(bars);
  // barrier addresses
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t done_bar = bar0 + 8u * (2 * STAGES + 4);

  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;  // in the CTA pair
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), CG * TC_EPI_WARPS);
    }
    mbar_init(done_bar, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (KIND == 1) {
      tma_prefetch_desc(&tmA2);
      tma_prefetch_desc(&tmB2);
    }
  }
  if (warp == 1) {
    if (CG == 2) {
      tmem_alloc_pair(smem_u32(s_tmem), L::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(s_tmem), L::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (CG == 2) cluster_sync();  // the peer's barriers are initialised before either signals them
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  // CG = 2: tiles are 256 rows (128 per CTA of the pair), walked per cluster.
  const int tiles_m = (M + TC_BM * CG - 1) / (TC_BM * CG);
  const int tiles_n = (N + BN - 1) / BN;
  const int tiles_per = tiles_m * tiles_n;  // per problem of a batch
  const int num_tiles = BATCH ? tiles_per * bp.batch : tiles_per;
  const int first_tile = static_cast<int>(blockIdx.x) / CG;
  const int tile_stride = static_cast<int>(gridDim.x) / CG;
  const int KB = (K + L::BK - 1) / L::BK;

  if (warp == 0) {
    // ── TMA producer ──────────────────────────────────────────────────────
    if (lane == 0 && !silence_producer) {
      int stage = 0;
      uint32_t phase = 0, issued = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = first_tile; tile < num_tiles && ok; tile += tile_stride) {
        const int bidx = BATCH ? tile / tiles_per : 0;
        int mb, nb;
        tile_coords<16 / CG>(tile - bidx * tiles_per, tiles_m, tiles_n, mb, nb);
        // this CTA's 128 rows of A and (CG = 2) its half of the tile's B columns
        const int m0 = (mb * CG + static_cast<int>(rank)) * TC_BM;
        const int n0 = nb * BN + static_cast<int>(rank) * L::B_ROWS;
        const int abc = bp.a_bc ? bidx : 0, bbc = bp.b_bc ? bidx : 0;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, budget, s_abort)) {
            ok = false;
            break;
          }
          // CG = 2: both CTAs' bytes complete on the leader's full barrier, for which
          // the leader alone announces the pair's total.
          const uint32_t fb = CG == 2 ? mapa_shared(full_bar(stage), 0) : full_bar(stage);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), CG * L::STAGE_BYTES);
          // stage layout: KIND 0 [A][B]; KIND 1 [A_hi][A_lo][B_hi][B_lo] (B_hi and B_lo
          // adjacent: one N = 2*BN MMA reads both)
          const uint32_t sA = sbase + stage * L::STAGE_BYTES;
          const uint32_t sB = sA + L::NPART * L::A_BYTES;
          const int k0 = kb * L::BK;
          // (the second CTA's half of a ragged pair tile may start past M or N and read
          // the zero fill: the debug checks take the pair tile's extent for a pair)
          load_operand<A_MN, L::BK, TC_BM, BATCH, CG>(sA, &tmA, fb, m0, k0, abc, SITE_TC_LOAD_A,
                                                      CG == 2 ? tiles_m * TC_BM * CG : M, K);
          load_operand<B_MN, L::BK, L::B_ROWS, BATCH, CG>(sB, &tmB, fb, n0, k0, bbc, SITE_TC_LOAD_B,
                                                         CG == 2 ? tiles_n * BN : N, K);
          if (KIND == 1) {
            load_operand<A_MN, L::BK, TC_BM, BATCH>(sA + L::A_BYTES, &tmA2, fb, m0, k0, abc,
                                                    SITE_TC_LOAD_A, M, K);
            load_operand<B_MN, L::BK, BN, BATCH>(sB + L::B_BYTES, &tmB2, fb, n0, k0, bbc,
                                                 SITE_TC_LOAD_B, N, K);
          }
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Let every copy this thread issued land before the CTA may exit.  (CG = 2: the
      // other CTA's copies complete on the leader's barrier; it waits instead for the
      // leader's MMAs to have consumed them, which its `empty` barriers record.)
      for (int s = 0; s < STAGES; ++s)
        if ((issued >> s) & 1u) {
          if (leader)
            mbar_wait_drain(full_bar(s), (issued_parity >> s) & 1u, budget);
          else
            mbar_wait_drain(empty_bar(s), (issued_parity >> s) & 1u, budget);
        }
    }
  } else if (warp == 1) {
    // ── MMA issuer (one thread; CG = 2: the leader's, for the pair) ──────────
    if (lane == 0 && leader) {
      constexpr uint32_t IDESC = make_idesc(FMT, A_MN, B_MN, TC_BM * CG, BN);
      // 3xTF32: Ah * [Bh | Bl] as one N = 2*BN MMA (the two products land side by side:
      // columns [0, BN) hold Ah*Bh, [BN, 2*BN) Ah*Bl), then Al * Bh added to the second
      // half.  The large term and the two small ones are accumulated apart and added in
      // the epilogue.
      constexpr uint32_t IDESC_WIDE = make_idesc(FMT, A_MN, B_MN, TC_BM, 2 * BN);
      constexpr uint32_t ACC_COLS = (KIND == 1 ? 2 : 1) * BN;  // TMEM columns per buffer
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      // Each run of KCH k-blocks goes into one TMEM accumulator buffer (KIND 0: the
      // whole K, one run per tile; 3xTF32: runs of TC_TF32_CHUNK_KB, see above).
      const int KCH = KIND == 1 ? TC_TF32_CHUNK_KB : KB;
      for (int tile = first_tile; tile < num_tiles && ok; tile += tile_stride) {
        for (int kc = 0; kc < KB && ok; kc += KCH) {
          if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, budget, s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + static_cast<uint32_t>(acc * ACC_COLS);
          const int kend = min(KB, kc + KCH);
          for (int kb = kc; kb < kend; ++kb) {
            if (!mbar_wait(full_bar(stage), phase, budget, s_abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sA = sbase + stage * L::STAGE_BYTES;
            const uint32_t sB = sA + L::NPART * L::A_BYTES;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t ad = operand_desc<A_MN, L::BK>(sA, ks);
              const uint64_t bd = operand_desc<B_MN, L::BK>(sB, ks);
              const uint32_t accum = (kb != kc || ks != 0) ? 1u : 0u;
              if (CG == 2) {
                mma_f16_pair(d, ad, bd, IDESC, accum);
              } else if (KIND == 0) {
                mma_f16(d, ad, bd, IDESC, accum);
              } else {
                const uint64_t ad_lo = operand_desc<A_MN, L::BK>(sA + L::A_BYTES, ks);
                mma_tf32(d, ad, bd, IDESC_WIDE, accum);  // [Ah*Bh | Ah*Bl]
                mma_tf32(d + BN, ad_lo, bd, IDESC, 1u);  // Ah*Bl + Al*Bh
              }
            }
            // smem slot free (in both CTAs of a pair) once these MMAs have read it
            if (CG == 2)
              mma_commit_pair(empty_bar(stage), 0x3);
            else
              mma_commit(empty_bar(stage));
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          // this run's sum ready for the epilogue (of both CTAs of a pair)
          if (CG == 2)
            mma_commit_pair(tfull_bar(acc), 0x3);
          else
            mma_commit(tfull_bar(acc));
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1u;
        }
      }
      // Every MMA issued above must complete before TMEM is released.
      if (CG == 2)
        mma_commit_pair(done_bar, 0x1);
      else
        mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0, budget);
    }
    __syncwarp();
  } else {
    // ── epilogue warps 2..9: lane quarter warp%4, column half (warp-2)/4 ──────
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    // 3xTF32: the tile's K arrives as runs of TC_TF32_CHUNK_KB k-blocks, each in one
    // TMEM buffer.  This warp adds its 32 rows x BN/2 columns of every run into
    // registers (fp32, round to nearest) and frees the buffer at once; after the
    // last run it applies the epilogue to the sums and stores them.  Returns false
    // when a bounded wait gave up.
    auto epi_tile_runs = [&](int tile) -> bool {
      constexpr int HC = BN / 2;
      float sum[HC];
      const int KCH = TC_TF32_CHUNK_KB;
      for (int kc = 0; kc < KB; kc += KCH) {
        if (!mbar_wait(tfull_bar(acc), acc_phase, budget, s_abort)) return false;
        tc_fence_after();
        // buffer acc: columns [0, BN) the Ah*Bh sums, [BN, 2*BN) the small terms
        const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(acc * 2 * BN + half * HC);
#pragma unroll
        for (int i = 0; i < HC; i += 16) {
          uint32_t r[16], t[16];
          tmem_ld16(tb + i, r);
          tmem_ld16(tb + BN + i, t);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float run = __uint_as_float(r[j]) + __uint_as_float(t[j]);
            sum[i + j] = kc == 0 ? run : sum[i + j] + run;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar(acc));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      const int bidx = BATCH ? tile / tiles_per : 0;
      int mb, nb;
      tile_coords<16 / CG>(tile - bidx * tiles_per, tiles_m, tiles_n, mb, nb);
      EpiParams epb = ep;
      if (BATCH) {
        const int esz_c = ep.dtype_c == OJX_F32 ? 4 : 2;
        const int esz_o = ep.dtype_operand == OJX_F32 ? 4 : 2;
        epb.dst[0] = static_cast<char*>(ep.dst[0]) + bidx * bp.stride_c * esz_c;
        if (ep.operand)
          epb.operand = static_cast<const char*>(ep.operand) + bidx * bp.stride_op * esz_o;
      }
      const int64_t row = static_cast<int64_t>(mb) * TC_BM + q * 32 + lane;
      const int n0 = nb * BN + half * HC;
      if (STORE_TMA) {
        const uint32_t stage_box = sout + static_cast<uint32_t>((warp - 2) * L::STAGE_OUT_BYTES);
        const int row0 = mb * TC_BM + q * 32;
        if (ep.dtype_c == OJX_F32) {
#pragma unroll
          for (int c = 0; c < HC; c += 32) {
            if (n0 + c < N) {
              float v[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = sum[c + j];
              epi_chunk_tma_regs<4, BATCH>(epb, smaps, v, row, M, n0 + c, N, stage_box, lane, row0,
                                           bidx);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < HC; c += 64) {
            if (n0 + c < N) {
              float v[64];
#pragma unroll
              for (int j = 0; j < 64; ++j) v[j] = sum[c + j];
              epi_chunk_tma_regs<2, BATCH>(epb, smaps, v, row, M, n0 + c, N, stage_box, lane, row0,
                                           bidx);
            }
          }
        }
      } else if (row < M) {
#pragma unroll
        for (int c = 0; c < HC; c += 16) {
          if (n0 + c < N) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = sum[c + j];
            store_row16f(epb, v, row, n0 + c, N);
          }
        }
      }
      return true;
    };
    for (int tile = first_tile; tile < num_tiles; tile += tile_stride) {
      if (KIND == 1) {
        if (!epi_tile_runs(tile)) break;
        continue;
      }
      if (!mbar_wait(tfull_bar(acc), acc_phase, budget, s_abort)) break;
      tc_fence_after();
      const int bidx = BATCH ? tile / tiles_per : 0;
      int mb, nb;
      tile_coords<16 / CG>(tile - bidx * tiles_per, tiles_m, tiles_n, mb, nb);
      // Problem bidx of a batch: its C and epilogue operand (ep is a copy, so
      // only the pointers of the fields the epilogue reads move).
      EpiParams epb = ep;
      if (BATCH) {
        const int esz_c = ep.dtype_c == OJX_F32 ? 4 : 2;
        const int esz_o = ep.dtype_operand == OJX_F32 ? 4 : 2;
        epb.dst[0] = static_cast<char*>(ep.dst[0]) + bidx * bp.stride_c * esz_c;
        if (ep.operand)
          epb.operand = static_cast<const char*>(ep.operand) + bidx * bp.stride_op * esz_o;
      }
      // this CTA's 128 rows of the tile (CG = 2: rank 1 holds the second 128)
      const int mrow = (mb * CG + static_cast<int>(rank)) * TC_BM;
      const int64_t row = static_cast<int64_t>(mrow) + q * 32 + lane;
      const int n0 = nb * BN + half * (BN / 2);
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(acc * BN + half * (BN / 2));
      if (STORE_TMA) {
        const uint32_t stage_box = sout + static_cast<uint32_t>((warp - 2) * L::STAGE_OUT_BYTES);
        const int row0 = mrow + q * 32;
        if (ep.dtype_c == OJX_F32) {
#pragma unroll 1
          for (int c = 0; c < BN / 2; c += 32) {
            if (n0 + c >= N) break;
            epi_chunk_tma<4, BATCH>(epb, smaps, tbase + c, row, M, n0 + c, N, stage_box, lane, row0,
                                    bidx);
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < BN / 2; c += 64) {
            if (n0 + c >= N) break;
            epi_chunk_tma<2, BATCH>(epb, smaps, tbase + c, row, M, n0 + c, N, stage_box, lane, row0,
                                    bidx);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          const int col0 = n0 + c;
          if (col0 >= N) break;  // uniform across the warp
          uint32_t r0[16], r1[16];
          tmem_ld16(tbase + c, r0);
          tmem_ld16(tbase + c + 16, r1);
          tmem_wait_ld();
          if (row < M) {
            store_row16(epb, r0, row, col0, N);
            if (col0 + 16 < N) store_row16(epb, r1, row, col0 + 16, N);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (CG == 2)  // the leader's MMA waits for both CTAs' epilogue warps
          mbar_arrive_cluster(mapa_shared(tempty_bar(acc), 0));
        else
          mbar_arrive(tempty_bar(acc));
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // Every tensor store has completed (and, for stores into other GPUs' memory,
    // is visible system-wide) before the kernel completes: the cross-rank barrier
    // that follows an all-gathering GEMM relies on it.
    if (STORE_TMA && lane == 0) bulk_wait_all();
    __syncwarp();
    if (ep.n_dst > 1) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  // A pair leaves together: the leader's MMAs (complete once its MMA thread passed
  // its done barrier) read the other CTA's shared memory and write its TMEM.
  if (CG == 2) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if (CG == 2)
      tmem_dealloc_pair(tmem_base, L::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

// fp32 -> (hi, lo) tf32 parts, K-major [R][Kp], zero for k >= K.
// Element (r, k) of the logical operand is src[r*ld + k] (trans == 0) or
// src[k*ld + r] (trans == 1).  tf32 rounding: cvt.rna (round to nearest, ties away).
// blockIdx.z selects one matrix of a batch: src_bs / dst_bs elements apart.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__global__ void __launch_bounds__(256) split_tf32_kernel(const float* __restrict__ src, int64_t ld,
                                                         int trans, int R, int K, int Kp,
                                                         float* __restrict__ hi,
                                                         float* __restrict__ lo, int64_t src_bs,
                                                         int64_t dst_bs) {
  __shared__ float tile[32][33];
  src += blockIdx.z * src_bs;
  hi += blockIdx.z * dst_bs;
  lo += blockIdx.z * dst_bs;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const int k0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  if (!trans) {
    for (int i = ty; i < 32; i += 8) {
      const int r = r0 + i, k = k0 + tx;
      if (r < R && k < Kp) {
        const float v = (k < K) ? src[static_cast<int64_t>(r) * ld + k] : 0.0f;
        const float h = to_tf32(v);
        const int64_t o = static_cast<int64_t>(r) * Kp + k;
        hi[o] = h;
        lo[o] = to_tf32(v - h);
      }
    }
  } else {
    for (int i = ty; i < 32; i += 8) {
      const int k = k0 + i, r = r0 + tx;
      tile[i][tx] = (k < K && r < R) ? src[static_cast<int64_t>(k) * ld + r] : 0.0f;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
      const int r = r0 + i, k = k0 + tx;
      if (r < R && k < Kp) {
        const float v = tile[tx][i];
        const float h = to_tf32(v);
        const int64_t o = static_cast<int64_t>(r) * Kp + k;
        hi[o] = h;
        lo[o] = to_tf32(v - h);
      }
    }
  }
}

// ── host side ────────────────────────────────────────────────────────────────

EpiParams make_epi(const ojx_gemm_desc& d, const Dests* dests) {
  EpiParams ep{};
  ep.c = d.c;
  ep.ldc = d.ldc;
  ep.operand = d.operand;
  ep.ld_operand = d.ld_operand;
  ep.dtype_c = d.dtype_c;
  ep.dtype_operand = d.dtype_operand;
  ep.operand_kind = d.operand_kind;
  ep.binary_op = d.binary_op;
  ep.operand_is_lhs = d.operand_is_lhs;
  ep.n_unary = d.n_unary;
  ep.unary_packed = 0;
  for (int i = 0; i < d.n_unary && i < OJX_MAX_UNARY; ++i)
    ep.unary_packed |= (static_cast<uint32_t>(d.unary[i]) & 15u) << (4 * i);
  ep.m_rows = d.M;
  ep.n_cols = d.N;
  ep.n_dst = 1;
  ep.col_offset = 0;
  for (int i = 0; i < OJX_MAX_PEERS; ++i) ep.dst[i] = d.c;
  if (dests) {
    ep.n_dst = dests->n;
    ep.col_offset = dests->col_offset;
    for (int i = 0; i < dests->n && i < OJX_MAX_PEERS; ++i) ep.dst[i] = dests->p[i];
  }
  return ep;
}

template <int KIND, int FMT, int A_MN, int B_MN, int BN, int STAGES, int STORE_TMA, int BATCH>
static int run_tc(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& a2,
                  const CUtensorMap& b2, const EpiParams& ep, const StoreMaps& sm, int M, int N,
                  int K, const BatchParams& bp, cudaStream_t s) {
  using L = TcLayout<KIND, BN, STAGES, STORE_TMA>;
  auto kern = tc_gemm_kernel<KIND, FMT, A_MN, B_MN, BN, STAGES, STORE_TMA, BATCH>;
  int st = ensure_smem_attr(reinterpret_cast<const void*>(kern), L::SMEM_BYTES);
  if (st) return st;
  const DeviceProps& p = current_props();
  const long tiles = static_cast<long>((M + TC_BM - 1) / TC_BM) * ((N + BN - 1) / BN) *
                     (BATCH ? bp.batch : 1);
  const int grid = static_cast<int>(std::min<long>(tiles, p.sm_count));
  const int silence = g_silence_producer_once.exchange(0);
  kern<<<grid, TC_THREADS, L::SMEM_BYTES, s>>>(a, b, a2, b2, ep, sm, M, N, K, g_wait_budget.load(),
                                               silence, bp);
  g_launches.fetch_add(1);
  return cuda_status(cudaGetLastError(), "tc_gemm launch");
}

// Clusters of 2 that can be resident at once for this kernel and launch shape (cached
// per kernel and device).  Returns 0 if none, or -status on a CUDA error.
static int pair_clusters(const void* kern, cudaLaunchConfig_t* cfg) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int>* cache = new std::map<std::pair<const void*, int>, int>();
  const int dev = current_props().device;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache->find({kern, dev});
  if (it != cache->end()) return it->second;
  cfg->gridDim = dim3(2 * (current_props().sm_count / 2));
  int n = 0;
  const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, cfg);
  if (e != cudaSuccess) return -cuda_status(e, "cudaOccupancyMaxActiveClusters");
  (*cache)[{kern, dev}] = n;
  return n;
}

// CTA-pair instance (cta_group::2, clusters of 2): launched with exactly as many
// clusters as can be resident at once (an SM count the pairs cannot tile, or GPCs
// with an odd number of SMs, leave some SMs out), so that no cluster starts late and
// runs its tiles after the others have finished.
template <int FMT, int A_MN, int B_MN, int BN, int STAGES>
static int run_tc_pair(const CUtensorMap& a, const CUtensorMap& b, const EpiParams& ep,
                       const StoreMaps& sm, int M, int N, int K, cudaStream_t s) {
  using L = TcLayout<0, BN, STAGES, 1, 2>;
  auto kern = tc_gemm_kernel<0, FMT, A_MN, B_MN, BN, STAGES, 1, 0, 2>;
  int st = ensure_smem_attr(reinterpret_cast<const void*>(kern), L::SMEM_BYTES);
  if (st) return st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = L::SMEM_BYTES;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int clusters = pair_clusters(reinterpret_cast<const void*>(kern), &cfg);
  if (clusters <= 0) return clusters < 0 ? -clusters : set_error(OJX_ERR_UNSUPPORTED, "no CTA pair fits");
  const long tiles = static_cast<long>((M + 255) / 256) * ((N + BN - 1) / BN);
  cfg.gridDim = dim3(static_cast<unsigned>(2 * std::min<long>(tiles, clusters)));
  const BatchParams bp{};
  const int silence = g_silence_producer_once.exchange(0);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, b, a, b, ep, sm, M, N, K,
                                           g_wait_budget.load(), silence, bp);
  g_launches.fetch_add(1);
  if (e != cudaSuccess) return cuda_status(e, "tc_gemm pair launch");
  return cuda_status(cudaGetLastError(), "tc_gemm pair launch");
}

// Output tensor maps for the TMA-store epilogue: destination i is the [M, N] block
// at ep.dst[i] + col_offset with row stride ldc.  Returns false (no error) when an
// address or the stride is not 16-byte aligned; the register-store epilogue is
// used then.
static bool make_store_maps(const EpiParams& ep, int M, int N, StoreMaps* sm,
                            const BatchInfo* bi = nullptr) {
  const int esz = ep.dtype_c == OJX_F32 ? 4 : 2;
  if ((ep.ldc * esz) % 16 != 0 || (ep.col_offset * esz) % 16 != 0) return false;
  if (bi && (bi->stride_c * esz) % 16 != 0) return false;
  const CUtensorMapDataType dt = ep.dtype_c == OJX_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : ep.dtype_c == OJX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  for (int i = 0; i < ep.n_dst; ++i) {
    const char* base = static_cast<const char*>(ep.dst[i]) + ep.col_offset * esz;
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
    const int st = bi ? make_tmap_3d_sw128(&sm->m[i], dt, esz, base, N, M, bi->batch, ep.ldc * esz,
                                           bi->stride_c * esz, 128 / esz, 32)
                      : make_tmap_2d_sw128(&sm->m[i], dt, esz, base, N, M, ep.ldc * esz, 128 / esz, 32);
    if (st != OJX_OK) return false;
  }
  return true;
}

bool tc_gemm_supported(const ojx_gemm_desc& d) {
  if (d.dtype_a != d.dtype_b || (d.dtype_a != OJX_BF16 && d.dtype_a != OJX_F16)) return false;
  if (d.K <= 0 || d.M > INT32_MAX || d.N > INT32_MAX || d.K > INT32_MAX) return false;
  if (reinterpret_cast<uintptr_t>(d.a) % 16 || reinterpret_cast<uintptr_t>(d.b) % 16) return false;
  if ((d.lda * 2) % 16 || (d.ldb * 2) % 16) return false;
  return true;
}

// Rank-2 map of one operand, or for a batch the rank-3 map over all its matrices
// (one matrix when stride == 0: every problem reads the same one).
static int operand_map(CUtensorMap* m, CUtensorMapDataType dt, int esz, const void* base,
                       uint64_t inner, uint64_t outer, int64_t ld, const BatchInfo* bi,
                       int64_t stride, uint32_t box_inner, uint32_t box_outer) {
  if (!bi) return make_tmap_2d_sw128(m, dt, esz, base, inner, outer, ld * esz, box_inner, box_outer);
  const uint64_t nb = stride ? static_cast<uint64_t>(bi->batch) : 1;
  const uint64_t bs = stride ? static_cast<uint64_t>(stride) * esz
                             : (outer * ld * esz + 15) / 16 * 16;  // never stepped over
  return make_tmap_3d_sw128(m, dt, esz, base, inner, outer, nb, ld * esz, bs, box_inner, box_outer);
}

static BatchParams batch_params(const BatchInfo* bi, bool a_batched, bool b_batched) {
  BatchParams bp{};
  bp.batch = bi ? static_cast<int>(bi->batch) : 1;
  bp.a_bc = bi && a_batched ? 1 : 0;
  bp.b_bc = bi && b_batched ? 1 : 0;
  bp.stride_c = bi ? bi->stride_c : 0;
  bp.stride_op = bi ? bi->stride_op : 0;
  return bp;
}

int launch_tc_gemm(const ojx_gemm_desc& d, cudaStream_t s, const Dests* dests, const BatchInfo* bi) {
  const int M = static_cast<int>(d.M), N = static_cast<int>(d.N), K = static_cast<int>(d.K);
  const CUtensorMapDataType tdt =
      d.dtype_a == OJX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const DeviceProps& p = current_props();
  // BN = 256 unless that leaves most SMs idle.
  const long tiles256 =
      static_cast<long>((M + 127) / 128) * ((N + 255) / 256) * (bi ? bi->batch : 1);
  const int BN = tiles256 >= p.sm_count ? 256 : 128;
  CUtensorMap ta, tb;
  int st;
  // CTA pairs (256 x 256 tiles, cta_group::2), on request (OJX_GEMM_FLAG_PAIR), for
  // unbatched problems with A row-major that fill every pair at least once; each SM
  // then loads 32 KB per k-block instead of 48 KB.  Measured on this GPU: 1.6-2.4 %
  // faster than one-CTA tiles in short runs (8192^3, the FFN shape), but at 32768^3,
  // where a run sits at the 1000 W power limit, the pairs held the SM clock at
  // 900-920 MHz against 1260-1275 MHz and were 25 % slower.  One-CTA tiles stay the
  // default.
  const bool pair = !bi && !d.trans_a && BN == 256 && (d.flags & OJX_GEMM_FLAG_PAIR) &&
                    static_cast<long>((M + 255) / 256) * ((N + 255) / 256) >= p.sm_count / 2;
  if (pair) {
    const EpiParams ep = make_epi(d, dests);
    StoreMaps sm;
    if (make_store_maps(ep, M, N, &sm)) {
      if ((st = operand_map(&ta, tdt, 2, d.a, K, M, d.lda, nullptr, 0, 64, 128))) return st;
      if (!d.trans_b)
        st = operand_map(&tb, tdt, 2, d.b, N, K, d.ldb, nullptr, 0, 64, 64);
      else
        st = operand_map(&tb, tdt, 2, d.b, K, N, d.ldb, nullptr, 0, 64, 128);
      if (st) return st;
      const bool bf = d.dtype_a == OJX_BF16;
      if (bf && !d.trans_b) return run_tc_pair<1, 0, 1, 256, 6>(ta, tb, ep, sm, M, N, K, s);
      if (bf) return run_tc_pair<1, 0, 0, 256, 6>(ta, tb, ep, sm, M, N, K, s);
      if (!d.trans_b) return run_tc_pair<0, 0, 1, 256, 6>(ta, tb, ep, sm, M, N, K, s);
      return run_tc_pair<0, 0, 0, 256, 6>(ta, tb, ep, sm, M, N, K, s);
    }
  }
  // A: K-major [M,K] (box 64k x 128m) or MN-major [K,M] (box 64m x 64k).
  if (!d.trans_a)
    st = operand_map(&ta, tdt, 2, d.a, K, M, d.lda, bi, bi ? bi->stride_a : 0, 64, 128);
  else
    st = operand_map(&ta, tdt, 2, d.a, M, K, d.lda, bi, bi ? bi->stride_a : 0, 64, 64);
  if (st) return st;
  // B: MN-major [K,N] (box 64n x 64k) or K-major [N,K] (box 64k x BN).
  if (!d.trans_b)
    st = operand_map(&tb, tdt, 2, d.b, N, K, d.ldb, bi, bi ? bi->stride_b : 0, 64, 64);
  else
    st = operand_map(&tb, tdt, 2, d.b, K, N, d.ldb, bi, bi ? bi->stride_b : 0, 64, BN);
  if (st) return st;
  const EpiParams ep = make_epi(d, dests);
  StoreMaps sm;
  const bool tma_out = make_store_maps(ep, M, N, &sm, bi);
  if (bi && !tma_out)
    return set_error(OJX_ERR_UNSUPPORTED, "batched tcgen05 GEMM needs 16-byte aligned C rows and strides");
  const BatchParams bp = batch_params(bi, bi && bi->stride_a, bi && bi->stride_b);
  const int fmt = d.dtype_a == OJX_BF16 ? 1 : 0;
  const int am = d.trans_a ? 1 : 0, bm = d.trans_b ? 0 : 1;
#define OJX_TC_CASE(FMTV, AMN, BMN, BNV)                                                        \
  if (fmt == FMTV && am == AMN && bm == BMN && BN == BNV) {                                      \
    constexpr int STG = BNV == 256 ? 4 : 6;                                                      \
    if (bi) return run_tc<0, FMTV, AMN, BMN, BNV, STG, 1, 1>(ta, tb, ta, tb, ep, sm, M, N, K, bp, s); \
    return tma_out ? run_tc<0, FMTV, AMN, BMN, BNV, STG, 1, 0>(ta, tb, ta, tb, ep, sm, M, N, K, bp, s) \
                   : run_tc<0, FMTV, AMN, BMN, BNV, STG, 0, 0>(ta, tb, ta, tb, ep, sm, M, N, K, bp, s); \
  }
#define OJX_TC_BN(FMTV, AMN, BMN) \
  OJX_TC_CASE(FMTV, AMN, BMN, 256) OJX_TC_CASE(FMTV, AMN, BMN, 128)
  OJX_TC_BN(1, 0, 1) OJX_TC_BN(1, 0, 0) OJX_TC_BN(1, 1, 1) OJX_TC_BN(1, 1, 0)
  OJX_TC_BN(0, 0, 1) OJX_TC_BN(0, 0, 0) OJX_TC_BN(0, 1, 1) OJX_TC_BN(0, 1, 0)
#undef OJX_TC_BN
#undef OJX_TC_CASE
  return set_error(OJX_ERR_UNSUPPORTED, "no tcgen05 GEMM instance for this layout");
}

int launch_tc_gemm_3xtf32(const ojx_gemm_desc& d, cudaStream_t s, const BatchInfo* bi) {
  const int M = static_cast<int>(d.M), N = static_cast<int>(d.N), K = static_cast<int>(d.K);
  const int Kp = (K + 3) / 4 * 4;  // 16-byte row stride for TMA
  // distinct A / B matrices of a batch (1 when one matrix is shared)
  const int64_t nA = bi && bi->stride_a ? bi->batch : 1;
  const int64_t nB = bi && bi->stride_b ? bi->batch : 1;
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t a_part = al(static_cast<size_t>(M) * Kp * 4 * nA);
  const size_t b_part = al(static_cast<size_t>(N) * Kp * 4 * nB);
  char* ws = static_cast<char*>(stream_workspace(s, 2 * a_part + 2 * b_part, 0, false));
  if (!ws) return workspace_error();
  float* a_hi = reinterpret_cast<float*>(ws);
  float* a_lo = reinterpret_cast<float*>(ws + a_part);
  float* b_hi = reinterpret_cast<float*>(ws + 2 * a_part);
  float* b_lo = reinterpret_cast<float*>(ws + 2 * a_part + b_part);
  // A -> [nA][M][Kp]; op(B)^T -> [nB][N][Kp] (the MMA's B operand is N x K, K-major).
  dim3 blk(256);
  split_tf32_kernel<<<dim3((Kp + 31) / 32, (M + 31) / 32, static_cast<unsigned>(nA)), blk, 0, s>>>(
      static_cast<const float*>(d.a), d.lda, d.trans_a ? 1 : 0, M, K, Kp, a_hi, a_lo,
      bi ? bi->stride_a : 0, static_cast<int64_t>(M) * Kp);
  g_launches.fetch_add(1);
  split_tf32_kernel<<<dim3((Kp + 31) / 32, (N + 31) / 32, static_cast<unsigned>(nB)), blk, 0, s>>>(
      static_cast<const float*>(d.b), d.ldb, d.trans_b ? 0 : 1, N, K, Kp, b_hi, b_lo,
      bi ? bi->stride_b : 0, static_cast<int64_t>(N) * Kp);
  g_launches.fetch_add(1);
  int st = cuda_status(cudaGetLastError(), "split_tf32 launch");
  if (st) return st;
  constexpr int BN = 128;
  CUtensorMap ta, tb, ta2, tb2;
  const auto F = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  auto map = [&](CUtensorMap* m, const float* base, int rows, int64_t n, uint32_t box_rows) {
    if (!bi) return make_tmap_2d_sw128(m, F, 4, base, Kp, rows, Kp * 4ull, 32, box_rows);
    return make_tmap_3d_sw128(m, F, 4, base, Kp, rows, n, Kp * 4ull, static_cast<uint64_t>(rows) * Kp * 4,
                              32, box_rows);
  };
  if ((st = map(&ta, a_hi, M, nA, 128))) return st;
  if ((st = map(&ta2, a_lo, M, nA, 128))) return st;
  if ((st = map(&tb, b_hi, N, nB, BN))) return st;
  if ((st = map(&tb2, b_lo, N, nB, BN))) return st;
  const EpiParams ep = make_epi(d);
  StoreMaps sm;
  const bool tma_out = make_store_maps(ep, M, N, &sm, bi);
  const BatchParams bp = batch_params(bi, nA > 1, nB > 1);
  if (bi) {
    if (!tma_out)
      return set_error(OJX_ERR_UNSUPPORTED, "batched 3xTF32 GEMM needs 16-byte aligned C rows and strides");
    return run_tc<1, 2, 0, 0, BN, 3, 1, 1>(ta, tb, ta2, tb2, ep, sm, M, N, Kp, bp, s);
  }
  if (tma_out) return run_tc<1, 2, 0, 0, BN, 3, 1, 0>(ta, tb, ta2, tb2, ep, sm, M, N, Kp, bp, s);
  return run_tc<1, 2, 0, 0, BN, 3, 0, 0>(ta, tb, ta2, tb2, ep, sm, M, N, Kp, bp, s);
}

}  // namespace ojx
