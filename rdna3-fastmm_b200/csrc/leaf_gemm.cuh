// Leaf products of the reduced-rank linear: R independent FP16 GEMMs
//   P[r][m][n] = sum_k L[r][m][k] * Rt[r][n][k]
// on the 5th-generation tensor cores (tcgen05) of sm_100a.  With kBf16 the
// planes and products are BF16 instead (same kind::f16 MMA, BF16 operand
// formats in the instruction descriptor, BF16 rounding in the epilogue).
//
// Structure (one CTA per SM, persistent over the (r, tile_m, tile_n) grid):
//   warp 0      TMA producer: 3-D tensor maps over the stacked planes, one
//               128x64 L tile and one BNx64 Rt tile per stage (128-byte
//               swizzle), STAGES-deep ring guarded by full/empty mbarriers.
//   warp 1      MMA issuer (one elected thread): 4 x tcgen05.mma m128nBNk16
//               per stage into an FP32 accumulator in tensor memory; two
//               accumulators (2 x BN columns) so the epilogue of one tile
//               overlaps the main loop of the next.  Also owns TMEM alloc.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, round to FP16,
//               16-byte stores of P.
// Out-of-range rows/columns/K are zero-filled by TMA, so ragged shapes need
// no special casing in the main loop; the epilogue masks its stores.
// Every wait is bounded (mbar_wait_bounded); on a timeout all roles unwind,
// drain what they issued, and the CTA frees its tensor memory and returns.
#pragma once

#include "fmm_common.cuh"

namespace fmm {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;

template <int BN, int STAGES>
struct LeafGemmConfig {
  static constexpr int kBN = BN;
  static constexpr int kStages = STAGES;
  static constexpr uint32_t kABytes = kGemmBM * kGemmBK * 2;  // 16 KiB
  static constexpr uint32_t kBBytes = BN * kGemmBK * 2;       // 32 KiB at BN=256
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
  // tiles + 1 KiB slack for the 1024-byte alignment + barrier block
  static constexpr size_t kSmemBytes = size_t(STAGES) * kStageBytes + 1024 + 256;
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation must be a power of two");
};

struct LeafGemmParams {
  int64_t bm, bn, bk;
  int64_t ldp;
  // rows between consecutive planes of L and P (>= bm): bm for a whole
  // launch, the full plane height when a launch covers a band of rows
  int64_t plane_rows;
  int32_t rank;
  int32_t tiles_m, tiles_n;
  int32_t group_m;
  int32_t serpentine;  // odd groups sweep the N-tiles in reverse
  // 2-SM kernel, 256-column tiles: the last `tail_rows` (1..32) rows of every
  // plane are computed transposed, P^T = Rt * L_tail^T, in `tail_tiles`
  // 256-row tiles over bn per batch (0, 0: no transposed tail)
  int32_t tail_rows, tail_tiles;
  uint16_t* P;  // FP16 (or BF16) products
  uint64_t timeout_ns;
};

// Tile t -> (r, tm, tn): batches in order, inside a batch groups of
// `group_m` M-tiles sweep the N-tiles so concurrently running CTAs share L
// rows and Rt columns in L2; with `serpentine` every odd group sweeps them in
// reverse, so a group starts on the Rt columns its predecessor used last.
__device__ __forceinline__ void leaf_tile_coords(const LeafGemmParams& p, int t, int& r, int& tm,
                                                 int& tn) {
  const int per_batch = p.tiles_m * p.tiles_n;
  r = t / per_batch;
  const int local = t - r * per_batch;
  const int per_group = p.group_m * p.tiles_n;
  const int group = local / per_group;
  const int first_m = group * p.group_m;
  const int group_rows = min(p.tiles_m - first_m, p.group_m);
  const int in_group = local - group * per_group;
  tm = first_m + in_group % group_rows;
  tn = in_group / group_rows;
  if (p.serpentine && (group & 1)) tn = p.tiles_n - 1 - tn;
}

// Columns the MMA computes for N tile tn: the whole tile, or for the ragged
// last tile the remainder rounded up to `granule` (a valid MMA N for the
// instruction shape), so no tensor-core time goes to columns past bn.  Every
// column the epilogue stores (below ldp = bn rounded up to 8) lies inside it.
__device__ __forceinline__ int tile_n_columns(const LeafGemmParams& p, int tn, int tile_n, int granule) {
  const int64_t rem = p.bn - static_cast<int64_t>(tn) * tile_n;
  if (rem >= tile_n) return tile_n;
  return static_cast<int>((rem + granule - 1) / granule * granule);
}

// 2-SM kernel: tile t -> batch r and either a regular tile (tm, tn) of the
// rows above the transposed tail, or (transposed) tail tile tm over bn.  Each
// batch runs its regular tiles (leaf_tile_coords' order) and then its tail
// tiles, which re-read the batch's Rt planes while they are still in L2.
__device__ __forceinline__ void pair_tile_coords(const LeafGemmParams& p, int t, int& r, int& tm, int& tn,
                                                 bool& transposed) {
  const int regular = p.tiles_m * p.tiles_n;
  const int per_batch = regular + p.tail_tiles;
  r = t / per_batch;
  const int local = t - r * per_batch;
  transposed = local >= regular;
  if (transposed) {
    tm = local - regular;
    tn = 0;
    return;
  }
  int rr;
  leaf_tile_coords(p, r * regular + local, rr, tm, tn);
}

template <class Cfg, bool kBf16 = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    leaf_gemm_kernel(const __grid_constant__ CUtensorMap tmap_l,
                     const __grid_constant__ CUtensorMap tmap_r, const LeafGemmParams p) {
  constexpr int BN = Cfg::kBN;
  constexpr int STAGES = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t a_base = base;
  const uint32_t b_base = base + STAGES * Cfg::kABytes;
  uint8_t* ctrl = smem + STAGES * Cfg::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ctrl);
  const uint32_t full_bar = smem_u32(bars);                   // [STAGES]
  const uint32_t empty_bar = smem_u32(bars + STAGES);         // [STAGES]
  const uint32_t tfull_bar = smem_u32(bars + 2 * STAGES);     // [2]
  const uint32_t tempty_bar = smem_u32(bars + 2 * STAGES + 2);  // [2]
  const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar + 8 * s, 1);
      mbar_init(empty_bar + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar + 8 * b, 1);
      mbar_init(tempty_bar + 8 * b, 4);  // one arrival per epilogue warp
    }
    mbar_init(drain_bar, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmap_l);
    prefetch_tmap(&tmap_r);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = p.rank * p.tiles_m * p.tiles_n;
  const int k_blocks = static_cast<int>((p.bk + kGemmBK - 1) / kGemmBK);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        int r, tm, tn;
        leaf_tile_coords(p, t, r, tm, tn);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait_bounded(empty_bar + 8 * stage, phase ^ 1u, abort, p.timeout_ns, 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar + 8 * stage, Cfg::kStageBytes);
          tma_load_3d(a_base + stage * Cfg::kABytes, &tmap_l, full_bar + 8 * stage,
                      kb * kGemmBK, tm * kGemmBM, r);
          tma_load_3d(b_base + stage * Cfg::kBBytes, &tmap_r, full_bar + 8 * stage,
                      kb * kGemmBK, tn * BN, r);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // drain: the last min(STAGES, issued) loads may still be landing
        int s = stage;
        uint32_t ph = phase;
        for (int n = 0; n < STAGES && n < issued; ++n) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1u;
          }
          volatile int no_abort = 0;
          mbar_wait_bounded(full_bar + 8 * s, ph, &no_abort, p.timeout_ns, 5);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        int r, tm, tn;
        leaf_tile_coords(p, t, r, tm, tn);
        // M = 128, cta_group::1: N a multiple of 16
        const uint32_t idesc =
            idesc_kind_f16<kBf16>(kGemmBM, static_cast<uint32_t>(tile_n_columns(p, tn, BN, 16)));
        if (!mbar_wait_bounded(tempty_bar + 8 * acc, acc_phase ^ 1u, abort, p.timeout_ns, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait_bounded(full_bar + 8 * stage, phase, abort, p.timeout_ns, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_base + stage * Cfg::kABytes;
          const uint32_t b_addr = b_base + stage * Cfg::kBBytes;
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk) {
            const uint64_t a_desc = smem_desc_k_sw128(a_addr + kk * 32);
            const uint64_t b_desc = smem_desc_k_sw128(b_addr + kk * 32);
            tc_mma_f16(d_tmem, a_desc, b_desc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          tc_commit(empty_bar + 8 * stage);  // frees the stage once read
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(tfull_bar + 8 * acc);  // accumulator ready for the epilogue
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        // drain our own tensor-core work before the CTA frees TMEM
        tc_commit(drain_bar);
        volatile int no_abort = 0;
        mbar_wait_bounded(drain_bar, 0, &no_abort, p.timeout_ns, 6);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      int r, tm, tn;
      leaf_tile_coords(p, t, r, tm, tn);
      int ready = 0;
      if (lane == 0)
        ready = mbar_wait_bounded(tfull_bar + 8 * acc, acc_phase, abort, p.timeout_ns, 4) ? 1 : 0;
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tm) * kGemmBM + row_in_tile;
      uint16_t* prow = p.P + (static_cast<int64_t>(r) * p.plane_rows + row) * p.ldp;
      const uint32_t t_addr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const int n_cols = tile_n_columns(p, tn, BN, 16);
#pragma unroll 1
      for (int c = 0; c < n_cols; c += 32) {
        uint32_t v[32];
        tc_ld_32x32b_x32(t_addr + c, v);
        tc_wait_ld();
        const int64_t col = static_cast<int64_t>(tn) * BN + c;
        if (row < p.bm) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int64_t c8 = col + q * 8;
            if (c8 + 8 <= p.ldp) {
              uint4 pk;
              uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                w[e] = pack2_rn<kBf16>(__uint_as_float(v[q * 8 + 2 * e]),
                                       __uint_as_float(v[q * 8 + 2 * e + 1]));
              *reinterpret_cast<uint4*>(prow + c8) = pk;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar + 8 * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs on a TPC computes one 256 x BN tile with
// tcgen05.mma.cta_group::2 (M = 256).  CTA r of the pair holds rows
// [128 r, 128 r + 128) of the L tile and rows [BN/2 r, BN/2 r + BN/2) of the
// Rt tile in its own shared memory; the tensor cores of the pair read both
// halves, so each SM stages half of the B operand it would need alone -- per
// 64-deep stage 16 KiB of L and BN*64 B of Rt per SM, i.e. about 128 B/clk of
// shared-memory traffic at the full MMA rate instead of 192.
//
// Roles (both CTAs unless noted):
//   warp 0   TMA producer: waits on its own `empty` stage barrier (released by
//            the pair's multicast commit), loads its halves; the bytes complete
//            on the EVEN CTA's `full` barrier (.cta_group::2 TMA), where the even
//            CTA's producer has posted the expected byte count of both halves.
//   warp 1   TMEM allocation for the pair (both CTAs); in the even CTA one
//            thread issues the MMAs and the multicast commits.
//   warps 2-5 epilogue: each CTA drains its own 128 accumulator lanes and
//            signals the even CTA's `tmem_empty` barrier (8 arrivals); the
//            products leave as 16-byte row stores, or (TMA_STORE) as 32 x 32
//            blocks staged in shared memory and written by TMA stores.
// No TMA multicast is used: every CTA loads only its own halves.  Leaves with
// bk >= 1024 run 128-deep k-blocks in 3 stages (two 64-deep atom columns per
// operand and stage, half the barrier round trips per FLOP) with the TMA-store
// epilogue; the host picks the configuration (fmm_api.cu).  With 256-column
// tiles a short last M tile of 1..32 rows is computed transposed (tail tiles
// after each batch's regular tiles, pair_tile_coords): A = 128 Rt rows a CTA,
// B = 16 L tail rows a CTA, N = 32, and the epilogue writes the tail rows of P
// column by column.
template <int BN, int STAGES, int BK = kGemmBK, bool TMA_STORE = false>
struct LeafGemmPairConfig {
  static constexpr int kBN = BN;
  static constexpr int kStages = STAGES;
  // Epilogue: per-lane 16-byte row stores (false), or each warp stages 32 x 32
  // FP16 blocks in shared memory (64-byte swizzle, two buffers a warp) and
  // writes them with TMA stores (true)
  static constexpr bool kTmaStore = TMA_STORE;
  static constexpr uint32_t kStoreBufBytes = 32 * 32 * 2;
  static constexpr uint32_t kStoreBytes = TMA_STORE ? 4 * 2 * kStoreBufBytes : 0;
  // k-block depth 64 or 128: one or two 64-deep columns of 128-byte swizzle
  // atoms per operand and stage
  static constexpr int kBK = BK;
  static constexpr int kAtomK = 64;  // k per swizzle-atom column (128-byte rows)
  static constexpr int kAtoms = BK / kAtomK;
  static constexpr uint32_t kAAtomBytes = kGemmBM * kAtomK * 2;
  static constexpr uint32_t kBAtomBytes = (BN / 2) * kAtomK * 2;
  static constexpr int kTileM = 2 * kGemmBM;              // 256 rows per pair
  static constexpr uint32_t kABytes = kGemmBM * BK * 2;   // this CTA's L half: 16 KiB at BK=64
  static constexpr uint32_t kBBytes = (BN / 2) * BK * 2;  // this CTA's Rt half
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  // two accumulators of BN columns; the allocation is a power of two
  static constexpr uint32_t kTmemCols = 2 * BN <= 256 ? 256 : 512;
  // stages + store buffers + 1 KiB slack for the 1024-byte alignment + the
  // barrier block (2 * STAGES + 5 barriers, the TMEM slot and the abort flag)
  static constexpr size_t kSmemBytes =
      size_t(STAGES) * kStageBytes + kStoreBytes + 1024 + 8 * (2 * STAGES + 8);
  static_assert(2 * BN <= 512 && BN % 32 == 0, "two BN-column accumulators must fit in TMEM");
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
  static_assert(BK == 64 || BK == 128, "k-block depth");
};

template <class Cfg, bool kBf16 = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    leaf_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_l,
                          const __grid_constant__ CUtensorMap tmap_r,
                          const __grid_constant__ CUtensorMap tmap_r16,
                          const __grid_constant__ CUtensorMap tmap_p,
                          const __grid_constant__ CUtensorMap tmap_l16, const LeafGemmParams p) {
  constexpr int BN = Cfg::kBN;
  constexpr int STAGES = Cfg::kStages;
  constexpr int BK = Cfg::kBK;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t a_base = base;
  const uint32_t b_base = base + STAGES * Cfg::kABytes;
  const uint32_t store_base = base + STAGES * Cfg::kStageBytes;  // kTmaStore: 8 buffers of 2 KiB
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::kStageBytes + Cfg::kStoreBytes);
  const uint32_t full_bar = smem_u32(bars);                     // [STAGES], used in CTA 0
  const uint32_t empty_bar = smem_u32(bars + STAGES);           // [STAGES], each CTA
  const uint32_t tfull_bar = smem_u32(bars + 2 * STAGES);       // [2], each CTA
  const uint32_t tempty_bar = smem_u32(bars + 2 * STAGES + 2);  // [2], used in CTA 0
  const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t cta = cluster_cta_rank();  // 0 = even CTA (issues the MMAs)
  const int pair = blockIdx.x / 2;
  const int pairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar + 8 * s, 1);
      mbar_init(empty_bar + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar + 8 * b, 1);
      mbar_init(tempty_bar + 8 * b, 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(drain_bar, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmap_l);
    prefetch_tmap(&tmap_r);
    prefetch_tmap(&tmap_r16);
    if constexpr (Cfg::kTmaStore) prefetch_tmap(&tmap_p);
    if (p.tail_rows > 0) prefetch_tmap(&tmap_l16);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Transposed tail (256-column tiles only: its A operand is a 128-row box of
  // the Rt map): rows [rows_main, bm) of every plane come from tail tiles
  // P^T = Rt * L_tail^T with M = 256 Rt rows and N = 32 (16 L rows per CTA,
  // zero-filled past bm); the regular tiles cover rows [0, rows_main).
  constexpr bool kTailOk = BN == Cfg::kTileM;
  const int tail_rows = kTailOk ? p.tail_rows : 0;
  const int64_t rows_main = p.bm - tail_rows;
  const int tiles_m = static_cast<int>((rows_main + Cfg::kTileM - 1) / Cfg::kTileM);
  const int tiles_n = static_cast<int>((p.bn + BN - 1) / BN);
  LeafGemmParams q = p;
  q.tiles_m = tiles_m;
  q.tiles_n = tiles_n;
  q.tail_rows = tail_rows;
  q.tail_tiles = tail_rows > 0 ? p.tail_tiles : 0;
  const int total_tiles = p.rank * (tiles_m * tiles_n + q.tail_tiles);
  const int k_blocks = static_cast<int>((p.bk + BK - 1) / BK);

  if (warp == 0) {
    // ------------------------------------------------------------ producers
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int issued = 0;
      for (int t = pair; t < total_tiles && ok; t += pairs) {
        int r, tm, tn;
        bool tr;
        pair_tile_coords(q, t, r, tm, tn, tr);
        const int a_row = tm * Cfg::kTileM + static_cast<int>(cta) * kGemmBM;
        // Each CTA supplies half of the N columns the pair's MMA computes.  A
        // ragged last tile loads exactly its half in 16-row boxes: a BN/2-row
        // box would fetch rows that belong to the other CTA's half.  A
        // transposed tail tile takes its A rows from Rt and 16 L tail rows a CTA.
        const int n_cols = tr ? 32 : tile_n_columns(q, tn, BN, 32);
        const int half = n_cols / 2;
        const int b_row = tr ? static_cast<int>(rows_main) + static_cast<int>(cta) * 16
                             : tn * BN + static_cast<int>(cta) * half;
        const uint32_t stage_tx = 2u * (Cfg::kABytes + static_cast<uint32_t>(half) * BK * 2u);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait_bounded_cluster(empty_bar + 8 * stage, phase ^ 1u, abort, p.timeout_ns, 11)) {
            ok = false;
            break;
          }
          const uint32_t full_even = map_to_cta(full_bar + 8 * stage, 0);
          if (cta == 0) mbar_arrive_expect_tx(full_bar + 8 * stage, stage_tx);
#pragma unroll
          for (int at = 0; at < Cfg::kAtoms; ++at) {
            const int k0 = kb * BK + at * Cfg::kAtomK;
            const uint32_t a_dst = a_base + stage * Cfg::kABytes + at * Cfg::kAAtomBytes;
            const uint32_t b_dst = b_base + stage * Cfg::kBBytes + at * Cfg::kBAtomBytes;
            if (tr) {
              tma_load_3d_pair(a_dst, &tmap_r, full_even, k0, a_row, r);
              tma_load_3d_pair(b_dst, &tmap_l16, full_even, k0, b_row, r);
              continue;
            }
            tma_load_3d_pair(a_dst, &tmap_l, full_even, k0, a_row, r);
            if (n_cols == BN) {
              tma_load_3d_pair(b_dst, &tmap_r, full_even, k0, b_row, r);
            } else {
              for (int j = 0; j < half; j += 16)
                tma_load_3d_pair(b_dst + static_cast<uint32_t>(j) * Cfg::kAtomK * 2u, &tmap_r16, full_even,
                                 k0, b_row + j, r);
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && issued > 0) {
        // loads may still be landing in this CTA's shared memory: give them
        // time to finish (they complete on the even CTA's barrier, which this
        // CTA cannot wait on) before the CTA unwinds
        const uint64_t start = globaltimer_ns();
        while (globaltimer_ns() - start < 200000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (cta == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int t = pair; t < total_tiles && ok; t += pairs) {
        int r, tm, tn;
        bool tr;
        pair_tile_coords(q, t, r, tm, tn, tr);
        // M = 256, cta_group::2: N a multiple of 32 (16 columns from each CTA)
        const uint32_t idesc = idesc_kind_f16<kBf16>(
            Cfg::kTileM, static_cast<uint32_t>(tr ? 32 : tile_n_columns(q, tn, BN, 32)));
        if (!mbar_wait_bounded_cluster(tempty_bar + 8 * acc, acc_phase ^ 1u, abort, p.timeout_ns, 12)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait_bounded_cluster(full_bar + 8 * stage, phase, abort, p.timeout_ns, 13)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_base + stage * Cfg::kABytes;
          const uint32_t b_addr = b_base + stage * Cfg::kBBytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // 16-deep step kk: atom column kk / (kAtomK / 16), 32 bytes per step inside it
            constexpr int kSteps = Cfg::kAtomK / 16;
            const uint32_t a_off = (kk / kSteps) * Cfg::kAAtomBytes + (kk % kSteps) * 32;
            const uint32_t b_off = (kk / kSteps) * Cfg::kBAtomBytes + (kk % kSteps) * 32;
            tc_mma_f16_pair(d_tmem, smem_desc_k_sw128(a_addr + a_off),
                            smem_desc_k_sw128(b_addr + b_off), idesc,
                            (kb > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          tc_commit_pair_multicast(empty_bar + 8 * stage, 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair_multicast(tfull_bar + 8 * acc, 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        tc_commit_pair_multicast(drain_bar, 0x1);
        volatile int no_abort = 0;
        mbar_wait_bounded(drain_bar, 0, &no_abort, p.timeout_ns, 16);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row_in_tile = static_cast<int>(cta) * kGemmBM + quarter * 32 + lane;
    const uint32_t tempty_even = map_to_cta(tempty_bar, 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    int chunk = 0;  // kTmaStore: running count of this warp's staged blocks (buffer = chunk & 1)
    for (int t = pair; t < total_tiles; t += pairs) {
      int r, tm, tn;
      bool tr;
      pair_tile_coords(q, t, r, tm, tn, tr);
      int ready = 0;
      if (lane == 0)
        ready = mbar_wait_bounded_cluster(tfull_bar + 8 * acc, acc_phase, abort, p.timeout_ns, 14) ? 1 : 0;
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tm) * Cfg::kTileM + row_in_tile;
      uint16_t* prow = p.P + (static_cast<int64_t>(r) * p.plane_rows + row) * p.ldp;
      const uint32_t t_addr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (tr) {
        // transposed tail: this lane holds Rt row (P column) col for the 32 L
        // tail rows (TMEM columns); for each valid tail row the warp writes 32
        // consecutive columns of P
        uint32_t v[32];
        tc_ld_32x32b_x32(t_addr, v);
        tc_wait_ld();
        const int64_t col = static_cast<int64_t>(tm) * Cfg::kTileM + row_in_tile;
        if (col < p.bn) {
          uint16_t* pc = p.P + (static_cast<int64_t>(r) * p.plane_rows + rows_main) * p.ldp + col;
#pragma unroll
          for (int n = 0; n < 32; ++n)
            if (n < tail_rows)
              pc[n * p.ldp] = static_cast<uint16_t>(pack2_rn<kBf16>(__uint_as_float(v[n]), 0.0f) & 0xFFFFu);
        }
      }
      const int n_cols = tr ? 0 : tile_n_columns(q, tn, BN, 32);
#pragma unroll 1
      for (int c = 0; c < n_cols; c += 32) {
        uint32_t v[32];
        tc_ld_32x32b_x32(t_addr + c, v);
        tc_wait_ld();
        const int64_t col = static_cast<int64_t>(tn) * BN + c;
        if constexpr (Cfg::kTmaStore) {
          // this lane's row of a 32 x 32 FP16 block, 64-byte swizzled: 16-byte
          // chunk j of row l sits at l * 64 + ((j ^ ((l >> 1) & 3)) << 4), the
          // layout a SWIZZLE_64B tensor map reads (and conflict-free per 8 lanes)
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            w[e] = pack2_rn<kBf16>(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
          const uint32_t buf = store_base + static_cast<uint32_t>((quarter * 2 + (chunk & 1)) * Cfg::kStoreBufBytes);
          // the store issued from this buffer two blocks ago must have read it
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j)
            st_shared_v4(buf + static_cast<uint32_t>(lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)), w[4 * j],
                         w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          // rows past bm and columns past ldp fall outside the tensor map and are
          // not written; a block that lies wholly outside is not issued at all
          const int64_t row0 = static_cast<int64_t>(tm) * Cfg::kTileM + static_cast<int>(cta) * kGemmBM +
                               quarter * 32;
          if (lane == 0 && row0 < p.bm && col < p.ldp) {
            tma_store_3d(&tmap_p, buf, static_cast<int32_t>(col), static_cast<int32_t>(row0), r);
            bulk_commit_group();
          }
          ++chunk;
        } else {
          if (row < p.bm) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const int64_t c8 = col + g * 8;
              if (c8 + 8 <= p.ldp) {
                uint4 pk;
                uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  w[e] = pack2_rn<kBf16>(__uint_as_float(v[g * 8 + 2 * e]),
                                         __uint_as_float(v[g * 8 + 2 * e + 1]));
                *reinterpret_cast<uint4*>(prow + c8) = pk;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty_even + 8 * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // the staged blocks' stores must finish (reading shared memory and writing
    // P) before the CTA leaves
    if constexpr (Cfg::kTmaStore) {
      if (lane == 0) bulk_wait_group_all();
      __syncwarp();
    }
  }

  tc_fence_before();
  cluster_sync_all();  // nobody leaves while the pair may still touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace fmm
