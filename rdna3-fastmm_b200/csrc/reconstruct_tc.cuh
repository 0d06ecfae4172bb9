// Output side of the rank-343 <8,8,8> scheme on the tensor cores.
//
// For every plane position p (row i, column j of the 8 x 8 output blocks),
//   C[block o](p) = sum_r W[o][r] * P[r](p),   W: 64 x 343, entries -1/0/+1,
// which for a tile of 128 consecutive positions is the product
//   D[128 x 64] = P_tile[128 x 343] * W^T[343 x 64]
// -- the reference's MFMA reconstruction (generated/rank343_8x8x8.py
// output_transform_mfma_kernel), here with tcgen05.mma kind::f16 into tensor
// memory.  P's planes are position-contiguous, so the A operand is MN-major:
// each K-block of 64 products arrives as two TMA boxes {64 positions, 1 row,
// 64 products} (128-byte swizzle), i.e. two 64-position atoms 8 KiB apart
// (LBO) with 8-product groups 1 KiB apart (SBO).  Products past 343 and
// positions past the row pitch are zero-filled by TMA.  W^T (FP16, K-major,
// 64 x 384 zero-padded) is loaded once per CTA.
//
// Structure (one persistent CTA per SM, as the leaf GEMM):
//   warp 0      TMA producer (coefficients once, then STAGES-deep ring of P)
//   warp 1      MMA issuer: 4 x m128n64k16 per K-block, 6 K-blocks per tile,
//               two 64-column accumulators so epilogue and main loop overlap
//   warps 2..5  epilogue: tcgen05.ld, optional bias, one rounding to the
//               output format, transposed through shared memory into 16-byte
//               runs along each of the 64 output blocks.
// Every wait is bounded; on a timeout all roles unwind and TMEM is freed.
#pragma once

#include "fmm_common.cuh"
#include "transforms.cuh"

namespace fmm {

constexpr int kRcM = 128;       // positions per tile
constexpr int kRcN = 64;        // output blocks
constexpr int kRcK = 64;        // products per K-block
constexpr int kRcRank = 343;
constexpr int kRcKBlocks = (kRcRank + kRcK - 1) / kRcK;  // 6
constexpr int kRcKPadded = kRcKBlocks * kRcK;            // 384
constexpr int kRcThreads = 192;

template <int STAGES>
struct ReconstructTcConfig {
  static constexpr int kStages = STAGES;
  static constexpr uint32_t kBoxBytes = 64 * kRcK * 2;           // 8 KiB: 64 positions x 64 products
  static constexpr uint32_t kABytes = 2 * kBoxBytes;              // one K-block of a 128-position tile
  static constexpr uint32_t kBBytes = kRcN * kRcK * 2;            // 8 KiB of W^T per K-block
  static constexpr uint32_t kCoefBytes = kRcKBlocks * kBBytes;    // 48 KiB, resident
  static constexpr uint32_t kTmemCols = 2 * kRcN;                 // 128
  static constexpr uint32_t kOutBytes = kRcM * kRcN * 2;          // 16 KiB epilogue transpose
  static constexpr size_t kSmemBytes =
      size_t(STAGES) * kABytes + kCoefBytes + kOutBytes + 1024 + 256;
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

struct ReconstructTcParams {
  int64_t bm, bn;
  int64_t M, N, ldc;
  int32_t tiles_per_row;
  int32_t total_tiles;
  int32_t vector_stores;  // bn, ldc multiples of 8 and C 16-byte aligned
  const uint16_t* bias;
  uint16_t* C;
  uint64_t timeout_ns;
};

template <class Cfg, bool kHalfOut>
__global__ void __launch_bounds__(kRcThreads, 1)
    reconstruct_tc_kernel(const __grid_constant__ CUtensorMap tmap_p,
                          const __grid_constant__ CUtensorMap tmap_w, const ReconstructTcParams p) {
  constexpr int STAGES = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t a_base = base;
  const uint32_t w_base = base + STAGES * Cfg::kABytes;
  uint16_t* out_stage = reinterpret_cast<uint16_t*>(smem + STAGES * Cfg::kABytes + Cfg::kCoefBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::kABytes + Cfg::kCoefBytes +
                                               Cfg::kOutBytes);
  const uint32_t full_bar = smem_u32(bars);                     // [STAGES]
  const uint32_t empty_bar = smem_u32(bars + STAGES);           // [STAGES]
  const uint32_t tfull_bar = smem_u32(bars + 2 * STAGES);       // [2]
  const uint32_t tempty_bar = smem_u32(bars + 2 * STAGES + 2);  // [2]
  const uint32_t coef_bar = smem_u32(bars + 2 * STAGES + 4);
  const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 5);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 6);
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
      mbar_init(tempty_bar + 8 * b, 4);
    }
    mbar_init(coef_bar, 1);
    mbar_init(drain_bar, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmap_p);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(coef_bar, Cfg::kCoefBytes);
      for (int kb = 0; kb < kRcKBlocks; ++kb)
        tma_load_3d(w_base + kb * Cfg::kBBytes, &tmap_w, coef_bar, kb * kRcK, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
        const int i = t / p.tiles_per_row;
        const int j0 = (t - i * p.tiles_per_row) * kRcM;
        for (int kb = 0; kb < kRcKBlocks; ++kb) {
          if (!mbar_wait_bounded(empty_bar + 8 * stage, phase ^ 1u, abort, p.timeout_ns, 11)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar + 8 * stage, Cfg::kABytes);
          const uint32_t dst = a_base + stage * Cfg::kABytes;
          tma_load_3d(dst, &tmap_p, full_bar + 8 * stage, j0, i, kb * kRcK);
          tma_load_3d(dst + Cfg::kBoxBytes, &tmap_p, full_bar + 8 * stage, j0 + 64, i, kb * kRcK);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // drain what may still be landing (the coefficient block and, after an
      // abort, the last min(STAGES, issued) stages)
      volatile int no_abort = 0;
      mbar_wait_bounded(coef_bar, 0, &no_abort, p.timeout_ns, 15);
      if (!ok) {
        int s = stage;
        uint32_t ph = phase;
        for (int n = 0; n < STAGES && n < issued; ++n) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1u;
          }
          mbar_wait_bounded(full_bar + 8 * s, ph, &no_abort, p.timeout_ns, 15);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32_a_mn(kRcM, kRcN);
      bool ok = mbar_wait_bounded(coef_bar, 0, abort, p.timeout_ns, 12);
      if (ok) tc_fence_after();
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued_any = false;
      for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
        if (!mbar_wait_bounded(tempty_bar + 8 * acc, acc_phase ^ 1u, abort, p.timeout_ns, 13)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kRcN);
        for (int kb = 0; kb < kRcKBlocks; ++kb) {
          if (!mbar_wait_bounded(full_bar + 8 * stage, phase, abort, p.timeout_ns, 14)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_base + stage * Cfg::kABytes;
          const uint32_t w_addr = w_base + kb * Cfg::kBBytes;
#pragma unroll
          for (int kk = 0; kk < kRcK / 16; ++kk) {
            // 16 products = two 8-product groups (1 KiB each) of both atoms
            const uint64_t a_desc = smem_desc_mn_sw128(a_addr + kk * 2048, Cfg::kBoxBytes, 1024);
            const uint64_t b_desc = smem_desc_k_sw128(w_addr + kk * 32);
            tc_mma_f16(d_tmem, a_desc, b_desc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          tc_commit(empty_bar + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(tfull_bar + 8 * acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        tc_commit(drain_bar);
        volatile int no_abort = 0;
        mbar_wait_bounded(drain_bar, 0, &no_abort, p.timeout_ns, 16);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Each warp owns 32 positions (its TMEM lane quarter).  The 64 outputs of
    // a position are rounded in registers, written to this warp's 4 KiB slab
    // of shared memory as [output][position], and stored back to C as 16-byte
    // runs of 8 positions (4 lanes per output block), 8 store instructions
    // per warp per tile instead of 64 two-byte ones.
    const int quarter = warp & 3;
    uint16_t* slab = out_stage + quarter * 32 * kRcN;  // [64 outputs][32 positions]
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      const int64_t i = t / p.tiles_per_row;
      const int64_t j_base = (t - i * p.tiles_per_row) * kRcM + quarter * 32;
      const int64_t j = j_base + lane;
      int ready = 0;
      if (lane == 0)
        ready = mbar_wait_bounded(tfull_bar + 8 * acc, acc_phase, abort, p.timeout_ns, 17) ? 1 : 0;
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready) break;
      tc_fence_after();
      const uint32_t t_addr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * kRcN);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t v[32];
        tc_ld_32x32b_x32(t_addr + half * 32, v);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int o = half * 32 + c;  // output block (o / 8, o % 8)
          float y = __uint_as_float(v[c]);
          if (p.bias != nullptr) {
            const int64_t col = (o % 8) * p.bn + j;
            y = __fadd_rn(y, (j < p.bn && col < p.N) ? widen_in<kHalfOut>(p.bias[col]) : 0.0f);
          }
          slab[o * 32 + lane] = round_out<kHalfOut>(y);
        }
      }
      // the accumulator is in registers/shared memory now: hand it back
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar + 8 * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
      // lane l stores positions [8 (l % 4), +8) of output blocks l / 4 + 8 s
      const int chunk = lane & 3;
      const int64_t jc = j_base + chunk * 8;
#pragma unroll
      for (int step = 0; step < kRcN / 8; ++step) {
        const int o = step * 8 + (lane >> 2);
        const int64_t row = (o / 8) * p.bm + i;
        const int64_t col = (o % 8) * p.bn + jc;
        const uint16_t* src = slab + o * 32 + chunk * 8;
        if (row < p.M) {
          uint16_t* dst = p.C + row * p.ldc + col;
          if (p.vector_stores && jc + 8 <= p.bn && col + 8 <= p.N) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (jc + e < p.bn && col + e < p.N) dst[e] = src[e];
          }
        }
      }
      __syncwarp();  // the slab is rewritten by the next tile
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace fmm
