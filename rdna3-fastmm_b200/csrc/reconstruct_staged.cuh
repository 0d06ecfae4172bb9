// Recombination of the circuit schemes (rank 7, 48, 49) with the product
// planes staged in shared memory by TMA.
//
// The register version (reconstruct_kernel) keeps all R product vectors of a
// position in registers before the circuit runs; for R = 48/49 that is 160+
// registers a thread, 3 resident blocks and about 0.65 of the copy peak.  Here
// one TMA box {TP positions, 1 row, R planes} brings a whole tile of products
// into shared memory per stage, a producer warp keeps STAGES tiles in flight,
// and TP / 64 compute warps evaluate the same generated circuit on two
// positions a thread, reading each product from shared memory when the circuit
// first needs it (under 100 registers, so several CTAs share an SM).  Product
// planes are FP16, or BF16 with kBfPlanes (TMA moves them as 2-byte elements
// either way).  The
// arithmetic, its order and the rounding are reconstruct_kernel's (the same
// Prog::run and store_output_vector), so the outputs are bit-identical.
//
// Every mbarrier wait is bounded; on a timeout the roles unwind, the producer
// drains its in-flight copies, and the CTA returns.
#pragma once

#include "fmm_common.cuh"
#include "transforms.cuh"

namespace fmm {

template <class Prog, int STAGES, int TP = 256>
struct StagedReconstructConfig {
  static constexpr int kR = Prog::kInputs;
  static constexpr int kTP = TP;  // positions per tile (TMA box along x, <= 256)
  static constexpr int kVec = 2;
  static constexpr int kComputeWarps = kTP / kVec / 32;
  static constexpr int kThreads = 32 * (kComputeWarps + 1);
  static constexpr uint32_t kTileBytes = uint32_t(kR) * kTP * 2;
  static constexpr size_t kSmemBytes = size_t(STAGES) * kTileBytes + 16 * STAGES + 16;
  static_assert(kR <= 256 && kTP <= 256 && kTP % 64 == 0, "one TMA box spans a tile");
};

struct StagedReconstructParams {
  int64_t bm, bn;
  int64_t M, N, ldc;
  int32_t tiles_per_row, total_tiles;
  int vector_flags;  // bit 0: vector stores into C, bit 1: vector bias loads
  const uint16_t* bias;
  uint16_t* C;
  uint64_t timeout_ns;
};

template <class Prog, int S, int STAGES, bool kHalfOut, int TP = 256, int MIN_BLOCKS = 1,
          bool kBfPlanes = false>
__global__ void __launch_bounds__(StagedReconstructConfig<Prog, STAGES, TP>::kThreads, MIN_BLOCKS)
    reconstruct_staged_kernel(const __grid_constant__ CUtensorMap tmap_p,
                              const StagedReconstructParams p) {
  using Cfg = StagedReconstructConfig<Prog, STAGES, TP>;
  extern __shared__ __align__(128) uint8_t staged_smem[];
  const uint16_t* tiles = reinterpret_cast<const uint16_t*>(staged_smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(staged_smem + size_t(STAGES) * Cfg::kTileBytes);
  const uint32_t full_bar = smem_u32(bars);             // [STAGES]
  const uint32_t empty_bar = smem_u32(bars + STAGES);   // [STAGES]
  volatile int* abort = reinterpret_cast<volatile int*>(bars + 2 * STAGES);
  const uint32_t tiles_base = smem_u32(staged_smem);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar + 8 * s, 1);
      mbar_init(empty_bar + 8 * s, Cfg::kComputeWarps);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmap_p);
  }
  __syncthreads();

  if (warp == Cfg::kComputeWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
        const int i = t / p.tiles_per_row;
        const int j0 = (t - i * p.tiles_per_row) * Cfg::kTP;
        if (!mbar_wait_bounded(empty_bar + 8 * stage, phase ^ 1u, abort, p.timeout_ns, 21)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(full_bar + 8 * stage, Cfg::kTileBytes);
        tma_load_3d(tiles_base + stage * Cfg::kTileBytes, &tmap_p, full_bar + 8 * stage, j0, i, 0);
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {
        // drain the copies that may still be landing before the CTA exits
        int s = stage;
        uint32_t ph = phase;
        volatile int no_abort = 0;
        for (int n = 0; n < STAGES && n < issued; ++n) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1u;
          }
          mbar_wait_bounded(full_bar + 8 * s, ph, &no_abort, p.timeout_ns, 23);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ compute
    int stage = 0;
    uint32_t phase = 0;
    const int pos = threadIdx.x * Cfg::kVec;  // position within the tile
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      const int64_t i = t / p.tiles_per_row;
      const int64_t j = (t - i * p.tiles_per_row) * Cfg::kTP + pos;
      // every lane waits (and so acquires the TMA's writes) itself
      const bool ready = mbar_wait_bounded(full_bar + 8 * stage, phase, abort, p.timeout_ns, 22);
      if (!__all_sync(0xffffffffu, ready)) break;
      const uint16_t* tile = tiles + size_t(stage) * Cfg::kR * Cfg::kTP;
      auto in = [&](int r) -> VecF<2> {
        return unpack_plane<kBfPlanes, 2>(*reinterpret_cast<const unsigned*>(tile + r * Cfg::kTP + pos));
      };
      // Interior tile (the same for every thread of the CTA): row i of every
      // block row lies inside C, every column block's span of the tile lies
      // inside C, 4-byte stores, no bias.  Each output is then one store
      // through one of S row pointers at a fixed column offset, without the
      // per-output bounds and alignment checks of the general path (same
      // values, same rounding).
      const int64_t j0 = j - pos;
      const bool interior = (p.vector_flags & 1) && p.bias == nullptr && i + (S - 1) * p.bm < p.M &&
                            (S - 1) * p.bn + j0 + Cfg::kTP <= p.N;
      if (interior) {
        uint16_t* rowp[S];
#pragma unroll
        for (int br = 0; br < S; ++br) rowp[br] = p.C + (br * p.bm + i) * p.ldc + j;
        auto out = [&](int o, const VecF<2>& x) {
          store_out_vec<kHalfOut, 2>(rowp[o / S] + (o % S) * p.bn, x);
        };
        Prog::template run<VecF<2>>(in, out);
      } else if (j < p.bn) {
        auto out = [&](int o, const VecF<2>& x) {
          store_output_vector<S, 2, kHalfOut>(o, x, i, j, p.bm, p.bn, p.bias, p.C, p.M, p.N, p.ldc,
                                              p.vector_flags);
        };
        Prog::template run<VecF<2>>(in, out);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar + 8 * stage);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
}

}  // namespace fmm
