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
// reconstruct_staged_gather_kernel (end of this file) is the same pipeline for
// the row-sharded linear: it writes each tile's output rows into several
// gather buffers at once with bulk async copies.
//
// Every mbarrier wait is bounded; on a timeout the roles unwind, the producer
// drains its in-flight copies, and the CTA returns.
#pragma once

#include "fmm_common.cuh"
#include "transforms.cuh"

namespace fmm {

template <class Prog, int STAGES, int TP = 256>
struct StagedReconstructConfig {
  static constexpr int kStages = STAGES;
  static constexpr int kR = Prog::kInputs;
  static constexpr int kTP = TP;  // positions per tile (TMA box along x, <= 256)
  static constexpr int kBoxTP = TP;  // one box a tile
  static constexpr int kBoxes = 1;
  static constexpr int kVec = 2;
  static constexpr int kComputeWarps = kTP / kVec / 32;
  static constexpr int kThreads = 32 * (kComputeWarps + 1);
  static constexpr uint32_t kTileBytes = uint32_t(kR) * kTP * 2;
  static constexpr uint32_t kBoxBytes = kTileBytes;
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

// Producer of both staged kernels (one thread): kBoxes TMA boxes {kBoxTP
// positions, 1 row, R planes} per tile (box b at b * kBoxBytes, positions
// j0 + b * kBoxTP) into a ring of STAGES slots.  On a timeout it drains the
// copies that may still be landing before the CTA exits.
template <class Cfg>
__device__ __forceinline__ void staged_produce(const CUtensorMap* tmap_p, int total_tiles, int tiles_per_row,
                                               uint32_t full_bar, uint32_t empty_bar, uint32_t tiles_base,
                                               volatile int* abort, uint64_t timeout_ns) {
  constexpr int STAGES = Cfg::kStages;
  int stage = 0;
  uint32_t phase = 0;
  int issued = 0;
  bool ok = true;
  for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
    const int i = t / tiles_per_row;
    const int j0 = (t - i * tiles_per_row) * Cfg::kTP;
    if (!mbar_wait_bounded(empty_bar + 8 * stage, phase ^ 1u, abort, timeout_ns, 21)) {
      ok = false;
      break;
    }
    mbar_arrive_expect_tx(full_bar + 8 * stage, Cfg::kTileBytes);
#pragma unroll
    for (int b = 0; b < Cfg::kBoxes; ++b)
      tma_load_3d(tiles_base + stage * Cfg::kTileBytes + b * Cfg::kBoxBytes, tmap_p, full_bar + 8 * stage,
                  j0 + b * Cfg::kBoxTP, i, 0);
    ++issued;
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1u;
    }
  }
  if (!ok) {
    int s = stage;
    uint32_t ph = phase;
    volatile int no_abort = 0;
    for (int n = 0; n < STAGES && n < issued; ++n) {
      if (--s < 0) {
        s = STAGES - 1;
        ph ^= 1u;
      }
      mbar_wait_bounded(full_bar + 8 * s, ph, &no_abort, timeout_ns, 23);
    }
  }
}

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
    if (lane == 0)
      staged_produce<Cfg>(&tmap_p, p.total_tiles, p.tiles_per_row, full_bar, empty_bar, tiles_base, abort,
                          p.timeout_ns);
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

// ---------------------------------------------------------------------------
// The staged reconstruct fused with the all-gather of a row-sharded linear.
// Producer and circuit are reconstruct_staged_kernel's; the outputs of a tile
// (S*S row segments of TP positions, each contiguous in C) are rounded into a
// shared-memory staging buffer, and then bulk async copies (cp.async.bulk
// shared -> global, no tensor map, no multicast) write every segment into
// every destination -- this rank's gather buffer and the peers' buffers mapped
// into this process -- one copy per (output, destination) pair, each issued by
// its own compute thread.  The TMA units move the bytes, so a few SMs keep
// NVLink busy while the others compute.  Two staging buffers alternate: a
// thread rewrites a buffer only after its copy from two tiles earlier has
// finished reading it (wait_group.read) and every compute thread has passed
// the barrier behind that wait.  The kernel ends once every copy has completed,
// with a system-scope fence.  The host runs it only when bn, N and ldc are
// multiples of 8 and the destinations 16-byte aligned, so each copy starts on
// a 16-byte boundary and moves a multiple of 16 bytes.  Values and rounding
// are the general store path's, so the gathered output is bit-identical to
// fmm_reconstruct's.  Shared memory is sized so that one CTA occupies an SM:
// the grid is the SM budget in force, and the SMs outside it stay whole for a
// leaf GEMM running beside it.
template <class Prog, int STAGES, int TP = 512>
struct StagedGatherConfig {
  static constexpr int kStages = STAGES;
  static constexpr int kR = Prog::kInputs;
  static constexpr int kTP = TP;       // positions per tile
  static constexpr int kBoxTP = 256;   // positions per TMA box
  static constexpr int kBoxes = TP / kBoxTP;
  static constexpr int kVec = 2;
  static constexpr int kComputeWarps = kTP / kVec / 32;
  static constexpr int kThreads = 32 * (kComputeWarps + 1);
  static constexpr uint32_t kBoxBytes = uint32_t(kR) * kBoxTP * 2;
  static constexpr uint32_t kTileBytes = kBoxes * kBoxBytes;
  static constexpr uint32_t kOutBufBytes = uint32_t(Prog::kOutputs) * TP * 2;
  // tiles, two staging buffers, then the barrier block
  static constexpr size_t kSmemBytes = size_t(STAGES) * kTileBytes + 2 * kOutBufBytes + 16 * STAGES + 16;
  static_assert(TP % kBoxTP == 0, "whole boxes per tile");
  static_assert(Prog::kOutputs * kMaxGatherDests <= kComputeWarps * 32,
                "one copy per (output, destination) pair and compute thread");
  static_assert(2 * kSmemBytes > 228 * 1024, "one CTA per SM");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
};

template <class Prog, int S, int STAGES, bool kHalfOut, int TP = 512, bool kBfPlanes = false>
__global__ void __launch_bounds__(StagedGatherConfig<Prog, STAGES, TP>::kThreads, 1)
    reconstruct_staged_gather_kernel(const __grid_constant__ CUtensorMap tmap_p,
                                     const StagedReconstructParams p, const GatherDests dests) {
  using Cfg = StagedGatherConfig<Prog, STAGES, TP>;
  constexpr int kOut = Prog::kOutputs;
  constexpr int kComputeThreads = Cfg::kComputeWarps * 32;
  extern __shared__ __align__(128) uint8_t gather_smem[];
  const uint16_t* tiles = reinterpret_cast<const uint16_t*>(gather_smem);
  const uint32_t tiles_base = smem_u32(gather_smem);
  const uint32_t out_base = tiles_base + STAGES * Cfg::kTileBytes;  // [2][kOut][TP] elements
  uint64_t* bars = reinterpret_cast<uint64_t*>(gather_smem + size_t(STAGES) * Cfg::kTileBytes + 2 * Cfg::kOutBufBytes);
  const uint32_t full_bar = smem_u32(bars);
  const uint32_t empty_bar = smem_u32(bars + STAGES);
  volatile int* abort = reinterpret_cast<volatile int*>(bars + 2 * STAGES);
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
    if (lane == 0)
      staged_produce<Cfg>(&tmap_p, p.total_tiles, p.tiles_per_row, full_bar, empty_bar, tiles_base, abort,
                          p.timeout_ns);
    return;
  }

  // ------------------------------------------------------------ compute + copies
  const int ct = threadIdx.x;            // compute thread
  const int pos = ct * Cfg::kVec;        // position within the tile
  const int my_out = ct % kOut;          // the (output, destination) pair whose copy this thread issues
  uint16_t* my_dest = ct / kOut < dests.n ? dests.p[ct / kOut] : nullptr;
  int stage = 0;
  uint32_t phase = 0;
  int n = 0;  // tiles done: staging buffer n & 1
  for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++n) {
    const int64_t i = t / p.tiles_per_row;
    const int64_t j0 = (t - i * p.tiles_per_row) * Cfg::kTP;
    const int64_t j = j0 + pos;
    const bool ready = mbar_wait_bounded(full_bar + 8 * stage, phase, abort, p.timeout_ns, 24);
    // this thread's copy from two tiles ago has read the buffer about to be
    // rewritten; the barrier makes that true for every thread, and all compute
    // threads leave together if a wait gave up
    bulk_wait_group_read<1>();
    if (!named_barrier_and(1, kComputeThreads, ready)) break;
    const uint32_t buf = out_base + static_cast<uint32_t>(n & 1) * Cfg::kOutBufBytes;
    if (j < p.bn) {
      // this thread's box and its position inside the box
      const uint16_t* box = tiles + size_t(stage) * Cfg::kTileBytes / 2 +
                            size_t(pos / Cfg::kBoxTP) * Cfg::kBoxBytes / 2 + pos % Cfg::kBoxTP;
      auto in = [&](int r) -> VecF<2> {
        return unpack_plane<kBfPlanes, 2>(*reinterpret_cast<const unsigned*>(box + r * Cfg::kBoxTP));
      };
      auto out = [&](int o, const VecF<2>& x) {
        VecF<2> y = x;
        if (p.bias != nullptr)
          y = vadd(x, load_bias_vector<2, kHalfOut>(p.bias, j, (o % S) * p.bn + j, p.bn, p.N, p.vector_flags));
        st_shared_b32(buf + static_cast<uint32_t>((o * Cfg::kTP + pos) * 2), pack2_rn<!kHalfOut>(y.v[0], y.v[1]));
      };
      Prog::template run<VecF<2>>(in, out);
    }
    fence_proxy_async_smem();
    named_barrier_sync(1, kComputeThreads);
    if (lane == 0) mbar_arrive(empty_bar + 8 * stage);  // the product tile is consumed
    if (my_dest != nullptr) {
      const int64_t row = (my_out / S) * p.bm + i;
      const int64_t c0 = (my_out % S) * p.bn + j0;
      int64_t cols = p.bn - j0;
      if (p.N - c0 < cols) cols = p.N - c0;
      if (Cfg::kTP < cols) cols = Cfg::kTP;
      if (row < p.M && cols > 0)
        bulk_store_global(my_dest + row * p.ldc + c0, buf + static_cast<uint32_t>(my_out * Cfg::kTP * 2),
                          static_cast<uint32_t>(cols * 2));
    }
    bulk_commit_group();
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1u;
    }
  }
  // every copy complete (its writes performed) before the fence and the exit
  bulk_wait_group_all();
  __threadfence_system();
}

}  // namespace fmm
