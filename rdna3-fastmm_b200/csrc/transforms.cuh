// Block transforms (HBM-bound streaming kernels) for the reduced-rank linear.
//
// The scheme-specific arithmetic comes from generated/fmm_schemes.cuh; this
// file supplies the vector type it runs on, the block addressing with zero
// padding, and the stores.  Every kernel reads each source element once and
// writes each destination element once, with 8- or 16-byte vector accesses on
// the aligned fast path.
#pragma once

#include "fmm_common.cuh"

namespace fmm {

template <int N>
struct VecF {
  float v[N];
};

// One FP32 rounding per certificate operation, never contracted or
// reassociated.  Pairs of lanes go through sm_100's packed FP32 instructions
// (add/sub/mul.rn.f32x2: two independent IEEE single-precision operations,
// round to nearest even, denormals kept -- the same results as two scalar
// __fadd_rn / __fsub_rn / __fmul_rn), which halves the arithmetic issue of the
// transforms and reconstructs; an odd last lane uses the scalar intrinsic.
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack_f32x2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <int N, class Op2, class Op1>
__device__ __forceinline__ VecF<N> vbinary(const VecF<N>& a, const VecF<N>& b, Op2 op2, Op1 op1) {
  VecF<N> r;
#pragma unroll
  for (int i = 0; i + 1 < N; i += 2)
    unpack_f32x2(op2(pack_f32x2(a.v[i], a.v[i + 1]), pack_f32x2(b.v[i], b.v[i + 1])), r.v[i], r.v[i + 1]);
  if constexpr (N % 2 == 1) r.v[N - 1] = op1(a.v[N - 1], b.v[N - 1]);
  return r;
}

template <int N>
__device__ __forceinline__ VecF<N> vadd(const VecF<N>& a, const VecF<N>& b) {
  return vbinary<N>(a, b, [](uint64_t x, uint64_t y) { return add_f32x2(x, y); },
                    [](float x, float y) { return __fadd_rn(x, y); });
}
template <int N>
__device__ __forceinline__ VecF<N> vsub(const VecF<N>& a, const VecF<N>& b) {
  return vbinary<N>(a, b, [](uint64_t x, uint64_t y) { return sub_f32x2(x, y); },
                    [](float x, float y) { return __fsub_rn(x, y); });
}
// Unary minus as 0 - x: a zero operand yields +0, matching the reference's
// Triton kernels (they lower `-x` to a subtraction from zero).
template <int N>
__device__ __forceinline__ VecF<N> vneg(const VecF<N>& a) {
  VecF<N> zero;
#pragma unroll
  for (int i = 0; i < N; ++i) zero.v[i] = 0.0f;
  return vsub(zero, a);
}
// Scaling by a power of two (or a small dyadic): exact, so x/2 == x*0.5.
template <int N>
__device__ __forceinline__ VecF<N> vscale(const VecF<N>& a, float c) {
  VecF<N> cv;
#pragma unroll
  for (int i = 0; i < N; ++i) cv.v[i] = c;
  return vbinary<N>(a, cv, [](uint64_t x, uint64_t y) { return mul_f32x2(x, y); },
                    [](float x, float y) { return __fmul_rn(x, y); });
}

// The same operations lane by lane in scalar FP32 instructions, for circuits
// whose packed form needs more registers than a thread has: the rank-343
// input sides (64 inputs and ~240 gates a position).
template <int N>
struct VecFs {
  float v[N];
};
template <int N>
__device__ __forceinline__ VecFs<N> vadd(const VecFs<N>& a, const VecFs<N>& b) {
  VecFs<N> r;
#pragma unroll
  for (int i = 0; i < N; ++i) r.v[i] = __fadd_rn(a.v[i], b.v[i]);
  return r;
}
template <int N>
__device__ __forceinline__ VecFs<N> vsub(const VecFs<N>& a, const VecFs<N>& b) {
  VecFs<N> r;
#pragma unroll
  for (int i = 0; i < N; ++i) r.v[i] = __fsub_rn(a.v[i], b.v[i]);
  return r;
}
template <int N>
__device__ __forceinline__ VecFs<N> vneg(const VecFs<N>& a) {
  VecFs<N> r;
#pragma unroll
  for (int i = 0; i < N; ++i) r.v[i] = __fsub_rn(0.0f, a.v[i]);
  return r;
}
template <int N>
__device__ __forceinline__ VecFs<N> vscale(const VecFs<N>& a, float c) {
  VecFs<N> r;
#pragma unroll
  for (int i = 0; i < N; ++i) r.v[i] = __fmul_rn(a.v[i], c);
  return r;
}
template <int N>
__device__ __forceinline__ VecFs<N> to_scalar_math(const VecF<N>& a) {
  VecFs<N> r;
#pragma unroll
  for (int i = 0; i < N; ++i) r.v[i] = a.v[i];
  return r;
}
template <int N>
__device__ __forceinline__ VecF<N> to_packed_math(const VecFs<N>& a) {
  VecF<N> r;
#pragma unroll
  for (int i = 0; i < N; ++i) r.v[i] = a.v[i];
  return r;
}
// Programs with this many inputs run in scalar FP32 (see VecFs).
constexpr int kScalarMathInputs = 64;

template <int N>
struct VecIO;

template <>
struct VecIO<2> {
  using BF = unsigned int;  // 2 x bf16
  using H = unsigned int;   // 2 x fp16
};
template <>
struct VecIO<4> {
  using BF = uint2;   // 4 x bf16
  using H = uint2;    // 4 x fp16
};
template <>
struct VecIO<8> {
  using BF = uint4;
  using H = uint4;
};

template <int N>
__device__ __forceinline__ VecF<N> unpack_bf16(const typename VecIO<N>::BF& raw) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  VecF<N> r;
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    r.v[2 * i] = f.x;
    r.v[2 * i + 1] = f.y;
  }
  return r;
}

template <int N>
__device__ __forceinline__ VecF<N> unpack_half(const typename VecIO<N>::H& raw) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
  VecF<N> r;
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    float2 f = __half22float2(h[i]);
    r.v[2 * i] = f.x;
    r.v[2 * i + 1] = f.y;
  }
  return r;
}

// 16-bit element types of the operands: BF16 (kHalf = false) or FP16.
template <bool kHalf, int N>
__device__ __forceinline__ VecF<N> unpack_in(const typename VecIO<N>::BF& raw) {
  if constexpr (kHalf) {
    return unpack_half<N>(raw);
  } else {
    return unpack_bf16<N>(raw);
  }
}

template <int N>
__device__ __forceinline__ void store_half_vec(__half* p, const VecF<N>& x) {
  typename VecIO<N>::H raw;
  __half2* h = reinterpret_cast<__half2*>(&raw);
#pragma unroll
  for (int i = 0; i < N / 2; ++i) h[i] = __floats2half2_rn(x.v[2 * i], x.v[2 * i + 1]);
  *reinterpret_cast<typename VecIO<N>::H*>(p) = raw;
}

template <int N>
__device__ __forceinline__ void store_bf16_vec(__nv_bfloat16* p, const VecF<N>& x) {
  typename VecIO<N>::BF raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < N / 2; ++i) h[i] = __floats2bfloat162_rn(x.v[2 * i], x.v[2 * i + 1]);
  *reinterpret_cast<typename VecIO<N>::BF*>(p) = raw;
}

// Plane element type: FP16 (kBfPlanes = false) or BF16, round to nearest even.
template <bool kBfPlanes, int N>
__device__ __forceinline__ void store_plane_vec(uint16_t* p, const VecF<N>& x) {
  if constexpr (kBfPlanes) {
    store_bf16_vec<N>(reinterpret_cast<__nv_bfloat16*>(p), x);
  } else {
    store_half_vec<N>(reinterpret_cast<__half*>(p), x);
  }
}
template <bool kBfPlanes, int N>
__device__ __forceinline__ VecF<N> unpack_plane(const typename VecIO<N>::H& raw) {
  if constexpr (kBfPlanes) {
    return unpack_bf16<N>(raw);
  } else {
    return unpack_half<N>(raw);
  }
}

// Output element (BF16 or FP16), round to nearest even.
template <bool kHalf>
__device__ __forceinline__ uint16_t round_out(float x) {
  if constexpr (kHalf) {
    return __half_as_ushort(__float2half_rn(x));
  } else {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
}
template <bool kHalf>
__device__ __forceinline__ float widen_in(uint16_t bits) {
  if constexpr (kHalf) {
    return __half2float(__ushort_as_half(bits));
  } else {
    return __bfloat162float(__ushort_as_bfloat16(bits));
  }
}
template <bool kHalf, int N>
__device__ __forceinline__ void store_out_vec(uint16_t* p, const VecF<N>& x) {
  if constexpr (kHalf) {
    store_half_vec<N>(reinterpret_cast<__half*>(p), x);
  } else {
    store_bf16_vec<N>(reinterpret_cast<__nv_bfloat16*>(p), x);
  }
}

// ---------------------------------------------------------------------------
// Input-side transform: src [rows, cols] BF16 or FP16 (leading dim ld) is cut
// into S x S zero-padded blocks of [brows, bcols]; Prog combines them into
// Prog::kOutputs planes dst[o][brows][ldd], FP16 (or BF16 with kBfPlanes).
//
// kWeight = false: activation side, input q is block (q / S, q % S) of A.
// kWeight = true : weight side; the program's input q is block (q / S, q % S)
//                  of B = weight^T, which is block (q % S, q / S) of weight,
//                  and rows/cols here are weight's (N, K).  The planes come out
//                  as Rt[r][n][k], the K-major transpose of the reference's
//                  Rw[r][k][n], without any transposition in memory.
//
// Thread mapping: one thread per VEC consecutive plane columns of one plane
// row; consecutive threads take consecutive vectors, so every block load and
// plane store of a warp is one contiguous span.  All S*S source vectors are
// loaded (packed, 2 bytes per element) before any arithmetic, so each thread
// has every load in flight at once; the generated program then unpacks them
// as it needs them.  This memory-level parallelism is what keeps the rank-48/49
// transforms near HBM bandwidth.  Columns in [bcols, ldd) are padding and are
// written as zeros.
struct TransformArgs {
  const uint16_t* src;
  int64_t rows, cols, ld;
  uint16_t* dst;  // FP16 or BF16 plane elements
  int64_t brows, bcols, ldd;
  int vector_loads;
};

// Body shared by the single and the paired launch: `block` / `blocks` are the
// CTA index and count this transform owns.
template <class Prog, int S, int VEC, bool kWeight, bool kHalfIn, bool kBfPlanes>
__device__ __forceinline__ void block_transform_body(const TransformArgs& a, uint32_t block,
                                                     uint32_t blocks) {
  using Raw = typename VecIO<VEC>::BF;
  const uint16_t* __restrict__ src = a.src;
  uint16_t* __restrict__ dst = a.dst;
  const int64_t rows = a.rows, cols = a.cols, ld = a.ld;
  const int64_t brows = a.brows, bcols = a.bcols, ldd = a.ldd;
  const int vector_loads = a.vector_loads;
  const int64_t plane = brows * ldd;
  const uint32_t vecs_per_row = static_cast<uint32_t>(ldd / VEC);
  const uint32_t total = static_cast<uint32_t>(brows) * vecs_per_row;
  for (uint32_t idx = block * blockDim.x + threadIdx.x; idx < total; idx += blocks * blockDim.x) {
    const uint32_t i = idx / vecs_per_row;
    const int64_t j = static_cast<int64_t>(idx - i * vecs_per_row) * VEC;
    Raw raw[Prog::kInputs];
    // interior vectors (every source block in range, aligned source): one
    // test per thread, then S*S unconditional vector loads back to back
    const bool interior = vector_loads && (S - 1) * brows + i < rows && j + VEC <= bcols &&
                          (S - 1) * bcols + j + VEC <= cols;
    if (interior) {
#pragma unroll
      for (int q = 0; q < Prog::kInputs; ++q) {
        const int br = kWeight ? (q % S) : (q / S);
        const int bc = kWeight ? (q / S) : (q % S);
        raw[q] = __ldg(reinterpret_cast<const Raw*>(src + (br * brows + i) * ld + bc * bcols + j));
      }
    } else {
      // ragged edge or unaligned source: element loads with zero padding
#pragma unroll
      for (int q = 0; q < Prog::kInputs; ++q) {
        const int br = kWeight ? (q % S) : (q / S);
        const int bc = kWeight ? (q / S) : (q % S);
        const int64_t r = br * brows + i;
        const int64_t c0 = bc * bcols + j;
        uint16_t* e = reinterpret_cast<uint16_t*>(&raw[q]);
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          const bool ok = r < rows && j + k < bcols && c0 + k < cols;
          e[k] = ok ? src[r * ld + c0 + k] : uint16_t(0);  // +0 in both formats
        }
      }
    }
    if constexpr (Prog::kInputs >= kScalarMathInputs) {
      auto in = [&](int q) -> VecFs<VEC> { return to_scalar_math(unpack_in<kHalfIn, VEC>(raw[q])); };
      auto out = [&](int o, const VecFs<VEC>& x) {
        store_plane_vec<kBfPlanes, VEC>(dst + o * plane + static_cast<int64_t>(i) * ldd + j, to_packed_math(x));
      };
      Prog::template run<VecFs<VEC>>(in, out);
    } else {
      auto in = [&](int q) -> VecF<VEC> { return unpack_in<kHalfIn, VEC>(raw[q]); };
      auto out = [&](int o, const VecF<VEC>& x) {
        store_plane_vec<kBfPlanes, VEC>(dst + o * plane + static_cast<int64_t>(i) * ldd + j, x);
      };
      Prog::template run<VecF<VEC>>(in, out);
    }
  }
}

template <class Prog, int S, int VEC, bool kWeight, int THREADS = 256, int MIN_BLOCKS = 1,
          bool kHalfIn = false, bool kBfPlanes = false>
__global__ void __launch_bounds__(THREADS, MIN_BLOCKS) block_transform_kernel(const TransformArgs a) {
  block_transform_body<Prog, S, VEC, kWeight, kHalfIn, kBfPlanes>(a, blockIdx.x, gridDim.x);
}

// The activation-side and the weight-side transform of one dynamic linear in
// a single launch: CTAs [0, left_blocks) run the left transform, the rest the
// weight transform.  Both stream HBM; sharing a launch lets the small left
// transform's ramp and tail overlap the weight transform instead of
// serialising with it.
template <class Left, class Right, int S, int VEC, int THREADS, int MIN_BLOCKS, bool kHalfIn,
          bool kBfPlanes = false>
__global__ void __launch_bounds__(THREADS, MIN_BLOCKS) paired_transform_kernel(
    const TransformArgs left, const TransformArgs weight, uint32_t left_blocks) {
  if (blockIdx.x < left_blocks) {
    block_transform_body<Left, S, VEC, false, kHalfIn, kBfPlanes>(left, blockIdx.x, left_blocks);
  } else {
    block_transform_body<Right, S, VEC, true, kHalfIn, kBfPlanes>(weight, blockIdx.x - left_blocks,
                                                                  gridDim.x - left_blocks);
  }
}

// ---------------------------------------------------------------------------
// Output side: recombine one vector position (plane row i, columns j..j+VEC)
// of the R product planes into the S*S output blocks of C.  Output o is C
// block (o / S, o % S); bias[bc*bn + c] is added after the whole
// recombination, then rounded to nearest even (BF16 or FP16).  `raw` holds the
// R product vectors, already loaded.  Shared by the reconstruct kernel and the
// fused rank-7 epilogue of the leaf GEMM, so both round identically.
// Bias of one output vector, widened to FP32: one vector load when the
// vector is interior and the bias aligned (bit 1 of `vector_flags`), else
// element loads with zeros past the edges.
template <int VEC, bool kHalfOut>
__device__ __forceinline__ VecF<VEC> load_bias_vector(const uint16_t* __restrict__ bias, int64_t j,
                                                      int64_t c0, int64_t bn, int64_t N,
                                                      int vector_flags) {
  if ((vector_flags & 2) && j + VEC <= bn && c0 + VEC <= N)
    return unpack_in<kHalfOut, VEC>(__ldg(reinterpret_cast<const typename VecIO<VEC>::BF*>(bias + c0)));
  VecF<VEC> b;
#pragma unroll
  for (int e = 0; e < VEC; ++e)
    b.v[e] = (j + e < bn && c0 + e < N) ? widen_in<kHalfOut>(bias[c0 + e]) : 0.0f;
  return b;
}

// Store output o (C block (o / S, o % S)) of one vector position: optional
// bias, then one rounding to the output format; ragged edges element-wise.
// `vector_stores`: bit 0 = C rows allow vector stores, bit 1 = bias allows
// vector loads.
template <int S, int VEC, bool kHalfOut>
__device__ __forceinline__ void store_output_vector(int o, const VecF<VEC>& x, int64_t i, int64_t j,
                                                    int64_t bm, int64_t bn,
                                                    const uint16_t* __restrict__ bias,
                                                    uint16_t* __restrict__ C, int64_t M, int64_t N,
                                                    int64_t ldc, int vector_stores) {
  const int br = o / S, bc = o % S;
  const int64_t row = br * bm + i;
  if (row >= M) return;
  const int64_t c0 = bc * bn + j;
  VecF<VEC> y = x;
  if (bias != nullptr) y = vadd(x, load_bias_vector<VEC, kHalfOut>(bias, j, c0, bn, N, vector_stores));
  uint16_t* dst = C + row * ldc + c0;
  if ((vector_stores & 1) && j + VEC <= bn && c0 + VEC <= N) {
    store_out_vec<kHalfOut, VEC>(dst, y);
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e)
      if (j + e < bn && c0 + e < N) dst[e] = round_out<kHalfOut>(y.v[e]);
  }
}

template <class Prog, int S, int VEC, bool kHalfOut, bool kBfPlanes>
__device__ __forceinline__ void recombine_vector(const typename VecIO<VEC>::H (&raw)[Prog::kInputs],
                                                 int64_t i, int64_t j, int64_t bm, int64_t bn,
                                                 const uint16_t* __restrict__ bias,
                                                 uint16_t* __restrict__ C, int64_t M, int64_t N,
                                                 int64_t ldc, int vector_stores) {
  auto in = [&](int r) -> VecF<VEC> { return unpack_plane<kBfPlanes, VEC>(raw[r]); };
  // Interior vector: row i of every block row and this vector's columns in
  // every column block lie inside C (N <= S * bn, so they also lie inside the
  // block), stores are vector stores and a bias is read with vector loads.
  // Each output is then one store at a fixed offset from this position's
  // element of output block (0, 0), without store_output_vector's per-output
  // tests (same values, same rounding).
  const bool interior = (vector_stores & 1) && (bias == nullptr || (vector_stores & 2)) &&
                        i + (S - 1) * bm < M && (S - 1) * bn + j + VEC <= N;
  if (interior) {
    uint16_t* base = C + i * ldc + j;
    const int64_t row_step = bm * ldc;
    auto out = [&](int o, const VecF<VEC>& x) {
      const int br = o / S, bc = o % S;
      VecF<VEC> y = x;
      if (bias != nullptr)
        y = vadd(x, unpack_in<kHalfOut, VEC>(
                        __ldg(reinterpret_cast<const typename VecIO<VEC>::BF*>(bias + bc * bn + j))));
      store_out_vec<kHalfOut, VEC>(base + br * row_step + bc * bn, y);
    };
    Prog::template run<VecF<VEC>>(in, out);
  } else {
    auto out = [&](int o, const VecF<VEC>& x) {
      store_output_vector<S, VEC, kHalfOut>(o, x, i, j, bm, bn, bias, C, M, N, ldc, vector_stores);
    };
    Prog::template run<VecF<VEC>>(in, out);
  }
}

// Unfused reconstruct: P[r][bm][ldp] (FP16, or BF16 with kBfPlanes) -> C[M,N].
// All R product vectors are loaded before the arithmetic, as in the input
// side.  The rank-7 reconstruct; rank 48/49 use the TMA-staged form
// (reconstruct_staged.cuh) unless FMM_RECONSTRUCT_VARIANT=register.
template <class Prog, int S, int VEC, int THREADS = 256, int MIN_BLOCKS = 1, bool kHalfOut = false,
          bool kBfPlanes = false>
__global__ void __launch_bounds__(THREADS, MIN_BLOCKS) reconstruct_kernel(
    const uint16_t* __restrict__ P, int64_t bm, int64_t bn, int64_t ldp,
    const uint16_t* __restrict__ bias, uint16_t* __restrict__ C, int64_t M, int64_t N,
    int64_t ldc, int vector_stores) {
  using Raw = typename VecIO<VEC>::H;
  const int64_t plane = bm * ldp;
  const uint32_t vecs_per_row = static_cast<uint32_t>((bn + VEC - 1) / VEC);
  const uint32_t total = static_cast<uint32_t>(bm) * vecs_per_row;
  for (uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += gridDim.x * blockDim.x) {
    const uint32_t i = idx / vecs_per_row;
    const int64_t j = static_cast<int64_t>(idx - i * vecs_per_row) * VEC;
    Raw raw[Prog::kInputs];
#pragma unroll
    for (int r = 0; r < Prog::kInputs; ++r)
      raw[r] = __ldg(reinterpret_cast<const Raw*>(P + r * plane + static_cast<int64_t>(i) * ldp + j));
    recombine_vector<Prog, S, VEC, kHalfOut, kBfPlanes>(raw, i, j, bm, bn, bias, C, M, N, ldc,
                                                        vector_stores);
  }
}

// ---------------------------------------------------------------------------
// Reconstruct fused with the all-gather of a row-sharded linear: every output
// vector is stored into `n` copies of the gathered output at once -- this
// rank's own buffer and its peers' buffers mapped into this process (NVLink
// peer memory), each pointer already offset to this rank's first row.  The
// arithmetic and rounding are reconstruct_kernel's; only the store fans out,
// so the transfer over NVLink overlaps the recombination vector by vector and
// no separate collective runs.  A system-scope fence at the end orders the
// peer stores before whatever the caller uses to signal completion.
constexpr int kMaxGatherDests = 8;
struct GatherDests {
  uint16_t* p[kMaxGatherDests];
  int n;
};

template <int S, int VEC, bool kHalfOut>
__device__ __forceinline__ void store_output_vector_all(int o, const VecF<VEC>& x, int64_t i, int64_t j,
                                                        int64_t bm, int64_t bn,
                                                        const uint16_t* __restrict__ bias,
                                                        const GatherDests& dests, int64_t M, int64_t N,
                                                        int64_t ldc, int vector_stores) {
  const int br = o / S, bc = o % S;
  const int64_t row = br * bm + i;
  if (row >= M) return;
  const int64_t c0 = bc * bn + j;
  VecF<VEC> y = x;
  if (bias != nullptr) y = vadd(x, load_bias_vector<VEC, kHalfOut>(bias, j, c0, bn, N, vector_stores));
  const int64_t offset = row * ldc + c0;
  if ((vector_stores & 1) && j + VEC <= bn && c0 + VEC <= N) {
    for (int d = 0; d < dests.n; ++d) store_out_vec<kHalfOut, VEC>(dests.p[d] + offset, y);
  } else {
    for (int d = 0; d < dests.n; ++d) {
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        if (j + e < bn && c0 + e < N) dests.p[d][offset + e] = round_out<kHalfOut>(y.v[e]);
    }
  }
}

template <class Prog, int S, int VEC, int THREADS = 256, int MIN_BLOCKS = 1, bool kHalfOut = false,
          bool kBfPlanes = false>
__global__ void __launch_bounds__(THREADS, MIN_BLOCKS) reconstruct_gather_kernel(
    const uint16_t* __restrict__ P, int64_t bm, int64_t bn, int64_t ldp,
    const uint16_t* __restrict__ bias, const GatherDests dests, int64_t M, int64_t N, int64_t ldc,
    int vector_stores) {
  using Raw = typename VecIO<VEC>::H;
  const int64_t plane = bm * ldp;
  const uint32_t vecs_per_row = static_cast<uint32_t>((bn + VEC - 1) / VEC);
  const uint32_t total = static_cast<uint32_t>(bm) * vecs_per_row;
  for (uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += gridDim.x * blockDim.x) {
    const uint32_t i = idx / vecs_per_row;
    const int64_t j = static_cast<int64_t>(idx - i * vecs_per_row) * VEC;
    Raw raw[Prog::kInputs];
#pragma unroll
    for (int r = 0; r < Prog::kInputs; ++r)
      raw[r] = __ldg(reinterpret_cast<const Raw*>(P + r * plane + static_cast<int64_t>(i) * ldp + j));
    auto in = [&](int r) -> VecF<VEC> { return unpack_plane<kBfPlanes, VEC>(raw[r]); };
    auto out = [&](int o, const VecF<VEC>& x) {
      store_output_vector_all<S, VEC, kHalfOut>(o, x, i, j, bm, bn, bias, dests, M, N, ldc,
                                                vector_stores);
    };
    Prog::template run<VecF<VEC>>(in, out);
  }
  __threadfence_system();
}

// ---------------------------------------------------------------------------
// Right transform of a contiguous B[K, N] (the plain-mm API): the program's
// input q is block (q / S, q % S) of B and the planes come out K-major,
// Rt[r][n][k], so each block is transposed on the way.  A CTA owns TK x TN
// positions (k0.., n0..) inside the blocks.
//   load:    the S*S input tiles are read with lanes along n (each B row
//            segment is contiguous) and written to shared memory transposed,
//            tile[q][n][k], rows padded by 2 elements against bank conflicts;
//   compute: each thread takes VEC consecutive k at one n -- one vector read
//            per input from shared memory -- and stores VEC elements of every
//            output plane; the lanes of a warp cover TK / VEC consecutive
//            vectors of one n, so each plane store is one contiguous run of
//            2*TK bytes.
// Shared memory: S*S * TN * (TK + 2) * 2 bytes (dynamic).
template <int S, int TK, int TN>
struct KnTile {
  static constexpr int kQ = S * S;
  static constexpr int kPitch = TK + 2;
  static constexpr size_t kBytes = size_t(kQ) * TN * kPitch * 2;
};

template <class Prog, int S, bool kHalfIn, int TK, int TN, int VEC, int THREADS, int MIN_BLOCKS,
          bool kBfPlanes = false>
__global__ void __launch_bounds__(THREADS, MIN_BLOCKS) right_transform_kn_kernel(
    const uint16_t* __restrict__ B, int64_t K, int64_t N, int64_t ldb, uint16_t* __restrict__ dst,
    int64_t bk, int64_t bn, int64_t ldk, int vector_loads) {
  using T = KnTile<S, TK, TN>;
  static_assert(TN % 8 == 0, "16-byte source chunks");
  extern __shared__ uint16_t kn_tile[];  // [kQ][TN][kPitch]
  const int64_t k0 = static_cast<int64_t>(blockIdx.x) * TK;
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * TN;
  // 16-byte chunks of 8 consecutive n; a chunk whose source row is in range
  // and whose 8 columns all lie inside the block (and B) is one vector load,
  // anything else goes element by element with zero padding
  constexpr int kChunks = TN / 8;
  for (int idx = threadIdx.x; idx < T::kQ * TK * kChunks; idx += THREADS) {
    const int q = idx / (TK * kChunks);
    const int kk = (idx / kChunks) % TK;
    const int nn = (idx % kChunks) * 8;
    const int64_t k = k0 + kk, n = n0 + nn;
    const int64_t row = (q / S) * bk + k, col = (q % S) * bn + n;
    uint16_t* to = kn_tile + (q * TN + nn) * T::kPitch + kk;
    if (vector_loads && k < bk && row < K && n + 8 <= bn && col + 8 <= N) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(B + row * ldb + col));
      const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
      for (int t = 0; t < 8; ++t) to[t * T::kPitch] = e[t];
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const bool ok = k < bk && n + t < bn && row < K && col + t < N;
        to[t * T::kPitch] = ok ? B[row * ldb + col + t] : uint16_t(0);
      }
    }
  }
  __syncthreads();
  const int64_t plane = bn * ldk;
  constexpr int kVecs = TK / VEC;  // vectors along k per n
  using Raw = typename VecIO<VEC>::BF;
  for (int idx = threadIdx.x; idx < TN * kVecs; idx += THREADS) {
    const int nn = idx / kVecs;
    const int kk = (idx % kVecs) * VEC;
    const int64_t n = n0 + nn, k = k0 + kk;
    if (n >= bn || k >= ldk) continue;
    auto load = [&](int q) -> VecF<VEC> {
      Raw raw;
      uint16_t* e = reinterpret_cast<uint16_t*>(&raw);
      const uint16_t* src = kn_tile + (q * TN + nn) * T::kPitch + kk;
#pragma unroll
      for (int v = 0; v < VEC; ++v) e[v] = src[v];
      return unpack_in<kHalfIn, VEC>(raw);
    };
    auto store = [&](int o, const VecF<VEC>& x) {
      store_plane_vec<kBfPlanes, VEC>(dst + o * plane + n * ldk + k, x);
    };
    if constexpr (Prog::kInputs >= kScalarMathInputs) {
      auto in = [&](int q) -> VecFs<VEC> { return to_scalar_math(load(q)); };
      auto out = [&](int o, const VecFs<VEC>& x) { store(o, to_packed_math(x)); };
      Prog::template run<VecFs<VEC>>(in, out);
    } else {
      Prog::template run<VecF<VEC>>(load, store);
    }
  }
}

}  // namespace fmm
