// C ABI of libfmm_sm100.so: argument checking, launch geometry, TMA tensor
// maps, and the per-scheme dispatch of the generated transforms.
//
// Nothing here allocates device memory or synchronises the stream (except
// fmm_device_status, whose job is to synchronise and read the status word).

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "fmm_common.cuh"
#include "transforms.cuh"
#include "generated/fmm_schemes.cuh"
#include "leaf_gemm.cuh"
#include "reconstruct_tc.cuh"
#include "reconstruct_staged.cuh"

// Scratch of fmm_linear_noalloc: the L, Rt and P planes of one call live in
// this array instead of caller-provided buffers.  It is part of the module, so
// every GPU that loads this library holds it until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FMM_NOALLOC_SCRATCH_BYTES];

namespace fmm {

namespace {

thread_local std::string t_last_error;
uint64_t g_timeout_ns = 2000000000ull;  // 2 s per wait
int g_sm_budget = 0;                     // 0: every SM; else the most SMs one launch may fill

int fail(int code, const std::string& what) {
  t_last_error = what;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(FMM_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

bool aligned(const void* p, size_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

int scheme_size(int scheme) {
  switch (scheme) {
    case FMM_SCHEME_RANK7: return 2;
    case FMM_SCHEME_RANK48: return 4;
    case FMM_SCHEME_RANK49: return 4;
    case FMM_SCHEME_RANK343: return 8;
    default: return 0;
  }
}

int dims_for(int scheme, int64_t M, int64_t K, int64_t N, fmm_dims* d) {
  const int s = scheme_size(scheme);
  if (s == 0) return fail(FMM_ERR_UNSUPPORTED, "unknown scheme id " + std::to_string(scheme));
  if (M < 1 || K < 1 || N < 1) return fail(FMM_ERR_INVALID_ARGUMENT, "matrix dimensions must be positive");
  d->scheme_size = s;
  d->rank = scheme;
  d->bm = ceil_div(M, s);
  d->bk = ceil_div(K, s);
  d->bn = ceil_div(N, s);
  d->ldk = round_up(d->bk, 8);
  d->ldp = round_up(d->bn, 8);
  d->left_elements = d->rank * d->bm * d->ldk;
  d->right_elements = d->rank * d->bn * d->ldk;
  d->product_elements = d->rank * d->bm * d->ldp;
  // 32-bit per-plane vector indices in the streaming kernels; TMA coordinates
  if (d->bm * d->ldk > (int64_t(1) << 31) || d->bn * d->ldk > (int64_t(1) << 31) ||
      d->bm * d->ldp > (int64_t(1) << 31) || d->bm > (int64_t(1) << 30) ||
      d->bn > (int64_t(1) << 30))
    return fail(FMM_ERR_TOO_LARGE, "transform planes exceed 2^31 elements");
  return FMM_OK;
}

struct DeviceInfo {
  int sm_count = 0;
  bool gemm_configured = false;
  bool pair256_configured = false;
  bool pair128_configured = false;
  bool pair192_configured = false;
  bool pair256k128_configured = false;
  void* noalloc_scratch = nullptr;  // device address of g_noalloc_scratch
  void* rank343_wt = nullptr;       // device address of g_rank343_wt, once uploaded
  bool reconstruct_tc_configured = false;
};

constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::mutex g_device_mutex;

int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FMM_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_device_mutex);
  DeviceInfo& info = g_devices[dev];
  if (info.sm_count == 0) {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    if (major != 10 || minor != 0)
      return fail(FMM_ERR_UNSUPPORTED, "libfmm_sm100 needs an sm_100 (B200) device; found sm_" +
                                           std::to_string(major) + std::to_string(minor));
    info.sm_count = sms;
  }
  *out = &info;
  return FMM_OK;
}

// SMs a launch may fill: all of them, or the budget set by fmm_set_sm_budget
// (kept even so that SM pairs of the 2-SM GEMM stay whole).
int usable_sms(const DeviceInfo* info) {
  int sms = info->sm_count;
  if (g_sm_budget > 0 && g_sm_budget < sms) sms = g_sm_budget & ~1;
  return sms < 2 ? 2 : sms;
}

// ------------------------------------------------------------------ dispatch
// Launch shapes were swept on B200 with random data (threads per block,
// minimum resident blocks, grid cap in blocks per SM); with every input
// preloaded these reach 91-98 % of the measured copy bandwidth.  The K x N
// right transform (plain-mm API) was swept separately: small 32 (k) x 8 (n)
// tiles with two k per thread and many resident blocks won for every scheme
// (16384^2: rank 7 4.8, rank 48/49 4.2, rank 343 2.4 TB/s).  The rank-48/49
// reconstruct runs TMA-staged (kOutStages > 0): timed right after the leaf
// GEMM that writes its products, 2 stages of 256 positions and 4 CTAs per SM
// beat the register kernel by 12-25 % (3 stages x 2 CTAs, fewer compute warps
// per SM, lost to it; 128-position tiles and single stages were slower).
template <int SCHEME>
struct SchemeTraits;
template <>
struct SchemeTraits<FMM_SCHEME_RANK7> {
  using Left = gen::Rank7Left;
  using Right = gen::Rank7Right;
  using Output = gen::Rank7Output;
  static constexpr int S = 2;
  static constexpr int VEC = 8;
  static constexpr int kInThreads = 256, kInBlocks = 1, kInGrid = 64;
  static constexpr int kOutVec = 8, kOutThreads = 128, kOutBlocks = 4, kOutGrid = 64;
  static constexpr int kOutStages = 0;
  static constexpr bool kTensorCoreOutput = false;
  static constexpr int kKnTK = 32, kKnTN = 8, kKnVec = 2, kKnThreads = 128, kKnBlocks = 4;
};
template <>
struct SchemeTraits<FMM_SCHEME_RANK48> {
  using Left = gen::Rank48Left;
  using Right = gen::Rank48Right;
  using Output = gen::Rank48Output;
  static constexpr int S = 4;
  static constexpr int VEC = 4;
  static constexpr int kInThreads = 128, kInBlocks = 4, kInGrid = 64;
  static constexpr int kOutVec = 4, kOutThreads = 128, kOutBlocks = 3, kOutGrid = 16;
  static constexpr int kOutStages = 2, kOutStagedBlocks = 4;
  static constexpr bool kTensorCoreOutput = false;
  static constexpr int kKnTK = 32, kKnTN = 8, kKnVec = 2, kKnThreads = 128, kKnBlocks = 4;
};
template <>
struct SchemeTraits<FMM_SCHEME_RANK49> {
  using Left = gen::Rank49Left;
  using Right = gen::Rank49Right;
  using Output = gen::Rank49Output;
  static constexpr int S = 4;
  static constexpr int VEC = 4;
  static constexpr int kInThreads = 128, kInBlocks = 4, kInGrid = 64;
  static constexpr int kOutVec = 4, kOutThreads = 128, kOutBlocks = 3, kOutGrid = 64;
  static constexpr int kOutStages = 2, kOutStagedBlocks = 4;
  static constexpr bool kTensorCoreOutput = false;
  static constexpr int kKnTK = 32, kKnTN = 8, kKnVec = 2, kKnThreads = 128, kKnBlocks = 4;
};
// Rank 343: 64 inputs and 343 planes per position.  The input side keeps two
// elements per thread (64 packed inputs plus the circuit fit in registers);
// the output side is a tensor-core product with the coefficient matrix
// (reconstruct_tc.cuh).
template <>
struct SchemeTraits<FMM_SCHEME_RANK343> {
  using Left = gen::Rank343Left;
  using Right = gen::Rank343Right;
  using Output = gen::Rank343OutputCoefficients;
  static constexpr int S = 8;
  static constexpr int VEC = 2;
  static constexpr int kInThreads = 128, kInBlocks = 1, kInGrid = 16;
  static constexpr bool kTensorCoreOutput = true;
  static constexpr int kKnTK = 32, kKnTN = 8, kKnVec = 2, kKnThreads = 128, kKnBlocks = 1;
};

int streaming_grid(const DeviceInfo* info, int64_t work_items, int threads, int blocks_per_sm) {
  const int64_t blocks = ceil_div(work_items, threads);
  const int64_t cap = int64_t(usable_sms(info)) * blocks_per_sm;
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

template <int SCHEME>
TransformArgs transform_args(const void* src, int64_t rows, int64_t cols, int64_t ld, void* dst,
                             int64_t brows, int64_t bcols, int64_t ldd) {
  using T = SchemeTraits<SCHEME>;
  const bool vec = (bcols % T::VEC == 0) && (ld % T::VEC == 0) && aligned(src, 2 * T::VEC);
  TransformArgs a;
  a.src = static_cast<const uint16_t*>(src);
  a.rows = rows;
  a.cols = cols;
  a.ld = ld;
  a.dst = static_cast<uint16_t*>(dst);
  a.brows = brows;
  a.bcols = bcols;
  a.ldd = ldd;
  a.vector_loads = vec ? 1 : 0;
  return a;
}

// Precision of one launch (the dtype argument of the C ABI): operand and
// output elements FP16 or BF16, plane elements BF16 only for
// FMM_DTYPE_BF16_BF16 (FP16 otherwise).
template <int PREC>
struct Precision {
  static constexpr bool kHalf = PREC == FMM_DTYPE_F16;
  static constexpr bool kBfPlanes = PREC == FMM_DTYPE_BF16_BF16;
};

template <int SCHEME, bool kWeight, int PREC>
int launch_input_transform(const void* src, int64_t rows, int64_t cols, int64_t ld, void* dst,
                           int64_t brows, int64_t bcols, int64_t ldd, cudaStream_t stream) {
  using T = SchemeTraits<SCHEME>;
  constexpr bool kHalf = Precision<PREC>::kHalf, kBf = Precision<PREC>::kBfPlanes;
  DeviceInfo* info = nullptr;
  if (int rc = device_info(&info)) return rc;
  const TransformArgs a = transform_args<SCHEME>(src, rows, cols, ld, dst, brows, bcols, ldd);
  const int64_t items = brows * (ldd / T::VEC);
  using Prog = typename std::conditional<kWeight, typename T::Right, typename T::Left>::type;
  block_transform_kernel<Prog, T::S, T::VEC, kWeight, T::kInThreads, T::kInBlocks, kHalf, kBf>
      <<<streaming_grid(info, items, T::kInThreads, T::kInGrid), T::kInThreads, 0, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, kWeight ? "weight transform launch" : "left transform launch");
  return FMM_OK;
}

// Left and weight transform of a dynamic linear in one launch; each gets a
// share of the CTAs proportional to its vectors (at least one).
template <int SCHEME, int PREC>
int launch_paired_transform(const void* A, int64_t M, int64_t K, int64_t lda, void* L, const void* W,
                            int64_t N, int64_t ldw, void* Rt, const fmm_dims& d, cudaStream_t stream) {
  using T = SchemeTraits<SCHEME>;
  constexpr bool kHalf = Precision<PREC>::kHalf, kBf = Precision<PREC>::kBfPlanes;
  DeviceInfo* info = nullptr;
  if (int rc = device_info(&info)) return rc;
  const TransformArgs left = transform_args<SCHEME>(A, M, K, lda, L, d.bm, d.bk, d.ldk);
  const TransformArgs weight = transform_args<SCHEME>(W, N, K, ldw, Rt, d.bn, d.bk, d.ldk);
  const int64_t left_items = d.bm * (d.ldk / T::VEC);
  const int64_t weight_items = d.bn * (d.ldk / T::VEC);
  int total = streaming_grid(info, left_items + weight_items, T::kInThreads, T::kInGrid);
  if (total < 2) total = 2;
  int64_t left_blocks = (int64_t(total) * left_items) / (left_items + weight_items);
  if (left_blocks < 1) left_blocks = 1;
  if (left_blocks > total - 1) left_blocks = total - 1;
  paired_transform_kernel<typename T::Left, typename T::Right, T::S, T::VEC, T::kInThreads,
                          T::kInBlocks, kHalf, kBf>
      <<<total, T::kInThreads, 0, stream>>>(left, weight, static_cast<uint32_t>(left_blocks));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "paired transform launch");
  return FMM_OK;
}

template <class Coefs, bool kHalf>
int launch_reconstruct_tc(const void* P, const fmm_dims& d, int64_t M, int64_t N, const void* bias,
                          void* C, int64_t ldc, DeviceInfo* info, cudaStream_t stream);

template <int SCHEME, int PREC>
int launch_reconstruct_staged(const void* P, const fmm_dims& d, int64_t M, int64_t N, const void* bias,
                              void* C, int64_t ldc, DeviceInfo* info, cudaStream_t stream);

template <int SCHEME, int PREC>
int launch_reconstruct_staged_gather(const void* P, const fmm_dims& d, int64_t M, int64_t N, const void* bias,
                                     const GatherDests& dests, int64_t ldc, DeviceInfo* info,
                                     cudaStream_t stream);

// FMM_RECONSTRUCT_VARIANT=register keeps the circuit schemes on the register
// reconstruct (the TMA-staged one is the default where a scheme has stages).
bool staged_reconstruct_enabled() {
  const char* v = std::getenv("FMM_RECONSTRUCT_VARIANT");
  return v == nullptr || std::string(v) != "register";
}

template <int SCHEME, int PREC>
int launch_reconstruct(const void* P, const fmm_dims& d, int64_t M, int64_t N, const void* bias,
                       void* C, int64_t ldc, cudaStream_t stream) {
  using T = SchemeTraits<SCHEME>;
  constexpr bool kHalf = Precision<PREC>::kHalf, kBf = Precision<PREC>::kBfPlanes;
  DeviceInfo* info = nullptr;
  if (int rc = device_info(&info)) return rc;
  if constexpr (T::kTensorCoreOutput) {
    return launch_reconstruct_tc<typename T::Output, kHalf>(P, d, M, N, bias, C, ldc, info, stream);
  } else {
    if constexpr (T::kOutStages > 0) {
      if (staged_reconstruct_enabled() && aligned(P, 16) && d.ldp % 8 == 0)
        return launch_reconstruct_staged<SCHEME, PREC>(P, d, M, N, bias, C, ldc, info, stream);
    }
    constexpr int V = T::kOutVec;
    const bool vec = (d.bn % V == 0) && (ldc % V == 0) && aligned(C, 2 * V);
    const bool vec_bias = (d.bn % V == 0) && bias != nullptr && aligned(bias, 2 * V);
    const int64_t items = d.bm * ceil_div(d.bn, V);
    const int grid = streaming_grid(info, items, T::kOutThreads, T::kOutGrid);
    reconstruct_kernel<typename T::Output, T::S, V, T::kOutThreads, T::kOutBlocks, kHalf, kBf>
        <<<grid, T::kOutThreads, 0, stream>>>(
            static_cast<const uint16_t*>(P), d.bm, d.bn, d.ldp, static_cast<const uint16_t*>(bias),
            static_cast<uint16_t*>(C), M, N, ldc, (vec ? 1 : 0) | (vec_bias ? 2 : 0));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "reconstruct launch");
    return FMM_OK;
  }
}

template <int SCHEME, int PREC>
int launch_reconstruct_gather(const void* P, const fmm_dims& d, int64_t M, int64_t N,
                              const void* bias, const GatherDests& dests, int64_t ldc,
                              cudaStream_t stream) {
  using T = SchemeTraits<SCHEME>;
  constexpr bool kHalf = Precision<PREC>::kHalf, kBf = Precision<PREC>::kBfPlanes;
  if constexpr (T::kTensorCoreOutput) {
    return fail(FMM_ERR_UNSUPPORTED, "the gathering reconstruct covers the circuit schemes (7, 48, 49)");
  } else {
    constexpr int V = T::kOutVec;
    DeviceInfo* info = nullptr;
    if (int rc = device_info(&info)) return rc;
    if constexpr (T::kOutStages > 0) {
      // staged tiles with bulk-copy stores: every output row segment starts on
      // a 16-byte boundary and moves a multiple of 16 bytes
      bool bulk = staged_reconstruct_enabled() && aligned(P, 16) && d.ldp % 8 == 0 && d.bn % 8 == 0 &&
                  N % 8 == 0 && ldc % 8 == 0;
      for (int k = 0; k < dests.n; ++k) bulk = bulk && aligned(dests.p[k], 16);
      if (bulk)
        return launch_reconstruct_staged_gather<SCHEME, PREC>(P, d, M, N, bias, dests, ldc, info, stream);
    }
    bool vec = (d.bn % V == 0) && (ldc % V == 0);
    for (int k = 0; k < dests.n; ++k) vec = vec && aligned(dests.p[k], 2 * V);
    const bool vec_bias = (d.bn % V == 0) && bias != nullptr && aligned(bias, 2 * V);
    const int64_t items = d.bm * ceil_div(d.bn, V);
    const int grid = streaming_grid(info, items, T::kOutThreads, T::kOutGrid);
    reconstruct_gather_kernel<typename T::Output, T::S, V, T::kOutThreads, T::kOutBlocks, kHalf, kBf>
        <<<grid, T::kOutThreads, 0, stream>>>(static_cast<const uint16_t*>(P), d.bm, d.bn, d.ldp,
                                              static_cast<const uint16_t*>(bias), dests, M, N, ldc,
                                              (vec ? 1 : 0) | (vec_bias ? 2 : 0));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "gathering reconstruct launch");
    return FMM_OK;
  }
}

template <class Kernel>
int ensure_smem_attribute(bool& done, Kernel kernel, size_t bytes);

template <int SCHEME, int PREC>
int launch_right_kn(const void* B, int64_t K, int64_t N, int64_t ldb, void* dst, const fmm_dims& d,
                    cudaStream_t stream) {
  using T = SchemeTraits<SCHEME>;
  constexpr bool kHalf = Precision<PREC>::kHalf, kBf = Precision<PREC>::kBfPlanes;
  constexpr int TK = T::kKnTK, TN = T::kKnTN;
  using Tile = KnTile<T::S, TK, TN>;
  auto kernel = right_transform_kn_kernel<typename T::Right, T::S, kHalf, TK, TN, T::kKnVec, T::kKnThreads,
                                           T::kKnBlocks, kBf>;
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (Tile::kBytes > 48 * 1024 && dev >= 0 && dev < kMaxDevices) {
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (int rc = ensure_smem_attribute(configured[dev], kernel, Tile::kBytes)) return rc;
  }
  const dim3 grid(static_cast<unsigned>(ceil_div(d.ldk, TK)), static_cast<unsigned>(ceil_div(d.bn, TN)));
  const bool vec = (ldb % 8 == 0) && (d.bn % 8 == 0) && aligned(B, 16);
  kernel<<<grid, T::kKnThreads, Tile::kBytes, stream>>>(static_cast<const uint16_t*>(B), K, N, ldb,
                                                        static_cast<uint16_t*>(dst), d.bk, d.bn, d.ldk,
                                                        vec ? 1 : 0);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "right transform (K x N) launch");
  return FMM_OK;
}

// Runtime (scheme, dtype) -> template instance.  BF16 planes exist for rank 49
// only, the one scheme whose reference plan offers them (Rank49Plan's
// (bfloat16, bfloat16) precision pair).
template <template <int, int> class F, class... Args>
int dispatch(int scheme, int dtype, Args... args) {
  const bool half = dtype == FMM_DTYPE_F16;
  if (dtype == FMM_DTYPE_BF16_BF16 && scheme != FMM_SCHEME_RANK49)
    return fail(FMM_ERR_UNSUPPORTED, "BF16 planes (FMM_DTYPE_BF16_BF16) are offered for rank 49 only");
  switch (scheme) {
    case FMM_SCHEME_RANK7:
      return half ? F<FMM_SCHEME_RANK7, FMM_DTYPE_F16>::run(args...)
                  : F<FMM_SCHEME_RANK7, FMM_DTYPE_BF16>::run(args...);
    case FMM_SCHEME_RANK48:
      return half ? F<FMM_SCHEME_RANK48, FMM_DTYPE_F16>::run(args...)
                  : F<FMM_SCHEME_RANK48, FMM_DTYPE_BF16>::run(args...);
    case FMM_SCHEME_RANK343:
      // FP16 inputs and output only, as the reference plan (precision_pairs)
      if (!half) return fail(FMM_ERR_UNSUPPORTED, "rank 343 takes FP16 operands only");
      return F<FMM_SCHEME_RANK343, FMM_DTYPE_F16>::run(args...);
    default:
      if (dtype == FMM_DTYPE_BF16_BF16) return F<FMM_SCHEME_RANK49, FMM_DTYPE_BF16_BF16>::run(args...);
      return half ? F<FMM_SCHEME_RANK49, FMM_DTYPE_F16>::run(args...)
                  : F<FMM_SCHEME_RANK49, FMM_DTYPE_BF16>::run(args...);
  }
}
template <int SC, int H>
struct LeftOp {
  static int run(const void* A, int64_t M, int64_t K, int64_t lda, void* L, const fmm_dims* d,
                 cudaStream_t s) {
    return launch_input_transform<SC, false, H>(A, M, K, lda, L, d->bm, d->bk, d->ldk, s);
  }
};
template <int SC, int H>
struct PairedOp {
  static int run(const void* A, int64_t M, int64_t K, int64_t lda, void* L, const void* W, int64_t N,
                 int64_t ldw, void* Rt, const fmm_dims* d, cudaStream_t s) {
    return launch_paired_transform<SC, H>(A, M, K, lda, L, W, N, ldw, Rt, *d, s);
  }
};
template <int SC, int H>
struct WeightOp {
  static int run(const void* W, int64_t N, int64_t K, int64_t ldw, void* Rt, const fmm_dims* d,
                 cudaStream_t s) {
    return launch_input_transform<SC, true, H>(W, N, K, ldw, Rt, d->bn, d->bk, d->ldk, s);
  }
};
template <int SC, int H>
struct RightKnOp {
  static int run(const void* B, int64_t K, int64_t N, int64_t ldb, void* Rt, const fmm_dims* d,
                 cudaStream_t s) {
    return launch_right_kn<SC, H>(B, K, N, ldb, Rt, *d, s);
  }
};
template <int SC, int H>
struct ReconstructGatherOp {
  static int run(const void* P, const fmm_dims* d, int64_t M, int64_t N, const void* bias,
                 const GatherDests* dests, int64_t ldc, cudaStream_t s) {
    return launch_reconstruct_gather<SC, H>(P, *d, M, N, bias, *dests, ldc, s);
  }
};
template <int SC, int H>
struct ReconstructOp {
  static int run(const void* P, const fmm_dims* d, int64_t M, int64_t N, const void* bias, void* C,
                 int64_t ldc, cudaStream_t s) {
    return launch_reconstruct<SC, H>(P, *d, M, N, bias, C, ldc, s);
  }
};

int check_dtype(int dtype) {
  if (dtype != FMM_DTYPE_BF16 && dtype != FMM_DTYPE_F16 && dtype != FMM_DTYPE_BF16_BF16)
    return fail(FMM_ERR_UNSUPPORTED,
                "dtype must be FMM_DTYPE_BF16, FMM_DTYPE_F16 or FMM_DTYPE_BF16_BF16");
  return FMM_OK;
}

// ------------------------------------------------------------------ TMA maps
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000* out) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return fail(FMM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  *out = g_encode;
  return FMM_OK;
}

// Stacked 16-bit planes [batch][plane_rows][pitch] as a 3-D map over (k, row,
// batch), covering the first `rows` rows of every plane (rows <= plane_rows;
// `base` may point into a plane to start the band further down); box = 64
// K-elements (128 B, swizzled) x box_rows rows x 1 plane.  TMA copies the
// 2-byte elements without conversion, so the FP16 map serves BF16 planes too.
int plane_map(CUtensorMap* map, const void* base, int64_t k, int64_t rows, int64_t pitch,
              int64_t batch, uint32_t box_rows, int64_t plane_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (int rc = tensor_map_encoder(&encode)) return rc;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(pitch * 2),
                           static_cast<cuuint64_t>(pitch * 2 * plane_rows)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kGemmBK), box_rows, 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims,
                      strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return FMM_OK;
}

// Generic 3-D FP16 tiled map (128-byte swizzle); strides in bytes.
int tiled_map_3d(CUtensorMap* map, const void* base, const int64_t (&dims)[3],
                 const int64_t (&strides)[2], const uint32_t (&box)[3],
                 CUtensorMapSwizzle swizzle) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (int rc = tensor_map_encoder(&encode)) return rc;
  cuuint64_t d[3] = {static_cast<cuuint64_t>(dims[0]), static_cast<cuuint64_t>(dims[1]),
                     static_cast<cuuint64_t>(dims[2])};
  cuuint64_t st[2] = {static_cast<cuuint64_t>(strides[0]), static_cast<cuuint64_t>(strides[1])};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), d, st, b,
                      elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return FMM_OK;
}

using GemmCfg = LeafGemmConfig<256, 4>;
using PairCfg256 = LeafGemmPairConfig<256, 7>;
using PairCfg192 = LeafGemmPairConfig<192, 7>;
using PairCfg128 = LeafGemmPairConfig<128, 8>;
using PairCfg256K128 = LeafGemmPairConfig<256, 3, 128>;
// the same two tiles with the TMA-store epilogue (one stage fewer for the
// epilogue's 16 KiB of shared-memory store buffers)
using PairCfg256Tma = LeafGemmPairConfig<256, 6, 64, true>;
using PairCfg256K128Tma = LeafGemmPairConfig<256, 3, 128, true>;
// narrower pair tiles with 128-deep k-blocks (TMA-store epilogue only): 3
// stages of 56 KiB at BN = 192, 4 of 48 KiB at BN = 128
using PairCfg192K128Tma = LeafGemmPairConfig<192, 3, 128, true>;
using PairCfg128K128Tma = LeafGemmPairConfig<128, 4, 128, true>;

enum GemmVariant {
  kVariantSingle = 0,
  kVariantPair256 = 1,
  kVariantPair128 = 2,
  kVariantPair192 = 3,
  kVariantPair256K128 = 4,  // 256x256 pair tile, 128-deep k-blocks in 3 stages
  kVariantPair192K128 = 5,  // 256x192 pair tile, 128-deep k-blocks in 3 stages
  kVariantPair128K128 = 6,  // 256x128 pair tile, 128-deep k-blocks in 4 stages
};

bool deep_k_variant(int variant) {
  return variant == kVariantPair256K128 || variant == kVariantPair192K128 || variant == kVariantPair128K128;
}

// Estimated relative cost of a variant: whole waves of full-tile equivalents
// over the SMs (or SM pairs), times the padded work one SM does per tile,
// divided by the variant's measured throughput relative to the 1-SM 128x256
// tile on B200 leaf shapes (a pair stages half of B per SM; 256x192 pairs
// measured 0.90 - 0.97 of one SM, 256x128 pairs slower still and only used
// when forced).  The ragged last N tile counts only the columns its MMA
// computes (the remainder rounded up to 16, or 32 for a pair).
double variant_cost(int variant, int64_t rank, int64_t bm, int64_t bn, int sms) {
  const bool pair = variant != kVariantSingle;
  const int64_t tm = pair ? 256 : 128;
  const int64_t tn = variant == kVariantPair128 ? 128 : (variant == kVariantPair192 ? 192 : 256);
  const int64_t granule = pair ? 32 : 16;
  const int64_t units = pair ? sms / 2 : sms;
  const double efficiency = variant == kVariantSingle    ? 1.0
                            : variant == kVariantPair256 ? 1.15
                            : variant == kVariantPair192 ? 0.95
                                                         : 0.70;
  const int64_t full_n = bn / tn;
  const int64_t last_cols = round_up(bn - full_n * tn, granule);
  const double n_tiles = double(full_n) + double(last_cols) / double(tn);
  const double waves = std::ceil(double(rank * ceil_div(bm, tm)) * n_tiles / double(units));
  return waves * double(tm * tn / (pair ? 2 : 1)) / efficiency;
}

int choose_variant(int64_t rank, int64_t bm, int64_t bn, int sms) {
  if (const char* forced = std::getenv("FMM_LEAF_GEMM_VARIANT")) {
    const std::string v(forced);
    if (v == "single") return kVariantSingle;
    if (v == "pair256") return kVariantPair256;
    if (v == "pair192") return kVariantPair192;
    if (v == "pair128") return kVariantPair128;
    if (v == "pair256k128") return kVariantPair256K128;
    if (v == "pair192k128") return kVariantPair192K128;
    if (v == "pair128k128") return kVariantPair128K128;
  }
  int best = kVariantSingle;
  double best_cost = variant_cost(kVariantSingle, rank, bm, bn, sms);
  for (int v : {kVariantPair256, kVariantPair192}) {
    const double c = variant_cost(v, rank, bm, bn, sms);
    if (c < best_cost) {
      best = v;
      best_cost = c;
    }
  }
  return best;
}

// Epilogue of the 256 x 256 pair GEMM: per-lane row stores, or shared-memory
// staged TMA stores (16 KiB of buffers).  The 128-deep configuration keeps its
// 3 stages either way and takes the TMA stores; the 64-deep one would lose one
// of its 7 stages and keeps the row stores.  FMM_LEAF_GEMM_EPILOGUE=rows|tma
// forces either.
bool tma_store_epilogue(int variant) {
  if (const char* v = std::getenv("FMM_LEAF_GEMM_EPILOGUE")) {
    if (std::string(v) == "tma") return true;
    if (std::string(v) == "rows") return false;
  }
  return deep_k_variant(variant);
}

template <class Kernel>
int ensure_smem_attribute(bool& done, Kernel kernel, size_t bytes) {
  if (done) return FMM_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(leaf GEMM)");
  done = true;
  return FMM_OK;
}

template <class Cfg, bool kBf16>
int launch_pair(const void* L, const void* Rt, const LeafGemmParams& prm, int64_t ldk, int sms,
                cudaStream_t stream) {
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FMM_ERR_UNSUPPORTED, "device index out of range");
  CUtensorMap map_l, map_r, map_r16;
  if (int rc = plane_map(&map_l, L, prm.bk, prm.bm, ldk, prm.rank, kGemmBM, prm.plane_rows)) return rc;
  if (int rc = plane_map(&map_r, Rt, prm.bk, prm.bn, ldk, prm.rank, Cfg::kBN / 2, prm.bn)) return rc;
  // 16-row boxes for the ragged last N tile's halves
  if (int rc = plane_map(&map_r16, Rt, prm.bk, prm.bn, ldk, prm.rank, 16, prm.bn)) return rc;
  // P[rank][bm][ldp] for the TMA-store epilogue: boxes of 32 columns x 32 rows,
  // 64-byte swizzle (unused by the row-store epilogue)
  // 16-row boxes of L for the transposed tail tiles' B operand (rows past bm
  // read as zeros)
  CUtensorMap map_l16 = map_l;
  if (prm.tail_rows > 0) {
    if (int rc = plane_map(&map_l16, L, prm.bk, prm.bm, ldk, prm.rank, 16, prm.plane_rows)) return rc;
  }
  CUtensorMap map_p = map_l;
  if constexpr (Cfg::kTmaStore) {
    if (int rc = tiled_map_3d(&map_p, prm.P, {prm.ldp, prm.bm, int64_t(prm.rank)},
                              {prm.ldp * 2, prm.plane_rows * prm.ldp * 2}, {32u, 32u, 1u},
                              CU_TENSOR_MAP_SWIZZLE_64B))
      return rc;
  }
  {
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (int rc = ensure_smem_attribute(configured[dev], leaf_gemm_pair_kernel<Cfg, kBf16>, Cfg::kSmemBytes))
      return rc;
  }
  const int64_t tiles =
      int64_t(prm.rank) * (ceil_div(prm.bm - prm.tail_rows, Cfg::kTileM) * ceil_div(prm.bn, Cfg::kBN) + prm.tail_tiles);
  const int64_t pairs = tiles < sms / 2 ? tiles : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, leaf_gemm_pair_kernel<Cfg, kBf16>, map_l, map_r, map_r16, map_p, map_l16, prm);
  if (e != cudaSuccess) return cuda_fail(e, "leaf GEMM (pair) launch");
  return FMM_OK;
}

// ------------------------------------------------------------------ rank-343 output
// W^T of the rank-343 scheme as FP16 [64 outputs][384 products] (+-1 / 0,
// zero past product 343): one copy per device in static device memory,
// uploaded on the first rank-343 reconstruct on that device.
static __device__ __align__(1024) uint16_t g_rank343_wt[kRcN * kRcKPadded];

using RcCfg = ReconstructTcConfig<6>;

template <class Coefs>
int upload_coefficients(DeviceInfo* info) {
  static_assert(Coefs::kOutputs == kRcN && Coefs::kInputs == kRcRank, "rank-343 coefficient table");
  std::lock_guard<std::mutex> lock(g_device_mutex);
  if (info->rank343_wt != nullptr) return FMM_OK;
  std::vector<uint16_t> host(size_t(kRcN) * kRcKPadded, 0);
  for (int o = 0; o < kRcN; ++o)
    for (int r = 0; r < kRcRank; ++r)
      host[size_t(o) * kRcKPadded + r] =
          Coefs::kW[o][r] > 0 ? uint16_t(0x3C00) : (Coefs::kW[o][r] < 0 ? uint16_t(0xBC00) : uint16_t(0));
  cudaError_t e = cudaMemcpyToSymbol(g_rank343_wt, host.data(), host.size() * sizeof(uint16_t));
  if (e != cudaSuccess) return cuda_fail(e, "upload of the rank-343 coefficients");
  void* addr = nullptr;
  e = cudaGetSymbolAddress(&addr, g_rank343_wt);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_rank343_wt)");
  info->rank343_wt = addr;
  return FMM_OK;
}

template <class Coefs, bool kHalf>
int launch_reconstruct_tc(const void* P, const fmm_dims& d, int64_t M, int64_t N, const void* bias,
                          void* C, int64_t ldc, DeviceInfo* info, cudaStream_t stream) {
  if (int rc = upload_coefficients<Coefs>(info)) return rc;
  CUtensorMap map_p, map_w;
  // P[343][bm][ldp] as (position, row, product); box 64 positions x 1 row x 64 products
  if (int rc = tiled_map_3d(&map_p, P, {d.ldp, d.bm, kRcRank}, {d.ldp * 2, d.bm * d.ldp * 2},
                            {64u, 1u, static_cast<uint32_t>(kRcK)}, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int rc = tiled_map_3d(&map_w, info->rank343_wt, {kRcKPadded, kRcN, 1},
                            {int64_t(kRcKPadded) * 2, int64_t(kRcKPadded) * kRcN * 2},
                            {static_cast<uint32_t>(kRcK), static_cast<uint32_t>(kRcN), 1u},
                            CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  {
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (int rc = ensure_smem_attribute(info->reconstruct_tc_configured,
                                       reconstruct_tc_kernel<RcCfg, kHalf>, RcCfg::kSmemBytes))
      return rc;
  }
  ReconstructTcParams prm;
  prm.bm = d.bm;
  prm.bn = d.bn;
  prm.M = M;
  prm.N = N;
  prm.ldc = ldc;
  const int64_t per_row = ceil_div(d.bn, kRcM);
  if (d.bm * per_row > 0x7fffffff) return fail(FMM_ERR_TOO_LARGE, "too many reconstruct tiles");
  prm.tiles_per_row = static_cast<int32_t>(per_row);
  prm.total_tiles = static_cast<int32_t>(d.bm * per_row);
  prm.vector_stores = (d.bn % 8 == 0 && ldc % 8 == 0 && aligned(C, 16)) ? 1 : 0;
  prm.bias = static_cast<const uint16_t*>(bias);
  prm.C = static_cast<uint16_t*>(C);
  prm.timeout_ns = g_timeout_ns;
  const int sms = usable_sms(info);
  const int grid = prm.total_tiles < sms ? prm.total_tiles : sms;
  reconstruct_tc_kernel<RcCfg, kHalf><<<grid, kRcThreads, RcCfg::kSmemBytes, stream>>>(map_p, map_w, prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rank-343 reconstruct launch");
  return FMM_OK;
}

// TMA-staged reconstruct of a circuit scheme: persistent CTAs, one box of
// 256 positions x R products per tile (unswizzled, so plane r of a tile sits at
// r * 256 elements in shared memory), two positions a compute thread.
template <int SCHEME, int PREC>
int launch_reconstruct_staged(const void* P, const fmm_dims& d, int64_t M, int64_t N, const void* bias,
                              void* C, int64_t ldc, DeviceInfo* info, cudaStream_t stream) {
  using T = SchemeTraits<SCHEME>;
  using Prog = typename T::Output;
  using Cfg = StagedReconstructConfig<Prog, T::kOutStages>;
  auto kernel = reconstruct_staged_kernel<Prog, T::S, T::kOutStages, Precision<PREC>::kHalf, Cfg::kTP,
                                          T::kOutStagedBlocks, Precision<PREC>::kBfPlanes>;
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FMM_ERR_UNSUPPORTED, "device index out of range");
  {
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (int rc = ensure_smem_attribute(configured[dev], kernel, Cfg::kSmemBytes)) return rc;
  }
  CUtensorMap map_p;
  if (int rc = tiled_map_3d(&map_p, P, {d.ldp, d.bm, int64_t(Cfg::kR)}, {d.ldp * 2, d.bm * d.ldp * 2},
                            {uint32_t(Cfg::kTP), 1u, uint32_t(Cfg::kR)}, CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  StagedReconstructParams prm;
  prm.bm = d.bm;
  prm.bn = d.bn;
  prm.M = M;
  prm.N = N;
  prm.ldc = ldc;
  const int64_t per_row = ceil_div(d.bn, Cfg::kTP);
  if (d.bm * per_row > 0x7fffffff) return fail(FMM_ERR_TOO_LARGE, "too many reconstruct tiles");
  prm.tiles_per_row = static_cast<int32_t>(per_row);
  prm.total_tiles = static_cast<int32_t>(d.bm * per_row);
  const bool vec = (d.bn % Cfg::kVec == 0) && (ldc % Cfg::kVec == 0) && aligned(C, 2 * Cfg::kVec);
  const bool vec_bias = (d.bn % Cfg::kVec == 0) && bias != nullptr && aligned(bias, 2 * Cfg::kVec);
  prm.vector_flags = (vec ? 1 : 0) | (vec_bias ? 2 : 0);
  prm.bias = static_cast<const uint16_t*>(bias);
  prm.C = static_cast<uint16_t*>(C);
  prm.timeout_ns = g_timeout_ns;
  const int64_t cap = int64_t(usable_sms(info)) * T::kOutStagedBlocks;
  const int grid = static_cast<int>(prm.total_tiles < cap ? prm.total_tiles : cap);
  kernel<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(map_p, prm);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "staged reconstruct launch");
  return FMM_OK;
}

// The staged reconstruct fused with the gather (bulk-copy stores into every
// destination): 512-position tiles (two TMA boxes) in 3 stages, 8 compute
// warps, one CTA per SM, the grid the SM budget in force (fmm_set_sm_budget),
// so a leaf GEMM launched beside it with the complementary budget keeps its
// SMs whole.
constexpr int kGatherStages = 3;

template <int SCHEME, int PREC>
int launch_reconstruct_staged_gather(const void* P, const fmm_dims& d, int64_t M, int64_t N, const void* bias,
                                     const GatherDests& dests, int64_t ldc, DeviceInfo* info,
                                     cudaStream_t stream) {
  using T = SchemeTraits<SCHEME>;
  using Prog = typename T::Output;
  using Cfg = StagedGatherConfig<Prog, kGatherStages>;
  auto kernel = reconstruct_staged_gather_kernel<Prog, T::S, kGatherStages, Precision<PREC>::kHalf, Cfg::kTP,
                                                 Precision<PREC>::kBfPlanes>;
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FMM_ERR_UNSUPPORTED, "device index out of range");
  {
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (int rc = ensure_smem_attribute(configured[dev], kernel, Cfg::kSmemBytes)) return rc;
  }
  CUtensorMap map_p;
  if (int rc = tiled_map_3d(&map_p, P, {d.ldp, d.bm, int64_t(Cfg::kR)}, {d.ldp * 2, d.bm * d.ldp * 2},
                            {uint32_t(Cfg::kBoxTP), 1u, uint32_t(Cfg::kR)}, CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  StagedReconstructParams prm;
  prm.bm = d.bm;
  prm.bn = d.bn;
  prm.M = M;
  prm.N = N;
  prm.ldc = ldc;
  const int64_t per_row = ceil_div(d.bn, Cfg::kTP);
  if (d.bm * per_row > 0x7fffffff) return fail(FMM_ERR_TOO_LARGE, "too many reconstruct tiles");
  prm.tiles_per_row = static_cast<int32_t>(per_row);
  prm.total_tiles = static_cast<int32_t>(d.bm * per_row);
  const bool vec_bias = (d.bn % Cfg::kVec == 0) && bias != nullptr && aligned(bias, 2 * Cfg::kVec);
  prm.vector_flags = vec_bias ? 2 : 0;  // bit 0 (vector stores into C) is unused: copies write C
  prm.bias = static_cast<const uint16_t*>(bias);
  prm.C = nullptr;
  prm.timeout_ns = g_timeout_ns;
  const int64_t cap = usable_sms(info);
  const int grid = static_cast<int>(prm.total_tiles < cap ? prm.total_tiles : cap);
  kernel<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(map_p, prm, dests);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "staged gathering reconstruct launch");
  return FMM_OK;
}

// The 1-SM GEMM (small or ragged leaves).
template <bool kBf16>
int launch_single(const void* L, const void* Rt, const LeafGemmParams& prm, int64_t ldk, int sms,
                  cudaStream_t stream) {
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FMM_ERR_UNSUPPORTED, "device index out of range");
  CUtensorMap map_l, map_r;
  if (int rc = plane_map(&map_l, L, prm.bk, prm.bm, ldk, prm.rank, kGemmBM, prm.plane_rows)) return rc;
  if (int rc = plane_map(&map_r, Rt, prm.bk, prm.bn, ldk, prm.rank, GemmCfg::kBN, prm.bn)) return rc;
  {
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (int rc = ensure_smem_attribute(configured[dev], leaf_gemm_kernel<GemmCfg, kBf16>, GemmCfg::kSmemBytes))
      return rc;
  }
  const int64_t tiles = int64_t(prm.rank) * prm.tiles_m * prm.tiles_n;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  leaf_gemm_kernel<GemmCfg, kBf16><<<grid, kGemmThreads, GemmCfg::kSmemBytes, stream>>>(map_l, map_r, prm);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "leaf GEMM launch");
  return FMM_OK;
}

// M-tiles per group of the tile order (a group sweeps all N-tiles of its
// M-tiles before the next group starts, so the group's L rows and the
// weight planes' N-tiles are reused from L2): 16, or FMM_LEAF_GEMM_GROUP_M.
int leaf_group_m() {
  if (const char* v = std::getenv("FMM_LEAF_GEMM_GROUP_M")) {
    const int g = std::atoi(v);
    if (g >= 1 && g <= 4096) return g;
  }
  return 16;
}

// Serpentine N order across tile groups (on; FMM_LEAF_GEMM_SERPENTINE=0 turns
// it off): a group starts on the weight-plane columns its predecessor used
// last, which cut the c5b launch's DRAM reads from 4.87 to 4.19 GB (ncu, one
// full-size launch); its time moved less than the run-to-run noise.
int leaf_serpentine() {
  const char* v = std::getenv("FMM_LEAF_GEMM_SERPENTINE");
  return (v != nullptr && std::string(v) == "0") ? 0 : 1;
}

// One GEMM launch over rows [row0, row0 + rows) of every plane (planes of
// `plane_rows` rows), with the given variant and epilogue.
template <bool kBf16>
int launch_leaf_band(int variant, bool tma_store, int rank, const uint16_t* L, const void* Rt,
                     int64_t row0, int64_t rows, int64_t plane_rows, int64_t bn, int64_t bk,
                     uint16_t* P, int sms, cudaStream_t stream, int64_t transposed_tail = 0) {
  const int64_t ldk = round_up(bk, 8), ldp = round_up(bn, 8);
  const uint16_t* band_l = L + row0 * ldk;
  LeafGemmParams prm;
  prm.bm = rows;
  prm.bn = bn;
  prm.bk = bk;
  prm.ldp = ldp;
  prm.plane_rows = plane_rows;
  prm.rank = rank;
  prm.tiles_m = static_cast<int32_t>(ceil_div(rows, kGemmBM));
  prm.tiles_n = static_cast<int32_t>(ceil_div(bn, GemmCfg::kBN));
  prm.group_m = leaf_group_m();
  prm.serpentine = leaf_serpentine();
  prm.tail_rows = static_cast<int32_t>(transposed_tail);
  prm.tail_tiles = transposed_tail > 0 ? static_cast<int32_t>(ceil_div(bn, 256)) : 0;
  prm.P = P + row0 * ldp;
  prm.timeout_ns = g_timeout_ns;
  if (variant == kVariantPair256) {
    return tma_store ? launch_pair<PairCfg256Tma, kBf16>(band_l, Rt, prm, ldk, sms, stream)
                     : launch_pair<PairCfg256, kBf16>(band_l, Rt, prm, ldk, sms, stream);
  }
  if (variant == kVariantPair256K128) {
    return tma_store ? launch_pair<PairCfg256K128Tma, kBf16>(band_l, Rt, prm, ldk, sms, stream)
                     : launch_pair<PairCfg256K128, kBf16>(band_l, Rt, prm, ldk, sms, stream);
  }
  // the narrow 128-deep configurations exist with the TMA-store epilogue only
  if (variant == kVariantPair192K128) return launch_pair<PairCfg192K128Tma, kBf16>(band_l, Rt, prm, ldk, sms, stream);
  if (variant == kVariantPair128K128) return launch_pair<PairCfg128K128Tma, kBf16>(band_l, Rt, prm, ldk, sms, stream);
  if constexpr (!kBf16) {
    if (variant == kVariantPair192) return launch_pair<PairCfg192, false>(band_l, Rt, prm, ldk, sms, stream);
    if (variant == kVariantPair128) return launch_pair<PairCfg128, false>(band_l, Rt, prm, ldk, sms, stream);
  }
  return launch_single<kBf16>(band_l, Rt, prm, ldk, sms, stream);
}

// Rows of a short last M tile of the 2-SM GEMM, run as a second, 1-SM launch
// of 128-row tiles over the planes' last rows (one SM instead of two for each
// of their tiles) when FMM_LEAF_GEMM_TAIL=1 and the planes' last 256-row tile
// holds at most 128 rows.  Off by default: on c4 (bm = 2054, a 6-row last
// tile) the two launches measured 0.7 % slower than one (0.591 vs 0.587 ms,
// GEMM alone, three interleaved rounds) -- the second launch's partial waves
// cost what the narrower tiles save.
int64_t split_tail_rows(int variant, int64_t bm) {
  if (variant == kVariantSingle) return 0;
  const int64_t tail = bm % 256;
  if (bm < 256 || tail == 0 || tail > 128) return 0;
  const char* v = std::getenv("FMM_LEAF_GEMM_TAIL");
  return (v != nullptr && std::string(v) == "1") ? tail : 0;
}

// Rows of a short last M tile (1..32 rows) that the 256 x 256 pair kernels
// compute transposed inside the same launch: P^T = Rt * L_tail^T in 256 x 32
// tiles over bn, an eighth of a regular tile's MMA work, instead of padding
// the rows to a whole 256-row tile (c4: bm = 2054, 6 rows).
// FMM_LEAF_GEMM_TAIL=0 pads them as before; =1 selects the 1-SM band above.
int64_t transposed_tail_rows(int variant, int64_t bm) {
  if (variant != kVariantPair256 && variant != kVariantPair256K128) return 0;
  const int64_t tail = bm % 256;
  if (bm < 256 || tail == 0 || tail > 32) return 0;
  const char* v = std::getenv("FMM_LEAF_GEMM_TAIL");
  if (v != nullptr && (std::string(v) == "0" || std::string(v) == "1")) return 0;
  return tail;
}

// FP16 planes (kBf16 = false) or BF16 planes.  The BF16 form carries the
// 1-SM configuration and every 128-deep pair configuration; a forced narrower
// 64-deep pair variant runs as the 256 x 256 pair there.
template <bool kBf16>
int launch_leaf_gemm(int rank, const void* L, const void* Rt, int64_t bm, int64_t bn, int64_t bk,
                     void* P, cudaStream_t stream) {
  if (rank < 1 || bm < 1 || bn < 1 || bk < 1)
    return fail(FMM_ERR_INVALID_ARGUMENT, "leaf GEMM dimensions must be positive");
  if (!aligned(L, 16) || !aligned(Rt, 16) || !aligned(P, 16))
    return fail(FMM_ERR_MISALIGNED, "leaf GEMM planes must be 16-byte aligned");
  DeviceInfo* info = nullptr;
  if (int rc = device_info(&info)) return rc;
  if (int64_t(rank) * ceil_div(bm, kGemmBM) * ceil_div(bn, 128) > (int64_t(1) << 30))
    return fail(FMM_ERR_TOO_LARGE, "too many GEMM tiles");
  const int sms = usable_sms(info);
  int variant = choose_variant(rank, bm, bn, sms);
  // 128-deep k-blocks with the TMA-store epilogue, from bk = 1024 up (at most
  // 6 % of the last k-block's MMA work is zero padding there): measured
  // against 64-deep k-blocks in 7 stages with row stores (GEMM alone, full
  // clock, L2 flushed, 3 interleaved rounds): c2 0.256 -> 0.240 ms, c5a
  // 0.594 -> 0.557, c5b 4.11-4.17 -> 3.95-4.09 (against 64-deep k-blocks with
  // the TMA stores there, the previous choice).  A forced
  // FMM_LEAF_GEMM_VARIANT keeps its own k-depth.
  if (bk >= 1024 && std::getenv("FMM_LEAF_GEMM_VARIANT") == nullptr) {
    if (variant == kVariantPair256) variant = kVariantPair256K128;
    if (variant == kVariantPair192) variant = kVariantPair192K128;
    if (variant == kVariantPair128) variant = kVariantPair128K128;
  }
  if (kBf16 && (variant == kVariantPair192 || variant == kVariantPair128)) variant = kVariantPair256;
  const bool tma_store = tma_store_epilogue(variant);
  const uint16_t* l16 = static_cast<const uint16_t*>(L);
  uint16_t* p16 = static_cast<uint16_t*>(P);
  const int64_t tail = split_tail_rows(variant, bm);
  const int64_t transposed = tail == 0 ? transposed_tail_rows(variant, bm) : 0;
  if (int rc = launch_leaf_band<kBf16>(variant, tma_store, rank, l16, Rt, 0, bm - tail, bm, bn, bk, p16, sms,
                                       stream, transposed))
    return rc;
  if (tail == 0) return FMM_OK;
  // the short last band: same stream, after the 2-SM launch
  return launch_leaf_band<kBf16>(kVariantSingle, false, rank, l16, Rt, bm - tail, tail, bm, bn, bk, p16, sms,
                                 stream);
}

// Device address of g_noalloc_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  DeviceInfo* info = nullptr;
  if (int rc = device_info(&info)) return rc;
  std::lock_guard<std::mutex> lock(g_device_mutex);
  if (info->noalloc_scratch == nullptr) {
    void* address = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&address, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    info->noalloc_scratch = address;
  }
  *out = info->noalloc_scratch;
  return FMM_OK;
}

__global__ void bounded_wait_probe_kernel(uint64_t timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // nothing ever arrives: the wait must give up after timeout_ns
    mbar_wait_bounded(smem_u32(&bar), 0, &abort_flag, timeout_ns, 7);
  }
  __syncthreads();
}

}  // namespace
}  // namespace fmm

using namespace fmm;

extern "C" {

int fmm_version(void) { return 100; }

const char* fmm_last_error_string(void) { return t_last_error.c_str(); }

int fmm_plan_dims(int scheme, int64_t M, int64_t K, int64_t N, fmm_dims* out) {
  if (out == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null output");
  return dims_for(scheme, M, K, N, out);
}

int fmm_transform_a(int scheme, int dtype, const void* A, int64_t M, int64_t K, int64_t lda,
                    void* L, fmm_stream_t stream) {
  fmm_dims d;
  if (int rc = dims_for(scheme, M, K, 1, &d)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (A == nullptr || L == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  if (lda < K) return fail(FMM_ERR_INVALID_ARGUMENT, "lda < K");
  if (!aligned(L, 16)) return fail(FMM_ERR_MISALIGNED, "L must be 16-byte aligned");
  return dispatch<LeftOp>(scheme, dtype, A, M, K, lda, L, &d, reinterpret_cast<cudaStream_t>(stream));
}

int fmm_transform_w(int scheme, int dtype, const void* W, int64_t N, int64_t K, int64_t ldw,
                    void* Rt, fmm_stream_t stream) {
  fmm_dims d;
  if (int rc = dims_for(scheme, 1, K, N, &d)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (W == nullptr || Rt == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldw < K) return fail(FMM_ERR_INVALID_ARGUMENT, "ldw < K");
  if (!aligned(Rt, 16)) return fail(FMM_ERR_MISALIGNED, "Rt must be 16-byte aligned");
  return dispatch<WeightOp>(scheme, dtype, W, N, K, ldw, Rt, &d, reinterpret_cast<cudaStream_t>(stream));
}

int fmm_transform_aw(int scheme, int dtype, const void* A, int64_t M, int64_t K, int64_t lda,
                     void* L, const void* W, int64_t N, int64_t ldw, void* Rt, fmm_stream_t stream) {
  fmm_dims d;
  if (int rc = dims_for(scheme, M, K, N, &d)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (A == nullptr || L == nullptr || W == nullptr || Rt == nullptr)
    return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  if (lda < K || ldw < K) return fail(FMM_ERR_INVALID_ARGUMENT, "lda or ldw < K");
  if (!aligned(L, 16) || !aligned(Rt, 16))
    return fail(FMM_ERR_MISALIGNED, "L and Rt must be 16-byte aligned");
  return dispatch<PairedOp>(scheme, dtype, A, M, K, lda, L, W, N, ldw, Rt, &d,
                            reinterpret_cast<cudaStream_t>(stream));
}

int fmm_transform_b(int scheme, int dtype, const void* B, int64_t K, int64_t N, int64_t ldb,
                    void* Rt, fmm_stream_t stream) {
  fmm_dims d;
  if (int rc = dims_for(scheme, 1, K, N, &d)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (B == nullptr || Rt == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldb < N) return fail(FMM_ERR_INVALID_ARGUMENT, "ldb < N");
  if (!aligned(Rt, 16)) return fail(FMM_ERR_MISALIGNED, "Rt must be 16-byte aligned");
  return dispatch<RightKnOp>(scheme, dtype, B, K, N, ldb, Rt, &d, reinterpret_cast<cudaStream_t>(stream));
}

int fmm_leaf_gemm(int rank, const void* L, const void* Rt, int64_t bm, int64_t bn, int64_t bk,
                  void* P, fmm_stream_t stream) {
  if (L == nullptr || Rt == nullptr || P == nullptr)
    return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  return launch_leaf_gemm<false>(rank, L, Rt, bm, bn, bk, P, reinterpret_cast<cudaStream_t>(stream));
}

int fmm_leaf_gemm_bf16(int rank, const void* L, const void* Rt, int64_t bm, int64_t bn, int64_t bk,
                       void* P, fmm_stream_t stream) {
  if (L == nullptr || Rt == nullptr || P == nullptr)
    return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  return launch_leaf_gemm<true>(rank, L, Rt, bm, bn, bk, P, reinterpret_cast<cudaStream_t>(stream));
}

int fmm_reconstruct(int scheme, int dtype, const void* P, int64_t M, int64_t N, const void* bias,
                    void* C, int64_t ldc, fmm_stream_t stream) {
  fmm_dims d;
  if (int rc = dims_for(scheme, M, 1, N, &d)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (P == nullptr || C == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  if (ldc < N) return fail(FMM_ERR_INVALID_ARGUMENT, "ldc < N");
  if (!aligned(P, 16)) return fail(FMM_ERR_MISALIGNED, "P must be 16-byte aligned");
  return dispatch<ReconstructOp>(scheme, dtype, P, &d, M, N, bias, C, ldc,
                                 reinterpret_cast<cudaStream_t>(stream));
}

int fmm_reconstruct_gather(int scheme, int dtype, const void* P, int64_t M, int64_t N,
                           const void* bias, void* const* dests, int ndest, int64_t ldc,
                           fmm_stream_t stream) {
  fmm_dims d;
  if (int rc = dims_for(scheme, M, 1, N, &d)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (P == nullptr || dests == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  if (ndest < 1 || ndest > kMaxGatherDests)
    return fail(FMM_ERR_INVALID_ARGUMENT, "ndest must be in [1, 8]");
  if (ldc < N) return fail(FMM_ERR_INVALID_ARGUMENT, "ldc < N");
  if (!aligned(P, 16)) return fail(FMM_ERR_MISALIGNED, "P must be 16-byte aligned");
  GatherDests list = {};
  list.n = ndest;
  for (int k = 0; k < ndest; ++k) {
    if (dests[k] == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null destination");
    list.p[k] = static_cast<uint16_t*>(dests[k]);
  }
  return dispatch<ReconstructGatherOp>(scheme, dtype, P, &d, M, N, bias, &list, ldc,
                                       reinterpret_cast<cudaStream_t>(stream));
}

int fmm_linear(int scheme, int dtype, const void* A, const void* W, const void* bias, void* C,
               int64_t M, int64_t K, int64_t N, void* L, void* Rt, void* P, unsigned int flags,
               fmm_stream_t stream) {
  fmm_dims d;
  if (int rc = dims_for(scheme, M, K, N, &d)) return rc;
  if (int rc = check_dtype(dtype)) return rc;
  if (A == nullptr || C == nullptr || L == nullptr || Rt == nullptr || P == nullptr)
    return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  const bool prepacked = (flags & FMM_LINEAR_PREPACKED) != 0;
  if (!prepacked && W == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null weight");
  if (!prepacked && !(flags & FMM_RIGHT_KN)) {
    // native [N, K] weight: both input-side transforms in one launch
    if (int rc = fmm_transform_aw(scheme, dtype, A, M, K, K, L, W, N, K, Rt, stream)) return rc;
  } else {
    if (int rc = fmm_transform_a(scheme, dtype, A, M, K, K, L, stream)) return rc;
    if (!prepacked) {
      if (int rc = fmm_transform_b(scheme, dtype, W, K, N, N, Rt, stream)) return rc;
    }
  }
  const int gemm = dtype == FMM_DTYPE_BF16_BF16
                       ? fmm_leaf_gemm_bf16(static_cast<int>(d.rank), L, Rt, d.bm, d.bn, d.bk, P, stream)
                       : fmm_leaf_gemm(static_cast<int>(d.rank), L, Rt, d.bm, d.bn, d.bk, P, stream);
  if (gemm != FMM_OK) return gemm;
  return fmm_reconstruct(scheme, dtype, P, M, N, bias, C, N, stream);
}

int fmm_linear_noalloc(int scheme, const void* A, const void* W, const void* bias, void* C,
                       int64_t M, int64_t K, int64_t N, fmm_stream_t stream) {
  // BF16 linears only: rank 343 takes FP16 operands, so it has no BF16 form to run here
  if (scheme != FMM_SCHEME_RANK7 && scheme != FMM_SCHEME_RANK48 && scheme != FMM_SCHEME_RANK49)
    return fail(FMM_ERR_UNSUPPORTED, "fmm_linear_noalloc: scheme " + std::to_string(scheme) +
                                         " is not a BF16 linear scheme (7, 48 or 49)");
  fmm_dims d;
  if (int rc = dims_for(scheme, M, K, N, &d)) return rc;
  if (A == nullptr || W == nullptr || C == nullptr)
    return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  const int64_t left = round_up(d.left_elements * 2, 256);
  const int64_t right = round_up(d.right_elements * 2, 256);
  const int64_t products = round_up(d.product_elements * 2, 256);
  const int64_t needed = left + right + products;
  if (needed > static_cast<int64_t>(FMM_NOALLOC_SCRATCH_BYTES))
    return fail(FMM_ERR_TOO_LARGE,
                "fmm_linear_noalloc: this shape needs " + std::to_string(needed) +
                    " bytes of scratch, more than its fixed " +
                    std::to_string(static_cast<long long>(FMM_NOALLOC_SCRATCH_BYTES)) +
                    "; use fmm_linear with caller-provided planes");
  void* base = nullptr;
  if (int rc = noalloc_scratch(&base)) return rc;
  unsigned char* bytes = static_cast<unsigned char*>(base);
  // Every plane element the GEMM and the reconstruct read is written earlier
  // in the same call (pitch padding included), so nothing is cleared first.
  return fmm_linear(scheme, FMM_DTYPE_BF16, A, W, bias, C, M, K, N, bytes, bytes + left,
                    bytes + left + right, 0u, stream);
}

// ------------------------------------------------------------------ peer memory (IPC)
static_assert(sizeof(cudaIpcMemHandle_t) == FMM_IPC_HANDLE_BYTES, "IPC handle size");

int fmm_ipc_export(const void* ptr, unsigned char* handle, uint64_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr)
    return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  static PFN_cuMemGetAddressRange_v3020 range = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 3020, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  if (range == nullptr) return fail(FMM_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(FMM_ERR_INVALID_ARGUMENT, "pointer is not device memory of this context");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return FMM_OK;
}

int fmm_ipc_import(const unsigned char* handle, uint64_t offset, void** base, void** ptr) {
  if (handle == nullptr || base == nullptr || ptr == nullptr)
    return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* mapped = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&mapped, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *base = mapped;
  *ptr = static_cast<unsigned char*>(mapped) + offset;
  return FMM_OK;
}

int fmm_ipc_close(void* base) {
  if (base == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return FMM_OK;
}

int fmm_copy_async(void* dst, const void* src, uint64_t bytes, fmm_stream_t stream) {
  if (dst == nullptr || src == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null pointer");
  if (bytes == 0) return FMM_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice,
                                  reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync (device to device)");
  return FMM_OK;
}

int fmm_set_sm_budget(int sms) {
  if (sms < 0) return fail(FMM_ERR_INVALID_ARGUMENT, "SM budget must be >= 0");
  g_sm_budget = sms;
  return FMM_OK;
}

int fmm_set_wait_timeout_ns(uint64_t timeout_ns) {
  if (timeout_ns == 0) return fail(FMM_ERR_INVALID_ARGUMENT, "timeout must be positive");
  g_timeout_ns = timeout_ns;
  return FMM_OK;
}

int fmm_device_status(int device, uint32_t* status, uint32_t* site, int reset) {
  if (status == nullptr) return fail(FMM_ERR_INVALID_ARGUMENT, "null status");
  int previous = 0;
  cudaError_t e = cudaGetDevice(&previous);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (device != previous && (e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  int rc = FMM_OK;
  unsigned int value = 0, where = 0;
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) rc = cuda_fail(e, "cudaDeviceSynchronize");
  if (rc == FMM_OK && (e = cudaMemcpyFromSymbol(&value, g_status, sizeof(value))) != cudaSuccess)
    rc = cuda_fail(e, "read status");
  if (rc == FMM_OK && (e = cudaMemcpyFromSymbol(&where, g_timeout_site, sizeof(where))) != cudaSuccess)
    rc = cuda_fail(e, "read timeout site");
  if (rc == FMM_OK && reset) {
    const unsigned int zero = 0;
    if ((e = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero))) != cudaSuccess ||
        (e = cudaMemcpyToSymbol(g_timeout_site, &zero, sizeof(zero))) != cudaSuccess)
      rc = cuda_fail(e, "clear status");
  }
  if (device != previous) cudaSetDevice(previous);
  *status = value;
  if (site != nullptr) *site = where;
  return rc;
}

int fmm_test_bounded_wait(uint64_t timeout_ns, fmm_stream_t stream) {
  if (timeout_ns == 0 || timeout_ns > 10000000000ull)
    return fail(FMM_ERR_INVALID_ARGUMENT, "probe timeout must be in (0, 10 s]");
  bounded_wait_probe_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(timeout_ns);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bounded wait probe launch");
  return FMM_OK;
}

}  // extern "C"
