/*
 * fmm_sm100.h -- C ABI of libfmm_sm100.so, the B200 (sm_100a) kernels behind
 * the rdna3_fastmm operator surface.
 *
 * The reference (chelokot/rdna3-fastmm) has no C layer: its plans launch
 * generated Triton kernels and torch.bmm directly from Python.  Each entry
 * point below replaces one of those launches; the citation names the
 * reference call it stands in for (paths are inside the reference project).
 *
 * Conventions for every entry point:
 *   - all pointers are caller-owned device pointers; nothing is allocated,
 *     freed, retained or synchronised (work is queued on `stream`);
 *   - BF16 tensors are row-major with the given leading dimension in
 *     elements; planes (FP16, or BF16 with FMM_DTYPE_BF16_BF16) are stacked
 *     [rank][rows][pitch] with
 *     pitch = round_up(cols, 8) elements (fmm_plan_dims), which keeps every
 *     row 16-byte aligned for TMA; plane buffers must be 16-byte aligned;
 *   - the return value is FMM_OK or an FMM_ERR_* code; fmm_last_error_string
 *     describes the last failure of the calling thread.
 *
 * Transformed planes use the layout [rank][rows][cols]:
 *   left  (activations)  L[r][bm][ldk]   -- as the reference's L[r][bm][bk]
 *   right (weight)       Rt[r][bn][ldk]  -- the TRANSPOSE of the reference's
 *                                           Rw[r][bk][bn], i.e. K-major, the
 *                                           operand layout tcgen05 reads
 *   products             P[r][bm][ldp]   -- as the reference's P[r][bm][bn]
 */
#ifndef FMM_SM100_H
#define FMM_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* fmm_stream_t; /* == cudaStream_t */

#define FMM_OK 0
#define FMM_ERR_INVALID_ARGUMENT 1
#define FMM_ERR_MISALIGNED 2
#define FMM_ERR_UNSUPPORTED 3
#define FMM_ERR_CUDA 4
#define FMM_ERR_DEVICE_TIMEOUT 5
#define FMM_ERR_TOO_LARGE 6

/* scheme ids: the rank of the block scheme */
#define FMM_SCHEME_RANK7 7   /* <2,2,2> rank 7 (Strassen-Winograd form)  */
#define FMM_SCHEME_RANK48 48 /* <4,4,4> rank 48 dyadic-rational SLP        */
#define FMM_SCHEME_RANK49 49 /* <4,4,4> rank 49 (rank 7 (x) rank 7)        */
#define FMM_SCHEME_RANK343 343 /* <8,8,8> rank 343, FP16 only (reference     */
                               /* Rank343Plan, runtime.py:883-962)          */

/* bits of the device status word */
#define FMM_STATUS_TIMEOUT 1u

/* precision of a call (the `dtype` argument): the element type of A,
 * weight/B, bias and C, and of the L, Rt and P planes.
 *   FMM_DTYPE_BF16       BF16 operands and output, FP16 planes
 *                        (the reference's (bfloat16, float16) precision pair)
 *   FMM_DTYPE_F16        FP16 operands, output and planes
 *                        (the reference's (float16, float16) pair)
 *   FMM_DTYPE_BF16_BF16  BF16 operands, output and planes -- rank 49 only,
 *                        the reference's (bfloat16, bfloat16) pair of
 *                        Rank49Plan (src/rdna3_fastmm/runtime.py:852-858);
 *                        FMM_ERR_UNSUPPORTED for the other schemes */
#define FMM_DTYPE_BF16 0
#define FMM_DTYPE_F16 1
#define FMM_DTYPE_BF16_BF16 2

/* fmm_linear flags */
#define FMM_LINEAR_PREPACKED 1u /* `Rt` already holds the packed right planes; W is ignored */
#define FMM_RIGHT_KN 2u         /* W is a contiguous right matrix B[K,N] (plain mm), not weight[N,K] */

typedef struct fmm_dims {
  int64_t scheme_size; /* s                      */
  int64_t rank;        /* R                      */
  int64_t bm, bk, bn;  /* ceil(M/s), ceil(K/s), ceil(N/s) */
  int64_t ldk;         /* pitch of L and Rt rows = round_up(bk, 8) */
  int64_t ldp;         /* pitch of P rows        = round_up(bn, 8) */
  int64_t left_elements;    /* R*bm*ldk */
  int64_t right_elements;   /* R*bn*ldk */
  int64_t product_elements; /* R*bm*ldp */
} fmm_dims;

/* Library version (major*10000 + minor*100 + patch). */
int fmm_version(void);

/* Text of the calling thread's last error ("" if none). */
const char* fmm_last_error_string(void);

/* Block dimensions and plane sizes for an M x K x N linear.
 * Replaces MatrixShape.from_dimensions (src/rdna3_fastmm/runtime.py:56-89). */
int fmm_plan_dims(int scheme, int64_t M, int64_t K, int64_t N, fmm_dims* out);

/* A[M,K] (BF16 or FP16 per dtype, lda) -> L[R][bm][ldk] (FP16, or BF16 for
 * FMM_DTYPE_BF16_BF16).
 * Replaces left_transform_kernel (src/rdna3_fastmm/runtime.py:597-615;
 * src/rdna3_fastmm/generated/rank7_2x2x2.py:9-62 and the rank-48/49 twins). */
int fmm_transform_a(int scheme, int dtype, const void* A, int64_t M, int64_t K, int64_t lda,
                    void* L, fmm_stream_t stream);

/* weight[N,K] (dtype, ldw) -> Rt[R][bn][ldk] (planes per dtype), the transform of
 * B = weight^T stored K-major.  Used per call (dynamic) and once (prepack).
 * Replaces right_transform_weight_kernel (src/rdna3_fastmm/runtime.py:637-655;
 * src/rdna3_fastmm/generated/rank7_2x2x2.py:121-204 and twins). */
int fmm_transform_w(int scheme, int dtype, const void* W, int64_t N, int64_t K, int64_t ldw,
                    void* Rt, fmm_stream_t stream);

/* fmm_transform_a and fmm_transform_w of one dynamic linear in a single
 * launch (the two input-side transforms share the GPU instead of running
 * back to back): A[M,K] -> L and weight[N,K] -> Rt, same layouts and
 * numerics as the two calls.  Replaces the consecutive left_transform_kernel
 * and right_transform_weight_kernel launches of src/rdna3_fastmm/linear.py:84-115
 * (src/rdna3_fastmm/runtime.py:597-655); fmm_linear uses it for a native
 * [N, K] weight. */
int fmm_transform_aw(int scheme, int dtype, const void* A, int64_t M, int64_t K, int64_t lda,
                     void* L, const void* W, int64_t N, int64_t ldw, void* Rt, fmm_stream_t stream);

/* Contiguous right matrix B[K,N] (dtype, ldb) -> Rt[R][bn][ldk] (planes per dtype), the
 * same planes as fmm_transform_w of weight = B^T (transposed on chip).  The
 * plain-mm API, per call and for pack_right.
 * Replaces right_transform_kernel (src/rdna3_fastmm/runtime.py:617-635;
 * src/rdna3_fastmm/generated/rank7_2x2x2.py:65-118 and twins). */
int fmm_transform_b(int scheme, int dtype, const void* B, int64_t K, int64_t N, int64_t ldb,
                    void* Rt, fmm_stream_t stream);

/* P[r] = L[r] * Rt[r]^T for r < rank: FP16 operands, FP32 accumulation in
 * tensor memory, FP16 products.  tcgen05 + TMA, persistent over 148 SMs.
 * Replaces torch.bmm(L, Rw, out=P) (src/rdna3_fastmm/runtime.py:728-732). */
int fmm_leaf_gemm(int rank, const void* L, const void* Rt, int64_t bm, int64_t bn, int64_t bk,
                  void* P, fmm_stream_t stream);

/* fmm_leaf_gemm with BF16 planes: BF16 L and Rt, FP32 accumulation in tensor
 * memory, BF16 products (round to nearest even) -- the leaf products of the
 * FMM_DTYPE_BF16_BF16 precision.
 * Replaces torch.bmm(L, Rw, out=P) on BF16 planes, which the reference runs
 * for Rank49Plan's (bfloat16, bfloat16) pair (src/rdna3_fastmm/runtime.py:728-732,
 * 852-858). */
int fmm_leaf_gemm_bf16(int rank, const void* L, const void* Rt, int64_t bm, int64_t bn, int64_t bk,
                       void* P, fmm_stream_t stream);

/* P[R][bm][ldp] (planes per dtype) -> C[M,N] (dtype, ldc) with optional bias[N] (dtype,
 * may be NULL): FP32 recombination, bias added last, round to nearest even.
 * Replaces output_transform_kernel / output_transform_bias_kernel
 * (src/rdna3_fastmm/runtime.py:657-698). */
int fmm_reconstruct(int scheme, int dtype, const void* P, int64_t M, int64_t N, const void* bias,
                    void* C, int64_t ldc, fmm_stream_t stream);

/* Row-sharded linear, output transform fused with the all-gather: like
 * fmm_reconstruct, but every output element is stored into all `ndest`
 * destinations (1..8) at once -- this rank's own gather buffer and the
 * peers' buffers mapped into this process (CUDA IPC peer
 * pointers reached over NVLink), each pointing at this rank's first row of
 * the gathered [rows, N] output, with leading dimension `ldc`.  The stores
 * end with a system-scope fence; the caller signals peers (a barrier on the
 * same stream) before they read.  Rank 48/49 with bn, N and ldc multiples of 8
 * and 16-byte-aligned destinations run 512-position tiles staged in shared
 * memory, whose row segments go to every destination as bulk async copies
 * (one CTA per SM; the grid is the fmm_set_sm_budget budget, so a GEMM
 * launched beside it with the complementary budget keeps its SMs); other
 * cases store element vectors from registers.  Circuit schemes only (7, 48,
 * 49); rank 343 returns FMM_ERR_UNSUPPORTED.  No reference counterpart: the reference is
 * single-GPU; this replaces the reconstruct + NCCL all-gather pair of the
 * multi-GPU form (rdna3_fastmm/distributed.py). */
int fmm_reconstruct_gather(int scheme, int dtype, const void* P, int64_t M, int64_t N,
                           const void* bias, void* const* dests, int ndest, int64_t ldc,
                           fmm_stream_t stream);

/* Peer memory for fmm_reconstruct_gather, by CUDA IPC (plain peer mappings,
 * no multicast object): export writes the 64-byte IPC handle of the
 * allocation containing `ptr` and ptr's byte offset inside it; another
 * process imports it (peer access enabled on first use) and receives the
 * mapping's base (for fmm_ipc_close) and the address at `offset`.  No
 * reference counterpart (the reference is single-GPU). */
#define FMM_IPC_HANDLE_BYTES 64
int fmm_ipc_export(const void* ptr, unsigned char* handle, uint64_t* offset);
int fmm_ipc_import(const unsigned char* handle, uint64_t offset, void** base, void** ptr);
int fmm_ipc_close(void* base);

/* Queue one device-to-device copy of `bytes` on `stream`; `dst` may be a
 * peer's buffer mapped by fmm_ipc_import, so the copy engines carry it over
 * NVLink while the SMs compute (the copy-engine gather of a row-sharded
 * linear).  One cudaMemcpyAsync; nothing is allocated.  No reference
 * counterpart (the reference is single-GPU). */
int fmm_copy_async(void* dst, const void* src, uint64_t bytes, fmm_stream_t stream);

/* The whole product through the scheme, using the caller's planes (L, Rt, P
 * sized by fmm_plan_dims): C = A * weight^T (+ bias) for F.linear, or, with
 * FMM_RIGHT_KN, C = A * B for a contiguous B[K,N].  With FMM_LINEAR_PREPACKED,
 * W is ignored (may be NULL) and Rt holds planes made earlier by
 * fmm_transform_w / fmm_transform_b.
 * Replaces _LinearPlan.run_linear / run_linear_packed and _Plan.run /
 * run_packed (src/rdna3_fastmm/runtime.py:278-341, 700-777). */
int fmm_linear(int scheme, int dtype, const void* A, const void* W, const void* bias, void* C,
               int64_t M, int64_t K, int64_t N, void* L, void* Rt, void* P, unsigned int flags,
               fmm_stream_t stream);

/* Size of the fixed scratch array behind fmm_linear_noalloc (32 MiB). */
#define FMM_NOALLOC_SCRATCH_BYTES (32u << 20)

/* BF16 fmm_linear without caller planes and without any allocation: for callers
 * that are handed device buffers for A, weight, bias and C but cannot
 * allocate device memory themselves -- a plugin whose host application owns
 * and budgets all device memory, or a loop that must never call cudaMalloc
 * because cudaMalloc can synchronise the device.  The L, Rt and P planes live
 * in one fixed FMM_NOALLOC_SCRATCH_BYTES array inside this library, which
 * every GPU that loads the library keeps until the process exits; shapes
 * whose planes do not fit (see fmm_plan_dims) return FMM_ERR_TOO_LARGE.
 * The first call on a device looks up that array's device address (with the
 * device current); make that first call before any stream capture.  All
 * calls on a device share the one array, so calls that overlap on the GPU
 * (on different streams, or from different threads) race; serialise them.
 * Nothing in the array has to start at zero: each call writes every plane
 * element it later reads.  Schemes 7, 48 and 49 only (BF16 operands); any other
 * scheme id returns FMM_ERR_UNSUPPORTED.  No counterpart in the reference (its
 * Python plans always allocate through PyTorch). */
int fmm_linear_noalloc(int scheme, const void* A, const void* W, const void* bias, void* C,
                       int64_t M, int64_t K, int64_t N, fmm_stream_t stream);

/* Most SMs any later launch of this library may fill (0 = all, the default;
 * odd values round down to even).  Leaving SMs free lets work on other
 * streams -- an NCCL all-gather of finished output rows, for instance -- run
 * alongside the persistent leaf GEMM.  Process-wide.  No counterpart in the
 * reference. */
int fmm_set_sm_budget(int sms);

/* Upper bound, in nanoseconds, of every device-side wait (default 2 s).  A
 * wait that runs out records FMM_STATUS_TIMEOUT and unwinds the kernel.  No
 * counterpart in the reference (it has no device-side waits). */
int fmm_set_wait_timeout_ns(uint64_t timeout_ns);

/* Synchronise `device` and read its status word; clear it when `reset`.
 * `site` (may be NULL) receives where the first timeout happened.  No
 * counterpart in the reference. */
int fmm_device_status(int device, uint32_t* status, uint32_t* site, int reset);

/* Test hook for the bounded waits: launches one CTA that waits, with
 * `timeout_ns`, on an mbarrier nothing arrives on.  The wait must run out and
 * the kernel must return; the caller then reads FMM_STATUS_TIMEOUT with
 * fmm_device_status.  No counterpart in the reference. */
int fmm_test_bounded_wait(uint64_t timeout_ns, fmm_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FMM_SM100_H */
