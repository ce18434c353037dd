/*
 * flash_kmeans_b200.h -- C ABI of the B200 (sm_100a) Lloyd-iteration kernels.
 *
 * This is the drop-in boundary under the Python package `flash_kmeans`
 * (flash-kmeans_b200/flash_kmeans/).  Every entry point takes plain device
 * pointers, element strides and sizes, launches on the caller's CUDA stream
 * (`stream` is a cudaStream_t; NULL means the legacy default stream) and never
 * synchronises.  Buffers are caller-owned; scratch memory is the caller's
 * `workspace` (size from the matching *_workspace_size query).  Nothing is
 * allocated.  Global mutable state: one-time per-device lookups (driver entry
 * point, SM count, kernel attributes, the address of fk_assign_static_scratch's
 * array), all thread-safe, and that 16 MiB static array itself, which only
 * fk_assign_static_scratch uses (its calls share it).  One host thread may
 * drive several devices by switching the current device.
 *
 * Errors: functions return FK_OK (0) or an fk_status code; fk_last_error()
 * returns a thread-local message for the last failure.  Kernels that can
 * detect bad data or a stalled pipeline report it asynchronously through the
 * optional `dev_status` word (an int32 in device memory, zero on entry):
 * the caller reads it back at its next synchronisation point.
 *
 * Reference interfaces replaced (paths inside svg-project/flash-kmeans):
 *   fk_row_sqnorm          <- x_sq precompute, flash_kmeans/kmeans_triton_impl.py:84-87
 *                             and flash_kmeans/interface.py:240-245
 *   fk_assign              <- euclid_assign_triton, flash_kmeans/assign_euclid_triton.py:1238-1412
 *                             (kernels _euclid_assign_kernel :804-917 and
 *                             _euclid_assign_kernel_split_d :933-1030)
 *   fk_centroid_accumulate <- triton_centroid_update_sorted_euclid accumulate phase,
 *                             flash_kmeans/centroid_update_triton.py:316-376
 *                             (kernel _centroid_update_chunk_kernel :188-263)
 *   fk_centroid_finalize   <- the same function's finalize, centroid_update_triton.py:378-386,
 *                             plus the shift of kmeans_triton_impl.py:16 and the
 *                             c_sq of assign_euclid_triton.py:1282-1283
 *   fk_pack_rows           <- no reference counterpart: repacks rows whose
 *                             stride is not a multiple of 16 bytes for TMA
 *   fk_assign_dot          <- cosine_assign_triton, flash_kmeans/assign_euclid_triton.py:1415-1498
 *                             (kernels _cosine_assign_kernel :1038-1131 and its split-D
 *                             variant :1137-1231), used by batch_kmeans_Cosine / _Dot
 *   fk_assign_dot_accumulate
 *                          <- cosine_assign_triton + the accumulate phase of
 *                             triton_centroid_update_sorted_cosine, as paired in
 *                             _cosine_iter / _dot_iter, kmeans_triton_impl.py:19-35
 *   fk_row_normalize       <- F.normalize of x in batch_kmeans_Cosine,
 *                             flash_kmeans/kmeans_triton_impl.py:135
 *   fk_centroid_finalize_normalized
 *                          <- the cosine update's finalize: _centroid_update_torch_native
 *                             with mode='cosine', flash_kmeans/torch_fallback.py:101-109
 *                             (triton_centroid_update_sorted_cosine,
 *                             centroid_update_triton.py:268-313)
 */
#ifndef FLASH_KMEANS_B200_H
#define FLASH_KMEANS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FK_ABI_VERSION 2

/* element types.  FK_F32_XSPLIT is accepted by the *_accumulate entry points
 * only: float32 x whose tf32 hi halves and exact rests the workspace holds,
 * split once by fk_assign_accumulate_split_x (see there). */
enum fk_dtype { FK_F16 = 0, FK_BF16 = 1, FK_F32 = 2, FK_I32 = 3, FK_I64 = 4, FK_F32_XSPLIT = 5 };

/* host-side status codes */
enum fk_status {
  FK_OK = 0,
  FK_ERR_INVALID_ARG = 1, /* null pointer, negative size, bad stride, dtype mismatch */
  FK_ERR_UNSUPPORTED = 2, /* layout/size the kernels do not take (e.g. rows not 16-byte aligned) */
  FK_ERR_WORKSPACE = 3,   /* workspace missing, too small or misaligned */
  FK_ERR_CUDA = 4,        /* a CUDA runtime call or kernel launch failed */
  FK_ERR_TMA = 5          /* tensor-map encoding failed */
};

/* device-side codes written to *dev_status (first error wins) */
enum fk_device_status {
  FK_DEV_OK = 0,
  FK_DEV_BAD_LABEL = 101,      /* a cluster id outside [0, K) was fed to the update */
  FK_DEV_WAIT_TIMEOUT = 102    /* a pipeline wait in the assign kernel exceeded its limit */
};

int fk_abi_version(void);
const char* fk_status_string(int status);
const char* fk_last_error(void);
/* SM count of the current device (cached); <0 on error. */
int fk_device_sm_count(void);

/* 1 if (ptr, strides) can be read by the TMA-based assignment directly:
 * unit innermost stride, 16-byte aligned base, 16-byte multiple outer strides. */
int fk_tma_compatible(const void* ptr, int dtype, int64_t D, const int64_t* strides3);

/* Row squared norms out[b,n] = sum_d x[b,n,d]^2.
 * out_dtype == dtype: rounded like `(x ** 2).sum(-1)` evaluated in that dtype
 * (per-element square rounded, float32 accumulation, one final rounding);
 * out_dtype == FK_F32: computed entirely in float32. */
int fk_row_sqnorm(const void* x, int dtype, int64_t B, int64_t N, int64_t D,
                  const int64_t* x_strides3, void* out, int out_dtype,
                  const int64_t* out_strides2, void* stream);

/* out = F.normalize(x, p=2, dim=-1) in x's dtype: norm accumulated in float32
 * and rounded to the dtype, clamped below by 1e-12 taken in the dtype, each
 * element divided in float32 and rounded.  out may alias x. */
int fk_row_normalize(const void* x, int dtype, int64_t B, int64_t N, int64_t D,
                     const int64_t* x_strides3, void* out, const int64_t* out_strides3,
                     void* stream);

/* Copy x (B,N,D, any strides) into a contiguous (B,N,Dp) buffer, Dp >= D, with
 * zeros in columns [D, Dp).  Used to make rows TMA-addressable. */
int fk_pack_rows(const void* x, int dtype, int64_t B, int64_t N, int64_t D,
                 const int64_t* x_strides3, void* out, int64_t Dp, void* stream);

/* Nearest centroid by squared Euclidean distance.
 *   x (B,N,D), centroids (B,K,D): dtype FK_F16 / FK_BF16 / FK_F32, TMA-compatible.
 *   x_sq (B,N): xsq_dtype; c_sq (B,K) optional (NULL -> computed from centroids).
 *   out (B,N) int32.  counts (B,K) int32 optional: if given, out's histogram is
 *   ADDED to it (the update's histogram, fused).
 * Distance rounding follows the reference's torch path: with x_sq in x's
 * 16-bit dtype the chain is round(round(x_sq - round(2*round(x.c))) + c_sq) in
 * that dtype, overflow to inf included (the centroid operand of the tensor
 * cores is -2c, staged in the workspace); otherwise float32 (for float32 x
 * the dot products are 3xTF32 on the tensor cores).  Ties resolve to the
 * lowest centroid index; a NaN distance wins at its first column, as argmin.
 * Requires K <= 1<<20, N < 2^31.  The workspace (fk_assign_workspace_size)
 * holds the padded c_sq and, for 16-bit x, -2c (about B*K*D*2 bytes); for
 * float32 x, the centroids' tf32 hi and lo halves (about B*K*D*8 bytes). */
size_t fk_assign_workspace_size(int64_t B, int64_t K, int64_t D, int dtype);
int fk_assign(const void* x, const void* centroids, const void* x_sq, const void* c_sq,
              int32_t* out, int32_t* counts, int dtype, int xsq_dtype, int csq_dtype,
              int64_t B, int64_t N, int64_t K, int64_t D, const int64_t* x_strides3,
              const int64_t* c_strides3, const int64_t* xsq_strides2,
              const int64_t* csq_strides2, const int64_t* out_strides2, void* workspace,
              size_t workspace_bytes, int32_t* dev_status, void* stream);

/* Centroid of the largest dot product (cosine / dot-product k-means):
 * out[b,n] = argmax_k x[b,n].c[b,k] with float32 (16-bit inputs) or 3xTF32
 * (float32 inputs) dot products, lowest index on ties.  Same conventions and
 * workspace (fk_assign_workspace_size) as fk_assign, without x_sq / c_sq;
 * counts optional as there. */
int fk_assign_dot(const void* x, const void* centroids, int32_t* out, int32_t* counts, int dtype,
                  int64_t B, int64_t N, int64_t K, int64_t D, const int64_t* x_strides3,
                  const int64_t* c_strides3, const int64_t* out_strides2, void* workspace,
                  size_t workspace_bytes, int32_t* dev_status, void* stream);

/* Assignment fused with the centroid accumulation of one Lloyd iteration
 * (replaces the pair euclid_assign_triton + triton_centroid_update_sorted_euclid
 * in _euclid_iter, flash_kmeans/kmeans_triton_impl.py:11-17, up to the
 * finalize).  Same arguments as fk_assign plus `sums` (B,K,D float32
 * contiguous); `counts` (B,K int32) is required.  Labels are written to `out`,
 * their histogram is ADDED to `counts` and the rows of x are ADDED to
 * sums[label].  When a batch's K x D float32 sums (plus K counts) fit in
 * 200 KiB of shared memory it runs fk_assign then the privatised sum of
 * fk_centroid_accumulate; else with 16-bit x and D <= 128 it is one kernel
 * that reads x once; otherwise fk_assign then fk_centroid_accumulate. */
size_t fk_assign_accumulate_workspace_size(int64_t B, int64_t N, int64_t K, int64_t D, int dtype);

/* How fk_assign_accumulate accumulates for these sizes (no counterpart in
 * the reference, which always sorts): FK_ACC_PRIVATISED (a batch's K x D
 * float32 sums fit in shared memory), FK_ACC_FUSED (16-bit x, D <= 128: one
 * kernel), FK_ACC_SORTED (assignment, then counting sort + segmented sum). */
enum fk_acc_method { FK_ACC_PRIVATISED = 0, FK_ACC_FUSED = 1, FK_ACC_SORTED = 2 };
int fk_assign_accumulate_method(int64_t K, int64_t D, int dtype);
int fk_assign_accumulate(const void* x, const void* centroids, const void* x_sq, const void* c_sq,
                         int32_t* out, int32_t* counts, float* sums, int dtype, int xsq_dtype,
                         int csq_dtype, int64_t B, int64_t N, int64_t K, int64_t D,
                         const int64_t* x_strides3, const int64_t* c_strides3,
                         const int64_t* xsq_strides2, const int64_t* csq_strides2,
                         const int64_t* out_strides2, void* workspace, size_t workspace_bytes,
                         int32_t* dev_status, void* stream);

/* fk_assign_dot fused with the accumulation of one cosine / dot-product Lloyd
 * iteration (replaces cosine_assign_triton + the accumulate phase of
 * triton_centroid_update_sorted_cosine in _cosine_iter / _dot_iter,
 * flash_kmeans/kmeans_triton_impl.py:19-35).  Arguments as fk_assign_dot
 * plus `sums`; `counts` is required; sums and counts are ADDED to, by the
 * method fk_assign_accumulate_method names; workspace
 * fk_assign_accumulate_workspace_size.  Follow with
 * fk_centroid_finalize_normalized. */
int fk_assign_dot_accumulate(const void* x, const void* centroids, int32_t* out, int32_t* counts,
                             float* sums, int dtype, int64_t B, int64_t N, int64_t K, int64_t D,
                             const int64_t* x_strides3, const int64_t* c_strides3,
                             const int64_t* out_strides2, void* workspace, size_t workspace_bytes,
                             int32_t* dev_status, void* stream);

/* Float32 x split once for many Lloyd iterations (no counterpart in the
 * reference, whose float32 assignment is plain TF32).  The 3xTF32 assignment
 * needs x as tf32 hi = x rounded to 10 explicit mantissa bits and the exact
 * rest lo = x - hi; fk_assign_accumulate / fk_assign_dot_accumulate split each
 * x tile in shared memory on every call.  With dtype FK_F32_XSPLIT they
 * instead load both halves from the workspace (x itself still feeds the
 * centroid sums), which this call fills from x: a (2B, N, Dx) float32 array,
 * Dx = D rounded up to 4, at the end of a workspace of
 * fk_assign_accumulate_workspace_size(B, N, K, D, FK_F32_XSPLIT) bytes
 * (2*B*N*Dx*4 bytes more than FK_F32's).  Call it again whenever x changes;
 * labels, sums and counts are the same as with FK_F32. */
int fk_assign_accumulate_split_x(const float* x, int64_t B, int64_t N, int64_t K, int64_t D,
                                 const int64_t* x_strides3, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* fk_assign for callers that cannot allocate (no counterpart in the reference).
 * Some hosts give a plugin only its inputs and outputs: a serving framework's
 * custom-op interface without a workspace hook, a memory pool that forbids side
 * allocations, or a latency-bound loop where cudaMalloc/cudaFree (which can
 * synchronise the device) is not acceptable.  Same arguments and results as
 * fk_assign, minus the workspace: the scratch is a 16 MiB file-scope device
 * array that every GPU loading this library keeps until exit.
 * Limit: fk_assign_workspace_size(B, K, D, dtype) <= 16 MiB (e.g. B=32,
 * K=1000, D=128 float16 takes 8.3 MiB); larger sizes return FK_ERR_WORKSPACE.
 * The first call on a device looks the array up (cudaGetSymbolAddress) and
 * should come before any stream capture.  All calls on a device share the
 * array (each call rewrites what it reads); calls that overlap on the GPU race
 * on it.  Allocates nothing. */
int fk_assign_static_scratch(const void* x, const void* centroids, const void* x_sq,
                             const void* c_sq, int32_t* out, int32_t* counts, int dtype,
                             int xsq_dtype, int csq_dtype, int64_t B, int64_t N, int64_t K,
                             int64_t D, const int64_t* x_strides3, const int64_t* c_strides3,
                             const int64_t* xsq_strides2, const int64_t* csq_strides2,
                             const int64_t* out_strides2, int32_t* dev_status, void* stream);

/* Per-cluster float32 sums (B,K,D contiguous) and int32 counts (B,K contiguous)
 * of the rows of x grouped by ids (B,N; FK_I32 or FK_I64), ADDED to `sums`
 * and `counts`.  `hist` (B,K) optional: the histogram of exactly these ids
 * (e.g. produced by fk_assign's `counts`); NULL -> computed here.
 * When a batch's K x D float32 sums plus K counts fit in 200 KiB, each CTA
 * accumulates its share of the points in shared memory and adds its partial
 * sums once (the workspace is then unused); otherwise grouping is a counting
 * sort (histogram, scan, scatter) followed by a segmented sum over the sorted
 * order. */
size_t fk_centroid_accumulate_workspace_size(int64_t B, int64_t N, int64_t K);
int fk_centroid_accumulate(const void* x, int dtype, int64_t B, int64_t N, int64_t K, int64_t D,
                           const int64_t* x_strides3, const void* ids, int ids_dtype,
                           const int64_t* ids_strides2, const int32_t* hist, float* sums,
                           int32_t* counts, void* workspace, size_t workspace_bytes,
                           int32_t* dev_status, void* stream);

/* new = counts ? sums / counts : old, cast to dtype (reference finalize).
 * Optional outputs: csq_out (B,K) float32 = (new ** 2).sum(-1) rounded in dtype;
 * shift_out (one float32) = max_k ||new_k - old_k|| rounded in dtype.
 * reset_accumulators != 0: sums and counts are set to zero after being read,
 * ready for the next iteration's accumulation.
 * `new_centroids` may not alias `old_centroids`. */
int fk_centroid_finalize(float* sums, int32_t* counts, const void* old_centroids,
                         void* new_centroids, int dtype, int64_t B, int64_t K, int64_t D,
                         const int64_t* old_strides3, const int64_t* new_strides3,
                         float* csq_out, float* shift_out, int reset_accumulators, void* stream);

/* Cosine / dot-product finalize: m = counts ? sums / counts : old (float32),
 * new = (m / max(||m||, 1e-12)) cast to dtype; shift_out as in
 * fk_centroid_finalize; reset_accumulators as there. */
int fk_centroid_finalize_normalized(float* sums, int32_t* counts, const void* old_centroids,
                                    void* new_centroids, int dtype, int64_t B, int64_t K,
                                    int64_t D, const int64_t* old_strides3,
                                    const int64_t* new_strides3, float* shift_out,
                                    int reset_accumulators, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FLASH_KMEANS_B200_H */
