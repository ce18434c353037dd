// Shared types and helpers for the sm_100a Flash-KMeans kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "flash_kmeans_b200.h"

namespace fk {

// --------------------------------------------------------------- element types
template <typename T>
struct Elem;

template <>
struct Elem<__half> {
  static constexpr int kBytes = 2;
  static constexpr uint32_t kMmaFmt = 0;  // kind::f16, A/B format f16
  static constexpr int kDtype = FK_F16;
  static constexpr float kMaxFinite = 65504.0f;
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
  __device__ __forceinline__ static float round(float v) { return __half2float(__float2half_rn(v)); }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kBytes = 2;
  static constexpr uint32_t kMmaFmt = 1;  // kind::f16, A/B format bf16
  static constexpr int kDtype = FK_BF16;
  static constexpr float kMaxFinite = 3.38953139e38f;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  __device__ __forceinline__ static float round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
};

template <>
struct Elem<float> {
  static constexpr int kBytes = 4;
  static constexpr uint32_t kMmaFmt = 2;  // kind::tf32
  static constexpr int kDtype = FK_F32;
  static constexpr float kMaxFinite = 3.40282347e38f;
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
  __device__ __forceinline__ static float round(float v) { return v; }
};

__host__ __device__ inline int dtype_bytes(int dt) {
  return dt == FK_F16 || dt == FK_BF16 ? 2 : (dt == FK_F32 || dt == FK_I32 ? 4 : (dt == FK_I64 ? 8 : 0));
}

// Load one element of a runtime-typed float array as float.
__device__ __forceinline__ float load_f(const void* p, int64_t i, int dt) {
  if (dt == FK_F16) return __half2float(static_cast<const __half*>(p)[i]);
  if (dt == FK_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_f(void* p, int64_t i, int dt, float v) {
  if (dt == FK_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else if (dt == FK_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ float round_to(float v, int dt) {
  if (dt == FK_F16) return __half2float(__float2half_rn(v));
  if (dt == FK_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------ host side
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int check_launch(const char* what);
int sm_count_current();
int current_device();

// cuTensorMapEncodeTiled resolved once through the runtime's driver entry
// point (no link-time dependency on libcuda).
// `sw64`: the 64-byte swizzle (box rows of 64 bytes) instead of the 128-byte one.
int encode_tmap_3d(CUtensorMap* map, const void* base, int dtype, uint64_t d0, uint64_t d1,
                   uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                   uint32_t box1, bool sw64 = false);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Privatised centroid accumulation (fk_update.cu): true when one batch's
// K x D float32 sums and K counts fit in a CTA's shared memory.
bool segsum_priv_fits(int64_t K, int64_t D);
// sums[b][ids] += rows of x; counts[b][ids] += 1 unless counts is null.
int segsum_priv(const void* x, int dtype, const int64_t* xs, const void* ids, int ids_dtype,
                const int64_t* is, int64_t B, int64_t N, int64_t K, int64_t D, float* sums,
                int32_t* counts, int32_t* status, cudaStream_t s);

}  // namespace fk
