// Per-row squared norms (x_sq, kmeans_triton_impl.py:84-87) and row packing.
#include "fk_common.cuh"

namespace fk {

// One warp per row.  Same-dtype output follows `(x ** 2).sum(-1)` in that
// dtype: each square rounded to the dtype, float32 accumulation, one final
// rounding.  Float32 output squares and sums in float32.
template <typename T, bool SAME>
__global__ void row_sqnorm_kernel(const T* __restrict__ x, int64_t sxb, int64_t sxn, int64_t sxd,
                                  void* out, int out_dtype, int64_t sob, int64_t son, int N,
                                  int D, int64_t rows) {
  const int wpb = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5); r < rows;
       r += static_cast<int64_t>(gridDim.x) * wpb) {
    const int64_t b = r / N;
    const int64_t n = r % N;
    const T* row = x + b * sxb + n * sxn;
    float acc = 0.0f;
    if (sxd == 1) {
#pragma unroll 4
      for (int d = lane; d < D; d += 32) {
        const float e = Elem<T>::to_f(row[d]);
        acc += SAME ? Elem<T>::round(e * e) : e * e;
      }
    } else {
      for (int d = lane; d < D; d += 32) {
        const float e = Elem<T>::to_f(row[d * sxd]);
        acc += SAME ? Elem<T>::round(e * e) : e * e;
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) store_f(out, b * sob + n * son, out_dtype, acc);
  }
}

// Vector path: rows of 16-byte aligned records, LPR = D * sizeof(T) / 16
// lanes per row (a power of two <= 32), so one warp covers 32 / LPR rows per
// step with one 16-byte load per lane; the lanes of a row combine their
// partial sums with a segmented shuffle tree.  Each warp issues the loads of
// kSteps steps before reducing any of them (bytes in flight for an HBM-bound
// pass), and FLAT (batches laid out back to back in x and out) addresses
// row r directly instead of dividing it into (batch, point).
template <typename T, bool SAME, int LPR, bool FLAT>
__global__ void row_sqnorm_vec_kernel(const T* __restrict__ x, int64_t sxb, int64_t sxn,
                                      void* out, int out_dtype, int64_t sob, int64_t son, int N,
                                      int64_t rows) {
  constexpr int E = 16 / sizeof(T);  // elements per lane
  constexpr int RPW = 32 / LPR;      // rows per warp step
  constexpr int kSteps = 4;
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, part = lane % LPR;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t step = warps * RPW;
  auto xoff = [&](int64_t r) -> int64_t {
    if constexpr (FLAT) return r * sxn;
    const int64_t b = r / N;
    return b * sxb + (r - b * N) * sxn;
  };
  auto ooff = [&](int64_t r) -> int64_t {
    if constexpr (FLAT) return r * son;
    const int64_t b = r / N;
    return b * sob + (r - b * N) * son;
  };
  for (int64_t r0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW;
       r0 < rows; r0 += step * kSteps) {
    uint4 v[kSteps];
#pragma unroll
    for (int u = 0; u < kSteps; ++u) {
      const int64_t r = r0 + u * step + sub;
      v[u] = r < rows ? __ldcs(reinterpret_cast<const uint4*>(x + xoff(r) + part * E))
                      : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kSteps; ++u) {
      const int64_t r = r0 + u * step + sub;
      float acc = 0.0f;
      const T* e = reinterpret_cast<const T*>(&v[u]);
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const float f = Elem<T>::to_f(e[i]);
        acc += SAME ? Elem<T>::round(f * f) : f * f;
      }
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (part == 0 && r < rows) store_f(out, ooff(r), out_dtype, acc);
    }
  }
}

// F.normalize(x, p=2, dim=-1) in x's dtype (kmeans_triton_impl.py:135): the
// norm is accumulated in float32 and rounded to the dtype, clamped below by
// eps = 1e-12 taken in the dtype (0 for float16), and each element is divided
// in float32 and rounded.  One warp per row.
template <typename T>
__global__ void row_normalize_kernel(const T* __restrict__ x, int64_t sxb, int64_t sxn,
                                     int64_t sxd, T* __restrict__ out, int64_t sob, int64_t son,
                                     int64_t sod, int N, int D, int64_t rows) {
  const int wpb = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const float eps = Elem<T>::round(1e-12f);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5); r < rows;
       r += static_cast<int64_t>(gridDim.x) * wpb) {
    const int64_t b = r / N, n = r % N;
    const T* row = x + b * sxb + n * sxn;
    T* dst = out + b * sob + n * son;
    float ss = 0.0f;
    for (int d = lane; d < D; d += 32) {
      const float e = Elem<T>::to_f(row[d * sxd]);
      ss = __fmaf_rn(e, e, ss);
    }
    ss = warp_sum(ss);
    const float den = fmaxf(Elem<T>::round(sqrtf(ss)), eps);
    for (int d = lane; d < D; d += 32)
      dst[d * sod] = Elem<T>::from_f(__fdiv_rn(Elem<T>::to_f(row[d * sxd]), den));
  }
}

// Vector path of row_normalize_kernel (contiguous rows of 16-byte aligned
// records, LPR = D * sizeof(T) / 16 lanes per row, a power of two <= 32): each
// lane squares and sums its 16 bytes in float32, a segmented shuffle tree
// combines the row's lanes, and the lane divides the elements it still holds.
// Same rounding steps as the scalar kernel (float32 sum, norm rounded to the
// dtype and clamped, one rounded division per element); the float32 summation
// order differs, as it does from torch's.  FLAT: batches back to back.
template <typename T, int LPR, bool FLAT>
__global__ void row_normalize_vec_kernel(const T* __restrict__ x, int64_t sxb, int64_t sxn,
                                         T* __restrict__ out, int64_t sob, int64_t son, int N,
                                         int64_t rows) {
  constexpr int E = 16 / sizeof(T);
  constexpr int RPW = 32 / LPR;
  constexpr int kSteps = 2;
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, part = lane % LPR;
  const float eps = Elem<T>::round(1e-12f);
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t step = warps * RPW;
  auto off = [&](int64_t r, int64_t sb, int64_t sn) -> int64_t {
    if constexpr (FLAT) return r * sn;
    const int64_t b = r / N;
    return b * sb + (r - b * N) * sn;
  };
  for (int64_t r0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW;
       r0 < rows; r0 += step * kSteps) {
    uint4 v[kSteps];
#pragma unroll
    for (int u = 0; u < kSteps; ++u) {
      const int64_t r = r0 + u * step + sub;
      v[u] = r < rows ? __ldcs(reinterpret_cast<const uint4*>(x + off(r, sxb, sxn) + part * E))
                      : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kSteps; ++u) {
      const int64_t r = r0 + u * step + sub;
      T* e = reinterpret_cast<T*>(&v[u]);
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const float f = Elem<T>::to_f(e[i]);
        ss = __fmaf_rn(f, f, ss);
      }
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float den = fmaxf(Elem<T>::round(sqrtf(ss)), eps);
#pragma unroll
      for (int i = 0; i < E; ++i) e[i] = Elem<T>::from_f(__fdiv_rn(Elem<T>::to_f(e[i]), den));
      if (r < rows) __stcs(reinterpret_cast<uint4*>(out + off(r, sob, son) + part * E), v[u]);
    }
  }
}

template <typename T>
static int row_normalize_vec(const void* x, int64_t B, int64_t N, int64_t D, const int64_t* xs,
                             void* out, const int64_t* os, int64_t blocks, cudaStream_t s,
                             bool* done) {
  constexpr int64_t eb = sizeof(T);
  const int64_t lpr = D * eb / 16;
  *done = xs[2] == 1 && os[2] == 1 && (D * eb) % 16 == 0 && (lpr & (lpr - 1)) == 0 && lpr <= 32 &&
          reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
          (xs[1] * eb) % 16 == 0 && (os[1] * eb) % 16 == 0 &&
          (B == 1 || ((xs[0] * eb) % 16 == 0 && (os[0] * eb) % 16 == 0));
  if (!*done) return FK_OK;
  const bool flat = B == 1 || (xs[0] == N * xs[1] && os[0] == N * os[1]);
  const T* xt = static_cast<const T*>(x);
  T* ot = static_cast<T*>(out);
  const int64_t rows = B * N;
#define FK_RN2(L, F)                                                                              \
  row_normalize_vec_kernel<T, L, F><<<static_cast<int>(blocks), 256, 0, s>>>(                     \
      xt, xs[0], xs[1], ot, os[0], os[1], static_cast<int>(N), rows);
#define FK_RN(L)                                                                                  \
  if (lpr == L) {                                                                                 \
    if (flat) {                                                                                   \
      FK_RN2(L, true)                                                                             \
    } else {                                                                                      \
      FK_RN2(L, false)                                                                            \
    }                                                                                             \
  }
  FK_RN(1) FK_RN(2) FK_RN(4) FK_RN(8) FK_RN(16) FK_RN(32)
#undef FK_RN
#undef FK_RN2
  return check_launch("row_normalize_vec_kernel");
}

template <typename T>
__global__ void pack_rows_kernel(const T* __restrict__ x, int64_t sxb, int64_t sxn, int64_t sxd,
                                 T* __restrict__ out, int N, int D, int Dp, int64_t total) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(i % Dp);
    const int64_t rn = i / Dp;
    const int64_t n = rn % N;
    const int64_t b = rn / N;
    out[i] = d < D ? x[b * sxb + n * sxn + d * sxd] : Elem<T>::from_f(0.0f);
  }
}

template <typename T>
static int row_sqnorm_typed(const void* x, int dtype, int64_t B, int64_t N, int64_t D,
                            const int64_t* xs, void* out, int out_dtype, const int64_t* os,
                            cudaStream_t s) {
  const int64_t rows = B * N;
  const int threads = 256;
  int64_t blocks = (rows + 7) / 8;
  const int sms = sm_count_current();
  const int64_t cap = sms > 0 ? static_cast<int64_t>(sms) * 16 : 2048;
  if (blocks > cap) blocks = cap;
  const int64_t eb = sizeof(T);
  const int64_t lpr = D * eb / 16;
  const bool vec = xs[2] == 1 && (D * eb) % 16 == 0 && (lpr & (lpr - 1)) == 0 && lpr <= 32 &&
                   reinterpret_cast<uintptr_t>(x) % 16 == 0 && (xs[1] * eb) % 16 == 0 &&
                   (B == 1 || (xs[0] * eb) % 16 == 0);
  if (vec) {
    const bool same = out_dtype == dtype;
    const bool flat = (B == 1 || xs[0] == N * xs[1]) && (B == 1 || os[0] == N * os[1]);
    const T* xt = static_cast<const T*>(x);
#define FK_SQN2(L, F)                                                                             \
  if (same)                                                                                       \
    row_sqnorm_vec_kernel<T, true, L, F><<<static_cast<int>(blocks), threads, 0, s>>>(            \
        xt, xs[0], xs[1], out, out_dtype, os[0], os[1], static_cast<int>(N), rows);               \
  else                                                                                            \
    row_sqnorm_vec_kernel<T, false, L, F><<<static_cast<int>(blocks), threads, 0, s>>>(           \
        xt, xs[0], xs[1], out, out_dtype, os[0], os[1], static_cast<int>(N), rows);
#define FK_SQN(L)                                                                                 \
  if (lpr == L) {                                                                                 \
    if (flat) {                                                                                   \
      FK_SQN2(L, true)                                                                            \
    } else {                                                                                      \
      FK_SQN2(L, false)                                                                           \
    }                                                                                             \
    return check_launch("row_sqnorm_vec_kernel");                                               \
  }
    FK_SQN(1) FK_SQN(2) FK_SQN(4) FK_SQN(8) FK_SQN(16) FK_SQN(32)
#undef FK_SQN
#undef FK_SQN2
  }
  if (out_dtype == dtype)
    row_sqnorm_kernel<T, true><<<static_cast<int>(blocks), threads, 0, s>>>(
        static_cast<const T*>(x), xs[0], xs[1], xs[2], out, out_dtype, os[0], os[1],
        static_cast<int>(N), static_cast<int>(D), rows);
  else
    row_sqnorm_kernel<T, false><<<static_cast<int>(blocks), threads, 0, s>>>(
        static_cast<const T*>(x), xs[0], xs[1], xs[2], out, out_dtype, os[0], os[1],
        static_cast<int>(N), static_cast<int>(D), rows);
  return check_launch("row_sqnorm_kernel");
}

template <typename T>
static int pack_rows_typed(const void* x, int64_t B, int64_t N, int64_t D, const int64_t* xs,
                           void* out, int64_t Dp, cudaStream_t s) {
  const int64_t total = B * N * Dp;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int sms = sm_count_current();
  const int64_t cap = sms > 0 ? static_cast<int64_t>(sms) * 32 : 4096;
  if (blocks > cap) blocks = cap;
  pack_rows_kernel<T><<<static_cast<int>(blocks), threads, 0, s>>>(
      static_cast<const T*>(x), xs[0], xs[1], xs[2], static_cast<T*>(out), static_cast<int>(N),
      static_cast<int>(D), static_cast<int>(Dp), total);
  return check_launch("pack_rows_kernel");
}

}  // namespace fk

using namespace fk;

extern "C" int fk_row_sqnorm(const void* x, int dtype, int64_t B, int64_t N, int64_t D,
                             const int64_t* x_strides3, void* out, int out_dtype,
                             const int64_t* out_strides2, void* stream) {
  if (B < 0 || N < 0 || D <= 0) return fail(FK_ERR_INVALID_ARG, "fk_row_sqnorm: bad sizes");
  if (B == 0 || N == 0) return FK_OK;
  if (!x || !out || !x_strides3 || !out_strides2)
    return fail(FK_ERR_INVALID_ARG, "fk_row_sqnorm: null pointer argument");
  if (out_dtype != dtype && out_dtype != FK_F32)
    return fail(FK_ERR_INVALID_ARG, "fk_row_sqnorm: out dtype must equal x dtype or be f32");
  if (N >= (1ll << 31) || D >= (1ll << 31))
    return fail(FK_ERR_UNSUPPORTED, "fk_row_sqnorm: sizes exceed 32-bit");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case FK_F16:
      return row_sqnorm_typed<__half>(x, dtype, B, N, D, x_strides3, out, out_dtype, out_strides2, s);
    case FK_BF16:
      return row_sqnorm_typed<__nv_bfloat16>(x, dtype, B, N, D, x_strides3, out, out_dtype,
                                             out_strides2, s);
    case FK_F32:
      return row_sqnorm_typed<float>(x, dtype, B, N, D, x_strides3, out, out_dtype, out_strides2, s);
    default:
      return fail(FK_ERR_INVALID_ARG, "fk_row_sqnorm: unsupported dtype %d", dtype);
  }
}

extern "C" int fk_row_normalize(const void* x, int dtype, int64_t B, int64_t N, int64_t D,
                                const int64_t* x_strides3, void* out, const int64_t* out_strides3,
                                void* stream) {
  if (B < 0 || N < 0 || D <= 0) return fail(FK_ERR_INVALID_ARG, "fk_row_normalize: bad sizes");
  if (B == 0 || N == 0) return FK_OK;
  if (!x || !out || !x_strides3 || !out_strides3)
    return fail(FK_ERR_INVALID_ARG, "fk_row_normalize: null pointer argument");
  if (N >= (1ll << 31) || D >= (1ll << 31))
    return fail(FK_ERR_UNSUPPORTED, "fk_row_normalize: N and D must be below 2^31");
  const int64_t rows = B * N;
  int64_t blocks = (rows + 7) / 8;
  const int sms = sm_count_current();
  const int64_t cap = sms > 0 ? static_cast<int64_t>(sms) * 16 : 2048;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t* xs = x_strides3;
  const int64_t* os = out_strides3;
  {
    bool done = false;
    int st = FK_OK;
    if (dtype == FK_F16)
      st = row_normalize_vec<__half>(x, B, N, D, xs, out, os, blocks, s, &done);
    else if (dtype == FK_BF16)
      st = row_normalize_vec<__nv_bfloat16>(x, B, N, D, xs, out, os, blocks, s, &done);
    else if (dtype == FK_F32)
      st = row_normalize_vec<float>(x, B, N, D, xs, out, os, blocks, s, &done);
    if (done || st != FK_OK) return st;
  }
  switch (dtype) {
    case FK_F16:
      row_normalize_kernel<__half><<<static_cast<int>(blocks), 256, 0, s>>>(
          static_cast<const __half*>(x), xs[0], xs[1], xs[2], static_cast<__half*>(out), os[0],
          os[1], os[2], static_cast<int>(N), static_cast<int>(D), rows);
      break;
    case FK_BF16:
      row_normalize_kernel<__nv_bfloat16><<<static_cast<int>(blocks), 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), xs[0], xs[1], xs[2],
          static_cast<__nv_bfloat16*>(out), os[0], os[1], os[2], static_cast<int>(N),
          static_cast<int>(D), rows);
      break;
    case FK_F32:
      row_normalize_kernel<float><<<static_cast<int>(blocks), 256, 0, s>>>(
          static_cast<const float*>(x), xs[0], xs[1], xs[2], static_cast<float*>(out), os[0],
          os[1], os[2], static_cast<int>(N), static_cast<int>(D), rows);
      break;
    default:
      return fail(FK_ERR_INVALID_ARG, "fk_row_normalize: unsupported dtype %d", dtype);
  }
  return check_launch("row_normalize_kernel");
}

extern "C" int fk_pack_rows(const void* x, int dtype, int64_t B, int64_t N, int64_t D,
                            const int64_t* x_strides3, void* out, int64_t Dp, void* stream) {
  if (B < 0 || N < 0 || D <= 0 || Dp < D) return fail(FK_ERR_INVALID_ARG, "fk_pack_rows: bad sizes");
  if (B == 0 || N == 0) return FK_OK;
  if (!x || !out || !x_strides3) return fail(FK_ERR_INVALID_ARG, "fk_pack_rows: null pointer");
  if (N >= (1ll << 31) || Dp >= (1ll << 31))
    return fail(FK_ERR_UNSUPPORTED, "fk_pack_rows: sizes exceed 32-bit");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case FK_F16: return pack_rows_typed<__half>(x, B, N, D, x_strides3, out, Dp, s);
    case FK_BF16: return pack_rows_typed<__nv_bfloat16>(x, B, N, D, x_strides3, out, Dp, s);
    case FK_F32: return pack_rows_typed<float>(x, B, N, D, x_strides3, out, Dp, s);
    default: return fail(FK_ERR_INVALID_ARG, "fk_pack_rows: unsupported dtype %d", dtype);
  }
}
