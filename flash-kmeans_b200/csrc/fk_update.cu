// Centroid update (replaces triton_centroid_update_sorted_euclid and its
// _centroid_update_chunk_kernel, flash_kmeans/centroid_update_triton.py:188-386).
//
// The reference sorts the labels with torch.sort and has each program walk
// 256 sorted points, gathering rows and issuing one atomic per run of equal
// labels.  Here the grouping is a counting sort built for the case at hand
// (labels are small integers in [0, K)): histogram -> per-batch exclusive
// scan -> scatter of point indices.  A segmented-sum kernel then walks the
// sorted order 32 points per warp, each lane owning 4 consecutive columns,
// accumulating in float32 registers and flushing one (vector) atomic per run
// boundary.  The finalize kernel divides, keeps empty clusters, casts, and
// also produces the next iteration's ||c||^2 and the centre shift.
#include "fk_common.cuh"

namespace fk {

template <typename I>
__global__ void hist_kernel(const I* __restrict__ ids, int64_t sib, int64_t sin, int N, int K,
                            int64_t total, int32_t* __restrict__ hist, int* status) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = i / N, n = i % N;
    const int64_t id = static_cast<int64_t>(ids[b * sib + n * sin]);
    if (id < 0 || id >= K) {
      if (status) atomicCAS(status, 0, FK_DEV_BAD_LABEL);
      continue;
    }
    atomicAdd(hist + b * K + id, 1);
  }
}

// One 1024-thread block per batch: offs = exclusive scan of hist, cursor =
// offs, counts += hist.
__global__ void scan_kernel(const int32_t* __restrict__ hist, int32_t* __restrict__ offs,
                            int32_t* __restrict__ cursor, int32_t* __restrict__ counts, int K) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry_s;
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int32_t* h = hist + static_cast<int64_t>(b) * K;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (int base = 0; base < K; base += blockDim.x) {
    const int k = base + tid;
    const int32_t v = k < K ? h[k] : 0;
    int32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[w] = incl;
    __syncthreads();
    if (w == 0) {
      const int nw = blockDim.x >> 5;
      int32_t t = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      if (lane < nw) warp_tot[lane] = t;  // inclusive over warps
    }
    __syncthreads();
    const int32_t carry = carry_s;
    const int32_t before = (w > 0 ? warp_tot[w - 1] : 0) + incl - v;
    if (k < K) {
      const int64_t o = static_cast<int64_t>(b) * K + k;
      offs[o] = carry + before;
      cursor[o] = carry + before;
      if (counts) counts[o] += v;
    }
    __syncthreads();
    if (tid == blockDim.x - 1) carry_s = carry + warp_tot[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
}

template <typename I>
__global__ void scatter_kernel(const I* __restrict__ ids, int64_t sib, int64_t sin, int N, int K,
                               int64_t total, int32_t* __restrict__ cursor,
                               int32_t* __restrict__ perm, int32_t* __restrict__ sid) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = i / N, n = i % N;
    const int64_t id = static_cast<int64_t>(ids[b * sib + n * sin]);
    if (id < 0 || id >= K) continue;
    const int32_t pos = atomicAdd(cursor + b * K + id, 1);
    perm[b * N + pos] = static_cast<int32_t>(n);
    sid[b * N + pos] = static_cast<int32_t>(id);
  }
}

// 16-byte vector of T: raw load, then widen-and-add into float accumulators.
template <typename T>
struct Vec16 {
  static constexpr int kElems = 16 / sizeof(T);
  __device__ __forceinline__ static uint4 load(const T* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
  }
  __device__ __forceinline__ static void add(float (&acc)[kElems], const uint4& u);
};
template <>
__device__ __forceinline__ void Vec16<__half>::add(float (&acc)[8], const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}
template <>
__device__ __forceinline__ void Vec16<__nv_bfloat16>::add(float (&acc)[8], const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[2 * i] += __uint_as_float(w[i] << 16);
    acc[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <>
__device__ __forceinline__ void Vec16<float>::add(float (&acc)[4], const uint4& u) {
  acc[0] += __uint_as_float(u.x);
  acc[1] += __uint_as_float(u.y);
  acc[2] += __uint_as_float(u.z);
  acc[3] += __uint_as_float(u.w);
}

constexpr int kSegWarps = 8;
constexpr int kSegPos = 64;    // sorted positions per warp
constexpr int kSegUnroll = 8;  // rows per lane group loaded before use

template <int E>
__device__ __forceinline__ void flush_run(float* dst, int d0, int D, bool vec, const float (&acc)[E]) {
  if (vec && d0 + E <= D) {
#pragma unroll
    for (int i = 0; i < E; i += 4)
      atomicAdd(reinterpret_cast<float4*>(dst + i),
                make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]));
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (d0 + e < D) atomicAdd(dst + e, acc[e]);
  }
}

// grid (ceil(N / (8 warps * 64)), column slices, B).  A warp walks 64
// consecutive sorted points.  Its lanes form 32/L groups of L lanes; a group
// owns a contiguous share of the 64 points and reads each row slice as L
// 16-byte vectors, so one load instruction fetches 32/L rows and
// kSegUnroll instructions are in flight before any value is used.  Runs of
// equal labels are summed in registers and flushed with vector atomics.
// Rows must be 16-byte aligned; columns past D inside the last vector are
// read (row padding) but never stored.
template <typename T, int L>
__global__ void __launch_bounds__(kSegWarps * 32)
    segsum_kernel(const T* __restrict__ x, int64_t sxb, int64_t sxn,
                  const int32_t* __restrict__ perm, const int32_t* __restrict__ sid,
                  const int32_t* __restrict__ offs, const int32_t* __restrict__ hist, int N, int K,
                  int D, float* __restrict__ sums, bool vflush) {
  constexpr int E = Vec16<T>::kElems;
  constexpr int G = 32 / L;          // row groups per warp
  constexpr int PG = kSegPos / G;    // points per group
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t hb = static_cast<int64_t>(b) * K;
  const int total_b = offs[hb + K - 1] + hist[hb + K - 1];
  const int p0 = blockIdx.x * (kSegWarps * kSegPos) + warp * kSegPos;
  if (p0 >= total_b) return;
  const int np = min(kSegPos, total_b - p0);
  const int64_t pb = static_cast<int64_t>(b) * N + p0;
  int my_n0 = 0, my_n1 = 0, my_i0 = -1, my_i1 = -1;
  if (lane < np) { my_n0 = __ldg(perm + pb + lane); my_i0 = __ldg(sid + pb + lane); }
  if (lane + 32 < np) { my_n1 = __ldg(perm + pb + lane + 32); my_i1 = __ldg(sid + pb + lane + 32); }
  const int g = lane / L;
  const int d0 = blockIdx.y * (L * E) + (lane % L) * E;
  const bool lane_active = d0 < D;
  const int ng = max(0, min(PG, np - g * PG));  // points of this lane's group
  const T* xb = x + b * sxb;
  auto fetch = [&](int q, int a0, int a1) {  // value of position q from a per-lane pair
    const int s0 = __shfl_sync(0xffffffffu, a0, q & 31);
    const int s1 = __shfl_sync(0xffffffffu, a1, q & 31);
    return (q >> 5) ? s1 : s0;
  };
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  int cur = fetch(g * PG, my_i0, my_i1);
  const int steps = min(PG, np);  // group 0 has the most points
  for (int j0 = 0; j0 < steps; j0 += kSegUnroll) {
    uint4 v[kSegUnroll];
#pragma unroll
    for (int u = 0; u < kSegUnroll; ++u) {
      const int j = j0 + u;
      const int n = fetch(g * PG + (j < PG ? j : 0), my_n0, my_n1);
      v[u] = (j < ng && lane_active) ? Vec16<T>::load(xb + static_cast<int64_t>(n) * sxn + d0)
                                     : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kSegUnroll; ++u) {
      const int j = j0 + u;
      const int id = fetch(g * PG + (j < PG ? j : 0), my_i0, my_i1);
      if (j < ng) {
        if (id != cur) {
          if (lane_active) flush_run<E>(sums + (hb + cur) * D + d0, d0, D, vflush, acc);
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] = 0.f;
          cur = id;
        }
        Vec16<T>::add(acc, v[u]);
      }
    }
  }
  if (ng > 0 && lane_active) flush_run<E>(sums + (hb + cur) * D + d0, d0, D, vflush, acc);
}

// Fallback for rows that are not 16-byte aligned: one warp per 64 points,
// lane = column (strided), scalar loads.
template <typename T>
__global__ void __launch_bounds__(kSegWarps * 32)
    segsum_scalar_kernel(const T* __restrict__ x, int64_t sxb, int64_t sxn, int64_t sxd,
                         const int32_t* __restrict__ perm, const int32_t* __restrict__ sid,
                         const int32_t* __restrict__ offs, const int32_t* __restrict__ hist, int N,
                         int K, int D, float* __restrict__ sums) {
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t hb = static_cast<int64_t>(b) * K;
  const int total_b = offs[hb + K - 1] + hist[hb + K - 1];
  const int p0 = blockIdx.x * (kSegWarps * kSegPos) + warp * kSegPos;
  if (p0 >= total_b) return;
  const int np = min(kSegPos, total_b - p0);
  const int64_t pb = static_cast<int64_t>(b) * N + p0;
  const T* xb = x + b * sxb;
  for (int d = blockIdx.y * 32 + lane; d < D; d += 32 * gridDim.y) {
    float acc = 0.f;
    int cur = __ldg(sid + pb);
    for (int j = 0; j < np; ++j) {
      const int id = __ldg(sid + pb + j);
      if (id != cur) {
        atomicAdd(sums + (hb + cur) * D + d, acc);
        acc = 0.f;
        cur = id;
      }
      acc += Elem<T>::to_f(xb[static_cast<int64_t>(__ldg(perm + pb + j)) * sxn + d * sxd]);
    }
    atomicAdd(sums + (hb + cur) * D + d, acc);
  }
}

// One warp per (b, k): reference finalize (centroid_update_triton.py:378-385,
// torch_fallback.py:101-108) plus ||c_new||^2 and the shift.  Lane l owns
// columns 4l..4l+3 of every 128-column slice (float4 loads of the sums).
template <typename T>
__device__ __forceinline__ void fin_elem(float sumv, int32_t cnt, float fc, T ov, T* dst,
                                         float& ss, float& cs) {
  const T nv = cnt > 0 ? Elem<T>::from_f(sumv / fc) : ov;
  *dst = nv;
  const float nf = Elem<T>::to_f(nv);
  const float df = Elem<T>::round(nf - Elem<T>::to_f(ov));
  ss += df * df;
  cs += Elem<T>::round(nf * nf);
}

template <typename T>
__global__ void finalize_kernel(float* __restrict__ sums, int32_t* __restrict__ counts,
                                const T* __restrict__ old, int64_t sob, int64_t sok, int64_t sod,
                                T* __restrict__ out, int64_t snb, int64_t snk, int64_t snd, int B,
                                int K, int D, float* __restrict__ csq_out,
                                float* __restrict__ shift_out, bool reset) {
  const int wpb = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(B) * K;
  const bool vec = (D % 4 == 0) && sod == 1 && snd == 1;
  float wmax = 0.f;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5); r < rows;
       r += static_cast<int64_t>(gridDim.x) * wpb) {
    const int64_t b = r / K, k = r % K;
    const int32_t cnt = counts[r];
    const float fc = static_cast<float>(cnt);
    float* s = sums + r * D;
    const T* o = old + b * sob + k * sok;
    T* nw = out + b * snb + k * snk;
    float ss = 0.f, cs = 0.f;
    if (vec) {
      for (int d = lane * 4; d < D; d += 128) {
        const float4 sv = *reinterpret_cast<const float4*>(s + d);
        if (reset) *reinterpret_cast<float4*>(s + d) = make_float4(0.f, 0.f, 0.f, 0.f);
        const float svs[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) fin_elem<T>(svs[e], cnt, fc, o[d + e], nw + d + e, ss, cs);
      }
    } else {
      for (int d = lane; d < D; d += 32) {
        const float sv = s[d];
        if (reset) s[d] = 0.f;
        fin_elem<T>(sv, cnt, fc, o[d * sod], nw + d * snd, ss, cs);
      }
    }
    ss = warp_sum(ss);
    cs = warp_sum(cs);
    if (reset && lane == 0) counts[r] = 0;
    if (lane == 0) {
      if (csq_out) csq_out[r] = Elem<T>::round(cs);
      wmax = fmaxf(wmax, Elem<T>::round(sqrtf(ss)));
    }
  }
  // one atomic per block for the shift (non-negative floats order as uints)
  __shared__ float blk_max[32];
  if (lane == 0) blk_max[threadIdx.x >> 5] = wmax;
  __syncthreads();
  if (threadIdx.x == 0 && shift_out) {
    float m = 0.f;
    for (int w = 0; w < wpb; ++w) m = fmaxf(m, blk_max[w]);
    atomicMax(reinterpret_cast<unsigned int*>(shift_out), __float_as_uint(m));
  }
}

static int grid_for(int64_t work, int per_block, int cap_per_sm) {
  int64_t blocks = (work + per_block - 1) / per_block;
  const int sms = sm_count_current();
  const int64_t cap = sms > 0 ? static_cast<int64_t>(sms) * cap_per_sm : 4096;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

template <typename I>
static int hist_scatter(const void* ids, const int64_t* is, int64_t B, int64_t N, int64_t K,
                        int32_t* hist, bool do_hist, int32_t* offs, int32_t* cursor, int32_t* perm,
                        int32_t* sid, int32_t* counts, int32_t* status, cudaStream_t s) {
  const int64_t total = B * N;
  const I* id = static_cast<const I*>(ids);
  if (do_hist) {
    hist_kernel<I><<<grid_for(total, 256, 8), 256, 0, s>>>(id, is[0], is[1], (int)N, (int)K, total,
                                                           hist, status);
    int st = check_launch("hist_kernel");
    if (st) return st;
  }
  scan_kernel<<<static_cast<int>(B), 1024, 0, s>>>(hist, offs, cursor, counts, (int)K);
  int st = check_launch("scan_kernel");
  if (st) return st;
  scatter_kernel<I><<<grid_for(total, 256, 8), 256, 0, s>>>(id, is[0], is[1], (int)N, (int)K, total,
                                                             cursor, perm, sid);
  return check_launch("scatter_kernel");
}

template <typename T, int L>
static void launch_segsum(const T* x, const int64_t* xs, int64_t B, int64_t N, int64_t K, int64_t D,
                          const int32_t* perm, const int32_t* sid, const int32_t* offs,
                          const int32_t* hist, float* sums, bool vflush, cudaStream_t s) {
  constexpr int E = 16 / sizeof(T);
  dim3 grid(static_cast<unsigned>((N + kSegWarps * kSegPos - 1) / (kSegWarps * kSegPos)),
            static_cast<unsigned>((D + L * E - 1) / (L * E)), static_cast<unsigned>(B));
  segsum_kernel<T, L><<<grid, kSegWarps * 32, 0, s>>>(x, xs[0], xs[1], perm, sid, offs, hist,
                                                      (int)N, (int)K, (int)D, sums, vflush);
}

template <typename T>
static int segsum_typed(const void* x, const int64_t* xs, int64_t B, int64_t N, int64_t K,
                        int64_t D, const int32_t* perm, const int32_t* sid, const int32_t* offs,
                        const int32_t* hist, float* sums, cudaStream_t s) {
  constexpr int E = 16 / sizeof(T);
  const bool vload = xs[2] == 1 && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                     ((xs[1] * static_cast<int64_t>(sizeof(T))) % 16 == 0) &&
                     ((xs[0] * static_cast<int64_t>(sizeof(T))) % 16 == 0 || B == 1) &&
                     xs[1] >= (D + E - 1) / E * E;
  const bool vflush = (D % 4 == 0) && (reinterpret_cast<uintptr_t>(sums) % 16 == 0);
  const T* xt = static_cast<const T*>(x);
  if (vload) {
    const int64_t vecs = (D + E - 1) / E;  // 16-byte vectors per row
    if (vecs <= 8)
      launch_segsum<T, 8>(xt, xs, B, N, K, D, perm, sid, offs, hist, sums, vflush, s);
    else if (vecs <= 16)
      launch_segsum<T, 16>(xt, xs, B, N, K, D, perm, sid, offs, hist, sums, vflush, s);
    else
      launch_segsum<T, 32>(xt, xs, B, N, K, D, perm, sid, offs, hist, sums, vflush, s);
  } else {
    dim3 grid(static_cast<unsigned>((N + kSegWarps * kSegPos - 1) / (kSegWarps * kSegPos)),
              static_cast<unsigned>(D > 32 * 16 ? 16 : (D + 31) / 32), static_cast<unsigned>(B));
    segsum_scalar_kernel<T><<<grid, kSegWarps * 32, 0, s>>>(xt, xs[0], xs[1], xs[2], perm, sid,
                                                           offs, hist, (int)N, (int)K, (int)D, sums);
  }
  return check_launch("segsum_kernel");
}

}  // namespace fk

using namespace fk;

// workspace: hist | offs | cursor (B*K int32 each) | perm | sid (B*N int32 each)
extern "C" size_t fk_centroid_accumulate_workspace_size(int64_t B, int64_t N, int64_t K) {
  if (B <= 0 || N < 0 || K <= 0) return 256;
  const size_t bk = align_up(static_cast<size_t>(B * K) * 4, 256);
  const size_t bn = align_up(static_cast<size_t>(B * N) * 4, 256);
  return 3 * bk + 2 * bn + 256;
}

extern "C" int fk_centroid_accumulate(const void* x, int dtype, int64_t B, int64_t N, int64_t K,
                                      int64_t D, const int64_t* x_strides3, const void* ids,
                                      int ids_dtype, const int64_t* ids_strides2,
                                      const int32_t* hist, float* sums, int32_t* counts,
                                      void* workspace, size_t workspace_bytes,
                                      int32_t* dev_status, void* stream) {
  if (B < 0 || N < 0 || K <= 0 || D <= 0)
    return fail(FK_ERR_INVALID_ARG, "fk_centroid_accumulate: bad sizes");
  if (B == 0 || N == 0) return FK_OK;
  if (!x || !ids || !sums || !counts || !x_strides3 || !ids_strides2)
    return fail(FK_ERR_INVALID_ARG, "fk_centroid_accumulate: null pointer argument");
  if (ids_dtype != FK_I32 && ids_dtype != FK_I64)
    return fail(FK_ERR_INVALID_ARG, "fk_centroid_accumulate: ids must be int32 or int64");
  if (N >= (1ll << 31) || K >= (1ll << 31) || B >= 65536)
    return fail(FK_ERR_UNSUPPORTED, "fk_centroid_accumulate: sizes exceed kernel limits");
  const size_t need = fk_centroid_accumulate_workspace_size(B, N, K);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(FK_ERR_WORKSPACE, "fk_centroid_accumulate: workspace needs %zu bytes", need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  const size_t bk = align_up(static_cast<size_t>(B * K) * 4, 256);
  const size_t bn = align_up(static_cast<size_t>(B * N) * 4, 256);
  int32_t* whist = reinterpret_cast<int32_t*>(w);
  int32_t* offs = reinterpret_cast<int32_t*>(w + bk);
  int32_t* cursor = reinterpret_cast<int32_t*>(w + 2 * bk);
  int32_t* perm = reinterpret_cast<int32_t*>(w + 3 * bk);
  int32_t* sid = reinterpret_cast<int32_t*>(w + 3 * bk + bn);
  const bool do_hist = hist == nullptr;
  int32_t* h = do_hist ? whist : const_cast<int32_t*>(hist);
  if (counts == h) counts = nullptr;  // counts already is this call's histogram
  if (do_hist) {
    cudaError_t e = cudaMemsetAsync(whist, 0, static_cast<size_t>(B * K) * 4, s);
    if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  }
  int st = ids_dtype == FK_I32
               ? hist_scatter<int32_t>(ids, ids_strides2, B, N, K, h, do_hist, offs, cursor, perm,
                                       sid, counts, dev_status, s)
               : hist_scatter<int64_t>(ids, ids_strides2, B, N, K, h, do_hist, offs, cursor, perm,
                                       sid, counts, dev_status, s);
  if (st) return st;
  switch (dtype) {
    case FK_F16:
      return segsum_typed<__half>(x, x_strides3, B, N, K, D, perm, sid, offs, h, sums, s);
    case FK_BF16:
      return segsum_typed<__nv_bfloat16>(x, x_strides3, B, N, K, D, perm, sid, offs, h, sums, s);
    case FK_F32:
      return segsum_typed<float>(x, x_strides3, B, N, K, D, perm, sid, offs, h, sums, s);
    default:
      return fail(FK_ERR_INVALID_ARG, "fk_centroid_accumulate: unsupported dtype %d", dtype);
  }
}

extern "C" int fk_centroid_finalize(float* sums, int32_t* counts, const void* old_centroids,
                                    void* new_centroids, int dtype, int64_t B, int64_t K,
                                    int64_t D, const int64_t* old_strides3,
                                    const int64_t* new_strides3, float* csq_out, float* shift_out,
                                    int reset_accumulators, void* stream) {
  if (B < 0 || K <= 0 || D <= 0) return fail(FK_ERR_INVALID_ARG, "fk_centroid_finalize: bad sizes");
  if (!sums || !counts || !old_centroids || !new_centroids || !old_strides3 || !new_strides3)
    return fail(FK_ERR_INVALID_ARG, "fk_centroid_finalize: null pointer argument");
  if (old_centroids == new_centroids)
    return fail(FK_ERR_INVALID_ARG, "fk_centroid_finalize: new_centroids aliases old_centroids");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (shift_out) {
    cudaError_t e = cudaMemsetAsync(shift_out, 0, sizeof(float), s);
    if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  }
  if (B == 0) return FK_OK;
  const int64_t rows = B * K;
  const int grid = grid_for(rows, 8, 16);
  const int64_t* os = old_strides3;
  const int64_t* ns = new_strides3;
  switch (dtype) {
    case FK_F16:
      finalize_kernel<__half><<<grid, 256, 0, s>>>(
          sums, counts, static_cast<const __half*>(old_centroids), os[0], os[1], os[2],
          static_cast<__half*>(new_centroids), ns[0], ns[1], ns[2], (int)B, (int)K, (int)D, csq_out,
          shift_out, reset_accumulators != 0);
      break;
    case FK_BF16:
      finalize_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          sums, counts, static_cast<const __nv_bfloat16*>(old_centroids), os[0], os[1], os[2],
          static_cast<__nv_bfloat16*>(new_centroids), ns[0], ns[1], ns[2], (int)B, (int)K, (int)D,
          csq_out, shift_out, reset_accumulators != 0);
      break;
    case FK_F32:
      finalize_kernel<float><<<grid, 256, 0, s>>>(
          sums, counts, static_cast<const float*>(old_centroids), os[0], os[1], os[2],
          static_cast<float*>(new_centroids), ns[0], ns[1], ns[2], (int)B, (int)K, (int)D, csq_out,
          shift_out, reset_accumulators != 0);
      break;
    default:
      return fail(FK_ERR_INVALID_ARG, "fk_centroid_finalize: unsupported dtype %d", dtype);
  }
  return check_launch("finalize_kernel");
}
