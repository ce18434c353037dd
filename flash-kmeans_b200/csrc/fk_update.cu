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
// boundary.  When one batch's K x D float32 sums fit in shared memory no sort
// is needed: each CTA accumulates its contiguous range of points privately in
// shared memory and adds its partial sums to the global ones once.  The
// finalize kernel divides, keeps empty clusters, casts, and also produces the
// next iteration's ||c||^2 and the centre shift.
#include <algorithm>
#include <type_traits>

#include "fk_common.cuh"
#include "fk_ptx.cuh"

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

constexpr int kSegWarps = 8;
constexpr int kSegPos = 64;  // sorted positions per warp (scalar fallback)

// ---------------------------------------------------------------------------
// Gathered segmented sums with bulk copies.  Block = 1 producer warp + 4
// consumer warps and handles a contiguous range of sorted positions of one
// batch and one column slice (grid (chunks, slices, B)).  The range is cut in
// stages of R rows; consumer warp w owns a contiguous run of stages and two
// private ring slots (double buffer).  The producer warp fetches the stage's
// point indices (one per lane) and each lane issues one cp.async.bulk of its
// row slice into the slot, completion counted in bytes on the slot's "full"
// mbarrier -- hundreds of rows in flight per SM without register cost.  A
// consumer sums runs of equal labels from shared memory (lane owns 4
// consecutive columns of each 128-column sub-chunk) and flushes one vector
// atomic per lane at each run boundary and at the end.
// ---------------------------------------------------------------------------
constexpr int kBulkConsumers = 4;
constexpr int kBulkSlots = 2 * kBulkConsumers;
constexpr int kBulkThreads = (1 + kBulkConsumers) * 32;
constexpr int kBulkStageBytes = 8192;

struct BulkParams {
  int64_t sxb, sxn;          // element strides of x (batch, row); unit column stride
  const int32_t* perm;       // (B, N) sorted point index
  const int32_t* sid;        // (B, N) sorted label
  const int32_t* offs;       // (B, K) exclusive scan of hist
  const int32_t* hist;       // (B, K)
  float* sums;               // (B, K, D)
  int N, K, D;
  int slice_elems;           // columns per slice (grid.y)
  int slice_bytes;           // smem bytes reserved per row (multiple of 16)
  int rows;                  // R rows per stage
  int pos_per_block;
  bool vflush;
  int* status;
};

template <typename T, int NSUB>
__global__ void __launch_bounds__(kBulkThreads)
    segsum_bulk_kernel(const T* __restrict__ x, const BulkParams p) {
  extern __shared__ __align__(128) uint8_t sm_raw[];
  uint8_t* slots = sm_raw;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm_raw + kBulkSlots * kBulkStageBytes);
  uint64_t* empty = full + kBulkSlots;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kBulkSlots);
  constexpr int esz = sizeof(T);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const int slice0 = blockIdx.y * p.slice_elems;
  const int64_t hb = static_cast<int64_t>(b) * p.K;
  const int total_b = p.offs[hb + p.K - 1] + p.hist[hb + p.K - 1];
  const int P0 = blockIdx.x * p.pos_per_block;
  const int P1 = min(P0 + p.pos_per_block, total_b);
  if (P0 >= P1) return;  // whole block leaves before any barrier is used
  const int R = p.rows;
  const int nst = (P1 - P0 + R - 1) / R;
  const int per = (nst + kBulkConsumers - 1) / kBulkConsumers;
  // bytes actually copied per row: the slice, cut at the 16-byte-padded row end
  const int rem = (p.D - slice0) * esz;
  const int copy_bytes = min(p.slice_bytes, (rem + 15) & ~15);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kBulkSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 32);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int last_par[kBulkSlots];
    for (int i = 0; i < kBulkSlots; ++i) last_par[i] = -1;
    bool ok = true;
    const T* xb = x + b * p.sxb + slice0;
    const int32_t* pm = p.perm + static_cast<int64_t>(b) * p.N;
    // Issue order: round r of every consumer, r = 0, 1, ...  The point indices
    // of the next stage are loaded before waiting for the current slot.
    const int nissue = per * kBulkConsumers;
    auto stage_of = [&](int j, int& t, int& slot, uint32_t& ph) {
      const int r = j / kBulkConsumers, w = j % kBulkConsumers;
      t = w * per + r;
      slot = 2 * w + (r & 1);
      ph = static_cast<uint32_t>((r >> 1) & 1);
      return t < min((w + 1) * per, nst);
    };
    auto load_idx = [&](int t, int& a, int& c) {
      const int q0 = P0 + t * R;
      const int nr = min(R, P1 - q0);
      a = lane < nr ? __ldg(pm + q0 + lane) : 0;
      c = lane + 32 < nr ? __ldg(pm + q0 + 32 + lane) : 0;
    };
    int na = 0, nc = 0, t_nx = 0, slot_nx = 0;
    uint32_t ph_nx = 0;
    int j = 0;
    while (j < nissue && !stage_of(j, t_nx, slot_nx, ph_nx)) ++j;
    if (j < nissue) load_idx(t_nx, na, nc);
    while (ok && j < nissue) {
      const int t = t_nx, slot = slot_nx;
      const uint32_t ph = ph_nx;
      const int ca = na, cc = nc;
      int jn = j + 1;
      while (jn < nissue && !stage_of(jn, t_nx, slot_nx, ph_nx)) ++jn;
      if (jn < nissue) load_idx(t_nx, na, nc);  // in flight during the wait below
      j = jn;
      const bool got = mbar_wait(&empty[slot], ph ^ 1, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      const int q0 = P0 + t * R;
      const int nr = min(R, P1 - q0);
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(nr * copy_bytes));
      __syncwarp();
      uint8_t* dst = slots + slot * kBulkStageBytes;
      if (lane < nr)
        bulk_load(dst + lane * p.slice_bytes, xb + static_cast<int64_t>(ca) * p.sxn,
                  static_cast<uint32_t>(copy_bytes), &full[slot]);
      if (lane + 32 < nr)
        bulk_load(dst + (lane + 32) * p.slice_bytes, xb + static_cast<int64_t>(cc) * p.sxn,
                  static_cast<uint32_t>(copy_bytes), &full[slot]);
      if (lane == 0) last_par[slot] = static_cast<int>(ph);
    }
    if (!ok && lane == 0) {
      for (int i = 0; i < kBulkSlots; ++i) {
        if (last_par[i] < 0) continue;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[i], static_cast<uint32_t>(last_par[i])) &&
               globaltimer_ns() - t0 < 200000000ull) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int w = warp - 1;
    const int t_begin = w * per;
    const int t_end = min(t_begin + per, nst);
    float acc[NSUB][4];
#pragma unroll
    for (int s2 = 0; s2 < NSUB; ++s2)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[s2][e] = 0.f;
    int cur = -1;
    auto flush = [&](int id) {
#pragma unroll
      for (int s2 = 0; s2 < NSUB; ++s2) {
        const int col = slice0 + s2 * 128 + lane * 4;
        float* dst = p.sums + (hb + id) * p.D + col;
        if (col + 4 <= p.D && col - slice0 + 4 <= p.slice_elems && p.vflush) {
          atomicAdd(reinterpret_cast<float4*>(dst),
                    make_float4(acc[s2][0], acc[s2][1], acc[s2][2], acc[s2][3]));
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (col + e < p.D && col - slice0 + e < p.slice_elems) atomicAdd(dst + e, acc[s2][e]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[s2][e] = 0.f;
      }
    };
    const int32_t* sd = p.sid + static_cast<int64_t>(b) * p.N;
    for (int t = t_begin, r = 0; t < t_end; ++t, ++r) {
      const int slot = 2 * w + (r & 1);
      const uint32_t ph = static_cast<uint32_t>((r >> 1) & 1);
      const int q0 = P0 + t * R;
      const int nr = min(R, P1 - q0);
      const int id_lo = lane < nr ? __ldg(sd + q0 + lane) : -1;
      const int id_hi = lane + 32 < nr ? __ldg(sd + q0 + 32 + lane) : -1;
      const bool got = mbar_wait(&full[slot], ph, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT);
      if (!__all_sync(0xffffffffu, got)) break;
      const uint8_t* base = slots + slot * kBulkStageBytes;
      // add row i's slice (lane's 4 columns of each 128-column sub-chunk)
      auto add_row = [&](float (&a)[NSUB][4], int i) {
        const uint8_t* row = base + i * p.slice_bytes;
#pragma unroll
        for (int s2 = 0; s2 < NSUB; ++s2) {
          const int off = (s2 * 128 + lane * 4) * esz;
          if (off < p.slice_bytes) {
            if constexpr (esz == 2) {
              const uint2 u = *reinterpret_cast<const uint2*>(row + off);
              if constexpr (std::is_same<T, __half>::value) {
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
                a[s2][0] += f0.x; a[s2][1] += f0.y; a[s2][2] += f1.x; a[s2][3] += f1.y;
              } else {
                a[s2][0] += __uint_as_float(u.x << 16); a[s2][1] += __uint_as_float(u.x & 0xFFFF0000u);
                a[s2][2] += __uint_as_float(u.y << 16); a[s2][3] += __uint_as_float(u.y & 0xFFFF0000u);
              }
            } else {
              const float4 u = *reinterpret_cast<const float4*>(row + off);
              a[s2][0] += u.x; a[s2][1] += u.y; a[s2][2] += u.z; a[s2][3] += u.w;
            }
          }
        }
      };
      auto id_at = [&](int i) {
        return __shfl_sync(0xffffffffu, i < 32 ? id_lo : id_hi, i & 31);
      };
      int i = 0;
      while (i < nr) {
        const int id = id_at(i);
        if (id != cur) {
          if (cur >= 0) flush(cur);
          cur = id;
        }
        // labels are sorted: rows i..i+7 share a label iff rows i and i+7 do.
        // Then sum them with independent loads into a second accumulator.
        if (i + 8 <= nr && id_at(i + 7) == id) {
          float t8[NSUB][4];
#pragma unroll
          for (int s2 = 0; s2 < NSUB; ++s2)
#pragma unroll
            for (int e = 0; e < 4; ++e) t8[s2][e] = 0.f;
#pragma unroll
          for (int u = 0; u < 8; u += 2) {
            add_row(acc, i + u);
            add_row(t8, i + u + 1);
          }
#pragma unroll
          for (int s2 = 0; s2 < NSUB; ++s2)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[s2][e] += t8[s2][e];
          i += 8;
        } else {
          add_row(acc, i);
          i += 1;
        }
      }
      mbar_arrive(&empty[slot]);
    }
    if (cur >= 0) flush(cur);
  }
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

// Four consecutive elements of T as one vector load / store.
template <typename T>
struct Quad;
template <>
struct Quad<__half> {
  __device__ __forceinline__ static void load(const __half* p, float (&f)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    f[0] = a.x; f[1] = a.y; f[2] = c.x; f[3] = c.y;
  }
  __device__ __forceinline__ static void store(__half* p, const float (&f)[4]) {
    const __half2 a = __floats2half2_rn(f[0], f[1]), c = __floats2half2_rn(f[2], f[3]);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&c);
    *reinterpret_cast<uint2*>(p) = u;
  }
};
template <>
struct Quad<__nv_bfloat16> {
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float (&f)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    f[0] = __uint_as_float(u.x << 16); f[1] = __uint_as_float(u.x & 0xFFFF0000u);
    f[2] = __uint_as_float(u.y << 16); f[3] = __uint_as_float(u.y & 0xFFFF0000u);
  }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, const float (&f)[4]) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]), c = __floats2bfloat162_rn(f[2], f[3]);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&c);
    *reinterpret_cast<uint2*>(p) = u;
  }
};
template <>
struct Quad<float> {
  __device__ __forceinline__ static void load(const float* p, float (&f)[4]) {
    const float4 u = *reinterpret_cast<const float4*>(p);
    f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
  }
  __device__ __forceinline__ static void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};

// One warp per (b, k) row: the reference finalize (centroid_update_triton.py:378-385,
// torch_fallback.py:101-108) -- new = cnt ? sums / cnt : old, cast -- plus the
// next ||c||^2 with the reference's rounding, the row's shift
// round(||round(new - old)||), and optionally zeroing sums/counts for the next
// iteration.  Vector path: lane owns 4 consecutive columns per 128.
template <typename T>
__global__ void finalize_kernel(float* __restrict__ sums, int32_t* __restrict__ counts,
                                const T* __restrict__ old, int64_t sob, int64_t sok, int64_t sod,
                                T* __restrict__ out, int64_t snb, int64_t snk, int64_t snd, int B,
                                int K, int D, float* __restrict__ csq_out,
                                float* __restrict__ shift_out, bool reset, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t wpb = blockDim.x >> 5;
  float wmax = 0.f;
  // warp per row, grid-stride; the shift below costs one same-address atomic
  // per block
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5);
       r < static_cast<int64_t>(B) * K; r += static_cast<int64_t>(gridDim.x) * wpb) {
    const int64_t b = r / K, k = r % K;
    const int32_t cnt = counts[r];
    const float fc = static_cast<float>(cnt);
    float* s = sums + r * D;
    const T* o = old + b * sob + k * sok;
    T* nw = out + b * snb + k * snk;
    float ss = 0.f, cs = 0.f;
    if (vec) {
      for (int d = lane * 4; d < D; d += 128) {
        float sv[4], ov[4], nv[4];
        Quad<float>::load(s + d, sv);
        Quad<T>::load(o + d, ov);
        if (reset) *reinterpret_cast<float4*>(s + d) = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          nv[e] = cnt > 0 ? Elem<T>::round(sv[e] / fc) : ov[e];
          const float df = Elem<T>::round(nv[e] - ov[e]);
          ss += df * df;
          cs += Elem<T>::round(nv[e] * nv[e]);
        }
        Quad<T>::store(nw + d, nv);
      }
    } else {
      for (int d = lane; d < D; d += 32) {
        const float sv = s[d];
        if (reset) s[d] = 0.f;
        const float ov = Elem<T>::to_f(o[d * sod]);
        const float nv = cnt > 0 ? Elem<T>::round(sv / fc) : ov;
        nw[d * snd] = Elem<T>::from_f(nv);
        const float df = Elem<T>::round(nv - ov);
        ss += df * df;
        cs += Elem<T>::round(nv * nv);
      }
    }
    ss = warp_sum(ss);
    cs = warp_sum(cs);
    if (lane == 0) {
      if (reset) counts[r] = 0;
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
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) m = fmaxf(m, blk_max[w]);
    atomicMax(reinterpret_cast<unsigned int*>(shift_out), __float_as_uint(m));
  }
}

// Cosine / dot-product finalize (_centroid_update_torch_native with
// mode='cosine', torch_fallback.py:101-109): per (b, k) row the float32 mean
// (the old centroid, as float32, when the cluster is empty) is L2-normalised
// in float32 (F.normalize: / max(||m||, 1e-12)) and cast to the dtype; the
// shift is round(||round(new - old)||) as for the Euclidean finalize.  Warp per
// row, grid-stride.
template <typename T>
__global__ void finalize_normalized_kernel(const float* __restrict__ sums,
                                           const int32_t* __restrict__ counts,
                                           const T* __restrict__ old, int64_t sob, int64_t sok,
                                           int64_t sod, T* __restrict__ out, int64_t snb,
                                           int64_t snk, int64_t snd, int B, int K, int D,
                                           float* __restrict__ shift_out) {
  const int lane = threadIdx.x & 31;
  const int64_t wpb = blockDim.x >> 5;
  float wmax = 0.f;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5);
       r < static_cast<int64_t>(B) * K; r += static_cast<int64_t>(gridDim.x) * wpb) {
    const int64_t b = r / K, k = r % K;
    const int32_t cnt = counts[r];
    const float fc = static_cast<float>(cnt);
    const float* sm = sums + r * D;
    const T* o = old + b * sob + k * sok;
    T* nw = out + b * snb + k * snk;
    float ss = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float m = cnt > 0 ? __fdiv_rn(sm[d], fc) : Elem<T>::to_f(o[d * sod]);
      ss = __fmaf_rn(m, m, ss);
    }
    const float den = fmaxf(sqrtf(warp_sum(ss)), 1e-12f);
    float ds = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float ov = Elem<T>::to_f(o[d * sod]);
      const float m = cnt > 0 ? __fdiv_rn(sm[d], fc) : ov;
      const float nv = Elem<T>::round(__fdiv_rn(m, den));
      nw[d * snd] = Elem<T>::from_f(nv);
      const float df = Elem<T>::round(nv - ov);
      ds = __fmaf_rn(df, df, ds);
    }
    ds = warp_sum(ds);
    if (lane == 0) wmax = fmaxf(wmax, Elem<T>::round(sqrtf(ds)));
  }
  __shared__ float blk_max[32];
  if (lane == 0) blk_max[threadIdx.x >> 5] = wmax;
  __syncthreads();
  if (threadIdx.x == 0 && shift_out) {
    float m = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) m = fmaxf(m, blk_max[w]);
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


// ------------------------------------------------ privatised segmented sum
// For K x D small enough that a batch's float32 sums (and K counts) fit in
// shared memory.  CTA c takes the contiguous point range
// [c*total/grid, (c+1)*total/grid) of the flattened (B, N) points, one batch
// segment at a time, in chunks of kPrivChunk points:
//   A. labels are read (coalesced) and counted per cluster with
//      warp-aggregated shared atomics (__match_any_sync: one atomic per
//      distinct label of a warp), each point getting its slot in its bin;
//   B. one warp scans the bins (and adds them to the private counts);
//   C. the chunk's point indices are scattered into label order;
//   D. each warp walks a contiguous range of that order, loading rows 4 at a
//      time (each lane 4 consecutive columns of a 128-column group) and
//      summing them in registers, with one shared-memory flush per run of
//      equal labels.
// Float atomics thus happen once per run, not once per point, so clusters
// holding most of the points (skewed data) cost least instead of
// serialising.  At the end of a segment the private sums are added to the
// global ones (one vector atomic per non-zero group of 4) and the counts with
// one atomic each.  x is read once.  The private rows are padded to a
// multiple of 128 columns and each 128-column group is stored transposed
// (column 4i+e at slot 32e+i) so a warp's flush touches 32 consecutive words
// per instruction.
constexpr int kPrivThreads = 512;
constexpr int kPrivChunk = 4096;
constexpr size_t kPrivMaxSmem = 200 * 1024;
static_assert(kPrivChunk % kPrivThreads == 0, "chunk must be a multiple of the block");

// Per-warp staging of the privatised sum: two 2 KB buffers of rows.
constexpr int kPrivStageBuf = 2048;
constexpr size_t kPrivStageBytes = static_cast<size_t>(kPrivThreads / 32) * 2 * kPrivStageBuf;

static int64_t priv_row(int64_t D) { return (D + 127) / 128 * 128; }

static size_t priv_smem_bytes(int64_t K, int64_t D) {
  return static_cast<size_t>(K * priv_row(D) + 3 * K + 3 * kPrivChunk + 4) * 4;
}

// Whether the staged (cp.async) variant applies: rows of D * esize bytes, a
// power of two between 64 bytes and one 2 KB buffer, 16-byte aligned, and
// room for the staging buffers next to the private sums.
static bool priv_staged(int64_t K, int64_t D, int64_t row_bytes, bool aligned) {
  return aligned && row_bytes >= 64 && row_bytes <= kPrivStageBuf &&
         (row_bytes & (row_bytes - 1)) == 0 &&
         align_up(priv_smem_bytes(K, D), 16) + kPrivStageBytes <= kPrivMaxSmem;
}

bool segsum_priv_fits(int64_t K, int64_t D) {
  return D <= 512 && priv_smem_bytes(K, D) <= kPrivMaxSmem;
}

// 16-byte asynchronous global -> shared copy (L2 only), and its group
// bookkeeping: a warp keeps one batch of rows in flight while it sums the
// previous one, without holding the rows in registers.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(gsrc))
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Four consecutive columns d..d+3 of a row as float (missing ones 0).
template <typename T>
__device__ __forceinline__ void load4_f(const T* row, int d, int D, int64_t sxd, bool vec,
                                        float (&f)[4]) {
  if (vec) {  // D % 4 == 0, unit stride, 4-element aligned rows
    if constexpr (std::is_same<T, float>::value) {
      const float4 v = *reinterpret_cast<const float4*>(row + d);
      f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
    } else {
      const uint2 v = *reinterpret_cast<const uint2*>(row + d);
      const T* h = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e) f[e] = Elem<T>::to_f(h[e]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) f[e] = d + e < D ? Elem<T>::to_f(row[(d + e) * sxd]) : 0.f;
  }
}

// NG = number of 128-column groups of a row (1, 2 or 4); STAGED: rows reach
// shared memory through per-warp cp.async batches (see priv_staged).
template <typename T, typename I, int NG, bool STAGED>
__global__ void __launch_bounds__(kPrivThreads) segsum_priv_kernel(
    const T* __restrict__ x, int64_t sxb, int64_t sxn, int64_t sxd, const I* __restrict__ ids,
    int64_t sib, int64_t sin, int N, int K, int D, int64_t total, float* __restrict__ sums,
    int32_t* __restrict__ counts, bool vec_x, bool vec_sums, int* status) {
  extern __shared__ float priv_sh[];
  const int R = (D + 127) / 128 * 128;  // padded row
  float* ssum = priv_sh;                                                  // [K][R]
  int* scnt = reinterpret_cast<int*>(priv_sh + static_cast<size_t>(K) * R);  // [K]
  int* bin = scnt + K;                                                    // [K]
  int* start = bin + K;                                                   // [K]
  int* slab = start + K;                                                  // [chunk] label
  int* sslot = slab + kPrivChunk;                                         // [chunk] slot in bin
  int* perm = sslot + kPrivChunk;                                         // [chunk] sorted
  int* s_nvalid = perm + kPrivChunk;
  uint8_t* wstage = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(s_nvalid + 1) + 15) & ~static_cast<uintptr_t>(15));
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * total / gridDim.x;
  const int64_t end = static_cast<int64_t>(blockIdx.x + 1) * total / gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int KD = K * D;
  const int KR = K * R;
  for (int k = threadIdx.x; k < K; k += blockDim.x) bin[k] = 0;
  int64_t p0 = begin;
  while (p0 < end) {
    const int b = static_cast<int>(p0 / N);
    const int64_t p1 = min(end, static_cast<int64_t>(b + 1) * N);  // this batch's part
    for (int i = threadIdx.x; i < KR; i += blockDim.x) ssum[i] = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) scnt[k] = 0;
    __syncthreads();
    const T* xb = x + static_cast<int64_t>(b) * sxb;
    const I* ib = ids + static_cast<int64_t>(b) * sib;
    for (int64_t c0 = p0; c0 < p1; c0 += kPrivChunk) {
      const int P = static_cast<int>(p1 - c0 < kPrivChunk ? p1 - c0 : kPrivChunk);
      const int64_t n0 = c0 - static_cast<int64_t>(b) * N;  // chunk start within the batch
      // A. labels (all of this thread's loads issued first), bin counts, slots
      constexpr int kPer = kPrivChunk / kPrivThreads;
      int64_t lraw[kPer];
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int j = r * kPrivThreads + threadIdx.x;
        lraw[r] = j < P ? static_cast<int64_t>(ib[(n0 + j) * sin]) : -1;
      }
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int j = r * kPrivThreads + threadIdx.x;
        int lab = -1;
        if (j < P) {
          const int64_t l = lraw[r];
          if (l >= 0 && l < K) lab = static_cast<int>(l);
          else if (status) atomicCAS(status, 0, FK_DEV_BAD_LABEL);
          slab[j] = lab;
        }
        const unsigned act = __ballot_sync(0xffffffffu, lab >= 0);
        if (lab >= 0) {
          const unsigned grp = __match_any_sync(act, lab);
          const int leader = __ffs(grp) - 1;
          int base = 0;
          if (lane == leader) base = atomicAdd(&bin[lab], __popc(grp));
          base = __shfl_sync(grp, base, leader);
          sslot[j] = base + __popc(grp & ((1u << lane) - 1u));
        }
      }
      __syncthreads();
      // B. exclusive scan of the bins
      if (warp == 0) {
        int carry = 0;
        for (int k0 = 0; k0 < K; k0 += 32) {
          const int k = k0 + lane;
          const int v = k < K ? bin[k] : 0;
          int incl = v;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
          }
          if (k < K) {
            start[k] = carry + incl - v;
            scnt[k] += v;
            bin[k] = 0;
          }
          carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) *s_nvalid = carry;
      }
      __syncthreads();
      // C. scatter into label order
      for (int j = threadIdx.x; j < P; j += blockDim.x) {
        const int lab = slab[j];
        if (lab >= 0) perm[start[lab] + sslot[j]] = j;
      }
      __syncthreads();
      // D. runs of equal labels, summed in registers
      const int nv = *s_nvalid;
      const int per = (nv + nwarps - 1) / nwarps;
      const int q0 = warp * per;
      const int q1 = min(nv, q0 + per);
      float acc[NG][4];
#pragma unroll
      for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
      int cur = -1;
      auto flush = [&]() {
        float* dst = ssum + cur * R + lane;  // slot 32e + lane of each group
#pragma unroll
        for (int g = 0; g < NG; ++g)
          if (g * 128 + lane * 4 < D) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              atomicAdd(dst + g * 128 + 32 * e, acc[g][e]);
              acc[g][e] = 0.f;
            }
          }
      };
      if constexpr (STAGED) {
        // Batches of RB rows (one 2 KB buffer) in sorted order; batch b+1's
        // copies are in flight while batch b is summed from shared memory.
        // The chunk is in label order, so a row's label follows from the
        // run bounds (start[] of the scan): one label lookup per run, none
        // per row, and four rows' loads issued before their adds.  A run
        // wholly inside this warp's range [q0, q1) belongs to no other warp
        // in this chunk and is flushed with plain read-add-writes; only the
        // first and last run, which a neighbour may share, use atomics
        // (shared float atomics cost about 70 cycles each).
        const int rowb = D * static_cast<int>(sizeof(T));
        const int RB = kPrivStageBuf / rowb;
        uint8_t* wst = wstage + static_cast<size_t>(warp) * 2 * kPrivStageBuf;
        auto issue = [&](int qb, int buf) {
#pragma unroll
          for (int i = 0; i < kPrivStageBuf / 512; ++i) {
            const int byte = i * 512 + lane * 16;
            const int q = qb + byte / rowb;
            if (q < q1) {
              const int j = perm[q];
              cp_async16(wst + buf * kPrivStageBuf + byte,
                         reinterpret_cast<const uint8_t*>(xb + (n0 + j) * sxn) + (byte % rowb));
            }
          }
          cp_async_commit();
        };
        auto run_end = [&](int k) { return k + 1 < K ? start[k + 1] : nv; };
        int bound = 0;
        if (q0 < q1) {
          cur = slab[perm[q0]];
          bound = run_end(cur);
        }
        auto flush_run = [&]() {
          float* dst = ssum + cur * R + lane;
          const bool own = start[cur] >= q0 && bound <= q1;
#pragma unroll
          for (int g = 0; g < NG; ++g)
            if (g * 128 + lane * 4 < D) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float* w = dst + g * 128 + 32 * e;
                if (own) *w += acc[g][e];
                else atomicAdd(w, acc[g][e]);
                acc[g][e] = 0.f;
              }
            }
        };
        if (q0 < q1) issue(q0, 0);
        int buf = 0;
        for (int qb = q0; qb < q1; qb += RB, buf ^= 1) {
          if (qb + RB < q1) issue(qb + RB, buf ^ 1);
          else cp_async_commit();  // keep one group per step
          cp_async_wait<1>();      // batch qb has landed (this lane's copies)
          __syncwarp();            // ... and every lane's
          const uint8_t* rows = wst + buf * kPrivStageBuf;
          const int nr = min(RB, q1 - qb);
          for (int r0 = 0; r0 < nr; r0 += 4) {
            float f[4][NG][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const T* row = reinterpret_cast<const T*>(rows + (r0 + u) * rowb);
#pragma unroll
              for (int g = 0; g < NG; ++g) {
                const int d = g * 128 + lane * 4;
                if (r0 + u < nr && d < D) {
                  load4_f<T>(row, d, D, 1, true, f[u][g]);
                } else {
#pragma unroll
                  for (int e = 0; e < 4; ++e) f[u][g][e] = 0.f;
                }
              }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int q = qb + r0 + u;
              if (r0 + u >= nr) break;
              if (q >= bound) {  // the run ended before q: flush it, enter q's run
                flush_run();
                cur = slab[perm[q]];
                bound = run_end(cur);
              }
#pragma unroll
              for (int g = 0; g < NG; ++g)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[g][e] += f[u][g][e];
            }
          }
          __syncwarp();  // the buffer is refilled two steps later
        }
        cp_async_wait<0>();
        if (cur >= 0) flush_run();
        cur = -1;
      } else {
      // rows loaded per warp before summing (more would lower occupancy)
      constexpr int kB = 4;
      for (int q = q0; q < q1; q += kB) {
        float f[kB][NG][4];
        int lab[kB];
#pragma unroll
        for (int u = 0; u < kB; ++u) {
          lab[u] = -1;
          if (q + u < q1) {
            const int j = perm[q + u];
            lab[u] = slab[j];
            const T* row = xb + (n0 + j) * sxn;
#pragma unroll
            for (int g = 0; g < NG; ++g) {
              const int d = g * 128 + lane * 4;
              if (d < D) load4_f<T>(row, d, D, sxd, vec_x, f[u][g]);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kB; ++u) {
          if (lab[u] < 0) continue;
          if (lab[u] != cur) {
            if (cur >= 0) flush();
            cur = lab[u];
          }
#pragma unroll
          for (int g = 0; g < NG; ++g)
            if (g * 128 + lane * 4 < D) {
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[g][e] += f[u][g][e];
            }
        }
      }
      }
      if (cur >= 0) flush();
      __syncthreads();
    }
    // private slot of (cluster k, column d): k*R + (d & ~127) + 32*(d & 3) + (d & 127)/4
    float* gs = sums + static_cast<int64_t>(b) * KD;
    if (vec_sums && D % 4 == 0) {
      for (int i = threadIdx.x * 4; i < KD; i += blockDim.x * 4) {
        const int k = i / D, d = i - k * D;  // d % 4 == 0
        const float* src = ssum + k * R + (d & ~127) + ((d & 127) >> 2);
        const float4 v = make_float4(src[0], src[32], src[64], src[96]);
        if (v.x != 0.f || v.y != 0.f || v.z != 0.f || v.w != 0.f)
          atomicAdd(reinterpret_cast<float4*>(gs + i), v);
      }
    } else {
      for (int i = threadIdx.x; i < KD; i += blockDim.x) {
        const int k = i / D, d = i - k * D;
        const float v = ssum[k * R + (d & ~127) + 32 * (d & 3) + ((d & 127) >> 2)];
        if (v != 0.f) atomicAdd(gs + i, v);
      }
    }
    if (counts) {
      int32_t* gc = counts + static_cast<int64_t>(b) * K;
      for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const int c = scnt[k];
        if (c) atomicAdd(gc + k, c);
      }
    }
    __syncthreads();
    p0 = p1;
  }
}

template <typename T, typename I, int NG, bool STAGED>
static int launch_priv_ng(const void* x, const int64_t* xs, const void* ids, const int64_t* is,
                          int64_t B, int64_t N, int64_t K, int64_t D, float* sums,
                          int32_t* counts, int32_t* status, cudaStream_t s) {
  const size_t smem = STAGED ? align_up(priv_smem_bytes(K, D), 16) + kPrivStageBytes + 16
                             : priv_smem_bytes(K, D);
  auto kern = segsum_priv_kernel<T, I, NG, STAGED>;
  static bool attr_done[64] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return fail(FK_ERR_CUDA, "segsum_priv: no current device");
  if (!attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kPrivMaxSmem));
    if (e != cudaSuccess) return fail(FK_ERR_CUDA, "segsum_priv attribute: %s", cudaGetErrorString(e));
    attr_done[dev] = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPrivThreads, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int sms = sm_count_current();
  const int64_t total = B * N;
  int64_t grid = static_cast<int64_t>(sms > 0 ? sms : 148) * per_sm;
  // each CTA zeroes and flushes K x D values per batch segment: keep a few
  // chunks of points per CTA at least
  grid = std::min<int64_t>(grid, std::max<int64_t>(1, total / (2 * kPrivChunk)));
  const bool vec_x = xs[2] == 1 && D % 4 == 0 &&
                     reinterpret_cast<uintptr_t>(x) % (4 * sizeof(T)) == 0 &&
                     (xs[1] * static_cast<int64_t>(sizeof(T))) % (4 * sizeof(T)) == 0 &&
                     (xs[0] * static_cast<int64_t>(sizeof(T))) % (4 * sizeof(T)) == 0;
  const bool vec_sums = (K * D) % 4 == 0 && reinterpret_cast<uintptr_t>(sums) % 16 == 0;
  kern<<<static_cast<int>(grid), kPrivThreads, smem, s>>>(
      static_cast<const T*>(x), xs[0], xs[1], xs[2], static_cast<const I*>(ids), is[0], is[1],
      static_cast<int>(N), static_cast<int>(K), static_cast<int>(D), total, sums, counts, vec_x,
      vec_sums, status);
  return check_launch("segsum_priv_kernel");
}

template <typename T, typename I>
static int launch_priv_typed(const void* x, const int64_t* xs, const void* ids, const int64_t* is,
                             int64_t B, int64_t N, int64_t K, int64_t D, float* sums,
                             int32_t* counts, int32_t* status, cudaStream_t s) {
  const int64_t eb = sizeof(T);
  const bool aligned = xs[2] == 1 && D % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                       (xs[1] * eb) % 16 == 0 && (B == 1 || (xs[0] * eb) % 16 == 0);
  if (priv_staged(K, D, D * eb, aligned)) {
    if (D <= 128) return launch_priv_ng<T, I, 1, true>(x, xs, ids, is, B, N, K, D, sums, counts, status, s);
    if (D <= 256) return launch_priv_ng<T, I, 2, true>(x, xs, ids, is, B, N, K, D, sums, counts, status, s);
    return launch_priv_ng<T, I, 4, true>(x, xs, ids, is, B, N, K, D, sums, counts, status, s);
  }
  if (D <= 128) return launch_priv_ng<T, I, 1, false>(x, xs, ids, is, B, N, K, D, sums, counts, status, s);
  if (D <= 256) return launch_priv_ng<T, I, 2, false>(x, xs, ids, is, B, N, K, D, sums, counts, status, s);
  return launch_priv_ng<T, I, 4, false>(x, xs, ids, is, B, N, K, D, sums, counts, status, s);
}

int segsum_priv(const void* x, int dtype, const int64_t* xs, const void* ids, int ids_dtype,
                const int64_t* is, int64_t B, int64_t N, int64_t K, int64_t D, float* sums,
                int32_t* counts, int32_t* status, cudaStream_t s) {
  const bool i32 = ids_dtype == FK_I32;
  switch (dtype) {
    case FK_F16:
      return i32 ? launch_priv_typed<__half, int32_t>(x, xs, ids, is, B, N, K, D, sums, counts, status, s)
                 : launch_priv_typed<__half, int64_t>(x, xs, ids, is, B, N, K, D, sums, counts, status, s);
    case FK_BF16:
      return i32 ? launch_priv_typed<__nv_bfloat16, int32_t>(x, xs, ids, is, B, N, K, D, sums, counts, status, s)
                 : launch_priv_typed<__nv_bfloat16, int64_t>(x, xs, ids, is, B, N, K, D, sums, counts, status, s);
    case FK_F32:
      return i32 ? launch_priv_typed<float, int32_t>(x, xs, ids, is, B, N, K, D, sums, counts, status, s)
                 : launch_priv_typed<float, int64_t>(x, xs, ids, is, B, N, K, D, sums, counts, status, s);
    default:
      return fail(FK_ERR_INVALID_ARG, "segsum_priv: unsupported dtype %d", dtype);
  }
}

template <typename T>
static int bulk_smem_attr(int nsub, int smem) {
  static bool done[4][64] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return fail(FK_ERR_CUDA, "bad current device");
  if (done[nsub - 1][dev]) return FK_OK;
  cudaError_t e;
  switch (nsub) {
    case 1: e = cudaFuncSetAttribute(segsum_bulk_kernel<T, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 2: e = cudaFuncSetAttribute(segsum_bulk_kernel<T, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    case 3: e = cudaFuncSetAttribute(segsum_bulk_kernel<T, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
    default: e = cudaFuncSetAttribute(segsum_bulk_kernel<T, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); break;
  }
  if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaFuncSetAttribute(segsum): %s", cudaGetErrorString(e));
  done[nsub - 1][dev] = true;
  return FK_OK;
}

template <typename T>
static int segsum_typed(const void* x, const int64_t* xs, int64_t B, int64_t N, int64_t K,
                        int64_t D, const int32_t* perm, const int32_t* sid, const int32_t* offs,
                        const int32_t* hist, float* sums, int* status, cudaStream_t s) {
  constexpr int E = 16 / sizeof(T);
  const bool aligned = xs[2] == 1 && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       ((xs[1] * static_cast<int64_t>(sizeof(T))) % 16 == 0) &&
                       ((xs[0] * static_cast<int64_t>(sizeof(T))) % 16 == 0 || B == 1) &&
                       xs[1] >= (D + E - 1) / E * E;
  const bool vflush = (D % 4 == 0) && (reinterpret_cast<uintptr_t>(sums) % 16 == 0);
  const T* xt = static_cast<const T*>(x);
  if (aligned) {
    // column slice: up to 512 columns and 1024 bytes, a multiple of 128 columns
    const int max_cols = (1024 / static_cast<int>(sizeof(T))) >= 512 ? 512 : 1024 / static_cast<int>(sizeof(T));
    const int64_t Dpad = (D + E - 1) / E * E;
    int slice = static_cast<int>(Dpad < max_cols ? Dpad : max_cols);
    const int nsub = (slice + 127) / 128;
    slice = slice < nsub * 128 ? slice : nsub * 128;
    const int slice_bytes = (slice * static_cast<int>(sizeof(T)) + 15) & ~15;
    BulkParams bp;
    bp.sxb = xs[0];
    bp.sxn = xs[1];
    bp.perm = perm;
    bp.sid = sid;
    bp.offs = offs;
    bp.hist = hist;
    bp.sums = sums;
    bp.N = static_cast<int>(N);
    bp.K = static_cast<int>(K);
    bp.D = static_cast<int>(D);
    bp.slice_elems = slice;
    bp.slice_bytes = slice_bytes;
    bp.rows = kBulkStageBytes / slice_bytes < 64 ? kBulkStageBytes / slice_bytes : 64;
    const int nslices = static_cast<int>((D + slice - 1) / slice);
    const int sms = sm_count_current() > 0 ? sm_count_current() : 148;
    const int64_t unit = static_cast<int64_t>(bp.rows) * kBulkConsumers;
    int64_t target_blocks = static_cast<int64_t>(sms) * 9;  // ~3 waves of 3 blocks per SM
    int64_t ppb = (N * B * nslices + target_blocks - 1) / target_blocks;
    ppb = (ppb + unit - 1) / unit * unit;
    if (ppb < unit) ppb = unit;
    bp.pos_per_block = static_cast<int>(ppb);
    bp.vflush = vflush;
    bp.status = status;
    const size_t smem = kBulkSlots * kBulkStageBytes + 2 * kBulkSlots * 8 + 16;
    int st = bulk_smem_attr<T>(nsub, static_cast<int>(smem));
    if (st != FK_OK) return st;
    dim3 grid(static_cast<unsigned>((N + ppb - 1) / ppb), static_cast<unsigned>(nslices),
              static_cast<unsigned>(B));
    switch (nsub) {
      case 1: segsum_bulk_kernel<T, 1><<<grid, kBulkThreads, smem, s>>>(xt, bp); break;
      case 2: segsum_bulk_kernel<T, 2><<<grid, kBulkThreads, smem, s>>>(xt, bp); break;
      case 3: segsum_bulk_kernel<T, 3><<<grid, kBulkThreads, smem, s>>>(xt, bp); break;
      default: segsum_bulk_kernel<T, 4><<<grid, kBulkThreads, smem, s>>>(xt, bp); break;
    }
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype != FK_F16 && dtype != FK_BF16 && dtype != FK_F32)
    return fail(FK_ERR_INVALID_ARG, "fk_centroid_accumulate: unsupported dtype %d", dtype);
  if (segsum_priv_fits(K, D)) {
    // no sort needed; `hist`, when given, is the histogram of these very ids,
    // so counting here adds the same numbers to `counts`
    return segsum_priv(x, dtype, x_strides3, ids, ids_dtype, ids_strides2, B, N, K, D, sums,
                       counts == hist ? nullptr : counts, dev_status, s);
  }
  const size_t need = fk_centroid_accumulate_workspace_size(B, N, K);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(FK_ERR_WORKSPACE, "fk_centroid_accumulate: workspace needs %zu bytes", need);
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
      return segsum_typed<__half>(x, x_strides3, B, N, K, D, perm, sid, offs, h, sums, dev_status, s);
    case FK_BF16:
      return segsum_typed<__nv_bfloat16>(x, x_strides3, B, N, K, D, perm, sid, offs, h, sums, dev_status, s);
    case FK_F32:
      return segsum_typed<float>(x, x_strides3, B, N, K, D, perm, sid, offs, h, sums, dev_status, s);
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
  // 8 rows (warps) per block, up to 16 blocks per SM: about one row per warp
  // at B*K = 32000, so every row's loads are in flight at once (4 blocks per
  // SM left each warp seven dependent rows: 16.5 us at B=32, K=1000, D=128)
  const int grid = grid_for(rows, 8, 16);
  const int64_t* os = old_strides3;
  const int64_t* ns = new_strides3;
  const int64_t eb = dtype_bytes(dtype);
  const bool vec = D % 4 == 0 && os[2] == 1 && ns[2] == 1 && os[1] % 4 == 0 && ns[1] % 4 == 0 &&
                   (os[0] % 4 == 0 || B == 1) && (ns[0] % 4 == 0 || B == 1) &&
                   reinterpret_cast<uintptr_t>(old_centroids) % (4 * eb) == 0 &&
                   reinterpret_cast<uintptr_t>(new_centroids) % (4 * eb) == 0 &&
                   reinterpret_cast<uintptr_t>(sums) % 16 == 0;
  switch (dtype) {
    case FK_F16:
      finalize_kernel<__half><<<grid, 256, 0, s>>>(
          sums, counts, static_cast<const __half*>(old_centroids), os[0], os[1], os[2],
          static_cast<__half*>(new_centroids), ns[0], ns[1], ns[2], (int)B, (int)K, (int)D, csq_out,
          shift_out, false, vec);
      break;
    case FK_BF16:
      finalize_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          sums, counts, static_cast<const __nv_bfloat16*>(old_centroids), os[0], os[1], os[2],
          static_cast<__nv_bfloat16*>(new_centroids), ns[0], ns[1], ns[2], (int)B, (int)K, (int)D,
          csq_out, shift_out, false, vec);
      break;
    case FK_F32:
      finalize_kernel<float><<<grid, 256, 0, s>>>(
          sums, counts, static_cast<const float*>(old_centroids), os[0], os[1], os[2],
          static_cast<float*>(new_centroids), ns[0], ns[1], ns[2], (int)B, (int)K, (int)D, csq_out,
          shift_out, false, vec);
      break;
    default:
      return fail(FK_ERR_INVALID_ARG, "fk_centroid_finalize: unsupported dtype %d", dtype);
  }
  int st = check_launch("finalize_kernel");
  if (st != FK_OK || !reset_accumulators) return st;
  // Zero the accumulators after the kernel has read them: a memset streams
  // the 4*B*K*D bytes at full bandwidth, while zero stores issued by the
  // finalize right behind its reads of the same (atomically updated) lines
  // tripled its time.
  cudaError_t e = cudaMemsetAsync(sums, 0, static_cast<size_t>(rows * D) * sizeof(float), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(counts, 0, static_cast<size_t>(rows) * sizeof(int32_t), s);
  if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  return FK_OK;
}

extern "C" int fk_centroid_finalize_normalized(float* sums, int32_t* counts,
                                               const void* old_centroids, void* new_centroids,
                                               int dtype, int64_t B, int64_t K, int64_t D,
                                               const int64_t* old_strides3,
                                               const int64_t* new_strides3, float* shift_out,
                                               int reset_accumulators, void* stream) {
  if (B < 0 || K <= 0 || D <= 0)
    return fail(FK_ERR_INVALID_ARG, "fk_centroid_finalize_normalized: bad sizes");
  if (!sums || !counts || !old_centroids || !new_centroids || !old_strides3 || !new_strides3)
    return fail(FK_ERR_INVALID_ARG, "fk_centroid_finalize_normalized: null pointer argument");
  if (old_centroids == new_centroids)
    return fail(FK_ERR_INVALID_ARG, "fk_centroid_finalize_normalized: new_centroids aliases old_centroids");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (shift_out) {
    cudaError_t e = cudaMemsetAsync(shift_out, 0, sizeof(float), s);
    if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  }
  if (B == 0) return FK_OK;
  const int64_t rows = B * K;
  const int grid = grid_for(rows, 8, 4);
  const int64_t* os = old_strides3;
  const int64_t* ns = new_strides3;
  switch (dtype) {
    case FK_F16:
      finalize_normalized_kernel<__half><<<grid, 256, 0, s>>>(
          sums, counts, static_cast<const __half*>(old_centroids), os[0], os[1], os[2],
          static_cast<__half*>(new_centroids), ns[0], ns[1], ns[2], (int)B, (int)K, (int)D, shift_out);
      break;
    case FK_BF16:
      finalize_normalized_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          sums, counts, static_cast<const __nv_bfloat16*>(old_centroids), os[0], os[1], os[2],
          static_cast<__nv_bfloat16*>(new_centroids), ns[0], ns[1], ns[2], (int)B, (int)K, (int)D,
          shift_out);
      break;
    case FK_F32:
      finalize_normalized_kernel<float><<<grid, 256, 0, s>>>(
          sums, counts, static_cast<const float*>(old_centroids), os[0], os[1], os[2],
          static_cast<float*>(new_centroids), ns[0], ns[1], ns[2], (int)B, (int)K, (int)D, shift_out);
      break;
    default:
      return fail(FK_ERR_INVALID_ARG, "fk_centroid_finalize_normalized: unsupported dtype %d", dtype);
  }
  int st = check_launch("finalize_normalized_kernel");
  if (st != FK_OK || !reset_accumulators) return st;
  cudaError_t e = cudaMemsetAsync(sums, 0, static_cast<size_t>(rows * D) * sizeof(float), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(counts, 0, static_cast<size_t>(rows) * sizeof(int32_t), s);
  if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  return FK_OK;
}
