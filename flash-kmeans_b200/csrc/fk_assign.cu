// Nearest-centroid assignment on sm_100a (replaces _euclid_assign_kernel and
// _euclid_assign_kernel_split_d, flash_kmeans/assign_euclid_triton.py:804-1030).
//
// One persistent CTA per SM walks a contiguous range of (batch, 128-point tile)
// work items (contiguous, so the CTAs stream different batches' centroids at
// any moment).  Per item it streams the batch's centroids in tiles of 256
// through a TMA ring and computes the 128 x 256 cross products x.c^T with
// tcgen05.mma into one of two TMEM accumulators (2 x 256 of the 512 columns),
// so the epilogue of tile j overlaps the MMAs of tile j+1.  The epilogue reads
// its TMEM lane (= its point) with tcgen05.ld, 32 columns at a time with the
// next chunk's load in flight, forms the distance with the reference torch
// path's rounding and keeps a running argmin; the (B,N,K) distance matrix
// never exists.  Nothing is written but one int32 label per point (and,
// optionally, +1 on that label's count, or with fused accumulation the point's
// row added to its cluster's float32 sum).
//
// Roles (warps): 0 = TMA producer, 1 = TMEM owner + MMA issuer, 2-3 idle
// (the three form warpgroup 0, which gives most of its registers away),
// 4..11 = epilogue (warp w reads TMEM lanes 32*(w%4).. and column half
// (w-4)/4 of each 256-column tile), then 4 more warps: f32 split converters
// (3xTF32 mode) or sum warps (fused accumulation).
//
// Modes:
//   0  16-bit x with x_sq in the same dtype: dist = r(r(x_sq - r(2 r(x.c))) + c_sq),
//      r = round to that dtype, evaluated two columns at a time on packed
//      half2 / bfloat162 registers.  This is the reference torch path's op
//      chain (torch_fallback.py:41-45) with no clamp, overflow of 2 r(x.c)
//      to inf included: the centroid operand is -2c (staged by the host), so
//      the accumulator holds -2 x.c and one conversion rounds it.
//   1  16-bit x, float32 x_sq: the same -2 x.c rounded to the 16-bit dtype (the
//      bmm output dtype), then the float32 chain (type promotion of
//      torch_fallback.py:41-45).
//   2  float32 x: cross = 3xTF32 (hi*hi + hi*lo + lo*hi, hi = tf32-rounded
//      value, lo = exact remainder, split in shared memory by the 4 extra warps),
//      float32 chain.
//   3  16-bit x, dot-product argmax (cosine / dot k-means, replaces
//      _cosine_assign_kernel, assign_euclid_triton.py:1038-1131): the float32
//      cross itself, maximised (ArgmaxSaved); padding columns are set to -inf
//      in the chunk that crosses K, so they never win even when every real
//      score is negative.  No c_sq.
//   4  float32 x, dot-product argmax with the 3xTF32 cross of mode 2.
// Split-D: when the x tile (128 points x D) does not fit twice in shared
// memory (more than two 128-byte column chunks) the x chunk travels with each
// centroid chunk instead of staying resident.
#include <atomic>
#include <mutex>
#include <type_traits>

#include "fk_common.cuh"
#include "fk_ptx.cuh"

namespace fk {

constexpr int kRows = 128;            // points per tile (MMA M)
constexpr int kCent = 256;            // centroids per tile (MMA N); 128 for K <= 128
constexpr int kTmemCols = 512;        // accumulators: kTmemCols / tile width of them
constexpr int kChunkB = 128;          // bytes per row chunk = one 128B swizzle span
constexpr int kXChunk = kRows * kChunkB;   // 16 KB
constexpr int kW64MinD = 512;          // float32 rows from here on take the 64-byte-row ring
// Warpgroup 0 = TMA producer (warp 0), MMA issuer (warp 1), two idle warps;
// warpgroups 1-2 = epilogue; warpgroup 3 (when present) = split converters or
// sum warps.  Roles follow warpgroups so each can get its own register budget.
constexpr int kEpiWarp0 = 4;           // epilogue warps start here (EPI of them)
constexpr int kConvWarps = 4;          // fp32 split warps / sum warps after the epilogue
constexpr int kResidentChunks = 2;    // resident x: at most 2 chunks (D <= 128 for 16-bit)

// Bytes of the workspace's c_sq part: B x (K padded to 256-column tiles) x 4.
inline size_t assign_csq_bytes(int64_t B, int64_t K) {
  const int64_t kpad = (K + kCent - 1) / kCent * kCent;
  return align_up(static_cast<size_t>(B * kpad * 4), 256);
}

// Modes 2 and 4 split float32 operands into tf32 hi/lo parts (converter warps).
constexpr bool split_mode(int mode) { return mode == 2 || mode == 4; }

template <int MODE, bool XRES, int STAGES, bool FUSE = false, int EPI = 8, int KC = kCent,
          bool RESC = false>
struct Layout {
  // Narrow tiles (K <= 128, resident centroids): the two epilogue warpgroups
  // take alternate point tiles and each thread reduces all 128 columns of its
  // point, so no column-group merge is needed and a warpgroup has two tile
  // periods for its tile.  Wide tiles: both warpgroups share every tile, one
  // column group each, merged through shared memory.
  static constexpr bool kAlt = RESC && KC < kCent;
  static constexpr int kGroups = kAlt ? 1 : EPI / 4;  // column groups of each centroid tile
  static constexpr int kSplit = split_mode(MODE) ? 2 : 1;  // hi/lo copies for 3xTF32
  // Rows of a chunk: 128 bytes (128-byte swizzle), or 64 bytes (64-byte
  // swizzle) in the four-stage form of the 3xTF32 modes: their stages hold hi
  // and lo copies of both operands, so four 64-byte-row stages fit where two
  // 128-byte-row ones do (used for long rows, where the deeper ring hides the
  // loads; short rows keep fewer, wider stages).
  static constexpr int kRowB = (split_mode(MODE) && STAGES == 4) ? 64 : kChunkB;
  static constexpr int kKSteps = kRowB / 32;           // MMA K steps (32 bytes) per chunk
  static constexpr int kCChunk = KC * kRowB;           // one column chunk of a centroid tile
  static constexpr int kXChunkL = kRows * kRowB;       // one column chunk of a point tile
  // Fused accumulation comes in two forms: with 256-column tiles (large K)
  // four sum warps add each point's row to its cluster's sums with vector
  // atomics; with 128-column tiles (K <= 128) the tensor core adds a one-hot
  // matrix times the tile's x into a TMEM sums accumulator (kOneHot).
  static constexpr bool kOneHot = FUSE && KC < kCent;
  static constexpr bool kSumWarps = FUSE && !kOneHot;
  // TMEM accumulators.  The one-hot form keeps 128 columns for the sums and
  // uses two accumulators, so with alternating warpgroups each accumulator
  // (and its barriers) belongs to one warpgroup: a warpgroup only waits for
  // phases whose predecessor it observed itself.
  static constexpr int kAcc = kOneHot ? 2 : kTmemCols / KC;
  static constexpr int kSumsCol = kAcc * KC;            // first TMEM column of the sums
  // resident x tile buffers: a third one lets the fused sum warps hold a tile,
  // or (narrow tiles, one centroid tile per point tile) lets x loads run
  // further ahead of the short per-tile MMA work; with resident centroids
  // (RESC) the ring is small and five x tiles fit; next to the two one-hot
  // buffers four fit (three with the shared-memory argmin slots).  A one-hot
  // tile holds its x buffer until its sums MMAs finish.
  // mode 0 keeps its saved chunk in registers in the one-hot form; the other
  // modes 0, 3 and 4 use shared-memory slots
  static constexpr bool kRegSave = kOneHot && MODE == 0;
  static constexpr bool kSmemSave = (MODE == 0 && !kRegSave) || MODE >= 3;
  static constexpr int XB = RESC ? (kOneHot ? (kSmemSave ? 3 : 4) : 5) : ((FUSE || KC < kCent) ? 3 : 2);
  static constexpr int x_off = 0;
  static constexpr int x_bytes = XRES ? XB * kResidentChunks * kXChunk : 0;
  static constexpr int st_c = 0;                          // centroid chunk (hi)
  static constexpr int st_clo = kCChunk;                  // centroid chunk lo (3xTF32, TMA-loaded)
  static constexpr int st_x = kCChunk * kSplit;           // x chunk (split-D)
  static constexpr int st_xlo = st_x + kXChunkL;          // x chunk lo (3xTF32, converter warps)
  static constexpr int stage_bytes = kCChunk * kSplit + (XRES ? 0 : kXChunkL * kSplit);
  static constexpr int stages_off = x_off + x_bytes;
  // one-hot operands [warpgroup][point chunk 0..1][centroid row][64 points],
  // 16-bit, 128-byte swizzle (K-major A operand of the sums MMA).  One buffer
  // per epilogue warpgroup: a warpgroup rewrites its buffer once the sums MMAs
  // of its previous tile (two tiles back) are done, so the two warpgroups do
  // not wait on each other's sums.
  static constexpr int kOhBufs = 2;
  static constexpr int oh_off = stages_off + STAGES * stage_bytes;
  static constexpr int oh_bytes = kOneHot ? kOhBufs * 2 * kXChunk : 0;
  static constexpr int hist_off = oh_off + oh_bytes;  // counts per epilogue warpgroup, K <= 128
  static constexpr int hist_bytes = kOneHot ? 2 * 128 * 4 : 0;
  static constexpr int merge_off = hist_off + hist_bytes;
  // [parity][group 1..G-1][row] (value, index) candidates for the merge
  static constexpr int merge_bytes = 2 * (kGroups - 1) * kRows * 8;
  static constexpr int lab_off = merge_off + merge_bytes;
  static constexpr int lab_bytes = kSumWarps ? 2 * kRows * 4 : 0;  // [parity][row] label or -1
  // modes 0, 3, 4: each epilogue thread's saved chunk (16 packed distances,
  // or 16 float32 scores), as [unit 0..3][epilogue thread] 16-byte units
  // (conflict-free stores)
  static constexpr int save_stride = EPI * 32;  // in 16-byte units
  static constexpr int save_off = lab_off + lab_bytes;
  static constexpr int save_bytes = kSmemSave ? 4 * save_stride * 16 : 0;
  static constexpr int bar_off = save_off + save_bytes;
  // x_full[XB] x_empty[XB] c_full[S] c_empty[S] conv_full[S] acc_full[A] acc_empty[A]
  // merge_full[2] merge_empty[2] lab_full[2] lab_empty[2] final[1]
  // oh_full[2] oh_empty[2] sums_full[1] sums_empty[1] wg_bar[2] sums_full_odd[1]
  static constexpr int nbars = 2 * XB + 3 * STAGES + 2 * kAcc + 4 + 4 + 1 + 9;
  static constexpr int misc_off = bar_off + nbars * 8;
  static constexpr int total = misc_off + 16 + 1024;  // + slack for 1024-byte alignment
  static constexpr bool kExtra = split_mode(MODE) || kSumWarps;  // warpgroup 3
  static constexpr int threads = (kEpiWarp0 + EPI + (kExtra ? kConvWarps : 0)) * 32;
  // Register budgets (setmaxnreg).  kLaunchRegs is what ptxas gives a thread
  // under __launch_bounds__(threads, 1); the host checks the kernel's actual
  // count before launching.  Control warps shrink to kCtlRegs, the extra
  // warpgroup to kExtraRegs, and the epilogue takes the rest (the budgets
  // are the smallest at which ptxas reports no spills for each instance).
  static constexpr int kLaunchRegs = threads == 384 ? 168 : 128;
  static constexpr int kCtlRegs = (kAlt && MODE != 0) ? 80 : 72;
  static constexpr int kExtraRegs = FUSE ? 96 : 72;
  static constexpr int kEpiRegs =
      ((threads * kLaunchRegs - 128 * kCtlRegs - (kExtra ? 128 * kExtraRegs : 0)) / (EPI * 32)) & ~7;
  static_assert(EPI == 8, "two epilogue warpgroups");
  static_assert(!kOneHot || kAlt, "one-hot accumulation runs with alternating warpgroups");
  static_assert(!kAlt || kAcc % 2 == 0, "alternating warpgroups need an even accumulator ring");
  static_assert(threads == 384 || threads == 512, "three or four warpgroups");
  static_assert(kEpiRegs <= 256 && kEpiRegs >= kLaunchRegs, "epilogue register budget");
};

struct AssignParams {
  const void* xsq;
  int64_t sxq_b, sxq_n;
  int xsq_dtype;
  const void* csq;  // (B, Kpad) in the distance dtype, +inf beyond K
  int64_t kpad;
  int32_t* out;
  int64_t so_b, so_n;
  int32_t* counts;  // (B, K) or null
  float* sums;      // (B, K, D) contiguous, only with FUSE
  int D;
  bool sums_vec;    // D % 4 == 0 and 16-byte aligned sums: float4 atomics
  int N, K;
  int nd;           // 128-byte column chunks per row
  int dch;          // elements per chunk
  int ntn;          // point tiles per batch
  int nkt;          // centroid tiles
  int total_tiles;
  int* status;
  int lo_b;         // 3xTF32 modes: the centroids' lo halves are batches lo_b.. of tmap_c
  int xlo_b;        // 3xTF32 modes: 0 -> the converter warps split each x chunk; > 0 -> x
                    // arrives split, its lo halves are batches xlo_b.. of tmap_x
};

__device__ __forceinline__ bool drain_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// ---------------------------------------------------------------- epilogue math
// Packed 16-bit helpers (mode 0).  In modes 0 and 1 the MMA's centroid
// operand is -2c, so the float32 accumulator holds -2 x.c exactly and one
// round-to-nearest conversion gives round(-2 * round(x.c)): the reference's
// `2 * bmm(x, c^T)` in the 16-bit dtype, overflow to inf included (the two
// differ only when x.c is a float16 subnormal, |x.c| < 2^-14).
template <typename T>
struct Pack2;

#define FK_PACK2_OPS(SFX, INF2)                                                                  \
  static constexpr uint32_t kInf2 = INF2;                                                        \
  /* round(round(x_sq + round(acc)) + c_sq) for two columns, lo = even column */                 \
  __device__ __forceinline__ static uint32_t dist(float a0, float a1, uint32_t xsq2,             \
                                                  uint32_t csq2) {                               \
    uint32_t r;                                                                                  \
    asm("{\n\t.reg .b32 t;\n\t"                                                                  \
        "cvt.rn." SFX ".f32 t, %2, %1;\n\t"                                                      \
        "add.rn." SFX " t, %3, t;\n\t"                                                           \
        "add.rn." SFX " %0, t, %4;\n\t}"                                                         \
        : "=r"(r)                                                                                \
        : "f"(a0), "f"(a1), "r"(xsq2), "r"(csq2));                                               \
    return r;                                                                                    \
  }                                                                                              \
  /* minimum that propagates NaN (argmin takes the first NaN) */                                 \
  __device__ __forceinline__ static uint32_t min2(uint32_t a, uint32_t b) {                      \
    uint32_t r;                                                                                  \
    asm("min.NaN." SFX " %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));                               \
    return r;                                                                                    \
  }                                                                                              \
  /* a strict improvement of the chunk minimum mm over best2, or its first NaN         */        \
  __device__ __forceinline__ static bool improves(uint32_t best2, uint32_t mm) {                 \
    uint32_t r;                                                                                  \
    asm("{\n\t.reg .pred p, q, n;\n\t"                                                           \
        "setp.nan." SFX " n|q, %1, %1;\n\t"                                                      \
        "setp.ltu.and." SFX " p|q, %2, %1, !n;\n\t"                                              \
        "selp.u32 %0, 1, 0, p;\n\t}"                                                            \
        : "=r"(r)                                                                                \
        : "r"(best2), "r"(mm));                                                                  \
    return r != 0;                                                                               \
  }                                                                                              \
  /* on a strict improvement of the chunk minimum mm over best2 (or the first NaN),    */        \
  /* store the chunk's 16 packed distances as four 16-byte units `STRIDE` bytes apart  */        \
  /* at shared address `saddr`, and take mm and `tag` as the new best and saved chunk. */        \
  template <int STRIDE>                                                                          \
  __device__ __forceinline__ static void save_if_better(uint32_t& best2, int& chunk,             \
                                                        uint32_t mm, int tag, uint32_t saddr,    \
                                                        const uint32_t (&d)[16]) {               \
    asm volatile(                                                                                \
        "{\n\t.reg .pred p, q, n;\n\t"                                                           \
        "setp.nan." SFX " n|q, %0, %0;\n\t"                                                      \
        "setp.ltu.and." SFX " p|q, %2, %0, !n;\n\t"                                              \
        "@p st.shared.v4.b32 [%4], {%6, %7, %8, %9};\n\t"                                        \
        "@p st.shared.v4.b32 [%4+%5], {%10, %11, %12, %13};\n\t"                                 \
        "@p st.shared.v4.b32 [%4+2*%5], {%14, %15, %16, %17};\n\t"                               \
        "@p st.shared.v4.b32 [%4+3*%5], {%18, %19, %20, %21};\n\t"                               \
        "selp.b32 %0, %2, %0, p;\n\t"                                                            \
        "selp.b32 %1, %3, %1, p;\n\t}"                                                           \
        : "+r"(best2), "+r"(chunk)                                                               \
        : "r"(mm), "r"(tag), "r"(saddr), "n"(STRIDE), "r"(d[0]), "r"(d[1]), "r"(d[2]),           \
          "r"(d[3]), "r"(d[4]), "r"(d[5]), "r"(d[6]), "r"(d[7]), "r"(d[8]), "r"(d[9]),           \
          "r"(d[10]), "r"(d[11]), "r"(d[12]), "r"(d[13]), "r"(d[14]), "r"(d[15])                 \
        : "memory");                                                                             \
  }

template <>
struct Pack2<__half> {
  FK_PACK2_OPS("f16x2", 0x7C007C00u)
  static constexpr unsigned short kOne = 0x3C00;  // 1.0
  __device__ __forceinline__ static float lo(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFFu)));
  }
  __device__ __forceinline__ static float hi(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16)));
  }
  __device__ __forceinline__ static uint32_t splat(float v) {
    const __half2 h = __float2half2_rn(v);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};

template <>
struct Pack2<__nv_bfloat16> {
  FK_PACK2_OPS("bf16x2", 0x7F807F80u)
  static constexpr unsigned short kOne = 0x3F80;  // 1.0
  __device__ __forceinline__ static float lo(uint32_t v) { return __uint_as_float(v << 16); }
  __device__ __forceinline__ static float hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
  __device__ __forceinline__ static uint32_t splat(float v) {
    const __nv_bfloat162 h = __float2bfloat162_rn(v);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};
#undef FK_PACK2_OPS

// Round a float to the 16-bit type and back (mode 1 cross rounding).
template <typename T>
__device__ __forceinline__ float round16(float v) {
  return Elem<T>::round(v);
}

// Candidate (vo, io) beats (val, idx) under argmin's rules: the first NaN
// wins, otherwise the smaller value, then the lower index.
__device__ __forceinline__ bool argmin_better(float vo, int io, float val, int idx) {
  const bool nv = vo != vo, nc = val != val;
  if (nv || nc) return nv && (!nc || io < idx);
  return vo < val || (vo == val && io < idx);
}

// Running argmin over a thread's row for the float32-chain modes, split into
// kChains independent chains (column j goes to chain j % kChains) so
// consecutive updates do not wait on each other.  Columns are visited in
// increasing order within a chain and updates need a strictly smaller value,
// so each chain keeps its lowest-index minimum; result() merges the chains by
// (value, index).  A chain remembers the local position of its best column
// inside its 32-column chunk plus the chunk id, which is refreshed once per
// chunk where the best value changed.
constexpr int kChains = 4;

// Running argmin for mode 0 at about one ALU operation per column pair: each
// 32-column chunk is reduced to its minimum with a tree of packed NaN-
// propagating min operations and compared once with the running best.  When
// the chunk minimum is strictly below the best (or is the row's first NaN),
// the thread stores the chunk's 16 packed distances in its own shared-memory
// slot with predicated stores (no branch).  The saved chunk is then the first
// chunk holding the final minimum (later chunks that only tie are not
// saved), so the first column equal to the minimum inside it (the first NaN
// if the minimum is NaN) is argmin's lowest-index answer; result() finds it
// once per point tile.
template <typename T>
struct ArgminSaved {
  uint32_t best2;  // running minimum, in both halves
  int chunk;       // col >> 5 of the saved chunk, -1 while nothing is saved
  uint32_t saddr;  // shared address of this thread's first 16-byte unit
  __device__ __forceinline__ void init(uint32_t slot_addr) {
    best2 = Pack2<T>::kInf2;
    chunk = -1;
    saddr = slot_addr;
  }
  template <int STRIDE>
  __device__ __forceinline__ void chunk32(const uint32_t (&v)[32], const uint4 (&cq)[4],
                                          uint32_t xsq2, int col0) {
    const uint32_t* cw = reinterpret_cast<const uint32_t*>(cq);
    uint32_t d[16];
#pragma unroll
    for (int pp = 0; pp < 16; ++pp)
      d[pp] = Pack2<T>::dist(__uint_as_float(v[2 * pp]), __uint_as_float(v[2 * pp + 1]), xsq2, cw[pp]);
    uint32_t m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = Pack2<T>::min2(d[i], d[i + 8]);
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = Pack2<T>::min2(m[i], m[i + 4]);
    m[0] = Pack2<T>::min2(m[0], m[2]);
    m[1] = Pack2<T>::min2(m[1], m[3]);
    m[0] = Pack2<T>::min2(m[0], m[1]);
    const uint32_t mm = Pack2<T>::min2(m[0], __byte_perm(m[0], 0, 0x1032));  // both halves
    Pack2<T>::template save_if_better<STRIDE>(best2, chunk, mm, col0 >> 5, saddr, d);
  }
  // first_col: the lowest column this thread visits (the answer when every
  // distance it saw was +inf, matching argmin's first index)
  template <int STRIDE>
  __device__ __forceinline__ void result(float& val, int& idx, int first_col) const {
    val = __int_as_float(0x7f800000);
    idx = first_col;
    if (chunk < 0) return;
    val = Pack2<T>::lo(best2);
    uint32_t w[16];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(w[4 * u]), "=r"(w[4 * u + 1]), "=r"(w[4 * u + 2]), "=r"(w[4 * u + 3])
                   : "r"(saddr + u * STRIDE)
                   : "memory");
    int pos = 31;
    if (val != val) {  // the first NaN of the saved chunk
#pragma unroll
      for (int pp = 15; pp >= 0; --pp) {
        const float h = Pack2<T>::hi(w[pp]), l = Pack2<T>::lo(w[pp]);
        if (h != h) pos = 2 * pp + 1;
        if (l != l) pos = 2 * pp;
      }
    } else {
#pragma unroll
      for (int pp = 15; pp >= 0; --pp) {
        if (Pack2<T>::hi(w[pp]) == val) pos = 2 * pp + 1;
        if (Pack2<T>::lo(w[pp]) == val) pos = 2 * pp;
      }
    }
    idx = chunk * 32 + pos;
  }
};

// Mode 0 with the saved chunk in registers (narrow one-hot tiles, where the
// shared-memory slots would cost an x tile buffer): the same rule as
// ArgminSaved, the winning chunk's 16 packed distances copied to w[] on each
// strict improvement instead of stored.
template <typename T>
struct ArgminRegs {
  uint32_t best2;
  int chunk;
  uint32_t w[16];
  __device__ __forceinline__ void init(uint32_t) {
    best2 = Pack2<T>::kInf2;
    chunk = -1;
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = 0u;
  }
  template <int STRIDE>
  __device__ __forceinline__ void chunk32(const uint32_t (&v)[32], const uint4 (&cq)[4],
                                          uint32_t xsq2, int col0) {
    const uint32_t* cw = reinterpret_cast<const uint32_t*>(cq);
    uint32_t d[16];
#pragma unroll
    for (int pp = 0; pp < 16; ++pp)
      d[pp] = Pack2<T>::dist(__uint_as_float(v[2 * pp]), __uint_as_float(v[2 * pp + 1]), xsq2, cw[pp]);
    uint32_t m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = Pack2<T>::min2(d[i], d[i + 8]);
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = Pack2<T>::min2(m[i], m[i + 4]);
    m[0] = Pack2<T>::min2(m[0], m[2]);
    m[1] = Pack2<T>::min2(m[1], m[3]);
    m[0] = Pack2<T>::min2(m[0], m[1]);
    const uint32_t mm = Pack2<T>::min2(m[0], __byte_perm(m[0], 0, 0x1032));  // both halves
    const bool p = Pack2<T>::improves(best2, mm);
    best2 = p ? mm : best2;
    chunk = p ? (col0 >> 5) : chunk;
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = p ? d[i] : w[i];
  }
  template <int STRIDE>
  __device__ __forceinline__ void result(float& val, int& idx, int first_col) const {
    val = __int_as_float(0x7f800000);
    idx = first_col;
    if (chunk < 0) return;
    val = Pack2<T>::lo(best2);
    int pos = 31;
    if (val != val) {  // the first NaN of the saved chunk
#pragma unroll
      for (int pp = 15; pp >= 0; --pp) {
        const float h = Pack2<T>::hi(w[pp]), l = Pack2<T>::lo(w[pp]);
        if (h != h) pos = 2 * pp + 1;
        if (l != l) pos = 2 * pp;
      }
    } else {
#pragma unroll
      for (int pp = 15; pp >= 0; --pp) {
        if (Pack2<T>::hi(w[pp]) == val) pos = 2 * pp + 1;
        if (Pack2<T>::lo(w[pp]) == val) pos = 2 * pp;
      }
    }
    idx = chunk * 32 + pos;
  }
};

template <typename T, int MODE>
struct ArgminF32 {  // modes 1 and 2: one column per register, float32 chain
  float best[kChains];
  int loc[kChains], chunk[kChains];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int c = 0; c < kChains; ++c) {
      best[c] = __int_as_float(0x7f800000);
      loc[c] = 0;
      chunk[c] = 0;
    }
  }
  __device__ __forceinline__ void chunk32(const uint32_t (&v)[32], const float* cs, float xsq,
                                          int col0) {
    float prev[kChains];
#pragma unroll
    for (int c = 0; c < kChains; ++c) prev[c] = best[c];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int c = j % kChains;
      // mode 1: the accumulator is -2 x.c (operand -2c) and round16 gives the
      // reference's float16 `2 * bmm(...)`, then the float32 chain;
      // mode 2: float32 cross products, x_sq - 2 * cross rounded once
      float d;
      if constexpr (MODE == 1)
        d = __fadd_rn(__fadd_rn(xsq, round16<T>(__uint_as_float(v[j]))), cs[j]);
      else
        d = __fadd_rn(__fmaf_rn(-2.0f, __uint_as_float(v[j]), xsq), cs[j]);
      const bool lt = d < best[c];
      best[c] = fminf(best[c], d);
      loc[c] = lt ? j : loc[c];
    }
#pragma unroll
    for (int c = 0; c < kChains; ++c) chunk[c] = (best[c] != prev[c]) ? (col0 >> 5) : chunk[c];
  }
  __device__ __forceinline__ void result(float& val, int& idx) const {
    val = __int_as_float(0x7f800000);
    idx = 0x7fffffff;
#pragma unroll
    for (int c = 0; c < kChains; ++c) {
      const int i = (chunk[c] << 5) + loc[c];
      if (best[c] < val || (best[c] == val && i < idx)) {
        val = best[c];
        idx = i;
      }
    }
  }
};

// Modes 3 and 4 (dot-product argmax): float32 scores straight from TMEM.  Per
// 16-column half of a chunk a tree of fmaxf gives the half's maximum; only a
// strictly larger maximum replaces the running best (so the earliest half
// keeps a tie) and then the half's 16 scores go to this thread's shared-memory
// slot.  result() scans the saved half for the first score equal to the best.
// Padding columns (>= K, zero-filled centroid rows) only occur in the chunk
// that crosses K: that chunk sets them to -inf first (a warp-uniform branch).
// A point whose scores are all NaN keeps nothing and reports its first
// column with +inf, so the merge gives column 0, as argmax over NaNs does.
struct ArgmaxSaved {
  float best;   // running maximum
  int part;     // col >> 4 of the saved half chunk, -1 while nothing is saved
  uint4* slot;  // this thread's four 16-byte units, `stride` units apart
  int stride;
  __device__ __forceinline__ void init(uint4* s, int st) {
    best = __int_as_float(0xff800000);
    part = -1;
    slot = s;
    stride = st;
  }
  __device__ __forceinline__ void half16(const uint32_t* v, int part16) {
    float m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmaxf(__uint_as_float(v[i]), __uint_as_float(v[i + 8]));
#pragma unroll
    for (int i = 0; i < 4; ++i) m[i] = fmaxf(m[i], m[i + 4]);
    const float mm = fmaxf(fmaxf(m[0], m[2]), fmaxf(m[1], m[3]));
    if (mm > best) {
      best = mm;
      part = part16;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        slot[u * stride] = make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
    }
  }
  __device__ __forceinline__ void chunk32(uint32_t (&v)[32], int col0, int K) {
    if (col0 + 32 > K) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = (col0 + j < K) ? v[j] : 0xff800000u;
    }
    half16(v, col0 >> 4);
    half16(v + 16, (col0 >> 4) + 1);
  }
  // val is the negated score, so the group merge (smallest value, then lowest
  // column) is the argmax with first-index ties
  __device__ __forceinline__ void result(float& val, int& idx, int first_col) const {
    val = __int_as_float(0x7f800000);
    idx = first_col;
    if (part < 0) return;
    val = -best;
    int pos = 15;
#pragma unroll
    for (int u = 3; u >= 0; --u) {
      const uint4 q = slot[u * stride];
      if (__uint_as_float(q.w) == best) pos = 4 * u + 3;
      if (__uint_as_float(q.z) == best) pos = 4 * u + 2;
      if (__uint_as_float(q.y) == best) pos = 4 * u + 1;
      if (__uint_as_float(q.x) == best) pos = 4 * u;
    }
    idx = part * 16 + pos;
  }
};

// --------------------------------------------------------------------- kernel
// RESC (resident centroids; 16-bit, resident x, nkt * nd <= STAGES): stage
// s = kt * nd + dc holds that chunk of the current batch's centroids.  The
// producer loads the chunks only when a CTA's tile range enters a new batch
// (batch bi of the CTA: fill bi of every stage); the MMA waits for them once
// per batch and releases them after the batch's last tile.
template <typename T, int MODE, bool XRES, int STAGES, bool FUSE, int EPI, int KC, bool RESC>
__global__ void __launch_bounds__(Layout<MODE, XRES, STAGES, FUSE, EPI, KC, RESC>::threads, 1)
    assign_kernel(const __grid_constant__ CUtensorMap tmap_x,
                  const __grid_constant__ CUtensorMap tmap_c, const AssignParams p) {
  using L = Layout<MODE, XRES, STAGES, FUSE, EPI, KC, RESC>;
  static_assert(!RESC || (XRES && !split_mode(MODE)), "resident centroids need resident x, 16-bit");
  constexpr int kCent = KC;                 // this instance's tile width
  constexpr int kAcc = L::kAcc;
  constexpr int kCChunk = L::kCChunk;
  constexpr int kEpiWarps = EPI;
  constexpr int kGroups = L::kGroups;
  constexpr int kGCols = kCent / kGroups;   // columns per group
  constexpr int kGChunks = kGCols / 32;     // 32-column TMEM loads per group
  constexpr int kConvWarp0 = kEpiWarp0 + EPI;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Each CTA takes a contiguous range of (batch, 128-point) tiles, so at any
  // moment the CTAs stream different batches' centroid tiles; round-robin
  // assignment made all CTAs hit the same batch's centroids in the same L2
  // slices at once.
  const int t_begin = static_cast<int>((static_cast<int64_t>(blockIdx.x) * p.total_tiles) / gridDim.x);
  const int t_end = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * p.total_tiles) / gridDim.x);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bar_off);
  uint64_t* x_full = bars;
  uint64_t* x_empty = bars + L::XB;
  uint64_t* c_full = bars + 2 * L::XB;
  uint64_t* c_empty = c_full + STAGES;
  uint64_t* conv_full = c_empty + STAGES;
  uint64_t* acc_full = conv_full + STAGES;
  uint64_t* acc_empty = acc_full + kAcc;
  uint64_t* merge_full = acc_empty + kAcc;
  uint64_t* merge_empty = merge_full + 2;
  uint64_t* lab_full = merge_empty + 2;
  uint64_t* lab_empty = lab_full + 2;
  uint64_t* final_bar = lab_empty + 2;
  uint64_t* oh_full = final_bar + 1;     // one-hot operand of a tile written (128 points)
  uint64_t* oh_empty = oh_full + 2;      // its sums MMAs done (buffer and x tile free)
  uint64_t* sums_full = oh_empty + 2;    // a batch's sums complete in TMEM
  uint64_t* sums_empty = sums_full + 1;  // the epilogue has added them to global memory
  uint64_t* wg_bar = sums_empty + 1;     // [2] barriers of each epilogue warpgroup's 128 threads
  uint64_t* sums_full_odd = wg_bar + 2;  // sums_full of the CTA's odd batches (one-hot)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::misc_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::misc_off + 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::XB; ++i) {
      mbar_init(&x_full[i], 1);
      // with FUSE the resident x tile is also read by the 128 sum threads
      // (the points' rows) before it may be overwritten
      mbar_init(&x_empty[i], L::kSumWarps ? 1 + 128 : 1);
    }
    for (int i = 0; i < kAcc; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], L::kAlt ? 4 : kEpiWarps * 32);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&lab_full[i], 128);
      mbar_init(&lab_empty[i], 128);
      if (kGroups > 1) {
        mbar_init(&merge_full[i], (kGroups - 1) * 128);
        mbar_init(&merge_empty[i], 128);
      }
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&c_full[s], 1);
      mbar_init(&c_empty[s], 1);
      mbar_init(&conv_full[s], kConvWarps * 32);
    }
    mbar_init(final_bar, L::kOneHot ? 2 : 1);   // one commit per MMA-issuing thread
    for (int i = 0; i < 2; ++i) {
      mbar_init(&oh_full[i], 4);
      mbar_init(&oh_empty[i], 1);
    }
    mbar_init(sums_full, 1);
    mbar_init(sums_full_odd, 1);
    // one warpgroup reads a batch's sums (one-hot form)
    mbar_init(sums_empty, 128);
    mbar_init(&wg_bar[0], 128);
    mbar_init(&wg_bar[1], 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if constexpr (L::kOneHot) {
    // one-hot buffers start all zero (each tile then sets one element per
    // point and clears the element it set in the buffer's previous use);
    // counts zero
    uint4* oh = reinterpret_cast<uint4*>(smem + L::oh_off);
    for (int i = threadIdx.x; i < L::oh_bytes / 16; i += blockDim.x) oh[i] = make_uint4(0, 0, 0, 0);
    int* hist = reinterpret_cast<int*>(smem + L::hist_off);
    for (int i = threadIdx.x; i < L::hist_bytes / 4; i += blockDim.x) hist[i] = 0;
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_c);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Each role's branch first moves its warpgroup's register budget
  // (setmaxnreg, inside the branch so the compiler knows each role's limit):
  // the control warps and the extra warpgroup give registers to the epilogue.

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    setmaxnreg_dec<L::kCtlRegs>();
    if (lane == 0) {
      int stage = 0;
      uint32_t sph = 0;
      int xb = 0;
      uint32_t xph = 0;
      int last_par[STAGES];
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      int last_xpar[L::XB];
      for (int i = 0; i < L::XB; ++i) last_xpar[i] = -1;
      int bi = -1, prev_b = -1;  // RESC: batch count of this CTA, last batch loaded
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; ++t) {
        const int b = t / p.ntn;
        const int row0 = (t % p.ntn) * kRows;
        if constexpr (XRES) {
          if (!mbar_wait(&x_empty[xb], xph ^ 1, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&x_full[xb], p.nd * kXChunk);
          for (int dc = 0; dc < p.nd; ++dc)
            tma_load_3d(smem + L::x_off + (xb * kResidentChunks + dc) * kXChunk, &tmap_x,
                        &x_full[xb], dc * p.dch, row0, b);
          last_xpar[xb] = static_cast<int>(xph);
          if (++xb == L::XB) { xb = 0; xph ^= 1; }
        }
        if constexpr (RESC) {
          if (b != prev_b) {
            ++bi;
            prev_b = b;
            for (int kt = 0; ok && kt < p.nkt; ++kt)
              for (int dc = 0; ok && dc < p.nd; ++dc) {
                const int sc = kt * p.nd + dc;
                // the previous batch's chunk is released after its last tile
                if (!mbar_wait(&c_empty[sc], static_cast<uint32_t>(bi & 1) ^ 1u, abort_flag,
                               p.status, FK_DEV_WAIT_TIMEOUT)) {
                  ok = false;
                  break;
                }
                mbar_arrive_expect_tx(&c_full[sc], kCChunk);
                tma_load_3d(smem + L::stages_off + sc * L::stage_bytes + L::st_c, &tmap_c,
                            &c_full[sc], dc * p.dch, kt * kCent, b);
                last_par[sc] = bi & 1;
              }
          }
        } else {
          for (int kt = 0; ok && kt < p.nkt; ++kt) {
            for (int dc = 0; dc < p.nd; ++dc) {
              if (!mbar_wait(&c_empty[stage], sph ^ 1, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT)) {
                ok = false;
                break;
              }
              uint8_t* st = smem + L::stages_off + stage * L::stage_bytes;
              const int xparts = (split_mode(MODE) && p.xlo_b) ? 2 : 1;
              mbar_arrive_expect_tx(&c_full[stage],
                                    kCChunk * L::kSplit + (XRES ? 0 : L::kXChunkL * xparts));
              tma_load_3d(st + L::st_c, &tmap_c, &c_full[stage], dc * p.dch, kt * kCent, b);
              if constexpr (split_mode(MODE))   // the centroids come split (hi, lo) per call
                tma_load_3d(st + L::st_clo, &tmap_c, &c_full[stage], dc * p.dch, kt * kCent,
                            b + p.lo_b);
              if constexpr (!XRES)
                tma_load_3d(st + L::st_x, &tmap_x, &c_full[stage], dc * p.dch, row0, b);
              if constexpr (split_mode(MODE) && !XRES) {
                if (p.xlo_b)   // x split once per fit: its lo half from the second half of tmap_x
                  tma_load_3d(st + L::st_xlo, &tmap_x, &c_full[stage], dc * p.dch, row0,
                              b + p.xlo_b);
              }
              last_par[stage] = static_cast<int>(sph);
              if (++stage == STAGES) { stage = 0; sph ^= 1; }
            }
          }
        }
      }
      if (!ok) {
        // Let every load already issued land before the CTA can exit.
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) drain_wait(&c_full[s], static_cast<uint32_t>(last_par[s]), 200000000ull);
        for (int i = 0; i < L::XB; ++i)
          if (last_xpar[i] >= 0) drain_wait(&x_full[i], static_cast<uint32_t>(last_xpar[i]), 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    setmaxnreg_dec<L::kCtlRegs>();
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(Elem<T>::kMmaFmt, kRows, kCent);
      int stage = 0;
      uint32_t sph = 0;
      int xb = 0;
      uint32_t xph = 0;
      int ab = 0;
      uint32_t aph = 0;
      int bi = -1, prev_b = -1;  // RESC: as in the producer
      bool ok = true;
      if constexpr (!L::kOneHot) {
      for (int t = t_begin; ok && t < t_end; ++t) {
        bool new_batch = false, last_of_batch = false;
        if constexpr (RESC) {
          const int b = t / p.ntn;
          new_batch = b != prev_b;
          if (new_batch) {
            ++bi;
            prev_b = b;
          }
          last_of_batch = t + 1 == t_end || (t + 1) / p.ntn != b;
        }
        if constexpr (XRES) {
          if (!mbar_wait(&x_full[xb], xph, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        for (int kt = 0; ok && kt < p.nkt; ++kt) {
          if (!mbar_wait(&acc_empty[ab], aph ^ 1, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * kCent);
          for (int dc = 0; dc < p.nd; ++dc) {
            const int sc = RESC ? kt * p.nd + dc : stage;
            uint64_t* ready = (split_mode(MODE) && !p.xlo_b) ? &conv_full[sc] : &c_full[sc];
            if (!RESC || new_batch) {
              if (!mbar_wait(ready, RESC ? static_cast<uint32_t>(bi & 1) : sph, abort_flag,
                             p.status, FK_DEV_WAIT_TIMEOUT)) {
                ok = false;
                break;
              }
            }
            tc_fence_after();
            uint8_t* st = smem + L::stages_off + sc * L::stage_bytes;
            const uint32_t a_addr =
                XRES ? smem_u32(smem + L::x_off + (xb * kResidentChunks + dc) * kXChunk)
                     : smem_u32(st + L::st_x);
            const uint32_t b_addr = smem_u32(st + L::st_c);
#pragma unroll
            for (int ks = 0; ks < L::kKSteps; ++ks) {
              const uint32_t acc = (dc > 0 || ks > 0) ? 1u : 0u;
              const uint32_t off = static_cast<uint32_t>(ks * 32);
              if constexpr (split_mode(MODE)) {
                const uint32_t alo = smem_u32(st + L::st_xlo);
                const uint32_t blo = smem_u32(st + L::st_clo);
                auto sd = [](uint32_t a) {
                  if constexpr (L::kRowB == 64) return smem_desc_sw64(a);
                  else return smem_desc_sw128(a);
                };
                mma_tf32(d_tmem, sd(a_addr + off), sd(b_addr + off), idesc, acc);
                mma_tf32(d_tmem, sd(a_addr + off), sd(blo + off), idesc, 1u);
                mma_tf32(d_tmem, sd(alo + off), sd(b_addr + off), idesc, 1u);
              } else {
                mma_f16(d_tmem, smem_desc_sw128(a_addr + off), smem_desc_sw128(b_addr + off),
                        idesc, acc);
              }
            }
            if constexpr (RESC) {
              if (last_of_batch) mma_commit(&c_empty[sc]);
            } else {
              mma_commit(&c_empty[stage]);
              if (++stage == STAGES) { stage = 0; sph ^= 1; }
            }
          }
          if (!ok) break;
          mma_commit(&acc_full[ab]);
          if (++ab == kAcc) { ab = 0; aph ^= 1; }
        }
        if constexpr (XRES) {
          if (ok) {
            mma_commit(&x_empty[xb]);
            if (++xb == L::XB) { xb = 0; xph ^= 1; }
          }
        }
      }
      } else {
        // One-hot form (K <= 128: one centroid tile, resident): this thread
        // issues the assignment MMAs only; warp 2 issues the sums MMAs, so the
        // two instruction streams do not wait behind each other.  A tile's x
        // buffer is released by its sums MMAs (its assignment MMAs are done
        // before its labels, hence its one-hot operand, exist).
        for (int td = t_begin; ok && td < t_end; ++td) {
          if (!mbar_wait(&x_full[xb], xph, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT) ||
              !mbar_wait(&acc_empty[ab], aph ^ 1, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int b = td / p.ntn;
          const bool new_batch = b != prev_b;
          if (new_batch) {
            ++bi;
            prev_b = b;
          }
          const bool last_of_batch = td + 1 == t_end || (td + 1) / p.ntn != b;
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * kCent);
          for (int dc = 0; dc < p.nd; ++dc) {
            if (new_batch && !mbar_wait(&c_full[dc], static_cast<uint32_t>(bi & 1), abort_flag,
                                        p.status, FK_DEV_WAIT_TIMEOUT)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr =
                smem_u32(smem + L::x_off + (xb * kResidentChunks + dc) * kXChunk);
            const uint32_t b_addr = smem_u32(smem + L::stages_off + dc * L::stage_bytes + L::st_c);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint32_t off = static_cast<uint32_t>(ks * 32);
              mma_f16(d_tmem, smem_desc_sw128(a_addr + off), smem_desc_sw128(b_addr + off), idesc,
                      (dc > 0 || ks > 0) ? 1u : 0u);
            }
            if (last_of_batch) mma_commit(&c_empty[dc]);
          }
          if (!ok) break;
          mma_commit(&acc_full[ab]);
          if (++ab == kAcc) { ab = 0; aph ^= 1; }
          if (++xb == L::XB) { xb = 0; xph ^= 1; }
        }
      }
      // All MMAs this thread issued must finish before TMEM is released.
      mma_commit(final_bar);
      drain_wait(final_bar, 0, 1000000000ull);
    }
  } else if (L::kOneHot && warp == 2) {
    // --------------------------------------------- sums MMAs (one-hot form)
    setmaxnreg_dec<L::kCtlRegs>();
    if constexpr (L::kOneHot) {
    if (lane == 0) {
      bool ok = true;
      // One-hot accumulation: the sums MMAs of tile t run once the epilogue
      // has written the labels of t as a one-hot operand:
      // sums[k][d] += sum_p onehot[k][p] * x[p][d] into the TMEM sums columns,
      // A = one-hot (K-major: points contiguous per centroid), B = the tile's
      // x buffer read MN-major (dims contiguous per point; LBO = the 64-dim
      // chunk stride, SBO = 8 points).  A batch's last tile commits sums_full
      // (sums_full_odd for the CTA's odd batches); the next batch's first sums
      // MMA waits until the epilogue has read them (sums_empty).
      int ohn = 0, fln = 0;       // one-hot buffers consumed, flushes done
      bool sums_on = false;       // the current batch's sums already started
      auto sums_mma = [&](int tt, int xbuf) -> bool {
        {
          constexpr uint32_t idesc_s = instr_desc(Elem<T>::kMmaFmt, kRows, 128) | (1u << 16);
          if (!sums_on && fln > 0) {
            if (!mbar_wait(sums_empty, static_cast<uint32_t>((fln - 1) & 1), abort_flag, p.status,
                           FK_DEV_WAIT_TIMEOUT))
              return false;
            tc_fence_after();
          }
          const int par = ohn & 1;   // tile ohn of the CTA: its warpgroup's buffer
          if (!mbar_wait(&oh_full[par], static_cast<uint32_t>((ohn >> 1) & 1), abort_flag,
                         p.status, FK_DEV_WAIT_TIMEOUT))
            return false;
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + L::oh_off + par * 2 * kXChunk);
          const uint32_t b0 = smem_u32(smem + L::x_off + xbuf * kResidentChunks * kXChunk);
#pragma unroll
          for (int s = 0; s < 8; ++s)   // 16 points per MMA
            mma_f16(tmem_base + static_cast<uint32_t>(L::kSumsCol),
                    smem_desc_sw128(a0 + (s >> 2) * kXChunk + (s & 3) * 32),
                    smem_desc_sw128_mn(b0 + s * 16 * kChunkB, kXChunk, 1024), idesc_s,
                    (sums_on || s > 0) ? 1u : 0u);
          sums_on = true;
          mma_commit(&oh_empty[par]);
          mma_commit(&x_empty[xbuf]);
          ++ohn;
          if (tt + 1 == t_end || (tt + 1) / p.ntn != tt / p.ntn) {
            mma_commit((fln & 1) ? sums_full_odd : sums_full);
            ++fln;
            sums_on = false;
          }
        }
        return true;
      };
      int xs = 0;   // x buffer of tile ts
      for (int ts = t_begin; ok && ts < t_end; ++ts) {
        ok = sums_mma(ts, xs);
        if (++xs == L::XB) xs = 0;
      }
      (void)ok;
      // All MMAs this thread issued must finish before TMEM is released.
      mma_commit(final_bar);
      drain_wait(final_bar, 0, 1000000000ull);
    }
    }
  } else if (warp < kEpiWarp0) {
    // idle warps of warpgroup 0: straight to the final barrier
    setmaxnreg_dec<L::kCtlRegs>();
  } else if (warp < kEpiWarp0 + kEpiWarps) {
    // ------------------------------------------------------------- epilogue
    setmaxnreg_inc<L::kEpiRegs>();
    const int ew = warp - kEpiWarp0;
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int wg = ew >> 2;          // epilogue warpgroup
    const int h = L::kAlt ? 0 : wg;  // column group: kGCols columns of each tile
    const int row = q * 32 + lane;   // point within the tile
    uint2* merge = reinterpret_cast<uint2*>(smem + L::merge_off);
    // alternating warpgroups: warpgroup wg takes the CTA's tiles wg, wg+2, ...
    constexpr int kStep = L::kAlt ? 2 : 1;
    const int it0 = L::kAlt ? wg : 0;
    int ab = it0 % kAcc;
    uint32_t aph = static_cast<uint32_t>((it0 / kAcc) & 1);
    int it = it0;                    // tile index within the CTA's range
    bool ok = true;
    int wsn = 0;                     // alternating: uses of this warpgroup's barrier
    int prev_lab = -1;               // one-hot: the element this thread set in its buffer
    // x_sq of this thread's point in tile t (0 past N), fetched one tile
    // ahead so the tile's first distances do not wait on an HBM read
    auto load_xsq = [&](int t) -> float {
      const int n = (t % p.ntn) * kRows + row;
      return (n < p.N && p.xsq) ? load_f(p.xsq, (t / p.ntn) * p.sxq_b + n * p.sxq_n, p.xsq_dtype)
                                : 0.0f;
    };
    // bounded barrier of this warpgroup's 128 threads (alternating form)
    auto wg_sync = [&]() -> bool {
      uint64_t* bar = &wg_bar[wg];
      mbar_arrive(bar);
      const bool got = mbar_wait(bar, static_cast<uint32_t>(wsn & 1), abort_flag, p.status,
                                 FK_DEV_WAIT_TIMEOUT);
      ++wsn;
      return __all_sync(0xffffffffu, got);
    };
    float xsq_next = t_begin + it0 < t_end ? load_xsq(t_begin + it0) : 0.0f;
    for (int t = t_begin + it0; ok && t < t_end; t += kStep, it += kStep) {
      const int b = t / p.ntn;
      const int n = (t % p.ntn) * kRows + row;
      const bool valid = n < p.N;
      const float xsq_f = xsq_next;
      if (t + kStep < t_end) xsq_next = load_xsq(t + kStep);
      if constexpr (L::kAlt) {   // one accumulator per tile, used in tile order
        ab = it % kAcc;
        aph = static_cast<uint32_t>((it / kAcc) & 1);
      }

      using Argmin = typename std::conditional<
          MODE == 0,
          typename std::conditional<L::kRegSave, ArgminRegs<T>, ArgminSaved<T>>::type,
          typename std::conditional<(MODE >= 3), ArgmaxSaved, ArgminF32<T, MODE>>::type>::type;
      constexpr int kSaveStride = L::save_stride * 16;  // bytes between a slot's 16-byte units
      Argmin am;
      if constexpr (MODE == 0)
        am.init(smem_u32(smem + L::save_off) + static_cast<uint32_t>((ew * 32 + lane) * 16));
      else if constexpr (MODE >= 3)
        am.init(reinterpret_cast<uint4*>(smem + L::save_off) + ew * 32 + lane, L::save_stride);
      else
        am.init();
      uint32_t xsq2 = 0u;
      if constexpr (MODE == 0) xsq2 = Pack2<T>::splat(xsq_f);  // exact: x_sq holds a T value
      const uint8_t* csq_row =
          static_cast<const uint8_t*>(p.csq) +
          static_cast<size_t>(b) * p.kpad * (MODE == 0 ? 2 : 4);
      // Wait for accumulator `ab` (warp-uniform outcome: tcgen05.ld is .sync.aligned).
      auto acc_wait = [&]() -> bool {
        const bool got = mbar_wait(&acc_full[ab], aph, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT);
        if (!__all_sync(0xffffffffu, got)) return false;
        tc_fence_after();
        return true;
      };
      // (alternating form: one arrival per warp once all its lanes' loads
      // are done, instead of 128 arrivals on one shared word)
      auto acc_release = [&]() {
        tc_fence_before();
        if constexpr (L::kAlt) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[ab]);
        } else {
          mbar_arrive(&acc_empty[ab]);
        }
        if (++ab == kAcc) { ab = 0; aph ^= 1; }
      };

      if constexpr (MODE == 0) {
        // Per centroid tile the warp loads its whole column slice (kCh
        // 32-column chunks, kCh*32 registers) with back-to-back TMEM loads and
        // one wait, hands the accumulator back at once and reduces from
        // registers, so the accumulator is held only for the loads.  The chunk
        // loop is unrolled (TMEM addresses and c_sq offsets are constants);
        // each chunk's c_sq words are fetched one chunk ahead.
        constexpr int kCh = kGCols / 32;
        const uint32_t tq = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            static_cast<uint32_t>(h * kGCols);
        const uint4* cs0 = reinterpret_cast<const uint4*>(csq_row) + h * kGCols / 8;
        uint32_t v[kCh][32];
        uint4 cq[2][4];
        for (int kt = 0; kt < p.nkt; ++kt) {
          if (!acc_wait()) {
            ok = false;
            break;
          }
          const uint32_t tt = tq + static_cast<uint32_t>(ab * kCent);
#pragma unroll
          for (int c = 0; c < kCh; ++c) tmem_ld32(tt + c * 32, v[c]);
          const uint4* ct = cs0 + kt * (kCent / 8);
#pragma unroll
          for (int i = 0; i < 4; ++i) cq[0][i] = __ldg(ct + i);
#pragma unroll
          for (int c = 0; c < kCh; ++c) tmem_ld_wait(v[c]);  // the first waits for all
          acc_release();
          const int colt = kt * kCent + h * kGCols;
#pragma unroll
          for (int c = 0; c < kCh; ++c) {
            if (c + 1 < kCh) {
#pragma unroll
              for (int i = 0; i < 4; ++i) cq[(c + 1) & 1][i] = __ldg(ct + (c + 1) * 4 + i);
            }
            am.template chunk32<kSaveStride>(v[c], cq[c & 1], xsq2, colt + c * 32);
          }
        }
        if (!ok) break;
      } else {
        // Modes 1-4: the chunks in (centroid tile, chunk) order; the TMEM load
        // of chunk g+1 is in flight while chunk g is reduced; a tile's
        // accumulator is released once its last chunk is in registers.  The
        // float32 chains load their c_sq words when reducing.
        const int nchunks = p.nkt * kGChunks;
        uint32_t va[32], vb[32];
        auto issue = [&](int g, uint32_t(&v)[32]) -> bool {
          const int ch = g % kGChunks;
          if (ch == 0 && !acc_wait()) return false;
          tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                        static_cast<uint32_t>(ab * kCent + h * kGCols + ch * 32),
                    v);
          return true;
        };
        auto landed = [&](int g, uint32_t(&v)[32]) {
          tmem_ld_wait(v);
          if (g % kGChunks == kGChunks - 1) acc_release();
        };
        auto reduce = [&](int g, uint32_t(&v)[32]) {
          const int col0 = (g / kGChunks) * kCent + h * kGCols + (g % kGChunks) * 32;
          if constexpr (MODE >= 3) {
            am.chunk32(v, col0, p.K);
          } else {
            const float4* src = reinterpret_cast<const float4*>(csq_row + col0 * 4);
            float4 c4[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) c4[i] = __ldg(src + i);
            am.chunk32(v, reinterpret_cast<const float*>(c4), xsq_f, col0);
          }
        };
        if (!issue(0, va)) {
          ok = false;
          break;
        }
        landed(0, va);
#pragma unroll 1
        for (int g = 0; g < nchunks; g += 2) {
          if (!issue(g + 1, vb)) {
            ok = false;
            break;
          }
          reduce(g, va);
          landed(g + 1, vb);
          const bool more = g + 2 < nchunks;
          if (more && !issue(g + 2, va)) {
            ok = false;
            break;
          }
          reduce(g + 1, vb);
          if (more) landed(g + 2, va);
        }
        if (!ok) break;
      }

      // Per-thread winner: (value, lowest column on ties; the first NaN wins).
      float val;
      int idx;
      if constexpr (MODE == 0)
        am.template result<kSaveStride>(val, idx, h * kGCols);
      else if constexpr (MODE >= 3)
        am.result(val, idx, h * kGCols);
      else
        am.result(val, idx);

      // Merge the column groups (wide tiles): groups 1.. publish, group 0 decides.
      const int par = it & 1;
      const uint32_t mph = static_cast<uint32_t>((it >> 1) & 1);
      bool decide = true;
      if constexpr (kGroups > 1) {
        uint2* mslots = merge + par * (kGroups - 1) * kRows;
        if (h != 0) {
          const bool got = mbar_wait(&merge_empty[par], mph ^ 1, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          mslots[(h - 1) * kRows + row] = make_uint2(__float_as_uint(val), static_cast<uint32_t>(idx));
          mbar_arrive(&merge_full[par]);
          decide = false;
        } else {
          const bool got = mbar_wait(&merge_full[par], mph, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int gg = 1; gg < kGroups; ++gg) {
            const uint2 o = mslots[(gg - 1) * kRows + row];
            const float vo = __uint_as_float(o.x);
            const int io = static_cast<int>(o.y);
            if (argmin_better(vo, io, val, idx)) {
              val = vo;
              idx = io;
            }
          }
          mbar_arrive(&merge_empty[par]);
        }
      }
      if (decide) {
        if (valid) {
          p.out[b * p.so_b + static_cast<int64_t>(n) * p.so_n] = idx;
          if (p.counts && !L::kOneHot) atomicAdd(p.counts + static_cast<int64_t>(b) * p.K + idx, 1);
        }
        if constexpr (L::kOneHot) {
          // Count the point in this warpgroup's shared counts (warp-aggregated
          // atomics), then mark it in the warpgroup's one-hot buffer once the
          // sums MMAs of the warpgroup's previous tile are done with it: clear
          // the element this thread set there, set (label, point) to 1.
          const int lab = valid ? idx : -1;
          int* hist = reinterpret_cast<int*>(smem + L::hist_off) + wg * 128;
          const unsigned grp = __match_any_sync(0xffffffffu, lab);
          if (lab >= 0 && lane == __ffs(grp) - 1) atomicAdd(hist + lab, __popc(grp));
          const int use = it >> 1;   // uses of this warpgroup's buffer so far
          if (use > 0) {
            const bool got2 = mbar_wait(&oh_empty[wg], static_cast<uint32_t>((use - 1) & 1), abort_flag,
                                        p.status, FK_DEV_WAIT_TIMEOUT);
            if (!__all_sync(0xffffffffu, got2)) {
              ok = false;
              break;
            }
          }
          uint8_t* ob = smem + L::oh_off + wg * 2 * kXChunk + (row >> 6) * kXChunk;
          const int pb = (row & 63) * 2;  // byte of this point within a 128-byte row
          auto elem = [&](int k) -> unsigned short* {
            return reinterpret_cast<unsigned short*>(ob + k * kChunkB + (((pb >> 4) ^ (k & 7)) << 4) +
                                                     (pb & 15));
          };
          if (prev_lab >= 0) *elem(prev_lab) = 0;
          if (lab >= 0) *elem(lab) = Pack2<T>::kOne;
          prev_lab = lab;
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&oh_full[wg]);   // one arrival per warp
        }
        if constexpr (L::kSumWarps && XRES) {
          // hand the label (or -1 past N) to the sum warps
          const bool got2 = mbar_wait(&lab_empty[par], mph ^ 1, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT);
          if (!__all_sync(0xffffffffu, got2)) {
            ok = false;
            break;
          }
          reinterpret_cast<int*>(smem + L::lab_off)[par * kRows + row] = valid ? idx : -1;
          mbar_arrive(&lab_full[par]);
        }
      }
      if constexpr (L::kOneHot) {
        // This warpgroup's last tile of the batch: add its shared counts to
        // the global counts and reset them (a barrier of the warpgroup on
        // each side: every count added before, none of the next batch's
        // before the reset).
        if (t + kStep >= t_end || (t + kStep) / p.ntn != b) {
          if (!wg_sync()) {
            ok = false;
            break;
          }
          int* hist = reinterpret_cast<int*>(smem + L::hist_off) + wg * 128;
          const int cnt = hist[row];
          if (cnt && p.counts && row < p.K)
            atomicAdd(p.counts + static_cast<int64_t>(b) * p.K + row, cnt);
          hist[row] = 0;
          if (!wg_sync()) {
            ok = false;
            break;
          }
        }
        // The batch's last tile: add the TMEM sums (lanes = centroids, 128
        // dimension columns) to the global sums.  Batches alternate between
        // two sums_full barriers (batch j of the CTA: barrier j & 1, phase
        // (j >> 1) & 1), so a warpgroup that never saw the previous batch's
        // completion cannot mistake it for this one's.
        if (t + 1 == t_end || (t + 1) / p.ntn != b) {
          const int j = b - t_begin / p.ntn;
          uint64_t* sf = (j & 1) ? sums_full_odd : sums_full;
          const bool got3 =
              mbar_wait(sf, static_cast<uint32_t>((j >> 1) & 1), abort_flag, p.status, FK_DEV_WAIT_TIMEOUT);
          if (!__all_sync(0xffffffffu, got3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ta = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                              static_cast<uint32_t>(L::kSumsCol);
          float* dst = p.sums + (static_cast<int64_t>(b) * p.K + row) * p.D;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t sa[32], sb[32];
            tmem_ld32(ta + half * 64, sa);
            tmem_ld32(ta + half * 64 + 32, sb);
            tmem_ld_wait(sa);
            tmem_ld_wait(sb);
            if (half == 1) {
              tc_fence_before();
              mbar_arrive(sums_empty);
            }
            if (row < p.K) {
              const int d0 = half * 64;
#pragma unroll
              for (int jj = 0; jj < 32; jj += 4) {
                if (p.sums_vec) {   // D % 4 == 0: whole float4 groups, 16-byte aligned
                  if (d0 + jj < p.D)
                    atomicAdd(reinterpret_cast<float4*>(dst + d0 + jj),
                              make_float4(__uint_as_float(sa[jj]), __uint_as_float(sa[jj + 1]),
                                          __uint_as_float(sa[jj + 2]), __uint_as_float(sa[jj + 3])));
                  if (d0 + 32 + jj < p.D)
                    atomicAdd(reinterpret_cast<float4*>(dst + d0 + 32 + jj),
                              make_float4(__uint_as_float(sb[jj]), __uint_as_float(sb[jj + 1]),
                                          __uint_as_float(sb[jj + 2]), __uint_as_float(sb[jj + 3])));
                } else {
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    if (d0 + jj + e < p.D) atomicAdd(dst + d0 + jj + e, __uint_as_float(sa[jj + e]));
                    if (d0 + 32 + jj + e < p.D)
                      atomicAdd(dst + d0 + 32 + jj + e, __uint_as_float(sb[jj + e]));
                  }
                }
              }
            }
          }
        }
      }
    }
  } else if (L::kSumWarps && XRES) {
    // ------------------------------------------- sum warps (fused accumulation)
    // Sum warp w adds rows 32w..32w+31 of every tile, one point at a time:
    // lane l takes columns 4l..4l+3 of the point's row (still resident in the
    // tile's x buffer, 128-byte swizzle: 16-byte unit u of row r sits at
    // r*128 + ((u ^ (r % 8)) * 16) of each 64-column chunk), so one float4
    // atomic instruction covers 512 contiguous bytes of sums[label] (16 full
    // sectors) instead of 32 scattered half-sectors.  Once its labels are
    // read the warp releases the label slot; once its rows are in registers
    // it releases the x buffer.  Runs concurrently with the next tile's
    // epilogue.
    if constexpr (L::kExtraRegs < L::kLaunchRegs) setmaxnreg_dec<L::kExtraRegs>();
    if constexpr (L::kSumWarps && XRES && sizeof(T) == 2) {
    const int sw = warp - kConvWarp0;  // 0..3
    const int col = 4 * lane;
    const int dc = col / p.dch;
    const int ub = (col % p.dch) * 2;  // byte of column `col` within its chunk
    const bool lane_on = col < p.D;
    const bool lane_vec = p.sums_vec && col + 4 <= p.D;
    int it = 0, xi = 0;
    for (int t = t_begin; t < t_end; ++t, ++it) {
      const int b = t / p.ntn;
      const int par = it & 1;
      const uint32_t mph = static_cast<uint32_t>((it >> 1) & 1);
      const bool got = mbar_wait(&lab_full[par], mph, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT);
      if (!__all_sync(0xffffffffu, got)) break;
      const int lab_mine = reinterpret_cast<const int*>(smem + L::lab_off)[par * kRows + sw * 32 + lane];
      mbar_arrive(&lab_empty[par]);
      const uint8_t* xsrc = smem + L::x_off + (xi * kResidentChunks + dc) * kXChunk + (ub & 15);
      float* const sums_b = p.sums + static_cast<int64_t>(b) * p.K * p.D + col;
      // The warp's 32 rows go to registers first and the x buffer is released
      // before any atomic is issued, so the producer can refill it while the
      // atomics drain (dot modes: 0.78 -> 0.70 ms at B=32, N=75600, K=1000).
      uint2 rows[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int r = sw * 32 + i;
        rows[i] = lane_on ? *reinterpret_cast<const uint2*>(xsrc + r * kChunkB +
                                                            (((ub >> 4) ^ (r & 7)) << 4))
                          : make_uint2(0u, 0u);
      }
      mbar_arrive(&x_empty[xi]);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int lab = __shfl_sync(0xffffffffu, lab_mine, i);
        if (lab < 0 || !lane_on) continue;
        const uint2 q = rows[i];
        const float f0 = Pack2<T>::lo(q.x), f1 = Pack2<T>::hi(q.x);
        const float f2 = Pack2<T>::lo(q.y), f3 = Pack2<T>::hi(q.y);
        float* dst = sums_b + static_cast<int64_t>(lab) * p.D;
        if (lane_vec) {
          atomicAdd(reinterpret_cast<float4*>(dst), make_float4(f0, f1, f2, f3));
        } else {
          atomicAdd(dst, f0);
          if (col + 1 < p.D) atomicAdd(dst + 1, f1);
          if (col + 2 < p.D) atomicAdd(dst + 2, f2);
          if (col + 3 < p.D) atomicAdd(dst + 3, f3);
        }
      }
      if (++xi == L::XB) xi = 0;
    }
    }
  } else if (split_mode(MODE)) {
    // ------------------------------------- 3xTF32 split converters (modes 2, 4)
    // Each stage's x chunk is split in place into tf32 hi and the exact lo
    // rest (the centroid chunks arrive already split, from the workspace).
    // With x split once per fit (p.xlo_b > 0) both halves arrive by TMA and
    // these warps have nothing to do.
    if constexpr (L::kExtraRegs < L::kLaunchRegs) setmaxnreg_dec<L::kExtraRegs>();
    const int ct = threadIdx.x - kConvWarp0 * 32;  // 0..127
    int stage = 0;
    uint32_t sph = 0;
    bool ok = p.xlo_b == 0;
    for (int t = t_begin; ok && t < t_end; ++t) {
      for (int kt = 0; ok && kt < p.nkt; ++kt) {
        for (int dc = 0; dc < p.nd; ++dc) {
          const bool got = mbar_wait(&c_full[stage], sph, abort_flag, p.status, FK_DEV_WAIT_TIMEOUT);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + L::stages_off + stage * L::stage_bytes;
          // hi = value rounded to tf32 (10 explicit mantissa bits), lo = exact rest
          auto split = [&](int hi_off, int lo_off, int nfloat4) {
            float4* hi = reinterpret_cast<float4*>(st + hi_off);
            float4* lo = reinterpret_cast<float4*>(st + lo_off);
            for (int i = ct; i < nfloat4; i += kConvWarps * 32) {
              float4 v = hi[i];
              float4 vh, vl;
              uint32_t u;
              u = (__float_as_uint(v.x) + 0x1000u) & 0xFFFFE000u; vh.x = __uint_as_float(u); vl.x = v.x - vh.x;
              u = (__float_as_uint(v.y) + 0x1000u) & 0xFFFFE000u; vh.y = __uint_as_float(u); vl.y = v.y - vh.y;
              u = (__float_as_uint(v.z) + 0x1000u) & 0xFFFFE000u; vh.z = __uint_as_float(u); vl.z = v.z - vh.z;
              u = (__float_as_uint(v.w) + 0x1000u) & 0xFFFFE000u; vh.w = __uint_as_float(u); vl.w = v.w - vh.w;
              hi[i] = vh;
              lo[i] = vl;
            }
          };
          split(L::st_x, L::st_xlo, L::kXChunkL / 16);   // the centroids arrive split
          fence_proxy_async_smem();
          mbar_arrive(&conv_full[stage]);
          if (++stage == STAGES) { stage = 0; sph ^= 1; }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ------------------------------------------------------------------ host side
template <typename T, int MODE, bool XRES, bool FUSE = false, int KC = kCent, bool RESC = false,
          bool W64 = false>
static int launch_assign(const CUtensorMap& tx, const CUtensorMap& tc, const AssignParams& p,
                         cudaStream_t stream) {
  // centroid ring depth (the narrow-tile ring holds as many bytes in twice the
  // stages; resident centroids need one stage per chunk of the batch)
  constexpr int STAGES = RESC ? kResidentChunks
                              : (split_mode(MODE) ? (W64 ? 4 : 2) : (FUSE ? 3 : (KC < kCent ? 6 : 4)));
  constexpr int EPI = 8;  // epilogue warps: 4 TMEM lane quarters x 2 column halves
  using L = Layout<MODE, XRES, STAGES, FUSE, EPI, KC, RESC>;
  static_assert(L::total <= 232448, "shared memory budget");
  if (RESC && p.nkt * p.nd > STAGES) return fail(FK_ERR_UNSUPPORTED, "resident centroids do not fit");
  auto kern = assign_kernel<T, MODE, XRES, STAGES, FUSE, EPI, KC, RESC>;
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return fail(FK_ERR_CUDA, "bad current device %d", dev);
  // Once per device and instance (only a successful set-up is remembered):
  // allow the dynamic shared memory, and check that the launch allocation
  // covers the warpgroups' register budgets (setmaxnreg.inc would otherwise
  // wait forever for registers that do not exist).
  static std::atomic<bool> ready[64];
  static std::mutex setup_mu;
  if (!ready[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(setup_mu);
    if (!ready[dev].load(std::memory_order_relaxed)) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::total);
      if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, kern);
      if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
      const long budget = 128L * L::kCtlRegs + 32L * EPI * L::kEpiRegs +
                          (L::kExtra ? 128L * L::kExtraRegs : 0L);
      if (static_cast<long>(fa.numRegs) * L::threads < budget || fa.numRegs > L::kLaunchRegs)
        return fail(FK_ERR_UNSUPPORTED,
                    "assign_kernel register split: %d registers x %d threads at launch, budgets "
                    "need %ld",
                    fa.numRegs, L::threads, budget);
      ready[dev].store(true, std::memory_order_release);
    }
  }
  const int sms = sm_count_current();
  if (sms <= 0) return fail(FK_ERR_CUDA, "could not query SM count");
  const int grid = p.total_tiles < sms ? p.total_tiles : sms;
  kern<<<grid, L::threads, L::total, stream>>>(tx, tc, p);
  return check_launch("assign_kernel");
}

// Stages the centroid-side operands of a Euclidean assignment:
// * csq_out (B, kpad): per-centroid squared norms in the epilogue's distance
//   dtype, +inf past K.  Modes 0/1 follow (c ** 2).sum(-1) in the 16-bit dtype
//   (torch_fallback.py:23), mode 2 float32; a caller-provided c_sq is
//   converted instead.
// * cneg (B, K, dp), modes 0/1 only: -2c in the 16-bit dtype, the MMA's
//   centroid operand (exact; saturated to the largest finite value where 2|c|
//   leaves the range).
// One warp per padded centroid row.
template <typename T, int MODE>
__global__ void prep_centroids_kernel(const T* __restrict__ c, int64_t scb, int64_t sck,
                                      int64_t scd, const void* csq_in, int csq_dtype, int64_t sqb,
                                      int64_t sqk, void* csq_out, int64_t kpad, T* cneg,
                                      int64_t dp, int B, int K, int D) {
  const int warps_per_block = blockDim.x >> 5;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t total = static_cast<int64_t>(B) * kpad;
  for (int64_t r = gw; r < total; r += static_cast<int64_t>(gridDim.x) * warps_per_block) {
    const int b = static_cast<int>(r / kpad);
    const int k = static_cast<int>(r % kpad);
    float v = __int_as_float(0x7f800000);
    if (k < K) {
      const T* row = c + b * scb + k * sck;
      T* nrow = cneg ? cneg + (static_cast<int64_t>(b) * K + k) * dp : nullptr;
      float acc = 0.0f;
      for (int d = lane; d < D; d += 32) {
        const float e = Elem<T>::to_f(row[d * scd]);
        acc += (MODE == 2) ? e * e : Elem<T>::round(e * e);
        if (nrow) nrow[d] = Elem<T>::from_f(fminf(fmaxf(-2.0f * e, -Elem<T>::kMaxFinite),
                                                  Elem<T>::kMaxFinite));
      }
      acc = warp_sum(acc);
      v = csq_in ? load_f(csq_in, b * sqb + k * sqk, csq_dtype)
                 : ((MODE == 2) ? acc : Elem<T>::round(acc));
    }
    if (lane == 0) {
      if (MODE == 0)
        static_cast<T*>(csq_out)[r] = Elem<T>::from_f(v);
      else
        static_cast<float*>(csq_out)[r] = v;
    }
  }
}

// c_sq given, 16-bit centroids stored densely (rows of D elements back to
// back, D a multiple of 8, 16-byte aligned): the -2c operand 16 bytes per
// thread step (the same per-element saturated -2e as prep_centroids_kernel),
// then the padded c_sq copy.  This is the Lloyd engine's steady state.
template <typename T, int MODE>
__global__ void prep_centroids_flat_kernel(const T* __restrict__ c, T* __restrict__ cneg,
                                           int64_t units, const void* __restrict__ csq_in,
                                           int csq_dtype, int64_t sqb, int64_t sqk,
                                           void* __restrict__ csq_out, int64_t kpad, int K,
                                           int64_t csq_total) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nth = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t u = tid; u < units; u += nth) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(c) + u);
    T* e = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      e[i] = Elem<T>::from_f(fminf(fmaxf(-2.0f * Elem<T>::to_f(e[i]), -Elem<T>::kMaxFinite),
                                   Elem<T>::kMaxFinite));
    reinterpret_cast<uint4*>(cneg)[u] = v;
  }
  for (int64_t r = tid; r < csq_total; r += nth) {
    const int64_t b = r / kpad;
    const int k = static_cast<int>(r - b * kpad);
    const float v = k < K ? load_f(csq_in, b * sqb + k * sqk, csq_dtype) : __int_as_float(0x7f800000);
    if (MODE == 0)
      static_cast<T*>(csq_out)[r] = Elem<T>::from_f(v);
    else
      static_cast<float*>(csq_out)[r] = v;
  }
}

// 3xTF32 modes: the centroids split once per call into tf32 hi parts
// (rounded to 10 explicit mantissa bits) and exact lo rests, each dense
// (B, K, dp) with zero padding, lo at hi + lo_off: the split the converter
// warps apply to the x chunks, done here once instead of for every point tile.
__global__ void split_centroids_kernel(const float* __restrict__ c, int64_t scb, int64_t sck,
                                       int64_t scd, float* __restrict__ hi, int64_t dp, int K,
                                       int D, int64_t total, int64_t lo_off) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / dp;
    const int d = static_cast<int>(i - row * dp);
    const int64_t b = row / K;
    const int k = static_cast<int>(row - b * K);
    const float v = d < D ? c[b * scb + k * sck + d * scd] : 0.0f;
    const float h = __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
    hi[i] = h;
    hi[lo_off + i] = v - h;
  }
}

// c_sq given: one thread per padded element (convert, +inf beyond K).
template <typename T, int MODE>
__global__ void copy_csq_kernel(const void* __restrict__ csq_in, int csq_dtype, int64_t sqb,
                                int64_t sqk, void* __restrict__ csq_out, int64_t kpad, int K,
                                int64_t total) {
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < total;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = r / kpad;
    const int k = static_cast<int>(r % kpad);
    const float v = k < K ? load_f(csq_in, b * sqb + k * sqk, csq_dtype) : __int_as_float(0x7f800000);
    if (MODE == 0)
      static_cast<T*>(csq_out)[r] = Elem<T>::from_f(v);
    else
      static_cast<float*>(csq_out)[r] = v;
  }
}

template <typename T>
static int assign_typed(const void* x, const void* cent, const void* x_sq, const void* c_sq,
                        int32_t* out, int32_t* counts, int xsq_dtype, int csq_dtype, int64_t B,
                        int64_t N, int64_t K, int64_t D, const int64_t* xs, const int64_t* cs,
                        const int64_t* xqs, const int64_t* cqs, const int64_t* os, void* ws,
                        int32_t* status, cudaStream_t stream, float* sums = nullptr,
                        bool dot = false, bool xsplit = false) {
  constexpr int eb = Elem<T>::kBytes;
  const bool is16 = eb == 2;
  const int mode = dot ? (is16 ? 3 : 4) : (is16 ? (xsq_dtype == Elem<T>::kDtype ? 0 : 1) : 2);
  // elements per chunk row: 128 bytes, or 64 in the four-stage 3xTF32 form
  // (float32 rows of at least kW64MinD elements)
  const bool w64 = !is16 && D >= kW64MinD;
  const int dch = (w64 ? 64 : kChunkB) / eb;
  const int nd = static_cast<int>((D + dch - 1) / dch);
  const bool xres = is16 && nd <= kResidentChunks;
  // K <= 128 (one centroid tile either way): 128-column tiles, so the epilogue
  // skips the padding half of a 256-column tile and TMEM holds four accumulators
  // (with fused sums the narrow kernel accumulates them on the tensor core)
  const bool narrow = is16 && K <= kCent / 2;
  const int kc = narrow ? kCent / 2 : kCent;
  const int nkt = static_cast<int>((K + kc - 1) / kc);
  const int64_t kpad = static_cast<int64_t>(nkt) * kc;

  // 1) padded c_sq in the distance dtype and, for the 16-bit Euclidean modes,
  //    the -2c operand (the dot-product modes stage nothing: their epilogue
  //    masks the padding columns itself)
  const int64_t dp = static_cast<int64_t>(align_up(static_cast<size_t>(D), 8));
  T* cneg = nullptr;
  if (!dot && is16)
    cneg = reinterpret_cast<T*>(static_cast<uint8_t*>(ws) + assign_csq_bytes(B, K));
  // float32 (3xTF32 modes): the centroids' hi and lo halves, (2B, K, dp)
  float* csplit = nullptr;
  if (!is16) {
    csplit = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + assign_csq_bytes(B, K));
    const int64_t total = B * K * dp;
    const int sms = sm_count_current();
    const int64_t cap = sms > 0 ? static_cast<int64_t>(sms) * 8 : 1024;
    const int blocks = static_cast<int>((total + 255) / 256 < cap ? (total + 255) / 256 : cap);
    split_centroids_kernel<<<blocks, 256, 0, stream>>>(static_cast<const float*>(cent), cs[0], cs[1],
                                                       cs[2], csplit, dp, (int)K, (int)D, total,
                                                       total);
    int st = check_launch("split_centroids_kernel");
    if (st != FK_OK) return st;
  }
  if (dot) {
    // nothing to stage
  } else if (c_sq && mode == 2) {
    const int64_t total = B * kpad;
    const int blocks = static_cast<int>((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    copy_csq_kernel<T, 2><<<blocks, 256, 0, stream>>>(c_sq, csq_dtype, cqs[0], cqs[1], ws, kpad,
                                                       (int)K, total);
    int st = check_launch("copy_csq_kernel");
    if (st != FK_OK) return st;
  } else if (c_sq && cneg && dp == D && cs[2] == 1 && cs[1] == D && (B == 1 || cs[0] == K * D) &&
             reinterpret_cast<uintptr_t>(cent) % 16 == 0) {
    // steady state of the Lloyd engine: dense centroids, c_sq from the update
    const int64_t units = B * K * D / 8;
    const int64_t csq_total = B * kpad;
    const int64_t work = units > csq_total ? units : csq_total;
    const int sms = sm_count_current();
    const int64_t cap = sms > 0 ? static_cast<int64_t>(sms) * 8 : 1024;
    const int blocks = static_cast<int>((work + 255) / 256 < cap ? (work + 255) / 256 : cap);
    const T* c = static_cast<const T*>(cent);
    if constexpr (eb == 2) {   // cneg exists for 16-bit centroids only (8 per 16 bytes)
      if (mode == 0)
        prep_centroids_flat_kernel<T, 0><<<blocks, 256, 0, stream>>>(
            c, cneg, units, c_sq, csq_dtype, cqs[0], cqs[1], ws, kpad, (int)K, csq_total);
      else
        prep_centroids_flat_kernel<T, 1><<<blocks, 256, 0, stream>>>(
            c, cneg, units, c_sq, csq_dtype, cqs[0], cqs[1], ws, kpad, (int)K, csq_total);
    }
    int st = check_launch("prep_centroids_flat_kernel");
    if (st != FK_OK) return st;
  } else {
    const int threads = 256;
    const int64_t rows = B * kpad;
    const int blocks = static_cast<int>(rows / 8 + 1 < 4096 ? rows / 8 + 1 : 4096);
    const T* c = static_cast<const T*>(cent);
    const int64_t sqb = c_sq ? cqs[0] : 0, sqk = c_sq ? cqs[1] : 0;
    if (mode == 0)
      prep_centroids_kernel<T, 0><<<blocks, threads, 0, stream>>>(
          c, cs[0], cs[1], cs[2], c_sq, csq_dtype, sqb, sqk, ws, kpad, cneg, dp, (int)B, (int)K,
          (int)D);
    else if (mode == 1)
      prep_centroids_kernel<T, 1><<<blocks, threads, 0, stream>>>(
          c, cs[0], cs[1], cs[2], c_sq, csq_dtype, sqb, sqk, ws, kpad, cneg, dp, (int)B, (int)K,
          (int)D);
    else
      prep_centroids_kernel<T, 2><<<blocks, threads, 0, stream>>>(
          c, cs[0], cs[1], cs[2], c_sq, csq_dtype, sqb, sqk, ws, kpad, nullptr, dp, (int)B,
          (int)K, (int)D);
    int st = check_launch("prep_centroids_kernel");
    if (st != FK_OK) return st;
  }

  // 2) tensor maps: x as (D, N, B), centroids (or -2c) as (D, K, B), 128-byte swizzle
  CUtensorMap tx, tc;
  // (x split once per fit: its hi halves are batches [0, B), the lo halves [B, 2B))
  int st = encode_tmap_3d(&tx, x, Elem<T>::kDtype, D, N, xsplit ? 2 * B : B, xs[1] * eb, xs[0] * eb,
                          dch, kRows, w64);
  if (st != FK_OK) return st;
  if (cneg)
    st = encode_tmap_3d(&tc, cneg, Elem<T>::kDtype, D, K, B, dp * eb, K * dp * eb, dch, kc);
  else if (csplit)  // hi halves in batches [0, B), lo halves in [B, 2B)
    st = encode_tmap_3d(&tc, csplit, Elem<T>::kDtype, D, K, 2 * B, dp * eb, K * dp * eb, dch, kc, w64);
  else
    st = encode_tmap_3d(&tc, cent, Elem<T>::kDtype, D, K, B, cs[1] * eb, cs[0] * eb, dch, kc, w64);
  if (st != FK_OK) return st;

  AssignParams p;
  p.xsq = x_sq;
  p.sxq_b = xqs ? xqs[0] : 0;  // x_sq is not used by the dot-product modes
  p.sxq_n = xqs ? xqs[1] : 0;
  p.xsq_dtype = xsq_dtype;
  p.csq = ws;
  p.kpad = kpad;
  p.out = out;
  p.so_b = os[0];
  p.so_n = os[1];
  p.counts = counts;
  p.sums = sums;
  p.D = static_cast<int>(D);
  p.sums_vec = (D % 4 == 0) && (reinterpret_cast<uintptr_t>(sums) % 16 == 0);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.nd = nd;
  p.dch = dch;
  p.ntn = static_cast<int>((N + kRows - 1) / kRows);
  p.nkt = nkt;
  p.total_tiles = static_cast<int>(B * p.ntn);
  p.status = status;
  p.lo_b = static_cast<int>(B);
  p.xlo_b = xsplit ? static_cast<int>(B) : 0;

  if (dot) {
    if constexpr (Elem<T>::kBytes == 2) {
      if (sums) {
        if (!xres) return fail(FK_ERR_UNSUPPORTED, "fused sums need a resident x tile");
        return narrow ? launch_assign<T, 3, true, true, kCent / 2, true>(tx, tc, p, stream)
                      : launch_assign<T, 3, true, true>(tx, tc, p, stream);
      }
      if (narrow)
        return xres ? launch_assign<T, 3, true, false, kCent / 2, true>(tx, tc, p, stream)
                    : launch_assign<T, 3, false, false, kCent / 2>(tx, tc, p, stream);
      return xres ? launch_assign<T, 3, true>(tx, tc, p, stream)
                  : launch_assign<T, 3, false>(tx, tc, p, stream);
    } else {
      if (sums) return fail(FK_ERR_UNSUPPORTED, "fused sums need 16-bit x");
      return w64 ? launch_assign<T, 4, false, false, kCent, false, true>(tx, tc, p, stream)
                 : launch_assign<T, 4, false>(tx, tc, p, stream);
    }
  }
  if constexpr (Elem<T>::kBytes == 2) {
    if (sums) {  // fused centroid sums: resident x tiles only (checked by the caller)
      if (!xres) return fail(FK_ERR_UNSUPPORTED, "fused sums need a resident x tile");
      if (narrow)  // K <= 128: one-hot sums on the tensor core
        return mode == 0 ? launch_assign<T, 0, true, true, kCent / 2, true>(tx, tc, p, stream)
                         : launch_assign<T, 1, true, true, kCent / 2, true>(tx, tc, p, stream);
      return mode == 0 ? launch_assign<T, 0, true, true>(tx, tc, p, stream)
                       : launch_assign<T, 1, true, true>(tx, tc, p, stream);
    }
    if (narrow) {  // one centroid tile: resident in the stages when x is resident
      if (mode == 0) return xres ? launch_assign<T, 0, true, false, kCent / 2, true>(tx, tc, p, stream)
                                 : launch_assign<T, 0, false, false, kCent / 2>(tx, tc, p, stream);
      return xres ? launch_assign<T, 1, true, false, kCent / 2, true>(tx, tc, p, stream)
                  : launch_assign<T, 1, false, false, kCent / 2>(tx, tc, p, stream);
    }
    if (mode == 0) return xres ? launch_assign<T, 0, true>(tx, tc, p, stream)
                               : launch_assign<T, 0, false>(tx, tc, p, stream);
    return xres ? launch_assign<T, 1, true>(tx, tc, p, stream)
                : launch_assign<T, 1, false>(tx, tc, p, stream);
  } else {
    return w64 ? launch_assign<T, 2, false, false, kCent, false, true>(tx, tc, p, stream)
               : launch_assign<T, 2, false>(tx, tc, p, stream);
  }
}

}  // namespace fk

using namespace fk;

// Workspace of fk_assign: c_sq padded to whole 256-column tiles (4 bytes per
// entry covers every mode), then for 16-bit x the -2c operand (B, K, D
// rounded up to 8 elements).
extern "C" size_t fk_assign_workspace_size(int64_t B, int64_t K, int64_t D, int dtype) {
  if (B <= 0 || K <= 0 || D <= 0) return 256;
  size_t bytes = assign_csq_bytes(B, K);
  if (dtype == FK_F16 || dtype == FK_BF16)
    bytes += align_up(static_cast<size_t>(B * K) * align_up(static_cast<size_t>(D), 8) * 2, 256);
  else  // float32: the centroids' tf32 hi and lo halves
    bytes += align_up(static_cast<size_t>(B * K) * align_up(static_cast<size_t>(D), 8) * 8, 256);
  return bytes + 256;
}

// fk_assign and fk_assign_dot: validation, TMA-friendly strides, dispatch.
static int assign_entry(const char* fn, bool dot, const void* x, const void* centroids,
                        const void* x_sq, const void* c_sq, int32_t* out, int32_t* counts,
                        int dtype, int xsq_dtype, int csq_dtype, int64_t B, int64_t N, int64_t K,
                        int64_t D, const int64_t* x_strides3, const int64_t* c_strides3,
                        const int64_t* xsq_strides2, const int64_t* csq_strides2,
                        const int64_t* out_strides2, void* workspace, size_t workspace_bytes,
                        int32_t* dev_status, void* stream, bool xsplit = false) {
  if (B < 0 || N < 0 || K <= 0 || D <= 0)
    return fail(FK_ERR_INVALID_ARG, "%s: bad sizes B=%lld N=%lld K=%lld D=%lld", fn,
                (long long)B, (long long)N, (long long)K, (long long)D);
  if (B == 0 || N == 0) return FK_OK;
  if (!x || !centroids || (!dot && !x_sq) || !out || !x_strides3 || !c_strides3 ||
      (!dot && !xsq_strides2) || !out_strides2)
    return fail(FK_ERR_INVALID_ARG, "%s: null pointer argument", fn);
  if (c_sq && !csq_strides2) return fail(FK_ERR_INVALID_ARG, "%s: c_sq without strides", fn);
  if (dtype != FK_F16 && dtype != FK_BF16 && dtype != FK_F32)
    return fail(FK_ERR_INVALID_ARG, "%s: x dtype must be f16, bf16 or f32", fn);
  if (!dot && xsq_dtype != FK_F16 && xsq_dtype != FK_BF16 && xsq_dtype != FK_F32)
    return fail(FK_ERR_INVALID_ARG, "%s: x_sq dtype must be floating", fn);
  if (c_sq && csq_dtype != FK_F16 && csq_dtype != FK_BF16 && csq_dtype != FK_F32)
    return fail(FK_ERR_INVALID_ARG, "%s: c_sq dtype must be floating", fn);
  if (K > (1 << 20)) return fail(FK_ERR_UNSUPPORTED, "%s: K=%lld above 2^20", fn, (long long)K);
  if (N >= (1ll << 31) || B * ((N + kRows - 1) / kRows) >= (1ll << 31))
    return fail(FK_ERR_UNSUPPORTED, "%s: problem too large for 32-bit tile indices", fn);
  // Strides of size-1 dimensions are irrelevant; give TMA valid ones.
  const int64_t eb = dtype == FK_F32 ? 4 : 2;
  const int64_t row_al = 16 / eb;
  int64_t xs[3] = {x_strides3[0], x_strides3[1], x_strides3[2]};
  int64_t cs[3] = {c_strides3[0], c_strides3[1], c_strides3[2]};
  if (D == 1) { xs[2] = 1; cs[2] = 1; }
  if (N == 1) xs[1] = (D + row_al - 1) / row_al * row_al;
  if (K == 1) cs[1] = (D + row_al - 1) / row_al * row_al;
  if (B == 1) { xs[0] = N * xs[1]; cs[0] = K * cs[1]; }
  x_strides3 = xs;
  c_strides3 = cs;
  if (!fk_tma_compatible(x, dtype, D, x_strides3))
    return fail(FK_ERR_UNSUPPORTED, "%s: x rows not TMA-addressable (pack with fk_pack_rows)", fn);
  if (!fk_tma_compatible(centroids, dtype, D, c_strides3))
    return fail(FK_ERR_UNSUPPORTED, "%s: centroid rows not TMA-addressable", fn);
  const size_t need = fk_assign_workspace_size(B, K, D, dtype);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(FK_ERR_WORKSPACE, "%s: workspace needs %zu bytes, 256-aligned", fn, need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case FK_F16:
      return assign_typed<__half>(x, centroids, x_sq, c_sq, out, counts, xsq_dtype, csq_dtype, B, N,
                                  K, D, x_strides3, c_strides3, xsq_strides2, csq_strides2,
                                  out_strides2, workspace, dev_status, s, nullptr, dot);
    case FK_BF16:
      return assign_typed<__nv_bfloat16>(x, centroids, x_sq, c_sq, out, counts, xsq_dtype,
                                         csq_dtype, B, N, K, D, x_strides3, c_strides3,
                                         xsq_strides2, csq_strides2, out_strides2, workspace,
                                         dev_status, s, nullptr, dot);
    default:
      return assign_typed<float>(x, centroids, x_sq, c_sq, out, counts, xsq_dtype, csq_dtype, B, N,
                                 K, D, x_strides3, c_strides3, xsq_strides2, csq_strides2,
                                 out_strides2, workspace, dev_status, s, nullptr, dot, xsplit);
  }
}

extern "C" int fk_assign(const void* x, const void* centroids, const void* x_sq, const void* c_sq,
                         int32_t* out, int32_t* counts, int dtype, int xsq_dtype, int csq_dtype,
                         int64_t B, int64_t N, int64_t K, int64_t D, const int64_t* x_strides3,
                         const int64_t* c_strides3, const int64_t* xsq_strides2,
                         const int64_t* csq_strides2, const int64_t* out_strides2, void* workspace,
                         size_t workspace_bytes, int32_t* dev_status, void* stream) {
  return assign_entry("fk_assign", false, x, centroids, x_sq, c_sq, out, counts, dtype, xsq_dtype,
                      csq_dtype, B, N, K, D, x_strides3, c_strides3, xsq_strides2, csq_strides2,
                      out_strides2, workspace, workspace_bytes, dev_status, stream);
}

extern "C" int fk_assign_dot(const void* x, const void* centroids, int32_t* out, int32_t* counts,
                             int dtype, int64_t B, int64_t N, int64_t K, int64_t D,
                             const int64_t* x_strides3, const int64_t* c_strides3,
                             const int64_t* out_strides2, void* workspace, size_t workspace_bytes,
                             int32_t* dev_status, void* stream) {
  return assign_entry("fk_assign_dot", true, x, centroids, nullptr, nullptr, out, counts, dtype,
                      FK_F32, FK_F32, B, N, K, D, x_strides3, c_strides3, nullptr, nullptr,
                      out_strides2, workspace, workspace_bytes, dev_status, stream);
}

// ---------------------------------------------------------------------------
// fk_assign_accumulate: assignment plus centroid sums/counts in one pass.
// 16-bit x with D <= 128 (x tile resident in shared memory): one kernel; each
// point's row is added to sums[label] right after its label is decided, so x
// is read once per Lloyd iteration.  Other layouts: fk_assign with a workspace
// histogram followed by fk_centroid_accumulate (counting-sort path).
// ---------------------------------------------------------------------------
// How fk_assign_accumulate accumulates:
//   fused (16-bit x with D <= 128, x read once): with K <= 128 the narrow
//     assignment kernel also multiplies each tile's one-hot label matrix with
//     the resident x tile on the tensor core into TMEM sums, added to the
//     global sums once per batch and CTA; with larger K, when a batch's K x D
//     float32 sums do not fit in shared memory, the sum warps of the
//     assignment kernel add each point's resident row with vector atomics;
//   privatised: K x D small enough for shared memory otherwise; fk_assign
//     (labels only) then the privatised segmented sum, which reads x a second
//     time but adds each CTA's partial sums to the global ones once;
//   sorted: otherwise fk_assign then fk_centroid_accumulate's counting sort.
// 16-bit x whose tile stays resident in shared memory (D <= 128)
static bool assign_accumulate_resident16(int64_t D, int dtype) {
  if (dtype != FK_F16 && dtype != FK_BF16) return false;
  const int64_t nd = (D * 2 + kChunkB - 1) / kChunkB;
  return nd <= kResidentChunks;
}

// fused: one kernel reads x once; with K <= 128 the sums are a one-hot
// product on the tensor core, otherwise (when a batch's K x D sums do not fit
// in shared memory) the sum warps add rows with vector atomics
static bool assign_accumulate_fused(int64_t K, int64_t D, int dtype) {
  if (!assign_accumulate_resident16(D, dtype)) return false;
  return K <= kCent / 2 || !segsum_priv_fits(K, D);
}

static bool assign_accumulate_priv(int64_t K, int64_t D, int dtype) {
  return !assign_accumulate_fused(K, D, dtype) && segsum_priv_fits(K, D);
}

extern "C" int fk_assign_accumulate_method(int64_t K, int64_t D, int dtype) {
  if (dtype == FK_F32_XSPLIT) dtype = FK_F32;
  if (assign_accumulate_fused(K, D, dtype)) return FK_ACC_FUSED;
  return assign_accumulate_priv(K, D, dtype) ? FK_ACC_PRIVATISED : FK_ACC_SORTED;
}

// FK_F32_XSPLIT: x's tf32 hi halves and exact rests, (2B, N, Dx) float32 with
// Dx = D rounded up to 4 (16-byte rows for TMA), after FK_F32's workspace.
static int64_t xsplit_row(int64_t D) { return (D + 3) / 4 * 4; }

static size_t xsplit_offset(int64_t B, int64_t N, int64_t K, int64_t D) {
  return align_up(fk_assign_accumulate_workspace_size(B, N, K, D, FK_F32), 256);
}

extern "C" size_t fk_assign_accumulate_workspace_size(int64_t B, int64_t N, int64_t K, int64_t D,
                                                      int dtype) {
  if (dtype == FK_F32_XSPLIT) {
    const size_t rows = (B > 0 && N > 0) ? static_cast<size_t>(2 * B * N) : 0;
    return xsplit_offset(B, N, K, D) + align_up(rows * xsplit_row(D > 0 ? D : 1) * 4, 256);
  }
  const size_t wa = fk_assign_workspace_size(B, K, D, dtype);
  if (assign_accumulate_priv(K, D, dtype) || assign_accumulate_fused(K, D, dtype)) return wa;
  return wa + align_up(static_cast<size_t>(B > 0 && K > 0 ? B * K : 1) * 4, 256) +
         fk_centroid_accumulate_workspace_size(B, N, K);
}

// fk_assign_accumulate and fk_assign_dot_accumulate: the method of
// fk_assign_accumulate_method (privatised sum after the assignment, sums
// fused into the assignment, or assignment then counting sort + segmented sum).
static int assign_accumulate_entry(const char* fn, bool dot, const void* x, const void* centroids,
                                   const void* x_sq, const void* c_sq, int32_t* out,
                                   int32_t* counts, float* sums, int dtype, int xsq_dtype,
                                   int csq_dtype, int64_t B, int64_t N, int64_t K, int64_t D,
                                   const int64_t* x_strides3, const int64_t* c_strides3,
                                   const int64_t* xsq_strides2, const int64_t* csq_strides2,
                                   const int64_t* out_strides2, void* workspace,
                                   size_t workspace_bytes, int32_t* dev_status, void* stream) {
  if (!counts || !sums) return fail(FK_ERR_INVALID_ARG, "%s: counts and sums are required", fn);
  if (B < 0 || N < 0 || K <= 0 || D <= 0) return fail(FK_ERR_INVALID_ARG, "%s: bad sizes", fn);
  if (B == 0 || N == 0) return FK_OK;
  const size_t need = fk_assign_accumulate_workspace_size(B, N, K, D, dtype);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(FK_ERR_WORKSPACE, "%s: workspace needs %zu bytes, 256-aligned", fn, need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // FK_F32_XSPLIT: the assignment reads x's halves from the workspace, the
  // sums read x itself
  const bool xsplit = dtype == FK_F32_XSPLIT;
  if (xsplit) dtype = FK_F32;
  const void* xa = x;
  const int64_t* xa_strides = x_strides3;
  int64_t xs_split[3] = {0, 0, 1};
  if (xsplit) {
    const int64_t dx = xsplit_row(D);
    xs_split[0] = N * dx;
    xs_split[1] = dx;
    xa = static_cast<uint8_t*>(workspace) + xsplit_offset(B, N, K, D);
    xa_strides = xs_split;
  }
  auto assign = [&](int32_t* cnt, size_t ws_bytes) {
    return assign_entry(fn, dot, xa, centroids, x_sq, c_sq, out, cnt, dtype, xsq_dtype, csq_dtype,
                        B, N, K, D, xa_strides, c_strides3, xsq_strides2, csq_strides2,
                        out_strides2, workspace, ws_bytes, dev_status, stream, xsplit);
  };
  if (assign_accumulate_priv(K, D, dtype)) {
    int st = assign(nullptr, workspace_bytes);
    if (st != FK_OK) return st;
    return segsum_priv(x, dtype, x_strides3, out, FK_I32, out_strides2, B, N, K, D, sums, counts,
                       dev_status, s);
  }
  if (!assign_accumulate_fused(K, D, dtype)) {
    const size_t wa = fk_assign_workspace_size(B, K, D, dtype);
    int32_t* hist = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + wa);
    void* wu = static_cast<uint8_t*>(workspace) + wa + align_up(static_cast<size_t>(B * K) * 4, 256);
    cudaError_t e = cudaMemsetAsync(hist, 0, static_cast<size_t>(B * K) * 4, s);
    if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    int st = assign(hist, wa);
    if (st != FK_OK) return st;
    return fk_centroid_accumulate(x, dtype, B, N, K, D, x_strides3, out, FK_I32, out_strides2,
                                  hist, sums, counts, wu,
                                  fk_centroid_accumulate_workspace_size(B, N, K), dev_status,
                                  stream);
  }
  // fused path: same validation as fk_assign
  if (!x || !centroids || (!dot && !x_sq) || !out || !x_strides3 || !c_strides3 ||
      (!dot && !xsq_strides2) || !out_strides2)
    return fail(FK_ERR_INVALID_ARG, "%s: null pointer argument", fn);
  if (c_sq && !csq_strides2) return fail(FK_ERR_INVALID_ARG, "%s: c_sq without strides", fn);
  if (!dot && xsq_dtype != FK_F16 && xsq_dtype != FK_BF16 && xsq_dtype != FK_F32)
    return fail(FK_ERR_INVALID_ARG, "%s: x_sq dtype must be floating", fn);
  if (c_sq && csq_dtype != FK_F16 && csq_dtype != FK_BF16 && csq_dtype != FK_F32)
    return fail(FK_ERR_INVALID_ARG, "%s: c_sq dtype must be floating", fn);
  if (K > (1 << 20)) return fail(FK_ERR_UNSUPPORTED, "%s: K above 2^20", fn);
  if (N >= (1ll << 31) || B * ((N + kRows - 1) / kRows) >= (1ll << 31))
    return fail(FK_ERR_UNSUPPORTED, "%s: problem too large", fn);
  const int64_t row_al = 8;
  int64_t xs[3] = {x_strides3[0], x_strides3[1], x_strides3[2]};
  int64_t cs[3] = {c_strides3[0], c_strides3[1], c_strides3[2]};
  if (D == 1) { xs[2] = 1; cs[2] = 1; }
  if (N == 1) xs[1] = (D + row_al - 1) / row_al * row_al;
  if (K == 1) cs[1] = (D + row_al - 1) / row_al * row_al;
  if (B == 1) { xs[0] = N * xs[1]; cs[0] = K * cs[1]; }
  if (!fk_tma_compatible(x, dtype, D, xs))
    return fail(FK_ERR_UNSUPPORTED, "%s: x rows not TMA-addressable", fn);
  if (!fk_tma_compatible(centroids, dtype, D, cs))
    return fail(FK_ERR_UNSUPPORTED, "%s: centroid rows not TMA-addressable", fn);
  if (dtype == FK_F16)
    return assign_typed<__half>(x, centroids, x_sq, c_sq, out, counts, xsq_dtype, csq_dtype, B, N, K,
                                D, xs, cs, xsq_strides2, csq_strides2, out_strides2, workspace,
                                dev_status, s, sums, dot);
  return assign_typed<__nv_bfloat16>(x, centroids, x_sq, c_sq, out, counts, xsq_dtype, csq_dtype, B,
                                     N, K, D, xs, cs, xsq_strides2, csq_strides2, out_strides2,
                                     workspace, dev_status, s, sums, dot);
}

extern "C" int fk_assign_accumulate(const void* x, const void* centroids, const void* x_sq,
                                    const void* c_sq, int32_t* out, int32_t* counts, float* sums,
                                    int dtype, int xsq_dtype, int csq_dtype, int64_t B, int64_t N,
                                    int64_t K, int64_t D, const int64_t* x_strides3,
                                    const int64_t* c_strides3, const int64_t* xsq_strides2,
                                    const int64_t* csq_strides2, const int64_t* out_strides2,
                                    void* workspace, size_t workspace_bytes, int32_t* dev_status,
                                    void* stream) {
  return assign_accumulate_entry("fk_assign_accumulate", false, x, centroids, x_sq, c_sq, out,
                                 counts, sums, dtype, xsq_dtype, csq_dtype, B, N, K, D, x_strides3,
                                 c_strides3, xsq_strides2, csq_strides2, out_strides2, workspace,
                                 workspace_bytes, dev_status, stream);
}

extern "C" int fk_assign_dot_accumulate(const void* x, const void* centroids, int32_t* out,
                                        int32_t* counts, float* sums, int dtype, int64_t B,
                                        int64_t N, int64_t K, int64_t D,
                                        const int64_t* x_strides3, const int64_t* c_strides3,
                                        const int64_t* out_strides2, void* workspace,
                                        size_t workspace_bytes, int32_t* dev_status, void* stream) {
  return assign_accumulate_entry("fk_assign_dot_accumulate", true, x, centroids, nullptr, nullptr,
                                 out, counts, sums, dtype, FK_F32, FK_F32, B, N, K, D, x_strides3,
                                 c_strides3, nullptr, nullptr, out_strides2, workspace,
                                 workspace_bytes, dev_status, stream);
}

// ---------------------------------------------------------------------------
// fk_assign_accumulate_split_x: x's tf32 hi halves and exact rests, once per
// fit, into the FK_F32_XSPLIT workspace (hi = the split_centroids_kernel rule).
// ---------------------------------------------------------------------------
namespace fk {
__device__ __forceinline__ float tf32_hi(float v) {
  return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
}

// dense x (rows of D % 4 == 0 floats back to back): four floats per thread step
__global__ void split_rows_flat_kernel(const float4* __restrict__ x, float4* __restrict__ out,
                                       int64_t n4) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = __ldcs(x + i);
    float4 h, l;
    h.x = tf32_hi(v.x); l.x = v.x - h.x;
    h.y = tf32_hi(v.y); l.y = v.y - h.y;
    h.z = tf32_hi(v.z); l.z = v.z - h.z;
    h.w = tf32_hi(v.w); l.w = v.w - h.w;
    __stcs(out + i, h);
    __stcs(out + n4 + i, l);
  }
}
// rows with their own batch and row strides (unit column stride, D % 4 == 0,
// 16-byte aligned rows, e.g. one block of a larger buffer): one warp per row
// step, so the row's batch and index cost one division per row, not per element
__global__ void split_rows_vec_kernel(const float* __restrict__ x, int64_t sxb, int64_t sxn,
                                      float4* __restrict__ out, int N, int d4, int64_t rows) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t lo_off = rows * d4;
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += nw) {
    const int64_t b = r / N;
    const float4* src = reinterpret_cast<const float4*>(x + b * sxb + (r - b * N) * sxn);
    float4* dst = out + r * d4;
    for (int j = lane; j < d4; j += 32) {
      const float4 v = __ldcs(src + j);
      float4 h, l;
      h.x = tf32_hi(v.x); l.x = v.x - h.x;
      h.y = tf32_hi(v.y); l.y = v.y - h.y;
      h.z = tf32_hi(v.z); l.z = v.z - h.z;
      h.w = tf32_hi(v.w); l.w = v.w - h.w;
      __stcs(dst + j, h);
      __stcs(dst + lo_off + j, l);
    }
  }
}
}  // namespace fk

extern "C" int fk_assign_accumulate_split_x(const float* x, int64_t B, int64_t N, int64_t K,
                                            int64_t D, const int64_t* x_strides3, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  if (B < 0 || N < 0 || K <= 0 || D <= 0)
    return fail(FK_ERR_INVALID_ARG, "fk_assign_accumulate_split_x: bad sizes");
  if (B == 0 || N == 0) return FK_OK;
  if (!x || !x_strides3) return fail(FK_ERR_INVALID_ARG, "fk_assign_accumulate_split_x: null x");
  if (N >= (1ll << 31)) return fail(FK_ERR_UNSUPPORTED, "fk_assign_accumulate_split_x: N >= 2^31");
  const size_t need = fk_assign_accumulate_workspace_size(B, N, K, D, FK_F32_XSPLIT);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(FK_ERR_WORKSPACE, "fk_assign_accumulate_split_x: workspace needs %zu bytes, 256-aligned",
                need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* out = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + xsplit_offset(B, N, K, D));
  const int64_t dx = xsplit_row(D);
  const int64_t xs0 = B == 1 ? N * x_strides3[1] : x_strides3[0];
  const bool dense = D == dx && x_strides3[2] == 1 && (N == 1 || x_strides3[1] == D) &&
                     xs0 == N * D && reinterpret_cast<uintptr_t>(x) % 16 == 0;
  const int sms = sm_count_current();
  const int64_t cap = sms > 0 ? static_cast<int64_t>(sms) * 8 : 1024;
  if (dense) {
    const int64_t n4 = B * N * D / 4;
    const int blocks = static_cast<int>((n4 + 255) / 256 < cap ? (n4 + 255) / 256 : cap);
    split_rows_flat_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4*>(x),
                                                  reinterpret_cast<float4*>(out), n4);
    return check_launch("split_rows_flat_kernel");
  }
  if (D == dx && x_strides3[2] == 1 && xs0 % 4 == 0 && (N == 1 || x_strides3[1] % 4 == 0) &&
      reinterpret_cast<uintptr_t>(x) % 16 == 0) {
    const int64_t rows = B * N;   // eight rows per 256-thread block step
    const int blocks = static_cast<int>((rows + 7) / 8 < cap ? (rows + 7) / 8 : cap);
    split_rows_vec_kernel<<<blocks, 256, 0, s>>>(x, xs0, N == 1 ? 0 : x_strides3[1],
                                                 reinterpret_cast<float4*>(out), static_cast<int>(N),
                                                 static_cast<int>(D / 4), rows);
    return check_launch("split_rows_vec_kernel");
  }
  // any strides: one element per thread step, zeros in columns [D, Dx)
  const int64_t total = B * N * dx;
  const int blocks = static_cast<int>((total + 255) / 256 < cap ? (total + 255) / 256 : cap);
  split_centroids_kernel<<<blocks, 256, 0, s>>>(x, xs0, N == 1 ? dx : x_strides3[1], x_strides3[2],
                                                out, dx, static_cast<int>(N), static_cast<int>(D),
                                                total, total);
  return check_launch("split_centroids_kernel");
}

// ---------------------------------------------------------------------------
// fk_assign_static_scratch: fk_assign for callers that cannot allocate.
//
// Some hosts hand a plugin only its input and output buffers: an inference
// server's custom-op interface with no workspace hook, a framework whose
// memory pool forbids side allocations, or a latency-bound loop where
// cudaMalloc/cudaFree (which can synchronise the device) is not acceptable.
// This entry point needs no caller workspace: its scratch (what
// fk_assign_workspace_size reports: the padded per-centroid squared norms
// and, for 16-bit x, the -2c operand) lives in the file-scope device array
// below, which every GPU that loads this library holds until the process
// exits.
//
// * Limit: kAssignStaticScratchBytes = 16 MiB, i.e.
//   fk_assign_workspace_size(B, K, D, dtype) <= 16 MiB (for example B=32,
//   K=1000, D=128 float16 needs 8.3 MiB); larger problems are rejected with
//   FK_ERR_WORKSPACE before anything is launched.
// * The first call on a device looks up the array's device address for that
//   device (cudaGetSymbolAddress, with that device current); make that first
//   call before any stream capture.  A failed lookup is not remembered: the
//   next call tries again.
// * All calls on a device share the one array and it keeps the last call's
//   contents; every call rewrites all the scratch it reads, so nothing needs
//   clearing, but calls that overlap on the GPU (different streams, or
//   different host threads on the same device) race on it.
// * No cudaMalloc, cudaFree or allocating library routine is called.
// ---------------------------------------------------------------------------
namespace fk {

constexpr size_t kAssignStaticScratchBytes = size_t(16) << 20;
static __device__ __align__(256) uint8_t g_assign_static_scratch[kAssignStaticScratchBytes];

// Per-device address of the array; only a successful lookup is kept.
static std::atomic<void*> g_static_scratch_ptr[64];
static std::mutex g_static_scratch_mu;

static int static_scratch_for_current_device(void** out) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return fail(FK_ERR_CUDA, "fk_assign_static_scratch: bad current device");
  void* ptr = g_static_scratch_ptr[dev].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    std::lock_guard<std::mutex> lock(g_static_scratch_mu);
    ptr = g_static_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (ptr == nullptr) {
      // runs with `dev` current: the caller's current device is this slot's device
      const cudaError_t e = cudaGetSymbolAddress(&ptr, g_assign_static_scratch);
      if (e != cudaSuccess || ptr == nullptr)
        return fail(FK_ERR_CUDA,
                    "fk_assign_static_scratch: cudaGetSymbolAddress failed on device %d: %s", dev,
                    cudaGetErrorString(e));
      g_static_scratch_ptr[dev].store(ptr, std::memory_order_release);
    }
  }
  *out = ptr;
  return FK_OK;
}

}  // namespace fk

extern "C" int fk_assign_static_scratch(const void* x, const void* centroids, const void* x_sq,
                                        const void* c_sq, int32_t* out, int32_t* counts,
                                        int dtype, int xsq_dtype, int csq_dtype, int64_t B,
                                        int64_t N, int64_t K, int64_t D,
                                        const int64_t* x_strides3, const int64_t* c_strides3,
                                        const int64_t* xsq_strides2, const int64_t* csq_strides2,
                                        const int64_t* out_strides2, int32_t* dev_status,
                                        void* stream) {
  if (B < 0 || N < 0 || K <= 0 || D <= 0)
    return fail(FK_ERR_INVALID_ARG, "fk_assign_static_scratch: bad sizes B=%lld N=%lld K=%lld D=%lld",
                (long long)B, (long long)N, (long long)K, (long long)D);
  if (B == 0 || N == 0) return FK_OK;
  const size_t need = fk_assign_workspace_size(B, K, D, dtype);
  if (need > kAssignStaticScratchBytes)
    return fail(FK_ERR_WORKSPACE,
                "fk_assign_static_scratch: B=%lld, K=%lld, D=%lld needs %zu bytes of scratch; the "
                "static scratch holds %zu; use fk_assign with a workspace",
                (long long)B, (long long)K, (long long)D, need, kAssignStaticScratchBytes);
  void* scratch = nullptr;
  const int st = static_scratch_for_current_device(&scratch);
  if (st != FK_OK) return st;
  return fk_assign(x, centroids, x_sq, c_sq, out, counts, dtype, xsq_dtype, csq_dtype, B, N, K, D,
                   x_strides3, c_strides3, xsq_strides2, csq_strides2, out_strides2, scratch,
                   kAssignStaticScratchBytes, dev_status, stream);
}
