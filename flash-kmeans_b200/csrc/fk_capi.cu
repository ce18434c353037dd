// C-ABI plumbing: status strings, thread-local error text, device queries and
// TMA tensor-map encoding.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "fk_common.cuh"

namespace fk {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FK_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return FK_OK;
}

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

int sm_count_current() {
  // per-device cache; concurrent first calls store the same value
  static std::atomic<int> cache[64];
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return -1;
  int v = cache[dev].load(std::memory_order_acquire);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    cache[dev].store(v, std::memory_order_release);
  }
  return v;
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

int encode_tmap_3d(CUtensorMap* map, const void* base, int dtype, uint64_t d0, uint64_t d1,
                   uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                   uint32_t box1, bool sw64) {
  auto enc = get_encode();
  if (!enc) return fail(FK_ERR_TMA, "cuTensorMapEncodeTiled not available from the driver");
  CUtensorMapDataType dt = dtype == FK_F16    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                           : dtype == FK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r =
      enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          sw64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FK_ERR_TMA,
                "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu strides %llu %llu box %u x %u",
                (int)r, (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2,
                (unsigned long long)stride1_bytes, (unsigned long long)stride2_bytes, box0, box1);
  return FK_OK;
}

}  // namespace fk

using namespace fk;

extern "C" int fk_abi_version(void) { return FK_ABI_VERSION; }

extern "C" const char* fk_status_string(int status) {
  switch (status) {
    case FK_OK: return "ok";
    case FK_ERR_INVALID_ARG: return "invalid argument";
    case FK_ERR_UNSUPPORTED: return "unsupported layout or size";
    case FK_ERR_WORKSPACE: return "workspace too small or misaligned";
    case FK_ERR_CUDA: return "CUDA error";
    case FK_ERR_TMA: return "tensor map encoding failed";
    case FK_DEV_BAD_LABEL: return "cluster id outside [0, K)";
    case FK_DEV_WAIT_TIMEOUT: return "assignment pipeline wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* fk_last_error(void) { return g_last_error; }

extern "C" int fk_device_sm_count(void) { return sm_count_current(); }

extern "C" int fk_tma_compatible(const void* ptr, int dtype, int64_t D, const int64_t* s) {
  if (!ptr || !s || D <= 0) return 0;
  const int64_t eb = dtype_bytes(dtype);
  if (eb != 2 && eb != 4) return 0;
  if (reinterpret_cast<uintptr_t>(ptr) % 16) return 0;
  if (s[2] != 1) return 0;
  if ((s[1] * eb) % 16 || (s[0] * eb) % 16) return 0;
  if (s[1] < D || s[0] < 0) return 0;
  if (s[1] * eb >= (1ll << 40) || s[0] * eb >= (1ll << 40)) return 0;
  return 1;
}
