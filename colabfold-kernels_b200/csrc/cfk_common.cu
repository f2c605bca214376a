// Tensor-map construction and the device status word shared by every kernel of the library.
#include "cfk_common.cuh"

#include <cudaTypedefs.h>
#include <atomic>
#include <mutex>

namespace cfk {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}
}  // namespace

int make_tensor_map(CUtensorMap* map, const void* base, int dtype, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  auto fn = encode_fn();
  if (fn == nullptr) return CFK_ERR_TMA;
  CUtensorMapDataType dt = dtype == CFK_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : dtype == CFK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  cuuint64_t gdim[5];
  cuuint64_t gstr[4];
  cuuint32_t bdim[5];
  cuuint32_t estr[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estr[i] = 1;
    if (i + 1 < rank) gstr[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdim, gstr, bdim, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CFK_OK : CFK_ERR_TMA;
}

namespace {
std::atomic<long long> g_launches{0};
constexpr int kMaxDevices = 64;
int* g_status[kMaxDevices] = {};
std::mutex g_status_mutex;
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// One int32 per device, allocated on first use on that device and kept for the life of the process.
int* device_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mutex);
  if (g_status[dev] == nullptr) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    g_status[dev] = p;
  }
  return g_status[dev];
}

}  // namespace cfk

extern "C" int cfk_last_device_status(int reset) {
  int* p = cfk::device_status_word();
  if (p == nullptr) return CFK_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return CFK_ERR_LAUNCH;
  if (reset && v != 0) cudaMemset(p, 0, sizeof(int));
  return v;
}

extern "C" long long cfk_launch_count(int reset) {
  return reset ? cfk::g_launches.exchange(0) : cfk::g_launches.load();
}

extern "C" const char* cfk_version() { return "cfk_b200 0.1 (sm_100a)"; }
