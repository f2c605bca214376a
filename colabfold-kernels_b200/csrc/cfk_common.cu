// Tensor-map construction and the device status word shared by every kernel of the library.
#include "cfk_common.cuh"
#include "cfk_ptx.cuh"

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
volatile int* g_mirror[kMaxDevices] = {};  // pinned host copies of the status words
std::mutex g_status_mutex;
}  // namespace

int note_launch() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CFK_OK;
  volatile int* m = g_mirror[dev];
  return (m != nullptr && *m != 0) ? CFK_ERR_DEVICE_WAIT : CFK_OK;
}

// 16 bytes per device (layout in cfk_common.cuh), allocated with their pinned host mirror on first use on that device
// and kept for the life of the process.
int* device_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mutex);
  if (g_status[dev] == nullptr) {
    int* p = nullptr;
    int* host = nullptr;
    int* host_dev = nullptr;
    if (cudaMalloc(&p, 16) != cudaSuccess) return nullptr;
    if (cudaHostAlloc(&host, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess) {
      *host = 0;
      if (cudaHostGetDevicePointer(&host_dev, host, 0) != cudaSuccess) host_dev = nullptr;
    }
    unsigned long long words[2] = {0ull, reinterpret_cast<unsigned long long>(host_dev)};
    if (cudaMemcpy(p, words, 16, cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaFree(p);
      return nullptr;
    }
    g_mirror[dev] = host_dev != nullptr ? host : nullptr;
    g_status[dev] = p;
  }
  return g_status[dev];
}

namespace {
// One CTA waits, with a limit of the given number of clocks, on an mbarrier that nothing arrives on, reports the
// timeout and returns.
__global__ void wait_selftest_kernel(int* status, long long limit_clocks, int code) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    const long long t0 = clock64();
    bool flipped = false;
    while (!flipped && clock64() - t0 < limit_clocks) flipped = mbar_try_wait(&bar, 0);
    if (!flipped) report_timeout(status, code);
  }
}
}  // namespace

}  // namespace cfk

extern "C" int cfk_last_device_status(int reset) {
  int* p = cfk::device_status_word();
  if (p == nullptr) return CFK_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return CFK_ERR_LAUNCH;
  if (reset && v != 0) {
    cudaMemset(p, 0, sizeof(int));
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < cfk::kMaxDevices && cfk::g_mirror[dev] != nullptr)
      *cfk::g_mirror[dev] = 0;
  }
  return v;
}

extern "C" int cfk_debug_wait_timeout(int64_t limit_clocks, int code, void* stream) {
  if (limit_clocks <= 0 || limit_clocks > (1ll << 24) || code <= 0) return CFK_ERR_SHAPE;
  int* status = cfk::device_status_word();
  if (status == nullptr) return CFK_ERR_LAUNCH;
  cfk::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, limit_clocks, code);
  return cfk::check_launch();
}

extern "C" long long cfk_launch_count(int reset) {
  return reset ? cfk::g_launches.exchange(0) : cfk::g_launches.load();
}

extern "C" const char* cfk_version() { return "cfk_b200 0.2 (sm_100a)"; }
