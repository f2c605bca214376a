// Shared host-side helpers of the C-ABI library: status codes, dtype tags, launch checks and
// TMA tensor-map construction.  No torch types, no allocation.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/cfk_b200.h"

namespace cfk {

// Device-side status word (16 bytes of device memory per device): word 0 is 0 or the id of the first bounded wait that
// ran out; bytes 8..15 hold the device-visible address of a pinned host int that receives a copy of that id, so that
// the host entry points can see a pending timeout without synchronising.
__device__ __forceinline__ void report_timeout(int* status, int code) {
  if (status == nullptr) return;
  if (atomicCAS(status, 0, code) == 0) {
    int* mirror = *reinterpret_cast<int* const*>(status + 2);
    if (mirror != nullptr) {
      *reinterpret_cast<volatile int*>(mirror) = code;
      __threadfence_system();
    }
  }
}

// Every kernel launch of the library goes through check_launch(): it counts the launch (cfk_launch_count), turns a
// refused launch into CFK_ERR_LAUNCH, and answers CFK_ERR_DEVICE_WAIT while a timeout reported by an earlier kernel
// on this device has not been read and cleared with cfk_last_device_status(1): kernels launched in that state return
// at once and write nothing, so their outputs must not be taken for results.
int note_launch();
inline int check_launch() {
  const int pending = note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return CFK_ERR_LAUNCH;
  return pending;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline size_t dtype_size(int dtype) {
  return dtype == CFK_F32 ? 4 : dtype == CFK_BF16 ? 2 : dtype == CFK_E4M3 ? 1 : 0;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda dependency).
// dims/strides are innermost-first; strides[i] is the byte stride of dimension i+1.
// Returns CFK_OK or CFK_ERR_TMA.
int make_tensor_map(CUtensorMap* map, const void* base, int dtype, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);

// The per-device status word kernels report bounded-wait timeouts into.
int* device_status_word();

}  // namespace cfk
