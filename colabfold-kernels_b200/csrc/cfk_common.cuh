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

// Device-side status word layout (one int32 per library, see cfk_status.cu): 0 = ok, else the id of the
// first wait that ran out of polls.
__device__ __forceinline__ void report_timeout(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// Every kernel launch of the library goes through check_launch(): it counts the launch (cfk_launch_count)
// and turns a refused launch into a status.
void note_launch();
inline int check_launch() {
  note_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CFK_OK : CFK_ERR_LAUNCH;
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
