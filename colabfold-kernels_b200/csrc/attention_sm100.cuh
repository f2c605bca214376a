// Pieces shared by the tcgen05 attention forward and backward kernels.
#pragma once
#include <cfloat>

#include "attention_problem.cuh"
#include "cfk_common.cuh"
#include "cfk_ptx.cuh"

namespace cfk {

constexpr int kBQ = 128;  // query rows per tile = TMEM lanes = UMMA M
constexpr int kBK = 128;  // keys per tile

// Natural-log-domain mask floor.  A power of two, so that floor * log2(e) is exact and
// fma(floor, log2e, -(floor*log2e)) == 0: a row whose keys are all masked gets p == 1 for every key
// (the uniform mean the reference defines), and adding it to any sane logit rounds to the floor itself.
__device__ constexpr float kFloorNat = -8.507059173023462e37f;  // -2^126
__device__ constexpr float kLog2eF = 1.4426950408889634f;
__device__ constexpr float kNegRef = -0.7f * FLT_MAX;  // the reference's log2-domain floor, reported as lse of masked rows
// A running maximum is replaced (and the accumulator rescaled) only when it grows by more than this:
// probabilities then stay below 2^8, harmless in fp32/bf16, and most steps skip the TMEM round trip.
__device__ constexpr float kRescaleSlack = 5.545177444479562f;  // 8 ln 2

__device__ __forceinline__ uint64_t desc_k_major(uint32_t saddr, uint32_t row_bytes) {
  const uint32_t swz = row_bytes == 128 ? kSwz128 : row_bytes == 64 ? kSwz64 : kSwz32;
  return make_smem_desc(saddr, 16, 8 * row_bytes, swz);
}
// MN-major operand whose rows (one per K index) are row_bytes long; atom_stride is the byte distance
// between successive row_bytes-wide blocks along MN (unused when the operand is one block wide).
__device__ __forceinline__ uint64_t desc_mn_major(uint32_t saddr, uint32_t row_bytes, uint32_t atom_stride) {
  const uint32_t swz = row_bytes == 128 ? kSwz128 : row_bytes == 64 ? kSwz64 : kSwz32;
  return make_smem_desc(saddr, atom_stride, 8 * row_bytes, swz);
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Deadline-bounded mbarrier wait: polls until the phase flips or ~2^30 clocks (about half a second) have passed.
__device__ __forceinline__ bool mbar_wait_deadline(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > (1ll << 30)) return false;
  }
}

// Tensor maps for a [nb, s, h, d] tensor given by element strides, box = [d, rows] with swizzle = row bytes.
inline int make_qkv_map(CUtensorMap* m, const void* base, const Strides& st, int nb, int h, int s, int d,
                        int rows, int dtype = CFK_BF16) {
  const size_t es = dtype_size(dtype);
  uint64_t dims[4] = {uint64_t(d), uint64_t(s), uint64_t(h), uint64_t(nb)};
  uint64_t strides[3] = {uint64_t(st.s) * es, uint64_t(st.h) * es, uint64_t(st.b) * es};
  uint32_t box[4] = {uint32_t(d), uint32_t(rows), 1, 1};
  return make_tensor_map(m, base, dtype, 4, dims, strides, box, int(d * es));
}

}  // namespace cfk
