// Outer-product-mean tail: out = (x + bias) / (eps + norm) + residual, one streaming pass.
// x [m, f] bf16 is the product of the two GEMMs (outer product over the MSA depth, then the output weights),
// norm [m] fp32 the number of sequences that cover both residues.  Math: src/colabfold_kernels/opm.py:69-88,116-119.
#include "cfk_common.cuh"
#include "cfk_ptx.cuh"

namespace cfk {
namespace {

__global__ void opm_finish_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ bias,
                                  const float* __restrict__ norm, const __nv_bfloat16* __restrict__ residual,
                                  __nv_bfloat16* __restrict__ out, int64_t m, int f, float eps) {
  const int64_t total = m * (f / 8);
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row = idx / (f / 8);
    const int c = int(idx % (f / 8)) * 8;
    const float inv = 1.0f / (eps + norm[row]);
    const uint4 xv = *reinterpret_cast<const uint4*>(x + row * f + c);
    const uint4 bv = *reinterpret_cast<const uint4*>(bias + c);
    uint4 rv = make_uint4(0, 0, 0, 0);
    if (residual != nullptr) rv = *reinterpret_cast<const uint4*>(residual + row * f + c);
    const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w}, bs[4] = {bv.x, bv.y, bv.z, bv.w}, rs[4] = {rv.x, rv.y, rv.z, rv.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = (bf16lo_to_f32(xs[e]) + bf16lo_to_f32(bs[e])) * inv + bf16lo_to_f32(rs[e]);
      const float hi = (bf16hi_to_f32(xs[e]) + bf16hi_to_f32(bs[e])) * inv + bf16hi_to_f32(rs[e]);
      o[e] = pack_bf16x2(lo, hi);
    }
    *reinterpret_cast<uint4*>(out + row * f + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace
}  // namespace cfk

extern "C" int cfk_opm_finish(const void* x, const void* bias, const float* norm, const void* residual, void* out,
                              int64_t m, int f, float eps, void* stream) {
  using namespace cfk;
  if (!x || !bias || !norm || !out) return CFK_ERR_NULL;
  if (m < 0 || f <= 0 || f % 8 != 0) return CFK_ERR_SHAPE;
  if (m == 0) return CFK_OK;
  const int64_t total = m * (f / 8);
  const int blocks = int(total / 256 + 1 < 148 * 16 ? total / 256 + 1 : 148 * 16);
  opm_finish_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(bias), norm,
      static_cast<const __nv_bfloat16*>(residual), static_cast<__nv_bfloat16*>(out), m, f, eps);
  return check_launch();
}
