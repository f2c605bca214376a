// C-ABI entry points of the attention family: argument checks, layout -> stride translation, and
// the choice between the tcgen05 kernels (bf16, head dim 16/32/64, keys a multiple of 8) and the
// fp32-math kernels (everything else).
#include "attention_problem.cuh"
#include "cfk_common.cuh"

namespace cfk {
int attention_fwd_simt(const AttnProblem& p, int dtype, cudaStream_t st);
int attention_bwd_simt(const AttnBwdProblem& bp, int dtype, float* delta, cudaStream_t st);
bool attention_sm100_supported(const AttnProblem& p, int dtype);
int attention_fwd_sm100(const AttnProblem& p, cudaStream_t st);
bool attention_bwd_sm100_supported(const AttnBwdProblem& bp, int dtype);
size_t attention_bwd_sm100_workspace(const AttnProblem& p);
int attention_bwd_sm100(const AttnBwdProblem& bp, float* delta, void* workspace, cudaStream_t st);

namespace {
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace
}  // namespace cfk

using namespace cfk;

extern "C" int cfk_attention_fwd(const void* q, const void* k, const void* v, const void* bias, const uint8_t* kmask,
                                 void* out, float* lse, int n, int h, int sq, int sk, int d, int dtype, int seq_major,
                                 float scale, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || kmask == nullptr || out == nullptr) return CFK_ERR_NULL;
  if (n < 0 || h <= 0 || sq <= 0 || sk <= 0 || d <= 0) return CFK_ERR_SHAPE;
  if (dtype != CFK_F32 && dtype != CFK_BF16) return CFK_ERR_DTYPE;
  if (n == 0) return CFK_OK;
  AttnProblem p{};
  p.q = q; p.k = k; p.v = v; p.bias = bias; p.kmask = kmask; p.out = out; p.lse = lse;
  p.sq_ = p.so_ = seq_major ? strides_seq_major(h, sq, d) : strides_heads_major(h, sq, d);
  p.sk_ = p.sv_ = seq_major ? strides_seq_major(h, sk, d) : strides_heads_major(h, sk, d);
  p.nb = n; p.h = h; p.sq = sq; p.sk = sk; p.d = d; p.scale = scale;
  auto st = static_cast<cudaStream_t>(stream);
  if (attention_sm100_supported(p, dtype)) return attention_fwd_sm100(p, st);
  return attention_fwd_simt(p, dtype, st);
}

extern "C" int cfk_packed_attention_fwd(const void* pk, const void* bias, const uint8_t* kmask, const void* gate_bias,
                                        void* out, float* lse, const int32_t* trim_limits, int x, int y, int g, int h,
                                        int d, int dtype, int column, float scale, void* stream) {
  if (pk == nullptr || kmask == nullptr || out == nullptr) return CFK_ERR_NULL;
  if (x <= 0 || y <= 0 || h <= 0 || d <= 0 || (g != 3 && g != 4)) return CFK_ERR_SHAPE;
  if ((g == 4) != (gate_bias != nullptr)) return CFK_ERR_NULL;
  if (dtype != CFK_F32 && dtype != CFK_BF16) return CFK_ERR_DTYPE;
  const size_t es = dtype_size(dtype);
  const int64_t slot = int64_t(h) * d, pos = int64_t(g) * slot;
  AttnProblem p{};
  const char* base = static_cast<const char*>(pk);
  p.q = base; p.k = base + slot * es; p.v = base + 2 * slot * es;
  p.gate = g == 4 ? base + 3 * slot * es : nullptr;
  p.gate_bias = gate_bias; p.bias = bias; p.kmask = kmask; p.out = out; p.lse = lse; p.trim = trim_limits;
  // rows: batch X (stride Y*pos), sequence Y (stride pos); columns: batch Y (stride pos), sequence X (stride Y*pos)
  const Strides in = column ? Strides{pos, int64_t(y) * pos, d} : Strides{int64_t(y) * pos, pos, d};
  const Strides outs = column ? Strides{slot, int64_t(y) * slot, d} : Strides{int64_t(y) * slot, slot, d};
  p.sq_ = p.sk_ = p.sv_ = p.sg_ = in;
  p.so_ = outs;
  p.nb = column ? y : x; p.h = h; p.sq = p.sk = column ? x : y; p.d = d; p.scale = scale;
  auto st = static_cast<cudaStream_t>(stream);
  if (attention_sm100_supported(p, dtype)) return attention_fwd_sm100(p, st);
  return attention_fwd_simt(p, dtype, st);
}

extern "C" int cfk_packed_attention_fwd_qk8(const void* pk, const void* qk8, const void* bias, const uint8_t* kmask,
                                            const void* gate_bias, void* out, float* lse, const int32_t* trim_limits,
                                            int x, int y, int g, int h, int d, int column, float scale, void* stream) {
  if (pk == nullptr || qk8 == nullptr || kmask == nullptr || out == nullptr) return CFK_ERR_NULL;
  if (x <= 0 || y <= 0 || h <= 0 || d <= 0 || (g != 1 && g != 2)) return CFK_ERR_SHAPE;
  if ((g == 2) != (gate_bias != nullptr)) return CFK_ERR_NULL;
  const int64_t slot = int64_t(h) * d, pos = int64_t(g) * slot, pos8 = 2 * slot;
  AttnProblem p{};
  const char* base = static_cast<const char*>(pk);
  const char* base8 = static_cast<const char*>(qk8);
  p.q = base8; p.k = base8 + slot;          // one byte per element
  p.v = base; p.gate = g == 2 ? base + slot * 2 : nullptr;
  p.gate_bias = gate_bias; p.bias = bias; p.kmask = kmask; p.out = out; p.lse = lse; p.trim = trim_limits;
  const Strides in = column ? Strides{pos, int64_t(y) * pos, d} : Strides{int64_t(y) * pos, pos, d};
  const Strides in8 = column ? Strides{pos8, int64_t(y) * pos8, d} : Strides{int64_t(y) * pos8, pos8, d};
  const Strides outs = column ? Strides{slot, int64_t(y) * slot, d} : Strides{int64_t(y) * slot, slot, d};
  p.sq_ = p.sk_ = in8;
  p.sv_ = p.sg_ = in;
  p.so_ = outs;
  p.nb = column ? y : x; p.h = h; p.sq = p.sk = column ? x : y; p.d = d; p.scale = scale;
  p.qk_e4m3 = 1;
  // no second path: the e4m3 scores exist only on the tensor-core kernel
  if (!attention_sm100_supported(p, CFK_BF16)) return CFK_ERR_UNSUPPORTED;
  return attention_fwd_sm100(p, static_cast<cudaStream_t>(stream));
}

namespace cfk {
namespace {
// one warp per batch row: the last live key, then (block 0 after a grid-wide atomicMax) the global limit
__global__ void trim_limits_kernel(const uint8_t* kmask, int32_t* limits, int batch, int s) {
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b >= batch) return;
  int last = 0;
  for (int i = lane; i < s; i += 32)
    if (kmask[int64_t(b) * s + i]) last = i + 1;
  for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  if (lane == 0) {
    limits[b] = last;
    atomicMax(&limits[batch], last);
  }
}
}  // namespace
}  // namespace cfk

extern "C" int cfk_trim_limits(const uint8_t* kmask, int32_t* limits, int batch, int s, void* stream) {
  if (kmask == nullptr || limits == nullptr) return CFK_ERR_NULL;
  if (batch <= 0 || s <= 0) return CFK_ERR_SHAPE;
  auto st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(limits + batch, 0, sizeof(int32_t), st) != cudaSuccess) return CFK_ERR_LAUNCH;
  trim_limits_kernel<<<(batch + 7) / 8, 256, 0, st>>>(kmask, limits, batch, s);
  return check_launch();
}

extern "C" size_t cfk_attention_bwd_workspace_bytes(int n, int h, int sq, int sk, int d, int dtype) {
  AttnProblem p{};
  p.nb = n; p.h = h; p.sq = sq; p.sk = sk; p.d = d;
  size_t delta = align_up(sizeof(float) * size_t(n) * h * sq, 256);
  (void)dtype;
  return delta + attention_bwd_sm100_workspace(p);
}

extern "C" int cfk_attention_bwd(const void* q, const void* k, const void* v, const void* bias, const uint8_t* kmask,
                                 const void* out, const void* dout, const float* lse, void* dq, void* dk, void* dv,
                                 float* dbias, int n, int h, int sq, int sk, int d, int dtype, int seq_major,
                                 float scale, void* workspace, size_t workspace_bytes, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || kmask == nullptr || out == nullptr || dout == nullptr ||
      lse == nullptr || dq == nullptr || dk == nullptr || dv == nullptr || workspace == nullptr)
    return CFK_ERR_NULL;
  if (n <= 0 || h <= 0 || sq <= 0 || sk <= 0 || d <= 0) return CFK_ERR_SHAPE;
  if (dtype != CFK_F32 && dtype != CFK_BF16) return CFK_ERR_DTYPE;
  if (workspace_bytes < cfk_attention_bwd_workspace_bytes(n, h, sq, sk, d, dtype)) return CFK_ERR_WORKSPACE;
  AttnBwdProblem bp{};
  AttnProblem& p = bp.f;
  p.q = q; p.k = k; p.v = v; p.bias = bias; p.kmask = kmask; p.out = const_cast<void*>(out);
  p.lse = const_cast<float*>(lse);
  p.sq_ = p.so_ = seq_major ? strides_seq_major(h, sq, d) : strides_heads_major(h, sq, d);
  p.sk_ = p.sv_ = seq_major ? strides_seq_major(h, sk, d) : strides_heads_major(h, sk, d);
  p.nb = n; p.h = h; p.sq = sq; p.sk = sk; p.d = d; p.scale = scale;
  bp.dout = dout; bp.dq = dq; bp.dk = dk; bp.dv = dv; bp.dbias = dbias;
  bp.sdo = bp.sdq = p.sq_;
  bp.sdk = bp.sdv = p.sk_;
  auto st = static_cast<cudaStream_t>(stream);
  float* delta = static_cast<float*>(workspace);
  if (attention_bwd_sm100_supported(bp, dtype)) {
    char* rest = static_cast<char*>(workspace) + align_up(sizeof(float) * size_t(n) * h * sq, 256);
    return attention_bwd_sm100(bp, delta, rest, st);
  }
  return attention_bwd_simt(bp, dtype, delta, st);
}
