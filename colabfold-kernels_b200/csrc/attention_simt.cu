// fp32-math attention forward and backward for every shape and dtype the tensor-core kernels do
// not take: float32 tensors (where tensor-core rounding would miss the 1e-4 bound), head dims that
// are not 16/32/64, key counts that are not a multiple of 8.  One warp owns one query row (or, in
// the dK/dV pass, one key row); K/V (or Q/dO) tiles of 32 rows are staged in shared memory.
// Math: src/colabfold_kernels/tri_flash.py:132-167,215-239 (forward), :313-355 (backward).
#include <cfloat>

#include "attention_problem.cuh"
#include "cfk_common.cuh"

namespace cfk {

namespace {

constexpr int kWarps = 8;
constexpr int kTile = 32;
constexpr int kMaxD = 128;
__device__ constexpr float kNeg = -0.7f * FLT_MAX;
__device__ constexpr float kLog2e = 1.4426950408889634f;

template <typename T>
__device__ __forceinline__ float ldf(const void* base, int64_t idx) {
  if constexpr (sizeof(T) == 4) return static_cast<const float*>(base)[idx];
  else return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
}
template <typename T>
__device__ __forceinline__ void stf(void* base, int64_t idx, float v) {
  if constexpr (sizeof(T) == 4) static_cast<float*>(base)[idx] = v;
  else static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Stage `rows` rows of a [.., s, .., d] tensor starting at sequence position s0 into shared memory as
// float [kTile][d + 1]; rows past `limit` read as zero.
template <typename T>
__device__ __forceinline__ void stage_tile(float* dst, const void* src, int64_t base, int64_t stride_s, int s0,
                                           int limit, int d) {
  for (int idx = threadIdx.x; idx < kTile * d; idx += blockDim.x) {
    const int r = idx / d, c = idx - r * d;
    const int s = s0 + r;
    dst[r * (d + 1) + c] = s < limit ? ldf<T>(src, base + s * stride_s + c) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) attn_fwd_simt_kernel(AttnProblem p) {
  extern __shared__ float sm[];
  const int d = p.d, dp1 = d + 1;
  float* ks = sm;
  float* vs = ks + kTile * dp1;
  float* qs = vs + kTile * dp1;  // [kWarps][d]
  const int b = blockIdx.z, h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qrow = blockIdx.x * kWarps + warp;
  const bool qvalid = qrow < p.sq;
  const int64_t qbase = b * p.sq_.b + h * p.sq_.h + int64_t(qrow) * p.sq_.s;
  for (int c = lane; c < d; c += 32) qs[warp * d + c] = qvalid ? ldf<T>(p.q, qbase + c) : 0.f;
  int sk_eff = p.sk;
  bool zero_row = false;
  if (p.trim != nullptr) {
    sk_eff = p.trim[b];
    zero_row = sk_eff == 0 || qrow >= p.trim[p.nb];
  }
  float m = -INFINITY, l = 0.f;
  float o[kMaxD / 32] = {0.f, 0.f, 0.f, 0.f};
  const int64_t kbase = b * p.sk_.b + h * p.sk_.h, vbase = b * p.sv_.b + h * p.sv_.h;
  for (int k0 = 0; k0 < sk_eff; k0 += kTile) {
    __syncthreads();
    stage_tile<T>(ks, p.k, kbase, p.sk_.s, k0, p.sk, d);
    stage_tile<T>(vs, p.v, vbase, p.sv_.s, k0, p.sk, d);
    __syncthreads();
    const int key = k0 + lane;
    float s = -INFINITY;
    if (key < p.sk) {
      float dot = 0.f;
      for (int c = 0; c < d; ++c) dot = fmaf(qs[warp * d + c], ks[lane * dp1 + c], dot);
      float bias = 0.f;
      if (p.bias != nullptr && qvalid) bias = ldf<T>(p.bias, (int64_t(h) * p.sq + qrow) * p.sk + key);
      s = (dot * p.scale + bias) * kLog2e;
      if (!p.kmask[int64_t(b) * p.sk + key]) s = kNeg;
    }
    const float m_new = fmaxf(m, wmax(s));
    const float corr = exp2f(m - m_new);
    const float pl = exp2f(s - m_new);
    l = l * corr + wsum(pl);
#pragma unroll
    for (int i = 0; i < kMaxD / 32; ++i) o[i] *= corr;
    for (int j = 0; j < kTile; ++j) {
      const float pj = __shfl_sync(0xffffffffu, pl, j);
#pragma unroll
      for (int i = 0; i < kMaxD / 32; ++i)
        if (lane + 32 * i < d) o[i] = fmaf(pj, vs[j * dp1 + lane + 32 * i], o[i]);
    }
    m = m_new;
  }
  if (!qvalid) return;
  const float inv = zero_row ? 0.f : 1.0f / l;
  const int64_t obase = b * p.so_.b + h * p.so_.h + int64_t(qrow) * p.so_.s;
  const int64_t gbase = b * p.sg_.b + h * p.sg_.h + int64_t(qrow) * p.sg_.s;
#pragma unroll
  for (int i = 0; i < kMaxD / 32; ++i) {
    const int c = lane + 32 * i;
    if (c < d) {
      float val = zero_row ? 0.f : o[i] * inv;
      if (p.gate != nullptr) {
        const float g = ldf<T>(p.gate, gbase + c) + ldf<T>(p.gate_bias, int64_t(h) * d + c);
        val *= 1.0f / (1.0f + expf(-g));
      }
      stf<T>(p.out, obase + c, val);
    }
  }
  if (p.lse != nullptr && lane == 0) p.lse[(int64_t(b) * p.h + h) * p.sq + qrow] = m + log2f(l);
}

// delta[b,h,q] = sum_d out * dout (tri_flash.py:380)
template <typename T>
__global__ void attn_delta_kernel(const void* out, Strides so, const void* dout, Strides sdo, float* delta, int nb,
                                  int h, int sq, int d) {
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = int64_t(nb) * h * sq;
  if (warp >= total) return;
  const int q = warp % sq, hh = (warp / sq) % h, b = warp / (int64_t(sq) * h);
  float s = 0.f;
  for (int c = lane; c < d; c += 32)
    s += ldf<T>(out, b * so.b + hh * so.h + int64_t(q) * so.s + c) * ldf<T>(dout, b * sdo.b + hh * sdo.h + int64_t(q) * sdo.s + c);
  s = wsum(s);
  if (lane == 0) delta[warp] = s;
}

// The same for bf16 tensors whose rows are 16-byte aligned and a power-of-two multiple of 8 wide: d/8 threads per row,
// one 16-byte load of out and of dout each, rows walked in memory order so that a warp reads contiguous bytes.
__global__ void attn_delta_bf16_vec_kernel(const __nv_bfloat16* __restrict__ out, Strides so,
                                           const __nv_bfloat16* __restrict__ dout, Strides sdo, float* __restrict__ delta,
                                           int nb, int h, int sq, int tpr, int heads_inner) {
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = int64_t(nb) * h * sq * tpr;
  const int64_t gc = gid < total ? gid : total - 1;  // clamped so that whole warps reach the shuffles
  const int chunk = int(gc % tpr);
  const int64_t rowid = gc / tpr;
  int q, hh, b;
  if (heads_inner) {  // [b, s, h, d]
    hh = int(rowid % h);
    q = int((rowid / h) % sq);
    b = int(rowid / (int64_t(h) * sq));
  } else {  // [b, h, s, d]
    q = int(rowid % sq);
    hh = int((rowid / sq) % h);
    b = int(rowid / (int64_t(h) * sq));
  }
  const uint4 a = *reinterpret_cast<const uint4*>(out + b * so.b + hh * so.h + int64_t(q) * so.s + chunk * 8);
  const uint4 g = *reinterpret_cast<const uint4*>(dout + b * sdo.b + hh * sdo.h + int64_t(q) * sdo.s + chunk * 8);
  const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w};
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    s = fmaf(__uint_as_float(aw[e] << 16), __uint_as_float(gw[e] << 16), s);
    s = fmaf(__uint_as_float(aw[e] & 0xffff0000u), __uint_as_float(gw[e] & 0xffff0000u), s);
  }
  for (int off = tpr >> 1; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (chunk == 0 && gid < total) delta[(int64_t(b) * h + hh) * sq + q] = s;
}

// The probability and score gradient of one (query, key) pair, the way the flash backward rebuilds them
// (tri_flash.py:336-343): masked logits are constants, a fully masked row was the uniform 1/Sk.
__device__ __forceinline__ void p_and_ds(float dot, float bias, float scale, bool live, bool inb, float lse, float dp,
                                         float delta, int sk, float& pr, float& ds) {
  const float s = live ? (dot * scale + bias) * kLog2e : kNeg;
  pr = !inb ? 0.f : (lse <= kNeg * 0.5f ? 1.0f / sk : exp2f(s - lse));
  ds = live ? pr * (dp - delta) : 0.f;
}

// dQ (and dBias through fp32 atomics): one warp per query row, sweeping key tiles.
template <typename T>
__global__ void __launch_bounds__(kWarps * 32) attn_bwd_dq_simt_kernel(AttnBwdProblem bp, const float* delta) {
  extern __shared__ float sm[];
  const AttnProblem& p = bp.f;
  const int d = p.d, dp1 = d + 1;
  float* ks = sm;
  float* vs = ks + kTile * dp1;
  float* qs = vs + kTile * dp1;   // [kWarps][d]
  float* dos = qs + kWarps * d;   // [kWarps][d]
  const int b = blockIdx.z, h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qrow = blockIdx.x * kWarps + warp;
  const bool qvalid = qrow < p.sq;
  const int64_t qbase = b * p.sq_.b + h * p.sq_.h + int64_t(qrow) * p.sq_.s;
  const int64_t dobase = b * bp.sdo.b + h * bp.sdo.h + int64_t(qrow) * bp.sdo.s;
  for (int c = lane; c < d; c += 32) {
    qs[warp * d + c] = qvalid ? ldf<T>(p.q, qbase + c) : 0.f;
    dos[warp * d + c] = qvalid ? ldf<T>(bp.dout, dobase + c) : 0.f;
  }
  const int64_t row = (int64_t(b) * p.h + h) * p.sq + qrow;
  const float lse = qvalid ? p.lse[row] : 0.f;
  const float dl = qvalid ? delta[row] : 0.f;
  float dq[kMaxD / 32] = {0.f, 0.f, 0.f, 0.f};
  const int64_t kbase = b * p.sk_.b + h * p.sk_.h, vbase = b * p.sv_.b + h * p.sv_.h;
  for (int k0 = 0; k0 < p.sk; k0 += kTile) {
    __syncthreads();
    stage_tile<T>(ks, p.k, kbase, p.sk_.s, k0, p.sk, d);
    stage_tile<T>(vs, p.v, vbase, p.sv_.s, k0, p.sk, d);
    __syncthreads();
    const int key = k0 + lane;
    const bool inb = key < p.sk && qvalid;
    const bool live = inb && p.kmask[int64_t(b) * p.sk + key];
    float dot = 0.f, dpv = 0.f;
    for (int c = 0; c < d; ++c) {
      dot = fmaf(qs[warp * d + c], ks[lane * dp1 + c], dot);
      dpv = fmaf(dos[warp * d + c], vs[lane * dp1 + c], dpv);
    }
    const float bias = (p.bias != nullptr && inb) ? ldf<T>(p.bias, (int64_t(h) * p.sq + qrow) * p.sk + key) : 0.f;
    float pr, ds;
    p_and_ds(dot, bias, p.scale, live, inb, lse, dpv, dl, p.sk, pr, ds);
    if (bp.dbias != nullptr && live) atomicAdd(&bp.dbias[(int64_t(h) * p.sq + qrow) * p.sk + key], ds);
    for (int j = 0; j < kTile; ++j) {
      const float dsj = __shfl_sync(0xffffffffu, ds, j);
#pragma unroll
      for (int i = 0; i < kMaxD / 32; ++i)
        if (lane + 32 * i < d) dq[i] = fmaf(dsj, ks[j * dp1 + lane + 32 * i], dq[i]);
    }
  }
  if (!qvalid) return;
  const int64_t dqbase = b * bp.sdq.b + h * bp.sdq.h + int64_t(qrow) * bp.sdq.s;
#pragma unroll
  for (int i = 0; i < kMaxD / 32; ++i)
    if (lane + 32 * i < d) stf<T>(bp.dq, dqbase + lane + 32 * i, dq[i] * p.scale);
}

// dK and dV: one warp per key row, sweeping query tiles; no atomics.
template <typename T>
__global__ void __launch_bounds__(kWarps * 32) attn_bwd_dkv_simt_kernel(AttnBwdProblem bp, const float* delta) {
  extern __shared__ float sm[];
  const AttnProblem& p = bp.f;
  const int d = p.d, dp1 = d + 1;
  float* qs = sm;                  // [kTile][d+1]
  float* dos = qs + kTile * dp1;   // [kTile][d+1]
  float* kr = dos + kTile * dp1;   // [kWarps][d]
  float* vr = kr + kWarps * d;     // [kWarps][d]
  float* ls = vr + kWarps * d;     // [kTile] lse
  float* dls = ls + kTile;         // [kTile] delta
  const int b = blockIdx.z, h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int key = blockIdx.x * kWarps + warp;
  const bool kvalid = key < p.sk;
  const int64_t kbase = b * p.sk_.b + h * p.sk_.h + int64_t(key) * p.sk_.s;
  const int64_t vbase = b * p.sv_.b + h * p.sv_.h + int64_t(key) * p.sv_.s;
  for (int c = lane; c < d; c += 32) {
    kr[warp * d + c] = kvalid ? ldf<T>(p.k, kbase + c) : 0.f;
    vr[warp * d + c] = kvalid ? ldf<T>(p.v, vbase + c) : 0.f;
  }
  const bool klive = kvalid && p.kmask[int64_t(b) * p.sk + key];
  float dk[kMaxD / 32] = {0.f, 0.f, 0.f, 0.f}, dv[kMaxD / 32] = {0.f, 0.f, 0.f, 0.f};
  const int64_t qbase = b * p.sq_.b + h * p.sq_.h, dobase = b * bp.sdo.b + h * bp.sdo.h;
  const int64_t rowbase = (int64_t(b) * p.h + h) * p.sq;
  for (int q0 = 0; q0 < p.sq; q0 += kTile) {
    __syncthreads();
    stage_tile<T>(qs, p.q, qbase, p.sq_.s, q0, p.sq, d);
    stage_tile<T>(dos, bp.dout, dobase, bp.sdo.s, q0, p.sq, d);
    if (threadIdx.x < kTile) {
      const int q = q0 + threadIdx.x;
      ls[threadIdx.x] = q < p.sq ? p.lse[rowbase + q] : 0.f;
      dls[threadIdx.x] = q < p.sq ? delta[rowbase + q] : 0.f;
    }
    __syncthreads();
    const int q = q0 + lane;
    const bool inb = kvalid && q < p.sq;
    const bool live = inb && klive;
    float dot = 0.f, dpv = 0.f;
    for (int c = 0; c < d; ++c) {
      dot = fmaf(qs[lane * dp1 + c], kr[warp * d + c], dot);
      dpv = fmaf(dos[lane * dp1 + c], vr[warp * d + c], dpv);
    }
    const float bias = (p.bias != nullptr && inb) ? ldf<T>(p.bias, (int64_t(h) * p.sq + q) * p.sk + key) : 0.f;
    float pr, ds;
    p_and_ds(dot, bias, p.scale, live, inb, ls[lane], dpv, dls[lane], p.sk, pr, ds);
    for (int j = 0; j < kTile; ++j) {
      const float pj = __shfl_sync(0xffffffffu, pr, j);
      const float dsj = __shfl_sync(0xffffffffu, ds, j);
#pragma unroll
      for (int i = 0; i < kMaxD / 32; ++i)
        if (lane + 32 * i < d) {
          dv[i] = fmaf(pj, dos[j * dp1 + lane + 32 * i], dv[i]);
          dk[i] = fmaf(dsj, qs[j * dp1 + lane + 32 * i], dk[i]);
        }
    }
  }
  if (!kvalid) return;
  const int64_t dkbase = b * bp.sdk.b + h * bp.sdk.h + int64_t(key) * bp.sdk.s;
  const int64_t dvbase = b * bp.sdv.b + h * bp.sdv.h + int64_t(key) * bp.sdv.s;
#pragma unroll
  for (int i = 0; i < kMaxD / 32; ++i)
    if (lane + 32 * i < d) {
      stf<T>(bp.dk, dkbase + lane + 32 * i, dk[i] * p.scale);
      stf<T>(bp.dv, dvbase + lane + 32 * i, dv[i]);
    }
}

template <typename T>
int fwd_impl(const AttnProblem& p, cudaStream_t st) {
  const size_t smem = (2 * kTile * (p.d + 1) + kWarps * p.d) * sizeof(float);
  dim3 grid((p.sq + kWarps - 1) / kWarps, p.h, p.nb);
  attn_fwd_simt_kernel<T><<<grid, kWarps * 32, smem, st>>>(p);
  return check_launch();
}

template <typename T>
int bwd_impl(const AttnBwdProblem& bp, float* delta, cudaStream_t st) {
  const AttnProblem& p = bp.f;
  const int64_t rows = int64_t(p.nb) * p.h * p.sq;
  attn_delta_kernel<T><<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, st>>>(p.out, p.so_, bp.dout, bp.sdo,
                                                                                      delta, p.nb, p.h, p.sq, p.d);
  int rc = check_launch();
  if (rc != CFK_OK) return rc;
  if (bp.dbias != nullptr) cudaMemsetAsync(bp.dbias, 0, sizeof(float) * size_t(p.h) * p.sq * p.sk, st);
  const size_t smem_q = (2 * kTile * (p.d + 1) + 2 * kWarps * p.d) * sizeof(float);
  attn_bwd_dq_simt_kernel<T><<<dim3((p.sq + kWarps - 1) / kWarps, p.h, p.nb), kWarps * 32, smem_q, st>>>(bp, delta);
  rc = check_launch();
  if (rc != CFK_OK) return rc;
  const size_t smem_k = (2 * kTile * (p.d + 1) + 2 * kWarps * p.d + 2 * kTile) * sizeof(float);
  attn_bwd_dkv_simt_kernel<T><<<dim3((p.sk + kWarps - 1) / kWarps, p.h, p.nb), kWarps * 32, smem_k, st>>>(bp, delta);
  return check_launch();
}

}  // namespace

// delta[b,h,q] = sum_d out * dout for bf16 tensors (shared with the tcgen05 backward); the caller checks the launch
void launch_attn_delta_bf16(const AttnBwdProblem& bp, float* delta, cudaStream_t st) {
  const AttnProblem& p = bp.f;
  const int64_t rows = int64_t(p.nb) * p.h * p.sq;
  const int tpr = p.d / 8;
  auto vec_ok = [](const void* ptr, const Strides& s) {
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && s.b % 8 == 0 && s.h % 8 == 0 && s.s % 8 == 0;
  };
  if (p.d % 8 == 0 && tpr <= 32 && (tpr & (tpr - 1)) == 0 && vec_ok(p.out, p.so_) && vec_ok(bp.dout, bp.sdo)) {
    const int64_t threads = rows * tpr;
    attn_delta_bf16_vec_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(p.out), p.so_, static_cast<const __nv_bfloat16*>(bp.dout), bp.sdo, delta, p.nb, p.h,
        p.sq, tpr, p.so_.h < p.so_.s);
    return;
  }
  attn_delta_kernel<__nv_bfloat16><<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, st>>>(
      p.out, p.so_, bp.dout, bp.sdo, delta, p.nb, p.h, p.sq, p.d);
}

int attention_fwd_simt(const AttnProblem& p, int dtype, cudaStream_t st) {
  if (p.d > kMaxD) return CFK_ERR_UNSUPPORTED;
  if (dtype == CFK_F32) return fwd_impl<float>(p, st);
  if (dtype == CFK_BF16) return fwd_impl<__nv_bfloat16>(p, st);
  return CFK_ERR_DTYPE;
}

// delta: nb*h*sq floats of scratch.
int attention_bwd_simt(const AttnBwdProblem& bp, int dtype, float* delta, cudaStream_t st) {
  if (bp.f.d > kMaxD) return CFK_ERR_UNSUPPORTED;
  if (dtype == CFK_F32) return bwd_impl<float>(bp, delta, st);
  if (dtype == CFK_BF16) return bwd_impl<__nv_bfloat16>(bp, delta, st);
  return CFK_ERR_DTYPE;
}

}  // namespace cfk
