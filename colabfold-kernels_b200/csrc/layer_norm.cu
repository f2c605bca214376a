// LayerNorm forward and backward over the last axis: a pure HBM-streaming kernel.
// One warp owns a row; each lane holds C/32 values in registers (128-bit loads where the width
// allows), the two row statistics are warp-shuffle reductions in fp32, and several rows per warp
// are in flight so the loads of one row overlap the arithmetic of the previous.
// Math: src/colabfold_kernels/tri_mul.py:463-485,515-520; backward: grads.py:25-39.
#include <mutex>
#include "cfk_common.cuh"

namespace cfk {
namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kRowsInFlight = 4;

template <typename T>
struct Io;
template <>
struct Io<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};
template <>
struct Io<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

// V contiguous elements per lane and chunk; a row is C = 32 * V * CHUNKS wide: lane l owns elements
// [ (chunk*32 + l) * V , +V ) so that every chunk is one fully coalesced warp access.
template <typename T, int V>
__device__ __forceinline__ void load_vec(const T* p, float (&out)[V]) {
  if constexpr (sizeof(T) * V == 16) {
    uint4 raw = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) out[i] = Io<T>::load(e + i);
  } else if constexpr (sizeof(T) * V == 8) {
    uint2 raw = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) out[i] = Io<T>::load(e + i);
  } else if constexpr (sizeof(T) * V == 4) {
    uint32_t raw = *reinterpret_cast<const uint32_t*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) out[i] = Io<T>::load(e + i);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) out[i] = Io<T>::load(p + i);
  }
}
template <typename T, int V>
__device__ __forceinline__ void store_vec(T* p, const float (&in)[V]) {
  if constexpr (sizeof(T) * V == 16 || sizeof(T) * V == 8 || sizeof(T) * V == 4) {
    alignas(16) T e[V];
#pragma unroll
    for (int i = 0; i < V; ++i) Io<T>::store(e + i, in[i]);
    if constexpr (sizeof(T) * V == 16) *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(e);
    else if constexpr (sizeof(T) * V == 8) *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(e);
    else *reinterpret_cast<uint32_t*>(p) = *reinterpret_cast<const uint32_t*>(e);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) Io<T>::store(p + i, in[i]);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, int V, int CHUNKS>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
ln_fwd_kernel(const T* __restrict__ x, const float* __restrict__ scale, const float* __restrict__ offset,
              T* __restrict__ y, int64_t m, float eps) {
  constexpr int C = 32 * V * CHUNKS;
  const int lane = threadIdx.x & 31;
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  float sc[CHUNKS][V], of[CHUNKS][V];
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    load_vec<float, V>(scale + (c * 32 + lane) * V, sc[c]);
    load_vec<float, V>(offset + (c * 32 + lane) * V, of[c]);
  }
  for (int64_t row0 = warp * kRowsInFlight; row0 < m; row0 += nwarps * kRowsInFlight) {
    float v[kRowsInFlight][CHUNKS][V];
#pragma unroll
    for (int r = 0; r < kRowsInFlight; ++r) {
      const int64_t row = row0 + r;
      if (row < m) {
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) load_vec<T, V>(x + row * C + (c * 32 + lane) * V, v[r][c]);
      }
    }
#pragma unroll
    for (int r = 0; r < kRowsInFlight; ++r) {
      const int64_t row = row0 + r;
      if (row >= m) break;
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < CHUNKS; ++c)
#pragma unroll
        for (int i = 0; i < V; ++i) s += v[r][c][i];
      const float mean = warp_sum(s) * (1.0f / C);
      float q = 0.f;
#pragma unroll
      for (int c = 0; c < CHUNKS; ++c)
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const float d = v[r][c][i] - mean;
          v[r][c][i] = d;
          q += d * d;
        }
      const float rstd = rsqrtf(warp_sum(q) * (1.0f / C) + eps);
#pragma unroll
      for (int c = 0; c < CHUNKS; ++c) {
        float o[V];
#pragma unroll
        for (int i = 0; i < V; ++i) o[i] = v[r][c][i] * rstd * sc[c][i] + of[c][i];
        store_vec<T, V>(y + row * C + (c * 32 + lane) * V, o);
      }
    }
  }
}

// Any width: lanes stride over the row (used when c is not 32 * {1,2,4,8} * k).
template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
ln_fwd_generic_kernel(const T* __restrict__ x, const float* __restrict__ scale, const float* __restrict__ offset,
                      T* __restrict__ y, int64_t m, int c, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  for (int64_t row = warp; row < m; row += nwarps) {
    const T* xr = x + row * c;
    float s = 0.f;
    for (int i = lane; i < c; i += 32) s += Io<T>::load(xr + i);
    const float mean = warp_sum(s) / c;
    float q = 0.f;
    for (int i = lane; i < c; i += 32) {
      const float d = Io<T>::load(xr + i) - mean;
      q += d * d;
    }
    const float rstd = rsqrtf(warp_sum(q) / c + eps);
    for (int i = lane; i < c; i += 32)
      Io<T>::store(y + row * c + i, (Io<T>::load(xr + i) - mean) * rstd * scale[i] + offset[i]);
  }
}

// Backward.  dx is per row; dscale/doffset are column sums over all rows: each warp keeps its lanes'
// column partials in registers, blocks combine them in shared memory and write one partial row per block
// to the workspace, and a second tiny kernel folds the partial rows (deterministic, no atomics).
template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
ln_bwd_kernel(const T* __restrict__ x, const float* __restrict__ scale, const T* __restrict__ dy, T* __restrict__ dx,
              float* __restrict__ partial, int64_t m, int c, float eps) {
  extern __shared__ float sm[];  // [warps][2][c] per-warp partials
  const int lane = threadIdx.x & 31;
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  constexpr int kMaxPer = 16;  // c <= 512
  float ds_acc[kMaxPer], do_acc[kMaxPer];
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) ds_acc[j] = do_acc[j] = 0.f;
  for (int64_t row = warp; row < m; row += nwarps) {
    const T* xr = x + row * c;
    const T* gr = dy + row * c;
    float s = 0.f;
    for (int i = lane; i < c; i += 32) s += Io<T>::load(xr + i);
    const float mean = warp_sum(s) / c;
    float q = 0.f;
    for (int i = lane; i < c; i += 32) {
      const float d = Io<T>::load(xr + i) - mean;
      q += d * d;
    }
    const float rstd = rsqrtf(warp_sum(q) / c + eps);
    float a = 0.f, b = 0.f;
    int j = 0;
    for (int i = lane; i < c; i += 32, ++j) {
      const float xhat = (Io<T>::load(xr + i) - mean) * rstd;
      const float g = Io<T>::load(gr + i);
      const float dxhat = g * scale[i];
      a += dxhat;
      b += dxhat * xhat;
      if (j < kMaxPer) {
        ds_acc[j] += g * xhat;
        do_acc[j] += g;
      }
    }
    a = warp_sum(a) / c;
    b = warp_sum(b) / c;
    for (int i = lane; i < c; i += 32) {
      const float xhat = (Io<T>::load(xr + i) - mean) * rstd;
      const float dxhat = Io<T>::load(gr + i) * scale[i];
      Io<T>::store(dx + row * c + i, rstd * (dxhat - a - xhat * b));
    }
  }
  float* mine = sm + (threadIdx.x >> 5) * 2 * c;
  int j = 0;
  for (int i = lane; i < c; i += 32, ++j) {
    mine[i] = j < kMaxPer ? ds_acc[j] : 0.f;
    mine[c + i] = j < kMaxPer ? do_acc[j] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * c; i += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsPerBlock; ++w) s += sm[w * 2 * c + i];
    partial[static_cast<int64_t>(blockIdx.x) * 2 * c + i] = s;
  }
}

__global__ void ln_bwd_fold_kernel(const float* __restrict__ partial, float* __restrict__ dscale,
                                   float* __restrict__ doffset, int nblocks, int c) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * c) return;
  float s = 0.f;
  for (int b = 0; b < nblocks; ++b) s += partial[static_cast<int64_t>(b) * 2 * c + i];
  if (i < c) dscale[i] = s;
  else doffset[i - c] = s;
}

// SM count of the current device (asked for on every call: a process may drive several devices)
int sm_count() {
  int dev = 0, v = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  return v;
}

constexpr int kBwdBlocksPerSm = 2;

template <typename T>
int launch_fwd(const T* x, const float* scale, const float* offset, T* y, int64_t m, int c, float eps,
               cudaStream_t st) {
  const int64_t warps_needed = (m + kRowsInFlight - 1) / kRowsInFlight;
  int64_t blocks = (warps_needed + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  dim3 grid(static_cast<unsigned>(blocks)), block(kWarpsPerBlock * 32);
  constexpr int V = 16 / sizeof(T);  // 128-bit accesses
  const bool vec_ok = aligned16(x) && aligned16(y) && aligned16(scale) && aligned16(offset);
  if (vec_ok && c == 32 * V) ln_fwd_kernel<T, V, 1><<<grid, block, 0, st>>>(x, scale, offset, y, m, eps);
  else if (vec_ok && c == 64 * V) ln_fwd_kernel<T, V, 2><<<grid, block, 0, st>>>(x, scale, offset, y, m, eps);
  else if (vec_ok && c == 16 * V) ln_fwd_kernel<T, V / 2, 1><<<grid, block, 0, st>>>(x, scale, offset, y, m, eps);
  else if (vec_ok && c == 8 * V) ln_fwd_kernel<T, V / 4, 1><<<grid, block, 0, st>>>(x, scale, offset, y, m, eps);
  else {
    int64_t gb = (m + kWarpsPerBlock - 1) / kWarpsPerBlock;
    if (gb > cap) gb = cap;
    ln_fwd_generic_kernel<T><<<dim3(static_cast<unsigned>(gb)), block, 0, st>>>(x, scale, offset, y, m, c, eps);
  }
  return check_launch();
}

}  // namespace
}  // namespace cfk

extern "C" int cfk_layer_norm(const void* x, const float* scale, const float* offset, void* y, int64_t m, int c,
                              int dtype, float eps, void* stream) {
  using namespace cfk;
  if (x == nullptr || scale == nullptr || offset == nullptr || y == nullptr) return CFK_ERR_NULL;
  if (m < 0 || c <= 0) return CFK_ERR_SHAPE;
  if (m == 0) return CFK_OK;
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == CFK_BF16)
    return launch_fwd(static_cast<const __nv_bfloat16*>(x), scale, offset, static_cast<__nv_bfloat16*>(y), m, c, eps, st);
  if (dtype == CFK_F32) return launch_fwd(static_cast<const float*>(x), scale, offset, static_cast<float*>(y), m, c, eps, st);
  return CFK_ERR_DTYPE;
}

extern "C" size_t cfk_layer_norm_bwd_workspace_bytes(int64_t m, int c) {
  (void)m;
  return static_cast<size_t>(cfk::sm_count()) * cfk::kBwdBlocksPerSm * 2 * static_cast<size_t>(c) * sizeof(float);
}

extern "C" int cfk_layer_norm_bwd(const void* x, const float* scale, const void* dy, void* dx, float* dscale,
                                  float* doffset, int64_t m, int c, int dtype, float eps, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  using namespace cfk;
  if (x == nullptr || scale == nullptr || dy == nullptr || dx == nullptr || dscale == nullptr || doffset == nullptr ||
      workspace == nullptr)
    return CFK_ERR_NULL;
  if (m <= 0 || c <= 0 || c > 512) return CFK_ERR_SHAPE;
  if (workspace_bytes < cfk_layer_norm_bwd_workspace_bytes(m, c)) return CFK_ERR_WORKSPACE;
  auto st = static_cast<cudaStream_t>(stream);
  const int blocks = sm_count() * kBwdBlocksPerSm;
  float* partial = static_cast<float*>(workspace);
  const size_t smem = kWarpsPerBlock * 2 * static_cast<size_t>(c) * sizeof(float);
  if (dtype == CFK_BF16)
    ln_bwd_kernel<__nv_bfloat16><<<blocks, kWarpsPerBlock * 32, smem, st>>>(
        static_cast<const __nv_bfloat16*>(x), scale, static_cast<const __nv_bfloat16*>(dy),
        static_cast<__nv_bfloat16*>(dx), partial, m, c, eps);
  else if (dtype == CFK_F32)
    ln_bwd_kernel<float><<<blocks, kWarpsPerBlock * 32, smem, st>>>(static_cast<const float*>(x), scale,
                                                                    static_cast<const float*>(dy),
                                                                    static_cast<float*>(dx), partial, m, c, eps);
  else
    return CFK_ERR_DTYPE;
  int rc = check_launch();
  if (rc != CFK_OK) return rc;
  ln_bwd_fold_kernel<<<(2 * c + 127) / 128, 128, 0, st>>>(partial, dscale, doffset, blocks, c);
  return check_launch();
}

// ---- LayerNorm backward with built-in scratch -----------------------------------------------------------
// The same two kernels as cfk_layer_norm_bwd, with the per-block partial sums in a fixed array that is part of
// this module's device image instead of a caller workspace: the entry allocates nothing, on the device or through
// any library.
namespace cfk {
namespace {

constexpr int kStaticMaxC = 256;       // widest row the built-in scratch takes
constexpr int kStaticMaxBlocks = 512;  // most blocks it takes (the launch uses 2 per SM)
static __device__ __align__(256) float g_ln_bwd_partial[static_cast<size_t>(kStaticMaxBlocks) * 2 * kStaticMaxC];  // 1 MiB

constexpr int kStaticMaxDevices = 64;
float* g_ln_bwd_partial_addr[kStaticMaxDevices] = {};  // device address of the array, per device
std::mutex g_ln_bwd_partial_mutex;

// Set-up, once per device and with that device current: the array's name is not a device address in host code,
// the runtime has to be asked for it.  This also makes the runtime load this module's image on the device.
int static_partial(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kStaticMaxDevices) return CFK_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_ln_bwd_partial_mutex);
  if (g_ln_bwd_partial_addr[dev] == nullptr) {
    float* ptr = nullptr;
    if (cudaGetSymbolAddress((void**)&ptr, g_ln_bwd_partial) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      return CFK_ERR_LAUNCH;
    }
    g_ln_bwd_partial_addr[dev] = ptr;
  }
  *out = g_ln_bwd_partial_addr[dev];
  return CFK_OK;
}

}  // namespace
}  // namespace cfk

extern "C" int cfk_layer_norm_bwd_static(const void* x, const float* scale, const void* dy, void* dx, float* dscale,
                                         float* doffset, int64_t m, int c, int dtype, float eps, void* stream) {
  using namespace cfk;
  if (x == nullptr || scale == nullptr || dy == nullptr || dx == nullptr || dscale == nullptr || doffset == nullptr)
    return CFK_ERR_NULL;
  if (m <= 0 || c <= 0) return CFK_ERR_SHAPE;
  if (dtype != CFK_BF16 && dtype != CFK_F32) return CFK_ERR_DTYPE;
  const int blocks = sm_count() * kBwdBlocksPerSm;
  if (c > kStaticMaxC || blocks > kStaticMaxBlocks) return CFK_ERR_WORKSPACE;  // beyond the built-in scratch
  float* partial = nullptr;
  int rc = static_partial(&partial);
  if (rc != CFK_OK) return rc;
  // Nothing has to start at zero: every block overwrites its whole row of 2*c partial sums before the fold reads it.
  auto st = static_cast<cudaStream_t>(stream);
  const size_t smem = kWarpsPerBlock * 2 * static_cast<size_t>(c) * sizeof(float);
  if (dtype == CFK_BF16)
    ln_bwd_kernel<__nv_bfloat16><<<blocks, kWarpsPerBlock * 32, smem, st>>>(
        static_cast<const __nv_bfloat16*>(x), scale, static_cast<const __nv_bfloat16*>(dy),
        static_cast<__nv_bfloat16*>(dx), partial, m, c, eps);
  else
    ln_bwd_kernel<float><<<blocks, kWarpsPerBlock * 32, smem, st>>>(static_cast<const float*>(x), scale,
                                                                    static_cast<const float*>(dy),
                                                                    static_cast<float*>(dx), partial, m, c, eps);
  rc = check_launch();
  if (rc != CFK_OK) return rc;
  ln_bwd_fold_kernel<<<(2 * c + 127) / 128, 128, 0, st>>>(partial, dscale, doffset, blocks, c);
  return check_launch();
}
