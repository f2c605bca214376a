// Row-block GEMM engine (see rowgemm_sm100.cuh).  Math of the callers:
//   LayerNorm rows:            src/colabfold_kernels/transition.py:20-26
//   gated dual projection:     tri_mul.py:25-46,70-107
//   tri-mul epilogue:          tri_mul.py:325-340
//   LN -> packed projection:   packed_attn.py:190-231; output projection: packed_attn.py:321-344
//   OPM projection:            opm.py:21-30
#include "rowgemm_sm100.cuh"

#include <cuda_fp8.h>

namespace cfk {
namespace {

constexpr int kRows = 128;
constexpr int kThreadsRg = 384;
constexpr int kAtom = kRows * 128;  // one 64-column K-major atom of an A tile: 16 KB

struct Layout {  // byte offsets inside the (1024-aligned) dynamic shared memory, computed on the host
  int w[2];       // weights of accumulator i: [chunk][atom][K rows][128 B]
  int w_chunk[2]; // bytes per chunk
  int a[2];       // A tile of source i: [stage][K/64 atoms][16 KB]
  int a_stage[2]; // bytes per stage
  int ln[2];      // float [2][K]: LayerNorm scale, offset of source i
  int stage_out;  // channel-major output staging: [n_chunk][128 * itemsize]
  int bars;
  int tmem;
  int total;
};

struct KernelArgs {
  RowGemmParams p;
  Layout l;
  int64_t ntiles, tiles_per_outer;
};

__device__ __forceinline__ float act_sigmoid(float x) { return sigmoid_fast(x); }

__global__ void __launch_bounds__(kThreadsRg, 1)
rowgemm_kernel(const __grid_constant__ CUtensorMap tw0, const __grid_constant__ CUtensorMap tw1, const KernelArgs ka) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const RowGemmParams& p = ka.p;
  const Layout& L = ka.l;
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(p.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* w_full = bars;            // weights resident
  uint64_t* a_full = bars + 1;        // [2]
  uint64_t* a_empty = bars + 3;       // [2]
  uint64_t* acc_full = bars + 5;      // [2]
  uint64_t* acc_empty = bars + 7;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsrc = p.src[1].x != nullptr ? 2 : 1;
  const int nacc = p.dual ? 2 : 1;

  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_full[i], 4);
      mbar_init(&a_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tw0);
    if (p.dual) tma_prefetch_desc(&tw1);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // LayerNorm parameters of each source into shared memory (floats)
  for (int i = 0; i < nsrc; ++i) {
    if (p.src[i].ln_scale == nullptr) continue;
    float* dst = reinterpret_cast<float*>(smem + L.ln[i]);
    for (int k = threadIdx.x; k < p.src[i].k; k += blockDim.x) {
      dst[k] = p.src[i].ln_scale[k];
      dst[p.src[i].k + k] = p.src[i].ln_offset[k];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ weight loader (once)
    if (lane == 0) {
      const int atoms = p.n_chunk / 64;
      uint32_t bytes = 0;
      for (int i = 0; i < nacc; ++i) bytes += uint32_t(p.chunks) * L.w_chunk[i];
      mbar_arrive_expect_tx(w_full, bytes);
      for (int i = 0; i < nacc; ++i) {
        const int kw = p.src[(i == 1 && nsrc == 2) ? 1 : 0].k;
        for (int c = 0; c < p.chunks; ++c) {
          const int cg = p.chunk0 + c;
          const int slot = cg / p.chunks_per_slot;
          const int col = (cg % p.chunks_per_slot) * p.n_chunk;
          for (int a = 0; a < atoms; ++a)
            tma_load_3d(smem + L.w[i] + c * L.w_chunk[i] + a * kw * 128, i == 0 ? &tw0 : &tw1, w_full, col + a * 64, 0, slot);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(kRows, uint32_t(p.n_chunk), 1, 1, 0, 1);
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      bool ok = mbar_wait_deadline(w_full, 0);
      if (!ok) report_timeout(p.status, 901);
      uint32_t it = 0, cc = 0;
      for (int64_t tile = blockIdx.x; tile < ka.ntiles && ok; tile += gridDim.x, ++it) {
        const int stage = it & 1;
        ok = mbar_wait_deadline(&a_full[stage], (it >> 1) & 1);
        if (!ok) { report_timeout(p.status, 902); break; }
        for (int c = 0; c < p.chunks && ok; ++c, ++cc) {
          const int buf = cc & 1;
          ok = mbar_wait_deadline(&acc_empty[buf], ((cc >> 1) & 1) ^ 1);
          if (!ok) { report_timeout(p.status, 903); break; }
          tc_fence_after();
          for (int i = 0; i < nacc; ++i) {
            const int s = (i == 1 && nsrc == 2) ? 1 : 0;
            const int kw = p.src[s].k;
            const uint32_t a_lo = desc_lo(smem_u32(smem + L.a[s] + stage * L.a_stage[s]), 16);
            const uint32_t w_lo = desc_lo(smem_u32(smem + L.w[i] + c * L.w_chunk[i]), uint32_t(kw) * 128);
            const uint32_t d = tmem + buf * 256 + i * 128;
            // one 64-column atom of A per outer iteration, four K = 16 steps inside it
            uint32_t al = a_lo, wl = w_lo;
#pragma unroll 1
            for (int at = 0; at < kw / 64; ++at, al += kAtom >> 4, wl += 512) {
#pragma unroll
              for (int q = 0; q < 4; ++q) mma_f16_ss2(d, al + q * 2, hi, wl + q * 128, hi, idesc, (at | q) != 0);
            }
          }
          mma_commit(&acc_full[buf]);
        }
        if (ok) mma_commit(&a_empty[stage]);
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------------ prologue: build the A tiles
    const int trow = (warp - 4) * 32 + lane;
    bool ok = true;
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < ka.ntiles; tile += gridDim.x, ++it) {
      const int stage = it & 1;
      if (ok && !mbar_wait_deadline(&a_empty[stage], ((it >> 1) & 1) ^ 1)) {
        report_timeout(p.status, 904);
        ok = false;
      }
      const int64_t o = tile / ka.tiles_per_outer;
      const int64_t r = (tile % ka.tiles_per_outer) * kRows + trow;
      const bool valid = r < p.inner;
      for (int s = 0; s < nsrc; ++s) {
        const RowSource& src = p.src[s];
        uint8_t* dst = smem + L.a[s] + stage * L.a_stage[s];
        const float* lnp = reinterpret_cast<const float*>(smem + L.ln[s]);
        const int K = src.k;
        if (!src.channel_major) {
          // row-major bf16 row, processed in 64-column pieces held as packed pairs
          const __nv_bfloat16* xr = static_cast<const __nv_bfloat16*>(src.x) + (o * src.stride_outer + r * src.stride_inner) * K;
          float mean = 0.f, rstd = 1.f;
          if (src.ln_scale != nullptr) {
            float sum = 0.f, sq = 0.f;
            if (valid) {
              for (int c = 0; c < K / 8; ++c) {
                const uint4 w = *reinterpret_cast<const uint4*>(xr + c * 8);
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float a = bf16lo_to_f32(ww[e]), b = bf16hi_to_f32(ww[e]);
                  sum += a + b;
                  sq = fmaf(a, a, fmaf(b, b, sq));
                }
              }
            }
            mean = sum / K;
            // two-pass form on the second read keeps the variance accurate
            float var = 0.f;
            if (valid) {
              for (int c = 0; c < K / 8; ++c) {
                const uint4 w = *reinterpret_cast<const uint4*>(xr + c * 8);
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float a = bf16lo_to_f32(ww[e]) - mean, b = bf16hi_to_f32(ww[e]) - mean;
                  var = fmaf(a, a, fmaf(b, b, var));
                }
              }
            }
            (void)sq;
            rstd = rsqrtf(var / K + p.eps);
          }
          for (int c = 0; c < K / 8; ++c) {
            uint4 w = make_uint4(0, 0, 0, 0);
            if (valid) {
              w = *reinterpret_cast<const uint4*>(xr + c * 8);
              if (src.ln_scale != nullptr) {
                uint32_t ww[4] = {w.x, w.y, w.z, w.w};
                const float4 s0 = *reinterpret_cast<const float4*>(lnp + c * 8), s1 = *reinterpret_cast<const float4*>(lnp + c * 8 + 4);
                const float4 o0 = *reinterpret_cast<const float4*>(lnp + K + c * 8), o1 = *reinterpret_cast<const float4*>(lnp + K + c * 8 + 4);
                const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                const float of[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float a = fmaf((bf16lo_to_f32(ww[e]) - mean) * rstd, sc[2 * e], of[2 * e]);
                  const float b = fmaf((bf16hi_to_f32(ww[e]) - mean) * rstd, sc[2 * e + 1], of[2 * e + 1]);
                  ww[e] = pack_bf16x2(a, b);
                }
                w = make_uint4(ww[0], ww[1], ww[2], ww[3]);
              }
            }
            *reinterpret_cast<uint4*>(dst + (c >> 3) * kAtom + swz_off(trow, c & 7, 128)) = w;
          }
        } else {
          // channel-major source [K, rows]: lanes read consecutive rows of one channel (coalesced); K <= 128
          const int64_t m = o * p.inner + r, mtot = p.outer * p.inner;
          float v[128];
#pragma unroll
          for (int k = 0; k < 128; ++k) {
            float t = 0.f;
            if (k < K && valid)
              t = src.dtype == CFK_F32 ? static_cast<const float*>(src.x)[int64_t(k) * mtot + m]
                                       : __bfloat162float(static_cast<const __nv_bfloat16*>(src.x)[int64_t(k) * mtot + m]);
            v[k] = t;
          }
          float mean = 0.f, rstd = 1.f;
          if (src.ln_scale != nullptr) {
            float sum = 0.f;
#pragma unroll
            for (int k = 0; k < 128; ++k) sum += v[k];
            mean = sum / K;
            float var = 0.f;
#pragma unroll
            for (int k = 0; k < 128; ++k) {
              const float d = k < K ? v[k] - mean : 0.f;
              var = fmaf(d, d, var);
            }
            rstd = rsqrtf(var / K + p.eps);
          }
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (c * 8 < K) {
              uint32_t ww[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float a = v[c * 8 + 2 * e], b = v[c * 8 + 2 * e + 1];
                if (src.ln_scale != nullptr && valid) {
                  a = fmaf((a - mean) * rstd, lnp[c * 8 + 2 * e], lnp[K + c * 8 + 2 * e]);
                  b = fmaf((b - mean) * rstd, lnp[c * 8 + 2 * e + 1], lnp[K + c * 8 + 2 * e + 1]);
                }
                ww[e] = pack_bf16x2(a, b);
              }
              *reinterpret_cast<uint4*>(dst + (c >> 3) * kAtom + swz_off(trow, c & 7, 128)) = make_uint4(ww[0], ww[1], ww[2], ww[3]);
            }
          }
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[stage]);
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ epilogue
    const int quad = warp & 3, trow = quad * 32 + lane;
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    bool ok = true;
    uint32_t cc = 0;
    const bool two_out = p.mode == kModeLinear && p.dual;
    for (int64_t tile = blockIdx.x; tile < ka.ntiles; tile += gridDim.x) {
      const int64_t o = tile / ka.tiles_per_outer;
      const int64_t r = (tile % ka.tiles_per_outer) * kRows + trow;
      const bool valid = r < p.inner;
      const int64_t src_row = o * p.src[0].stride_outer + r * p.src[0].stride_inner;
      const int64_t out_row = o * p.inner + r;
      float mk = valid ? 1.f : 0.f;
      if (p.rowmask != nullptr && valid) {
        const float m = p.rowmask_dtype == CFK_F32 ? static_cast<const float*>(p.rowmask)[src_row]
                                                   : __bfloat162float(static_cast<const __nv_bfloat16*>(p.rowmask)[src_row]);
        mk = fmaxf(m, 0.f);
      }
      for (int c = 0; c < p.chunks; ++c, ++cc) {
        const int buf = cc & 1;
        if (ok && !mbar_wait_deadline(&acc_full[buf], (cc >> 1) & 1)) {
          report_timeout(p.status, 905);
          ok = false;
        }
        tc_fence_after();
        const int cg = p.chunk0 + c;
        const int bcol = (cg / p.chunks_per_slot) * p.bias_slot_stride + (cg % p.chunks_per_slot) * p.n_chunk;  // bias index
        const int arr = two_out ? 0 : cg / p.chunks_per_array;
        const int ocol = (cg % p.chunks_per_array) * p.n_chunk;
        for (int sub = 0; sub < p.n_chunk / 32; ++sub) {
          float y[2][32];
          tmem_ld_x32(tmem + lane_addr + buf * 256 + sub * 32, reinterpret_cast<uint32_t(&)[32]>(y[0]));
          if (p.dual) tmem_ld_x32(tmem + lane_addr + buf * 256 + 128 + sub * 32, reinterpret_cast<uint32_t(&)[32]>(y[1]));
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            if (i == 1 && !p.dual) break;
            if (p.bias[i] != nullptr) {
              const __nv_bfloat16* b = static_cast<const __nv_bfloat16*>(p.bias[i]) + bcol + sub * 32;
#pragma unroll
              for (int j = 0; j < 32; ++j) y[i][j] += __bfloat162float(b[j]);
            }
          }
          if (p.mode == kModeGdp) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float g = y[1][j];
              const float a = p.swish ? g * act_sigmoid(g) : act_sigmoid(g);
              y[0][j] = mk * y[0][j] * a;
            }
          } else if (p.mode == kModeEpi) {
#pragma unroll
            for (int j = 0; j < 32; ++j) y[0][j] = valid ? y[0][j] * act_sigmoid(y[1][j]) : 0.f;
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              y[0][j] *= mk;
              y[1][j] *= mk;
            }
          }
          const int nouts = two_out ? 2 : 1;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            if (i >= nouts) break;
            const int a_idx = two_out ? i : arr;
            const int col = ocol + sub * 32;
            if (!ok || p.out[a_idx] == nullptr) continue;
            if (p.out_channel_major) {
              // [n, outer, inner_pad]: lanes write consecutive rows of one channel
              if (r < p.inner_pad) {
                const int64_t plane = p.outer * p.inner_pad;
                if (p.out_dtype == CFK_E4M3) {
                  uint8_t* dst = static_cast<uint8_t*>(p.out[a_idx]) + o * p.inner_pad + r;
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    if (col + j < p.n_valid)
                      dst[int64_t(col + j) * plane] =
                          uint8_t(__nv_cvt_float2_to_fp8x2(make_float2(y[i][j] * p.out_scale, 0.f), __NV_SATFINITE, __NV_E4M3) & 0xff);
                } else {
                  __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out[a_idx]) + o * p.inner_pad + r;
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    if (col + j < p.n_valid) dst[int64_t(col + j) * plane] = __float2bfloat16_rn(y[i][j]);
                }
              }
            } else if (valid) {
              if (i == 0 && p.residual != nullptr) {
                const __nv_bfloat16* res = static_cast<const __nv_bfloat16*>(p.residual) + out_row * p.ldo + col;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col + j < p.n_valid) y[0][j] += __bfloat162float(res[j]);
              }
              if (i == 0 && p.add_source1) {
                const RowSource& s1 = p.src[1];
                const __nv_bfloat16* xr = static_cast<const __nv_bfloat16*>(s1.x) +
                                          (o * s1.stride_outer + r * s1.stride_inner) * s1.k + col;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col + j < p.n_valid) y[0][j] += __bfloat162float(xr[j]);
              }
              if (p.out_dtype == CFK_E4M3) {
                uint8_t* dst = static_cast<uint8_t*>(p.out[a_idx]) + out_row * p.ldo + col;
#pragma unroll
                for (int j = 0; j < 32; j += 2)
                  if (col + j < p.n_valid)
                    *reinterpret_cast<uint16_t*>(dst + j) = uint16_t(__nv_cvt_float2_to_fp8x2(
                        make_float2(y[i][j] * p.out_scale, y[i][j + 1] * p.out_scale), __NV_SATFINITE, __NV_E4M3));
              } else {
                __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out[a_idx]) + out_row * p.ldo + col;
#pragma unroll
                for (int j = 0; j < 32; j += 8)
                  if (col + j < p.n_valid)
                    *reinterpret_cast<uint4*>(dst + j) =
                        make_uint4(pack_bf16x2(y[i][j], y[i][j + 1]), pack_bf16x2(y[i][j + 2], y[i][j + 3]),
                                   pack_bf16x2(y[i][j + 4], y[i][j + 5]), pack_bf16x2(y[i][j + 6], y[i][j + 7]));
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int launch_rowgemm(const RowGemmParams& prm, const CUtensorMap& tw0, const CUtensorMap& tw1, cudaStream_t st) {
  KernelArgs ka{};
  ka.p = prm;
  const RowGemmParams& p = ka.p;
  const int nsrc = p.src[1].x != nullptr ? 2 : 1;
  const int nacc = p.dual ? 2 : 1;
  int off = 0;
  for (int i = 0; i < 2; ++i) {
    const int kw = p.src[(i == 1 && nsrc == 2) ? 1 : 0].k;
    ka.l.w[i] = off;
    ka.l.w_chunk[i] = (p.n_chunk / 64) * kw * 128;
    if (i < nacc) off += p.chunks * ka.l.w_chunk[i];
  }
  for (int i = 0; i < 2; ++i) {
    ka.l.a[i] = off;
    ka.l.a_stage[i] = (p.src[i].k / 64) * kAtom;
    if (i < nsrc) off += 2 * ka.l.a_stage[i];
  }
  for (int i = 0; i < 2; ++i) {
    ka.l.ln[i] = off;
    if (i < nsrc) off += 2 * p.src[i].k * 4;
  }
  ka.l.stage_out = off;
  ka.l.bars = (off + 15) & ~15;
  ka.l.tmem = ka.l.bars + 9 * 8;
  ka.l.total = ka.l.tmem + 16 + 1024;
  if (ka.l.total > 232448) return CFK_ERR_UNSUPPORTED;
  ka.tiles_per_outer = (p.inner_pad + kRows - 1) / kRows;
  ka.ntiles = p.outer * ka.tiles_per_outer;
  if (ka.ntiles == 0) return CFK_OK;
  if (cudaFuncSetAttribute(rowgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ka.l.total) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = int(ka.ntiles < sms ? ka.ntiles : sms);
  rowgemm_kernel<<<grid, kThreadsRg, ka.l.total, st>>>(tw0, tw1, ka);
  return check_launch();
}

// weights [slots, K, N] bf16 row-major: box = 64 columns x K rows, 128-byte swizzle (MN-major B operand atoms)
int make_weight_map(CUtensorMap* m, const void* w, int slots, int k, int n) {
  uint64_t dims[3] = {uint64_t(n), uint64_t(k), uint64_t(slots)};
  uint64_t strides[2] = {uint64_t(n) * 2, uint64_t(n) * k * 2};
  uint32_t box[3] = {64, uint32_t(k), 1};
  return make_tensor_map(m, w, CFK_BF16, 3, dims, strides, box, 128);
}

}  // namespace cfk
