// Per-head attention bias from a LayerNorm-ed activation: bias[h, m] = (LN(x) wb)[m, h] (packed_attn.py:225-229).
// The op reads 2 a bytes per row and writes 2 h (h = 4 or 8 heads): it is HBM-bound on the read, and with so few
// output columns a tensor-core tile would be all padding, so this is a CUDA-core kernel: a block stages 128 rows in
// shared memory with coalesced 16-byte loads, then thread = row accumulates, in one pass over its row, the fp32
// statistics and the dot with up to eight scale-folded weight columns (packed f32x2 FMAs, the weights broadcast from
// shared memory), and applies mean, rstd and the offset's dot at the end.  The result leaves
// channel-major: consecutive threads write consecutive rows of one head.
// Row blocks of 128 follow `keep` (transition.py:29-38): a block it marks nowhere is written as zeros, a block that is
// negative throughout is left unwritten.
#include "cfk_common.cuh"
#include "cfk_ptx.cuh"

namespace cfk {
namespace {

constexpr int kRowsHb = 128;

template <int A>
__global__ void __launch_bounds__(kRowsHb) ln_head_bias_kernel(const __nv_bfloat16* __restrict__ x,
                                                               const float* __restrict__ ln_scale,
                                                               const float* __restrict__ ln_offset,
                                                               const __nv_bfloat16* __restrict__ wb, const void* keep,
                                                               int keep_dtype, __nv_bfloat16* __restrict__ out, int64_t m,
                                                               int h, int hp, float eps) {
  constexpr int kPitch = A * 2 + 16;             // bytes per staged row: the 16 spare bytes spread the rows over banks
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* xs = smem;                                            // [128][kPitch]
  float2* ws = reinterpret_cast<float2*>(smem + kRowsHb * kPitch);  // [A][4]: eight weight columns of the current group
  float2* gb = ws + A * 4;                                       // [A]: LayerNorm scale, offset
  __shared__ float s_top[kRowsHb / 32], s_sw[8], s_tw[8];
  const int t = threadIdx.x;
  for (int k = t; k < A; k += kRowsHb) gb[k] = make_float2(ln_scale[k], ln_offset[k]);
  // the weights of one group of eight heads in shared memory: w'[k][h] = scale[k] wb[k][h], their column sums and the
  // offset's dot with wb (one head per thread, the k loop split over 16 threads and combined by shuffle)
  auto stage_weights = [&](int h0) {
    for (int i = t; i < A * 4; i += kRowsHb) {
      const int k = i >> 2, j = (i & 3) * 2 + h0;
      const float g = gb[k].x;
      ws[i] = make_float2(j < h ? g * __bfloat162float(wb[k * hp + j]) : 0.f,
                          j + 1 < h ? g * __bfloat162float(wb[k * hp + j + 1]) : 0.f);
    }
    {
      const int hh = t >> 4, part = t & 15;  // 8 heads x 16 threads
      float sw = 0.f, tw = 0.f;
      if (h0 + hh < h)
        for (int k = part; k < A; k += 16) {
          const float wv = __bfloat162float(wb[k * hp + h0 + hh]);
          sw = fmaf(gb[k].x, wv, sw);
          tw = fmaf(gb[k].y, wv, tw);
        }
      for (int off = 8; off > 0; off >>= 1) {
        sw += __shfl_xor_sync(0xffffffffu, sw, off);
        tw += __shfl_xor_sync(0xffffffffu, tw, off);
      }
      if (part == 0) {
        s_sw[hh] = sw;
        s_tw[hh] = tw;
      }
    }
  };
  __syncthreads();
  if (h <= 8) stage_weights(0);
  const int64_t ntiles = (m + kRowsHb - 1) / kRowsHb;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t r0 = tile * kRowsHb;
    const int64_t row = r0 + t;
    // ---- the block's class: largest keep value over its rows (> 0 compute, == 0 zeros, < 0 leave alone)
    float top = 1.f;
    if (keep != nullptr) {
      float v = -1.f;
      if (row < m)
        v = keep_dtype == CFK_F32 ? static_cast<const float*>(keep)[row]
                                  : __bfloat162float(static_cast<const __nv_bfloat16*>(keep)[row]);
      for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
      if ((t & 31) == 0) s_top[t >> 5] = v;
      __syncthreads();
      top = fmaxf(fmaxf(s_top[0], s_top[1]), fmaxf(s_top[2], s_top[3]));
    }
    if (top < 0.f) {
      __syncthreads();
      continue;
    }
    if (top == 0.f) {
      if (row < m)
        for (int hh = 0; hh < h; ++hh) out[int64_t(hh) * m + row] = __float2bfloat16_rn(0.f);
      __syncthreads();
      continue;
    }
    // ---- stage the rows: 16-byte pieces, consecutive threads on consecutive pieces
    constexpr int kPieces = A / 8;  // per row
    for (int i = t; i < kRowsHb * kPieces; i += kRowsHb) {
      const int r = i / kPieces, c = i % kPieces;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r0 + r < m) v = __ldg(reinterpret_cast<const uint4*>(x + (r0 + r) * A) + c);
      *reinterpret_cast<uint4*>(xs + r * kPitch + c * 16) = v;
    }
    __syncthreads();
    const uint8_t* mine = xs + t * kPitch;
    // ---- eight heads at a time, one pass over the row: with w'[k][h] = scale[k] wb[k][h] (fp32, in shared memory)
    //   (LN(x) wb)[h] = rstd * (sum_k x[k] w'[k][h] - mean * sum_k w'[k][h]) + sum_k offset[k] wb[k][h]
    // so the dot runs on the raw row while the statistics accumulate beside it (the normalised row is not rounded to
    // bf16 on the way, which only brings the result closer to exact arithmetic)
    for (int h0 = 0; h0 < h; h0 += 8) {
      if (h > 8) {  // more than one group of eight heads: the group's weights are set up per pass
        __syncthreads();
        stage_weights(h0);
        __syncthreads();
      }
      uint64_t acc[4] = {0, 0, 0, 0};
      float sum = 0.f, sq = 0.f;
#pragma unroll 2
      for (int c = 0; c < kPieces; ++c) {
        const uint4 w = *reinterpret_cast<const uint4*>(mine + c * 16);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = c * 8 + 2 * e;
          const float y0 = bf16lo_to_f32(ww[e]), y1 = bf16hi_to_f32(ww[e]);
          sum += y0 + y1;
          sq = fmaf(y0, y0, fmaf(y1, y1, sq));
          const uint64_t b0 = f2_pack(y0, y0), b1 = f2_pack(y1, y1);
          const ulonglong2* w0 = reinterpret_cast<const ulonglong2*>(ws + k * 4);
          const ulonglong2 p0 = w0[0], p1 = w0[1], q0 = w0[2], q1 = w0[3];
          acc[0] = f2_fma(b0, p0.x, acc[0]);
          acc[1] = f2_fma(b0, p0.y, acc[1]);
          acc[2] = f2_fma(b0, p1.x, acc[2]);
          acc[3] = f2_fma(b0, p1.y, acc[3]);
          acc[0] = f2_fma(b1, q0.x, acc[0]);
          acc[1] = f2_fma(b1, q0.y, acc[1]);
          acc[2] = f2_fma(b1, q1.x, acc[2]);
          acc[3] = f2_fma(b1, q1.y, acc[3]);
        }
      }
      const float mean = sum * (1.0f / A);
      // second moment about the mean from the raw sums; the row is bf16 data, so fp32 sums leave this difference exact
      // to far below the data's own precision unless |mean| exceeds the spread a thousandfold
      const float var = fmaxf(sq * (1.0f / A) - mean * mean, 0.f);
      const float rstd = rsqrtf(var + eps);
      if (row < m) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float lo, hi;
          f2_unpack(acc[j], lo, hi);
          const int ha = h0 + 2 * j;
          if (ha < h) out[int64_t(ha) * m + row] = __float2bfloat16_rn(fmaf(rstd, lo - mean * s_sw[2 * j], s_tw[2 * j]));
          if (ha + 1 < h) out[int64_t(ha + 1) * m + row] = __float2bfloat16_rn(fmaf(rstd, hi - mean * s_sw[2 * j + 1], s_tw[2 * j + 1]));
        }
      }
    }
    __syncthreads();  // the staged rows are read no more
  }
}

template <int A>
int launch_hb(const void* x, const float* ln_scale, const float* ln_offset, const void* wb, const void* keep, int keep_dtype,
              void* out, int64_t m, int h, int hp, float eps, cudaStream_t st) {
  const int smem = kRowsHb * (A * 2 + 16) + A * 4 * 8 + A * 8;
  auto kern = ln_head_bias_kernel<A>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int per_sm = 227 * 1024 / (smem + 1024) < 8 ? 227 * 1024 / (smem + 1024) : 8;
  const int64_t ntiles = (m + kRowsHb - 1) / kRowsHb;
  const int64_t want = int64_t(sms) * per_sm;
  const int grid = int(ntiles < want ? ntiles : want);
  kern<<<grid, kRowsHb, smem, st>>>(static_cast<const __nv_bfloat16*>(x), ln_scale, ln_offset,
                                    static_cast<const __nv_bfloat16*>(wb), keep, keep_dtype, static_cast<__nv_bfloat16*>(out),
                                    m, h, hp, eps);
  return check_launch();
}

}  // namespace
}  // namespace cfk

using namespace cfk;

extern "C" int cfk_ln_head_bias(const void* x, const float* ln_scale, const float* ln_offset, const void* wb,
                                const void* keep, int keep_dtype, void* bias_out, int64_t m, int a, int h, int h_padded,
                                float eps, void* stream) {
  if (!x || !ln_scale || !ln_offset || !wb || !bias_out) return CFK_ERR_NULL;
  if (m < 0 || h <= 0 || h > h_padded || h_padded > 64) return CFK_ERR_SHAPE;
  if (a != 64 && a != 128 && a != 256) return CFK_ERR_UNSUPPORTED;
  if (keep != nullptr && keep_dtype != CFK_F32 && keep_dtype != CFK_BF16) return CFK_ERR_DTYPE;
  if (m == 0) return CFK_OK;
  if (!aligned16(x)) return CFK_ERR_ALIGN;
  if (device_status_word() == nullptr) return CFK_ERR_LAUNCH;
  auto st = static_cast<cudaStream_t>(stream);
  switch (a) {
    case 64: return launch_hb<64>(x, ln_scale, ln_offset, wb, keep, keep_dtype, bias_out, m, h, h_padded, eps, st);
    case 128: return launch_hb<128>(x, ln_scale, ln_offset, wb, keep, keep_dtype, bias_out, m, h, h_padded, eps, st);
    default: return launch_hb<256>(x, ln_scale, ln_offset, wb, keep, keep_dtype, bias_out, m, h, h_padded, eps, st);
  }
}
