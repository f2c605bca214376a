// Per-head attention bias from a LayerNorm-ed activation: bias[h, m] = (LN(x) wb)[m, h] (packed_attn.py:225-229).
// The op reads 2 a bytes per row and writes 2 h (h = 4 or 8 heads): it is bound by the read of x.
//
// LayerNorm is folded around the dot, LN(x) wb = rstd * (x w' - mean * s) + t with w'[k][h] = scale[k] wb[k][h] (bf16,
// prepared once per CTA), s[h] = sum_k w'[k][h], t[h] = sum_k offset[k] wb[k][h]: the dot runs on the RAW 128-row tile as TMA
// lands it (one accumulator of 16 ... 64 columns, a / 16 MMAs per tile), while thread = row takes the row's sum and sum
// of squares from the same tile, and the epilogue is eight values per thread.  (A CUDA-core version of the dot -
// thread = row, packed FMAs against weights broadcast from shared memory - spent 1 770 instructions per row and ran at a
// quarter of the copy bandwidth.)  The result leaves channel-major: consecutive threads write consecutive rows of a head.
// Row blocks of 128 follow `keep` (transition.py:29-38): a block it marks nowhere is written as zeros, a block that is
// negative throughout is left unwritten.  Every mbarrier wait is deadline-bounded.
#include "attention_sm100.cuh"

namespace cfk {
namespace {

constexpr int kRowsHb = 128;
constexpr int kThreadsHb = 320;     // warp 0 producer, warp 1 MMA issuer, warps 2-5 and 6-9: thread = row, tiles in turn
constexpr int kStagesHb = 3;
constexpr int kMaxTilesHb = 1024;

// Up to two weight matrices side by side ([a, hp0] giving columns 0 .. h0-1 into out0, [a, hp1] giving h1 more into
// out1), optional biases, an optional row mask, rows addressed as (outer, inner) with strides so that a transposed read
// (the MSA with rows running along the depth for a fixed residue) is the same kernel, outputs [h, outer, inner_pad].
struct HbParams {
  const float* ln_scale;
  const float* ln_offset;
  const __nv_bfloat16* w0;   // [a, hp0]
  const __nv_bfloat16* w1;   // [a, hp1] or null
  const __nv_bfloat16* b0;   // [h0] or null
  const __nv_bfloat16* b1;   // [h1] or null
  const __nv_bfloat16* mask; // per source row, or null; negative counts as zero
  const void* keep;
  int keep_dtype;
  __nv_bfloat16* out0;       // [h0, outer, inner_pad]
  __nv_bfloat16* out1;       // [h1, outer, inner_pad]
  int64_t outer, inner, inner_pad, stride_outer, stride_inner, tiles_per_outer, ntiles;
  int h0, hp0, h1, hp1, n;   // n = h0 + h1 rounded up to 16: accumulator columns
  float eps;
  int* status;
};

template <int A>
__global__ void __launch_bounds__(kThreadsHb, 1)
ln_head_bias_kernel(const __grid_constant__ CUtensorMap tm_x, const HbParams prm) {
  constexpr int kTile = kRowsHb * A * 2;          // A / 64 atoms of [128 rows][64 channels]
  constexpr int kOffW = kStagesHb * kTile;        // w' as the K-major B operand: A / 64 atoms of [64 rows n][64 channels]
  constexpr int kWBytes = (A / 64) * 64 * 128;
  constexpr int kOffCst = kOffW + kWBytes;        // float2 [64]: s, t
  constexpr int kOffBar = kOffCst + 64 * 8;
  constexpr int kOffTmem = kOffBar + (2 * kStagesHb + 4 + 1) * 8;
  constexpr int kOffCls = kOffTmem + 16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;                     // [3] the tile has landed
  uint64_t* s_free = full + kStagesHb;       // [3] ... and neither the MMAs nor the row threads read it any more
  uint64_t* acc_full = s_free + kStagesHb;   // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint64_t* w_ready = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  float2* cst = reinterpret_cast<float2*>(smem + kOffCst);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = prm.ntiles;
  const int h = prm.h0 + prm.h1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStagesHb; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(w_ready, 8);
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  // tile classes from keep: 1 compute, 0 zeros, -1 leave alone
  const int8_t* cls = nullptr;
  if (prm.keep != nullptr) {
    int8_t* w = reinterpret_cast<int8_t*>(smem + kOffCls);
    for (int i = warp;; i += kThreadsHb / 32) {
      const int64_t tile = blockIdx.x + int64_t(i) * gridDim.x;
      if (tile >= ntiles) break;
      float top = -1.f;
      const int64_t o = tile / prm.tiles_per_outer, r0 = (tile % prm.tiles_per_outer) * kRowsHb;
      for (int j = lane; j < kRowsHb; j += 32) {
        const int64_t r = r0 + j;
        if (r < prm.inner) {
          const int64_t src = o * prm.stride_outer + r * prm.stride_inner;
          top = fmaxf(top, prm.keep_dtype == CFK_F32 ? static_cast<const float*>(prm.keep)[src]
                                                     : __bfloat162float(static_cast<const __nv_bfloat16*>(prm.keep)[src]));
        } else if (r < prm.inner_pad) {
          top = fmaxf(top, 0.f);
        }
      }
      for (int off = 16; off > 0; off >>= 1) top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, off));
      if (lane == 0) w[i] = top > 0.f ? 1 : (top == 0.f ? 0 : -1);
    }
    cls = w;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto next_computed = [&](uint32_t& seq) -> int64_t {
    for (;; ++seq) {
      const int64_t tile = blockIdx.x + int64_t(seq) * gridDim.x;
      if (tile >= ntiles) return -1;
      if (cls == nullptr || cls[seq] == 1) return tile;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      uint32_t seq = 0, ti = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        const int st = ti % kStagesHb;
        ok = mbar_wait_deadline(&s_free[st], ((ti / kStagesHb) & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 1801); break; }
        mbar_arrive_expect_tx(&full[st], kTile);
        const int o = int(tile / prm.tiles_per_outer), r0 = int(tile % prm.tiles_per_outer) * kRowsHb;
#pragma unroll
        for (int a = 0; a < A / 64; ++a) tma_load_3d(smem + st * kTile + a * (kRowsHb * 128), &tm_x, &full[st], a * 64, r0, o);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer: acc[row][head] = x w'
    if (lane == 0) {
      const uint32_t idesc = make_idesc(kRowsHb, uint32_t(prm.n), 1, 1, 0, 0);   // both operands K-major
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      const uint32_t wk = desc_lo(smem_u32(smem + kOffW), 16);
      bool ok = mbar_wait_deadline(w_ready, 0);
      if (!ok) report_timeout(prm.status, 1802);
      uint32_t seq = 0, ti = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        const int st = ti % kStagesHb, ab = ti & 1;
        ok = mbar_wait_deadline(&full[st], (ti / kStagesHb) & 1);
        if (!ok) { report_timeout(prm.status, 1803); break; }
        ok = mbar_wait_deadline(&acc_empty[ab], ((ti >> 1) & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 1804); break; }
        tc_fence_after();
        const uint32_t xk = desc_lo(smem_u32(smem + st * kTile), 16);
#pragma unroll
        for (int kk = 0; kk < A / 16; ++kk)
          mma_f16_ss2(tmem + ab * 64, xk + (kk / 4) * ((kRowsHb * 128) >> 4) + (kk % 4) * 2, hi,
                      wk + (kk / 4) * ((64 * 128) >> 4) + (kk % 4) * 2, hi, idesc, kk > 0);
        mma_commit(&acc_full[ab]);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ row threads
    // two groups of four warps take the computed tiles in turn (group = accumulator buffer): a group alone is one warp per
    // scheduler, and every dependent instruction of its statistics pass and epilogue would wait in the open
    const int grp = (warp - 2) >> 2;
    const int quad = warp & 3;                      // TMEM lane quarter of this warp
    const int trow = quad * 32 + lane;
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const int pt = (warp - 2) * 32 + lane;
    bool ok = true;
    // column n of the two weight matrices side by side
    auto weight = [&](int k, int n) -> float {
      return __bfloat162float(n < prm.h0 ? prm.w0[k * prm.hp0 + n] : prm.w1[k * prm.hp1 + (n - prm.h0)]);
    };
    // ---- once: w'[n][k] = scale[k] w[k][n] as a K-major tile (rows n, 128-byte swizzle), s[n], t[n] (+ bias)
    for (int i = pt; i < 64 * (A / 8); i += 256) {   // 16-byte pieces: 8 consecutive k of one row n
      const int n = i / (A / 8), p = i % (A / 8);
      uint32_t v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int k = p * 8 + 2 * e;
        v[e] = pack_bf16x2(n < h ? prm.ln_scale[k] * weight(k, n) : 0.f, n < h ? prm.ln_scale[k + 1] * weight(k + 1, n) : 0.f);
      }
      *reinterpret_cast<uint4*>(smem + kOffW + (p >> 3) * (64 * 128) + swz_off(n, p & 7, 128)) = make_uint4(v[0], v[1], v[2], v[3]);
    }
    if (pt < 64) {
      float s = 0.f, t = 0.f;
      if (pt < h) {
        for (int k = 0; k < A; ++k) {
          const float w = weight(k, pt);
          s += __bfloat162float(__float2bfloat16_rn(prm.ln_scale[k] * w));
          t = fmaf(prm.ln_offset[k], w, t);
        }
        if (pt < prm.h0 && prm.b0 != nullptr) t += __bfloat162float(prm.b0[pt]);
        if (pt >= prm.h0 && prm.b1 != nullptr) t += __bfloat162float(prm.b1[pt - prm.h0]);
      }
      cst[pt] = make_float2(s, t);
    }
    fence_proxy_async();
    named_bar_sync(2, 256);
    if (lane == 0) mbar_arrive(w_ready);

    const int64_t plane = prm.outer * prm.inner_pad;
    // where column n of the accumulator goes
    auto dst = [&](int n, int64_t at) -> __nv_bfloat16* {
      return n < prm.h0 ? prm.out0 + int64_t(n) * plane + at : prm.out1 + int64_t(n - prm.h0) * plane + at;
    };
    uint32_t seq = 0, ti = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++seq) {
      const int64_t o = tile / prm.tiles_per_outer;
      const int64_t r = (tile % prm.tiles_per_outer) * kRowsHb + trow;
      const bool in_pad = r < prm.inner_pad;          // a position of the output
      const bool valid = r < prm.inner;               // ... that is a row of x
      const int64_t at = o * prm.inner_pad + r;
      if (cls != nullptr && cls[seq] != 1) {
        if (cls[seq] == 0 && in_pad && grp == int(seq & 1))
          for (int hh = 0; hh < h; ++hh) *dst(hh, at) = __float2bfloat16_rn(0.f);
        continue;
      }
      if (int(ti & 1) != grp) {  // the other group's tile
        ++ti;
        continue;
      }
      float mk = valid ? 1.f : 0.f;
      if (valid && prm.mask != nullptr) mk = fmaxf(__bfloat162float(prm.mask[o * prm.stride_outer + r * prm.stride_inner]), 0.f);
      const int st = ti % kStagesHb, ab = ti & 1;
      if (ok && !mbar_wait_deadline(&full[st], (ti / kStagesHb) & 1)) {
        report_timeout(prm.status, 1805);
        ok = false;
      }
      // ---- the row's statistics from the raw tile (fp32 sums over bf16 data, one pass)
      const uint8_t* xs = smem + st * kTile;
      float s0 = 0.f, s1 = 0.f, q0 = 0.f, q1 = 0.f;
#pragma unroll
      for (int c = 0; c < A / 8; ++c) {
        const uint4 w = *reinterpret_cast<const uint4*>(xs + (c >> 3) * (kRowsHb * 128) + swz_off(trow, c & 7, 128));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = bf16lo_to_f32(ww[e]), b = bf16hi_to_f32(ww[e]);
          s0 += a; s1 += b;
          q0 = fmaf(a, a, q0); q1 = fmaf(b, b, q1);
        }
      }
      const float mean = (s0 + s1) * (1.0f / A);
      const float var = fmaxf((q0 + q1) * (1.0f / A) - mean * mean, 0.f);
      const float rstd = rsqrtf(var + prm.eps);
      // ---- epilogue: rstd * (acc - mean s) + t, eight heads at a time
      if (ok && !mbar_wait_deadline(&acc_full[ab], (ti >> 1) & 1)) {
        report_timeout(prm.status, 1806);
        ok = false;
      }
      tc_fence_after();
      const float nmr = -mean * rstd * mk, rm = rstd * mk;   // mk * (rstd * (acc - mean s) + t) = rm acc + nmr s + mk t
      for (int hb = 0; hb < h; hb += 16) {
        uint32_t acc[16];
        tmem_ld_x16(tmem + lane_addr + ab * 64 + hb, acc);
        tmem_wait_ld();
        if (in_pad) {
          __nv_bfloat16* p = hb < prm.h0 ? prm.out0 + int64_t(hb) * plane + at : prm.out1 + int64_t(hb - prm.h0) * plane + at;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (hb + j == prm.h0) p = prm.out1 - int64_t(j) * plane + at;   // the second output starts here
            if (hb + j < h) {
              const float2 c = cst[hb + j];
              p[int64_t(j) * plane] = __float2bfloat16_rn(fmaf(rm, __uint_as_float(acc[j]), fmaf(nmr, c.x, mk * c.y)));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc_empty[ab]);
        mbar_arrive(&s_free[st]);
      }
      ++ti;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

template <int A>
int launch_hb(const void* x, HbParams prm, cudaStream_t st) {
  prm.tiles_per_outer = (prm.inner_pad + kRowsHb - 1) / kRowsHb;
  prm.ntiles = prm.outer * prm.tiles_per_outer;
  prm.n = (prm.h0 + prm.h1 + 15) / 16 * 16;
  prm.status = device_status_word();
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  if (prm.ntiles == 0) return CFK_OK;
  CUtensorMap tx;
  {
    const uint64_t row = uint64_t(A) * 2;
    uint64_t dims[3] = {uint64_t(A), uint64_t(prm.inner), uint64_t(prm.outer)};
    uint64_t str[2] = {uint64_t(prm.stride_inner) * row,
                       (prm.outer > 1 ? uint64_t(prm.stride_outer) : uint64_t(prm.inner) * uint64_t(prm.stride_inner)) * row};
    uint32_t box[3] = {64, kRowsHb, 1};
    int rc = make_tensor_map(&tx, x, CFK_BF16, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  const int smem = kStagesHb * kRowsHb * A * 2 + (A / 64) * 64 * 128 + 64 * 8 + (2 * kStagesHb + 5) * 8 + 16 + kMaxTilesHb + 1024;
  auto kern = ln_head_bias_kernel<A>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = int(prm.ntiles < sms ? prm.ntiles : sms);
  if (prm.keep != nullptr && (prm.ntiles + grid - 1) / grid > kMaxTilesHb) return CFK_ERR_UNSUPPORTED;
  kern<<<grid, kThreadsHb, smem, st>>>(tx, prm);
  return check_launch();
}

int launch_hb_any(const void* x, int a, const HbParams& prm, cudaStream_t st) {
  switch (a) {
    case 64: return launch_hb<64>(x, prm, st);
    case 128: return launch_hb<128>(x, prm, st);
    case 256: return launch_hb<256>(x, prm, st);
    default: return CFK_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace cfk

using namespace cfk;

extern "C" int cfk_ln_head_bias(const void* x, const float* ln_scale, const float* ln_offset, const void* wb,
                                const void* keep, int keep_dtype, void* bias_out, int64_t m, int a, int h, int h_padded,
                                float eps, void* stream) {
  if (!x || !ln_scale || !ln_offset || !wb || !bias_out) return CFK_ERR_NULL;
  if (m < 0 || h <= 0 || h > h_padded || h > 64 || m > INT32_MAX) return CFK_ERR_SHAPE;
  if (a != 64 && a != 128 && a != 256) return CFK_ERR_UNSUPPORTED;
  if (keep != nullptr && keep_dtype != CFK_F32 && keep_dtype != CFK_BF16) return CFK_ERR_DTYPE;
  if (m == 0) return CFK_OK;
  if (!aligned16(x)) return CFK_ERR_ALIGN;
  HbParams prm{};
  prm.ln_scale = ln_scale; prm.ln_offset = ln_offset;
  prm.w0 = static_cast<const __nv_bfloat16*>(wb); prm.h0 = h; prm.hp0 = h_padded;
  prm.keep = keep; prm.keep_dtype = keep_dtype;
  prm.out0 = static_cast<__nv_bfloat16*>(bias_out);
  prm.outer = 1; prm.inner = m; prm.inner_pad = m; prm.stride_outer = 0; prm.stride_inner = 1;
  prm.eps = eps;
  return launch_hb_any(x, a, prm, static_cast<cudaStream_t>(stream));
}

// The two outer-product-mean projections written channel-major with the MSA depth contiguous, [k, r, pitch]: x [s, r, c]
// is read with rows running along s for a fixed residue, so that the fused outer product mean takes both results as
// K-major operands without a transposed copy.
extern "C" int cfk_opm_projection_cm(const void* x, const float* ln_scale, const float* ln_offset, const void* lw,
                                     const void* lb, const void* rw, const void* rb, const void* mask, void* left,
                                     void* right, int64_t s, int64_t r, int c, int k, int64_t pitch, float eps,
                                     void* stream) {
  if (!x || !ln_scale || !ln_offset || !lw || !lb || !rw || !rb || !mask || !left || !right) return CFK_ERR_NULL;
  if (s < 0 || r < 0 || k <= 0 || k > 32 || pitch < s || s > INT32_MAX || r > INT32_MAX) return CFK_ERR_SHAPE;
  if (c != 64 && c != 128 && c != 256) return CFK_ERR_UNSUPPORTED;
  if (s == 0 || r == 0) return CFK_OK;
  if (!aligned16(x)) return CFK_ERR_ALIGN;
  HbParams prm{};
  prm.ln_scale = ln_scale; prm.ln_offset = ln_offset;
  prm.w0 = static_cast<const __nv_bfloat16*>(lw); prm.h0 = k; prm.hp0 = k;
  prm.w1 = static_cast<const __nv_bfloat16*>(rw); prm.h1 = k; prm.hp1 = k;
  prm.b0 = static_cast<const __nv_bfloat16*>(lb); prm.b1 = static_cast<const __nv_bfloat16*>(rb);
  prm.mask = static_cast<const __nv_bfloat16*>(mask);
  prm.out0 = static_cast<__nv_bfloat16*>(left); prm.out1 = static_cast<__nv_bfloat16*>(right);
  prm.outer = r; prm.inner = s; prm.inner_pad = pitch; prm.stride_outer = 1; prm.stride_inner = r;
  prm.eps = eps;
  return launch_hb_any(x, c, prm, static_cast<cudaStream_t>(stream));
}
