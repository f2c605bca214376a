// Triangle-multiplication output at 128 channels in one pass without rewriting a tile (tri_mul.py:303-451):
//   out = (LN(x_cm^T) wo + bo) * sigmoid(LN(act) wg + bg) (+ act)
// with x_cm [128, M] the channel-major contraction result and act [M, 128] the module input.
//
// LayerNorm is folded around the GEMMs instead of being applied to the tiles: with w'[k][f] = scale[k] w[k][f] (rounded to
// bf16, prepared once per CTA in shared memory), s[f] = sum_k w'[k][f] and t[f] = sum_k offset[k] w[k][f] + bias[f],
//   LN(x) w + bias = rstd * (x w' - mean * s) + t
// so both GEMMs run on the RAW tiles as TMA lands them: the channel-major tile [128 channels][128 rows] is an MN-major A
// operand as it is (no transpose through registers), the row-major act tile is a K-major A operand and stays intact for
// the residual, and no thread waits for a normalised tile before the MMAs start.  The statistics (mean, rstd per row of
// both tiles) are computed by the worker warps beside the MMAs and applied in the epilogue.  s uses the same bf16 w'
// the tensor core multiplies by, so mean * s cancels the mean's part of x w' to fp32 rounding.
//
// A persistent CTA walks 128-row tiles.  Warp 0: TMA producer (weights once, then two stages of (x_cm tile, act tile)).
// Warp 1: MMA issuer (two GEMMs of 8 MMAs N = 128 per tile into one of two accumulator pairs).  Warps 4-11: weight
// preparation, statistics, epilogue (thread = row, group = 64-column half); the result is written over the stage's dead
// x_cm tile as swizzled 64-column atoms and stored by TMA.  Every mbarrier wait is deadline-bounded.
#include "attention_sm100.cuh"
#include "rowgemm_sm100.cuh"

namespace cfk {
namespace {

constexpr int kCe = 128;
constexpr int kRowsE = 128;
constexpr int kThreadsE = 384;
constexpr int kMaxTilesE = 1024;                 // tiles per CTA when row blocks may be skipped
constexpr int kAtomE = 128 * 128;                  // 16 KB: 128 lines of 128 bytes
constexpr int kOffWE = 0;                          // wo' then wg': two atoms each ([128 k][64 f])
constexpr int kOffStE = kOffWE + 4 * kAtomE;       // two stages of (x_cm tile: 2 atoms by rows; act tile: 2 atoms by k)
constexpr int kStageE = 4 * kAtomE;
constexpr int kOffRedX = kOffStE + 2 * kStageE;    // float2 [4][128]: partial (sum, sum of squares) of x_cm rows
constexpr int kOffRedA = kOffRedX + 4 * 128 * 8;   // float2 [2][128]: of act rows
constexpr int kOffCst = kOffRedA + 2 * 128 * 8;    // float4 [128]: s, t of the output path, s, t of the gate path
constexpr int kOffBarE = kOffCst + 128 * 16;
constexpr int kNumBarsE = 2 + 2 + 2 + 2 + 2;
constexpr int kOffTmemE = kOffBarE + kNumBarsE * 8;
constexpr int kOffClsE = kOffTmemE + 16;
constexpr int kSmemE = kOffClsE + kMaxTilesE + 1024;
static_assert(kSmemE <= 232448, "shared memory budget");

struct EpiParams {
  const float* ln_scale;     // centre LayerNorm over the channels of x_cm
  const float* ln_offset;
  const float* in_scale;     // LayerNorm of act for the gate, or null (act is used as it is)
  const float* in_offset;
  const __nv_bfloat16* bo;
  const __nv_bfloat16* bg;
  int64_t m;
  float eps;
  int add_input;
  const void* keep;          // [M] or null: 128-row blocks it marks nowhere are not computed
  int keep_dtype;
  const __nv_bfloat16* act;  // for the rows of a block that is not computed
  __nv_bfloat16* out;
  int* status;
};

__global__ void __launch_bounds__(kThreadsE, 1)
trimul_epi128_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_wo, const __grid_constant__ CUtensorMap tm_wg,
                     const __grid_constant__ CUtensorMap tm_out, const EpiParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBarE);
  uint64_t* w_full = bars;            // the weights have landed
  uint64_t* w_ready = w_full + 1;     // ... and are scaled
  uint64_t* full = w_ready + 1;       // [2] a stage has landed
  uint64_t* s_free = full + 2;        // [2] ... and nothing reads or stores from it any more
  uint64_t* acc_full = s_free + 2;    // [2]
  uint64_t* acc_empty = acc_full + 2; // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemE);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = (prm.m + kRowsE - 1) / kRowsE;

  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    mbar_init(w_ready, 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&s_free[i], 2);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_wo);
    tma_prefetch_desc(&tm_wg);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // Row-block skipping (transition.py:29-38): 1 compute, 0 no row kept (the result is act, or zeros), -1 keep negative
  // throughout (left unwritten)
  const int8_t* cls = nullptr;
  if (prm.keep != nullptr) {
    int8_t* w = reinterpret_cast<int8_t*>(smem + kOffClsE);
    for (int i = warp;; i += kThreadsE / 32) {
      const int64_t tile = blockIdx.x + int64_t(i) * gridDim.x;
      if (tile >= ntiles) break;
      float top = -1.f;
      for (int j = lane; j < kRowsE; j += 32) {
        const int64_t r = tile * kRowsE + j;
        if (r < prm.m)
          top = fmaxf(top, prm.keep_dtype == CFK_F32 ? static_cast<const float*>(prm.keep)[r]
                                                     : __bfloat162float(static_cast<const __nv_bfloat16*>(prm.keep)[r]));
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
      mbar_arrive_expect_tx(w_full, 4 * kAtomE);
      for (int a = 0; a < 2; ++a) {
        tma_load_2d(smem + kOffWE + a * kAtomE, &tm_wo, w_full, a * 64, 0);
        tma_load_2d(smem + kOffWE + (2 + a) * kAtomE, &tm_wg, w_full, a * 64, 0);
      }
      bool ok = true;
      uint32_t ti = 0, seq = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        const int st = ti & 1;
        ok = mbar_wait_deadline(&s_free[st], ((ti >> 1) & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 1701); break; }
        uint8_t* base = smem + kOffStE + st * kStageE;
        const int r0 = int(tile * kRowsE);
        mbar_arrive_expect_tx(&full[st], kStageE);
        for (int a = 0; a < 2; ++a) {
          tma_load_2d(base + a * kAtomE, &tm_x, &full[st], r0 + a * 64, 0);        // [128 channels][64 rows]
          tma_load_2d(base + (2 + a) * kAtomE, &tm_a, &full[st], a * 64, r0);      // [128 rows][64 channels]
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_x = make_idesc(kRowsE, kCe, 1, 1, 1, 1);   // A = x_cm tile MN-major, B = wo' MN-major
      constexpr uint32_t idesc_g = make_idesc(kRowsE, kCe, 1, 1, 0, 1);   // A = act tile K-major, B = wg' MN-major
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      const uint32_t wo = desc_lo(smem_u32(smem + kOffWE), kAtomE), wg = desc_lo(smem_u32(smem + kOffWE + 2 * kAtomE), kAtomE);
      bool ok = mbar_wait_deadline(w_ready, 0);
      if (!ok) report_timeout(prm.status, 1702);
      uint32_t ti = 0, seq = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        const int st = ti & 1;
        ok = mbar_wait_deadline(&full[st], (ti >> 1) & 1);
        if (!ok) { report_timeout(prm.status, 1703); break; }
        ok = mbar_wait_deadline(&acc_empty[st], ((ti >> 1) & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 1704); break; }
        tc_fence_after();
        const uint32_t xa = desc_lo(smem_u32(smem + kOffStE + st * kStageE), kAtomE);
        const uint32_t aa = desc_lo(smem_u32(smem + kOffStE + st * kStageE + 2 * kAtomE), 16);
        const uint32_t d = tmem + st * 256;
#pragma unroll
        for (int kk = 0; kk < kCe / 16; ++kk) mma_f16_ss2(d, xa + kk * 128, hi, wo + kk * 128, hi, idesc_x, kk > 0);
#pragma unroll
        for (int kk = 0; kk < kCe / 16; ++kk)
          mma_f16_ss2(d + 128, aa + (kk / 4) * (kAtomE >> 4) + (kk % 4) * 2, hi, wg + kk * 128, hi, idesc_g, kk > 0);
        mma_commit(&acc_full[st]);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ workers
    const int grp = (warp - 4) >> 2, quad = warp & 3;
    const int trow = quad * 32 + lane;
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const int pt = (warp - 4) * 32 + lane;
    float2* redx = reinterpret_cast<float2*>(smem + kOffRedX);
    float2* reda = reinterpret_cast<float2*>(smem + kOffRedA);
    float4* cst = reinterpret_cast<float4*>(smem + kOffCst);
    bool ok = true;
#define CFK_EP_WAIT(bar, parity, code)                            \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    // ---- once: scale the weights' rows by the LayerNorm scales and take the column constants
    CFK_EP_WAIT(w_full, 0, 1705)
    {
      const int which = pt >> 7, f = pt & 127;   // 0: output path (wo, centre LayerNorm), 1: gate path (wg, input LayerNorm)
      const float* sc = which ? prm.in_scale : prm.ln_scale;
      const float* of = which ? prm.in_offset : prm.ln_offset;
      uint8_t* wb = smem + kOffWE + which * 2 * kAtomE + (f >> 6) * kAtomE;
      float s = 0.f, t = 0.f;
      for (int k = 0; k < kCe; ++k) {
        __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(wb + k * 128 + ((((f & 63) >> 3) ^ (k & 7)) << 4) + (f & 7) * 2);
        const float w = __bfloat162float(*e);
        const float g = sc != nullptr ? sc[k] : 1.f, o = of != nullptr ? of[k] : 0.f;
        const __nv_bfloat16 ws = __float2bfloat16_rn(g * w);
        *e = ws;
        s += __bfloat162float(ws);
        t = fmaf(o, w, t);
      }
      t += __bfloat162float(which ? prm.bg[f] : prm.bo[f]);
      float* c = reinterpret_cast<float*>(&cst[f]);
      c[which * 2] = s;
      c[which * 2 + 1] = t;
    }
    fence_proxy_async();
    named_bar_sync(2, 256);
    if (lane == 0) mbar_arrive(w_ready);

    uint32_t ti = 0, seq = 0;
    int prev_st = -1;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++seq) {
      if (cls != nullptr && cls[seq] != 1) {
        if (cls[seq] == 0) {  // no row kept: the input rows (or zeros) in 16-byte pieces, straight from these threads
          for (int idx = pt; idx < kRowsE * (kCe / 8); idx += 256) {
            const int64_t r = tile * kRowsE + idx / (kCe / 8);
            if (r < prm.m) {
              const int64_t off = r * kCe + (idx % (kCe / 8)) * 8;
              uint4 v = make_uint4(0, 0, 0, 0);
              if (prm.add_input) v = *reinterpret_cast<const uint4*>(prm.act + off);
              *reinterpret_cast<uint4*>(prm.out + off) = v;
            }
          }
        }
        continue;
      }
      const int st = ti & 1;
      uint8_t* xs = smem + kOffStE + st * kStageE;          // x_cm tile, later the result
      const uint8_t* as = xs + 2 * kAtomE;                  // act tile
      CFK_EP_WAIT(&full[st], (ti >> 1) & 1, 1706)
      // ---- partial statistics.  x_cm: thread (row pair, channel quarter) reads two adjacent rows of 32 channels;
      // act: thread (row, half) reads 64 channels of its row as 16-byte pieces
      {
        const int rp = pt & 63, cq = pt >> 6, r = 2 * rp;
        const uint8_t* base = xs + (r >> 6) * kAtomE + (r & 7) * 2;
        float s0 = 0.f, s1 = 0.f, q0 = 0.f, q1 = 0.f;
#pragma unroll 8
        for (int i = 0; i < 32; ++i) {
          const int c = cq * 32 + i;
          const uint32_t w = *reinterpret_cast<const uint32_t*>(base + c * 128 + ((((r & 63) >> 3) ^ (c & 7)) << 4));
          const float a = bf16lo_to_f32(w), b = bf16hi_to_f32(w);
          s0 += a; s1 += b;
          q0 = fmaf(a, a, q0); q1 = fmaf(b, b, q1);
        }
        redx[cq * 128 + r] = make_float2(s0, q0);
        redx[cq * 128 + r + 1] = make_float2(s1, q1);
      }
      if (prm.in_scale != nullptr) {
        float s = 0.f, q = 0.f;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const uint4 w = *reinterpret_cast<const uint4*>(as + grp * kAtomE + swz_off(trow, p, 128));
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float a = bf16lo_to_f32(ww[e]), b = bf16hi_to_f32(ww[e]);
            s += a + b;
            q = fmaf(a, a, fmaf(b, b, q));
          }
        }
        reda[grp * 128 + trow] = make_float2(s, q);
      }
      named_bar_sync(2, 256);
      if (trow == 0 && prev_st >= 0) {  // this group's store of the tile before has read its atom: hand the stage back
        tma_wait_group_read<0>();
        mbar_arrive(&s_free[prev_st]);
      }
      float mean_x, rstd_x, mean_a = 0.f, rstd_a = 1.f;
      {
        const float2 a = redx[trow], b = redx[128 + trow], c = redx[256 + trow], d = redx[384 + trow];
        mean_x = ((a.x + b.x) + (c.x + d.x)) * (1.0f / kCe);
        const float var = fmaxf(((a.y + b.y) + (c.y + d.y)) * (1.0f / kCe) - mean_x * mean_x, 0.f);
        rstd_x = rsqrtf(var + prm.eps);
      }
      if (prm.in_scale != nullptr) {
        const float2 a = reda[trow], b = reda[128 + trow];
        mean_a = (a.x + b.x) * (1.0f / kCe);
        const float var = fmaxf((a.y + b.y) * (1.0f / kCe) - mean_a * mean_a, 0.f);
        rstd_a = rsqrtf(var + prm.eps);
      }
      named_bar_sync(2, 256);  // every partial has been read: the next tile may overwrite them
      // ---- epilogue: this group's 64 columns
      CFK_EP_WAIT(&acc_full[st], (ti >> 1) & 1, 1707)
      tc_fence_after();
#pragma unroll 1
      for (int hb = 0; hb < 2; ++hb) {
        uint32_t rx[32], rg[32];
        tmem_ld_x32(tmem + lane_addr + st * 256 + grp * 64 + hb * 32, rx);
        tmem_ld_x32(tmem + lane_addr + st * 256 + 128 + grp * 64 + hb * 32, rg);
        tmem_wait_ld();
        if (hb == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[st]);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int piece = hb * 4 + q;   // 16-byte piece of this group's 64 columns
          uint4 raw = make_uint4(0, 0, 0, 0);
          if (prm.add_input) raw = *reinterpret_cast<const uint4*>(as + grp * kAtomE + swz_off(trow, piece, 128));
          const uint32_t rr[4] = {raw.x, raw.y, raw.z, raw.w};
          uint32_t y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = q * 8 + 2 * e, f = grp * 64 + hb * 32 + j;
            const float4 c0 = cst[f], c1 = cst[f + 1];
            const float x0 = fmaf(rstd_x, fmaf(-mean_x, c0.x, __uint_as_float(rx[j])), c0.y);
            const float x1 = fmaf(rstd_x, fmaf(-mean_x, c1.x, __uint_as_float(rx[j + 1])), c1.y);
            const float g0 = fmaf(rstd_a, fmaf(-mean_a, c0.z, __uint_as_float(rg[j])), c0.w);
            const float g1 = fmaf(rstd_a, fmaf(-mean_a, c1.z, __uint_as_float(rg[j + 1])), c1.w);
            y[e] = pack_bf16x2(fmaf(x0, sigmoid_fast(g0), bf16lo_to_f32(rr[e])), fmaf(x1, sigmoid_fast(g1), bf16hi_to_f32(rr[e])));
          }
          // over the dead x_cm tile: atom = this group's 64 columns, row = this thread's
          *reinterpret_cast<uint4*>(xs + grp * kAtomE + swz_off(trow, piece, 128)) = make_uint4(y[0], y[1], y[2], y[3]);
        }
      }
      fence_proxy_async();
      named_bar_sync(3 + grp, 128);
      if (trow == 0) {  // one thread per group stores the group's atom; it hands the stage back at the next tile
        if (ok) tma_store_2d(&tm_out, xs + grp * kAtomE, grp * 64, int(tile * kRowsE));
        tma_commit_group();
      }
      prev_st = st;
      ++ti;
    }
    if (trow == 0) {
      if (prev_st >= 0) {
        tma_wait_group_read<0>();
        mbar_arrive(&s_free[prev_st]);
      }
      tma_wait_group<0>();
    }
#undef CFK_EP_WAIT
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// Returns CFK_ERR_UNSUPPORTED for what the general engine should take instead.
int trimul_epi128_launch(const void* x_cm, const void* act, const float* in_scale, const float* in_offset, const float* ln_scale,
                         const float* ln_offset, const void* wo, const void* bo, const void* wg, const void* bg, void* out,
                         const void* keep, int keep_dtype, int64_t m, float eps, int add_input, cudaStream_t st) {
  if (m % 8 != 0 || m > INT32_MAX) return CFK_ERR_UNSUPPORTED;
  if (!aligned16(x_cm) || !aligned16(act) || !aligned16(wo) || !aligned16(wg) || !aligned16(out)) return CFK_ERR_UNSUPPORTED;
  EpiParams prm{ln_scale, ln_offset, in_scale, in_offset, static_cast<const __nv_bfloat16*>(bo),
                static_cast<const __nv_bfloat16*>(bg), m, eps, add_input, keep, keep_dtype,
                static_cast<const __nv_bfloat16*>(act), static_cast<__nv_bfloat16*>(out), device_status_word()};
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  CUtensorMap tx, ta, two, twg, to;
  {
    uint64_t dims[2] = {uint64_t(m), uint64_t(kCe)};
    uint64_t str[1] = {uint64_t(m) * 2};
    uint32_t box[2] = {64, kCe};
    int rc = make_tensor_map(&tx, x_cm, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  for (int i = 0; i < 2; ++i) {
    uint64_t dims[2] = {uint64_t(kCe), uint64_t(m)};
    uint64_t str[1] = {uint64_t(kCe) * 2};
    uint32_t box[2] = {64, kRowsE};
    int rc = make_tensor_map(i ? &to : &ta, i ? out : act, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  for (int i = 0; i < 2; ++i) {
    uint64_t dims[2] = {uint64_t(kCe), uint64_t(kCe)};
    uint64_t str[1] = {uint64_t(kCe) * 2};
    uint32_t box[2] = {64, kCe};
    int rc = make_tensor_map(i ? &twg : &two, i ? wg : wo, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  if (cudaFuncSetAttribute(trimul_epi128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemE) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ntiles = (m + kRowsE - 1) / kRowsE;
  const int grid = int(ntiles < sms ? ntiles : sms);
  if (keep != nullptr && (ntiles + grid - 1) / grid > kMaxTilesE) return CFK_ERR_UNSUPPORTED;
  trimul_epi128_kernel<<<grid, kThreadsE, kSmemE, st>>>(tx, ta, two, twg, to, prm);
  return check_launch();
}

}  // namespace cfk
