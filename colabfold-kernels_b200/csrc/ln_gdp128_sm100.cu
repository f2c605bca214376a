// LayerNorm -> gated dual projection of the pair representation at 128 channels, channel-major bf16 outputs
// (tri_mul.py:222-300: left, right = mask * (LN(x) wp + bp) * sigmoid(LN(x) wg + bg), split in halves, each [128, ., .']).
//
// The general row-GEMM engine computes D[row][channel] and turns it channel-major through 2-byte shared-memory stores
// with the bias, the gate and the mask applied per element from per-column vectors; it runs this op at a quarter of the
// copy bandwidth.  Here the GEMM is issued transposed, D^T[channel][row] = W^T LN(x)^T: the weights in their natural
// [K, N] layout are the MN-major A operand (M = 128 output channels), the normalised row tile [128 rows][128] is the
// K-major B operand (N = 128 rows).  A TMEM lane is then an output channel: its biases are two scalars per thread, the
// 128 rows of the tile are contiguous along the thread's columns, and a thread writes its channel's rows as 16-byte
// pieces of a swizzled [channel][64 rows] staging atom that one TMA store moves to the channel-major output.
//
// A persistent CTA walks 128-row tiles (rows along the pair's inner axis, or along its outer axis for the transposed
// read of incoming edges).  Warp 0: TMA producer (the four 128 x 128 weight blocks once, then double-buffered row tiles).
// Warp 1: MMA issuer: per tile the left pair (projection, gate) into TMEM columns [0, 256) and the right pair into
// [256, 512), 8 + 8 MMAs of N = 128 each.  Warps 4-11: LayerNorm in place (two lanes per row, fp32 statistics, bf16 out),
// one tile ahead of the epilogue; epilogue thread = channel, group = 64-row half.  Tiles follow the mask as the engine's do:
// a tile whose mask is zero throughout is written as zeros without being read, one that is negative throughout is
// left unwritten (transition.py:29-38).  Every mbarrier wait is deadline-bounded.
#include "attention_sm100.cuh"
#include "rowgemm_sm100.cuh"

namespace cfk {
namespace {

constexpr int kKc = 128;                  // input channels
constexpr int kRowsG = 128;
constexpr int kThreadsG = 384;
constexpr int kMaxTilesG = 512;
constexpr int kWBlock = kKc * 128 * 2;    // one 128 x 128 weight block: two atoms of [128 k][64 channels]
constexpr int kTileXG = kRowsG * kKc * 2; // two atoms of [128 rows][64 k]
constexpr int kStageG = 128 * 128;        // staging atom: [128 channels][64 rows]
constexpr int kOffWG = 0;
constexpr int kOffXG = kOffWG + 4 * kWBlock;
constexpr int kOffOG = kOffXG + 2 * kTileXG;
constexpr int kOffMaskG = kOffOG + 2 * kStageG;          // float [2][128]: the tile's row mask (0 for rows past the end)
constexpr int kOffBarG = kOffMaskG + 2 * kRowsG * 4;
constexpr int kNumBarsG = 6 + 1 + 4;
constexpr int kOffTmemG = kOffBarG + kNumBarsG * 8;
constexpr int kOffClsG = kOffTmemG + 16;
constexpr int kSmemG = kOffClsG + kMaxTilesG + 1024;
static_assert(kSmemG <= 232448, "shared memory budget");

struct GdpParams {
  const float* ln_scale;
  const float* ln_offset;
  const __nv_bfloat16* bp;    // [256]
  const __nv_bfloat16* bg;    // [256]
  const __nv_bfloat16* mask;  // indexed by source row
  int64_t outer, inner, inner_pad, stride_outer, stride_inner;  // strides in rows of x
  int64_t ntiles, tiles_per_outer;
  float eps;
  int* status;
};

__global__ void __launch_bounds__(kThreadsG, 1)
ln_gdp128_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_wp,
                 const __grid_constant__ CUtensorMap tm_wg, const __grid_constant__ CUtensorMap tm_l,
                 const __grid_constant__ CUtensorMap tm_r, const GdpParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBarG);
  uint64_t* x_full = bars;            // [2] the tile has landed
  uint64_t* x_ready = x_full + 2;     // [2] ... and is normalised
  uint64_t* x_free = x_ready + 2;     // [2] every MMA of the tile has completed
  uint64_t* w_full = x_free + 2;      // the weights are resident
  uint64_t* acc_full = w_full + 1;    // [2] left pair, right pair
  uint64_t* acc_empty = acc_full + 2; // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemG);
  float* maskf = reinterpret_cast<float*>(smem + kOffMaskG);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = prm.ntiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_ready[i], 8);
      mbar_init(&x_free[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    mbar_init(w_full, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_wp);
    tma_prefetch_desc(&tm_wg);
    tma_prefetch_desc(&tm_l);
    tma_prefetch_desc(&tm_r);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // tile classes from the mask: 1 compute, 0 zero throughout (or all padding rows), -1 negative throughout
  int8_t* cls = reinterpret_cast<int8_t*>(smem + kOffClsG);
  for (int i = warp;; i += kThreadsG / 32) {
    const int64_t tile = blockIdx.x + int64_t(i) * gridDim.x;
    if (tile >= ntiles) break;
    const int64_t o = tile / prm.tiles_per_outer;
    const int64_t r0 = (tile % prm.tiles_per_outer) * kRowsG;
    float top = -1.f;
    for (int j = lane; j < kRowsG; j += 32) {
      const int64_t r = r0 + j;
      float v = -1.f;
      if (r < prm.inner) v = __bfloat162float(prm.mask[o * prm.stride_outer + r * prm.stride_inner]);
      else if (r < prm.inner_pad) v = 0.f;
      top = fmaxf(top, v);
    }
    for (int off = 16; off > 0; off >>= 1) top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, off));
    if (lane == 0) cls[i] = top > 0.f ? 1 : (top == 0.f ? 0 : -1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto next_computed = [&](uint32_t& seq) -> int64_t {
    for (;; ++seq) {
      const int64_t tile = blockIdx.x + int64_t(seq) * gridDim.x;
      if (tile >= ntiles) return -1;
      if (cls[seq] == 1) return tile;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // weight blocks in the order the issuer uses them: projection left, gate left, projection right, gate right
      mbar_arrive_expect_tx(w_full, 4 * kWBlock);
      for (int blk = 0; blk < 4; ++blk)
        for (int a = 0; a < 2; ++a)
          tma_load_2d(smem + kOffWG + blk * kWBlock + a * (kWBlock / 2), (blk & 1) ? &tm_wg : &tm_wp, w_full,
                      (blk >> 1) * 128 + a * 64, 0);
      bool ok = true;
      uint32_t seq = 0, ti = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        const int xb = ti & 1;
        ok = mbar_wait_deadline(&x_free[xb], ((ti >> 1) & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 1601); break; }
        const int o = int(tile / prm.tiles_per_outer), r0 = int(tile % prm.tiles_per_outer) * kRowsG;
        mbar_arrive_expect_tx(&x_full[xb], kTileXG);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(smem + kOffXG + xb * kTileXG + a * (kTileXG / 2), &tm_x, &x_full[xb], a * 64, r0, o);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer: D^T[channel][row] = W^T LN(x)^T
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(128, kRowsG, 1, 1, 1, 0);   // A = weights MN-major, B = rows K-major
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      bool ok = mbar_wait_deadline(w_full, 0);
      if (!ok) report_timeout(prm.status, 1602);
      uint32_t seq = 0, ti = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        const int xb = ti & 1;
        ok = mbar_wait_deadline(&x_ready[xb], (ti >> 1) & 1);
        if (!ok) { report_timeout(prm.status, 1603); break; }
        const uint32_t xk = desc_lo(smem_u32(smem + kOffXG + xb * kTileXG), 16);
        for (int set = 0; set < 2 && ok; ++set) {
          ok = mbar_wait_deadline(&acc_empty[set], (ti & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 1604); break; }
          tc_fence_after();
          for (int part = 0; part < 2; ++part) {   // projection, gate
            const uint32_t wa = desc_lo(smem_u32(smem + kOffWG + (set * 2 + part) * kWBlock), kWBlock / 2);
            const uint32_t d = tmem + set * 256 + part * 128;
#pragma unroll
            for (int kk = 0; kk < kKc / 16; ++kk)
              mma_f16_ss2(d, wa + kk * 128, hi, xk + (kk / 4) * ((kTileXG / 2) >> 4) + (kk % 4) * 2, hi, idesc, kk > 0);
          }
          mma_commit(&acc_full[set]);
        }
        if (ok) mma_commit(&x_free[xb]);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ workers
    const int grp = (warp - 4) >> 2, quad = warp & 3;
    const int ch = quad * 32 + lane;                          // epilogue: thread = output channel, group = 64-row half
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const int pt = (warp - 4) * 32 + lane;                    // LayerNorm: two adjacent lanes share a row
    const int lrow = pt >> 1, half = pt & 1;
    uint8_t* stage = smem + kOffOG + grp * kStageG;
    bool ok = true;
#define CFK_GD_WAIT(bar, parity, code)                            \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    // this thread's biases: projection and gate of the left and of the right half
    const float bpl = __bfloat162float(prm.bp[ch]), bpr = __bfloat162float(prm.bp[128 + ch]);
    const float bgl = __bfloat162float(prm.bg[ch]), bgr = __bfloat162float(prm.bg[128 + ch]);
    // LayerNorm of local tile index u (tile number `tile`) into its buffer, and the tile's row mask
    auto layer_norm = [&](uint32_t u, int64_t tile) {
      const int xb = u & 1;
      uint8_t* xt = smem + kOffXG + xb * kTileXG;
      const int64_t o = tile / prm.tiles_per_outer;
      const int64_t r = (tile % prm.tiles_per_outer) * kRowsG + lrow;
      CFK_GD_WAIT(&x_full[xb], (u >> 1) & 1, 1605)
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < kKc / 16; ++j) {
        const int c = 2 * j + half;
        const uint4 w = *reinterpret_cast<const uint4*>(xt + (c / 8) * (kTileXG / 2) + swz_off(lrow, c % 8, 128));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) ps += bf16lo_to_f32(ww[e]) + bf16hi_to_f32(ww[e]);
      }
      const float mean = (ps + __shfl_xor_sync(0xffffffffu, ps, 1)) * (1.0f / kKc);
      float pv = 0.f;
#pragma unroll
      for (int j = 0; j < kKc / 16; ++j) {
        const int c = 2 * j + half;
        const uint4 w = *reinterpret_cast<const uint4*>(xt + (c / 8) * (kTileXG / 2) + swz_off(lrow, c % 8, 128));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = bf16lo_to_f32(ww[e]) - mean, b = bf16hi_to_f32(ww[e]) - mean;
          pv = fmaf(a, a, fmaf(b, b, pv));
        }
      }
      const float rstd = rsqrtf((pv + __shfl_xor_sync(0xffffffffu, pv, 1)) * (1.0f / kKc) + prm.eps);
#pragma unroll 2
      for (int j = 0; j < kKc / 16; ++j) {
        const int c = 2 * j + half;
        uint4* ptr = reinterpret_cast<uint4*>(xt + (c / 8) * (kTileXG / 2) + swz_off(lrow, c % 8, 128));
        const uint4 w = *ptr;
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(prm.ln_scale + c * 8));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(prm.ln_scale + c * 8 + 4));
        const float4 o0 = __ldg(reinterpret_cast<const float4*>(prm.ln_offset + c * 8));
        const float4 o1 = __ldg(reinterpret_cast<const float4*>(prm.ln_offset + c * 8 + 4));
        const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float oo[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
        uint32_t y[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          y[e] = pack_bf16x2(fmaf((bf16lo_to_f32(ww[e]) - mean) * rstd, gg[2 * e], oo[2 * e]),
                             fmaf((bf16hi_to_f32(ww[e]) - mean) * rstd, gg[2 * e + 1], oo[2 * e + 1]));
        *ptr = make_uint4(y[0], y[1], y[2], y[3]);
      }
      if (half == 0) {
        float mk = 0.f;  // rows past the end (zero-filled by TMA, so their normalised value is the offset) count as masked
        if (r < prm.inner) mk = fmaxf(__bfloat162float(prm.mask[o * prm.stride_outer + r * prm.stride_inner]), 0.f);
        maskf[xb * kRowsG + lrow] = mk;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_ready[xb]);
    };

    uint32_t seq = 0, ti = 0;
    // the first computed tile is normalised before the loop, every later one during the iteration before its own
    {
      uint32_t s0 = 0;
      const int64_t first = next_computed(s0);
      if (first >= 0) layer_norm(0, first);
    }
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++seq) {
      const int o = int(tile / prm.tiles_per_outer), r0 = int(tile % prm.tiles_per_outer) * kRowsG;
      if (cls[seq] != 1) {
        if (cls[seq] == 0) {
          // zero throughout: both outputs get zeros for the tile's rows (up to the padded extent), from the staging atoms
          if (ch == 0) tma_wait_group_read<0>();
          named_bar_sync(3 + grp, 128);
#pragma unroll
          for (int q = 0; q < 8; ++q) *reinterpret_cast<uint4*>(stage + swz_off(ch, q, 128)) = make_uint4(0, 0, 0, 0);
          fence_proxy_async();
          named_bar_sync(3 + grp, 128);
          if (ch == 0) {
            if (r0 + grp * 64 < prm.inner_pad) {   // a store never starts past the padded extent
              tma_store_3d(&tm_l, stage, r0 + grp * 64, o, 0);
              tma_store_3d(&tm_r, stage, r0 + grp * 64, o, 0);
            }
            tma_commit_group();
          }
        }
        continue;
      }
      {
        uint32_t sn = seq + 1;
        const int64_t nxt = next_computed(sn);
        if (nxt >= 0) layer_norm(ti + 1, nxt);
      }
      // the row masks of this tile were written by other threads during its LayerNorm (an iteration ago)
      named_bar_sync(2, 256);
      const float* mk = maskf + (ti & 1) * kRowsG + grp * 64;
#pragma unroll 1
      for (int set = 0; set < 2; ++set) {
        const float b_p = set ? bpr : bpl, b_g = set ? bgr : bgl;
        const uint64_t half2 = f2_pack(0.5f, 0.5f), hbg = f2_pack(0.5f * b_g, 0.5f * b_g), bp2 = f2_pack(b_p, b_p);
        CFK_GD_WAIT(&acc_full[set], ti & 1, 1606)
        tc_fence_after();
        if (ch == 0) tma_wait_group_read<0>();   // the store this group issued last has read the staging atom
        named_bar_sync(3 + grp, 128);
#pragma unroll 1
        for (int hb = 0; hb < 2; ++hb) {           // 32 rows at a time
          uint32_t rp[32], rg[32];
          tmem_ld_x32(tmem + lane_addr + set * 256 + grp * 64 + hb * 32, rp);
          tmem_ld_x32(tmem + lane_addr + set * 256 + 128 + grp * 64 + hb * 32, rg);
          tmem_wait_ld();
          if (hb == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[set]);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t y[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // two rows at a time in packed fp32: sigmoid(g + bg) = 0.5 tanh(0.5 (g + bg)) + 0.5, then mask (p + bp) sigmoid
              const int j = q * 8 + 2 * e;
              const uint64_t t = f2_fma(f2_pack(__uint_as_float(rg[j]), __uint_as_float(rg[j + 1])), half2, hbg);
              float t0, t1;
              f2_unpack(t, t0, t1);
              const uint64_t sg = f2_fma(f2_pack(tanh_approx(t0), tanh_approx(t1)), half2, half2);
              const uint64_t u = f2_add(f2_pack(__uint_as_float(rp[j]), __uint_as_float(rp[j + 1])), bp2);
              const uint64_t m2 = *reinterpret_cast<const uint64_t*>(mk + hb * 32 + j);
              float v0, v1;
              f2_unpack(f2_mul(f2_mul(m2, u), sg), v0, v1);
              y[e] = pack_bf16x2(v0, v1);
            }
            *reinterpret_cast<uint4*>(stage + swz_off(ch, hb * 4 + q, 128)) = make_uint4(y[0], y[1], y[2], y[3]);
          }
        }
        fence_proxy_async();
        named_bar_sync(3 + grp, 128);
        if (ch == 0) {
          if (ok && r0 + grp * 64 < prm.inner_pad) tma_store_3d(set ? &tm_r : &tm_l, stage, r0 + grp * 64, o, 0);
          tma_commit_group();
        }
      }
      ++ti;
    }
    if (ch == 0) tma_wait_group<0>();
#undef CFK_GD_WAIT
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// x [outer, inner, 128] read with the given row strides, wp / wg [128, 256], left / right [128, outer, inner_pad] bf16.
// Returns CFK_ERR_UNSUPPORTED for what the general engine should take instead.
int ln_gdp128_launch(const void* x, const float* ln_scale, const float* ln_offset, const void* wp, const void* bp,
                     const void* wg, const void* bg, const void* mask, void* left, void* right, int64_t outer, int64_t inner,
                     int64_t inner_pad, int64_t stride_outer, int64_t stride_inner, float eps, cudaStream_t st) {
  if ((inner_pad * 2) % 16 != 0 || outer > INT32_MAX || inner_pad > INT32_MAX) return CFK_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(wp) || !aligned16(wg) || !aligned16(left) || !aligned16(right) || !aligned16(ln_scale) ||
      !aligned16(ln_offset))
    return CFK_ERR_UNSUPPORTED;
  GdpParams prm{};
  prm.ln_scale = ln_scale; prm.ln_offset = ln_offset;
  prm.bp = static_cast<const __nv_bfloat16*>(bp); prm.bg = static_cast<const __nv_bfloat16*>(bg);
  prm.mask = static_cast<const __nv_bfloat16*>(mask);
  prm.outer = outer; prm.inner = inner; prm.inner_pad = inner_pad;
  prm.stride_outer = stride_outer; prm.stride_inner = stride_inner;
  prm.tiles_per_outer = (inner_pad + kRowsG - 1) / kRowsG;
  prm.ntiles = outer * prm.tiles_per_outer;
  prm.eps = eps;
  prm.status = device_status_word();
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  if (prm.ntiles == 0) return CFK_OK;
  CUtensorMap tx, twp, twg, tl, tr;
  {
    const uint64_t row = uint64_t(kKc) * 2;
    uint64_t dims[3] = {uint64_t(kKc), uint64_t(inner), uint64_t(outer)};
    uint64_t str[2] = {uint64_t(stride_inner) * row, (outer > 1 ? uint64_t(stride_outer) : uint64_t(inner) * uint64_t(stride_inner)) * row};
    uint32_t box[3] = {64, kRowsG, 1};
    int rc = make_tensor_map(&tx, x, CFK_BF16, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  for (int i = 0; i < 2; ++i) {
    uint64_t dims[2] = {256, uint64_t(kKc)};
    uint64_t str[1] = {256 * 2};
    uint32_t box[2] = {64, kKc};
    int rc = make_tensor_map(i ? &twg : &twp, i ? wg : wp, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  for (int i = 0; i < 2; ++i) {
    uint64_t dims[3] = {uint64_t(inner_pad), uint64_t(outer), 128};
    uint64_t str[2] = {uint64_t(inner_pad) * 2, uint64_t(outer) * uint64_t(inner_pad) * 2};
    uint32_t box[3] = {64, 1, 128};
    int rc = make_tensor_map(i ? &tr : &tl, i ? right : left, CFK_BF16, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  if (cudaFuncSetAttribute(ln_gdp128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemG) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = int(prm.ntiles < sms ? prm.ntiles : sms);
  if ((prm.ntiles + grid - 1) / grid > kMaxTilesG) return CFK_ERR_UNSUPPORTED;
  ln_gdp128_kernel<<<grid, kThreadsG, kSmemG, st>>>(tx, twp, twg, tl, tr, prm);
  return check_launch();
}

}  // namespace cfk
