// Fused LayerNorm -> Linear -> relu -> Linear (+ x) transition for sm_100a: both GEMMs on tcgen05 with the hidden
// activation kept on chip (src/colabfold_kernels/transition.py:68-92,102-138 streams the hidden layer in chunks through
// registers; here a chunk goes TMEM -> registers -> shared memory and is the A operand of the second GEMM).
//
// A persistent CTA walks 128-row tiles of x [M, C].  Per tile:
//   producer (warp 0)    TMA: the x tile as 64-column K-major atoms; per hidden chunk of HC columns (128 at 128
//                        channels, 64 at 256) the weights w1[:, chunk] ([C][HC], MN-major B) and w2[chunk, :]
//                        ([HC][C], MN-major B) into two rings
//   workers (warps 4-11) LayerNorm of the landed tile in place (thread = row, fp32 statistics, bf16 out: the reference
//                        rounds the normed tile before the dot, transition.py:76-80); per chunk: acc1 -> + b1 -> relu
//                        -> bf16 -> H tile in shared memory; per tile: acc2 + b2 (+ x) -> out
//   issuers (warps 1, 2) per chunk n: acc1[n & 1] = LN(x) w1[:, n]  (C / 16 MMAs of N = HC) from warp 1 and
//                        acc2 += H[n] w2[n, :]  (HC / 16 MMAs of N = C) from warp 2
// TMEM columns: acc1 [0, HC) and [HC, 2 HC), acc2 [2 HC, 2 HC + C).
// Every mbarrier wait is deadline-bounded and reports into the status word instead of hanging.
#include "attention_sm100.cuh"

namespace cfk {
namespace {

constexpr int kRowsT = 128;   // rows per tile = TMEM lanes
constexpr int kMaxTilesT = 768;   // tiles per CTA when row blocks may be skipped
constexpr int kThreadsT = 384;   // warps 0-3 control, 4-7 and 8-11 two worker groups

template <int C>
struct TrCfg {
  static constexpr int kAtoms = C / 64;                  // 64-column atoms of an x tile / of a w2 chunk
  static constexpr int kTileX = kRowsT * C * 2;          // x tile
  // hidden columns per chunk: an N = 64 MMA costs its issue floor, not its tensor time, so 128 wherever the shared
  // memory allows it (at 256 channels the x tile and the weight chunks leave no room)
  static constexpr int kHC = C == 128 ? 128 : 64;
  static constexpr int kGroupsPerChunk = kHC / 64;       // worker groups that share one chunk's epilogue
  static constexpr int kW1 = C * kHC * 2;                // w1 chunk: kHC / 64 atoms of [C rows][64 columns]
  static constexpr int kW2 = kHC * C * 2;                // w2 chunk: kAtoms atoms of [kHC rows][64 columns]
  static constexpr int kH = kRowsT * kHC * 2;            // H tile: kHC / 64 atoms of [128 rows][64 columns]
  static constexpr int kWRing = 2;                       // ring depth of each weight ring
  // H buffers: one per worker group when the groups take chunks in turn; one when both work on every chunk (the second
  // GEMM of a chunk has long completed when the next chunk's activations are ready to be written)
  static constexpr int kHBufs = kGroupsPerChunk == 2 ? 1 : 2;
  static constexpr int kXBufs = C == 128 ? 2 : 1;        // x tiles in flight
  static constexpr int kOffX = 0;
  static constexpr int kOffW1 = kOffX + kXBufs * kTileX;
  static constexpr int kOffW2 = kOffW1 + kWRing * kW1;
  static constexpr int kOffH = kOffW2 + kWRing * kW2;
  static constexpr int kOffBar = kOffH + kHBufs * kH;
  static constexpr int kNumBars = 6 + 4 * kWRing + 4 + 4 + 2 + 2;
  static constexpr int kOffTmem = kOffBar + kNumBars * 8;
  static constexpr int kOffCls = kOffTmem + 16;           // int8 [kMaxTilesT]: class of each tile this CTA visits
  static constexpr int kSmem = kOffCls + kMaxTilesT + 1024;
  static constexpr int kColAcc2 = 2 * kHC;
  static_assert(kSmem <= 232448, "shared memory budget");
  static_assert(kOffW1 % 1024 == 0 && kOffW2 % 1024 == 0 && kOffH % 1024 == 0, "swizzled tiles start on their atom");
};

struct TrParams {
  const __nv_bfloat16* x;
  const float* ln_scale;
  const float* ln_offset;
  const __nv_bfloat16* b1;   // [hdim]
  const __nv_bfloat16* b2;   // [C]
  __nv_bfloat16* out;        // [M, C]
  int64_t m;
  int hdim;
  float eps;
  int add_input;
  const void* keep;            // [M] rows that matter (or null): 128-row blocks it marks nowhere are not computed
  int keep_dtype;
  int* status;
};

template <int C>
__global__ void __launch_bounds__(kThreadsT, 1)
transition_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w1,
                  const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_out,
                  const TrParams prm) {
  using T = TrCfg<C>;
  constexpr int WR = T::kWRing, HB = T::kHBufs, XB = T::kXBufs, kHC = T::kHC, GPC = T::kGroupsPerChunk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + T::kOffBar);
  uint64_t* x_full = bars;             // [2] the x tile has landed
  uint64_t* x_ready = x_full + 2;      // [2] ... and is normalised (a valid A operand)
  uint64_t* x_free = x_ready + 2;      // [2] the tile's result has been read out of the buffer by the TMA store
  uint64_t* w1_full = x_free + 2;      // [WR]
  uint64_t* w1_empty = w1_full + WR;   // [WR]
  uint64_t* w2_full = w1_empty + WR;   // [WR]
  uint64_t* w2_empty = w2_full + WR;   // [WR]
  uint64_t* acc1_full = w2_empty + WR; // [2]
  uint64_t* acc1_empty = acc1_full + 2;// [2]
  uint64_t* h_full = acc1_empty + 2;   // [2] (HB used)
  uint64_t* h_empty = h_full + 2;      // [2]
  uint64_t* acc2_full = h_empty + 2;   // every MMA of the tile has completed (the x tile is free as well)
  uint64_t* acc2_empty = acc2_full + 1;
  uint64_t* x_dead = acc2_empty + 1;   // the tile's first GEMMs have completed: the normalised tile is no longer read
  uint64_t* xraw_full = x_dead + 1;    // the raw rows of the tile have landed again (for the residual)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + T::kOffTmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = (prm.m + kRowsT - 1) / kRowsT;
  const int nchunks = prm.hdim / kHC;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_ready[i], 8);
      mbar_init(&x_free[i], 1);
    }
    for (int i = 0; i < WR; ++i) {
      mbar_init(&w1_full[i], 1);
      mbar_init(&w1_empty[i], 1);
      mbar_init(&w2_full[i], 1);
      mbar_init(&w2_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc1_full[i], 1);
      mbar_init(&acc1_empty[i], 4 * GPC);
      mbar_init(&h_full[i], 4 * GPC);
      mbar_init(&h_empty[i], 1);
    }
    mbar_init(acc2_full, 1);
    mbar_init(acc2_empty, 1);
    mbar_init(x_dead, 1);
    mbar_init(xraw_full, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w1);
    tma_prefetch_desc(&tm_w2);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // Row-block skipping (transition.py:29-38): the class of every tile this CTA will visit - 1 compute, 0 no row kept
  // (the result is x, or zeros without the residual), -1 keep negative throughout (left unwritten) - worked out once
  // by all warps so that every role takes the same decision.
  const int8_t* cls = nullptr;
  if (prm.keep != nullptr) {
    int8_t* w = reinterpret_cast<int8_t*>(smem + T::kOffCls);
    for (int i = warp;; i += kThreadsT / 32) {
      const int64_t tile = blockIdx.x + int64_t(i) * gridDim.x;
      if (tile >= ntiles) break;
      float top = -1.f;
      for (int j = lane; j < kRowsT; j += 32) {
        const int64_t r = tile * kRowsT + j;
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
  // the next tile this CTA computes at or after its local index seq (-1: none); seq is left on it
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
      uint32_t ti = 0, cc = 0;
      // the x tile of local tile index u into its buffer, once the result of the tile that used the buffer before
      // has been stored out of it
      auto load_x = [&](uint32_t u, int64_t tile) {
        const int xb = u % XB;
        if (!mbar_wait_deadline(&x_free[xb], ((u / XB) & 1) ^ 1)) { report_timeout(prm.status, 1101); return false; }
        mbar_arrive_expect_tx(&x_full[xb], T::kTileX);
#pragma unroll
        for (int a = 0; a < T::kAtoms; ++a)
          tma_load_2d(smem + T::kOffX + xb * T::kTileX + a * (kRowsT * 128), &tm_x, &x_full[xb], a * 64, int(tile * kRowsT));
        return true;
      };
      uint32_t seq = 0;
      int64_t tile = next_computed(seq);
      if (tile >= 0) ok = load_x(0, tile);
      for (; tile >= 0 && ok; ++ti) {
        const int xb = ti % XB;
        uint32_t seq_next = seq + 1;
        const int64_t next = next_computed(seq_next);
        for (int n = 0; n < nchunks && ok; ++n, ++cc) {
          const int slot = cc % WR;
          const uint32_t par = ((cc / WR) & 1) ^ 1;
          ok = mbar_wait_deadline(&w1_empty[slot], par);
          if (!ok) { report_timeout(prm.status, 1102); break; }
          mbar_arrive_expect_tx(&w1_full[slot], T::kW1);
#pragma unroll
          for (int a = 0; a < kHC / 64; ++a)
            tma_load_2d(smem + T::kOffW1 + slot * T::kW1 + a * (C * 128), &tm_w1, &w1_full[slot], n * kHC + a * 64, 0);
          ok = mbar_wait_deadline(&w2_empty[slot], par);
          if (!ok) { report_timeout(prm.status, 1103); break; }
          mbar_arrive_expect_tx(&w2_full[slot], T::kW2);
#pragma unroll
          for (int a = 0; a < T::kAtoms; ++a)
            tma_load_2d(smem + T::kOffW2 + slot * T::kW2 + a * (kHC * 128), &tm_w2, &w2_full[slot], a * 64, n * kHC);
          // with two buffers the next tile's rows land under this tile's GEMMs
          if (XB == 2 && n == nchunks / 2 && next >= 0) ok = load_x(ti + 1, next);
        }
        if (ok && prm.add_input) {
          // the raw rows again, over the normalised tile, for the residual: from L2, under the tile's last GEMMs
          ok = mbar_wait_deadline(x_dead, ti & 1);
          if (!ok) { report_timeout(prm.status, 1104); break; }
          mbar_arrive_expect_tx(xraw_full, T::kTileX);
#pragma unroll
          for (int a = 0; a < T::kAtoms; ++a)
            tma_load_2d(smem + T::kOffX + xb * T::kTileX + a * (kRowsT * 128), &tm_x, xraw_full, a * 64, int(tile * kRowsT));
        }
        if (XB == 1 && ok && next >= 0) ok = load_x(ti + 1, next);
        tile = next;
        seq = seq_next;
      }
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------------ MMA issuers: warp 1 the first GEMMs, warp 2 the
    // second (what bounds a chunk is the issuing thread's own chain of waits, MMAs and commits, so the two chains run
    // side by side; they share no accumulator)
    if (lane == 0) {
      constexpr uint32_t idesc1 = make_idesc(kRowsT, kHC, 1, 1, 0, 1);  // A = LN(x) K-major, B = w1 chunk MN-major
      constexpr uint32_t idesc2 = make_idesc(kRowsT, C, 1, 1, 0, 1);    // A = H K-major, B = w2 chunk MN-major
      constexpr uint32_t hi128 = desc_hi(1024, kSwz128);
      const uint32_t x_k = desc_lo(smem_u32(smem + T::kOffX), 16);
      const uint32_t w1_mn = desc_lo(smem_u32(smem + T::kOffW1), C * 128);     // atoms of 64 columns, C * 128 bytes apart
      const uint32_t w2_mn = desc_lo(smem_u32(smem + T::kOffW2), kHC * 128);   // atoms of 64 columns, kHC * 128 bytes apart
      const uint32_t h_k = desc_lo(smem_u32(smem + T::kOffH), 16);
      bool ok = true;
      uint32_t ti = 0, c1 = 0, c2 = 0;  // tiles done, chunks whose first / second GEMM has been issued
      auto gemm1 = [&](uint32_t xoff) {
        const int slot = c1 % WR, buf = c1 & 1;
        if (!mbar_wait_deadline(&w1_full[slot], (c1 / WR) & 1)) { report_timeout(prm.status, 1201); return false; }
        if (!mbar_wait_deadline(&acc1_empty[buf], ((c1 >> 1) & 1) ^ 1)) { report_timeout(prm.status, 1202); return false; }
        tc_fence_after();
        const uint32_t b = w1_mn + slot * (T::kW1 >> 4);
        // K step kk: 16 columns of the x tile (32 bytes into the row, the next atom 16 KB on) against 16 rows of the
        // weight chunk (2048 bytes on)
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk)
          mma_f16_ss2(tmem + buf * kHC, x_k + xoff + (kk / 4) * ((kRowsT * 128) >> 4) + (kk % 4) * 2, hi128, b + kk * 128, hi128, idesc1,
                      kk > 0);
        mma_commit(&w1_empty[slot]);
        mma_commit(&acc1_full[buf]);
        ++c1;
        return true;
      };
      auto gemm2 = [&](bool first) {
        const int slot = c2 % WR, hb = c2 % HB;
        if (!mbar_wait_deadline(&w2_full[slot], (c2 / WR) & 1)) { report_timeout(prm.status, 1203); return false; }
        if (!mbar_wait_deadline(&h_full[hb], (c2 / HB) & 1)) { report_timeout(prm.status, 1204); return false; }
        tc_fence_after();
        const uint32_t a = h_k + hb * (T::kH >> 4), b = w2_mn + slot * (T::kW2 >> 4);
#pragma unroll
        for (int kk = 0; kk < kHC / 16; ++kk)
          mma_f16_ss2(tmem + T::kColAcc2, a + (kk / 4) * ((kRowsT * 128) >> 4) + (kk % 4) * 2, hi128, b + kk * 128, hi128, idesc2,
                      (kk > 0 || !first) ? 1u : 0u);
        mma_commit(&w2_empty[slot]);
        mma_commit(&h_empty[hb]);
        ++c2;
        return true;
      };
      uint32_t seq = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        if (warp == 1) {
          const int xb = ti % XB;
          ok = mbar_wait_deadline(&x_ready[xb], (ti / XB) & 1);
          if (!ok) { report_timeout(prm.status, 1205); break; }
          tc_fence_after();
          for (int n = 0; n < nchunks && ok; ++n) ok = gemm1(xb * (T::kTileX >> 4));
          if (ok) mma_commit(x_dead);
        } else {
          // acc2 of the tile before has been read out
          ok = mbar_wait_deadline(acc2_empty, (ti & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 1206); break; }
          tc_fence_after();
          for (int n = 0; n < nchunks && ok; ++n) ok = gemm2(n == 0);
          if (ok) mma_commit(acc2_full);
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ workers: two groups of 128 threads, thread = row
    // of the tile.  Group g normalises and finally writes column half g of the row.  With 64-column chunks it owns the
    // chunks n with (chunks so far + n) % 2 == g, with them acc1[g] and H[g]; with 128-column chunks it takes column
    // half g of every chunk.  Either way two warps per scheduler hide the dependent chains one warp cannot.
    const int g = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    // the statistics' partial sums cross the groups through the H buffers, which no MMA reads between two tiles
    float* red_sum = reinterpret_cast<float*>(smem + T::kOffH);
    float* red_var = red_sum + 2 * kRowsT;
    bool ok = true;
#define CFK_TR_WAIT(bar, parity, code)                            \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    uint32_t ti = 0, ce = 0, seq = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++seq) {
      if (cls != nullptr && cls[seq] != 1) {
        // not computed: the result is the input (or zeros), copied by these warps in 16-byte pieces; a block whose
        // keep is negative throughout is left alone
        if (cls[seq] == 0) {
          constexpr int kPieces = C / 8;
          for (int idx = (warp - 4) * 32 + lane; idx < kRowsT * kPieces; idx += 256) {
            const int64_t r = tile * kRowsT + idx / kPieces;
            if (r < prm.m) {
              const int64_t off = r * C + (idx % kPieces) * 8;
              uint4 v = make_uint4(0, 0, 0, 0);
              if (prm.add_input) v = *reinterpret_cast<const uint4*>(prm.x + off);
              *reinterpret_cast<uint4*>(prm.out + off) = v;
            }
          }
        }
        continue;
      }
      const int xb = ti % XB;
      uint8_t* xt = smem + T::kOffX + xb * T::kTileX;
      constexpr int kHalf = C / 16;   // 8-column pieces of this group's half of the row
      // ---- LayerNorm of the row in place (three passes over this group's C bytes of it in shared memory)
      CFK_TR_WAIT(&x_full[xb], (ti / XB) & 1, 1301)
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        const int ch = g * kHalf + i;
        const uint4 w = *reinterpret_cast<const uint4*>(xt + (ch / 8) * (kRowsT * 128) + swz_off(row, ch % 8, 128));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) sum += bf16lo_to_f32(ww[e]) + bf16hi_to_f32(ww[e]);
      }
      red_sum[g * kRowsT + row] = sum;
      named_bar_sync(2, 256);
      const float mean = (red_sum[row] + red_sum[kRowsT + row]) * (1.0f / C);
      float var = 0.f;
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        const int ch = g * kHalf + i;
        const uint4 w = *reinterpret_cast<const uint4*>(xt + (ch / 8) * (kRowsT * 128) + swz_off(row, ch % 8, 128));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = bf16lo_to_f32(ww[e]) - mean, b = bf16hi_to_f32(ww[e]) - mean;
          var = fmaf(a, a, fmaf(b, b, var));
        }
      }
      red_var[g * kRowsT + row] = var;
      named_bar_sync(2, 256);
      const float rstd = rsqrtf((red_var[row] + red_var[kRowsT + row]) * (1.0f / C) + prm.eps);
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        const int ch = g * kHalf + i;
        uint4* ptr = reinterpret_cast<uint4*>(xt + (ch / 8) * (kRowsT * 128) + swz_off(row, ch % 8, 128));
        const uint4 w = *ptr;
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(prm.ln_scale + ch * 8));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(prm.ln_scale + ch * 8 + 4));
        const float4 o0 = __ldg(reinterpret_cast<const float4*>(prm.ln_offset + ch * 8));
        const float4 o1 = __ldg(reinterpret_cast<const float4*>(prm.ln_offset + ch * 8 + 4));
        const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float oo[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
        uint32_t y[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          y[e] = pack_bf16x2(fmaf((bf16lo_to_f32(ww[e]) - mean) * rstd, gg[2 * e], oo[2 * e]),
                             fmaf((bf16hi_to_f32(ww[e]) - mean) * rstd, gg[2 * e + 1], oo[2 * e + 1]));
        *ptr = make_uint4(y[0], y[1], y[2], y[3]);
      }
      fence_proxy_async();
      // both groups have read the partial sums before a chunk epilogue writes an H buffer over them
      named_bar_sync(2, 256);
      if (lane == 0) mbar_arrive(&x_ready[xb]);

      // ---- per hidden chunk of this group: relu(acc1 + b1) as bf16 into the H tile (the second GEMM's A operand)
#pragma unroll 1
      for (int n = 0; n < nchunks; ++n, ++ce) {
        if (GPC == 1 && int(ce & 1) != g) continue;   // 64-column chunks: the groups take them in turn
        const int buf = ce & 1, hb = ce % HB;
        const int coff = GPC == 2 ? g * 64 : 0;       // 128-column chunks: this group's half of every chunk
        CFK_TR_WAIT(&acc1_full[buf], (ce >> 1) & 1, 1302)
        tc_fence_after();
        uint32_t r0[32], r1[32];
        tmem_ld_x32(tmem + lane_addr + buf * kHC + coff, r0);
        tmem_ld_x32(tmem + lane_addr + buf * kHC + coff + 32, r1);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc1_empty[buf]);
        uint32_t hp[32];
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint4 bw = __ldg(reinterpret_cast<const uint4*>(prm.b1 + n * kHC + coff + ch * 8));
          const uint32_t bb[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int col = ch * 8 + 2 * e;
            const float a0 = __uint_as_float(col < 32 ? r0[col] : r1[col - 32]) + bf16lo_to_f32(bb[e]);
            const float a1 = __uint_as_float(col + 1 < 32 ? r0[col + 1] : r1[col + 1 - 32]) + bf16hi_to_f32(bb[e]);
            hp[ch * 4 + e] = pack_bf16x2(fmaxf(a0, 0.f), fmaxf(a1, 0.f));
          }
        }
        // the second GEMM of the chunk that used this H buffer before has read it
        CFK_TR_WAIT(&h_empty[hb], ((ce / HB) & 1) ^ 1, 1303)
        uint8_t* ht = smem + T::kOffH + hb * T::kH + (coff / 64) * (kRowsT * 128);
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)
          *reinterpret_cast<uint4*>(ht + swz_off(row, ch, 128)) = make_uint4(hp[ch * 4], hp[ch * 4 + 1], hp[ch * 4 + 2], hp[ch * 4 + 3]);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_full[hb]);
      }

      // ---- the tile's result: acc2 + b2 (+ the raw rows, which the producer has loaded again over the normalised
      // tile) written in place into the tile's shared memory and stored by TMA (rows past M are clipped by the map)
      CFK_TR_WAIT(acc2_full, ti & 1, 1304)
      if (prm.add_input) CFK_TR_WAIT(xraw_full, ti & 1, 1305)
      tc_fence_after();
#pragma unroll 1
      for (int i = 0; i < C / 64; ++i) {
        const int cb = g * (C / 64) + i;
        uint32_t r[32];
        tmem_ld_x32(tmem + lane_addr + T::kColAcc2 + cb * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          const int col = cb * 32 + ch * 8;
          uint4* ptr = reinterpret_cast<uint4*>(xt + (col / 64) * (kRowsT * 128) + swz_off(row, (col % 64) / 8, 128));
          const uint4 bw = __ldg(reinterpret_cast<const uint4*>(prm.b2 + col));
          const uint32_t bb[4] = {bw.x, bw.y, bw.z, bw.w};
          uint4 xw = make_uint4(0, 0, 0, 0);
          if (prm.add_input) xw = *ptr;
          const uint32_t xx[4] = {xw.x, xw.y, xw.z, xw.w};
          uint32_t y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            y[e] = pack_bf16x2(__uint_as_float(r[ch * 8 + 2 * e]) + bf16lo_to_f32(bb[e]) + bf16lo_to_f32(xx[e]),
                               __uint_as_float(r[ch * 8 + 2 * e + 1]) + bf16hi_to_f32(bb[e]) + bf16hi_to_f32(xx[e]));
          *ptr = make_uint4(y[0], y[1], y[2], y[3]);
        }
      }
      tc_fence_before();
      fence_proxy_async();
      named_bar_sync(1, 256);
      if (warp == 4 && lane == 0) {
        mbar_arrive(acc2_empty);  // every thread has read its part of the accumulator
        if (ok) {
#pragma unroll
          for (int a = 0; a < T::kAtoms; ++a)
            tma_store_2d(&tm_out, xt + a * (kRowsT * 128), a * 64, int(tile * kRowsT));
          tma_commit_group();
          tma_wait_group_read<0>();
        }
        mbar_arrive(&x_free[xb]);  // the store has read the buffer
      }
      ++ti;
    }
    if (warp == 4 && lane == 0) tma_wait_group<0>();
#undef CFK_TR_WAIT
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int C>
int launch(const TrParams& prm, const void* w1, const void* w2, cudaStream_t st) {
  using T = TrCfg<C>;
  CUtensorMap tx, tw1, tw2;
  {
    uint64_t dims[2] = {uint64_t(C), uint64_t(prm.m)};
    uint64_t str[1] = {uint64_t(C) * 2};
    uint32_t box[2] = {64, kRowsT};
    int rc = make_tensor_map(&tx, prm.x, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  {
    uint64_t dims[2] = {uint64_t(prm.hdim), uint64_t(C)};
    uint64_t str[1] = {uint64_t(prm.hdim) * 2};
    uint32_t box[2] = {64, uint32_t(C)};
    int rc = make_tensor_map(&tw1, w1, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  {
    uint64_t dims[2] = {uint64_t(C), uint64_t(prm.hdim)};
    uint64_t str[1] = {uint64_t(C) * 2};
    uint32_t box[2] = {64, uint32_t(T::kHC)};
    int rc = make_tensor_map(&tw2, w2, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  CUtensorMap to;
  {
    uint64_t dims[2] = {uint64_t(C), uint64_t(prm.m)};
    uint64_t str[1] = {uint64_t(C) * 2};
    uint32_t box[2] = {64, kRowsT};
    int rc = make_tensor_map(&to, prm.out, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  if (cudaFuncSetAttribute(transition_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, T::kSmem) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ntiles = (prm.m + kRowsT - 1) / kRowsT;
  const int grid = int(ntiles < sms ? ntiles : sms);
  if (prm.keep != nullptr && (ntiles + grid - 1) / grid > kMaxTilesT) return CFK_ERR_UNSUPPORTED;
  transition_kernel<C><<<grid, kThreadsT, T::kSmem, st>>>(tx, tw1, tw2, to, prm);
  return check_launch();
}

}  // namespace
}  // namespace cfk

using namespace cfk;

extern "C" int cfk_transition(const void* x, const float* ln_scale, const float* ln_offset, const void* w1, const void* b1,
                              const void* w2, const void* b2, const void* keep, int keep_dtype, void* out, int64_t m, int c,
                              int hdim, float eps, int add_input, void* stream) {
  if (!x || !ln_scale || !ln_offset || !w1 || !b1 || !w2 || !b2 || !out) return CFK_ERR_NULL;
  if (m < 0 || hdim <= 0 || hdim % 64 != 0) return CFK_ERR_SHAPE;
  if (c == 128 && hdim % 128 != 0) return CFK_ERR_UNSUPPORTED;  // 128-column hidden chunks at 128 channels
  if (c != 128 && c != 256) return CFK_ERR_UNSUPPORTED;
  if (keep != nullptr && keep_dtype != CFK_F32 && keep_dtype != CFK_BF16) return CFK_ERR_DTYPE;
  if (m == 0) return CFK_OK;
  if (!aligned16(x) || !aligned16(w1) || !aligned16(w2) || !aligned16(out) || !aligned16(b1) || !aligned16(b2) ||
      !aligned16(ln_scale) || !aligned16(ln_offset))
    return CFK_ERR_ALIGN;
  TrParams prm{static_cast<const __nv_bfloat16*>(x), ln_scale, ln_offset, static_cast<const __nv_bfloat16*>(b1),
               static_cast<const __nv_bfloat16*>(b2), static_cast<__nv_bfloat16*>(out), m, hdim, eps, add_input, keep,
               keep_dtype, device_status_word()};
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  auto st = static_cast<cudaStream_t>(stream);
  return c == 128 ? launch<128>(prm, w1, w2, st) : launch<256>(prm, w1, w2, st);
}
