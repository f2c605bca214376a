// LayerNorm -> gated dual projection of the pair representation at 128 channels, channel-major bf16 outputs
// (tri_mul.py:222-300: left, right = mask * (LN(x) wp + bp) * sigmoid(LN(x) wg + bg), split in halves, each [128, ., .']).
//
// The general row-GEMM engine computes D[row][channel] and turns it channel-major through 2-byte shared-memory stores
// with the bias, the gate and the mask applied per element from per-column vectors; it runs this op at a quarter of the
// copy bandwidth.  Here the GEMM is issued transposed, D^T[channel][row] = W^T x^T: the weights in their natural
// [K, N] layout are the MN-major A operand (M = 128 output channels), the row tile [128 rows][128] is the K-major B
// operand (N = 128 rows).  A TMEM lane is then an output channel, the 128 rows of the tile are contiguous along the
// thread's columns, and a thread writes its channel's rows as 16-byte pieces of a swizzled [channel][64 rows] staging
// atom that one TMA store moves to the channel-major output.
//
// LayerNorm is folded around the GEMM instead of being applied to the tile: with w'[k][f] = scale[k] w[k][f] (rounded
// to bf16, prepared once per CTA in shared memory), s[f] = sum_k w'[k][f] and t[f] = sum_k offset[k] w[k][f] + bias[f],
//   LN(x) w + bias = rstd * (x w' - mean * s + std * t),   std = 1 / rstd
// so the MMAs run on the RAW tile as TMA lands it.  The rank-two correction is one more K step on the tensor core: the
// weights get 16 extra K rows holding s and t, the row tile a 16-wide extra tile whose row holds -mean and std, each
// fp32 value split into a bf16 head and a bf16 remainder with all four cross products present (relative error about
// 2^-17).  What is left per element is rstd (times the mask): out = (mask rstd) p' sigmoid(rstd g').
//
// A persistent CTA walks 128-row tiles (rows along the pair's inner axis, or along its outer axis for the transposed
// read of incoming edges).  Warp 0: TMA producer (the four 128 x 128 weight blocks once, then the row tile).  Warp 1:
// MMA issuer: per tile the left pair (projection, gate) into TMEM columns [0, 256) and the right pair into [256, 512),
// 8 + 8 MMAs of N = 128 on the raw tile and two correction steps each.  Warps 2-3: one store thread per worker group.
// Warps 4-11: weight preparation; the statistics of the next tile (two lanes per row, fp32 sum and sum of squares)
// between the two halves of a tile's epilogue, which is when the next tile has landed in the single tile buffer;
// epilogue thread = channel, group = 64-row half.  Tiles follow the mask as the engine's do: a tile whose mask is zero
// throughout is written as zeros without being read, one that is negative throughout is left unwritten
// (transition.py:29-38).  Every mbarrier wait is deadline-bounded.
#include "attention_sm100.cuh"
#include "rowgemm_sm100.cuh"

namespace cfk {
namespace {

constexpr int kKc = 128;                  // input channels
constexpr int kRowsG = 128;
constexpr int kThreadsG = 384;
constexpr int kMaxTilesG = 512;
constexpr int kWBlock = kKc * 128 * 2;    // one 128 x 128 weight block: two atoms of [128 k][64 channels]
constexpr int kWxBlock = 16 * 128 * 2;    // its correction rows: two atoms of [16 k][64 channels]
constexpr int kTileXG = kRowsG * kKc * 2; // two atoms of [128 rows][64 k]
constexpr int kStageG = 128 * 128;        // staging atom: [128 channels][64 rows]
constexpr int kOffWG = 0;
constexpr int kOffWxG = kOffWG + 4 * kWBlock;
constexpr int kOffXG = kOffWxG + 4 * kWxBlock;
constexpr int kOffBxG = kOffXG + kTileXG;                // correction entries of the tile's rows: [128 rows][64 bytes]
constexpr int kOffOG = kOffBxG + kRowsG * 64;
constexpr int kOffRowG = kOffOG + 2 * kStageG;           // float4 [2][64]: per row pair (mask rstd) x 2, (rstd / 2) x 2
constexpr int kOffBarG = kOffRowG + 2 * 64 * 16;
constexpr int kNumBarsG = 4 + 4 + 4;
constexpr int kOffTmemG = kOffBarG + kNumBarsG * 8;
constexpr int kOffClsG = kOffTmemG + 16;
constexpr int kSmemG = kOffClsG + kMaxTilesG + 1024;
static_assert(kSmemG <= 232448, "shared memory budget");

constexpr int kMaxPartsG = 8;
// Where the two outputs go: one tensor map per part of the channel axis.  One part: the caller's [128, outer, inner']
// arrays.  P parts (the row-sharded triangle multiplication, which wants channel shards next): part p is channels
// [p * 128 / P, (p + 1) * 128 / P) and goes into rank p's receive buffer [P, 128 / P, outer, inner'] at this rank's
// index - the all-to-all over channels happens in this kernel's stores, over NVLink peer memory, with no pass of its own.
struct GdpOutMaps {
  CUtensorMap l[kMaxPartsG];
  CUtensorMap r[kMaxPartsG];
};

struct GdpParams {
  const float* ln_scale;
  const float* ln_offset;
  const __nv_bfloat16* bp;    // [256]
  const __nv_bfloat16* bg;    // [256]
  const __nv_bfloat16* mask;  // indexed by source row
  int64_t outer, inner, inner_pad, stride_outer, stride_inner;  // strides in rows of x
  int64_t ntiles, tiles_per_outer;
  float eps;
  int parts;                  // parts of the channel axis, each with its own output maps
  int* status;
};

__global__ void __launch_bounds__(kThreadsG, 1)
ln_gdp128_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_wp,
                 const __grid_constant__ CUtensorMap tm_wg, const __grid_constant__ GdpOutMaps om, const GdpParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBarG);
  uint64_t* x_full = bars;            // the tile has landed
  uint64_t* x_free = x_full + 1;      // every MMA of the tile has completed and its statistics are taken
  uint64_t* bx_ready = x_free + 1;    // the correction entries of the tile's rows are written
  uint64_t* w_full = bx_ready + 1;    // the weights have landed
  uint64_t* w_ready = w_full + 1;     // ... and are scaled
  uint64_t* acc_full = w_ready + 1;   // [2] left pair, right pair
  uint64_t* acc_empty = acc_full + 2; // [2]
  uint64_t* stg_full = acc_empty + 2; // [2] a group's staging atom is written
  uint64_t* stg_free = stg_full + 2;  // [2] ... and its store has read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemG);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = prm.ntiles;

  if (threadIdx.x == 0) {
    mbar_init(x_full, 1);
    mbar_init(x_free, 9);
    mbar_init(bx_ready, 8);
    mbar_init(w_full, 1);
    mbar_init(w_ready, 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
      mbar_init(&stg_full[i], 4);
      mbar_init(&stg_free[i], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_wp);
    tma_prefetch_desc(&tm_wg);
    for (int q = 0; q < prm.parts; ++q) {
      tma_prefetch_desc(&om.l[q]);
      tma_prefetch_desc(&om.r[q]);
    }
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
        ok = mbar_wait_deadline(x_free, (ti & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 1601); break; }
        const int o = int(tile / prm.tiles_per_outer), r0 = int(tile % prm.tiles_per_outer) * kRowsG;
        mbar_arrive_expect_tx(x_full, kTileXG);
        for (int a = 0; a < 2; ++a) tma_load_3d(smem + kOffXG + a * (kTileXG / 2), &tm_x, x_full, a * 64, r0, o);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer: D^T[channel][row] = W'^T x^T
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(128, kRowsG, 1, 1, 1, 0);   // A = weights MN-major, B = rows K-major
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      constexpr uint32_t hi_bx = desc_hi(8 * 64, kSwz64);               // correction entries: 64-byte rows
      const uint32_t xk = desc_lo(smem_u32(smem + kOffXG), 16), bxk = desc_lo(smem_u32(smem + kOffBxG), 16);
      bool ok = mbar_wait_deadline(w_ready, 0);
      if (!ok) report_timeout(prm.status, 1602);
      uint32_t seq = 0, ti = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        ok = mbar_wait_deadline(x_full, ti & 1);
        if (!ok) { report_timeout(prm.status, 1603); break; }
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
          if (set == 0) {  // the correction steps need the rows' statistics; the steps above did not
            ok = mbar_wait_deadline(bx_ready, ti & 1);
            if (!ok) { report_timeout(prm.status, 1607); break; }
            tc_fence_after();
          }
          for (int part = 0; part < 2; ++part)
            mma_f16_ss2(tmem + set * 256 + part * 128,
                        desc_lo(smem_u32(smem + kOffWxG + (set * 2 + part) * kWxBlock), kWxBlock / 2), hi, bxk, hi_bx, idesc, 1);
          mma_commit(&acc_full[set]);
        }
        if (ok) mma_commit(x_free);
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------------ store threads: warp 2 for group 0, warp 3 for 1
    if (lane == 0) {
      const int grp = warp - 2;
      const uint8_t* stage = smem + kOffOG + grp * kStageG;
      bool ok = true;
      uint32_t sc = 0, seq = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++seq) {
        if (cls[seq] < 0) continue;
        const int o = int(tile / prm.tiles_per_outer), r0 = int(tile % prm.tiles_per_outer) * kRowsG;
        const bool inside = r0 + grp * 64 < prm.inner_pad;   // a store never starts past the padded extent
        const int nst = cls[seq] == 1 ? 2 : 1;               // a zero tile: one atom of zeros goes to both outputs
        for (int set = 0; set < nst; ++set, ++sc) {
          ok = mbar_wait_deadline(&stg_full[grp], sc & 1);
          if (!ok) { report_timeout(prm.status, 1608); break; }
          if (inside) {
            // part q: rows q * 128 / parts .. of the atom (a multiple of 8 lines, so the swizzle phase is the atom's)
            const int part_bytes = (128 / prm.parts) * 128;
            for (int q = 0; q < prm.parts; ++q) {
              if (nst == 1) {
                tma_store_3d(&om.l[q], stage + q * part_bytes, r0 + grp * 64, o, 0);
                tma_store_3d(&om.r[q], stage + q * part_bytes, r0 + grp * 64, o, 0);
              } else {
                tma_store_3d(set ? &om.r[q] : &om.l[q], stage + q * part_bytes, r0 + grp * 64, o, 0);
              }
            }
          }
          tma_commit_group();
          tma_wait_group_read<0>();
          mbar_arrive(&stg_free[grp]);
        }
      }
      tma_wait_group<0>();
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ workers
    const int grp = (warp - 4) >> 2, quad = warp & 3;
    const int ch = quad * 32 + lane;                          // epilogue: thread = output channel, group = 64-row half
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const int pt = (warp - 4) * 32 + lane;                    // statistics: two adjacent lanes share a row
    const int lrow = pt >> 1, half = pt & 1;
    uint8_t* stage = smem + kOffOG + grp * kStageG;
    float* rowc = reinterpret_cast<float*>(smem + kOffRowG);
    bool ok = true;
#define CFK_GD_WAIT(bar, parity, code)                            \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    // head and remainder of an fp32 value as two bf16
    auto split = [](float v, __nv_bfloat16& hd, __nv_bfloat16& rm) {
      hd = __float2bfloat16_rn(v);
      rm = __float2bfloat16_rn(v - __bfloat162float(hd));
    };
    // ---- once: scale the weights' rows by the LayerNorm scales and write the correction rows.  Thread (side, f) owns
    // output channel f of the side's projection and gate blocks.  Correction rows: 0-3 = s head, s rem, s head, s rem;
    // 4-7 = t head, t rem, t head, t rem; 8-15 = 0 (and the entries of a row of the tile: -mean head, head, rem, rem;
    // std head, head, rem, rem; 0 ...), so that the K step adds (-mean) * s + std * t with every cross product.
    CFK_GD_WAIT(w_full, 0, 1605)
    {
      const int side = pt >> 7, f = pt & 127;
#pragma unroll 1
      for (int part = 0; part < 2; ++part) {
        const int blk = side * 2 + part;
        uint8_t* wb = smem + kOffWG + blk * kWBlock + (f >> 6) * (kWBlock / 2);
        float s = 0.f, t = 0.f;
#pragma unroll 4
        for (int k = 0; k < kKc; ++k) {
          __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(wb + k * 128 + ((((f & 63) >> 3) ^ (k & 7)) << 4) + (f & 7) * 2);
          const float w = __bfloat162float(*e);
          const __nv_bfloat16 ws = __float2bfloat16_rn(__ldg(prm.ln_scale + k) * w);
          *e = ws;
          s += __bfloat162float(ws);
          t = fmaf(__ldg(prm.ln_offset + k), w, t);
        }
        t += __bfloat162float(part ? prm.bg[side * 128 + f] : prm.bp[side * 128 + f]);
        __nv_bfloat16 sh, sr, th, tr;
        split(s, sh, sr);
        split(t, th, tr);
        uint8_t* xb = smem + kOffWxG + blk * kWxBlock + (f >> 6) * (kWxBlock / 2);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const __nv_bfloat16 v = k >= 8 ? __float2bfloat16_rn(0.f) : (k < 4 ? ((k & 1) ? sr : sh) : ((k & 1) ? tr : th));
          *reinterpret_cast<__nv_bfloat16*>(xb + k * 128 + ((((f & 63) >> 3) ^ (k & 7)) << 4) + (f & 7) * 2) = v;
        }
      }
      if (pt < kRowsG) {  // K = 8 .. 15 of the rows' correction entries stay zero
        *reinterpret_cast<uint4*>(smem + kOffBxG + swz_off(pt, 0, 64)) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(smem + kOffBxG + swz_off(pt, 1, 64)) = make_uint4(0, 0, 0, 0);
      }
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive(w_ready);

    // Statistics of local tile u (tile number `tile`) from the raw tile: the rows' correction entries for the tensor
    // core and the per-row factors of the epilogue (rows past the end are zero-filled by TMA and count as masked)
    auto row_stats = [&](uint32_t u, int64_t tile) {
      const uint8_t* xt = smem + kOffXG;
      const int64_t o = tile / prm.tiles_per_outer;
      const int64_t r = (tile % prm.tiles_per_outer) * kRowsG + lrow;
      float mk = 0.f;   // fetched before the wait for the tile, so that its latency runs under it
      if (half == 0 && r < prm.inner) mk = fmaxf(__bfloat162float(prm.mask[o * prm.stride_outer + r * prm.stride_inner]), 0.f);
      CFK_GD_WAIT(x_full, u & 1, 1609)
      uint64_t s2 = f2_pack(0.f, 0.f), q2 = s2, s2b = s2, q2b = s2;
#pragma unroll
      for (int j = 0; j < kKc / 16; ++j) {
        const int c = 2 * j + half;
        const uint4 w = *reinterpret_cast<const uint4*>(xt + (c / 8) * (kTileXG / 2) + swz_off(lrow, c % 8, 128));
        const uint64_t v0 = f2_pack(bf16lo_to_f32(w.x), bf16hi_to_f32(w.x)), v1 = f2_pack(bf16lo_to_f32(w.y), bf16hi_to_f32(w.y));
        const uint64_t v2 = f2_pack(bf16lo_to_f32(w.z), bf16hi_to_f32(w.z)), v3 = f2_pack(bf16lo_to_f32(w.w), bf16hi_to_f32(w.w));
        s2 = f2_add(s2, v0);
        s2b = f2_add(s2b, v1);
        q2 = f2_fma(v0, v0, q2);
        q2b = f2_fma(v1, v1, q2b);
        s2 = f2_add(s2, v2);
        s2b = f2_add(s2b, v3);
        q2 = f2_fma(v2, v2, q2);
        q2b = f2_fma(v3, v3, q2b);
      }
      float s0, s1, q0, q1;
      f2_unpack(f2_add(s2, s2b), s0, s1);
      f2_unpack(f2_add(q2, q2b), q0, q1);
      float ps = s0 + s1, pq = q0 + q1;
      ps += __shfl_xor_sync(0xffffffffu, ps, 1);
      pq += __shfl_xor_sync(0xffffffffu, pq, 1);
      if (half == 0) {
        const float mean = ps * (1.0f / kKc);
        const float var = fmaxf(pq * (1.0f / kKc) - mean * mean, 0.f) + prm.eps;
        const float rstd = rsqrtf(var);
        float* rc = rowc + (u & 1) * 256 + (lrow >> 1) * 4 + (lrow & 1);
        rc[0] = mk * rstd;
        rc[2] = 0.5f * rstd;
        __nv_bfloat16 mh, mr, dh, dr;
        split(-mean, mh, mr);
        split(var * rstd, dh, dr);
        auto two = [](__nv_bfloat16 v) { return uint32_t(__bfloat16_as_ushort(v)) * 0x10001u; };
        *reinterpret_cast<uint4*>(smem + kOffBxG + swz_off(lrow, 0, 64)) = make_uint4(two(mh), two(mr), two(dh), two(dr));
        fence_proxy_async();
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bx_ready);
        mbar_arrive(x_free);
      }
    };

    uint32_t seq = 0, ti = 0, sc = 0;
    {
      uint32_t s0 = 0;
      const int64_t first = next_computed(s0);
      if (first >= 0) row_stats(0, first);
    }
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++seq) {
      if (cls[seq] != 1) {
        if (cls[seq] == 0) {
          // zero throughout: both outputs get zeros for the tile's rows (up to the padded extent), from the staging atom
          CFK_GD_WAIT(&stg_free[grp], (sc & 1) ^ 1, 1610)
#pragma unroll
          for (int q = 0; q < 8; ++q) *reinterpret_cast<uint4*>(stage + swz_off(ch, q, 128)) = make_uint4(0, 0, 0, 0);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(&stg_full[grp]);
          ++sc;
        }
        continue;
      }
      // the row factors of this tile were written by other threads (between the halves of the tile before, or before
      // the loop)
      named_bar_sync(2, 256);
      const float4* rc4 = reinterpret_cast<const float4*>(rowc + (ti & 1) * 256) + grp * 32;
#pragma unroll 1
      for (int set = 0; set < 2; ++set) {
        if (set == 1) {  // by now the next tile has landed in the tile buffer: its statistics, one tile ahead
          uint32_t sn = seq + 1;
          const int64_t nxt = next_computed(sn);
          if (nxt >= 0) row_stats(ti + 1, nxt);
        }
        const uint64_t half2 = f2_pack(0.5f, 0.5f);
        CFK_GD_WAIT(&acc_full[set], ti & 1, 1606)
        tc_fence_after();
        uint32_t y[32];   // the 64 rows of this thread's channel, packed: the wait for the staging atom comes after them
#pragma unroll
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
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // two rows at a time in packed fp32: g + bg = rstd g', sigmoid(z) = 0.5 tanh(0.5 z) + 0.5, then
              // (mask rstd) p' sigmoid
              const int j = q * 8 + 2 * e;
              const float4 c = rc4[hb * 16 + q * 4 + e];
              const uint64_t t = f2_mul(f2_pack(__uint_as_float(rg[j]), __uint_as_float(rg[j + 1])), f2_pack(c.z, c.w));
              float t0, t1;
              f2_unpack(t, t0, t1);
              const uint64_t sg = f2_fma(f2_pack(tanh_approx(t0), tanh_approx(t1)), half2, half2);
              const uint64_t u = f2_mul(f2_pack(__uint_as_float(rp[j]), __uint_as_float(rp[j + 1])), f2_pack(c.x, c.y));
              float v0, v1;
              f2_unpack(f2_mul(u, sg), v0, v1);
              y[hb * 16 + q * 4 + e] = pack_bf16x2(v0, v1);
            }
          }
        }
        CFK_GD_WAIT(&stg_free[grp], (sc & 1) ^ 1, 1611)   // the store this group handed over last has read the atom
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<uint4*>(stage + swz_off(ch, q, 128)) = make_uint4(y[q * 4], y[q * 4 + 1], y[q * 4 + 2], y[q * 4 + 3]);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&stg_full[grp]);
        ++sc;
      }
      ++ti;
    }
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

// x [outer, inner, 128] read with the given row strides, wp / wg [128, 256].  parts == 1: left_ptrs[0] / right_ptrs[0] are
// left / right [128, outer, inner_pad] bf16.  parts == P > 1: left_ptrs[q] / right_ptrs[q] are rank q's receive buffers
// [P, 128 / P, outer, inner_pad] (peer mappings for q != rank), and this rank's channel part q lands at index `rank` there.
// Returns CFK_ERR_UNSUPPORTED for what the general engine should take instead.
int ln_gdp128_launch(const void* x, const float* ln_scale, const float* ln_offset, const void* wp, const void* bp,
                     const void* wg, const void* bg, const void* mask, void* const* left_ptrs, void* const* right_ptrs,
                     int rank, int parts, int64_t outer, int64_t inner, int64_t inner_pad, int64_t stride_outer,
                     int64_t stride_inner, float eps, cudaStream_t st) {
  if ((inner_pad * 2) % 16 != 0 || outer > INT32_MAX || inner_pad > INT32_MAX) return CFK_ERR_UNSUPPORTED;
  if (parts < 1 || parts > kMaxPartsG || 128 % parts != 0 || (128 / parts) % 8 != 0 || rank < 0 || rank >= parts)
    return CFK_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(wp) || !aligned16(wg) || !aligned16(ln_scale) || !aligned16(ln_offset)) return CFK_ERR_UNSUPPORTED;
  for (int q = 0; q < parts; ++q)
    if (!left_ptrs[q] || !right_ptrs[q] || !aligned16(left_ptrs[q]) || !aligned16(right_ptrs[q])) return CFK_ERR_UNSUPPORTED;
  GdpParams prm{};
  prm.ln_scale = ln_scale; prm.ln_offset = ln_offset;
  prm.bp = static_cast<const __nv_bfloat16*>(bp); prm.bg = static_cast<const __nv_bfloat16*>(bg);
  prm.mask = static_cast<const __nv_bfloat16*>(mask);
  prm.outer = outer; prm.inner = inner; prm.inner_pad = inner_pad;
  prm.stride_outer = stride_outer; prm.stride_inner = stride_inner;
  prm.tiles_per_outer = (inner_pad + kRowsG - 1) / kRowsG;
  prm.ntiles = outer * prm.tiles_per_outer;
  prm.eps = eps;
  prm.parts = parts;
  prm.status = device_status_word();
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  if (prm.ntiles == 0) return CFK_OK;
  CUtensorMap tx, twp, twg;
  GdpOutMaps om{};
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
  const int cpart = 128 / parts;
  const uint64_t part_elems = uint64_t(cpart) * uint64_t(outer) * uint64_t(inner_pad);   // one rank's share of a buffer
  for (int i = 0; i < 2; ++i)
    for (int q = 0; q < parts; ++q) {
      uint64_t dims[3] = {uint64_t(inner_pad), uint64_t(outer), uint64_t(cpart)};
      uint64_t str[2] = {uint64_t(inner_pad) * 2, uint64_t(outer) * uint64_t(inner_pad) * 2};
      uint32_t box[3] = {64, 1, uint32_t(cpart)};
      char* base = static_cast<char*>(i ? right_ptrs[q] : left_ptrs[q]) + (parts > 1 ? uint64_t(rank) * part_elems * 2 : 0);
      int rc = make_tensor_map(i ? &om.r[q] : &om.l[q], base, CFK_BF16, 3, dims, str, box, 128);
      if (rc != CFK_OK) return rc;
    }
  if (cudaFuncSetAttribute(ln_gdp128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemG) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = int(prm.ntiles < sms ? prm.ntiles : sms);
  if ((prm.ntiles + grid - 1) / grid > kMaxTilesG) return CFK_ERR_UNSUPPORTED;
  ln_gdp128_kernel<<<grid, kThreadsG, kSmemG, st>>>(tx, twp, twg, om, prm);
  return check_launch();
}

}  // namespace cfk
