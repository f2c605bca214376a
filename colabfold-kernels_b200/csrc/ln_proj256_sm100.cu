// LayerNorm -> packed projection at 256 input channels (the MSA side of the Evoformer): p[m, s*n + j] = (LN(x) w[s])[m, j]
// (packed_attn.py:190-231, 234-305).  The general row-GEMM engine serves this shape with 64-column chunks (a 64 KB
// activation tile and 64 KB weight chunks leave it no room for more) and is then bound by its MMA issue: 256
// instructions of N = 64 per tile at the issue floor.  This kernel takes 128-column chunks - half the instructions -
// by spending the shared memory differently: one activation tile (normalised in place), a two-slot ring of 64 KB weight
// chunks streamed from L2, and two 16 KB output staging atoms.
//
// A persistent CTA walks 128-row tiles.  Warp 0: TMA producer (tile, weight chunks).  Warp 1: MMA issuer, one chunk =
// 16 MMAs of M = 128, N = 128 into one of two accumulators.  Warps 4-11: LayerNorm in place (two lanes per row, halves
// combined by shuffle; fp32 statistics, bf16 out as the reference rounds the normed tile, packed_attn.py:215-220), then
// per chunk both groups of four warps drain the accumulator (group = 64-column half), round to bf16 into their staging
// atom and store it by TMA.  Row blocks follow `keep` (transition.py:29-38).  Every mbarrier wait is deadline-bounded.
#include "attention_sm100.cuh"
#include "rowgemm_sm100.cuh"

namespace cfk {
namespace {

constexpr int kA = 256;                  // input channels
constexpr int kRowsP = 128;
constexpr int kNC = 128;                 // output columns per chunk
constexpr int kThreadsP = 384;
constexpr int kMaxTilesP = 512;          // tiles per CTA when row blocks may be skipped
constexpr int kTileXP = kRowsP * kA * 2;           // 4 atoms of [128 rows][64 columns]
constexpr int kWChunk = kA * kNC * 2;              // 2 atoms of [256 rows][64 columns]
constexpr int kStageOut = kRowsP * 128;            // one staging atom: [128 rows][64 columns]
constexpr int kOffXP = 0;
constexpr int kOffWP = kOffXP + kTileXP;
constexpr int kOffOP = kOffWP + 2 * kWChunk;
constexpr int kOffBarP = kOffOP + 2 * kStageOut;
constexpr int kNumBarsP = 3 + 4 + 4;
constexpr int kOffTmemP = kOffBarP + kNumBarsP * 8;
constexpr int kOffClsP = kOffTmemP + 16;
constexpr int kSmemP = kOffClsP + kMaxTilesP + 1024;
static_assert(kSmemP <= 232448, "shared memory budget");

struct ProjParams {
  const float* ln_scale;
  const float* ln_offset;
  __nv_bfloat16* out;   // [m, ldo]
  int64_t m, ldo;
  int chunks, chunks_per_slot;   // chunks = slots * chunks_per_slot
  float eps;
  const void* keep;
  int keep_dtype;
  int* status;
};

__global__ void __launch_bounds__(kThreadsP, 1)
ln_proj256_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                  const __grid_constant__ CUtensorMap tm_out, const ProjParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBarP);
  uint64_t* x_full = bars;            // the tile has landed
  uint64_t* x_ready = x_full + 1;     // ... and is normalised
  uint64_t* x_dead = x_ready + 1;     // every MMA of the tile has completed: the buffer is free
  uint64_t* w_full = x_dead + 1;      // [2]
  uint64_t* w_empty = w_full + 2;     // [2]
  uint64_t* acc_full = w_empty + 2;   // [2]
  uint64_t* acc_empty = acc_full + 2; // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemP);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = (prm.m + kRowsP - 1) / kRowsP;

  if (threadIdx.x == 0) {
    mbar_init(x_full, 1);
    mbar_init(x_ready, 8);
    mbar_init(x_dead, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  // the class of every tile this CTA will visit: 1 compute, 0 no row kept (zeros), -1 negative throughout (unwritten)
  const int8_t* cls = nullptr;
  if (prm.keep != nullptr) {
    int8_t* w = reinterpret_cast<int8_t*>(smem + kOffClsP);
    for (int i = warp;; i += kThreadsP / 32) {
      const int64_t tile = blockIdx.x + int64_t(i) * gridDim.x;
      if (tile >= ntiles) break;
      float top = -1.f;
      for (int j = lane; j < kRowsP; j += 32) {
        const int64_t r = tile * kRowsP + j;
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
      bool ok = true;
      uint32_t seq = 0, ti = 0, cc = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        ok = mbar_wait_deadline(x_dead, (ti & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 1501); break; }
        mbar_arrive_expect_tx(x_full, kTileXP);
#pragma unroll
        for (int a = 0; a < kA / 64; ++a)
          tma_load_2d(smem + kOffXP + a * (kRowsP * 128), &tm_x, x_full, a * 64, int(tile * kRowsP));
        for (int c = 0; c < prm.chunks && ok; ++c, ++cc) {
          const int slot = cc & 1;
          ok = mbar_wait_deadline(&w_empty[slot], ((cc >> 1) & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 1502); break; }
          mbar_arrive_expect_tx(&w_full[slot], kWChunk);
          const int ws = c / prm.chunks_per_slot, col = (c % prm.chunks_per_slot) * kNC;
          tma_load_3d(smem + kOffWP + slot * kWChunk, &tm_w, &w_full[slot], col, 0, ws);
          tma_load_3d(smem + kOffWP + slot * kWChunk + kWChunk / 2, &tm_w, &w_full[slot], col + 64, 0, ws);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(kRowsP, kNC, 1, 1, 0, 1);   // A = LN(x) K-major, B = weight chunk MN-major
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      const uint32_t x_k = desc_lo(smem_u32(smem + kOffXP), 16);
      bool ok = true;
      uint32_t seq = 0, ti = 0, cc = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        ok = mbar_wait_deadline(x_ready, ti & 1);
        if (!ok) { report_timeout(prm.status, 1503); break; }
        for (int c = 0; c < prm.chunks && ok; ++c, ++cc) {
          const int slot = cc & 1, buf = cc & 1;
          ok = mbar_wait_deadline(&w_full[slot], (cc >> 1) & 1);
          if (!ok) { report_timeout(prm.status, 1504); break; }
          ok = mbar_wait_deadline(&acc_empty[buf], ((cc >> 1) & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 1505); break; }
          tc_fence_after();
          const uint32_t b = desc_lo(smem_u32(smem + kOffWP + slot * kWChunk), kWChunk / 2);  // atoms of 64 columns, 32 KB apart
#pragma unroll
          for (int kk = 0; kk < kA / 16; ++kk)
            mma_f16_ss2(tmem + buf * kNC, x_k + (kk / 4) * ((kRowsP * 128) >> 4) + (kk % 4) * 2, hi, b + kk * 128, hi, idesc, kk > 0);
          mma_commit(&w_empty[slot]);
          mma_commit(&acc_full[buf]);
        }
        if (ok) mma_commit(x_dead);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ workers
    const int grp = (warp - 4) >> 2, quad = warp & 3;
    const int trow = quad * 32 + lane;                       // epilogue: thread = row, group = 64-column half
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const int pt = (warp - 4) * 32 + lane;                   // LayerNorm: two adjacent lanes share a row
    const int lrow = pt >> 1, half = pt & 1;
    uint8_t* stage = smem + kOffOP + grp * kStageOut;
    uint8_t* xt = smem + kOffXP;
    bool ok = true;
#define CFK_LP_WAIT(bar, parity, code)                            \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    uint32_t seq = 0, ti = 0, cc = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++seq) {
      if (cls != nullptr && cls[seq] != 1) {
        if (cls[seq] == 0) {  // no row kept: zeros, straight from these threads
          const int pieces = int(prm.ldo / 8);
          for (int64_t idx = pt; idx < int64_t(kRowsP) * pieces; idx += 256) {
            const int64_t r = tile * kRowsP + idx / pieces;
            if (r < prm.m) *reinterpret_cast<uint4*>(prm.out + r * prm.ldo + (idx % pieces) * 8) = make_uint4(0, 0, 0, 0);
          }
        }
        continue;
      }
      // ---- LayerNorm in place: this thread's 16-byte pieces of its row are the odd or the even ones
      CFK_LP_WAIT(x_full, ti & 1, 1506)
      float ps = 0.f;
#pragma unroll 4
      for (int j = 0; j < kA / 16; ++j) {
        const int ch = 2 * j + half;
        const uint4 w = *reinterpret_cast<const uint4*>(xt + (ch / 8) * (kRowsP * 128) + swz_off(lrow, ch % 8, 128));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) ps += bf16lo_to_f32(ww[e]) + bf16hi_to_f32(ww[e]);
      }
      const float mean = (ps + __shfl_xor_sync(0xffffffffu, ps, 1)) * (1.0f / kA);
      float pv = 0.f;
#pragma unroll 4
      for (int j = 0; j < kA / 16; ++j) {
        const int ch = 2 * j + half;
        const uint4 w = *reinterpret_cast<const uint4*>(xt + (ch / 8) * (kRowsP * 128) + swz_off(lrow, ch % 8, 128));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = bf16lo_to_f32(ww[e]) - mean, b = bf16hi_to_f32(ww[e]) - mean;
          pv = fmaf(a, a, fmaf(b, b, pv));
        }
      }
      const float rstd = rsqrtf((pv + __shfl_xor_sync(0xffffffffu, pv, 1)) * (1.0f / kA) + prm.eps);
#pragma unroll 2
      for (int j = 0; j < kA / 16; ++j) {
        const int ch = 2 * j + half;
        uint4* ptr = reinterpret_cast<uint4*>(xt + (ch / 8) * (kRowsP * 128) + swz_off(lrow, ch % 8, 128));
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
      __syncwarp();
      if (lane == 0) mbar_arrive(x_ready);

      // ---- per chunk: this group's 64 columns of the accumulator -> bf16 -> staging atom -> TMA store
#pragma unroll 1
      for (int c = 0; c < prm.chunks; ++c, ++cc) {
        const int buf = cc & 1;
        CFK_LP_WAIT(&acc_full[buf], (cc >> 1) & 1, 1507)
        tc_fence_after();
        uint32_t r0[32], r1[32];
        tmem_ld_x32(tmem + lane_addr + buf * kNC + grp * 64, r0);
        tmem_ld_x32(tmem + lane_addr + buf * kNC + grp * 64 + 32, r1);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        // the store this group issued one chunk ago has read the staging atom
        if (trow == 0) tma_wait_group_read<0>();
        named_bar_sync(3 + grp, 128);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t* r = q < 4 ? r0 : r1;
          const int o = (q & 3) * 8;
          *reinterpret_cast<uint4*>(stage + swz_off(trow, q, 128)) =
              make_uint4(pack_bf16x2(__uint_as_float(r[o]), __uint_as_float(r[o + 1])),
                         pack_bf16x2(__uint_as_float(r[o + 2]), __uint_as_float(r[o + 3])),
                         pack_bf16x2(__uint_as_float(r[o + 4]), __uint_as_float(r[o + 5])),
                         pack_bf16x2(__uint_as_float(r[o + 6]), __uint_as_float(r[o + 7])));
        }
        fence_proxy_async();
        named_bar_sync(3 + grp, 128);
        if (trow == 0) {
          if (ok) tma_store_2d(&tm_out, stage, c * kNC + grp * 64, int(tile * kRowsP));
          tma_commit_group();
        }
      }
      ++ti;
    }
    if (trow == 0) tma_wait_group<0>();
#undef CFK_LP_WAIT
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

// x [m, 256], w [slots, 256, n] (n a multiple of 128), out [m, slots * n] bf16.  Returns CFK_ERR_UNSUPPORTED for what the
// general engine should take instead.
int ln_proj256_launch(const void* x, const float* ln_scale, const float* ln_offset, const void* w, const void* keep,
                      int keep_dtype, void* out, int64_t m, int slots, int n, float eps, cudaStream_t st) {
  if (n % kNC != 0 || slots <= 0) return CFK_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(w) || !aligned16(out) || !aligned16(ln_scale) || !aligned16(ln_offset)) return CFK_ERR_UNSUPPORTED;
  ProjParams prm{ln_scale, ln_offset, static_cast<__nv_bfloat16*>(out), m, int64_t(slots) * n, slots * (n / kNC), n / kNC, eps,
                 keep, keep_dtype, device_status_word()};
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  CUtensorMap tx, tw, to;
  {
    uint64_t dims[2] = {uint64_t(kA), uint64_t(m)};
    uint64_t str[1] = {uint64_t(kA) * 2};
    uint32_t box[2] = {64, kRowsP};
    int rc = make_tensor_map(&tx, x, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  {
    uint64_t dims[3] = {uint64_t(n), uint64_t(kA), uint64_t(slots)};
    uint64_t str[2] = {uint64_t(n) * 2, uint64_t(kA) * uint64_t(n) * 2};
    uint32_t box[3] = {64, kA, 1};
    int rc = make_tensor_map(&tw, w, CFK_BF16, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  {
    uint64_t dims[2] = {uint64_t(prm.ldo), uint64_t(m)};
    uint64_t str[1] = {uint64_t(prm.ldo) * 2};
    uint32_t box[2] = {64, kRowsP};
    int rc = make_tensor_map(&to, out, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  if (cudaFuncSetAttribute(ln_proj256_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemP) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ntiles = (m + kRowsP - 1) / kRowsP;
  const int grid = int(ntiles < sms ? ntiles : sms);
  if (keep != nullptr && (ntiles + grid - 1) / grid > kMaxTilesP) return CFK_ERR_UNSUPPORTED;
  ln_proj256_kernel<<<grid, kThreadsP, kSmemP, st>>>(tx, tw, to, prm);
  return check_launch();
}

}  // namespace cfk
