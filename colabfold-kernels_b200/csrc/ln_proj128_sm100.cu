// LayerNorm -> packed projection at 128 input channels and up to 512 output columns (the pair side of the Evoformer:
// q, k, v and gate of the triangle attention, packed_attn.py:190-231, 234-305): p[m, s*n + j] = (LN(x) w[s])[m, j].
//
// All the weights (128 KB) stay in shared memory and LayerNorm is folded around the GEMM instead of being applied to the
// tile: with w'[k][f] = scale[k] w[k][f] (rounded to bf16, prepared once per CTA in shared memory), s[f] = sum_k w'[k][f]
// and t[f] = sum_k offset[k] w[k][f],
//   LN(x) w = rstd * (x w' - mean * s + std * t),   std = 1 / rstd
// so the MMAs run on the RAW tile as TMA lands it and nothing waits for a normalised tile.  The rank-two correction
// (- mean * s + std * t) is itself one more K step on the tensor core: the A operand gets a 16-wide extra tile whose row
// holds -mean and std, the B operand 16 extra rows holding s and t, each fp32 value split into a bf16 head and a bf16
// remainder with all four cross products present (head*head, head*rem, rem*head, rem*rem: relative error about 2^-17).
// The epilogue is then one multiplication by rstd per element: no per-column constants are read, which matters because
// a load of a constant that the 32 threads of a warp share still costs the shared-memory pipe as much as a full load,
// and that pipe, not HBM, bounded the first form of this kernel.  s uses the same bf16 w' the tensor core multiplies
// by, so mean * s cancels the mean's part of x w' to fp32 rounding.
//
// A persistent CTA walks 128-row tiles.  Warp 0: TMA producer (weights once, then the activation tile).  Warp 1: MMA
// issuer, per 256 output columns 8 MMAs of M = 128, N = 256 on the raw tile plus the correction step (N = 128 for an odd
// last chunk) into one of two accumulators.  Warps 2-3: one store thread per worker group (TMA store of the group's
// staging atom, then the hand-back once the store has read it).  Warps 4-11: weight preparation, the statistics of
// the thread's own row (fp32 sum and sum of squares from the raw tile) and its correction entries, and per chunk both
// groups of four warps drain the accumulator (group = 64-column half), scale by rstd and round to bf16 into their
// staging atom.  Row blocks follow `keep` (transition.py:29-38).  Every mbarrier wait is deadline-bounded.
#include "attention_sm100.cuh"
#include "rowgemm_sm100.cuh"

namespace cfk {
namespace {

constexpr int kK8 = 128;                 // input channels
constexpr int kRows8 = 128;
constexpr int kNC8 = 128;                // output columns per chunk
constexpr int kMaxChunks8 = 4;
constexpr int kThreads8 = 384;
constexpr int kMaxTiles8 = 256;          // tiles per CTA when row blocks may be skipped
constexpr int kAtom8 = 128 * 128;        // 16 KB: 128 lines of 128 bytes
constexpr int kOffW8 = 0;                              // chunk c: atoms 2c, 2c + 1 ([128 k][64 columns])
constexpr int kWxAtom8 = 16 * 128;                     // correction rows of 64 columns: 16 lines of 128 bytes
constexpr int kOffWx8 = kOffW8 + 2 * kMaxChunks8 * kAtom8;  // chunk c: atoms 2c, 2c + 1 ([16 k][64 columns])
constexpr int kOffX8 = kOffWx8 + 2 * kMaxChunks8 * kWxAtom8;  // the activation tile: 2 atoms ([128 rows][64 channels])
constexpr int kOffAx8 = kOffX8 + 2 * kAtom8;           // correction entries of the tile's rows: [128 rows][64 bytes]
constexpr int kOffO8 = kOffAx8 + 128 * 64;             // one staging atom per group ([128 rows][64 columns])
constexpr int kOffBar8 = kOffO8 + 2 * kAtom8;
constexpr int kNumBars8 = 5 + 2 + 2 + 2 + 2;
constexpr int kOffTmem8 = kOffBar8 + kNumBars8 * 8;
constexpr int kOffCls8 = kOffTmem8 + 16;
constexpr int kSmem8 = kOffCls8 + kMaxTiles8 + 1024;
static_assert(kSmem8 <= 232448, "shared memory budget");

struct Proj8Params {
  const float* ln_scale;
  const float* ln_offset;
  __nv_bfloat16* out;   // [m, ldo]
  int64_t m, ldo;
  int chunks, chunks_per_slot;   // chunks = slots * chunks_per_slot, at most 4
  float eps;
  const void* keep;
  int keep_dtype;
  int* status;
};

__global__ void __launch_bounds__(kThreads8, 1)
ln_proj128_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                  const __grid_constant__ CUtensorMap tm_out, const Proj8Params prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar8);
  uint64_t* w_full = bars;            // the weights have landed
  uint64_t* w_ready = w_full + 1;     // ... and are scaled
  uint64_t* x_full = w_ready + 1;     // the tile has landed
  uint64_t* x_free = x_full + 1;      // its MMAs have completed and every worker warp has its statistics
  uint64_t* ax_ready = x_free + 1;    // the correction entries of the tile's rows are written
  uint64_t* acc_full = ax_ready + 1;  // [2]
  uint64_t* acc_empty = acc_full + 2; // [2]
  uint64_t* stg_full = acc_empty + 2; // [2] a group's staging atom is written
  uint64_t* stg_free = stg_full + 2;  // [2] ... and its store has read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t ntiles = (prm.m + kRows8 - 1) / kRows8;

  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    mbar_init(w_ready, 8);
    mbar_init(x_full, 1);
    mbar_init(x_free, 9);
    mbar_init(ax_ready, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
      mbar_init(&stg_full[i], 4);
      mbar_init(&stg_free[i], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // the class of every tile this CTA will visit: 1 compute, 0 no row kept (zeros), -1 negative throughout (unwritten)
  const int8_t* cls = nullptr;
  if (prm.keep != nullptr) {
    int8_t* w = reinterpret_cast<int8_t*>(smem + kOffCls8);
    for (int i = warp;; i += kThreads8 / 32) {
      const int64_t tile = blockIdx.x + int64_t(i) * gridDim.x;
      if (tile >= ntiles) break;
      float top = -1.f;
      for (int j = lane; j < kRows8; j += 32) {
        const int64_t r = tile * kRows8 + j;
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
      mbar_arrive_expect_tx(w_full, uint32_t(prm.chunks) * 2 * kAtom8);
      for (int c = 0; c < prm.chunks; ++c) {
        const int ws = c / prm.chunks_per_slot, col = (c % prm.chunks_per_slot) * kNC8;
        tma_load_3d(smem + kOffW8 + (2 * c) * kAtom8, &tm_w, w_full, col, 0, ws);
        tma_load_3d(smem + kOffW8 + (2 * c + 1) * kAtom8, &tm_w, w_full, col + 64, 0, ws);
      }
      bool ok = true;
      uint32_t seq = 0, ti = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        ok = mbar_wait_deadline(x_free, (ti & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 1801); break; }
        mbar_arrive_expect_tx(x_full, 2 * kAtom8);
        tma_load_2d(smem + kOffX8, &tm_x, x_full, 0, int(tile * kRows8));
        tma_load_2d(smem + kOffX8 + kAtom8, &tm_x, x_full, 64, int(tile * kRows8));
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc1 = make_idesc(kRows8, kNC8, 1, 1, 0, 1);       // A = raw x tile K-major, B = w' MN-major
      constexpr uint32_t idesc2 = make_idesc(kRows8, 2 * kNC8, 1, 1, 0, 1);   // two chunks at once
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      constexpr uint32_t hi_ax = desc_hi(8 * 64, kSwz64);   // correction entries: 64-byte rows
      const uint32_t x_k = desc_lo(smem_u32(smem + kOffX8), 16), ax_k = desc_lo(smem_u32(smem + kOffAx8), 16);
      bool ok = mbar_wait_deadline(w_ready, 0);
      if (!ok) report_timeout(prm.status, 1802);
      uint32_t seq = 0, ti = 0, cc = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq), ++ti) {
        ok = mbar_wait_deadline(x_full, ti & 1);
        if (!ok) { report_timeout(prm.status, 1803); break; }
        for (int c = 0; c < prm.chunks && ok; c += 2, ++cc) {
          const int buf = cc & 1;
          ok = mbar_wait_deadline(&acc_empty[buf], ((cc >> 1) & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 1804); break; }
          tc_fence_after();
          const uint32_t b = desc_lo(smem_u32(smem + kOffW8 + (2 * c) * kAtom8), kAtom8);  // atoms of 64 columns, 16 KB apart
          const uint32_t idesc = c + 1 < prm.chunks ? idesc2 : idesc1;
#pragma unroll
          for (int kk = 0; kk < kK8 / 16; ++kk)
            mma_f16_ss2(tmem + buf * 2 * kNC8, x_k + (kk / 4) * (kAtom8 >> 4) + (kk % 4) * 2, hi, b + kk * 128, hi, idesc, kk > 0);
          if (c == 0) {  // the correction step needs the rows' statistics; the steps above did not
            ok = mbar_wait_deadline(ax_ready, ti & 1);
            if (!ok) { report_timeout(prm.status, 1810); break; }
            tc_fence_after();
          }
          mma_f16_ss2(tmem + buf * 2 * kNC8, ax_k, hi_ax, desc_lo(smem_u32(smem + kOffWx8 + (2 * c) * kWxAtom8), kWxAtom8), hi, idesc, 1);
          mma_commit(&acc_full[buf]);
        }
        if (ok) mma_commit(x_free);
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------------ store threads: warp 2 for group 0, warp 3 for 1
    if (lane == 0) {
      const int grp = warp - 2;
      const uint8_t* stage = smem + kOffO8 + grp * kAtom8;
      bool ok = true;
      uint32_t seq = 0, sc = 0;
      for (int64_t tile = next_computed(seq); tile >= 0 && ok; tile = next_computed(++seq)) {
        for (int c = 0; c < prm.chunks; ++c, ++sc) {
          ok = mbar_wait_deadline(&stg_full[grp], sc & 1);
          if (!ok) { report_timeout(prm.status, 1808); break; }
          tma_store_2d(&tm_out, stage, c * kNC8 + grp * 64, int(tile * kRows8));
          tma_commit_group();
          tma_wait_group_read<0>();
          mbar_arrive(&stg_free[grp]);
        }
      }
      tma_wait_group<0>();
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ workers
    const int grp = (warp - 4) >> 2, quad = warp & 3;
    const int trow = quad * 32 + lane;                       // thread = row, group = 64-column half of every chunk
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const int pt = (warp - 4) * 32 + lane;
    uint8_t* stage = smem + kOffO8 + grp * kAtom8;
    bool ok = true;
#define CFK_P8_WAIT(bar, parity, code)                            \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    // head and remainder of an fp32 value as two bf16
    auto split = [](float v, __nv_bfloat16& hd, __nv_bfloat16& rm) {
      hd = __float2bfloat16_rn(v);
      rm = __float2bfloat16_rn(v - __bfloat162float(hd));
    };
    // ---- once: scale the weights' rows by the LayerNorm scales and write the correction rows.  Thread (group, j, h)
    // owns column grp * 64 + j of chunks 2h and 2h + 1.  Correction rows: 0-3 = s head, s rem, s head, s rem;
    // 4-7 = t head, t rem, t head, t rem; 8-15 = 0 (and the entries of a row: -mean head, head, rem, rem; std head,
    // head, rem, rem; 0 ...), so that the K step adds (-mean) * s + std * t with every cross product.
    const int cj = trow & 63, chh = trow >> 6;
    CFK_P8_WAIT(w_full, 0, 1805)
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = 2 * chh + u;
      if (c < prm.chunks) {
        uint8_t* wb = smem + kOffW8 + (2 * c + grp) * kAtom8;
        float s = 0.f, t = 0.f;
#pragma unroll 4
        for (int k = 0; k < kK8; ++k) {
          __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(wb + k * 128 + (((cj >> 3) ^ (k & 7)) << 4) + (cj & 7) * 2);
          const float w = __bfloat162float(*e);
          const __nv_bfloat16 ws = __float2bfloat16_rn(__ldg(prm.ln_scale + k) * w);
          *e = ws;
          s += __bfloat162float(ws);
          t = fmaf(__ldg(prm.ln_offset + k), w, t);
        }
        __nv_bfloat16 sh, sr, th, tr;
        split(s, sh, sr);
        split(t, th, tr);
        uint8_t* xb = smem + kOffWx8 + (2 * c + grp) * kWxAtom8;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const __nv_bfloat16 v = k >= 8 ? __float2bfloat16_rn(0.f) : (k < 4 ? ((k & 1) ? sr : sh) : ((k & 1) ? tr : th));
          *reinterpret_cast<__nv_bfloat16*>(xb + k * 128 + (((cj >> 3) ^ (k & 7)) << 4) + (cj & 7) * 2) = v;
        }
      }
    }
    if (grp == 0) {  // K = 8 .. 15 of the rows' correction entries stay zero
      *reinterpret_cast<uint4*>(smem + kOffAx8 + swz_off(trow, 1, 64)) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(smem + kOffAx8 + swz_off(trow, 0, 64)) = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive(w_ready);

    uint32_t seq = 0, ti = 0, cc = 0, sc = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++seq) {
      if (cls != nullptr && cls[seq] != 1) {
        if (cls[seq] == 0) {  // no row kept: zeros, straight from these threads
          const int pieces = int(prm.ldo / 8);
          for (int64_t idx = pt; idx < int64_t(kRows8) * pieces; idx += 256) {
            const int64_t r = tile * kRows8 + idx / pieces;
            if (r < prm.m) *reinterpret_cast<uint4*>(prm.out + r * prm.ldo + (idx % pieces) * 8) = make_uint4(0, 0, 0, 0);
          }
        }
        continue;
      }
      // ---- statistics of this thread's row from the raw tile (fp32 sum and sum of squares over the 128 channels)
      CFK_P8_WAIT(x_full, ti & 1, 1806)
      float rstd;
      {
        const uint8_t* xt = smem + kOffX8;
        uint64_t s2a = f2_pack(0.f, 0.f), s2b = s2a, q2a = s2a, q2b = s2a;   // packed pairs, two chains
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const uint4 w = *reinterpret_cast<const uint4*>(xt + (p >> 3) * kAtom8 + swz_off(trow, p & 7, 128));
          const uint64_t v0 = f2_pack(bf16lo_to_f32(w.x), bf16hi_to_f32(w.x)), v1 = f2_pack(bf16lo_to_f32(w.y), bf16hi_to_f32(w.y));
          const uint64_t v2 = f2_pack(bf16lo_to_f32(w.z), bf16hi_to_f32(w.z)), v3 = f2_pack(bf16lo_to_f32(w.w), bf16hi_to_f32(w.w));
          s2a = f2_add(s2a, v0);
          s2b = f2_add(s2b, v1);
          q2a = f2_fma(v0, v0, q2a);
          q2b = f2_fma(v1, v1, q2b);
          s2a = f2_add(s2a, v2);
          s2b = f2_add(s2b, v3);
          q2a = f2_fma(v2, v2, q2a);
          q2b = f2_fma(v3, v3, q2b);
        }
        float s0, s1, q0, q1;
        f2_unpack(f2_add(s2a, s2b), s0, s1);
        f2_unpack(f2_add(q2a, q2b), q0, q1);
        const float mean = (s0 + s1) * (1.0f / kK8);
        const float var = fmaxf((q0 + q1) * (1.0f / kK8) - mean * mean, 0.f) + prm.eps;
        rstd = rsqrtf(var);
        if (grp == 0) {  // the row's correction entries (the other group computes the same numbers for its own epilogue)
          __nv_bfloat16 mh, mr, dh, dr;
          split(-mean, mh, mr);
          split(var * rstd, dh, dr);
          auto two = [](__nv_bfloat16 v) { return uint32_t(__bfloat16_as_ushort(v)) * 0x10001u; };
          *reinterpret_cast<uint4*>(smem + kOffAx8 + swz_off(trow, 0, 64)) = make_uint4(two(mh), two(mr), two(dh), two(dr));
          fence_proxy_async();
        }
      }
      __syncwarp();
      if (lane == 0) {
        if (grp == 0) mbar_arrive(ax_ready);
        mbar_arrive(x_free);
      }
      const uint64_t r2 = f2_pack(rstd, rstd);

      // ---- per chunk: this group's 64 columns of the accumulator -> * rstd -> bf16 -> staging atom -> the store thread
#pragma unroll 1
      for (int c = 0; c < prm.chunks; ++c, ++sc) {
        const int buf = cc & 1, hf = c & 1;
        if (hf == 0) {
          CFK_P8_WAIT(&acc_full[buf], (cc >> 1) & 1, 1807)
          tc_fence_after();
        }
        uint32_t r0[32], r1[32];
        tmem_ld_x32(tmem + lane_addr + buf * 2 * kNC8 + hf * kNC8 + grp * 64, r0);
        tmem_ld_x32(tmem + lane_addr + buf * 2 * kNC8 + hf * kNC8 + grp * 64 + 32, r1);
        tmem_wait_ld();
        if (hf == 1 || c + 1 == prm.chunks) {  // both halves of the accumulator are in registers
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
          ++cc;
        }
        CFK_P8_WAIT(&stg_free[grp], (sc & 1) ^ 1, 1809)  // the store of the chunk before has read the staging atom
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t* r = q < 4 ? r0 : r1;
          const int o = (q & 3) * 8;
          float a0, a1, a2, a3, a4, a5, a6, a7;
          f2_unpack(f2_mul(r2, f2_pack(__uint_as_float(r[o]), __uint_as_float(r[o + 1]))), a0, a1);
          f2_unpack(f2_mul(r2, f2_pack(__uint_as_float(r[o + 2]), __uint_as_float(r[o + 3]))), a2, a3);
          f2_unpack(f2_mul(r2, f2_pack(__uint_as_float(r[o + 4]), __uint_as_float(r[o + 5]))), a4, a5);
          f2_unpack(f2_mul(r2, f2_pack(__uint_as_float(r[o + 6]), __uint_as_float(r[o + 7]))), a6, a7);
          *reinterpret_cast<uint4*>(stage + swz_off(trow, q, 128)) =
              make_uint4(pack_bf16x2(a0, a1), pack_bf16x2(a2, a3), pack_bf16x2(a4, a5), pack_bf16x2(a6, a7));
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&stg_full[grp]);
      }
      ++ti;
    }
#undef CFK_P8_WAIT
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// x [m, 128], w [slots, 128, n] (n a multiple of 128, slots * n <= 512), out [m, slots * n] bf16.  Returns
// CFK_ERR_UNSUPPORTED for what the general engine should take instead.
int ln_proj128_launch(const void* x, const float* ln_scale, const float* ln_offset, const void* w, const void* keep,
                      int keep_dtype, void* out, int64_t m, int slots, int n, float eps, cudaStream_t st) {
  if (n % kNC8 != 0 || slots <= 0 || int64_t(slots) * n > kMaxChunks8 * kNC8 || m > INT32_MAX) return CFK_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(w) || !aligned16(out)) return CFK_ERR_UNSUPPORTED;
  Proj8Params prm{ln_scale, ln_offset, static_cast<__nv_bfloat16*>(out), m, int64_t(slots) * n, slots * (n / kNC8), n / kNC8, eps,
                  keep, keep_dtype, device_status_word()};
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  CUtensorMap tx, tw, to;
  {
    uint64_t dims[2] = {uint64_t(kK8), uint64_t(m)};
    uint64_t str[1] = {uint64_t(kK8) * 2};
    uint32_t box[2] = {64, kRows8};
    int rc = make_tensor_map(&tx, x, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  {
    uint64_t dims[3] = {uint64_t(n), uint64_t(kK8), uint64_t(slots)};
    uint64_t str[2] = {uint64_t(n) * 2, uint64_t(kK8) * uint64_t(n) * 2};
    uint32_t box[3] = {64, kK8, 1};
    int rc = make_tensor_map(&tw, w, CFK_BF16, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  {
    uint64_t dims[2] = {uint64_t(prm.ldo), uint64_t(m)};
    uint64_t str[1] = {uint64_t(prm.ldo) * 2};
    uint32_t box[2] = {64, kRows8};
    int rc = make_tensor_map(&to, out, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  if (cudaFuncSetAttribute(ln_proj128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem8) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ntiles = (m + kRows8 - 1) / kRows8;
  const int grid = int(ntiles < sms ? ntiles : sms);
  if (keep != nullptr && (ntiles + grid - 1) / grid > kMaxTiles8) return CFK_ERR_UNSUPPORTED;
  ln_proj128_kernel<<<grid, kThreads8, kSmem8, st>>>(tx, tw, to, prm);
  return check_launch();
}

}  // namespace cfk
