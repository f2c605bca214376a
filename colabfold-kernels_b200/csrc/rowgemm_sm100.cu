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
constexpr int kThreadsRg = 640;  // 4 control warps, 8 prologue warps, 2 x 4 epilogue warps
constexpr int kAtom = kRows * 128;  // one 64-column K-major atom of an A tile: 16 KB

struct Layout {  // byte offsets inside the (1024-aligned) dynamic shared memory, computed on the host
  int w[2];        // weights of accumulator i: [chunk][atom][K rows][128 B]
  int w_chunk[2];  // bytes per chunk
  int a[2];        // tile of source i inside a stage (TMA lands here; LayerNorm rewrites it in place)
  int a_bytes[2];  // bytes TMA writes for source i
  int stage0;      // first stage
  int stage_bytes;
  int nstages;
  int o0;          // ring of output staging buffers (a residual chunk lands here first and is updated in place)
  int o_bytes;     // bytes per buffer
  int o_arr;       // bytes per output array inside a buffer (two arrays when both accumulators are outputs)
  int no;          // buffers in the ring (1 or 2)
  int cls;         // int8 [kMaxTilesPerCta] tile classes when rows may be skipped, else -1
  int bars;
  int tmem;
  int total;
};

struct KernelArgs {
  RowGemmParams p;
  Layout l;
  int64_t ntiles, tiles_per_outer;
  int direct[2];  // channel-major source i is gathered with plain loads instead of TMA
  int stream_w;   // weights do not stay resident: chunk cc uses slot cc % 2 of a two-chunk ring, refilled from L2
  int out_tma;    // outputs leave through the staging ring and TMA stores (else straight from registers)
  int resid_tma;  // 0: none (or plain loads); 1: residual chunk by TMA (map tr); 2: raw rows of source 1 by TMA (map tx1)
};

constexpr int kMaxStages = 4;
constexpr int kMaxTilesPerCta = 1024;  // with row-block skipping: tile classes of one CTA live in shared memory

__device__ __forceinline__ float act_sigmoid(float x) { return sigmoid_fast(x); }

// Compile-time shape of one kernel variant (each is a separate, small instruction stream):
//   MODE   RowGemmMode;  DUAL  two accumulators per chunk
//   SRC0   source 0 is 0: row-major, 1: channel-major bf16 by TMA, 2: channel-major fp32 by TMA, 3: channel-major by plain loads
//   OUT    0: row-major through the staging ring, 1: channel-major through the staging ring, 2: straight from registers
//   E4M3   outputs are e4m3 (else bf16)
//   KEEP   row-block skipping compiled in (a variant without it keeps the epilogue's registers free)
template <int MODE, int DUAL, int SRC0, int OUT, int E4M3, int KEEP>
__global__ void __launch_bounds__(kThreadsRg, 1)
rowgemm_kernel(const __grid_constant__ CUtensorMap tw0, const __grid_constant__ CUtensorMap tw1,
               const __grid_constant__ CUtensorMap tx0, const __grid_constant__ CUtensorMap tx1,
               const __grid_constant__ CUtensorMap to0, const __grid_constant__ CUtensorMap to1,
               const __grid_constant__ CUtensorMap tr, const KernelArgs ka) {
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
  uint64_t* w_full = bars;                       // weights resident
  uint64_t* raw_full = bars + 1;                 // [kMaxStages] TMA tile landed
  uint64_t* a_full = raw_full + kMaxStages;      // [kMaxStages] tile is a valid UMMA operand
  uint64_t* a_empty = a_full + kMaxStages;       // [kMaxStages] MMAs reading the stage have completed
  uint64_t* acc_full = a_empty + kMaxStages;     // [2]
  uint64_t* acc_empty = acc_full + 2;            // [2]
  uint64_t* o_full = acc_empty + 2;              // [2] residual chunk landed in the staging buffer
  uint64_t* o_empty = o_full + 2;                // [2] the TMA store out of the buffer has read it
  uint64_t* ws_full = o_empty + 2;               // [2] streamed weights: chunk landed in ring slot
  uint64_t* ws_empty = ws_full + 2;              // [2] ... and the MMAs reading it have completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.tmem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsrc = p.src[1].x != nullptr ? 2 : 1;
  constexpr int nacc = DUAL ? 2 : 1;
  const int NS = L.nstages, NO = L.no;

  if (threadIdx.x == 0) {
    mbar_init(w_full, 1);
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&a_full[i], 8);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], L.no == 2 ? 4 : 8);  // the epilogue warps that read one accumulator: one group or both
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 1);
      mbar_init(&ws_full[i], 1);
      mbar_init(&ws_empty[i], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tw0);
    tma_prefetch_desc(&tx0);
    if (DUAL) tma_prefetch_desc(&tw1);
    if (nsrc == 2) tma_prefetch_desc(&tx1);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // Row-block skipping: the class of every tile this CTA will visit (1 compute, 0 padding, -1 leave unwritten), worked
  // out once by all warps so that every role takes the same decision.
  const int8_t* cls = nullptr;
  if (KEEP && L.cls >= 0) {
    int8_t* w = reinterpret_cast<int8_t*>(smem + L.cls);
    for (int i = warp;; i += kThreadsRg / 32) {
      const int64_t tile = blockIdx.x + int64_t(i) * gridDim.x;
      if (tile >= ka.ntiles) break;
      const int64_t o = tile / ka.tiles_per_outer;
      const int64_t r0 = (tile % ka.tiles_per_outer) * kRows;
      float top = -1.f;
      for (int j = lane; j < kRows; j += 32) {
        const int64_t r = r0 + j;
        float v = -1.f;  // rows past the padded extent
        if (r < p.inner) {
          const int64_t row = o * p.src[0].stride_outer + r * p.src[0].stride_inner;
          v = p.keep_dtype == CFK_F32 ? static_cast<const float*>(p.keep)[row]
                                      : __bfloat162float(static_cast<const __nv_bfloat16*>(p.keep)[row]);
        } else if (r < p.inner_pad) {
          v = 0.f;
        }
        top = fmaxf(top, v);
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

  if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 40;");
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer: weights once, then row tiles
    if (lane == 0) {
      const int atoms = p.n_chunk / 64;
      uint32_t bytes = 0;
      for (int i = 0; i < nacc; ++i) bytes += uint32_t(p.chunks) * L.w_chunk[i];
      if (!ka.stream_w) mbar_arrive_expect_tx(w_full, bytes);
      for (int i = 0; i < nacc && !ka.stream_w; ++i) {
        const int kw = p.src[(i == 1 && nsrc == 2) ? 1 : 0].k;
        for (int c = 0; c < p.chunks; ++c) {
          const int cg = p.chunk0 + c;
          const int slot = cg / p.chunks_per_slot;
          const int col = (cg % p.chunks_per_slot) * p.n_chunk;
          for (int a = 0; a < atoms; ++a)
            tma_load_3d(smem + L.w[i] + c * L.w_chunk[i] + a * kw * 128, i == 0 ? &tw0 : &tw1, w_full, col + a * 64, 0, slot);
        }
      }
      uint32_t it = 0, ti = 0;
      for (int64_t tile = blockIdx.x; tile < ka.ntiles; tile += gridDim.x, ++ti) {
        if (KEEP && cls != nullptr && cls[ti] != 1) continue;
        const int stage = it % NS;
        if (!mbar_wait_deadline(&a_empty[stage], ((it / NS) & 1) ^ 1)) { report_timeout(p.status, 906); break; }
        ++it;
        const int o = int(tile / ka.tiles_per_outer);
        const int r0 = int(tile % ka.tiles_per_outer) * kRows;
        uint8_t* base = smem + L.stage0 + stage * L.stage_bytes;
        mbar_arrive_expect_tx(&raw_full[stage], uint32_t(L.a_bytes[0] + (nsrc == 2 ? L.a_bytes[1] : 0)));
        for (int s = 0; s < nsrc; ++s) {
          const CUtensorMap* tm = s == 0 ? &tx0 : &tx1;
          if (s == 0 && SRC0 == 3) continue;
          if (s == 0 && SRC0 != 0) {
            tma_load_2d(base + L.a[s], tm, &raw_full[stage], o * int(p.inner) + r0, 0);
          } else {
            for (int a = 0; a < p.src[s].k / 64; ++a)
              tma_load_3d(base + L.a[s] + a * kAtom, tm, &raw_full[stage], a * 64, r0, o);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(kRows, uint32_t(p.n_chunk), 1, 1, 0, 1);
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      bool ok = ka.stream_w ? true : mbar_wait_deadline(w_full, 0);
      if (!ok) report_timeout(p.status, 901);
      uint32_t it = 0, cc = 0, ti = 0;
      for (int64_t tile = blockIdx.x; tile < ka.ntiles && ok; tile += gridDim.x, ++ti) {
        if (KEEP && cls != nullptr && cls[ti] != 1) continue;
        const int stage = it % NS;
        ok = mbar_wait_deadline(&a_full[stage], (it / NS) & 1);
        if (!ok) { report_timeout(p.status, 902); break; }
        ++it;
        for (int c = 0; c < p.chunks && ok; ++c, ++cc) {
          const int buf = cc & 1;
          ok = mbar_wait_deadline(&acc_empty[buf], ((cc >> 1) & 1) ^ 1);
          if (!ok) { report_timeout(p.status, 903); break; }
          const int wslot = ka.stream_w ? int(cc & 1) : c;  // streamed: ring slot of this chunk
          if (ka.stream_w) {
            ok = mbar_wait_deadline(&ws_full[wslot], (cc >> 1) & 1);
            if (!ok) { report_timeout(p.status, 909); break; }
          }
          tc_fence_after();
          for (int i = 0; i < nacc; ++i) {
            const int s = (i == 1 && nsrc == 2) ? 1 : 0;
            const int kw = p.src[s].k;
            const uint32_t a_lo = desc_lo(smem_u32(smem + L.stage0 + stage * L.stage_bytes + L.a[s]), 16);
            const uint32_t w_lo = desc_lo(smem_u32(smem + L.w[i] + wslot * L.w_chunk[i]), uint32_t(kw) * 128);
            const uint32_t d = tmem + buf * 256 + i * 128;
            // one 64-column atom of A per outer iteration, four K = 16 steps inside it
            uint32_t al = a_lo, wl = w_lo;
#pragma unroll 1
            for (int at = 0; at < kw / 64; ++at, al += kAtom >> 4, wl += 512) {
#pragma unroll
              for (int q = 0; q < 4; ++q) mma_f16_ss2(d, al + q * 2, hi, wl + q * 128, hi, idesc, (at | q) != 0);
            }
          }
          if (ka.stream_w) mma_commit(&ws_empty[wslot]);
          mma_commit(&acc_full[buf]);
        }
        if (ok) mma_commit(&a_empty[stage]);
      }
    }
    __syncwarp();
  } else if (warp == 3) {
    // ------------------------------------------------------------------ weight streamer: chunk -> two-slot ring (from L2)
    if (lane == 0 && ka.stream_w) {
      const int atoms = p.n_chunk / 64;
      uint32_t cc = 0, ti = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < ka.ntiles && ok; tile += gridDim.x, ++ti) {
        if (KEEP && cls != nullptr && cls[ti] != 1) continue;
        for (int c = 0; c < p.chunks; ++c, ++cc) {
          const int wslot = cc & 1;
          if (!mbar_wait_deadline(&ws_empty[wslot], ((cc >> 1) & 1) ^ 1)) { report_timeout(p.status, 910); ok = false; break; }
          uint32_t bytes = 0;
          for (int i = 0; i < nacc; ++i) bytes += L.w_chunk[i];
          mbar_arrive_expect_tx(&ws_full[wslot], bytes);
          const int cg = p.chunk0 + c;
          const int slot = cg / p.chunks_per_slot;
          const int col = (cg % p.chunks_per_slot) * p.n_chunk;
          for (int i = 0; i < nacc; ++i) {
            const int kw = p.src[(i == 1 && nsrc == 2) ? 1 : 0].k;
            for (int a = 0; a < atoms; ++a)
              tma_load_3d(smem + L.w[i] + wslot * L.w_chunk[i] + a * kw * 128, i == 0 ? &tw0 : &tw1, &ws_full[wslot], col + a * 64, 0,
                          slot);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------------ residual producer: chunk -> staging buffer
    if (lane == 0 && ka.resid_tma != 0) {
      const CUtensorMap* tm = ka.resid_tma == 1 ? &tr : &tx1;
      const int atoms = p.n_chunk / 64;
      uint32_t cc = 0, ti = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < ka.ntiles && ok; tile += gridDim.x, ++ti) {
        if (KEEP && cls != nullptr && cls[ti] != 1) continue;
        const int o = int(tile / ka.tiles_per_outer);
        const int r0 = int(tile % ka.tiles_per_outer) * kRows;
        for (int c = 0; c < p.chunks; ++c, ++cc) {
          const int ob = cc % NO;
          if (!mbar_wait_deadline(&o_empty[ob], ((cc / NO) & 1) ^ 1)) { report_timeout(p.status, 907); ok = false; break; }
          const int ocol = ((p.chunk0 + c) % p.chunks_per_array) * p.n_chunk;
          mbar_arrive_expect_tx(&o_full[ob], uint32_t(atoms) * kAtom);
          for (int a = 0; a < atoms; ++a)
            tma_load_3d(smem + L.o0 + ob * L.o_bytes + a * kAtom, tm, &o_full[ob], ocol + a * 64, r0, o);
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------------ prologue: turn landed tiles into UMMA operands
    // Two adjacent lanes share a row: lane bit 0 picks the 16-byte chunks 0-3 or 4-7 of every 64-column atom (for a
    // channel-major source the even or odd 8-channel groups), and the halves combine their LayerNorm statistics by
    // shuffle (pairwise mean / sum of squared deviations).
    // register budgets: 128 x 40 + 256 x (104 + 112) stays inside the 640 x 96 the CTA is launched with
    asm volatile("setmaxnreg.inc.sync.aligned.u32 104;");
    const int pt = (warp - 4) * 32 + lane;
    const int trow = pt >> 1, half = pt & 1;
    bool ok = true;
    uint32_t it = 0, ti = 0;
    for (int64_t tile = blockIdx.x; tile < ka.ntiles; tile += gridDim.x, ++ti) {
      if (KEEP && cls != nullptr && cls[ti] != 1) continue;
      const int stage = it % NS;
      if (ok && !mbar_wait_deadline(&raw_full[stage], (it / NS) & 1)) {
        report_timeout(p.status, 904);
        ok = false;
      }
      ++it;
      const int64_t o = tile / ka.tiles_per_outer;
      const int64_t r = (tile % ka.tiles_per_outer) * kRows + trow;
      const bool valid = r < p.inner;
      uint8_t* base = smem + L.stage0 + stage * L.stage_bytes;
      bool wrote = false;
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        if (s >= nsrc) break;
        const RowSource& src = p.src[s];
        uint8_t* dst = base + L.a[s];
        const float* lns = src.ln_scale;
        const float* lno = src.ln_offset;
        const int K = src.k;
        const float inv_k = 1.f / K;
        if (s == 1 || SRC0 == 0) {
          // The TMA tile already is the K-major swizzled operand; rows past the end arrive as zeros and stay zeros.
          if (src.ln_scale == nullptr) continue;
          wrote = true;
          // my chunk j (0 .. K/16-1) is chunk (j & 3) + 4 * half of atom j >> 2
          // four independent partial sums keep the adds from forming one dependent chain
          float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
          for (int j = 0; j < K / 16; ++j) {
            const uint4 w = *reinterpret_cast<const uint4*>(dst + (j >> 2) * kAtom + swz_off(trow, (j & 3) + 4 * half, 128));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) ps[e] += bf16lo_to_f32(ww[e]) + bf16hi_to_f32(ww[e]);
          }
          const float mean_h = ((ps[0] + ps[1]) + (ps[2] + ps[3])) * (2.f * inv_k);
          float pm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
          for (int j = 0; j < K / 16; ++j) {
            const uint4 w = *reinterpret_cast<const uint4*>(dst + (j >> 2) * kAtom + swz_off(trow, (j & 3) + 4 * half, 128));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float a = bf16lo_to_f32(ww[e]) - mean_h, b = bf16hi_to_f32(ww[e]) - mean_h;
              pm[e] = fmaf(a, a, fmaf(b, b, pm[e]));
            }
          }
          const float m2 = (pm[0] + pm[1]) + (pm[2] + pm[3]);
          const float mean_o = __shfl_xor_sync(0xffffffffu, mean_h, 1), m2_o = __shfl_xor_sync(0xffffffffu, m2, 1);
          const float mean = 0.5f * (mean_h + mean_o);
          const float dm = mean_h - mean_o;
          const float var = (m2 + m2_o) * inv_k + 0.25f * dm * dm;
          const float rstd = rsqrtf(var + p.eps);
          if (valid) {
#pragma unroll 2
            for (int j = 0; j < K / 16; ++j) {
              const int c = (j >> 2) * 8 + (j & 3) + 4 * half;  // chunk of the row
              uint4* slot = reinterpret_cast<uint4*>(dst + (j >> 2) * kAtom + swz_off(trow, (j & 3) + 4 * half, 128));
              const uint4 w = *slot;
              uint32_t ww[4] = {w.x, w.y, w.z, w.w};
              const float4 s0 = __ldg(reinterpret_cast<const float4*>(lns + c * 8)), s1 = __ldg(reinterpret_cast<const float4*>(lns + c * 8 + 4));
              const float4 o0 = __ldg(reinterpret_cast<const float4*>(lno + c * 8)), o1 = __ldg(reinterpret_cast<const float4*>(lno + c * 8 + 4));
              const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
              const float of[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float a = fmaf((bf16lo_to_f32(ww[e]) - mean) * rstd, sc[2 * e], of[2 * e]);
                const float b = fmaf((bf16hi_to_f32(ww[e]) - mean) * rstd, sc[2 * e + 1], of[2 * e + 1]);
                ww[e] = pack_bf16x2(a, b);
              }
              *slot = make_uint4(ww[0], ww[1], ww[2], ww[3]);
            }
          }
        } else {
          // channel-major source [K, rows], K <= 128: the tile landed as [K][128 rows]; each thread gathers its half
          // of a row (the 8-channel groups g with g & 1 == half), normalises it and, once every thread holds its
          // values, the tile is rewritten in place as the K-major operand.
          wrote = true;
          // a bf16 tile is held as packed pairs (32 registers), anything else as floats
          constexpr bool packed = SRC0 == 1;
          float v[packed ? 1 : 64];
          uint32_t vp[packed ? 32 : 1];
          if (packed) {
            const unsigned short* raw = reinterpret_cast<const unsigned short*>(dst) + trow;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int k = (i >> 2) * 16 + half * 8 + (i & 3) * 2;  // even channel of the pair
              vp[i] = k < K ? uint32_t(raw[k * kRows]) | (uint32_t(raw[(k + 1) * kRows]) << 16) : 0u;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 64; ++i) {
              const int k = (i >> 3) * 16 + half * 8 + (i & 7);  // channel
              float t = 0.f;
              if (k < K) {
                if (SRC0 == 3) {
                  const int64_t m = o * p.inner + r, mtot = p.outer * p.inner;
                  if (valid)
                    t = src.dtype == CFK_F32 ? static_cast<const float*>(src.x)[int64_t(k) * mtot + m]
                                             : __bfloat162float(static_cast<const __nv_bfloat16*>(src.x)[int64_t(k) * mtot + m]);
                } else {
                  t = reinterpret_cast<const float*>(dst)[k * kRows + trow];
                }
              }
              v[i] = t;
            }
          }
          auto val = [&](int i) -> float {
            if (packed) return (i & 1) ? bf16hi_to_f32(vp[i >> 1]) : bf16lo_to_f32(vp[i >> 1]);
            return v[i];
          };
          float mean = 0.f, rstd = 1.f;
          if (src.ln_scale != nullptr) {
            float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < 64; ++i) ps[i & 3] += val(i);
            const float mean_h = ((ps[0] + ps[1]) + (ps[2] + ps[3])) * (2.f * inv_k);
            float pm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < 64; ++i) {
              const float d = ((i >> 3) * 16 + half * 8 + (i & 7)) < K ? val(i) - mean_h : 0.f;
              pm[i & 3] = fmaf(d, d, pm[i & 3]);
            }
            const float m2 = (pm[0] + pm[1]) + (pm[2] + pm[3]);
            const float mean_o = __shfl_xor_sync(0xffffffffu, mean_h, 1), m2_o = __shfl_xor_sync(0xffffffffu, m2, 1);
            mean = 0.5f * (mean_h + mean_o);
            const float dm = mean_h - mean_o;
            rstd = rsqrtf((m2 + m2_o) * inv_k + 0.25f * dm * dm + p.eps);
          }
          named_bar_sync(2, 256);
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const int c = 2 * g + half;  // 8-channel group = 16-byte chunk of the row
            if (c * 8 < K) {
              uint32_t ww[4];
              float sc[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f}, of[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
              if (src.ln_scale != nullptr) {
                const float4 s0 = __ldg(reinterpret_cast<const float4*>(lns + c * 8)), s1 = __ldg(reinterpret_cast<const float4*>(lns + c * 8 + 4));
                const float4 o0 = __ldg(reinterpret_cast<const float4*>(lno + c * 8)), o1 = __ldg(reinterpret_cast<const float4*>(lno + c * 8 + 4));
                sc[0] = s0.x; sc[1] = s0.y; sc[2] = s0.z; sc[3] = s0.w; sc[4] = s1.x; sc[5] = s1.y; sc[6] = s1.z; sc[7] = s1.w;
                of[0] = o0.x; of[1] = o0.y; of[2] = o0.z; of[3] = o0.w; of[4] = o1.x; of[5] = o1.y; of[6] = o1.z; of[7] = o1.w;
              }
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float a = fmaf((val(g * 8 + 2 * e) - mean) * rstd, sc[2 * e], of[2 * e]);
                const float b = fmaf((val(g * 8 + 2 * e + 1) - mean) * rstd, sc[2 * e + 1], of[2 * e + 1]);
                ww[e] = valid ? pack_bf16x2(a, b) : 0u;
              }
              *reinterpret_cast<uint4*>(dst + (c >> 3) * kAtom + swz_off(trow, c & 7, 128)) = make_uint4(ww[0], ww[1], ww[2], ww[3]);
            }
          }
        }
      }
      if (wrote) fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[stage]);
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------------ epilogue
    if (SRC0 != 0) {
      asm volatile("setmaxnreg.inc.sync.aligned.u32 104;");
    } else {
      asm volatile("setmaxnreg.inc.sync.aligned.u32 112;");
    }
    // Two groups of four warps.  With two staging buffers they take the chunks in turn (group = accumulator buffer =
    // staging buffer = chunk parity): while one group waits for its accumulator, its residual or its store, the other
    // is in its arithmetic.  With one staging buffer (or none) they share every chunk: group g takes the 32-column
    // pieces g, g + 2.
    const bool alt = NO == 2;
    const int quad = warp & 3, trow = quad * 32 + lane, grp = (warp - 12) >> 2;
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    bool ok = true;
    uint32_t cc = 0;
    constexpr bool two_out = MODE == kModeLinear && DUAL;
    constexpr int nouts = two_out ? 2 : 1;
    constexpr bool staged = OUT != 2;
    const bool out_cm = OUT == 1 || (OUT == 2 && p.out_channel_major);
    const bool row_add_direct = !staged && !out_cm && (p.residual != nullptr || p.add_source1);
    uint32_t ti = 0;
    for (int64_t tile = blockIdx.x; tile < ka.ntiles; tile += gridDim.x, ++ti) {
      const int64_t o = tile / ka.tiles_per_outer;
      const int r0 = int(tile % ka.tiles_per_outer) * kRows;
      const int64_t r = r0 + trow;
      const bool valid = r < p.inner;
      const int64_t src_row = o * p.src[0].stride_outer + r * p.src[0].stride_inner;
      const int64_t out_row = o * p.inner + r;
      if (KEEP && cls != nullptr && cls[ti] != 1) {
        // A padding tile gets its result without any of the work, straight from these threads (group g takes the
        // chunks of its parity): zeros, or the rows that would have been added.  A tile below zero is left alone.
        if (cls[ti] == 0) {
          for (int c = grp; c < p.chunks; c += 2) {
            const int cg = p.chunk0 + c;
            const int ocol = (cg % p.chunks_per_array) * p.n_chunk;
            for (int i = 0; i < nouts; ++i) {
              const int a_idx = two_out ? i : cg / p.chunks_per_array;
              if (p.out[a_idx] == nullptr) continue;
              if (out_cm) {
                if (r >= p.inner_pad) continue;
                const int64_t plane = p.outer * p.inner_pad;
                for (int j = 0; j < p.n_chunk && ocol + j < p.n_valid; ++j) {
                  if (E4M3) static_cast<uint8_t*>(p.out[a_idx])[int64_t(ocol + j) * plane + o * p.inner_pad + r] = 0;
                  else static_cast<__nv_bfloat16*>(p.out[a_idx])[int64_t(ocol + j) * plane + o * p.inner_pad + r] = __float2bfloat16_rn(0.f);
                }
              } else if (valid) {
                const __nv_bfloat16* add_row =
                    p.residual != nullptr ? static_cast<const __nv_bfloat16*>(p.residual) + out_row * p.ldo
                    : p.add_source1 ? static_cast<const __nv_bfloat16*>(p.src[1].x) +
                                          (o * p.src[1].stride_outer + r * p.src[1].stride_inner) * p.src[1].k
                                    : nullptr;
                for (int j = 0; j < p.n_chunk && ocol + j < p.n_valid; j += 8) {
                  if (E4M3) {
                    *reinterpret_cast<uint2*>(static_cast<uint8_t*>(p.out[a_idx]) + out_row * p.ldo + ocol + j) = make_uint2(0, 0);
                  } else {
                    const uint4 v = add_row != nullptr && i == 0 ? *reinterpret_cast<const uint4*>(add_row + ocol + j) : make_uint4(0, 0, 0, 0);
                    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out[a_idx]) + out_row * p.ldo + ocol + j) = v;
                  }
                }
              }
            }
          }
        }
        continue;
      }
      float mk = valid ? 1.f : 0.f;
      if (p.rowmask != nullptr && valid) {
        const float m = p.rowmask_dtype == CFK_F32 ? static_cast<const float*>(p.rowmask)[src_row]
                                                   : __bfloat162float(static_cast<const __nv_bfloat16*>(p.rowmask)[src_row]);
        mk = fmaxf(m, 0.f);
      }
      for (int c = 0; c < p.chunks; ++c, ++cc) {
        const int buf = cc & 1;
        if (alt && buf != grp) continue;  // the other group's chunk
        const int sub0 = alt ? 0 : grp, dsub = alt ? 1 : 2;
        const int cg = p.chunk0 + c;
        const int bcol = (cg / p.chunks_per_slot) * p.bias_slot_stride + (cg % p.chunks_per_slot) * p.n_chunk;  // bias index
        const int arr = two_out ? 0 : cg / p.chunks_per_array;
        const int ocol = (cg % p.chunks_per_array) * p.n_chunk;
        const int ob = cc % NO;
        uint8_t* obuf = smem + L.o0 + ob * L.o_bytes;
        // unstaged path: rows added to the result are fetched with plain loads, one 32-column piece ahead of use
        const __nv_bfloat16* rowp = nullptr;
        if (row_add_direct && valid)
          rowp = p.residual != nullptr
                     ? static_cast<const __nv_bfloat16*>(p.residual) + out_row * p.ldo + ocol
                     : static_cast<const __nv_bfloat16*>(p.src[1].x) +
                           (o * p.src[1].stride_outer + r * p.src[1].stride_inner) * p.src[1].k + ocol;
        uint4 nxt[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          nxt[q] = make_uint4(0, 0, 0, 0);
          if (rowp != nullptr && ocol + sub0 * 32 + q * 8 < p.n_valid) nxt[q] = *reinterpret_cast<const uint4*>(rowp + sub0 * 32 + q * 8);
        }
        if (ok && !mbar_wait_deadline(&acc_full[buf], (cc >> 1) & 1)) {
          report_timeout(p.status, 905);
          ok = false;
        }
        const bool landed = ka.resid_tma != 0;
        if (staged) {
          // The staging buffer is ours once its residual chunk has landed or, without one, once the store that last
          // used it has read it: with two buffers that store is this group's own previous one (its issuer waits and
          // the group meets), with one buffer o_empty says so.
          if (landed || !alt) {
            if (ok && !mbar_wait_deadline(landed ? &o_full[ob] : &o_empty[ob], landed ? (cc / NO) & 1 : ((cc / NO) & 1) ^ 1)) {
              report_timeout(p.status, 908);
              ok = false;
            }
          } else {
            if (trow == 0) tma_wait_group_read<0>();
            named_bar_sync(3 + grp, 128);
          }
        }
        tc_fence_after();
#pragma unroll 1
        for (int sub = sub0; sub < p.n_chunk / 32; sub += dsub) {
          float y[2][32];
          uint4 add[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            add[q] = nxt[q];
            const int cq = (sub + dsub) * 32 + q * 8;
            nxt[q] = make_uint4(0, 0, 0, 0);
            if (rowp != nullptr && cq < p.n_chunk && ocol + cq < p.n_valid) nxt[q] = *reinterpret_cast<const uint4*>(rowp + cq);
          }
          tmem_ld_x32(tmem + lane_addr + buf * 256 + sub * 32, reinterpret_cast<uint32_t(&)[32]>(y[0]));
          if (DUAL) tmem_ld_x32(tmem + lane_addr + buf * 256 + 128 + sub * 32, reinterpret_cast<uint32_t(&)[32]>(y[1]));
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            if (i == 1 && !DUAL) break;
            if (p.bias[i] == nullptr) continue;
            const __nv_bfloat16* b = static_cast<const __nv_bfloat16*>(p.bias[i]) + bcol + sub * 32;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (bcol + sub * 32 + q * 8 >= p.bias_len) break;
              const uint4 t = __ldg(reinterpret_cast<const uint4*>(b + q * 8));
              const uint32_t ww[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                y[i][q * 8 + 2 * e] += bf16lo_to_f32(ww[e]);
                y[i][q * 8 + 2 * e + 1] += bf16hi_to_f32(ww[e]);
              }
            }
          }
          if (MODE == kModeGdp) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float g = y[1][j];
              const float a = p.swish ? g * act_sigmoid(g) : act_sigmoid(g);
              y[0][j] = mk * y[0][j] * a;
            }
          } else if (MODE == kModeEpi) {
#pragma unroll
            for (int j = 0; j < 32; ++j) y[0][j] = valid ? y[0][j] * act_sigmoid(y[1][j]) : 0.f;
          } else {
            const float floor = p.relu ? 0.f : -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              y[0][j] = fmaxf(y[0][j], floor) * mk;
              if (DUAL) y[1][j] *= mk;
            }
          }
          if (row_add_direct) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 t = add[q];
              const uint32_t ww[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                y[0][q * 8 + 2 * e] += bf16lo_to_f32(ww[e]);
                y[0][q * 8 + 2 * e + 1] += bf16hi_to_f32(ww[e]);
              }
            }
          }
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            if (i >= nouts) break;
            const int a_idx = two_out ? i : arr;
            const int col = ocol + sub * 32;
            if (!ok || p.out[a_idx] == nullptr) continue;
            if (staged) {
              uint8_t* oa = obuf + i * L.o_arr;
              if (OUT == 1) {
                // [n_chunk channels][128 rows]: lanes write consecutive rows of one channel
                if (E4M3) {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    oa[(sub * 32 + j) * kRows + trow] =
                        uint8_t(__nv_cvt_float2_to_fp8x2(make_float2(y[i][j] * p.out_scale, 0.f), __NV_SATFINITE, __NV_E4M3) & 0xff);
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    reinterpret_cast<__nv_bfloat16*>(oa)[(sub * 32 + j) * kRows + trow] = __float2bfloat16_rn(y[i][j]);
                }
              } else {
                // [64-column atoms][128 rows][128 B], 128-byte swizzle; a landed residual chunk is updated in place
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const int cq = sub * 32 + q * 8;
                  uint4* slot = reinterpret_cast<uint4*>(oa + (cq >> 6) * kAtom + swz_off(trow, (cq & 63) >> 3, 128));
                  if (ka.resid_tma != 0) {
                    const uint4 t = *slot;
                    const uint32_t ww[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                      y[i][q * 8 + 2 * e] += bf16lo_to_f32(ww[e]);
                      y[i][q * 8 + 2 * e + 1] += bf16hi_to_f32(ww[e]);
                    }
                  }
                  *slot = make_uint4(pack_bf16x2(y[i][q * 8], y[i][q * 8 + 1]), pack_bf16x2(y[i][q * 8 + 2], y[i][q * 8 + 3]),
                                     pack_bf16x2(y[i][q * 8 + 4], y[i][q * 8 + 5]), pack_bf16x2(y[i][q * 8 + 6], y[i][q * 8 + 7]));
                }
              }
            } else if (out_cm) {
              // [n, outer, inner_pad]: lanes write consecutive rows of one channel
              if (r < p.inner_pad) {
                const int64_t plane = p.outer * p.inner_pad;
                if (E4M3) {
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
              if (E4M3) {
                uint8_t* dst = static_cast<uint8_t*>(p.out[a_idx]) + out_row * p.ldo + col;
                auto two = [&](int j) {
                  return uint32_t(__nv_cvt_float2_to_fp8x2(make_float2(y[i][j] * p.out_scale, y[i][j + 1] * p.out_scale),
                                                           __NV_SATFINITE, __NV_E4M3));
                };
                // 16 values per 16-byte store when the row allows it (pitch and column count in whole 16-byte pieces)
                const bool wide = (p.ldo % 16 == 0) && (p.n_valid % 16 == 0) && (reinterpret_cast<uintptr_t>(p.out[a_idx]) % 16 == 0);
#pragma unroll
                for (int j = 0; j < 32; j += 16) {
                  if (wide) {
                    if (col + j < p.n_valid)
                      *reinterpret_cast<uint4*>(dst + j) =
                          make_uint4(two(j) | (two(j + 2) << 16), two(j + 4) | (two(j + 6) << 16), two(j + 8) | (two(j + 10) << 16),
                                     two(j + 12) | (two(j + 14) << 16));
                  } else {
#pragma unroll
                    for (int jj = j; jj < j + 16; jj += 2)
                      if (col + jj < p.n_valid) *reinterpret_cast<uint16_t*>(dst + jj) = uint16_t(two(jj));
                  }
                }
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
        if (staged) {
          fence_proxy_async();
          if (alt) named_bar_sync(3 + grp, 128);
          else named_bar_sync(3, 256);
          if (trow == 0 && (alt || grp == 0)) {
            if (ok) {
              for (int i = 0; i < nouts; ++i) {
                const int a_idx = two_out ? i : arr;
                if (p.out[a_idx] == nullptr) continue;
                const CUtensorMap* tm = a_idx == 0 ? &to0 : &to1;
                if (OUT == 1) {
                  tma_store_3d(tm, obuf + i * L.o_arr, r0, int(o), ocol);
                } else {
                  for (int a = 0; a < p.n_chunk / 64; ++a)
                    if (ocol + a * 64 < p.n_valid) tma_store_3d(tm, obuf + i * L.o_arr + a * kAtom, ocol + a * 64, r0, int(o));
                }
              }
            }
            tma_commit_group();
            if (landed || !alt) {  // o_empty is waited for: by the residual producer, or by both groups (one buffer)
              tma_wait_group_read<0>();
              mbar_arrive(&o_empty[ob]);
            }
          }
        }
      }
    }
    if (staged && trow == 0) tma_wait_group<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

namespace {

// Bytes of one pipeline stage and whether a channel-major source must be gathered with plain loads (its row pitch or
// base address does not meet the 16-byte rule of TMA); bytes of one output staging buffer and whether the outputs can
// leave through it.
struct Plan {
  int a[2], a_bytes[2], stage_bytes;
  int direct[2];
  int out_tma, resid_tma, o_arr, o_bytes;
};

bool ptr_aligned16(const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; }

Plan make_plan(const RowGemmParams& p) {
  Plan s{};
  const int nsrc = p.src[1].x != nullptr ? 2 : 1;
  int off = 0;
  for (int i = 0; i < nsrc; ++i) {
    const RowSource& src = p.src[i];
    const int operand = (src.k / 64) * kAtom;
    int landed = operand;
    if (src.channel_major) {
      const int es = src.dtype == CFK_F32 ? 4 : 2;
      const int64_t mtot = p.outer * p.inner;
      s.direct[i] = ((mtot * es) % 16 != 0) || !ptr_aligned16(src.x);
      landed = s.direct[i] ? 0 : src.k * kRows * es;
    }
    s.a[i] = off;
    s.a_bytes[i] = landed;
    off += ((landed > operand ? landed : operand) + 1023) & ~1023;
  }
  s.stage_bytes = off;
  const bool two_out = p.mode == kModeLinear && p.dual;
  const int es = p.out_dtype == CFK_E4M3 ? 1 : 2;
  bool ok = ptr_aligned16(p.out[0]) && (p.out[1] == nullptr || ptr_aligned16(p.out[1]));
  if (p.out_channel_major) {
    ok = ok && (p.inner_pad * es) % 16 == 0;
    s.o_arr = p.n_chunk * kRows * es;
  } else {
    ok = ok && p.out_dtype == CFK_BF16 && (p.ldo * es) % 16 == 0;
    s.o_arr = (p.n_chunk / 64) * kAtom;
  }
  s.out_tma = ok;
  s.o_bytes = ok ? (two_out ? 2 : 1) * s.o_arr : 0;
  s.o_bytes = (s.o_bytes + 1023) & ~1023;
  if (ok && !p.out_channel_major && !two_out) {
    if (p.residual != nullptr && ptr_aligned16(p.residual)) s.resid_tma = 1;
    if (p.residual == nullptr && p.add_source1) s.resid_tma = 2;
  }
  return s;
}

constexpr int kSmemBudget = 232448;
constexpr int kSmemFixed = 1024 /*alignment slack*/ + 25 * 8 + 32;

}  // namespace

int rowgemm_chunks_that_fit(const RowGemmParams& p) {
  const int nsrc = p.src[1].x != nullptr ? 2 : 1;
  const int k0 = p.src[0].k, k1 = nsrc == 2 ? p.src[1].k : k0;
  const Plan sp = make_plan(p);
  const int per_chunk = (p.n_chunk / 64) * 128 * (k0 + (p.dual ? k1 : 0));
  // two stages keep loads in flight behind the math
  const int fixed = kSmemFixed + (p.keep != nullptr ? kMaxTilesPerCta : 0);
  int fit = (kSmemBudget - fixed - 2 * sp.stage_bytes - sp.o_bytes) / per_chunk;
  if (fit < 1) fit = (kSmemBudget - fixed - sp.stage_bytes - sp.o_bytes) / per_chunk;
  return fit;
}

// With `chunks` chunk weights resident, is there no room left for two stages and two output staging buffers while the
// two-slot weight ring would leave it?
bool rowgemm_resident_is_tight(const RowGemmParams& p, int chunks) {
  const int nsrc = p.src[1].x != nullptr ? 2 : 1;
  const int k0 = p.src[0].k, k1 = nsrc == 2 ? p.src[1].k : k0;
  const Plan sp = make_plan(p);
  const int per_chunk = (p.n_chunk / 64) * 128 * (k0 + (p.dual ? k1 : 0));
  const int fixed = kSmemFixed + (p.keep != nullptr ? kMaxTilesPerCta : 0);
  const int want = 2 * sp.stage_bytes + 2 * sp.o_bytes;
  return sp.o_bytes > 0 && kSmemBudget - fixed - chunks * per_chunk < want && kSmemBudget - fixed - 2 * per_chunk >= want;
}

bool rowgemm_stream_fits(const RowGemmParams& p) {
  const int nsrc = p.src[1].x != nullptr ? 2 : 1;
  const int k0 = p.src[0].k, k1 = nsrc == 2 ? p.src[1].k : k0;
  const Plan sp = make_plan(p);
  const int per_chunk = (p.n_chunk / 64) * 128 * (k0 + (p.dual ? k1 : 0));
  const int fixed = kSmemFixed + (p.keep != nullptr ? kMaxTilesPerCta : 0);
  return kSmemBudget - fixed - 2 * per_chunk - sp.stage_bytes - sp.o_bytes >= 0;
}

int launch_rowgemm(const RowGemmParams& prm, const CUtensorMap& tw0, const CUtensorMap& tw1, cudaStream_t st) {
  KernelArgs ka{};
  ka.p = prm;
  const RowGemmParams& p = ka.p;
  const int nsrc = p.src[1].x != nullptr ? 2 : 1;
  const int nacc = p.dual ? 2 : 1;
  ka.tiles_per_outer = (p.inner_pad + kRows - 1) / kRows;
  ka.ntiles = p.outer * ka.tiles_per_outer;
  if (ka.ntiles == 0) return CFK_OK;
  for (int i = 0; i < nsrc; ++i)
    if (p.src[i].ln_scale != nullptr && (!ptr_aligned16(p.src[i].ln_scale) || !ptr_aligned16(p.src[i].ln_offset))) return CFK_ERR_ALIGN;
  for (int i = 0; i < nacc; ++i)
    if (p.bias[i] != nullptr && !ptr_aligned16(p.bias[i])) return CFK_ERR_ALIGN;
  int off = 0;
  ka.stream_w = prm.stream_weights;
  for (int i = 0; i < 2; ++i) {
    const int kw = p.src[(i == 1 && nsrc == 2) ? 1 : 0].k;
    ka.l.w[i] = off;
    ka.l.w_chunk[i] = (p.n_chunk / 64) * kw * 128;
    if (i < nacc) off += (ka.stream_w ? 2 : p.chunks) * ka.l.w_chunk[i];
  }
  const Plan sp = make_plan(p);
  for (int i = 0; i < 2; ++i) {
    ka.l.a[i] = sp.a[i];
    ka.l.a_bytes[i] = sp.a_bytes[i];
    ka.direct[i] = sp.direct[i];
  }
  ka.out_tma = sp.out_tma;
  ka.resid_tma = sp.resid_tma;
  // shared memory: weights, then as many stages as fit (at least one), a second staging buffer before a third stage
  const int room = kSmemBudget - kSmemFixed - off - (p.keep != nullptr ? kMaxTilesPerCta : 0);
  int ns = 0, no = sp.out_tma ? 1 : 0;
  if (room >= 2 * sp.stage_bytes + 2 * sp.o_bytes) {
    no = sp.out_tma ? 2 : 0;
    ns = (room - no * sp.o_bytes) / sp.stage_bytes;
  } else {
    ns = (room - no * sp.o_bytes) / sp.stage_bytes;
  }
  if (ns < 1) return CFK_ERR_UNSUPPORTED;
  if (ns > kMaxStages) ns = kMaxStages;
  ka.l.stage0 = off;
  ka.l.stage_bytes = sp.stage_bytes;
  ka.l.nstages = ns;
  off += ns * sp.stage_bytes;
  ka.l.o0 = off;
  ka.l.o_bytes = sp.o_bytes;
  ka.l.o_arr = sp.o_arr;
  ka.l.no = no > 0 ? no : 1;
  off += no * sp.o_bytes;
  ka.l.bars = off;
  ka.l.tmem = ka.l.bars + 25 * 8;
  ka.l.cls = -1;
  int end = ka.l.tmem + 16;
  if (p.keep != nullptr) {
    ka.l.cls = end;
    end += kMaxTilesPerCta;
  }
  ka.l.total = end + 1024;
  if (ka.l.total > kSmemBudget) return CFK_ERR_UNSUPPORTED;

  // tensor maps of the sources, the outputs and the residual
  CUtensorMap tx[2], to[2], tr;
  for (int i = 0; i < 2; ++i) {
    const int si = i < nsrc ? i : 0;
    const RowSource& src = p.src[si];
    int rc;
    if (src.channel_major) {
      if (sp.direct[si]) {
        tx[i] = tw0;  // never used
        continue;
      }
      const int es = src.dtype == CFK_F32 ? 4 : 2;
      const uint64_t mtot = uint64_t(p.outer * p.inner);
      uint64_t dims[2] = {mtot, uint64_t(src.k)};
      uint64_t strides[1] = {mtot * es};
      uint32_t box[2] = {uint32_t(kRows), uint32_t(src.k)};
      rc = make_tensor_map(&tx[i], src.x, src.dtype, 2, dims, strides, box, 0);
    } else {
      if (!ptr_aligned16(src.x)) return CFK_ERR_ALIGN;
      const uint64_t row = uint64_t(src.k) * 2;
      uint64_t dims[3] = {uint64_t(src.k), uint64_t(p.inner), uint64_t(p.outer)};
      uint64_t strides[2] = {uint64_t(src.stride_inner) * row,
                             (p.outer > 1 ? uint64_t(src.stride_outer) : uint64_t(p.inner) * uint64_t(src.stride_inner)) * row};
      uint32_t box[3] = {64, uint32_t(kRows), 1};
      rc = make_tensor_map(&tx[i], src.x, CFK_BF16, 3, dims, strides, box, 128);
    }
    if (rc != CFK_OK) return rc;
  }
  to[0] = to[1] = tr = tw0;
  if (sp.out_tma) {
    const uint64_t es = p.out_dtype == CFK_E4M3 ? 1 : 2;
    for (int i = 0; i < 2; ++i) {
      if (p.out[i] == nullptr) continue;
      int rc;
      if (p.out_channel_major) {
        uint64_t dims[3] = {uint64_t(p.inner_pad), uint64_t(p.outer), uint64_t(p.n_valid)};
        uint64_t strides[2] = {uint64_t(p.inner_pad) * es, uint64_t(p.outer) * uint64_t(p.inner_pad) * es};
        uint32_t box[3] = {uint32_t(kRows), 1, uint32_t(p.n_chunk)};
        rc = make_tensor_map(&to[i], p.out[i], p.out_dtype, 3, dims, strides, box, 0);
      } else {
        uint64_t dims[3] = {uint64_t(p.n_valid), uint64_t(p.inner), uint64_t(p.outer)};
        uint64_t strides[2] = {uint64_t(p.ldo) * es, uint64_t(p.inner) * uint64_t(p.ldo) * es};
        uint32_t box[3] = {64, uint32_t(kRows), 1};
        rc = make_tensor_map(&to[i], p.out[i], CFK_BF16, 3, dims, strides, box, 128);
        if (rc == CFK_OK && i == 0 && sp.resid_tma == 1) rc = make_tensor_map(&tr, p.residual, CFK_BF16, 3, dims, strides, box, 128);
      }
      if (rc != CFK_OK) return rc;
    }
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = int(ka.ntiles < sms ? ka.ntiles : sms);
  if (p.keep != nullptr && (ka.ntiles + grid - 1) / grid > kMaxTilesPerCta) return CFK_ERR_UNSUPPORTED;
  const int src0 = !p.src[0].channel_major ? 0 : sp.direct[0] ? 3 : p.src[0].dtype == CFK_F32 ? 2 : 1;
  const int out = !sp.out_tma ? 2 : p.out_channel_major ? 1 : 0;
  const int e4m3 = p.out_dtype == CFK_E4M3;
  const int key = ((((p.mode * 2) + (p.dual ? 1 : 0)) * 4 + src0) * 3 + out) * 2 + e4m3;
  const int keep = p.keep != nullptr;
  int rc = CFK_ERR_UNSUPPORTED;
  // KEEP = 1 variants take any call; where a KEEP = 0 twin exists it serves the calls without row-block skipping
#define CFK_RG_VARIANT(MODE, DUAL, SRC0, OUT, E4M3, KEEP, ALSO_PLAIN)                                                  \
  if (rc != CFK_OK && key == (((((MODE)*2) + (DUAL)) * 4 + (SRC0)) * 3 + (OUT)) * 2 + (E4M3) &&                         \
      (keep == (KEEP) || ((KEEP) == 1 && !(ALSO_PLAIN)))) {                                                            \
    auto kern = rowgemm_kernel<MODE, DUAL, SRC0, OUT, E4M3, KEEP>;                                                     \
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, ka.l.total) != cudaSuccess)            \
      return CFK_ERR_LAUNCH;                                                                                           \
    /* the in-kernel register re-split must fit the registers the CTA is launched with, or it would wait forever */  \
    cudaFuncAttributes fa;                                                                                             \
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess || fa.numRegs * kThreadsRg < 128 * 40 + 256 * (104 + 112))    \
      return CFK_ERR_LAUNCH;                                                                                           \
    kern<<<grid, kThreadsRg, ka.l.total, st>>>(tw0, tw1, tx[0], tx[1], to[0], to[1], tr, ka);                          \
    rc = CFK_OK;                                                                                                       \
  }
  // gated dual projection (with or without LayerNorm): row-major or channel-major outputs, bf16 or e4m3
  CFK_RG_VARIANT(kModeGdp, 1, 0, 0, 0, 1, 0)
  CFK_RG_VARIANT(kModeGdp, 1, 0, 1, 0, 1, 0)
  CFK_RG_VARIANT(kModeGdp, 1, 0, 1, 1, 1, 0)
  CFK_RG_VARIANT(kModeGdp, 1, 0, 2, 0, 1, 0)
  CFK_RG_VARIANT(kModeGdp, 1, 0, 2, 1, 1, 0)
  // triangle-multiplication epilogue: channel-major contraction result
  CFK_RG_VARIANT(kModeEpi, 1, 1, 0, 0, 0, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 1, 0, 0, 1, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 2, 0, 0, 0, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 2, 0, 0, 1, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 3, 0, 0, 0, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 3, 0, 0, 1, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 1, 2, 0, 0, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 1, 2, 0, 1, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 2, 2, 0, 0, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 2, 2, 0, 1, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 3, 2, 0, 0, 1)
  CFK_RG_VARIANT(kModeEpi, 1, 3, 2, 0, 1, 1)
  // single projections (LayerNorm -> projection, head bias, output projection)
  CFK_RG_VARIANT(kModeLinear, 0, 0, 0, 0, 0, 1)
  CFK_RG_VARIANT(kModeLinear, 0, 0, 0, 0, 1, 1)
  CFK_RG_VARIANT(kModeLinear, 0, 0, 1, 0, 0, 1)
  CFK_RG_VARIANT(kModeLinear, 0, 0, 1, 0, 1, 1)
  CFK_RG_VARIANT(kModeLinear, 0, 0, 2, 0, 0, 1)
  CFK_RG_VARIANT(kModeLinear, 0, 0, 2, 0, 1, 1)
  CFK_RG_VARIANT(kModeLinear, 0, 0, 2, 1, 0, 1)
  CFK_RG_VARIANT(kModeLinear, 0, 0, 2, 1, 1, 1)
  // two projections of one normed tile (outer-product-mean projection)
  CFK_RG_VARIANT(kModeLinear, 1, 0, 0, 0, 0, 1)
  CFK_RG_VARIANT(kModeLinear, 1, 0, 2, 0, 0, 1)
#undef CFK_RG_VARIANT
  if (rc != CFK_OK) return rc;
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
