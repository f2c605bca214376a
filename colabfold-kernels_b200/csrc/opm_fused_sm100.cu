// Fused deep outer product mean for sm_100a: out[i, j, :] = ((sum_s a[s, i, :] (x) b[s, j, :]) . w + bias) / (eps + norm[i, j])
// (+ residual), with the outer product kept on chip (src/colabfold_kernels/opm.py:122-162 `opm_outer` never writes the
// product either: per left channel c it forms g = l_c^T r, rounds it to the input type and multiplies by w[c*E:(c+1)*E]).
//
// Operands arrive channel-major with the MSA depth contiguous: left [32, ri, s'], right [32, rj, s'] (what
// cfk_opm_projection_cm writes), so that both are K-major GEMM operands straight from TMA.
//
// A persistent CTA walks tiles of 16 residues i x 8 residues j.  Per tile and per group q of 8 left channels:
//   first GEMM   G[(a', i), (b, j')] = sum_s left[q*8 + a', i, s] right[b, j', s]      M = 128, N = 256, K = depth
//   drain        thread (a', i) rounds its 256 values to bf16 and writes them as row (j', i), columns a'*32 + b of a
//                [128][256] K-major tile in shared memory: the (i, j) pairs become rows, the (a, b) pairs the
//                contracted axis, without a transpose through lanes (a thread only moves its own values)
//   second GEMM  acc2[(j', i), f] += tile . w[q*256 : (q+1)*256, f]                     M = 128, N = 128, K = 256
// and per tile the epilogue (bias, normaliser, residual, bf16) straight from TMEM to global memory.
// TMEM columns: G [0, 256), acc2 [256, 384).  Warps: 0 operand producer, 1 first-GEMM issuer, 2 second-GEMM issuer,
// 3 weight producer, 4-11 two worker groups (column halves).  Every mbarrier wait is deadline-bounded.
#include "attention_sm100.cuh"

namespace cfk {
namespace {

constexpr int kTI = 16;                 // residues i per tile
constexpr int kTJ = 8;                  // residues j per tile
constexpr int kCh = 32;                 // channels of each projection
constexpr int kQ = 4;                   // groups of 8 left channels
constexpr int kF = 128;                 // output channels
constexpr int kThreadsO = 384;
constexpr int kStageA = 128 * 128;      // [a' * 16 + i][64 s] bf16
constexpr int kStageB = 256 * 128;      // [b * 8 + j'][64 s] bf16
constexpr int kStageBytes = kStageA + kStageB;
constexpr int kStagesO = 3;
constexpr int kOffA2 = kStagesO * kStageBytes;   // [4 atoms of 64 columns][128 rows][128 B]
constexpr int kA2Bytes = 4 * 128 * 128;
constexpr int kOffWr = kOffA2 + kA2Bytes;        // ring of two weight pieces [32 k][128 f] as two 64-column atoms
constexpr int kWPiece = 32 * 128 * 2;
constexpr int kOffBarO = kOffWr + 2 * kWPiece;
constexpr int kNumBarsO = 2 * kStagesO + 4 + 4 + 2;
constexpr int kOffTmemO = kOffBarO + kNumBarsO * 8;
constexpr int kSmemO = kOffTmemO + 16 + 1024;
static_assert(kSmemO <= 232448, "shared memory budget");
constexpr int kColAcc2O = 256;

struct OpmParams {
  const __nv_bfloat16* bias;      // [128]
  const float* norm;              // [ri, rj]
  const __nv_bfloat16* residual;  // [ri, rj, 128] or null
  __nv_bfloat16* out;             // [ri, rj, 128]
  int ri, rj, depth;
  float eps;
  int* status;
};

__global__ void __launch_bounds__(kThreadsO, 1)
opm_fused_kernel(const __grid_constant__ CUtensorMap tm_l, const __grid_constant__ CUtensorMap tm_r,
                 const __grid_constant__ CUtensorMap tm_w, const OpmParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBarO);
  uint64_t* full = bars;                 // [3] operand stage landed
  uint64_t* empty = full + kStagesO;     // [3] ... and read by its MMAs
  uint64_t* g_full = empty + kStagesO;   // the first GEMM of a channel group has completed
  uint64_t* g_empty = g_full + 1;        // ... and every worker has read it out of TMEM
  uint64_t* a2_full = g_empty + 1;       // the rounded product is in shared memory
  uint64_t* a2_empty = a2_full + 1;      // ... and the second GEMM has read it
  uint64_t* w_full = a2_empty + 1;       // [2]
  uint64_t* w_empty = w_full + 2;        // [2]
  uint64_t* acc2_full = w_empty + 2;
  uint64_t* acc2_empty = acc2_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemO);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntj = (prm.rj + kTJ - 1) / kTJ;
  const int64_t ntiles = int64_t((prm.ri + kTI - 1) / kTI) * ntj;
  const int nks = (prm.depth + 63) / 64;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStagesO; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(g_full, 1);
    mbar_init(g_empty, 8);
    mbar_init(a2_full, 8);
    mbar_init(a2_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 1);
    }
    mbar_init(acc2_full, 1);
    mbar_init(acc2_empty, 8);
    fence_mbar_init();
    tma_prefetch_desc(&tm_l);
    tma_prefetch_desc(&tm_r);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ operand producer
    if (lane == 0) {
      bool ok = true;
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int i0 = int(tile / ntj) * kTI, j0 = int(tile % ntj) * kTJ;
        for (int q = 0; q < kQ && ok; ++q) {
          for (int ks = 0; ks < nks; ++ks, ++it) {
            const int stage = it % kStagesO;
            ok = mbar_wait_deadline(&empty[stage], ((it / kStagesO) & 1) ^ 1);
            if (!ok) { report_timeout(prm.status, 1401); break; }
            uint8_t* base = smem + stage * kStageBytes;
            mbar_arrive_expect_tx(&full[stage], kStageBytes);
            // rows a' * 16 + i of the left operand, rows b * 8 + j' of the right one; depth past the end reads zeros
            tma_load_3d(base, &tm_l, &full[stage], ks * 64, i0, q * 8);
            tma_load_3d(base + kStageA, &tm_r, &full[stage], ks * 64, j0, 0);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 3) {
    // ------------------------------------------------------------------ weight producer: pieces of 32 rows of w
    if (lane == 0) {
      bool ok = true;
      uint32_t wc = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        for (int p = 0; p < kQ * 8 && ok; ++p, ++wc) {
          const int slot = wc & 1;
          ok = mbar_wait_deadline(&w_empty[slot], ((wc >> 1) & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 1402); break; }
          uint8_t* base = smem + kOffWr + slot * kWPiece;
          mbar_arrive_expect_tx(&w_full[slot], kWPiece);
          tma_load_2d(base, &tm_w, &w_full[slot], 0, p * 32);
          tma_load_2d(base + kWPiece / 2, &tm_w, &w_full[slot], 64, p * 32);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ first GEMM: G = left_q . right^T over the depth
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(128, 256, 1, 1, 0, 0);
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      bool ok = true;
      uint32_t it = 0, gc = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        for (int q = 0; q < kQ && ok; ++q, ++gc) {
          ok = mbar_wait_deadline(g_empty, (gc & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 1403); break; }
          tc_fence_after();
          for (int ks = 0; ks < nks; ++ks, ++it) {
            const int stage = it % kStagesO;
            ok = mbar_wait_deadline(&full[stage], (it / kStagesO) & 1);
            if (!ok) { report_timeout(prm.status, 1404); break; }
            tc_fence_after();
            const uint32_t a = desc_lo(smem_u32(smem + stage * kStageBytes), 16);
            const uint32_t b = desc_lo(smem_u32(smem + stage * kStageBytes + kStageA), 16);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) mma_f16_ss2(tmem, a + kk * 2, hi, b + kk * 2, hi, idesc, (ks | kk) != 0);
            mma_commit(&empty[stage]);
          }
          if (ok) mma_commit(g_full);
        }
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------------ second GEMM: acc2 += rounded product . w_q
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(128, kF, 1, 1, 0, 1);   // A K-major, B = w piece MN-major
      constexpr uint32_t hi = desc_hi(1024, kSwz128);
      const uint32_t a2 = desc_lo(smem_u32(smem + kOffA2), 16);
      bool ok = true;
      uint32_t ti = 0, gc = 0, wc = 0;
      for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++ti) {
        ok = mbar_wait_deadline(acc2_empty, (ti & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 1405); break; }
        for (int q = 0; q < kQ && ok; ++q, ++gc) {
          ok = mbar_wait_deadline(a2_full, gc & 1);
          if (!ok) { report_timeout(prm.status, 1406); break; }
          for (int p = 0; p < 8; ++p, ++wc) {
            const int slot = wc & 1;
            ok = mbar_wait_deadline(&w_full[slot], (wc >> 1) & 1);
            if (!ok) { report_timeout(prm.status, 1407); break; }
            tc_fence_after();
            // piece p: columns [p * 32, p * 32 + 32) of the tile = atom p / 2, 64 bytes into its rows for odd p
            const uint32_t a = a2 + (p >> 1) * ((128 * 128) >> 4) + (p & 1) * 4;
            const uint32_t b = desc_lo(smem_u32(smem + kOffWr + slot * kWPiece), kWPiece / 2);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) mma_f16_ss2(tmem + kColAcc2O, a + kk * 2, hi, b + kk * 128, hi, idesc, (q | p | kk) != 0);
            mma_commit(&w_empty[slot]);
          }
          if (ok) mma_commit(a2_empty);
        }
        if (ok) mma_commit(acc2_full);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ workers
    const int g = (warp - 4) >> 2;   // column half
    const int quad = warp & 3;
    const int row = quad * 32 + lane;                 // TMEM lane
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const int ap = row >> 4, il = row & 15;           // first GEMM: lane = a' * 16 + i
    const int jl = row >> 4;                          // second GEMM: lane = j' * 16 + i
    bool ok = true;
#define CFK_OPM_WAIT(bar, parity, code)                           \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    uint32_t ti = 0, gc = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++ti) {
      const int i0 = int(tile / ntj) * kTI, j0 = int(tile % ntj) * kTJ;
      for (int q = 0; q < kQ; ++q, ++gc) {
        CFK_OPM_WAIT(g_full, gc & 1, 1408)
        CFK_OPM_WAIT(a2_empty, (gc & 1) ^ 1, 1409)
        tc_fence_after();
#pragma unroll 1
        for (int rd = 0; rd < 2; ++rd) {
          // 64 columns = right channels b0 .. b0 + 7 (column = b * 8 + j')
          uint32_t r0[32], r1[32];
          tmem_ld_x32(tmem + lane_addr + g * 128 + rd * 64, r0);
          tmem_ld_x32(tmem + lane_addr + g * 128 + rd * 64 + 32, r1);
          tmem_wait_ld();
          if (rd == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(g_empty);
          }
          // row (j', i) of the tile, columns a' * 32 + b0 .. + 7: atom a' / 2, 16-byte piece (a' % 2) * 4 + b0 / 8
          const int piece = (ap & 1) * 4 + g * 2 + rd;
          uint8_t* atom = smem + kOffA2 + (ap >> 1) * (128 * 128);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 v = make_uint4(
                pack_bf16x2(__uint_as_float(r0[j]), __uint_as_float(r0[8 + j])),
                pack_bf16x2(__uint_as_float(r0[16 + j]), __uint_as_float(r0[24 + j])),
                pack_bf16x2(__uint_as_float(r1[j]), __uint_as_float(r1[8 + j])),
                pack_bf16x2(__uint_as_float(r1[16 + j]), __uint_as_float(r1[24 + j])));
            *reinterpret_cast<uint4*>(atom + swz_off(j * 16 + il, piece, 128)) = v;
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(a2_full);
      }
      // ---- the tile's result: (acc2 + bias) / (eps + norm) (+ residual), thread = pair (i, j'), this group's 64 columns
      const int gi = i0 + il, gj = j0 + jl;
      const bool valid = gi < prm.ri && gj < prm.rj;
      const int64_t pair = int64_t(gi) * prm.rj + gj;
      const float inv = valid ? 1.0f / (prm.eps + __ldg(prm.norm + pair)) : 0.f;
      // the residual row is fetched before the wait for the second GEMM, so that its latency runs under that wait
      uint4 xpre[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        xpre[u] = make_uint4(0, 0, 0, 0);
        if (valid && prm.residual != nullptr) xpre[u] = *reinterpret_cast<const uint4*>(prm.residual + pair * kF + g * 64 + u * 8);
      }
      CFK_OPM_WAIT(acc2_full, ti & 1, 1410)
      tc_fence_after();
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {
        uint32_t r[32];
        tmem_ld_x32(tmem + lane_addr + kColAcc2O + g * 64 + cb * 32, r);
        tmem_wait_ld();
        if (cb == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc2_empty);
        }
        if (valid && ok) {
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const int col = g * 64 + cb * 32 + ch * 8;
            const uint4 bw = __ldg(reinterpret_cast<const uint4*>(prm.bias + col));
            const uint32_t bb[4] = {bw.x, bw.y, bw.z, bw.w};
            const uint4 xw = xpre[cb * 4 + ch];
            const uint32_t xx[4] = {xw.x, xw.y, xw.z, xw.w};
            uint32_t y[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              y[e] = pack_bf16x2(fmaf(__uint_as_float(r[ch * 8 + 2 * e]) + bf16lo_to_f32(bb[e]), inv, bf16lo_to_f32(xx[e])),
                                 fmaf(__uint_as_float(r[ch * 8 + 2 * e + 1]) + bf16hi_to_f32(bb[e]), inv, bf16hi_to_f32(xx[e])));
            *reinterpret_cast<uint4*>(prm.out + pair * kF + col) = make_uint4(y[0], y[1], y[2], y[3]);
          }
        }
      }
    }
#undef CFK_OPM_WAIT
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// norm[i, j] = sum_s ml[s, i] mr[s, j] in fp32 (the mask overlap count the mean divides by): 64 x 64 outputs per block,
// 4 x 4 per thread, the depth in slices of 32 through shared memory.
template <typename T>
__global__ void __launch_bounds__(256) opm_norm_kernel(const T* __restrict__ ml, const T* __restrict__ mr,
                                                       float* __restrict__ norm, int depth, int ri, int rj) {
  __shared__ float sl[32][64], sr[32][64];
  const int i0 = blockIdx.y * 64, j0 = blockIdx.x * 64;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float acc[4][4] = {};
  for (int s0 = 0; s0 < depth; s0 += 32) {
    for (int e = threadIdx.x; e < 32 * 64; e += 256) {
      const int s = s0 + (e >> 6), c = e & 63;
      sl[e >> 6][c] = (s < depth && i0 + c < ri) ? float(ml[int64_t(s) * ri + i0 + c]) : 0.f;
      sr[e >> 6][c] = (s < depth && j0 + c < rj) ? float(mr[int64_t(s) * rj + j0 + c]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int s = 0; s < 32; ++s) {
      float a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a[u] = sl[s][ty * 4 + u];
        b[u] = sr[s][tx * 4 + u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(a[u], b[v], acc[u][v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int i = i0 + ty * 4 + u, j = j0 + tx * 4 + v;
      if (i < ri && j < rj) norm[int64_t(i) * rj + j] = acc[u][v];
    }
}

}  // namespace
}  // namespace cfk

using namespace cfk;

extern "C" int cfk_opm_norm(const void* mask_left, const void* mask_right, int mask_dtype, float* norm, int depth, int ri,
                            int rj, void* stream) {
  if (!mask_left || !mask_right || !norm) return CFK_ERR_NULL;
  if (depth < 0 || ri < 0 || rj < 0) return CFK_ERR_SHAPE;
  if (mask_dtype != CFK_BF16 && mask_dtype != CFK_F32) return CFK_ERR_DTYPE;
  if (ri == 0 || rj == 0) return CFK_OK;
  if (device_status_word() == nullptr) return CFK_ERR_LAUNCH;
  auto st = static_cast<cudaStream_t>(stream);
  dim3 grid((rj + 63) / 64, (ri + 63) / 64);
  if (mask_dtype == CFK_F32)
    opm_norm_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(mask_left), static_cast<const float*>(mask_right),
                                                 norm, depth, ri, rj);
  else
    opm_norm_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(mask_left),
                                                         static_cast<const __nv_bfloat16*>(mask_right), norm, depth, ri, rj);
  return check_launch();
}

extern "C" int cfk_opm_fused(const void* left_cm, const void* right_cm, const void* w, const void* bias, const float* norm,
                             const void* residual, void* out, int ri, int rj, int depth, int64_t pitch, int c, int f,
                             float eps, void* stream) {
  if (!left_cm || !right_cm || !w || !bias || !norm || !out) return CFK_ERR_NULL;
  if (ri < 0 || rj < 0 || depth <= 0 || pitch < depth) return CFK_ERR_SHAPE;
  if (c != kCh || f != kF) return CFK_ERR_UNSUPPORTED;
  if (pitch % 8 != 0) return CFK_ERR_ALIGN;
  if (ri == 0 || rj == 0) return CFK_OK;
  if (!aligned16(left_cm) || !aligned16(right_cm) || !aligned16(w) || !aligned16(bias) || !aligned16(out) ||
      (residual && !aligned16(residual)))
    return CFK_ERR_ALIGN;
  OpmParams prm{static_cast<const __nv_bfloat16*>(bias), norm, static_cast<const __nv_bfloat16*>(residual),
                static_cast<__nv_bfloat16*>(out), ri, rj, depth, eps, device_status_word()};
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  CUtensorMap tl, tr, tw;
  {
    uint64_t dims[3] = {uint64_t(depth), uint64_t(ri), uint64_t(kCh)};
    uint64_t str[2] = {uint64_t(pitch) * 2, uint64_t(ri) * uint64_t(pitch) * 2};
    uint32_t box[3] = {64, kTI, 8};
    int rc = make_tensor_map(&tl, left_cm, CFK_BF16, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  {
    uint64_t dims[3] = {uint64_t(depth), uint64_t(rj), uint64_t(kCh)};
    uint64_t str[2] = {uint64_t(pitch) * 2, uint64_t(rj) * uint64_t(pitch) * 2};
    uint32_t box[3] = {64, kTJ, kCh};
    int rc = make_tensor_map(&tr, right_cm, CFK_BF16, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  {
    uint64_t dims[2] = {uint64_t(kF), uint64_t(kCh * kCh)};
    uint64_t str[1] = {uint64_t(kF) * 2};
    uint32_t box[2] = {64, 32};
    int rc = make_tensor_map(&tw, w, CFK_BF16, 2, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  if (cudaFuncSetAttribute(opm_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemO) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ntiles = int64_t((ri + kTI - 1) / kTI) * ((rj + kTJ - 1) / kTJ);
  const int grid = int(ntiles < sms ? ntiles : sms);
  opm_fused_kernel<<<grid, kThreadsO, kSmemO, static_cast<cudaStream_t>(stream)>>>(tl, tr, tw, prm);
  return check_launch();
}
