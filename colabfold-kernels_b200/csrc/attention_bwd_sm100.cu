// Bias-fused flash attention backward for sm_100a (recompute based): TMA-staged tiles, tcgen05 MMAs, TMEM.
//
// One CTA owns one 128-key block of one head for G = 3 batch rows: their K/V tiles stay in shared memory and
// their dK/dV accumulators stay in TMEM while the CTA sweeps the query blocks.  A "step" is one (query block i,
// batch row g) pair:
//   MMA issuers    warp 1: S = Q K^T and dP = dO V^T into TMEM (one step ahead), then, once the softmax warps have
//                  published P and dS (bf16, shared memory): dV_g += P^T dO, dK_g += dS^T Q; warp 3 (which also
//                  produces the bias tiles) issues dQ = dS K of the same step beside them
//   softmax warps  8 warps, thread = (query row, half of the 128 keys): p = 2^(s*log2e - lse) from the forward's
//                  lse, ds = p * (dp - delta); dBias accumulates over the G batch rows in registers and is
//                  flushed with vector atomics during the block's last step; the previous step's dQ tile goes
//                  TMEM -> shared, from where a reducer warp sends it to the fp32 scratch by TMA reduce-add
// The bias tile is shared by the G steps of a query block.  dK/dV leave TMEM once, at the end.
// TMEM columns: S [0,128) dP [128,256) dQ [256,288) | batch row g: dK [288+64g, +32) dV [320+64g, +32).
// Math: src/colabfold_kernels/tri_flash.py:313-355,380,434-446.
#include "attention_sm100.cuh"

namespace cfk {

void launch_attn_delta_bf16(const AttnBwdProblem& bp, float* delta, cudaStream_t st);

namespace {

constexpr int D = 32;
constexpr int G = 3;
constexpr int kQdoStages = 3;
constexpr int kRowBytes = D * 2;
constexpr int kTile = kBQ * kRowBytes;      // 8 KB: one Q / dO / K / V tile
constexpr int kTileBig = kBQ * kBK * 2;     // 32 KB: bias, P, dS tiles (two 64-key halves of 128-byte rows)
constexpr int kTileDq = kBQ * D * 4;        // 16 KB fp32 staging
constexpr int kOffK = 0;
constexpr int kOffV = kOffK + G * kTile;
constexpr int kOffQ = kOffV + G * kTile;
constexpr int kOffDo = kOffQ + kQdoStages * kTile;
constexpr int kOffBias = kOffDo + kQdoStages * kTile;
constexpr int kOffP = kOffBias + kTileBig;
constexpr int kOffDs = kOffP + kTileBig;
constexpr int kOffDq = kOffDs + kTileBig;               // [2][kTileDq]
constexpr int kOffMask = kOffDq + 2 * kTileDq;          // float [G][128]
constexpr int kOffBar = kOffMask + G * 128 * 4;
constexpr int kNumBars = G + 2 * kQdoStages + 2 + 2 + 2 + 4;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kSmem = kOffTmem + 16 + 1024;
static_assert(kSmem <= 232448, "shared memory budget");
constexpr int kColS = 0, kColDp = 128, kColDq = 256, kColAcc = 288;
constexpr int kThreads = 384;
constexpr int kSoftmaxThreads = 256;

struct BwdParams {
  AttnBwdProblem bp;
  const float* delta;  // [nb, h, sq]
  float* dq_acc;       // [nb, h, sq, D] fp32, zeroed
  int* status;
  int has_bias;
};

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                      const __grid_constant__ CUtensorMap tm_bias, const __grid_constant__ CUtensorMap tm_dq,
                      const BwdParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const AttnProblem& p = prm.bp.f;
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* kv_full = bars;                      // [G]
  uint64_t* qdo_full = kv_full + G;              // [kQdoStages]
  uint64_t* qdo_empty = qdo_full + kQdoStages;   // [kQdoStages]
  uint64_t* bias_full = qdo_empty + kQdoStages;  // [1] (+1 pad)
  uint64_t* bias_empty = bias_full + 1;
  uint64_t* sdp_full = bias_empty + 1;           // S and dP of a step are in TMEM
  uint64_t* sdp_empty = sdp_full + 1;            // ... and have been read into registers
  uint64_t* pds_full = sdp_empty + 1;            // P and dS of a step are in shared memory
  uint64_t* gemm_done = pds_full + 1;            // the three output GEMMs of a step have completed
  uint64_t* dq_staged = gemm_done + 1;           // [2] a dQ tile is in its staging buffer
  uint64_t* dq_free = dq_staged + 2;             // [2] the reduce out of a staging buffer has read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b0 = blockIdx.x * G;
  const int gcount = min(G, p.nb - b0);
  const int k0 = blockIdx.y * kBK;
  const int head = blockIdx.z;
  const int ni = (p.sq + kBQ - 1) / kBQ;
  const int nsteps = ni * gcount;

  if (threadIdx.x == 0) {
    for (int i = 0; i < G; ++i) mbar_init(&kv_full[i], 1);
    for (int i = 0; i < kQdoStages; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    mbar_init(bias_full, 1);
    mbar_init(bias_empty, 8);
    mbar_init(sdp_full, 1);
    mbar_init(sdp_empty, 8);
    mbar_init(pds_full, 8);
    mbar_init(gemm_done, 2);  // the dV/dK issuer and the dQ issuer each commit once per step
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dq_staged[i], 8);
      mbar_init(&dq_free[i], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_bias);
    tma_prefetch_desc(&tm_dq);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 40;");
    if (warp == 0) {
      // ---------------------------------------------------------------- TMA producer
      if (lane == 0) {
        for (int g = 0; g < gcount; ++g) {
          mbar_arrive_expect_tx(&kv_full[g], 2 * kTile);
          tma_load_4d(smem + kOffK + g * kTile, &tm_k, &kv_full[g], 0, k0, head, b0 + g);
          tma_load_4d(smem + kOffV + g * kTile, &tm_v, &kv_full[g], 0, k0, head, b0 + g);
        }
        int step = 0;
        bool ok = true;
        for (int i = 0; i < ni && ok; ++i) {
          for (int g = 0; g < gcount; ++g, ++step) {
            const int st = step % kQdoStages;
            ok = mbar_wait_deadline(&qdo_empty[st], ((step / kQdoStages) & 1) ^ 1);
            if (!ok) { report_timeout(prm.status, 602); break; }
            mbar_arrive_expect_tx(&qdo_full[st], 2 * kTile);
            tma_load_4d(smem + kOffQ + st * kTile, &tm_q, &qdo_full[st], 0, i * kBQ, head, b0 + g);
            tma_load_4d(smem + kOffDo + st * kTile, &tm_do, &qdo_full[st], 0, i * kBQ, head, b0 + g);
          }
        }
      }
      __syncwarp();
    } else if (warp == 3) {
      // ---------------------------------------------------------------- bias tile per query block + the dQ GEMM
      // One thread with two duties it polls for: the bias producer (its own warp, so that waiting for the single bias
      // buffer never holds back the Q / dO prefetch) and a second MMA issuer.  dQ = dS K of a step goes out from here
      // while the other issuer sends dV and dK: small MMAs cost an issuing thread ~58 clocks each whatever their tensor
      // time, two issuing warps ~41.
      if (lane == 0) {
        constexpr uint32_t idesc_q = make_idesc(kBQ, D, 1, 1, 0, 1);     // dQ: A = dS (K-major), B = K (MN-major)
        constexpr uint32_t kTile16 = kTile >> 4;
        constexpr uint32_t hi64 = desc_hi(8 * kRowBytes, kSwz64);
        constexpr uint32_t hi128 = desc_hi(1024, kSwz128);
        const uint32_t k_mn = desc_lo(smem_u32(smem + kOffK), 0);
        const uint32_t ds_k = desc_lo(smem_u32(smem + kOffDs), 16);
        const int nbias = prm.has_bias ? ni : 0;
        int bi = 0, t = 0, g = 0;
        long long t0 = clock64();
        while (bi < nbias || t < nsteps) {
          bool moved = false;
          if (bi < nbias && mbar_test(bias_empty, (bi & 1) ^ 1)) {
            mbar_arrive_expect_tx(bias_full, kTileBig);
            tma_load_3d(smem + kOffBias, &tm_bias, bias_full, k0, bi * kBQ, head);
            tma_load_3d(smem + kOffBias + kTileBig / 2, &tm_bias, bias_full, k0 + 64, bi * kBQ, head);
            ++bi;
            moved = true;
          }
          if (t < nsteps && mbar_test(pds_full, t & 1)) {
            tc_fence_after();
            const uint32_t bk = k_mn + g * kTile16;
            // dQ = dS K: A K-major (64 keys per 128-byte row, second half 16 KB on), a K step is 16 keys
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              mma_f16_ss2(tmem + kColDq, ds_k + (kk / 4) * (kTileBig / 32) + (kk % 4) * 2, hi128, bk + kk * 64, hi64, idesc_q,
                          kk > 0);
            mma_commit(gemm_done);
            ++t;
            if (++g == gcount) g = 0;
            moved = true;
          }
          if (moved) {
            t0 = clock64();
          } else if (clock64() - t0 > (1ll << 30)) {
            report_timeout(prm.status, 601);
            break;
          }
        }
      }
      __syncwarp();
    } else if (warp == 2) {
      // ---------------------------------------------------------------- dQ reducer: staging buffer -> fp32 scratch
      if (lane == 0) {
        for (int tp = 0; tp < nsteps; ++tp) {
          if (!mbar_wait_deadline(&dq_staged[tp & 1], (tp >> 1) & 1)) { report_timeout(prm.status, 603); break; }
          const int ip = tp / gcount, gp = tp - ip * gcount;
          tma_reduce_add_4d(&tm_dq, smem + kOffDq + (tp & 1) * kTileDq, 0, ip * kBQ, head, b0 + gp);
          tma_commit_group();
          tma_wait_group_read<0>();
          mbar_arrive(&dq_free[tp & 1]);
        }
        tma_wait_group<0>();
      }
      __syncwarp();
    } else if (warp == 1) {
      // ---------------------------------------------------------------- MMA issuer
      if (lane == 0) {
        constexpr uint32_t idesc_s = make_idesc(kBQ, kBK, 1, 1, 0, 0);   // S, dP: both operands K-major
        constexpr uint32_t idesc_t = make_idesc(kBK, D, 1, 1, 1, 1);     // dV, dK: A = P^T / dS^T (MN-major), B MN-major
        constexpr uint32_t kTile16 = kTile >> 4;
        // low descriptor words (start address >> 4, leading byte offset); the high words are constants
        constexpr uint32_t hi64 = desc_hi(8 * kRowBytes, kSwz64);   // Q, dO, K, V tiles: 64-byte rows
        constexpr uint32_t hi128 = desc_hi(1024, kSwz128);          // P, dS tiles: 128-byte rows
        const uint32_t q_k = desc_lo(smem_u32(smem + kOffQ), 16), do_k = desc_lo(smem_u32(smem + kOffDo), 16);
        const uint32_t k_k = desc_lo(smem_u32(smem + kOffK), 16), v_k = desc_lo(smem_u32(smem + kOffV), 16);
        const uint32_t q_mn = desc_lo(smem_u32(smem + kOffQ), 0), do_mn = desc_lo(smem_u32(smem + kOffDo), 0);
        const uint32_t k_mn = desc_lo(smem_u32(smem + kOffK), 0);
        const uint32_t p_mn = desc_lo(smem_u32(smem + kOffP), kTileBig / 2);
        const uint32_t ds_mn = desc_lo(smem_u32(smem + kOffDs), kTileBig / 2);
        const uint32_t ds_k = desc_lo(smem_u32(smem + kOffDs), 16);
        int s_g = 0, s_st = 0, o_g = 0, o_st = 0;
        uint32_t s_par = 0, s_first = 1, se_par = 1, pf_par = 0, o_first = 1;
        bool ok = true;
        auto issue_sdp = [&]() {
          if (s_first && !mbar_wait_deadline(&kv_full[s_g], 0)) { report_timeout(prm.status, 701); return false; }
          if (!mbar_wait_deadline(&qdo_full[s_st], s_par)) { report_timeout(prm.status, 702); return false; }
          if (!mbar_wait_deadline(sdp_empty, se_par)) { report_timeout(prm.status, 703); return false; }
          tc_fence_after();
          const uint32_t aq = q_k + s_st * kTile16, ad = do_k + s_st * kTile16;
          const uint32_t bk = k_k + s_g * kTile16, bv = v_k + s_g * kTile16;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) mma_f16_ss2(tmem + kColS, aq + 2 * kk, hi64, bk + 2 * kk, hi64, idesc_s, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) mma_f16_ss2(tmem + kColDp, ad + 2 * kk, hi64, bv + 2 * kk, hi64, idesc_s, kk > 0);
          mma_commit(sdp_full);
          se_par ^= 1;
          if (++s_g == gcount) { s_g = 0; s_first = 0; }
          if (++s_st == kQdoStages) { s_st = 0; s_par ^= 1; }
          return true;
        };
        auto issue_out = [&]() {
          if (!mbar_wait_deadline(pds_full, pf_par)) { report_timeout(prm.status, 704); return false; }
          tc_fence_after();
          const uint32_t bdo = do_mn + o_st * kTile16, bq = q_mn + o_st * kTile16;
          const uint32_t d_k = tmem + kColAcc + o_g * 64, d_v = d_k + 32;
          const uint32_t acc0 = o_first ^ 1;  // the first query block overwrites the dK/dV accumulators
          // dV_g += P^T dO and dK_g += dS^T Q: A MN-major, a K step is 16 query rows = 2048 bytes of P/dS,
          // 1024 bytes of dO/Q
#pragma unroll
          for (int kk = 0; kk < kBQ / 16; ++kk)
            mma_f16_ss2(d_v, p_mn + kk * 128, hi128, bdo + kk * 64, hi64, idesc_t, kk > 0 ? 1u : acc0);
#pragma unroll
          for (int kk = 0; kk < kBQ / 16; ++kk)
            mma_f16_ss2(d_k, ds_mn + kk * 128, hi128, bq + kk * 64, hi64, idesc_t, kk > 0 ? 1u : acc0);
          // (dQ = dS K of the step is issued by the second issuer, warp 3)
          mma_commit(&qdo_empty[o_st]);
          mma_commit(gemm_done);
          pf_par ^= 1;
          if (++o_g == gcount) { o_g = 0; o_first = 0; }
          if (++o_st == kQdoStages) o_st = 0;
          return true;
        };
        ok = issue_sdp();
        for (int t = 0; t < nsteps && ok; ++t) {
          if (t + 1 < nsteps) ok = issue_sdp();
          if (ok) ok = issue_out();
        }
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------------ softmax warps (256 threads)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 232;");
    const int sw = warp - 4;            // 0..7
    const int quad = warp & 3;          // TMEM lane quadrant
    const int half = sw >> 2;           // which 64 keys of the block
    const int row = quad * 32 + lane;   // query row in the tile (S, dP, dQ) and key row (dK, dV epilogue)
    const int stid = threadIdx.x - 128; // 0..255
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    float* mask_all = reinterpret_cast<float*>(smem + kOffMask);
    bool ok = true;
#define CFK_BWD_WAIT(bar, parity, code)                           \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    // additive key masks of the G batch rows for this key block: 0 live, floor masked, -inf past Sk
    for (int idx = stid; idx < gcount * 128; idx += kSoftmaxThreads) {
      const int g = idx >> 7, key = k0 + (idx & 127);
      float add = -INFINITY;
      if (key < p.sk) add = p.kmask[int64_t(b0 + g) * p.sk + key] ? 0.f : kFloorNat;
      mask_all[idx] = add;
    }
    named_bar_sync(1, kSoftmaxThreads);

    const float scale = p.scale;
    float acc[64];  // dBias of this thread's (query row, 64 keys), summed over the G batch rows of a query block
    int t = 0;
    // forward statistics of a step's row, fetched one step ahead of their use (rows past Sq get lse = +inf, which
    // makes p and ds exactly zero)
    auto fetch_stats = [&](int step, float& lse_out, float& dlt_out) {
      lse_out = INFINITY;
      dlt_out = 0.f;
      const int ii = step / gcount, gg = step - ii * gcount, qq = ii * kBQ + row;
      if (step < nsteps && qq < p.sq) {
        const int64_t r = (int64_t(b0 + gg) * p.h + head) * p.sq + qq;
        lse_out = p.lse[r];
        dlt_out = prm.delta[r];
      }
    };
    float lse_next, dlt_next;
    fetch_stats(0, lse_next, dlt_next);
    for (int i = 0; i < ni; ++i) {
      const int q = i * kBQ + row;
#pragma unroll
      for (int c = 0; c < 64; ++c) acc[c] = 0.f;
      if (prm.has_bias) CFK_BWD_WAIT(bias_full, i & 1, 801)
      const bool flush_ok = prm.bp.dbias != nullptr && q < p.sq;
      float* dbias_row = prm.bp.dbias + (int64_t(head) * p.sq + q) * p.sk + k0 + half * 64;
#pragma unroll 1
      for (int g = 0; g < gcount; ++g, ++t) {
        const float lse = lse_next, dlt = dlt_next;
        fetch_stats(t + 1, lse_next, dlt_next);
        CFK_BWD_WAIT(sdp_full, t & 1, 802)
        tc_fence_after();
        const float* madd = mask_all + g * 128 + half * 64;
        const uint8_t* bias_tile = smem + kOffBias + half * (kTileBig / 2);
        // a row whose keys were all masked: the forward was the uniform mean, so p = 1/Sk on every real key and
        // ds = 0.  Handled by rewriting the inputs of the common formula (s := -mask so that s + mask = 0,
        // lse := log2(Sk), dp := delta); whole batch rows are dead or alive, so the branch is warp-uniform.
        const bool dead = lse <= kNegRef * 0.5f;
        const bool any_dead = __any_sync(0xffffffffu, dead);
        const float neg_lse = dead ? -__log2f(float(p.sk)) : -lse;
        uint32_t pk[32], dk[32];
        // two chunks of 32 keys keep the live registers (scores, dP, dBias sums, packed outputs) under the budget
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          float s[32], dp[32];
          tmem_ld_x32(tmem + lane_addr + kColS + half * 64 + hc * 32, reinterpret_cast<uint32_t(&)[32]>(s));
          tmem_ld_x32(tmem + lane_addr + kColDp + half * 64 + hc * 32, reinterpret_cast<uint32_t(&)[32]>(dp));
          tmem_wait_ld();
          if (hc == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sdp_empty);
          }
          // packed fp32 pairs from here on: two keys per FMA-pipe instruction
          const uint64_t scale2 = f2_pack(scale, scale);
          if (prm.has_bias) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint4 w = *reinterpret_cast<const uint4*>(bias_tile + swz_off(row, hc * 4 + c, 128));
              const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float lo, hi;
                f2_unpack(f2_fma(f2_pack(s[c * 8 + 2 * e], s[c * 8 + 2 * e + 1]), scale2,
                                 f2_pack(bf16lo_to_f32(ww[e]), bf16hi_to_f32(ww[e]))), lo, hi);
                s[c * 8 + 2 * e] = lo;
                s[c * 8 + 2 * e + 1] = hi;
              }
            }
            // the last step of a query block has now read the whole bias tile: release it, so that the next block's
            // tile loads behind the rest of this step
            if (hc == 1 && g == gcount - 1) {
              __syncwarp();
              if (lane == 0) mbar_arrive(bias_empty);
            }
          } else {
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              float lo, hi;
              f2_unpack(f2_mul(f2_pack(s[2 * c], s[2 * c + 1]), scale2), lo, hi);
              s[2 * c] = lo;
              s[2 * c + 1] = hi;
            }
          }
          if (any_dead) {
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const float a = madd[hc * 32 + c];
              if (dead) {
                s[c] = a == -INFINITY ? 0.f : -a;
                dp[c] = dlt;
              }
            }
          }
          const uint64_t l2e2 = f2_pack(kLog2eF, kLog2eF), nlse2 = f2_pack(neg_lse, neg_lse), ndlt2 = f2_pack(-dlt, -dlt);
          // Stage by stage over the whole chunk (32 independent elements per stage) instead of element by element:
          // the exponentials and the arithmetic around them then overlap instead of waiting on one another.
#pragma unroll
          for (int c = 0; c < 8; ++c) {  // exponent arguments, in place of the scores
            const float4 a = *reinterpret_cast<const float4*>(madd + hc * 32 + c * 4);
            f2_unpack(f2_fma(f2_add(f2_pack(s[c * 4 + 0], s[c * 4 + 1]), f2_pack(a.x, a.y)), l2e2, nlse2), s[c * 4 + 0], s[c * 4 + 1]);
            f2_unpack(f2_fma(f2_add(f2_pack(s[c * 4 + 2], s[c * 4 + 3]), f2_pack(a.z, a.w)), l2e2, nlse2), s[c * 4 + 2], s[c * 4 + 3]);
          }
#pragma unroll
          for (int c = 0; c < 32; ++c) s[c] = ex2_approx(s[c]);  // p
#pragma unroll
          for (int c = 0; c < 16; ++c)  // ds, in place of dp
            f2_unpack(f2_mul(f2_pack(s[2 * c], s[2 * c + 1]), f2_add(f2_pack(dp[2 * c], dp[2 * c + 1]), ndlt2)), dp[2 * c], dp[2 * c + 1]);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            pk[hc * 16 + c] = pack_bf16x2(s[2 * c], s[2 * c + 1]);
            dk[hc * 16 + c] = pack_bf16x2(dp[2 * c], dp[2 * c + 1]);
          }
          if (g == gcount - 1) {
            // last batch row of the query block: the finished dBias sums leave as vector atomics during the math
#pragma unroll
            for (int c = 0; c < 8; ++c)
              if (flush_ok && k0 + half * 64 + hc * 32 + c * 4 < p.sk)
                red_add_v4(dbias_row + hc * 32 + c * 4, acc[hc * 32 + c * 4 + 0] + dp[c * 4 + 0], acc[hc * 32 + c * 4 + 1] + dp[c * 4 + 1],
                           acc[hc * 32 + c * 4 + 2] + dp[c * 4 + 2], acc[hc * 32 + c * 4 + 3] + dp[c * 4 + 3]);
          } else {
#pragma unroll
            for (int c = 0; c < 16; ++c)
              f2_unpack(f2_add(f2_pack(acc[hc * 32 + 2 * c], acc[hc * 32 + 2 * c + 1]), f2_pack(dp[2 * c], dp[2 * c + 1])),
                        acc[hc * 32 + 2 * c], acc[hc * 32 + 2 * c + 1]);
          }
          if (hc == 0 && t > 0) {
            // the previous step's output GEMMs are complete: its dQ tile can leave TMEM, P/dS can be overwritten
            CFK_BWD_WAIT(gemm_done, (t - 1) & 1, 803)
            tc_fence_after();
            uint32_t r[16];
            tmem_ld_x16(tmem + lane_addr + kColDq + half * 16, r);
            tmem_wait_ld();
            CFK_BWD_WAIT(&dq_free[(t - 1) & 1], (((t - 1) >> 1) & 1) ^ 1, 805)
            // 128-byte rows, 128-byte swizzle (the reduce's tensor map undoes it): conflict-free 16-byte stores
            uint8_t* stg = smem + kOffDq + ((t - 1) & 1) * kTileDq;
#pragma unroll
            for (int c = 0; c < 4; ++c)
              *reinterpret_cast<float4*>(stg + swz_off(row, half * 4 + c, 128)) =
                  make_float4(__uint_as_float(r[c * 4]) * scale, __uint_as_float(r[c * 4 + 1]) * scale,
                              __uint_as_float(r[c * 4 + 2]) * scale, __uint_as_float(r[c * 4 + 3]) * scale);
          }
          // this chunk's P and dS into shared memory (64 keys = one 128-byte swizzled row of this thread's half)
          {
            uint8_t* p_row = smem + kOffP + half * (kTileBig / 2);
            uint8_t* ds_row = smem + kOffDs + half * (kTileBig / 2);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t off = swz_off(row, hc * 4 + c, 128);
              *reinterpret_cast<uint4*>(p_row + off) =
                  make_uint4(pk[hc * 16 + c * 4], pk[hc * 16 + c * 4 + 1], pk[hc * 16 + c * 4 + 2], pk[hc * 16 + c * 4 + 3]);
              *reinterpret_cast<uint4*>(ds_row + off) =
                  make_uint4(dk[hc * 16 + c * 4], dk[hc * 16 + c * 4 + 1], dk[hc * 16 + c * 4 + 2], dk[hc * 16 + c * 4 + 3]);
            }
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          if (t > 0) mbar_arrive(&dq_staged[(t - 1) & 1]);
          mbar_arrive(pds_full);
        }
      }
    }
    // ---------------------------------------------------------------- tail: last dQ tile, then dK / dV
    if (nsteps > 0) {
      CFK_BWD_WAIT(gemm_done, (nsteps - 1) & 1, 804)
      tc_fence_after();
      uint32_t r[16];
      tmem_ld_x16(tmem + lane_addr + kColDq + half * 16, r);
      tmem_wait_ld();
      CFK_BWD_WAIT(&dq_free[(nsteps - 1) & 1], (((nsteps - 1) >> 1) & 1) ^ 1, 806)
      uint8_t* stg = smem + kOffDq + ((nsteps - 1) & 1) * kTileDq;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<float4*>(stg + swz_off(row, half * 4 + c, 128)) =
            make_float4(__uint_as_float(r[c * 4]) * scale, __uint_as_float(r[c * 4 + 1]) * scale,
                        __uint_as_float(r[c * 4 + 2]) * scale, __uint_as_float(r[c * 4 + 3]) * scale);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_staged[(nsteps - 1) & 1]);
      const int key = k0 + row;
      // tcgen05.ld is warp-collective: every lane loads, only the lanes whose key exists store
#pragma unroll 1
      for (int g = 0; g < gcount; ++g) {
        uint32_t rk[16], rv[16];
        tmem_ld_x16(tmem + lane_addr + kColAcc + g * 64 + half * 16, rk);
        tmem_ld_x16(tmem + lane_addr + kColAcc + g * 64 + 32 + half * 16, rv);
        tmem_wait_ld();
        if (ok && key < p.sk) {
          const int b = b0 + g;
          __nv_bfloat16* dk_out = static_cast<__nv_bfloat16*>(prm.bp.dk) + b * prm.bp.sdk.b + head * prm.bp.sdk.h +
                                  int64_t(key) * prm.bp.sdk.s + half * 16;
          __nv_bfloat16* dv_out = static_cast<__nv_bfloat16*>(prm.bp.dv) + b * prm.bp.sdv.b + head * prm.bp.sdv.h +
                                  int64_t(key) * prm.bp.sdv.s + half * 16;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint4 wk, wv;
            wk.x = pack_bf16x2(__uint_as_float(rk[c * 8 + 0]) * scale, __uint_as_float(rk[c * 8 + 1]) * scale);
            wk.y = pack_bf16x2(__uint_as_float(rk[c * 8 + 2]) * scale, __uint_as_float(rk[c * 8 + 3]) * scale);
            wk.z = pack_bf16x2(__uint_as_float(rk[c * 8 + 4]) * scale, __uint_as_float(rk[c * 8 + 5]) * scale);
            wk.w = pack_bf16x2(__uint_as_float(rk[c * 8 + 6]) * scale, __uint_as_float(rk[c * 8 + 7]) * scale);
            wv.x = pack_bf16x2(__uint_as_float(rv[c * 8 + 0]), __uint_as_float(rv[c * 8 + 1]));
            wv.y = pack_bf16x2(__uint_as_float(rv[c * 8 + 2]), __uint_as_float(rv[c * 8 + 3]));
            wv.z = pack_bf16x2(__uint_as_float(rv[c * 8 + 4]), __uint_as_float(rv[c * 8 + 5]));
            wv.w = pack_bf16x2(__uint_as_float(rv[c * 8 + 6]), __uint_as_float(rv[c * 8 + 7]));
            *reinterpret_cast<uint4*>(dk_out + c * 8) = wk;
            *reinterpret_cast<uint4*>(dv_out + c * 8) = wv;
          }
        }
      }
    }
#undef CFK_BWD_WAIT
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dq_acc [nb, h, sq, D] fp32 -> dq in the caller's layout, bf16
__global__ void dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, Strides sdq, int nb,
                                  int h, int sq) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // one thread per 8 elements
  const int64_t total = int64_t(nb) * h * sq * (D / 8);
  if (idx >= total) return;
  const int c = idx % (D / 8);
  const int64_t r = idx / (D / 8);
  const int q = r % sq, hh = (r / sq) % h, b = r / (int64_t(sq) * h);
  const float4 a = *reinterpret_cast<const float4*>(acc + r * D + c * 8);
  const float4 bb = *reinterpret_cast<const float4*>(acc + r * D + c * 8 + 4);
  uint4 w = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(bb.x, bb.y), pack_bf16x2(bb.z, bb.w));
  *reinterpret_cast<uint4*>(dq + b * sdq.b + hh * sdq.h + int64_t(q) * sdq.s + c * 8) = w;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

bool attention_sm100_supported(const AttnProblem& p, int dtype);

bool attention_bwd_sm100_supported(const AttnBwdProblem& bp, int dtype) {
  if (!attention_sm100_supported(bp.f, dtype)) return false;
  if (bp.f.gate != nullptr) return false;
  auto ok16 = [](const void* ptr) { return ptr == nullptr || aligned16(ptr); };
  if (!ok16(bp.dout) || !ok16(bp.dq) || !ok16(bp.dk) || !ok16(bp.dv) || !ok16(bp.dbias)) return false;
  auto st8 = [](const Strides& s) { return s.b % 8 == 0 && s.s % 8 == 0 && s.h % 8 == 0; };
  return st8(bp.sdo) && st8(bp.sdq) && st8(bp.sdk) && st8(bp.sdv) && bp.f.nb <= 3 * 65535;
}

// fp32 dQ accumulator [nb, h, sq, D]
size_t attention_bwd_sm100_workspace(const AttnProblem& p) {
  return align_up(sizeof(float) * size_t(p.nb) * p.h * p.sq * D, 256);
}

// workspace layout handed in by the C entry: delta [nb,h,sq] fp32 (256-aligned) | dq accumulator
int attention_bwd_sm100(const AttnBwdProblem& bp, float* delta, void* workspace, cudaStream_t st) {
  const AttnProblem& p = bp.f;
  float* dq_acc = static_cast<float*>(workspace);
  launch_attn_delta_bf16(bp, delta, st);
  int rc = check_launch();
  if (rc != CFK_OK) return rc;
  if (cudaMemsetAsync(dq_acc, 0, sizeof(float) * size_t(p.nb) * p.h * p.sq * D, st) != cudaSuccess) return CFK_ERR_LAUNCH;
  if (bp.dbias != nullptr &&
      cudaMemsetAsync(bp.dbias, 0, sizeof(float) * size_t(p.h) * p.sq * p.sk, st) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  CUtensorMap tq, tk, tv, tdo, tb, tdq;
  rc = make_qkv_map(&tq, p.q, p.sq_, p.nb, p.h, p.sq, D, kBQ);
  if (rc == CFK_OK) rc = make_qkv_map(&tk, p.k, p.sk_, p.nb, p.h, p.sk, D, kBK);
  if (rc == CFK_OK) rc = make_qkv_map(&tv, p.v, p.sv_, p.nb, p.h, p.sk, D, kBK);
  if (rc == CFK_OK) rc = make_qkv_map(&tdo, bp.dout, bp.sdo, p.nb, p.h, p.sq, D, kBQ);
  if (rc != CFK_OK) return rc;
  if (p.bias != nullptr) {
    uint64_t dims[3] = {uint64_t(p.sk), uint64_t(p.sq), uint64_t(p.h)};
    uint64_t strides[2] = {uint64_t(p.sk) * 2, uint64_t(p.sk) * p.sq * 2};
    uint32_t box[3] = {64, kBQ, 1};
    rc = make_tensor_map(&tb, p.bias, CFK_BF16, 3, dims, strides, box, 128);
    if (rc != CFK_OK) return rc;
  } else {
    tb = tq;
  }
  {
    uint64_t dims[4] = {uint64_t(D), uint64_t(p.sq), uint64_t(p.h), uint64_t(p.nb)};
    uint64_t strides[3] = {uint64_t(D) * 4, uint64_t(p.sq) * D * 4, uint64_t(p.h) * p.sq * D * 4};
    uint32_t box[4] = {uint32_t(D), kBQ, 1, 1};
    rc = make_tensor_map(&tdq, dq_acc, CFK_F32, 4, dims, strides, box, 128);
    if (rc != CFK_OK) return rc;
  }
  BwdParams prm{bp, delta, dq_acc, device_status_word(), p.bias != nullptr};
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  if (cudaFuncSetAttribute(attn_bwd_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  dim3 grid((p.nb + G - 1) / G, (p.sk + kBK - 1) / kBK, p.h);
  attn_bwd_sm100_kernel<<<grid, kThreads, kSmem, st>>>(tq, tk, tv, tdo, tb, tdq, prm);
  rc = check_launch();
  if (rc != CFK_OK) return rc;
  const int64_t total = int64_t(p.nb) * p.h * p.sq * (D / 8);
  dq_convert_kernel<<<unsigned((total + 255) / 256), 256, 0, st>>>(dq_acc, static_cast<__nv_bfloat16*>(bp.dq), bp.sdq,
                                                                    p.nb, p.h, p.sq);
  return check_launch();
}

}  // namespace cfk
