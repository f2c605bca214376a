// Bias-fused flash attention forward for sm_100a: TMA-staged tiles, tcgen05 MMAs, TMEM accumulators.
//
// One CTA owns a 128-query tile of one head for G batch rows that share the same [128 x Sk] slice of the
// per-head bias (the bias is read once per key block and reused for G score tiles).  Warp roles:
//   warp 0      TMA producer: Q tiles (once), bias tile per key block, K/V tiles per (key block, batch row)
//   warp 1      MMA issuer:   S = Q K^T into TMEM (double buffered), then O += P V (P staged in shared memory)
//   warps 2-5   softmax group 0 (batch rows 0, 2, ...), one thread per query row = one TMEM lane
//   warps 6-9   softmax group 1 (batch rows 1, 3, ...)
// Softmax is online in the natural-log domain with a lazily updated reference maximum; masked keys are an
// additive per-key floor, keys past Sk an additive -inf.  Every barrier wait is deadline-bounded and reports
// into the status word instead of hanging.
// Math: src/colabfold_kernels/tri_flash.py:132-167,215-239; gate: packed_attn.py:157-158.
#include "attention_sm100.cuh"

namespace cfk {

namespace {

template <int D>
struct FwdCfg {
  static constexpr int G = D <= 32 ? 4 : 2;        // batch rows per CTA
  static constexpr int kStages = D <= 32 ? 3 : 2;  // K/V ring depth
  static constexpr int kRowBytes = D * 2;
  static constexpr int kTileQkv = kBQ * kRowBytes;
  static constexpr int kTileBias = kBQ * kBK * 2;  // two 64-key halves, 128-byte swizzled rows
  static constexpr int kTileP = kBQ * kBK * 2;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + G * kTileQkv;
  static constexpr int kOffV = kOffK + kStages * kTileQkv;
  static constexpr int kOffBias = kOffV + kStages * kTileQkv;
  static constexpr int kOffP = kOffBias + 2 * kTileBias;
  static constexpr int kOffMask = kOffP + 2 * kTileP;          // float [2 groups][2 buffers][128]
  static constexpr int kOffFlag = kOffMask + 2 * 2 * 128 * 4;  // int [2 groups][2 buffers][4 warps]
  static constexpr int kOffBar = kOffFlag + 2 * 2 * 4 * 4;
  static constexpr int kNumBars = G + 2 * kStages + 4 + 4 + 4;
  static constexpr int kOffTmem = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffTmem + 16;
  static constexpr int kTmemCols = 512;
  static constexpr int kColS = 0;    // S buffers at columns 0 and 128
  static constexpr int kColO = 256;  // O_g at 256 + g * D
  static_assert(256 + G * D <= 512, "TMEM budget");
  static_assert(kSmemBytes + 1024 <= 232448, "shared memory budget");
};

constexpr int kThreads = 320;

struct FwdParams {
  AttnProblem p;
  int* status;
  int has_bias;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_bias,
                      const FwdParams prm) {
  using C = FwdCfg<D>;
  constexpr int G = C::G;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment: swizzled tiles and UMMA descriptors assume it
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const AttnProblem& p = prm.p;
  {
    // an earlier CTA gave up: do not pile on (one thread reads, so the whole CTA takes the same branch)
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* q_full = bars;                      // [G]
  uint64_t* kv_full = q_full + G;               // [kStages]
  uint64_t* kv_empty = kv_full + C::kStages;    // [kStages]
  uint64_t* bias_full = kv_empty + C::kStages;  // [2]
  uint64_t* bias_empty = bias_full + 2;         // [2]
  uint64_t* s_full = bias_empty + 2;            // [2]
  uint64_t* s_empty = s_full + 2;               // [2]
  uint64_t* p_full = s_empty + 2;               // [2]
  uint64_t* pv_done = p_full + 2;               // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b0 = blockIdx.x * G;
  const int gcount = min(G, p.nb - b0);
  const int q0 = blockIdx.y * kBQ;
  const int head = blockIdx.z;
  const int nj = (p.sk + kBK - 1) / kBK;
  const int nsteps = nj * gcount;
  const int ngroups = gcount >= 2 ? 2 : 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < G; ++i) mbar_init(&q_full[i], 1);
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bias_full[i], 1);
      mbar_init(&bias_empty[i], 4 * ngroups);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_bias);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      for (int g = 0; g < gcount; ++g) {
        mbar_arrive_expect_tx(&q_full[g], C::kTileQkv);
        tma_load_4d(smem + C::kOffQ + g * C::kTileQkv, &tm_q, &q_full[g], 0, q0, head, b0 + g);
      }
      int step = 0;
      for (int j = 0; j < nj && ok; ++j) {
        if (prm.has_bias) {
          const int bb = j & 1;
          ok = mbar_wait_deadline(&bias_empty[bb], ((j >> 1) & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 101); break; }
          mbar_arrive_expect_tx(&bias_full[bb], C::kTileBias);
          uint8_t* dst = smem + C::kOffBias + bb * C::kTileBias;
          tma_load_3d(dst, &tm_bias, &bias_full[bb], j * kBK, q0, head);
          tma_load_3d(dst + C::kTileBias / 2, &tm_bias, &bias_full[bb], j * kBK + 64, q0, head);
        }
        for (int g = 0; g < gcount; ++g, ++step) {
          const int st = step % C::kStages;
          ok = mbar_wait_deadline(&kv_empty[st], ((step / C::kStages) & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 102); break; }
          mbar_arrive_expect_tx(&kv_full[st], 2 * C::kTileQkv);
          tma_load_4d(smem + C::kOffK + st * C::kTileQkv, &tm_k, &kv_full[st], 0, j * kBK, head, b0 + g);
          tma_load_4d(smem + C::kOffV + st * C::kTileQkv, &tm_v, &kv_full[st], 0, j * kBK, head, b0 + g);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc(kBQ, kBK, 1, 1, 0, 0);
      constexpr uint32_t idesc_pv = make_idesc(kBQ, D, 1, 1, 0, 1);
      const uint32_t q_base = smem_u32(smem + C::kOffQ), k_base = smem_u32(smem + C::kOffK);
      const uint32_t v_base = smem_u32(smem + C::kOffV), p_base = smem_u32(smem + C::kOffP);
      uint32_t s_uses[2] = {0, 0}, p_uses[2] = {0, 0};
      bool ok = true;
      auto issue_s = [&](int t) {
        const int g = t % gcount, buf = g & 1, st = t % C::kStages;
        if (!mbar_wait_deadline(&q_full[g], 0)) { report_timeout(prm.status, 201); return false; }
        if (!mbar_wait_deadline(&kv_full[st], (t / C::kStages) & 1)) { report_timeout(prm.status, 202); return false; }
        if (!mbar_wait_deadline(&s_empty[buf], (s_uses[buf] & 1) ^ 1)) { report_timeout(prm.status, 203); return false; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = desc_k_major(q_base + g * C::kTileQkv + kk * 32, C::kRowBytes);
          const uint64_t b = desc_k_major(k_base + st * C::kTileQkv + kk * 32, C::kRowBytes);
          mma_f16_ss(tmem + C::kColS + buf * kBK, a, b, idesc_s, kk > 0);
        }
        mma_commit(&s_full[buf]);
        ++s_uses[buf];
        return true;
      };
      auto issue_pv = [&](int t) {
        const int g = t % gcount, j = t / gcount, buf = g & 1, st = t % C::kStages;
        if (!mbar_wait_deadline(&p_full[buf], p_uses[buf] & 1)) { report_timeout(prm.status, 204); return false; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t a =
              desc_k_major(p_base + buf * C::kTileP + (kk / 4) * (C::kTileP / 2) + (kk % 4) * 32, 128);
          const uint64_t b = desc_mn_major(v_base + st * C::kTileQkv + kk * 16 * C::kRowBytes, C::kRowBytes, 0);
          mma_f16_ss(tmem + C::kColO + g * D, a, b, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&kv_empty[st]);
        mma_commit(&pv_done[buf]);
        ++p_uses[buf];
        return true;
      };
      ok = issue_s(0);
      for (int t = 0; t < nsteps && ok; ++t) {
        if (t + 1 < nsteps) ok = issue_s(t + 1);
        if (ok) ok = issue_pv(t);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax groups
    const int grp = (warp - 2) >> 2;           // 0 or 1
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may touch
    const int row = quad * 32 + lane;          // query row inside the tile = TMEM lane
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const int gtid = quad * 32 + lane;         // 0..127 inside the group (distinct per thread)
    float* mask_buf = reinterpret_cast<float*>(smem + C::kOffMask) + grp * 2 * 128;
    int* flag_buf = reinterpret_cast<int*>(smem + C::kOffFlag) + grp * 2 * 4;
    constexpr int kMine = (G + 1) / 2;
    float m_ref[kMine], l_sum[kMine];
#pragma unroll
    for (int i = 0; i < kMine; ++i) { m_ref[i] = 0.f; l_sum[i] = 0.f; }
    uint32_t uses = 0;  // steps this group has processed: parity of s_full / pv_done for its buffer
    bool ok = true;
    const float scale = p.scale;
    // A wait that runs out clears `ok`; later waits are then skipped but every thread still walks the
    // same loop (named barriers stay matched) and nothing is stored.
#define CFK_SOFTMAX_WAIT(bar, parity, code)                       \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    const int jmax = grp < ngroups ? nj : 0;
    for (int j = 0; j < jmax; ++j) {
      const int k0 = j * kBK;
      const uint8_t* bias_tile = smem + C::kOffBias + (j & 1) * C::kTileBias;
      if (prm.has_bias) CFK_SOFTMAX_WAIT(&bias_full[j & 1], (j >> 1) & 1, 301)
#pragma unroll
      for (int gi = 0; gi < kMine; ++gi) {
        const int g = grp + 2 * gi;
        if (g >= gcount) break;
        const int b = b0 + g;
        // additive key mask for this (batch row, key block): 0 live, floor masked, -inf past Sk
        const int mb = uses & 1;
        {
          const int key = k0 + gtid;
          float add = 0.f;
          if (key >= p.sk) add = -INFINITY;
          else if (p.kmask[int64_t(b) * p.sk + key] == 0) add = kFloorNat;
          mask_buf[mb * 128 + gtid] = add;
          const unsigned any = __ballot_sync(0xffffffffu, add != 0.f);
          if (lane == 0) flag_buf[mb * 4 + quad] = any != 0;
        }
        named_bar_sync(1 + grp, 128);
        const bool any_mask = (flag_buf[mb * 4 + 0] | flag_buf[mb * 4 + 1] | flag_buf[mb * 4 + 2] | flag_buf[mb * 4 + 3]) != 0;

        CFK_SOFTMAX_WAIT(&s_full[grp], uses & 1, 302)
        tc_fence_after();
        float s[kBK];
#pragma unroll
        for (int c = 0; c < kBK / 32; ++c)
          tmem_ld_x32(tmem + lane_addr + C::kColS + grp * kBK + c * 32, reinterpret_cast<uint32_t(&)[32]>(s[c * 32]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[grp]);

        // logits t = scale * s + bias (+ mask), row maximum
        float mx = -INFINITY;
        if (prm.has_bias) {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const uint4 w = *reinterpret_cast<const uint4*>(bias_tile + (c / 8) * (C::kTileBias / 2) + swz_off(row, c % 8, 128));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              s[c * 8 + 2 * i] = fmaf(s[c * 8 + 2 * i], scale, bf16lo_to_f32(ww[i]));
              s[c * 8 + 2 * i + 1] = fmaf(s[c * 8 + 2 * i + 1], scale, bf16hi_to_f32(ww[i]));
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < kBK; ++i) s[i] *= scale;
        }
        if (any_mask) {
#pragma unroll
          for (int c = 0; c < kBK / 4; ++c) {
            const float4 a = *reinterpret_cast<const float4*>(mask_buf + mb * 128 + c * 4);
            s[c * 4 + 0] += a.x; s[c * 4 + 1] += a.y; s[c * 4 + 2] += a.z; s[c * 4 + 3] += a.w;
          }
        }
#pragma unroll
        for (int i = 0; i < kBK; ++i) mx = fmaxf(mx, s[i]);

        // lazily updated reference maximum
        float corr = 1.0f;
        bool need = false;
        if (j == 0) {
          m_ref[gi] = mx;
        } else if (mx > m_ref[gi] + kRescaleSlack) {
          corr = ex2_approx(fmaf(m_ref[gi], kLog2eF, -mx * kLog2eF));
          m_ref[gi] = mx;
          need = true;
        }
        const float neg_m = -m_ref[gi] * kLog2eF;
        float sum = 0.f;
        uint32_t pk[kBK / 2];
#pragma unroll
        for (int i = 0; i < kBK / 2; ++i) {
          const float e0 = ex2_approx(fmaf(s[2 * i], kLog2eF, neg_m));
          const float e1 = ex2_approx(fmaf(s[2 * i + 1], kLog2eF, neg_m));
          sum += e0 + e1;
          pk[i] = pack_bf16x2(e0, e1);
        }
        l_sum[gi] = l_sum[gi] * corr + sum;

        // the previous P V of this buffer must be complete before P is overwritten or O is rescaled
        if (uses > 0) {
          CFK_SOFTMAX_WAIT(&pv_done[grp], (uses - 1) & 1, 303)
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
          for (int c = 0; c < D / 16; ++c) {
            uint32_t r[16];
            tmem_ld_x16(tmem + lane_addr + C::kColO + g * D + c * 16, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
            tmem_st_x16(tmem + lane_addr + C::kColO + g * D + c * 16, r);
          }
          tmem_wait_st();
        }
        uint8_t* p_tile = smem + C::kOffP + grp * C::kTileP;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint4 w = make_uint4(pk[c * 4], pk[c * 4 + 1], pk[c * 4 + 2], pk[c * 4 + 3]);
          *reinterpret_cast<uint4*>(p_tile + (c / 8) * (C::kTileP / 2) + swz_off(row, c % 8, 128)) = w;
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[grp]);
        ++uses;
      }
      if (prm.has_bias) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&bias_empty[j & 1]);
      }
    }
    // ---------------------------------------------------------------- epilogue: O / l, gate, store
    if (uses > 0) {
      CFK_SOFTMAX_WAIT(&pv_done[grp], (uses - 1) & 1, 304)
      tc_fence_after();
    }
#undef CFK_SOFTMAX_WAIT
    if (ok) {
      const int q = q0 + row;
#pragma unroll
      for (int gi = 0; gi < kMine; ++gi) {
        const int g = grp + 2 * gi;
        if (g >= gcount) break;
        const int b = b0 + g;
        float o[D];
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t r[16];
          tmem_ld_x16(tmem + lane_addr + C::kColO + g * D + c * 16, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[c * 16 + i] = __uint_as_float(r[i]);
        }
        if (q < p.sq) {
          bool zero_row = false;
          if (p.trim != nullptr) zero_row = p.trim[b] == 0 || q >= p.trim[p.nb];
          const float inv = zero_row ? 0.f : 1.0f / l_sum[gi];
          const __nv_bfloat16* gate =
              p.gate == nullptr ? nullptr
                                : static_cast<const __nv_bfloat16*>(p.gate) + b * p.sg_.b + head * p.sg_.h + int64_t(q) * p.sg_.s;
          const __nv_bfloat16* gb =
              p.gate == nullptr ? nullptr : static_cast<const __nv_bfloat16*>(p.gate_bias) + int64_t(head) * D;
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + b * p.so_.b + head * p.so_.h + int64_t(q) * p.so_.s;
#pragma unroll
          for (int c = 0; c < D / 8; ++c) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = o[c * 8 + i] * inv;
            if (gate != nullptr) {
              const uint4 gw = *reinterpret_cast<const uint4*>(gate + c * 8);
              const uint4 bw = *reinterpret_cast<const uint4*>(gb + c * 8);
              const uint32_t gg[4] = {gw.x, gw.y, gw.z, gw.w}, bb[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                v[2 * i] *= sigmoid_fast(bf16lo_to_f32(gg[i]) + bf16lo_to_f32(bb[i]));
                v[2 * i + 1] *= sigmoid_fast(bf16hi_to_f32(gg[i]) + bf16hi_to_f32(bb[i]));
              }
            }
            uint4 w = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                                 pack_bf16x2(v[6], v[7]));
            *reinterpret_cast<uint4*>(out + c * 8) = w;
          }
          if (p.lse != nullptr) {
            const float m = m_ref[gi];
            p.lse[(int64_t(b) * p.h + head) * p.sq + q] =
                m < -1e30f ? kNegRef : fmaf(m, kLog2eF, __log2f(l_sum[gi]));
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int D>
int launch(const AttnProblem& p, cudaStream_t st) {
  using C = FwdCfg<D>;
  CUtensorMap tq, tk, tv, tb;
  int rc = make_qkv_map(&tq, p.q, p.sq_, p.nb, p.h, p.sq, D, kBQ);
  if (rc == CFK_OK) rc = make_qkv_map(&tk, p.k, p.sk_, p.nb, p.h, p.sk, D, kBK);
  if (rc == CFK_OK) rc = make_qkv_map(&tv, p.v, p.sv_, p.nb, p.h, p.sk, D, kBK);
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
  FwdParams prm{p, device_status_word(), p.bias != nullptr};
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  static bool attr_set = false;
  const int smem = C::kSmemBytes + 1024;
  if (!attr_set) {
    if (cudaFuncSetAttribute(attn_fwd_sm100_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return CFK_ERR_LAUNCH;
    attr_set = true;
  }
  dim3 grid((p.nb + C::G - 1) / C::G, (p.sq + kBQ - 1) / kBQ, p.h);
  attn_fwd_sm100_kernel<D><<<grid, kThreads, smem, st>>>(tq, tk, tv, tb, prm);
  return check_launch();
}

}  // namespace

bool attention_sm100_supported(const AttnProblem& p, int dtype) {
  if (dtype != CFK_BF16) return false;
  if (p.d != 32) return false;
  if (p.sk % 8 != 0 || p.h > 65535 || (p.sq + kBQ - 1) / kBQ > 65535) return false;
  auto ok16 = [](const void* ptr) { return ptr == nullptr || aligned16(ptr); };
  if (!ok16(p.q) || !ok16(p.k) || !ok16(p.v) || !ok16(p.bias) || !ok16(p.out) || !ok16(p.gate) || !ok16(p.gate_bias))
    return false;
  auto st8 = [](const Strides& s) { return s.b % 8 == 0 && s.s % 8 == 0 && s.h % 8 == 0; };
  return st8(p.sq_) && st8(p.sk_) && st8(p.sv_) && st8(p.so_) && (p.gate == nullptr || st8(p.sg_));
}

int attention_fwd_sm100(const AttnProblem& p, cudaStream_t st) {
  switch (p.d) {
    case 32: return launch<32>(p, st);
    default: return CFK_ERR_UNSUPPORTED;
  }
}

}  // namespace cfk
