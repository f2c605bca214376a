// Bias-fused flash attention forward for sm_100a: TMA-staged tiles, tcgen05 MMAs, TMEM accumulators.
//
// One CTA owns a 128-query tile of one head for G batch rows that share the same [128 x Sk] slice of the
// per-head bias (the bias is read once per key block and reused for G score tiles).  A "step" is one
// (key block j, batch row g) pair; steps alternate between two softmax groups so that one group's
// exponentials overlap the other's MMAs.  Warp roles (warpgroup 0 hands its registers to the others):
//   warp 0      TMA producer: Q tiles (once), bias tile per key block, K and V tiles per step
//   warp 1      MMA issuer:   S = Q K^T + the mask step (SS, two steps ahead)
//   warp 2      key-mask producer: per step the additive key mask (0 / floor / lower floor) in shared memory
//   warp 3      MMA issuer:   O += P V (TS: P is read from TMEM)
//   warps 4-7   softmax group 0 (batch rows 0, 2, ...), one thread per query row = one TMEM lane
//   warps 8-11  softmax group 1 (batch rows 1, 3, ...)
// TMEM columns: S0 [0,128) S1 [128,256) | P0 [256,320) P1 [320,384) (bf16 pairs) | O_g [384 + g*D, +D).
// Softmax is online with a lazily updated reference maximum; masked keys are an additive per-key floor, keys past
// Sk a lower one.  Every barrier wait is deadline-bounded and reports into the status word instead of hanging.
// The MMA-issuing thread is scalar code on one lane: it only adds constants to descriptors built once, because
// every extra instruction there delays the tensor pipe.
//
// At head dim 32 the softmax warps' instruction stream, not the tensor pipe, sets the pace (64 tensor flops per score
// against one ex2 and a handful of fp32 instructions), so the key mask is added by the tensor pipe: after Q K^T the
// scores accumulator receives one K = 16 step [1 0 ..] x [mask 0 ..]^T (a column of ones beside Q, the additive mask in
// accumulator units beside K).  (The bias was tried the same way - eight K = 16 steps (I / scale) x bias tile - and
// dropped: an M = 128 MMA reads 8 KB of shared memory whatever it computes, and eight of them per step cost more of
// the shared-memory path than the bias add costs the softmax warps.)
// Math: src/colabfold_kernels/tri_flash.py:132-167,215-239; gate: packed_attn.py:157-158.
#include <cmath>
#include <cstring>

#include "attention_sm100.cuh"

namespace cfk {

namespace {

// F8: q and k arrive in e4m3 (the scores run on the f8f6f4 MMA path, one K = 32 step per 32 head channels); v, P and
// the output stay bf16.
template <int D, int F8>
struct FwdCfg {
  static constexpr int G = 128 / D;  // batch rows per CTA: their O accumulators fill 128 TMEM columns
  static constexpr int kStages = 4;  // K ring and V ring depth
  static constexpr int kRowBytes = D * 2;                 // v rows
  static constexpr int kTileV = kBQ * kRowBytes;
  static constexpr int kRowBytesQK = D * (F8 ? 1 : 2);    // q and k rows
  static constexpr int kTileQK = kBQ * kRowBytesQK;
  static constexpr int kTileBias = kBQ * kBK * 2;  // two 64-key halves, 128-byte swizzled rows
  static constexpr int kMaskSlots = 4;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + G * kTileQK;
  static constexpr int kOffV = kOffK + kStages * kTileQK;
  static constexpr int kOffBias = kOffV + kStages * kTileV;
  static_assert(kOffV % 1024 == 0 && kOffBias % 1024 == 0, "swizzled tiles start on their atom");
  static constexpr int kTileAug = kBQ * 32;  // [128 rows][16 bf16]: the extra K = 16 step (32-byte rows, 32-byte swizzle)
  static constexpr int kOffQaug = kOffBias + 2 * kTileBias;        // column of ones
  static constexpr int kOffKaug = kOffQaug + kTileAug;             // [kMaskSlots] additive key masks
  static constexpr int kOffFlag = kOffKaug + kMaskSlots * kTileAug;
  static_assert(kOffQaug % 1024 == 0 && kOffKaug % 1024 == 0, "swizzled tiles start on their atom");
  static constexpr int kOffState = kOffFlag + 16;                   // float [2][G][128]: reference max, row sum
  static constexpr int kOffBar = kOffState + 2 * G * 128 * 4;
  static constexpr int kNumBars = G + 4 * kStages + 4 + 4 + 4 + 2 * kMaskSlots;
  static constexpr int kOffTmem = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffTmem + 16;
  static constexpr int kTmemCols = 512;
  static constexpr int kColS = 0, kColP = 256, kColO = 384;
  static_assert(kColO + G * D <= 512, "TMEM budget");
  static_assert(kSmemBytes + 1024 <= 232448, "shared memory budget");
  static_assert(kMaskSlots * 4 <= 16, "flag area");
};

constexpr int kThreads = 384;

struct FwdParams {
  AttnProblem p;
  int* status;
  int has_bias;
};

// bf16 bits of the additive key mask in accumulator units (before the scale): a masked key -2^100, a key past Sk -2^126.
constexpr uint32_t kMaskedBf16 = 0xF180u, kPastEndBf16 = 0xFE80u;
// A row maximum (scale * accumulator + bias) below this saw masked keys only.  Such a row's logits are all the same
// number F = fl(-scale * 2^100): the exponent argument is then formed as (t - m) * 2^-90 - exact, 0 on the row's real
// keys and hugely negative past Sk - instead of fma(t, log2 e, -m log2 e), whose rounding residue would be of the
// order of 2^73 there.  The row then averages its real keys, as the reference defines.
constexpr float kDeadNat = -1e25f;
constexpr float kDeadLk = 8.077935669463161e-28f;  // 2^-90

template <int D, int F8>
__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_bias,
                      const FwdParams prm) {
  using C = FwdCfg<D, F8>;
  constexpr int G = C::G;
  constexpr int ST = C::kStages;
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
  uint64_t* q_full = bars;                 // [G]
  uint64_t* k_full = q_full + G;           // [ST]
  uint64_t* k_empty = k_full + ST;         // [ST]
  uint64_t* v_full = k_empty + ST;         // [ST]
  uint64_t* v_empty = v_full + ST;         // [ST]
  uint64_t* bias_full = v_empty + ST;      // [2]
  uint64_t* bias_empty = bias_full + 2;    // [2]
  uint64_t* s_full = bias_empty + 2;       // [2]
  uint64_t* s_empty = s_full + 2;          // [2]
  uint64_t* p_full = s_empty + 2;          // [2]
  uint64_t* pv_done = p_full + 2;          // [2]
  uint64_t* mask_full = pv_done + 2;       // [kMaskSlots]
  uint64_t* mask_empty = mask_full + C::kMaskSlots;
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
    for (int i = 0; i < ST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bias_full[i], 1);
      mbar_init(&bias_empty[i], 4 * ngroups);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    for (int i = 0; i < C::kMaskSlots; ++i) {
      mbar_init(&mask_full[i], 1);
      mbar_init(&mask_empty[i], 1);  // released by the scores issuer's commit
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_bias);
  }
  {
    // constant operands: a column of ones, and zeros in the mask ring beyond its first column
    for (int idx = threadIdx.x; idx < 128 * 2; idx += kThreads) {
      const int r = idx >> 1, chunk = idx & 1;
      *reinterpret_cast<uint4*>(smem + C::kOffQaug + swz_off(r, chunk, 32)) = make_uint4(chunk == 0 ? 0x3F80u : 0u, 0, 0, 0);
    }
    for (int idx = threadIdx.x; idx < C::kMaskSlots * 128 * 2; idx += kThreads)
      *reinterpret_cast<uint4*>(smem + C::kOffKaug + idx * 16) = make_uint4(0, 0, 0, 0);
    fence_proxy_async();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 64;");  // (168 - 64) * 128 registers released ...
    if (warp == 0) {
      // ---------------------------------------------------------------- TMA producer: Q, bias, K
      if (lane == 0) {
        bool ok = true;
        for (int g = 0; g < gcount; ++g) {
          mbar_arrive_expect_tx(&q_full[g], C::kTileQK);
          tma_load_4d(smem + C::kOffQ + g * C::kTileQK, &tm_q, &q_full[g], 0, q0, head, b0 + g);
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
            const int st = step % ST;
            ok = mbar_wait_deadline(&k_empty[st], ((step / ST) & 1) ^ 1);
            if (!ok) { report_timeout(prm.status, 102); break; }
            mbar_arrive_expect_tx(&k_full[st], C::kTileQK);
            tma_load_4d(smem + C::kOffK + st * C::kTileQK, &tm_k, &k_full[st], 0, j * kBK, head, b0 + g);
            // the V slot of a step frees long before its K slot is wanted again (the scores run two steps ahead of
            // P V), so waiting for it here never holds a K load back
            ok = mbar_wait_deadline(&v_empty[st], ((step / ST) & 1) ^ 1);
            if (!ok) { report_timeout(prm.status, 103); break; }
            mbar_arrive_expect_tx(&v_full[st], C::kTileV);
            tma_load_4d(smem + C::kOffV + st * C::kTileV, &tm_v, &v_full[st], 0, j * kBK, head, b0 + g);
          }
        }
      }
      __syncwarp();
    } else if (warp == 1 || warp == 3) {
      // ---------------------------------------------------------------- MMA issuers: warp 1 the scores, warp 3 P V
      // Two threads, because what bounds a step is the issuing thread's own instruction chain (waits, descriptor
      // arithmetic, commits: ~650 clocks per scores step and as much per P V step when one thread did both in turn),
      // not the tensor pipe, which is a tenth busy.  The two chains touch different TMEM columns and barriers.
      if (lane == 0) {
        constexpr uint32_t idesc_s = F8 ? make_idesc(kBQ, kBK, 0, 0, 0, 0) : make_idesc(kBQ, kBK, 1, 1, 0, 0);
        constexpr uint32_t idesc_pv = make_idesc(kBQ, D, 1, 1, 0, 1);
        // the mask step: both operands K-major, 32-byte rows
        constexpr uint32_t idesc_aug = make_idesc(kBQ, kBK, 1, 1, 0, 0);
        const uint64_t qaug_desc = desc_k_major(smem_u32(smem + C::kOffQaug), 32);
        const uint64_t kaug_desc0 = desc_k_major(smem_u32(smem + C::kOffKaug), 32);
        int m_slot = 0;
        uint32_t m_par = 0;
        constexpr uint32_t kTile16 = C::kTileQK >> 4, kTile16V = C::kTileV >> 4;
        const uint64_t q_desc0 = desc_k_major(smem_u32(smem + C::kOffQ), C::kRowBytesQK);
        const uint64_t k_desc0 = desc_k_major(smem_u32(smem + C::kOffK), C::kRowBytesQK);
        const uint64_t v_desc0 = desc_mn_major(smem_u32(smem + C::kOffV), C::kRowBytes, 0);
        // Scalar state advanced by increments only: one lane runs this, and every division or re-derivation
        // here would sit between two MMAs.
        int s_g = 0, s_st = 0, p_g = 0, p_st = 0;
        uint32_t k_par = 0, v_par = 0, s_first = 1, p_first = 1;
        uint32_t se_par0 = 1, se_par1 = 1, pf_par0 = 0, pf_par1 = 0;
        bool ok = true;
        auto issue_s = [&]() {
          const int buf = s_g & 1;
          if (s_first && !mbar_wait_deadline(&q_full[s_g], 0)) { report_timeout(prm.status, 201); return false; }
          if (!mbar_wait_deadline(&k_full[s_st], k_par)) { report_timeout(prm.status, 202); return false; }
          if (!mbar_wait_deadline(&s_empty[buf], buf ? se_par1 : se_par0)) { report_timeout(prm.status, 203); return false; }
          if (!mbar_wait_deadline(&mask_full[m_slot], m_par)) { report_timeout(prm.status, 206); return false; }
          tc_fence_after();
          const uint64_t a = q_desc0 + uint64_t(s_g * kTile16), b = k_desc0 + uint64_t(s_st * kTile16);
          const uint32_t d = tmem + C::kColS + buf * kBK;
#pragma unroll
          for (int kk = 0; kk < D / (F8 ? 32 : 16); ++kk) {  // 32 bytes of the row per MMA either way
            if (F8) mma_f8_ss(d, a + 2 * kk, b + 2 * kk, idesc_s, kk > 0);
            else mma_f16_ss(d, a + 2 * kk, b + 2 * kk, idesc_s, kk > 0);
          }
          mma_f16_ss(d, qaug_desc, kaug_desc0 + uint64_t(m_slot * (C::kTileAug >> 4)), idesc_aug, 1);
          mma_commit(&mask_empty[m_slot]);
          if (++m_slot == C::kMaskSlots) { m_slot = 0; m_par ^= 1; }
          mma_commit(&k_empty[s_st]);
          mma_commit(&s_full[buf]);
          if (buf) se_par1 ^= 1; else se_par0 ^= 1;
          if (++s_g == gcount) { s_g = 0; s_first = 0; }
          if (++s_st == ST) { s_st = 0; k_par ^= 1; }
          return true;
        };
        auto issue_pv = [&]() {
          const int buf = p_g & 1;
          if (!mbar_wait_deadline(&v_full[p_st], v_par)) { report_timeout(prm.status, 204); return false; }
          if (!mbar_wait_deadline(&p_full[buf], buf ? pf_par1 : pf_par0)) { report_timeout(prm.status, 205); return false; }
          tc_fence_after();
          const uint64_t b = v_desc0 + uint64_t(p_st * kTile16V);
          const uint32_t d = tmem + C::kColO + p_g * D, a = tmem + C::kColP + buf * (kBK / 2);
          const uint32_t acc0 = p_first ^ 1;  // key block 0 overwrites the accumulator
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_f16_ts(d, a + kk * 8, b + uint64_t(kk * ((16 * C::kRowBytes) >> 4)), idesc_pv, kk > 0 ? 1u : acc0);
          mma_commit(&v_empty[p_st]);
          mma_commit(&pv_done[buf]);
          if (buf) pf_par1 ^= 1; else pf_par0 ^= 1;
          if (++p_g == gcount) { p_g = 0; p_first = 0; }
          if (++p_st == ST) { p_st = 0; v_par ^= 1; }
          return true;
        };
        // the scores of a step go out as soon as their buffer has been read (one per softmax group: two steps ahead)
        if (warp == 1) {
          for (int t = 0; t < nsteps && ok; ++t) ok = issue_s();
        } else {
          for (int t = 0; t < nsteps && ok; ++t) ok = issue_pv();
        }
      }
      __syncwarp();
    } else {
      // ---------------------------------------------------------------- key-mask producer
      // Per step the first column of a [128 keys][16] bf16 operand (the rest stays zero): 0 live, -2^100 masked,
      // -2^126 past Sk.  The mask bytes of the next step are fetched before this step's slot is waited for, so the
      // global-memory latency is off the path.
      bool ok = true;
      auto fetch = [&](int t) -> uint32_t {
        const int g = t % gcount, j = t / gcount, key = j * kBK + lane * 4;
        // Sk is a multiple of 8, so a group of four keys is in or out as a whole
        if (t >= nsteps || key >= p.sk) return 0xffffffffu;  // placeholder, not used for keys past Sk
        return *reinterpret_cast<const uint32_t*>(p.kmask + int64_t(b0 + g) * p.sk + key);
      };
      uint32_t w_next = fetch(0);
      for (int t = 0; t < nsteps && ok; ++t) {
        const int j = t / gcount, slot = t % C::kMaskSlots;
        const uint32_t w = w_next;
        w_next = fetch(t + 1);
        if (lane == 0) ok = mbar_wait_deadline(&mask_empty[slot], ((t / C::kMaskSlots) & 1) ^ 1);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) { if (lane == 0) report_timeout(prm.status, 501); break; }
        const bool in = j * kBK + lane * 4 < p.sk;
        const uint32_t m0 = !in ? kPastEndBf16 : (w & 0x000000ffu) ? 0u : kMaskedBf16;
        const uint32_t m1 = !in ? kPastEndBf16 : (w & 0x0000ff00u) ? 0u : kMaskedBf16;
        const uint32_t m2 = !in ? kPastEndBf16 : (w & 0x00ff0000u) ? 0u : kMaskedBf16;
        const uint32_t m3 = !in ? kPastEndBf16 : (w & 0xff000000u) ? 0u : kMaskedBf16;
        uint8_t* tile = smem + C::kOffKaug + slot * C::kTileAug;
        *reinterpret_cast<uint4*>(tile + swz_off(lane * 4 + 0, 0, 32)) = make_uint4(m0, 0, 0, 0);
        *reinterpret_cast<uint4*>(tile + swz_off(lane * 4 + 1, 0, 32)) = make_uint4(m1, 0, 0, 0);
        *reinterpret_cast<uint4*>(tile + swz_off(lane * 4 + 2, 0, 32)) = make_uint4(m2, 0, 0, 0);
        *reinterpret_cast<uint4*>(tile + swz_off(lane * 4 + 3, 0, 32)) = make_uint4(m3, 0, 0, 0);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&mask_full[slot]);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax groups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;");  // ... cover the (216 - 168) * 256 taken here
    const int grp = (warp - 4) >> 2;           // 0 or 1
    const int quad = warp & 3;                 // TMEM lane quadrant this warp may touch
    const int row = quad * 32 + lane;          // query row inside the tile = TMEM lane
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    // running (reference maximum, row sum) of each batch row this thread serves: [g][row], private to the thread
    float* st_m = reinterpret_cast<float*>(smem + C::kOffState) + row;
    float* st_l = st_m + G * 128;
    uint32_t uses = 0;  // steps this group has processed: parity of s_full / pv_done for its buffer
    bool ok = true;
    const float scale = p.scale;
    // A wait that runs out clears `ok`; later waits are then skipped but every thread still walks the
    // same loop and nothing is stored.
#define CFK_SOFTMAX_WAIT(bar, parity, code)                       \
  if (ok && !mbar_wait_deadline((bar), (parity))) {               \
    report_timeout(prm.status, (code));                           \
    ok = false;                                                   \
  }
    const int jmax = grp < ngroups ? nj : 0;
    for (int j = 0; j < jmax; ++j) {
      const uint8_t* bias_tile = smem + C::kOffBias + (j & 1) * C::kTileBias;
      if (prm.has_bias) CFK_SOFTMAX_WAIT(&bias_full[j & 1], (j >> 1) & 1, 301)
#pragma unroll 1
      for (int g = grp; g < gcount; g += 2) {

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

        // logits t = scale * s + bias (the mask is in s already); packed fp32 pairs: two keys per FMA-pipe instruction
        const uint64_t scale2 = f2_pack(scale, scale);
        if (prm.has_bias) {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const uint4 w = *reinterpret_cast<const uint4*>(bias_tile + (c / 8) * (C::kTileBias / 2) + swz_off(row, c % 8, 128));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
              f2_unpack(f2_fma(f2_pack(s[c * 8 + 2 * i], s[c * 8 + 2 * i + 1]), scale2,
                               f2_pack(bf16lo_to_f32(ww[i]), bf16hi_to_f32(ww[i]))), s[c * 8 + 2 * i], s[c * 8 + 2 * i + 1]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < kBK; i += 2) f2_unpack(f2_mul(f2_pack(s[i], s[i + 1]), scale2), s[i], s[i + 1]);
        }
        float mx;
        {
          // four independent chains of three-input maxima: one instruction per two scores
          float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
          for (int i = 0; i < kBK; i += 8) {
            m0 = fmax3(m0, s[i], s[i + 1]); m1 = fmax3(m1, s[i + 2], s[i + 3]);
            m2 = fmax3(m2, s[i + 4], s[i + 5]); m3 = fmax3(m3, s[i + 6], s[i + 7]);
          }
          mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
        }

        // lazily updated reference maximum
        float corr = 1.0f, m_ref = mx, l_run = 0.f;
        bool need = false;
        if (j > 0) {
          m_ref = st_m[g * 128];
          l_run = st_l[g * 128];
          if (mx > m_ref + kRescaleSlack) {
            corr = ex2_approx(fmaf(m_ref, kLog2eF, -mx * kLog2eF));
            m_ref = mx;
            need = true;
          }
        }
        // exponent arguments fma(t, lk, -m lk); a row that has seen masked keys only takes lk = 2^-90 (see kDeadNat)
        const float lk = m_ref < kDeadNat ? kDeadLk : kLog2eF;
        const float neg_m = -m_ref * lk;
        uint32_t pk[kBK / 2];
        {
          // Software-pipelined by hand and pinned (volatile): each slot issues the two exponentials of one pair of keys,
          // the multiply-add that prepares the pair two slots on, and the sum and bf16 pack of the pair three slots
          // back.  The XU pipe (16 ex2 per clock and SM, 8 clocks per warp instruction) is the busiest unit of this
          // kernel; a warp issues in order, so exponentials written as one run would leave the other pipes idle.
          const uint64_t l2e2 = f2_pack(lk, lk), negm2 = f2_pack(neg_m, neg_m);
          uint64_t sum_a = f2_pack(0.f, 0.f), sum_b = sum_a;
          constexpr int NP = kBK / 2, kAhead = 2, kBehind = 3;
          uint64_t v[NP];
#pragma unroll
          for (int i = 0; i < kAhead; ++i) v[i] = f2_fma_pinned(f2_pack(s[2 * i], s[2 * i + 1]), l2e2, negm2);
#pragma unroll
          for (int i = 0; i < NP + kBehind; ++i) {
            if (i < NP) v[i] = f2_ex2_pinned(v[i]);
            if (i + kAhead < NP)
              v[i + kAhead] = f2_fma_pinned(f2_pack(s[2 * (i + kAhead)], s[2 * (i + kAhead) + 1]), l2e2, negm2);
            if (i >= kBehind) {
              const int k = i - kBehind;
              if (k & 1) sum_b = f2_add_pinned(sum_b, v[k]); else sum_a = f2_add_pinned(sum_a, v[k]);
              pk[k] = f2_pack_bf16_pinned(v[k]);
            }
          }
          float t0, t1;
          f2_unpack(f2_add(sum_a, sum_b), t0, t1);
          st_m[g * 128] = m_ref;
          st_l[g * 128] = l_run * corr + (t0 + t1);
        }

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
        }
        // P (bf16 pairs) into this group's TMEM operand buffer: column c holds keys 2c, 2c+1
#pragma unroll
        for (int c = 0; c < kBK / 32; ++c)
          tmem_st_x16(tmem + lane_addr + C::kColP + grp * (kBK / 2) + c * 16, reinterpret_cast<uint32_t(&)[16]>(pk[c * 16]));
        tmem_wait_st();
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
    // the gate rows of this group's batch rows are fetched before the wait for the last P V, so that their latency
    // runs under it instead of after it
    constexpr int kMine = (C::G + 1) / 2;   // batch rows of one group: grp, grp + 2, ...
    uint4 gpre[kMine][D / 8];
    {
      const int q = q0 + row;
#pragma unroll
      for (int k = 0; k < kMine; ++k) {
        const int g = grp + 2 * k;
#pragma unroll
        for (int c = 0; c < D / 8; ++c) gpre[k][c] = make_uint4(0, 0, 0, 0);
        if (ok && p.gate != nullptr && g < gcount && q < p.sq) {
          const __nv_bfloat16* gate = static_cast<const __nv_bfloat16*>(p.gate) + (b0 + g) * p.sg_.b + head * p.sg_.h + int64_t(q) * p.sg_.s;
#pragma unroll
          for (int c = 0; c < D / 8; ++c) gpre[k][c] = *reinterpret_cast<const uint4*>(gate + c * 8);
        }
      }
    }
    if (uses > 0) {
      CFK_SOFTMAX_WAIT(&pv_done[grp], (uses - 1) & 1, 304)
      tc_fence_after();
    }
#undef CFK_SOFTMAX_WAIT
    if (ok) {
      const int q = q0 + row;
#pragma unroll
      for (int k = 0; k < kMine; ++k) {
        const int g = grp + 2 * k;
        if (g >= gcount) break;
        const int b = b0 + g;
        const float m_ref = st_m[g * 128], l_run = st_l[g * 128];
        float o[D];
#pragma unroll
        for (int c = 0; c < D / 16; ++c) tmem_ld_x16(tmem + lane_addr + C::kColO + g * D + c * 16, reinterpret_cast<uint32_t(&)[16]>(o[c * 16]));
        tmem_wait_ld();
        if (q < p.sq) {
          bool zero_row = false;
          if (p.trim != nullptr) zero_row = p.trim[b] == 0 || q >= p.trim[p.nb];
          const float inv = zero_row ? 0.f : 1.0f / l_run;
          const __nv_bfloat16* gb =
              p.gate == nullptr ? nullptr : static_cast<const __nv_bfloat16*>(p.gate_bias) + int64_t(head) * D;
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + b * p.so_.b + head * p.so_.h + int64_t(q) * p.so_.s;
#pragma unroll
          for (int c = 0; c < D / 8; ++c) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = o[c * 8 + i] * inv;
            if (p.gate != nullptr) {
              const uint4 gw = gpre[k][c];
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
          if (p.lse != nullptr)
            p.lse[(int64_t(b) * p.h + head) * p.sq + q] = m_ref < kDeadNat ? kNegRef : fmaf(m_ref, kLog2eF, __log2f(l_run));
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

template <int D, int F8>
int launch(const AttnProblem& p, cudaStream_t st) {
  using C = FwdCfg<D, F8>;
  CUtensorMap tq, tk, tv, tb;
  const int qk_dtype = F8 ? CFK_E4M3 : CFK_BF16;
  int rc = make_qkv_map(&tq, p.q, p.sq_, p.nb, p.h, p.sq, D, kBQ, qk_dtype);
  if (rc == CFK_OK) rc = make_qkv_map(&tk, p.k, p.sk_, p.nb, p.h, p.sk, D, kBK, qk_dtype);
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
  const int smem = C::kSmemBytes + 1024;
  if (cudaFuncSetAttribute(attn_fwd_sm100_kernel<D, F8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  dim3 grid((p.nb + C::G - 1) / C::G, (p.sq + kBQ - 1) / kBQ, p.h);
  attn_fwd_sm100_kernel<D, F8><<<grid, kThreads, smem, st>>>(tq, tk, tv, tb, prm);
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
  if (reinterpret_cast<uintptr_t>(p.kmask) % 4 != 0) return false;
  auto st8 = [](const Strides& s) { return s.b % 8 == 0 && s.s % 8 == 0 && s.h % 8 == 0; };
  auto st16 = [](const Strides& s) { return s.b % 16 == 0 && s.s % 16 == 0 && s.h % 16 == 0; };  // one-byte elements
  if (p.qk_e4m3 ? !(st16(p.sq_) && st16(p.sk_)) : !(st8(p.sq_) && st8(p.sk_))) return false;
  return st8(p.sv_) && st8(p.so_) && (p.gate == nullptr || st8(p.sg_));
}

int attention_fwd_sm100(const AttnProblem& p, cudaStream_t st) {
  if (p.d != 32 || !(p.scale > 0.f)) return CFK_ERR_UNSUPPORTED;
  return p.qk_e4m3 ? launch<32, 1>(p, st) : launch<32, 0>(p, st);
}

}  // namespace cfk
