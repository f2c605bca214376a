// Triangle-multiplication contraction as a persistent tcgen05 batched GEMM:
//   out[c, i, j] = alpha * sum_k a[c, i, k] * b[c, j, k],   a [C,I,K], b [C,J,K] (bf16 or e4m3), out [C,I,J] bf16.
// One CTA per SM walks 128 x 256 output tiles (c outermost, so the tiles in flight share operands in L2).
//   warp 0     TMA producer: 128-byte-wide K slices of A (128 rows) and B (256 rows) into a 4-stage ring
//   warp 1     MMA issuer: four K=32-byte tcgen05.mma per slice into one of two 256-column TMEM accumulators
//   warps 2-5  epilogue: TMEM -> registers -> bf16 -> swizzled shared staging -> TMA store, overlapped with the
//              next tile's main loop through the second accumulator
// bf16 and e4m3 differ only in the tensor-map element type and the instruction descriptor: both move 128-byte
// rows and advance the descriptors by 32 bytes per MMA.
// Math: src/colabfold_kernels/contract.py:1-4,56-57 (e4m3) and the XLA batched GEMM of tri_mul.py:6-7 (bf16).
#include "attention_sm100.cuh"

namespace cfk {
namespace {

constexpr int kTM = 128, kTN = 256;
constexpr int kStages = 4;
constexpr int kSliceA = kTM * 128, kSliceB = kTN * 128;  // bytes per stage
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStages * kSliceA;
constexpr int kOffStage = kOffB + kStages * kSliceB;  // epilogue staging: two [128 x 128 B] boxes
constexpr int kStageBytes = 2 * kTM * 128;
constexpr int kOffBar = kOffStage + kStageBytes;
constexpr int kNumBars = 2 * kStages + 4;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr int kSmem = kOffTmem + 16 + 1024;
static_assert(kSmem <= 232448, "shared memory budget");
constexpr int kThreads = 192;

struct ContractParams {
  int C, I, J, K;       // K in ELEMENTS
  int k_per_slice;      // elements per 128-byte slice (64 bf16, 128 e4m3)
  int is_f8;
  float alpha;
  int* status;
  int opm;              // 1: rows are (i, 32 channels), columns (j, 32 channels); the product is stored as [i, j, 32, 32]
  int part_rows;        // > 0: b is [parts, C, part_rows, K] (an all-gather's output); a multiple of 128
  // Operands and product as an all-to-all over the channel axis leaves / wants them (4-D tensor maps
  // {x, rows, c, part}).  mode 0: plain 3-D; 1: split by rows, [parts, C, rows / parts, X] with `div` rows per part
  // (a multiple of 128); 2: split along K, [parts, C, rows, K / parts] with `div` elements per part (a multiple of
  // the 128-byte slice).  The product only takes modes 0 and 1.
  int a_mode, a_div, b_mode, b_div, o_div;
  int o_peer;           // > 0: part q of the product (rows [q o_div, (q + 1) o_div)) is stored through peer map q
};

// The exchanged form's product with the all-to-all back to row shards done by the stores: one 3-D map {J, o_div, C} per
// destination rank, based at this rank's index of that rank's receive buffer [parts, C, o_div, J] (NVLink peer memory
// for the other ranks; plain TMA stores, no multicast).
constexpr int kMaxPeerParts = 8;
struct ContractPeerMaps {
  CUtensorMap o[kMaxPeerParts];
};

__global__ void __launch_bounds__(kThreads, 1)
contract_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_o, const __grid_constant__ ContractPeerMaps pm,
                const ContractParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = *reinterpret_cast<volatile int*>(prm.status);
    __syncthreads();
    if (s_abort != 0) return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int ti = (prm.I + kTM - 1) / kTM, tj = (prm.J + kTN - 1) / kTN;
  const int ntiles = prm.C * ti * tj;
  const int nslices = (prm.K + prm.k_per_slice - 1) / prm.k_per_slice;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_o);
    for (int q = 0; q < prm.o_peer; ++q) tma_prefetch_desc(&pm.o[q]);
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
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int c = tile / (ti * tj), rem = tile % (ti * tj), i0 = (rem / tj) * kTM, j0 = (rem % tj) * kTN;
        for (int s = 0; s < nslices; ++s, ++it) {
          const int st = it % kStages;
          ok = mbar_wait_deadline(&empty[st], ((it / kStages) & 1) ^ 1);
          if (!ok) { report_timeout(prm.status, 401); break; }
          mbar_arrive_expect_tx(&full[st], kSliceA + kSliceB);
          const int kx = s * prm.k_per_slice;
          if (prm.a_mode == 1)
            tma_load_4d(smem + kOffA + st * kSliceA, &tm_a, &full[st], kx, i0 % prm.a_div, c, i0 / prm.a_div);
          else if (prm.a_mode == 2)
            tma_load_4d(smem + kOffA + st * kSliceA, &tm_a, &full[st], kx % prm.a_div, i0, c, kx / prm.a_div);
          else
            tma_load_3d(smem + kOffA + st * kSliceA, &tm_a, &full[st], kx, i0, c);
          if (prm.b_mode == 2) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
              tma_load_4d(smem + kOffB + st * kSliceB + h * (128 * 128), &tm_b, &full[st], kx % prm.b_div, j0 + h * 128, c,
                          kx / prm.b_div);
          } else if (prm.part_rows > 0) {
            // rows j0 .. j0+255 of the gathered operand: two 128-row boxes, each inside one part
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int j = j0 + h * 128;
              tma_load_4d(smem + kOffB + st * kSliceB + h * (128 * 128), &tm_b, &full[st], s * prm.k_per_slice,
                          j % prm.part_rows, c, j / prm.part_rows);
            }
          } else {
            tma_load_3d(smem + kOffB + st * kSliceB, &tm_b, &full[st], s * prm.k_per_slice, j0, c);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // a product no wider than 128 columns (the outer product mean's output weights) runs N = 128 instructions: the
      // rows of the B box past J are fill values and their half of the accumulator would only hold zeros
      const uint32_t nn = prm.J <= 128 ? 128u : uint32_t(kTN);
      const uint32_t idesc = prm.is_f8 ? make_idesc(kTM, nn, 0, 0, 0, 0) : make_idesc(kTM, nn, 1, 1, 0, 0);
      const uint32_t a_base = smem_u32(smem + kOffA), b_base = smem_u32(smem + kOffB);
      int it = 0, n = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++n) {
        const int acc = n & 1;
        ok = mbar_wait_deadline(&acc_empty[acc], ((n >> 1) & 1) ^ 1);
        if (!ok) { report_timeout(prm.status, 402); break; }
        tc_fence_after();
        for (int s = 0; s < nslices; ++s, ++it) {
          const int st = it % kStages;
          ok = mbar_wait_deadline(&full[st], (it / kStages) & 1);
          if (!ok) { report_timeout(prm.status, 403); break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t a = desc_k_major(a_base + st * kSliceA + kk * 32, 128);
            const uint64_t b = desc_k_major(b_base + st * kSliceB + kk * 32, 128);
            if (prm.is_f8) mma_f8_ss(tmem + acc * kTN, a, b, idesc, (s | kk) != 0);
            else mma_f16_ss(tmem + acc * kTN, a, b, idesc, (s | kk) != 0);
          }
          mma_commit(&empty[st]);
        }
        if (ok) mma_commit(&acc_full[acc]);
      }
    }
    __syncwarp();
  } else {
    const int quad = warp & 3, row = quad * 32 + lane;
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const bool issuer = warp == 2 && lane == 0;
    uint8_t* stage = smem + kOffStage;
    int n = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++n) {
      const int c = tile / (ti * tj), rem = tile % (ti * tj), i0 = (rem / tj) * kTM, j0 = (rem % tj) * kTN;
      const int acc = n & 1;
      if (ok && !mbar_wait_deadline(&acc_full[acc], (n >> 1) & 1)) {
        report_timeout(prm.status, 404);
        ok = false;
      }
      tc_fence_after();
#pragma unroll 1
      for (int half = 0; half < (prm.J <= 128 ? 1 : 2); ++half) {
        if (issuer) tma_wait_group_read<0>();  // the previous store has finished reading the staging tile
        named_bar_sync(1, 128);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t r[32];
          tmem_ld_x32(tmem + lane_addr + acc * kTN + half * 128 + cc * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r[q * 8 + 0]) * prm.alpha, __uint_as_float(r[q * 8 + 1]) * prm.alpha);
            w.y = pack_bf16x2(__uint_as_float(r[q * 8 + 2]) * prm.alpha, __uint_as_float(r[q * 8 + 3]) * prm.alpha);
            w.z = pack_bf16x2(__uint_as_float(r[q * 8 + 4]) * prm.alpha, __uint_as_float(r[q * 8 + 5]) * prm.alpha);
            w.w = pack_bf16x2(__uint_as_float(r[q * 8 + 6]) * prm.alpha, __uint_as_float(r[q * 8 + 7]) * prm.alpha);
            const int chunk = cc * 4 + q;  // 16-byte chunk inside the 256-byte half row
            if (prm.opm)  // four [128 rows x 32 columns] sub-tiles, one per residue j: 64-byte swizzled rows
              *reinterpret_cast<uint4*>(stage + (chunk / 4) * (kTM * 64) + swz_off(row, chunk % 4, 64)) = w;
            else
              *reinterpret_cast<uint4*>(stage + (chunk / 8) * (kTM * 128) + swz_off(row, chunk % 8, 128)) = w;
          }
        }
        fence_proxy_async();
        named_bar_sync(1, 128);
        if (issuer && ok) {
          if (prm.opm) {
            // 4-D map (e, c, j, i) in memory order: a sub-tile is the 32 x 32 blocks of one j for the tile's four i
#pragma unroll
            for (int sub = 0; sub < 4; ++sub)
              tma_store_4d(&tm_o, stage + sub * (kTM * 64), 0, 0, (j0 + half * 128) / 32 + sub, i0 / 32);
          } else if (prm.o_peer > 0) {
            const CUtensorMap* m = &pm.o[i0 / prm.o_div];
            tma_store_3d(m, stage, j0 + half * 128, i0 % prm.o_div, c);
            tma_store_3d(m, stage + kTM * 128, j0 + half * 128 + 64, i0 % prm.o_div, c);
          } else if (prm.o_div > 0) {
            tma_store_4d(&tm_o, stage, j0 + half * 128, i0 % prm.o_div, c, i0 / prm.o_div);
            tma_store_4d(&tm_o, stage + kTM * 128, j0 + half * 128 + 64, i0 % prm.o_div, c, i0 / prm.o_div);
          } else {
            tma_store_3d(&tm_o, stage, j0 + half * 128, i0, c);
            tma_store_3d(&tm_o, stage + kTM * 128, j0 + half * 128 + 64, i0, c);
          }
          tma_commit_group();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
    if (issuer) tma_wait_group<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace
}  // namespace cfk

using namespace cfk;

namespace {
// opm_ri > 0: a is [(opm_ri x 32), k], b [(opm_rj x 32), k] and the product is stored as out[opm_ri, opm_rj, 32, 32]
// parts > 1: b is [parts, c, j / parts, k], the layout an all-gather of per-rank [c, j / parts, k] operands leaves
// xmode / xparts (exchanged form): mode 1 = operands split by rows over xparts, mode 2 = split along K; the product
// is then stored split by rows, [xparts, C, I / xparts, J]
int contract_impl(const void* a, const void* b, void* out, int c, int i, int j, int k, int dtype, float alpha, int opm_ri,
                  int opm_rj, int parts, void* stream, int xmode = 0, int xparts = 1, void* const* out_ptrs = nullptr,
                  int rank = 0) {
  if (out_ptrs != nullptr) {
    if (xmode == 0 || xparts > kMaxPeerParts || rank < 0 || rank >= xparts) return CFK_ERR_UNSUPPORTED;
    for (int q = 0; q < xparts; ++q)
      if (out_ptrs[q] == nullptr || !aligned16(out_ptrs[q])) return CFK_ERR_ALIGN;
    out = out_ptrs[rank];   // the 4-D map below is built but not used
  }
  if (a == nullptr || b == nullptr || out == nullptr) return CFK_ERR_NULL;
  if (c <= 0 || i <= 0 || j <= 0 || k <= 0) return CFK_ERR_SHAPE;
  if (dtype != CFK_BF16 && dtype != CFK_E4M3) return CFK_ERR_DTYPE;
  const int es = dtype == CFK_BF16 ? 2 : 1;
  // TMA strides are multiples of 16 bytes: K rows of the operands, J rows of the bf16 product
  if ((int64_t(k) * es) % 16 != 0 || j % 8 != 0) return CFK_ERR_SHAPE;
  if (!aligned16(a) || !aligned16(b) || !aligned16(out)) return CFK_ERR_ALIGN;
  CUtensorMap ta, tb, to;
  ContractPeerMaps pm{};
  int a_div = 0, b_div = 0, o_div = 0, part_rows = 0;
  if (xmode != 0) {
    const int kps = 128 / es;
    if (xparts <= 0 || i % xparts != 0 || (i / xparts) % kTM != 0) return CFK_ERR_SHAPE;
    o_div = i / xparts;
    if (xmode == 1) {
      if (j % xparts != 0 || (j / xparts) % 128 != 0) return CFK_ERR_SHAPE;
      a_div = i / xparts;
      b_div = j / xparts;
    } else {
      if (k % xparts != 0 || (k / xparts) % kps != 0) return CFK_ERR_SHAPE;
      a_div = b_div = k / xparts;
    }
    auto map4 = [&](CUtensorMap* m, const void* base, int rows) {
      // xmode 1: [parts, C, rows / parts, K]; xmode 2: [parts, C, rows, K / parts]
      const uint64_t rr = xmode == 1 ? uint64_t(rows / xparts) : uint64_t(rows);
      const uint64_t kk = xmode == 1 ? uint64_t(k) : uint64_t(k / xparts);
      uint64_t dims[4] = {kk, rr, uint64_t(c), uint64_t(xparts)};
      uint64_t str[3] = {kk * es, rr * kk * es, uint64_t(c) * rr * kk * es};
      uint32_t box[4] = {uint32_t(128 / es), 128, 1, 1};
      return make_tensor_map(m, base, dtype, 4, dims, str, box, 128);
    };
    int rc = map4(&ta, a, i);
    if (rc == CFK_OK) rc = map4(&tb, b, j);
    if (rc != CFK_OK) return rc;
    uint64_t dims[4] = {uint64_t(j), uint64_t(o_div), uint64_t(c), uint64_t(xparts)};
    uint64_t str[3] = {uint64_t(j) * 2, uint64_t(o_div) * j * 2, uint64_t(c) * o_div * j * 2};
    uint32_t box[4] = {64, kTM, 1, 1};
    rc = make_tensor_map(&to, out, CFK_BF16, 4, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
    if (out_ptrs != nullptr) {
      const uint64_t share = uint64_t(c) * o_div * j * 2;   // bytes one source rank fills of a receive buffer
      for (int q = 0; q < xparts; ++q) {
        uint64_t d3[3] = {uint64_t(j), uint64_t(o_div), uint64_t(c)};
        uint64_t s3[2] = {uint64_t(j) * 2, uint64_t(o_div) * j * 2};
        uint32_t b3[3] = {64, kTM, 1};
        rc = make_tensor_map(&pm.o[q], static_cast<char*>(out_ptrs[q]) + uint64_t(rank) * share, CFK_BF16, 3, d3, s3, b3, 128);
        if (rc != CFK_OK) return rc;
      }
    }
  } else {
  {
    uint64_t dims[3] = {uint64_t(k), uint64_t(i), uint64_t(c)};
    uint64_t str[2] = {uint64_t(k) * es, uint64_t(i) * k * es};
    uint32_t box[3] = {uint32_t(128 / es), kTM, 1};
    int rc = make_tensor_map(&ta, a, dtype, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  if (parts > 1) {
    if (j % parts != 0 || (j / parts) % 128 != 0) return CFK_ERR_SHAPE;
    part_rows = j / parts;
    // a box past the last part (J not a multiple of 256) reads the fill value, as the 3-D map does past J
    uint64_t dims[4] = {uint64_t(k), uint64_t(part_rows), uint64_t(c), uint64_t(parts)};
    uint64_t str[3] = {uint64_t(k) * es, uint64_t(part_rows) * k * es, uint64_t(c) * part_rows * k * es};
    uint32_t box[4] = {uint32_t(128 / es), 128, 1, 1};
    int rc = make_tensor_map(&tb, b, dtype, 4, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  } else {
    uint64_t dims[3] = {uint64_t(k), uint64_t(j), uint64_t(c)};
    uint64_t str[2] = {uint64_t(k) * es, uint64_t(j) * k * es};
    uint32_t box[3] = {uint32_t(128 / es), kTN, 1};
    int rc = make_tensor_map(&tb, b, dtype, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  if (opm_ri > 0) {
    // out [ri, rj, 32, 32] in memory order (e, c, j, i): a store box of 32 e x 32 c x 1 j x 4 i is one [128 rows][32
    // columns] sub-tile of the staging buffer
    uint64_t dims[4] = {32, 32, uint64_t(opm_rj), uint64_t(opm_ri)};
    uint64_t str[3] = {32 * 2, 32 * 32 * 2, uint64_t(opm_rj) * 32 * 32 * 2};
    uint32_t box[4] = {32, 32, 1, 4};
    int rc = make_tensor_map(&to, out, CFK_BF16, 4, dims, str, box, 64);
    if (rc != CFK_OK) return rc;
  } else {
    uint64_t dims[3] = {uint64_t(j), uint64_t(i), uint64_t(c)};
    uint64_t str[2] = {uint64_t(j) * 2, uint64_t(i) * j * 2};
    uint32_t box[3] = {64, kTM, 1};
    int rc = make_tensor_map(&to, out, CFK_BF16, 3, dims, str, box, 128);
    if (rc != CFK_OK) return rc;
  }
  }
  // exchanged form: the b boxes of mode 1 go through the gathered operand's path (two 128-row boxes, part = row / div)
  ContractParams prm{c, i, j, k, 128 / es, dtype == CFK_E4M3, alpha, device_status_word(), opm_ri > 0,
                     xmode == 1 ? b_div : part_rows, xmode, a_div, xmode == 2 ? 2 : 0, b_div, o_div,
                     out_ptrs != nullptr ? xparts : 0};
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  // a function attribute belongs to the current device: set on every launch, as the other launchers do
  if (cudaFuncSetAttribute(contract_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return CFK_ERR_LAUNCH;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ntiles = int64_t(c) * ((i + kTM - 1) / kTM) * ((j + kTN - 1) / kTN);
  const int grid = int(ntiles < sms ? ntiles : sms);
  contract_kernel<<<grid, kThreads, kSmem, static_cast<cudaStream_t>(stream)>>>(ta, tb, to, pm, prm);
  return check_launch();
}
}  // namespace

extern "C" int cfk_contract(const void* a, const void* b, void* out, int c, int i, int j, int k, int dtype, float alpha,
                            void* stream) {
  return contract_impl(a, b, out, c, i, j, k, dtype, alpha, 0, 0, 1, stream);
}

extern "C" int cfk_contract_gathered(const void* a, const void* b, void* out, int c, int i, int j, int k, int dtype,
                                     float alpha, int parts, void* stream) {
  if (parts <= 0) return CFK_ERR_SHAPE;
  return contract_impl(a, b, out, c, i, j, k, dtype, alpha, 0, 0, parts, stream);
}

extern "C" int cfk_contract_exchanged(const void* a, const void* b, void* out, int c, int i, int j, int k, int dtype,
                                      float alpha, int parts, int split_k, void* stream) {
  if (parts <= 0) return CFK_ERR_SHAPE;
  return contract_impl(a, b, out, c, i, j, k, dtype, alpha, 0, 0, 1, stream, split_k ? 2 : 1, parts);
}

extern "C" int cfk_contract_exchanged_peer(const void* a, const void* b, void* const* out_ptrs, int rank, int c, int i, int j,
                                           int k, int dtype, float alpha, int parts, int split_k, void* stream) {
  if (parts <= 0) return CFK_ERR_SHAPE;
  if (out_ptrs == nullptr) return CFK_ERR_NULL;
  return contract_impl(a, b, nullptr, c, i, j, k, dtype, alpha, 0, 0, 1, stream, split_k ? 2 : 1, parts, out_ptrs, rank);
}

extern "C" int cfk_opm_outer_product(const void* a, const void* b, void* out, int ri, int rj, int s, int dtype, void* stream) {
  if (ri <= 0 || rj <= 0 || s <= 0) return CFK_ERR_SHAPE;
  return contract_impl(a, b, out, 1, ri * 32, rj * 32, s, dtype, 1.0f, ri, rj, 1, stream);
}
