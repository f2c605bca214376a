// Row-block GEMM with fused prologue and epilogue: the shared engine of the HBM-bound projection kernels
// (gated dual projection, LayerNorm -> gated dual projection, triangle-multiplication epilogue, LayerNorm ->
// packed projection, output projection, outer-product-mean projection).
//
// A persistent CTA walks 128-row tiles.  Per tile:
//   producer thread     TMA loads of the tile of every source into a ring of shared-memory stages: a row-major
//                       source (optionally through a pair transpose) lands directly as the 128-byte-swizzled
//                       K-major UMMA operand, a channel-major source as [K][128 rows]
//   prologue warps (4)  one thread per row: LayerNorm the landed row in fp32 and rewrite it in place as bf16
//                       (a channel-major tile is transposed into the operand layout on the way)
//   MMA issuer          for every 128-column chunk of the output: acc0 = A0 W0 (and acc1 = A1 W1) with the
//                       weights resident in shared memory in their natural [K, N] layout (MN-major B operand)
//   epilogue warps (4)  TMEM -> registers -> bias / activation / mask / residual -> bf16 (or e4m3) -> global
//                       (row-major: straight from registers; channel-major: transposed through shared memory
//                       and written by TMA)
#pragma once
#include "attention_sm100.cuh"

namespace cfk {

enum RowGemmMode : int {
  kModeLinear = 0,  // out_i = rowmask * (acc_i + b_i) (+ residual)        (one or two independent outputs)
  kModeGdp = 1,     // out = rowmask * (acc0 + b0) * act(acc1 + b1)
  kModeEpi = 2,     // out = (acc0 + b0) * sigmoid(acc1 + b1) (+ residual | + raw rows of source 1)
};

struct RowSource {
  const void* x;           // nullptr: unused (source 1 then shares source 0's tile)
  const float* ln_scale;   // nullptr: no LayerNorm
  const float* ln_offset;
  int64_t stride_outer;    // row index of (outer o, inner r) = o * stride_outer + r * stride_inner   (row-major source)
  int64_t stride_inner;
  int channel_major;       // 1: x is [K, rows] (bf16 or fp32), rows indexed o * inner + r
  int dtype;               // CFK_BF16 / CFK_F32 (fp32 only for a channel-major source)
  int k;                   // 64, 128 or 256
};

struct RowGemmParams {
  RowSource src[2];
  int64_t outer, inner, inner_pad;  // tiles = outer * ceil(inner_pad / 128); rows r >= inner are zero padding
  float eps;
  int mode, swish;                  // swish: act = x * sigmoid(x) instead of sigmoid (GDP only)
  int relu;                         // kModeLinear: max(y, 0) after the bias
  int dual;                         // two accumulators per chunk
  int n_chunk;                      // columns per accumulator and chunk: 16..128, multiple of 16
  int chunks;                       // chunks handled per tile (weights of all of them stay resident)
  int chunk0;                       // global index of this launch's first chunk (launches may split the chunk list)
  int stream_weights;               // 1: all chunks in one launch, their weights streamed through a two-chunk ring
  int chunks_per_slot;              // global chunk c -> weight slot c / chunks_per_slot, column (c % chunks_per_slot) * n_chunk
  int bias_slot_stride;             // bias index = slot * bias_slot_stride + column
  const void* bias[2];              // bf16 [N] per accumulator or nullptr (indexed by absolute output column)
  int bias_len;                     // entries of each bias vector
  const void* rowmask;              // [rows] in src[0] order (bf16 or fp32 by rowmask_dtype) or nullptr
  int rowmask_dtype;
  // Row-block skipping (transition.py:29-38 of the reference): keep[rows] in src[0] order, or nullptr.  A 128-row tile
  // whose largest keep is > 0 is computed as usual; == 0 (padding) it gets zeros - or the residual / raw source-1 rows
  // where one is added - without any of the work; < 0 it is not written at all.  Rows in [inner, inner_pad) count as 0.
  const void* keep;
  int keep_dtype;
  // row-major output: out[i][row * ldo + col0[i] + chunk columns]; chunk c of accumulator i lands in array
  // (c / chunks_per_array), column (c % chunks_per_array) * n_chunk
  void* out[2];
  int64_t ldo;
  int chunks_per_array;
  int out_dtype;                    // CFK_BF16 or CFK_E4M3 (saturating, times out_scale)
  float out_scale;
  int out_channel_major;            // 1: out[array] is [n, outer, inner_pad] (lanes store consecutive rows of a channel)
  int n_valid;                      // real columns per array (columns past it are not stored)
  const void* residual;             // row-major [rows, ldo] (same dtype as out) or nullptr
  int add_source1;                  // kModeEpi: add the raw rows of source 1
  int* status;
};

int rowgemm_chunks_that_fit(const RowGemmParams& prm);
bool rowgemm_resident_is_tight(const RowGemmParams& prm, int chunks);  // resident weights leave < 2 stages + 2 staging buffers
bool rowgemm_stream_fits(const RowGemmParams& prm);    // room for a two-chunk weight ring, one stage and the staging buffer  // chunks whose weights fit beside two pipeline stages
int launch_rowgemm(const RowGemmParams& prm, const CUtensorMap& tw0, const CUtensorMap& tw1, cudaStream_t st);
int make_weight_map(CUtensorMap* m, const void* w, int slots, int k, int n);

// LayerNorm -> packed projection at 256 input channels with 128-column chunks (ln_proj256_sm100.cu); returns
// CFK_ERR_UNSUPPORTED for shapes the general engine should take.
int ln_proj256_launch(const void* x, const float* ln_scale, const float* ln_offset, const void* w, const void* keep,
                      int keep_dtype, void* out, int64_t m, int slots, int n, float eps, cudaStream_t st);

// LayerNorm -> packed projection at 128 input channels and at most 512 output columns, weights resident and LayerNorm
// folded around the GEMM (ln_proj128_sm100.cu); returns CFK_ERR_UNSUPPORTED for shapes the general engine should take.
int ln_proj128_launch(const void* x, const float* ln_scale, const float* ln_offset, const void* w, const void* keep,
                      int keep_dtype, void* out, int64_t m, int slots, int n, float eps, cudaStream_t st);

// LayerNorm -> gated dual projection at 128 channels in and 128 + 128 out, channel-major bf16 (ln_gdp128_sm100.cu);
// returns CFK_ERR_UNSUPPORTED for shapes the general engine should take.
int ln_gdp128_launch(const void* x, const float* ln_scale, const float* ln_offset, const void* wp, const void* bp,
                     const void* wg, const void* bg, const void* mask, void* const* left_ptrs, void* const* right_ptrs,
                     int rank, int parts, int64_t outer, int64_t inner, int64_t inner_pad, int64_t stride_outer,
                     int64_t stride_inner, float eps, cudaStream_t st);

// Triangle-multiplication output at 128 channels with LayerNorm folded around the GEMMs (trimul_epi128_sm100.cu);
// returns CFK_ERR_UNSUPPORTED for shapes the general engine should take.
int trimul_epi128_launch(const void* x_cm, const void* act, const float* in_scale, const float* in_offset, const float* ln_scale,
                         const float* ln_offset, const void* wo, const void* bo, const void* wg, const void* bg, void* out,
                         const void* keep, int keep_dtype, int64_t m, float eps, int add_input, cudaStream_t st);

}  // namespace cfk
