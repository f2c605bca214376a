// C-ABI entry points of the projection family, all on the row-block GEMM engine.
#include "rowgemm_sm100.cuh"

using namespace cfk;

namespace cfk {
namespace {

bool k_ok(int k) { return k == 64 || k == 128 || k == 256; }

// Runs the chunk list in as many launches as the shared-memory budget needs (weights of a launch stay resident).
int run_chunks(RowGemmParams prm, int total_chunks, const void* w0, const void* w1, int slots, int n_cols,
               cudaStream_t st) {
  const int nsrc = prm.src[1].x != nullptr ? 2 : 1;
  const int k0 = prm.src[0].k, k1 = nsrc == 2 ? prm.src[1].k : k0;
  prm.chunks = 1;
  CUtensorMap tw0, tw1;
  int rc = make_weight_map(&tw0, w0, slots, k0, n_cols);
  if (rc != CFK_OK) return rc;
  if (prm.dual) {
    rc = make_weight_map(&tw1, w1, slots, k1, n_cols);
    if (rc != CFK_OK) return rc;
  } else {
    tw1 = tw0;
  }
  int fit = rowgemm_chunks_that_fit(prm);
  if (fit < 1) return CFK_ERR_UNSUPPORTED;
  prm.status = device_status_word();
  if (prm.status == nullptr) return CFK_ERR_LAUNCH;
  if ((fit < total_chunks || (total_chunks > 1 && rowgemm_resident_is_tight(prm, total_chunks))) && rowgemm_stream_fits(prm)) {
    // The weights of all chunks do not fit beside the pipeline, or fit only by squeezing it to one output staging
    // buffer (every store then waits for its own read): rather than one launch per group of chunks (each reading the
    // activations again from HBM), one launch streams the chunk weights from L2 through a two-slot ring.
    prm.chunk0 = 0;
    prm.chunks = total_chunks;
    prm.stream_weights = 1;
    return launch_rowgemm(prm, tw0, tw1, st);
  }
  for (int c0 = 0; c0 < total_chunks; c0 += fit) {
    prm.chunk0 = c0;
    prm.chunks = total_chunks - c0 < fit ? total_chunks - c0 : fit;
    rc = launch_rowgemm(prm, tw0, tw1, st);
    if (rc != CFK_OK) return rc;
  }
  return CFK_OK;
}

RowSource row_major(const void* x, int k, const float* scale, const float* offset) {
  RowSource s{};
  s.x = x; s.k = k; s.ln_scale = scale; s.ln_offset = offset; s.stride_outer = 0; s.stride_inner = 1; s.dtype = CFK_BF16;
  return s;
}

}  // namespace
}  // namespace cfk

extern "C" int cfk_gated_dual_proj(const void* x, const void* wp, const void* bp, const void* wg, const void* bg,
                                   const void* mask, void* out0, void* out1, int64_t m, int k, int p, int split,
                                   int channel_major, int activation, void* stream) {
  if (!x || !wp || !bp || !wg || !bg || !mask || !out0 || (split && !out1)) return CFK_ERR_NULL;
  if (m < 0 || p <= 0 || p % 8 != 0 || (split && p % 16 != 0)) return CFK_ERR_SHAPE;
  if (!k_ok(k)) return CFK_ERR_UNSUPPORTED;
  if (m == 0) return CFK_OK;
  const int width = split ? p / 2 : p;  // columns per output array
  RowGemmParams prm{};
  prm.src[0] = row_major(x, k, nullptr, nullptr);
  prm.outer = 1; prm.inner = m; prm.inner_pad = m;
  prm.mode = kModeGdp; prm.swish = activation == 1; prm.dual = 1;
  prm.n_chunk = width >= 128 ? 128 : 64;
  if (width % prm.n_chunk != 0 && split) return CFK_ERR_UNSUPPORTED;
  const int cpa = (width + prm.n_chunk - 1) / prm.n_chunk;
  prm.chunks_per_array = cpa;
  prm.chunks_per_slot = split ? 2 * cpa : cpa;
  prm.bias_slot_stride = 0;
  prm.bias[0] = bp; prm.bias[1] = bg; prm.bias_len = p;
  prm.rowmask = mask; prm.rowmask_dtype = CFK_BF16;
  prm.out[0] = out0; prm.out[1] = out1;
  prm.ldo = width; prm.out_dtype = CFK_BF16; prm.out_scale = 1.f;
  prm.out_channel_major = channel_major; prm.n_valid = width;
  return run_chunks(prm, split ? 2 * cpa : cpa, wp, wg, 1, p, static_cast<cudaStream_t>(stream));
}

extern "C" int cfk_ln_gated_dual_proj(const void* x, const float* ln_scale, const float* ln_offset, const void* wp,
                                      const void* bp, const void* wg, const void* bg, const void* mask, void* left,
                                      void* right, int64_t a, int64_t b, int k, int p, int transpose, int pad, int fp8,
                                      float fp8_scale, float eps, void* stream) {
  if (!x || !ln_scale || !ln_offset || !wp || !bp || !wg || !bg || !mask || !left || !right) return CFK_ERR_NULL;
  if (a <= 0 || b < 0 || p <= 0 || p % 16 != 0 || pad < 1) return CFK_ERR_SHAPE;
  if (fp8 && !(fp8_scale > 0.f)) return CFK_ERR_SHAPE;
  if (!k_ok(k)) return CFK_ERR_UNSUPPORTED;
  const int ci = p / 2;
  RowGemmParams prm{};
  prm.src[0] = row_major(x, k, ln_scale, ln_offset);
  if (b == 0) {  // 2-D [M, K]
    prm.outer = 1; prm.inner = a;
  } else if (!transpose) {  // pair [A, B, K]: block rows run along b of row a
    prm.outer = a; prm.inner = b; prm.src[0].stride_outer = b; prm.src[0].stride_inner = 1;
  } else {  // read transposed: outer b, rows run along a
    prm.outer = b; prm.inner = a; prm.src[0].stride_outer = 1; prm.src[0].stride_inner = b;
  }
  prm.inner_pad = (prm.inner + pad - 1) / pad * pad;
  prm.eps = eps;
  if (k == 128 && p == 256 && !fp8) {  // the triangle multiplication's shape has a kernel of its own
    const int rc = ln_gdp128_launch(x, ln_scale, ln_offset, wp, bp, wg, bg, mask, &left, &right, 0, 1, prm.outer, prm.inner,
                                    prm.inner_pad, prm.src[0].stride_outer, prm.src[0].stride_inner, eps,
                                    static_cast<cudaStream_t>(stream));
    if (rc != CFK_ERR_UNSUPPORTED) return rc;
  }
  prm.mode = kModeGdp; prm.dual = 1;
  prm.n_chunk = ci >= 128 ? 128 : 64;
  if (ci % prm.n_chunk != 0) return CFK_ERR_UNSUPPORTED;
  const int cpa = ci / prm.n_chunk;
  prm.chunks_per_array = cpa; prm.chunks_per_slot = 2 * cpa; prm.bias_slot_stride = 0;
  prm.bias[0] = bp; prm.bias[1] = bg; prm.bias_len = p;
  prm.rowmask = mask; prm.rowmask_dtype = CFK_BF16;
  prm.out[0] = left; prm.out[1] = right;
  prm.ldo = ci; prm.out_dtype = fp8 ? CFK_E4M3 : CFK_BF16; prm.out_scale = fp8 ? fp8_scale : 1.f;
  prm.out_channel_major = 1; prm.n_valid = ci;
  // the mask doubles as the row-block filter: a tile of zeros skips the work, a tile below zero is left unwritten
  prm.keep = mask; prm.keep_dtype = CFK_BF16;
  return run_chunks(prm, 2 * cpa, wp, wg, 1, p, static_cast<cudaStream_t>(stream));
}

extern "C" int cfk_ln_gated_dual_proj_peer(const void* x, const float* ln_scale, const float* ln_offset, const void* wp,
                                           const void* bp, const void* wg, const void* bg, const void* mask,
                                           void* const* left_ptrs, void* const* right_ptrs, int rank, int parts, int64_t a,
                                           int64_t b, int k, int p, int transpose, int pad, float eps, void* stream) {
  if (!x || !ln_scale || !ln_offset || !wp || !bp || !wg || !bg || !mask || !left_ptrs || !right_ptrs) return CFK_ERR_NULL;
  if (a <= 0 || b <= 0 || pad < 1 || parts < 1 || rank < 0 || rank >= parts) return CFK_ERR_SHAPE;
  if (k != 128 || p != 256) return CFK_ERR_UNSUPPORTED;
  const int64_t outer = transpose ? b : a, inner = transpose ? a : b;
  const int64_t inner_pad = (inner + pad - 1) / pad * pad;
  return ln_gdp128_launch(x, ln_scale, ln_offset, wp, bp, wg, bg, mask, left_ptrs, right_ptrs, rank, parts, outer, inner,
                          inner_pad, transpose ? 1 : b, transpose ? b : 1, eps, static_cast<cudaStream_t>(stream));
}

extern "C" int cfk_trimul_epilogue(const void* x_cm, int x_cm_dtype, const void* act, const float* in_scale,
                                   const float* in_offset, const float* ln_scale, const float* ln_offset,
                                   const void* wo, const void* bo, const void* wg, const void* bg, const void* residual,
                                   const void* keep, int keep_dtype, void* out, int64_t m, int c, int ca, int o, float eps,
                                   int add_input, void* stream) {
  if (!x_cm || !act || !ln_scale || !ln_offset || !wo || !bo || !wg || !bg || !out) return CFK_ERR_NULL;
  if (m < 0 || o <= 0 || o % 8 != 0) return CFK_ERR_SHAPE;
  if (!(c == 64 || c == 128) || !k_ok(ca) || (add_input && ca != o)) return CFK_ERR_UNSUPPORTED;
  if (x_cm_dtype != CFK_BF16 && x_cm_dtype != CFK_F32) return CFK_ERR_DTYPE;
  if (m == 0) return CFK_OK;
  if (c == 128 && ca == 128 && o == 128 && x_cm_dtype == CFK_BF16 && residual == nullptr &&
      (in_scale == nullptr) == (in_offset == nullptr)) {  // the block's shape has a kernel of its own
    const int rc = trimul_epi128_launch(x_cm, act, in_scale, in_offset, ln_scale, ln_offset, wo, bo, wg, bg, out, keep,
                                        keep_dtype, m, eps, add_input, static_cast<cudaStream_t>(stream));
    if (rc != CFK_ERR_UNSUPPORTED) return rc;
  }
  RowGemmParams prm{};
  prm.src[0].x = x_cm; prm.src[0].k = c; prm.src[0].channel_major = 1; prm.src[0].dtype = x_cm_dtype;
  prm.src[0].ln_scale = ln_scale; prm.src[0].ln_offset = ln_offset; prm.src[0].stride_outer = 0; prm.src[0].stride_inner = 1;
  prm.src[1] = row_major(act, ca, in_scale, in_offset);
  prm.outer = 1; prm.inner = m; prm.inner_pad = m; prm.eps = eps;
  prm.mode = kModeEpi; prm.dual = 1;
  prm.n_chunk = o >= 128 ? 128 : 64;
  const int cpa = (o + prm.n_chunk - 1) / prm.n_chunk;
  prm.chunks_per_array = cpa; prm.chunks_per_slot = cpa; prm.bias_slot_stride = 0;
  prm.bias[0] = bo; prm.bias[1] = bg; prm.bias_len = o;
  prm.out[0] = out; prm.ldo = o; prm.out_dtype = CFK_BF16; prm.out_scale = 1.f; prm.n_valid = o;
  prm.residual = residual; prm.add_source1 = add_input;
  prm.keep = keep; prm.keep_dtype = keep_dtype;
  // the two weights have different K (c and ca): separate maps inside run_chunks use src[0].k and src[1].k
  return run_chunks(prm, cpa, wo, wg, 1, o, static_cast<cudaStream_t>(stream));
}

extern "C" int cfk_ln_projection(const void* x, const float* ln_scale, const float* ln_offset, const void* w,
                                 const void* keep, int keep_dtype, void* p_out, int64_t m, int a, int g, int n, int f8,
                                 float f8_scale, float eps, void* stream) {
  if (!x || !ln_scale || !ln_offset || !w || !p_out) return CFK_ERR_NULL;
  if (m < 0 || g <= 0 || n <= 0 || n % 8 != 0) return CFK_ERR_SHAPE;
  if (!k_ok(a)) return CFK_ERR_UNSUPPORTED;
  if (m == 0) return CFK_OK;
  if (a == 256 && !f8) {  // the MSA shape has a kernel of its own (128-column chunks)
    const int rc = ln_proj256_launch(x, ln_scale, ln_offset, w, keep, keep_dtype, p_out, m, g, n, eps,
                                     static_cast<cudaStream_t>(stream));
    if (rc != CFK_ERR_UNSUPPORTED) return rc;
  }
  if (a == 128 && !f8) {  // the pair shape has a kernel of its own (weights resident, LayerNorm folded around the GEMM)
    const int rc = ln_proj128_launch(x, ln_scale, ln_offset, w, keep, keep_dtype, p_out, m, g, n, eps,
                                     static_cast<cudaStream_t>(stream));
    if (rc != CFK_ERR_UNSUPPORTED) return rc;
  }
  RowGemmParams prm{};
  prm.src[0] = row_major(x, a, ln_scale, ln_offset);
  prm.outer = 1; prm.inner = m; prm.inner_pad = m; prm.eps = eps;
  prm.mode = kModeLinear; prm.dual = 0;
  // 256 input channels: 64-column chunks leave room for two stages and two staging buffers beside the weight ring
  prm.n_chunk = (n >= 128 && a != 256) ? 128 : 64;
  if (n % prm.n_chunk != 0 && g > 1) return CFK_ERR_UNSUPPORTED;
  const int cps = (n + prm.n_chunk - 1) / prm.n_chunk;
  prm.chunks_per_slot = cps; prm.chunks_per_array = g * cps; prm.bias_slot_stride = 0;
  prm.out[0] = p_out; prm.ldo = int64_t(g) * n; prm.n_valid = g * n;
  prm.out_dtype = f8 ? CFK_E4M3 : CFK_BF16; prm.out_scale = f8 ? f8_scale : 1.f;
  prm.keep = keep; prm.keep_dtype = keep_dtype;
  return run_chunks(prm, g * cps, w, nullptr, g, n, static_cast<cudaStream_t>(stream));
}

extern "C" int cfk_transition_hidden(const void* x, const float* ln_scale, const float* ln_offset, const void* w1,
                                     const void* b1, const void* keep, int keep_dtype, void* h_out, int64_t m, int c,
                                     int hdim, float eps, void* stream) {
  if (!x || !ln_scale || !ln_offset || !w1 || !b1 || !h_out) return CFK_ERR_NULL;
  if (m < 0 || hdim <= 0 || hdim % 64 != 0) return CFK_ERR_SHAPE;
  if (!k_ok(c)) return CFK_ERR_UNSUPPORTED;
  if (m == 0) return CFK_OK;
  RowGemmParams prm{};
  prm.src[0] = row_major(x, c, ln_scale, ln_offset);
  prm.outer = 1; prm.inner = m; prm.inner_pad = m; prm.eps = eps;
  prm.mode = kModeLinear; prm.dual = 0; prm.relu = 1;
  prm.n_chunk = (hdim % 128 == 0 && c != 256) ? 128 : 64;  // as in cfk_ln_projection
  const int cps = hdim / prm.n_chunk;
  prm.chunks_per_slot = cps; prm.chunks_per_array = cps; prm.bias_slot_stride = 0;
  prm.bias[0] = b1; prm.bias_len = hdim;
  prm.out[0] = h_out; prm.ldo = hdim; prm.n_valid = hdim; prm.out_dtype = CFK_BF16; prm.out_scale = 1.f;
  prm.keep = keep; prm.keep_dtype = keep_dtype;
  return run_chunks(prm, cps, w1, nullptr, 1, hdim, static_cast<cudaStream_t>(stream));
}

extern "C" int cfk_output_projection(const void* o, const void* w, const void* b, const void* residual, const void* keep,
                                     int keep_dtype, void* out, int64_t m, int k, int c, void* stream) {
  if (!o || !w || !b || !out) return CFK_ERR_NULL;
  if (m < 0 || c <= 0 || c % 8 != 0) return CFK_ERR_SHAPE;
  if (!k_ok(k)) return CFK_ERR_UNSUPPORTED;
  if (m == 0) return CFK_OK;
  RowGemmParams prm{};
  prm.src[0] = row_major(o, k, nullptr, nullptr);
  prm.outer = 1; prm.inner = m; prm.inner_pad = m;
  prm.mode = kModeLinear; prm.dual = 0;
  prm.n_chunk = (c >= 128 && k != 256) ? 128 : 64;  // as in cfk_ln_projection
  const int cps = (c + prm.n_chunk - 1) / prm.n_chunk;
  prm.chunks_per_slot = cps; prm.chunks_per_array = cps;
  prm.bias[0] = b; prm.bias_len = c;
  prm.out[0] = out; prm.ldo = c; prm.n_valid = c; prm.out_dtype = CFK_BF16; prm.out_scale = 1.f;
  prm.residual = residual;
  prm.keep = keep; prm.keep_dtype = keep_dtype;
  return run_chunks(prm, cps, w, nullptr, 1, c, static_cast<cudaStream_t>(stream));
}

extern "C" int cfk_opm_projection(const void* x, const float* ln_scale, const float* ln_offset, const void* lw,
                                  const void* lb, const void* rw, const void* rb, const void* mask, void* left,
                                  void* right, int64_t m, int c, int k, float eps, void* stream) {
  if (!x || !ln_scale || !ln_offset || !lw || !lb || !rw || !rb || !mask || !left || !right) return CFK_ERR_NULL;
  if (m < 0 || k <= 0 || k % 8 != 0 || k > 128) return CFK_ERR_SHAPE;
  if (!k_ok(c)) return CFK_ERR_UNSUPPORTED;
  if (m == 0) return CFK_OK;
  RowGemmParams prm{};
  prm.src[0] = row_major(x, c, ln_scale, ln_offset);
  prm.outer = 1; prm.inner = m; prm.inner_pad = m; prm.eps = eps;
  prm.mode = kModeLinear; prm.dual = 1;  // two independent outputs from one normed tile
  prm.n_chunk = k > 64 ? 128 : 64;
  prm.chunks_per_slot = 1; prm.chunks_per_array = 1;
  prm.bias[0] = lb; prm.bias[1] = rb; prm.bias_len = k;
  prm.rowmask = mask; prm.rowmask_dtype = CFK_BF16;
  prm.out[0] = left; prm.out[1] = right; prm.ldo = k; prm.n_valid = k; prm.out_dtype = CFK_BF16; prm.out_scale = 1.f;
  return run_chunks(prm, 1, lw, rw, 1, k, static_cast<cudaStream_t>(stream));
}

