// One description of an attention problem for every layout the library accepts: heads-major
// [n,h,s,d], seq-major [n,s,h,d], and the packed projection [X,Y,G,H,D] read in place by rows or
// columns.  All four are the same kernel with different element strides.
#pragma once
#include <cstdint>

namespace cfk {

struct Strides {
  int64_t b, s, h;  // element strides of batch, sequence position and head; the head dim is contiguous
};

struct AttnProblem {
  const void* q;
  const void* k;
  const void* v;
  const void* gate;       // packed slot 3 or nullptr
  const void* gate_bias;  // [h, d] or nullptr
  const void* bias;       // [h, sq, sk] or nullptr
  const uint8_t* kmask;   // [nb, sk]
  void* out;
  float* lse;             // [nb, h, sq] or nullptr
  const int32_t* trim;    // nullptr, or [nb + 1]: per-batch last live key + 1, then the global limit
  Strides sq_, sk_, sv_, sg_, so_;
  int nb, h, sq, sk, d;
  float scale;
  int qk_e4m3;            // q and k are float8 e4m3 (strides in elements of that type); v, gate and out stay bf16
};

struct AttnBwdProblem {
  AttnProblem f;  // forward tensors (out = forward output)
  const void* dout;
  void* dq;
  void* dk;
  void* dv;
  float* dbias;  // [h, sq, sk] fp32 or nullptr
  Strides sdo, sdq, sdk, sdv;
};

inline Strides strides_heads_major(int h, int s, int d) { return {int64_t(h) * s * d, d, int64_t(s) * d}; }
inline Strides strides_seq_major(int h, int s, int d) { return {int64_t(s) * h * d, int64_t(h) * d, d}; }

}  // namespace cfk
