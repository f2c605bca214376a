// Placeholder dispatch for the tcgen05 attention backward (filled in by the kernel below).
#include "attention_sm100.cuh"

namespace cfk {

bool attention_bwd_sm100_supported(const AttnBwdProblem& bp, int dtype) {
  (void)bp;
  (void)dtype;
  return false;
}
size_t attention_bwd_sm100_workspace(const AttnProblem& p) {
  (void)p;
  return 0;
}
int attention_bwd_sm100(const AttnBwdProblem& bp, void* workspace, cudaStream_t st) {
  (void)bp;
  (void)workspace;
  (void)st;
  return CFK_ERR_UNSUPPORTED;
}

}  // namespace cfk
