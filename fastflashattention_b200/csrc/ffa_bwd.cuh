// ffa_bwd.cuh — deterministic attention backward for sm_100a (placeholder).
#pragma once
#include "ffa_common.cuh"
namespace ffa {
int launch_bwd(const BwdArgs& a, cudaStream_t stream) {
  (void)a; (void)stream;
  return set_error(FFA_ERR_UNSUPPORTED, "backward not built yet");
}
}  // namespace ffa
