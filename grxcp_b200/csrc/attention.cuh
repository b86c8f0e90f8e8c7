// Host/device interface of the fused attention forward kernel.
#pragma once

#include <cuda_runtime.h>

namespace grx {

struct AttnArgs {
  int batch, heads, seq_q, seq_k;
  const void* q; long long q_sb, q_sh, q_ss;  // element strides; headDim contiguous
  const void* k; long long k_sb, k_sh, k_ss;
  const void* v; long long v_sb, v_sh, v_ss;
  void* o; long long o_sb, o_sh, o_ss;
  float* lse;          // [batch, heads, seq_q] or null
  float scale;
  int causal;
  int* err_word;
  unsigned long long timeout_ns;
};

// headDim 128, bf16. cudaErrorNotSupported when a stride or base address
// defeats TMA (16-byte rule).
cudaError_t launch_attention_fwd(const AttnArgs& a, int num_sms, cudaStream_t s);

}  // namespace grx
