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

// Attention backward (attention_bwd.cu): dQ, dK, dV from Q, K, V, O, dO and
// the forward's LSE. All bf16 [batch, heads, seq, 128] with element strides;
// lse fp32 [batch, heads, seq_q]. ws: at least attention_bwd_workspace_bytes.
struct AttnBwdArgs {
  int batch, heads, seq_q, seq_k;
  const void* q; long long q_sb, q_sh, q_ss;
  const void* k; long long k_sb, k_sh, k_ss;
  const void* v; long long v_sb, v_sh, v_ss;
  const void* o; long long o_sb, o_sh, o_ss;
  const void* dout; long long do_sb, do_sh, do_ss;
  const float* lse;
  void* dq; long long dq_sb, dq_sh, dq_ss;
  void* dk; long long dk_sb, dk_sh, dk_ss;
  void* dv; long long dv_sb, dv_sh, dv_ss;
  float scale;
  int causal;
  int* err_word;
  unsigned long long timeout_ns;
};
size_t attention_bwd_workspace_bytes(const AttnBwdArgs& a);
cudaError_t launch_attention_bwd(const AttnBwdArgs& a, void* ws, size_t ws_bytes, cudaStream_t s);

}  // namespace grx
