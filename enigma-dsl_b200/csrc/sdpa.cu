// sdpa.cu — bf16 attention dispatcher: tensor-core FlashAttention kernel for
// head_dim 64 / 128 (sdpa_tc.cu), CUDA-core online softmax otherwise (sdpa_simt.cu).
#include "common.cuh"

namespace enigma {
cudaError_t sdpa_simt_bf16_launch(const void* Q, const void* K, const void* V, void* O, int64_t B,
                                  int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D,
                                  float scale, bool causal, cudaStream_t s);
bool sdpa_tc_supported(const void* Q, const void* K, const void* V, const void* O, int64_t B,
                       int64_t Hq, int64_t Sq, int64_t Sk, int64_t D);
cudaError_t sdpa_tc_bf16_launch(const void* Q, const void* K, const void* V, void* O, int64_t B,
                                int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D,
                                float scale, bool causal, cudaStream_t s);

cudaError_t sdpa_bf16_launch(const void* Q, const void* K, const void* V, void* O, int64_t B,
                             int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D,
                             float scale, bool causal, cudaStream_t s) {
  if (sdpa_tc_supported(Q, K, V, O, B, Hq, Sq, Skv, D)) {
    note_kernel("sdpa_fwd_tc_kernel");
    return sdpa_tc_bf16_launch(Q, K, V, O, B, Hq, Hkv, Sq, Skv, D, scale, causal, s);
  }
  note_kernel("sdpa_simt_kernel");
  return sdpa_simt_bf16_launch(Q, K, V, O, B, Hq, Hkv, Sq, Skv, D, scale, causal, s);
}
}  // namespace enigma
