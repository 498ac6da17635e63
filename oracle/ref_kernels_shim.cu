// Test infrastructure, not part of the product: C-linkage entry points over the reference's own
// attention launchers, so that the GPU tests can load the reference's kernels -- compiled from the
// reference's sources for sm_100a by oracle/build_ref.sh into oracle/_ref/ -- with ctypes and use
// them as a second checker beside the stock CPU path.  The launchers (C++ linkage) are:
//   launch_flash_attention_hfma2   src/cuda/fp16_flash_attention_hfma2.cu:269-286 (non-causal fp16,
//                                  D in {40, 64, 80, 128, 160}, strided [B, H, S, D] views)
//   launch_attention_fp16          src/cuda/fp16_attention.cu:328-386 (fp16, D = 128, Sq = Sk,
//                                  contiguous, legacy default stream)
//   launch_attention_fp32          src/cuda/fp32_attention.cu:200-221 (fp32, non-causal, D <= 128,
//                                  Sq = Sk, contiguous, legacy default stream)
#include <cstdint>
#include <cuda_runtime.h>

bool launch_flash_attention_hfma2(const void* q, const void* k, const void* v, void* o, int B, int H, int Sq, int Sk,
                                  int D, const int64_t* qs, const int64_t* ks, const int64_t* vs, const int64_t* os,
                                  float scale, cudaStream_t stream);
void launch_attention_fp16(const void* q, const void* k, const void* v, void* output, int B, int H, int S, int D,
                           float scale_f32, bool causal);
void launch_attention_fp32(const float* input, const float* weight, const float* value, float* output, int B, int H,
                           int S, int D, float scale);

extern "C" {

// 0: launched; 1: the launcher declined the head dim.
int ref_flash_hfma2(const void* q, const void* k, const void* v, void* o, int B, int H, int Sq, int Sk, int D,
                    const int64_t* qs, const int64_t* ks, const int64_t* vs, const int64_t* os, float scale,
                    void* stream) {
  return launch_flash_attention_hfma2(q, k, v, o, B, H, Sq, Sk, D, qs, ks, vs, os, scale,
                                      static_cast<cudaStream_t>(stream))
             ? 0
             : 1;
}

void ref_attention_fp16(const void* q, const void* k, const void* v, void* o, int B, int H, int S, int D, float scale,
                        int causal) {
  launch_attention_fp16(q, k, v, o, B, H, S, D, scale, causal != 0);
}

void ref_attention_fp32(const float* q, const float* k, const float* v, float* o, int B, int H, int S, int D,
                        float scale) {
  launch_attention_fp32(q, k, v, o, B, H, S, D, scale);
}

}  // extern "C"
