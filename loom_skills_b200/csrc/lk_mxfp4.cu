// MXFP4 (split planes) x FP8 prefill GEMM on tcgen05 -- replaces g_gemm_mxfp4s_{store,swiglu}_f8_m256_rdna4
// (gen_mxfp4s.py:50-500).
#include "lk_common.cuh"
#include "lk_internal.h"

namespace lk {

int gemm_mxfp4s(int mode, int order, int rows, int k, int n, const uint8_t* x8, const float* s8, const uint8_t* w,
                const uint8_t* ws, const uint8_t* w2, const uint8_t* w2s, float* y, cudaStream_t s) {
  (void)mode; (void)order; (void)rows; (void)k; (void)n; (void)x8; (void)s8; (void)w; (void)ws; (void)w2; (void)w2s;
  (void)y; (void)s;
  return LK_EUNSUPPORTED;
}

}  // namespace lk
