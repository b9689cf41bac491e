// Per-token MoE routing shared by the router kernel (lk_moe.cu) and the fused decode MoE kernels (lk_moeq8.cu).
#pragma once
#include "lk_common.cuh"

namespace lk {

// One token's routing by one warp (gen_moe.py:76-253 route_decode, _softmax_weight_*, scaled): lane l holds experts
// l, l + 32, ... (E <= 256). gating 1: softmax over all experts, top-k, optional renormalisation over the picked
// (w / max(sum, 6.1e-5)); 2: sigmoid (+ bias for the ranking only); 3: top-k on logit + bias, softmax over the picked.
// Top-k by ku rounds of (max, lowest index): ties go to the lower expert. Writes ids[0..ku) and wts[0..ku) (times
// scale). Shared by the router kernel and the fused decode MoE kernels, so both route bit for bit alike.
LK_DEV void route_token(int lane, int E, int ku, int gating, int norm, float scale, const float* __restrict__ logits,
                        const float* __restrict__ bias, int32_t* __restrict__ ids, float* __restrict__ wts) {
  auto wmax = [](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
  };
  auto wsum = [](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
  };
  float lg[8], prob[8], sc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = lane + 32 * j;
    lg[j] = e < E ? __ldg(logits + e) : -INFINITY;
  }
  if (gating == 1) {
    float m = lg[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) m = fmaxf(m, lg[j]);
    m = wmax(m);
    float den = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      prob[j] = lane + 32 * j < E ? expf(lg[j] - m) : 0.f;
      den += prob[j];
    }
    den = wsum(den);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      prob[j] = prob[j] / den;
      sc[j] = lg[j];   // softmax is monotonic in the logit: rank on the exact input
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = lane + 32 * j;
      const bool in = e < E;
      const float b = (bias && in) ? __ldg(bias + e) : 0.f;
      if (gating == 2) {
        prob[j] = in ? 1.0f / (1.0f + expf(-lg[j])) : 0.f;
        sc[j] = in ? prob[j] + b : -INFINITY;
      } else {
        prob[j] = in ? lg[j] + b : -INFINITY;
        sc[j] = prob[j];
      }
    }
  }
  // Ranking keys: the score's bits mapped so that unsigned order is float order (-0 as +0, NaN below everything,
  // as fmaxf ignores it); a slot past E never ranks. Each round is one warp max and one warp min (redux) over keys:
  // the highest score, then the lowest expert index holding it -- the lowest-index tie rule.
  auto okey = [](float v) {
    const uint32_t b = __float_as_uint(v + 0.0f);
    return v != v ? 0u : ((b & 0x80000000u) ? ~b : (b | 0x80000000u));
  };
  const uint32_t kPicked = okey(-INFINITY);
  uint32_t key[8];
  int my[8];   // round each held expert was picked in, or -1
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    key[j] = lane + 32 * j < E ? okey(sc[j]) : 0u;
    my[j] = -1;
  }
  float sel_sum = 0.f;
  for (int r = 0; r < ku; ++r) {
    uint32_t km = key[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) km = max(km, key[j]);
    km = __reduce_max_sync(0xffffffffu, km);
    uint32_t c = 0xffffffffu;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (lane + 32 * j < E && key[j] == km) c = min(c, uint32_t(lane + 32 * j));
    const int cand = int(__reduce_min_sync(0xffffffffu, c));
    float pw = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (lane + 32 * j == cand) {
        my[j] = r;
        key[j] = kPicked;   // as a picked score of -inf
        pw = prob[j];
      }
    if (lane == (cand & 31)) ids[r] = cand;
    sel_sum += __shfl_sync(0xffffffffu, pw, cand & 31);   // the picked probability, summed in round order
  }
  float m3 = 0.f, den3 = 1.f;
  if (gating == 3) {   // softmax over the picked
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (my[j] >= 0) m = fmaxf(m, prob[j]);
    m3 = wmax(m);
    float d = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (my[j] >= 0) d += expf(prob[j] - m3);
    den3 = wsum(d);
  }
  const float den = norm ? fmaxf(sel_sum, 6.103515625e-05f) : 1.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (my[j] >= 0) {
      const float wv = gating == 3 ? expf(prob[j] - m3) / den3 : prob[j] / den;
      wts[my[j]] = wv * scale;
    }
}

}  // namespace lk
