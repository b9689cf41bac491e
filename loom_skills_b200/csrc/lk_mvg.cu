// Decode matvec for every GGUF format the reference decodes (formats.py:5-17) -- the formats k_mv does not cover
// (Q5_0, Q8_0, Q3_K, Q5_K, Q6_K, IQ4_XS, ggml 17-byte MXFP4) and any k of a whole number of blocks (a Q4_0 row of
// 704 values, for example) -- dense and per MoE assignment, with the expert epilogue:
//
//   g_mv_{fmt}_k{K}... (gen_llm.py:1159-1378)       y[t][n] (+)= sum_k x[t][k] W[n][k]  (swiglu: act(x.Wg, x.Wu))
//   g_moe_gu_{fmt} / g_moe_dn_{fmt} (gen_moe.py:535-727)
//
// The numerics are the reference's f32 decode: each 32-value group is dequantised to its exact f32 values (gguf's
// dequantize_blocks, lk_formats.cuh) and multiplied with the f32 activations, f32 accumulation.
//
// Design: a CTA of 8 warps owns 16 output rows (2 per warp) and up to TOK tokens; lane l takes the groups l, l + 32, ...
// of each row, decodes them from the packed bytes (byte loads: these blocks start at any even offset) and runs them
// against every token's activations, read straight from global memory (the CTA's rows share them in L1). A warp
// reduces its rows' partial sums by shuffles. Instruction-bound by design (the decode plus one FMA per value and
// token): the general path, where the Q4 formats' k_mv / k_mv_q8_rows are the tuned ones.
#include "lk_common.cuh"
#include "lk_formats.cuh"
#include "lk_internal.h"

namespace lk {
namespace {

constexpr int kGWarps = 8, kGRowsPerWarp = 2, kGRows = kGWarps * kGRowsPerWarp;

template <int XT>
LK_DEV void load_x32(const void* x, int64_t off, float (&xv)[32]) {
  if (XT == LK_F32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + off);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = __ldg(p + i);
      xv[4 * i] = f.x;
      xv[4 * i + 1] = f.y;
      xv[4 * i + 2] = f.z;
      xv[4 * i + 3] = f.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = __ldg(p + i);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (XT == LK_BF16) {
          xv[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
          xv[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
          xv[8 * i + 2 * j] = f.x;
          xv[8 * i + 2 * j + 1] = f.y;
        }
      }
    }
  }
}

template <int FMT, int XT, bool SWIGLU, bool MOE, int TOK>
__global__ void __launch_bounds__(kGWarps * 32) k_mvg(const MvArgs a) {
  constexpr int NW = SWIGLU ? 2 : 1;
  constexpr int gpb = fmt_qk(FMT) / 32;   // 32-value groups per block
  constexpr int bb = fmt_block_bytes(FMT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = a.k / 32;
  int xrow0, ntok, yrow0, e = 0;
  int64_t wbase = 0, w2base = 0;   // first weight row of this CTA's expert (MoE) in w / w2
  if (MOE) {
    const int asg = blockIdx.y;
    e = min(max(a.ids[asg], 0), a.n_experts - 1);
    wbase = int64_t(e) * a.rows_per_expert;
    w2base = int64_t(e) * a.rows_per_expert2 + a.w2_row_offset;
    xrow0 = asg / a.x_div;
    ntok = 1;
    yrow0 = asg;
  } else {
    xrow0 = blockIdx.y * TOK;
    ntok = min(TOK, a.tokens - xrow0);
    yrow0 = xrow0;
    w2base = a.w2_row_offset;
  }
  const uint8_t* w2 = a.w2 ? a.w2 : a.w;
#pragma unroll 1
  for (int rr = 0; rr < kGRowsPerWarp; ++rr) {
    const int row = blockIdx.x * kGRows + warp * kGRowsPerWarp + rr;
    if (row >= a.n) break;
    const uint8_t* wr[2] = {a.w + (wbase + row) * a.row_bytes, w2 + (w2base + row) * a.row_bytes};
    float acc[NW][TOK];
#pragma unroll
    for (int wi = 0; wi < NW; ++wi)
#pragma unroll
      for (int t = 0; t < TOK; ++t) acc[wi][t] = 0.f;
    for (int gi = lane; gi < groups; gi += 32) {
#pragma unroll
      for (int wi = 0; wi < NW; ++wi) {
        float v[32];
        group_values<FMT>(wr[wi] + (gi / gpb) * bb, gi % gpb, v);
#pragma unroll
        for (int t = 0; t < TOK; ++t) {
          if (t >= ntok) break;
          float xv[32];
          load_x32<XT>(a.x, int64_t(xrow0 + t) * a.k + gi * 32, xv);
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            s0 = fmaf(v[i], xv[i], s0);
            s1 = fmaf(v[i + 1], xv[i + 1], s1);
          }
          acc[wi][t] += s0 + s1;
        }
      }
    }
#pragma unroll
    for (int wi = 0; wi < NW; ++wi)
#pragma unroll
      for (int t = 0; t < TOK; ++t)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[wi][t] += __shfl_xor_sync(0xFFFFFFFFu, acc[wi][t], o);
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < TOK; ++t) {
        if (t >= ntok) break;
        float g = acc[0][t], u = acc[NW - 1][t];
        if (MOE && a.epi.bias) {
          g += __ldg(a.epi.bias + int64_t(e) * a.n + row);
          if (SWIGLU) u += __ldg(a.epi.bias2 + int64_t(e) * a.n + row);
        }
        const float val = SWIGLU ? act_apply(a.epi.act, g, u, a.epi.alpha, a.epi.limit) : g;
        float* yp = a.y + int64_t(yrow0 + t) * a.n + row;
        *yp = a.accumulate ? *yp + val : val;
      }
    }
  }
}

template <int FMT, int XT, bool SWIGLU, bool MOE, int TOK>
int launch_g(const MvArgs& a, int groups, cudaStream_t s) {
  const dim3 grid((a.n + kGRows - 1) / kGRows, groups);
  k_mvg<FMT, XT, SWIGLU, MOE, TOK><<<grid, kGWarps * 32, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

template <int FMT, int XT>
int mvg_x(const MvArgs& a, cudaStream_t s) {
  if (a.ids)
    return a.swiglu ? launch_g<FMT, XT, true, true, 1>(a, a.tokens, s) : launch_g<FMT, XT, false, true, 1>(a, a.tokens, s);
  if (a.tokens == 1)
    return a.swiglu ? launch_g<FMT, XT, true, false, 1>(a, 1, s) : launch_g<FMT, XT, false, false, 1>(a, 1, s);
  const int g = (a.tokens + 7) / 8;
  return a.swiglu ? launch_g<FMT, XT, true, false, 8>(a, g, s) : launch_g<FMT, XT, false, false, 8>(a, g, s);
}

template <int FMT>
int mvg_f(const MvArgs& a, cudaStream_t s) {
  switch (a.x_dtype) {
    case LK_F32: return mvg_x<FMT, LK_F32>(a, s);
    case LK_F16: return mvg_x<FMT, LK_F16>(a, s);
    case LK_BF16: return mvg_x<FMT, LK_BF16>(a, s);
  }
  return LK_EINVAL;
}

}  // namespace

int mv_generic(int fmt, const MvArgs& a, cudaStream_t s) {
  switch (fmt) {
    case LK_Q4_0: return mvg_f<LK_Q4_0>(a, s);
    case LK_IQ4_NL: return mvg_f<LK_IQ4_NL>(a, s);
    case LK_Q4_K: return mvg_f<LK_Q4_K>(a, s);
    case LK_Q5_0: return mvg_f<LK_Q5_0>(a, s);
    case LK_Q8_0: return mvg_f<LK_Q8_0>(a, s);
    case LK_Q5_K: return mvg_f<LK_Q5_K>(a, s);
    case LK_Q6_K: return mvg_f<LK_Q6_K>(a, s);
    case LK_IQ4_XS: return mvg_f<LK_IQ4_XS>(a, s);
    case LK_Q3_K: return mvg_f<LK_Q3_K>(a, s);
    case LK_MXFP4: return mvg_f<LK_MXFP4>(a, s);
  }
  return LK_EUNSUPPORTED;
}

}  // namespace lk
