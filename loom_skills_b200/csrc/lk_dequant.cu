// Standalone block dequantisation and the activation producers (row scale to f16, fp8 twin).
//
// lk_dequant   replaces the value helpers @g_<fmt>_values (quant_values.loom:18-91, 386-408; gen_llm.py:288-315,
//              786-895) and the GEMM's f16 staging dequant16 (gen_gemm.py:281-532, moe_q4_0.py:11-38).
// row scales   g_row_scale_f16 (gen_llm.py:1843-1912) and its fp8 twin (gen_mxfp4s.py:852-870, 887-938).
// act * up     g_silu_mul (gen_llm.py:5717-5745) and its GEGLU form (gen_llm.py:5670-5716).
#include <algorithm>

#include "lk_common.cuh"
#include "lk_formats.cuh"
#include "lk_internal.h"

namespace lk {

__constant__ float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

// one thread = one 32-value group; writes 32 outputs (exact f32 values, or the GEMM's f16 staging)
template <int FMT, bool F16OUT>
__global__ void k_dequant(const uint8_t* __restrict__ w, const uint8_t* __restrict__ ws, int64_t groups,
                          void* __restrict__ out) {
  int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= groups) return;
  float v[32];
  __half h[32];
  if (FMT == LK_MXFP4S) {   // nibble plane (pairs order: element 2i low nibble, 2i+1 high) + scale plane
    const uint8_t* b = w + gid * 16;
    int e = ws[gid];
    float s = e >= 1 ? __uint_as_float(uint32_t(e) << 23) : __uint_as_float(0x00400000u);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      int lo = b[i] & 15, hi = b[i] >> 4;
      v[2 * i] = ((lo & 8) ? -kE2M1[lo & 7] : kE2M1[lo & 7]) * s;
      v[2 * i + 1] = ((hi & 8) ? -kE2M1[hi & 7] : kE2M1[hi & 7]) * s;
    }
    if (F16OUT)
#pragma unroll
      for (int i = 0; i < 32; ++i) h[i] = __float2half_rn(v[i]);
  } else {
    constexpr int gpb = fmt_qk(FMT) / 32;   // groups per block
    const uint8_t* b = w + (gid / gpb) * fmt_block_bytes(FMT);
    const int j = int(gid % gpb);
    if (F16OUT) group_f16<FMT>(b, j, h);
    else group_values<FMT>(b, j, v);
  }
  if (F16OUT) {
    uint4* o = reinterpret_cast<uint4*>(static_cast<__half*>(out) + gid * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = reinterpret_cast<uint4*>(h)[i];
  } else {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + gid * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

template <int FMT>
static int launch_dequant(const void* w, const void* ws, int64_t groups, void* out, bool f16, cudaStream_t s) {
  int threads = 128;
  int64_t blocks = (groups + threads - 1) / threads;
  if (f16)
    k_dequant<FMT, true><<<unsigned(blocks), threads, 0, s>>>((const uint8_t*)w, (const uint8_t*)ws, groups, out);
  else
    k_dequant<FMT, false><<<unsigned(blocks), threads, 0, s>>>((const uint8_t*)w, (const uint8_t*)ws, groups, out);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

int dequant(int fmt, const void* w, const void* ws, int64_t n, void* out, int out_dtype, cudaStream_t s) {
  int64_t groups = n / 32;
  bool f16 = out_dtype == LK_F16;
  switch (fmt) {
    case LK_Q4_0: return launch_dequant<LK_Q4_0>(w, ws, groups, out, f16, s);
    case LK_IQ4_NL: return launch_dequant<LK_IQ4_NL>(w, ws, groups, out, f16, s);
    case LK_Q4_K: return launch_dequant<LK_Q4_K>(w, ws, groups, out, f16, s);
    case LK_MXFP4: return launch_dequant<LK_MXFP4>(w, ws, groups, out, f16, s);
    case LK_MXFP4S: return launch_dequant<LK_MXFP4S>(w, ws, groups, out, f16, s);
    case LK_Q5_0: return launch_dequant<LK_Q5_0>(w, ws, groups, out, f16, s);
    case LK_Q8_0: return launch_dequant<LK_Q8_0>(w, ws, groups, out, f16, s);
    case LK_Q5_K: return launch_dequant<LK_Q5_K>(w, ws, groups, out, f16, s);
    case LK_Q6_K: return launch_dequant<LK_Q6_K>(w, ws, groups, out, f16, s);
    case LK_IQ4_XS: return launch_dequant<LK_IQ4_XS>(w, ws, groups, out, f16, s);
    case LK_Q3_K: return launch_dequant<LK_Q3_K>(w, ws, groups, out, f16, s);
    case LK_IQ3_S: return launch_dequant<LK_IQ3_S>(w, ws, groups, out, f16, s);
  }
  return LK_EINVAL;
}

// ---------------------------------------------------------------------------------------------------------------
// row scales: one 256-thread block per row
// ---------------------------------------------------------------------------------------------------------------
template <bool BF16>
LK_DEV float load_x(const void* x, int64_t i) {
  if (BF16) return bf2f(static_cast<const uint16_t*>(x)[i]);
  return static_cast<const float*>(x)[i];
}

LK_DEV float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < (blockDim.x >> 5) ? red[l] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <bool BF16, bool F8>
__global__ void __launch_bounds__(256) k_row_scale(int k, const void* __restrict__ x, float* __restrict__ scales,
                                                   __half* __restrict__ x16, uint8_t* __restrict__ x8,
                                                   float* __restrict__ s8) {
  __shared__ float red[8];
  int64_t row = blockIdx.x;
  const int64_t base = row * k;
  float m = 0.0f;
  for (int i = threadIdx.x; i < k; i += 256) m = fmaxf(m, fabsf(load_x<BF16>(x, base + i)));
  m = block_max(m, red);
  int biased = int((__float_as_uint(m) >> 23) & 255);
  int e = min(max(biased - 127 - 13, 0), 100);
  float s = __uint_as_float(uint32_t(127 - e) << 23), inv = __uint_as_float(uint32_t(127 + e) << 23);
  float fs = 0.0f, finv = 0.0f;
  if (F8) {
    fs = __uint_as_float(uint32_t(min(max(261 - biased, 1), 254)) << 23);
    finv = __uint_as_float(uint32_t(min(max(biased - 15, 1), 254)) << 23);
  }
  for (int i = threadIdx.x; i < k; i += 256) {
    float v = load_x<BF16>(x, base + i);
    if (x16) x16[base + i] = __float2half_rn(v * s);
    if (F8) {
      // e4m3, round to nearest even, saturating finite (the fptrunc of the producer twin)
      __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(v * fs, __NV_SATFINITE, __NV_E4M3);
      x8[base + i] = q;
    }
  }
  if (threadIdx.x == 0) {
    if (scales) {
      scales[2 * row] = s;
      scales[2 * row + 1] = inv;
    }
    if (F8) {
      s8[2 * row] = fs;
      s8[2 * row + 1] = finv;
    }
  }
}

// 8 consecutive values of row `src` from column 8 * v (16 or 32 bytes, one or two vector loads)
template <bool BF16>
LK_DEV void load8(const void* x, int64_t off, float (&v)[8]) {
  if (BF16) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + off);
    const float4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// The same row scale with one warp per output row (8 rows per CTA) and 16-byte vector accesses; k % 8 == 0. GATHER:
// output row r is the row scale of x[rowmap[r] / ku] (a zero row where rowmap[r] < 0) -- the MoE gate/up activations
// in bucket order, so the grouped GEMM reads plain tiles instead of gathering rows.
template <bool BF16, bool F8, bool GATHER>
__global__ void __launch_bounds__(256) k_row_scale_w(int rows, int k, const void* __restrict__ x,
                                                     const int32_t* __restrict__ rowmap, int ku,
                                                     float* __restrict__ scales, __half* __restrict__ x16,
                                                     uint8_t* __restrict__ x8, float* __restrict__ s8) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  int64_t src = row;
  if (GATHER) {
    const int a = __ldg(rowmap + row);
    src = a >= 0 ? a / ku : -1;
  }
  const int nv = k / 8;
  float m = 0.0f;
  if (src >= 0)
#pragma unroll 4
    for (int i = lane; i < nv; i += 32) {
      float v[8];
      load8<BF16>(x, src * k + 8 * i, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int biased = int((__float_as_uint(m) >> 23) & 255);
  const int e = min(max(biased - 127 - 13, 0), 100);
  const float s = __uint_as_float(uint32_t(127 - e) << 23), inv = __uint_as_float(uint32_t(127 + e) << 23);
  float fs = 0.0f, finv = 0.0f;
  if (F8) {
    fs = __uint_as_float(uint32_t(min(max(261 - biased, 1), 254)) << 23);
    finv = __uint_as_float(uint32_t(min(max(biased - 15, 1), 254)) << 23);
  }
  const int64_t base = row * k;
#pragma unroll 2
  for (int i = lane; i < nv; i += 32) {
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (src >= 0) load8<BF16>(x, src * k + 8 * i, v);
    if (x16) {
      uint32_t h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        h[j] = uint32_t(__half_as_ushort(__float2half_rn(v[2 * j] * s))) |
               (uint32_t(__half_as_ushort(__float2half_rn(v[2 * j + 1] * s))) << 16);
      *reinterpret_cast<uint4*>(x16 + base + 8 * i) = make_uint4(h[0], h[1], h[2], h[3]);
    }
    if (F8) {   // pairs through the two-value conversion: the same e4m3 rounding, half the instructions
      uint32_t q[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 8; j += 2)
        q[j >> 2] |= uint32_t(__nv_cvt_float2_to_fp8x2(make_float2(v[j] * fs, v[j + 1] * fs), __NV_SATFINITE,
                                                       __NV_E4M3))
                     << (8 * (j & 3));
      *reinterpret_cast<uint2*>(x8 + base + 8 * i) = make_uint2(q[0], q[1]);
    }
  }
  if (lane == 0) {
    if (scales) {
      scales[2 * row] = s;
      scales[2 * row + 1] = inv;
    }
    if (F8) {
      s8[2 * row] = fs;
      s8[2 * row + 1] = finv;
    }
  }
}

// The same row scale for long rows (2048 < k <= 8192, k % 8 == 0): one 128-thread CTA per output row, each thread's
// up to NV vectors of 8 values held in registers between the max and the conversion, so the row is read once.
template <bool BF16, bool F8, bool GATHER, int NV>
__global__ void __launch_bounds__(128) k_row_scale_b(int k, const void* __restrict__ x, const int32_t* __restrict__ rowmap,
                                                     int ku, float* __restrict__ scales, __half* __restrict__ x16,
                                                     uint8_t* __restrict__ x8, float* __restrict__ s8) {
  __shared__ float red[4];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  int64_t src = row;
  if (GATHER) {
    const int a = __ldg(rowmap + row);
    src = a >= 0 ? a / ku : -1;
  }
  const int nv = k / 8;
  float v[NV][8];
  float m = 0.0f;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const int i = threadIdx.x + 128 * u;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[u][j] = 0.0f;
    if (src >= 0 && i < nv) load8<BF16>(x, src * k + 8 * i, v[u]);
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[u][j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const int biased = int((__float_as_uint(m) >> 23) & 255);
  const int e = min(max(biased - 127 - 13, 0), 100);
  const float s = __uint_as_float(uint32_t(127 - e) << 23), inv = __uint_as_float(uint32_t(127 + e) << 23);
  float fs = 0.0f, finv = 0.0f;
  if (F8) {
    fs = __uint_as_float(uint32_t(min(max(261 - biased, 1), 254)) << 23);
    finv = __uint_as_float(uint32_t(min(max(biased - 15, 1), 254)) << 23);
  }
  const int64_t base = row * k;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    const int i = threadIdx.x + 128 * u;
    if (i >= nv) break;
    if (x16) {
      uint32_t h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        h[j] = uint32_t(__half_as_ushort(__float2half_rn(v[u][2 * j] * s))) |
               (uint32_t(__half_as_ushort(__float2half_rn(v[u][2 * j + 1] * s))) << 16);
      *reinterpret_cast<uint4*>(x16 + base + 8 * i) = make_uint4(h[0], h[1], h[2], h[3]);
    }
    if (F8) {
      uint32_t q[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 8; j += 2)
        q[j >> 2] |= uint32_t(__nv_cvt_float2_to_fp8x2(make_float2(v[u][j] * fs, v[u][j + 1] * fs), __NV_SATFINITE,
                                                       __NV_E4M3))
                     << (8 * (j & 3));
      *reinterpret_cast<uint2*>(x8 + base + 8 * i) = make_uint2(q[0], q[1]);
    }
  }
  if (threadIdx.x == 0) {
    if (scales) {
      scales[2 * row] = s;
      scales[2 * row + 1] = inv;
    }
    if (F8) {
      s8[2 * row] = fs;
      s8[2 * row + 1] = finv;
    }
  }
}

template <bool GATHER, int NV>
static cudaError_t launch_row_scale_b(int rows, int k, const void* x, bool bf, const int32_t* rowmap, int ku,
                                      float* scales, __half* h, uint8_t* x8, float* s8, cudaStream_t s) {
  if (x8) {
    if (bf) k_row_scale_b<true, true, GATHER, NV><<<rows, 128, 0, s>>>(k, x, rowmap, ku, scales, h, x8, s8);
    else k_row_scale_b<false, true, GATHER, NV><<<rows, 128, 0, s>>>(k, x, rowmap, ku, scales, h, x8, s8);
  } else {
    if (bf) k_row_scale_b<true, false, GATHER, NV><<<rows, 128, 0, s>>>(k, x, rowmap, ku, scales, h, nullptr, nullptr);
    else k_row_scale_b<false, false, GATHER, NV><<<rows, 128, 0, s>>>(k, x, rowmap, ku, scales, h, nullptr, nullptr);
  }
  return cudaGetLastError();
}

template <bool GATHER>
static cudaError_t launch_row_scale_w(int rows, int k, const void* x, bool bf, const int32_t* rowmap, int ku,
                                      float* scales, __half* h, uint8_t* x8, float* s8, cudaStream_t s) {
  // one pass for long rows (measured: 2880-wide e4m3 rows 129 -> 74 us; 2048-wide rows are faster on the warp form)
  if (k > 2048 && k <= 4096) return launch_row_scale_b<GATHER, 4>(rows, k, x, bf, rowmap, ku, scales, h, x8, s8, s);
  if (k > 4096 && k <= 8192) return launch_row_scale_b<GATHER, 8>(rows, k, x, bf, rowmap, ku, scales, h, x8, s8, s);
  const dim3 grid((rows + 7) / 8);
  if (x8) {
    if (bf) k_row_scale_w<true, true, GATHER><<<grid, 256, 0, s>>>(rows, k, x, rowmap, ku, scales, h, x8, s8);
    else k_row_scale_w<false, true, GATHER><<<grid, 256, 0, s>>>(rows, k, x, rowmap, ku, scales, h, x8, s8);
  } else {
    if (bf) k_row_scale_w<true, false, GATHER><<<grid, 256, 0, s>>>(rows, k, x, rowmap, ku, scales, h, nullptr, nullptr);
    else k_row_scale_w<false, false, GATHER><<<grid, 256, 0, s>>>(rows, k, x, rowmap, ku, scales, h, nullptr, nullptr);
  }
  return cudaGetLastError();
}

static bool al(const void* p, uintptr_t b) { return (reinterpret_cast<uintptr_t>(p) & (b - 1)) == 0; }

int row_scale(int rows, int k, const void* x, int x_dtype, float* scales, uint16_t* x16, uint8_t* x8, float* s8,
              cudaStream_t s) {
  bool bf = x_dtype == LK_BF16;
  __half* h = reinterpret_cast<__half*>(x16);
  if (k % 8 == 0 && al(x, 16) && al(x16, 16) && al(x8, 8))   // vector form (null outputs are aligned)
    return launch_row_scale_w<false>(rows, k, x, bf, nullptr, 1, scales, h, x8, s8, s) == cudaSuccess ? LK_OK
                                                                                                      : LK_ECUDA;
  if (x8) {
    if (bf) k_row_scale<true, true><<<rows, 256, 0, s>>>(k, x, scales, h, x8, s8);
    else k_row_scale<false, true><<<rows, 256, 0, s>>>(k, x, scales, h, x8, s8);
  } else {
    if (bf) k_row_scale<true, false><<<rows, 256, 0, s>>>(k, x, scales, h, nullptr, nullptr);
    else k_row_scale<false, false><<<rows, 256, 0, s>>>(k, x, scales, h, nullptr, nullptr);
  }
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

// the gate/up activations of the MoE in bucket order (k % 8 == 0 and aligned operands, checked by the caller)
int row_scale_gather(int rows, int k, int ku, const int32_t* rowmap, const void* x, int x_dtype, float* scales,
                     uint16_t* x16, uint8_t* x8, float* s8, cudaStream_t s) {
  return launch_row_scale_w<true>(rows, k, x, x_dtype == LK_BF16, rowmap, ku, scales, reinterpret_cast<__half*>(x16),
                                  x8, s8, s) == cudaSuccess
             ? LK_OK
             : LK_ECUDA;
}

// f[t][c] = act(f[t][c]) * u[t][c] over [tokens][n] f32 rows (n % 4 == 0, 16-byte aligned), four values a thread
__global__ void __launch_bounds__(256) k_act_mul(int64_t quads, int act, float4* __restrict__ f,
                                                 const float4* __restrict__ u) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < quads; i += int64_t(gridDim.x) * blockDim.x) {
    float4 g = f[i];
    const float4 v = __ldg(u + i);
    g.x = act_apply(act, g.x, v.x, 0.f, 0.f);
    g.y = act_apply(act, g.y, v.y, 0.f, 0.f);
    g.z = act_apply(act, g.z, v.z, 0.f, 0.f);
    g.w = act_apply(act, g.w, v.w, 0.f, 0.f);
    f[i] = g;
  }
}

int act_mul(int tokens, int n, int act, float* f, const float* u, cudaStream_t s) {
  const int64_t quads = int64_t(tokens) * n / 4;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = std::min<int64_t>((quads + 255) / 256, int64_t(sms) * 8);
  k_act_mul<<<int(blocks), 256, 0, s>>>(quads, act, reinterpret_cast<float4*>(f), reinterpret_cast<const float4*>(u));
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

}  // namespace lk
