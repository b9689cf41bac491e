// Decode expert matvecs for MXFP4S experts: the reference's expert_mv (gen_moe.py:535-727) over the MXFP4S weight
// format (split planes, gen_llm.py:844-895), f32 accumulation of f32 activations as its decode path does.
//   mode 0 (gate/up; expert e holds f gate rows, then f up rows): act[a][j] = act(g + bg, u + bu) (SiLU default),
//          g = Wg[e][j] . x[a / ku], u = Wu[e][j] . x[a / ku]
//   mode 1 (down; expert e holds h rows):                        y[a][j] = Wd[e][j] . x[a] (+ bd)
// with e = ids[a] and W the exact MXFP4 values: e2m1 code * 2^(s - 127), s the row's E8M0 byte of the 32-value block.
//
// Design. One CTA per (16 output rows, assignment); a warp computes 2 of the rows (a gate/up pair counts as one). The
// CTA first stages the assignment's activation row in shared memory as f32, each 128-byte block in 16-byte granules
// swizzled by the block index (granule q of block b at q ^ (b % 8)), so the lanes of a warp, which read the same
// granule of 32 consecutive blocks, spread over eight bank groups. Lane l owns the 32-value blocks l + 32 i of every
// row (i < BPL = ceil(k / 1024)). Per block a lane loads the block's 16 nibble bytes (consecutive lanes read
// consecutive 16-byte segments of the row) and its E8M0 byte, the loads of the warp's rows going out before any of
// their arithmetic. Each nibble becomes an exact f16 -- the e2m1 sign, exponent and mantissa bits placed in the f16
// sign, low exponent and top mantissa bits give value * 2^-14, e = 0 landing on the f16 subnormal 0.5 * 2^-14 --
// then an f32 for an f32 FMA against the activation. The block's sum takes its scale, and the row's warp-reduced
// total is multiplied by 2^14.
// Measured at one token of gpt-oss shapes (a MoE layer, CUDA events): 8 rows per warp 56 us, 4 rows 50 us, 2 rows
// 42-45 us; with the activations in registers instead of shared memory (one CTA per SM) 72 us. ncu counts it
// instruction-bound (issue 64 % of cycles, DRAM 16 %): about 4.4 instructions per weight value.
#include "lk_common.cuh"
#include "lk_internal.h"

namespace lk {
namespace {

constexpr int kMxMvWarps = 8;
constexpr int kMxMvRowsPerWarp = 2;
constexpr int kMxMvRowsPerCta = kMxMvWarps * kMxMvRowsPerWarp;

struct MxMvArgs {
  const uint8_t* w;     // nibble plane [n_experts * rows_per_expert][k / 2]
  const uint8_t* ws;    // E8M0 plane [n_experts * rows_per_expert][k / 32]
  const void* x;        // activations [tokens][k]
  float* y;             // [assignments][n]
  const int32_t* ids;   // expert of each assignment
  int n, k, x_div, n_experts, rows_per_expert, x_dtype;
  ExpertEpi epi;        // gate/up activation, per-expert biases [n_experts][n]
};

// f16 bit patterns of the 2 nibbles held in the low 4 bits of each 16-bit half of r: value * 2^-14, sign included
LK_DEV uint32_t e2m1x2_f16(uint32_t r) { return ((r << 9) & 0x0E000E00u) | ((r << 12) & 0x80008000u); }

LK_DEV float2 h2f2(uint32_t h) { return __half22float2(*reinterpret_cast<const __half2*>(&h)); }

// E8M0 byte -> 2^(e - 127) (e = 0: 2^-127, a subnormal)
LK_DEV float e8m0_scale(uint32_t e) { return e >= 1 ? __uint_as_float(e << 23) : __uint_as_float(0x00400000u); }

// granule g (values 4g .. 4g + 3) of the staged activation block whose 16-byte granules start at xb, key = b % 8
LK_DEV float4 xgran(const float4* xb, int key, int g) { return xb[g ^ key]; }

// sum of the 32 products of one block (16 nibble bytes q against the staged activations), times 2^-14
template <int ORDER>
LK_DEV float block_dot(const uint4 q, const float4* xb, int key) {
  const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {   // bytes 4i .. 4i + 3
    const uint32_t lo4 = wv[i] & 0x0F0F0F0Fu, hi4 = (wv[i] >> 4) & 0x0F0F0F0Fu;
    const float2 l01 = h2f2(e2m1x2_f16(prmt(lo4, 0u, 0x4140u))), l23 = h2f2(e2m1x2_f16(prmt(lo4, 0u, 0x4342u)));
    const float2 h01 = h2f2(e2m1x2_f16(prmt(hi4, 0u, 0x4140u))), h23 = h2f2(e2m1x2_f16(prmt(hi4, 0u, 0x4342u)));
    if (ORDER == LK_ORDER_PAIRS) {   // byte b: element 2b (low nibble), 2b + 1 (high): values 8i .. 8i + 7
      const float4 xa = xgran(xb, key, 2 * i), xc = xgran(xb, key, 2 * i + 1);
      s0 = fmaf(l01.x, xa.x, s0);
      s1 = fmaf(h01.x, xa.y, s1);
      s0 = fmaf(l01.y, xa.z, s0);
      s1 = fmaf(h01.y, xa.w, s1);
      s0 = fmaf(l23.x, xc.x, s0);
      s1 = fmaf(h23.x, xc.y, s1);
      s0 = fmaf(l23.y, xc.z, s0);
      s1 = fmaf(h23.y, xc.w, s1);
    } else {   // split16 (ggml): byte b: element b (low nibble), b + 16 (high): values 4i .. 4i + 3, 16 + 4i ..
      const float4 xa = xgran(xb, key, i), xc = xgran(xb, key, 4 + i);
      s0 = fmaf(l01.x, xa.x, s0);
      s0 = fmaf(l01.y, xa.y, s0);
      s0 = fmaf(l23.x, xa.z, s0);
      s0 = fmaf(l23.y, xa.w, s0);
      s1 = fmaf(h01.x, xc.x, s1);
      s1 = fmaf(h01.y, xc.y, s1);
      s1 = fmaf(h23.x, xc.z, s1);
      s1 = fmaf(h23.y, xc.w, s1);
    }
  }
  return s0 + s1;
}

LK_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// RB output rows per load batch: the rows' blocks are all requested before any is used
template <int MODE, int ORDER, int BPL>
__global__ void __launch_bounds__(kMxMvWarps * 32, 2) k_moe_mv_mx(const MxMvArgs p) {
  constexpr int RB = MODE == 0 ? 2 : (kMxMvRowsPerWarp < 4 ? kMxMvRowsPerWarp : 4);   // output rows per batch
  constexpr int NW = MODE == 0 ? 2 : 1;   // weight rows per output row
  const int a = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.k / 32;
  const int e = min(max(p.ids[a], 0), p.n_experts - 1);
  const int tok = a / p.x_div;

  // the activation row as f32 in shared memory: granule g of block b (values 32b + 4g ..) at 16 (8b + (g ^ b % 8))
  __shared__ float4 xs[4096 / 4];
  for (int gi = threadIdx.x; gi < nb * 8; gi += kMxMvWarps * 32) {
    const int b = gi >> 3, g = gi & 7;
    const int64_t off = int64_t(tok) * p.k + 4 * int64_t(gi);
    float4 f;
    if (p.x_dtype == LK_F32) {
      f = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + off));
    } else {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.x) + off));
      if (p.x_dtype == LK_BF16) {
        f = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                        __uint_as_float(u.y & 0xffff0000u));
      } else {
        const float2 f0 = h2f2(u.x), f1 = h2f2(u.y);
        f = make_float4(f0.x, f0.y, f1.x, f1.y);
      }
    }
    xs[8 * b + (g ^ (b & 7))] = f;
  }
  __syncthreads();

  const int64_t rb = p.k / 2;   // nibble bytes per row
  const int j0 = blockIdx.x * kMxMvRowsPerCta + warp * kMxMvRowsPerWarp;
#pragma unroll 1
  for (int r0 = 0; r0 < kMxMvRowsPerWarp; r0 += RB) {
    uint4 q[RB][NW][BPL];
    uint32_t sc[RB][NW][BPL];
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
      for (int wi = 0; wi < NW; ++wi)
#pragma unroll
        for (int i = 0; i < BPL; ++i) {
          const int j = j0 + r0 + r, b = lane + 32 * i;
          q[r][wi][i] = make_uint4(0u, 0u, 0u, 0u);
          sc[r][wi][i] = 127u;
          if (j < p.n && b < nb) {
            const int64_t row = int64_t(e) * p.rows_per_expert + j + (wi ? p.n : 0);
            q[r][wi][i] = __ldg(reinterpret_cast<const uint4*>(p.w + row * rb) + b);
            sc[r][wi][i] = __ldg(p.ws + row * nb + b);
          }
        }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      float acc[NW];
#pragma unroll
      for (int wi = 0; wi < NW; ++wi) {
        acc[wi] = 0.f;
#pragma unroll
        for (int i = 0; i < BPL; ++i)
          if (lane + 32 * i < nb) {
            const int b = lane + 32 * i;
            acc[wi] = fmaf(block_dot<ORDER>(q[r][wi][i], xs + 8 * b, b & 7), e8m0_scale(sc[r][wi][i]), acc[wi]);
          }
        acc[wi] = warp_sum(acc[wi]) * 16384.0f;
      }
      const int j = j0 + r0 + r;
      if (lane == 0 && j < p.n) {
        float g = acc[0], u = acc[NW - 1];
        if (p.epi.bias) {   // per-expert output biases (gpt-oss ffn_{gate,up,down}_exps.bias)
          g += __ldg(p.epi.bias + int64_t(e) * p.n + j);
          if (MODE == 0) u += __ldg(p.epi.bias2 + int64_t(e) * p.n + j);
        }
        p.y[int64_t(a) * p.n + j] = MODE == 0 ? act_apply(p.epi.act, g, u, p.epi.alpha, p.epi.limit) : g;
      }
    }
  }
}

template <int MODE, int ORDER>
int launch_mx_mv(const MxMvArgs& a, int assignments, cudaStream_t s) {
  const dim3 grid((a.n + kMxMvRowsPerCta - 1) / kMxMvRowsPerCta, assignments);
  const int bpl = (a.k / 32 + 31) / 32;
  switch (bpl) {
    case 1: k_moe_mv_mx<MODE, ORDER, 1><<<grid, kMxMvWarps * 32, 0, s>>>(a); break;
    case 2: k_moe_mv_mx<MODE, ORDER, 2><<<grid, kMxMvWarps * 32, 0, s>>>(a); break;
    case 3: k_moe_mv_mx<MODE, ORDER, 3><<<grid, kMxMvWarps * 32, 0, s>>>(a); break;
    case 4: k_moe_mv_mx<MODE, ORDER, 4><<<grid, kMxMvWarps * 32, 0, s>>>(a); break;
    default: return LK_EUNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

}  // namespace

int moe_expert_mv_mx(int mode, int order, int n, int k, int assignments, int ku, int n_experts, const int32_t* ids,
                     const void* x, int x_dtype, const uint8_t* w, const uint8_t* ws, float* y, cudaStream_t s,
                     const ExpertEpi* epi) {
  MxMvArgs a{};
  if (epi) a.epi = *epi;
  a.w = w;
  a.ws = ws;
  a.x = x;
  a.y = y;
  a.ids = ids;
  a.n = n;
  a.k = k;
  a.x_div = mode == 0 ? ku : 1;
  a.n_experts = n_experts;
  a.rows_per_expert = mode == 0 ? 2 * n : n;
  a.x_dtype = x_dtype;
  if (mode == 0)
    return order == LK_ORDER_PAIRS ? launch_mx_mv<0, LK_ORDER_PAIRS>(a, assignments, s)
                                   : launch_mx_mv<0, LK_ORDER_SPLIT16>(a, assignments, s);
  return order == LK_ORDER_PAIRS ? launch_mx_mv<1, LK_ORDER_PAIRS>(a, assignments, s)
                                 : launch_mx_mv<1, LK_ORDER_SPLIT16>(a, assignments, s);
}

}  // namespace lk
