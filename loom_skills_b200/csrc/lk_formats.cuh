// Per-format decoding of one 32-value group of GGUF block weights, shared by the standalone dequantisation and the
// generic-format decode matvec. Formats and value rules (the reference's format table formats.py:5-17 and
// gen_gemm.py:16-39; values as gguf-py 0.19.0's dequantize_blocks computes them, which the reference's numpy path
// calls, make_kernel_tests.py:45-47; the GEMM staging as gen_gemm.py:281-532):
//
//   Q4_0   18 B / 32   d, 16 nibble bytes                      d (q - 8)
//   IQ4_NL 18 B / 32   d, 16 nibble bytes                      d kvalue[q]
//   Q5_0   22 B / 32   d, u32 qh, 16 nibble bytes              d (q - 16), q = nibble | bit i of qh << 4
//   Q8_0   34 B / 32   d, 32 int8 codes                        d q
//   MXFP4  17 B / 32   E8M0 e, 16 nibble bytes (ggml)          2 e2m1[q] 2^(e - 128)
//   Q4_K  144 B / 256  d, dmin, 12 B scales/mins, 128 B nibbles        d sc q - dmin m   (groups of 32)
//   Q5_K  176 B / 256  as Q4_K plus qh[32] (bit g: the 5th bit of group g)   d sc q - dmin m
//   Q6_K  210 B / 256  ql[128], qh[64], int8 sc[16], d         (d sc) (q - 32)          (sub-blocks of 16)
//   IQ4_XS 136 B / 256 d, u16 scales_h, 4 B scales_l, qs[128]  d (ls - 32) kvalue[q]    (groups of 32)
//   Q3_K  110 B / 256  hmask[32], qs[64], 12 B scales, d       (d (ls - 32)) (q2 - 4 !hbit) (sub-blocks of 16)
//   IQ3_S 110 B / 256  d, qs[64], qh[8], signs[32], scales[4]  (d (1 + 2 s)) (+-grid[qs | qh bit << 8][i])  (groups of 32)
//
// Every value is an exact f32 product (the integer factors are at most 24 significant bits together), except the
// K-quants' d sc q - dmin m, which rounds once as gguf's does. Byte loads only: blocks of these sizes start at any
// even (MXFP4: any) byte offset.
#pragma once
#include "lk_common.cuh"
// kIq3sGrid[512]: the IQ3_S codebook, one u32 of four magnitudes per entry (written by build.py at build time)
#include "lk_iq3s_grid.inc"

namespace lk {

__host__ __device__ constexpr int fmt_qk(int fmt) {
  return (fmt == LK_Q4_K || fmt == LK_Q5_K || fmt == LK_Q6_K || fmt == LK_IQ4_XS || fmt == LK_Q3_K || fmt == LK_IQ3_S)
             ? 256
             : 32;
}
__host__ __device__ constexpr int fmt_block_bytes(int fmt) {
  return fmt == LK_Q4_0 || fmt == LK_IQ4_NL ? 18
         : fmt == LK_Q5_0                  ? 22
         : fmt == LK_Q8_0                  ? 34
         : fmt == LK_MXFP4                 ? 17
         : fmt == LK_Q4_K                  ? 144
         : fmt == LK_Q5_K                  ? 176
         : fmt == LK_Q6_K                  ? 210
         : fmt == LK_IQ4_XS                ? 136
         : fmt == LK_Q3_K                  ? 110
         : fmt == LK_IQ3_S                 ? 110
                                           : 0;
}

LK_DEV float f16_at(const uint8_t* p) { return h2f(uint16_t(p[0] | (p[1] << 8))); }
// the IQ4 codebook value of nibble q: a byte permute of the biased table words (no indexed array, which would live
// in local memory)
LK_DEV int iq4_value(int q) {
  const uint32_t lo = prmt(kIq4Biased0, kIq4Biased1, uint32_t(q & 7));
  const uint32_t hi = prmt(kIq4Biased2, kIq4Biased3, uint32_t(q & 7));
  return int(((q & 8) ? hi : lo) & 0xffu) - 128;
}
// twice the E2M1 magnitude of code bits q & 7 (0 1 2 3 4 6 8 12), by a byte permute
LK_DEV int e2m1_x2(int q) { return int(prmt(0x03020100u, 0x0C080604u, uint32_t(q & 7)) & 0xffu); }

// The 32 values of group j (0 for 32-value formats, 0..7 of a super-block) as exact integer codes and the f32
// scale / offset they combine with: value_i = a_i * q_i - c_i. Per format: a and c are per group or per 16-value
// half (lo: values 0..15, hi: 16..31).
struct GroupCodes {
  int q[32];
  float a_lo, a_hi, c_lo, c_hi;
};

template <int FMT>
LK_DEV void group_codes(const uint8_t* b, int j, GroupCodes& g) {
  if (FMT == LK_Q4_0 || FMT == LK_IQ4_NL || FMT == LK_Q5_0) {
    const float d = f16_at(b);
    const uint8_t* qs = b + (FMT == LK_Q5_0 ? 6 : 2);
    const uint32_t qh = FMT == LK_Q5_0 ? uint32_t(b[2]) | (uint32_t(b[3]) << 8) | (uint32_t(b[4]) << 16) |
                                             (uint32_t(b[5]) << 24)
                                       : 0u;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int nib = i < 16 ? (qs[i] & 15) : (qs[i - 16] >> 4);
      g.q[i] = FMT == LK_Q4_0   ? nib - 8
               : FMT == LK_IQ4_NL ? iq4_value(nib)
                                  : (nib | int(((qh >> i) & 1u) << 4)) - 16;
    }
    g.a_lo = g.a_hi = d;
    g.c_lo = g.c_hi = 0.f;
  } else if (FMT == LK_Q8_0) {
    const float d = f16_at(b);
#pragma unroll
    for (int i = 0; i < 32; ++i) g.q[i] = int(int8_t(b[2 + i]));
    g.a_lo = g.a_hi = d;
    g.c_lo = g.c_hi = 0.f;
  } else if (FMT == LK_MXFP4) {
    const int e = b[0];
    // ggml_e8m0_to_fp32_half: 2^(e - 128), the e2m1 table doubled to integers (0 1 2 3 4 6 8 12)
    const float half_scale = __uint_as_float(e < 2 ? (0x00200000u << e) : (uint32_t(e - 1) << 23));
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int nib = i < 16 ? (b[1 + i] & 15) : (b[1 + i - 16] >> 4);
      g.q[i] = (nib & 8) ? -e2m1_x2(nib) : e2m1_x2(nib);
    }
    g.a_lo = g.a_hi = half_scale;
    g.c_lo = g.c_hi = 0.f;
  } else if (FMT == LK_Q4_K || FMT == LK_Q5_K) {
    const float d = f16_at(b), dmin = f16_at(b + 2);
    int sc, m;
    q4k_scale_min(b + 4, j, sc, m);
    const uint8_t* qs = b + (FMT == LK_Q5_K ? 48 : 16) + 32 * (j >> 1);
    const int sh = 4 * (j & 1);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      int q = (qs[i] >> sh) & 15;
      if (FMT == LK_Q5_K) q |= ((b[16 + i] >> j) & 1) << 4;
      g.q[i] = q;
    }
    g.a_lo = g.a_hi = d * float(sc);
    g.c_lo = g.c_hi = dmin * float(m);
  } else if (FMT == LK_Q6_K) {
    const float d = f16_at(b + 208);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int v = 32 * j + i, h = v >> 7, r = v & 127;
      const int lo = (b[64 * h + (r & 63)] >> (4 * (r >> 6))) & 15;
      const int hi = (b[128 + 32 * h + (r & 31)] >> (2 * (r >> 5))) & 3;
      g.q[i] = (lo | (hi << 4)) - 32;
    }
    g.a_lo = d * float(int8_t(b[192 + 2 * j]));
    g.a_hi = d * float(int8_t(b[192 + 2 * j + 1]));
    g.c_lo = g.c_hi = 0.f;
  } else if (FMT == LK_IQ4_XS) {
    const float d = f16_at(b);
    const int sh = b[2] | (b[3] << 8);
    const int ls = ((b[4 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((sh >> (2 * j)) & 3) << 4);
    const uint8_t* qs = b + 8 + 16 * j;
#pragma unroll
    for (int i = 0; i < 32; ++i) g.q[i] = iq4_value(i < 16 ? (qs[i] & 15) : (qs[i - 16] >> 4));
    g.a_lo = g.a_hi = d * float(ls - 32);
    g.c_lo = g.c_hi = 0.f;
  } else if (FMT == LK_Q3_K) {
    const float d = f16_at(b + 108);
    const uint8_t* sc = b + 96;
    float a[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {   // the group's two 16-value sub-blocks
      const int s = 2 * j + hh;
      const int ls = (sc[s & 7] >> (4 * (s >> 3))) & 15, hs = (sc[8 + (s & 3)] >> (2 * (s >> 2))) & 3;
      a[hh] = d * float((ls | (hs << 4)) - 32);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int v = 32 * j + i;
      const int q2 = (b[32 + 32 * (v >> 7) + (v & 31)] >> (2 * ((v & 127) >> 5))) & 3;
      const int hb = (b[v & 31] >> (v >> 5)) & 1;
      g.q[i] = q2 - (hb ? 0 : 4);
    }
    g.a_lo = a[0];
    g.a_hi = a[1];
    g.c_lo = g.c_hi = 0.f;
  } else if (FMT == LK_IQ3_S) {
    // group j: 8 codebook entries of 4 magnitudes, entry c = qs[8j + c] | (bit c of qh[j]) << 8; the sign of value i
    // is bit i % 8 of signs[4j + i / 8]; the scale d (1 + 2 s), s the j-th nibble of scales[4]
    const float d = f16_at(b);
    const uint8_t* qs = b + 2 + 8 * j;
    const int qh = b[66 + j];
    const uint8_t* sg = b + 74 + 4 * j;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint32_t e = __ldg(&kIq3sGrid[qs[c] | (((qh >> c) & 1) << 8)]);
      const int sb = sg[c >> 1] >> (4 * (c & 1));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = int((e >> (8 * i)) & 0xffu);
        g.q[4 * c + i] = ((sb >> i) & 1) ? -m : m;
      }
    }
    g.a_lo = g.a_hi = d * float(1 + 2 * ((b[106 + (j >> 1)] >> (4 * (j & 1))) & 15));
    g.c_lo = g.c_hi = 0.f;
  }
}

// exact f32 values of the group (gguf's dequantize_blocks)
template <int FMT>
LK_DEV void group_values(const uint8_t* b, int j, float (&v)[32]) {
  GroupCodes g;
  group_codes<FMT>(b, j, g);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float a = i < 16 ? g.a_lo : g.a_hi, c = i < 16 ? g.c_lo : g.c_hi;
    v[i] = (FMT == LK_Q4_K || FMT == LK_Q5_K) ? __fsub_rn(__fmul_rn(a, float(g.q[i])), c)
                                                : __fmul_rn(a, float(g.q[i]));
  }
}

// the prefill GEMM's f16 staging: Q4_K / Q5_K fma_f16(q, f16(d sc), f16(-dmin m)) (gen_gemm.py:445-532), Q6_K
// fma_f16(q + 32, f16(d sc), f16(-32 d sc)) (gen_gemm.py:369-444), every other format one rounding of the exact value
template <int FMT>
LK_DEV void group_f16(const uint8_t* b, int j, __half (&h)[32]) {
  GroupCodes g;
  group_codes<FMT>(b, j, g);
  if (FMT == LK_Q4_K || FMT == LK_Q5_K || FMT == LK_Q6_K) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float a = i < 16 ? g.a_lo : g.a_hi;
      const float c = FMT == LK_Q6_K ? -32.0f * a : -(i < 16 ? g.c_lo : g.c_hi);
      const int q = FMT == LK_Q6_K ? g.q[i] + 32 : g.q[i];
      h[i] = __hfma(__int2half_rn(q), __float2half_rn(a), __float2half_rn(c));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) h[i] = __float2half_rn(__fmul_rn(i < 16 ? g.a_lo : g.a_hi, float(g.q[i])));
  }
}

// Gate and up weights in two formats (LK_FMT_PAIR(gate, up): the reference's "GATE+UP" kernels, gen_moe.py:537-552,
// 1129-1141, and gen_gemm.py:535-545 fmt2). Kernels instantiated with kFmtPair read each weight's format at run time;
// the switch is uniform across a warp (a warp's rows belong to one weight).
constexpr int kFmtPair = -1;

// the 32 values of group gi of a packed row (row: its first byte) in format `fmt`, chosen at run time; zeros for a
// format without a decoder here
LK_DEV void row_group_values(int fmt, const uint8_t* row, int gi, float (&v)[32]) {
  switch (fmt) {
#define LK_ROW_GROUP(F)                                                                              \
  case F:                                                                                            \
    group_values<F>(row + (gi / (fmt_qk(F) / 32)) * fmt_block_bytes(F), gi % (fmt_qk(F) / 32), v); \
    return;
    LK_ROW_GROUP(LK_Q4_0)
    LK_ROW_GROUP(LK_IQ4_NL)
    LK_ROW_GROUP(LK_Q4_K)
    LK_ROW_GROUP(LK_Q5_0)
    LK_ROW_GROUP(LK_Q8_0)
    LK_ROW_GROUP(LK_Q5_K)
    LK_ROW_GROUP(LK_Q6_K)
    LK_ROW_GROUP(LK_IQ4_XS)
    LK_ROW_GROUP(LK_Q3_K)
    LK_ROW_GROUP(LK_IQ3_S)
    LK_ROW_GROUP(LK_MXFP4)
#undef LK_ROW_GROUP
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = 0.f;
}

}  // namespace lk
