// Device pieces of the int8-activation decode matvecs (lk_mvq8.cu: dense; lk_moeq8.cu: the MoE expert matvecs):
//   quant_half / quant_groups / quant_flat
//                  g_quant_q8 (gen_llm.py:683-750) of activation rows into shared memory
//   XUnit / load_xunit / unit_dot
//                  one lane's (chunk, page) unit of 64 values: its activation codes and group meta held in registers,
//                  and its dot with one packed weight row's unit (@g_<fmt>_icodes, gen_llm.py:521-680)
// A unit is one 32-byte nibble page of a Q4_K super-block (with the super-block's 16-byte header) or two consecutive
// 18-byte Q4_0 blocks, 36 bytes at a 4-byte aligned offset: both formats spend 144 bytes per 256 values.
#pragma once
#include "lk_common.cuh"

namespace lk {
namespace q8 {

LK_DEV int dp4a_us(uint32_t a, uint32_t b, int c) {   // unsigned bytes of a . signed bytes of b + c
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// exact int -> float for |v| < 2^22 without a conversion instruction
LK_DEV float i2f_small(int v) { return __int_as_float(0x4B400000 + v) - 12582912.0f; }

// the Q4_K (scale, min) pairs of groups (2pg, 2pg + 1) as "2^23 + value" floats: f[0..1] scales, f[2..3] minima.
// pg is constant per thread: byte half h = pg & 1 of each scale word, the 4-bit-plus-2-bit form for pg >= 2.
LK_DEV void q4k_pair_magic(uint4 hd, uint32_t hsel, uint32_t big_mask, float (&f)[4]) {
  const uint32_t a = prmt(hd.y, 0u, hsel), b = prmt(hd.z, 0u, hsel), c = prmt(hd.w, 0u, hsel);
  const uint32_t sc_lo = a & 0x3F3Fu, m_lo = b & 0x3F3Fu;
  const uint32_t sc_hi = (c & 0x0F0Fu) | ((a >> 2) & 0x3030u);
  const uint32_t m_hi = ((c >> 4) & 0x0F0Fu) | ((b >> 2) & 0x3030u);
  const uint32_t v = ((sc_hi & big_mask) | (sc_lo & ~big_mask)) | (((m_hi & big_mask) | (m_lo & ~big_mask)) << 16);
  f[0] = __uint_as_float(prmt(v, 0x4B000000u, 0x7650u));
  f[1] = __uint_as_float(prmt(v, 0x4B000000u, 0x7651u));
  f[2] = __uint_as_float(prmt(v, 0x4B000000u, 0x7652u));
  f[3] = __uint_as_float(prmt(v, 0x4B000000u, 0x7653u));
}

// where a row kernel's activation codes come from: lk_quant_q8's buffer, or x of this type quantised in the kernel
// (distinct from the LK_* dtype ids, among which LK_F32 is 0)
enum { kXinCodes = 0, kXinF32 = 1, kXinBF16 = 2 };

// bytes of the shared copy of the quantised activation row (codes, then the group meta), 128-byte rounded
__host__ __device__ inline int xq_smem_bytes(int k) { return (k + k / 4 + 127) / 128 * 128; }

// g_quant_q8 of one 16-value half-group (the other half of its 32-value group in lane t ^ 1, which must run the same
// call): d = amax / 127, q = round(x / d) (halves away from zero; 0 for an all-zero group), the 16 codes stored at
// codes[hg * 16 ..], and for even hg the group meta (f16-rounded d, sum of q) at meta[hg / 2]. The codes and meta are
// k_quant_q8's bit for bit:
//  - y = x * (1/d) (both correctly rounded) is within 2 units in the last place of the quotient x / d, |y| <= 127;
//  - adding 1.5 * 2^23 rounds y to the nearest integer m (ties to even) in the low mantissa bits, whose low byte is
//    then the two's-complement code; f = y - m is exact (Sterbenz), |f| <= 1/2;
//  - where |f| lies within 2^-14 of 1/2 (y near a rounding boundary, where y and x / d could round apart or the tie
//    rules differ) or is NaN, the half-group is recomputed with the exact quotient and roundf.
// Codes are packed by byte permutes; their sum is a dp4a. `store` false: the shuffles only (a lane past the end).
LK_DEV void quant_half(const float (&v)[16], int hg, bool store, int8_t* codes, float* meta) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
  const float d = amax / 127.0f;
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  if (amax > 0.0f) {   // ordered compare: a NaN maximum gives codes 0, like the reference
    const float r = __frcp_rn(d);
    constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23
    bool exact = false;
    uint32_t tb[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float y = __fmul_rn(v[i], r);
      const float tm = __fadd_rn(y, kMagic);
      const float f = __fsub_rn(y, __fsub_rn(tm, kMagic));
      exact |= !(fabsf(f) < 0.49993896484375f);   // within 2^-14 of a half, or NaN
      tb[i] = __float_as_uint(tm);
    }
    if (exact) {
#pragma unroll
      for (int i = 0; i < 16; ++i) tb[i] = uint32_t(int(roundf(v[i] / d)));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = __byte_perm(__byte_perm(tb[4 * i], tb[4 * i + 1], 0x0040), __byte_perm(tb[4 * i + 2], tb[4 * i + 3], 0x0040),
                         0x5410);
  }
  int sum = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) sum = __dp4a(int(w[i]), 0x01010101, sum);
  sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
  if (!store) return;
  reinterpret_cast<uint4*>(codes)[hg] = make_uint4(w[0], w[1], w[2], w[3]);
  if ((hg & 1) == 0) reinterpret_cast<float2*>(meta)[hg >> 1] = make_float2(__half2float(__float2half_rn(d)), float(sum));
}

// the 16 values of half-group hg of x (f32 or bf16), read-only loads
template <int XIN>
LK_DEV void load_half(const void* x, int hg, uint32_t (&raw)[XIN == kXinBF16 ? 8 : 16]) {
  constexpr int kWords = XIN == kXinBF16 ? 8 : 16;
  const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(x) + int64_t(hg) * 4 * kWords);
#pragma unroll
  for (int i = 0; i < kWords / 4; ++i) {
    const uint4 u = __ldg(p + i);
    raw[4 * i] = u.x;
    raw[4 * i + 1] = u.y;
    raw[4 * i + 2] = u.z;
    raw[4 * i + 3] = u.w;
  }
}
template <int XIN>
LK_DEV void unpack_half(const uint32_t (&raw)[XIN == kXinBF16 ? 8 : 16], float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i)
    v[i] = XIN == kXinBF16 ? __uint_as_float((i & 1) ? (raw[i >> 1] & 0xffff0000u) : (raw[i >> 1] << 16))
                           : __uint_as_float(raw[i]);
}

// g_quant_q8 of a row of k = 4096 NIT values by 256 threads: thread t takes the half-groups t + 256 j, j < NIT, with
// all of its loads issued before any arithmetic (x comes from an earlier kernel: read-only loads). Codes [k] and meta
// [k/32][2] as k_quant_q8 writes them.
template <int XIN, int NIT>
LK_DEV void quant_groups(const void* x, int t, int8_t* codes, float* meta) {
  static_assert(XIN == kXinF32 || XIN == kXinBF16, "an activation type to quantise");
  uint32_t raw[NIT][XIN == kXinBF16 ? 8 : 16];
#pragma unroll
  for (int j = 0; j < NIT; ++j) load_half<XIN>(x, t + 256 * j, raw[j]);
#pragma unroll
  for (int j = 0; j < NIT; ++j) {
    float v[16];
    unpack_half<XIN>(raw[j], v);
    quant_half(v, t + 256 * j, true, codes, meta);
  }
}

// g_quant_q8 of `rows` consecutive rows of k values (k % 32 == 0) as one flat vector, by 256 threads: the same codes
// and meta layout as k_quant_q8 on [rows][k] (codes [rows][k], then meta [rows][k/32][2]). Rounds of 256 half-groups
// go in batches (4 for bf16, 2 for f32) whose loads are all issued before their arithmetic; every thread runs the same
// rounds (lanes past the end take part in the pair shuffles only).
template <int XIN>
LK_DEV void quant_flat(const void* x, int nvals, int t, int8_t* codes, float* meta) {
  static_assert(XIN == kXinF32 || XIN == kXinBF16, "an activation type to quantise");
  constexpr int kW = XIN == kXinBF16 ? 8 : 16;
  constexpr int kB = XIN == kXinBF16 ? 4 : 2;
  const int nhg = nvals / 16;
  for (int base = 0; base < nhg; base += kB * 256) {
    uint32_t raw[kB][kW];
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const int hg = base + b * 256 + t;
      if (hg < nhg) {
        load_half<XIN>(x, hg, raw[b]);
      } else {
#pragma unroll
        for (int i = 0; i < kW; ++i) raw[b][i] = 0u;
      }
    }
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      if (base + b * 256 >= nhg) break;   // the same for every thread
      const int hg = base + b * 256 + t;
      float v[16];
      unpack_half<XIN>(raw[b], v);
      quant_half(v, hg, hg < nhg, codes, meta);
    }
  }
}

// One lane's activation unit: chunk c, page pg = 64 codes (xa: the first 32, xb: the next 32) and the two groups'
// meta folded into the factors unit_dot needs.
struct XUnit {
  uint32_t xa[8], xb[8];
  float dx0, dx1, b0, b1;   // Q4_0: b0, b1 unused
  int s0x8, s1x8;           // Q4_0: 8 x the groups' code sums (codes are q - 8)
};

// codes / meta: one activation row's codes [k] and group meta [k/32][2]. SMEM: in shared memory (quantised by this
// CTA); else read-only global loads of lk_quant_q8's buffer
template <int FMT, bool SMEM>
LK_DEV void load_xunit(const uint8_t* codes, const float* meta, int c, int pg, XUnit& u) {
  auto ld16 = [](const void* q) {
    return SMEM ? *reinterpret_cast<const uint4*>(q) : __ldg(reinterpret_cast<const uint4*>(q));
  };
  const uint8_t* xw = codes + c * 256 + 64 * pg;
  const uint4 v0 = ld16(xw), v1 = ld16(xw + 16), v2 = ld16(xw + 32), v3 = ld16(xw + 48);
  u.xa[0] = v0.x; u.xa[1] = v0.y; u.xa[2] = v0.z; u.xa[3] = v0.w;
  u.xa[4] = v1.x; u.xa[5] = v1.y; u.xa[6] = v1.z; u.xa[7] = v1.w;
  u.xb[0] = v2.x; u.xb[1] = v2.y; u.xb[2] = v2.z; u.xb[3] = v2.w;
  u.xb[4] = v3.x; u.xb[5] = v3.y; u.xb[6] = v3.z; u.xb[7] = v3.w;
  const uint4 mu = ld16(meta + c * 16 + 4 * pg);
  const float4 mt = make_float4(__uint_as_float(mu.x), __uint_as_float(mu.y), __uint_as_float(mu.z),
                                __uint_as_float(mu.w));
  u.dx0 = mt.x;
  if (FMT == LK_Q4_0) {
    u.dx1 = mt.z;
    u.b0 = u.b1 = 0.f;
    u.s0x8 = 8 * int(mt.y);
    u.s1x8 = 8 * int(mt.w);
  } else {
    u.dx1 = mt.z * 0.0625f;   // high nibbles: the dot is 16 x
    u.b0 = mt.x * mt.y;
    u.b1 = mt.z * mt.w;
    u.s0x8 = u.s1x8 = 0;
  }
}

// Page selectors of lane page pg for q4k_pair_magic
LK_DEV uint32_t q4k_hsel(int pg) { return (pg & 1) ? 0x4432u : 0x4410u; }
LK_DEV uint32_t q4k_big(int pg) { return (pg >> 1) ? 0xFFFFFFFFu : 0u; }

// sum over the unit's 64 values of weight x activation, for the packed chunk `sb` (144 bytes in shared memory).
// Per 64 values: 3 (Q4_K) or 9 (Q4_0) shared loads, 16 nibble masks and 16 dp4a; the high nibbles are used in place
// (16 x code), their group's integer dot is 16x and the 1/16 is in that group's scale.
template <int FMT>
LK_DEV float unit_dot(const uint8_t* sb, const XUnit& u, int pg, uint32_t hsel, uint32_t big) {
  if (FMT == LK_Q4_0) {
    // blocks 2 pg, 2 pg + 1 of the chunk: [d_a | 16 nibble bytes | d_b | 16 nibble bytes] from byte 36 pg
    const uint32_t* bw = reinterpret_cast<const uint32_t*>(sb + 36 * pg);
    uint32_t v[9];
#pragma unroll
    for (int j = 0; j < 9; ++j) v[j] = bw[j];
    const float da = h2f(uint16_t(v[0] & 0xffffu)), db = h2f(uint16_t(v[4] >> 16));
    int la = 0, ha = 0, lb = 0, hb = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {   // byte i of a block: element i (low nibble), element 16 + i (high)
      const uint32_t qa = __funnelshift_r(v[j], v[j + 1], 16), qb = v[5 + j];
      la = dp4a_us(qa & 0x0F0F0F0Fu, u.xa[j], la);
      ha = dp4a_us(qa & 0xF0F0F0F0u, u.xa[4 + j], ha);
      lb = dp4a_us(qb & 0x0F0F0F0Fu, u.xb[j], lb);
      hb = dp4a_us(qb & 0xF0F0F0F0u, u.xb[4 + j], hb);
    }
    // sum((q - 8) x) = dot - 8 sum(x); the high nibbles' dot is 16 x, exactly
    return da * u.dx0 * i2f_small(la + (ha >> 4) - u.s0x8) + db * u.dx1 * i2f_small(lb + (hb >> 4) - u.s1x8);
  } else {
    const uint4 hd = *reinterpret_cast<const uint4*>(sb);
    const uint4 q0 = *reinterpret_cast<const uint4*>(sb + 16 + 32 * pg);
    const uint4 q1 = *reinterpret_cast<const uint4*>(sb + 32 + 32 * pg);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    float f[4];
    q4k_pair_magic(hd, hsel, big, f);
    const float d = h2f(uint16_t(hd.x & 0xffffu)), dmin = h2f(uint16_t(hd.x >> 16));
    const float nd = -8388608.0f * d, ndm = -8388608.0f * dmin;
    int i0 = 0, i1 = 0, i2 = 0, i3 = 0;
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      i0 = dp4a_us(w[j] & 0x0F0F0F0Fu, u.xa[j], i0);
      i1 = dp4a_us(w[j] & 0xF0F0F0F0u, u.xb[j], i1);
      i2 = dp4a_us(w[j + 1] & 0x0F0F0F0Fu, u.xa[j + 1], i2);
      i3 = dp4a_us(w[j + 1] & 0xF0F0F0F0u, u.xb[j + 1], i3);
    }
    // d*sc = fma(d, 2^23 + sc, -d*2^23), exact; the same for the minima
    return fmaf(d, f[0], nd) * (u.dx0 * i2f_small(i0 + i2)) + fmaf(d, f[1], nd) * (u.dx1 * i2f_small(i1 + i3)) -
           fmaf(dmin, f[2], ndm) * u.b0 - fmaf(dmin, f[3], ndm) * u.b1;
  }
}

}  // namespace q8
}  // namespace lk
