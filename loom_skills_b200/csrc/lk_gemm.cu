// Prefill GEMM over GGUF block weights on the 5th-generation tensor cores (tcgen05 + TMEM), dense and MoE-grouped.
//
// Replaces g_gemm_{fmt}_{store,acc,swiglu}[_m128|_m256] (gen_gemm.py:535-704, 706, 1224; dispatch gen_llm.py:4568-4622)
// and the grouped expert GEMMs g_moe_ggu_{fmt}[_fused]_k{H} / g_moe_gdn_{fmt}_k{F} (gen_moe.py:1126-1228,
// moe_q4_0.py:126-146) with their bias / activation epilogue (gen_moe.py:958-1007):
//   Y = (X16 . W16^T) * inv[row]  (+ y | act(G + bg, U + bu) | + bd).
//
// One persistent kernel (k_gemm_p, below) walks output tiles with warp-specialised roles: a TMA producer (A tiles of
// X16, 128-byte swizzle -- MoE gate/up: TMA gather4 of the routed token rows -- and the weights' packed bytes, one
// 2-D box of BN rows x 144 bytes per 256 k), an MMA issuer (tcgen05.mma kind::f16 from one lane, accumulators in
// TMEM), dequantisation warps that write the reference's one-rounding f16 staging (f16(d*(q-8)), f16(d*kvalue),
// fma_f16(q, f16(d*sc), f16(-dmin*m))) into the UMMA K-major 128-byte-swizzle B layout, and epilogue warps.
#include <mutex>

#include <atomic>

#include "lk_common.cuh"
#include "lk_formats.cuh"
#include "lk_internal.h"

namespace lk {

constexpr int kBM = 128, kBK = 64;
constexpr int kDqWarps = 8;

enum { kDense = 0, kGather = 1, kSorted = 2 };

constexpr int kStgStride = 36;   // floats per row of the epilogue's 32 x 32 staging tile (16-byte aligned rows)

struct GemmArgs {
  const float* scales;  // [rows or xrows][2]
  // outputs: tile (row, col) goes to dst[d][row * ld + col_off + col] for every d < ndst (one destination: y with
  // ld = n; the all-gather form: every rank's y, ld = the full width, col_off = this rank's first column)
  float* dst[kMaxPeers];
  int ndst;
  int64_t ld;
  int col_off;
  int rows, k, n;
  // weights: wmap / w2map cover [rows][row_bytes / 4] u32 of the (expert-stacked) packed weights; an expert's
  // first row is e * rows_per_expert (w2: e * rows_per_expert2 + w2_row_offset)
  int rows_per_expert, rows_per_expert2, w2_row_offset;
  // MoE
  const int32_t* tile_info;   // [max_tiles][2]
  const int32_t* rowmap;      // [max_tiles*64]
  int max_tiles;
  int xrows, ku, n_experts;
  int n_fast;                 // persistent dense kernel: walk the n tiles of an m tile first (large A, small W)
  // persistent dense store / acc: K split into ksplit ranges of kps packed stages (256 values) each; every range is
  // a work item of its own. The ranges of an output tile meet in y in a fixed order: range 0 stores (acc: adds to y),
  // range s adds its partial after range s - 1 has (turnstile: kflags[tile] = kepoch * 64 + ranges done).
  int ksplit, kps;
  unsigned long long* kflags;
  unsigned long long kepoch;
  ExpertEpi epi;              // gate/up activation and per-expert biases (bias index: expert * n + column)
  // window producer (formats whose packed rows are not 16-byte aligned 144-byte chunks): the weights' base
  // pointers and packed row stride
  const uint8_t* wp;
  const uint8_t* w2p;
  int64_t rb;
  // gate and up in two formats (kernels instantiated with kFmtPair): each weight's format, packed bytes of a
  // 256-value chunk, and the up weight's row stride
  int fmt, fmt2, cb, cb2;
  int64_t rb2;
  // store modes: y = act(y, acc * scale + bias) -- the second pass of a gate/up pair in two formats, whose first pass
  // stored the gate's products (plus its bias) in y (epi.act / alpha / limit choose the activation)
  int act_mul;
};

// packed bytes of one 256-value chunk of a row, and the bytes a window of it takes in shared memory: the chunk
// copied from its 16-byte aligned start, so up to 15 bytes before and after it
__host__ __device__ constexpr int chunk_bytes(int fmt) { return 256 / fmt_qk(fmt) * fmt_block_bytes(fmt); }
__host__ __device__ constexpr int window_bytes(int fmt) { return (chunk_bytes(fmt) + 15 + 15) / 16 * 16; }
// shared-memory bytes of one row's chunk: the TMA box form's 144, a window of the format's chunk, or for a format pair
// the largest window of any format (Q8_0's)
__host__ __device__ constexpr int row_slot_bytes(int fmt, bool win) {
  return !win ? kChunkBytes : fmt == kFmtPair ? window_bytes(LK_Q8_0) : window_bytes(fmt);
}

LK_DEV uint32_t hsub2u(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
LK_DEV uint32_t hmul2u(uint32_t a, __half2 b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), b);
  return *reinterpret_cast<uint32_t*>(&r);
}
LK_DEV uint32_t hfma2u(uint32_t a, __half2 b, __half2 c) {
  __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), b, c);
  return *reinterpret_cast<uint32_t*>(&r);
}

// N little-endian words from a 2-byte aligned shared-memory address: N + 1 aligned loads and funnel shifts (the
// load past the end stays inside the CTA's shared memory: the row windows are followed by the staging buffers)
template <int N>
LK_DEV void ld_words_2a(const uint8_t* p, uint32_t (&w)[N]) {
  // explicit shared-memory loads: the aligned address is formed as an integer, and a generic load through it would
  // not be known to be shared
  const uint32_t a = smem_u32(p), base = a & ~3u, sh = (a & 3u) * 8u;
  uint32_t v[N + 1];
#pragma unroll
  for (int i = 0; i <= N; ++i) asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v[i]) : "r"(base + 4u * i));
#pragma unroll
  for (int i = 0; i < N; ++i) w[i] = __funnelshift_r(v[i], v[i + 1], sh);
}

// Word-wise f16 staging of one 32-value group for the formats whose codes sit in whole bytes or nibble/bit planes
// (Q8_0, Q5_0, Q5_K, Q6_K): 4 codes per 32-bit word, f16(1024 + code) by a byte permute, the exact code (or centred
// code) by one f16 subtraction, then the reference's single rounding -- one f16 multiply by d (Q8_0, Q5_0), or the
// f16 fma of the K-quants with f16(d sc) and f16(-dmin m) / f16(-32 d sc) -- the same operations group_f16 does value
// by value. words[i] = codes of values 4i..4i+3; s / o: the scale and offset of values 0..15 (s[0], o[0]) and 16..31.
LK_DEV void stage_words(const uint32_t (&c)[8], uint32_t bias, const __half2 (&s)[2], const __half2 (&o)[2], bool fma,
                        uint8_t* b_tile, int r, int c0) {
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const __half2 sc = s[cc >> 1], of = o[cc >> 1];
    uint32_t h[4] = {prmt(c[2 * cc], 0x64646464u, 0x4140u), prmt(c[2 * cc], 0x64646464u, 0x4342u),
                     prmt(c[2 * cc + 1], 0x64646464u, 0x4140u), prmt(c[2 * cc + 1], 0x64646464u, 0x4342u)};
    uint4 out;
    uint32_t* po = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int t = 0; t < 4; ++t) po[t] = fma ? hfma2u(hsub2u(h[t], bias), sc, of) : hmul2u(hsub2u(h[t], bias), sc);
    *reinterpret_cast<uint4*>(b_tile + sw128(r, c0 + cc)) = out;
  }
}

template <int FMT>
LK_DEV void dequant_group_words(const uint8_t* chunk, int j, uint8_t* b_tile, int r, int c0) {
  uint32_t c[8];
  __half2 s[2], o[2];
  if (FMT == LK_Q8_0) {   // int8 codes: code ^ 0x80 = code + 128; f16(1152 + code) - 1152 = code; f16(d code)
    const uint8_t* b = chunk + 34 * j;
    ld_words_2a(b + 2, c);
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] ^= 0x80808080u;
    const __half d = __ushort_as_half(*reinterpret_cast<const uint16_t*>(b));
    s[0] = s[1] = __halves2half2(d, d);
    stage_words(c, 0x64806480u, s, s, false, b_tile, r, c0);
  } else if (FMT == LK_Q5_0) {   // nibble | bit i of qh << 4; f16(1024 + code) - 1040 = code - 16; f16(d (code - 16))
    const uint8_t* b = chunk + 22 * j;
    uint32_t qh[1], qs[4];
    ld_words_2a(b + 2, qh);
    ld_words_2a(b + 6, qs);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t hb = (qh[0] >> (4 * i)) & 15u;
      c[i] = ((i < 4 ? qs[i] : qs[i - 4] >> 4) & 0x0F0F0F0Fu) |
             ((hb & 1u) << 4) | ((hb & 2u) << 11) | ((hb & 4u) << 18) | ((hb & 8u) << 25);
    }
    const __half d = __ushort_as_half(*reinterpret_cast<const uint16_t*>(b));
    s[0] = s[1] = __halves2half2(d, d);
    stage_words(c, 0x64106410u, s, s, false, b_tile, r, c0);
  } else if (FMT == LK_Q5_K) {   // Q4_K's nibble pages | bit j of qh[l] << 4; fma(code, f16(d sc), f16(-dmin m))
    int sc, m;
    q4k_scale_min(chunk + 4, j, sc, m);
    uint32_t qs[8], qh[8];
    ld_words_2a(chunk + 48 + 32 * (j >> 1), qs);
    ld_words_2a(chunk + 16, qh);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      c[i] = ((qs[i] >> (4 * (j & 1))) & 0x0F0F0F0Fu) | (((qh[i] >> j) & 0x01010101u) << 4);
    s[0] = s[1] = __float2half2_rn(f16_at(chunk) * float(sc));
    o[0] = o[1] = __float2half2_rn(-(f16_at(chunk + 2) * float(m)));
    stage_words(c, 0x64006400u, s, o, true, b_tile, r, c0);
  } else {   // Q6_K: ql nibble | 2 bits of qh << 4 (0..63); fma(code, f16(d sc), f16(-32 d sc)) per 16 values
    const int h = j >> 2, jj = j & 3;
    uint32_t ql[8], qh[8];
    ld_words_2a(chunk + 64 * h + 32 * (jj & 1), ql);
    ld_words_2a(chunk + 128 + 32 * h, qh);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      c[i] = ((ql[i] >> (4 * (jj >> 1))) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * jj)) & 0x03030303u) << 4);
    const float d = f16_at(chunk + 208);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float a = d * float(int8_t(chunk[192 + 2 * j + t]));
      s[t] = __float2half2_rn(a);
      o[t] = __float2half2_rn(-32.0f * a);
    }
    stage_words(c, 0x64006400u, s, o, true, b_tile, r, c0);
  }
}

// One 32-value group (j of the 256-value chunk) of any format into 4 swizzled 16-byte chunks of the B tile, with the
// reference's staging (group_f16: one rounding, or the K-quants' f16 fma)
template <int FMT>
LK_DEV void dequant_group_any(const uint8_t* chunk, int j, uint8_t* b_tile, int r, int c0) {
  if (FMT == LK_Q8_0 || FMT == LK_Q5_0 || FMT == LK_Q5_K || FMT == LK_Q6_K) {
    dequant_group_words<FMT>(chunk, j, b_tile, r, c0);
    return;
  }
  __half h[32];
  if (fmt_qk(FMT) == 32) group_f16<FMT>(chunk + j * fmt_block_bytes(FMT), 0, h);
  else group_f16<FMT>(chunk, j, h);
#pragma unroll
  for (int cc = 0; cc < 4; ++cc)
    *reinterpret_cast<uint4*>(b_tile + sw128(r, c0 + cc)) = reinterpret_cast<const uint4*>(h)[cc];
}

// 16-byte chunk `c` of row `r` of a K-major 128-byte-swizzled tile


// 8 codes (bytes of t0, t1; low nibble only) -> 8 f16 (1024 + code), natural k order
LK_DEV void magic8(uint32_t t0, uint32_t t1, uint32_t (&h)[4]) {
  h[0] = prmt(t0, 0x64646464u, 0x4140u);
  h[1] = prmt(t0, 0x64646464u, 0x4342u);
  h[2] = prmt(t1, 0x64646464u, 0x4140u);
  h[3] = prmt(t1, 0x64646464u, 0x4342u);
}

// Dequantise one 32-value group of one weight row into 4 swizzled 16-byte chunks of the B tile.
//   raw    : the row's 144-byte packed chunk (256 values) in shared memory
//   j      : group within the chunk (0..7); b_tile: the B stage; r: tile row; c0: first 16-byte chunk (0 or 4)
// Register arithmetic only: scales are formed in f16 (exact products rounded once), no conversion instructions.
template <int FMT>
LK_DEV void dequant_group(const uint8_t* raw, int j, uint8_t* b_tile, int r, int c0) {
  if (FMT == LK_Q4_K) {
    const uint8_t* qs = raw + 16 + 32 * (j >> 1);
    uint4 a = *reinterpret_cast<const uint4*>(qs);
    uint4 b = *reinterpret_cast<const uint4*>(qs + 16);
    uint4 hd = *reinterpret_cast<const uint4*>(raw);
    uint32_t sh = (j & 1) * 4;
    uint32_t c[8] = {(a.x >> sh) & 0x0F0F0F0Fu, (a.y >> sh) & 0x0F0F0F0Fu, (a.z >> sh) & 0x0F0F0F0Fu,
                     (a.w >> sh) & 0x0F0F0F0Fu, (b.x >> sh) & 0x0F0F0F0Fu, (b.y >> sh) & 0x0F0F0F0Fu,
                     (b.z >> sh) & 0x0F0F0F0Fu, (b.w >> sh) & 0x0F0F0F0Fu};
    uint32_t sc, m;
    q4k_scale_min_w(hd.y, hd.z, hd.w, j, sc, m);
    // f16(d * sc) and f16(-dmin * m): the f16 product of exact operands rounds once, like the f32 product + fptrunc
    __half a16 = __hmul(__ushort_as_half(uint16_t(hd.x & 0xffffu)), small_int_half(sc));
    __half c16 = __hneg(__hmul(__ushort_as_half(uint16_t(hd.x >> 16)), small_int_half(m)));
    __half2 scale = __halves2half2(a16, a16), offset = __halves2half2(c16, c16);
    const uint32_t k1024 = 0x64006400u;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t h[4];
      magic8(c[2 * cc], c[2 * cc + 1], h);
      uint4 out;
      out.x = hfma2u(hsub2u(h[0], k1024), scale, offset);
      out.y = hfma2u(hsub2u(h[1], k1024), scale, offset);
      out.z = hfma2u(hsub2u(h[2], k1024), scale, offset);
      out.w = hfma2u(hsub2u(h[3], k1024), scale, offset);
      *reinterpret_cast<uint4*>(b_tile + sw128(r, c0 + cc)) = out;
    }
    return;
  }
  // Q4_0 / IQ4_NL: 18-byte block j at raw + 18j: f16 d, then 16 code bytes (2-byte aligned)
  const uint16_t* p16 = reinterpret_cast<const uint16_t*>(raw + 18 * j);
  uint32_t q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = uint32_t(p16[1 + 2 * i]) | (uint32_t(p16[2 + 2 * i]) << 16);
  __half dh = __ushort_as_half(p16[0]);
  __half2 scale = __halves2half2(dh, dh);
  const uint32_t koff = FMT == LK_Q4_0 ? 0x64086408u : 0x64806480u;   // f16 1032 (1024 + 8) | 1152 (1024 + 128)
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    // chunk cc: values 8cc .. 8cc+7 = (cc < 2 ? low : high) nibbles of bytes 8*(cc&1) .. +7
    uint32_t w0 = q[2 * (cc & 1)], w1 = q[2 * (cc & 1) + 1];
    uint32_t t0 = ((cc >= 2) ? (w0 >> 4) : w0) & 0x0F0F0F0Fu;
    uint32_t t1 = ((cc >= 2) ? (w1 >> 4) : w1) & 0x0F0F0F0Fu;
    if (FMT == LK_IQ4_NL) {
      t0 = iq4_lookup4(t0);
      t1 = iq4_lookup4(t1);
    }
    uint32_t h[4];
    magic8(t0, t1, h);
    uint4 out;
    // exact centred code (q - 8, or the kvalue), then one f16 multiply by d: the reference's single rounding
    out.x = hmul2u(hsub2u(h[0], koff), scale);
    out.y = hmul2u(hsub2u(h[1], koff), scale);
    out.z = hmul2u(hsub2u(h[2], koff), scale);
    out.w = hmul2u(hsub2u(h[3], koff), scale);
    *reinterpret_cast<uint4*>(b_tile + sw128(r, c0 + cc)) = out;
  }
}

// dequant_group / dequant_group_any of the format `fmt` read at run time (format pairs)
LK_DEV void dequant_group_rt(int fmt, const uint8_t* chunk, int j, uint8_t* b_tile, int r, int c0) {
  switch (fmt) {
    case LK_Q4_0: dequant_group<LK_Q4_0>(chunk, j, b_tile, r, c0); return;
    case LK_IQ4_NL: dequant_group<LK_IQ4_NL>(chunk, j, b_tile, r, c0); return;
    case LK_Q4_K:   // the box form's register decode where the window left the 144-byte chunk 16-byte aligned
      if ((reinterpret_cast<uintptr_t>(chunk) & 15) == 0) dequant_group<LK_Q4_K>(chunk, j, b_tile, r, c0);
      else dequant_group_any<LK_Q4_K>(chunk, j, b_tile, r, c0);
      return;
    case LK_Q5_0: dequant_group_any<LK_Q5_0>(chunk, j, b_tile, r, c0); return;
    case LK_Q8_0: dequant_group_any<LK_Q8_0>(chunk, j, b_tile, r, c0); return;
    case LK_Q5_K: dequant_group_any<LK_Q5_K>(chunk, j, b_tile, r, c0); return;
    case LK_Q6_K: dequant_group_any<LK_Q6_K>(chunk, j, b_tile, r, c0); return;
    case LK_IQ4_XS: dequant_group_any<LK_IQ4_XS>(chunk, j, b_tile, r, c0); return;
    case LK_Q3_K: dequant_group_any<LK_Q3_K>(chunk, j, b_tile, r, c0); return;
    case LK_IQ3_S: dequant_group_any<LK_IQ3_S>(chunk, j, b_tile, r, c0); return;
    case LK_MXFP4: dequant_group_any<LK_MXFP4>(chunk, j, b_tile, r, c0); return;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Persistent dense GEMM: one CTA per SM walks the output tiles (tile t = blockIdx.x + i * gridDim.x; m fastest, so
// the CTAs in flight share weight tiles in L2). The rings run on across tile boundaries, and the two TMEM
// accumulator buffers (2 x 256 columns) let four dedicated epilogue warps drain tile i while the tensor core already
// accumulates tile i + 1:
//   warp 0        producer (A boxes, packed weight boxes)
//   warp 1        TMEM allocation, MMA issue; waits acc_empty[buf] before reusing an accumulator buffer
//   warps 2-9     dequantise B stages
//   warps 10-13   epilogue: acc_full[buf] -> tcgen05.ld -> scale (silu * u) -> shared staging -> coalesced stores
//                 -> acc_empty[buf]
// ---------------------------------------------------------------------------------------------------------------
constexpr int kEpWarps = 4;
constexpr int kGemmPThreads = (2 + kDqWarps + kEpWarps) * 32;
constexpr int kStgBytes = kEpWarps * 32 * kStgStride * 4;


// NBUF accumulator buffers of MH * NW * BN columns each (512 TMEM columns in all); SAP / SBP / SRP stages of the A,
// B and packed-weight rings
// WIN: the packed chunks come by per-row bulk copies of 16-byte aligned windows (any format, any row stride, a last
// chunk of fewer than 256 values) instead of one 2-D TMA box of 144-byte chunks per stage.
// Split-K turnstiles: one 64-bit flag per output tile of a launch, taken from a ring of slots, so that launches in
// flight on other streams use other flags. A flag holds epoch * 64 + (K ranges already added); every launch has its
// own epoch, and one launch's flags end at epoch * 64 + ksplit, a value no range of a later replay waits for.
constexpr int kKFlags = 1 << 16;
__device__ unsigned long long g_kflags[kKFlags];

// Waits until *flag == want (acquire); false when it gave up after about 2 s (the caller records the error and carries
// on, so a missing predecessor cannot hang the GPU).
LK_DEV bool turnstile_wait(const unsigned long long* flag, unsigned long long want) {
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
    if (v == want) return true;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > 2000000000ull) return false;
    __nanosleep(64);
  }
}

template <int FMT, int BN, int NW, int MODE, int GROUP, int MH, int NBUF, int SAP, int SBP, int SRP, bool WIN>
__global__ void __launch_bounds__(kGemmPThreads, 1)
    k_gemm_p(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
             const __grid_constant__ CUtensorMap w2map, const GemmArgs p) {
  constexpr int kTM = kBM * MH;
  constexpr int kRowsB = BN * NW;
  constexpr int kABytes = kTM * kBK * 2;
  constexpr int kBBytes = kRowsB * kBK * 2;
  constexpr int kCB = WIN ? chunk_bytes(FMT) : kChunkBytes;    // packed bytes of a 256-value chunk
  constexpr int kRW = row_slot_bytes(FMT, WIN);                // shared-memory bytes of one row's chunk
  constexpr int kRBytes = kRowsB * kRW;
  static_assert(WIN || chunk_bytes(FMT) == kChunkBytes, "the TMA box form streams 144-byte chunks");
  static_assert(FMT != kFmtPair || (WIN && NW == 2), "a format pair is a gate/up kernel of the window form");
  // window form: the packed source of row r's chunk of k stage ks (gate rows r < BN, up rows after them) and its length
  auto win_src = [&](int r, int wrow, int w2row, int ks, uintptr_t& src, uint32_t& clen) {
    const bool up = r >= BN;
    const int cb = FMT == kFmtPair ? (up ? p.cb2 : p.cb) : kCB;
    const int64_t rb = (FMT == kFmtPair && up) ? p.rb2 : p.rb;
    const int64_t c0b = int64_t(ks >> 2) * cb;
    clen = uint32_t(min(int64_t(cb), rb - c0b));
    src = reinterpret_cast<uintptr_t>(up ? p.w2p : p.wp) + uintptr_t((int64_t(up ? w2row : wrow) + r % BN) * rb + c0b);
  };
  constexpr int kSAp = SAP;
  constexpr int kSBp = SBP;
  constexpr uint32_t kAcc = MH * NW * BN;   // accumulator columns of one tile
  static_assert(NBUF * kAcc == 512, "the accumulator buffers fill the 512 TMEM columns");
  static_assert(kRowsB == 2 * kDqWarps * 16 || kRowsB == kDqWarps * 16, "one or two rows per dequant thread");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + kSAp * kABytes;
  uint8_t* sR = sB + kSBp * kBBytes;
  float* stg_all = reinterpret_cast<float*>(sR + SRP * kRBytes);
  uint64_t* full_a = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(stg_all) + kStgBytes);
  uint64_t* empty_a = full_a + kSAp;
  uint64_t* full_b = empty_a + kSAp;
  uint64_t* empty_b = full_b + kSBp;
  uint64_t* full_r = empty_b + kSBp;
  uint64_t* empty_r = full_r + SRP;
  uint64_t* acc_full = empty_r + SRP;    // [NBUF]
  uint64_t* acc_empty = acc_full + NBUF;   // [NBUF]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + NBUF);
  int* stbl = reinterpret_cast<int*>(tmem_slot + 4);   // MoE super-tile table [3][kMaxExperts]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kstages = p.k / kBK;
  const int mt = (p.rows + kTM - 1) / kTM, nt = (p.n + BN - 1) / BN;
  // tiles: dense m x n; grouped (super-tile, n) with the n tiles of a super-tile consecutive
  const int ntiles =
      GROUP == kDense ? mt * nt * p.ksplit : moe_super_table(p.tile_info, p.max_tiles, p.n_experts, stbl) * nt;
  const int my_tiles = ntiles > int(blockIdx.x) ? (ntiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
  // tile t -> first output row, first weight row of the tile inside the expert block, expert, valid rows, and the
  // k stages [ks0, ks1) it accumulates (dense: split ranges start on packed-stage boundaries)
  int ks0 = 0, ks1 = kstages;
  auto tile_of = [&](int t, int& m0, int& n0, int& e, int& valid) {
    if (GROUP == kDense) {
      const int tt = t % (mt * nt), si = t / (mt * nt);
      const int mi = p.n_fast ? tt / nt : tt % mt, ni = p.n_fast ? tt % nt : tt / mt;
      m0 = mi * kTM;
      n0 = ni * BN;
      e = 0;
      valid = min(kTM, p.rows - m0);
      ks0 = si * p.kps * 4;
      ks1 = min(kstages, ks0 + p.kps * 4);
    } else {
      int first, rows;
      moe_super_lookup(p.tile_info, stbl, t / nt, e, first, rows);
      e = min(e, p.n_experts - 1);
      m0 = first * 64;
      n0 = (t % nt) * BN;
      valid = rows;
    }
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSAp; ++i) {
      mbar_init(&full_a[i], 1);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < kSBp; ++i) {
      mbar_init(&full_b[i], kDqWarps);
      mbar_init(&empty_b[i], 1);
    }
    for (int i = 0; i < SRP; ++i) {
      mbar_init(&full_r[i], 1);
      mbar_init(&empty_r[i], kDqWarps);
    }
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpWarps);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, NBUF * kAcc);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&amap);
      prefetch_tensormap(&wmap);
      if (NW == 2) prefetch_tensormap(&w2map);
    }
    int ga = 0, gr = 0;
    for (int li = 0; li < my_tiles; ++li) {
      int m0, n0, e, valid;
      tile_of(int(blockIdx.x) + li * int(gridDim.x), m0, n0, e, valid);
      const int wrow = e * p.rows_per_expert + n0, w2row = e * p.rows_per_expert2 + p.w2_row_offset + n0;
      int arow[4] = {0, 0, 0, 0};
      if (GROUP == kGather) {   // the routed token rows of this tile: 4 per lane, out-of-range -> zero rows
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = lane * 4 + j;
          const int a = r < valid ? p.rowmap[m0 + r] : -1;
          arow[j] = a >= 0 ? a / p.ku : p.xrows;
        }
      }
      for (int ks = ks0; ks < ks1; ++ks) {
        if ((ks & 3) == 0) {
          const int sr = gr % SRP;
          if (gr >= SRP && !mbar_wait(&empty_r[sr], ((gr / SRP) - 1) & 1)) atomicOr(&g_status, 1u);
          if (WIN) {
            // every lane copies the chunk of rows lane, lane + 32, ... (those inside n): the 16-byte aligned window
            // around the row's chunk bytes. Lane 0 announces the stage's total bytes before any copy is issued.
            uint32_t mine = 0;
#pragma unroll
            for (int i = 0; i < kRowsB / 32; ++i) {
              const int r = lane + 32 * i, rl = r % BN;
              if (n0 + rl >= p.n) continue;
              uintptr_t src;
              uint32_t clen;
              win_src(r, wrow, w2row, ks, src, clen);
              mine += uint32_t(((src + clen + 15) & ~uintptr_t(15)) - (src & ~uintptr_t(15)));
            }
            uint32_t total = mine;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xFFFFFFFFu, total, o);
            if (lane == 0) mbar_expect_tx(&full_r[sr], total);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < kRowsB / 32; ++i) {
              const int r = lane + 32 * i, rl = r % BN;
              if (n0 + rl >= p.n) continue;
              uintptr_t src;
              uint32_t clen;
              win_src(r, wrow, w2row, ks, src, clen);
              const uintptr_t a0 = src & ~uintptr_t(15);
              bulk_g2s(sR + sr * kRBytes + r * kRW, reinterpret_cast<const void*>(a0),
                       uint32_t(((src + clen + 15) & ~uintptr_t(15)) - a0), &full_r[sr]);
            }
          } else if (lane == 0) {
            mbar_expect_tx(&full_r[sr], uint32_t(kRBytes));
            tma_load_2d(sR + sr * kRBytes, &wmap, (ks >> 2) * (kChunkBytes / 4), wrow, &full_r[sr]);
            if (NW == 2)
              tma_load_2d(sR + sr * kRBytes + BN * kChunkBytes, &w2map, (ks >> 2) * (kChunkBytes / 4), w2row,
                          &full_r[sr]);
          }
          __syncwarp();
          ++gr;
        }
        const int sa = ga % kSAp;
        if (ga >= kSAp && !mbar_wait(&empty_a[sa], ((ga / kSAp) - 1) & 1)) atomicOr(&g_status, 1u);
        if (lane == 0) mbar_expect_tx(&full_a[sa], kABytes);
        __syncwarp();
        if (GROUP == kGather) {
          tma_gather4(sA + sa * kABytes + lane * 4 * 128, &amap, ks * kBK, arow[0], arow[1], arow[2], arow[3],
                      &full_a[sa]);
        } else if (lane == 0) {
          tma_load_2d(sA + sa * kABytes, &amap, ks * kBK, m0, &full_a[sa]);
        }
        __syncwarp();
        ++ga;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_f16(kBM, BN, 0);
    const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
    int ga = 0, gb = 0;
    for (int li = 0; li < my_tiles; ++li) {
      int m0, n0, e, valid;
      tile_of(int(blockIdx.x) + li * int(gridDim.x), m0, n0, e, valid);
      const int buf = li % NBUF;
      if (li >= NBUF && !mbar_wait(&acc_empty[buf], ((li / NBUF) - 1) & 1)) atomicOr(&g_status, 1u);
      tc_fence_after();
      const uint32_t tacc = tmem + buf * kAcc;
      for (int ks = ks0; ks < ks1; ++ks) {
        const int sa = ga % kSAp, sb = gb % kSBp;
        if (!mbar_wait(&full_a[sa], (ga / kSAp) & 1)) atomicOr(&g_status, 1u);
        if (!mbar_wait(&full_b[sb], (gb / kSBp) & 1)) atomicOr(&g_status, 1u);
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
#pragma unroll
            for (int mh = 0; mh < MH; ++mh) {
              uint64_t ad = sdesc_k128(a_base + sa * kABytes + mh * (kBM * 128) + kk * 32);
#pragma unroll
              for (int wi = 0; wi < NW; ++wi) {
                uint64_t bd = sdesc_k128(b_base + sb * kBBytes + wi * BN * 128 + kk * 32);
                umma_f16(tacc + (mh * NW + wi) * BN, ad, bd, idesc, ks != ks0 || kk != 0);
              }
            }
          }
          umma_commit(&empty_a[sa]);
          umma_commit(&empty_b[sb]);
          if (ks == ks1 - 1) umma_commit(&acc_full[buf]);
        }
        __syncwarp();
        ++ga;
        ++gb;
      }
    }
  } else if (warp < 2 + kDqWarps) {
    // ------------------------------------------------------------------ dequant warps
    const int dt = threadIdx.x - 64;   // 0..255
    constexpr int kGroupsPerThread = kRowsB * 2 / (kDqWarps * 32);
    int gb = 0, gr = 0;
    for (int li = 0; li < my_tiles; ++li) {
      int m0, n0, e, valid;
      tile_of(int(blockIdx.x) + li * int(gridDim.x), m0, n0, e, valid);
      const int wrow = e * p.rows_per_expert + n0, w2row = e * p.rows_per_expert2 + p.w2_row_offset + n0;
      for (int ks = ks0; ks < ks1; ++ks) {
        const int sub = ks & 3, sr = gr % SRP, sb = gb % kSBp;
        // a chunk's last stage: its fourth, or the tile's last (a row whose last chunk holds fewer than 256 values)
        const bool chunk_end = sub == 3 || ks == ks1 - 1;
        if (sub == 0 && !mbar_wait(&full_r[sr], (gr / SRP) & 1)) atomicOr(&g_status, 1u);
        if (gb >= kSBp && !mbar_wait(&empty_b[sb], ((gb / kSBp) - 1) & 1)) atomicOr(&g_status, 1u);
        uint8_t* bt = sB + sb * kBBytes;
#pragma unroll
        for (int gi = 0; gi < kGroupsPerThread; ++gi) {
          const int item = dt * kGroupsPerThread + gi;   // (row, half) pairs
          const int r = item >> 1, h = item & 1;
          if (WIN) {
            // the row's chunk starts (src mod 16) bytes into its window; rows past n hold stale bytes whose
            // columns are never stored
            uintptr_t src;
            uint32_t clen;
            win_src(r, wrow, w2row, ks, src, clen);
            const uint8_t* chunk = sR + sr * kRBytes + r * kRW + (src & 15);
            if (FMT == kFmtPair) dequant_group_rt(r < BN ? p.fmt : p.fmt2, chunk, 2 * sub + h, bt, r, 4 * h);
            else if (FMT == LK_Q4_0 || FMT == LK_IQ4_NL) dequant_group<FMT>(chunk, 2 * sub + h, bt, r, 4 * h);
            else dequant_group_any<FMT>(chunk, 2 * sub + h, bt, r, 4 * h);
          } else {
            dequant_group<FMT>(sR + sr * kRBytes + r * kChunkBytes, 2 * sub + h, bt, r, 4 * h);
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&full_b[sb]);
          if (chunk_end) mbar_arrive(&empty_r[sr]);
        }
        ++gb;
        if (chunk_end) ++gr;
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue warps
    const int q = warp & 3;                    // TMEM lane quadrant this warp may read
    float* stg = stg_all + (warp - 2 - kDqWarps) * (32 * kStgStride);
    const int sr = lane >> 3, sc = 4 * (lane & 7);
    for (int li = 0; li < my_tiles; ++li) {
      int m0, n0, e, valid_rows;
      tile_of(int(blockIdx.x) + li * int(gridDim.x), m0, n0, e, valid_rows);
      const int nb_rows = min(BN, p.n - n0);
      // rows stored: a dense tile's valid rows; a MoE super-tile's whole 64-row tiles (one, or two when paired),
      // padding rows included -- their zero products give act(biases) -- as the reference's grouped tiles write
      const int store_rows = GROUP == kDense ? valid_rows : (valid_rows > 64 ? 128 : 64);
      const float* bcol = p.epi.bias ? p.epi.bias + int64_t(e) * p.n + n0 : nullptr;
      const float* b2col = p.epi.bias2 ? p.epi.bias2 + int64_t(e) * p.n + n0 : nullptr;
      const int buf = li % NBUF;
      if (!mbar_wait(&acc_full[buf], (li / NBUF) & 1)) atomicOr(&g_status, 1u);
      tc_fence_after();
      // split K: this item's K range and output tile; range s > 0 waits until ranges 0 .. s - 1 have added theirs
      const bool ksp = GROUP == kDense && p.ksplit > 1;
      const int item = int(blockIdx.x) + li * int(gridDim.x);
      const int kt = ksp ? item % (mt * nt) : 0, ksi = ksp ? item / (mt * nt) : 0;
      if (ksp && ksi > 0) {
        if (warp == 2 + kDqWarps && lane == 0 &&
            !turnstile_wait(p.kflags + kt, (p.kepoch << 6) | uint64_t(ksi)))
          atomicOr(&g_status, 4u);
        asm volatile("bar.sync 3, 128;" ::: "memory");   // the four epilogue warps
      }
#pragma unroll 1
      for (int mh = 0; mh < MH; ++mh) {
        const int row = mh * kBM + 32 * q + lane;
        int srow = row < valid_rows ? m0 + row : -1;
        if (GROUP == kGather && srow >= 0) {
          const int a = p.rowmap[srow];
          srow = a >= 0 ? a / p.ku : -1;
        }
        const float inv = srow >= 0 ? p.scales[2 * int64_t(srow) + 1] : 0.f;
        const uint32_t tbase = tmem + buf * kAcc + (uint32_t(32 * q) << 16) + mh * NW * BN;
#pragma unroll 1
        for (int col = 0; col < BN; col += 32) {
          float v[32];
          tmem_ld32(tbase + col, v);
          if (NW == 2) {
            float u[32];
            tmem_ld32(tbase + BN + col, u);
            if (bcol) {   // per-expert biases (columns past n read nothing: they are never stored)
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const bool in = col + i < nb_rows;
                v[i] = fmaf(v[i], inv, in ? __ldg(bcol + col + i) : 0.f);
                u[i] = fmaf(u[i], inv, in ? __ldg(b2col + col + i) : 0.f);
              }
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = act_apply(p.epi.act, v[i], u[i], p.epi.alpha, p.epi.limit);
            } else if (p.epi.act != LK_ACT_SILU) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = act_apply(p.epi.act, v[i] * inv, u[i] * inv, p.epi.alpha, p.epi.limit);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = silu(v[i] * inv) * (u[i] * inv);
            }
          } else if (bcol) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = fmaf(v[i], inv, col + i < nb_rows ? __ldg(bcol + col + i) : 0.f);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= inv;
          }
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(stg + lane * kStgStride + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          __syncwarp();
          const bool col_ok = col + sc < nb_rows;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int rr = 4 * j + sr;
            const int trow = mh * kBM + 32 * q + rr;
            float4 o = *reinterpret_cast<const float4*>(stg + rr * kStgStride + sc);
            if (col_ok && trow < store_rows) {
              const int64_t off = int64_t(m0 + trow) * p.ld + p.col_off + n0 + col + sc;
              if (ksp) {
                // K ranges meet in dst[0] (this rank's own y) in range order; the last range stores the finished
                // tile to every destination
                if (ksi > 0 || MODE == LK_ACC) {
                  const float4 old = __ldcg(reinterpret_cast<const float4*>(p.dst[0] + off));
                  o.x += old.x;
                  o.y += old.y;
                  o.z += old.z;
                  o.w += old.w;
                }
                if (ksi < p.ksplit - 1) {
                  *reinterpret_cast<float4*>(p.dst[0] + off) = o;
                  continue;
                }
              } else if (MODE == LK_ACC) {
                float4 old = *reinterpret_cast<const float4*>(p.dst[0] + off);
                o.x += old.x;
                o.y += old.y;
                o.z += old.z;
                o.w += old.w;
              } else if (MODE == LK_STORE && p.act_mul) {
                const float4 g = *reinterpret_cast<const float4*>(p.dst[0] + off);
                o.x = act_apply(p.epi.act, g.x, o.x, p.epi.alpha, p.epi.limit);
                o.y = act_apply(p.epi.act, g.y, o.y, p.epi.alpha, p.epi.limit);
                o.z = act_apply(p.epi.act, g.z, o.z, p.epi.alpha, p.epi.limit);
                o.w = act_apply(p.epi.act, g.w, o.w, p.epi.alpha, p.epi.limit);
              }
#pragma unroll
              for (int d = 0; d < kMaxPeers; ++d)
                if (d < p.ndst) *reinterpret_cast<float4*>(p.dst[d] + off) = o;
            }
          }
          __syncwarp();
        }
      }
      if (ksp) {   // every epilogue warp's stores of the range are issued: pass the turnstile on
        asm volatile("bar.sync 3, 128;" ::: "memory");
        if (warp == 2 + kDqWarps && lane == 0) {
          __threadfence();
          asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p.kflags + kt), "l"((p.kepoch << 6) | uint64_t(ksi + 1))
                       : "memory");
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, NBUF * kAcc);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D tensor map over a row-major [rows][cols] matrix; box = box_cols x box_rows elements
int make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, int64_t rows, int64_t cols,
             int box_cols, int box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LK_ECUDA;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols * elem_bytes)};
  cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LK_OK : LK_EINVAL;
}

// any tiled tensor map (dims, strides in bytes, box and element strides given in full), zero out-of-range fill
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
                 const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* estr, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LK_ECUDA;
  CUresult r = fn(map, dt, cuuint32_t(rank), const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LK_OK : LK_EINVAL;
}

struct GemmMaps {
  CUtensorMap a, w, w2;
};

template <int FMT, int BN, int NW, int MODE, int GROUP, int MH, int NBUF, int SAP, int SBP, int SRP, bool WIN>
static int launch_gemm_p(const GemmMaps& m, const GemmArgs& a, cudaStream_t s) {
  constexpr int kRowsB = BN * NW;
  constexpr int kABytes = kBM * MH * kBK * 2, kBBytes = kRowsB * kBK * 2;
  constexpr int kRBytes = kRowsB * row_slot_bytes(FMT, WIN);
  constexpr int smem = 1024 + SAP * kABytes + SBP * kBBytes + SRP * kRBytes + kStgBytes +
                       (2 * (SAP + SBP + SRP) + 2 * NBUF) * 8 + 16 + 3 * kMaxExperts * 4;
  static_assert(smem <= 227 * 1024, "persistent GEMM CTA exceeds shared memory");
  auto kern = k_gemm_p<FMT, BN, NW, MODE, GROUP, MH, NBUF, SAP, SBP, SRP, WIN>;
  static unsigned configured = 0;
  if (!once_per_device(configured)) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // dense: the exact tile count (with the K ranges); grouped: a bound (at most one super-tile per schedule tile)
  const int ntiles = (GROUP == kDense ? (a.rows + kBM * MH - 1) / (kBM * MH) * a.ksplit : a.rows / 64) *
                     ((a.n + BN - 1) / BN);
  kern<<<min(ntiles, sms), kGemmPThreads, smem, s>>>(m.a, m.w, m.w2, a);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

// tile shape per mode: (BN, NW, MH)
//   dense store/acc  128 x 1 x 2   a 256 x 128 tile, two M=128 accumulators sharing each dequantised B stage
//   ... at most 128 rows  256 x 1 x 1   a 128 x 256 tile: no padded M half, twice the weight rows per stage
//   dense swiglu     128 x 2 x 1   128 rows x 128 columns of gate and of up
//   grouped gate/up  128 x 2 x 1   (MoE super-tiles hold at most 128 rows of one expert; gathered or sorted rows)
//   grouped down     256 x 1 x 1
template <int FMT>
static int gemm_fmt(int mode, int group, bool short_m, const GemmMaps& m, const GemmArgs& a, cudaStream_t s) {
  if (group == kDense) {   // persistent kernel
    if (mode == LK_SWIGLU) return launch_gemm_p<FMT, 128, 2, LK_SWIGLU, kDense, 1, 2, 4, 2, 2, false>(m, a, s);
    if (short_m)
      return mode == LK_ACC ? launch_gemm_p<FMT, 256, 1, LK_ACC, kDense, 1, 2, 4, 2, 2, false>(m, a, s)
                            : launch_gemm_p<FMT, 256, 1, LK_STORE, kDense, 1, 2, 4, 2, 2, false>(m, a, s);
    if (mode == LK_ACC) return launch_gemm_p<FMT, 128, 1, LK_ACC, kDense, 2, 2, 3, 4, 2, false>(m, a, s);
    return launch_gemm_p<FMT, 128, 1, LK_STORE, kDense, 2, 2, 3, 4, 2, false>(m, a, s);
  }
  if (group == kGather) return launch_gemm_p<FMT, 128, 2, LK_SWIGLU, kGather, 1, 2, 4, 2, 2, false>(m, a, s);
  if (mode == LK_SWIGLU_SORTED) return launch_gemm_p<FMT, 128, 2, LK_SWIGLU, kSorted, 1, 2, 4, 2, 2, false>(m, a, s);
  return launch_gemm_p<FMT, 256, 1, LK_STORE, kSorted, 1, 2, 4, 2, 2, false>(m, a, s);
}

// the window form: 128 weight rows per stage in every mode (a window of a large chunk -- Q8_0's 272 bytes, Q6_K's
// 210 -- takes up to 288 bytes a row), so the rings fit shared memory:
//   dense swiglu 64 x 2 x 1; dense store/acc 128 x 1 x 2 (at most 128 rows: 128 x 1 x 1); grouped gate/up 64 x 2 x 1;
//   grouped down 128 x 1 x 1
template <int FMT>
static int gemm_fmt_win(int mode, int group, bool short_m, const GemmMaps& m, const GemmArgs& a, cudaStream_t s) {
  if (group == kDense) {
    if (mode == LK_SWIGLU) return launch_gemm_p<FMT, 64, 2, LK_SWIGLU, kDense, 1, 4, 4, 4, 2, true>(m, a, s);
    if (short_m)
      return mode == LK_ACC ? launch_gemm_p<FMT, 128, 1, LK_ACC, kDense, 1, 4, 4, 4, 2, true>(m, a, s)
                            : launch_gemm_p<FMT, 128, 1, LK_STORE, kDense, 1, 4, 4, 4, 2, true>(m, a, s);
    if (mode == LK_ACC) return launch_gemm_p<FMT, 128, 1, LK_ACC, kDense, 2, 2, 2, 4, 2, true>(m, a, s);
    return launch_gemm_p<FMT, 128, 1, LK_STORE, kDense, 2, 2, 2, 4, 2, true>(m, a, s);
  }
  if (group == kGather) return launch_gemm_p<FMT, 64, 2, LK_SWIGLU, kGather, 1, 4, 4, 4, 2, true>(m, a, s);
  if (mode == LK_SWIGLU_SORTED) return launch_gemm_p<FMT, 64, 2, LK_SWIGLU, kSorted, 1, 4, 4, 4, 2, true>(m, a, s);
  return launch_gemm_p<FMT, 128, 1, LK_STORE, kSorted, 1, 4, 4, 4, 2, true>(m, a, s);
}

// gate and up weights in two formats: the gate/up kernels of the window form, each weight decoded in its own format
static int gemm_pair_win(int group, const GemmMaps& m, const GemmArgs& a, cudaStream_t s) {
  if (group == kDense) return launch_gemm_p<kFmtPair, 64, 2, LK_SWIGLU, kDense, 1, 4, 4, 4, 2, true>(m, a, s);
  if (group == kGather) return launch_gemm_p<kFmtPair, 64, 2, LK_SWIGLU, kGather, 1, 4, 4, 4, 2, true>(m, a, s);
  return launch_gemm_p<kFmtPair, 64, 2, LK_SWIGLU, kSorted, 1, 4, 4, 4, 2, true>(m, a, s);
}

// K ranges for a dense store / acc GEMM of `tiles` output tiles and kp packed stages on `sms` persistent CTAs: the
// count whose rounds x (stages per range + 1, + 1 more when split: the read-add-write of y) is least -- the + 1
// stands for a tile's fill and epilogue -- with no empty range; the smallest such count on ties
static int choose_ksplit(int tiles, int kp, int sms) {
  int best = 1;
  int64_t best_cost = INT64_MAX;
  for (int sp = 1; sp <= std::min(kp, 32); ++sp) {
    const int per = (kp + sp - 1) / sp;
    if ((kp + per - 1) / per != sp) continue;
    const int64_t rounds = (int64_t(tiles) * sp + sms - 1) / sms;
    const int64_t cost = rounds * (per + 1 + (sp > 1 ? 1 : 0));
    if (cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

int gemm(int fmt, int mode, int rows, int k, int n, const uint16_t* x16, const float* scales, const void* w,
         const void* w2, float* y, cudaStream_t s, const int32_t* tile_info, const int32_t* rowmap, int xrows, int ku,
         int n_experts, int64_t expert_stride, int64_t w2_offset, const OutSpec* out, const ExpertEpi* epi,
         bool act_mul) {
  if ((fmt >> 16) && !out && (mode == LK_SWIGLU ? !tile_info : mode == LK_SWIGLU_SORTED)) {
    // a gate/up pair on dense or bucket-sorted rows: two passes of the single-format kernels -- the gate's products
    // (+ its bias) stored in y, then the up weight's with the activation applied against them in the epilogue --
    // where each weight can take its own kernel (a Q4_K one keeps its 16-byte aligned rows); else the pair kernel
    const int fg = fmt & 0xffff, fu = fmt >> 16;
    auto own = [&](int f, const void* p) { return f != LK_Q4_K || (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (own(fg, w) && own(fu, w2)) {
      const ExpertEpi e0 = epi ? *epi : ExpertEpi{};
      const ExpertEpi eg{e0.bias, nullptr, LK_ACT_SILU, 0.f, 0.f}, eu{e0.bias2, nullptr, e0.act, e0.alpha, e0.limit};
      // LK_STORE: dense rows, or with a schedule the sorted-row store the down projection uses (A = x16[r], scales[r])
      int rc = gemm(fg, LK_STORE, rows, k, n, x16, scales, w, nullptr, y, s, tile_info, rowmap, xrows, ku, n_experts,
                    lk_row_bytes(fg, k) * n, 0, nullptr, &eg);
      if (rc == LK_OK)
        rc = gemm(fu, LK_STORE, rows, k, n, x16, scales, w2, nullptr, y, s, tile_info, rowmap, xrows, ku, n_experts,
                  lk_row_bytes(fu, k) * n, 0, nullptr, &eu, true);
      return rc;
    }
  }
  GemmArgs a{};
  a.act_mul = act_mul;
  a.scales = scales;
  if (epi) a.epi = *epi;
  if (out) {
    for (int d = 0; d < out->ndst; ++d) a.dst[d] = out->dst[d];
    a.ndst = out->ndst;
    a.ld = out->ld;
    a.col_off = out->col_off;
  } else {
    a.dst[0] = y;
    a.ndst = 1;
    a.ld = n;
    a.col_off = 0;
  }
  a.rows = rows;
  a.k = k;
  a.n = n;
  // LK_FMT_PAIR(gate, up): the gate's format in the low 16 bits, the up weight's above (gate/up modes only)
  const bool pair = (fmt >> 16) != 0;
  a.fmt = fmt & 0xffff;
  a.fmt2 = pair ? fmt >> 16 : a.fmt;
  fmt = a.fmt;
  const int64_t rb = lk_row_bytes(a.fmt, k);
  a.rb2 = lk_row_bytes(a.fmt2, k);
  a.cb = chunk_bytes(a.fmt);
  a.cb2 = chunk_bytes(a.fmt2);
  if (pair && mode != LK_SWIGLU && mode != LK_SWIGLU_SORTED) return LK_EINVAL;
  // rasterise so the larger operand is read once: n tiles of an m tile first when the activations outweigh the
  // weights (each A tile is then reused from L2 across the n tiles)
  a.n_fast = int64_t(rows) * k * 2 > int64_t(n) * (mode == LK_SWIGLU ? rb + a.rb2 : rb);
  int group = kDense;
  int64_t wrows = n, w2rows = n;
  a.rows_per_expert = a.rows_per_expert2 = 0;
  if (tile_info) {
    group = mode == LK_SWIGLU ? kGather : kSorted;
    a.tile_info = tile_info;
    a.rowmap = rowmap;
    a.max_tiles = rows / 64;
    a.xrows = xrows;
    a.ku = ku;
    a.n_experts = n_experts;
    a.rows_per_expert = int(expert_stride / rb);
    a.rows_per_expert2 = w2 ? n : a.rows_per_expert;
    wrows = int64_t(n_experts) * a.rows_per_expert;
    w2rows = int64_t(n_experts) * a.rows_per_expert2;
  }
  a.w2_row_offset = (mode != LK_STORE && mode != LK_ACC && !w2) ? int(w2_offset / rb) : 0;
  // the window producer: every format but the Q4 family's 144-byte chunks in 16-byte aligned rows
  const bool win = pair || !((fmt == LK_Q4_0 || fmt == LK_Q4_K || fmt == LK_IQ4_NL) && k % 256 == 0 &&
                     (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(w2) & 15) == 0);
  a.wp = static_cast<const uint8_t*>(w);
  a.w2p = static_cast<const uint8_t*>(w2 ? w2 : w);
  a.rb = rb;
  // at most 128 rows (dense store / acc): 128-row tiles of 256 weight rows (window form: 128)
  const bool short_m = group == kDense && mode != LK_SWIGLU && rows <= kBM;
  // weight rows per tile (per weight): the TMA form 256 for grouped down and short dense, 128 otherwise; the window
  // form 128, 64 per weight for gate/up
  const bool gu = mode == LK_SWIGLU || mode == LK_SWIGLU_SORTED;
  const int bn = win ? (gu ? 64 : 128) : (((group == kSorted && mode == LK_STORE) || short_m) ? 256 : 128);
  const int tm = (group == kDense && mode != LK_SWIGLU && !short_m) ? 2 * kBM : kBM;   // tile rows
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int kp = (k + 255) / 256;   // packed chunks of 256 values (the last one may be shorter)
  a.ksplit = 1;
  a.kps = kp;
  // dense store / acc: split K where the rounds of the persistent grid come out shorter (few tiles, or a last round
  // that would run nearly empty); the ranges meet in dst[0] in order
  const int dense_tiles = ((rows + tm - 1) / tm) * ((n + bn - 1) / bn);
  if (group == kDense && mode != LK_SWIGLU && rows > 0 && !act_mul) {
    a.ksplit = choose_ksplit(dense_tiles, kp, sms);
    a.kps = (kp + a.ksplit - 1) / a.ksplit;
  }
  GemmMaps m;
  int rc = group == kGather ? make_map(&m.a, x16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xrows, k, kBK, 1,
                                       CU_TENSOR_MAP_SWIZZLE_128B)   // one-row boxes for gather4
                            : make_map(&m.a, x16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, rows, k, kBK, tm,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == LK_OK && !win)
    rc = make_map(&m.w, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, wrows, rb / 4, kChunkBytes / 4, bn,
                  CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc == LK_OK && !win)
    rc = w2 ? make_map(&m.w2, w2, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w2rows, rb / 4, kChunkBytes / 4, bn,
                       CU_TENSOR_MAP_SWIZZLE_NONE)
            : (m.w2 = m.w, LK_OK);
  if (rc != LK_OK) return rc;
  if (win) m.w = m.w2 = m.a;   // unused by the window form
  if (a.ksplit > 1) {   // turnstile flags for the dense tiles of this launch (range 0 stores, the others add in order)
    static unsigned long long* base[32] = {};
    static std::atomic<unsigned long long> epoch{0};
    static std::atomic<unsigned> slot{0};
    if (dev >= 32) return LK_EUNSUPPORTED;
    if (!base[dev] && cudaGetSymbolAddress(reinterpret_cast<void**>(&base[dev]), g_kflags) != cudaSuccess)
      return LK_ECUDA;
    unsigned s0 = slot.fetch_add(unsigned(dense_tiles)) % kKFlags;
    if (s0 + unsigned(dense_tiles) > unsigned(kKFlags)) s0 = 0;
    a.kflags = base[dev] + s0;
    a.kepoch = ++epoch;
  }
  if (pair) return gemm_pair_win(group, m, a, s);
  if (!win) {
    switch (fmt) {
      case LK_Q4_0: return gemm_fmt<LK_Q4_0>(mode, group, short_m, m, a, s);
      case LK_Q4_K: return gemm_fmt<LK_Q4_K>(mode, group, short_m, m, a, s);
      case LK_IQ4_NL: return gemm_fmt<LK_IQ4_NL>(mode, group, short_m, m, a, s);
    }
    return LK_EUNSUPPORTED;
  }
  switch (fmt) {
    case LK_Q4_0: return gemm_fmt_win<LK_Q4_0>(mode, group, short_m, m, a, s);
    case LK_IQ4_NL: return gemm_fmt_win<LK_IQ4_NL>(mode, group, short_m, m, a, s);
    case LK_Q5_0: return gemm_fmt_win<LK_Q5_0>(mode, group, short_m, m, a, s);
    case LK_Q8_0: return gemm_fmt_win<LK_Q8_0>(mode, group, short_m, m, a, s);
    case LK_Q5_K: return gemm_fmt_win<LK_Q5_K>(mode, group, short_m, m, a, s);
    case LK_Q6_K: return gemm_fmt_win<LK_Q6_K>(mode, group, short_m, m, a, s);
    case LK_IQ4_XS: return gemm_fmt_win<LK_IQ4_XS>(mode, group, short_m, m, a, s);
    case LK_Q3_K: return gemm_fmt_win<LK_Q3_K>(mode, group, short_m, m, a, s);
    case LK_IQ3_S: return gemm_fmt_win<LK_IQ3_S>(mode, group, short_m, m, a, s);
    case LK_MXFP4: return gemm_fmt_win<LK_MXFP4>(mode, group, short_m, m, a, s);
  }
  return LK_EUNSUPPORTED;
}

LK_STATUS_READER(status_gemm)

}  // namespace lk
