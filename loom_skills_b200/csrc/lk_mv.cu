// Decode matvec for GGUF block weights (tokens < 64): y[t][n] (+)= sum_k x[t][k] W[n][k].
//
// Replaces g_mv_{fmt}_k{K}[_t{TG}][_r{R}] and its swiglu pair (gen_llm.py:1159-1378) and the MoE expert matvecs
// g_moe_gu_/g_moe_dn_ (gen_moe.py:535-727).
//
// Design (HBM-bound). A CTA owns 16 weight rows and up to 8 tokens. A producer warp streams, per stage, one 2-D TMA
// box of the rows' packed bytes per consumer warp (16 rows x 144 bytes = 256 k each; 8 consumers for one dense token,
// 4 otherwise) plus the matching slice of each token's activations (1-D bulk copies) into a 4-stage shared-memory
// ring. Each consumer warp takes one 256-value chunk of every
// stage: they convert their activation slice to f16 once (with per-32-value group sums), then unpack nibbles in
// registers straight into the A fragments of warp-level f16 MMAs (16 rows x 16 k x 8 tokens) -- the weights never
// go back to shared memory. Codes enter the MMA as exact small-integer f16 values, made from a (1024 + code) bit
// pattern minus its offset: q - 8 (Q4_0), the kvalue (IQ4_NL, from the codebook byte kvalue + 128), q or 16 q (Q4_K
// low / high nibbles). The per-32-value group scale is applied in f32 afterwards:
//     Q4_0 / IQ4_NL: sum_k d v_k x_k = d * D;   Q4_K: sum_k (a q_k - c) x_k = a * D - c * S,   S = sum x_k
// with a = d*sc, c = dmin*m per group. Centred codes keep D free of the cancellation a (1024 + q) offset would cause:
// the f32 accumulation of exact codes is as precise as the reference's f32 dequant-then-dot (gen_llm.py:1281-1357).
//
// Kernels: k_mv (token tiles of up to 8, one CTA per 16 rows), k_mv_rows (persistent: one dense token, or MoE expert
// matvecs per assignment, optionally with the router folded in), k_mv_grp (persistent: MoE expert matvecs of 128 to
// 1024 assignments grouped by expert, 8 to the MMA's token columns). mv_x picks one by shape.
#include <mutex>

#include "lk_common.cuh"
#include "lk_internal.h"
#include "lk_route.cuh"

namespace lk {

// consumer warps per CTA (CONS below; one 256-value chunk of each stage apiece): 8 for one token of a dense matvec --
// more warps in flight per SM hide the TMA and decode latency (measured: Q4_0 4096 x 4096 fp16 6.83 -> 5.98 us, the
// bf16 decode step 1885 -> 1982 GB/s) -- and 4 for token tiles of 8, whose larger stages must fit, and for the MoE
// expert matvecs, whose short rows (one stage at K = 2048) ran slower with 8 (27 -> 31 us for configs[2] at M = 1)
constexpr int mv_consumers(int tok, bool moe) { return tok == 1 && !moe ? 8 : 4; }
constexpr int kMvRows = 16;
// ring depth: 4 stages, or 2 when a stage is large (two weights and 8 f32 tokens) so the CTA fits shared memory
constexpr int mv_stages(int stage_bytes) { return 4 * stage_bytes <= 150 * 1024 ? 4 : 2; }
constexpr int kMvChunkTile = kMvRows * kChunkBytes;             // 2304: 16 rows x 144 bytes (one TMA box)
constexpr int kAcStride = 10;                                   // float2 stride of a row of the (a, c') table
constexpr int kXStride = 272;                                   // f16 row stride of a consumer's x tile

LK_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D = A * B (zero accumulator input)
LK_DEV void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

LK_DEV uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

LK_DEV uint32_t hsub2u(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
// bytes of t (code in the low or high nibble, other nibble zero) -> A fragment halves (byte - off) for 4 consecutive k:
// the f16 bit pattern of 1024 + byte, minus the f16 pair koff2 = (1024 + off) -- exact for every byte
LK_DEV void code_frag(uint32_t t, uint32_t koff2, uint32_t& first, uint32_t& second) {
  first = hsub2u(prmt(t, 0x64646464u, 0x4140u), koff2);
  second = hsub2u(prmt(t, 0x64646464u, 0x4342u), koff2);
}
constexpr uint32_t kMagic1024 = 0x64006400u;   // f16 pair (1024, 1024)

LK_DEV uint32_t lds_u16x2(const uint8_t* p) {   // 2-byte aligned 4 bytes
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
  return uint32_t(q[0]) | (uint32_t(q[1]) << 16);
}

// acc += a * D - c' * S for the lane's D elements: rows g, g+8 x tokens 2tig, 2tig+1. With one token only the
// token-0 column carries data (elements 0 and 2).
template <int TOK>
LK_DEV void group_epilogue_d(float (&acc)[4], const float (&d)[4], float a_g, float a_g8) {   // no offset term
  acc[0] = fmaf(a_g, d[0], acc[0]);
  acc[2] = fmaf(a_g8, d[2], acc[2]);
  if (TOK > 1) {
    acc[1] = fmaf(a_g, d[1], acc[1]);
    acc[3] = fmaf(a_g8, d[3], acc[3]);
  }
}
template <int TOK>
LK_DEV void group_epilogue(float (&acc)[4], const float (&d)[4], float2 s01, float a_g, float c_g, float a_g8,
                           float c_g8) {
  acc[0] = fmaf(a_g, d[0], fmaf(-c_g, s01.x, acc[0]));
  acc[2] = fmaf(a_g8, d[2], fmaf(-c_g8, s01.x, acc[2]));
  if (TOK > 1) {
    acc[1] = fmaf(a_g, d[1], fmaf(-c_g, s01.y, acc[1]));
    acc[3] = fmaf(a_g8, d[3], fmaf(-c_g8, s01.y, acc[3]));
  }
}

// 4 bytes (values 0..255) of w -> f32, without a conversion instruction
LK_DEV float byte_f32(uint32_t w, uint32_t sel) {
  return __uint_as_float(prmt(w, 0x4B000000u, sel)) - 8388608.0f;
}

// B fragment (token g, 4 consecutive k) from a consumer's f16 x tile; zero for lanes past the token count
LK_DEV void bfrag(const __half* xt, int g, int kk, bool valid, uint32_t& b0, uint32_t& b1) {
  if (valid) {
    uint2 v = *reinterpret_cast<const uint2*>(xt + g * kXStride + kk);
    b0 = v.x;
    b1 = v.y;
  } else {
    b0 = b1 = 0;
  }
}

// A lane's 8 activations of a 256-value chunk as f32, from the raw words it loaded (f32: two uint4, else one).
template <int XT>
LK_DEV void x8_f32(const uint4* r, float (&f)[8]) {
  if (XT == LK_F32) {
    f[0] = __uint_as_float(r[0].x); f[1] = __uint_as_float(r[0].y);
    f[2] = __uint_as_float(r[0].z); f[3] = __uint_as_float(r[0].w);
    f[4] = __uint_as_float(r[1].x); f[5] = __uint_as_float(r[1].y);
    f[6] = __uint_as_float(r[1].z); f[7] = __uint_as_float(r[1].w);
  } else {
    uint32_t w[4] = {r[0].x, r[0].y, r[0].z, r[0].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (XT == LK_BF16) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      } else {
        float2 h = __half22float2(*reinterpret_cast<__half2*>(&w[i]));
        f[2 * i] = h.x;
        f[2 * i + 1] = h.y;
      }
    }
  }
}

// One token of a chunk: the lane's 8 f32 activations into the f16 tile (and, for f32, the residual tile) and the
// token's per-group sums S[8].
template <int XT>
LK_DEV void put_x8(const float (&f)[8], int lane, __half* xt, __half* xl, float* S);

// Convert this chunk's activations (ntok tokens x 256 values) to the f16 tile(s) and per-group sums S[t][8].
template <int XT, int TOK>
LK_DEV void stage_x(const uint8_t* xraw, int xraw_stride, int ntok, int lane, __half* xt, __half* xl, float* S) {
#pragma unroll
  for (int t = 0; t < TOK; ++t) {
    if (t >= ntok) break;
    constexpr int NR = XT == LK_F32 ? 2 : 1;
    const uint4* p = reinterpret_cast<const uint4*>(xraw + t * xraw_stride) + NR * lane;
    uint4 r[NR];
#pragma unroll
    for (int j = 0; j < NR; ++j) r[j] = p[j];
    float f[8];
    x8_f32<XT>(r, f);
    put_x8<XT>(f, lane, xt + t * kXStride, xl + t * kXStride, S + t * 8);
  }
}

template <int XT>
LK_DEV void put_x8(const float (&f)[8], int lane, __half* xt, __half* xl, float* S) {
  uint32_t hp[4], lp[4];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    hp[i] = h2u(h);
    if (XT == LK_F32) {
      float2 hf = __half22float2(h);
      lp[i] = h2u(__floats2half2_rn(f[2 * i] - hf.x, f[2 * i + 1] - hf.y));
    }
    s += f[2 * i] + f[2 * i + 1];
  }
  *reinterpret_cast<uint4*>(xt + 8 * lane) = make_uint4(hp[0], hp[1], hp[2], hp[3]);
  if (XT == LK_F32) *reinterpret_cast<uint4*>(xl + 8 * lane) = make_uint4(lp[0], lp[1], lp[2], lp[3]);
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  if ((lane & 3) == 0) S[lane >> 2] = s;   // group lane/4
}

// One 256-value chunk of 16 rows (row r at rb + r*144, one TMA box) against the staged x tile.
template <int FMT, int XT, int NW, int TOK>
LK_DEV void mv_chunk(const uint8_t* rb0, const uint8_t* rb1, const __half* xt, const __half* xl, const float* S,
                     bool xvalid, int g, int tig, int lane, float2* actab, float (&acc)[NW][4]) {
  constexpr int RS = kChunkBytes;
  // S for tokens 2tig, 2tig+1 of group j (with one token, token 0's for every lane)
  auto sums = [&](int j) {
    return TOK == 1 ? make_float2(S[j], 0.f) : make_float2(S[(2 * tig) * 8 + j], S[(2 * tig + 1) * 8 + j]);
  };
  if (FMT == LK_Q4_K) {
    // cooperative header decode: lane -> (row lane/2, groups 4*(lane&1) .. +3), four groups at a time with byte-wise
    // bit operations. Low-nibble groups (even j) hold (a, c); high-nibble groups (odd j, whose codes the MMA sees as
    // 16 q) hold (a / 16, c).
#pragma unroll
    for (int wi = 0; wi < NW; ++wi) {
      const uint8_t* rb = wi ? rb1 : rb0;
      const int r = lane >> 1, hh = lane & 1;
      uint4 hv = *reinterpret_cast<const uint4*>(rb + r * RS);
      float d = h2f(uint16_t(hv.x & 0xffff)), dmin = h2f(uint16_t(hv.x >> 16));
      uint32_t sc4 = hh ? ((hv.w & 0x0F0F0F0Fu) | ((hv.y >> 2) & 0x30303030u)) : (hv.y & 0x3F3F3F3Fu);
      uint32_t m4 = hh ? (((hv.w >> 4) & 0x0F0F0F0Fu) | ((hv.z >> 2) & 0x30303030u)) : (hv.z & 0x3F3F3F3Fu);
      float4 lo, hi;
      float a0 = d * byte_f32(sc4, 0x7650u), a1 = d * byte_f32(sc4, 0x7651u);
      float a2 = d * byte_f32(sc4, 0x7652u), a3 = d * byte_f32(sc4, 0x7653u);
      lo = make_float4(a0, dmin * byte_f32(m4, 0x7650u), a1 * 0.0625f, dmin * byte_f32(m4, 0x7651u));
      hi = make_float4(a2, dmin * byte_f32(m4, 0x7652u), a3 * 0.0625f, dmin * byte_f32(m4, 0x7653u));
      float4* dst = reinterpret_cast<float4*>(actab + wi * 16 * kAcStride + r * kAcStride + 4 * hh);
      dst[0] = lo;
      dst[1] = hi;
    }
    __syncwarp();
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float dl[NW][4], dh[NW][4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t bl0, bl1, bh0, bh1;
        int kk = 64 * p + 16 * h + 4 * tig;
        bfrag(xt, g, kk, xvalid, bl0, bl1);
        bfrag(xt, g, kk + 32, xvalid, bh0, bh1);
        uint32_t ll0 = 0, ll1 = 0, lh0 = 0, lh1 = 0;
        if (XT == LK_F32) {
          bfrag(xl, g, kk, xvalid, ll0, ll1);
          bfrag(xl, g, kk + 32, xvalid, lh0, lh1);
        }
#pragma unroll
        for (int wi = 0; wi < NW; ++wi) {
          const uint8_t* rb = wi ? rb1 : rb0;
          int off = 16 + 32 * p + 16 * h + 4 * tig;
          uint32_t w0 = *reinterpret_cast<const uint32_t*>(rb + g * RS + off);
          uint32_t w8 = *reinterpret_cast<const uint32_t*>(rb + (g + 8) * RS + off);
          uint32_t f0, s0, f8, s8;
          code_frag(w0 & 0x0F0F0F0Fu, kMagic1024, f0, s0);
          code_frag(w8 & 0x0F0F0F0Fu, kMagic1024, f8, s8);
          if (h == 0) mma16816_z(dl[wi], f0, f8, s0, s8, bl0, bl1);
          else mma16816(dl[wi], f0, f8, s0, s8, bl0, bl1);
          if (XT == LK_F32) mma16816(dl[wi], f0, f8, s0, s8, ll0, ll1);
          code_frag(w0 & 0xF0F0F0F0u, kMagic1024, f0, s0);
          code_frag(w8 & 0xF0F0F0F0u, kMagic1024, f8, s8);
          if (h == 0) mma16816_z(dh[wi], f0, f8, s0, s8, bh0, bh1);
          else mma16816(dh[wi], f0, f8, s0, s8, bh0, bh1);
          if (XT == LK_F32) mma16816(dh[wi], f0, f8, s0, s8, lh0, lh1);
        }
      }
      float2 sl = sums(2 * p), sh = sums(2 * p + 1);
#pragma unroll
      for (int wi = 0; wi < NW; ++wi) {
        float4 r0 = *reinterpret_cast<const float4*>(&actab[wi * 16 * kAcStride + g * kAcStride + 2 * p]);
        float4 r8 = *reinterpret_cast<const float4*>(&actab[wi * 16 * kAcStride + (g + 8) * kAcStride + 2 * p]);
        group_epilogue<TOK>(acc[wi], dl[wi], sl, r0.x, r0.y, r8.x, r8.y);
        group_epilogue<TOK>(acc[wi], dh[wi], sh, r0.z, r0.w, r8.z, r8.w);
      }
    }
    __syncwarp();   // the table is rewritten by the next chunk
  } else {
    constexpr uint32_t kOff2 = FMT == LK_Q4_0 ? 0x64086408u : 0x64806480u;   // f16 pairs 1024 + (8 | 128 bias)
#pragma unroll 2
    for (int j = 0; j < 8; ++j) {
      uint32_t b00, b01, b10, b11, l00 = 0, l01 = 0, l10 = 0, l11 = 0;
      int kk = 32 * j + 4 * tig;
      bfrag(xt, g, kk, xvalid, b00, b01);
      bfrag(xt, g, kk + 16, xvalid, b10, b11);
      if (XT == LK_F32) {
        bfrag(xl, g, kk, xvalid, l00, l01);
        bfrag(xl, g, kk + 16, xvalid, l10, l11);
      }
#pragma unroll
      for (int wi = 0; wi < NW; ++wi) {
        const uint8_t* blk = (wi ? rb1 : rb0) + 18 * j;
        const uint8_t* p0 = blk + g * RS;
        const uint8_t* p8 = blk + (g + 8) * RS;
        float d0 = h2f(*reinterpret_cast<const uint16_t*>(p0));
        float d8 = h2f(*reinterpret_cast<const uint16_t*>(p8));
        uint32_t w0 = lds_u16x2(p0 + 2 + 4 * tig), w8 = lds_u16x2(p8 + 2 + 4 * tig);
        uint32_t t0 = w0 & 0x0F0F0F0Fu, t8 = w8 & 0x0F0F0F0Fu;
        uint32_t u0 = (w0 >> 4) & 0x0F0F0F0Fu, u8 = (w8 >> 4) & 0x0F0F0F0Fu;
        if (FMT == LK_IQ4_NL) {
          t0 = iq4_lookup4(t0);
          t8 = iq4_lookup4(t8);
          u0 = iq4_lookup4(u0);
          u8 = iq4_lookup4(u8);
        }
        float dd[4];
        uint32_t f0, s0, f8, s8;
        code_frag(t0, kOff2, f0, s0);
        code_frag(t8, kOff2, f8, s8);
        mma16816_z(dd, f0, f8, s0, s8, b00, b01);
        if (XT == LK_F32) mma16816(dd, f0, f8, s0, s8, l00, l01);
        code_frag(u0, kOff2, f0, s0);
        code_frag(u8, kOff2, f8, s8);
        mma16816(dd, f0, f8, s0, s8, b10, b11);
        if (XT == LK_F32) mma16816(dd, f0, f8, s0, s8, l10, l11);
        group_epilogue_d<TOK>(acc[wi], dd, d0, d8);
      }
    }
  }
}

template <int FMT, int XT, bool SWIGLU, bool MOE, int TOK, int CONS = mv_consumers(TOK, MOE)>
__global__ void __launch_bounds__((CONS + 1) * 32, (SWIGLU && XT == LK_F32) ? 1 : 2) k_mv(const __grid_constant__ CUtensorMap wmap,
                                                        const __grid_constant__ CUtensorMap w2map, MvArgs a) {
  constexpr int kMvConsumers = CONS, kMvStageChunks = CONS;
  constexpr int kMvWBytes = kMvStageChunks * kMvChunkTile;   // one weight's chunk tiles per stage
  constexpr int NW = SWIGLU ? 2 : 1;
  constexpr int XE = XT == LK_F32 ? 4 : 2;                          // activation element bytes
  constexpr int kXStageBytes = TOK * kMvStageChunks * 256 * XE;     // raw activations per stage
  constexpr int kStageBytes = NW * kMvWBytes + kXStageBytes;
  constexpr int kMvStages = mv_stages(kStageBytes);
  constexpr int kXT = (XT == LK_F32 ? 2 : 1) * TOK * kXStride;      // f16 elements of a consumer's x tile(s)
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kMvStages * kStageBytes);
  uint64_t* empty = full + kMvStages;
  float2* actab_all = reinterpret_cast<float2*>(empty + kMvStages);    // [consumers][NW][16][kAcStride]
  float* red = reinterpret_cast<float*>(actab_all + kMvConsumers * NW * 16 * kAcStride);   // [consumers][NW][32][4]
  float* S_all = red + kMvConsumers * NW * 32 * 4;                                  // [consumers][TOK][8]
  __half* xt_all = reinterpret_cast<__half*>(S_all + kMvConsumers * TOK * 8);       // [consumers][kXT]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * kMvRows;
  int wrow = r0, w2row = r0 + a.w2_row_offset;
  int xrow0, ntok, yrow0, e = 0;
  if (MOE) {
    int asg = blockIdx.y;
    e = min(max(a.ids[asg], 0), a.n_experts - 1);
    wrow = e * a.rows_per_expert + r0;
    w2row = e * a.rows_per_expert2 + a.w2_row_offset + r0;
    xrow0 = asg / a.x_div;
    ntok = 1;
    yrow0 = asg;
  } else {
    xrow0 = blockIdx.y * TOK;
    ntok = min(TOK, a.tokens - xrow0);
    yrow0 = xrow0;
  }
  const int kchunks = a.k / kChunkValues;
  const int nstages = (kchunks + kMvStageChunks - 1) / kMvStageChunks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMvStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMvConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kMvConsumers) {
    // producer: stage st = chunks [4 st, 4 st + 4) of the 16 rows, and the same k range of every token
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      if (NW == 2) prefetch_tensormap(&w2map);
      const uint8_t* xbase = static_cast<const uint8_t*>(a.x) + int64_t(xrow0) * a.k * XE;
      for (int st = 0; st < nstages; ++st) {
        int s = st % kMvStages;
        if (st >= kMvStages && !mbar_wait(&empty[s], ((st / kMvStages) - 1) & 1)) atomicOr(&g_status, 1u);
        int c0 = st * kMvStageChunks;
        int nch = min(kMvStageChunks, kchunks - c0);
        uint32_t xbytes = uint32_t(nch) * 256u * XE;
        mbar_expect_tx(&full[s], uint32_t(NW * nch * kMvChunkTile) + xbytes * ntok);
        uint8_t* stg = ring + s * kStageBytes;
        // one box per chunk: a [16 rows][144 bytes] tile, whose 36-word row stride spreads the rows over the banks
        for (int c = 0; c < nch; ++c) {
          tma_load_2d(stg + c * kMvChunkTile, &wmap, (c0 + c) * (kChunkBytes / 4), wrow, &full[s]);
          if (NW == 2)
            tma_load_2d(stg + kMvWBytes + c * kMvChunkTile, &w2map, (c0 + c) * (kChunkBytes / 4), w2row, &full[s]);
        }
        for (int t = 0; t < ntok; ++t)
          bulk_g2s(stg + NW * kMvWBytes + t * (kMvStageChunks * 256 * XE), xbase + (int64_t(t) * a.k + c0 * 256) * XE,
                   xbytes, &full[s]);
      }
    }
    return;
  }

  // consumers
  const int g = lane >> 2, tig = lane & 3;
  float acc[NW][4];
#pragma unroll
  for (int wi = 0; wi < NW; ++wi)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[wi][i] = 0.f;
  const bool xvalid = g < ntok;
  float2* actab = actab_all + warp * NW * 16 * kAcStride;
  float* S = S_all + warp * TOK * 8;
  __half* xt = xt_all + warp * kXT;
  __half* xl = xt + TOK * kXStride;
  for (int st = 0; st < nstages; ++st) {
    int s = st % kMvStages;
    if (!mbar_wait(&full[s], (st / kMvStages) & 1)) atomicOr(&g_status, 1u);
    int c = st * kMvStageChunks + warp;
    if (c < kchunks) {
      const uint8_t* stg = ring + s * kStageBytes;
      stage_x<XT, TOK>(stg + NW * kMvWBytes + warp * 256 * XE, kMvStageChunks * 256 * XE, ntok, lane, xt, xl, S);
      __syncwarp();
      const uint8_t* rb0 = stg + warp * kMvChunkTile;
      mv_chunk<FMT, XT, NW, TOK>(rb0, rb0 + kMvWBytes, xt, xl, S, xvalid, g, tig, lane, actab, acc);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // reduce the consumers' partial sums; warp 0 stores
#pragma unroll
  for (int wi = 0; wi < NW; ++wi)
    *reinterpret_cast<float4*>(red + ((warp * NW + wi) * 32 + lane) * 4) =
        make_float4(acc[wi][0], acc[wi][1], acc[wi][2], acc[wi][3]);
  asm volatile("bar.sync 1, %0;" ::"r"(kMvConsumers * 32));
  if (warp != 0) return;
  float out[NW][4];
#pragma unroll
  for (int wi = 0; wi < NW; ++wi)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kMvConsumers; ++w) sum += red[((w * NW + wi) * 32 + lane) * 4 + i];
      out[wi][i] = sum;
    }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int row = r0 + g + (i >= 2 ? 8 : 0);
    int tok = 2 * tig + (i & 1);
    if (row >= a.n || tok >= ntok) continue;
    float g = out[0][i], u = out[NW - 1][i];
    if (MOE && a.epi.bias) {   // per-expert output biases (gen_moe.py:535 expert_mv bias=True)
      g += __ldg(a.epi.bias + int64_t(e) * a.n + row);
      if (SWIGLU) u += __ldg(a.epi.bias2 + int64_t(e) * a.n + row);
    }
    float v = SWIGLU ? act_apply(a.epi.act, g, u, a.epi.alpha, a.epi.limit) : g;
    float* yp = a.y + int64_t(yrow0 + tok) * a.n + row;
    *yp = a.accumulate ? *yp + v : v;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Persistent one-token dense form (the decode step's shape): the same chunk math, with the activation row converted to
// its f16 chunk tiles (and group sums) once per CTA instead of once per stage, and the CTAs walking 16-row blocks
// round-robin, so the producer's TMA ring runs on across row blocks while the consumers finish the previous one.
// Per row block the 8 consumer warps' partial sums meet in shared memory; warp 0 stores the 16 outputs.
// MOE: per-assignment expert matvecs: the blocks are (assignment, 16-row block) pairs, each block's rows taken from
// its assignment's expert, with the expert epilogue (biases, activation). The activation row is the one token's for
// every assignment (the gate/up matvecs of one decode token), or with XPER row a / x_div of the assignment a (its
// token's row for gate/up, its own for down), each CTA then walking a contiguous range of blocks and converting the
// row again where its range crosses into another assignment.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kRowsCons = 8;
template <bool SWIGLU>
constexpr int rows_stages() { return SWIGLU ? 2 : 3; }

template <int FMT, int XT, bool SWIGLU, bool MOE, bool XPER, bool ROUTE>
__global__ void __launch_bounds__((kRowsCons + 1) * 32, SWIGLU ? 1 : 2)
    k_mv_rows(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap w2map, MvArgs a) {
  constexpr int NW = SWIGLU ? 2 : 1, NST = rows_stages<SWIGLU>();
  constexpr int kWB = kRowsCons * kMvChunkTile;                     // one weight's chunk tiles per stage
  constexpr int kStageBytes = NW * kWB;
  constexpr int kXT = (XT == LK_F32 ? 2 : 1) * kXStride;            // f16 elements of one chunk's x tile(s)
  constexpr int XE = XT == LK_F32 ? 4 : 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * kStageBytes);
  uint64_t* empty = full + NST;
  float2* actab_all = reinterpret_cast<float2*>(empty + NST);                                  // [cons][NW][16][st]
  float* red = reinterpret_cast<float*>(actab_all + kRowsCons * NW * 16 * kAcStride);        // [cons][NW][32][4]
  float* S_all = red + kRowsCons * NW * 32 * 4;                                               // [kchunks][8]
  const int kchunks = a.k / kChunkValues;
  __half* xt_all = reinterpret_cast<__half*>(S_all + kchunks * 8);                          // [kchunks][kXT]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nrb = (a.n + kMvRows - 1) / kMvRows;           // 16-row blocks of one output row
  const int nblk = MOE ? a.tokens * nrb : nrb;              // MoE: a.tokens = assignments
  const int nstages = (kchunks + kRowsCons - 1) / kRowsCons;
  // blocks of this CTA: round-robin, or with XPER a contiguous range (fewer activation rows to restage)
  const int b0 = XPER ? int(int64_t(blockIdx.x) * nblk / gridDim.x) : blockIdx.x;
  const int b1 = XPER ? int(int64_t(blockIdx.x + 1) * nblk / gridDim.x) : nblk;
  const int bstep = XPER ? 1 : gridDim.x;
  // ROUTE: every CTA routes the token itself (one warp, the router's own code) before anything else; CTA 0 stores
  // the routing for the launches after this one
  __shared__ int32_t s_ids[8];
  __shared__ float s_wts[8];
  if (ROUTE && warp == 0) {
    route_token(lane, a.n_experts, a.x_div, a.gating, a.norm, a.rscale, a.logits, a.rbias, s_ids, s_wts);
    __syncwarp();
    if (blockIdx.x == 0 && lane < a.x_div) {
      a.ids_out[lane] = s_ids[lane];
      a.wts_out[lane] = s_wts[lane];
    }
  }
  // block blk: its expert (MoE), first weight row in w and w2, first output row
  auto expert_of = [&](int blk) {
    return MOE ? min(max(ROUTE ? s_ids[blk / nrb] : __ldg(a.ids + blk / nrb), 0), a.n_experts - 1) : 0;
  };
  auto wrow_of = [&](int blk) { return expert_of(blk) * a.rows_per_expert + (blk % nrb) * kMvRows; };
  auto w2row_of = [&](int blk) {
    return expert_of(blk) * a.rows_per_expert2 + a.w2_row_offset + (blk % nrb) * kMvRows;
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRowsCons);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kRowsCons) {   // producer: stage (block, st) = chunks [8 st, 8 st + 8) of the block's 16 rows
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      if (NW == 2) prefetch_tensormap(&w2map);
      int i = 0;
      for (int blk = b0; blk < b1; blk += bstep) {
        const int wr = wrow_of(blk), w2r = NW == 2 ? w2row_of(blk) : 0;
        for (int st = 0; st < nstages; ++st, ++i) {
          const int s = i % NST;
          if (i >= NST && !mbar_wait(&empty[s], ((i / NST) - 1) & 1)) atomicOr(&g_status, 1u);
          const int c0 = st * kRowsCons, nch = min(kRowsCons, kchunks - c0);
          mbar_expect_tx(&full[s], uint32_t(NW * nch * kMvChunkTile));
          uint8_t* stg = smem + s * kStageBytes;
          for (int c = 0; c < nch; ++c) {
            tma_load_2d(stg + c * kMvChunkTile, &wmap, (c0 + c) * (kChunkBytes / 4), wr, &full[s]);
            if (NW == 2)
              tma_load_2d(stg + kWB + c * kMvChunkTile, &w2map, (c0 + c) * (kChunkBytes / 4), w2r, &full[s]);
          }
        }
      }
    }
    return;
  }
  // consumers: the activation row as f16 chunk tiles and group sums (once, or per assignment with XPER)
  auto stage_row = [&](int xrow) {
    for (int c = warp; c < kchunks; c += kRowsCons)
      stage_x<XT, 1>(static_cast<const uint8_t*>(a.x) + (int64_t(xrow) * a.k + int64_t(c) * 256) * XE, 0, 1, lane,
                     xt_all + c * kXT, xt_all + c * kXT + kXStride, S_all + c * 8);
    asm volatile("bar.sync 1, %0;" ::"r"(kRowsCons * 32) : "memory");
  };
  if (!XPER) stage_row(0);
  int staged = -1;   // the assignment whose row the tiles hold (XPER)
  const int g = lane >> 2, tig = lane & 3;
  float2* actab = actab_all + warp * NW * 16 * kAcStride;
  int i = 0;
  for (int blk = b0; blk < b1; blk += bstep) {
    if (XPER && (blk / nrb) / a.x_div != staged) {   // the previous block's last bar.sync has every warp done
      staged = (blk / nrb) / a.x_div;                  // with the old tiles
      stage_row(staged);
    }
    float acc[NW][4];
#pragma unroll
    for (int wi = 0; wi < NW; ++wi)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[wi][e] = 0.f;
    for (int st = 0; st < nstages; ++st, ++i) {
      const int s = i % NST;
      if (!mbar_wait(&full[s], (i / NST) & 1)) atomicOr(&g_status, 1u);
      const int c = st * kRowsCons + warp;
      if (c < kchunks) {
        const uint8_t* rb0 = smem + s * kStageBytes + warp * kMvChunkTile;
        mv_chunk<FMT, XT, NW, 1>(rb0, rb0 + kWB, xt_all + c * kXT, xt_all + c * kXT + kXStride, S_all + c * 8, g == 0,
                                 g, tig, lane, actab, acc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int wi = 0; wi < NW; ++wi)
      *reinterpret_cast<float4*>(red + ((warp * NW + wi) * 32 + lane) * 4) =
          make_float4(acc[wi][0], acc[wi][1], acc[wi][2], acc[wi][3]);
    asm volatile("bar.sync 1, %0;" ::"r"(kRowsCons * 32) : "memory");
    if (warp == 0 && tig == 0) {   // token 0: elements 0 (row g) and 2 (row g + 8)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = (blk % nrb) * kMvRows + g + 8 * h;
        float out[NW];
#pragma unroll
        for (int wi = 0; wi < NW; ++wi) {
          float sum = 0.f;
#pragma unroll
          for (int w = 0; w < kRowsCons; ++w) sum += red[((w * NW + wi) * 32 + lane) * 4 + 2 * h];
          out[wi] = sum;
        }
        if (row < a.n) {
          if (MOE && a.epi.bias) {   // per-expert output biases (gen_moe.py:535 expert_mv bias=True)
            const int e = expert_of(blk);
            out[0] += __ldg(a.epi.bias + int64_t(e) * a.n + row);
            if (SWIGLU) out[NW - 1] += __ldg(a.epi.bias2 + int64_t(e) * a.n + row);
          }
          const float v = SWIGLU ? act_apply(a.epi.act, out[0], out[NW - 1], a.epi.alpha, a.epi.limit) : out[0];
          float* yp = a.y + (MOE ? int64_t(blk / nrb) * a.n : 0) + row;
          *yp = a.accumulate ? *yp + v : v;
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kRowsCons * 32) : "memory");   // red is rewritten by the next block
  }
}

int make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, int64_t rows, int64_t cols,
             int box_cols, int box_rows, CUtensorMapSwizzle swz);

template <int FMT, int XT, bool SWIGLU, bool MOE, int TOK>
static int launch_mv(const CUtensorMap& wm, const CUtensorMap& w2m, const MvArgs& a, int groups, cudaStream_t s) {
  constexpr int kMvConsumers = mv_consumers(TOK, MOE), kMvStageChunks = kMvConsumers;
  constexpr int kMvWBytes = kMvStageChunks * kMvChunkTile;
  constexpr int NW = SWIGLU ? 2 : 1;
  constexpr int XE = XT == LK_F32 ? 4 : 2;
  constexpr int kStageBytes = NW * kMvWBytes + TOK * kMvStageChunks * 256 * XE;
  constexpr int kXT = (XT == LK_F32 ? 2 : 1) * TOK * kXStride;
  constexpr int kMvStages = mv_stages(kStageBytes);
  static_assert(kMvStages * kStageBytes + 64 * 1024 <= 227 * 1024, "matvec CTA exceeds shared memory");
  constexpr int smem = kMvStages * kStageBytes + 2 * kMvStages * 8 + kMvConsumers * NW * 16 * kAcStride * 8 +
                       kMvConsumers * NW * 32 * 4 * 4 + kMvConsumers * TOK * 8 * 4 + kMvConsumers * kXT * 2;
  auto kern = k_mv<FMT, XT, SWIGLU, MOE, TOK>;
  static unsigned configured = 0;
  if (!once_per_device(configured)) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((a.n + kMvRows - 1) / kMvRows, groups);
  kern<<<grid, (kMvConsumers + 1) * 32, smem, s>>>(wm, w2m, a);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

template <int FMT, int XT, bool SWIGLU, bool MOE, bool XPER = false, bool ROUTE = false>
static int launch_mv_rows(const CUtensorMap& wm, const CUtensorMap& w2m, const MvArgs& a, cudaStream_t s) {
  constexpr int NW = SWIGLU ? 2 : 1, NST = rows_stages<SWIGLU>();
  constexpr int kXT = (XT == LK_F32 ? 2 : 1) * kXStride;
  const int kchunks = a.k / kChunkValues;
  const int smem = NST * NW * kRowsCons * kMvChunkTile + 2 * NST * 8 + kRowsCons * NW * 16 * kAcStride * 8 +
                   kRowsCons * NW * 32 * 4 * 4 + kchunks * 8 * 4 + kchunks * kXT * 2;
  if (smem > 200 * 1024) return LK_EUNSUPPORTED;   // rows past ~40k values: the per-stage form below
  auto kern = k_mv_rows<FMT, XT, SWIGLU, MOE, XPER, ROUTE>;
  static int configured[32] = {};   // the largest shared-memory size set per device
  static std::mutex mu;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  if (dev >= 32) return LK_EUNSUPPORTED;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (configured[dev] < smem) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return LK_ECUDA;
      configured[dev] = smem;
    }
  }
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (kRowsCons + 1) * 32, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int nblk = (a.n + kMvRows - 1) / kMvRows * (MOE ? a.tokens : 1);
  kern<<<min(nblk, per_sm * sms), (kRowsCons + 1) * 32, smem, s>>>(wm, w2m, a);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

// ---------------------------------------------------------------------------------------------------------------
// Expert-grouped form of the per-assignment expert matvecs (MoE decode at several tokens). The assignments are grouped
// by expert, at most 8 to a group, so a 16-row block of an expert's weights is read once for all the assignments of
// its group: the group's activation rows fill the MMA's 8 token columns, which the per-assignment form leaves empty.
// Every CTA groups the assignments itself and deterministically (warp 0 in rounds of 32 over the assignments: counts
// per expert, one scan, stable placement), so all CTAs see the same groups without scratch memory or another launch.
// The work items are (group, 16-row block) pairs, a contiguous range of them per CTA, so a CTA restages the activation
// tiles only where its range crosses into another group (the rows of a group loaded together, then converted). Each assignment's outputs are its own row y[a][n], computed by
// the same chunk math as the per-assignment form (an MMA column depends on its own activations only).
// ---------------------------------------------------------------------------------------------------------------
constexpr int kGrpTok = 8;      // assignments of one group (the MMA's token columns)
constexpr int kGrpMaxA = 1024;  // assignments one launch can group
constexpr int kGrpMinA = 128;   // below this the per-assignment form measured faster (configs[2] shapes)
template <int FMT, int XT, bool SWIGLU>
__global__ void __launch_bounds__((kRowsCons + 1) * 32, SWIGLU ? 1 : 2)
    k_mv_grp(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap w2map, MvArgs a) {
  constexpr int NW = SWIGLU ? 2 : 1, NST = rows_stages<SWIGLU>();
  constexpr int kWB = kRowsCons * kMvChunkTile;
  constexpr int kStageBytes = NW * kWB;
  constexpr int kXT = (XT == LK_F32 ? 2 : 1) * kGrpTok * kXStride;   // f16 elements of one chunk's x tiles
  constexpr int XE = XT == LK_F32 ? 4 : 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * kStageBytes);
  uint64_t* empty = full + NST;
  float2* actab_all = reinterpret_cast<float2*>(empty + NST);                                  // [cons][NW][16][st]
  float* red = reinterpret_cast<float*>(actab_all + kRowsCons * NW * 16 * kAcStride);        // [cons][NW][32][4]
  float* S_all = red + kRowsCons * NW * 32 * 4;                                               // [kchunks][8][8]
  const int kchunks = a.k / kChunkValues;
  __half* xt_all = reinterpret_cast<__half*>(S_all + kchunks * kGrpTok * 8);                // [kchunks][kXT]
  __shared__ int s_cnt[256];            // assignments per expert, then the placement cursor
  __shared__ int s_order[kGrpMaxA];     // the assignments in (expert, assignment) order
  __shared__ int s_grp[kGrpMaxA];       // group: expert | count << 8 | first place in s_order << 12
  __shared__ int s_ngrp;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int A = a.tokens, E = a.n_experts;
  if (warp == 0) {
    auto expert_at = [&](int i) { return i < A ? min(max(__ldg(a.ids + i), 0), E - 1) : -1; };
    for (int e = lane; e < E; e += 32) s_cnt[e] = 0;
    __syncwarp();
    for (int b = 0; b < A; b += 32) {   // counts: the first lane of each expert's peers adds them
      const int e = expert_at(b + lane);
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e >= 0 && (peers & ((1u << lane) - 1)) == 0) s_cnt[e] += __popc(peers);
      __syncwarp();
    }
    const int per = (E + 31) / 32;   // lane owns experts [lane * per, lane * per + per)
    int pos = 0, grp = 0;
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < E) {
        pos += s_cnt[e];
        grp += (s_cnt[e] + kGrpTok - 1) / kGrpTok;
      }
    }
    int pinc = pos, ginc = grp;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int p = __shfl_up_sync(0xffffffffu, pinc, o), q = __shfl_up_sync(0xffffffffu, ginc, o);
      if (lane >= o) {
        pinc += p;
        ginc += q;
      }
    }
    int pb = pinc - pos, gb = ginc - grp;
    if (lane == 31) s_ngrp = ginc;
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < E) {
        const int c = s_cnt[e];
        for (int q = 0; q < c; q += kGrpTok) s_grp[gb++] = e | (min(kGrpTok, c - q) << 8) | ((pb + q) << 12);
        s_cnt[e] = pb;
        pb += c;
      }
    }
    __syncwarp();
    for (int b = 0; b < A; b += 32) {   // stable placement, in assignment order within each expert
      const int e = expert_at(b + lane);
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int rank = __popc(peers & ((1u << lane) - 1));
      if (e >= 0) s_order[s_cnt[e] + rank] = b + lane;
      __syncwarp();
      if (e >= 0 && rank == 0) s_cnt[e] += __popc(peers);
      __syncwarp();
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRowsCons);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int nrb = (a.n + kMvRows - 1) / kMvRows;
  const int nitems = s_ngrp * nrb;
  const int it0 = int(int64_t(blockIdx.x) * nitems / gridDim.x), it1 = int(int64_t(blockIdx.x + 1) * nitems / gridDim.x);
  const int nstages = (kchunks + kRowsCons - 1) / kRowsCons;
  if (warp == kRowsCons) {   // producer: stage (item, st) = chunks [8 st, 8 st + 8) of the item's 16 expert rows
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      if (NW == 2) prefetch_tensormap(&w2map);
      int i = 0;
      for (int it = it0; it < it1; ++it) {
        const int e = s_grp[it / nrb] & 0xff, r0 = (it % nrb) * kMvRows;
        const int wr = e * a.rows_per_expert + r0, w2r = e * a.rows_per_expert2 + a.w2_row_offset + r0;
        for (int st = 0; st < nstages; ++st, ++i) {
          const int s = i % NST;
          if (i >= NST && !mbar_wait(&empty[s], ((i / NST) - 1) & 1)) atomicOr(&g_status, 1u);
          const int c0 = st * kRowsCons, nch = min(kRowsCons, kchunks - c0);
          mbar_expect_tx(&full[s], uint32_t(NW * nch * kMvChunkTile));
          uint8_t* stg = smem + s * kStageBytes;
          for (int c = 0; c < nch; ++c) {
            tma_load_2d(stg + c * kMvChunkTile, &wmap, (c0 + c) * (kChunkBytes / 4), wr, &full[s]);
            if (NW == 2)
              tma_load_2d(stg + kWB + c * kMvChunkTile, &w2map, (c0 + c) * (kChunkBytes / 4), w2r, &full[s]);
          }
        }
      }
    }
    return;
  }
  const int g = lane >> 2, tig = lane & 3;
  float2* actab = actab_all + warp * NW * 16 * kAcStride;
  int staged = -1, i = 0;
  for (int it = it0; it < it1; ++it) {
    const int gi = it / nrb, gw = s_grp[gi], e = gw & 0xff, ng = (gw >> 8) & 15, first = gw >> 12;
    if (gi != staged) {   // the previous item's last bar.sync has every warp done with the old tiles
      staged = gi;
      constexpr int NR = XT == LK_F32 ? 2 : 1, TB = kGrpTok / NR;   // rows loaded together: 8 words per lane
      for (int c = warp; c < kchunks; c += kRowsCons) {
        __half* xt = xt_all + c * kXT;
        for (int t0 = 0; t0 < ng; t0 += TB) {
          uint4 r[TB][NR];
#pragma unroll
          for (int t = 0; t < TB; ++t)
            if (t0 + t < ng) {
              const int xrow = s_order[first + t0 + t] / a.x_div;
              const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.x) +
                                                              (int64_t(xrow) * a.k + int64_t(c) * 256) * XE) +
                               NR * lane;
#pragma unroll
              for (int j = 0; j < NR; ++j) r[t][j] = __ldg(p + j);
            }
#pragma unroll
          for (int t = 0; t < TB; ++t)
            if (t0 + t < ng) {
              const int u = t0 + t;
              float f[8];
              x8_f32<XT>(r[t], f);
              put_x8<XT>(f, lane, xt + u * kXStride, xt + (kGrpTok + u) * kXStride, S_all + (c * kGrpTok + u) * 8);
            }
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kRowsCons * 32) : "memory");
    }
    float acc[NW][4];
#pragma unroll
    for (int wi = 0; wi < NW; ++wi)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[wi][q] = 0.f;
    for (int st = 0; st < nstages; ++st, ++i) {
      const int s = i % NST;
      if (!mbar_wait(&full[s], (i / NST) & 1)) atomicOr(&g_status, 1u);
      const int c = st * kRowsCons + warp;
      if (c < kchunks) {
        const uint8_t* rb0 = smem + s * kStageBytes + warp * kMvChunkTile;
        const __half* xt = xt_all + c * kXT;
        mv_chunk<FMT, XT, NW, kGrpTok>(rb0, rb0 + kWB, xt, xt + kGrpTok * kXStride, S_all + c * kGrpTok * 8, g < ng,
                                       g, tig, lane, actab, acc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int wi = 0; wi < NW; ++wi)
      *reinterpret_cast<float4*>(red + ((warp * NW + wi) * 32 + lane) * 4) =
          make_float4(acc[wi][0], acc[wi][1], acc[wi][2], acc[wi][3]);
    asm volatile("bar.sync 1, %0;" ::"r"(kRowsCons * 32) : "memory");
    if (warp == 0) {   // element q: row g (q < 2) or g + 8, token column 2 tig + (q & 1)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int row = (it % nrb) * kMvRows + g + (q >= 2 ? 8 : 0), tok = 2 * tig + (q & 1);
        float out[NW];
#pragma unroll
        for (int wi = 0; wi < NW; ++wi) {
          float sum = 0.f;
#pragma unroll
          for (int w = 0; w < kRowsCons; ++w) sum += red[((w * NW + wi) * 32 + lane) * 4 + q];
          out[wi] = sum;
        }
        if (row < a.n && tok < ng) {
          if (a.epi.bias) {   // per-expert output biases (gen_moe.py:535 expert_mv bias=True)
            out[0] += __ldg(a.epi.bias + int64_t(e) * a.n + row);
            if (SWIGLU) out[NW - 1] += __ldg(a.epi.bias2 + int64_t(e) * a.n + row);
          }
          const float v = SWIGLU ? act_apply(a.epi.act, out[0], out[NW - 1], a.epi.alpha, a.epi.limit) : out[0];
          float* yp = a.y + int64_t(s_order[first + tok]) * a.n + row;
          *yp = a.accumulate ? *yp + v : v;
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kRowsCons * 32) : "memory");   // red and the x tiles are rewritten next
  }
}

template <int FMT, int XT, bool SWIGLU>
static int launch_mv_grp(const CUtensorMap& wm, const CUtensorMap& w2m, const MvArgs& a, cudaStream_t s) {
  constexpr int NW = SWIGLU ? 2 : 1, NST = rows_stages<SWIGLU>();
  constexpr int kXT = (XT == LK_F32 ? 2 : 1) * kGrpTok * kXStride;
  const int kchunks = a.k / kChunkValues;
  const int smem = NST * NW * kRowsCons * kMvChunkTile + 2 * NST * 8 + kRowsCons * NW * 16 * kAcStride * 8 +
                   kRowsCons * NW * 32 * 4 * 4 + kchunks * kGrpTok * 8 * 4 + kchunks * kXT * 2;
  if (smem > 200 * 1024 || a.n_experts > 256 || a.tokens > kGrpMaxA) return LK_EUNSUPPORTED;
  auto kern = k_mv_grp<FMT, XT, SWIGLU>;
  static int configured[32] = {};
  static std::mutex mu;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  if (dev >= 32) return LK_EUNSUPPORTED;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (configured[dev] < smem) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return LK_ECUDA;
      configured[dev] = smem;
    }
  }
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (kRowsCons + 1) * 32, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  // at most min(A, E + A / 8) groups
  const int max_items = min(a.tokens, a.n_experts + a.tokens / kGrpTok) * ((a.n + kMvRows - 1) / kMvRows);
  kern<<<min(max_items, per_sm * sms), (kRowsCons + 1) * 32, smem, s>>>(wm, w2m, a);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

template <int FMT, int XT>
static int mv_x(const CUtensorMap& wm, const CUtensorMap& w2m, const MvArgs& a, int groups, cudaStream_t s) {
  if (!a.ids && a.tokens == 1) {   // the decode step's shape: the persistent form where its shared memory fits
    const int rc = a.swiglu ? launch_mv_rows<FMT, XT, true, false>(wm, w2m, a, s)
                            : launch_mv_rows<FMT, XT, false, false>(wm, w2m, a, s);
    if (rc != LK_EUNSUPPORTED) return rc;
  }
  if (a.ids && a.swiglu && a.x_div == a.tokens) {   // the gate/up expert matvecs of one token: all read x row 0
    const int rc = launch_mv_rows<FMT, XT, true, true>(wm, w2m, a, s);
    if (rc != LK_EUNSUPPORTED) return rc;
  }
  if (a.ids && a.x_div < a.tokens && a.tokens >= kGrpMinA && a.tokens <= kGrpMaxA) {   // several tokens: by expert
    const int rc = a.swiglu ? launch_mv_grp<FMT, XT, true>(wm, w2m, a, s) : launch_mv_grp<FMT, XT, false>(wm, w2m, a, s);
    if (rc != LK_EUNSUPPORTED) return rc;
  }
  if (a.ids && a.swiglu && a.tokens <= 256) {   // gate/up of a few tokens: row a / ku of x
    const int rc = launch_mv_rows<FMT, XT, true, true, true>(wm, w2m, a, s);
    if (rc != LK_EUNSUPPORTED) return rc;
  }
  if (a.ids && !a.swiglu && a.x_div == 1 && a.tokens <= 256) {   // the down matvecs at decode sizes: row a of x
    const int rc = launch_mv_rows<FMT, XT, false, true, true>(wm, w2m, a, s);
    if (rc != LK_EUNSUPPORTED) return rc;
  }
  if (a.ids) {
    if (a.swiglu) return launch_mv<FMT, XT, true, true, 1>(wm, w2m, a, groups, s);
    return launch_mv<FMT, XT, false, true, 1>(wm, w2m, a, groups, s);
  }
  if (a.tokens == 1) {
    if (a.swiglu) return launch_mv<FMT, XT, true, false, 1>(wm, w2m, a, groups, s);
    return launch_mv<FMT, XT, false, false, 1>(wm, w2m, a, groups, s);
  }
  if (a.swiglu) return launch_mv<FMT, XT, true, false, 8>(wm, w2m, a, groups, s);
  return launch_mv<FMT, XT, false, false, 8>(wm, w2m, a, groups, s);
}

template <int FMT>
static int mv_f(const CUtensorMap& wm, const CUtensorMap& w2m, const MvArgs& a, int groups, cudaStream_t s) {
  switch (a.x_dtype) {
    case LK_F16: return mv_x<FMT, LK_F16>(wm, w2m, a, groups, s);
    case LK_BF16: return mv_x<FMT, LK_BF16>(wm, w2m, a, groups, s);
    case LK_F32: return mv_x<FMT, LK_F32>(wm, w2m, a, groups, s);
  }
  return LK_EINVAL;
}

template <int FMT>
static int routed_f(const CUtensorMap& wm, const CUtensorMap& w2m, const MvArgs& a, cudaStream_t s) {
  switch (a.x_dtype) {
    case LK_F16: return launch_mv_rows<FMT, LK_F16, true, true, false, true>(wm, w2m, a, s);
    case LK_BF16: return launch_mv_rows<FMT, LK_BF16, true, true, false, true>(wm, w2m, a, s);
    case LK_F32: return launch_mv_rows<FMT, LK_F32, true, true, false, true>(wm, w2m, a, s);
  }
  return LK_EINVAL;
}

int mv_routed(int fmt, const MvArgs& a, cudaStream_t s) {
  CUtensorMap wm, w2m;
  int rc = make_map(&wm, a.w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, int64_t(a.n_experts) * a.rows_per_expert,
                    a.row_bytes / 4, kChunkBytes / 4, kMvRows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc == LK_OK)
    rc = make_map(&w2m, a.w2, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, int64_t(a.n_experts) * a.rows_per_expert2,
                  a.row_bytes / 4, kChunkBytes / 4, kMvRows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != LK_OK) return rc;
  switch (fmt) {
    case LK_Q4_0: return routed_f<LK_Q4_0>(wm, w2m, a, s);
    case LK_Q4_K: return routed_f<LK_Q4_K>(wm, w2m, a, s);
    case LK_IQ4_NL: return routed_f<LK_IQ4_NL>(wm, w2m, a, s);
  }
  return LK_EUNSUPPORTED;
}

int mv(int fmt, const MvArgs& a, int groups, cudaStream_t s) {
  // weight maps: the packed rows as u32 columns, 16 rows x 576 bytes per box; MoE experts stacked as rows
  int64_t rows = a.ids ? int64_t(a.n_experts) * a.rows_per_expert : a.n;
  int64_t rows2 = a.ids ? int64_t(a.n_experts) * a.rows_per_expert2 : a.n;
  CUtensorMap wm, w2m;
  int rc = make_map(&wm, a.w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, rows, a.row_bytes / 4, kChunkBytes / 4, kMvRows,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc == LK_OK)
    rc = a.w2 ? make_map(&w2m, a.w2, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, rows2, a.row_bytes / 4, kChunkBytes / 4,
                         kMvRows, CU_TENSOR_MAP_SWIZZLE_NONE)
              : (w2m = wm, LK_OK);
  if (rc != LK_OK) return rc;
  switch (fmt) {
    case LK_Q4_0: return mv_f<LK_Q4_0>(wm, w2m, a, groups, s);
    case LK_Q4_K: return mv_f<LK_Q4_K>(wm, w2m, a, groups, s);
    case LK_IQ4_NL: return mv_f<LK_IQ4_NL>(wm, w2m, a, groups, s);
  }
  return LK_EUNSUPPORTED;
}

LK_STATUS_READER(status_mv)

}  // namespace lk
