// Decode matvec for GGUF block weights (tokens < 64): y[t][n] (+)= sum_k x[t][k] W[n][k].
//
// Replaces g_mv_{fmt}_k{K}[_t{TG}][_r{R}] and its swiglu pair (gen_llm.py:1159-1378) and the MoE expert matvecs
// g_moe_gu_/g_moe_dn_ (gen_moe.py:535-727).
//
// Design (HBM-bound): a CTA owns 16 weight rows and up to 8 tokens. A producer warp streams the rows' packed bytes
// into a shared-memory ring with 1-D bulk copies (TMA), 576 contiguous bytes per row per stage; four consumer warps
// each take one 256-value chunk of every stage. A consumer unpacks nibbles in registers straight into the A fragments
// of warp-level f16 MMAs (16 rows x 16 k x 8 tokens): the weights never go back to shared memory, so the only shared
// memory traffic is the bulk copy in and one read. Codes enter the MMA exactly as (1024 + code) f16 values; the
// per-32-value group scale is applied in f32 afterwards:
//     sum_k (a*q_k - c) x_k = a * D - (1024 a + c) * S,   D = sum (1024 + q_k) x_k,  S = sum x_k
// with S from a second MMA against a ones operand. Q4_0: a = d, c = 8d; IQ4_NL: codes are the biased codebook bytes
// (kvalue + 128), a = d, offset 1152 a; Q4_K: a = d*sc, c = dmin*m per group. The f32 accumulation of exact codes
// is more precise than the reference's f32 per-value dequant-then-dot (gen_llm.py:1281-1357).
#include "lk_common.cuh"
#include "lk_internal.h"

namespace lk {

constexpr int kMvConsumers = 4;
constexpr int kMvThreads = (kMvConsumers + 1) * 32;
constexpr int kMvRows = 16;
constexpr int kMvStageChunks = 4;                   // 256-value chunks per stage (one per consumer warp)
constexpr int kMvStages = 4;
constexpr int kMvRowStageBytes = kMvStageChunks * kChunkBytes;   // 576

LK_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

LK_DEV uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// B fragment of 4 consecutive activations x[kk .. kk+3] of one token (f16 MMA operand); f32 inputs split hi + lo
template <int XT>
struct BFrag {
  uint32_t b0, b1, l0, l1;
  LK_DEV void load(const void* xrow, int kk, bool valid) {
    b0 = b1 = l0 = l1 = 0;
    if (!valid) return;
    if (XT == LK_F16) {
      uint2 v = __ldg(reinterpret_cast<const uint2*>(static_cast<const __half*>(xrow) + kk));
      b0 = v.x;
      b1 = v.y;
    } else if (XT == LK_BF16) {
      uint2 v = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(xrow) + kk));
      b0 = h2u(__floats2half2_rn(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u)));
      b1 = h2u(__floats2half2_rn(__uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u)));
    } else {
      float4 v = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(xrow) + kk));
      __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
      b0 = h2u(h0);
      b1 = h2u(h1);
      float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
      l0 = h2u(__floats2half2_rn(v.x - f0.x, v.y - f0.y));
      l1 = h2u(__floats2half2_rn(v.z - f1.x, v.w - f1.y));
    }
  }
};

// D += A(code word pair) * B, for both hi and lo parts of an f32 activation
template <int XT>
LK_DEV void mma_codes(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, const BFrag<XT>& b) {
  mma16816(d, a0, a1, a2, a3, b.b0, b.b1);
  if (XT == LK_F32) mma16816(d, a0, a1, a2, a3, b.l0, b.l1);
}

constexpr uint32_t kOnes = 0x3C003C00u;   // f16x2 (1, 1)

// nibble codes (bits 0-3 of each byte) -> the A fragment halves (1024 + code) for 4 consecutive k
LK_DEV void code_frag(uint32_t t, uint32_t& first, uint32_t& second) {
  first = prmt(t, 0x64646464u, 0x4140u);
  second = prmt(t, 0x64646464u, 0x4342u);
}

template <int FMT>
LK_DEV uint32_t nib_bytes(uint32_t w, bool hi) {
  uint32_t t = (hi ? (w >> 4) : w) & 0x0F0F0F0Fu;
  if (FMT == LK_IQ4_NL) t = iq4_lookup4(t);
  return t;
}

LK_DEV uint32_t lds_u16x2(const uint8_t* p) {   // 2-byte aligned 4 bytes
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
  return uint32_t(q[0]) | (uint32_t(q[1]) << 16);
}

struct Acc {
  float v[4];
};

LK_DEV void group_epilogue(Acc& acc, const float (&d)[4], const float (&s)[4], float a_g, float c_g, float a_g8,
                           float c_g8) {
  acc.v[0] = fmaf(a_g, d[0], fmaf(-c_g, s[0], acc.v[0]));
  acc.v[1] = fmaf(a_g, d[1], fmaf(-c_g, s[1], acc.v[1]));
  acc.v[2] = fmaf(a_g8, d[2], fmaf(-c_g8, s[2], acc.v[2]));
  acc.v[3] = fmaf(a_g8, d[3], fmaf(-c_g8, s[3], acc.v[3]));
}

// One 256-value chunk of 16 rows (rows at `rb + r * rstride`) against the B operand at k0.
template <int FMT, int XT, int NW>
LK_DEV void mv_chunk(const uint8_t* rb0, const uint8_t* rb1, int rstride, const void* xrow, bool xvalid, int k0,
                     int g, int tig, int lane, float2* actab, Acc (&acc)[NW]) {
  if (FMT == LK_Q4_K) {
    // cooperative header decode: lane -> (row lane/2, groups 4*(lane&1) .. +3); (a, c') per row and group
#pragma unroll
    for (int wi = 0; wi < NW; ++wi) {
      const uint8_t* rb = wi ? rb1 : rb0;
      int r = lane >> 1, j0 = (lane & 1) * 4;
      uint4 hv = *reinterpret_cast<const uint4*>(rb + r * rstride);
      const uint8_t* hb = reinterpret_cast<const uint8_t*>(&hv);
      float d = h2f(uint16_t(hv.x & 0xffff)), dmin = h2f(uint16_t(hv.x >> 16));
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        int sc, m;
        q4k_scale_min(hb + 4, j0 + jj, sc, m);
        float a = d * float(sc);
        actab[wi * 128 + r * 8 + j0 + jj] = make_float2(a, fmaf(1024.0f, a, dmin * float(m)));
      }
    }
    __syncwarp();
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float dl[NW][4], dh[NW][4], sl[4], sh[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sl[i] = sh[i] = 0.f;
#pragma unroll
        for (int wi = 0; wi < NW; ++wi) dl[wi][i] = dh[wi][i] = 0.f;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        BFrag<XT> bl, bh;
        int kk = k0 + 64 * p + 16 * h + 4 * tig;
        bl.load(xrow, kk, xvalid);
        bh.load(xrow, kk + 32, xvalid);
        mma_codes<XT>(sl, kOnes, kOnes, kOnes, kOnes, bl);
        mma_codes<XT>(sh, kOnes, kOnes, kOnes, kOnes, bh);
#pragma unroll
        for (int wi = 0; wi < NW; ++wi) {
          const uint8_t* rb = wi ? rb1 : rb0;
          int off = 16 + 32 * p + 16 * h + 4 * tig;
          uint32_t w0 = *reinterpret_cast<const uint32_t*>(rb + g * rstride + off);
          uint32_t w8 = *reinterpret_cast<const uint32_t*>(rb + (g + 8) * rstride + off);
          uint32_t f0, s0, f8, s8;
          code_frag(nib_bytes<FMT>(w0, false), f0, s0);
          code_frag(nib_bytes<FMT>(w8, false), f8, s8);
          mma_codes<XT>(dl[wi], f0, f8, s0, s8, bl);
          code_frag(nib_bytes<FMT>(w0, true), f0, s0);
          code_frag(nib_bytes<FMT>(w8, true), f8, s8);
          mma_codes<XT>(dh[wi], f0, f8, s0, s8, bh);
        }
      }
#pragma unroll
      for (int wi = 0; wi < NW; ++wi) {
        float2 lo0 = actab[wi * 128 + g * 8 + 2 * p], lo8 = actab[wi * 128 + (g + 8) * 8 + 2 * p];
        float2 hi0 = actab[wi * 128 + g * 8 + 2 * p + 1], hi8 = actab[wi * 128 + (g + 8) * 8 + 2 * p + 1];
        group_epilogue(acc[wi], dl[wi], sl, lo0.x, lo0.y, lo8.x, lo8.y);
        group_epilogue(acc[wi], dh[wi], sh, hi0.x, hi0.y, hi8.x, hi8.y);
      }
    }
    __syncwarp();   // the table is rewritten by the next chunk
  } else {
    constexpr float kOff = FMT == LK_Q4_0 ? 1032.0f : 1152.0f;   // magic 1024 + (8 | 128 codebook bias)
#pragma unroll 2
    for (int j = 0; j < 8; ++j) {
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      float dd[NW][4];
      BFrag<XT> b0, b1;
      int kk = k0 + 32 * j + 4 * tig;
      b0.load(xrow, kk, xvalid);
      b1.load(xrow, kk + 16, xvalid);
      mma_codes<XT>(s, kOnes, kOnes, kOnes, kOnes, b0);
      mma_codes<XT>(s, kOnes, kOnes, kOnes, kOnes, b1);
#pragma unroll
      for (int wi = 0; wi < NW; ++wi) {
        const uint8_t* rb = (wi ? rb1 : rb0) + 18 * j;
        const uint8_t* p0 = rb + g * rstride;
        const uint8_t* p8 = rb + (g + 8) * rstride;
        float d0 = h2f(*reinterpret_cast<const uint16_t*>(p0));
        float d8 = h2f(*reinterpret_cast<const uint16_t*>(p8));
        uint32_t w0 = lds_u16x2(p0 + 2 + 4 * tig), w8 = lds_u16x2(p8 + 2 + 4 * tig);
#pragma unroll
        for (int i = 0; i < 4; ++i) dd[wi][i] = 0.f;
        uint32_t f0, s0, f8, s8;
        code_frag(nib_bytes<FMT>(w0, false), f0, s0);
        code_frag(nib_bytes<FMT>(w8, false), f8, s8);
        mma_codes<XT>(dd[wi], f0, f8, s0, s8, b0);
        code_frag(nib_bytes<FMT>(w0, true), f0, s0);
        code_frag(nib_bytes<FMT>(w8, true), f8, s8);
        mma_codes<XT>(dd[wi], f0, f8, s0, s8, b1);
        group_epilogue(acc[wi], dd[wi], s, d0, kOff * d0, d8, kOff * d8);
      }
    }
  }
}

template <int FMT, int XT, bool SWIGLU, bool MOE>
__global__ void __launch_bounds__(kMvThreads) k_mv(MvArgs a) {
  constexpr int NW = SWIGLU ? 2 : 1;
  constexpr int kStageBytes = NW * kMvRows * kMvRowStageBytes;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kMvStages * kStageBytes);
  uint64_t* empty = full + kMvStages;
  float2* actab_all = reinterpret_cast<float2*>(empty + kMvStages);   // [consumers][NW][16][8]
  float* red = reinterpret_cast<float*>(actab_all + kMvConsumers * NW * 128);   // [consumers][NW][32][4]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * kMvRows;
  const int nrows = min(kMvRows, a.n - r0);
  const uint8_t* wb = a.w;
  const uint8_t* w2b = a.w2;
  int xrow0, ntok, yrow0;
  if (MOE) {
    int asg = blockIdx.y;
    int e = min(max(a.ids[asg], 0), a.n_experts - 1);
    wb = a.w + int64_t(e) * a.expert_stride;
    if (SWIGLU) w2b = a.w2 ? a.w2 + int64_t(e) * a.expert_stride : wb + a.w2_offset;
    xrow0 = asg / a.x_div;
    ntok = 1;
    yrow0 = asg;
  } else {
    xrow0 = blockIdx.y * 8;
    ntok = min(8, a.tokens - xrow0);
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
    // producer: stage st holds chunks [st*4, st*4+4) of every row
    for (int st = 0; st < nstages; ++st) {
      int s = st % kMvStages;
      if (st >= kMvStages) {
        if (!mbar_wait(&empty[s], ((st / kMvStages) - 1) & 1)) atomicOr(&g_status, 1u);
      }
      int c0 = st * kMvStageChunks;
      int nch = min(kMvStageChunks, kchunks - c0);
      uint32_t bytes = uint32_t(nch) * kChunkBytes;
      if (lane == 0) mbar_expect_tx(&full[s], bytes * nrows * NW);
      __syncwarp();
      if (lane < NW * kMvRows) {
        int wi = lane / kMvRows, r = lane % kMvRows;
        if (r < nrows) {
          const uint8_t* src = (wi ? w2b : wb) + int64_t(r0 + r) * a.row_bytes + int64_t(c0) * kChunkBytes;
          uint8_t* dst = ring + s * kStageBytes + wi * kMvRows * kMvRowStageBytes + r * kMvRowStageBytes;
          bulk_g2s(dst, src, bytes, &full[s]);
        }
      }
    }
    return;
  }

  // consumers
  const int g = lane >> 2, tig = lane & 3;
  Acc acc[NW];
#pragma unroll
  for (int wi = 0; wi < NW; ++wi)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[wi].v[i] = 0.f;
  const bool xvalid = g < ntok;
  const void* xrow = static_cast<const uint8_t*>(a.x) +
                     (int64_t(xrow0) + (xvalid ? g : 0)) * a.k * (a.x_dtype == LK_F32 ? 4 : 2);
  float2* actab = actab_all + warp * NW * 128;
  for (int st = 0; st < nstages; ++st) {
    int s = st % kMvStages;
    if (!mbar_wait(&full[s], (st / kMvStages) & 1)) atomicOr(&g_status, 1u);
    int c = st * kMvStageChunks + warp;
    if (c < kchunks) {
      const uint8_t* rb0 = ring + s * kStageBytes + warp * kChunkBytes;
      const uint8_t* rb1 = rb0 + kMvRows * kMvRowStageBytes;
      mv_chunk<FMT, XT, NW>(rb0, rb1, kMvRowStageBytes, xrow, xvalid, c * kChunkValues, g, tig, lane, actab, acc);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // reduce the consumers' partial sums; warp 0 stores
#pragma unroll
  for (int wi = 0; wi < NW; ++wi)
    *reinterpret_cast<float4*>(red + ((warp * NW + wi) * 32 + lane) * 4) =
        make_float4(acc[wi].v[0], acc[wi].v[1], acc[wi].v[2], acc[wi].v[3]);
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
    float v = SWIGLU ? silu(out[0][i]) * out[NW - 1][i] : out[0][i];
    float* yp = a.y + int64_t(yrow0 + tok) * a.n + row;
    *yp = a.accumulate ? *yp + v : v;
  }
}

template <int FMT, int XT, bool SWIGLU, bool MOE>
static int launch_mv(const MvArgs& a, int groups, cudaStream_t s) {
  constexpr int NW = SWIGLU ? 2 : 1;
  constexpr int kStageBytes = NW * kMvRows * kMvRowStageBytes;
  constexpr int smem = kMvStages * kStageBytes + 2 * kMvStages * 8 + kMvConsumers * NW * 128 * 8 +
                       kMvConsumers * NW * 32 * 4 * 4;
  auto kern = k_mv<FMT, XT, SWIGLU, MOE>;
  static unsigned configured = 0;   // one bit per device
  if (!once_per_device(configured)) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((a.n + kMvRows - 1) / kMvRows, groups);
  kern<<<grid, kMvThreads, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

template <int FMT, int XT>
static int mv_x(const MvArgs& a, int groups, cudaStream_t s) {
  bool moe = a.ids != nullptr;
  if (a.swiglu) return moe ? launch_mv<FMT, XT, true, true>(a, groups, s) : launch_mv<FMT, XT, true, false>(a, groups, s);
  return moe ? launch_mv<FMT, XT, false, true>(a, groups, s) : launch_mv<FMT, XT, false, false>(a, groups, s);
}

template <int FMT>
static int mv_f(const MvArgs& a, int groups, cudaStream_t s) {
  switch (a.x_dtype) {
    case LK_F16: return mv_x<FMT, LK_F16>(a, groups, s);
    case LK_BF16: return mv_x<FMT, LK_BF16>(a, groups, s);
    case LK_F32: return mv_x<FMT, LK_F32>(a, groups, s);
  }
  return LK_EINVAL;
}

int mv(int fmt, const MvArgs& a, int groups, cudaStream_t s) {
  switch (fmt) {
    case LK_Q4_0: return mv_f<LK_Q4_0>(a, groups, s);
    case LK_Q4_K: return mv_f<LK_Q4_K>(a, groups, s);
    case LK_IQ4_NL: return mv_f<LK_IQ4_NL>(a, groups, s);
  }
  return LK_EUNSUPPORTED;
}

LK_STATUS_READER(status_mv)

}  // namespace lk
