// Decode matvec on int8 activations for the formats with integer weight codes beyond the Q4 pair: the reference's
// ICODES set (formats.py:22-31: Q8_0, Q5_0, Q5_K, Q6_K by default; IQ4_NL and IQ4_XS under its IQ4_Q8 choice), each
// format's @g_<fmt>_icodes helper (gen_llm.py:521-680, 898-1000) with the dot of iq_dot (gen_llm.py:1017-1050):
//
//   per 32-value group, the weight codes (int8) . the activation codes (lk_quant_q8's) as an exact integer dot, then
//     ONE_SCALE (Q8_0, IQ4_NL, IQ4_XS)   (scale * d_x) * dot
//     with a minimum (Q5_0, Q5_K)        (dot * scale - sum_x * minimum) * d_x
//     Q6_K (a scale per 16 values)        fma(dot_hi, scale_hi, dot_lo * scale_lo) * d_x
//
// k_mvq8g: a producer warp streams stages of (8 rows) x (a chunk of 2048 values) into a 4-slot shared-memory ring --
// one bulk copy per row of the 16-byte-aligned window around the row's chunk bytes, since these blocks (34, 22, 176,
// 210, 18, 136 bytes) start at any even offset -- and 8 consumer warps take one row each: lane l decodes the groups
// l, l + 32, ... of the chunk from shared memory (aligned word loads realigned by funnel shifts), reads the activation codes of up to 8 tokens from
// global memory (the whole row of codes is shared by every warp: it stays in L1), and runs 8 dp4a per group and token.
// A CTA walks whole row blocks (all chunks of 8 rows) so each row's sum stays in registers; the first stage is
// requested before griddepcontrol.wait (the weights never depend on the previous kernel).
#include <mutex>

#include "lk_common.cuh"
#include "lk_formats.cuh"
#include "lk_internal.h"

namespace lk {
namespace {

constexpr int kGRows = 8;                    // rows per stage = consumer warps
constexpr int kGThreads = 32 * (1 + kGRows);
constexpr int kGStages = 4;
constexpr int kGChunk = 2048;                // values of a row per stage

LK_DEV void gq_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LK_DEV void gq_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

LK_DEV float f16_2a(const uint8_t* p) { return h2f(*reinterpret_cast<const uint16_t*>(p)); }
// N little-endian words from a 2-byte aligned shared-memory address: N + 1 explicit shared loads of the aligned words
// around them and funnel shifts (the load past the end stays inside the CTA's shared memory: every row window has
// slack behind it, then the barriers)
template <int N>
LK_DEV void ldw(const uint8_t* p, uint32_t (&w)[N]) {
  const uint32_t a = smem_u32(p), base = a & ~3u, sh = (a & 3u) * 8u;
  uint32_t v[N + 1];
#pragma unroll
  for (int i = 0; i <= N; ++i) asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v[i]) : "r"(base + 4u * i));
#pragma unroll
  for (int i = 0; i < N; ++i) w[i] = __funnelshift_r(v[i], v[i + 1], sh);
}

// The int8 codes of one 32-value group (word i = values 4i..4i+3, one per byte) and its factors: sc the scale, mn
// the minimum (Q5_0, Q5_K) or the second 16 values' scale (Q6_K)
struct ICodes {
  uint32_t w[8];
  float sc, mn;
};

enum { kOneScale = 0, kMinimum = 1, kTwoScales = 2 };
__host__ __device__ constexpr int icode_kind(int fmt) {
  return fmt == LK_Q6_K ? kTwoScales
         : (fmt == LK_Q5_0 || fmt == LK_Q5_K || fmt == LK_Q4_0 || fmt == LK_Q4_K) ? kMinimum
                                                                                   : kOneScale;
}

// group j of the block at b (@g_<fmt>_icodes)
template <int FMT>
LK_DEV void group_icodes(const uint8_t* b, int j, ICodes& o) {
  if (FMT == LK_Q4_0) {   // gen_llm.py:536-552: nibbles 0..15, minimum 8 d
    const float d = f16_2a(b);
    uint32_t q[4];
    ldw(b + 2, q);
#pragma unroll
    for (int i = 0; i < 8; ++i) o.w[i] = (i < 4 ? q[i] : q[i - 4] >> 4) & 0x0F0F0F0Fu;
    o.sc = d;
    o.mn = 8.0f * d;
  } else if (FMT == LK_Q4_K) {   // gen_llm.py:554-577: the nibble page of group j, scale d sc, minimum dmin m
    uint32_t sc, m, hd[4], qs[8];
    ldw(b, hd);
    q4k_scale_min_w(hd[1], hd[2], hd[3], j, sc, m);
    o.sc = h2f(uint16_t(hd[0] & 0xffffu)) * float(sc);
    o.mn = h2f(uint16_t(hd[0] >> 16)) * float(m);
    ldw(b + 16 + 32 * (j >> 1), qs);
#pragma unroll
    for (int i = 0; i < 8; ++i) o.w[i] = (qs[i] >> (4 * (j & 1))) & 0x0F0F0F0Fu;
  } else if (FMT == LK_Q8_0) {   // gen_llm.py:523-534: int8 codes, scale d
    o.sc = f16_2a(b);
    ldw(b + 2, o.w);
    o.mn = 0.f;
  } else if (FMT == LK_Q5_0) {   // gen_llm.py:943-985: nibble | bit i of qh << 4 (0..31), minimum 16 d
    const float d = f16_2a(b);
    uint32_t hq[5];   // qh, then the 16 nibble bytes
    ldw(b + 2, hq);
    const uint32_t qh = hq[0];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t q = hq[1 + (i & 3)];
      const uint32_t hb = (qh >> (4 * i)) & 15u;
      o.w[i] = ((i < 4 ? q : q >> 4) & 0x0F0F0F0Fu) |
               ((hb & 1u) << 4) | ((hb & 2u) << 11) | ((hb & 4u) << 18) | ((hb & 8u) << 25);
    }
    o.sc = d;
    o.mn = 16.0f * d;
  } else if (FMT == LK_Q5_K) {   // gen_llm.py:579-615: Q4_K's nibbles | bit j of qh[l] << 4, scale d sc, minimum dmin m
    uint32_t sc, m, hd[4], qh[8], qs[8];
    ldw(b, hd);
    q4k_scale_min_w(hd[1], hd[2], hd[3], j, sc, m);
    o.sc = h2f(uint16_t(hd[0] & 0xffffu)) * float(sc);
    o.mn = h2f(uint16_t(hd[0] >> 16)) * float(m);
    ldw(b + 16, qh);
    ldw(b + 48 + 32 * (j >> 1), qs);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      o.w[i] = ((qs[i] >> (4 * (j & 1))) & 0x0F0F0F0Fu) | (((qh[i] >> j) & 0x01010101u) << 4);
  } else if (FMT == LK_Q6_K) {   // gen_llm.py:617-680: signed (q - 32), d sc of each 16 values
    const int half = j >> 2, jj = j & 3;
    const uint8_t* ql = b + 64 * half + 32 * (jj & 1);
    const uint8_t* qh = b + 128 + 32 * half;
    const uint8_t* sc = b + 192 + 8 * half + 2 * jj;
    const float d = f16_2a(b + 208);
    uint32_t wl[8], wh[8];
    ldw(ql, wl);
    ldw(qh, wh);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t c = ((wl[i] >> (4 * (jj >> 1))) & 0x0F0F0F0Fu) |
                         (((wh[i] >> (2 * jj)) & 0x03030303u) << 4);   // 0..63 per byte
      // c - 32 per byte: flip bit 5; bytes below 32 also get bits 6 and 7 (their two's complement)
      o.w[i] = (c ^ 0x20202020u) | ((~c & 0x20202020u) * 7u);
    }
    o.sc = float(int8_t(sc[0])) * d;
    o.mn = float(int8_t(sc[1])) * d;
  } else if (FMT == LK_IQ4_NL || FMT == LK_IQ4_XS) {   // gen_llm.py:898-940: codebook values, one scale
    const uint8_t* qs;
    if (FMT == LK_IQ4_NL) {
      o.sc = f16_2a(b);
      qs = b + 2;
    } else {
      const int sh = *reinterpret_cast<const uint16_t*>(b + 2);
      const int ls = ((b[4 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((sh >> (2 * j)) & 3) << 4);
      o.sc = f16_2a(b) * float(ls - 32);
      qs = b + 8 + 16 * j;
    }
    uint32_t q[4];
    ldw(qs, q);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      o.w[i] = iq4_lookup4((i < 4 ? q[i] : q[i - 4] >> 4) & 0x0F0F0F0Fu) ^ 0x80808080u;   // biased bytes -> int8
    o.mn = 0.f;
  }
}

// the group's contribution for one token: x codes xw[8], the activation group's f16-rounded d and code sum
template <int FMT>
LK_DEV float group_dot(const ICodes& c, const uint32_t (&xw)[8], float dx, float xsum) {
  if (icode_kind(FMT) == kTwoScales) {
    int lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lo = __dp4a(int(c.w[i]), int(xw[i]), lo);
      hi = __dp4a(int(c.w[4 + i]), int(xw[4 + i]), hi);
    }
    return fmaf(__int2float_rn(hi), c.mn, __int2float_rn(lo) * c.sc) * dx;
  }
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) s = __dp4a(int(c.w[i]), int(xw[i]), s);
  if (icode_kind(FMT) == kOneScale) return (c.sc * dx) * __int2float_rn(s);
  return (__int2float_rn(s) * c.sc - xsum * c.mn) * dx;
}

struct GqArgs {
  const uint8_t* w;
  const uint8_t* codes;   // [tokens][k] int8
  const float* meta;      // [tokens][k/32][2]
  float* y;
  int n, k, ntok, accumulate;
  int64_t rb;             // packed bytes of a row
  int cb;                 // packed bytes of a full chunk (kGChunk values)
  int nkc;                // chunks per row
  int row_slot;           // shared-memory bytes of one row's window
  // per MoE assignment a (kGMoeDn / kGMoeGu): expert ids[a], activation row a / x_div, output row a; the second
  // weight's rows (gate/up) at e * rows_per_expert2 + w2_row_offset of w2
  const int32_t* ids;
  const uint8_t* w2;
  int assignments, x_div, n_experts, rows_per_expert, rows_per_expert2, w2_row_offset;
  int act;
  float alpha, limit;
};

enum { kGDense = 0, kGMoeDn = 1, kGMoeGu = 2 };

template <int FMT, int NT, int MODE>
__global__ void __launch_bounds__(kGThreads, 4) k_mvq8g(const GqArgs a) {
  constexpr int gpb = fmt_qk(FMT) / 32;   // 32-value groups per block
  constexpr int bb = fmt_block_bytes(FMT);
  constexpr int NW = MODE == kGMoeGu ? 2 : 1;   // weights per row block (gate and up)
  static_assert(MODE == kGDense || NT == 1, "one activation row per MoE assignment");
  extern __shared__ __align__(128) uint8_t smem[];
  const int slot = NW * kGRows * a.row_slot;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGStages * slot);
  uint64_t* empty = full + kGStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, G = gridDim.x;
  const int nrb = (a.n + kGRows - 1) / kGRows;   // row blocks of one output row
  const int nblk = MODE == kGDense ? nrb : a.assignments * nrb;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGRows);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // output row r (of n) of row block blk in weight wi: its packed chunk kc's source and length
  auto src_of = [&](int blk, int r, int wi, int kc, uintptr_t& src, uint32_t& len) {
    const int64_t c0 = int64_t(kc) * a.cb;
    len = uint32_t(min(int64_t(a.cb), a.rb - c0));
    int64_t wr = r;
    if (MODE != kGDense) {
      const int e = min(max(__ldg(a.ids + blk / nrb), 0), a.n_experts - 1);
      wr = wi ? int64_t(e) * a.rows_per_expert2 + a.w2_row_offset + r : int64_t(e) * a.rows_per_expert + r;
    }
    src = reinterpret_cast<uintptr_t>((wi ? a.w2 : a.w) + wr * a.rb + c0);
  };
  if (warp == 0) {
    gq_launch();
    if (MODE != kGDense) gq_wait();   // the expert ids come from the previous kernel
    int i = 0;
    for (int blk = cta; blk < nblk; blk += G) {
      for (int kc = 0; kc < a.nkc; ++kc, ++i) {
        if (i == 1) gq_wait();   // the first stage goes out before the previous grid ends
        const int s = i % kGStages;
        if (i >= kGStages && !mbar_wait(&empty[s], ((i / kGStages) - 1) & 1)) atomicOr(&g_status, 1u);
        const int r = (blk % nrb) * kGRows + (lane % kGRows);   // lanes 0-7 the first weight's rows, 8-15 the second's
        uintptr_t src = 0;
        uint32_t len = 0, bytes = 0;
        if (lane < NW * kGRows && r < a.n) {
          src_of(blk, r, lane / kGRows, kc, src, len);
          bytes = uint32_t(((src + len + 15) & ~uintptr_t(15)) - (src & ~uintptr_t(15)));
        }
        uint32_t total = bytes;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xFFFFFFFFu, total, o);
        if (lane == 0) mbar_expect_tx(&full[s], total);
        __syncwarp();
        if (bytes)
          bulk_g2s(smem + s * slot + lane * a.row_slot, reinterpret_cast<const void*>(src & ~uintptr_t(15)), bytes,
                   &full[s]);
        __syncwarp();
      }
    }
    return;
  }
  gq_wait();   // the activation codes come from the previous kernel
  const int cw = warp - 1, groups = a.k / 32;
  int i = 0;
  for (int blk = cta; blk < nblk; blk += G) {
    const int r = (blk % nrb) * kGRows + cw;
    const int xrow = MODE == kGDense ? 0 : (blk / nrb) / a.x_div;   // the assignment's activation row
    float acc[NW][NT];
#pragma unroll
    for (int wi = 0; wi < NW; ++wi)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[wi][t] = 0.f;
    for (int kc = 0; kc < a.nkc; ++kc, ++i) {
      const int s = i % kGStages;
      if (!mbar_wait(&full[s], (i / kGStages) & 1)) atomicOr(&g_status, 1u);
      if (r < a.n) {
        const int gc = min(kGChunk, a.k - kc * kGChunk) / 32, g0 = kc * (kGChunk / 32);
#pragma unroll
        for (int wi = 0; wi < NW; ++wi) {
          uintptr_t src;
          uint32_t len;
          src_of(blk, r, wi, kc, src, len);
          const uint8_t* chunk = smem + s * slot + (wi * kGRows + cw) * a.row_slot + (src & 15);
          for (int g = lane; g < gc; g += 32) {
            ICodes c;
            group_icodes<FMT>(chunk + (g / gpb) * bb, g % gpb, c);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              if (t >= a.ntok) break;
              const int64_t xr = MODE == kGDense ? t : xrow;
              const uint4* xp = reinterpret_cast<const uint4*>(a.codes + xr * a.k + int64_t(g0 + g) * 32);
              const uint4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
              const float2 m = __ldg(reinterpret_cast<const float2*>(a.meta) + xr * groups + g0 + g);
              const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
              acc[wi][t] += group_dot<FMT>(c, xw, m.x, m.y);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int wi = 0; wi < NW; ++wi)
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[wi][t] += __shfl_xor_sync(0xFFFFFFFFu, acc[wi][t], o);
    if (lane == 0 && r < a.n) {
      if (MODE == kGDense) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t >= a.ntok) break;
          float* yp = a.y + int64_t(t) * a.n + r;
          *yp = a.accumulate ? *yp + acc[0][t] : acc[0][t];
        }
      } else {
        a.y[int64_t(blk / nrb) * a.n + r] =
            MODE == kGMoeGu ? act_apply(a.act, acc[0][0], acc[NW - 1][0], a.alpha, a.limit) : acc[0][0];
      }
    }
  }
}

template <int FMT, int NT, int MODE>
int launch_gq(const GqArgs& a, cudaStream_t s) {
  const int smem = kGStages * (MODE == kGMoeGu ? 2 : 1) * kGRows * a.row_slot + 2 * kGStages * 8;
  auto kern = k_mvq8g<FMT, NT, MODE>;
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
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGThreads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int nblk = (a.n + kGRows - 1) / kGRows * (MODE == kGDense ? 1 : a.assignments);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(min(nblk, per_sm * sms), 1, 1);
  cfg.blockDim = dim3(kGThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? LK_OK : LK_ECUDA;
}

template <int FMT>
void chunk_geometry(GqArgs& a) {
  a.rb = lk_row_bytes(FMT, a.k);
  a.cb = kGChunk / fmt_qk(FMT) * fmt_block_bytes(FMT);
  a.nkc = (a.k + kGChunk - 1) / kGChunk;
  a.row_slot = (a.cb + 15 + 15) / 16 * 16;
}

template <int FMT>
int mvq8g_moe(GqArgs a, int mode, cudaStream_t s) {
  chunk_geometry<FMT>(a);
  a.ntok = 1;
  return mode == 0 ? launch_gq<FMT, 1, kGMoeGu>(a, s) : launch_gq<FMT, 1, kGMoeDn>(a, s);
}

template <int FMT>
int mvq8g_f(GqArgs a, int tokens, cudaStream_t s) {
  chunk_geometry<FMT>(a);
  float* y = a.y;
  const uint8_t* codes = a.codes;
  const float* meta = a.meta;
  for (int t0 = 0; t0 < tokens; t0 += 8) {   // token tiles of 8 (one launch each; one token: the NT = 1 kernel)
    a.ntok = min(8, tokens - t0);
    a.y = y + int64_t(t0) * a.n;
    a.codes = codes + int64_t(t0) * a.k;
    a.meta = meta + int64_t(t0) * (a.k / 32) * 2;
    const int rc = a.ntok == 1 ? launch_gq<FMT, 1, kGDense>(a, s) : launch_gq<FMT, 8, kGDense>(a, s);
    if (rc != LK_OK) return rc;
  }
  return LK_OK;
}

}  // namespace

int moe_expert_mv_q8(int fmt, int mode, int n, int k, int assignments, int ku, int n_experts, int fused,
                     const int32_t* ids, const uint8_t* xq, int xrows, const void* w, const void* w2, int act,
                     float alpha, float limit, float* y, cudaStream_t s) {
  GqArgs a{};
  a.w = static_cast<const uint8_t*>(w);
  a.w2 = static_cast<const uint8_t*>(mode == 0 && !fused ? w2 : w);
  a.codes = xq;
  a.meta = reinterpret_cast<const float*>(xq + int64_t(xrows) * k);
  a.y = y;
  a.n = n;
  a.k = k;
  a.ids = ids;
  a.assignments = assignments;
  a.x_div = mode == 0 ? ku : 1;
  a.n_experts = n_experts;
  a.rows_per_expert = n * (mode == 0 && fused ? 2 : 1);
  a.rows_per_expert2 = mode == 0 && fused ? 2 * n : n;
  a.w2_row_offset = mode == 0 && fused ? n : 0;
  a.act = act;
  a.alpha = alpha;
  a.limit = limit;
  switch (fmt) {
    case LK_Q4_0: return mvq8g_moe<LK_Q4_0>(a, mode, s);
    case LK_Q4_K: return mvq8g_moe<LK_Q4_K>(a, mode, s);
    case LK_Q8_0: return mvq8g_moe<LK_Q8_0>(a, mode, s);
    case LK_Q5_0: return mvq8g_moe<LK_Q5_0>(a, mode, s);
    case LK_Q5_K: return mvq8g_moe<LK_Q5_K>(a, mode, s);
    case LK_Q6_K: return mvq8g_moe<LK_Q6_K>(a, mode, s);
  }
  return LK_EUNSUPPORTED;
}

bool mv_q8_generic_format(int fmt) {
  return fmt == LK_Q8_0 || fmt == LK_Q5_0 || fmt == LK_Q5_K || fmt == LK_Q6_K || fmt == LK_IQ4_NL ||
         fmt == LK_IQ4_XS;
}

int mv_q8_generic(int fmt, int n, int k, int tokens, int accumulate, const uint8_t* xq, const void* w, float* y,
                  cudaStream_t s) {
  GqArgs a{};
  a.w = static_cast<const uint8_t*>(w);
  a.codes = xq;
  a.meta = reinterpret_cast<const float*>(xq + int64_t(tokens) * k);
  a.y = y;
  a.n = n;
  a.k = k;
  a.accumulate = accumulate;
  switch (fmt) {
    case LK_Q8_0: return mvq8g_f<LK_Q8_0>(a, tokens, s);
    case LK_Q5_0: return mvq8g_f<LK_Q5_0>(a, tokens, s);
    case LK_Q5_K: return mvq8g_f<LK_Q5_K>(a, tokens, s);
    case LK_Q6_K: return mvq8g_f<LK_Q6_K>(a, tokens, s);
    case LK_IQ4_NL: return mvq8g_f<LK_IQ4_NL>(a, tokens, s);
    case LK_IQ4_XS: return mvq8g_f<LK_IQ4_XS>(a, tokens, s);
  }
  return LK_EUNSUPPORTED;
}

}  // namespace lk
