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
//
// k_mvs, the one-token dense form (the decode step's own shape): the same arithmetic, fed through shared memory.
// A producer warp bulk-copies stages of 8 consecutive rows -- the 16-byte-aligned window that covers the rows' bytes,
// one copy per weight -- into a 3-slot mbarrier ring, the first stage before griddepcontrol.wait; the 8 consumer warps
// stage x once as f32, then warp w takes row w of each stage (lane l its groups l, l + 32, ...), decoding from shared
// memory instead of global byte loads.
#include <mutex>

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

// group gi of a packed row of weight wi (0 gate / only weight, 1 up): FMT's decoder, or for kFmtPair the weight's
// own format read at run time
template <int FMT>
LK_DEV void mv_group(const MvArgs& a, int wi, const uint8_t* row, int gi, float (&v)[32]) {
  if (FMT == kFmtPair) {
    row_group_values(wi ? a.fmt2 : a.fmt, row, gi, v);
  } else {
    constexpr int gpb = fmt_qk(FMT) / 32;   // 32-value groups per block
    group_values<FMT>(row + (gi / gpb) * fmt_block_bytes(FMT), gi % gpb, v);
  }
}

template <int FMT, int XT, bool SWIGLU, bool MOE, int TOK>
__global__ void __launch_bounds__(kGWarps * 32) k_mvg(const MvArgs a) {
  constexpr int NW = SWIGLU ? 2 : 1;
  const int64_t rb2 = FMT == kFmtPair ? a.row_bytes2 : a.row_bytes;   // the second weight's row stride
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
    const uint8_t* wr[2] = {a.w + (wbase + row) * a.row_bytes, w2 + (w2base + row) * rb2};
    float acc[NW][TOK];
#pragma unroll
    for (int wi = 0; wi < NW; ++wi)
#pragma unroll
      for (int t = 0; t < TOK; ++t) acc[wi][t] = 0.f;
    for (int gi = lane; gi < groups; gi += 32) {
#pragma unroll
      for (int wi = 0; wi < NW; ++wi) {
        float v[32];
        mv_group<FMT>(a, wi, wr[wi], gi, v);
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

constexpr int kSRows = 8;                    // rows per stage = consumer warps
constexpr int kSThreads = 32 * (1 + kSRows);
constexpr int kSStages = 3;

LK_DEV void sgriddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LK_DEV void sgriddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// bytes of one weight's window in a slot: 8 rows and up to 15 bytes of slack at either end, 16-byte granules
__host__ __device__ inline int64_t mvs_window(int64_t rb) { return (kSRows * rb + 30 + 15) / 16 * 16; }

template <int FMT, int XT, bool SWIGLU>
__global__ void __launch_bounds__(kSThreads, 2) k_mvs(const MvArgs a, int nstages, int slot_bytes) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int64_t win = mvs_window(a.row_bytes);
  const int64_t rb2 = FMT == kFmtPair ? a.row_bytes2 : a.row_bytes;   // the second weight's row stride
  float* xs = reinterpret_cast<float*>(smem + kSStages * slot_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(xs + a.k);
  uint64_t* empty = full + kSStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, G = gridDim.x;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kSRows);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const uint8_t* w2 = a.w2 ? a.w2 : a.w;
  // the window of rows r0 .. r0 + rows of weight `src` (rows start at row_off in it): [floor16(start), ceil16(end))
  auto window = [&](const uint8_t* base, int64_t rb, int64_t row0, int rows, uintptr_t& lo, uint32_t& bytes) {
    const uintptr_t b = reinterpret_cast<uintptr_t>(base + row0 * rb);
    lo = b & ~uintptr_t(15);
    bytes = uint32_t(((b + uintptr_t(rows * rb) + 15) & ~uintptr_t(15)) - lo);
  };
  if (warp == 0) {
    if (lane == 0) {
      sgriddep_launch();
      for (int i = 0;; ++i) {
        const int st = cta + i * G;
        if (st >= nstages) break;
        if (i == 1) sgriddep_wait();   // the first stage goes out before the previous grid ends
        const int s = i % kSStages;
        if (i >= kSStages && !mbar_wait(&empty[s], ((i / kSStages) - 1) & 1)) atomicOr(&g_status, 1u);
        const int r0 = st * kSRows, rows = min(kSRows, a.n - r0);
        uintptr_t lo, lo2 = 0;
        uint32_t bytes, bytes2 = 0;
        window(a.w, a.row_bytes, r0, rows, lo, bytes);
        if (SWIGLU) window(w2, rb2, int64_t(a.w2_row_offset) + r0, rows, lo2, bytes2);
        mbar_expect_tx(&full[s], bytes + bytes2);
        bulk_g2s(smem + s * slot_bytes, reinterpret_cast<const void*>(lo), bytes, &full[s]);
        if (SWIGLU) bulk_g2s(smem + s * slot_bytes + win, reinterpret_cast<const void*>(lo2), bytes2, &full[s]);
      }
    }
    __syncwarp();
    return;
  }
  sgriddep_wait();   // x comes from the previous kernel
  for (int i = threadIdx.x - 32; i < a.k / 4; i += kSRows * 32) {   // x as f32 into shared memory
    float4 f;
    if (XT == LK_F32) {
      f = __ldg(reinterpret_cast<const float4*>(a.x) + i);
    } else {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(a.x) + i);
      if (XT == LK_BF16) {
        f = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                        __uint_as_float(u.y & 0xffff0000u));
      } else {
        const float2 p0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 p1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        f = make_float4(p0.x, p0.y, p1.x, p1.y);
      }
    }
    reinterpret_cast<float4*>(xs)[i] = f;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kSRows * 32) : "memory");   // consumer warps only
  const int cw = warp - 1, groups = a.k / 32;
  for (int i = 0;; ++i) {
    const int st = cta + i * G;
    if (st >= nstages) break;
    const int s = i % kSStages;
    if (!mbar_wait(&full[s], (i / kSStages) & 1)) atomicOr(&g_status, 1u);
    const int row = st * kSRows + cw;
    float acc[2] = {0.f, 0.f};
    if (row < a.n) {
      const uintptr_t b0 = reinterpret_cast<uintptr_t>(a.w + int64_t(st) * kSRows * a.row_bytes);
      const uintptr_t b1 = reinterpret_cast<uintptr_t>(w2 + (int64_t(a.w2_row_offset) + int64_t(st) * kSRows) * rb2);
      const uint8_t* rp[2] = {smem + s * slot_bytes + (b0 & 15) + int64_t(cw) * a.row_bytes,
                              smem + s * slot_bytes + win + (b1 & 15) + int64_t(cw) * rb2};
#pragma unroll
      for (int wi = 0; wi < (SWIGLU ? 2 : 1); ++wi) {
        float sacc = 0.f;
        for (int g = lane; g < groups; g += 32) {
          float v[32];
          mv_group<FMT>(a, wi, rp[wi], g, v);
          const float4* xp = reinterpret_cast<const float4*>(xs + g * 32);
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 xv = xp[q];
            s0 = fmaf(v[4 * q], xv.x, s0);
            s1 = fmaf(v[4 * q + 1], xv.y, s1);
            s0 = fmaf(v[4 * q + 2], xv.z, s0);
            s1 = fmaf(v[4 * q + 3], xv.w, s1);
          }
          sacc += s0 + s1;
        }
        acc[wi] = sacc;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc[0] += __shfl_xor_sync(0xFFFFFFFFu, acc[0], o);
      if (SWIGLU) acc[1] += __shfl_xor_sync(0xFFFFFFFFu, acc[1], o);
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&empty[s]);
      if (row < a.n) {
        const float val = SWIGLU ? act_apply(a.epi.act, acc[0], acc[1], a.epi.alpha, a.epi.limit) : acc[0];
        float* yp = a.y + row;
        *yp = a.accumulate ? *yp + val : val;
      }
    }
  }
}

// the streaming form's launch: 0 when it does not apply (the caller falls back to k_mvg)
template <int FMT, int XT, bool SWIGLU>
int launch_s(const MvArgs& a, cudaStream_t s, bool& done) {
  done = false;
  const int64_t win = mvs_window(a.row_bytes);
  const int64_t win2 = SWIGLU ? mvs_window(FMT == kFmtPair ? a.row_bytes2 : a.row_bytes) : 0;
  const int slot = int((win + win2 + 127) / 128 * 128);
  const int smem = kSStages * slot + a.k * 4 + 2 * kSStages * 8;
  if (smem > 110 * 1024 || a.k % 4) return LK_OK;   // two CTAs per SM, or not this form
  auto kern = k_mvs<FMT, XT, SWIGLU>;
  static int configured[32] = {};   // the largest shared-memory size set per device
  static std::mutex mu;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  if (dev >= 32) return LK_OK;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (configured[dev] < smem) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return LK_ECUDA;
      configured[dev] = smem;
    }
  }
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int nstages = (a.n + kSRows - 1) / kSRows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(min(nstages, 2 * sms), 1, 1);
  cfg.blockDim = dim3(kSThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  done = true;
  return cudaLaunchKernelEx(&cfg, kern, a, nstages, slot) == cudaSuccess ? LK_OK : LK_ECUDA;
}

template <int FMT, int XT, bool SWIGLU, bool MOE, int TOK>
int launch_g(const MvArgs& a, int groups, cudaStream_t s) {
  const dim3 grid((a.n + kGRows - 1) / kGRows, groups);
  k_mvg<FMT, XT, SWIGLU, MOE, TOK><<<grid, kGWarps * 32, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

template <int FMT, int XT>
int mvg_x(const MvArgs& a, cudaStream_t s) {
  if (!a.ids && a.tokens == 1) {   // one token, dense: the row-streaming form where its shared memory fits
    bool done = false;
    const int rc = a.swiglu ? launch_s<FMT, XT, true>(a, s, done) : launch_s<FMT, XT, false>(a, s, done);
    if (done || rc != LK_OK) return rc;
  }
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
  if (fmt >> 16) {   // LK_FMT_PAIR(gate, up): one kernel reads each weight in its own format
    MvArgs b = a;
    b.fmt = fmt & 0xffff;
    b.fmt2 = fmt >> 16;
    b.row_bytes = lk_row_bytes(b.fmt, a.k);
    b.row_bytes2 = lk_row_bytes(b.fmt2, a.k);
    return mvg_f<kFmtPair>(b, s);
  }
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
    case LK_IQ3_S: return mvg_f<LK_IQ3_S>(a, s);
    case LK_MXFP4: return mvg_f<LK_MXFP4>(a, s);
  }
  return LK_EUNSUPPORTED;
}

}  // namespace lk
