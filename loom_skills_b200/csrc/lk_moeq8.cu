// The decode MoE layer on int8 activations -- MOE_Q8=1, the reference's default with ACT_Q8 (gen_llm.py:5290-5302):
// the expert matvecs read Q8_1 codes of the router input and of the gate/up output and contract them with the weight
// codes by integer dot products. Reference pieces: route_decode (gen_moe.py:116-253), g_quant_q8 (gen_llm.py:683-750),
// expert_mv gate/up and down (gen_moe.py:535-727, the int8 forms of @g_<fmt>_icodes gen_llm.py:521-680), g_moe_wscale
// (gen_moe.py:1010-1045), g_moe_combine / shared_gated (gen_moe.py:730-777).
//
// Two launches instead of five (router, quantise x, gate/up, quantise act, down, combine):
//   k_moe_gu_q8   every CTA routes the tokens from their logits (route_token, the router kernel's code) and quantises
//                 x into shared memory; then a persistent walk over tiles of (assignment, 8 output rows): a producer warp
//                 bulk-copies the expert's 8 gate rows and 8 up rows per tile into a mbarrier ring, consumer warp w
//                 computes output row w: both dots over the lane's (chunk, page) units (unit_dot, lk_q8.cuh), a warp
//                 reduction, act(g + bg, u + bu) into act [assignments][f].
//   k_moe_dn_q8   one CTA per SM, launched as a programmatic dependent of the first: it routes the tokens again from the
//                 logits (the same code and inputs, so the same experts and weights) and streams the down rows of its
//                 tiles -- (token, 8 output rows) x the token's ku experts -- into a deep ring before
//                 griddepcontrol.wait, so the down weights arrive while the gate/up kernel runs. After the wait the CTA
//                 quantises act into shared memory; warp w dots row w of all ku experts' stages of a tile side by side
//                 with those assignments' codes and folds them into the combine in assignment order:
//                 acc = fmaf(w_k dsc[e], dn + bd, acc), from acc = sg[t] y[t] (accumulate) or 0 -- the combine's
//                 arithmetic, without the ys round trip.
// The gate/up kernel releases its dependents only after its own griddepcontrol.wait, so the logits the second kernel
// reads before its wait are complete.
#include <mutex>

#include "lk_common.cuh"
#include "lk_internal.h"
#include "lk_q8.cuh"
#include "lk_route.cuh"

namespace lk {
namespace {

constexpr int kQmWarps = 8;                     // consumer warps = output rows per stage
constexpr int kQmThreads = 32 * (1 + kQmWarps);
constexpr int kQmMaxAssign = 32;
constexpr int kQmMaxKu = 8;

struct MoeQ8Args {
  int tokens, h, f, E, ku;
  int gating, norm;
  float scale;
  const float* logits;   // [tokens][E]
  const float* rbias;    // router bias [E] or null
  const float* dscale;   // per-expert down scale [E] or null
  const void* x;         // [tokens][h]
  const uint8_t* wg;     // gate rows [E][f] (or fused: [E][2f], gate then up rows)
  const uint8_t* wu;     // up rows [E][f], or null (fused)
  const uint8_t* wd;     // down rows [E][h]
  int64_t rbh, rbf;      // packed bytes of a row of k = h / k = f
  const float* bg;       // [E][f] gate bias, or null
  const float* bu;       // [E][f] up bias
  const float* bd;       // [E][h] down bias, or null
  int act;
  float alpha, limit;
  float* actbuf;         // [tokens * ku][f]
  int32_t* ids;          // [tokens * ku] or null (written by the gate/up kernel)
  float* wts;            // [tokens * ku] or null
  const float* sg;       // [tokens] shared-expert gate, or null
  int accumulate;
  float* y;              // [tokens][h]
  int tiles;             // tiles of this launch
  int nst;               // ring stages
  int slot_bytes;
  int xs_off, ids_off;   // shared-memory offsets of the codes and of the routing
};

// smem: [ring: nst slots] [codes, then group meta] [ids[32], wts[32]] [full[nst], empty[nst]]
struct Smem {
  uint8_t* xs;
  float* meta;
  int32_t* ids;
  float* wts;
  uint64_t* full;
  uint64_t* empty;
};
LK_DEV Smem carve(uint8_t* smem, const MoeQ8Args& a, int nvals) {
  Smem m;
  m.xs = smem + a.xs_off;
  m.meta = reinterpret_cast<float*>(m.xs + nvals);
  m.ids = reinterpret_cast<int32_t*>(smem + a.ids_off);
  m.wts = reinterpret_cast<float*>(m.ids + kQmMaxAssign);
  m.full = reinterpret_cast<uint64_t*>(m.wts + kQmMaxAssign);
  m.empty = m.full + a.nst;
  return m;
}

LK_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LK_DEV void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

LK_DEV void init_ring(const Smem& m, int nst) {
  for (int i = 0; i < nst; ++i) {
    mbar_init(&m.full[i], 1);
    mbar_init(&m.empty[i], kQmWarps);
  }
  fence_mbar_init();
}

template <int FMT, int XIN, int UPL>
__global__ void __launch_bounds__(kQmThreads, 2) k_moe_gu_q8(const MoeQ8Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nx = a.tokens * a.h;
  const Smem m = carve(smem, a, nx);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, G = gridDim.x;
  if (threadIdx.x == 0) init_ring(m, a.nst);
  __syncthreads();
  griddep_wait();     // x and the logits come from earlier kernels
  griddep_launch();   // the down kernel may start: what it reads before its own wait is complete now
  if (warp == 0) {
    for (int t = 0; t < a.tokens; ++t)
      route_token(lane, a.E, a.ku, a.gating, a.norm, a.scale, a.logits + int64_t(t) * a.E, a.rbias, m.ids + t * a.ku,
                  m.wts + t * a.ku);
  } else {
    q8::quant_flat<XIN>(a.x, nx, threadIdx.x - 32, reinterpret_cast<int8_t*>(m.xs), m.meta);
  }
  __syncthreads();
  const int A = a.tokens * a.ku;
  if (cta == 0 && threadIdx.x < A && a.ids) {   // the layer's routing for the caller: combine weights after dscale
    const int e = m.ids[threadIdx.x];
    a.ids[threadIdx.x] = e;
    a.wts[threadIdx.x] = a.dscale ? m.wts[threadIdx.x] * __ldg(a.dscale + e) : m.wts[threadIdx.x];
  }
  const int ntr = (a.f + kQmWarps - 1) / kQmWarps;
  if (warp == 0) {   // producer: per tile the expert's gate rows r0.. and up rows r0.., one bulk copy each
    if (lane == 0) {
      for (int i = 0;; ++i) {
        const int tau = cta + i * G;
        if (tau >= a.tiles) break;
        const int as = tau / ntr, r0 = (tau % ntr) * kQmWarps;
        const int64_t e = m.ids[as];
        const int rows = min(kQmWarps, a.f - r0);
        const int s = i % a.nst;
        if (i >= a.nst && !mbar_wait(&m.empty[s], ((i / a.nst) - 1) & 1)) atomicOr(&g_status, 1u);
        const uint32_t bytes = uint32_t(rows * a.rbh);
        const uint8_t* gsrc = a.wu ? a.wg + (e * a.f + r0) * a.rbh : a.wg + (e * 2 * a.f + r0) * a.rbh;
        const uint8_t* usrc = a.wu ? a.wu + (e * a.f + r0) * a.rbh : a.wg + (e * 2 * a.f + a.f + r0) * a.rbh;
        uint8_t* dst = smem + s * a.slot_bytes;
        mbar_expect_tx(&m.full[s], 2 * bytes);
        bulk_g2s(dst, gsrc, bytes, &m.full[s]);
        bulk_g2s(dst + kQmWarps * a.rbh, usrc, bytes, &m.full[s]);
      }
    }
    __syncwarp();
    return;
  }
  const int cw = warp - 1, pg = lane & 3;
  const uint32_t hsel = q8::q4k_hsel(pg), big = q8::q4k_big(pg);
  for (int i = 0;; ++i) {
    const int tau = cta + i * G;
    if (tau >= a.tiles) break;
    const int as = tau / ntr, row = (tau % ntr) * kQmWarps + cw;
    const int t = as / a.ku;
    const int s = i % a.nst;
    if (!mbar_wait(&m.full[s], (i / a.nst) & 1)) atomicOr(&g_status, 1u);
    const int e = m.ids[as];
    float g = 0.f, u = 0.f;
    if (row < a.f) {
      const uint8_t* wr = smem + s * a.slot_bytes + cw * a.rbh;
      const uint8_t* codes = m.xs + t * a.h;
      const float* meta = m.meta + t * (a.h / 32) * 2;
#pragma unroll
      for (int j = 0; j < UPL; ++j) {
        const int c = (lane >> 2) + 8 * j;
        q8::XUnit xu;
        q8::load_xunit<FMT, true>(codes, meta, c, pg, xu);
        g += q8::unit_dot<FMT>(wr + c * kChunkBytes, xu, pg, hsel, big);
        u += q8::unit_dot<FMT>(wr + kQmWarps * a.rbh + c * kChunkBytes, xu, pg, hsel, big);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      g += __shfl_xor_sync(0xFFFFFFFFu, g, o);
      u += __shfl_xor_sync(0xFFFFFFFFu, u, o);
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&m.empty[s]);
      if (row < a.f) {
        if (a.bg) {
          g += __ldg(a.bg + int64_t(e) * a.f + row);
          u += __ldg(a.bu + int64_t(e) * a.f + row);
        }
        a.actbuf[int64_t(as) * a.f + row] = act_apply(a.act, g, u, a.alpha, a.limit);
      }
    }
  }
}

template <int FMT>
__global__ void __launch_bounds__(kQmThreads, 1) k_moe_dn_q8(const MoeQ8Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int A = a.tokens * a.ku;
  const Smem m = carve(smem, a, A * a.f);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, G = gridDim.x;
  if (threadIdx.x == 0) init_ring(m, a.nst);
  __syncthreads();
  if (warp == 0) {   // routing from the logits (complete: see the file comment), before the wait
    for (int t = 0; t < a.tokens; ++t)
      route_token(lane, a.E, a.ku, a.gating, a.norm, a.scale, a.logits + int64_t(t) * a.E, a.rbias, m.ids + t * a.ku,
                  m.wts + t * a.ku);
    __syncwarp();
    if (lane < A && a.dscale) m.wts[lane] *= __ldg(a.dscale + m.ids[lane]);
  }
  __syncthreads();
  const int ntr = (a.h + kQmWarps - 1) / kQmWarps;
  if (warp == 0) {   // producer: the down weights need nothing from the gate/up kernel
    if (lane == 0) {
      int i = 0;
      for (int j = 0;; ++j) {
        const int tau = cta + j * G;
        if (tau >= a.tiles) break;
        const int t = tau / ntr, r0 = (tau % ntr) * kQmWarps;
        const int rows = min(kQmWarps, a.h - r0);
        const uint32_t bytes = uint32_t(rows * a.rbf);
        for (int k = 0; k < a.ku; ++k, ++i) {
          const int64_t e = m.ids[t * a.ku + k];
          const int s = i % a.nst;
          if (i >= a.nst && !mbar_wait(&m.empty[s], ((i / a.nst) - 1) & 1)) atomicOr(&g_status, 1u);
          mbar_expect_tx(&m.full[s], bytes);
          bulk_g2s(smem + s * a.slot_bytes, a.wd + (e * a.h + r0) * a.rbf, bytes, &m.full[s]);
        }
      }
    }
    __syncwarp();
    return;
  }
  griddep_wait();   // act comes from the gate/up kernel
  q8::quant_flat<q8::kXinF32>(a.actbuf, A * a.f, threadIdx.x - 32, reinterpret_cast<int8_t*>(m.xs), m.meta);
  asm volatile("bar.sync 1, %0;" ::"r"(kQmWarps * 32) : "memory");   // consumer warps only
  const int cw = warp - 1, pg = lane & 3;
  const uint32_t hsel = q8::q4k_hsel(pg), big = q8::q4k_big(pg);
  const int U = a.f / 64;   // (chunk, page) units of a down row; lane l takes l, l + 32, ...
  int i = 0;                // this CTA's stage count so far (the producer's order)
  for (int j = 0;; ++j) {
    const int tau = cta + j * G;
    if (tau >= a.tiles) break;
    const int t = tau / ntr, row = (tau % ntr) * kQmWarps + cw;
    const bool valid = row < a.h;
    // the tile's ku stages are all in the ring at once (nst >= ku): wait for every one, then run the ku dots side by
    // side, so their shared-memory loads and integer dots overlap
    for (int k = 0; k < a.ku; ++k)
      if (!mbar_wait(&m.full[(i + k) % a.nst], ((i + k) / a.nst) & 1)) atomicOr(&g_status, 1u);
    float d[kQmMaxKu];
#pragma unroll
    for (int k = 0; k < kQmMaxKu; ++k) {
      d[k] = 0.f;
      if (k < a.ku && valid) {
        const int as = t * a.ku + k;
        const uint8_t* wr = smem + ((i + k) % a.nst) * a.slot_bytes + cw * a.rbf;
        const uint8_t* codes = m.xs + as * a.f;
        const float* meta = m.meta + as * (a.f / 32) * 2;
        for (int un = lane; un < U; un += 32) {
          const int c = un >> 2;
          q8::XUnit xu;
          q8::load_xunit<FMT, true>(codes, meta, c, pg, xu);
          d[k] += q8::unit_dot<FMT>(wr + c * kChunkBytes, xu, pg, hsel, big);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int k = 0; k < kQmMaxKu; ++k) d[k] += __shfl_xor_sync(0xFFFFFFFFu, d[k], o);
    __syncwarp();
    if (lane == 0) {
      float acc = 0.f;
      if (valid && a.accumulate) {
        acc = a.y[int64_t(t) * a.h + row];
        if (a.sg) acc *= __ldg(a.sg + t);
      }
      for (int k = 0; k < a.ku; ++k) {
        mbar_arrive(&m.empty[(i + k) % a.nst]);
        if (valid) {
          const int as = t * a.ku + k;
          float dk = d[0];
#pragma unroll
          for (int q = 1; q < kQmMaxKu; ++q)
            if (q == k) dk = d[q];
          if (a.bd) dk += __ldg(a.bd + int64_t(m.ids[as]) * a.h + row);
          acc = fmaf(m.wts[as], dk, acc);   // the combine's chain, in assignment order
        }
      }
      if (valid) a.y[int64_t(t) * a.h + row] = acc;
    }
    i += a.ku;
  }
}

struct Occ {
  const void* kern;
  int dev, smem, per_sm, sms;
};

// occupancy of (kernel, shared-memory size) on the current device, queried once
int occupancy(const void* kern, int smem, int& per_sm, int& sms) {
  static Occ cache[32];
  static int n = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (cache[i].kern == kern && cache[i].dev == dev && cache[i].smem == smem) {
      per_sm = cache[i].per_sm;
      sms = cache[i].sms;
      return LK_OK;
    }
  // the kernel's dynamic shared-memory limit only ever grows (a smaller later size must not undercut an earlier,
  // cached one)
  int top = smem;
  for (int i = 0; i < n; ++i)
    if (cache[i].kern == kern && cache[i].dev == dev) top = max(top, cache[i].smem);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, top) != cudaSuccess) return LK_ECUDA;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kQmThreads, smem) != cudaSuccess || per_sm < 1)
    return LK_ECUDA;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (n < 32) cache[n++] = Occ{kern, dev, smem, per_sm, sms};
  return LK_OK;
}

template <typename K>
int launch(K kern, const MoeQ8Args& a, int grid, int smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kQmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? LK_OK : LK_ECUDA;
}

int smem_bytes(int ring, int nvals, int nst, int& xs_off, int& ids_off) {
  xs_off = ring;
  ids_off = ring + (nvals + nvals / 4 + 127) / 128 * 128;
  return ids_off + 2 * kQmMaxAssign * 4 + 2 * nst * 8;
}

template <int FMT>
int run(const MoeFfnQ8& p, cudaStream_t s) {
  MoeQ8Args a{};
  a.tokens = p.tokens;
  a.h = p.h;
  a.f = p.f;
  a.E = p.n_experts;
  a.ku = p.ku;
  a.gating = p.gating;
  a.norm = p.norm;
  a.scale = p.scale;
  a.logits = p.logits;
  a.rbias = p.router_bias;
  a.dscale = p.down_scale;
  a.x = p.x;
  a.wg = static_cast<const uint8_t*>(p.w_gate);
  a.wu = static_cast<const uint8_t*>(p.w_up);
  a.wd = static_cast<const uint8_t*>(p.w_down);
  a.rbh = int64_t(p.h) / 256 * kChunkBytes;
  a.rbf = int64_t(p.f) / 256 * kChunkBytes;
  a.bg = p.b_gate;
  a.bu = p.b_up;
  a.bd = p.b_down;
  a.act = p.act;
  a.alpha = p.alpha;
  a.limit = p.limit;
  a.actbuf = p.act_buf;
  a.ids = p.ids;
  a.wts = p.wts;
  a.sg = p.sg;
  a.accumulate = p.accumulate;
  a.y = p.y;
  const int A = p.tokens * p.ku;

  // gate/up: 2 x 8 rows of k = h per stage, 3 stages (2 at h = 4096), two CTAs per SM
  MoeQ8Args g = a;
  g.slot_bytes = int((2 * kQmWarps * a.rbh + 127) / 128 * 128);
  g.nst = p.h <= 2048 ? 3 : 2;
  const int smem1 = smem_bytes(g.nst * g.slot_bytes, p.tokens * p.h, g.nst, g.xs_off, g.ids_off);
  g.tiles = A * ((p.f + kQmWarps - 1) / kQmWarps);
  const void* k1 = nullptr;
  const bool bf = p.x_dtype == LK_BF16;
  if (p.h == 2048) k1 = bf ? (const void*)k_moe_gu_q8<FMT, q8::kXinBF16, 1> : (const void*)k_moe_gu_q8<FMT, q8::kXinF32, 1>;
  else k1 = bf ? (const void*)k_moe_gu_q8<FMT, q8::kXinBF16, 2> : (const void*)k_moe_gu_q8<FMT, q8::kXinF32, 2>;
  int per_sm = 0, sms = 0;
  int rc = occupancy(k1, smem1, per_sm, sms);
  if (rc != LK_OK) return rc;
  const int grid1 = min(g.tiles, sms * min(per_sm, 2));
  if (p.h == 2048)
    rc = bf ? launch(k_moe_gu_q8<FMT, q8::kXinBF16, 1>, g, grid1, smem1, s)
            : launch(k_moe_gu_q8<FMT, q8::kXinF32, 1>, g, grid1, smem1, s);
  else
    rc = bf ? launch(k_moe_gu_q8<FMT, q8::kXinBF16, 2>, g, grid1, smem1, s)
            : launch(k_moe_gu_q8<FMT, q8::kXinF32, 2>, g, grid1, smem1, s);
  if (rc != LK_OK) return rc;

  // down + combine: 8 rows of k = f per stage, a ring of up to 64 KB, one CTA per SM
  MoeQ8Args d = a;
  d.slot_bytes = int((kQmWarps * a.rbf + 127) / 128 * 128);
  d.nst = max(p.ku, min(32, 65536 / d.slot_bytes));   // a tile's ku stages fit the ring at once
  const int smem2 = smem_bytes(d.nst * d.slot_bytes, A * p.f, d.nst, d.xs_off, d.ids_off);
  d.tiles = p.tokens * ((p.h + kQmWarps - 1) / kQmWarps);
  rc = occupancy((const void*)k_moe_dn_q8<FMT>, smem2, per_sm, sms);
  if (rc != LK_OK) return rc;
  return launch(k_moe_dn_q8<FMT>, d, min(d.tiles, sms), smem2, s);
}

}  // namespace

int moe_ffn_decode_q8(int fmt, const MoeFfnQ8& p, cudaStream_t s) {
  if (fmt == LK_Q4_K) return run<LK_Q4_K>(p, s);
  if (fmt == LK_Q4_0) return run<LK_Q4_0>(p, s);
  return LK_EUNSUPPORTED;
}

LK_STATUS_READER(status_moeq8)

}  // namespace lk
