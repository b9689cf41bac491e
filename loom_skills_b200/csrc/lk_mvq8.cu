// Decode matvec with int8 activations -- the reference's default decode numerics (ACT_Q8=1, gen_llm.py:514-518):
//
//   g_quant_q8 (gen_llm.py:683-750)   x [rows][k] -> codes int8 [rows][k/32][32], then at byte rows*k the group meta
//                                     [rows][k/32][2] f32 = (f16-rounded d, sum of codes); d = amax/127, q = round(x/d)
//   g_mv_{fmt}_q8 (gen_llm.py:1159-1378, @g_<fmt>_icodes :521-680)
//                                     y[t][n] (+)= sum over 32-groups g of  wscale_g * d_x[g] * dot(wcode_g, xcode_g)
//                                                                           - wmin_g  * d_x[g] * sum(xcode_g)
//
// k_mv_q8 contracts the 4-bit weight codes with the int8 activation codes by dp4a (4 products per instruction, integer
// exact), so a weight value costs about one instruction: a nibble mask per 4 values and a dp4a per 4 values. The high
// nibbles are used in place (16 * code, 0..240): their group's integer dot is 16x and the 1/16 goes into that group's
// f32 scale. Per 32-group the integer dot is scaled once in f32.
//
// CTA = 1 producer warp + 8 consumer warps, 64 weight rows, a K-range of 256-value chunks:
//   producer   TMA: per chunk one box of 64 rows x 144 bytes of packed weights, the chunk's activation codes
//              [tokens][256] and group meta [tokens][16 f32], into a 4-stage mbarrier ring. It issues the weight box
//              of the first stage before griddepcontrol.wait -- weights never depend on the previous kernel -- so
//              under programmatic dependent launch the weight stream starts while the previous kernel finishes.
//              Only one stage goes out early: loads still in flight on the SMs were measured to hold back the
//              previous grid's completion (the release of griddepcontrol.wait) by up to 2 us when every CTA
//              requested its whole ring up front; one stage per CTA keeps the overlap without the delay.
//   consumers  thread = (64-byte page / block pair p of the chunk, one row); partial sums over the 4 threads of a
//              row are combined by shuffles at the end. Small stages (37 KB of ring) keep 6 CTAs = 54 warps on an SM:
//              the per-thread work is a short dependent chain, so latency is hidden by warps, not by ILP alone.
//   split-K    small N runs S CTAs per row tile as one thread-block cluster; their partial sums meet in CTA 0's
//              shared memory (distributed shared memory reads, fixed order: deterministic).
#include <mutex>

#include "lk_common.cuh"
#include "lk_internal.h"
#include "lk_q8.cuh"

namespace lk {

int make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, int64_t rows, int64_t cols,
             int box_cols, int box_rows, CUtensorMapSwizzle swz);

namespace {

constexpr int kQConsumers = 8;
constexpr int kQThreads = 32 * (1 + kQConsumers);
// chunked matvec tiles: one token -- 64 rows, 4 stages; token tiles of 8 -- 128 rows (2 per thread, so each x load
// serves two rows), 3 stages, 96 registers: two CTAs per SM. Measured on the eight-token Qwen3-8B projections:
// 256 rows (151 registers, one CTA per SM) and forced two-CTA 256-row builds (spills) were slower.
constexpr int kQRows1 = 64, kQStages1 = 4, kQRows8 = 128, kQStages8 = 3;
constexpr int kPreWaitStages = 1;   // weight stages a CTA requests before griddepcontrol.wait (see above)

LK_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LK_DEV void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

using q8::dp4a_us;
using q8::i2f_small;
using q8::kXinBF16;
using q8::kXinCodes;
using q8::kXinF32;
using q8::xq_smem_bytes;
LK_DEV float u6_to_f(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.0f; }

LK_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
LK_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
LK_DEV float ld_dsmem_f32(const float* local_addr, uint32_t rank) {
  uint32_t a = smem_u32(local_addr), r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
  return v;
}

struct Q8Args {
  float* y;
  int n, k, ntok, accumulate;
  int nchunks, splits, cps;   // chunks of 256, CTAs per row tile (cluster size), chunks per split
};

// stage of the chunked kernel: QR weight rows of one 256-value chunk, then the chunk's x codes and meta of TOKB tokens
template <int TOKB, int QR>
constexpr int q8_stage_bytes() {
  return (QR * kChunkBytes + TOKB * 256 + TOKB * 64 + 127) / 128 * 128;
}
template <int TOKB, int QR, int QS>
constexpr int q8_smem_bytes() {
  return QS * q8_stage_bytes<TOKB, QR>() + 2 * QS * 8 + TOKB * QR * 4;
}

// Matvec over chunks of 256 values, for several tokens (tiles of TOKB) or for one token outside the row kernel's
// shapes. CTA (split, row tile) streams QR rows over its range of chunks through a QS-stage ring; a stage is one 2-D
// TMA box of the rows' 144-byte chunks plus the chunk's x codes and meta for the TOKB tokens. Consumer thread (rs, pg)
// owns page pg (64 values) of rows rs + 64 r, r < QR / 64: per stage it decodes those rows' weight words and scales
// into registers once, then for every token loads the page's x once and runs it against all its rows. Every one of
// the TOKB token rows is computed: rows past the tile's tokens are zero-filled by the TMA and never stored, and the
// unconditional loop lets the loads of later tokens go out ahead of the arithmetic of earlier ones. The split CTAs
// of a row tile form a cluster and reduce their partial sums through distributed shared memory.
template <int FMT, int TOKB, int QR, int QS>
__global__ void __launch_bounds__(kQThreads)
    k_mv_q8(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
            const __grid_constant__ CUtensorMap mmap, const Q8Args p) {
  constexpr int kStage = q8_stage_bytes<TOKB, QR>();
  constexpr int kWBytes = QR * kChunkBytes;
  constexpr int kRpt = QR / 64;   // rows per consumer thread
  static_assert(QR % 64 == 0 && QR <= 256, "64 to 256 rows per tile (one TMA box)");
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + QS * kStage);
  uint64_t* empty = full + QS;
  float* red = reinterpret_cast<float*>(empty + QS);   // [TOKB][QR] partial sums (split-K)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.y * QR;
  const int split = blockIdx.x;
  const int c0 = split * p.cps;
  const int nst = max(0, min(p.nchunks, c0 + p.cps) - c0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < QS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kQConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      griddep_launch();
      prefetch_tensormap(&wmap);
      const uint32_t bytes = kWBytes + TOKB * 256 + TOKB * 64;
      const int pre = min(kPreWaitStages, nst);
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full[i], bytes);
        tma_load_2d(smem + i * kStage, &wmap, (c0 + i) * (kChunkBytes / 4), row0, &full[i]);
      }
      griddep_wait();   // activations come from the previous kernel
      for (int i = 0; i < pre; ++i) {
        tma_load_2d(smem + i * kStage + kWBytes, &xmap, (c0 + i) * 256, 0, &full[i]);
        tma_load_2d(smem + i * kStage + kWBytes + TOKB * 256, &mmap, (c0 + i) * 16, 0, &full[i]);
      }
      for (int i = pre; i < nst; ++i) {
        const int s = i % QS;
        if (i >= QS && !mbar_wait(&empty[s], ((i / QS) - 1) & 1)) atomicOr(&g_status, 1u);
        mbar_expect_tx(&full[s], bytes);
        uint8_t* st = smem + s * kStage;
        tma_load_2d(st, &wmap, (c0 + i) * (kChunkBytes / 4), row0, &full[s]);
        tma_load_2d(st + kWBytes, &xmap, (c0 + i) * 256, 0, &full[s]);
        tma_load_2d(st + kWBytes + TOKB * 256, &mmap, (c0 + i) * 16, 0, &full[s]);
      }
    }
    __syncwarp();
  } else {
    griddep_wait();
    const int ct = threadIdx.x - 32;
    const int pg = ct & 3, rs = ct >> 2;
    const int ntok = min(p.ntok, TOKB);
    float acc[kRpt][TOKB];
#pragma unroll
    for (int r = 0; r < kRpt; ++r)
#pragma unroll
      for (int t = 0; t < TOKB; ++t) acc[r][t] = 0.f;

    for (int i = 0; i < nst; ++i) {
      const int s = i % QS;
      if (!mbar_wait(&full[s], (i / QS) & 1)) atomicOr(&g_status, 1u);
      const uint8_t* st = smem + s * kStage;
      const uint8_t* xs = st + kWBytes;
      const float* ms = reinterpret_cast<const float*>(st + kWBytes + TOKB * 256);
      // this thread's rows, page pg: eight nibble words each and their scales. Q4_K: words = the page's 32 bytes
      // (low nibbles group 2pg, high nibbles group 2pg + 1), sa / sb = d * sc of the two groups (sb / 16: the high
      // nibbles' dot is 16 x), ma / mb = dmin * m. Q4_0: words 0-3 = block 2pg's codes (realigned), 4-7 = block
      // 2pg + 1's, sa / sb = their d.
      uint32_t w[kRpt][8];
      float sa[kRpt], sb[kRpt], ma[kRpt], mb[kRpt];
#pragma unroll
      for (int r = 0; r < kRpt; ++r) {
        const uint8_t* wr = st + (rs + 64 * r) * kChunkBytes;
        if (FMT == LK_Q4_K) {
          const uint4 hd = *reinterpret_cast<const uint4*>(wr);
          const uint4 q0 = *reinterpret_cast<const uint4*>(wr + 16 + 32 * pg);
          const uint4 q1 = *reinterpret_cast<const uint4*>(wr + 32 + 32 * pg);
          w[r][0] = q0.x;
          w[r][1] = q0.y;
          w[r][2] = q0.z;
          w[r][3] = q0.w;
          w[r][4] = q1.x;
          w[r][5] = q1.y;
          w[r][6] = q1.z;
          w[r][7] = q1.w;
          uint32_t sc0, m0, sc1, m1;
          q4k_scale_min_w(hd.y, hd.z, hd.w, 2 * pg, sc0, m0);
          q4k_scale_min_w(hd.y, hd.z, hd.w, 2 * pg + 1, sc1, m1);
          const float d = h2f(uint16_t(hd.x & 0xffffu)), dmin = h2f(uint16_t(hd.x >> 16));
          sa[r] = d * u6_to_f(sc0);
          sb[r] = d * u6_to_f(sc1) * 0.0625f;
          ma[r] = dmin * u6_to_f(m0);
          mb[r] = dmin * u6_to_f(m1);
        } else {
          // block pair pg = blocks 2pg (bytes 36pg..+17: d, then codes starting 2 bytes into a word) and 2pg + 1
          const uint32_t* wv = reinterpret_cast<const uint32_t*>(wr + 36 * pg);
          uint32_t v[9];
#pragma unroll
          for (int j = 0; j < 9; ++j) v[j] = wv[j];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            w[r][j] = __funnelshift_r(v[j], v[j + 1], 16);   // codes of the even block, realigned
            w[r][4 + j] = v[5 + j];
          }
          sa[r] = h2f(uint16_t(v[0] & 0xffffu));
          sb[r] = h2f(uint16_t(v[4] >> 16));
          ma[r] = mb[r] = 0.f;
        }
      }
#pragma unroll
      for (int t = 0; t < TOKB; ++t) {
        const uint4* xw = reinterpret_cast<const uint4*>(xs + t * 256 + 64 * pg);
        const uint4 xa0 = xw[0], xa1 = xw[1], xb0 = xw[2], xb1 = xw[3];
        const float4 mt = *reinterpret_cast<const float4*>(ms + t * 16 + 4 * pg);   // d0, sum0, d1, sum1
        const uint32_t xa[8] = {xa0.x, xa0.y, xa0.z, xa0.w, xa1.x, xa1.y, xa1.z, xa1.w};
        const uint32_t xb[8] = {xb0.x, xb0.y, xb0.z, xb0.w, xb1.x, xb1.y, xb1.z, xb1.w};
#pragma unroll
        for (int r = 0; r < kRpt; ++r) {
          if (FMT == LK_Q4_K) {
            int i0 = 0, i1 = 0, i2 = 0, i3 = 0;   // four independent dp4a chains
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              i0 = dp4a_us(w[r][j] & 0x0F0F0F0Fu, xa[j], i0);
              i1 = dp4a_us(w[r][j] & 0xF0F0F0F0u, xb[j], i1);
              i2 = dp4a_us(w[r][j + 1] & 0x0F0F0F0Fu, xa[j + 1], i2);
              i3 = dp4a_us(w[r][j + 1] & 0xF0F0F0F0u, xb[j + 1], i3);
            }
            acc[r][t] += mt.x * (sa[r] * i2f_small(i0 + i2) - ma[r] * mt.y) +
                         mt.z * (sb[r] * i2f_small(i1 + i3) - mb[r] * mt.w);
          } else {
            // block a: elements 0-15 = low nibbles (x words 0-3), 16-31 = high nibbles (x words 4-7); block b alike
            int la = 0, ha = 0, lb = 0, hb = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              la = dp4a_us(w[r][j] & 0x0F0F0F0Fu, xa[j], la);
              ha = dp4a_us(w[r][j] & 0xF0F0F0F0u, xa[4 + j], ha);
              lb = dp4a_us(w[r][4 + j] & 0x0F0F0F0Fu, xb[j], lb);
              hb = dp4a_us(w[r][4 + j] & 0xF0F0F0F0u, xb[4 + j], hb);
            }
            // Q4_0 values are code - 8: sum((q - 8) x) = dot - 8 sum(x)
            const int ca = la + (ha >> 4) - 8 * int(mt.y), cb = lb + (hb >> 4) - 8 * int(mt.w);
            acc[r][t] += sa[r] * mt.x * i2f_small(ca) + sb[r] * mt.z * i2f_small(cb);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // the four threads of a row hold its four page / block-pair partial sums
#pragma unroll
    for (int r = 0; r < kRpt; ++r)
#pragma unroll
      for (int t = 0; t < TOKB; ++t) {
        acc[r][t] += __shfl_xor_sync(0xFFFFFFFFu, acc[r][t], 1);
        acc[r][t] += __shfl_xor_sync(0xFFFFFFFFu, acc[r][t], 2);
      }
    if (p.splits > 1) {
      if (pg == 0)
#pragma unroll
        for (int r = 0; r < kRpt; ++r)
#pragma unroll
          for (int t = 0; t < TOKB; ++t) red[t * QR + rs + 64 * r] = acc[r][t];
    } else if (pg == 0) {
#pragma unroll
      for (int r = 0; r < kRpt; ++r) {
        const int row = row0 + rs + 64 * r;
        if (row >= p.n) continue;
#pragma unroll
        for (int t = 0; t < TOKB; ++t) {
          if (t >= ntok) break;
          float* dst = p.y + int64_t(t) * p.n + row;
          *dst = p.accumulate ? *dst + acc[r][t] : acc[r][t];
        }
      }
    }
  }
  if (p.splits > 1) {
    // every CTA of the cluster reaches both barriers (no early exit above)
    cluster_sync();
    if (cluster_ctarank() == 0) {
      for (int e = threadIdx.x; e < TOKB * QR; e += kQThreads) {
        const int t = e / QR, r = e % QR, row = row0 + r;
        if (t >= p.ntok || row >= p.n) continue;
        float v = 0.f;
        for (int c = 0; c < p.splits; ++c) v += ld_dsmem_f32(red + e, uint32_t(c));
        float* dst = p.y + int64_t(t) * p.n + row;
        *dst = p.accumulate ? *dst + v : v;
      }
    }
    cluster_sync();
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Single-token Q4_K / Q4_0 matvec over whole rows (K % 4096 == 0): a persistent grid streams stages of 4 consecutive
// rows (one contiguous bulk copy each) round-robin over the CTAs. Each of the 4 consumer warps owns one row of the
// stage; lane l owns the K/2048 (chunk, page) units l + 32u of every row, so its activation codes and group meta are
// loaded into registers once per launch. Per stage a warp reduces its row's partial sums with shuffles and stores y.
// Both formats spend 144 bytes per 256 values, so a unit of 64 values is one 32-byte nibble page of a Q4_K
// super-block (with the super-block's 16-byte header) or two consecutive 18-byte Q4_0 blocks, 36 bytes at a 4-byte
// aligned offset: nine word loads, the first block's nibbles realigned by funnel shifts.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kRowWarps = 4;   // consumer warps = rows per stage
// rings per CTA for K = 4096 rows and for longer rows (measured on the 8-layer decode mix: 2 rings of the short
// form 4263 GB/s against 4207 with one; 3 or more rings, or 2 of the long form, were slower)
constexpr int kRingsShort = 2, kRingsLong = 1;
// stages per ring, weight stages a ring requests before griddepcontrol.wait, and the CTAs per SM the grid is sized
// for (capped by the occupancy)
constexpr int kStagesShort = 3, kStagesLong = 3;
constexpr int kRowPreWait = 1;
constexpr int kRowCtasPerSm = 2;

constexpr int kMaxSegs = 4;
struct RowArgs {
  // up to kMaxSegs weights sharing the activation: segment g has n[g] rows, stages start[g] .. start[g + 1] - 1
  const uint8_t* w[kMaxSegs];
  float* y[kMaxSegs];
  int n[kMaxSegs];
  int start[kMaxSegs + 1];
  int nseg;
  const uint8_t* xq;   // codes [1][k] then meta [1][k/32][2] (XIN == kXinCodes)
  const void* x;       // the activation row [1][k] of f32 / bf16, quantised by the kernel itself (other XIN)
  int k, accumulate;
  int64_t rb;          // bytes per packed row
  int sr;              // rows per stage
  int nstages;         // start[nseg]
  int prewait;         // weight stages a ring requests before griddepcontrol.wait
};
// segment of a global stage, and the stage's first row inside it
LK_DEV int seg_of(const RowArgs& p, int st, int& row0) {
  int g = 0;
#pragma unroll
  for (int j = 1; j < kMaxSegs; ++j)
    if (j < p.nseg && st >= p.start[j]) g = j;
  row0 = (st - p.start[g]) * p.sr;
  return g;
}

// bytes of one ring's shared memory: its stages, then full / empty barriers, per-row pair barriers and partial sums
__host__ __device__ inline int ring_bytes(int stage_bytes, int nst) {
  return (nst * stage_bytes + 2 * nst * 8 + nst * kRowWarps * 12 + 127) / 128 * 128;
}

// UPL units per lane over the whole row; HALVES warps per row (each takes UPL / HALVES of the units; the second
// hands its partial sum to the first through shared memory and a per-row mbarrier). A CTA runs RINGS independent
// rings (a producer warp, its consumer warps, its own stages and barriers); stages go round-robin over the
// gridDim.x * RINGS rings. Fewer, larger CTAs make the grid cheaper to launch, retire and hand over to the next grid.
// XIN == kXinCodes: the activation codes come from lk_quant_q8's buffer (p.xq). kXinF32 / kXinBF16: the consumer warps
// of the CTA first quantise the row p.x into shared memory together (the g_quant_q8 launch folded into the
// matvec's prologue; it overlaps the first weight stage's flight), then read their codes from there.
// k_quant_q8 reduces a group across a warp; here a group is one thread's, so the CTA's groups run side by side.
template <int FMT, int UPL, int HALVES, int RINGS, int XIN, int NST>
__global__ void __launch_bounds__(32 * RINGS * (1 + kRowWarps * HALVES))
    k_mv_q8_rows(const RowArgs p) {
  constexpr int kU = UPL / HALVES;             // units this lane computes
  constexpr int kCW = kRowWarps * HALVES;      // consumer warps per ring
  extern __shared__ __align__(128) uint8_t smem_all[];
  const int stage_bytes = int((int64_t(p.sr) * p.rb + 127) / 128 * 128);
  const int ring = (threadIdx.x >> 5) / (1 + kCW);
  uint8_t* smem = smem_all + ring * ring_bytes(stage_bytes, NST);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * stage_bytes);
  uint64_t* empty = full + NST;
  uint64_t* pair = empty + NST;                                    // [NST][kRowWarps]
  float* part = reinterpret_cast<float*>(pair + NST * kRowWarps);  // [NST][kRowWarps]
  const int warp = (threadIdx.x >> 5) % (1 + kCW), lane = threadIdx.x & 31;   // warp within the ring
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCW);
      for (int r = 0; r < kRowWarps; ++r) mbar_init(&pair[i * kRowWarps + r], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int vb = int(blockIdx.x) * RINGS + ring, vg = int(gridDim.x) * RINGS;   // this ring, all rings
  const int my_stages = p.nstages > vb ? (p.nstages - 1 - vb) / vg + 1 : 0;

  if (warp == 0) {
    if (lane == 0) {
      griddep_launch();
      for (int i = 0; i < my_stages; ++i) {
        const int s = i % NST;
        if (i == p.prewait) griddep_wait();   // the first stages go out before the previous grid ends
        if (i >= NST && !mbar_wait(&empty[s], ((i / NST) - 1) & 1)) atomicOr(&g_status, 1u);
        const int st = vb + i * vg;
        int r0;
        const int g = seg_of(p, st, r0);
        const int rows = min(p.sr, p.n[g] - r0);
        const uint32_t bytes = uint32_t(int64_t(rows) * p.rb);
        mbar_expect_tx(&full[s], bytes);
        bulk_g2s(smem + s * stage_bytes, p.w[g] + int64_t(r0) * p.rb, bytes, &full[s]);
      }
    }
    __syncwarp();
  } else {
    const int rslot = (warp - 1) % kRowWarps;  // this warp's row of every stage
    const int half = (warp - 1) / kRowWarps;   // which share of the row's units
    griddep_wait();                            // the activations come from the previous kernel
    const uint8_t* xq = p.xq;
    if constexpr (XIN != kXinCodes) {
      // every consumer warp of the CTA takes groups cw, cw + ncw, ... of the row; then all of them read the codes
      uint8_t* xs = smem_all + RINGS * ring_bytes(stage_bytes, NST);
      const int cw = ring * kCW + (warp - 1), ncw = RINGS * kCW;
      static_assert(RINGS * kCW == 8, "256 quantising threads");
      q8::quant_groups<XIN, UPL / 2>(p.x, cw * 32 + lane, reinterpret_cast<int8_t*>(xs), reinterpret_cast<float*>(xs + p.k));
      asm volatile("bar.sync 1, %0;" ::"r"(ncw * 32) : "memory");   // consumer warps only
      xq = xs;
    }
    // lane l owns the (chunk, page) units l + 32u: chunk l/4 + 8u, page l % 4 -- the same page for every unit
    const int pg = lane & 3;
    q8::XUnit xu[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      q8::load_xunit<FMT, XIN != kXinCodes>(xq, reinterpret_cast<const float*>(xq + p.k), (lane >> 2) + 8 * (half * kU + u),
                                            pg, xu[u]);
    const uint32_t hsel = q8::q4k_hsel(pg), big = q8::q4k_big(pg);
    for (int i = 0; i < my_stages; ++i) {
      const int s = i % NST;
      if (!mbar_wait(&full[s], (i / NST) & 1)) atomicOr(&g_status, 1u);
      const int st = vb + i * vg;
      int r0;
      const int g = seg_of(p, st, r0);
      const int row = r0 + rslot;
      float acc = 0.f;
      if (row < p.n[g]) {
        const uint8_t* wr = smem + s * stage_bytes + int64_t(rslot) * p.rb;
#pragma unroll
        for (int u = 0; u < kU; ++u)
          acc += q8::unit_dot<FMT>(wr + ((lane >> 2) + 8 * (half * kU + u)) * kChunkBytes, xu[u], pg, hsel, big);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
      __syncwarp();
      if (HALVES == 2 && half == 1) {
        if (lane == 0) {
          part[s * kRowWarps + rslot] = acc;
          mbar_arrive(&pair[s * kRowWarps + rslot]);   // release: the partial is visible to the row's first warp
          mbar_arrive(&empty[s]);
        }
      } else {
        if (HALVES == 2) {
          if (!mbar_wait(&pair[s * kRowWarps + rslot], (i / NST) & 1)) atomicOr(&g_status, 1u);
          acc += part[s * kRowWarps + rslot];
        }
        if (lane == 0) {
          mbar_arrive(&empty[s]);
          if (row < p.n[g]) p.y[g][row] = p.accumulate ? p.y[g][row] + acc : acc;
        }
      }
    }
  }
}

template <int FMT, int UPL, int HALVES, int RINGS, int XIN, int NST>
int launch_rows(RowArgs a, cudaStream_t s) {
  const int stage_bytes = int((int64_t(a.sr) * a.rb + 127) / 128 * 128);
  const int smem = RINGS * ring_bytes(stage_bytes, NST) + (XIN != kXinCodes ? xq_smem_bytes(a.k) : 0);
  constexpr int threads = 32 * RINGS * (1 + kRowWarps * HALVES);
  auto kern = k_mv_q8_rows<FMT, UPL, HALVES, RINGS, XIN, NST>;
  // the attribute and the occupancy query once per (device, shared-memory size): they cost host time on every call
  struct Entry {
    int dev, smem, per_sm, sms;
  };
  static Entry cache[16];
  static int ncache = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = 0, sms = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < ncache; ++i)
      if (cache[i].dev == dev && cache[i].smem == smem) {
        per_sm = cache[i].per_sm;
        sms = cache[i].sms;
      }
    if (per_sm == 0) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return LK_ECUDA;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
        return LK_ECUDA;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (ncache < 16) cache[ncache++] = Entry{dev, smem, per_sm, sms};
    }
  }
  cudaLaunchConfig_t cfg = {};
  // persistent: every resident CTA slot, once (no more CTAs than rings have stages)
  cfg.gridDim = dim3(min((a.nstages + RINGS - 1) / RINGS, sms * min(per_sm, kRowCtasPerSm)), 1, 1);
  a.prewait = kRowPreWait;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? LK_OK : LK_ECUDA;
}

// g_quant_q8: one warp per 32-value group, 8 groups per CTA
template <int XT>
__global__ void __launch_bounds__(256) k_quant_q8(int rows, int k, const void* x, int8_t* codes, float* meta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = k / 32;
  const int g = blockIdx.x * 8 + warp, row = blockIdx.y;
  griddep_launch();   // the next matvec may start streaming its weights now
  griddep_wait();     // x comes from the previous kernel
  if (g >= groups) return;
  const int64_t idx = int64_t(row) * k + g * 32 + lane;
  const float v = XT == LK_BF16 ? bf2f(static_cast<const uint16_t*>(x)[idx]) : static_cast<const float*>(x)[idx];
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  const float d = amax / 127.0f;
  int q = 0;
  if (amax > 0.0f) q = int(roundf(v / d));   // ordered compare: a NaN maximum gives code 0, like the reference
  codes[idx] = int8_t(q);
  int sum = q;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
  if (lane == 0) {
    float* m = meta + (int64_t(row) * groups + g) * 2;
    m[0] = __half2float(__float2half_rn(d));
    m[1] = float(sum);
  }
}

template <int FMT, int TOKB, int QR, int QS>
int launch_q8(const CUtensorMap& wm, const CUtensorMap& xm, const CUtensorMap& mm, const Q8Args& a, int row_tiles,
              cudaStream_t s) {
  constexpr int smem = q8_smem_bytes<TOKB, QR, QS>();
  static_assert(smem <= 227 * 1024, "chunked matvec CTA exceeds shared memory");
  auto kern = k_mv_q8<FMT, TOKB, QR, QS>;
  static unsigned configured = 0;
  if (!once_per_device(configured)) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, row_tiles, 1);
  cfg.blockDim = dim3(kQThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (a.splits > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = a.splits;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, wm, xm, mm, a) == cudaSuccess ? LK_OK : LK_ECUDA;
}

}  // namespace

int quant_q8(int rows, int k, const void* x, int x_dtype, uint8_t* xq, cudaStream_t s) {
  int8_t* codes = reinterpret_cast<int8_t*>(xq);
  float* meta = reinterpret_cast<float*>(xq + int64_t(rows) * k);
  dim3 grid((k / 32 + 7) / 8, rows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = x_dtype == LK_BF16 ? cudaLaunchKernelEx(&cfg, k_quant_q8<LK_BF16>, rows, k, x, codes, meta)
                                     : cudaLaunchKernelEx(&cfg, k_quant_q8<LK_F32>, rows, k, x, codes, meta);
  return e == cudaSuccess ? LK_OK : LK_ECUDA;
}

static bool rows_path(int fmt, int k, int tokens) {
  return (fmt == LK_Q4_K || fmt == LK_Q4_0) && tokens == 1 && k % 4096 == 0 && k <= 3 * 4096;
}

template <int XIN>
static int rows_dispatch(int fmt, int k, const RowArgs& ra, cudaStream_t s) {
  const bool q40 = fmt == LK_Q4_0;
  switch (k / 2048) {   // units (chunk, page) per lane
    case 2:
      return q40 ? launch_rows<LK_Q4_0, 2, 1, kRingsShort, XIN, kStagesShort>(ra, s)
                 : launch_rows<LK_Q4_K, 2, 1, kRingsShort, XIN, kStagesShort>(ra, s);
    case 4:
      return q40 ? launch_rows<LK_Q4_0, 4, 2, kRingsLong, XIN, kStagesLong>(ra, s)
                 : launch_rows<LK_Q4_K, 4, 2, kRingsLong, XIN, kStagesLong>(ra, s);
    case 6:
      return q40 ? launch_rows<LK_Q4_0, 6, 2, kRingsLong, XIN, kStagesLong>(ra, s)
                 : launch_rows<LK_Q4_K, 6, 2, kRingsLong, XIN, kStagesLong>(ra, s);
  }
  return LK_EUNSUPPORTED;
}

// xq: lk_quant_q8's buffer; or (xq == nullptr) x of x_dtype, quantised inside the matvec
static int mv_q8_rows(int fmt, int nseg, const int* ns, const void* const* ws, float* const* ys, int k, int accumulate,
                      const uint8_t* xq, cudaStream_t s, const void* x = nullptr, int x_dtype = LK_F32) {
  RowArgs ra{};
  ra.xq = xq;
  ra.x = x;
  ra.k = k;
  ra.accumulate = accumulate;
  ra.rb = int64_t(k) / 256 * kChunkBytes;   // Q4_K: k / 256 super-blocks; Q4_0: k / 32 blocks of 18 bytes, the same
  ra.sr = kRowWarps;
  ra.nseg = nseg;
  ra.start[0] = 0;
  for (int g = 0; g < nseg; ++g) {
    ra.w[g] = static_cast<const uint8_t*>(ws[g]);
    ra.y[g] = ys[g];
    ra.n[g] = ns[g];
    ra.start[g + 1] = ra.start[g] + (ns[g] + ra.sr - 1) / ra.sr;
  }
  ra.nstages = ra.start[nseg];
  if (xq) return rows_dispatch<kXinCodes>(fmt, k, ra, s);
  return x_dtype == LK_BF16 ? rows_dispatch<kXinBF16>(fmt, k, ra, s) : rows_dispatch<kXinF32>(fmt, k, ra, s);
}

// g_quant_q8 + g_mv_{fmt}_q8 of one token in one launch (the row-streaming kernel quantises x in its prologue)
int mv_q8_fused(int fmt, int nseg, const int* ns, const void* const* ws, float* const* ys, int k, int accumulate,
                const void* x, int x_dtype, cudaStream_t s) {
  if (!rows_path(fmt, k, 1) || nseg > kMaxSegs) return LK_EUNSUPPORTED;
  return mv_q8_rows(fmt, nseg, ns, ws, ys, k, accumulate, nullptr, s, x, x_dtype);
}

// Several weights sharing one activation (q | k | v of an attention layer): one launch over all their rows when the
// row-streaming kernel applies, else one launch each.
int mv_q8_multi(int fmt, int nseg, const int* ns, const void* const* ws, float* const* ys, int k, int tokens,
                int accumulate, const uint8_t* xq, cudaStream_t s) {
  if (rows_path(fmt, k, tokens) && nseg <= kMaxSegs) return mv_q8_rows(fmt, nseg, ns, ws, ys, k, accumulate, xq, s);
  for (int g = 0; g < nseg; ++g) {
    int rc = mv_q8(fmt, ns[g], k, tokens, accumulate, xq, ws[g], ys[g], s);
    if (rc != LK_OK) return rc;
  }
  return LK_OK;
}

int mv_q8(int fmt, int n, int k, int tokens, int accumulate, const uint8_t* xq, const void* w, float* y,
          cudaStream_t s) {
  if (fmt != LK_Q4_K && fmt != LK_Q4_0) return LK_EUNSUPPORTED;
  const int64_t rb = int64_t(k) / 256 * kChunkBytes;
  if (rows_path(fmt, k, tokens)) {
    const int ns[1] = {n};
    const void* ws[1] = {w};
    float* ys[1] = {y};
    return mv_q8_rows(fmt, 1, ns, ws, ys, k, accumulate, xq, s);
  }
  const int tokb = tokens <= 1 ? 1 : 8;
  CUtensorMap wm;
  const int qr = tokb == 1 ? kQRows1 : kQRows8;   // rows per tile (the weight box's height)
  int rc = make_map(&wm, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, n, rb / 4, kChunkBytes / 4, qr,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != LK_OK) return rc;
  Q8Args a{};
  a.n = n;
  a.k = k;
  a.accumulate = accumulate;
  a.nchunks = k / 256;
  const int row_tiles = (n + qr - 1) / qr;
  // split K until about one full wave of CTAs (one token: 6 per SM on 148 SMs; 8 tokens: 2 per SM), at most 8 CTAs
  // per cluster
  const int wave = tokb == 1 ? 888 : 296;
  int splits = (wave + row_tiles - 1) / row_tiles;
  splits = max(1, min(splits, min(8, a.nchunks)));
  a.cps = (a.nchunks + splits - 1) / splits;
  a.splits = (a.nchunks + a.cps - 1) / a.cps;
  const float* meta = reinterpret_cast<const float*>(xq + int64_t(tokens) * k);
  for (int t0 = 0; t0 < tokens; t0 += 8) {   // token tiles of 8 (one when tokens == 1)
    const int nt = min(8, tokens - t0);
    CUtensorMap xm, mm;
    rc = make_map(&xm, xq + int64_t(t0) * k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, nt, k, 256, tokb,
                  CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc == LK_OK)
      rc = make_map(&mm, meta + int64_t(t0) * (k / 16), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, nt, k / 16, 16, tokb,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != LK_OK) return rc;
    a.y = y + int64_t(t0) * n;
    a.ntok = nt;
    if (tokb == 1)
      rc = fmt == LK_Q4_K ? launch_q8<LK_Q4_K, 1, kQRows1, kQStages1>(wm, xm, mm, a, row_tiles, s)
                          : launch_q8<LK_Q4_0, 1, kQRows1, kQStages1>(wm, xm, mm, a, row_tiles, s);
    else
      rc = fmt == LK_Q4_K ? launch_q8<LK_Q4_K, 8, kQRows8, kQStages8>(wm, xm, mm, a, row_tiles, s)
                          : launch_q8<LK_Q4_0, 8, kQRows8, kQStages8>(wm, xm, mm, a, row_tiles, s);
    if (rc != LK_OK) return rc;
  }
  return LK_OK;
}

LK_STATUS_READER(status_q8)

}  // namespace lk
