// MXFP4 (split planes) weight x FP8 (e4m3) activation GEMM on the 5th-generation tensor cores with native block
// scaling: tcgen05.mma kind::mxf8f6f4.block_scale, e4m3 A, e2m1 B, one E8M0 scale per 32 k of every row.
//
// Replaces g_gemm_mxfp4s_{store,swiglu}[_pair]_f8_m256_rdna4 (gen_mxfp4s.py:50-500, launch signature gen_mxfp4s.py:101)
// and, grouped over the MoE tile schedule, the expert GEMMs of an MXFP4 MoE (gen_moe.py:1126-1228 layout).
//   y = (x8 . (W * 2^8)^T) * s8[row][1]   (the reference holds W at 2^8 times its value; s8[row][1] carries 2^-8)
// The reference decodes every nibble to an e5m2 byte and is exact only for block exponents 107..132
// (gen_mxfp4s.py:14-27); here the tensor core applies the block scales itself, exact for every E8M0 value.
//
// One CTA computes a 128-row x 256-column tile (swiglu: 128 columns of gate and of up), K in steps of 128:
//   warp 0      producer: A (x8) tiles by 2-D TMA with 128-byte swizzle (MoE gate/up: TMA gather4 of token rows), the
//               packed nibble rows (64 bytes per row per step) by 2-D TMA; out-of-range k is zero-filled by TMA
//   warp 1      allocates TMEM; copies scale factors into TMEM (tcgen05.cp 32x128b.warpx4) and issues the MMAs
//   warps 2-9   expand each packed row into the operand layout the MMA reads e2m1 from (16 values in the first 8 of
//               every 16 bytes, 128-byte swizzle; split16 blocks reordered to pairs), stage the row's four E8M0
//               bytes in the scale-factor atom (row 32j+i at byte 16i+4j), then run the epilogue.
#include "lk_common.cuh"
#include "lk_internal.h"

#include <algorithm>

namespace lk {

int make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, int64_t rows, int64_t cols,
             int box_cols, int box_rows, CUtensorMapSwizzle swz);
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
                 const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* estr, CUtensorMapSwizzle swz);

namespace {

constexpr int kBM = 128, kBK = 128;               // tile rows, k per stage (bytes of e4m3 A per row)
constexpr int kSA = 4, kSP = 3, kSB = 2;
constexpr int kXWarps = 8;
constexpr int kThreads = (2 + kXWarps) * 32;
constexpr int kRowsB = 256;                       // weight rows per tile (x NW weights)
constexpr int kABytes = kBM * kBK;                // 16 KB
constexpr int kPBytes = kRowsB * (kBK / 2);       // 16 KB of packed nibbles
constexpr int kBBytes = kRowsB * kBK;             // 32 KB expanded operand
constexpr int kSFBytes = kRowsB * 4;              // 1 KB: two 512-byte scale-factor atoms
constexpr uint32_t kColSFA = 256, kColSFB = 264;  // TMEM columns: accumulators 0..255, SFA 4, SFB 8 per stage
enum { kDense = 0, kGather = 1, kSorted = 2 };

struct MxArgs {
  const float* s8;              // [rows or xrows][2]
  float* y;                     // [rows][n]
  const uint8_t* ws;            // E8M0 plane of w  [rows of wmap][k/32]
  const uint8_t* ws2;           // E8M0 plane of w2 (or ws when fused)
  int rows, k, n;
  int sf_stride;                // bytes per scale row (k/32)
  int rows_per_expert, rows_per_expert2, w2_row_offset;
  const int32_t* tile_info;
  const int32_t* rowmap;
  int max_tiles, xrows, ku, n_experts;
  ExpertEpi epi;                // gate/up activation and per-expert biases (bias index: expert * n + column)
};

// The epilogue of 32 columns of one row: row scale, then act(g + bg, u + bu) (gate/up) or + bd (single weight), the
// biases of columns c0 .. c0 + 31 read where c0 + i < ncols (bias rows: the expert's, already offset)
template <int NW>
LK_DEV void mx_epilogue32(float (&v)[32], const float (&u)[32], float inv, const ExpertEpi& epi, const float* bcol,
                          const float* b2col, int c0, int ncols) {
  if (NW == 2) {
    if (bcol) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const bool in = c0 + i < ncols;
        v[i] = act_apply(epi.act, fmaf(v[i], inv, in ? __ldg(bcol + c0 + i) : 0.f),
                         fmaf(u[i], inv, in ? __ldg(b2col + c0 + i) : 0.f), epi.alpha, epi.limit);
      }
    } else if (epi.act != LK_ACT_SILU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = act_apply(epi.act, v[i] * inv, u[i] * inv, epi.alpha, epi.limit);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = silu(v[i] * inv) * (u[i] * inv);
    }
  } else if (bcol) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = fmaf(v[i], inv, c0 + i < ncols ? __ldg(bcol + c0 + i) : 0.f);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= inv;
  }
}

// split16 block bytes (element i low nibble of byte i, element i+16 high nibble) -> pairs order (element 2j low,
// 2j+1 high nibble of byte j), for one 32-value block held in 4 words
LK_DEV void split16_to_pairs(uint32_t (&w)[4]) {
  uint32_t e0 = prmt(w[0], w[1], 0x6420u), o0 = prmt(w[0], w[1], 0x7531u);   // even / odd bytes 0..7
  uint32_t e1 = prmt(w[2], w[3], 0x6420u), o1 = prmt(w[2], w[3], 0x7531u);   // even / odd bytes 8..15
  uint32_t lo0 = (e0 & 0x0F0F0F0Fu) | ((o0 & 0x0F0F0F0Fu) << 4), lo1 = (e1 & 0x0F0F0F0Fu) | ((o1 & 0x0F0F0F0Fu) << 4);
  uint32_t hi0 = ((e0 >> 4) & 0x0F0F0F0Fu) | (o0 & 0xF0F0F0F0u), hi1 = ((e1 >> 4) & 0x0F0F0F0Fu) | (o1 & 0xF0F0F0F0u);
  w[0] = lo0;
  w[1] = lo1;
  w[2] = hi0;
  w[3] = hi1;
}

template <int NW, int GROUP, int ORDER>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_mx(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
              const __grid_constant__ CUtensorMap w2map, const MxArgs p) {
  constexpr int BN = kRowsB / NW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + kSA * kABytes;
  uint8_t* sP = sB + kSB * kBBytes;
  uint8_t* sSF = sP + kSP * kPBytes;          // [kSB][1024]
  uint8_t* sSFA = sSF + kSB * kSFBytes;       // 512 bytes of 127 (2^0): the activations' block scales
  uint64_t* full_a = reinterpret_cast<uint64_t*>(sSFA + 512);
  uint64_t* empty_a = full_a + kSA;
  uint64_t* full_p = empty_a + kSA;
  uint64_t* empty_p = full_p + kSP;
  uint64_t* full_b = empty_p + kSP;
  uint64_t* empty_b = full_b + kSB;
  uint64_t* acc_full = empty_b + kSB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  int* tile_meta = reinterpret_cast<int*>(tmem_slot + 4);
  int* arow = tile_meta + 4;   // [128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int kstages = (p.k + kBK - 1) / kBK;
  const int kblocks = p.k / 32;
  int m0 = blockIdx.y * kBM;
  int valid_rows = min(kBM, p.rows - m0);
  int expert = 0;
  if (GROUP != kDense) {
    // super-tile s = blockIdx.y (the A ring is free scratch until the first TMA load)
    moe_super_tile(p.tile_info, p.max_tiles, p.n_experts, blockIdx.y, reinterpret_cast<int*>(sA), tile_meta);
    if (tile_meta[0] < 0) return;
    expert = min(tile_meta[0], p.n_experts - 1);
    m0 = tile_meta[1] * 64;
    valid_rows = tile_meta[2];
    if (GROUP == kGather && threadIdx.x < kBM) {
      int r = threadIdx.x;
      int a = r < valid_rows ? p.rowmap[m0 + r] : -1;
      arow[r] = a >= 0 ? a / p.ku : p.xrows;
    }
  }
  const int wrow = expert * p.rows_per_expert + n0;
  const int w2row = expert * p.rows_per_expert2 + p.w2_row_offset + n0;
  const int nb_rows = min(BN, p.n - n0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSA; ++i) {
      mbar_init(&full_a[i], 1);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < kSP; ++i) {
      mbar_init(&full_p[i], 1);
      mbar_init(&empty_p[i], kXWarps);
    }
    for (int i = 0; i < kSB; ++i) {
      mbar_init(&full_b[i], kXWarps);
      mbar_init(&empty_b[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (threadIdx.x >= 64 && threadIdx.x < 64 + 128) reinterpret_cast<uint32_t*>(sSFA)[threadIdx.x - 64] = 0x7F7F7F7Fu;
  fence_proxy_async();
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
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
    for (int ks = 0; ks < kstages; ++ks) {
      int sp = ks % kSP, sa = ks % kSA;
      if (ks >= kSP && !mbar_wait(&empty_p[sp], ((ks / kSP) - 1) & 1)) atomicOr(&g_status, 1u);
      if (lane == 0) {
        mbar_expect_tx(&full_p[sp], uint32_t(kPBytes));
        tma_load_2d(sP + sp * kPBytes, &wmap, ks * (kBK / 2), wrow, &full_p[sp]);
        if (NW == 2) tma_load_2d(sP + sp * kPBytes + BN * (kBK / 2), &w2map, ks * (kBK / 2), w2row, &full_p[sp]);
      }
      if (ks >= kSA && !mbar_wait(&empty_a[sa], ((ks / kSA) - 1) & 1)) atomicOr(&g_status, 1u);
      if (GROUP == kGather) {
        if (lane == 0) mbar_expect_tx(&full_a[sa], kABytes);
        __syncwarp();
        int r = lane * 4;
        tma_gather4(sA + sa * kABytes + r * 128, &amap, ks * kBK, arow[r], arow[r + 1], arow[r + 2], arow[r + 3],
                    &full_a[sa]);
      } else if (lane == 0) {
        mbar_expect_tx(&full_a[sa], kABytes);
        tma_load_2d(sA + sa * kABytes, &amap, ks * kBK, m0, &full_a[sa]);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ scale-factor copies + MMA issue
    const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
    if (lane == 0) tmem_cp_32x128_x4(tmem + kColSFA, sdesc_rows16(smem_u32(sSFA)));
    for (int ks = 0; ks < kstages; ++ks) {
      int sa = ks % kSA, sb = ks % kSB;
      if (!mbar_wait(&full_a[sa], (ks / kSA) & 1)) atomicOr(&g_status, 1u);
      if (!mbar_wait(&full_b[sb], (ks / kSB) & 1)) atomicOr(&g_status, 1u);
      tc_fence_after();
      if (lane == 0) {
        const uint32_t sfb = tmem + kColSFB + 8 * sb;
        tmem_cp_32x128_x4(sfb, sdesc_rows16(smem_u32(sSF + sb * kSFBytes)));
        tmem_cp_32x128_x4(sfb + 4, sdesc_rows16(smem_u32(sSF + sb * kSFBytes + 512)));
#pragma unroll
        for (int s = 0; s < kBK / 32; ++s) {
          uint64_t ad = sdesc_k128(a_base + sa * kABytes + s * 32);
#pragma unroll
          for (int wi = 0; wi < NW; ++wi) {
            uint64_t bd = sdesc_k128(b_base + sb * kBBytes + wi * BN * 128 + s * 32);
            uint32_t idesc = idesc_mx(kBM, BN, 0, 5, s, s);
            umma_mx(tmem + wi * BN, ad, bd, idesc, (tmem + kColSFA) | (uint32_t(s) << 30),
                    (sfb + 4 * wi) | (uint32_t(s) << 30), (ks | s) != 0);
          }
        }
        umma_commit(&empty_a[sa]);
        umma_commit(&empty_b[sb]);
        if (ks == kstages - 1) umma_commit(acc_full);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------------ operand expansion + scales, then epilogue
    const int r = threadIdx.x - 64;   // tile weight row 0..255
    const int wi = r / BN, rr = r % BN;
    const bool row_ok = n0 + rr < p.n;
    const uint8_t* sfrow = (wi ? p.ws2 : p.ws) + int64_t((wi ? w2row : wrow) + rr) * p.sf_stride;
    // block visiting order: q ^ perm[(r >> 1) & 3] with perm = {0, 2, 3, 1} (x -> alpha.x in GF(4)); both the
    // 64-byte-strided row reads and the swizzled chunk writes of 8 consecutive rows then hit 8 distinct bank groups
    const int qperm = (0x1320 >> (4 * ((r >> 1) & 3))) & 3;
    auto load_sf = [&](int ks) -> uint32_t {
      uint32_t v = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int b = ks * 4 + i;
        uint32_t e = (row_ok && b < kblocks) ? uint32_t(__ldg(sfrow + b)) : 0x7Fu;
        v |= e << (8 * i);
      }
      return v;
    };
    // the scale bytes of stage ks + kSfAhead are requested while stage ks is expanded (a register ring: the loads'
    // latency spans kSfAhead stages instead of one)
    constexpr int kSfAhead = 4;
    uint32_t sfr[kSfAhead];
#pragma unroll
    for (int j = 0; j < kSfAhead; ++j) sfr[j] = load_sf(j);
    for (int ks0 = 0; ks0 < kstages; ks0 += kSfAhead) {
#pragma unroll
      for (int j = 0; j < kSfAhead; ++j) {
        const int ks = ks0 + j;
        if (ks >= kstages) break;
        int sp = ks % kSP, sb = ks % kSB;
        if (!mbar_wait(&full_p[sp], (ks / kSP) & 1)) atomicOr(&g_status, 1u);
        if (ks >= kSB && !mbar_wait(&empty_b[sb], ((ks / kSB) - 1) & 1)) atomicOr(&g_status, 1u);
        const uint4* prow = reinterpret_cast<const uint4*>(sP + sp * kPBytes + r * (kBK / 2));
        uint8_t* bt = sB + sb * kBBytes;
#pragma unroll
        for (int qi = 0; qi < 4; ++qi) {   // 16 packed bytes = one 32-value block = two 16-value chunks
          const int q = qi ^ qperm;
          uint4 v = prow[q];
          uint32_t w[4] = {v.x, v.y, v.z, v.w};
          if (ORDER == LK_ORDER_SPLIT16) split16_to_pairs(w);
          *reinterpret_cast<uint4*>(bt + sw128(r, 2 * q)) = make_uint4(w[0], w[1], 0u, 0u);
          *reinterpret_cast<uint4*>(bt + sw128(r, 2 * q + 1)) = make_uint4(w[2], w[3], 0u, 0u);
        }
        // scale-factor atom: row 32j + i of a 128-row half at byte 16i + 4j, the four k blocks in its four bytes
        *reinterpret_cast<uint32_t*>(sSF + sb * kSFBytes + (r >> 7) * 512 + 16 * (r & 31) + 4 * ((r & 127) >> 5)) =
            sfr[j];
        sfr[j] = load_sf(ks + kSfAhead);   // past the last block: 127 (2^0) without a load
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&full_b[sb]);
          mbar_arrive(&empty_p[sp]);
        }
      }
    }
    // epilogue: quadrant q = TMEM lanes 32q..; the two warps of a quadrant split the columns
    if (!mbar_wait(acc_full, 0)) atomicOr(&g_status, 1u);
    tc_fence_after();
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int row = 32 * q + lane;
    const bool ok = row < valid_rows;
    // rows stored: a MoE super-tile's whole 64-row tiles, padding rows included (act of the biases, zero without)
    const bool store = GROUP == kDense ? ok : row < (valid_rows > 64 ? 128 : 64);
    float inv = 0.f;
    float* yrow = store ? p.y + int64_t(m0 + row) * p.n + n0 : nullptr;
    if (ok) {
      int grow = m0 + row;
      int srow = grow;
      if (GROUP == kGather) {
        int a = p.rowmap[grow];
        srow = a >= 0 ? a / p.ku : -1;
      }
      inv = srow >= 0 ? p.s8[2 * int64_t(srow) + 1] * 256.0f : 0.f;   // 2^8: the reference's weight pre-scale
    }
    const float* bcol = p.epi.bias ? p.epi.bias + int64_t(expert) * p.n + n0 : nullptr;
    const float* b2col = p.epi.bias2 ? p.epi.bias2 + int64_t(expert) * p.n + n0 : nullptr;
    constexpr int kCols = BN / 2;
    const uint32_t tbase = tmem + (uint32_t(32 * q) << 16);
#pragma unroll 1
    for (int cb = 0; cb < kCols; cb += 32) {
      int col = half * kCols + cb;
      float v[32], u[32];
      tmem_ld32(tbase + col, v);
      if (NW == 2) tmem_ld32(tbase + BN + col, u);
      mx_epilogue32<NW>(v, u, inv, p.epi, bcol, b2col, col, nb_rows);
      if (store) {
        if ((p.n & 3) == 0) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            if (col + i < nb_rows)
              *reinterpret_cast<float4*>(yrow + col + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (col + i < nb_rows) yrow[col + i] = v[i];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int NW, int GROUP, int ORDER>
int launch(const CUtensorMap& am, const CUtensorMap& wm, const CUtensorMap& w2m, const MxArgs& a, dim3 grid,
           cudaStream_t s) {
  constexpr int smem = 1024 + kSA * kABytes + kSB * kBBytes + kSP * kPBytes + kSB * kSFBytes + 512 + 256 + 32 + 512;
  static_assert(smem <= 227 * 1024, "MXFP4 GEMM CTA exceeds shared memory");
  auto kern = k_gemm_mx<NW, GROUP, ORDER>;
  static unsigned configured = 0;
  if (!once_per_device(configured)) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  kern<<<grid, kThreads, smem, s>>>(am, wm, w2m, a);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

template <int NW, int GROUP>
int launch_o(int order, const CUtensorMap& am, const CUtensorMap& wm, const CUtensorMap& w2m, const MxArgs& a,
             dim3 grid, cudaStream_t s) {
  if (order == LK_ORDER_SPLIT16) return launch<NW, GROUP, LK_ORDER_SPLIT16>(am, wm, w2m, a, grid, s);
  return launch<NW, GROUP, LK_ORDER_PAIRS>(am, wm, w2m, a, grid, s);
}

// ---------------------------------------------------------------------------------------------------------------
// Persistent dense MXFP4 x e4m3 GEMM for pairs-order nibbles: the tensor map unpacks the e2m1 operand itself.
//
// A TMA load of data type 16U4_ALIGN16B writes every 16 packed nibbles into the first 8 bytes of a 16-byte slot and
// leaves the other 8 alone: the layout kind::mxf8f6f4 reads e2m1 from. With the 128-byte swizzle the packed weight
// rows land in the MMA's K-major operand layout directly, so no warps rewrite them (the transaction count is the
// packed size). The map's K extent must be a multiple of 128 values: k = 128 q + 64 runs q stages over the first
// 128 q values and one tail stage over the LAST 128 values (a second map based (k - 128) / 2 bytes into each row),
// whose first 64 values, already counted, are skipped by starting that stage's MMAs at sub-step 2.
//
// One CTA per SM walks output tiles of 128 rows x 192 weight rows (swiglu: 96 gate + 96 up rows, one N = 192 MMA per
// 32 k) into two TMEM accumulators, so the epilogue of a tile overlaps the accumulation of the next. Grouped over the
// MoE schedule a tile's rows are one 128-row super-tile of an expert (its table built in shared memory at start):
// gate/up gathers the token rows of x8 by TMA gather4, down reads the sorted rows.
//   warp 0     TMA producer: A box 128 x 128 bytes (e4m3, 128-byte swizzle) and the weight boxes, unpacked
//   warp 1     TMEM owner; per stage copies the weights' scale-factor atoms into TMEM and issues the MMAs
//   warps 2-3  stage the E8M0 bytes of every weight row in the scale-factor atom (row 32j + i at byte 16i + 4j),
//              their loads issued kMxpSfAhead stages ahead of use
//   warps 4-7  epilogue: TMEM lane quarter w % 4, row scale, silu(g) * u or the plain product; each warp's 32 x 32
//              f32 blocks go through a 128-byte-swizzled shared tile and one TMA store (rows the tile does not
//              own, in a partly filled MoE super-tile, are stored by the threads instead)
// ---------------------------------------------------------------------------------------------------------------
constexpr int kMxpNT = 192;                  // weight rows per tile = accumulator columns
constexpr int kMxpS = 4;                     // stages (5 measured the same)
constexpr int kMxpA = kBM * kBK;             // 16 KB of e4m3
constexpr int kMxpB = kMxpNT * kBK;          // 24 KB of unpacked e2m1
constexpr int kMxpBtx = kMxpNT * kBK / 2;    // 12 KB of packed nibbles: the weight boxes' transaction bytes
constexpr int kMxpSF = 1024;                 // two scale-factor atoms: weight rows 0..127 and 128..255
constexpr int kMxpThreads = 256;
constexpr int kMxpSfAhead = 4;
constexpr uint32_t kMxpAcc1 = 256, kMxpColSFA = 192, kMxpColSFB = 200;   // TMEM: acc 0..191 / 256..447, scales
constexpr int kMxpStg = 4 * 32 * 32 * 4;     // epilogue staging: a 32 x 32 f32 block per epilogue warp
constexpr int kMxpSmem =
    1024 + kMxpS * (kMxpA + kMxpB + kMxpSF) + kMxpStg + 512 + 8 * (3 * kMxpS + 4) + 16 + 3 * kMaxExperts * 4;
static_assert(kMxpSmem <= 227 * 1024, "persistent MXFP4 GEMM CTA exceeds shared memory");
static_assert(kMxpColSFB + 8 * kMxpS <= kMxpAcc1, "scale-factor columns overlap the second accumulator");

struct MxpArgs {
  const float* s8;        // [rows][2]
  float* y;               // [rows][n]
  const uint8_t* ws;      // E8M0 plane of w  [n][k/32]
  const uint8_t* ws2;     // E8M0 plane of w2
  int rows, k, n;
  int sf_stride;          // k / 32
  int kmain;              // stages over the first 128 * kmain values
  int tail_sub;           // first MMA sub-step of the tail stage; 4 = no tail stage
  int m_tiles, n_tiles;   // dense: row tiles; grouped: m_tiles unused (super-tiles counted on the device)
  // grouped over the MoE schedule
  const int32_t* tile_info;
  const int32_t* rowmap;
  int max_tiles, xrows, ku, n_experts;
  int rows_per_expert, rows_per_expert2, w2_row_offset;
  ExpertEpi epi;          // gate/up activation and per-expert biases (bias index: expert * n + column)
};

template <int NW, int GROUP>
__global__ void __launch_bounds__(kMxpThreads, 1)
    k_gemm_mxp(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
               const __grid_constant__ CUtensorMap w2map, const __grid_constant__ CUtensorMap wtmap,
               const __grid_constant__ CUtensorMap w2tmap, const __grid_constant__ CUtensorMap ymap, const MxpArgs p) {
  constexpr int BNW = kMxpNT / NW;   // columns of each weight per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + kMxpS * kMxpA;
  uint8_t* sSF = sB + kMxpS * kMxpB;       // [kMxpS][1024]
  float* sStg = reinterpret_cast<float*>(sSF + kMxpS * kMxpSF);   // [4][32][32] f32, 1024-byte aligned
  uint8_t* sSFA = sSF + kMxpS * kMxpSF + kMxpStg;   // 512 bytes of 127 (2^0): the activations' block scales
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFA + 512);
  uint64_t* sfull = full + kMxpS;
  uint64_t* empty = sfull + kMxpS;
  uint64_t* accf = empty + kMxpS;          // [2]
  uint64_t* acce = accf + 2;               // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  int* stbl = reinterpret_cast<int*>(tmem_slot + 4);   // [3][kMaxExperts]: the MoE super-tile table

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nks = p.kmain + (p.tail_sub < 4 ? 1 : 0);
  const int msup = GROUP == kDense ? p.m_tiles : moe_super_table(p.tile_info, p.max_tiles, p.n_experts, stbl);
  const int ntiles = msup * p.n_tiles;
  const int my_tiles = int(blockIdx.x) < ntiles ? (ntiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
  // tile t: rows m0 .. m0 + vrows - 1 (dense: of x8 / y; grouped: sorted positions of expert `e`), columns n0 ..
  auto tile_of = [&](int t, int& m0, int& vrows, int& e, int& n0) {
    const int mt = t / p.n_tiles;
    n0 = (t - mt * p.n_tiles) * BNW;
    if (GROUP == kDense) {
      m0 = mt * kBM;
      vrows = min(kBM, p.rows - m0);
      e = 0;
    } else {
      int first;
      moe_super_lookup(p.tile_info, stbl, mt, e, first, vrows);
      e = min(max(e, 0), p.n_experts - 1);
      m0 = first * 64;
    }
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMxpS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&sfull[i], 2);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 4);
    }
    fence_mbar_init();
  }
  // the TMA never writes the 8-byte gaps of the unpacked weight tiles: zero them once; unused scale rows = 2^0
  for (int i = threadIdx.x; i < kMxpS * kMxpB / 16; i += kMxpThreads)
    reinterpret_cast<uint4*>(sB)[i] = make_uint4(0u, 0u, 0u, 0u);
  for (int i = threadIdx.x; i < kMxpS * kMxpSF / 4; i += kMxpThreads) reinterpret_cast<uint32_t*>(sSF)[i] = 0x7F7F7F7Fu;
  if (threadIdx.x < 128) reinterpret_cast<uint32_t*>(sSFA)[threadIdx.x] = 0x7F7F7F7Fu;
  fence_proxy_async();
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer (gather: every lane, 4 rows each)
    if (lane == 0) {
      prefetch_tensormap(&amap);
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&wtmap);
      if (NW == 2) {
        prefetch_tensormap(&w2map);
        prefetch_tensormap(&w2tmap);
      }
    }
    uint32_t g = 0;
    for (int ti = 0; ti < my_tiles; ++ti) {
      const int t = int(blockIdx.x) + ti * int(gridDim.x);
      int m0, vrows, e, n0;
      tile_of(t, m0, vrows, e, n0);
      const int wrow = e * p.rows_per_expert + n0;
      const int w2row = e * p.rows_per_expert2 + p.w2_row_offset + n0;
      int arow[4];   // gather: the token rows of tile rows 4 lane .. 4 lane + 3 (xrows: past the end, zero-filled)
      if (GROUP == kGather) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = 4 * lane + i;
          const int a = r < vrows ? __ldg(p.rowmap + m0 + r) : -1;
          arow[i] = a >= 0 ? a / p.ku : p.xrows;
        }
      }
      for (int ks = 0; ks < nks; ++ks, ++g) {
        const int s = int(g % kMxpS);
        if (g >= uint32_t(kMxpS) && !mbar_wait(&empty[s], ((g / kMxpS) - 1) & 1)) atomicOr(&g_status, 1u);
        const bool tail = ks == p.kmain;
        const int ka = tail ? p.k - kBK : ks * kBK;
        if (lane == 0) {
          mbar_expect_tx(&full[s], uint32_t(kMxpA + kMxpBtx));
          if (GROUP != kGather) tma_load_2d(sA + s * kMxpA, &amap, ka, m0, &full[s]);
          uint8_t* b = sB + s * kMxpB;
          tma_load_2d(b, tail ? &wtmap : &wmap, tail ? 0 : ks * kBK, wrow, &full[s]);
          if (NW == 2) tma_load_2d(b + BNW * kBK, tail ? &w2tmap : &w2map, tail ? 0 : ks * kBK, w2row, &full[s]);
        }
        __syncwarp();
        if (GROUP == kGather)
          tma_gather4(sA + s * kMxpA + 4 * lane * kBK, &amap, ka, arow[0], arow[1], arow[2], arow[3], &full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ scale-factor copies + MMA issue
    if (lane == 0) tmem_cp_32x128_x4(tmem + kMxpColSFA, sdesc_rows16(smem_u32(sSFA)));
    uint32_t g = 0;
    for (int ti = 0; ti < my_tiles; ++ti) {
      const int b = ti & 1;
      if (ti >= 2 && !mbar_wait(&acce[b], ((ti >> 1) - 1) & 1)) atomicOr(&g_status, 1u);
      tc_fence_after();
      const uint32_t acc = tmem + uint32_t(b) * kMxpAcc1;
      for (int ks = 0; ks < nks; ++ks, ++g) {
        const int s = int(g % kMxpS);
        const uint32_t ph = (g / kMxpS) & 1;
        if (!mbar_wait(&full[s], ph)) atomicOr(&g_status, 1u);
        if (!mbar_wait(&sfull[s], ph)) atomicOr(&g_status, 1u);
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sfb = tmem + kMxpColSFB + 8 * s;
          tmem_cp_32x128_x4(sfb, sdesc_rows16(smem_u32(sSF + s * kMxpSF)));
          tmem_cp_32x128_x4(sfb + 4, sdesc_rows16(smem_u32(sSF + s * kMxpSF + 512)));
          const int s0 = ks == p.kmain ? p.tail_sub : 0;
          const uint32_t a_base = smem_u32(sA + s * kMxpA), b_base = smem_u32(sB + s * kMxpB);
#pragma unroll
          for (int j = 0; j < kBK / 32; ++j) {
            if (j < s0) continue;
            umma_mx(acc, sdesc_k128(a_base + j * 32), sdesc_k128(b_base + j * 32), idesc_mx(kBM, kMxpNT, 0, 5, j, j),
                    (tmem + kMxpColSFA) | (uint32_t(j) << 30), sfb | (uint32_t(j) << 30), (ks | (j - s0)) != 0);
          }
          umma_commit(&empty[s]);
          if (ks == nks - 1) umma_commit(&accf[b]);
        }
        __syncwarp();
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------------ E8M0 scale staging
    const int jt = threadIdx.x - 64;   // tile weight rows jt, jt + 64, jt + 128
    const int total = my_tiles * nks;
    // two 16-bit loads per row per stage (row stride k/32 and block offsets are even); beyond the CTA's last stage
    // or past n: 2^0 without a load
    int cur_t = -1, wrow = 0, w2row = 0, n0 = 0;   // the tile whose weight rows are cached
    auto issue = [&](int q, uint32_t (&v)[3][2]) {
      const int ti = q / nks, ks = q - ti * nks;
      const int t = int(blockIdx.x) + ti * int(gridDim.x);
      if (q < total && t != cur_t) {
        int m0, vrows, e;
        tile_of(t, m0, vrows, e, n0);
        wrow = e * p.rows_per_expert + n0;
        w2row = e * p.rows_per_expert2 + p.w2_row_offset + n0;
        cur_t = t;
      }
      const int b0 = ks < p.kmain ? 4 * ks : (p.k - kBK) / 32;
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        const int r = jt + 64 * i;
        const int wi = r / BNW, rr = r - wi * BNW;
        const bool ok = q < total && n0 + rr < p.n;
        const uint16_t* src = reinterpret_cast<const uint16_t*>((wi ? p.ws2 : p.ws) +
                                                                int64_t((wi ? w2row : wrow) + rr) * p.sf_stride + b0);
        v[i][0] = ok ? uint32_t(__ldg(src)) : 0x7F7Fu;
        v[i][1] = ok ? uint32_t(__ldg(src + 1)) : 0x7F7Fu;
      }
    };
    uint32_t ring[kMxpSfAhead][3][2];
#pragma unroll
    for (int a = 0; a < kMxpSfAhead; ++a) issue(a, ring[a]);
    for (int q0 = 0; q0 < total; q0 += kMxpSfAhead) {
#pragma unroll
      for (int a = 0; a < kMxpSfAhead; ++a) {
        const int q = q0 + a;
        if (q < total) {
          const int s = q % kMxpS;
          if (q >= kMxpS && !mbar_wait(&empty[s], ((q / kMxpS) - 1) & 1)) atomicOr(&g_status, 1u);
          uint8_t* atom = sSF + s * kMxpSF;
#pragma unroll
          for (int i = 0; i < 3; ++i) {
            const int r = jt + 64 * i;
            *reinterpret_cast<uint32_t*>(atom + (r >> 7) * 512 + 16 * (r & 31) + 4 * ((r & 127) >> 5)) =
                ring[a][i][0] | (ring[a][i][1] << 16);
          }
          issue(q + kMxpSfAhead, ring[a]);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sfull[s]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (TMEM lanes 32 (w % 4) ..)
    const int qd = warp & 3;
    float* stg = sStg + qd * 1024;
    if (lane == 0) prefetch_tensormap(&ymap);
    for (int ti = 0; ti < my_tiles; ++ti) {
      const int t = int(blockIdx.x) + ti * int(gridDim.x);
      const int b = ti & 1;
      int m0, vrows, e, n0;
      tile_of(t, m0, vrows, e, n0);
      const int r = 32 * qd + lane;
      const bool ok = r < vrows;
      // rows stored: a MoE super-tile's whole 64-row tiles (padding rows give act of the biases, zero without)
      const int srows = GROUP == kDense ? vrows : (vrows > 64 ? 128 : 64);
      const float* bcol = p.epi.bias ? p.epi.bias + int64_t(e) * p.n + n0 : nullptr;
      const float* b2col = p.epi.bias2 ? p.epi.bias2 + int64_t(e) * p.n + n0 : nullptr;
      const int row = m0 + r;   // output row (grouped: sorted position)
      int srow = row;           // its activation scale row (gather: the token)
      if (GROUP == kGather && ok) {
        const int a = __ldg(p.rowmap + row);
        srow = a >= 0 ? a / p.ku : -1;
      }
      const float inv = ok && srow >= 0 ? __ldg(p.s8 + 2 * int64_t(srow) + 1) * 256.0f : 0.f;   // 2^8: weight pre-scale
      if (!mbar_wait(&accf[b], (ti >> 1) & 1)) atomicOr(&g_status, 1u);
      tc_fence_after();
      float* yrow = p.y + int64_t(ok ? row : 0) * p.n + n0;
      const uint32_t tb = tmem + uint32_t(b) * kMxpAcc1 + (uint32_t(32 * qd) << 16);
#pragma unroll 1
      for (int c = 0; c < BNW; c += 32) {
        float v[32], u[32];
        tmem_ld32(tb + c, v);
        if (NW == 2) tmem_ld32(tb + BNW + c, u);
        mx_epilogue32<NW>(v, u, inv, p.epi, bcol, b2col, c, p.n - n0);
        if (c + 32 >= BNW) {   // the tile's last TMEM read is done: hand the accumulator back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce[b]);
        }
        // the TMA store clips rows past p.rows and columns past n; a grouped super-tile owns its whole 64-row tiles
        // (srows, a multiple of 32), the rows past them belong to the next super-tile: its warps past srows store
        // nothing
        if (GROUP != kDense && 32 * qd >= srows) continue;
        if (GROUP == kDense || 32 * qd + 31 < srows) {
          if (m0 + 32 * qd >= p.rows || n0 + c >= p.n) continue;   // nothing of this block is in the output
          if (lane == 0) bulk_wait_group_read0();   // this warp's previous block has left the staging tile
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i)   // 16-byte chunk i of row `lane` at chunk i ^ (lane % 8): the 128-byte swizzle
            *reinterpret_cast<float4*>(stg + lane * 32 + ((i ^ (lane & 7)) << 2)) =
                make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&ymap, stg, n0 + c, m0 + 32 * qd);
            bulk_commit_group();
          }
        } else if (ok) {
          if ((p.n & 3) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              if (n0 + c + i < p.n)
                *reinterpret_cast<float4*>(yrow + c + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (n0 + c + i < p.n) yrow[c + i] = v[i];
          }
        }
      }
    }
    if (lane == 0) bulk_wait_group0();   // every TMA store of this warp has completed
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// 2-D map over MXFP4 nibble rows that unpacks 16 values per 16-byte slot: `vals` values per row from `base`, rows
// `row_bytes` apart, boxes of 128 values x box_rows rows, 128-byte swizzle
int make_map_u4(CUtensorMap* map, const void* base, int64_t rows, int64_t vals, int64_t row_bytes, int box_rows) {
  cuuint64_t dims[2] = {cuuint64_t(vals), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(row_bytes)};
  cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, base, dims, strides, box, estr,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

// the persistent kernel's conditions: dense, pairs order, k a multiple of 64 (at least 128), 32-byte aligned planes
// the persistent kernel's conditions: pairs order, k a multiple of 64 (at least 128), 32-byte aligned nibble planes,
// 2-byte aligned scale planes
bool mxp_applies(int order, int k, const uint8_t* w, const uint8_t* ws, const uint8_t* w2, const uint8_t* w2s) {
  auto al = [](const void* q, uintptr_t b) { return (reinterpret_cast<uintptr_t>(q) & (b - 1)) == 0; };
  return order == LK_ORDER_PAIRS && k >= kBK && k % 64 == 0 && al(w, 32) && al(ws, 2) && (!w2 || al(w2, 32)) &&
         (!w2s || al(w2s, 2));
}

template <int NW, int GROUP>
int launch_mxp(const CUtensorMap* m, const MxpArgs& a, int grid, cudaStream_t s) {
  auto kern = k_gemm_mxp<NW, GROUP>;
  static unsigned configured = 0;
  if (!once_per_device(configured)) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMxpSmem);
  kern<<<grid, kMxpThreads, kMxpSmem, s>>>(m[0], m[1], m[2], m[3], m[4], m[5], a);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

// dense (tile_info == nullptr) or grouped over the MoE schedule, arguments as gemm_mx
int gemm_mxp(int mode, int rows, int k, int n, const uint8_t* x8, const float* s8, const uint8_t* w,
             const uint8_t* ws, const uint8_t* w2, const uint8_t* w2s, float* y, cudaStream_t s,
             const int32_t* tile_info, const int32_t* rowmap, int xrows, int ku, int n_experts, int rows_per_expert,
             int w2_row_offset, const ExpertEpi* epi) {
  const int NW = mode == LK_STORE ? 1 : 2;   // swiglu: gathered or sorted gate/up rows
  const int bnw = kMxpNT / NW;
  const int group = tile_info ? (mode == LK_SWIGLU ? kGather : kSorted) : kDense;
  MxpArgs a{};
  if (epi) a.epi = *epi;
  a.s8 = s8;
  a.y = y;
  a.ws = ws;
  a.ws2 = w2s ? w2s : ws;
  a.rows = rows;
  a.k = k;
  a.n = n;
  a.sf_stride = k / 32;
  a.kmain = k / kBK;
  a.tail_sub = k % kBK ? (kBK - k % kBK) / 32 : 4;
  a.m_tiles = (rows + kBM - 1) / kBM;
  a.n_tiles = (n + bnw - 1) / bnw;
  int64_t wrows = n, w2rows = n;
  a.w2_row_offset = (NW == 2 && !w2) ? w2_row_offset : 0;
  if (tile_info) {
    a.tile_info = tile_info;
    a.rowmap = rowmap;
    a.max_tiles = rows / 64;
    a.xrows = xrows;
    a.ku = ku;
    a.n_experts = n_experts;
    a.rows_per_expert = rows_per_expert;
    a.rows_per_expert2 = w2 ? n : rows_per_expert;
    wrows = int64_t(n_experts) * rows_per_expert;
    w2rows = int64_t(n_experts) * a.rows_per_expert2;
  }
  const uint8_t* w2p = w2 ? w2 : w;
  CUtensorMap m[6];   // A, w, w2, w tail, w2 tail, y
  int rc = group == kGather
               ? make_map(&m[0], x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, xrows, k, kBK, 1, CU_TENSOR_MAP_SWIZZLE_128B)
               : make_map(&m[0], x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, k, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == LK_OK) rc = make_map_u4(&m[1], w, wrows, int64_t(a.kmain) * kBK, k / 2, bnw);
  if (rc == LK_OK) rc = make_map_u4(&m[2], w2p, w2rows, int64_t(a.kmain) * kBK, k / 2, bnw);
  if (rc == LK_OK) rc = make_map_u4(&m[3], w + (k - kBK) / 2, wrows, kBK, k / 2, bnw);
  if (rc == LK_OK) rc = make_map_u4(&m[4], w2p + (k - kBK) / 2, w2rows, kBK, k / 2, bnw);
  if (rc == LK_OK)
    rc = make_map(&m[5], y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, rows, n, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != LK_OK) return rc;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // grouped: at most rows / 128 + n_experts super-tiles (the count itself is known on the device only)
  const int64_t max_m = tile_info ? int64_t(rows) / kBM + n_experts : a.m_tiles;
  const int grid = int(std::min(int64_t(sms), max_m * a.n_tiles));
  if (group == kGather) return launch_mxp<2, kGather>(m, a, grid, s);
  if (group == kSorted) return NW == 2 ? launch_mxp<2, kSorted>(m, a, grid, s) : launch_mxp<1, kSorted>(m, a, grid, s);
  return NW == 2 ? launch_mxp<2, kDense>(m, a, grid, s) : launch_mxp<1, kDense>(m, a, grid, s);
}

}  // namespace

// dense (tile_info == nullptr) or grouped over the MoE schedule
int gemm_mx(int mode, int order, int rows, int k, int n, const uint8_t* x8, const float* s8, const uint8_t* w,
            const uint8_t* ws, const uint8_t* w2, const uint8_t* w2s, float* y, cudaStream_t s,
            const int32_t* tile_info, const int32_t* rowmap, int xrows, int ku, int n_experts, int rows_per_expert,
            int w2_row_offset, const ExpertEpi* epi) {
  if (mxp_applies(order, k, w, ws, w2, w2s))
    return gemm_mxp(mode, rows, k, n, x8, s8, w, ws, w2, w2s, y, s, tile_info, rowmap, xrows, ku, n_experts,
                    rows_per_expert, w2_row_offset, epi);
  const int NW = mode == LK_STORE ? 1 : 2;
  const int bn = kRowsB / NW;
  MxArgs a{};
  if (epi) a.epi = *epi;
  a.s8 = s8;
  a.y = y;
  a.rows = rows;
  a.k = k;
  a.n = n;
  a.sf_stride = k / 32;
  a.ws = ws;
  a.ws2 = w2s ? w2s : ws;
  int group = kDense;
  int64_t wrows = n, w2rows = n;
  a.rows_per_expert = a.rows_per_expert2 = 0;
  a.w2_row_offset = (NW == 2 && !w2) ? w2_row_offset : 0;
  if (tile_info) {
    group = mode == LK_SWIGLU ? kGather : kSorted;
    a.tile_info = tile_info;
    a.rowmap = rowmap;
    a.max_tiles = rows / 64;
    a.xrows = xrows;
    a.ku = ku;
    a.n_experts = n_experts;
    a.rows_per_expert = rows_per_expert;
    a.rows_per_expert2 = w2 ? n : rows_per_expert;
    wrows = int64_t(n_experts) * rows_per_expert;
    w2rows = int64_t(n_experts) * a.rows_per_expert2;
  }
  CUtensorMap am, wm, w2m;
  int rc = group == kGather ? make_map(&am, x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, xrows, k, kBK, 1,
                                       CU_TENSOR_MAP_SWIZZLE_128B)
                            : make_map(&am, x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, k, kBK, kBM,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == LK_OK)
    rc = make_map(&wm, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wrows, k / 2, kBK / 2, bn, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc == LK_OK)
    rc = w2 ? make_map(&w2m, w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w2rows, k / 2, kBK / 2, bn,
                       CU_TENSOR_MAP_SWIZZLE_NONE)
            : (w2m = wm, LK_OK);
  if (rc != LK_OK) return rc;
  dim3 grid((n + bn - 1) / bn, group == kDense ? (rows + kBM - 1) / kBM : rows / 64);
  if (NW == 2) {
    if (group == kGather) return launch_o<2, kGather>(order, am, wm, w2m, a, grid, s);
    if (group == kSorted) return launch_o<2, kSorted>(order, am, wm, w2m, a, grid, s);
    return launch_o<2, kDense>(order, am, wm, w2m, a, grid, s);
  }
  if (group == kSorted) return launch_o<1, kSorted>(order, am, wm, w2m, a, grid, s);
  return launch_o<1, kDense>(order, am, wm, w2m, a, grid, s);
}

int gemm_mxfp4s(int mode, int order, int rows, int k, int n, const uint8_t* x8, const float* s8, const uint8_t* w,
                const uint8_t* ws, const uint8_t* w2, const uint8_t* w2s, float* y, cudaStream_t s) {
  return gemm_mx(mode, order, rows, k, n, x8, s8, w, ws, w2, w2s, y, s, nullptr, nullptr, rows, 1, 1, 0, 0);
}

LK_STATUS_READER(status_mx)

}  // namespace lk
