// Shared device helpers for liblk (sm_100a): format constants, f16/bf16 bit helpers, mbarrier + bulk-copy (TMA)
// wrappers and the tcgen05 (5th-gen tensor core / TMEM) instruction wrappers used by the prefill GEMMs.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lk.h"

#define LK_DEV __device__ __forceinline__

namespace lk {

// ---------------------------------------------------------------------------------------------------------------
// formats: values and bytes per block (formats.py:5-17)
// ---------------------------------------------------------------------------------------------------------------
__host__ __device__ constexpr int qk_of(int fmt) { return fmt == LK_Q4_K ? 256 : 32; }
__host__ __device__ constexpr int block_bytes_of(int fmt) {
  return fmt == LK_Q4_K ? 144 : (fmt == LK_MXFP4 ? 17 : (fmt == LK_MXFP4S ? 16 : 18));
}
// 256 values of Q4_0, IQ4_NL and Q4_K all take 144 bytes: the unit every streamed chunk is counted in
constexpr int kChunkValues = 256;
constexpr int kChunkBytes = 144;

// IQ4_NL codebook (kvalues_iq4nl, quant_values.loom:18-36) biased by +128 so every entry is one unsigned byte
// (1..241): four little-endian words for a byte-permute lookup
constexpr uint32_t kIq4Biased0 = (1u) | (24u << 8) | (45u << 16) | (63u << 24);      // -127 -104 -83 -65
constexpr uint32_t kIq4Biased1 = (79u) | (93u << 8) | (106u << 16) | (118u << 24);   // -49 -35 -22 -10
constexpr uint32_t kIq4Biased2 = (129u) | (141u << 8) | (153u << 16) | (166u << 24); // 1 13 25 38
constexpr uint32_t kIq4Biased3 = (181u) | (197u << 8) | (217u << 16) | (241u << 24); // 53 69 89 113

LK_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// 4 nibble codes (bits 0-3 of each byte of `idx`) -> their biased IQ4 codebook bytes
LK_DEV uint32_t iq4_lookup4(uint32_t idx) {
  // byte i of the result = table[idx.byte_i]: low 3 bits pick within a half-table, bit 3 picks the half
  uint32_t sel = (idx & 0x7u) | ((idx >> 4) & 0x70u) | ((idx >> 8) & 0x700u) | ((idx >> 12) & 0x7000u);
  uint32_t lo = prmt(kIq4Biased0, kIq4Biased1, sel);
  uint32_t hi = prmt(kIq4Biased2, kIq4Biased3, sel);
  uint32_t hsel = 0x3210u | ((idx >> 1) & 0x4u) | ((idx >> 5) & 0x40u) | ((idx >> 9) & 0x400u) | ((idx >> 13) & 0x4000u);
  return prmt(lo, hi, hsel);
}

LK_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
LK_DEV float bf2f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// Q4_K 6-bit (scale, minimum) of group j from the three little-endian words of the 12-byte scale field
// (header bytes 4..15), register arithmetic only (gen_llm.py:234-266 @g_k_scale_minimum)
LK_DEV void q4k_scale_min_w(uint32_t s0, uint32_t s1, uint32_t s2, int j, uint32_t& sc, uint32_t& m) {
  uint32_t sh = 8u * uint32_t(j & 3);
  if (j < 4) {
    sc = (s0 >> sh) & 63u;
    m = (s1 >> sh) & 63u;
  } else {
    uint32_t lo = s2 >> sh;
    sc = (lo & 15u) | (((s0 >> sh) >> 2) & 48u);
    m = ((lo >> 4) & 15u) | (((s1 >> sh) >> 2) & 48u);
  }
}
// small integer (0..2047) -> f16 exactly, without a conversion instruction: bits of (1024 + v) minus 1024
LK_DEV __half small_int_half(uint32_t v) {
  return __hsub(__ushort_as_half(uint16_t(0x6400u | v)), __ushort_as_half(uint16_t(0x6400u)));
}

// Q4_K 6-bit (scale, minimum) of group j of a 12-byte scale field (gen_llm.py:234-266)
LK_DEV void q4k_scale_min(const uint8_t* s, int j, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// mbarrier + bulk async copies (TMA)
// ---------------------------------------------------------------------------------------------------------------
LK_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

LK_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
LK_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
LK_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

LK_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
LK_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
LK_DEV bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Device-side status word of this translation unit (bit 0: a bounded wait gave up). Each kernel file defines a
// reader with LK_STATUS_READER; lk_device_status() ORs them.
static __device__ unsigned int g_status;
#define LK_STATUS_READER(name)                                   \
  unsigned int name(bool clear) {                                \
    unsigned int v = 0;                                          \
    cudaMemcpyFromSymbol(&v, g_status, sizeof(v));               \
    if (clear) {                                                 \
      unsigned int z = 0;                                        \
      cudaMemcpyToSymbol(g_status, &z, sizeof(z));               \
    }                                                            \
    return v;                                                    \
  }

// Bounded wait: gives up after kSpinLimit polls and returns false (the caller records the error in g_status and
// carries on with uniform control flow), so a kernel never spins forever on a phase that will not complete.
constexpr uint32_t kSpinLimit = 1u << 26;
LK_DEV bool mbar_wait(uint64_t* bar, uint32_t phase) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, phase)) return true;
  return false;
}

// 1-D bulk copy global -> shared, completing on `bar` (both addresses and the size multiples of 16 bytes)
LK_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled TMA load through a tensor map (no multicast), completing on `bar`
LK_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// Four rows (row coordinates r0..r3, one-row boxes) gathered by one TMA instruction, completing on `bar`
LK_DEV void tma_gather4(void* dst, const CUtensorMap* map, int x, int r0, int r1, int r2, int r3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
      : "memory");
}
// 16-byte chunk `c` of row `r` of a K-major 128-byte-swizzled tile (1024-byte aligned)
LK_DEV uint32_t sw128(int r, int c) { return uint32_t((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)); }

LK_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 2-D tiled TMA store shared -> global through a tensor map; parts of the box outside the tensor are not written.
// Completion is tracked per thread by bulk async-groups (bulk_commit_group / bulk_wait_group*).
LK_DEV void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
LK_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// until no committed bulk group of this thread still reads its shared-memory source
LK_DEV void bulk_wait_group_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// until every committed bulk group of this thread has completed
LK_DEV void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue, commit, TMEM loads
// ---------------------------------------------------------------------------------------------------------------
LK_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
LK_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
LK_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
LK_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LK_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (f16 or bf16 inputs, f32 accumulate)
LK_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// kind::f8f6f4 (8-bit e4m3/e5m2 inputs, f32 accumulate)
LK_DEV void umma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// kind::mxf8f6f4 with block scale factors (one E8M0 byte per 32 k per row of A and of B) read from TMEM at sfa/sfb
// (bits 30-31 of each address: the byte of the 32-bit scale column, matching the instruction descriptor's sf ids)
LK_DEV void umma_mx(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa, uint32_t sfb,
                    uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}
// 32 rows x 16 bytes of shared memory -> 4 TMEM columns of lanes 0-31, replicated to all four lane quarters
LK_DEV void tmem_cp_32x128_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// Shared-memory descriptor of a dense, unswizzled block of 16-byte rows (8-row core matrices 128 bytes apart)
LK_DEV uint64_t sdesc_rows16(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFF);
  d |= uint64_t(128 >> 4) << 16;   // leading byte offset (one 16-byte column: unused)
  d |= uint64_t(128 >> 4) << 32;   // stride byte offset: next 8-row core matrix
  d |= uint64_t(1) << 46;          // version (sm_100); layout type 0 = no swizzle
  return d;
}
// Instruction descriptor, kind::mxf8f6f4.block_scale: A format fa, B format fb (0 e4m3, 1 e5m2, 5 e2m1), E8M0
// scales, K-major operands, sf ids of A and B
__host__ __device__ constexpr uint32_t idesc_mx(int m, int n, int fa, int fb, int sfa_id, int sfb_id) {
  return (uint32_t(sfb_id) << 4) | (uint32_t(fa) << 7) | (uint32_t(fb) << 10) | (uint32_t(n >> 3) << 17) |
         (1u << 23) | (uint32_t(m >> 4) << 24) | (uint32_t(sfa_id) << 29);
}

// arrive on `bar` when every previously issued tcgen05.mma of this thread has completed
LK_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle canonical layout: rows of 128 bytes,
// 8-row groups 1024 bytes apart (SBO), the 16-byte chunks of row r XOR-ed with (r % 8); version 1 (sm_100).
LK_DEV uint64_t sdesc_k128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFF);     // start address
  d |= uint64_t(1) << 16;                       // leading byte offset (unused for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;               // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;                       // descriptor version (sm_100)
  d |= uint64_t(2) << 61;                       // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: f32 accumulate, A and B both `ab` (0 = f16, 1 = bf16), both K-major
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, int ab) {
  return (1u << 4) | (uint32_t(ab) << 7) | (uint32_t(ab) << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}
// Instruction descriptor, kind::f8f6f4: f32 accumulate, A format fa, B format fb (0 = e4m3, 1 = e5m2), K-major
__host__ __device__ constexpr uint32_t idesc_f8(int m, int n, int fa, int fb) {
  return (1u << 4) | (uint32_t(fa) << 7) | (uint32_t(fb) << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// 32 lanes x 32 consecutive f32 columns of TMEM into registers (warp w reads lanes 32*(w%4) .. +31)
LK_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// true when `mask` already has the current device's bit; sets it (per-device one-time kernel attribute set-up)
inline bool once_per_device(unsigned& mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  unsigned bit = 1u << (dev & 31);
  if (mask & bit) return true;
  mask |= bit;
  return false;
}

LK_DEV float silu(float g) { return g / (1.0f + __expf(-g)); }

// The expert gate/up activation (gen_moe.py:27-64 act_scalar / act_vector; include/lk.h LK_ACT_*):
//   LK_ACT_SILU        silu(g) * u
//   LK_ACT_GELU        gelu_tanh(g) * u: 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))), GEGLU (make_kernel_tests.py:78-80)
//   LK_ACT_SWIGLU_OAI  x = min(g, limit), y = clamp(u, -limit, limit): x sigmoid(alpha x) (y + 1)   (gpt-oss)
LK_DEV float act_apply(int act, float g, float u, float alpha, float limit) {
  if (act == LK_ACT_GELU) return 0.5f * g * (1.0f + tanhf(0.7978845608028654f * fmaf(0.044715f * g, g * g, g))) * u;
  if (act == LK_ACT_SWIGLU_OAI) {
    const float x = fminf(g, limit), y = fmaxf(fminf(u, limit), -limit);
    return x / (1.0f + __expf(-alpha * x)) * (y + 1.0f);
  }
  return silu(g) * u;
}

// ---------------------------------------------------------------------------------------------------------------
// MoE schedule: 128-row super-tiles over the bucket's 64-row tiles
// ---------------------------------------------------------------------------------------------------------------
constexpr int kMaxExperts = 256;
constexpr int kMaxPeers = 8;   // ranks of one NVSwitch domain a GEMM epilogue can store to
// Super-tile `s` of a tile schedule laid out as the bucket writes it (the tiles of each expert contiguous, experts
// ascending, unused tiles (-1, 0)): consecutive tiles of one expert are paired from the start of its run, so expert e
// owns ceil(tiles_e / 2) super-tiles. Called by every thread of the CTA; `scratch` is 3 * kMaxExperts ints of shared
// memory that nothing else uses yet (the async proxy may write it afterwards). meta[0] = expert (-1: the schedule has
// fewer super-tiles than s + 1), meta[1] = first tile, meta[2] = valid rows (64 + rows of the second tile if paired).
// The whole super-tile table of a schedule, for kernels that walk many super-tiles: called by every thread of the
// CTA; tbl = 3 * kMaxExperts ints of shared memory that stay for the kernel's life: start[e] (first tile), count[e]
// (tiles), base[e] (first super-tile). Returns the number of super-tiles.
LK_DEV int moe_super_table(const int32_t* tile_info, int max_tiles, int n_experts, int* tbl) {
  int* start = tbl;
  int* count = tbl + kMaxExperts;
  int* base = tbl + 2 * kMaxExperts;
  for (int e = threadIdx.x; e < kMaxExperts; e += blockDim.x) {
    start[e] = 0x7FFFFFFF;
    count[e] = 0;
  }
  __syncthreads();
  for (int t = threadIdx.x; t < max_tiles; t += blockDim.x) {
    int e = __ldg(tile_info + 2 * t);
    if (e >= 0 && e < n_experts) {
      atomicMin(&start[e], t);
      atomicAdd(&count[e], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int v[kMaxExperts / 32], sum = 0;
#pragma unroll
    for (int i = 0; i < kMaxExperts / 32; ++i) {
      v[i] = (count[lane * (kMaxExperts / 32) + i] + 1) >> 1;
      sum += v[i];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += u;
    }
    int run = incl - sum;
#pragma unroll
    for (int i = 0; i < kMaxExperts / 32; ++i) {
      base[lane * (kMaxExperts / 32) + i] = run;
      run += v[i];
    }
  }
  __syncthreads();
  return base[kMaxExperts - 1] + ((count[kMaxExperts - 1] + 1) >> 1);
}
// Super-tile s of a table built by moe_super_table (s below the returned count): expert, first 64-row tile, valid
// rows.
LK_DEV void moe_super_lookup(const int32_t* tile_info, const int* tbl, int s, int& expert, int& first, int& rows) {
  const int* start = tbl;
  const int* count = tbl + kMaxExperts;
  const int* base = tbl + 2 * kMaxExperts;
  int lo = 0, hi = kMaxExperts;   // first e with base[e] > s
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (base[mid] <= s) lo = mid + 1;
    else hi = mid;
  }
  const int e = lo - 1;
  expert = e;
  first = start[e] + 2 * (s - base[e]);
  const bool pair = first + 1 < start[e] + count[e];
  rows = pair ? 64 + __ldg(tile_info + 2 * (first + 1) + 1) : __ldg(tile_info + 2 * first + 1);
}

LK_DEV void moe_super_tile(const int32_t* tile_info, int max_tiles, int n_experts, int s, int* scratch, int* meta) {
  int* start = scratch;
  int* count = scratch + kMaxExperts;
  int* base = scratch + 2 * kMaxExperts;
  for (int e = threadIdx.x; e < kMaxExperts; e += blockDim.x) {
    start[e] = 0x7FFFFFFF;
    count[e] = 0;
  }
  if (threadIdx.x == 0) meta[0] = -1;
  __syncthreads();
  for (int t = threadIdx.x; t < max_tiles; t += blockDim.x) {
    int e = __ldg(tile_info + 2 * t);
    if (e >= 0 && e < n_experts) {
      atomicMin(&start[e], t);
      atomicAdd(&count[e], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {   // exclusive scan of ceil(count / 2), 8 experts per lane
    const int lane = threadIdx.x;
    int v[kMaxExperts / 32], sum = 0;
#pragma unroll
    for (int i = 0; i < kMaxExperts / 32; ++i) {
      v[i] = (count[lane * (kMaxExperts / 32) + i] + 1) >> 1;
      sum += v[i];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += u;
    }
    int run = incl - sum;
#pragma unroll
    for (int i = 0; i < kMaxExperts / 32; ++i) {
      base[lane * (kMaxExperts / 32) + i] = run;
      run += v[i];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) {
    const int ns = (count[e] + 1) >> 1;
    if (s >= base[e] && s < base[e] + ns) {
      const int first = start[e] + 2 * (s - base[e]);
      const bool pair = first + 1 < start[e] + count[e];
      meta[0] = e;
      meta[1] = first;
      meta[2] = pair ? 64 + __ldg(tile_info + 2 * (first + 1) + 1) : __ldg(tile_info + 2 * first + 1);
    }
  }
  fence_proxy_async();
  __syncthreads();
}

}  // namespace lk
