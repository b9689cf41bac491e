// MoE routing, the GPU-built per-expert tile schedule, and the weighted combines.
//
// g_moe_route / g_moe_route_tr  gen_moe.py:116-253, 255-470   router logits, gating, top-k, weights
// g_moe_bucket                   gen_moe.py:829-955             tile_info / rowmap / pos
// g_moe_combine_sorted           gen_moe.py:1231-1280           y[t] (+)= sum_k w[t,k] ys[pos[t,k]]
// g_moe_combine                  gen_moe.py:730-762             y[t] (+)= sum_k w[t,k] ys[t*KU + k]
// shared_gated                   gen_moe.py:765-777             y[t] = sg[t] y[t] + sum_k ...
// g_moe_wscale                   gen_moe.py:1010-1045           w[t,k] *= scale[ids[t,k]]
// g_moe_shared_gate              gen_moe.py:780-823             sg[t] = sigmoid(x[t] . w)
#include "lk_common.cuh"
#include "lk_internal.h"
#include "lk_route.cuh"

namespace lk {

constexpr int kTile = 64;   // gen_moe.py:826 TILE
constexpr int kMaxRanks = 32;   // expert-parallel dispatch: ranks of one plan

// ---------------------------------------------------------------------------------------------------------------
// router: one 256-thread block per token; thread e owns expert e
// ---------------------------------------------------------------------------------------------------------------
template <bool BF16W>
__global__ void __launch_bounds__(256) k_route(int h, int E, int ku, int gating, int norm, float scale,
                                               const float* __restrict__ x, const void* __restrict__ router_w,
                                               const float* __restrict__ bias, int32_t* __restrict__ ids,
                                               float* __restrict__ wts) {
  __shared__ float logit[256];
  __shared__ float red_f[8];
  __shared__ int red_i[8];
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (router_w) {
    // warp w scores experts w, w+8, ...: lanes stride over h, then a warp sum
    const float* xr = x + int64_t(t) * h;
    for (int e = warp; e < E; e += 8) {
      float acc = 0.f;
      if (BF16W) {
        const uint16_t* wr = static_cast<const uint16_t*>(router_w) + int64_t(e) * h;
        for (int i = lane; i < h; i += 32) acc = fmaf(xr[i], bf2f(wr[i]), acc);
      } else {
        const float* wr = static_cast<const float*>(router_w) + int64_t(e) * h;
        for (int i = lane; i < h; i += 32) acc = fmaf(xr[i], wr[i], acc);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) logit[e] = acc;
    }
  } else {
    for (int e = tid; e < E; e += 256) logit[e] = x[int64_t(t) * E + e];
  }
  __syncthreads();
  const bool in = tid < E;
  const float lg = in ? logit[tid] : -INFINITY;
  auto bmax = [&](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red_f[warp] = v;
    __syncthreads();
    float r = red_f[0];
    for (int i = 1; i < 8; ++i) r = fmaxf(r, red_f[i]);
    return r;
  };
  auto bsum = [&](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red_f[warp] = v;
    __syncthreads();
    float r = 0.f;
    for (int i = 0; i < 8; ++i) r += red_f[i];
    return r;
  };
  auto bmin_i = [&](int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red_i[warp] = v;
    __syncthreads();
    int r = red_i[0];
    for (int i = 1; i < 8; ++i) r = min(r, red_i[i]);
    return r;
  };
  // probability (the weight's source) and selection score
  float prob, score;
  if (gating == 1) {
    float m = bmax(lg);
    float ex = in ? expf(lg - m) : 0.f;
    float den = bsum(ex);
    prob = ex / den;
    score = in ? lg : -INFINITY;   // softmax is monotonic in the logit: rank on the exact input
  } else if (gating == 2) {
    prob = in ? 1.0f / (1.0f + expf(-lg)) : 0.f;
    score = in ? prob + (bias ? bias[tid] : 0.f) : -INFINITY;
  } else {
    prob = in ? lg + (bias ? bias[tid] : 0.f) : -INFINITY;
    score = prob;
  }
  // ku rounds: the best score, ties to the lowest expert index
  int my_k = -1;
  float sc = score, sel_sum = 0.f;
  for (int r = 0; r < ku; ++r) {
    float best = bmax(sc);
    int cand = (in && sc == best) ? tid : 1 << 30;
    int winner = bmin_i(cand);
    if (tid == winner) {
      my_k = r;
      ids[int64_t(t) * ku + r] = tid;
      sc = -INFINITY;
    }
    sel_sum += bsum(tid == winner ? prob : 0.f);
  }
  float wv;
  if (gating == 3) {
    float m = bmax(my_k >= 0 ? prob : -INFINITY);
    float ex = my_k >= 0 ? expf(prob - m) : 0.f;
    float den = bsum(ex);
    wv = ex / den;
  } else {
    float den = norm ? fmaxf(sel_sum, 6.103515625e-05f) : 1.0f;
    wv = prob / den;
  }
  if (my_k >= 0) wts[int64_t(t) * ku + my_k] = wv * scale;
}

// router on given logits: one warp per token (8 per CTA); the per-token rules are route_token (lk_route.cuh)
__global__ void __launch_bounds__(256) k_route_w(int tokens, int E, int ku, int gating, int norm, float scale,
                                                 const float* __restrict__ logits, const float* __restrict__ bias,
                                                 int32_t* __restrict__ ids, float* __restrict__ wts) {
  const int lane = threadIdx.x & 31;
  const int64_t t = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= tokens) return;
  route_token(lane, E, ku, gating, norm, scale, logits + t * E, bias, ids + t * ku, wts + t * ku);
}

int moe_route(int tokens, int h, int E, int ku, int gating, int norm, float scale, const float* x,
              const void* router_w, int w_dtype, const float* bias, int32_t* ids, float* wts, cudaStream_t s) {
  if (!router_w) {
    k_route_w<<<(tokens + 7) / 8, 256, 0, s>>>(tokens, E, ku, gating, norm, scale, x, bias, ids, wts);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
  }
  if (w_dtype == LK_BF16)
    k_route<true><<<tokens, 256, 0, s>>>(h, E, ku, gating, norm, scale, x, router_w, bias, ids, wts);
  else
    k_route<false><<<tokens, 256, 0, s>>>(h, E, ku, gating, norm, scale, x, router_w, bias, ids, wts);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

// ---------------------------------------------------------------------------------------------------------------
// bucket: one 1024-thread block. Counting sort by expert, stable in the assignment index, so the schedule is
// deterministic (the reference's atomics give any order within an expert's rows). Warp w owns the contiguous
// assignments [w * chunk, (w + 1) * chunk): per-warp expert counts, one scan over the warps per expert, then each warp
// places its own assignments in rounds of 32 with no block-wide barrier (rank inside a round by __match_any_sync).
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_bucket(int tokens, int ku, int E, int max_tiles,
                                                 const int32_t* __restrict__ info, const int32_t* __restrict__ ids,
                                                 int32_t* __restrict__ tile_info, int32_t* __restrict__ rowmap,
                                                 int32_t* __restrict__ pos) {
  __shared__ int count[256];
  __shared__ int cursor[256];
  __shared__ int tbase[257];
  __shared__ int wcnt[32][256];   // per warp and expert: count, then the count in the warps before, then a cursor
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int A = tokens * ku;
  const int chunk = (A + 31) / 32;
  const int a0 = min(A, warp * chunk), a1 = min(A, a0 + chunk);
  for (int i = tid; i < 32 * 256; i += 1024) (&wcnt[0][0])[i] = 0;
  __syncthreads();
  auto expert_of = [&](int a) -> int {
    int t = a / ku;
    if (info && info[4 * t + 2] == 0) return -1;
    return min(max(ids[a], 0), E - 1);
  };
  for (int a = a0 + lane; a < a1; a += 32) {
    int e = expert_of(a);
    if (e >= 0) atomicAdd(&wcnt[warp][e], 1);
  }
  __syncthreads();
  if (tid < E) {   // exclusive scan over the warps: assignments of expert tid in the ranges before warp w
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = wcnt[w][tid];
      wcnt[w][tid] = run;
      run += c;
    }
    count[tid] = run;
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      tbase[e] = acc;
      acc += (count[e] + kTile - 1) / kTile;
    }
    tbase[E] = acc;
  }
  __syncthreads();
  const int total = tbase[E];
  if (tid < E) {
    int n = count[tid], tiles = (n + kTile - 1) / kTile;
    for (int j = 0; j < tiles; ++j) {
      int tile = tbase[tid] + j;
      if (tile < max_tiles) {
        tile_info[2 * tile] = tid;
        tile_info[2 * tile + 1] = min(kTile, n - j * kTile);
      }
    }
    cursor[tid] = tbase[tid] * kTile;
  }
  for (int u = total + tid; u < max_tiles; u += 1024) {
    tile_info[2 * u] = -1;
    tile_info[2 * u + 1] = 0;
  }
  // padding rows of used tiles and every row of unused tiles
  for (int e = 0; e < E; ++e) {
    int first = tbase[e] * kTile + count[e], end = tbase[e + 1] * kTile;
    for (int r = first + tid; r < end; r += 1024)
      if (r < max_tiles * kTile) rowmap[r] = -1;
  }
  for (int r = total * kTile + tid; r < max_tiles * kTile; r += 1024) rowmap[r] = -1;
  __syncthreads();
  // stable placement: warp-local rounds over the warp's own assignments, in ascending order
  for (int base = a0; base < a1; base += 32) {
    const int a = base + lane;
    const int e = a < a1 ? expert_of(a) : -2;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1));
    if (e >= 0) {
      const int off = cursor[e] + wcnt[warp][e] + rank;
      if (off < max_tiles * kTile) rowmap[off] = a;
      pos[a] = off;
    } else if (e == -1) {
      pos[a] = -1;
    }
    __syncwarp();
    if (e >= 0 && rank == 0) wcnt[warp][e] += __popc(peers);
    __syncwarp();
  }
}

int moe_bucket(int tokens, int ku, int E, int max_tiles, const int32_t* info, const int32_t* ids, int32_t* tile_info,
               int32_t* rowmap, int32_t* pos, cudaStream_t s) {
  k_bucket<<<1, 1024, 0, s>>>(tokens, ku, E, max_tiles, info, ids, tile_info, rowmap, pos);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

// ---------------------------------------------------------------------------------------------------------------
// expert-parallel dispatch (no reference counterpart: the reference runs on one device). Assignment a goes to rank
// ids[a] / n_local. k_rank_plan: one 1024-thread block, a stable counting sort of the assignments by rank, with
// k_bucket's structure (warp w owns a contiguous range of assignments; per-warp counts, one scan over the warps per
// rank, then warp-local placement rounds in ascending order): order[i] = the i-th assignment in (rank, a) order,
// pos[a] = its place in order, counts[r] = the assignments for rank r.
// k_gather_rows: row i of the send buffer = x[order[i] / ku] (f32 or bf16, 16-byte copies), eid[i] = the local expert
// ids[order[i]] % n_local.
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_rank_plan(int A, int n_local, int world, const int32_t* __restrict__ ids,
                                                    int32_t* __restrict__ order, int32_t* __restrict__ pos,
                                                    int32_t* __restrict__ counts) {
  __shared__ int wcnt[32][kMaxRanks];
  __shared__ int rbase[kMaxRanks + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = (A + 31) / 32;
  const int a0 = min(A, warp * chunk), a1 = min(A, a0 + chunk);
  auto rank_of = [&](int a) { return min(max(ids[a], 0) / n_local, world - 1); };
  if (tid < 32 * kMaxRanks) (&wcnt[0][0])[tid] = 0;
  __syncthreads();
  for (int a = a0 + lane; a < a1; a += 32) atomicAdd(&wcnt[warp][rank_of(a)], 1);
  __syncthreads();
  if (tid < world) {   // exclusive scan over the warps, per rank
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = wcnt[w][tid];
      wcnt[w][tid] = run;
      run += c;
    }
    counts[tid] = run;
    rbase[tid] = run;
  }
  __syncthreads();
  if (tid == 0) {   // rank bases
    int acc = 0;
    for (int r = 0; r < world; ++r) {
      const int c = rbase[r];
      rbase[r] = acc;
      acc += c;
    }
    rbase[world] = acc;
  }
  __syncthreads();
  for (int b = a0; b < a1; b += 32) {   // stable placement, warp-local rounds
    const int a = b + lane;
    const int r = a < a1 ? rank_of(a) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, r);
    const int rk = __popc(peers & ((1u << lane) - 1));
    if (r >= 0) {
      const int off = rbase[r] + wcnt[warp][r] + rk;
      order[off] = a;
      pos[a] = off;
    }
    __syncwarp();
    if (r >= 0 && rk == 0) wcnt[warp][r] += __popc(peers);
    __syncwarp();
  }
}

template <bool BF16>
__global__ void __launch_bounds__(256) k_gather_rows(int rows, int h, int ku, int n_local, const int32_t* __restrict__ order,
                                                     const int32_t* __restrict__ ids, const void* __restrict__ x,
                                                     void* __restrict__ out, int32_t* __restrict__ eid) {
  const int i = blockIdx.x;
  if (i >= rows) return;
  const int a = order[i];
  const int64_t bytes = int64_t(h) * (BF16 ? 2 : 4);
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(x) + int64_t(a / ku) * bytes);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(out) + int64_t(i) * bytes);
  for (int j = threadIdx.x; j < bytes / 16; j += 256) dst[j] = __ldg(src + j);
  if (threadIdx.x == 0 && eid) eid[i] = max(ids[a], 0) % n_local;
}

int moe_rank_plan(int assignments, int n_local, int world, const int32_t* ids, int32_t* order, int32_t* pos,
                  int32_t* counts, cudaStream_t s) {
  k_rank_plan<<<1, 1024, 0, s>>>(assignments, n_local, world, ids, order, pos, counts);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

int moe_gather_rows(int rows, int h, int ku, int n_local, const int32_t* order, const int32_t* ids, const void* x,
                    int x_dtype, void* out, int32_t* eid, cudaStream_t s) {
  if (x_dtype == LK_BF16) k_gather_rows<true><<<rows, 256, 0, s>>>(rows, h, ku, n_local, order, ids, x, out, eid);
  else k_gather_rows<false><<<rows, 256, 0, s>>>(rows, h, ku, n_local, order, ids, x, out, eid);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

// ---------------------------------------------------------------------------------------------------------------
// combines: block (t, c) covers columns 256 c .. 256 c + 255 of token t, one per thread (a token's columns spread over
// h / 256 CTAs, so a decode token's combine is not one CTA walking h); the fma chain runs over k in order, as the
// reference's
// ---------------------------------------------------------------------------------------------------------------
// sg != nullptr (shared_gated, gen_moe.py:765-777): the shared experts' output in y is scaled by the token's gate first
template <bool SORTED>
__global__ void __launch_bounds__(256) k_combine(int h, int ku, int accumulate, const float* __restrict__ ys,
                                                 const int32_t* __restrict__ pos, const float* __restrict__ wts,
                                                 const float* __restrict__ sg, float* __restrict__ y) {
  const int t = blockIdx.x;
  __shared__ float w[8];
  __shared__ int p[8];
  if (threadIdx.x < ku) {
    w[threadIdx.x] = wts[int64_t(t) * ku + threadIdx.x];
    p[threadIdx.x] = SORTED ? pos[int64_t(t) * ku + threadIdx.x] : t * ku + threadIdx.x;
  }
  __syncthreads();
  const int c = blockIdx.y * 256 + threadIdx.x;
  if (c >= h) return;
  float acc = accumulate ? y[int64_t(t) * h + c] : 0.f;
  if (sg) acc *= sg[t];
  for (int k = 0; k < ku; ++k) {
    float v = p[k] >= 0 ? ys[int64_t(p[k]) * h + c] : 0.f;
    acc = fmaf(w[k], v, acc);
  }
  y[int64_t(t) * h + c] = acc;
}

int moe_combine_sorted(int tokens, int rows, int h, int ku, int accumulate, const float* ys, const int32_t* pos,
                       const float* wts, float* y, cudaStream_t s) {
  (void)rows;
  k_combine<true><<<dim3(tokens, (h + 255) / 256), 256, 0, s>>>(h, ku, accumulate, ys, pos, wts, nullptr, y);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

int moe_combine(int tokens, int h, int ku, int accumulate, const float* ys, const float* wts, float* y,
                cudaStream_t s) {
  k_combine<false><<<dim3(tokens, (h + 255) / 256), 256, 0, s>>>(h, ku, accumulate, ys, nullptr, wts, nullptr, y);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

int moe_combine_g(int tokens, int h, int ku, const float* ys, const int32_t* pos, const float* wts, const float* sg,
                  float* y, cudaStream_t s) {
  const dim3 grid(tokens, (h + 255) / 256);
  if (pos) k_combine<true><<<grid, 256, 0, s>>>(h, ku, 1, ys, pos, wts, sg, y);
  else k_combine<false><<<grid, 256, 0, s>>>(h, ku, 1, ys, nullptr, wts, sg, y);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

// ---------------------------------------------------------------------------------------------------------------
// g_moe_wscale (gen_moe.py:1010-1045): wts[t][k] *= scale[ids[t][k]], one thread per assignment
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_wscale(int assignments, int E, const int32_t* __restrict__ ids,
                                                float* __restrict__ wts, const float* __restrict__ scale) {
  const int a = blockIdx.x * 256 + threadIdx.x;
  if (a >= assignments) return;
  const int e = min(max(ids[a], 0), E - 1);
  wts[a] *= scale[e];
}

int moe_wscale(int tokens, int ku, int n_experts, const int32_t* ids, float* wts, const float* scale, cudaStream_t s) {
  const int a = tokens * ku;
  k_wscale<<<(a + 255) / 256, 256, 0, s>>>(a, n_experts, ids, wts, scale);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

// ---------------------------------------------------------------------------------------------------------------
// g_moe_shared_gate (gen_moe.py:780-823): sg[t] = sigmoid(x[t] . w), one warp per token (8 per CTA), each lane over
// 4-value slices of h, f32 accumulation
// ---------------------------------------------------------------------------------------------------------------
template <bool BF16W>
__global__ void __launch_bounds__(256) k_shared_gate(int tokens, int h, const float* __restrict__ x,
                                                     const void* __restrict__ w, float* __restrict__ sg) {
  const int lane = threadIdx.x & 31;
  const int64_t t = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const float* xr = x + t * h;
  float acc = 0.f;
  for (int i = lane * 4; i < h; i += 128) {
    const float4 xv = __ldg(reinterpret_cast<const float4*>(xr + i));
    float4 wv;
    if (BF16W) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(w) + i));
      wv = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
    } else {
      wv = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(w) + i));
    }
    acc = fmaf(xv.x, wv.x, fmaf(xv.y, wv.y, fmaf(xv.z, wv.z, fmaf(xv.w, wv.w, acc))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) sg[t] = 1.0f / (1.0f + expf(-acc));
}

int moe_shared_gate(int tokens, int h, const float* x, const void* w, int w_dtype, float* sg, cudaStream_t s) {
  if (w_dtype == LK_BF16) k_shared_gate<true><<<(tokens + 7) / 8, 256, 0, s>>>(tokens, h, x, w, sg);
  else k_shared_gate<false><<<(tokens + 7) / 8, 256, 0, s>>>(tokens, h, x, w, sg);
  return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ECUDA;
}

}  // namespace lk
