// Internal launchers shared between the kernel files and the C-ABI layer (lk_api.cu). Validation happens in lk_api.cu;
// these assume their arguments were checked.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace lk {

// What a MoE expert kernel applies after its products: the activation of a gate/up pair (LK_ACT_*) and per-expert
// output biases ([n_experts][n] f32; bias: the gate's (gate/up) or the down projection's, bias2: the up projection's),
// as the reference's bias epilogues (gen_moe.py:958-1007 _gemm_bias_act; expert_mv(bias=...), gen_moe.py:535).
// Zero-initialised: SiLU, no biases.
struct ExpertEpi {
  const float* bias;
  const float* bias2;
  int act;
  float alpha, limit;
};

int dequant(int fmt, const void* w, const void* ws, int64_t n_values, void* out, int out_dtype, cudaStream_t s);
int row_scale(int rows, int k, const void* x, int x_dtype, float* scales, uint16_t* x16, uint8_t* x8, float* s8,
              cudaStream_t s);
int row_scale_gather(int rows, int k, int ku, const int32_t* rowmap, const void* x, int x_dtype, float* scales,
                     uint16_t* x16, uint8_t* x8, float* s8, cudaStream_t s);

// decode matvec, dense and per-assignment (MoE) forms
struct MvArgs {
  const uint8_t* w;      // packed rows of the first weight (expert 0 for MoE)
  const uint8_t* w2;     // second weight (swiglu) or nullptr
  const void* x;         // activations [x_rows][k]
  float* y;              // outputs [y_rows][n]
  int n, k;
  int tokens;            // dense: number of token rows
  int accumulate;
  int x_dtype;
  int64_t row_bytes;
  // MoE per-assignment mode (ids != nullptr): CTA column g = assignment, expert = ids[g],
  // x row = g / x_div (gu: x_div = ku; dn: 1), y row = g
  const int32_t* ids;
  int x_div;
  int n_experts;
  int rows_per_expert;    // weight rows of one expert in w (fused gate/up: 2n)
  int rows_per_expert2;   // weight rows of one expert in w2
  int w2_row_offset;      // first row of the second weight inside an expert (fused gate/up: n; else 0)
  int swiglu;
  ExpertEpi epi;          // MoE mode: activation and per-expert biases (dense: SiLU, no biases)
  // gate and up in two formats (mv_generic with an LK_FMT_PAIR id fills these): the formats and the up rows' stride
  int fmt, fmt2;
  int64_t row_bytes2;
  // the router folded into a one-token gate/up launch (mv_routed): the token's logits, router bias and settings;
  // ids_out / wts_out receive the routing (n_experts experts, top x_div)
  const float* logits;
  const float* rbias;
  int32_t* ids_out;
  float* wts_out;
  int gating, norm;
  float rscale;
};
// f = act(f) * u over [tokens][n] f32 (lk_silu_mul)
int act_mul(int tokens, int n, int act, float* f, const float* u, cudaStream_t s);
int mv(int fmt, const MvArgs& a, int groups, cudaStream_t s);
// every decodable format and any k of whole blocks (lk_mvg.cu): exact f32 values x f32 activations
int mv_generic(int fmt, const MvArgs& a, cudaStream_t s);
// the router and the gate/up expert matvecs of one decode token in one launch (Q4 formats, tuned layout)
int mv_routed(int fmt, const MvArgs& a, cudaStream_t s);

// where a GEMM stores its tile: dst[d][row * ld + col_off + col] for d < ndst (at most 8)
struct OutSpec {
  float* dst[8];
  int ndst;
  int64_t ld;
  int col_off;
};
int gemm(int fmt, int mode, int rows, int k, int n, const uint16_t* x16, const float* scales, const void* w,
         const void* w2, float* y, cudaStream_t s, const int32_t* tile_info, const int32_t* rowmap, int xrows, int ku,
         int n_experts, int64_t expert_stride, int64_t w2_offset, const OutSpec* out = nullptr,
         const ExpertEpi* epi = nullptr, bool act_mul = false);

int gemm_mxfp4s(int mode, int order, int rows, int k, int n, const uint8_t* x8, const float* s8, const uint8_t* w,
                const uint8_t* ws, const uint8_t* w2, const uint8_t* w2s, float* y, cudaStream_t s);
// decode expert matvecs over MXFP4S experts (lk_mvmx.cu)
int moe_expert_mv_mx(int mode, int order, int n, int k, int assignments, int ku, int n_experts, const int32_t* ids,
                     const void* x, int x_dtype, const uint8_t* w, const uint8_t* ws, float* y, cudaStream_t s,
                     const ExpertEpi* epi = nullptr);
int gemm_mx(int mode, int order, int rows, int k, int n, const uint8_t* x8, const float* s8, const uint8_t* w,
            const uint8_t* ws, const uint8_t* w2, const uint8_t* w2s, float* y, cudaStream_t s,
            const int32_t* tile_info, const int32_t* rowmap, int xrows, int ku, int n_experts, int rows_per_expert,
            int w2_row_offset, const ExpertEpi* epi = nullptr);

int moe_route(int tokens, int h, int n_experts, int ku, int gating, int norm, float scale, const float* x,
              const void* router_w, int w_dtype, const float* bias, int32_t* ids, float* wts, cudaStream_t s);
int moe_bucket(int tokens, int ku, int n_experts, int max_tiles, const int32_t* info, const int32_t* ids,
               int32_t* tile_info, int32_t* rowmap, int32_t* pos, cudaStream_t s);
int moe_combine_sorted(int tokens, int rows, int h, int ku, int accumulate, const float* ys, const int32_t* pos,
                       const float* wts, float* y, cudaStream_t s);
int moe_combine(int tokens, int h, int ku, int accumulate, const float* ys, const float* wts, float* y,
                cudaStream_t s);
// shared_gated combines (sg != nullptr: y = sg * y + sum), the down-scale fold and the shared-expert gate
int moe_combine_g(int tokens, int h, int ku, const float* ys, const int32_t* pos, const float* wts, const float* sg,
                  float* y, cudaStream_t s);
int moe_wscale(int tokens, int ku, int n_experts, const int32_t* ids, float* wts, const float* scale, cudaStream_t s);
// expert-parallel dispatch: the stable sort of assignments by destination rank, and the gather of the send rows
int moe_rank_plan(int assignments, int n_local, int world, const int32_t* ids, int32_t* order, int32_t* pos,
                  int32_t* counts, cudaStream_t s);
int moe_gather_rows(int rows, int h, int ku, int n_local, const int32_t* order, const int32_t* ids, const void* x,
                    int x_dtype, void* out, int32_t* eid, cudaStream_t s);
int moe_shared_gate(int tokens, int h, const float* x, const void* w, int w_dtype, float* sg, cudaStream_t s);

// int8-activation decode path (xq: codes [rows][k] int8, then [rows][k/32][2] f32 meta)
int quant_q8(int rows, int k, const void* x, int x_dtype, uint8_t* xq, cudaStream_t s);
int mv_q8(int fmt, int n, int k, int tokens, int accumulate, const uint8_t* xq, const void* w, float* y,
          cudaStream_t s);
int mv_q8_multi(int fmt, int nseg, const int* ns, const void* const* ws, float* const* ys, int k, int tokens,
                int accumulate, const uint8_t* xq, cudaStream_t s);
// the other formats with integer weight codes (Q8_0, Q5_0, Q5_K, Q6_K, IQ4_NL, IQ4_XS; lk_mvq8g.cu)
bool mv_q8_generic_format(int fmt);
// per-assignment expert matvecs on int8 activation codes (MOE_Q8; lk_mvq8g.cu): mode 0 gate/up with act, 1 down;
// xq holds xrows rows of lk_quant_q8 output
int moe_expert_mv_q8(int fmt, int mode, int n, int k, int assignments, int ku, int n_experts, int fused,
                     const int32_t* ids, const uint8_t* xq, int xrows, const void* w, const void* w2, int act,
                     float alpha, float limit, float* y, cudaStream_t s);
int mv_q8_generic(int fmt, int n, int k, int tokens, int accumulate, const uint8_t* xq, const void* w, float* y,
                  cudaStream_t s);
// one token: the activation row quantised inside the row-streaming matvec (no xq buffer); LK_EUNSUPPORTED off its
// shapes (Q4_0 / Q4_K, k % 4096 == 0, k <= 12288)
int mv_q8_fused(int fmt, int nseg, const int* ns, const void* const* ws, float* const* ys, int k, int accumulate,
                const void* x, int x_dtype, cudaStream_t s);

// the decode MoE layer on int8 activations in two launches (lk_moeq8.cu); arguments of lk_moe_ffn_decode_q8
struct MoeFfnQ8 {
  int tokens, h, f, n_experts, ku, gating, norm;
  float scale;
  const float* logits;
  const float* router_bias;
  const float* down_scale;
  const void* x;
  int x_dtype;
  const void* w_gate;
  const void* w_up;
  const void* w_down;
  const float* b_gate;
  const float* b_up;
  const float* b_down;
  int act;
  float alpha, limit;
  float* act_buf;
  int32_t* ids;
  float* wts;
  const float* sg;
  int accumulate;
  float* y;
};
int moe_ffn_decode_q8(int fmt, const MoeFfnQ8& p, cudaStream_t s);

// device status words of the kernel files (bit 0: a bounded wait gave up)
unsigned int status_q8(bool clear);
unsigned int status_mv(bool clear);
unsigned int status_gemm(bool clear);
unsigned int status_mx(bool clear);
unsigned int status_moeq8(bool clear);

}  // namespace lk
