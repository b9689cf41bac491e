/*
 * liblk -- the B200 (sm_100a) quantized-matmul hot path of loom-fun/loom-skills behind a C ABI.
 *
 * Every entry point replaces one kernel family that the reference's Python generators emit as Loom IR; the comment on
 * each names the reference interface (path:line relative to the loom-skills checkout) whose launch signature it keeps:
 * the same operands in the same order, the same layouts (packed GGUF blocks, [rows][k] activations, [rows][n] f32
 * outputs, [rows][2] (scale, inverse) row factors, MoE tile_info/rowmap/pos schedules).
 *
 * Conventions
 *  - All pointers are device pointers (cudaMalloc'd or views of them); the caller owns every buffer, as the
 *    reference's command programs do. Nothing here allocates device memory (lk_peer_alloc, the multi-GPU buffer
 *    set-up, excepted) or synchronises (lk_device_status excepted).
 *  - Work is enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream).
 *  - Return 0 (LK_OK) or a negative LK_E* code after host-side validation of formats, shapes and alignment. The
 *    reference has no runtime errors (its contracts are index.assume preconditions); violating one here is an error
 *    code, not undefined behaviour. A CUDA launch error is LK_ECUDA.
 *  - Weight formats use the ggml type ids (gguf.GGMLQuantizationType).
 */
#ifndef LK_H
#define LK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* lk_stream_t;   /* == cudaStream_t */

/* weight formats (ggml type ids); LK_MXFP4S = split planes (nibble plane + E8M0 scale plane), formats.py:11-14.
 * The Q4 family (Q4_0, Q4_K, IQ4_NL) and MXFP4S run on every kernel; Q5_0, Q8_0, Q3_K, Q5_K, Q6_K, IQ4_XS, IQ3_S
 * and the ggml 17-byte MXFP4 blocks (the reference's remaining formats, formats.py:5-17) on lk_dequant, the decode
 * matvecs (lk_mv, lk_moe_expert_mv) and the prefill GEMMs (lk_gemm, lk_moe_grouped_gemm). */
enum {
  LK_Q4_0 = 2, LK_Q5_0 = 6, LK_Q8_0 = 8, LK_Q3_K = 11, LK_Q4_K = 12, LK_Q5_K = 13, LK_Q6_K = 14, LK_IQ4_NL = 20,
  LK_IQ3_S = 21, LK_IQ4_XS = 23, LK_MXFP4 = 39, LK_MXFP4S = 1039
};
/* Gate and up weights in two formats (Q4_K_M's Q4_K gate and Q6_K up; unsloth's mixed quants): the reference's
 * "GATE+UP" format (gen_moe.py:537-552 expert_mv, :1129-1141 grouped_gemm; gen_gemm.py:535-545 gemm fmt2 and
 * :1224-1251 gemm_big256 fmt2). LK_FMT_PAIR(gate, up) goes where a gate/up entry point takes `fmt`: lk_mv with w2,
 * lk_gemm with LK_SWIGLU, lk_moe_expert_mv[_ex] mode 0 and lk_moe_grouped_gemm[_ex] with LK_SWIGLU /
 * LK_SWIGLU_SORTED, the gate and up in separate tensors (fused = 0), each weight with its own row stride and decode.
 * Either half is any format but LK_MXFP4S; k must be a whole number of both formats' blocks. A pair of one format is
 * that format. Any other entry point, mode or fused = 1 with a pair: LK_EINVAL. */
#define LK_FMT_PAIR(gate, up) ((int)(gate) | ((int)(up) << 16))
/* element types (ggml ids where ggml has one) */
enum { LK_F32 = 0, LK_F16 = 1, LK_BF16 = 30, LK_E4M3 = 1000 };
/* GEMM epilogues (gen_gemm.py:535 `mode`): y = acc, y += acc, y = silu(acc_w) * acc_w2. LK_SWIGLU_SORTED (grouped
 * GEMMs only; no counterpart in the reference, whose gate/up gathers token rows inside the GEMM): the swiglu gate/up
 * on activation rows already in bucket order (lk_moe_row_scale_gather's output), read as plain tiles. */
enum { LK_STORE = 0, LK_ACC = 1, LK_SWIGLU = 2, LK_SWIGLU_SORTED = 3 };
/* MXFP4 nibble order inside a 32-value block (gen_mxfp4s.py:1-7): OCP pairs, or ggml split16 */
enum { LK_ORDER_PAIRS = 0, LK_ORDER_SPLIT16 = 1 };
/* expert gate/up activations (gen_moe.py:27-64 act_scalar; cfg moe.act): silu(g) * u; GEGLU gelu_tanh(g) * u (the
 * gemma4 kit's ffn_act "gelu", make_kernel_tests.py:78-80); gpt-oss swiglu_oai: x = min(g, limit),
 * y = clamp(u, -limit, limit), x * sigmoid(alpha * x) * (y + 1) (llama.cpp ggml_swiglu_oai; alpha 1.702, limit 7) */
enum { LK_ACT_SILU = 0, LK_ACT_GELU = 1, LK_ACT_SWIGLU_OAI = 2 };

#define LK_OK 0
#define LK_EINVAL (-1)       /* unknown format / mode / dtype, bad shape, null pointer */
#define LK_EALIGN (-2)       /* a pointer or row stride is not aligned as the kernel's loads require */
#define LK_ECUDA (-3)        /* the launch failed (cudaGetLastError) */
#define LK_EUNSUPPORTED (-4) /* a valid combination this build has no kernel for */
#define LK_ERANGE (-5)       /* a size beyond a stated maximum */

const char* lk_strerror(int code);
int lk_version(void);
/* Device-side status (synchronous; no reference counterpart): bit 0 = a kernel's bounded wait on an mbarrier gave
 * up (its results are not valid). clear != 0 resets it. */
unsigned int lk_device_status(int clear);
/* packed bytes of one row of k values of `fmt` (gen_moe.py:70-71 row_bytes); -1 if k is not a block multiple */
int64_t lk_row_bytes(int fmt, int64_t k);

/* ---------------------------------------------------------------------------------------------------------------
 * Block dequantisation, standalone (bit-exact check and weight staging).
 * Replaces the value helpers @g_q4_0_values / @g_iq4_nl_values (quant_values.loom:18-91, 386-408), @g_q4_k_values
 * (gen_llm.py:288-315), MXFP4 / MXFP4S (gen_llm.py:786-895) and, for out_dtype LK_F16, the GEMM staging
 * dequant16 (gen_gemm.py:281-532, moe_q4_0.py:11-38).
 * out_dtype LK_F32: the exact values (== gguf.quants.dequantize); LK_F16: one rounding of the exact value, except Q4_K
 * whose staging is fma_f16(q, f16(d*sc), f16(-dmin*m)) as gen_gemm.py:526-532.
 * w_scales: the E8M0 scale plane for LK_MXFP4S (pairs order), else NULL. n_values % 32 == 0 (256 for Q4_K).
 */
int lk_dequant(int fmt, const void* w, const void* w_scales, int64_t n_values, void* out, int out_dtype,
               lk_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Activation producers.
 * lk_row_scale_f16: g_row_scale_f16 (gen_llm.py:1843-1912), launch(%rows, %k, %x, %scales, %x16):
 *   e = clamp(exponent(max|x[row]|) - 127 - 13, 0, 100); scales[row] = (2^-e, 2^e); x16 = f16(x * 2^-e).
 *   x_dtype LK_F32 or LK_BF16.
 * lk_row_scale_f8: the fp8 producer twin g_row_scale_f16_f8_rdna4 (gen_mxfp4s.py:852-870, 887-938),
 *   launch(..., %x16, %x8, %s8, %w16): additionally x8 = e4m3(x * 2^(134 - b)), s8 = (2^(134-b), 2^(b-142)),
 *   b = biased exponent of the row max; x16/scales are written only when non-NULL (the %w16 flag).
 */
int lk_row_scale_f16(int rows, int k, const void* x, int x_dtype, float* scales, uint16_t* x16, lk_stream_t stream);
int lk_row_scale_f8(int rows, int k, const void* x, int x_dtype, float* scales, uint16_t* x16, uint8_t* x8, float* s8,
                    lk_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Decode matvec (tokens < 64). Replaces g_mv_{fmt}_k{K}[_t{TG}][_r{R}] and its swiglu pair (gen_llm.py:1159-1378),
 * launch(%n, %tokens, %accumulate, %x, %w [, %w2], %y): y[t][n] (+)= sum_k x[t][k] W[n][k];
 * w2 != NULL: y[t][n] (+)= silu(x.Wg[n]) * (x.Wu[n]).  x: [tokens][k] of x_dtype (LK_F32, LK_F16 or LK_BF16),
 * W: [n] packed rows. Every format lk_dequant decodes but LK_MXFP4S, and LK_FMT_PAIR(gate, up) with w2; k a whole
 * number of the format's blocks. The Q4 family with k % 256 == 0 and 16-byte aligned w runs the tuned kernel.
 */
int lk_mv(int fmt, int n, int k, int tokens, int accumulate, const void* x, int x_dtype, const void* w,
          const void* w2, float* y, lk_stream_t stream);
/* lk_silu_mul: g_silu_mul (gen_llm.py:5717-5745; gen_llm.py:77, 6280-6283: the glue after two projections of a gate
 * and up in different formats), launch(%tokens, %n, %f, %u): f[t][c] = act(f[t][c]) * u[t][c] over [tokens][n] f32,
 * in place; act LK_ACT_SILU, or LK_ACT_GELU for the GEGLU form (gen_llm.py:5670-5716). n % 4 == 0; f, u 16-byte
 * aligned. The LK_FMT_PAIR kernels make the two projections and this glue one launch. */
int lk_silu_mul(int tokens, int n, float* f, const float* u, int act, lk_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Decode matvec with int8 activations: the reference's default decode numerics (ACT_Q8=1, gen_llm.py:514-518).
 * lk_quant_q8: g_quant_q8 (gen_llm.py:683-750), launch(%rows, %width, %x, %xq): per 32-value group d = amax/127,
 *   q = round(x/d) (halves away from zero; 0 for an all-zero group); xq = codes int8 [rows][k], then at byte rows*k
 *   the meta [rows][k/32][2] f32 = (d rounded to f16, sum of the group's codes). x_dtype LK_F32 or LK_BF16, k % 32 == 0.
 *   xq holds rows*k + rows*(k/32)*8 bytes.
 * lk_mv_q8: g_mv_{fmt}_k{K}[_t{TG}]_q8 (gen_llm.py:1159-1378 with the @g_<fmt>_icodes helpers, :521-680, 898-1000,
 *   and the dot of iq_dot, :1017-1050), launch(%n, %tokens, %accumulate, %xq, %w, %y):
 *   y[t][n] (+)= sum_k dequant(W)[n][k] * xcode[t][k] * d[t][k/32], the weight codes contracted with the activation
 *   codes in integer arithmetic per 32-group, then scaled in f32 as the reference does per format. xq: lk_quant_q8's
 *   output for `tokens` rows. Formats: Q4_0 and Q4_K (k % 256 == 0, w 16-byte aligned) on the tuned kernels; Q8_0,
 *   Q5_0, Q5_K, Q6_K (the reference's ICODES set, formats.py:22-31) and IQ4_NL, IQ4_XS (its IQ4_Q8 choice) with k a
 *   whole number of blocks and of 32-value groups, w 2-byte aligned. Other decodable formats (Q3_K, IQ3_S, MXFP4):
 *   LK_EUNSUPPORTED, as the reference has no integer codes for them.
 */
int lk_quant_q8(int rows, int k, const void* x, int x_dtype, uint8_t* xq, lk_stream_t stream);
int lk_mv_q8(int fmt, int n, int k, int tokens, int accumulate, const uint8_t* xq, const void* w, float* y,
             lk_stream_t stream);
/* lk_mv_q8_multi: lk_mv_q8 for up to 4 weights that share one activation (the q | k | v projections of an attention
 * layer; the reference reaches the same with one fused attn_qkv tensor, gen_llm.py:99-100, 6221): segment g has n[g]
 * rows in w[g] and writes y[g]. One launch over all segments where the kernel allows, else one per segment.
 * n, w, y are HOST arrays of nseg entries. */
int lk_mv_q8_multi(int fmt, int nseg, const int* n, const void* const* w, float* const* y, int k, int tokens,
                   int accumulate, const uint8_t* xq, lk_stream_t stream);
/* lk_mv_q8_fused / lk_mv_q8_fused_multi: g_quant_q8 (gen_llm.py:683-750) and g_mv_{fmt}_q8 (gen_llm.py:1159-1378) of
 * one token in one launch, launch(%n, %accumulate, %x, %w, %y): the activation row x [1][k] (LK_F32 or LK_BF16) is
 * quantised to Q8_1 codes inside the matvec -- each CTA quantises the row into its shared memory, the codes and group
 * meta bit for bit lk_quant_q8's -- and contracted with the weight codes as lk_mv_q8 does; no xq buffer exists.
 * Formats Q4_0 and Q4_K, k a multiple of 4096 up to 12288 (LK_EUNSUPPORTED otherwise: lk_quant_q8 + lk_mv_q8 cover
 * every other shape); x 16-byte aligned. The _multi form takes up to 4 weights that share x, as lk_mv_q8_multi. */
int lk_mv_q8_fused(int fmt, int n, int k, int accumulate, const void* x, int x_dtype, const void* w, float* y,
                   lk_stream_t stream);
int lk_mv_q8_fused_multi(int fmt, int nseg, const int* n, const void* const* w, float* const* y, int k, int accumulate,
                         const void* x, int x_dtype, lk_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Prefill GEMM (tcgen05 + TMEM). Replaces g_gemm_{fmt}_{store,acc,swiglu}[_m128|_m256] (gen_gemm.py:535-704,
 * 706, 1224), launch(%rows, %k, %n, %x, %scales, %w [, %w2], %y):
 *   Y[rows][n] (+)= (X16 . W16^T) * scales[row][1]; swiglu: silu(G) * U with G, U the two weights' products.
 * x16: [rows][k] f16 (lk_row_scale_f16's output), scales: [rows][2] f32, y: [rows][n] f32.
 * Formats: every one lk_dequant decodes (MXFP4S planes: lk_gemm_mxfp4s_f8); LK_SWIGLU also LK_FMT_PAIR(gate, up),
 * whose two weights the kernel decodes each in its own format. k % 64 == 0 and a whole number of the format's
 * blocks, n % 16 == 0; x16 16-byte aligned; w 16-byte aligned for Q4_K outside a pair, 2-byte otherwise (ggml MXFP4
 * any). Any rows >= 1.
 * Store / acc may split K into ranges where that shortens the persistent grid's rounds (few output tiles, or a last
 * round that would run nearly empty). The ranges meet in y in a fixed order: range 0 stores (acc: adds onto y), and
 * range s adds its partial once ranges 0..s-1 have, through a per-tile flag in liblk's device memory. The results are
 * the same from run to run, bit for bit.
 */
int lk_gemm(int fmt, int mode, int rows, int k, int n, const uint16_t* x16, const float* scales, const void* w,
            const void* w2, float* y, lk_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * MXFP4 (split planes) x FP8 GEMM. Replaces g_gemm_mxfp4s_{store,swiglu}_f8_m256_rdna4
 * (gen_mxfp4s.py:50-500; signature test tests/test_mxfp4s_f8.py:150-160),
 * launch(%rows, %k, %n, %x, %scales, %w, %ws [, %w2, %w2s], %y): y = (x8 . (W * 2^8)^T) * s8[row][1].
 * x8: [rows][k] e4m3, s8: [rows][2] (lk_row_scale_f8), w: nibble plane [n][k/2], ws: E8M0 plane [n][k/32].
 * k % 32 == 0 (the reference asks k % 128; gpt-oss's k = 2880 is not), n % 16 == 0. The block scales are applied
 * by the tensor core (exact for every E8M0 value; the reference's e5m2 decode covers exponents 107..132 only).
 */
int lk_gemm_mxfp4s_f8(int mode, int order, int rows, int k, int n, const uint8_t* x8, const float* s8,
                      const uint8_t* w, const uint8_t* ws, const uint8_t* w2, const uint8_t* w2s, float* y,
                      lk_stream_t stream);
/* The MXFP4 x FP8 GEMM grouped over the MoE tile schedule: the grouped-GEMM signature (gen_moe.py:1145-1146,
 * %xrows, %tile_info, %rowmap before %x) with the fp8 GEMM's operands (gen_mxfp4s.py:101). Rows, tiles, gather,
 * fused gate/up and skipped tiles as lk_moe_grouped_gemm; x8/s8 as lk_gemm_mxfp4s_f8 (gate/up: [xrows] token rows,
 * LK_SWIGLU_SORTED gate/up and down: [rows] sorted rows); w/ws per expert n rows (fused gate/up: 2n, gate then up) of k/2 nibble bytes and k/32
 * E8M0 bytes. */
int lk_moe_grouped_gemm_mxfp4s_f8(int mode, int order, int rows, int k, int n, int xrows, int ku, int n_experts,
                                  int fused, const int32_t* tile_info, const int32_t* rowmap, const uint8_t* x8,
                                  const float* s8, const uint8_t* w, const uint8_t* ws, const uint8_t* w2,
                                  const uint8_t* w2s, float* y, lk_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * MoE (gen_moe.py). Assignment a = t * ku + slot.
 * lk_moe_route: g_moe_route / g_moe_route_tr (gen_moe.py:116-253, 255-470), launch(%tokens, %h, %router_w, %bias,
 *   %ids, %wts). gating 1 softmax (+ top-k, renormalised when norm: w / max(sum, 6.1e-5)), 2 sigmoid (+ bias for the
 *   pick), 3 top-k of logit+bias weighted by a softmax over the picked. Ties: lowest expert index. `scale` multiplies
 *   the final weights (expert_weights_scale, gen_moe.py:111-113). router_w == NULL: x already holds the logits
 *   [tokens][n_experts] (f32); else x is [tokens][h] f32 and router_w [n_experts][h] of w_dtype (LK_F32/LK_BF16).
 *   n_experts <= 256, ku <= 8.
 * lk_moe_bucket: g_moe_bucket (gen_moe.py:829-955), launch(%tokens, %max_tiles, %info, %ids, %tile_info, %rowmap,
 *   %pos): 64-row tiles per expert in expert order; tile_info[max_tiles][2] = (expert, rows) or (-1, 0);
 *   rowmap[max_tiles*64] = a or -1; pos[tokens*ku] = row or -1. info == NULL: every token live, else live =
 *   info[t*4+2] != 0. Rows of one expert follow ascending a (deterministic; the reference orders them by atomics).
 * lk_moe_grouped_gemm: g_moe_ggu_{fmt}[_fused]_k{H} / g_moe_gdn_{fmt}_k{F} (gen_moe.py:1126-1228), launch(%rows,
 *   %k, %n, %xrows, %tile_info, %rowmap, %x, %scales, %w [, %w2], %y). mode LK_SWIGLU (gate/up): A rows gathered
 *   from x16[rowmap[r] / ku] (rowmap < 0 -> zero row), y[r] = silu(g) * u with g, u scaled by scales[token][1];
 *   fused: w holds per expert n gate rows then n up rows. mode LK_SWIGLU_SORTED: the same gate/up with A = sorted
 *   rows x16[r] and scales[r] (x16 [rows][k] from lk_moe_row_scale_gather; xrows is then not read). mode LK_STORE
 *   (down): A = sorted rows x16[r], y[r] = acc * scales[r][1]. Tiles with expert < 0 are skipped (their y rows are
 *   not written).
 * lk_moe_combine_sorted: g_moe_combine_sorted (gen_moe.py:1231-1280), launch(%tokens, %rows, %ys, %pos, %wts, %y):
 *   y[t] (+)= sum_k wts[t][k] * ys[pos[t][k]] (pos < 0 -> 0).
 * lk_moe_expert_mv: decode expert matvecs g_moe_gu_{fmt} / g_moe_dn_{fmt} (gen_moe.py:535-727): mode 0 (gu):
 *   y[a] = silu(Wg[e] x[a/ku]) * (Wu[e] x[a/ku]); mode 1 (dn): y[a] = Wd[e] x[a]; e = ids[a]. With Q4_0 / Q4_K /
 *   IQ4_NL experts, 128 to 1024 assignments over at most 256 experts (several decode tokens), the launch groups the
 *   assignments by expert and reads an expert's rows once for up to 8 of them; every y[a] is bit for bit the
 *   per-assignment result, and no scratch memory is used.
 * The gate/up forms of both (expert_mv mode 0, grouped LK_SWIGLU / LK_SWIGLU_SORTED) take LK_FMT_PAIR(gate, up) with
 *   fused = 0: w the gate experts [n_experts][n] rows, w2 the up experts, each in its own format.
 * lk_moe_combine: g_moe_combine (gen_moe.py:730-762): y[t] (+)= sum_k wts[t][k] ys[t*ku + k].
 */
int lk_moe_route(int tokens, int h, int n_experts, int ku, int gating, int norm, float scale, const float* x,
                 const void* router_w, int w_dtype, const float* bias, int32_t* ids, float* wts, lk_stream_t stream);
int lk_moe_bucket(int tokens, int ku, int n_experts, int max_tiles, const int32_t* info, const int32_t* ids,
                  int32_t* tile_info, int32_t* rowmap, int32_t* pos, lk_stream_t stream);
int lk_moe_grouped_gemm(int fmt, int mode, int rows, int k, int n, int xrows, int ku, int n_experts, int fused,
                        const int32_t* tile_info, const int32_t* rowmap, const uint16_t* x16, const float* scales,
                        const void* w, const void* w2, float* y, lk_stream_t stream);
/* lk_moe_row_scale_gather: the gate/up activations of a bucketed MoE in bucket order. No single counterpart in the
 * reference: it is the gather g_moe_ggu_* does on its A loads (gen_moe.py:1126-1228) moved into the row-scale
 * producer (g_row_scale_f16 / its fp8 twin, gen_llm.py:1843-1912, gen_mxfp4s.py:887-938). Row r of the outputs is
 * lk_row_scale_f16 / lk_row_scale_f8 of x[rowmap[r] / ku] (a zero row where rowmap[r] < 0), bit for bit; x16/scales
 * and x8/s8 are written when non-NULL. rows = the schedule's rows (max_tiles * 64); k % 8 == 0; x, x16 16-byte and
 * x8 8-byte aligned. Feed the outputs to the grouped GEMMs with LK_SWIGLU_SORTED. */
int lk_moe_row_scale_gather(int rows, int k, int ku, const int32_t* rowmap, const void* x, int x_dtype,
                            float* scales, uint16_t* x16, uint8_t* x8, float* s8, lk_stream_t stream);
int lk_moe_combine_sorted(int tokens, int rows, int h, int ku, int accumulate, const float* ys, const int32_t* pos,
                          const float* wts, float* y, lk_stream_t stream);
int lk_moe_expert_mv(int fmt, int mode, int n, int k, int assignments, int ku, int n_experts, int fused,
                     const int32_t* ids, const void* x, int x_dtype, const void* w, const void* w2, float* y,
                     lk_stream_t stream);
int lk_moe_combine(int tokens, int h, int ku, int accumulate, const float* ys, const float* wts, float* y,
                   lk_stream_t stream);
/* lk_moe_gate_up_routed: lk_moe_route (over the given logits) and lk_moe_expert_mv_ex mode 0 of ONE decode token in
 * one launch (g_moe_route + g_moe_gu_{fmt}, gen_moe.py:116-253, 535-727): every CTA routes the token with the router's
 * own code, then runs its gate/up expert rows; ids [ku] and wts [ku] receive the routing, bit for bit lk_moe_route's,
 * and y [ku][f] = act(Wg[e] x + bias, Wu[e] x + bias2) as lk_moe_expert_mv_ex gives. logits [n_experts] f32,
 * router_bias as lk_moe_route's (gating 2 / 3), x [h] of x_dtype; w / w2 / fused / biases as lk_moe_expert_mv_ex.
 * Formats Q4_0, Q4_K, IQ4_NL with h % 256 == 0 and 16-byte aligned x and weights; n_experts <= 256, ku <= 8
 * (LK_ERANGE beyond). A per-expert down scale (lk_moe_wscale) applies to wts afterwards as it does after the router. */
int lk_moe_gate_up_routed(int fmt, int h, int f, int n_experts, int ku, int gating, int norm, float scale,
                          const float* logits, const float* router_bias, const void* x, int x_dtype, const void* w,
                          const void* w2, int fused, const float* bias, const float* bias2, int act, float alpha,
                          float limit, int32_t* ids, float* wts, float* y, lk_stream_t stream);
/* lk_moe_expert_mv_q8: the decode expert matvecs on int8 activations, g_moe_gu_{fmt}_q8 / g_moe_dn_{fmt}_q8
 * (MOE_Q8, gen_llm.py:5290-5302; gen_moe.py:535-727 with iq): xq is lk_quant_q8's output for the activation rows --
 * mode 0 (gu): the tokens' rows (assignment a reads row a / ku; assignments % ku == 0), y[a] = act(Wg[e] x, Wu[e] x)
 * with w / w2 / fused as lk_moe_expert_mv; mode 1 (dn): one row per assignment (the quantised activations),
 * y[a] = Wd[e] x[a]; e = ids[a]. Per 32-value group an exact integer dot of the weight and activation codes, scaled in
 * f32 as lk_mv_q8 does. Formats: Q4_0, Q4_K, Q8_0, Q5_0, Q5_K, Q6_K (the reference's MoE int8 formats; no IQ4, no
 * biases); k a whole number of blocks and of 32-value groups; xq 16-byte, w 2-byte aligned. */
int lk_moe_expert_mv_q8(int fmt, int mode, int n, int k, int assignments, int ku, int n_experts, int fused,
                        const int32_t* ids, const uint8_t* xq, const void* w, const void* w2, int act, float alpha,
                        float limit, float* y, lk_stream_t stream);
/* lk_moe_expert_mv_mxfp4s: lk_moe_expert_mv over MXFP4S experts (the reference's expert_mv, gen_moe.py:535-727, with
 * the split-plane MXFP4S format of gen_llm.py:844-895; the MoE counterpart of lk_moe_grouped_gemm_mxfp4s_f8 at decode
 * sizes). w / ws: nibble plane [rows][k/2] and E8M0 plane [rows][k/32] of the stacked experts -- mode 0 (gu): per
 * expert n gate rows then n up rows of k values, y[a] = silu(Wg x[a/ku]) * (Wu x[a/ku]); mode 1 (dn): per expert n
 * rows, y[a] = Wd x[a]. order: LK_ORDER_PAIRS or LK_ORDER_SPLIT16. The activations (f32, f16 or bf16) are multiplied
 * in f32 with the exact MXFP4 values, f32 accumulation. k % 32 == 0 and k <= 4096 (LK_EUNSUPPORTED beyond);
 * assignments <= 65535 (LK_ERANGE beyond); x, w 16-byte aligned. */
int lk_moe_expert_mv_mxfp4s(int mode, int order, int n, int k, int assignments, int ku, int n_experts,
                            const int32_t* ids, const void* x, int x_dtype, const uint8_t* w, const uint8_t* ws,
                            float* y, lk_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * MoE epilogue variants: the same kernels with the reference's expert activation choice and per-expert output biases
 * (gen_moe.py:958-1007 _gemm_bias_act; expert_mv(bias=True, act=...), gen_moe.py:535-727). The biases are f32
 * [n_experts][n]: gate/up modes add bias (gate) and bias2 (up) to the two products before the activation, as
 * g_moe_ggu_* / g_moe_gu_* launch(..., %w, %w2, %bg, %bu, %y); down / store modes add bias (bias2 unused), as
 * launch(..., %w, %bd, %y). NULL biases: none. act: LK_ACT_* (gate/up modes; ignored otherwise); alpha, limit: the
 * swiglu_oai constants. The plain entry points above are these with LK_ACT_SILU and no biases.
 * A grouped GEMM writes every row of each live 64-row tile (rows past the tile's count hold the activation of zero
 * products plus the biases, zeros without biases, as the reference's tiles do) and no row of a dead tile.
 */
int lk_moe_grouped_gemm_ex(int fmt, int mode, int rows, int k, int n, int xrows, int ku, int n_experts, int fused,
                           const int32_t* tile_info, const int32_t* rowmap, const uint16_t* x16, const float* scales,
                           const void* w, const void* w2, const float* bias, const float* bias2, int act, float alpha,
                           float limit, float* y, lk_stream_t stream);
int lk_moe_grouped_gemm_mxfp4s_f8_ex(int mode, int order, int rows, int k, int n, int xrows, int ku, int n_experts,
                                     int fused, const int32_t* tile_info, const int32_t* rowmap, const uint8_t* x8,
                                     const float* s8, const uint8_t* w, const uint8_t* ws, const uint8_t* w2,
                                     const uint8_t* w2s, const float* bias, const float* bias2, int act, float alpha,
                                     float limit, float* y, lk_stream_t stream);
int lk_moe_expert_mv_ex(int fmt, int mode, int n, int k, int assignments, int ku, int n_experts, int fused,
                        const int32_t* ids, const void* x, int x_dtype, const void* w, const void* w2,
                        const float* bias, const float* bias2, int act, float alpha, float limit, float* y,
                        lk_stream_t stream);
int lk_moe_expert_mv_mxfp4s_ex(int mode, int order, int n, int k, int assignments, int ku, int n_experts,
                               const int32_t* ids, const void* x, int x_dtype, const uint8_t* w, const uint8_t* ws,
                               const float* bias, const float* bias2, int act, float alpha, float limit, float* y,
                               lk_stream_t stream);
/* lk_moe_wscale: g_moe_wscale (gen_moe.py:1010-1045), launch(%tokens, %ids, %wts, %scale): in place,
 *   wts[t][k] *= scale[clamp(ids[t][k], 0, n_experts - 1)] -- a per-expert down scale (ffn_down_exps.scale) folded
 *   into the combine weights before the experts run.
 * lk_moe_shared_gate: g_moe_shared_gate (gen_moe.py:780-823), launch(%tokens, %x, %w, %sg): sg[t] = sigmoid(x[t] . w)
 *   (the Qwen shared-expert gate ffn_gate_inp_shexp), x [tokens][h] f32, w [h] of w_dtype (LK_F32 / LK_BF16), f32
 *   accumulation; h % 32 == 0.
 * lk_moe_combine_gated / lk_moe_combine_sorted_gated: the combines made shared_gated (gen_moe.py:765-777):
 *   y[t] = sg[t] * y[t] + sum_k wts[t][k] * ys[...] -- y holds the shared experts' output on entry. */
int lk_moe_wscale(int tokens, int ku, int n_experts, const int32_t* ids, float* wts, const float* scale,
                  lk_stream_t stream);
/* lk_moe_ffn_decode_q8: the decode MoE layer on int8 activations -- MOE_Q8=1, the reference's default with ACT_Q8
 * (gen_llm.py:5290-5302) -- in two launches: routing of every token from `logits` (lk_moe_route's rules: gating,
 * norm, scale, router_bias), g_quant_q8 of x (gen_llm.py:683-750) and the int8 gate/up expert matvecs with
 * act(g + b_gate, u + b_up) into act_buf [tokens * ku][f] (gen_moe.py:535-727); then g_quant_q8 of act_buf, the
 * int8 down expert matvecs (+ b_down) and the weighted combine in assignment order (gen_moe.py:730-777, 1010-1045):
 *   y[t] = (accumulate ? (sg ? sg[t] : 1) y[t] : 0) + sum_k wts[t,k] dsc[e] (Wd[e] act_k + bd[e]),  e = ids[t,k]
 * the same fma chain as lk_moe_combine. Weights: w_gate / w_up [E][f] rows of k = h (w_up null: w_gate holds each
 * expert's f gate rows then f up rows), w_down [E][h] rows of k = f; Q4_0 or Q4_K. ids / wts (both or neither):
 * the routing, combine weights after down_scale. Limits: h a multiple of 2048 up to 4096, f % 256 == 0 and
 * f <= 4096 (LK_EUNSUPPORTED / LK_ERANGE beyond), tokens <= 4, ku <= 8, n_experts <= 256, tokens * ku * f <= 65536;
 * x, act_buf and the weights 16-byte aligned. */
int lk_moe_ffn_decode_q8(int fmt, int tokens, int h, int f, int n_experts, int ku, int gating, int norm, float scale,
                         const float* logits, const float* router_bias, const float* down_scale, const void* x,
                         int x_dtype, const void* w_gate, const void* w_up, const void* w_down, const float* b_gate,
                         const float* b_up, const float* b_down, int act, float alpha, float limit, float* act_buf,
                         int32_t* ids, float* wts, const float* sg, int accumulate, float* y, lk_stream_t stream);
int lk_moe_shared_gate(int tokens, int h, const float* x, const void* w, int w_dtype, float* sg, lk_stream_t stream);
int lk_moe_combine_gated(int tokens, int h, int ku, const float* ys, const float* wts, const float* sg, float* y,
                         lk_stream_t stream);
int lk_moe_combine_sorted_gated(int tokens, int rows, int h, int ku, const float* ys, const int32_t* pos,
                                const float* wts, const float* sg, float* y, lk_stream_t stream);

/* lk_moe_ffn_decode_noalloc: the decode MoE layer in one call that allocates nothing. No counterpart in the
 * reference. It runs lk_moe_route (gating 1 over the given logits [tokens][n_experts] f32, renormalised when norm),
 * then lk_moe_expert_mv in both modes (w_gu: per expert f gate rows then f up rows of h values; w_dn: per expert
 * h rows of f values), then lk_moe_combine into y [tokens][h] f32. Its four intermediates (ids, weights, activations,
 * expert outputs) live in one fixed device array inside liblk instead of buffers the caller allocates.
 * It is for callers that cannot call cudaMalloc: an embedding runtime with a fixed device-memory budget, a host
 * callback, or a process whose device allocator belongs to someone else.
 * Limits: tokens * ku <= 128, h <= 4096, f <= 4096 (LK_ERANGE beyond); h % 256 == f % 256 == 0.
 * Every call on a device shares the one array, so calls that overlap on the GPU (other streams, other host threads)
 * race. Nothing in the array needs to start at zero. The first call on a device looks up the array's address
 * (cudaGetSymbolAddress); make that call before any stream capture. */
int lk_moe_ffn_decode_noalloc(int fmt, int tokens, int h, int f, int n_experts, int ku, int norm,
                              const float* logits, const void* x, int x_dtype, const void* w_gu, const void* w_dn,
                              float* y, lk_stream_t stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Multi-GPU: N-sharded GEMM with the all-gather fused into the epilogue. No reference counterpart (the reference
 * runs on one device); the sharding is the one BASELINE.json asks for (output columns across the GPUs of one box).
 * lk_peer_alloc: a device buffer of `bytes` (cudaMalloc) and its 64-byte interprocess handle; lk_peer_open maps a
 *   peer rank's handle into this process with peer access enabled; lk_peer_close / lk_peer_free release them.
 * lk_gemm_allgather: the prefill GEMM of this rank's shard (n_local output columns from its slice of weight rows),
 *   every output tile stored to all n_dst ranks' y buffers ([rows][n_total] f32, this rank's included) at columns
 *   col_offset .. col_offset + n_local - 1: P2P stores over NVLink as each tile finishes. y_dst is a HOST array of
 *   n_dst (<= 8) device pointers, y_dst[0] this rank's own buffer: when K is split into ranges (the store case of
 *   lk_gemm), a tile's ranges meet there in order and the last range stores the finished tile to every buffer. The
 *   caller orders the call against readers of the y buffers (a barrier of the ranks before and after). mode LK_STORE
 *   or LK_SWIGLU (w2 = this rank's up shard).
 */
/* Expert-parallel dispatch (no reference counterpart). Assignment a goes to rank ids[a] / n_local.
 * lk_moe_rank_plan: a stable sort of the assignments by destination rank: order[i] = the i-th assignment in
 *   (rank, a) order, pos[a] = its place in order, counts[r] = the assignments for rank r. assignments <= 65536,
 *   world <= 32. The rows of rank r are order[sum(counts[< r]) ..]; the returned results, in the same order, combine
 *   with lk_moe_combine_sorted(pos).
 * lk_moe_gather_rows: out[i] = x[order[i] / ku] (rows of h values, LK_F32 or LK_BF16, 16-byte aligned, h * size a
 *   multiple of 16), eid[i] = ids[order[i]] % n_local (eid may be NULL). */
int lk_moe_rank_plan(int assignments, int n_local, int world, const int32_t* ids, int32_t* order, int32_t* pos,
                     int32_t* counts, lk_stream_t stream);
int lk_moe_gather_rows(int rows, int h, int ku, int n_local, const int32_t* order, const int32_t* ids, const void* x,
                       int x_dtype, void* out, int32_t* eid, lk_stream_t stream);

int lk_peer_alloc(int64_t bytes, void** ptr, void* handle64);
int lk_peer_open(const void* handle64, void** ptr);
int lk_peer_close(void* ptr);
int lk_peer_free(void* ptr);
int lk_gemm_allgather(int fmt, int mode, int rows, int k, int n_local, const uint16_t* x16, const float* scales,
                      const void* w, const void* w2, float* const* y_dst, int n_dst, int n_total, int col_offset,
                      lk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* LK_H */
