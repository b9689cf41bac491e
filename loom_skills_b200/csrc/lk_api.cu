// The C ABI of liblk: host-side validation, then the kernel launchers. See include/lk.h for the contract of each
// entry point and the reference interface it replaces.
#include "lk_common.cuh"
#include "lk_formats.cuh"
#include "lk_internal.h"

using namespace lk;

static bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
static bool q4_family(int fmt) { return fmt == LK_Q4_0 || fmt == LK_Q4_K || fmt == LK_IQ4_NL; }
static bool act_ok(int act) { return act == LK_ACT_SILU || act == LK_ACT_GELU || act == LK_ACT_SWIGLU_OAI; }
// formats the decode matvecs and GEMMs take: the Q4 family on the tuned kernels, the rest on the generic ones
static bool mv_format(int fmt) {
  return q4_family(fmt) || fmt == LK_Q5_0 || fmt == LK_Q8_0 || fmt == LK_Q3_K || fmt == LK_Q5_K || fmt == LK_Q6_K ||
         fmt == LK_IQ3_S ||
         fmt == LK_IQ4_XS || fmt == LK_MXFP4;
}
// the tuned Q4 kernels stream whole 256-value chunks by TMA: k % 256, 16-byte aligned rows
static bool tuned_q4(int fmt, int k, const void* w, const void* w2) {
  return q4_family(fmt) && k % 256 == 0 && aligned(w, 16) && (!w2 || aligned(w2, 16));
}
// LK_FMT_PAIR(gate, up) ids: the gate's format in the low 16 bits, the up weight's above; a pair of one format is
// that format
static int pair_norm(int fmt) { return (fmt >> 16) == (fmt & 0xffff) ? (fmt & 0xffff) : fmt; }
static bool is_pair(int fmt) { return (fmt >> 16) != 0; }
static int gate_fmt(int fmt) { return is_pair(fmt) ? (fmt & 0xffff) : fmt; }
static int up_fmt(int fmt) { return is_pair(fmt) ? (fmt >> 16) : fmt; }
// both formats of a (possibly paired) id decodable, k a whole number of both formats' blocks
static int pair_check(int fmt, int64_t k) {
  if (!mv_format(gate_fmt(fmt)) || !mv_format(up_fmt(fmt))) return LK_EUNSUPPORTED;
  if (k % fmt_qk(gate_fmt(fmt)) || k % fmt_qk(up_fmt(fmt))) return LK_EINVAL;
  return LK_OK;
}


extern "C" {

const char* lk_strerror(int code) {
  switch (code) {
    case LK_OK: return "ok";
    case LK_EINVAL: return "invalid argument (format, mode, dtype, shape or null pointer)";
    case LK_EALIGN: return "misaligned pointer or row stride";
    case LK_ECUDA: return "CUDA launch failed";
    case LK_EUNSUPPORTED: return "no kernel for this combination";
    case LK_ERANGE: return "size beyond the stated maximum";
  }
  return "unknown error";
}

int lk_version(void) { return 1; }

int64_t lk_row_bytes(int fmt, int64_t k) {
  const int qk = fmt == LK_MXFP4S ? 32 : fmt_qk(fmt), bb = fmt == LK_MXFP4S ? 16 : fmt_block_bytes(fmt);
  if (bb == 0 || k <= 0 || k % qk) return -1;
  return k / qk * bb;
}

// Reads (and optionally clears) the device-side status word: bit 0 = a kernel's bounded wait gave up. Synchronous.
unsigned int lk_device_status(int clear) {
  return status_mv(clear != 0) | status_gemm(clear != 0) | status_mx(clear != 0) | status_q8(clear != 0) |
         status_moeq8(clear != 0);
}

int lk_quant_q8(int rows, int k, const void* x, int x_dtype, uint8_t* xq, lk_stream_t stream) {
  if (rows < 0 || k <= 0 || k % 32) return LK_EINVAL;
  if (x_dtype != LK_F32 && x_dtype != LK_BF16) return LK_EINVAL;
  if (rows == 0) return LK_OK;
  if (!x || !xq) return LK_EINVAL;
  if (!aligned(xq, 16)) return LK_EALIGN;
  return quant_q8(rows, k, x, x_dtype, xq, (cudaStream_t)stream);
}

// the int8-activation matvec's formats: the Q4 pair on the tuned kernels (k % 256, 16-byte aligned rows), the other
// integer-code formats on k_mvq8g (k a whole number of blocks and of 32-value groups, 2-byte aligned blocks)
static int mv_q8_check(int fmt, int k, const void* w) {
  const bool gen = mv_q8_generic_format(fmt);
  if (fmt != LK_Q4_0 && fmt != LK_Q4_K && !gen) return mv_format(fmt) ? LK_EUNSUPPORTED : LK_EINVAL;
  if (k <= 0 || k % (gen ? fmt_qk(fmt) : 256) || k % 32) return LK_EINVAL;
  if (w && !aligned(w, gen ? 2 : 16)) return LK_EALIGN;
  return LK_OK;
}

int lk_mv_q8(int fmt, int n, int k, int tokens, int accumulate, const uint8_t* xq, const void* w, float* y,
             lk_stream_t stream) {
  if (int rc = mv_q8_check(fmt, k, nullptr)) return rc;
  if (n <= 0 || tokens < 0) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!xq || !w || !y) return LK_EINVAL;
  if (int rc = mv_q8_check(fmt, k, w)) return rc;
  if (!aligned(xq, 16)) return LK_EALIGN;
  if (mv_q8_generic_format(fmt)) return mv_q8_generic(fmt, n, k, tokens, accumulate, xq, w, y, (cudaStream_t)stream);
  return mv_q8(fmt, n, k, tokens, accumulate, xq, w, y, (cudaStream_t)stream);
}

int lk_mv_q8_multi(int fmt, int nseg, const int* n, const void* const* w, float* const* y, int k, int tokens,
                   int accumulate, const uint8_t* xq, lk_stream_t stream) {
  if (int rc = mv_q8_check(fmt, k, nullptr)) return rc;
  if (nseg <= 0 || nseg > 4 || !n || !w || !y) return LK_EINVAL;
  if (tokens < 0) return LK_EINVAL;
  for (int g = 0; g < nseg; ++g) {
    if (n[g] <= 0) return LK_EINVAL;
    if (tokens > 0 && (!w[g] || !y[g])) return LK_EINVAL;
    if (tokens > 0)
      if (int rc = mv_q8_check(fmt, k, w[g])) return rc;
  }
  if (tokens == 0) return LK_OK;
  if (!xq) return LK_EINVAL;
  if (!aligned(xq, 16)) return LK_EALIGN;
  if (mv_q8_generic_format(fmt)) {   // one launch per segment
    for (int g = 0; g < nseg; ++g)
      if (int rc = mv_q8_generic(fmt, n[g], k, tokens, accumulate, xq, w[g], y[g], (cudaStream_t)stream)) return rc;
    return LK_OK;
  }
  return mv_q8_multi(fmt, nseg, n, w, y, k, tokens, accumulate, xq, (cudaStream_t)stream);
}

int lk_mv_q8_fused_multi(int fmt, int nseg, const int* n, const void* const* w, float* const* y, int k, int accumulate,
                         const void* x, int x_dtype, lk_stream_t stream) {
  if (fmt != LK_Q4_0 && fmt != LK_Q4_K) return q4_family(fmt) ? LK_EUNSUPPORTED : LK_EINVAL;
  if (nseg <= 0 || nseg > 4 || !n || !w || !y) return LK_EINVAL;
  if (k <= 0 || k % 256) return LK_EINVAL;
  if (x_dtype != LK_F32 && x_dtype != LK_BF16) return LK_EINVAL;
  for (int g = 0; g < nseg; ++g) {
    if (n[g] <= 0 || !w[g] || !y[g]) return LK_EINVAL;
    if (!aligned(w[g], 16)) return LK_EALIGN;
  }
  if (!x) return LK_EINVAL;
  if (!aligned(x, 16)) return LK_EALIGN;
  if (k % 4096 || k > 3 * 4096) return LK_EUNSUPPORTED;
  return mv_q8_fused(fmt, nseg, n, w, y, k, accumulate, x, x_dtype, (cudaStream_t)stream);
}

int lk_mv_q8_fused(int fmt, int n, int k, int accumulate, const void* x, int x_dtype, const void* w, float* y,
                   lk_stream_t stream) {
  return lk_mv_q8_fused_multi(fmt, 1, &n, &w, &y, k, accumulate, x, x_dtype, stream);
}

int lk_dequant(int fmt, const void* w, const void* w_scales, int64_t n_values, void* out, int out_dtype,
               lk_stream_t stream) {
  if (!w || !out || n_values < 0) return LK_EINVAL;
  if (lk_row_bytes(fmt, 256) < 0) return LK_EINVAL;
  if (n_values % (fmt == LK_MXFP4S ? 32 : fmt_qk(fmt))) return LK_EINVAL;
  if (out_dtype != LK_F32 && out_dtype != LK_F16) return LK_EINVAL;
  if (fmt == LK_MXFP4S && !w_scales) return LK_EINVAL;
  if (!aligned(out, 16)) return LK_EALIGN;
  if (n_values == 0) return LK_OK;
  return dequant(fmt, w, w_scales, n_values, out, out_dtype, (cudaStream_t)stream);
}

// Zero-sized calls succeed before the pointer checks: an empty tensor has no storage (a null data pointer).
int lk_row_scale_f16(int rows, int k, const void* x, int x_dtype, float* scales, uint16_t* x16, lk_stream_t stream) {
  if (rows < 0 || k <= 0) return LK_EINVAL;
  if (x_dtype != LK_F32 && x_dtype != LK_BF16) return LK_EINVAL;
  if (rows == 0) return LK_OK;
  if (!x || !scales || !x16) return LK_EINVAL;
  return row_scale(rows, k, x, x_dtype, scales, x16, nullptr, nullptr, (cudaStream_t)stream);
}

int lk_row_scale_f8(int rows, int k, const void* x, int x_dtype, float* scales, uint16_t* x16, uint8_t* x8, float* s8,
                    lk_stream_t stream) {
  if (rows < 0 || k <= 0) return LK_EINVAL;
  if (x_dtype != LK_F32 && x_dtype != LK_BF16) return LK_EINVAL;
  if (rows == 0) return LK_OK;
  if (!x || !x8 || !s8) return LK_EINVAL;
  return row_scale(rows, k, x, x_dtype, scales, x16, x8, s8, (cudaStream_t)stream);
}

int lk_moe_row_scale_gather(int rows, int k, int ku, const int32_t* rowmap, const void* x, int x_dtype,
                            float* scales, uint16_t* x16, uint8_t* x8, float* s8, lk_stream_t stream) {
  if (rows < 0 || k <= 0 || k % 8 || ku <= 0) return LK_EINVAL;
  if (x_dtype != LK_F32 && x_dtype != LK_BF16) return LK_EINVAL;
  if (rows == 0) return LK_OK;
  if (!rowmap || !x || (!x16 && !x8) || (x16 && !scales) || (x8 && !s8)) return LK_EINVAL;
  if (!aligned(x, 16) || !aligned(x16, 16) || !aligned(x8, 8)) return LK_EALIGN;
  return row_scale_gather(rows, k, ku, rowmap, x, x_dtype, scales, x16, x8, s8, (cudaStream_t)stream);
}

int lk_silu_mul(int tokens, int n, float* f, const float* u, int act, lk_stream_t stream) {
  if (tokens < 0 || n <= 0 || n % 4) return LK_EINVAL;
  if (act != LK_ACT_SILU && act != LK_ACT_GELU) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!f || !u) return LK_EINVAL;
  if (!aligned(f, 16) || !aligned(u, 16)) return LK_EALIGN;
  return act_mul(tokens, n, act, f, u, (cudaStream_t)stream);
}

int lk_mv(int fmt, int n, int k, int tokens, int accumulate, const void* x, int x_dtype, const void* w, const void* w2,
          float* y, lk_stream_t stream) {
  fmt = pair_norm(fmt);
  if (!mv_format(gate_fmt(fmt)) || !mv_format(up_fmt(fmt))) return LK_EUNSUPPORTED;
  if (n <= 0 || k <= 0 || tokens < 0) return LK_EINVAL;
  if (int rc = pair_check(fmt, k)) return rc;
  if (is_pair(fmt) && !w2) return LK_EINVAL;   // a format pair is a gate/up matvec
  if (x_dtype != LK_F32 && x_dtype != LK_F16 && x_dtype != LK_BF16) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!x || !w || !y) return LK_EINVAL;
  if (!aligned(x, 16)) return LK_EALIGN;
  MvArgs a{};
  a.w = (const uint8_t*)w;
  a.w2 = (const uint8_t*)w2;
  a.x = x;
  a.y = y;
  a.n = n;
  a.k = k;
  a.tokens = tokens;
  a.accumulate = accumulate;
  a.x_dtype = x_dtype;
  a.row_bytes = lk_row_bytes(gate_fmt(fmt), k);
  a.swiglu = w2 != nullptr;
  if (tuned_q4(fmt, k, w, w2)) return mv(fmt, a, (tokens + 7) / 8, (cudaStream_t)stream);
  return mv_generic(fmt, a, (cudaStream_t)stream);
}

int lk_moe_expert_mv_mxfp4s_ex(int mode, int order, int n, int k, int assignments, int ku, int n_experts,
                               const int32_t* ids, const void* x, int x_dtype, const uint8_t* w, const uint8_t* ws,
                               const float* bias, const float* bias2, int act, float alpha, float limit, float* y,
                               lk_stream_t stream) {
  if (mode != 0 && mode != 1) return LK_EINVAL;
  if (order != LK_ORDER_PAIRS && order != LK_ORDER_SPLIT16) return LK_EINVAL;
  if (n <= 0 || k <= 0 || assignments < 0 || ku <= 0 || n_experts <= 0 || k % 32) return LK_EINVAL;
  if (x_dtype != LK_F32 && x_dtype != LK_F16 && x_dtype != LK_BF16) return LK_EINVAL;
  if (!act_ok(act)) return LK_EINVAL;
  if (mode == 0 && (!bias) != (!bias2)) return LK_EINVAL;
  if (k > 4096) return LK_EUNSUPPORTED;
  if (assignments > 65535) return LK_ERANGE;   // one grid row per assignment
  if (assignments == 0) return LK_OK;
  if (!ids || !x || !w || !ws || !y) return LK_EINVAL;
  if (!aligned(w, 16) || !aligned(x, 16)) return LK_EALIGN;
  ExpertEpi epi{bias, mode == 0 ? bias2 : nullptr, mode == 0 ? act : LK_ACT_SILU, alpha, limit};
  return moe_expert_mv_mx(mode, order, n, k, assignments, ku, n_experts, ids, x, x_dtype, w, ws, y,
                          (cudaStream_t)stream, &epi);
}

int lk_moe_expert_mv_mxfp4s(int mode, int order, int n, int k, int assignments, int ku, int n_experts,
                            const int32_t* ids, const void* x, int x_dtype, const uint8_t* w, const uint8_t* ws,
                            float* y, lk_stream_t stream) {
  return lk_moe_expert_mv_mxfp4s_ex(mode, order, n, k, assignments, ku, n_experts, ids, x, x_dtype, w, ws, nullptr,
                                    nullptr, LK_ACT_SILU, 0.f, 0.f, y, stream);
}

int lk_moe_expert_mv_ex(int fmt, int mode, int n, int k, int assignments, int ku, int n_experts, int fused,
                        const int32_t* ids, const void* x, int x_dtype, const void* w, const void* w2,
                        const float* bias, const float* bias2, int act, float alpha, float limit, float* y,
                        lk_stream_t stream) {
  fmt = pair_norm(fmt);
  if (!mv_format(gate_fmt(fmt)) || !mv_format(up_fmt(fmt))) return LK_EUNSUPPORTED;
  if (n <= 0 || k <= 0 || assignments < 0 || ku <= 0 || n_experts <= 0) return LK_EINVAL;
  if (mode != 0 && mode != 1) return LK_EINVAL;
  if (int rc = pair_check(fmt, k)) return rc;
  if (is_pair(fmt) && (mode != 0 || fused)) return LK_EINVAL;   // a pair: separate gate and up tensors
  if (x_dtype != LK_F32 && x_dtype != LK_F16 && x_dtype != LK_BF16) return LK_EINVAL;
  if (!act_ok(act)) return LK_EINVAL;
  if (mode == 0 && (!bias) != (!bias2)) return LK_EINVAL;
  if (assignments == 0) return LK_OK;
  if (!ids || !x || !w || !y) return LK_EINVAL;
  if (mode == 0 && !fused && !w2) return LK_EINVAL;
  if (!aligned(x, 16)) return LK_EALIGN;
  MvArgs a{};
  a.w = (const uint8_t*)w;
  a.w2 = (mode == 0 && !fused) ? (const uint8_t*)w2 : nullptr;
  a.x = x;
  a.y = y;
  a.n = n;
  a.k = k;
  a.tokens = assignments;
  a.x_dtype = x_dtype;
  a.row_bytes = lk_row_bytes(gate_fmt(fmt), k);
  a.ids = ids;
  a.x_div = mode == 0 ? ku : 1;
  a.n_experts = n_experts;
  a.rows_per_expert = n * ((mode == 0 && fused) ? 2 : 1);
  a.rows_per_expert2 = (mode == 0 && fused) ? 2 * n : n;   // fused: the up rows live in the same stacked tensor
  a.w2_row_offset = (mode == 0 && fused) ? n : 0;
  a.swiglu = mode == 0;
  a.epi = ExpertEpi{bias, mode == 0 ? bias2 : nullptr, mode == 0 ? act : LK_ACT_SILU, alpha, limit};
  if (tuned_q4(fmt, k, w, a.w2)) return mv(fmt, a, assignments, (cudaStream_t)stream);
  return mv_generic(fmt, a, (cudaStream_t)stream);
}

int lk_moe_expert_mv_q8(int fmt, int mode, int n, int k, int assignments, int ku, int n_experts, int fused,
                        const int32_t* ids, const uint8_t* xq, const void* w, const void* w2, int act, float alpha,
                        float limit, float* y, lk_stream_t stream) {
  if (fmt != LK_Q4_0 && fmt != LK_Q4_K && fmt != LK_Q8_0 && fmt != LK_Q5_0 && fmt != LK_Q5_K && fmt != LK_Q6_K)
    return mv_format(fmt) ? LK_EUNSUPPORTED : LK_EINVAL;
  if (n <= 0 || k <= 0 || assignments < 0 || ku <= 0 || n_experts <= 0) return LK_EINVAL;
  if (mode != 0 && mode != 1) return LK_EINVAL;
  if (k % fmt_qk(fmt) || k % 32) return LK_EINVAL;
  if (mode == 0 && assignments % ku) return LK_EINVAL;   // whole tokens of ku assignments
  if (!act_ok(act)) return LK_EINVAL;
  if (assignments == 0) return LK_OK;
  if (!ids || !xq || !w || !y) return LK_EINVAL;
  if (mode == 0 && !fused && !w2) return LK_EINVAL;
  if (!aligned(xq, 16) || !aligned(w, 2) || (mode == 0 && !fused && !aligned(w2, 2))) return LK_EALIGN;
  const int xrows = mode == 0 ? assignments / ku : assignments;
  return moe_expert_mv_q8(fmt, mode, n, k, assignments, ku, n_experts, fused, ids, xq, xrows, w, w2, act, alpha,
                          limit, y, (cudaStream_t)stream);
}

int lk_moe_gate_up_routed(int fmt, int h, int f, int n_experts, int ku, int gating, int norm, float scale,
                          const float* logits, const float* router_bias, const void* x, int x_dtype, const void* w,
                          const void* w2, int fused, const float* bias, const float* bias2, int act, float alpha,
                          float limit, int32_t* ids, float* wts, float* y, lk_stream_t stream) {
  if (!q4_family(fmt)) return mv_format(fmt) ? LK_EUNSUPPORTED : LK_EINVAL;
  if (h <= 0 || f <= 0 || n_experts <= 0 || ku <= 0 || h % 256) return LK_EINVAL;
  if (gating < 1 || gating > 3 || !act_ok(act)) return LK_EINVAL;
  if (n_experts > 256 || ku > 8 || ku > n_experts) return LK_ERANGE;
  if (x_dtype != LK_F32 && x_dtype != LK_F16 && x_dtype != LK_BF16) return LK_EINVAL;
  if (!logits || !x || !w || !ids || !wts || !y || (!fused && !w2)) return LK_EINVAL;
  if ((!bias) != (!bias2)) return LK_EINVAL;
  if (!aligned(x, 16) || !aligned(w, 16) || (!fused && !aligned(w2, 16))) return LK_EALIGN;
  MvArgs a{};
  a.w = (const uint8_t*)w;
  a.w2 = fused ? (const uint8_t*)w : (const uint8_t*)w2;
  a.x = x;
  a.y = y;
  a.n = f;
  a.k = h;
  a.tokens = ku;   // the token's assignments
  a.x_dtype = x_dtype;
  a.row_bytes = lk_row_bytes(fmt, h);
  a.x_div = ku;
  a.n_experts = n_experts;
  a.rows_per_expert = fused ? 2 * f : f;
  a.rows_per_expert2 = fused ? 2 * f : f;
  a.w2_row_offset = fused ? f : 0;
  a.swiglu = 1;
  a.epi = ExpertEpi{bias, bias2, act, alpha, limit};
  a.logits = logits;
  a.rbias = router_bias;
  a.ids_out = ids;
  a.wts_out = wts;
  a.gating = gating;
  a.norm = norm;
  a.rscale = scale;
  return mv_routed(fmt, a, (cudaStream_t)stream);
}

int lk_moe_expert_mv(int fmt, int mode, int n, int k, int assignments, int ku, int n_experts, int fused,
                     const int32_t* ids, const void* x, int x_dtype, const void* w, const void* w2, float* y,
                     lk_stream_t stream) {
  return lk_moe_expert_mv_ex(fmt, mode, n, k, assignments, ku, n_experts, fused, ids, x, x_dtype, w, w2, nullptr,
                             nullptr, LK_ACT_SILU, 0.f, 0.f, y, stream);
}

// the prefill GEMMs' weight contract: a whole number of 64-value stages and of the format's blocks; Q4_K alone keeps
// its 16-byte aligned rows (it takes the TMA box form), the others -- and either weight of a format pair, which takes
// the window form -- need 2-byte aligned blocks (MXFP4: any)
static int gemm_weight_check(int fmt, int k, const void* w, const void* w2) {
  if (int rc = pair_check(fmt, k)) return rc;
  if (k % 64) return LK_EINVAL;
  auto al = [&](int f) -> uintptr_t { return (f == LK_Q4_K && !is_pair(fmt)) ? 16 : f == LK_MXFP4 ? 1 : 2; };
  if (!aligned(w, al(gate_fmt(fmt))) || (w2 && !aligned(w2, al(up_fmt(fmt))))) return LK_EALIGN;
  return LK_OK;
}

int lk_gemm(int fmt, int mode, int rows, int k, int n, const uint16_t* x16, const float* scales, const void* w,
            const void* w2, float* y, lk_stream_t stream) {
  fmt = pair_norm(fmt);
  if (!mv_format(gate_fmt(fmt)) || !mv_format(up_fmt(fmt))) return LK_EUNSUPPORTED;
  if (mode != LK_STORE && mode != LK_ACC && mode != LK_SWIGLU) return LK_EINVAL;
  if (is_pair(fmt) && mode != LK_SWIGLU) return LK_EINVAL;
  if (rows < 0 || k <= 0 || n <= 0) return LK_EINVAL;
  if (n % 16) return LK_EINVAL;
  if (rows == 0) return LK_OK;
  if (!x16 || !scales || !w || !y) return LK_EINVAL;
  if (mode == LK_SWIGLU && !w2) return LK_EINVAL;
  if (int rc = gemm_weight_check(fmt, k, w, w2)) return rc;
  if (!aligned(x16, 16) || !aligned(y, 16)) return LK_EALIGN;
  return gemm(fmt, mode, rows, k, n, x16, scales, w, w2, y, (cudaStream_t)stream, nullptr, nullptr, rows, 1, 1, 0, 0);
}

int lk_gemm_allgather(int fmt, int mode, int rows, int k, int n_local, const uint16_t* x16, const float* scales,
                      const void* w, const void* w2, float* const* y_dst, int n_dst, int n_total, int col_offset,
                      lk_stream_t stream) {
  if (!q4_family(fmt)) return LK_EUNSUPPORTED;
  if (mode != LK_STORE && mode != LK_SWIGLU) return LK_EINVAL;
  if (rows < 0 || k <= 0 || n_local <= 0 || n_dst <= 0 || n_dst > kMaxPeers) return LK_EINVAL;
  if (k % 256 || n_local % 16 || n_total % 16 || col_offset % 16) return LK_EINVAL;
  if (col_offset < 0 || col_offset + n_local > n_total) return LK_EINVAL;
  if (rows == 0) return LK_OK;
  if (!x16 || !scales || !w || !y_dst) return LK_EINVAL;
  if (mode == LK_SWIGLU && !w2) return LK_EINVAL;
  if (!aligned(x16, 16) || !aligned(w, 16) || (w2 && !aligned(w2, 16))) return LK_EALIGN;
  OutSpec out{};
  for (int d = 0; d < n_dst; ++d) {
    if (!y_dst[d]) return LK_EINVAL;
    if (!aligned(y_dst[d], 16)) return LK_EALIGN;
    out.dst[d] = y_dst[d];
  }
  out.ndst = n_dst;
  out.ld = n_total;
  out.col_off = col_offset;
  return gemm(fmt, mode, rows, k, n_local, x16, scales, w, w2, y_dst[0], (cudaStream_t)stream, nullptr, nullptr,
              rows, 1, 1, 0, 0, &out);
}

int lk_moe_grouped_gemm_ex(int fmt, int mode, int rows, int k, int n, int xrows, int ku, int n_experts, int fused,
                           const int32_t* tile_info, const int32_t* rowmap, const uint16_t* x16, const float* scales,
                           const void* w, const void* w2, const float* bias, const float* bias2, int act, float alpha,
                           float limit, float* y, lk_stream_t stream) {
  fmt = pair_norm(fmt);
  if (!mv_format(gate_fmt(fmt)) || !mv_format(up_fmt(fmt))) return LK_EUNSUPPORTED;
  if (mode != LK_STORE && mode != LK_SWIGLU && mode != LK_SWIGLU_SORTED) return LK_EINVAL;
  if (is_pair(fmt) && (mode == LK_STORE || fused)) return LK_EINVAL;   // a pair: separate gate and up tensors
  if (rows < 0 || rows % 64 || k <= 0 || n <= 0 || xrows <= 0 || ku <= 0 || n_experts <= 0 || n_experts > kMaxExperts)
    return LK_EINVAL;
  if (!act_ok(act)) return LK_EINVAL;
  if (!tile_info || !rowmap || !x16 || !scales || !w || !y) return LK_EINVAL;
  const bool gu = mode != LK_STORE;   // gate/up: gathered or already sorted activation rows
  if (gu && !fused && !w2) return LK_EINVAL;
  if (gu && (!bias) != (!bias2)) return LK_EINVAL;   // gate and up biases come together
  if (n % 16) return LK_EINVAL;
  if (int rc = gemm_weight_check(fmt, k, w, w2)) return rc;
  if (!aligned(x16, 16) || !aligned(y, 16)) return LK_EALIGN;
  if (rows == 0) return LK_OK;
  int64_t rb = lk_row_bytes(gate_fmt(fmt), k);
  int64_t stride = rb * n * ((gu && fused) ? 2 : 1);
  const void* w2e = gu ? (fused ? nullptr : w2) : nullptr;
  ExpertEpi epi{bias, gu ? bias2 : nullptr, gu ? act : LK_ACT_SILU, alpha, limit};
  return gemm(fmt, mode, rows, k, n, x16, scales, w, w2e, y, (cudaStream_t)stream, tile_info, rowmap, xrows, ku,
              n_experts, stride, (gu && fused) ? rb * n : 0, nullptr, &epi);
}

int lk_moe_grouped_gemm(int fmt, int mode, int rows, int k, int n, int xrows, int ku, int n_experts, int fused,
                        const int32_t* tile_info, const int32_t* rowmap, const uint16_t* x16, const float* scales,
                        const void* w, const void* w2, float* y, lk_stream_t stream) {
  return lk_moe_grouped_gemm_ex(fmt, mode, rows, k, n, xrows, ku, n_experts, fused, tile_info, rowmap, x16, scales, w,
                                w2, nullptr, nullptr, LK_ACT_SILU, 0.f, 0.f, y, stream);
}

int lk_gemm_mxfp4s_f8(int mode, int order, int rows, int k, int n, const uint8_t* x8, const float* s8,
                      const uint8_t* w, const uint8_t* ws, const uint8_t* w2, const uint8_t* w2s, float* y,
                      lk_stream_t stream) {
  if (mode != LK_STORE && mode != LK_SWIGLU) return LK_EINVAL;
  if (order != LK_ORDER_PAIRS && order != LK_ORDER_SPLIT16) return LK_EINVAL;
  if (rows < 0 || k <= 0 || n <= 0) return LK_EINVAL;
  if (k % 32 || n % 16) return LK_EINVAL;
  if (rows == 0) return LK_OK;
  if (!x8 || !s8 || !w || !ws || !y) return LK_EINVAL;
  if (mode == LK_SWIGLU && (!w2 || !w2s)) return LK_EINVAL;
  if (!aligned(x8, 16) || !aligned(w, 16) || !aligned(y, 16)) return LK_EALIGN;
  if (w2 && !aligned(w2, 16)) return LK_EALIGN;
  return gemm_mxfp4s(mode, order, rows, k, n, x8, s8, w, ws, w2, w2s, y, (cudaStream_t)stream);
}

int lk_moe_grouped_gemm_mxfp4s_f8_ex(int mode, int order, int rows, int k, int n, int xrows, int ku, int n_experts,
                                     int fused, const int32_t* tile_info, const int32_t* rowmap, const uint8_t* x8,
                                     const float* s8, const uint8_t* w, const uint8_t* ws, const uint8_t* w2,
                                     const uint8_t* w2s, const float* bias, const float* bias2, int act, float alpha,
                                     float limit, float* y, lk_stream_t stream) {
  if (mode != LK_STORE && mode != LK_SWIGLU && mode != LK_SWIGLU_SORTED) return LK_EINVAL;
  if (order != LK_ORDER_PAIRS && order != LK_ORDER_SPLIT16) return LK_EINVAL;
  if (rows < 0 || rows % 64 || k <= 0 || n <= 0 || xrows <= 0 || ku <= 0 || n_experts <= 0 || n_experts > kMaxExperts)
    return LK_EINVAL;
  if (!act_ok(act)) return LK_EINVAL;
  if (k % 32 || n % 16) return LK_EINVAL;
  if (rows == 0) return LK_OK;
  if (!tile_info || !rowmap || !x8 || !s8 || !w || !ws || !y) return LK_EINVAL;
  const bool gu = mode != LK_STORE;
  const bool two = gu && !fused;
  if (two && (!w2 || !w2s)) return LK_EINVAL;
  if (gu && (!bias) != (!bias2)) return LK_EINVAL;
  if (!aligned(x8, 16) || !aligned(w, 16) || !aligned(y, 16) || (two && !aligned(w2, 16))) return LK_EALIGN;
  const int fuse = gu && fused;
  ExpertEpi epi{bias, gu ? bias2 : nullptr, gu ? act : LK_ACT_SILU, alpha, limit};
  return gemm_mx(mode, order, rows, k, n, x8, s8, w, ws, two ? w2 : nullptr, two ? w2s : nullptr, y,
                 (cudaStream_t)stream, tile_info, rowmap, xrows, ku, n_experts, fuse ? 2 * n : n, fuse ? n : 0, &epi);
}

int lk_moe_grouped_gemm_mxfp4s_f8(int mode, int order, int rows, int k, int n, int xrows, int ku, int n_experts,
                                  int fused, const int32_t* tile_info, const int32_t* rowmap, const uint8_t* x8,
                                  const float* s8, const uint8_t* w, const uint8_t* ws, const uint8_t* w2,
                                  const uint8_t* w2s, float* y, lk_stream_t stream) {
  return lk_moe_grouped_gemm_mxfp4s_f8_ex(mode, order, rows, k, n, xrows, ku, n_experts, fused, tile_info, rowmap, x8,
                                          s8, w, ws, w2, w2s, nullptr, nullptr, LK_ACT_SILU, 0.f, 0.f, y, stream);
}

int lk_moe_route(int tokens, int h, int n_experts, int ku, int gating, int norm, float scale, const float* x,
                 const void* router_w, int w_dtype, const float* bias, int32_t* ids, float* wts, lk_stream_t stream) {
  if (tokens < 0 || n_experts <= 0 || n_experts > 256 || ku <= 0 || ku > 8 || ku > n_experts) return LK_EINVAL;
  if (gating < 1 || gating > 3) return LK_EINVAL;
  if (router_w && (h <= 0 || (w_dtype != LK_F32 && w_dtype != LK_BF16))) return LK_EINVAL;
  if (gating == 1 && bias) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!x || !ids || !wts) return LK_EINVAL;
  return moe_route(tokens, h, n_experts, ku, gating, norm, scale, x, router_w, w_dtype, bias, ids, wts,
                   (cudaStream_t)stream);
}

int lk_moe_bucket(int tokens, int ku, int n_experts, int max_tiles, const int32_t* info, const int32_t* ids,
                  int32_t* tile_info, int32_t* rowmap, int32_t* pos, lk_stream_t stream) {
  if (tokens < 0 || ku <= 0 || n_experts <= 0 || n_experts > 256 || max_tiles <= 0) return LK_EINVAL;
  if (!ids || !tile_info || !rowmap || !pos) return LK_EINVAL;
  // worst case (gen_llm.py:5406-5411): every live expert's last tile partly filled
  int64_t a = int64_t(tokens) * ku;
  if (int64_t(max_tiles) < (a + 63) / 64 + (a < n_experts ? a : n_experts)) return LK_ERANGE;
  return moe_bucket(tokens, ku, n_experts, max_tiles, info, ids, tile_info, rowmap, pos, (cudaStream_t)stream);
}

int lk_moe_combine_sorted(int tokens, int rows, int h, int ku, int accumulate, const float* ys, const int32_t* pos,
                          const float* wts, float* y, lk_stream_t stream) {
  if (tokens < 0 || rows <= 0 || h <= 0 || ku <= 0 || ku > 8) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!ys || !pos || !wts || !y) return LK_EINVAL;
  return moe_combine_sorted(tokens, rows, h, ku, accumulate, ys, pos, wts, y, (cudaStream_t)stream);
}

int lk_moe_combine(int tokens, int h, int ku, int accumulate, const float* ys, const float* wts, float* y,
                   lk_stream_t stream) {
  if (tokens < 0 || h <= 0 || ku <= 0 || ku > 8) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!ys || !wts || !y) return LK_EINVAL;
  return moe_combine(tokens, h, ku, accumulate, ys, wts, y, (cudaStream_t)stream);
}

int lk_moe_combine_gated(int tokens, int h, int ku, const float* ys, const float* wts, const float* sg, float* y,
                         lk_stream_t stream) {
  if (tokens < 0 || h <= 0 || ku <= 0 || ku > 8) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!ys || !wts || !sg || !y) return LK_EINVAL;
  return moe_combine_g(tokens, h, ku, ys, nullptr, wts, sg, y, (cudaStream_t)stream);
}

int lk_moe_combine_sorted_gated(int tokens, int rows, int h, int ku, const float* ys, const int32_t* pos,
                                const float* wts, const float* sg, float* y, lk_stream_t stream) {
  if (tokens < 0 || rows <= 0 || h <= 0 || ku <= 0 || ku > 8) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!ys || !pos || !wts || !sg || !y) return LK_EINVAL;
  return moe_combine_g(tokens, h, ku, ys, pos, wts, sg, y, (cudaStream_t)stream);
}

int lk_moe_wscale(int tokens, int ku, int n_experts, const int32_t* ids, float* wts, const float* scale,
                  lk_stream_t stream) {
  if (tokens < 0 || ku <= 0 || n_experts <= 0) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!ids || !wts || !scale) return LK_EINVAL;
  return moe_wscale(tokens, ku, n_experts, ids, wts, scale, (cudaStream_t)stream);
}

int lk_moe_shared_gate(int tokens, int h, const float* x, const void* w, int w_dtype, float* sg, lk_stream_t stream) {
  if (tokens < 0 || h <= 0 || h % 32) return LK_EINVAL;
  if (w_dtype != LK_F32 && w_dtype != LK_BF16) return LK_EINVAL;
  if (tokens == 0) return LK_OK;
  if (!x || !w || !sg) return LK_EINVAL;
  if (!aligned(x, 16) || !aligned(w, 8)) return LK_EALIGN;
  return moe_shared_gate(tokens, h, x, w, w_dtype, sg, (cudaStream_t)stream);
}

int lk_moe_ffn_decode_q8(int fmt, int tokens, int h, int f, int n_experts, int ku, int gating, int norm, float scale,
                         const float* logits, const float* router_bias, const float* down_scale, const void* x,
                         int x_dtype, const void* w_gate, const void* w_up, const void* w_down, const float* b_gate,
                         const float* b_up, const float* b_down, int act, float alpha, float limit, float* act_buf,
                         int32_t* ids, float* wts, const float* sg, int accumulate, float* y, lk_stream_t stream) {
  if (fmt != LK_Q4_0 && fmt != LK_Q4_K) return (q4_family(fmt) || fmt_qk(fmt) > 0) ? LK_EUNSUPPORTED : LK_EINVAL;
  if (tokens < 0 || h <= 0 || f <= 0 || n_experts <= 0 || ku <= 0 || ku > n_experts) return LK_EINVAL;
  if (gating < 1 || gating > 3 || !act_ok(act) || (gating == 1 && router_bias)) return LK_EINVAL;
  if (x_dtype != LK_F32 && x_dtype != LK_BF16) return LK_EINVAL;
  if (h % 2048 || f % 256) return LK_EUNSUPPORTED;
  if (tokens > 4 || ku > 8 || n_experts > 256 || h > 4096 || f > 4096 || tokens * ku * f > 65536) return LK_ERANGE;
  if (tokens == 0) return LK_OK;
  if (!logits || !x || !w_gate || !w_down || !act_buf || !y) return LK_EINVAL;
  if ((b_gate == nullptr) != (b_up == nullptr) || (ids == nullptr) != (wts == nullptr)) return LK_EINVAL;
  if (!aligned(x, 16) || !aligned(act_buf, 16) || !aligned(w_gate, 16) || !aligned(w_down, 16) ||
      (w_up && !aligned(w_up, 16)))
    return LK_EALIGN;
  MoeFfnQ8 p{tokens, h, f, n_experts, ku, gating, norm ? 1 : 0, scale, logits, router_bias, down_scale, x, x_dtype,
             w_gate, w_up, w_down, b_gate, b_up, b_down, act, alpha, limit, act_buf, ids, wts, sg,
             accumulate ? 1 : 0, y};
  return moe_ffn_decode_q8(fmt, p, (cudaStream_t)stream);
}

int lk_moe_rank_plan(int assignments, int n_local, int world, const int32_t* ids, int32_t* order, int32_t* pos,
                     int32_t* counts, lk_stream_t stream) {
  if (assignments < 0 || assignments > 65536 || n_local <= 0 || world <= 0 || world > 32) return LK_EINVAL;
  if (!counts) return LK_EINVAL;
  if (assignments > 0 && (!ids || !order || !pos)) return LK_EINVAL;
  return moe_rank_plan(assignments, n_local, world, ids, order, pos, counts, (cudaStream_t)stream);
}

int lk_moe_gather_rows(int rows, int h, int ku, int n_local, const int32_t* order, const int32_t* ids, const void* x,
                       int x_dtype, void* out, int32_t* eid, lk_stream_t stream) {
  if (rows < 0 || h <= 0 || ku <= 0 || n_local <= 0) return LK_EINVAL;
  if (x_dtype != LK_F32 && x_dtype != LK_BF16) return LK_EINVAL;
  if ((int64_t(h) * (x_dtype == LK_BF16 ? 2 : 4)) % 16) return LK_EINVAL;
  if (rows == 0) return LK_OK;
  if (!order || !ids || !x || !out) return LK_EINVAL;
  if (!aligned(x, 16) || !aligned(out, 16)) return LK_EALIGN;
  return moe_gather_rows(rows, h, ku, n_local, order, ids, x, x_dtype, out, eid, (cudaStream_t)stream);
}

}  // extern "C"
