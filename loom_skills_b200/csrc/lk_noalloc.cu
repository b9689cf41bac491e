// The decode MoE layer without any allocation: the router, the fused gate/up expert matvecs with SwiGLU, the down
// expert matvecs and the weighted combine -- the same kernels, in the same order, as the caller-allocated decode path
// (lk_moe_route -> lk_moe_expert_mv x2 -> lk_moe_combine) -- with the layer's intermediates (routing ids and weights,
// per-assignment activations, per-assignment expert outputs) in one fixed array of device memory inside liblk.
//
// For callers that cannot allocate device memory: code that runs where cudaMalloc is not allowed or not wanted (an
// embedding runtime with a fixed device-memory budget, a host callback, a process whose allocator is owned by
// someone else) and so cannot provide the four scratch buffers the other entry points take.
#include <mutex>

#include "lk_common.cuh"
#include "lk_internal.h"

namespace lk {
namespace {

// Limits of the array: assignments (tokens * top-k) and the hidden / intermediate widths
constexpr int kNaMaxAssign = 128;
constexpr int kNaMaxDim = 4096;
constexpr size_t kNaActBytes = size_t(kNaMaxAssign) * kNaMaxDim * sizeof(float);   // [assignments][f]
constexpr size_t kNaYsBytes = size_t(kNaMaxAssign) * kNaMaxDim * sizeof(float);    // [assignments][h]
constexpr size_t kNaIdsBytes = size_t(kNaMaxAssign) * sizeof(int32_t);
constexpr size_t kNaWtsBytes = size_t(kNaMaxAssign) * sizeof(float);
constexpr size_t kNaBytes = kNaActBytes + kNaYsBytes + kNaIdsBytes + kNaWtsBytes;   // 4 MiB + 1 KiB

// Every call on a device shares this array. Nothing in it needs to start at zero: the router writes every id and
// weight, the matvecs store (not accumulate) every activation and expert output before the combine reads them.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNaBytes];

// The driver's current context, through the runtime's driver entry point (liblk links only the runtime)
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
CUcontext current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext c = nullptr;
  if (fn) fn(&c);
  return c;
}

// Address of the array on the current device, looked up once per device (cudaGetSymbolAddress, with that device
// current) and again whenever the device's context is no longer the one it was looked up in (after a
// cudaDeviceReset the runtime makes a new primary context, where the array has a new address). The first call on a
// device, and the first after a reset, must come before any stream capture.
int scratch_on_current_device(unsigned char** out) {
  static std::mutex mu;
  static unsigned char* ptrs[64] = {};
  static CUcontext ctxs[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LK_ECUDA;
  const CUcontext ctx = current_context();   // null before the runtime has made the device's context current
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev] || !ctx || ctxs[dev] != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return LK_ECUDA;
    ptrs[dev] = static_cast<unsigned char*>(p);
    ctxs[dev] = current_context();   // the context the lookup ran in (made current by it if none was)
  }
  *out = ptrs[dev];
  return LK_OK;
}

}  // namespace
}  // namespace lk

using namespace lk;

extern "C" int lk_moe_ffn_decode_noalloc(int fmt, int tokens, int h, int f, int n_experts, int ku, int norm,
                                         const float* logits, const void* x, int x_dtype, const void* w_gu,
                                         const void* w_dn, float* y, lk_stream_t stream) {
  if (fmt != LK_Q4_0 && fmt != LK_Q4_K && fmt != LK_IQ4_NL) return LK_EUNSUPPORTED;
  if (tokens < 0 || h <= 0 || f <= 0 || n_experts <= 0 || n_experts > kMaxExperts || ku <= 0 || ku > 8 ||
      ku > n_experts)
    return LK_EINVAL;
  if (h % 256 || f % 256) return LK_EINVAL;
  if (x_dtype != LK_F32 && x_dtype != LK_F16 && x_dtype != LK_BF16) return LK_EINVAL;
  if (int64_t(tokens) * ku > kNaMaxAssign || h > kNaMaxDim || f > kNaMaxDim) return LK_ERANGE;
  if (tokens == 0) return LK_OK;
  if (!logits || !x || !w_gu || !w_dn || !y) return LK_EINVAL;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_gu) | reinterpret_cast<uintptr_t>(w_dn)) & 15)
    return LK_EALIGN;
  unsigned char* base = nullptr;
  int rc = scratch_on_current_device(&base);
  if (rc != LK_OK) return rc;
  float* act = reinterpret_cast<float*>(base);
  float* ys = reinterpret_cast<float*>(base + kNaActBytes);
  int32_t* ids = reinterpret_cast<int32_t*>(base + kNaActBytes + kNaYsBytes);
  float* wts = reinterpret_cast<float*>(base + kNaActBytes + kNaYsBytes + kNaIdsBytes);
  cudaStream_t s = (cudaStream_t)stream;
  const int a = tokens * ku;

  rc = moe_route(tokens, 0, n_experts, ku, 1, norm, 1.0f, logits, nullptr, LK_F32, nullptr, ids, wts, s);
  if (rc != LK_OK) return rc;
  MvArgs gu{};
  gu.w = static_cast<const uint8_t*>(w_gu);
  gu.x = x;
  gu.y = act;
  gu.n = f;
  gu.k = h;
  gu.tokens = a;
  gu.x_dtype = x_dtype;
  gu.row_bytes = lk_row_bytes(fmt, h);
  gu.ids = ids;
  gu.x_div = ku;
  gu.n_experts = n_experts;
  gu.rows_per_expert = 2 * f;   // per expert: f gate rows, then f up rows
  gu.rows_per_expert2 = 2 * f;
  gu.w2_row_offset = f;
  gu.swiglu = 1;
  rc = mv(fmt, gu, a, s);
  if (rc != LK_OK) return rc;
  MvArgs dn{};
  dn.w = static_cast<const uint8_t*>(w_dn);
  dn.x = act;
  dn.y = ys;
  dn.n = h;
  dn.k = f;
  dn.tokens = a;
  dn.x_dtype = LK_F32;
  dn.row_bytes = lk_row_bytes(fmt, f);
  dn.ids = ids;
  dn.x_div = 1;
  dn.n_experts = n_experts;
  dn.rows_per_expert = h;
  dn.rows_per_expert2 = h;
  rc = mv(fmt, dn, a, s);
  if (rc != LK_OK) return rc;
  return moe_combine(tokens, h, ku, 0, ys, wts, y, s);
}
