"""Host-side mirror of the reference generators' op interface for the quantized-matmul path, on torch CUDA tensors.

Each function launches liblk kernels on the current CUDA stream through the C ABI (include/lk.h). The operand names,
order and meaning follow the reference's kernel launch signatures (paths relative to the loom-skills checkout):

  mv                 g_mv_{fmt}_k{K}...           gen_llm.py:1185-1194   (%n, %tokens, %accumulate, %x, %w[, %w2], %y)
  row_scale_f16      g_row_scale_f16              gen_llm.py:1843-1912   (%rows, %k, %x, %scales, %x16)
  row_scale_f8       g_row_scale_f16_f8_rdna4     gen_mxfp4s.py:887-938  (..., %x16, %x8, %s8, %w16)
  gemm               g_gemm_{fmt}_{mode}          gen_gemm.py:549-556    (%rows, %k, %n, %x, %scales, %w[, %w2], %y)
  gemm_mxfp4s_f8     g_gemm_mxfp4s_*_f8_m256      gen_mxfp4s.py:101      (%rows, %k, %n, %x, %scales, %w, %ws, ..., %y)
  moe_route          g_moe_route[_tr]             gen_moe.py:116-470     (%tokens, %h, %router_w, %bias, %ids, %wts)
  moe_bucket         g_moe_bucket                 gen_moe.py:829-955     (%tokens, %max_tiles, %info, %ids, %tile_info,
                                                                          %rowmap, %pos)
  moe_grouped_gemm   g_moe_ggu_* / g_moe_gdn_*    gen_moe.py:1126-1228   (%rows, %k, %n, %xrows, %tile_info, %rowmap,
                                                                          %x, %scales, %w[, %w2], %y)
  moe_combine_sorted g_moe_combine_sorted         gen_moe.py:1231-1280   (%tokens, %rows, %ys, %pos, %wts, %y)
  moe_expert_mv      g_moe_gu_* / g_moe_dn_*      gen_moe.py:535-727
  moe_combine        g_moe_combine                gen_moe.py:730-762     (+ shared_gated, gen_moe.py:765-777)
  moe_wscale         g_moe_wscale                 gen_moe.py:1010-1045   (%tokens, %ids, %wts, %scale)
  moe_shared_gate    g_moe_shared_gate            gen_moe.py:780-823     (%tokens, %x, %w, %sg)

The MoE expert kernels take the reference's activation choice (act: "silu", "gelu" -- GEGLU --, "swiglu_oai") and
per-expert output biases (gen_moe.py:958-1007, expert_mv bias=True).

Errors raise LkError (the C ABI's negative return codes). There is no CPU fallback: tensors must be on a CUDA device.
"""
import torch

from . import _lib as L

_DT = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}


def _fmt(fmt):
    """A format name, "gate+up" (two formats: the reference's GATE+UP, e.g. "q4_k+q6_k"), or an id."""
    if isinstance(fmt, str):
        g, _, u = fmt.partition("+")
        return L.fmt_pair(L.FMT_IDS[g], L.FMT_IDS[u]) if u else L.FMT_IDS[g]
    return int(fmt)


def _gate_fmt(fmt):
    """The gate's format of a (possibly paired) format: the down projection's default."""
    return fmt.partition("+")[0] if isinstance(fmt, str) else int(fmt) & 0xFFFF


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _act(act):
    return L.ACT_IDS[act] if isinstance(act, str) else int(act)


def _f32c(t):
    return None if t is None else t.contiguous().float()


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise L.LkError("liblk ops take CUDA tensors (there is no CPU path)")


def row_bytes(fmt, k):
    return int(L.load().lk_row_bytes(_fmt(fmt), k))


def device_status(clear=True):
    """Bit 0 set: a kernel's bounded wait gave up since the last clear (its results are invalid)."""
    return int(L.load().lk_device_status(1 if clear else 0))


def dequant(fmt, w, n_values, out_dtype=torch.float32, w_scales=None):
    """Packed blocks -> values (f32 exact, or the GEMM's f16 staging)."""
    _cuda(w, w_scales)
    out = torch.empty(n_values, dtype=out_dtype, device=w.device)
    L.check(L.load().lk_dequant(_fmt(fmt), _ptr(w), _ptr(w_scales), n_values, _ptr(out), _DT[out_dtype], _stream()),
            "lk_dequant")
    return out


def row_scale_f16(x):
    """x [rows][k] (f32 or bf16) -> (x16 [rows][k] f16, scales [rows][2] f32)."""
    _cuda(x)
    x = x.contiguous()
    rows, k = x.shape
    x16 = torch.empty(rows, k, dtype=torch.float16, device=x.device)
    sc = torch.empty(rows, 2, dtype=torch.float32, device=x.device)
    L.check(L.load().lk_row_scale_f16(rows, k, _ptr(x), _DT[x.dtype], _ptr(sc), _ptr(x16), _stream()),
            "lk_row_scale_f16")
    return x16, sc


def row_scale_f8(x, with_f16=False):
    """x [rows][k] -> (x8 e4m3 bytes [rows][k] uint8, s8 [rows][2]) (+ (x16, scales) when with_f16)."""
    _cuda(x)
    x = x.contiguous()
    rows, k = x.shape
    x8 = torch.empty(rows, k, dtype=torch.uint8, device=x.device)
    s8 = torch.empty(rows, 2, dtype=torch.float32, device=x.device)
    x16 = torch.empty(rows, k, dtype=torch.float16, device=x.device) if with_f16 else None
    sc = torch.empty(rows, 2, dtype=torch.float32, device=x.device) if with_f16 else None
    L.check(L.load().lk_row_scale_f8(rows, k, _ptr(x), _DT[x.dtype], _ptr(sc), _ptr(x16), _ptr(x8), _ptr(s8),
                                     _stream()), "lk_row_scale_f8")
    return (x8, s8, x16, sc) if with_f16 else (x8, s8)


def moe_row_scale_gather(x, rowmap, ku, f8=False):
    """The MoE gate/up activations in bucket order: row r = the row scale of x[rowmap[r] // ku] (zero row where
    rowmap[r] < 0). f8=False: (x16 [rows][k] f16, scales [rows][2]); f8=True: (x8 [rows][k] e4m3 bytes, s8 [rows][2])
    -- the operands of the grouped GEMMs' 'swiglu_sorted' mode."""
    _cuda(x, rowmap)
    x = x.contiguous()
    rows = rowmap.shape[0]
    k = x.shape[1]
    dev = x.device
    if f8:
        x8 = torch.empty(rows, k, dtype=torch.uint8, device=dev)
        s8 = torch.empty(rows, 2, dtype=torch.float32, device=dev)
        L.check(L.load().lk_moe_row_scale_gather(rows, k, ku, _ptr(rowmap), _ptr(x), _DT[x.dtype], None, None,
                                                 _ptr(x8), _ptr(s8), _stream()), "lk_moe_row_scale_gather")
        return x8, s8
    x16 = torch.empty(rows, k, dtype=torch.float16, device=dev)
    sc = torch.empty(rows, 2, dtype=torch.float32, device=dev)
    L.check(L.load().lk_moe_row_scale_gather(rows, k, ku, _ptr(rowmap), _ptr(x), _DT[x.dtype], _ptr(sc), _ptr(x16),
                                             None, None, _stream()), "lk_moe_row_scale_gather")
    return x16, sc


def mv(fmt, w, x, n, k, w2=None, y=None, accumulate=False):
    """Decode matvec: y[t][n] (+)= x[t] . W[n] (swiglu with w2). x [tokens][k] f32/f16/bf16."""
    _cuda(w, x, w2, y)
    x = x.contiguous()
    tokens = x.shape[0]
    if y is None:
        y = torch.empty(tokens, n, dtype=torch.float32, device=x.device)
    L.check(L.load().lk_mv(_fmt(fmt), n, k, tokens, 1 if accumulate else 0, _ptr(x), _DT[x.dtype], _ptr(w), _ptr(w2),
                           _ptr(y), _stream()), "lk_mv")
    return y


def silu_mul(f, u, act="silu"):
    """g_silu_mul: f = act(f) * u in place over [tokens][n] f32 (act "silu" or "gelu"); returns f."""
    _cuda(f, u)
    tokens, n = f.shape
    L.check(L.load().lk_silu_mul(tokens, n, _ptr(f), _ptr(u.contiguous()), _act(act), _stream()), "lk_silu_mul")
    return f


def gemm(fmt, mode, x16, scales, w, n, w2=None, y=None):
    """Prefill GEMM: y[rows][n] (+)= (x16 . W16^T) * scales[row][1]; mode 'store' | 'acc' | 'swiglu'."""
    _cuda(x16, scales, w, w2, y)
    rows, k = x16.shape
    if y is None:
        y = torch.empty(rows, n, dtype=torch.float32, device=x16.device)
    m = L.MODE_IDS[mode] if isinstance(mode, str) else int(mode)
    L.check(L.load().lk_gemm(_fmt(fmt), m, rows, k, n, _ptr(x16), _ptr(scales), _ptr(w), _ptr(w2), _ptr(y),
                             _stream()), "lk_gemm")
    return y


def gemm_mxfp4s_f8(mode, x8, s8, w, ws, n, w2=None, w2s=None, order=L.ORDER_PAIRS, y=None):
    """MXFP4 split planes x e4m3: y = (x8 . (W * 2^8)^T) * s8[row][1]."""
    _cuda(x8, s8, w, ws, w2, w2s, y)
    rows, k = x8.shape
    if y is None:
        y = torch.empty(rows, n, dtype=torch.float32, device=x8.device)
    m = L.MODE_IDS[mode] if isinstance(mode, str) else int(mode)
    L.check(L.load().lk_gemm_mxfp4s_f8(m, order, rows, k, n, _ptr(x8), _ptr(s8), _ptr(w), _ptr(ws), _ptr(w2),
                                       _ptr(w2s), _ptr(y), _stream()), "lk_gemm_mxfp4s_f8")
    return y


def moe_route(x, n_experts, ku, router_w=None, gating=1, norm=True, scale=1.0, bias=None):
    """Router top-k. router_w None: x is the logits [tokens][n_experts] (f32)."""
    _cuda(x, router_w, bias)
    x = x.contiguous().float()
    tokens = x.shape[0]
    ids = torch.empty(tokens, ku, dtype=torch.int32, device=x.device)
    wts = torch.empty(tokens, ku, dtype=torch.float32, device=x.device)
    h = x.shape[1] if router_w is not None else 0
    wdt = _DT[router_w.dtype] if router_w is not None else L.F32
    L.check(L.load().lk_moe_route(tokens, h, n_experts, ku, gating, 1 if norm else 0, scale, _ptr(x), _ptr(router_w),
                                  wdt, _ptr(bias), _ptr(ids), _ptr(wts), _stream()), "lk_moe_route")
    return ids, wts


def moe_gate_up_routed(fmt, x, logits, w, n, n_experts, ku, fused=True, w2=None, gating=1, norm=True, scale=1.0,
                       router_bias=None, act="silu", bias=None, bias2=None, alpha=1.702, limit=7.0):
    """The router and the gate/up expert matvecs of one decode token in one launch (lk_moe_gate_up_routed): returns
    (ids [1][ku], wts [1][ku], act [ku][n]) -- the routing bit for bit moe_route's, act as moe_expert_mv 'gu' gives."""
    _cuda(x, logits, w, w2, router_bias, bias, bias2)
    x = x.contiguous()
    h = x.shape[1]
    ids = torch.empty(1, ku, dtype=torch.int32, device=x.device)
    wts = torch.empty(1, ku, dtype=torch.float32, device=x.device)
    y = torch.empty(ku, n, dtype=torch.float32, device=x.device)
    L.check(L.load().lk_moe_gate_up_routed(_fmt(fmt), h, n, n_experts, ku, gating, 1 if norm else 0, scale,
                                           _ptr(logits.contiguous().float()), _ptr(_f32c(router_bias)), _ptr(x),
                                           _DT[x.dtype], _ptr(w), _ptr(w2), 1 if fused else 0, _ptr(_f32c(bias)),
                                           _ptr(_f32c(bias2)), _act(act), alpha, limit, _ptr(ids), _ptr(wts), _ptr(y),
                                           _stream()), "lk_moe_gate_up_routed")
    return ids, wts, y


def moe_max_tiles(tokens, ku, n_experts):
    """Worst-case schedule size (gen_llm.py:5406-5411)."""
    a = tokens * ku
    return (a + 63) // 64 + min(n_experts, a)


def moe_bucket(ids, n_experts, max_tiles=None, info=None):
    """-> (tile_info [max_tiles][2], rowmap [max_tiles*64], pos [tokens*ku]) int32."""
    _cuda(ids, info)
    tokens, ku = ids.shape
    if max_tiles is None:
        max_tiles = moe_max_tiles(tokens, ku, n_experts)
    dev = ids.device
    ti = torch.empty(max_tiles, 2, dtype=torch.int32, device=dev)
    rm = torch.empty(max_tiles * 64, dtype=torch.int32, device=dev)
    pos = torch.empty(tokens * ku, dtype=torch.int32, device=dev)
    L.check(L.load().lk_moe_bucket(tokens, ku, n_experts, max_tiles, _ptr(info), _ptr(ids.contiguous()), _ptr(ti),
                                   _ptr(rm), _ptr(pos), _stream()), "lk_moe_bucket")
    return ti, rm, pos


def moe_grouped_gemm(fmt, mode, tile_info, rowmap, x16, scales, w, n, ku, n_experts, fused=False, w2=None, y=None,
                     act="silu", bias=None, bias2=None, alpha=1.702, limit=7.0):
    """Grouped expert GEMM over the bucketed 64-row tiles. mode 'swiglu' (gate/up, x16 = token rows, gathered),
    'swiglu_sorted' (gate/up, x16 = sorted rows from moe_row_scale_gather) or 'store' (down, x16 = sorted rows).
    act / bias (gate, or down) / bias2 (up): the expert activation and per-expert biases [n_experts][n].
    y: [max_tiles*64][n]; every row of a live 64-row tile is written, no row of a dead tile."""
    _cuda(tile_info, rowmap, x16, scales, w, w2, y, bias, bias2)
    rows = rowmap.shape[0]
    xrows, k = x16.shape
    if y is None:
        y = torch.empty(rows, n, dtype=torch.float32, device=x16.device)
    m = L.MODE_IDS[mode] if isinstance(mode, str) else int(mode)
    bias, bias2 = _f32c(bias), _f32c(bias2)
    L.check(L.load().lk_moe_grouped_gemm_ex(_fmt(fmt), m, rows, k, n, xrows, ku, n_experts, 1 if fused else 0,
                                            _ptr(tile_info), _ptr(rowmap), _ptr(x16), _ptr(scales), _ptr(w), _ptr(w2),
                                            _ptr(bias), _ptr(bias2), _act(act), alpha, limit, _ptr(y), _stream()),
            "lk_moe_grouped_gemm_ex")
    return y


def moe_grouped_gemm_mxfp4s_f8(mode, tile_info, rowmap, x8, s8, w, ws, n, ku, n_experts, fused=False, w2=None,
                               w2s=None, order=L.ORDER_PAIRS, y=None, act="silu", bias=None, bias2=None, alpha=1.702,
                               limit=7.0):
    """MXFP4 x e4m3 grouped expert GEMM over the bucketed 64-row tiles; operands as gemm_mxfp4s_f8, rows, tiles,
    activation and biases as moe_grouped_gemm (gate/up: x8/s8 are token rows; down: sorted rows)."""
    _cuda(tile_info, rowmap, x8, s8, w, ws, w2, w2s, y, bias, bias2)
    rows = rowmap.shape[0]
    xrows, k = x8.shape
    if y is None:
        y = torch.empty(rows, n, dtype=torch.float32, device=x8.device)
    m = L.MODE_IDS[mode] if isinstance(mode, str) else int(mode)
    bias, bias2 = _f32c(bias), _f32c(bias2)
    L.check(L.load().lk_moe_grouped_gemm_mxfp4s_f8_ex(m, order, rows, k, n, xrows, ku, n_experts, 1 if fused else 0,
                                                      _ptr(tile_info), _ptr(rowmap), _ptr(x8), _ptr(s8), _ptr(w),
                                                      _ptr(ws), _ptr(w2), _ptr(w2s), _ptr(bias), _ptr(bias2),
                                                      _act(act), alpha, limit, _ptr(y), _stream()),
            "lk_moe_grouped_gemm_mxfp4s_f8_ex")
    return y


def moe_combine_sorted(ys, pos, wts, y=None, accumulate=False, sg=None):
    """y[t] (+)= sum_k wts[t,k] ys[pos[t,k]]; sg (shared_gated): y[t] = sg[t] y[t] + ... (y holds the shared output)."""
    _cuda(ys, pos, wts, y, sg)
    tokens, ku = wts.shape
    rows, h = ys.shape
    if sg is not None:
        L.check(L.load().lk_moe_combine_sorted_gated(tokens, rows, h, ku, _ptr(ys), _ptr(pos), _ptr(wts),
                                                     _ptr(sg.contiguous().float()), _ptr(y), _stream()),
                "lk_moe_combine_sorted_gated")
        return y
    if y is None:
        y = torch.empty(tokens, h, dtype=torch.float32, device=ys.device)
    L.check(L.load().lk_moe_combine_sorted(tokens, rows, h, ku, 1 if accumulate else 0, _ptr(ys), _ptr(pos),
                                           _ptr(wts), _ptr(y), _stream()), "lk_moe_combine_sorted")
    return y


def moe_expert_mv_q8(fmt, mode, ids, xq, w, n, k, ku, n_experts, fused=True, w2=None, y=None, act="silu", alpha=1.702,
                     limit=7.0):
    """Decode expert matvecs on int8 activations (MOE_Q8): xq = quant_q8 of the tokens' rows (mode 'gu') or of one
    row per assignment ('dn'); 'gu' -> act(Wg x, Wu x), 'dn' -> Wd x."""
    _cuda(ids, xq, w, w2, y)
    a = ids.numel()
    if y is None:
        y = torch.empty(a, n, dtype=torch.float32, device=xq.device)
    md = 0 if mode == "gu" else 1
    L.check(L.load().lk_moe_expert_mv_q8(_fmt(fmt), md, n, k, a, ku, n_experts, 1 if fused else 0,
                                         _ptr(ids.contiguous()), _ptr(xq), _ptr(w), _ptr(w2), _act(act), alpha, limit,
                                         _ptr(y), _stream()), "lk_moe_expert_mv_q8")
    return y


def moe_expert_mv(fmt, mode, ids, x, w, n, k, ku, n_experts, fused=True, w2=None, y=None, act="silu", bias=None,
                  bias2=None, alpha=1.702, limit=7.0):
    """Decode expert matvecs per assignment: mode 'gu' -> act(Wg x + bg, Wu x + bu); 'dn' -> Wd x (+ bd)."""
    _cuda(ids, x, w, w2, y, bias, bias2)
    a = ids.numel()
    if y is None:
        y = torch.empty(a, n, dtype=torch.float32, device=x.device)
    md = 0 if mode == "gu" else 1
    bias, bias2 = _f32c(bias), _f32c(bias2)
    L.check(L.load().lk_moe_expert_mv_ex(_fmt(fmt), md, n, k, a, ku, n_experts, 1 if fused else 0, _ptr(ids),
                                         _ptr(x.contiguous()), _DT[x.dtype], _ptr(w), _ptr(w2), _ptr(bias),
                                         _ptr(bias2), _act(act), alpha, limit, _ptr(y), _stream()),
            "lk_moe_expert_mv_ex")
    return y


def moe_expert_mv_mxfp4s(mode, ids, x, w, ws, n, k, ku, n_experts, order=L.ORDER_PAIRS, y=None, act="silu",
                         bias=None, bias2=None, alpha=1.702, limit=7.0):
    """Decode expert matvecs over MXFP4S experts per assignment: mode 'gu' (per expert n gate rows then n up rows)
    -> act(Wg x + bg, Wu x + bu); 'dn' -> Wd x (+ bd). w / ws: the stacked nibble and E8M0 planes."""
    _cuda(ids, x, w, ws, y, bias, bias2)
    a = ids.numel()
    if y is None:
        y = torch.empty(a, n, dtype=torch.float32, device=x.device)
    md = 0 if mode == "gu" else 1
    bias, bias2 = _f32c(bias), _f32c(bias2)
    L.check(L.load().lk_moe_expert_mv_mxfp4s_ex(md, int(order), n, k, a, ku, n_experts, _ptr(ids),
                                                _ptr(x.contiguous()), _DT[x.dtype], _ptr(w), _ptr(ws), _ptr(bias),
                                                _ptr(bias2), _act(act), alpha, limit, _ptr(y), _stream()),
            "lk_moe_expert_mv_mxfp4s_ex")
    return y


def moe_combine(ys, wts, y=None, accumulate=False, sg=None):
    """y[t] (+)= sum_k wts[t,k] ys[t*ku + k]; sg (shared_gated): y[t] = sg[t] y[t] + ... (y holds the shared output)."""
    _cuda(ys, wts, y, sg)
    tokens, ku = wts.shape
    h = ys.shape[1]
    if sg is not None:
        L.check(L.load().lk_moe_combine_gated(tokens, h, ku, _ptr(ys), _ptr(wts), _ptr(sg.contiguous().float()),
                                              _ptr(y), _stream()), "lk_moe_combine_gated")
        return y
    if y is None:
        y = torch.empty(tokens, h, dtype=torch.float32, device=ys.device)
    L.check(L.load().lk_moe_combine(tokens, h, ku, 1 if accumulate else 0, _ptr(ys), _ptr(wts), _ptr(y), _stream()),
            "lk_moe_combine")
    return y


def moe_wscale(ids, wts, scale):
    """g_moe_wscale: wts[t,k] *= scale[ids[t,k]] in place (a per-expert down scale folded into the combine weights)."""
    _cuda(ids, wts, scale)
    tokens, ku = wts.shape
    L.check(L.load().lk_moe_wscale(tokens, ku, scale.numel(), _ptr(ids), _ptr(wts), _ptr(scale.contiguous().float()),
                                   _stream()), "lk_moe_wscale")
    return wts


def moe_shared_gate(x, w):
    """g_moe_shared_gate: sg[t] = sigmoid(x[t] . w) (x f32 [tokens][h], w f32/bf16 [h])."""
    _cuda(x, w)
    x = x.contiguous().float()
    tokens, h = x.shape
    sg = torch.empty(tokens, dtype=torch.float32, device=x.device)
    L.check(L.load().lk_moe_shared_gate(tokens, h, _ptr(x), _ptr(w.contiguous()), _DT[w.dtype], _ptr(sg), _stream()),
            "lk_moe_shared_gate")
    return sg


def _route_and_gates(x, logits, n_experts, ku, norm, gating, router_bias, scale, down_scale, shared_gate_w):
    ids, wts = moe_route(logits, n_experts, ku, gating=gating, norm=norm, scale=scale, bias=router_bias)
    if down_scale is not None:
        moe_wscale(ids, wts, down_scale)
    sg = moe_shared_gate(x.float(), shared_gate_w) if shared_gate_w is not None else None
    return ids, wts, sg


def _combine_out(tokens, h, x, y_shared):
    """The combine's target: the shared experts' output (accumulated into, in place) or a new output."""
    if y_shared is not None:
        _cuda(y_shared)
        return y_shared, True
    return torch.empty(tokens, h, dtype=torch.float32, device=x.device), False


def _grouped_decode(fmt, fmt_down, x_dtype, h, f, n_experts):
    """Whether the expert-grouped matvecs (lk_mv.cu k_mv_grp: up to 1024 assignments, grouped by expert inside the
    launch) take both the gate/up and the down expert matvecs of a decode MoE layer: the tuned Q4 formats, at most 256
    experts, and the staged activation rows within the kernel's shared memory (gate/up: h values of x; down: f of the
    f32 activations)."""
    q4 = ("q4_0", "q4_k", "iq4_nl")
    if str(fmt) not in q4 or (fmt_down is not None and str(fmt_down) not in q4) or n_experts > 256:
        return False
    return h % 256 == 0 and f % 256 == 0 and h <= (2816 if x_dtype == torch.float32 else 5632) and f <= 3840


def moe_ffn(fmt, x, logits, w_gu, w_dn, h, f, n_experts, ku, norm=True, prefill=None, gating=1, router_bias=None,
            scale=1.0, act="silu", b_gate=None, b_up=None, b_down=None, down_scale=None, y_shared=None,
            shared_gate_w=None, alpha=1.702, limit=7.0, w_up=None, fmt_down=None, act_q8=False):
    """The routed expert FFN of one MoE layer (wiring of gen_llm.py:5324-5386): route (gating 1/2/3, router bias,
    expert_weights_scale) -> per-expert down scale folded into the weights (g_moe_wscale) -> bucket -> grouped gate/up
    (act + biases) -> row scale -> grouped down (+ bias) -> weighted combine (prefill), or per-assignment expert
    matvecs (decode). The combine adds into y_shared (the shared experts' output) when given -- scaled first by the
    shared-expert gate sigmoid(x . shared_gate_w) when that is given -- else into a new tensor.
    x [tokens][h] (bf16 / f32), logits [tokens][n_experts]; w_gu: per expert 2f rows (gate then up) of h values --
    or, with w_up given (GGUF's separate ffn_gate_exps / ffn_up_exps), per expert f gate rows, and w_up its f up rows;
    w_dn: per expert h rows of f values, in fmt_down when it differs from fmt (GGUF quants often keep ffn_down_exps in
    a wider format); fmt "gate+up" (e.g. "q4_k+q6_k", with w_up): gate and up experts in two formats, the down in
    fmt_down or the gate's; biases [n_experts][f] (gate, up) / [n_experts][h] (down). The reference
    switches to the GEMMs at 64 tokens (gen_llm.py:6107). Here the switch is at 192 assignments (tokens * ku), or at
    1024 where the expert-grouped matvecs take both projections (Q4_0 / Q4_K / IQ4_NL experts, see _grouped_decode):
    on configs[2] shapes (top-8 of 128 experts, bf16 x) those measured 143 / 191 / 224 / 314 us at 16 / 32 / 64 / 128
    tokens against 291 / 351 / 394 / 396 us for the GEMMs. `prefill` forces either path. act_q8 (decode only; the reference's MOE_Q8 numerics, gen_llm.py:5290-5302):
    x and the activations quantised to int8 codes (quant_q8) for the expert matvecs -- formats with integer codes,
    one format for gate and up, no biases."""
    tokens = x.shape[0]
    ep = dict(act=act, alpha=alpha, limit=limit)
    if prefill is None:
        grouped = not act_q8 and _grouped_decode(fmt, fmt_down, x.dtype, h, f, n_experts)
        prefill = tokens * ku > (1024 if grouped else 191)
    fused = w_up is None
    aligned = all(t is None or t.data_ptr() % 16 == 0 for t in (x, w_gu, w_up))
    if (not prefill and not act_q8 and tokens == 1 and fmt in ("q4_0", "q4_k", "iq4_nl") and h % 256 == 0
            and n_experts <= 256 and ku <= 8 and aligned and x.is_contiguous()):
        # one decode token: the router folded into the gate/up launch
        ids, wts, act_ = moe_gate_up_routed(fmt, x, logits, w_gu, f, n_experts, ku, fused=fused, w2=w_up,
                                            gating=gating, norm=norm, scale=scale, router_bias=router_bias,
                                            bias=b_gate, bias2=b_up, **ep)
        if down_scale is not None:
            moe_wscale(ids, wts, down_scale)
        sg = moe_shared_gate(x.float(), shared_gate_w) if shared_gate_w is not None else None
        y, acc = _combine_out(tokens, h, x, y_shared)
        ys = moe_expert_mv(fmt_down or _gate_fmt(fmt), "dn", ids.reshape(-1), act_, w_dn, h, f, ku, n_experts,
                           bias=b_down)
        return moe_combine(ys, wts, y=y, accumulate=acc, sg=sg)
    ids, wts, sg = _route_and_gates(x, logits, n_experts, ku, norm, gating, router_bias, scale, down_scale,
                                    shared_gate_w)
    y, acc = _combine_out(tokens, h, x, y_shared)
    if not prefill and act_q8:
        if b_gate is not None or b_up is not None or b_down is not None or "+" in str(fmt):
            raise L.LkError("the int8 expert matvecs take one gate/up format and no biases (gen_llm.py:5300-5302)")
        fi = ids.reshape(-1)
        act_ = moe_expert_mv_q8(fmt, "gu", fi, quant_q8(x), w_gu, f, h, ku, n_experts, fused=fused, w2=w_up, **ep)
        ys = moe_expert_mv_q8(fmt_down or fmt, "dn", fi, quant_q8(act_), w_dn, h, f, ku, n_experts)
        return moe_combine(ys, wts, y=y, accumulate=acc, sg=sg)
    if not prefill:
        act_ = moe_expert_mv(fmt, "gu", ids.reshape(-1), x, w_gu, f, h, ku, n_experts, fused=fused, w2=w_up,
                             bias=b_gate, bias2=b_up, **ep)
        ys = moe_expert_mv(fmt_down or _gate_fmt(fmt), "dn", ids.reshape(-1), act_, w_dn, h, f, ku, n_experts,
                           bias=b_down)
        return moe_combine(ys, wts, y=y, accumulate=acc, sg=sg)
    ti, rm, pos = moe_bucket(ids, n_experts)
    # the token rows row-scaled straight into bucket order: gate/up then reads plain tiles (no row gather)
    x16, sc = moe_row_scale_gather(x, rm, ku)
    act_ = moe_grouped_gemm(fmt, "swiglu_sorted", ti, rm, x16, sc, w_gu, f, ku, n_experts, fused=fused, w2=w_up,
                            bias=b_gate, bias2=b_up, **ep)
    a16, asc = row_scale_f16(act_)
    ys = moe_grouped_gemm(fmt_down or _gate_fmt(fmt), "store", ti, rm, a16, asc, w_dn, h, ku, n_experts, bias=b_down)
    return moe_combine_sorted(ys, pos, wts, y=y, accumulate=acc, sg=sg)


def moe_ffn_mxfp4s(x, logits, w_gu, ws_gu, w_dn, ws_dn, h, f, n_experts, ku, norm=True, order=L.ORDER_PAIRS,
                   prefill=None, gating=1, router_bias=None, scale=1.0, act="silu", b_gate=None, b_up=None,
                   b_down=None, down_scale=None, y_shared=None, shared_gate_w=None, alpha=1.702, limit=7.0):
    """The routed expert FFN of one MoE layer with MXFP4 experts (gpt-oss-like: gating=3 with the router bias,
    act='swiglu_oai' and the expert biases; gen_llm.py:5324-5386 wiring): the fp8 fusion of gen_mxfp4s.py:969-1110 --
    route -> bucket -> e4m3 row scale -> grouped gate/up (act + biases) -> e4m3 row scale -> grouped down (+ bias) ->
    weighted combine -- or, for at most 16 assignments, per-assignment expert matvecs on the unquantised activations
    (gen_moe.py:535-727). The reference switches at 64 tokens (gen_llm.py:6107); here the matvecs stream each
    assignment's expert on its own, which measured faster only up to about 20 assignments (gpt-oss shapes, matvecs /
    GEMMs: 4 assignments 45 / 83 us, 16: 139 / 165 us, 24: 196 / 170 us). `prefill` forces either path.
    w_gu / ws_gu: per expert 2f rows (gate then up) of h/2 nibble bytes / h/32 E8M0 bytes; w_dn / ws_dn: per
    expert h rows of f/2 / f/32 bytes. Routing options, down scale and shared output as moe_ffn."""
    tokens = x.shape[0]
    ids, wts, sg = _route_and_gates(x, logits, n_experts, ku, norm, gating, router_bias, scale, down_scale,
                                    shared_gate_w)
    y, acc = _combine_out(tokens, h, x, y_shared)
    ep = dict(act=act, alpha=alpha, limit=limit)
    if prefill is None:
        prefill = tokens * ku > 16
    if not prefill:
        act_ = moe_expert_mv_mxfp4s("gu", ids.reshape(-1), x, w_gu, ws_gu, f, h, ku, n_experts, order=order,
                                    bias=b_gate, bias2=b_up, **ep)
        ys = moe_expert_mv_mxfp4s("dn", ids.reshape(-1), act_, w_dn, ws_dn, h, f, ku, n_experts, order=order,
                                  bias=b_down)
        return moe_combine(ys, wts, y=y, accumulate=acc, sg=sg)
    ti, rm, pos = moe_bucket(ids, n_experts)
    x8, s8 = moe_row_scale_gather(x, rm, ku, f8=True)
    act_ = moe_grouped_gemm_mxfp4s_f8("swiglu_sorted", ti, rm, x8, s8, w_gu, ws_gu, f, ku, n_experts, fused=True,
                                      order=order, bias=b_gate, bias2=b_up, **ep)
    a8, as8 = row_scale_f8(act_)
    ys = moe_grouped_gemm_mxfp4s_f8("store", ti, rm, a8, as8, w_dn, ws_dn, h, ku, n_experts, order=order,
                                    bias=b_down)
    return moe_combine_sorted(ys, pos, wts, y=y, accumulate=acc, sg=sg)


def moe_ffn_decode_noalloc(fmt, x, logits, w_gu, w_dn, h, f, n_experts, ku, norm=True, y=None):
    """The decode MoE layer in one C-ABI call whose intermediates live in liblk's fixed device array (no allocation
    inside the call; only the output y is allocated here when not given). For callers that cannot allocate device
    memory. Limits: tokens * ku <= 128, h, f <= 4096; calls that overlap on the GPU race on the shared array."""
    _cuda(x, logits, w_gu, w_dn, y)
    x = x.contiguous()
    logits = logits.contiguous().float()
    tokens = x.shape[0]
    if y is None:
        y = torch.empty(tokens, h, dtype=torch.float32, device=x.device)
    L.check(L.load().lk_moe_ffn_decode_noalloc(_fmt(fmt), tokens, h, f, n_experts, ku, 1 if norm else 0,
                                               _ptr(logits), _ptr(x), _DT[x.dtype], _ptr(w_gu), _ptr(w_dn), _ptr(y),
                                               _stream()), "lk_moe_ffn_decode_noalloc")
    return y


def quant_q8(x, out=None):
    """g_quant_q8: x [rows][k] (f32 / bf16) -> xq uint8 holding int8 codes [rows][k], then the group meta
    [rows][k/32][2] f32 (f16-rounded d, sum of codes) -- the reference's single-buffer layout."""
    _cuda(x, out)
    x = x.contiguous()
    rows, k = x.shape
    xq = out if out is not None else torch.empty(rows * k + rows * (k // 32) * 8, dtype=torch.uint8, device=x.device)
    L.check(L.load().lk_quant_q8(rows, k, _ptr(x), _DT[x.dtype], _ptr(xq), _stream()), "lk_quant_q8")
    return xq


def q8_views(xq, rows, k):
    """(codes int8 [rows][k], meta f32 [rows][k/32][2]) views of a quant_q8 buffer."""
    codes = xq[:rows * k].view(torch.int8).view(rows, k)
    meta = xq[rows * k:rows * k + rows * (k // 32) * 8].view(torch.float32).view(rows, k // 32, 2)
    return codes, meta


def mv_q8(fmt, w, xq, n, k, tokens, y=None, accumulate=False):
    """Decode matvec on int8 activations (quant_q8's buffer for `tokens` rows): y[t][n] (+)= x_q8[t] . W[n]."""
    _cuda(w, xq, y)
    if y is None:
        y = torch.empty(tokens, n, dtype=torch.float32, device=xq.device)
    L.check(L.load().lk_mv_q8(_fmt(fmt), n, k, tokens, 1 if accumulate else 0, _ptr(xq), _ptr(w), _ptr(y),
                              _stream()), "lk_mv_q8")
    return y


def mv_q8_multi(fmt, ws, xq, ns, k, tokens, ys=None, accumulate=False):
    """mv_q8 over several weights sharing one activation (q | k | v): one launch where possible. Returns the ys."""
    import ctypes
    _cuda(xq, *ws)
    g = len(ws)
    if ys is None:
        ys = [torch.empty(tokens, n, dtype=torch.float32, device=xq.device) for n in ns]
    n_arr = (ctypes.c_int * g)(*ns)
    w_arr = (ctypes.c_void_p * g)(*[w.data_ptr() for w in ws])
    y_arr = (ctypes.c_void_p * g)(*[y.data_ptr() for y in ys])
    L.check(L.load().lk_mv_q8_multi(_fmt(fmt), g, n_arr, w_arr, y_arr, k, tokens, 1 if accumulate else 0, _ptr(xq),
                                    _stream()), "lk_mv_q8_multi")
    return ys


def mv_q8_fused(fmt, w, x, n, k, y=None, accumulate=False):
    """One token's decode matvec on int8 activations, quantised inside the matvec (g_quant_q8 folded into the
    kernel's prologue): the numerics of quant_q8 + mv_q8 in one launch. x [1][k] f32 / bf16."""
    _cuda(w, x, y)
    x = x.contiguous()
    if y is None:
        y = torch.empty(1, n, dtype=torch.float32, device=x.device)
    L.check(L.load().lk_mv_q8_fused(_fmt(fmt), n, k, 1 if accumulate else 0, _ptr(x), _DT[x.dtype], _ptr(w), _ptr(y),
                                    _stream()), "lk_mv_q8_fused")
    return y


def moe_rank_plan(ids, n_local, world):
    """lk_moe_rank_plan: assignments (ids [tokens][ku]) stably sorted by destination rank ids // n_local ->
    (order [A] int32, pos [A] int32, counts [world] int32)."""
    _cuda(ids)
    ids = ids.contiguous()
    a = ids.numel()
    order = torch.empty(a, dtype=torch.int32, device=ids.device)
    pos = torch.empty(a, dtype=torch.int32, device=ids.device)
    counts = torch.empty(world, dtype=torch.int32, device=ids.device)
    L.check(L.load().lk_moe_rank_plan(a, n_local, world, _ptr(ids), _ptr(order), _ptr(pos), _ptr(counts), _stream()),
            "lk_moe_rank_plan")
    return order, pos, counts


def moe_gather_rows(order, ids, x, ku, n_local):
    """lk_moe_gather_rows: (x[order // ku] rows, ids[order] % n_local as int32)."""
    _cuda(order, ids, x)
    x = x.contiguous()
    rows = order.numel()
    out = torch.empty(rows, x.shape[1], dtype=x.dtype, device=x.device)
    eid = torch.empty(rows, dtype=torch.int32, device=x.device)
    L.check(L.load().lk_moe_gather_rows(rows, x.shape[1], ku, n_local, _ptr(order), _ptr(ids.contiguous()), _ptr(x),
                                        _DT[x.dtype], _ptr(out), _ptr(eid), _stream()), "lk_moe_gather_rows")
    return out, eid


def moe_ffn_decode_q8(fmt, x, logits, w_gate, w_down, h, f, n_experts, ku, w_up=None, gating=1, norm=True,
                      scale=1.0, router_bias=None, down_scale=None, act="silu", alpha=1.702, limit=7.0, b_gate=None,
                      b_up=None, b_down=None, y=None, accumulate=False, sg=None, act_buf=None, routing=False):
    """lk_moe_ffn_decode_q8: the decode MoE layer on int8 activations (MOE_Q8=1, the reference's default decode
    numerics) in two launches -- routing from the logits, quantisation of x and the gate/up expert matvecs; then
    quantisation of act, the down expert matvecs and the weighted combine. w_up None: w_gate holds each expert's
    f gate rows then f up rows. Returns y [tokens][h] (and (ids, wts) with routing=True)."""
    _cuda(x, logits, w_gate, w_down)
    x = x.contiguous()
    tokens = x.shape[0]
    dev = x.device
    if y is None:
        if accumulate:
            raise ValueError("accumulate needs y")
        y = torch.empty(tokens, h, dtype=torch.float32, device=dev)
    if act_buf is None:
        act_buf = torch.empty(tokens * ku, f, dtype=torch.float32, device=dev)
    ids = wts = None
    if routing:
        ids = torch.empty(tokens, ku, dtype=torch.int32, device=dev)
        wts = torch.empty(tokens, ku, dtype=torch.float32, device=dev)
    lg = _f32c(logits)
    rb, ds = _f32c(router_bias), _f32c(down_scale)
    bg, bu, bd, sgc = _f32c(b_gate), _f32c(b_up), _f32c(b_down), _f32c(sg)
    L.check(L.load().lk_moe_ffn_decode_q8(
        _fmt(fmt), tokens, h, f, n_experts, ku, gating, 1 if norm else 0, float(scale), _ptr(lg), _ptr(rb), _ptr(ds),
        _ptr(x), _DT[x.dtype], _ptr(w_gate), _ptr(w_up), _ptr(w_down), _ptr(bg), _ptr(bu), _ptr(bd), _act(act),
        float(alpha), float(limit), _ptr(act_buf), _ptr(ids), _ptr(wts), _ptr(sgc), 1 if accumulate else 0, _ptr(y),
        _stream()), "lk_moe_ffn_decode_q8")
    return (y, ids, wts) if routing else y


def mv_q8_fused_multi(fmt, ws, x, ns, k, ys=None, accumulate=False):
    """mv_q8_fused over up to 4 weights sharing x (q | k | v) in one launch. Returns the ys."""
    import ctypes
    _cuda(x, *ws)
    x = x.contiguous()
    g = len(ws)
    if ys is None:
        ys = [torch.empty(1, n, dtype=torch.float32, device=x.device) for n in ns]
    n_arr = (ctypes.c_int * g)(*ns)
    w_arr = (ctypes.c_void_p * g)(*[w.data_ptr() for w in ws])
    y_arr = (ctypes.c_void_p * g)(*[y.data_ptr() for y in ys])
    L.check(L.load().lk_mv_q8_fused_multi(_fmt(fmt), g, n_arr, w_arr, y_arr, k, 1 if accumulate else 0, _ptr(x),
                                          _DT[x.dtype], _stream()), "lk_mv_q8_fused_multi")
    return ys
