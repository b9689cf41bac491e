"""GPU parity of the MXFP4 x FP8 GEMMs (dense and grouped over the MoE schedule) through the C ABI.

The kernels read the same e4m3 activations the oracle reads, so against the oracle's float64 product of those values
the only difference is the tensor core's f32 accumulation: relative L2 <= 1e-4 (TOL_SAME). Against the reference's
whole path from the f32 activations (its e4m3 producer, then the product) the north-star bar for fp8 activations
applies: relative L2 <= 2e-2 (TOL_F8). (The e4m3 rounding itself moves N(0,1) rows by about 2.6 % relative L2, so the
unquantised f32 product is not the comparison the reference makes.)
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

TOL_SAME = 1e-4
TOL_F8 = 2e-2


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from loom_skills_b200 import ops as _ops
    return _ops


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def mx_weights(n, k, seed, std=0.02, scale=1.0):
    w = (np.random.default_rng(seed).standard_normal((n, k)) * std * scale).astype(np.float32)
    nib, sc = O.quantize_mxfp4(w, "planar")
    return w, nib, sc


def to_split16(nib):
    """Pairs-order nibble plane -> ggml split16 order (byte i of a block: element i low, element i + 16 high)."""
    nib = np.asarray(nib, np.uint8)
    n = nib.shape[0]
    codes = np.stack([nib & 15, nib >> 4], -1).reshape(n, -1, 32)
    return (codes[..., :16] | (codes[..., 16:] << 4)).reshape(n, -1).astype(np.uint8)


def f8_rows(ops, x):
    x8, s8 = ops.row_scale_f8(dev(x))
    return x8, s8, host(x8), host(s8)


class TestDenseMxfp4:
    @pytest.mark.parametrize("rows,n,k", [(128, 256, 256), (200, 2880, 2880), (1, 512, 576), (300, 272, 1024),
                                          (256, 640, 4096)])
    @pytest.mark.parametrize("order", ["pairs", "split16"])
    def test_store(self, ops, rows, n, k, order):
        wf, nib, sc = mx_weights(n, k, 11)
        x = np.random.default_rng(12).standard_normal((rows, k)).astype(np.float32)
        x8, s8, hx8, hs8 = f8_rows(ops, x)
        wn = to_split16(nib) if order == "split16" else nib
        o = ops.L.ORDER_SPLIT16 if order == "split16" else ops.L.ORDER_PAIRS
        y = host(ops.gemm_mxfp4s_f8("store", x8, s8, dev(wn), dev(sc), n, order=o))
        ref = O.gemm_mxfp4_f8_ref(hx8, hs8, nib, sc, n, k)
        assert O.rel_l2(y, ref) < TOL_SAME, O.rel_l2(y, ref)
        # the whole reference path from the f32 activations (its own e4m3 producer on the CPU)
        rx8, rs8 = O.row_scale_f8(x)
        assert O.rel_l2(y, O.gemm_mxfp4_f8_ref(rx8, rs8, nib, sc, n, k)) < TOL_F8

    @pytest.mark.parametrize("scale_exp", [-60, -25, 30])
    def test_block_exponents_outside_e5m2_window(self, ops, scale_exp):
        """Block exponents far outside 107..132 (where the reference's e5m2 decode stops being exact)."""
        n, k, rows = 256, 512, 64
        _, nib, sc = mx_weights(n, k, 13, scale=2.0 ** scale_exp)
        assert sc.max() < 107 or sc.min() > 132
        x = np.random.default_rng(14).standard_normal((rows, k)).astype(np.float32)
        x8, s8, hx8, hs8 = f8_rows(ops, x)
        y = host(ops.gemm_mxfp4s_f8("store", x8, s8, dev(nib), dev(sc), n))
        ref = O.gemm_mxfp4_f8_ref(hx8, hs8, nib, sc, n, k)
        assert O.rel_l2(y, ref) < TOL_SAME, O.rel_l2(y, ref)

    @pytest.mark.parametrize("rows,n,k", [(128, 256, 512), (130, 2880, 2880)])
    def test_swiglu(self, ops, rows, n, k):
        _, g, gs = mx_weights(n, k, 21)
        _, u, us = mx_weights(n, k, 22)
        x = np.random.default_rng(23).standard_normal((rows, k)).astype(np.float32)
        x8, s8, hx8, hs8 = f8_rows(ops, x)
        y = host(ops.gemm_mxfp4s_f8("swiglu", x8, s8, dev(g), dev(gs), n, w2=dev(u), w2s=dev(us)))
        ref = O.silu(O.gemm_mxfp4_f8_ref(hx8, hs8, g, gs, n, k)) * O.gemm_mxfp4_f8_ref(hx8, hs8, u, us, n, k)
        assert O.rel_l2(y, ref) < TOL_SAME, O.rel_l2(y, ref)

    def test_empty_and_invalid(self, ops):
        x8 = torch.empty(0, 256, dtype=torch.uint8, device="cuda")
        s8 = torch.empty(0, 2, dtype=torch.float32, device="cuda")
        w = torch.zeros(64, 128, dtype=torch.uint8, device="cuda")
        ws = torch.zeros(64, 8, dtype=torch.uint8, device="cuda")
        assert ops.gemm_mxfp4s_f8("store", x8, s8, w, ws, 64).shape == (0, 64)
        x8 = torch.zeros(4, 48, dtype=torch.uint8, device="cuda")   # k % 32 != 0
        with pytest.raises(ops.L.LkError):
            ops.gemm_mxfp4s_f8("store", x8, torch.zeros(4, 2, device="cuda"), w[:, :24], ws[:, :1], 64)
        assert ops.L.load().lk_device_status(1) == 0


class TestGroupedMxfp4:
    @pytest.mark.parametrize("tokens,E,ku,h,f", [(37, 8, 4, 576, 320), (256, 4, 4, 2880, 704), (3, 8, 4, 2880, 320)])
    def test_gate_up_down(self, ops, tokens, E, ku, h, f):
        rng = np.random.default_rng(31)
        _, gu, gus = mx_weights(E * 2 * f, h, 32)          # per expert f gate rows then f up rows
        _, dn, dns = mx_weights(E * h, f, 33)
        x = rng.standard_normal((tokens, h)).astype(np.float32)
        logits = rng.standard_normal((tokens, E)).astype(np.float32)
        ids, wts = ops.moe_route(dev(logits), E, ku)
        ti, rm, pos = ops.moe_bucket(ids, E)
        x8, s8, hx8, hs8 = f8_rows(ops, x)
        act = ops.moe_grouped_gemm_mxfp4s_f8("swiglu", ti, rm, x8, s8, dev(gu), dev(gus), f, ku, E, fused=True)
        hact, hrm, hids = host(act), host(rm), host(ids).reshape(-1)
        live = np.nonzero(hrm >= 0)[0]
        assert live.size == tokens * ku
        a = hrm[live]
        e, t = hids[a], a // ku
        for ex in np.unique(e):
            sel = live[e == ex]
            tt = hrm[sel] // ku
            g = O.gemm_mxfp4_f8_ref(hx8[tt], hs8[tt], gu[ex * 2 * f:ex * 2 * f + f], gus[ex * 2 * f:ex * 2 * f + f], f, h)
            u = O.gemm_mxfp4_f8_ref(hx8[tt], hs8[tt], gu[ex * 2 * f + f:(ex + 1) * 2 * f],
                                    gus[ex * 2 * f + f:(ex + 1) * 2 * f], f, h)
            ref = O.silu(g) * u
            assert O.rel_l2(hact[sel], ref) < TOL_SAME, (ex, O.rel_l2(hact[sel], ref))
        # down: row-scaled sorted activations, rows of skipped tiles are never read by the combine
        act = torch.nan_to_num(act)
        a8, as8 = ops.row_scale_f8(act)
        ys = ops.moe_grouped_gemm_mxfp4s_f8("store", ti, rm, a8, as8, dev(dn), dev(dns), h, ku, E)
        hys, ha8, has8 = host(ys), host(a8), host(as8)
        for ex in np.unique(e):
            sel = live[e == ex]
            ref = O.gemm_mxfp4_f8_ref(ha8[sel], has8[sel], dn[ex * h:(ex + 1) * h], dns[ex * h:(ex + 1) * h], h, f)
            assert O.rel_l2(hys[sel], ref) < TOL_SAME, (ex, O.rel_l2(hys[sel], ref))
        assert ops.L.load().lk_device_status(1) == 0

    @pytest.mark.parametrize("tokens", [1, 4, 5, 40, 300])
    def test_moe_ffn_end_to_end(self, ops, tokens):
        E, ku, h, f = 8, 4, 576, 320
        rng = np.random.default_rng(41)
        _, gu, gus = mx_weights(E * 2 * f, h, 42)
        _, dn, dns = mx_weights(E * h, f, 43)
        x = rng.standard_normal((tokens, h)).astype(np.float32)
        logits = rng.standard_normal((tokens, E)).astype(np.float32)
        y = host(ops.moe_ffn_mxfp4s(dev(x), dev(logits), dev(gu), dev(gus), dev(dn), dev(dns), h, f, E, ku))
        ids, wts = O.route_ref(logits, ku)
        if tokens * ku > 16:   # the fp8 GEMM path
            ref = O.moe_ffn_mxfp4_ref(x, ids, wts, gu, gus, dn, dns, h, f)
            assert O.rel_l2(y, ref) < TOL_F8, O.rel_l2(y, ref)
        else:              # expert matvecs on the unquantised activations, f32 accumulation
            ref = O.moe_ffn_mxfp4_decode_ref(x, ids, wts, gu, gus, dn, dns, h, f)
            assert O.rel_l2(y, ref) < 1e-3, O.rel_l2(y, ref)
        assert ops.L.load().lk_device_status(1) == 0

    def test_moe_ffn_prefill_path_at_decode_sizes(self, ops):
        # the fp8 GEMM pipeline stays selectable for a few assignments (prefill=True)
        E, ku, h, f, tokens = 8, 4, 576, 320, 2
        rng = np.random.default_rng(44)
        _, gu, gus = mx_weights(E * 2 * f, h, 45)
        _, dn, dns = mx_weights(E * h, f, 46)
        x = rng.standard_normal((tokens, h)).astype(np.float32)
        logits = rng.standard_normal((tokens, E)).astype(np.float32)
        y = host(ops.moe_ffn_mxfp4s(dev(x), dev(logits), dev(gu), dev(gus), dev(dn), dev(dns), h, f, E, ku,
                                    prefill=True))
        ids, wts = O.route_ref(logits, ku)
        ref = O.moe_ffn_mxfp4_ref(x, ids, wts, gu, gus, dn, dns, h, f)
        assert O.rel_l2(y, ref) < TOL_F8, O.rel_l2(y, ref)


class TestExpertMvMxfp4:
    """Decode expert matvecs over MXFP4S experts (gen_moe.py:535-727 expert_mv with the MXFP4S format): f32
    accumulation of the activations against the exact MXFP4 values, so against the float64 product the bar is the
    f32 one (relative L2 <= 1e-4 here; the path's tolerance is 1e-3)."""

    @pytest.mark.parametrize("k", [2880, 64, 1024, 4096, 2080])
    @pytest.mark.parametrize("order", ["pairs", "split16"])
    @pytest.mark.parametrize("xdt", ["f32", "bf16", "f16"])
    def test_gate_up_and_down(self, ops, k, order, xdt):
        rng = np.random.default_rng(k + (order == "pairs") + 3 * (xdt == "bf16") + 5 * (xdt == "f16"))
        E, ku, tokens, f = 5, 2, 3, 200
        a = tokens * ku
        _, nib, sc = mx_weights(E * 2 * f, k, 81)
        ids = rng.integers(0, E, a).astype(np.int32)
        x = rng.standard_normal((tokens, k)).astype(np.float32)
        xt = dev(x).to({"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[xdt])
        xs = host(xt.float())
        od = ops.L.ORDER_PAIRS if order == "pairs" else ops.L.ORDER_SPLIT16
        nb = nib if order == "pairs" else to_split16(nib)
        act = host(ops.moe_expert_mv_mxfp4s("gu", dev(ids), xt, dev(nb), dev(sc), f, k, ku, E, order=od))
        W = O.dequant_mxfp4_planar(nib, sc, E * 2 * f, k).reshape(E, 2 * f, k)
        ref = np.empty((a, f))
        for i in range(a):
            v = W[ids[i]] @ xs[i // ku].astype(np.float64)
            g, u = v[:f], v[f:]
            ref[i] = g / (1.0 + np.exp(-g)) * u
        assert O.rel_l2(act, ref) < 1e-4, O.rel_l2(act, ref)
        # down: one activation row per assignment against per-expert h x 256 weights
        h, kd = 72, 256
        _, nd, sd = mx_weights(E * h, kd, 83)
        xd = rng.standard_normal((a, kd)).astype(np.float32)
        nbd = nd if order == "pairs" else to_split16(nd)
        y = host(ops.moe_expert_mv_mxfp4s("dn", dev(ids), dev(xd), dev(nbd), dev(sd), h, kd, ku, E, order=od))
        Wd = O.dequant_mxfp4_planar(nd, sd, E * h, kd).reshape(E, h, kd)
        refd = np.stack([Wd[ids[i]] @ xd[i].astype(np.float64) for i in range(a)])
        assert O.rel_l2(y, refd) < 1e-4, O.rel_l2(y, refd)
        assert ops.device_status() == 0

    def test_contract(self, ops):
        ids = torch.zeros(2, dtype=torch.int32, device="cuda")
        x = torch.zeros(1, 4128, device="cuda")
        w = torch.zeros(4, 4128 // 2, dtype=torch.uint8, device="cuda")
        ws = torch.zeros(4, 4128 // 32, dtype=torch.uint8, device="cuda")
        with pytest.raises(ops.L.LkError):   # k > 4096
            ops.moe_expert_mv_mxfp4s("gu", ids, x, w, ws, 2, 4128, 2, 1)
        with pytest.raises(ops.L.LkError):   # k % 32
            ops.moe_expert_mv_mxfp4s("dn", ids, x[:, :48], w, ws, 2, 48, 1, 1)
        assert ops.moe_expert_mv_mxfp4s("dn", ids[:0], x, w, ws, 4, 64, 1, 1).shape == (0, 4)
