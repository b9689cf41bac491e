"""GPU parity of the int8-activation decode path (the reference's default ACT_Q8=1 numerics) through the C ABI:
g_quant_q8 bit-exact against the oracle (codes and group meta), and the dp4a matvec against the float64 product of
the dequantised weights with the same int8 activations (relative L2 <= 1e-3; integer dots are exact, so the
difference is f32 rounding of the per-group scaling, ~1e-7)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

TOL = 1e-3


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


QUANT = {"q4_0": O.quantize_q4_0, "q4_k": O.quantize_q4_k}


def weights(fmt, n, k, seed):
    return QUANT[fmt]((np.random.default_rng(seed).standard_normal((n, k)) * 0.02).astype(np.float32))


class TestQuantQ8:
    @pytest.mark.parametrize("dtype", ["f32", "bf16"])
    def test_bit_exact(self, ops, golden, dtype):
        rng = np.random.default_rng(3)
        x = np.concatenate([golden["q8_in"][:, :512],
                            (rng.standard_normal((7, 512)) * rng.choice([1e-4, 1.0, 5e3], (7, 1)))]).astype(np.float32)
        x[3, 100:132] = 0.0
        xt = dev(x)
        if dtype == "bf16":
            xt = xt.to(torch.bfloat16)
            x = xt.float().cpu().numpy()
        xq = ops.quant_q8(xt)
        codes, meta = ops.q8_views(xq, x.shape[0], x.shape[1])
        rc, rm = O.quant_q8(x)
        assert np.array_equal(host(codes), rc)
        assert np.array_equal(host(meta).view(np.uint32), rm.view(np.uint32))


class TestMvQ8:
    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k"])
    @pytest.mark.parametrize("n,k,tokens", [(256, 256, 1), (4096, 4096, 1), (1000, 2048, 3), (64, 12288, 8),
                                            (300, 1024, 13), (1024, 4096, 1), (130, 8192, 1), (96, 12288, 1),
                                            (4099, 4096, 1), (200, 4096, 40), (129, 2048, 16)])
    def test_vs_oracle(self, ops, fmt, n, k, tokens):
        rng = np.random.default_rng(n + k + tokens)
        w = QUANT[fmt]((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
        x = rng.standard_normal((tokens, k)).astype(np.float32)
        xq = ops.quant_q8(dev(x))
        codes, meta = ops.q8_views(xq, tokens, k)
        y = host(ops.mv_q8(fmt, dev(w), xq, n, k, tokens))
        ref = O.mv_ref(fmt, w, O.dequant_q8(host(codes), host(meta)), n, k)
        assert O.rel_l2(y, ref) < TOL, O.rel_l2(y, ref)
        assert ops.device_status() == 0

    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k"])
    def test_golden_weights_and_accumulate(self, ops, golden, fmt):
        w, x = golden[f"mv_{fmt}_w"], golden[f"mv_{fmt}_x"]
        n, k = w.shape[0], x.shape[1]
        xq = ops.quant_q8(dev(x))
        codes, meta = ops.q8_views(xq, x.shape[0], k)
        xd = O.dequant_q8(host(codes), host(meta))
        y0 = np.random.default_rng(1).standard_normal((x.shape[0], n)).astype(np.float32)
        y = ops.mv_q8(fmt, dev(w), xq, n, k, x.shape[0], y=dev(y0), accumulate=True)
        ref = O.mv_ref(fmt, w, xd, n, k, y_old=y0)
        assert O.rel_l2(host(y), ref) < TOL
        # the q8 activations stay within the reference's own tolerance of the f32 product (make_kernel_tests q8 path)
        assert O.rel_l2(host(ops.mv_q8(fmt, dev(w), xq, n, k, x.shape[0])), golden[f"mv_{fmt}_y"]) < 2e-2

    def test_unsupported_and_empty(self, ops):
        # no integer codes for Q3_K / IQ3_S / MXFP4 (formats.py:22-31)
        xq = torch.zeros(256 + 8 * 8, dtype=torch.uint8, device="cuda")
        w = torch.zeros(4, 144, dtype=torch.uint8, device="cuda")
        for fmt in ("q3_k", "iq3_s", "mxfp4"):
            with pytest.raises(ops.L.LkError):
                ops.mv_q8(fmt, w, xq, 4, 256, 1)
        assert ops.mv_q8("q4_k", w, xq, 4, 256, 0).shape == (0, 4)


SCALE_OFFS = {"q5_0": [0], "q8_0": [0], "q5_k": [0, 2], "q6_k": [208], "iq4_xs": [0], "iq4_nl": [0], "q4_0": [0],
              "q4_k": [0, 2]}
GENERIC = ["q8_0", "q5_0", "q5_k", "q6_k", "iq4_nl", "iq4_xs"]


def blocks(fmt, rows, k, seed, lo=1e-3, hi=2e-2):
    """Random blocks of `fmt` (every code and sub-block scale) with finite f16 scales of both signs."""
    rng = np.random.default_rng(seed)
    nb = rows * k // O.QK[fmt]
    b = rng.integers(0, 256, (nb, O.BLOCK_BYTES[fmt]), dtype=np.uint8)
    for o in SCALE_OFFS[fmt]:
        b[:, o:o + 2] = (rng.uniform(lo, hi, nb) * rng.choice([-1, 1], nb)).astype(np.float16).view(np.uint8).reshape(-1, 2)
    return b.reshape(rows, -1)


class TestMvQ8Generic:
    """k_mvq8g: the reference's other integer-code formats (formats.py:22-31 ICODES, @g_<fmt>_icodes
    gen_llm.py:521-680, 898-1000) on lk_quant_q8 codes: exact integer dots, f32 scaling per format."""

    @pytest.mark.parametrize("fmt", GENERIC)
    @pytest.mark.parametrize("n,k,tokens", [(200, 2048, 1), (4096, 4096, 1), (130, 12288, 1), (300, 4096, 3),
                                            (96, 1024, 9), (1000, 2560, 8)])
    def test_vs_oracle(self, ops, fmt, n, k, tokens):
        rng = np.random.default_rng(n + k + tokens)
        w = blocks(fmt, n, k, n + tokens)
        x = rng.standard_normal((tokens, k)).astype(np.float32)
        xq = ops.quant_q8(dev(x))
        codes, meta = ops.q8_views(xq, tokens, k)
        y = host(ops.mv_q8(fmt, dev(w), xq, n, k, tokens))
        ref = O.mv_ref(fmt, w, O.dequant_q8(host(codes), host(meta)), n, k)
        assert O.rel_l2(y, ref) < 1e-5, O.rel_l2(y, ref)
        assert ops.device_status() == 0

    @pytest.mark.parametrize("fmt", ["q8_0", "q5_0", "iq4_nl"])
    def test_rows_of_32_value_blocks_and_accumulate(self, ops, fmt):
        # k = 704 (22 blocks of 32: the kbench down projection's width) at an odd 2-byte offset of 16 (w + 2 bytes)
        n, k, tokens = 77, 704, 2
        w = blocks(fmt, n, k, 5)
        buf = torch.zeros(w.size + 16, dtype=torch.uint8, device="cuda")
        buf[2:2 + w.size] = dev(w.reshape(-1))
        x = np.random.default_rng(6).standard_normal((tokens, k)).astype(np.float32)
        xq = ops.quant_q8(dev(x))
        codes, meta = ops.q8_views(xq, tokens, k)
        y0 = np.random.default_rng(7).standard_normal((tokens, n)).astype(np.float32)
        y = host(ops.mv_q8(fmt, buf[2:2 + w.size], xq, n, k, tokens, y=dev(y0), accumulate=True))
        ref = O.mv_ref(fmt, w, O.dequant_q8(host(codes), host(meta)), n, k, y_old=y0)
        assert O.rel_l2(y, ref) < 1e-5

    @pytest.mark.parametrize("fmt", ["q8_0", "q5_0", "q5_k", "q6_k"])
    def test_golden_within_the_q8_tolerance(self, ops, fmt):
        # gguf 0.19.0's float64 product of the golden blocks (tests/golden/golden_formats.npz): the int8 activations
        # stay within the reference's q8 tolerance of it
        import os
        with np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_formats.npz")) as z:
            w, x, yref = z[f"mv_{fmt}_w"], z[f"mv_{fmt}_x"], z[f"mv_{fmt}_y"]
        xq = ops.quant_q8(dev(x))
        y = host(ops.mv_q8(fmt, dev(w), xq, w.shape[0], x.shape[1], x.shape[0]))
        assert O.rel_l2(y, yref) < 2e-2

    def test_multi_segments(self, ops):
        k, tokens, ns = 4096, 1, [512, 128, 130]
        ws = [dev(blocks("q6_k", n, k, 30 + i)) for i, n in enumerate(ns)]
        xq = ops.quant_q8(dev(np.random.default_rng(31).standard_normal((tokens, k)).astype(np.float32)))
        ys = ops.mv_q8_multi("q6_k", ws, xq, ns, k, tokens)
        for w, n, y in zip(ws, ns, ys):
            assert torch.equal(y, ops.mv_q8("q6_k", w, xq, n, k, tokens))


class TestMoeExpertMvQ8:
    """lk_moe_expert_mv_q8 (MOE_Q8 for every format with integer codes) through ops.moe_ffn(act_q8=True): routing,
    quant_q8 of x, int8 gate/up with the activation, quant_q8 of the activations, int8 down, combine -- against the
    float64 oracle of the same numerics (moe_ffn_q8_ref)."""

    @pytest.mark.parametrize("fmt,fmt_down,fused,act", [("q6_k", None, True, "silu"), ("q4_k", "q6_k", False, "silu"),
                                                        ("q5_k", "q8_0", True, "gelu"), ("q8_0", "q5_0", False, "silu"),
                                                        ("q4_0", None, True, "swiglu_oai"), ("q5_0", "q4_k", True, "silu")])
    @pytest.mark.parametrize("tokens", [1, 3])
    def test_layer_vs_oracle(self, ops, fmt, fmt_down, fused, act, tokens):
        E, ku, H, F = 8, 4, 512, 256
        rng = np.random.default_rng(tokens * 10 + len(fmt))
        fd = fmt_down or fmt
        wg = np.stack([blocks(fmt, F, H, 100 + e) for e in range(E)])
        wu = np.stack([blocks(fmt, F, H, 200 + e) for e in range(E)])
        wd = np.stack([blocks(fd, H, F, 300 + e) for e in range(E)])
        w_gu = np.concatenate([wg, wu], axis=1)   # per expert F gate rows then F up rows
        x = rng.standard_normal((tokens, H)).astype(np.float32)
        lg = rng.standard_normal((tokens, E)).astype(np.float32)
        kw = dict(w_up=dev(wu)) if not fused else {}
        y = host(ops.moe_ffn(fmt, dev(x), dev(lg), dev(wg if not fused else w_gu), dev(wd), H, F, E, ku,
                             prefill=False, act=act, fmt_down=fmt_down, act_q8=True, **kw))
        ids, wts = O.route_ref(lg, ku)
        ref = O.moe_ffn_q8_ref(x, ids, wts, w_gu, wd, fmt, H, F, act={"silu": O.ACT_SILU, "gelu": O.ACT_GELU,
                               "swiglu_oai": O.ACT_SWIGLU_OAI}[act], fmt_down=fd)
        assert O.rel_l2(y, ref) < 1e-3, O.rel_l2(y, ref)
        assert ops.device_status() == 0

    def test_refusals(self, ops):
        ids = torch.zeros(4, dtype=torch.int32, device="cuda")
        xq = torch.zeros(4096, dtype=torch.uint8, device="cuda")
        w = torch.zeros(1024, dtype=torch.uint8, device="cuda")
        with pytest.raises(ops.L.LkError):   # no integer codes for IQ4 in the MoE (gen_llm.py:5300-5301)
            ops.moe_expert_mv_q8("iq4_nl", "dn", ids, xq, w, 32, 256, 4, 8)
        with pytest.raises(ops.L.LkError):   # gate/up: whole tokens of ku assignments
            ops.moe_expert_mv_q8("q6_k", "gu", ids[:3], xq, w, 32, 256, 2, 8)


class TestMvQ8Multi:
    @pytest.mark.parametrize("fmt,k,tokens", [("q4_k", 4096, 1), ("q4_k", 12288, 1), ("q4_0", 4096, 1),
                                              ("q4_0", 12288, 1), ("q4_k", 4096, 3)])
    def test_segments_match_single_launches(self, ops, fmt, k, tokens):
        rng = np.random.default_rng(k + tokens)
        ns = [512, 128, 130] if fmt == "q4_k" else [256, 64]
        ws = [QUANT[fmt]((rng.standard_normal((n, k)) * 0.02).astype(np.float32)) for n in ns]
        x = rng.standard_normal((tokens, k)).astype(np.float32)
        xq = ops.quant_q8(dev(x))
        codes, meta = ops.q8_views(xq, tokens, k)
        xd = O.dequant_q8(host(codes), host(meta))
        ys = ops.mv_q8_multi(fmt, [dev(w) for w in ws], xq, ns, k, tokens)
        for w, n, y in zip(ws, ns, ys):
            ref = O.mv_ref(fmt, w, xd, n, k)
            assert O.rel_l2(host(y), ref) < TOL, O.rel_l2(host(y), ref)
        assert ops.device_status() == 0


# ---------------------------------------------------------------------------------------------------------- fused
@pytest.mark.parametrize("fmt", ["q4_k", "q4_0"])
@pytest.mark.parametrize("k,n", [(4096, 1000), (8192, 512), (12288, 2048)])
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_fused_quantisation_equals_two_launches(ops, fmt, k, n, xdt):
    # the matvec that quantises x in its own prologue gives lk_quant_q8 + lk_mv_q8's result bit for bit
    rng = np.random.default_rng(k + n)
    w = dev(weights(fmt, n, k, 5))
    x = dev(rng.standard_normal((1, k)).astype(np.float32))
    if xdt == "bf16":
        x = x.to(torch.bfloat16)
    y2 = ops.mv_q8(fmt, w, ops.quant_q8(x), n, k, 1)
    y1 = ops.mv_q8_fused(fmt, w, x, n, k)
    assert torch.equal(y1, y2)
    codes, meta = O.quant_q8(x.float().cpu().numpy())
    ref = O.mv_ref(fmt, host(w), O.dequant_q8(codes, meta), n, k)
    assert O.rel_l2(host(y1), ref) < TOL
    assert ops.device_status() == 0


def test_fused_multi_and_accumulate(ops):
    k = 4096
    ns = [4096, 1024, 1024]
    rng = np.random.default_rng(9)
    ws = [dev(weights("q4_k", n, k, 20 + i)) for i, n in enumerate(ns)]
    x = dev(rng.standard_normal((1, k)).astype(np.float32)).to(torch.bfloat16)
    y0 = [dev(rng.standard_normal((1, n)).astype(np.float32)) for n in ns]
    ys = [t.clone() for t in y0]
    ops.mv_q8_fused_multi("q4_k", ws, x, ns, k, ys=ys, accumulate=True)
    ref = [t.clone() for t in y0]
    ops.mv_q8_multi("q4_k", ws, ops.quant_q8(x), ns, k, 1, ys=ref, accumulate=True)
    for a, b in zip(ys, ref):
        assert torch.equal(a, b)


def test_fused_shapes_outside_the_row_kernel_are_refused(ops):
    from loom_skills_b200 import _lib as L
    w = dev(weights("q4_k", 64, 1024, 3))
    x = torch.zeros(1, 1024, device="cuda")
    with pytest.raises(L.LkError, match="no kernel"):
        ops.mv_q8_fused("q4_k", w, x, 64, 1024)


def test_fused_quantisation_rounding_boundaries(ops):
    # activations whose x / d lie on or next to k + 1/2 (exact ties with d = 1; near ties with d = 100/127): the
    # in-kernel quantisation must round them as lk_quant_q8 does (codes compared through the matvec, bit for bit)
    k, n = 4096, 512
    rng = np.random.default_rng(17)
    x = np.empty((1, k), np.float32)
    g = x.reshape(-1, 32)
    half = rng.integers(-126, 126, g.shape).astype(np.float32) + 0.5
    g[0::2] = half[0::2]
    g[0::2, 0] = 127.0                                            # d = 127 / 127 = 1: x / d = x, exact ties
    d = np.float32(100.0) / np.float32(127.0)
    g[1::2] = (half[1::2] * d).astype(np.float32)                 # x / d within a few ulps of k + 1/2
    g[1::2] = np.nextafter(g[1::2], rng.choice([-np.inf, np.inf], g[1::2].shape)).astype(np.float32)
    g[1::2, 0] = 100.0
    w = dev(weights("q4_k", n, k, 9))
    for xt in (dev(x), dev(x).to(torch.bfloat16)):
        ref = ops.mv_q8("q4_k", w, ops.quant_q8(xt), n, k, 1)
        assert torch.equal(ops.mv_q8_fused("q4_k", w, xt, n, k), ref)


@pytest.mark.parametrize("k", [4096, 12288])
def test_fused_quantisation_special_values(ops, k):
    # all-zero groups, a NaN or an infinity inside a group, subnormal and huge magnitudes: the in-kernel quantisation
    # gives lk_quant_q8's codes (compared through the matvec; NaN outputs must sit in the same places)
    n = 256
    rng = np.random.default_rng(k)
    x = rng.standard_normal((1, k)).astype(np.float32)
    g = x.reshape(-1, 32)
    g[0] = 0.0
    g[1, 5] = np.nan
    g[2, 7] = np.inf
    g[3, 9] = -np.inf
    g[4] = rng.standard_normal(32).astype(np.float32) * np.float32(1e-40)   # subnormal values, d underflows
    g[5] = rng.standard_normal(32).astype(np.float32) * np.float32(3e38)
    g[6, :] = np.float32(1e-45)
    g[7, 3] = -np.float32(1e-45)
    w = dev(weights("q4_k", n, k, 13))
    for xt in (dev(x), dev(x).to(torch.bfloat16)):
        ref = ops.mv_q8("q4_k", w, ops.quant_q8(xt), n, k, 1)
        got = ops.mv_q8_fused("q4_k", w, xt, n, k)
        torch.testing.assert_close(got, ref, rtol=0, atol=0, equal_nan=True)
    assert ops.device_status() == 0
