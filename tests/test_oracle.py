"""Pins the CPU oracle (oracle/qmm_oracle.py) against the reference's golden vectors and against gguf 0.19.0.

Everything here runs on the CPU. The golden fixtures come from the reference's own functions
(tests/golden/make_golden.py), so a passing oracle reproduces the reference's numerics bit for bit where they are
integer/byte/exact-float work.
"""
import hashlib
import os

import numpy as np
import pytest

from oracle import qmm_oracle as O


def _bits_equal(a, b):
    a = np.ascontiguousarray(np.asarray(a, np.float32))
    b = np.ascontiguousarray(np.asarray(b, np.float32))
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def q4_0_bits_inputs():
    """Every finite F16 scale with codes i | (15-i) << 4: the input of kbench moe_q4_0/gen_bench.py:51-63."""
    bits = np.arange(65536, dtype=np.uint16)
    bits = bits[(bits & 0x7C00) != 0x7C00]
    raw = np.empty((len(bits), 18), np.uint8)
    raw[:, :2] = bits.astype("<u2").view(np.uint8).reshape(-1, 2)
    codes = np.arange(16, dtype=np.uint8)
    raw[:, 2:] = codes | ((15 - codes) << 4)
    return raw


class TestDequantGolden:
    def test_q4_0_reference_decoder(self, golden):
        got = O.dequant("q4_0", golden["q4_0_raw"].reshape(-1, 704 // 32 * 18), 704)
        assert _bits_equal(got.reshape(golden["q4_0_f32"].shape), golden["q4_0_f32"])

    def test_q4_0_all_finite_scales_f16_staging(self, golden):
        raw = q4_0_bits_inputs()
        assert hashlib.sha256(raw.tobytes()).digest() == golden["q4_0_bits_raw_sha256"].tobytes()
        with np.errstate(over="ignore"):
            got = O.dequant_f16("q4_0", raw, 32).view(np.uint16)
        assert np.array_equal(got[golden["q4_0_bits_rows"]], golden["q4_0_bits_sample"])
        assert hashlib.sha256(got.tobytes()).digest() == golden["q4_0_bits_sha256"].tobytes()

    @pytest.mark.parametrize("fmt,qk", [("q4_k", 256), ("iq4_nl", 32), ("mxfp4", 32), ("q4_0g", 32)])
    def test_gguf_blocks(self, golden, fmt, qk):
        f = "q4_0" if fmt == "q4_0g" else fmt
        got = O.dequant(f, golden[f"{fmt}_raw"], qk)
        assert _bits_equal(got, golden[f"{fmt}_f32"])

    def test_mxfp4_planar(self, golden):
        got = O.dequant("mxfp4_planar", (golden["mxfp4s_nib"], golden["mxfp4s_sc"]), 192)
        assert _bits_equal(got, golden["mxfp4s_f32"])
        known = O.dequant("mxfp4_planar", (golden["mxfp4s_known_nib"], golden["mxfp4s_known_sc"]), 32)
        assert known[0, :4].tolist() == [1.0, 2.0, -12.0, 12.0]
        assert _bits_equal(known, golden["mxfp4s_known_f32"])

    def test_mxfp4_bf8_decode(self, golden):
        e, q = golden["bf8_e"], golden["bf8_q"]
        codes = np.concatenate([q & 15, q >> 4], 1)
        got = O.mxfp4_e5m2_bytes(np.repeat(e[:, None], 32, 1), codes)
        assert np.array_equal(got, golden["bf8_bytes"])
        assert np.array_equal(O.e5m2_values(got), golden["bf8_values"])

    def test_e4m3(self, golden):
        r = O.e4m3_round(golden["e4m3_in"])
        assert np.array_equal(r, golden["e4m3_round"])
        # kbench gemm_mxfp4s/gen_bench.py:280 drops the sign of a negative zero; make_kernel_tests.py:2018 keeps it
        # (0x80), as the hardware conversion does -- the oracle follows the latter.
        negzero = (r == 0) & np.signbit(r)
        b = O.e4m3_bytes(r)
        assert np.array_equal(b[~negzero], golden["e4m3_bytes"][~negzero])
        assert negzero.any() and (b[negzero] == 0x80).all()
        assert np.array_equal(O.e4m3_values(golden["e4m3_bytes"]), np.abs(r) * np.where(golden["e4m3_bytes"] & 0x80, -1, 1))

    def test_e4m3_matches_ml_dtypes(self):
        ml = pytest.importorskip("ml_dtypes")
        v = np.random.default_rng(0).standard_normal(20000) * 40
        assert np.array_equal(O.e4m3_round(v), v.astype(ml.float8_e4m3fn).astype(np.float64))


class TestProductsGolden:
    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k", "iq4_nl"])
    def test_mv(self, golden, fmt):
        w, x = golden[f"mv_{fmt}_w"], golden[f"mv_{fmt}_x"]
        y = O.mv_ref(fmt, w, x, w.shape[0], 512)
        np.testing.assert_allclose(y, golden[f"mv_{fmt}_y"], rtol=1e-12, atol=1e-12)

    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k", "iq4_nl"])
    def test_row_scale_and_gemm(self, golden, fmt):
        x16, sc = O.row_scale_f16(golden[f"gemm_{fmt}_x"])
        assert np.array_equal(x16.view(np.uint16), golden[f"gemm_{fmt}_x16"].view(np.uint16))
        assert _bits_equal(sc, golden[f"gemm_{fmt}_scales"])
        w = golden[f"mv_{fmt}_w"]
        y = O.gemm_ref(fmt, w, x16, sc, w.shape[0], 512)
        np.testing.assert_allclose(y, golden[f"gemm_{fmt}_y"], rtol=1e-12, atol=1e-9)


class TestNegativeControls:
    """A planted mistake in the oracle (CPU only) must fail against the reference's golden vectors."""

    def test_nibble_swap_fails(self, golden):
        raw = golden["q4_0_raw"].reshape(-1, 18).copy()
        raw[:, 2:] = ((raw[:, 2:] & 15) << 4) | (raw[:, 2:] >> 4)
        got = O.dequant("q4_0", raw, 32).reshape(golden["q4_0_f32"].shape)
        assert not _bits_equal(got, golden["q4_0_f32"])

    def test_unsigned_scale_fails(self, golden):
        raw = golden["q4_0_raw"].reshape(-1, 18).copy()
        raw[:, 1] &= 0x7F
        got = O.dequant("q4_0", raw, 32).reshape(golden["q4_0_f32"].shape)
        assert not _bits_equal(got, golden["q4_0_f32"])


class TestQuantisers:
    def test_q4_0_matches_gguf(self):
        gq = pytest.importorskip("gguf.quants")
        from gguf import GGMLQuantizationType as T
        w = (np.random.default_rng(1).standard_normal((64, 4096)) * 0.02).astype(np.float32)
        assert np.array_equal(O.quantize_q4_0(w).reshape(-1), gq.quantize(w, T.Q4_0).reshape(-1))

    @pytest.mark.parametrize("fmt,ty", [("q4_k", 12), ("iq4_nl", 20), ("mxfp4", 39)])
    def test_own_quantisers_decode_like_gguf(self, fmt, ty):
        gq = pytest.importorskip("gguf.quants")
        from gguf import GGMLQuantizationType as T
        w = (np.random.default_rng(2).standard_normal((32, 1024)) * 0.02).astype(np.float32)
        raw = O.quantize_mxfp4(w, "ggml") if fmt == "mxfp4" else getattr(O, f"quantize_{fmt}")(w)
        assert raw.shape == (32, O.row_bytes(fmt, 1024))
        mine = O.dequant(fmt, raw, 1024)
        theirs = gq.dequantize(raw.reshape(-1), T(ty)).reshape(32, 1024)
        assert _bits_equal(mine, theirs)
        err = O.rel_l2(mine, w)
        assert err < {"q4_k": 0.12, "iq4_nl": 0.12, "mxfp4": 0.2}[fmt], err

    def test_mxfp4_layouts_agree(self):
        w = (np.random.default_rng(3).standard_normal((8, 256)) * 0.02).astype(np.float32)
        nib, sc = O.quantize_mxfp4(w, "planar")
        g = O.quantize_mxfp4(w, "ggml")
        a = O.dequant("mxfp4_planar", (nib, sc), 256)
        b = O.dequant("mxfp4", g, 256)
        np.testing.assert_array_equal(a, b)
        assert (sc >= 107).all() and (sc <= 132).all()      # N(0, 0.02) stays inside the bf8-exact range


class TestRowScale:
    def test_magnitudes(self):
        x = (np.random.default_rng(4).standard_normal((3, 512)) * np.array([[1e-3], [1.0], [3e5]])).astype(np.float32)
        x16, sc = O.row_scale_f16(x)
        e = np.clip(np.frexp(np.abs(x).max(1))[1] - 1 - 13, 0, 100)       # make_kernel_tests.py:1763
        np.testing.assert_array_equal(sc, np.stack([2.0 ** -e, 2.0 ** e], 1).astype(np.float32))
        assert np.isfinite(x16.astype(np.float32)).all()

    def test_f8_row_max_in_range(self):
        x = (np.random.default_rng(5).standard_normal((16, 2880)) * 3).astype(np.float32)
        x8, s8 = O.row_scale_f8(x)
        v = O.e4m3_values(x8)
        mx = np.abs(v).max(1)
        assert ((mx >= 128) & (mx <= 256)).all()
        np.testing.assert_allclose(v * (s8[:, 1:2].astype(np.float64) * 2.0 ** 8), x, rtol=0.07, atol=2e-4)


class TestMoE:
    def test_route_ties_lowest_index(self):
        lg = np.zeros((2, 16), np.float32)
        lg[1, [3, 9]] = 2.0
        ids, w = O.route_ref(lg, 4)
        assert ids[0].tolist() == [0, 1, 2, 3]
        assert ids[1].tolist() == [3, 9, 0, 1]
        np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)

    def test_bucket(self):
        rng = np.random.default_rng(6)
        t, ku, E = 37, 8, 16
        lg = rng.standard_normal((t, E)).astype(np.float32)
        ids, _ = O.route_ref(lg, ku)
        live = np.ones(t, np.int32)
        live[5] = 0
        mt = O.moe_max_tiles(t, ku, E)
        ti, rm, pos = O.bucket_ref(ids, E, mt, live)
        assert O.check_bucket(ids, E, mt, ti, rm, pos, live) is None
        assert (pos[5 * ku:6 * ku] == -1).all()
        used = ti[:, 0] >= 0
        assert ti[used, 1].sum() == (t - 1) * ku
        # a different order of rows within one expert is also valid
        e0 = ti[0, 0]
        rows = np.nonzero(rm[:64] >= 0)[0]
        rm2, pos2 = rm.copy(), pos.copy()
        rm2[rows] = rm[rows][::-1]
        pos2[rm2[rows]] = rows
        assert O.check_bucket(ids, E, mt, ti, rm2, pos2, live) is None
        rm2[rows[0]], rm2[-1] = -1, rm2[rows[0]]
        assert O.check_bucket(ids, E, mt, ti, rm2, pos2, live) is not None
        assert e0 >= 0


class TestQuantQ8:
    def test_matches_reference_q8_ref(self, golden):
        """quant_q8 + dequant_q8 == make_kernel_tests.py q8_ref (numerically; q8_ref's float codes can be -0.0)."""
        codes, meta = O.quant_q8(golden["q8_in"])
        got = O.dequant_q8(codes, meta).astype(np.float32)
        assert np.array_equal(got, golden["q8_deq"])

    def test_rounding_and_zero_groups(self):
        x = np.zeros((1, 64), np.float32)
        x[0, 0] = 127.0                       # d = 1: codes are round(x) half away from zero
        x[0, 1:6] = [0.5, -0.5, 1.5, -2.5, 0.49999997]
        codes, meta = O.quant_q8(x)
        assert codes[0, :6].tolist() == [127, 1, -1, 2, -3, 0]
        assert meta[0, 0, 0] == 1.0 and meta[0, 0, 1] == 127 + 1 - 1 + 2 - 3
        assert (codes[0, 32:] == 0).all() and meta[0, 1].tolist() == [0.0, 0.0]


# ---------------------------------------------------------------------------------------------------------- MoE pins
@pytest.fixture(scope="module")
def gmoe():
    with np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_moe.npz")) as z:
        return {k: z[k] for k in z.files}


def _digests_match(inputs, names, digests):
    import hashlib
    for name, d in zip(names, digests):
        got = hashlib.sha256(np.ascontiguousarray(inputs[str(name)]).tobytes()).digest()
        assert got == d.tobytes(), name


@pytest.mark.parametrize("case", ["r1", "r2", "r3", "r4", "r5", "r6"])
def test_route_ref_matches_reference_router(gmoe, case):
    # make_kernel_tests.py:3166-3186 route_ref, every gating / norm / bias / scale combination of the golden set
    gating, norm, has_bias, E, KU = (int(v) for v in gmoe[f"route_{case}_cfg"])
    ids, wts = O.route_ref(gmoe[f"route_{case}_logits"], KU, gating=gating, norm=bool(norm),
                           bias=gmoe[f"route_{case}_bias"] if has_bias else None,
                           scale=float(gmoe[f"route_{case}_scale"][0]))
    assert np.array_equal(ids, gmoe[f"route_{case}_ids"])
    np.testing.assert_allclose(wts, gmoe[f"route_{case}_wts"], rtol=2e-6, atol=1e-8)


def test_ffn_inputs_regenerate(gmoe):
    _digests_match(O.ffn_golden_inputs(), gmoe["ffn_digest_names"], gmoe["ffn_digests"])


@pytest.mark.parametrize("name,act,mx", [("silu", O.ACT_SILU, False), ("gelu", O.ACT_GELU, False),
                                         ("oai", O.ACT_SWIGLU_OAI, False), ("oai_mx", O.ACT_SWIGLU_OAI, True)])
def test_moe_ffn_ref_matches_reference_experts(gmoe, name, act, mx):
    # make_kernel_tests.py:3196-3215 experts_ref (decode precision); oai cases carry the per-expert biases
    fi = O.ffn_golden_inputs()
    E, H, F = 8, 512, 256
    kw = dict(b_gate=fi["bg"], b_up=fi["bu"], b_down=fi["bd"]) if name.startswith("oai") else {}
    if mx:
        wgu = O.dequant_mxfp4_planar(fi["mx_gu_nib"], fi["mx_gu_sc"], E * 2 * F, H).reshape(E, 2 * F, H)
        wdn = O.dequant_mxfp4_planar(fi["mx_dn_nib"], fi["mx_dn_sc"], E * H, F).reshape(E, H, F)
        y = O.moe_ffn_ref(fi["x"], fi["ids"], fi["wts"], wgu, wdn, None, H, F, E, act=act, **kw)
    else:
        y = O.moe_ffn_ref(fi["x"], fi["ids"], fi["wts"], fi["w_gu"], fi["w_dn"], "q4_0", H, F, E, act=act, **kw)
    assert O.rel_l2(y, gmoe[f"ffn_{name}_d_y"]) < 1e-6


def test_moe_chain_down_scale_and_shared_gate(gmoe):
    # make_kernel_tests.py:3268-3271: weights scaled per expert (g_moe_wscale), shared output gated (shared_gated)
    fi = O.ffn_golden_inputs()
    sg = O.shared_gate_ref(fi["x"], fi["wsg"])
    np.testing.assert_allclose(sg, gmoe["ffn_chain_sg"], rtol=1e-6)
    np.testing.assert_array_equal(O.wscale_ref(fi["ids"], fi["wts"], fi["dsc"]), gmoe["ffn_chain_wts_s"])
    y = O.moe_ffn_ref(fi["x"], fi["ids"], fi["wts"], fi["w_gu"], fi["w_dn"], "q4_0", 512, 256, 8, dsc=fi["dsc"],
                      y0=fi["y0"], sg=sg)
    assert O.rel_l2(y, gmoe["ffn_chain_y"]) < 1e-6


@pytest.fixture(scope="module")
def kbench():
    return O.kbench_moe_inputs(490)


def test_kbench_inputs_regenerate(gmoe, kbench):
    # the oracle draws the kbench moe_q4_0 inputs in the generator's own order (gen_bench.py:142-248)
    _digests_match(kbench, gmoe["kb_digest_names"], gmoe["kb_digests"])


def test_kbench_cases_from_oracle(gmoe, kbench):
    # the oracle's act / combine restatements reproduce the reference's F64 expectations of every kbench case
    H, F, U = O.KB_H, O.KB_F, O.KB_U
    gu, down = kbench["gu"], kbench["down"]
    for t in (1, 4):
        ids, x = kbench[f"decode_t{t}_ids"], kbench[f"decode_t{t}_x"]
        pair = np.stack([gu[e] @ x[a // U].astype(np.float64) for a, e in enumerate(ids.flat)])
        act = O.act_ref(pair[:, :F], pair[:, F:], O.ACT_GELU)
        assert O.rel_l2(act, gmoe[f"kb_decode_gu_t{t}"]) < 1e-6
    ti = np.array(O.KB_TILE_INFO)
    for t in (63, 65):
        rm, x, s = kbench[f"grouped_t{t}_rm"], kbench[f"grouped_t{t}_x"], kbench[f"grouped_t{t}_s"]
        ref = gmoe[f"kb_grouped_gu_t{t}"]
        assert (ref[192:] == O.KB_SENTINEL).all()          # the dead tile is never written
        e = ti[1, 0]
        W16 = gu[e].astype(np.float16).astype(np.float64)
        for q in range(17):
            src = rm[64 + q] // U
            pair = W16 @ x[src].astype(np.float64) * s[src, 1]
            np.testing.assert_allclose(O.act_ref(pair[:F], pair[F:], O.ACT_GELU)[gmoe["kb_cols_f"]], ref[64 + q],
                                       rtol=1e-6, atol=1e-9)
        assert (ref[64 + 17:128] == 0).all()               # padding rows of a live tile hold zeros
    y = O.combine_ref(kbench["dsc_ys"], O.wscale_ref(kbench["dsc_ids"], kbench["dsc_wts"], kbench["dsc_scales"]))
    assert O.rel_l2(y, gmoe["kb_dsc_y"]) < 1e-6


# ---------------------------------------------------------------------------------------------------------- formats
@pytest.fixture(scope="module")
def gfmt():
    with np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_formats.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("fmt", ["q5_0", "q8_0", "q3_k", "q5_k", "q6_k", "iq4_xs", "iq3_s"])
def test_remaining_formats_match_gguf(gfmt, fmt):
    # the oracle's restatement of gguf 0.19.0's dequantize_blocks, bit for bit on the golden blocks
    raw = gfmt[f"{fmt}_raw"]
    got = O.dequant(fmt, raw.reshape(-1), gfmt[f"{fmt}_f32"].size)
    assert _bits_equal(got, gfmt[f"{fmt}_f32"].reshape(-1))
    w, x = gfmt[f"mv_{fmt}_w"], gfmt[f"mv_{fmt}_x"]
    assert O.rel_l2(O.mv_ref(fmt, w, x, w.shape[0], 512), gfmt[f"mv_{fmt}_y"]) < 1e-12


@pytest.mark.parametrize("fmt", ["q5_k", "q6_k", "q8_0"])
def test_f16_staging_is_one_rounding_or_the_fma(gfmt, fmt):
    # Q8_0: one rounding of the exact value (gen_gemm.py:352-367); Q5_K / Q6_K: the f16 fma of gen_gemm.py:369-498,
    # whose f16 scale and offset each round once: within a few f16 steps of the group's largest value
    raw = gfmt[f"{fmt}_raw"]
    exact = O.dequant(fmt, raw.reshape(-1), gfmt[f"{fmt}_f32"].size).astype(np.float64)
    st = O.dequant_f16(fmt, raw.reshape(-1), exact.size).astype(np.float64)
    if fmt == "q8_0":
        assert np.array_equal(st, exact.astype(np.float16).astype(np.float64))
    else:
        gmax = np.abs(exact).reshape(-1, 16).max(-1, keepdims=True)
        assert np.all(np.abs(st - exact).reshape(-1, 16) <= gmax * 2.0 ** -8 + 2.0 ** -24)
