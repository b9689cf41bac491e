"""GPU parity of the MoE router and expert epilogues against vectors the reference's own code produced
(tests/golden/golden_moe.npz, written by tests/golden/make_golden.py):

* router: make_kernel_tests.py:3166-3186 route_ref -- gating 1 / 2 / 3, norm, selection / router bias, scale --
  through both router kernels (given logits; router weights);
* expert FFN: make_kernel_tests.py:3196-3215 experts_ref -- SiLU, GEGLU (gelu-tanh), gpt-oss swiglu_oai with
  per-expert biases, Q4_0 and MXFP4 experts -- on the decode path (expert matvecs) and the prefill path (bucketed
  grouped GEMMs), and the chain of :3268-3271 (g_moe_wscale down scale, shared-expert gate, shared output);
* the kbench moe_q4_0 cases (.github/devlab/kbench/moe_q4_0/gen_bench.py:185-248): hand-built tile_info with a full
  tile, 17- and 1-row tails and a dead tile, outputs pre-filled with sentinel 42, at the reference's own tolerances.

Bars: routing ids exact; weights within 2e-6 relative (f32 kernels against the reference's f64); products within
relative L2 1e-3 (f32/f16 accumulation) or 2e-2 (e4m3 activations, against the oracle's e4m3 chain); the kbench
cases at gen_bench.py's atol / rtol.
"""
import os

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


@pytest.fixture(scope="module")
def gmoe():
    with np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_moe.npz")) as z:
        return {k: z[k] for k in z.files}


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


# ---------------------------------------------------------------------------------------------------------- router
@pytest.mark.parametrize("case", ["r1", "r2", "r3", "r4", "r5", "r6"])
@pytest.mark.parametrize("with_router_w", [False, True])
def test_router_matches_reference(ops, gmoe, case, with_router_w):
    gating, norm, has_bias, E, KU = (int(v) for v in gmoe[f"route_{case}_cfg"])
    lg = gmoe[f"route_{case}_logits"]
    bias = dev(gmoe[f"route_{case}_bias"]) if has_bias else None
    scale = float(gmoe[f"route_{case}_scale"][0])
    if with_router_w:   # logits = x . I, exact in f32: the 256-thread router kernel with its own dot products
        ids, wts = ops.moe_route(dev(lg), E, KU, router_w=dev(np.eye(E, dtype=np.float32)), gating=gating,
                                 norm=bool(norm), scale=scale, bias=bias)
    else:
        ids, wts = ops.moe_route(dev(lg), E, KU, gating=gating, norm=bool(norm), scale=scale, bias=bias)
    assert np.array_equal(host(ids), gmoe[f"route_{case}_ids"])
    np.testing.assert_allclose(host(wts), gmoe[f"route_{case}_wts"], rtol=2e-6, atol=1e-8)


# ---------------------------------------------------------------------------------------------------------- expert FFN
def _ffn_given_routing(ops, prefill, fi, ids, wts, E, H, F, KU, act, biases, mx=False):
    """The expert FFN with the routing given: decode = expert matvecs + combine; prefill = bucket + row scale +
    grouped GEMMs + sorted combine (the wiring of ops.moe_ffn after its router)."""
    x = dev(fi["x"])
    idt, wt = dev(ids), dev(wts)
    bg, bu, bd = (dev(fi["bg"]), dev(fi["bu"]), dev(fi["bd"])) if biases else (None, None, None)
    if mx:
        wgu, sgu = dev(fi["mx_gu_nib"]), dev(fi["mx_gu_sc"])
        wdn, sdn = dev(fi["mx_dn_nib"]), dev(fi["mx_dn_sc"])
    else:
        wgu, wdn = dev(fi["w_gu"]), dev(fi["w_dn"])
    if not prefill:
        if mx:
            a = ops.moe_expert_mv_mxfp4s("gu", idt.reshape(-1), x, wgu, sgu, F, H, KU, E, act=act, bias=bg, bias2=bu)
            ys = ops.moe_expert_mv_mxfp4s("dn", idt.reshape(-1), a, wdn, sdn, H, F, KU, E, bias=bd)
        else:
            a = ops.moe_expert_mv("q4_0", "gu", idt.reshape(-1), x, wgu, F, H, KU, E, act=act, bias=bg, bias2=bu)
            ys = ops.moe_expert_mv("q4_0", "dn", idt.reshape(-1), a, wdn, H, F, KU, E, bias=bd)
        return host(ops.moe_combine(ys, wt))
    ti, rm, pos = ops.moe_bucket(idt, E)
    if mx:
        x8, s8 = ops.moe_row_scale_gather(x, rm, KU, f8=True)
        a = ops.moe_grouped_gemm_mxfp4s_f8("swiglu_sorted", ti, rm, x8, s8, wgu, sgu, F, KU, E, fused=True, act=act,
                                           bias=bg, bias2=bu)
        a8, as8 = ops.row_scale_f8(a)
        ys = ops.moe_grouped_gemm_mxfp4s_f8("store", ti, rm, a8, as8, wdn, sdn, H, KU, E, bias=bd)
    else:
        x16, sc = ops.moe_row_scale_gather(x, rm, KU)
        a = ops.moe_grouped_gemm("q4_0", "swiglu_sorted", ti, rm, x16, sc, wgu, F, KU, E, fused=True, act=act,
                                 bias=bg, bias2=bu)
        a16, asc = ops.row_scale_f16(a)
        ys = ops.moe_grouped_gemm("q4_0", "store", ti, rm, a16, asc, wdn, H, KU, E, bias=bd)
    return host(ops.moe_combine_sorted(ys, pos, wt))


@pytest.mark.parametrize("name,act,biases,mx", [("silu", "silu", False, False), ("gelu", "gelu", False, False),
                                                ("oai", "swiglu_oai", True, False),
                                                ("oai_mx", "swiglu_oai", True, True)])
@pytest.mark.parametrize("prefill", [False, True])
def test_expert_ffn_matches_reference(ops, gmoe, name, act, biases, mx, prefill):
    fi = O.ffn_golden_inputs()
    y = _ffn_given_routing(ops, prefill, fi, fi["ids"], fi["wts"], 8, 512, 256, 4, act, biases, mx)
    ref = gmoe[f"ffn_{name}_{'p' if prefill else 'd'}_y"]
    if mx and prefill:
        # the fp8 path quantises the activations to e4m3: against the oracle's e4m3 chain (the north-star 2e-2),
        # and within e4m3 rounding (3 mantissa bits) of the reference's f16-precision expectation
        ora = O.moe_ffn_mxfp4_ref(fi["x"], fi["ids"], fi["wts"], fi["mx_gu_nib"], fi["mx_gu_sc"], fi["mx_dn_nib"],
                                  fi["mx_dn_sc"], 512, 256, act=O.ACT_SWIGLU_OAI, b_gate=fi["bg"], b_up=fi["bu"],
                                  b_down=fi["bd"])
        assert O.rel_l2(y, ora) < 2e-2, O.rel_l2(y, ora)
        assert O.rel_l2(y, ref) < 6e-2, O.rel_l2(y, ref)
    else:
        assert O.rel_l2(y, ref) < TOL, O.rel_l2(y, ref)
    assert ops.device_status() == 0


@pytest.mark.parametrize("prefill", [False, True])
def test_chain_down_scale_shared_gate(ops, gmoe, prefill):
    fi = O.ffn_golden_inputs()
    ids, wts = dev(fi["ids"]), dev(fi["wts"]).clone()
    ops.moe_wscale(ids, wts, dev(fi["dsc"]))
    assert np.array_equal(host(wts), gmoe["ffn_chain_wts_s"])           # one f32 product each, as the reference's
    sg = ops.moe_shared_gate(dev(fi["x"]), dev(fi["wsg"]))
    np.testing.assert_allclose(host(sg), gmoe["ffn_chain_sg"], rtol=1e-5)
    # the routed experts on the scaled weights, added to the gated shared output
    x = dev(fi["x"])
    wgu, wdn = dev(fi["w_gu"]), dev(fi["w_dn"])
    y = dev(fi["y0"])
    if prefill:
        ti, rm, pos = ops.moe_bucket(ids, 8)
        x16, sc = ops.moe_row_scale_gather(x, rm, 4)
        a = ops.moe_grouped_gemm("q4_0", "swiglu_sorted", ti, rm, x16, sc, wgu, 256, 4, 8, fused=True)
        a16, asc = ops.row_scale_f16(a)
        ys = ops.moe_grouped_gemm("q4_0", "store", ti, rm, a16, asc, wdn, 512, 4, 8)
        ops.moe_combine_sorted(ys, pos, wts, y=y, sg=sg)
    else:
        a = ops.moe_expert_mv("q4_0", "gu", ids.reshape(-1), x, wgu, 256, 512, 4, 8)
        ys = ops.moe_expert_mv("q4_0", "dn", ids.reshape(-1), a, wdn, 512, 256, 4, 8)
        ops.moe_combine(ys, wts, y=y, sg=sg)
    assert O.rel_l2(host(y), gmoe["ffn_chain_y"]) < TOL


@pytest.mark.parametrize("prefill", [False, True])
def test_moe_ffn_full_wiring(ops, prefill):
    # ops.moe_ffn with every option of the reference's wiring: sigmoid gating with a selection bias, scale, GEGLU,
    # expert biases, down scale, shared output and gate -- against the oracle's float64 chain
    E, KU, H, F, t = 16, 4, 512, 256, 24
    rng = np.random.default_rng(5)
    w_gu = np.stack([O.quantize_q4_0((rng.standard_normal((2 * F, H)) * 0.02).astype(np.float32)) for _ in range(E)])
    w_dn = np.stack([O.quantize_q4_0((rng.standard_normal((H, F)) * 0.02).astype(np.float32)) for _ in range(E)])
    x = rng.standard_normal((t, H)).astype(np.float32)
    lg = rng.standard_normal((t, E)).astype(np.float32)
    rb = (rng.standard_normal(E) * 0.3).astype(np.float32)
    bg = (rng.standard_normal((E, F)) * 0.05).astype(np.float32)
    bu = (rng.standard_normal((E, F)) * 0.05).astype(np.float32)
    bd = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
    dsc = rng.uniform(0.5, 1.5, E).astype(np.float32)
    wsg = (rng.standard_normal(H) * 0.05).astype(np.float32)
    y0 = (rng.standard_normal((t, H)) * 0.1).astype(np.float32)
    y = dev(y0)
    ops.moe_ffn("q4_0", dev(x), dev(lg), dev(w_gu), dev(w_dn), H, F, E, KU, prefill=prefill, gating=2,
                router_bias=dev(rb), scale=2.5, act="gelu", b_gate=dev(bg), b_up=dev(bu), b_down=dev(bd),
                down_scale=dev(dsc), y_shared=y, shared_gate_w=dev(wsg))
    ids, wts = O.route_ref(lg, KU, gating=2, norm=True, bias=rb, scale=2.5)
    ref = O.moe_ffn_ref(x, ids, wts, w_gu, w_dn, "q4_0", H, F, E, act=O.ACT_GELU, b_gate=bg, b_up=bu, b_down=bd,
                        dsc=dsc, y0=y0, sg=O.shared_gate_ref(x, wsg))
    assert O.rel_l2(host(y), ref) < TOL, O.rel_l2(host(y), ref)


# ---------------------------------------------------------------------------------------------------------- kbench
@pytest.fixture(scope="module")
def kb():
    return O.kbench_moe_inputs(490)


@pytest.mark.parametrize("t", [1, 4])
def test_kbench_decode_gate_up_geglu(ops, gmoe, kb, t):
    H, F, E, U = O.KB_H, O.KB_F, O.KB_E, O.KB_U
    ids = dev(kb[f"decode_t{t}_ids"].reshape(-1))
    act = ops.moe_expert_mv("q4_0", "gu", ids, dev(kb[f"decode_t{t}_x"]), dev(kb["wg"]), F, H, U, E, act="gelu")
    np.testing.assert_allclose(host(act), gmoe[f"kb_decode_gu_t{t}"], atol=2e-5, rtol=2e-4)   # gen_bench.py:163


@pytest.mark.parametrize("t", [63, 65])
def test_kbench_grouped_gate_up_geglu(ops, gmoe, kb, t):
    # gen_bench.py:204-225: tile_info [[7,64],[0,17],[3,1],[-1,0]], token rows gathered by rowmap / U, sentinel 42
    H, F, E, U = O.KB_H, O.KB_F, O.KB_E, O.KB_U
    ti = dev(np.array(O.KB_TILE_INFO, np.int32))
    rm = dev(kb[f"grouped_t{t}_rm"])
    y = torch.full((256, F), O.KB_SENTINEL, dtype=torch.float32, device="cuda")
    ops.moe_grouped_gemm("q4_0", "swiglu", ti, rm, dev(kb[f"grouped_t{t}_x"]), dev(kb[f"grouped_t{t}_s"]),
                         dev(kb["wg"]), F, U, E, fused=True, y=y, act="gelu")
    yh = host(y)
    assert (yh[192:] == O.KB_SENTINEL).all()                          # the dead tile is not written
    np.testing.assert_allclose(yh[:, gmoe["kb_cols_f"]], gmoe[f"kb_grouped_gu_t{t}"], atol=5e-5, rtol=5e-4)
    for j, n in enumerate(O.KB_COUNTS[:3]):                          # padding rows of the live tiles: zero products
        assert (yh[j * 64 + n:(j + 1) * 64] == 0).all()


def test_kbench_down_scale_combine(ops, gmoe, kb):
    # gen_bench.py:239-248: g_moe_wscale then g_moe_combine
    wts = dev(kb["dsc_wts"]).clone()
    ops.moe_wscale(dev(kb["dsc_ids"]), wts, dev(kb["dsc_scales"]))
    assert np.array_equal(host(wts), gmoe["kb_dsc_wts_s"])
    y = host(ops.moe_combine(dev(kb["dsc_ys"]), wts))
    np.testing.assert_allclose(y, gmoe["kb_dsc_y"], atol=2e-5, rtol=2e-4)
