"""GPU parity of lk_moe_ffn_decode_q8, the decode MoE layer on int8 activations (MOE_Q8=1, gen_llm.py:5290-5302) in two
launches, through the C ABI.

Against the float64 oracle of the same numerics (moe_ffn_q8_ref: x quantised by g_quant_q8, act rounded to f32 and
quantised again per assignment, float64 products of the codes with the dequantised weights): relative L2 <= 1e-3
(the GPU's f32 group scaling and act differ from float64 by rounding; a code at an exact rounding tie can land one
step apart). The routing it returns is lk_moe_route's bit for bit (the same device code on the same logits), with
the down scale applied as lk_moe_wscale does. Cases: both Q4 formats, fused and separate gate/up, gating 1/2/3 with
router bias and scale, norm on and off, the three activations with biases, accumulate with the shared-expert gate,
f32 and bf16 x, 1-4 tokens, h = 2048 and 4096, the largest f the limits allow.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

TOL = 1e-3
QUANT = {"q4_0": O.quantize_q4_0, "q4_k": O.quantize_q4_k}
ACT = {"silu": O.ACT_SILU, "gelu": O.ACT_GELU, "swiglu_oai": O.ACT_SWIGLU_OAI}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from loom_skills_b200 import ops as _ops
    return _ops


def experts(fmt, E, h, f, seed):
    rng = np.random.default_rng(seed)
    q = QUANT[fmt]
    gu = q((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32))
    dn = q((rng.standard_normal((E * h, f)) * 0.02).astype(np.float32))
    return gu, dn


def split_gate_up(gu, E, f):
    """[E][2f] fused rows -> separate [E][f] gate and up tensors."""
    r = gu.reshape(E, 2 * f, -1)
    return np.ascontiguousarray(r[:, :f]).reshape(E * f, -1), np.ascontiguousarray(r[:, f:]).reshape(E * f, -1)


CASES = [
    # fmt, tokens, E, ku, h, f, gating, norm, act, biases, fused, xdt, accumulate
    ("q4_0", 1, 32, 8, 2048, 768, 1, True, "silu", False, True, "bf16", False),
    ("q4_k", 1, 32, 8, 2048, 768, 1, True, "silu", False, False, "f32", False),
    ("q4_0", 3, 16, 4, 2048, 512, 2, False, "gelu", True, True, "f32", True),
    ("q4_k", 4, 32, 4, 2048, 1024, 3, False, "swiglu_oai", True, False, "bf16", False),
    ("q4_k", 2, 8, 2, 4096, 768, 1, False, "silu", False, True, "bf16", True),
    ("q4_0", 4, 8, 8, 2048, 2048, 1, True, "silu", False, True, "f32", False),   # tokens * ku * f = 65536
]


@pytest.mark.parametrize("fmt,tokens,E,ku,h,f,gating,norm,act,biases,fused,xdt,accumulate", CASES)
def test_matches_the_oracle(ops, fmt, tokens, E, ku, h, f, gating, norm, act, biases, fused, xdt, accumulate):
    rng = np.random.default_rng(tokens * 100 + ku + h + f)
    gu, dn = experts(fmt, E, h, f, seed=E + f)
    x = rng.standard_normal((tokens, h)).astype(np.float32)
    lg = rng.standard_normal((tokens, E)).astype(np.float32)
    rbias = (rng.standard_normal(E) * 0.5).astype(np.float32) if gating != 1 else None
    dsc = rng.uniform(0.5, 1.5, E).astype(np.float32)
    bg = bu = bd = None
    if biases:
        bg, bu = (rng.standard_normal((E, f)) * 0.05).astype(np.float32), (rng.standard_normal((E, f)) * 0.05).astype(np.float32)
        bd = (rng.standard_normal((E, h)) * 0.05).astype(np.float32)
    y0 = rng.standard_normal((tokens, h)).astype(np.float32)
    sg = rng.uniform(0.2, 0.9, tokens).astype(np.float32)
    scale = 1.5 if gating == 2 else 1.0
    d = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()
    xt = d(x) if xdt == "f32" else d(x).to(torch.bfloat16)
    if fused:
        wg, wu = d(gu), None
    else:
        g_, u_ = split_gate_up(gu, E, f)
        wg, wu = d(g_), d(u_)
    y = d(y0).clone() if accumulate else None
    out, ids, wts = ops.moe_ffn_decode_q8(fmt, xt, d(lg), wg, d(dn), h, f, E, ku, w_up=wu, gating=gating, norm=norm,
                                         scale=scale, router_bias=d(rbias), down_scale=d(dsc), act=act,
                                         b_gate=d(bg), b_up=d(bu), b_down=d(bd), y=y, accumulate=accumulate,
                                         sg=d(sg) if accumulate else None, routing=True)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    # the routing: lk_moe_route's, bit for bit, then the down scale as lk_moe_wscale applies it
    rid, rw = ops.moe_route(d(lg), E, ku, gating=gating, norm=norm, scale=scale, bias=d(rbias))
    assert torch.equal(ids, rid)
    assert torch.equal(wts, rw * d(dsc)[rid.long()])
    ref = O.moe_ffn_q8_ref(xt.float().cpu().numpy(), ids.cpu().numpy(), rw.cpu().numpy(), gu.reshape(E, 2 * f, -1),
                           dn.reshape(E, h, -1), fmt, h, f, act=ACT[act], b_gate=bg, b_up=bu, b_down=bd, dsc=dsc,
                           y0=y0 if accumulate else None, sg=sg if accumulate else None)
    assert O.rel_l2(out.cpu().numpy(), ref) <= TOL


def test_two_calls_and_the_f32_path(ops):
    # two calls in a row on new inputs; and the int8 layer stays within the quantisation error of the f32-activation
    # decode layer (ops.moe_ffn, MOE_Q8=0) on the same weights
    fmt, E, ku, h, f = "q4_0", 32, 8, 2048, 768
    gu, dn = experts(fmt, E, h, f, seed=3)
    wg, wd = torch.from_numpy(gu).cuda(), torch.from_numpy(dn).cuda()
    rng = np.random.default_rng(4)
    for _ in range(2):
        x = torch.from_numpy(rng.standard_normal((1, h)).astype(np.float32)).cuda().to(torch.bfloat16)
        lg = torch.from_numpy(rng.standard_normal((1, E)).astype(np.float32)).cuda()
        y = ops.moe_ffn_decode_q8(fmt, x, lg, wg, wd, h, f, E, ku)
        y32 = ops.moe_ffn(fmt, x, lg, wg, wd, h, f, E, ku, prefill=False)
        err = float((y - y32).norm() / y32.norm())
        assert err < 3e-2, err
    assert ops.device_status() == 0


@pytest.mark.parametrize("kw,code", [
    (dict(h=1024), -4),              # h not a multiple of 2048
    (dict(f=700), -4),               # f % 256
    (dict(h=8192), -5),              # h above 4096
    (dict(f=4352), -5),              # f above 4096
    (dict(tokens=5), -5),            # more than 4 tokens
    (dict(ku=9, E=16), -5),          # more than 8 experts per token
    (dict(fmt="iq4_nl"), -4),        # no int8 codes for IQ4_NL (gen_llm.py:5300-5301)
])
def test_limits(ops, kw, code):
    from loom_skills_b200 import _lib as L
    p = dict(fmt="q4_0", tokens=1, E=8, ku=2, h=2048, f=512)
    p.update(kw)
    x = torch.zeros(p["tokens"], p["h"], device="cuda")
    lg = torch.zeros(p["tokens"], p["E"], device="cuda")
    w = torch.zeros(64, dtype=torch.uint8, device="cuda")
    with pytest.raises(L.LkError):
        ops.moe_ffn_decode_q8(p["fmt"], x, lg, w, w, p["h"], p["f"], p["E"], p["ku"])
    rc = L.load().lk_moe_ffn_decode_q8(L.FMT_IDS[p["fmt"]], p["tokens"], p["h"], p["f"], p["E"], p["ku"], 1, 1, 1.0,
                                       lg.data_ptr(), None, None, x.data_ptr(), L.F32, w.data_ptr(), None,
                                       w.data_ptr(), None, None, None, 0, 1.702, 7.0, x.data_ptr(), None, None, None,
                                       0, x.data_ptr(), None)
    assert rc == code
