"""GPU parity of lk_moe_gate_up_routed, the router folded into the gate/up expert matvecs of one decode token
(g_moe_route + g_moe_gu_{fmt}, gen_moe.py:116-253, 535-727), through the C ABI.

The launch routes with the router's own code and runs the same persistent expert matvec as the two-launch form, so
its ids and weights equal lk_moe_route's and its activations equal lk_moe_expert_mv_ex's, bit for bit; the layer it
feeds (ops.moe_ffn at one token) is also checked against the float64 oracle (relative L2 <= 1e-3).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

QUANT = {"q4_0": O.quantize_q4_0, "q4_k": O.quantize_q4_k, "iq4_nl": O.quantize_iq4_nl}
XDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from loom_skills_b200 import ops as _ops
    return _ops


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("fmt,xdt,gating,norm,fused,act,biases", [
    ("q4_0", "bf16", 1, True, True, "silu", False),
    ("q4_k", "f32", 2, False, False, "gelu", True),
    ("iq4_nl", "f16", 3, False, True, "swiglu_oai", True),
    ("q4_k", "bf16", 1, False, True, "silu", False),
])
def test_routed_equals_router_then_expert_matvecs(ops, fmt, xdt, gating, norm, fused, act, biases):
    E, ku, h, f = 32, 8, 1024, 512
    rng = np.random.default_rng(5 + gating)
    w = QUANT[fmt]((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32))
    if fused:
        wg, wu = dev(w), None
    else:
        r = w.reshape(E, 2 * f, -1)
        wg = dev(np.ascontiguousarray(r[:, :f]).reshape(E * f, -1))
        wu = dev(np.ascontiguousarray(r[:, f:]).reshape(E * f, -1))
    x = dev(rng.standard_normal((1, h)).astype(np.float32)).to(XDT[xdt])
    lg = dev(rng.standard_normal((1, E)).astype(np.float32))
    rb = dev((rng.standard_normal(E) * 0.5).astype(np.float32)) if gating != 1 else None
    bg = dev((rng.standard_normal((E, f)) * 0.05).astype(np.float32)) if biases else None
    bu = dev((rng.standard_normal((E, f)) * 0.05).astype(np.float32)) if biases else None
    scale = 1.5 if gating == 2 else 1.0
    for _ in range(2):   # two calls in a row
        ids, wts, y = ops.moe_gate_up_routed(fmt, x, lg, wg, f, E, ku, fused=fused, w2=wu, gating=gating, norm=norm,
                                             scale=scale, router_bias=rb, act=act, bias=bg, bias2=bu)
        rid, rw = ops.moe_route(lg, E, ku, gating=gating, norm=norm, scale=scale, bias=rb)
        ref = ops.moe_expert_mv(fmt, "gu", rid.reshape(-1), x, wg, f, h, ku, E, fused=fused, w2=wu, act=act, bias=bg,
                                bias2=bu)
        assert torch.equal(ids, rid) and torch.equal(wts, rw)
        assert torch.equal(y, ref)
    assert ops.device_status() == 0


def test_layer_at_one_token_vs_oracle(ops):
    E, ku, h, f = 128, 8, 2048, 768
    rng = np.random.default_rng(9)
    gu = O.quantize_q4_0((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32))
    dn = O.quantize_q4_0((rng.standard_normal((E * h, f)) * 0.02).astype(np.float32))
    x = rng.standard_normal((1, h)).astype(np.float32)
    lg = rng.standard_normal((1, E)).astype(np.float32)
    dsc = rng.uniform(0.5, 1.5, E).astype(np.float32)
    y = ops.moe_ffn("q4_0", dev(x), dev(lg), dev(gu), dev(dn), h, f, E, ku, prefill=False, down_scale=dev(dsc))
    ids, wts = O.route_ref(lg, ku)
    ref = O.moe_ffn_ref(x, ids, wts, gu.reshape(E, 2 * f, -1), dn.reshape(E, h, -1), "q4_0", h, f, E, dsc=dsc)
    assert O.rel_l2(y.cpu().numpy(), ref) < 1e-3


def test_refusals(ops):
    from loom_skills_b200 import _lib as L
    x = torch.zeros(1, 256, device="cuda")
    lg = torch.zeros(1, 16, device="cuda")
    w = torch.zeros(16 * 2 * 64, 144, dtype=torch.uint8, device="cuda")
    with pytest.raises(L.LkError):   # the tuned Q4 layout only
        ops.moe_gate_up_routed("q6_k", x, lg, w, 64, 16, 4)
    with pytest.raises(L.LkError):   # at most 8 experts per token
        ops.moe_gate_up_routed("q4_k", x, lg, w, 64, 16, 9)
