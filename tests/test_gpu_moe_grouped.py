"""GPU parity of the expert-grouped decode expert matvecs (g_moe_gu_{fmt} / g_moe_dn_{fmt} per assignment,
gen_moe.py:535-727, at several decode tokens), through the C ABI.

From 128 to 1024 assignments lk_moe_expert_mv_ex groups the assignments by expert inside the launch and reads each
16-row block of an expert once for up to 8 of them. Every assignment's row must equal, bit for bit, the per-assignment
form (the same call over slices of 8 assignments, which keep that form), and the layer built on them must match the
float64 oracle (relative L2 <= 1e-3).
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


@pytest.mark.parametrize("fmt,xdt,m,fused,act,biases", [
    ("q4_0", "bf16", 16, True, "silu", False),
    ("q4_k", "f32", 16, False, "gelu", True),
    ("iq4_nl", "f16", 64, True, "swiglu_oai", True),
    ("q4_k", "bf16", 128, True, "silu", False),
    ("q4_0", "f32", 17, False, "silu", True),   # 136 assignments: a partial round of 32 in the grouping
])
def test_grouped_equals_per_assignment(ops, fmt, xdt, m, fused, act, biases):
    E, ku, h, f = 32, 8, 1024, 512   # 32 experts: most experts serve several assignments
    rng = np.random.default_rng(11 + m)
    w = QUANT[fmt]((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32))
    wd = dev(QUANT[fmt]((rng.standard_normal((E * h, f)) * 0.02).astype(np.float32)))
    if fused:
        wg, wu = dev(w), None
    else:
        r = w.reshape(E, 2 * f, -1)
        wg = dev(np.ascontiguousarray(r[:, :f]).reshape(E * f, -1))
        wu = dev(np.ascontiguousarray(r[:, f:]).reshape(E * f, -1))
    x = dev(rng.standard_normal((m, h)).astype(np.float32)).to(XDT[xdt])
    ids = dev(np.stack([rng.permutation(E)[:ku] for _ in range(m)]).astype(np.int32).reshape(-1))
    bg = dev((rng.standard_normal((E, f)) * 0.05).astype(np.float32)) if biases else None
    bu = dev((rng.standard_normal((E, f)) * 0.05).astype(np.float32)) if biases else None
    bd = dev((rng.standard_normal((E, h)) * 0.05).astype(np.float32)) if biases else None
    ep = dict(fused=fused, w2=wu, act=act, bias=bg, bias2=bu)
    for _ in range(2):   # two calls in a row
        gu = ops.moe_expert_mv(fmt, "gu", ids, x, wg, f, h, ku, E, **ep)
        ref = torch.cat([ops.moe_expert_mv(fmt, "gu", ids[t * ku:(t + 1) * ku], x[t:t + 1], wg, f, h, ku, E, **ep)
                         for t in range(m)])
        assert torch.equal(gu, ref)
        dn = ops.moe_expert_mv(fmt, "dn", ids, gu, wd, h, f, ku, E, bias=bd)
        ref = torch.cat([ops.moe_expert_mv(fmt, "dn", ids[a:a + 8], gu[a:a + 8], wd, h, f, ku, E, bias=bd)
                         for a in range(0, m * ku, 8)])
        assert torch.equal(dn, ref)
    assert ops.device_status() == 0


@pytest.fixture(scope="module")
def layer_weights():
    E, h, f = 64, 1024, 512
    rng = np.random.default_rng(21)
    gu = O.quantize_q4_k((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32))
    dn = O.quantize_q4_k((rng.standard_normal((E * h, f)) * 0.02).astype(np.float32))
    return E, h, f, gu, dn


@pytest.mark.parametrize("m", [4, 32, 128])   # per-assignment form, grouped, grouped at the largest size
def test_layer_at_several_tokens_vs_oracle(ops, layer_weights, m):
    E, h, f, gu, dn = layer_weights
    ku = 8
    rng = np.random.default_rng(21 + m)
    x = rng.standard_normal((m, h)).astype(np.float32)
    lg = rng.standard_normal((m, E)).astype(np.float32)
    y = ops.moe_ffn("q4_k", dev(x), dev(lg), dev(gu), dev(dn), h, f, E, ku, prefill=False)
    ids, wts = O.route_ref(lg, ku)
    ref = O.moe_ffn_ref(x, ids, wts, gu.reshape(E, 2 * f, -1), dn.reshape(E, h, -1), "q4_k", h, f, E)
    assert O.rel_l2(y.cpu().numpy(), ref) < 1e-3
    assert ops.device_status() == 0


def test_one_expert_for_every_assignment(ops):
    """1024 assignments on one expert: 128 full groups of that expert."""
    E, ku, h, f, m = 4, 8, 512, 256, 128
    rng = np.random.default_rng(3)
    w = dev(O.quantize_q4_0((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32)))
    x = dev(rng.standard_normal((m, h)).astype(np.float32))
    ids = torch.full((m * ku,), 2, dtype=torch.int32, device="cuda")
    y = ops.moe_expert_mv("q4_0", "gu", ids, x, w, f, h, ku, E)
    ref = torch.cat([ops.moe_expert_mv("q4_0", "gu", ids[t * ku:(t + 1) * ku], x[t:t + 1], w, f, h, ku, E)
                     for t in range(m)])
    assert torch.equal(y, ref)
    assert ops.device_status() == 0
