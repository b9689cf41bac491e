"""GPU parity of gate and up weights in two formats -- the reference's "GATE+UP" kernels (gen_moe.py:537-552
expert_mv, :1129-1141 grouped_gemm; gen_gemm.py:535-545 and :1224-1251 gemm fmt2) and its dense fallback of two
projections + g_silu_mul (gen_llm.py:77, 6280-6283, 5717-5745) -- through the C ABI with LK_FMT_PAIR ids:

* lk_mv with a pair (one token: the row-streaming kernel; several: the general one) against the float64 oracle with
  each weight dequantised in its own format, and against two single-format projections + lk_silu_mul;
* lk_moe_expert_mv gate/up with a pair and the expert epilogue (biases, swiglu_oai);
* lk_gemm swiglu with a pair: the reference's f16 staging of each weight (bit for bit the oracle's dequant_f16) times
  the row-scaled activations, f32 sums, and the float64 oracle at the GEMM tolerance; a Q4_K gate at a 2-byte (not
  16-byte) aligned address;
* the grouped GEMMs (gathered and sorted gate/up rows) and the whole MoE layer, decode and prefill, with a Q4_K gate,
  a Q6_K up and a Q5_K down (Q4_K_M's mix).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

TOL = 1e-3
SCALE_OFFS = {"q5_0": [0], "q8_0": [0], "q3_k": [108], "q5_k": [0, 2], "q6_k": [208], "iq4_xs": [0], "iq3_s": [0],
              "q4_0": [0], "iq4_nl": [0], "q4_k": [0, 2]}


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


def blocks(fmt, rows, k, seed, lo=1e-3, hi=2e-2):
    """Random blocks of `fmt` with finite f16 scales of both signs at the format's scale offsets."""
    rng = np.random.default_rng(seed)
    nb = rows * k // O.QK[fmt]
    b = rng.integers(0, 256, (nb, O.BLOCK_BYTES[fmt]), dtype=np.uint8)
    for o in SCALE_OFFS[fmt]:
        b[:, o:o + 2] = (rng.uniform(lo, hi, nb) * rng.choice([-1, 1], nb)).astype(np.float16).view(np.uint8).reshape(-1, 2)
    return b.reshape(rows, -1)


PAIRS = [("q4_k", "q6_k"), ("q6_k", "q4_k"), ("q4_0", "q8_0"), ("iq4_xs", "q5_k"), ("q5_0", "iq4_nl"),
         ("q3_k", "q4_0"), ("iq3_s", "q4_k")]


@pytest.mark.parametrize("fg,fu", PAIRS)
@pytest.mark.parametrize("tokens,xdt", [(1, "bf16"), (1, "f32"), (3, "f32"), (9, "f16")])
def test_mv_pair(ops, fg, fu, tokens, xdt):
    n, k = 200, 2048
    w, w2 = blocks(fg, n, k, 1), blocks(fu, n, k, 2)
    x = np.random.default_rng(3).standard_normal((tokens, k)).astype(np.float32)
    xt = dev(x).to({"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[xdt])
    y = host(ops.mv(f"{fg}+{fu}", dev(w), xt, n, k, w2=dev(w2)))
    ref = O.mv_ref(fg, w, xt.float().cpu().numpy(), n, k, w2=w2, fmt2=fu)
    assert O.rel_l2(y, ref) < 1e-5, O.rel_l2(y, ref)
    assert ops.device_status() == 0


@pytest.mark.parametrize("fg,fu,k", [("q4_0", "q8_0", 704), ("q4_k", "q6_k", 768)])
def test_mv_pair_is_two_projections_and_silu_mul(ops, fg, fu, k):
    # the pair kernel against the reference's dense fallback: gate and up projections, then g_silu_mul; and accumulate.
    # A Q4_K projection alone runs the tuned kernel, which sums in another order: agreement to f32 rounding
    n = 96
    w, w2 = dev(blocks(fg, n, k, 5)), dev(blocks(fu, n, k, 6))
    x = dev(np.random.default_rng(7).standard_normal((2, k)).astype(np.float32))
    g, u = ops.mv(fg, w, x, n, k), ops.mv(fu, w2, x, n, k)
    two = host(ops.silu_mul(g, u))
    one = host(ops.mv(f"{fg}+{fu}", w, x, n, k, w2=w2))
    assert O.rel_l2(one, two) < 1e-6
    np.testing.assert_allclose(one, two, rtol=1e-4, atol=1e-4)
    y0 = np.random.default_rng(8).standard_normal((2, n)).astype(np.float32)
    ya = dev(y0)
    ops.mv(f"{fg}+{fu}", w, x, n, k, w2=w2, y=ya, accumulate=True)
    np.testing.assert_allclose(host(ya), y0 + one, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("act", ["silu", "gelu"])
def test_silu_mul(ops, act):
    rng = np.random.default_rng(9)
    f, u = rng.standard_normal((3, 1000)).astype(np.float32) * 4, rng.standard_normal((3, 1000)).astype(np.float32)
    out = host(ops.silu_mul(dev(f), dev(u), act=act))
    ref = O.act_ref(f.astype(np.float64), u.astype(np.float64), O.ACT_SILU if act == "silu" else O.ACT_GELU)
    np.testing.assert_allclose(out, ref, rtol=2e-6, atol=1e-6)


def test_expert_mv_pair_with_epilogue(ops):
    fg, fu, E, ku, H, F = "q4_k", "q6_k", 8, 2, 512, 256
    rng = np.random.default_rng(11)
    wg = np.stack([blocks(fg, F, H, 100 + e) for e in range(E)])
    wu = np.stack([blocks(fu, F, H, 200 + e) for e in range(E)])
    x = rng.standard_normal((3, H)).astype(np.float32)
    ids = rng.integers(0, E, (3, ku)).astype(np.int32)
    bg, bu = (rng.standard_normal((E, F)) * 0.05).astype(np.float32), (rng.standard_normal((E, F)) * 0.05).astype(np.float32)
    act = host(ops.moe_expert_mv(f"{fg}+{fu}", "gu", dev(ids.reshape(-1)), dev(x), dev(wg), F, H, ku, E, fused=False,
                                 w2=dev(wu), act="swiglu_oai", bias=dev(bg), bias2=dev(bu)))
    for a, e in enumerate(ids.reshape(-1)):
        g = O.dequant(fg, wg[e], H).reshape(F, H).astype(np.float64) @ x[a // ku].astype(np.float64)
        u = O.dequant(fu, wu[e], H).reshape(F, H).astype(np.float64) @ x[a // ku].astype(np.float64)
        assert O.rel_l2(act[a], O.act_ref(g + bg[e], u + bu[e], O.ACT_SWIGLU_OAI)) < TOL
    assert ops.device_status() == 0


def row_scaled(rows, k, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((rows, k)) * rng.choice([1.0, 3e4], (rows, 1))).astype(np.float32)
    return O.row_scale_f16(x)


def staged_swiglu(fg, fu, w, w2, x16, sc, n, k):
    """silu(G) * U with the reference's f16 staging of each weight, float64 sums."""
    xs = x16.astype(np.float64)
    g = (xs @ O.dequant_f16(fg, w, k).astype(np.float64).reshape(n, k).T) * sc[:, 1:2]
    u = (xs @ O.dequant_f16(fu, w2, k).astype(np.float64).reshape(n, k).T) * sc[:, 1:2]
    return O.silu(g) * u


@pytest.mark.parametrize("fg,fu", [("q4_k", "q6_k"), ("q6_k", "q4_k"), ("q4_0", "q5_k"), ("q8_0", "iq4_xs"),
                                   ("q3_k", "q5_0"), ("q5_k", "iq3_s")])
@pytest.mark.parametrize("rows,n,k", [(200, 272, 1024), (64, 128, 2048)])
def test_gemm_pair(ops, fg, fu, rows, n, k):
    w, w2 = blocks(fg, n, k, 41), blocks(fu, n, k, 42)
    x16, sc = row_scaled(rows, k, 43)
    y = host(ops.gemm(f"{fg}+{fu}", "swiglu", dev(x16), dev(sc), dev(w), n, w2=dev(w2)))
    assert O.rel_l2(y, staged_swiglu(fg, fu, w, w2, x16, sc, n, k)) < 1e-5
    assert O.rel_l2(y, O.gemm_ref(fg, w, x16, sc, n, k, mode="swiglu", w2=w2, fmt2=fu)) < TOL
    assert ops.device_status() == 0


def test_gemm_pair_q4k_at_two_byte_alignment(ops):
    # a Q4_K gate outside the TMA box form's 16-byte alignment: the one-kernel pair form (window copies of any 2-byte
    # aligned rows) rather than the two passes
    fg, fu, rows, n, k = "q4_k", "q8_0", 130, 144, 512
    w, w2 = blocks(fg, n, k, 51), blocks(fu, n, k, 52)
    buf = torch.zeros(w.size + 16, dtype=torch.uint8, device="cuda")
    buf[2:2 + w.size] = dev(w.reshape(-1))
    wv = buf[2:2 + w.size]
    assert wv.data_ptr() % 16 == 2
    x16, sc = row_scaled(rows, k, 53)
    y = host(ops.gemm(f"{fg}+{fu}", "swiglu", dev(x16), dev(sc), wv, n, w2=dev(w2)))
    assert O.rel_l2(y, staged_swiglu(fg, fu, w, w2, x16, sc, n, k)) < 1e-5


def moe_weights(E, H, F, fg, fu, fd, seed):
    wg = np.stack([blocks(fg, F, H, seed + e) for e in range(E)])
    wu = np.stack([blocks(fu, F, H, seed + 100 + e) for e in range(E)])
    wd = np.stack([blocks(fd, H, F, seed + 200 + e) for e in range(E)])
    return wg, wu, wd


def test_grouped_pair_gathered_equals_sorted(ops):
    # the gathered form (token rows by rowmap: the pair kernel) and the sorted form (moe_row_scale_gather's rows: two
    # single-format passes, the activation in the second's epilogue) agree on every live row, and match the oracle
    fg, fu, E, ku, H, F, tokens = "q4_k", "q6_k", 8, 4, 512, 256, 70
    rng = np.random.default_rng(60)
    wg, wu, _ = moe_weights(E, H, F, fg, fu, "q5_k", 600)
    x = rng.standard_normal((tokens, H)).astype(np.float32)
    ids = dev(rng.integers(0, E, (tokens, ku)).astype(np.int32))
    ti, rm, pos = ops.moe_bucket(ids, E)
    x16, sc = ops.row_scale_f16(dev(x))
    pf = f"{fg}+{fu}"
    yg = ops.moe_grouped_gemm(pf, "swiglu", ti, rm, x16, sc, dev(wg), F, ku, E, w2=dev(wu))
    s16, ssc = ops.moe_row_scale_gather(dev(x), rm, ku)
    ys = ops.moe_grouped_gemm(pf, "swiglu_sorted", ti, rm, s16, ssc, dev(wg), F, ku, E, w2=dev(wu))
    live = host(rm) >= 0
    assert O.rel_l2(host(yg)[live], host(ys)[live]) < 1e-6
    rmh, tih, x16h, sch = host(rm), host(ti), host(x16), host(sc)
    ref = np.zeros((live.sum(), F))
    out = host(ys)[live]
    j = 0
    for r in np.nonzero(live)[0]:
        e, t = tih[r // 64, 0], rmh[r] // ku
        ref[j] = staged_swiglu(fg, fu, wg[e], wu[e], x16h[t:t + 1], sch[t:t + 1], F, H)[0]
        j += 1
    assert O.rel_l2(out, ref) < 1e-5
    assert ops.device_status() == 0


@pytest.mark.parametrize("tokens,prefill", [(3, False), (70, True)])
def test_moe_layer_q4_k_m_mix(ops, tokens, prefill):
    # Q4_K_M's expert mix: Q4_K gate, Q6_K up, Q5_K down (fmt "gate+up", fmt_down), decode and prefill paths
    E, ku, H, F = 8, 4, 512, 256
    rng = np.random.default_rng(70 + tokens)
    wg, wu, wd = moe_weights(E, H, F, "q4_k", "q6_k", "q5_k", 700)
    x = rng.standard_normal((tokens, H)).astype(np.float32)
    lg = rng.standard_normal((tokens, E)).astype(np.float32)
    y = host(ops.moe_ffn("q4_k+q6_k", dev(x), dev(lg), dev(wg), dev(wd), H, F, E, ku, prefill=prefill, w_up=dev(wu),
                         fmt_down="q5_k"))
    ids, wts = O.route_ref(lg, ku)
    ref = O.moe_ffn_ref(x, ids, wts, wg, wd, "q4_k", H, F, E, w_up=wu, fmt_up="q6_k", fmt_down="q5_k")
    assert O.rel_l2(y, ref) < TOL, O.rel_l2(y, ref)
    assert ops.device_status() == 0
