"""GPU parity of the reference's remaining GGUF formats (formats.py:5-17: Q5_0, Q8_0, Q3_K, Q5_K, Q6_K, IQ4_XS, IQ3_S, and
ggml 17-byte MXFP4 on the decode path) and of rows that are not a multiple of 256 values (k % 32 only):

* lk_dequant against gguf 0.19.0's values bit for bit (tests/golden/golden_formats.npz) and the GEMM's f16 staging
  against the oracle bit for bit;
* the generic decode matvec (lk_mv, lk_moe_expert_mv) against gguf dequant + float64 products (golden) and the
  oracle, f32 / f16 / bf16 activations, 1 to 9 tokens, swiglu, accumulate, MoE assignments with the epilogue;
* the kbench moe_q4_0 down-projection decode cases (.github/devlab/kbench/moe_q4_0/gen_bench.py:169-173, F = 704) at
  the reference's own tolerances.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

TOL = 1e-3
FORMATS = ["q5_0", "q8_0", "q3_k", "q5_k", "q6_k", "iq4_xs", "iq3_s"]
SCALE_OFFS = {"q5_0": [0], "q8_0": [0], "q3_k": [108], "q5_k": [0, 2], "q6_k": [208], "iq4_xs": [0], "iq3_s": [0],
              "q4_0": [0], "iq4_nl": [0], "q4_k": [0, 2]}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from loom_skills_b200 import ops as _ops
    return _ops


@pytest.fixture(scope="module")
def gfmt():
    with np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_formats.npz")) as z:
        return {k: z[k] for k in z.files}


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def bits32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def blocks(fmt, rows, k, seed, lo=1e-3, hi=2e-2):
    """Random blocks of `fmt` with finite f16 scales of both signs at the format's scale offsets."""
    rng = np.random.default_rng(seed)
    nb = rows * k // O.QK[fmt]
    b = rng.integers(0, 256, (nb, O.BLOCK_BYTES[fmt]), dtype=np.uint8)
    for o in SCALE_OFFS[fmt]:
        b[:, o:o + 2] = (rng.uniform(lo, hi, nb) * rng.choice([-1, 1], nb)).astype(np.float16).view(np.uint8).reshape(-1, 2)
    return b.reshape(rows, -1)


@pytest.mark.parametrize("fmt", FORMATS)
def test_dequant_golden_bit_exact(ops, gfmt, fmt):
    raw = gfmt[f"{fmt}_raw"]
    out = ops.dequant(fmt, dev(raw.reshape(-1)), gfmt[f"{fmt}_f32"].size)
    assert np.array_equal(bits32(host(out)), bits32(gfmt[f"{fmt}_f32"].reshape(-1)))
    st = host(ops.dequant(fmt, dev(raw.reshape(-1)), gfmt[f"{fmt}_f32"].size, torch.float16)).view(np.uint16)
    assert np.array_equal(st, O.dequant_f16(fmt, raw.reshape(-1), gfmt[f"{fmt}_f32"].size).view(np.uint16))


@pytest.mark.parametrize("fmt", FORMATS)
def test_mv_golden(ops, gfmt, fmt):
    w, x = gfmt[f"mv_{fmt}_w"], gfmt[f"mv_{fmt}_x"]
    y = host(ops.mv(fmt, dev(w), dev(x), w.shape[0], 512))
    assert O.rel_l2(y, gfmt[f"mv_{fmt}_y"]) < 1e-6   # f32 values x f32 activations, f32 sums


@pytest.mark.parametrize("fmt", FORMATS + ["mxfp4"])
@pytest.mark.parametrize("xdt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("tokens", [1, 9])
def test_mv_vs_oracle(ops, fmt, xdt, tokens):
    n, k = 200, 2048
    if fmt == "mxfp4":
        w = O.quantize_mxfp4((np.random.default_rng(3).standard_normal((n, k)) * 0.02).astype(np.float32), "ggml")
    else:
        w = blocks(fmt, n, k, 3)
    x = np.random.default_rng(4).standard_normal((tokens, k)).astype(np.float32)
    xt = dev(x).to({"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[xdt])
    y = host(ops.mv(fmt, dev(w), xt, n, k))
    ref = O.mv_ref(fmt, w, xt.float().cpu().numpy(), n, k)
    assert O.rel_l2(y, ref) < 1e-5, O.rel_l2(y, ref)


@pytest.mark.parametrize("fmt", ["q6_k", "q8_0", "q4_0"])
def test_mv_swiglu_accumulate_odd_k(ops, fmt):
    # k = 704 (22 blocks of 32 for the 32-value formats; Q6_K: 768, three super-blocks)
    n, k = 96, 768 if fmt == "q6_k" else 704
    w, w2 = blocks(fmt, n, k, 5), blocks(fmt, n, k, 6)
    x = np.random.default_rng(7).standard_normal((3, k)).astype(np.float32)
    y0 = np.random.default_rng(8).standard_normal((3, n)).astype(np.float32)
    yt = dev(y0)
    ops.mv(fmt, dev(w), dev(x), n, k, w2=dev(w2), y=yt, accumulate=True)
    assert O.rel_l2(host(yt), O.mv_ref(fmt, w, x, n, k, w2=w2, y_old=y0)) < 1e-5


@pytest.mark.parametrize("fmt", ["q6_k", "q5_k", "iq4_xs", "q8_0"])
def test_expert_mv_with_epilogue(ops, fmt):
    E, ku, H, F = 8, 2, 512, 256
    rng = np.random.default_rng(11)
    w_gu = np.stack([blocks(fmt, 2 * F, H, 100 + e) for e in range(E)])
    w_dn = np.stack([blocks(fmt, H, F, 200 + e) for e in range(E)])
    x = rng.standard_normal((3, H)).astype(np.float32)
    ids = rng.integers(0, E, (3, ku)).astype(np.int32)
    bg, bu = (rng.standard_normal((E, F)) * 0.05).astype(np.float32), (rng.standard_normal((E, F)) * 0.05).astype(np.float32)
    bd = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
    act = ops.moe_expert_mv(fmt, "gu", dev(ids.reshape(-1)), dev(x), dev(w_gu), F, H, ku, E, act="swiglu_oai",
                            bias=dev(bg), bias2=dev(bu))
    ys = host(ops.moe_expert_mv(fmt, "dn", dev(ids.reshape(-1)), act, dev(w_dn), H, F, ku, E, bias=dev(bd)))
    act_h = host(act)
    for a, e in enumerate(ids.reshape(-1)):
        W = O.dequant(fmt, w_gu[e], H).reshape(2 * F, H).astype(np.float64)
        pr = W @ x[a // ku].astype(np.float64)
        ref = O.act_ref(pr[:F] + bg[e], pr[F:] + bu[e], O.ACT_SWIGLU_OAI)
        assert O.rel_l2(act_h[a], ref) < TOL
        D = O.dequant(fmt, w_dn[e], F).reshape(H, F).astype(np.float64)
        assert O.rel_l2(ys[a], D @ act_h[a].astype(np.float64) + bd[e]) < 1e-5


@pytest.fixture(scope="module")
def gmoe():
    with np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_moe.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("t", [1, 4])
def test_kbench_decode_down(ops, gmoe, t):
    # gen_bench.py:169-173: the down expert matvecs over F = 704 (22 Q4_0 blocks per row)
    kb = O.kbench_moe_inputs(490)
    H, F, E, U = O.KB_H, O.KB_F, O.KB_E, O.KB_U
    ys = ops.moe_expert_mv("q4_0", "dn", dev(kb[f"decode_t{t}_ids"].reshape(-1)), dev(kb[f"decode_t{t}_xdn"]),
                           dev(kb["wd"]), H, F, U, E)
    np.testing.assert_allclose(host(ys)[:, gmoe["kb_cols_h"]], gmoe[f"kb_decode_dn_t{t}"], atol=2e-5, rtol=2e-4)


# ---------------------------------------------------------------------------------------------------------- GEMM
def row_scaled(rows, k, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((rows, k)) * rng.choice([1.0, 3e4], (rows, 1))).astype(np.float32)
    return O.row_scale_f16(x)


@pytest.mark.parametrize("fmt", FORMATS + ["mxfp4", "q4_0", "iq4_nl"])
@pytest.mark.parametrize("rows,n,k", [(200, 272, 1024), (64, 512, 2048), (300, 192, 1536)])
def test_gemm_store(ops, fmt, rows, n, k):
    # the window form of the tcgen05 GEMM (Q4_0 / IQ4_NL take it when k is not a multiple of 256: 1536 is)
    if fmt == "mxfp4":
        w = O.quantize_mxfp4((np.random.default_rng(41).standard_normal((n, k)) * 0.02).astype(np.float32), "ggml")
    else:
        w = blocks(fmt, n, k, 41)
    x16, sc = row_scaled(rows, k, 42)
    y = host(ops.gemm(fmt, "store", dev(x16), dev(sc), dev(w), n))
    W16 = O.dequant_f16(fmt, w, k).astype(np.float64).reshape(n, k)
    ref16 = (x16.astype(np.float64) @ W16.T) * sc[:, 1:2]
    assert O.rel_l2(y, ref16) < 1e-5, O.rel_l2(y, ref16)          # the reference's staged weights, f32 sums
    assert O.rel_l2(y, O.gemm_ref(fmt, w, x16, sc, n, k)) < TOL
    assert ops.device_status() == 0


@pytest.mark.parametrize("fmt", ["q6_k", "q8_0", "q3_k"])
def test_gemm_swiglu_acc(ops, fmt):
    rows, n, k = 256, 320, 1024
    w, w2 = blocks(fmt, n, k, 51), blocks(fmt, n, k, 52)
    x16, sc = row_scaled(rows, k, 53)
    ys = host(ops.gemm(fmt, "swiglu", dev(x16), dev(sc), dev(w), n, w2=dev(w2)))
    assert O.rel_l2(ys, O.gemm_ref(fmt, w, x16, sc, n, k, mode="swiglu", w2=w2)) < TOL
    y0 = np.random.default_rng(54).standard_normal((rows, n)).astype(np.float32)
    ya = dev(y0)
    ops.gemm(fmt, "acc", dev(x16), dev(sc), dev(w), n, y=ya)
    assert O.rel_l2(host(ya), O.gemm_ref(fmt, w, x16, sc, n, k, mode="acc", y_old=y0)) < TOL


@pytest.mark.parametrize("fmt", ["q6_k", "q5_k"])
def test_grouped_gemms(ops, fmt):
    E, ku, H, F, tokens = 8, 4, 512, 256, 70
    rng = np.random.default_rng(60)
    w_gu = np.stack([blocks(fmt, 2 * F, H, 600 + e) for e in range(E)])
    w_dn = np.stack([blocks(fmt, H, F, 700 + e) for e in range(E)])
    x = rng.standard_normal((tokens, H)).astype(np.float32)
    lg = rng.standard_normal((tokens, E)).astype(np.float32)
    y = host(ops.moe_ffn(fmt, dev(x), dev(lg), dev(w_gu), dev(w_dn), H, F, E, ku, prefill=True))
    ids, wts = O.route_ref(lg, ku)
    ref = O.moe_ffn_ref(x, ids, wts, w_gu, w_dn, fmt, H, F, E)
    assert O.rel_l2(y, ref) < TOL, O.rel_l2(y, ref)


@pytest.mark.parametrize("t", [63, 65])
def test_kbench_grouped_down(ops, gmoe, t):
    # gen_bench.py:227-236: the grouped down GEMM over F = 704 (22 Q4_0 blocks a row), tile_info [[7,64],[0,17],
    # [3,1],[-1,0]], sorted rows (padding rows zero), row scales in {0.5, 1, 2}, sentinel 42
    kb = O.kbench_moe_inputs(490)
    H, F, E, U = O.KB_H, O.KB_F, O.KB_E, O.KB_U
    ti = dev(np.array(O.KB_TILE_INFO, np.int32))
    rm = dev(kb[f"grouped_t{t}_rm"])
    y = torch.full((256, H), O.KB_SENTINEL, dtype=torch.float32, device="cuda")
    ops.moe_grouped_gemm("q4_0", "store", ti, rm, dev(kb[f"grouped_t{t}_xd"]), dev(kb[f"grouped_t{t}_sd"]),
                         dev(kb["wd"]), H, U, E, y=y)
    yh = host(y)
    assert (yh[192:] == O.KB_SENTINEL).all()
    np.testing.assert_allclose(yh[:, gmoe["kb_cols_h"]], gmoe[f"kb_grouped_dn_t{t}"], atol=2e-5, rtol=2e-4)


@pytest.mark.parametrize("fmt", ["q6_k", "q5_0"])
def test_gemm_split_k_window_deterministic(ops, fmt):
    # few rows and narrow n on the window producer: K split into ranges that meet in y in a fixed order; against the
    # f64 product and bit for bit from run to run
    rows, n, k = 48, 512, 4096
    w = blocks(fmt, n, k, 91)
    x16, sc = row_scaled(rows, k, 92)
    wd, xd, sd = dev(w), dev(x16), dev(sc)
    y = ops.gemm(fmt, "store", xd, sd, wd, n)
    W16 = O.dequant_f16(fmt, w, k).astype(np.float64).reshape(n, k)
    ref16 = (x16.astype(np.float64) @ W16.T) * sc[:, 1:2]
    assert O.rel_l2(host(y), ref16) < 1e-5, O.rel_l2(host(y), ref16)
    for _ in range(3):
        assert torch.equal(ops.gemm(fmt, "store", xd, sd, wd, n), y)
    assert ops.device_status() == 0
