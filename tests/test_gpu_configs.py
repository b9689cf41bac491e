"""Parity at BASELINE.json's own config shapes: each config runs on the GPU at its full size and a row / column / token
subsample of the result is checked against the float64 oracle (the reference's numpy path), so every shape the bench
times is also a checked shape. Weights are seeded synthetic blocks (random f16 scales of the N(0, 0.02) weight size,
random codes); the values do not matter to the kernels' paths, only the layouts and shapes do.

  configs[0]  Q4_0 4096 x 4096 GEMV, M = 1, fp16 activations (f32 decode path) and the int8 path
  configs[1]  Q4_K decode at M = 1 / 8 over the Qwen3-8B-like shapes; prefill GEMMs at M = 64 / 2048
  configs[2]  Q4_0 MoE, 128 experts, top-8, H 2048, F 768, M = 1 / 16 / 256 / 4096
  configs[3]  MXFP4 x FP8 MoE, 32 experts, top-4, H = F = 2880, M = 1 / 32 / 1024 / 8192
  configs[4]  IQ4_NL GEMMs K 5120 / N 27648 and K 27648 / N 5120 at M = 4096
"""
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


def blocks32(rng, rows, k):
    """Random 18-byte blocks (Q4_0 / IQ4_NL): f16 scales +-[5e-4, 3e-3] of both signs, uniform code bytes."""
    nb = rows * k // 32
    raw = rng.integers(0, 256, (nb, 18), dtype=np.uint8)
    sc = (rng.uniform(5e-4, 3e-3, nb) * rng.choice([-1, 1], nb)).astype("<f2")
    raw[:, :2] = sc.view(np.uint8).reshape(-1, 2)
    return raw.reshape(rows, -1)


def blocks_q4k(rng, rows, k):
    """Random Q4_K super-blocks: d, dmin f16 of the N(0, 0.02) weight size, uniform scale bytes and nibbles."""
    nb = rows * k // 256
    raw = rng.integers(0, 256, (nb, 144), dtype=np.uint8)
    d = rng.uniform(2e-5, 1e-4, (nb, 2)).astype("<f2")
    raw[:, :4] = d.view(np.uint8).reshape(-1, 4)
    return raw.reshape(rows, -1)


def mxfp4_planes(rng, rows, k):
    nib = rng.integers(0, 256, (rows, k // 2), dtype=np.uint8)
    sc = rng.integers(117, 123, (rows, k // 32), dtype=np.uint8)
    return nib, sc


# ---------------------------------------------------------------------------------------------------------- configs[0]
def test_config0_q4_0_gemv_fp16(ops):
    rng = np.random.default_rng(100)
    n = k = 4096
    w = blocks32(rng, n, k)
    x = rng.standard_normal((1, k)).astype(np.float32).astype(np.float16)
    y = host(ops.mv("q4_0", dev(w), dev(x), n, k))
    ref = O.mv_ref("q4_0", w, x.astype(np.float32), n, k)
    assert O.rel_l2(y, ref) < TOL, O.rel_l2(y, ref)
    # the int8-activation path on the same weights (Q4_0 codes are opt-in int8 in the reference, formats.py:24-27)
    xq = ops.quant_q8(dev(x.astype(np.float32)))
    codes, meta = O.quant_q8(x.astype(np.float32))
    y8 = host(ops.mv_q8("q4_0", dev(w), xq, n, k, 1))
    ref8 = O.mv_ref("q4_0", w, O.dequant_q8(codes, meta), n, k)
    assert O.rel_l2(y8, ref8) < TOL, O.rel_l2(y8, ref8)


# ---------------------------------------------------------------------------------------------------------- configs[1]
SHAPES1 = [(4096, 4096), (4096, 1024), (4096, 24576), (12288, 4096)]   # (K, N)


@pytest.mark.parametrize("k,n", SHAPES1)
@pytest.mark.parametrize("m", [1, 8])
def test_config1_q4_k_decode(ops, k, n, m):
    rng = np.random.default_rng(k + n + m)
    w = blocks_q4k(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    xt = dev(x).to(torch.bfloat16)
    xb = xt.float().cpu().numpy()
    rows = np.sort(rng.choice(n, min(n, 512), replace=False))
    # the bench's int8 path (quantise + integer dot) and the bf16-activation path, full n, checked on 512 rows
    xq = ops.quant_q8(xt)
    codes, meta = O.quant_q8(xb)
    assert np.array_equal(host(xq)[:m * k].view(np.int8).reshape(m, k), codes)
    y8 = host(ops.mv_q8("q4_k", dev(w), xq, n, k, m))
    ref8 = O.mv_ref("q4_k", w[rows], O.dequant_q8(codes, meta), len(rows), k)
    assert O.rel_l2(y8[:, rows], ref8) < TOL, O.rel_l2(y8[:, rows], ref8)
    y = host(ops.mv("q4_k", dev(w), xt, n, k))
    ref = O.mv_ref("q4_k", w[rows], xb, len(rows), k)
    assert O.rel_l2(y[:, rows], ref) < TOL, O.rel_l2(y[:, rows], ref)


@pytest.mark.parametrize("k,n", SHAPES1)
@pytest.mark.parametrize("m", [64, 2048])
def test_config1_q4_k_prefill(ops, k, n, m):
    rng = np.random.default_rng(7 * k + n + m)
    w = blocks_q4k(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x16, sc = ops.row_scale_f16(dev(x).to(torch.bfloat16))
    y = host(ops.gemm("q4_k", "store", x16, sc, dev(w), n))
    rows = np.sort(rng.choice(m, min(m, 256), replace=False))
    cols = np.sort(rng.choice(n, 512, replace=False))
    ref = O.gemm_ref("q4_k", w[cols], host(x16)[rows], host(sc)[rows], len(cols), k)
    assert O.rel_l2(y[np.ix_(rows, cols)], ref) < TOL, O.rel_l2(y[np.ix_(rows, cols)], ref)
    assert ops.device_status() == 0


# ---------------------------------------------------------------------------------------------------------- configs[2]
@pytest.fixture(scope="module")
def moe2():
    rng = np.random.default_rng(2)
    E, H, F = 128, 2048, 768
    w_gu = blocks32(rng, E * 2 * F, H).reshape(E, 2 * F, -1)
    w_dn = blocks32(rng, E * H, F).reshape(E, H, -1)
    return w_gu, w_dn


@pytest.mark.parametrize("m", [1, 16, 256, 4096])
def test_config2_q4_0_moe(ops, moe2, m):
    E, KU, H, F = 128, 8, 2048, 768
    w_gu, w_dn = moe2
    rng = np.random.default_rng(20 + m)
    x = torch.from_numpy(rng.standard_normal((m, H)).astype(np.float32)).to(torch.bfloat16)
    lg = rng.standard_normal((m, E)).astype(np.float32)
    y = host(ops.moe_ffn("q4_0", x.cuda(), dev(lg), dev(w_gu), dev(w_dn), H, F, E, KU))
    toks = np.sort(rng.choice(m, min(m, 6), replace=False))
    ids, wts = O.route_ref(lg[toks], KU)
    ref = O.moe_ffn_ref(x.float().numpy()[toks], ids, wts, w_gu, w_dn, "q4_0", H, F, E)
    assert O.rel_l2(y[toks], ref) < TOL, O.rel_l2(y[toks], ref)
    assert ops.device_status() == 0


# ---------------------------------------------------------------------------------------------------------- configs[3]
@pytest.fixture(scope="module")
def moe3():
    rng = np.random.default_rng(3)
    E, H, F = 32, 2880, 2880
    gu = mxfp4_planes(rng, E * 2 * F, H)
    dn = mxfp4_planes(rng, E * H, F)
    return gu, dn


@pytest.mark.parametrize("m", [1, 32, 1024, 8192])
def test_config3_mxfp4_moe(ops, moe3, m):
    E, KU, H, F = 32, 4, 2880, 2880
    (nib_gu, sc_gu), (nib_dn, sc_dn) = moe3
    rng = np.random.default_rng(30 + m)
    x = rng.standard_normal((m, H)).astype(np.float32)
    lg = rng.standard_normal((m, E)).astype(np.float32)
    y = host(ops.moe_ffn_mxfp4s(dev(x), dev(lg), dev(nib_gu), dev(sc_gu), dev(nib_dn), dev(sc_dn), H, F, E, KU))
    toks = np.sort(rng.choice(m, min(m, 2), replace=False))
    ids, wts = O.route_ref(lg[toks], KU)
    used = np.unique(ids)
    # the oracle on the touched experts only (their rows of the stacked planes)
    gsel = np.concatenate([np.arange(e * 2 * F, (e + 1) * 2 * F) for e in used])
    dsel = np.concatenate([np.arange(e * H, (e + 1) * H) for e in used])
    remap = {int(e): i for i, e in enumerate(used)}
    lids = np.vectorize(remap.get)(ids)
    if m * KU <= 16:   # expert matvecs on the unquantised activations
        ref = O.moe_ffn_mxfp4_decode_ref(x[toks], lids, wts, nib_gu[gsel], sc_gu[gsel], nib_dn[dsel], sc_dn[dsel], H, F)
        tol = TOL
    else:              # e4m3 activations through the fp8 GEMMs
        ref = O.moe_ffn_mxfp4_ref(x[toks], lids, wts, nib_gu[gsel], sc_gu[gsel], nib_dn[dsel], sc_dn[dsel], H, F)
        tol = 2e-2
    assert O.rel_l2(y[toks], ref) < tol, O.rel_l2(y[toks], ref)
    assert ops.device_status() == 0


# ---------------------------------------------------------------------------------------------------------- configs[4]
@pytest.mark.parametrize("k,n", [(5120, 27648), (27648, 5120)])
def test_config4_iq4_nl_gemm(ops, k, n):
    rng = np.random.default_rng(k)
    m = 4096
    w = blocks32(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x16, sc = ops.row_scale_f16(dev(x).to(torch.bfloat16))
    y = host(ops.gemm("iq4_nl", "store", x16, sc, dev(w), n))
    rows = np.sort(rng.choice(m, 128, replace=False))
    cols = np.sort(rng.choice(n, 256, replace=False))
    ref = O.gemm_ref("iq4_nl", w[cols], host(x16)[rows], host(sc)[rows], len(cols), k)
    assert O.rel_l2(y[np.ix_(rows, cols)], ref) < TOL, O.rel_l2(y[np.ix_(rows, cols)], ref)
    assert ops.device_status() == 0
