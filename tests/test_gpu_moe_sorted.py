"""GPU parity of the MoE gate/up on activations row-scaled straight into bucket order (lk_moe_row_scale_gather, then
the grouped GEMMs' LK_SWIGLU_SORTED mode) through the C ABI.

lk_moe_row_scale_gather must equal the reference row scale of the gathered token rows bit for bit (the oracle's
row_scale_f16 / row_scale_f8 on x[rowmap // ku], zero rows for unused schedule rows). The sorted gate/up then reads the
very bytes the gathering gate/up reads, so its output must equal the gather mode's bit for bit on every live row.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402


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


def bits32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def gathered(x, rowmap, ku):
    """Host restatement of the A rows the gathering gate/up reads: x[rowmap // ku], zero rows where rowmap < 0."""
    rm = np.asarray(rowmap)
    out = np.zeros((rm.size, x.shape[1]), np.float32)
    live = rm >= 0
    out[live] = x[rm[live] // ku]
    return out


def schedule(ops, tokens, E, ku, seed):
    rng = np.random.default_rng(seed)
    ids, _ = O.route_ref(rng.standard_normal((tokens, E)).astype(np.float32), ku)
    ti, rm, pos = ops.moe_bucket(dev(ids), E, ops.moe_max_tiles(tokens, ku, E))
    return ti, rm


class TestRowScaleGather:
    @pytest.mark.parametrize("dtype", ["f32", "bf16"])
    def test_f16_bit_exact(self, ops, dtype):
        tokens, E, ku, k = 45, 8, 4, 576
        rng = np.random.default_rng(5)
        x = (rng.standard_normal((tokens, k)) * rng.choice([1e-3, 1.0, 3e4], (tokens, 1))).astype(np.float32)
        xt = dev(x)
        if dtype == "bf16":
            xt = xt.to(torch.bfloat16)
            x = xt.float().cpu().numpy()
        ti, rm = schedule(ops, tokens, E, ku, 6)
        x16, sc = ops.moe_row_scale_gather(xt, rm, ku)
        rx16, rsc = O.row_scale_f16(gathered(x, host(rm), ku))
        assert np.array_equal(host(x16).view(np.uint16), rx16.view(np.uint16))
        assert np.array_equal(bits32(host(sc)), bits32(rsc))

    def test_f8_bit_exact(self, ops):
        tokens, E, ku, k = 70, 8, 4, 2880
        rng = np.random.default_rng(7)
        x = (rng.standard_normal((tokens, k)) * rng.choice([1e-2, 1.0, 50.0], (tokens, 1))).astype(np.float32)
        ti, rm = schedule(ops, tokens, E, ku, 8)
        x8, s8 = ops.moe_row_scale_gather(dev(x), rm, ku, f8=True)
        rx8, rs8 = O.row_scale_f8(gathered(x, host(rm), ku))
        assert np.array_equal(host(x8), rx8)
        assert np.array_equal(bits32(host(s8)), bits32(rs8))

    def test_invalid(self, ops):
        x = torch.zeros(4, 20, device="cuda")   # k % 8 != 0
        rm = torch.zeros(64, dtype=torch.int32, device="cuda")
        with pytest.raises(ops.L.LkError):
            ops.moe_row_scale_gather(x, rm, 1)


class TestSortedGateUp:
    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k", "iq4_nl"])
    def test_equals_gather(self, ops, fmt):
        tokens, E, ku, H, F = 150, 8, 4, 512, 320
        rng = np.random.default_rng(9)
        quant = {"q4_0": O.quantize_q4_0, "q4_k": O.quantize_q4_k, "iq4_nl": O.quantize_iq4_nl}[fmt]
        w_gu = quant((rng.standard_normal((E * 2 * F, H)) * 0.02).astype(np.float32))
        x = rng.standard_normal((tokens, H)).astype(np.float32)
        ti, rm = schedule(ops, tokens, E, ku, 10)
        x16, sc = ops.row_scale_f16(dev(x))
        act_g = host(ops.moe_grouped_gemm(fmt, "swiglu", ti, rm, x16, sc, dev(w_gu), F, ku, E, fused=True))
        xs, scs = ops.moe_row_scale_gather(dev(x), rm, ku)
        act_s = host(ops.moe_grouped_gemm(fmt, "swiglu_sorted", ti, rm, xs, scs, dev(w_gu), F, ku, E, fused=True))
        rows = np.nonzero(host(rm) >= 0)[0]   # the live rows (rows past a tile's count are never written)
        assert np.array_equal(bits32(act_s[rows]), bits32(act_g[rows]))
        assert ops.L.load().lk_device_status(1) == 0

    @pytest.mark.parametrize("order", ["pairs", "split16"])
    @pytest.mark.parametrize("h", [576, 2880])
    def test_mxfp4_equals_gather(self, ops, order, h):
        tokens, E, ku, F = 90, 8, 4, 320
        rng = np.random.default_rng(11)
        nib, sc = O.quantize_mxfp4((rng.standard_normal((E * 2 * F, h)) * 0.02).astype(np.float32), "planar")
        if order == "split16":
            codes = np.stack([nib & 15, nib >> 4], -1).reshape(nib.shape[0], -1, 32)
            nib = (codes[..., :16] | (codes[..., 16:] << 4)).reshape(nib.shape[0], -1).astype(np.uint8)
        o = ops.L.ORDER_SPLIT16 if order == "split16" else ops.L.ORDER_PAIRS
        x = rng.standard_normal((tokens, h)).astype(np.float32)
        ti, rm = schedule(ops, tokens, E, ku, 12)
        x8, s8 = ops.row_scale_f8(dev(x))
        act_g = host(ops.moe_grouped_gemm_mxfp4s_f8("swiglu", ti, rm, x8, s8, dev(nib), dev(sc), F, ku, E, fused=True,
                                                    order=o))
        xs, ss = ops.moe_row_scale_gather(dev(x), rm, ku, f8=True)
        act_s = host(ops.moe_grouped_gemm_mxfp4s_f8("swiglu_sorted", ti, rm, xs, ss, dev(nib), dev(sc), F, ku, E,
                                                    fused=True, order=o))
        rows = np.nonzero(host(rm) >= 0)[0]
        assert np.array_equal(bits32(act_s[rows]), bits32(act_g[rows]))
        assert ops.L.load().lk_device_status(1) == 0
