"""GPU parity: liblk kernels (through the C ABI) against the CPU oracle and the reference's golden vectors.

Bars: dequantised values, row scales, e4m3 bytes and MoE schedules bit-exact; products within relative L2 1e-3 of the
reference's float64 path (the north-star tolerance for f16/bf16/f32 accumulation).
"""
import hashlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

TOL = 1e-3   # relative L2, products with f16/bf16/f32 accumulation


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


QUANT = {"q4_0": O.quantize_q4_0, "q4_k": O.quantize_q4_k, "iq4_nl": O.quantize_iq4_nl}


def weights(fmt, n, k, seed, std=0.02):
    w = (np.random.default_rng(seed).standard_normal((n, k)) * std).astype(np.float32)
    return QUANT[fmt](w)


# ---------------------------------------------------------------------------------------------------------- dequant
class TestDequant:
    @pytest.mark.parametrize("fmt,qk", [("q4_k", 256), ("iq4_nl", 32), ("mxfp4", 32), ("q4_0g", 32)])
    def test_golden_f32_bit_exact(self, ops, golden, fmt, qk):
        f = "q4_0" if fmt == "q4_0g" else fmt
        raw = golden[f"{fmt}_raw"]
        out = ops.dequant(f, dev(raw.reshape(-1)), raw.shape[0] * qk)
        assert np.array_equal(bits32(host(out)), bits32(golden[f"{fmt}_f32"].reshape(-1)))

    def test_q4_0_reference_blocks(self, ops, golden):
        out = ops.dequant("q4_0", dev(golden["q4_0_raw"]), golden["q4_0_f32"].size)
        assert np.array_equal(bits32(host(out)), bits32(golden["q4_0_f32"].reshape(-1)))

    def test_q4_0_every_finite_scale_f16_staging(self, ops, golden):
        bits = np.arange(65536, dtype=np.uint16)
        bits = bits[(bits & 0x7C00) != 0x7C00]
        raw = np.empty((len(bits), 18), np.uint8)
        raw[:, :2] = bits.astype("<u2").view(np.uint8).reshape(-1, 2)
        codes = np.arange(16, dtype=np.uint8)
        raw[:, 2:] = codes | ((15 - codes) << 4)
        out = host(ops.dequant("q4_0", dev(raw.reshape(-1)), len(bits) * 32, torch.float16)).view(np.uint16)
        assert hashlib.sha256(out.tobytes()).digest() == golden["q4_0_bits_sha256"].tobytes()

    def test_mxfp4_planar(self, ops, golden):
        nib, sc = golden["mxfp4s_nib"], golden["mxfp4s_sc"]
        out = ops.dequant("mxfp4s", dev(nib.reshape(-1)), nib.size * 2, w_scales=dev(sc.reshape(-1)))
        assert np.array_equal(bits32(host(out)), bits32(golden["mxfp4s_f32"].reshape(-1)))

    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k", "iq4_nl"])
    def test_f16_staging_matches_oracle(self, ops, fmt):
        raw = weights(fmt, 64, 1024, 7)
        out = host(ops.dequant(fmt, dev(raw.reshape(-1)), 64 * 1024, torch.float16)).view(np.uint16)
        ref = O.dequant_f16(fmt, raw, 1024).reshape(-1).view(np.uint16)
        assert np.array_equal(out, ref)


# ---------------------------------------------------------------------------------------------------------- producers
class TestRowScale:
    @pytest.mark.parametrize("dtype", ["f32", "bf16"])
    @pytest.mark.parametrize("k", [768, 2880, 5120, 12288, 1000])   # warp form, one-pass CTA forms, scalar form
    def test_row_scale_f16_bit_exact(self, ops, dtype, k):
        rng = np.random.default_rng(3)
        x = (rng.standard_normal((37, k)) * rng.choice([1e-3, 1.0, 3e4, 3e6], (37, 1))).astype(np.float32)
        xt = dev(x)
        if dtype == "bf16":
            xt = xt.to(torch.bfloat16)
            x = xt.float().cpu().numpy()
        x16, sc = ops.row_scale_f16(xt)
        rx16, rsc = O.row_scale_f16(x)
        assert np.array_equal(host(x16).view(np.uint16), rx16.view(np.uint16))
        assert np.array_equal(bits32(host(sc)), bits32(rsc))

    @pytest.mark.parametrize("k", [2880, 768, 6144])
    def test_row_scale_f8_bit_exact(self, ops, k):
        rng = np.random.default_rng(4)
        x = (rng.standard_normal((19, k)) * rng.choice([1e-2, 1.0, 50.0], (19, 1))).astype(np.float32)
        x8, s8 = ops.row_scale_f8(dev(x))
        rx8, rs8 = O.row_scale_f8(x)
        assert np.array_equal(host(x8), rx8)
        assert np.array_equal(bits32(host(s8)), bits32(rs8))


# ---------------------------------------------------------------------------------------------------------- matvec
class TestMv:
    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k", "iq4_nl"])
    def test_golden(self, ops, golden, fmt):
        w, x = golden[f"mv_{fmt}_w"], golden[f"mv_{fmt}_x"]
        y = host(ops.mv(fmt, dev(w), dev(x), w.shape[0], 512))
        assert O.rel_l2(y, golden[f"mv_{fmt}_y"]) < TOL

    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k", "iq4_nl"])
    @pytest.mark.parametrize("xdt", ["f32", "f16", "bf16"])
    @pytest.mark.parametrize("tokens", [1, 3, 8, 13])
    def test_vs_oracle(self, ops, fmt, xdt, tokens):
        n, k = 272, 1280
        w = weights(fmt, n, k, 11)
        x = np.random.default_rng(12).standard_normal((tokens, k)).astype(np.float32)
        xt = dev(x).to({"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[xdt])
        y = host(ops.mv(fmt, dev(w), xt, n, k))
        ref = O.mv_ref(fmt, w, xt.float().cpu().numpy(), n, k)
        assert O.rel_l2(y, ref) < TOL, O.rel_l2(y, ref)

    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k"])
    def test_swiglu_and_accumulate(self, ops, fmt):
        n, k = 96, 2048
        w, w2 = weights(fmt, n, k, 21), weights(fmt, n, k, 22)
        x = np.random.default_rng(23).standard_normal((4, k)).astype(np.float32)
        y0 = np.random.default_rng(24).standard_normal((4, n)).astype(np.float32)
        yt = dev(y0)
        ops.mv(fmt, dev(w), dev(x), n, k, w2=dev(w2), y=yt, accumulate=True)
        ref = O.mv_ref(fmt, w, x, n, k, w2=w2, y_old=y0)
        assert O.rel_l2(host(yt), ref) < TOL

    def test_large_shapes(self, ops):
        # the Q4_K decode shapes of the bench (K=4096, N=4096; down K=12288) at M=1 and M=8
        for k, n, t in [(4096, 4096, 1), (12288, 512, 8)]:
            w = weights("q4_k", n, k, 31)
            x = np.random.default_rng(32).standard_normal((t, k)).astype(np.float32)
            xt = dev(x).to(torch.bfloat16)
            y = host(ops.mv("q4_k", dev(w), xt, n, k))
            assert O.rel_l2(y, O.mv_ref("q4_k", w, xt.float().cpu().numpy(), n, k)) < TOL

    @pytest.mark.parametrize("fmt,xdt,n,k", [("q4_k", "f32", 1000, 12288), ("q4_0", "bf16", 4104, 4096),
                                             ("iq4_nl", "f16", 130, 2304), ("q4_k", "bf16", 24576, 4096)])
    def test_one_token_row_blocks(self, ops, fmt, xdt, n, k):
        # the persistent one-token form: several 16-row blocks per CTA, a last partial block and a partial last stage,
        # swiglu with accumulate, and the plain product
        w, w2 = weights(fmt, n, k, 41), weights(fmt, n, k, 42)
        x = np.random.default_rng(43).standard_normal((1, k)).astype(np.float32)
        xt = dev(x).to({"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[xdt])
        xh = xt.float().cpu().numpy()
        y = host(ops.mv(fmt, dev(w), xt, n, k))
        assert O.rel_l2(y, O.mv_ref(fmt, w, xh, n, k)) < TOL
        y0 = np.random.default_rng(44).standard_normal((1, n)).astype(np.float32)
        yt = dev(y0)
        ops.mv(fmt, dev(w), xt, n, k, w2=dev(w2), y=yt, accumulate=True)
        assert O.rel_l2(host(yt), O.mv_ref(fmt, w, xh, n, k, w2=w2, y_old=y0)) < TOL
        assert ops.device_status() == 0

    def test_device_status_clear(self, ops):
        assert ops.device_status() == 0


# ---------------------------------------------------------------------------------------------------------- GEMM
def row_scaled(rows, k, seed, big=False):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    if big:
        x *= rng.choice([1.0, 3e5], (rows, 1)).astype(np.float32)
    return x, *O.row_scale_f16(x)


class TestGemm:
    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k", "iq4_nl"])
    def test_golden(self, ops, golden, fmt):
        w = golden[f"mv_{fmt}_w"]
        y = host(ops.gemm(fmt, "store", dev(golden[f"gemm_{fmt}_x16"]), dev(golden[f"gemm_{fmt}_scales"]), dev(w),
                          w.shape[0]))
        assert O.rel_l2(y, golden[f"gemm_{fmt}_y"]) < TOL

    @pytest.mark.parametrize("fmt", ["q4_0", "q4_k", "iq4_nl"])
    @pytest.mark.parametrize("rows,n,k", [(128, 256, 256), (200, 512, 1024), (1, 272, 512), (384, 1024, 2048)])
    def test_store(self, ops, fmt, rows, n, k):
        w = weights(fmt, n, k, 41)
        _, x16, sc = row_scaled(rows, k, 42, big=True)
        y = host(ops.gemm(fmt, "store", dev(x16), dev(sc), dev(w), n))
        ref = O.gemm_ref(fmt, w, x16, sc, n, k)
        assert O.rel_l2(y, ref) < TOL, O.rel_l2(y, ref)
        # against the f16-staged weights the tensor cores see: accumulation error only
        W16 = O.dequant_f16(fmt, w, k).astype(np.float64).reshape(n, k)
        ref16 = (x16.astype(np.float64) @ W16.T) * sc[:, 1:2]
        assert O.rel_l2(y, ref16) < 1e-5

    @pytest.mark.parametrize("fmt", ["q4_k", "q4_0"])
    def test_acc_and_swiglu(self, ops, fmt):
        rows, n, k = 256, 384, 1024
        w, w2 = weights(fmt, n, k, 51), weights(fmt, n, k, 52)
        _, x16, sc = row_scaled(rows, k, 53)
        y0 = np.random.default_rng(54).standard_normal((rows, n)).astype(np.float32)
        yt = dev(y0)
        ops.gemm(fmt, "acc", dev(x16), dev(sc), dev(w), n, y=yt)
        assert O.rel_l2(host(yt), O.gemm_ref(fmt, w, x16, sc, n, k, mode="acc", y_old=y0)) < TOL
        ys = host(ops.gemm(fmt, "swiglu", dev(x16), dev(sc), dev(w), n, w2=dev(w2)))
        assert O.rel_l2(ys, O.gemm_ref(fmt, w, x16, sc, n, k, mode="swiglu", w2=w2)) < TOL

    @pytest.mark.parametrize("fmt", ["q4_k", "q4_0", "iq4_nl"])
    @pytest.mark.parametrize("rows,n,k", [(64, 1024, 4096), (37, 512, 12288), (128, 272, 1024), (129, 256, 2048)])
    def test_short_rows_split_k(self, ops, fmt, rows, n, k):
        # at most 128 rows: 128 x 256 tiles; few tiles: K split into ranges that meet in y in a fixed order (range 0
        # stores -- acc: adds onto y -- and range s adds after range s - 1): the same bits on every run
        w = weights(fmt, n, k, 71)
        _, x16, sc = row_scaled(rows, k, 72, big=True)
        wd, xd, sd = dev(w), dev(x16), dev(sc)
        y = host(ops.gemm(fmt, "store", xd, sd, wd, n, y=dev(np.full((rows, n), 7.0, np.float32))))
        ref = O.gemm_ref(fmt, w, x16, sc, n, k)
        assert O.rel_l2(y, ref) < TOL, O.rel_l2(y, ref)
        for _ in range(4):
            assert np.array_equal(host(ops.gemm(fmt, "store", xd, sd, wd, n)), y)
        y0 = np.random.default_rng(73).standard_normal((rows, n)).astype(np.float32)
        ya = dev(y0)
        ops.gemm(fmt, "acc", xd, sd, wd, n, y=ya)
        ref_acc = O.gemm_ref(fmt, w, x16, sc, n, k, mode="acc", y_old=y0)
        assert O.rel_l2(host(ya), ref_acc) < TOL, O.rel_l2(host(ya), ref_acc)
        for _ in range(3):
            yb = dev(y0)
            ops.gemm(fmt, "acc", xd, sd, wd, n, y=yb)
            assert torch.equal(yb, ya)
        assert ops.device_status() == 0

    def test_split_k_graph_replays(self, ops):
        # the split-K turnstiles across CUDA-graph replays of one captured launch (its epoch is reused): every replay
        # gives the eager launch's bits
        fmt, rows, n, k = "q4_k", 64, 1024, 4096
        w = dev(weights(fmt, n, k, 81))
        _, x16, sc = row_scaled(rows, k, 82, big=True)
        xd, sd = dev(x16), dev(sc)
        y_eager = ops.gemm(fmt, "store", xd, sd, w, n)
        y = torch.full((rows, n), float("nan"), device="cuda")
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ops.gemm(fmt, "store", xd, sd, w, n, y=y)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                ops.gemm(fmt, "store", xd, sd, w, n, y=y)
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            y.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(y, y_eager)
        assert ops.device_status() == 0
        del g

    def test_empty_rows(self, ops):
        w = weights("q4_k", 256, 256, 1)
        y = ops.gemm("q4_k", "store", torch.empty(0, 256, dtype=torch.float16, device="cuda"),
                     torch.empty(0, 2, device="cuda"), dev(w), 256)
        assert y.shape == (0, 256)


# ---------------------------------------------------------------------------------------------------------- MoE
class TestMoE:
    def test_route(self, ops):
        rng = np.random.default_rng(61)
        lg = rng.standard_normal((300, 128)).astype(np.float32)
        lg[7, [5, 77]] = 9.0    # an exact tie: lowest index first
        ids, wts = ops.moe_route(dev(lg), 128, 8)
        rids, rwts = O.route_ref(lg, 8)
        assert np.array_equal(host(ids), rids)
        np.testing.assert_allclose(host(wts), rwts, rtol=2e-6, atol=1e-7)

    def test_route_with_router_weights(self, ops):
        rng = np.random.default_rng(62)
        h = rng.standard_normal((20, 256)).astype(np.float32)
        wr = (rng.standard_normal((32, 256)) * 0.1).astype(np.float32)
        ids, wts = ops.moe_route(dev(h), 32, 4, router_w=dev(wr))
        rids, rwts = O.route_ref(h.astype(np.float64) @ wr.T.astype(np.float64), 4)
        assert np.array_equal(host(ids), rids)
        np.testing.assert_allclose(host(wts), rwts, rtol=1e-5)

    @pytest.mark.parametrize("tokens,E,ku", [(1, 128, 8), (37, 16, 8), (513, 128, 8), (4096, 128, 8), (64, 32, 4)])
    def test_bucket_exact(self, ops, tokens, E, ku):
        rng = np.random.default_rng(tokens)
        ids, _ = O.route_ref(rng.standard_normal((tokens, E)).astype(np.float32), ku)
        info = np.zeros((tokens, 4), np.int32)
        info[:, 2] = 1
        if tokens > 5:
            info[3, 2] = 0
        mt = ops.moe_max_tiles(tokens, ku, E)
        ti, rm, pos = ops.moe_bucket(dev(ids), E, mt, info=dev(info))
        rti, rrm, rpos = O.bucket_ref(ids, E, mt, info[:, 2])
        assert np.array_equal(host(ti), rti)
        assert np.array_equal(host(rm), rrm)
        assert np.array_equal(host(pos), rpos)

    @pytest.mark.parametrize("tokens", [63, 65, 300])
    def test_grouped_gemms_and_combine(self, ops, tokens):
        E, ku, H, F, fmt = 16, 4, 512, 256, "q4_0"
        rng = np.random.default_rng(70 + tokens)
        w_gu = np.stack([weights(fmt, 2 * F, H, 100 + e) for e in range(E)])
        w_dn = np.stack([weights(fmt, H, F, 200 + e) for e in range(E)])
        x = rng.standard_normal((tokens, H)).astype(np.float32)
        ids, wts = O.route_ref(rng.standard_normal((tokens, E)).astype(np.float32), ku)
        x16, sc = O.row_scale_f16(x)
        mt = ops.moe_max_tiles(tokens, ku, E)
        ti, rm, pos = ops.moe_bucket(dev(ids), E, mt)
        act = ops.moe_grouped_gemm(fmt, "swiglu", ti, rm, dev(x16), dev(sc), dev(w_gu), F, ku, E, fused=True)
        rti, rrm, rpos = O.bucket_ref(ids, E, mt)
        W = {e: O.dequant(fmt, w_gu[e], H).reshape(2 * F, H).astype(np.float64) for e in range(E)}
        D = {e: O.dequant(fmt, w_dn[e], F).reshape(H, F).astype(np.float64) for e in range(E)}
        act_h = host(act)
        live = rrm >= 0
        ref_act = np.zeros((len(rrm), F))
        for r in np.nonzero(live)[0]:
            a = rrm[r]
            e = rti[r // 64, 0]
            pr = (x16[a // ku].astype(np.float64) @ W[e].T) * sc[a // ku, 1]
            ref_act[r] = O.silu(pr[:F]) * pr[F:]
        assert O.rel_l2(act_h[live], ref_act[live]) < TOL
        a16, asc = O.row_scale_f16(np.where(live[:, None], act_h, 0).astype(np.float32))
        ys = ops.moe_grouped_gemm(fmt, "store", ti, rm, dev(a16), dev(asc), dev(w_dn), H, ku, E)
        ys_h = host(ys)
        ref_ys = np.zeros((len(rrm), H))
        for r in np.nonzero(live)[0]:
            ref_ys[r] = (a16[r].astype(np.float64) @ D[rti[r // 64, 0]].T) * asc[r, 1]
        assert O.rel_l2(ys_h[live], ref_ys[live]) < TOL
        y = host(ops.moe_combine_sorted(ys, pos, dev(wts)))
        ref_y = np.zeros((tokens, H))
        for t in range(tokens):
            for kk in range(ku):
                ref_y[t] += wts[t, kk] * ys_h[rpos[t * ku + kk]]
        assert O.rel_l2(y, ref_y) < 1e-6

    @pytest.mark.parametrize("tokens", [1, 16, 24, 40, 256])
    def test_moe_ffn_end_to_end(self, ops, tokens):
        E, ku, H, F, fmt = 32, 8, 1024, 256, "q4_0"
        rng = np.random.default_rng(90 + tokens)
        w_gu = np.stack([weights(fmt, 2 * F, H, 300 + e) for e in range(E)])
        w_dn = np.stack([weights(fmt, H, F, 400 + e) for e in range(E)])
        x = torch.from_numpy(rng.standard_normal((tokens, H)).astype(np.float32)).to(torch.bfloat16)
        lg = rng.standard_normal((tokens, E)).astype(np.float32)
        y = host(ops.moe_ffn(fmt, x.cuda(), dev(lg), dev(w_gu), dev(w_dn), H, F, E, ku))
        ids, wts = O.route_ref(lg, ku)
        ref = O.moe_ffn_ref(x.float().numpy(), ids, wts, w_gu, w_dn, fmt, H, F, E)
        assert O.rel_l2(y, ref) < TOL, O.rel_l2(y, ref)

    def test_expert_mv_decode(self, ops):
        E, ku, H, F, fmt = 16, 4, 512, 256, "q4_k"
        rng = np.random.default_rng(95)
        w_gu = np.stack([weights(fmt, 2 * F, H, 500 + e) for e in range(E)])
        x = rng.standard_normal((3, H)).astype(np.float32)
        ids = rng.integers(0, E, (3, ku)).astype(np.int32)
        act = host(ops.moe_expert_mv(fmt, "gu", dev(ids.reshape(-1)), dev(x), dev(w_gu), F, H, ku, E))
        for a, e in enumerate(ids.reshape(-1)):
            W = O.dequant(fmt, w_gu[e], H).reshape(2 * F, H).astype(np.float64)
            pr = W @ x[a // ku].astype(np.float64)
            assert O.rel_l2(act[a], O.silu(pr[:F]) * pr[F:]) < TOL
