"""A GGUF written by gguf-py (the reference's reader, inspect_gguf.py) loaded by this repository's reader straight into
the kernels: a dense Q4_K projection through lk_mv / lk_gemm, and an MoE layer whose experts come as GGUF's separate
ffn_gate_exps / ffn_up_exps / ffn_down_exps tensors (Q6_K gate/up, Q8_0 down), against the float64 oracle."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
gguf = pytest.importorskip("gguf")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

TOL = 1e-3


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from loom_skills_b200 import ops as _ops
    return _ops


def rand_blocks(fmt, rows, k, seed, offs):
    rng = np.random.default_rng(seed)
    nb = rows * k // O.QK[fmt]
    b = rng.integers(0, 256, (nb, O.BLOCK_BYTES[fmt]), dtype=np.uint8)
    for o in offs:
        b[:, o:o + 2] = (rng.uniform(1e-3, 2e-2, nb) * rng.choice([-1, 1], nb)).astype(np.float16).view(np.uint8).reshape(-1, 2)
    return b.reshape(rows, -1)


def test_gguf_weights_into_the_kernels(ops, tmp_path):
    from loom_skills_b200.gguf_file import GGUFFile
    T = gguf.GGMLQuantizationType
    E, F, H, n = 8, 256, 512, 384
    rng = np.random.default_rng(3)
    q = O.quantize_q4_k((rng.standard_normal((n, H)) * 0.02).astype(np.float32))
    g = rand_blocks("q6_k", E * F, H, 4, [208]).reshape(E, F, -1)
    u = rand_blocks("q6_k", E * F, H, 5, [208]).reshape(E, F, -1)
    d = rand_blocks("q8_0", E * H, F, 6, [0]).reshape(E, H, -1)
    wr = gguf.GGUFWriter(str(tmp_path / "m.gguf"), "qwen3moe", split_max_tensors=2)
    wr.add_uint32("qwen3moe.expert_count", E)
    wr.add_uint32("qwen3moe.expert_used_count", 2)
    wr.add_tensor("blk.0.attn_q.weight", q, raw_dtype=T.Q4_K)
    wr.add_tensor("blk.1.ffn_gate_exps.weight", g, raw_dtype=T.Q6_K)
    wr.add_tensor("blk.1.ffn_up_exps.weight", u, raw_dtype=T.Q6_K)
    wr.add_tensor("blk.1.ffn_down_exps.weight", d, raw_dtype=T.Q8_0)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    f = GGUFFile(str(tmp_path / "m-00001-of-00002.gguf"))
    wq = f.to_device("blk.0.attn_q.weight")
    x = rng.standard_normal((5, H)).astype(np.float32)
    y = ops.mv("q4_k", wq, torch.from_numpy(x).cuda(), n, H).cpu().numpy()
    assert O.rel_l2(y, O.mv_ref("q4_k", q, x, n, H)) < TOL
    cfg = f.moe_config(1)
    assert cfg["experts"] == E and cfg["used"] == 2 and cfg["gating"] == 1 and cfg["norm_weights"]
    wg, wu, wd = (f.to_device(f"blk.1.ffn_{p}_exps.weight") for p in ("gate", "up", "down"))
    for tokens in (3, 40):   # expert matvecs, then the grouped GEMMs
        xt = rng.standard_normal((tokens, H)).astype(np.float32)
        lg = rng.standard_normal((tokens, E)).astype(np.float32)
        yt = ops.moe_ffn(f.tensors["blk.1.ffn_gate_exps.weight"].format, torch.from_numpy(xt).cuda(),
                         torch.from_numpy(lg).cuda(), wg, wd, H, F, E, cfg["used"], w_up=wu,
                         prefill=tokens > 8, norm=cfg["norm_weights"],
                         fmt_down=f.tensors["blk.1.ffn_down_exps.weight"].format).cpu().numpy()
        ids, wts = O.route_ref(lg, cfg["used"], norm=cfg["norm_weights"])
        # gate and up from their own tensors; the down projection is Q8_0
        Wg = O.dequant("q6_k", g, H).reshape(E, F, H).astype(np.float64)
        Wu = O.dequant("q6_k", u, H).reshape(E, F, H).astype(np.float64)
        Wd = O.dequant("q8_0", d, F).reshape(E, H, F).astype(np.float64)
        ref = O.moe_ffn_ref(xt, ids, wts, np.concatenate([Wg, Wu], 1), Wd, None, H, F, E)
        assert O.rel_l2(yt, ref) < TOL, (tokens, O.rel_l2(yt, ref))
