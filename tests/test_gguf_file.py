"""The GGUF reader (loom_skills_b200/gguf_file.py) against gguf-py 0.19.0 -- the package the reference reads GGUFs
with (inspect_gguf.py:21-60): files written by gguf-py's GGUFWriter, single and split (NAME-0000i-of-0000N.gguf,
formats.split_parts), read back by this repository's own parser and compared with gguf-py's GGUFReader: names, types,
shapes, tensor bytes, metadata; the MoE routing config of inspect_gguf.py:284-320; the MXFP4 plane repack. CPU only."""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

from loom_skills_b200 import gguf_file as G  # noqa: E402
from oracle import qmm_oracle as O  # noqa: E402

T = gguf.GGMLQuantizationType


def write(path, arch, tensors, meta, split_max_tensors=0):
    wr = gguf.GGUFWriter(str(path), arch, split_max_tensors=split_max_tensors)
    for k, (kind, v) in meta.items():
        getattr(wr, f"add_{kind}")(k, v)
    for name, (arr, ty) in tensors.items():
        if ty is None:
            wr.add_tensor(name, arr)
        else:
            wr.add_tensor(name, arr, raw_dtype=ty)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()


@pytest.fixture(scope="module")
def model():
    rng = np.random.default_rng(5)
    E, F, H = 4, 64, 256
    t = {
        "token_embd.weight": (O.quantize_q4_0((rng.standard_normal((96, H)) * 0.02).astype(np.float32)), T.Q4_0),
        "blk.0.attn_q.weight": (O.quantize_q4_k((rng.standard_normal((128, H)) * 0.02).astype(np.float32)), T.Q4_K),
        "blk.0.ffn_gate_exps.weight": (O.quantize_q4_0((rng.standard_normal((E * F, H)) * 0.02).astype(np.float32))
                                       .reshape(E, F, -1), T.Q4_0),
        "blk.0.ffn_up_exps.weight": (O.quantize_q4_0((rng.standard_normal((E * F, H)) * 0.02).astype(np.float32))
                                     .reshape(E, F, -1), T.Q4_0),
        "blk.0.ffn_down_exps.weight": (O.quantize_mxfp4((rng.standard_normal((E * H, F)) * 0.02).astype(np.float32),
                                                        "ggml").reshape(E, H, -1), T.MXFP4),
        "blk.0.ffn_gate_inp.weight": (rng.standard_normal((E, H)).astype(np.float32), None),
        "blk.0.ffn_gate_inp.bias": (rng.standard_normal(E).astype(np.float32), None),
        "blk.0.attn_norm.weight": (rng.standard_normal(H).astype(np.float16), None),
    }
    meta = {"gpt-oss.expert_count": ("uint32", E), "gpt-oss.expert_used_count": ("uint32", 2),
            "gpt-oss.expert_feed_forward_length": ("uint32", F), "gpt-oss.embedding_length": ("uint32", H),
            "general.name": ("string", "tiny")}
    return t, meta


@pytest.mark.parametrize("split", [0, 3])
def test_reads_what_gguf_py_writes(tmp_path, model, split):
    tensors, meta = model
    write(tmp_path / "m.gguf", "gpt-oss", tensors, meta, split_max_tensors=split)
    first = tmp_path / ("m-00001-of-00003.gguf" if split else "m.gguf")
    if split:
        assert len(list(tmp_path.glob("m-*.gguf"))) == 3
    f = G.GGUFFile(str(first))
    assert len(f.paths) == (3 if split else 1)
    assert f.arch == "gpt-oss" and f.field("general.name") == "tiny"
    assert f.field("gpt-oss.expert_count") == 4
    refs = {}
    for p in f.paths:
        for t in gguf.GGUFReader(p).tensors:
            refs[t.name] = t
    assert set(refs) == set(f.tensors) == set(tensors)
    for name, rt in refs.items():
        t = f.tensors[name]
        assert t.type == int(rt.tensor_type)
        assert t.dims == tuple(int(d) for d in rt.shape)
        assert np.array_equal(f.raw(name), np.asarray(rt.data).view(np.uint8).reshape(-1))
    # packed rows in the ops' layouts: experts stacked as rows
    assert f.rows("blk.0.ffn_gate_exps.weight").shape == (4 * 64, 256 // 32 * 18)
    assert np.array_equal(f.rows("blk.0.ffn_gate_exps.weight"), tensors["blk.0.ffn_gate_exps.weight"][0].reshape(256, -1))
    assert np.array_equal(f.rows("blk.0.attn_q.weight"), tensors["blk.0.attn_q.weight"][0])
    np.testing.assert_array_equal(f.array("blk.0.ffn_gate_inp.weight"), tensors["blk.0.ffn_gate_inp.weight"][0])
    np.testing.assert_array_equal(f.array("blk.0.attn_norm.weight"),
                                  tensors["blk.0.attn_norm.weight"][0].astype(np.float32))


def test_moe_config_and_mxfp4_planes(tmp_path, model):
    tensors, meta = model
    write(tmp_path / "m.gguf", "gpt-oss", tensors, meta)
    f = G.GGUFFile(str(tmp_path / "m.gguf"))
    cfg = f.moe_config()
    # gpt-oss: softmax of the picked biased logits, no norm, swiglu_oai (inspect_gguf.py:291), router bias present
    assert cfg["experts"] == 4 and cfg["used"] == 2 and cfg["ffn"] == 64
    assert cfg["gating"] == 3 and not cfg["norm_weights"] and cfg["act"] == "swiglu_oai" and cfg["router_bias"]
    assert not cfg["gate_up_fused"] and not cfg["expert_bias"]
    nib, sc = f.mxfp4_planes("blk.0.ffn_down_exps.weight")
    blk = tensors["blk.0.ffn_down_exps.weight"][0].reshape(-1, 17)
    assert nib.shape == (4 * 256, 64 // 2) and sc.shape == (4 * 256, 64 // 32)
    # the planes decode (split16 order) to the ggml blocks' exact values
    vals = O.dequant_mxfp4_planar(nib, sc, 4 * 256, 64, "split16")
    np.testing.assert_array_equal(vals, O.dequant("mxfp4", blk.reshape(-1), blk.shape[0] * 32).reshape(4 * 256, 64))


def test_rejects_a_missing_part_and_a_bad_file(tmp_path, model):
    tensors, meta = model
    write(tmp_path / "m.gguf", "gpt-oss", tensors, meta, split_max_tensors=3)
    (tmp_path / "m-00002-of-00003.gguf").unlink()
    with pytest.raises(G.GGUFError, match="missing parts"):
        G.GGUFFile(str(tmp_path / "m-00001-of-00003.gguf"))
    (tmp_path / "bad.gguf").write_bytes(b"NOPE" + bytes(64))
    with pytest.raises(G.GGUFError, match="not a GGUF"):
        G.GGUFFile(str(tmp_path / "bad.gguf"))


def test_split_parts_names():
    assert G.split_parts("/m/x-00001-of-00003.gguf") == [f"/m/x-0000{i}-of-00003.gguf" for i in (1, 2, 3)]
    assert G.split_parts("/m/x.gguf") == ["/m/x.gguf"]
