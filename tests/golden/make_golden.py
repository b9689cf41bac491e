"""Generate the golden fixtures in this directory from the reference's own Python code.

Run in a container that has the loom-skills checkout (read-only) and gguf-py 0.19.0:

    python tests/golden/make_golden.py /path/to/loom-skills

Every expected array here is produced by the REFERENCE's functions (or by gguf 0.19.0, the third-party package the
reference's numpy path calls), never by this repository's oracle, so the oracle and the CUDA kernels are both pinned
against them:

* Q4_0 blocks and their F64 decode: ``.github/devlab/kbench/moe_q4_0/gen_bench.py:19-35`` (weights, dequant_reference);
  the all-finite-F16-scale bit case ``gen_bench.py:51-63`` (dequant_bits_inputs) -- stored as a SHA-256 of the
  expected F16 bits plus a sample, since the full array is 4 MiB.
* Q4_K / IQ4_NL / MXFP4 (ggml blocks): ``gguf.quants.dequantize`` on seeded random blocks with finite scales
  (``make_kernel_tests.py:45-47`` is the reference's call site).
* MXFP4 split planes: ``skills/loom-port-llm/starter/st_tensors.py:26-35`` (dequant_mxfp4), including the known
  answer of ``tests/test_safetensors_source.py:200-205``.
* MXFP4 -> bf8 decode: ``tests/test_mxfp4s_f8.py:36-50`` (decode, e5m2) over the exact range e = 107..132.
* e4m3 rounding: ``.github/devlab/kbench/gemm_mxfp4s/gen_bench.py:268-281`` (e4m3_round, e4m3_bytes).
* small dense products: gguf dequant + float64 numpy matmul, as ``make_kernel_tests.py:231-238`` (matvec) and
  ``:1860-1876`` (GEMM with the row-scaled f16 activations and the inverse scale).
"""
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref):
    starter = os.path.join(ref, "skills/loom-port-llm/starter")
    sys.path.insert(0, starter)
    from gguf import GGMLQuantizationType as T
    from gguf.quants import dequantize
    q40 = _load(os.path.join(ref, ".github/devlab/kbench/moe_q4_0/gen_bench.py"), "q40_bench")
    argv, sys.argv = sys.argv, [sys.argv[0]]
    mx = _load(os.path.join(ref, ".github/devlab/kbench/gemm_mxfp4s/gen_bench.py"), "mx_bench")
    sys.argv = argv
    st = _load(os.path.join(starter, "st_tensors.py"), "st_tensors")
    f8t = _load(os.path.join(ref, "tests/test_mxfp4s_f8.py"), "test_mxfp4s_f8")
    out = {}

    # Q4_0: the reference's independent decoder on its own synthetic block generator
    rng = np.random.default_rng(47)
    raw, expected = q40.weights(rng, (2, 16, 704))
    out["q4_0_raw"] = np.asarray(raw).view(np.uint8)
    out["q4_0_f32"] = expected.astype(np.float32)   # d * (q - 8) is exact in f32
    braw, bexp = q40.dequant_bits_inputs()
    bexp = np.asarray(bexp).view(np.uint16)
    out["q4_0_bits_sha256"] = np.frombuffer(hashlib.sha256(bexp.tobytes()).digest(), np.uint8)
    sel = np.arange(0, bexp.size // 32, 97)
    out["q4_0_bits_rows"] = sel.astype(np.int64)
    out["q4_0_bits_sample"] = bexp.reshape(-1, 32)[sel]
    out["q4_0_bits_raw_sha256"] = np.frombuffer(hashlib.sha256(np.asarray(braw).view(np.uint8).tobytes()).digest(), np.uint8)

    # gguf 0.19.0 dequantisation of seeded random blocks (finite f16 scales)
    rng = np.random.default_rng(2024)
    for name, ty, bb, nb in [("q4_k", T.Q4_K, 144, 64), ("iq4_nl", T.IQ4_NL, 18, 512), ("mxfp4", T.MXFP4, 17, 512),
                             ("q4_0g", T.Q4_0, 18, 512)]:
        b = rng.integers(0, 256, (nb, bb), dtype=np.uint8)
        if name == "mxfp4":
            b[:, 0] = rng.integers(100, 140, nb)
        else:
            nsc = 2 if name == "q4_k" else 1
            sc = (rng.uniform(1e-4, 4e-2, (nb, nsc)) * rng.choice([-1, 1], (nb, nsc))).astype(np.float16)
            b[:, :2 * nsc] = sc.view(np.uint8).reshape(nb, 2 * nsc)
        out[f"{name}_raw"] = b
        out[f"{name}_f32"] = dequantize(b.reshape(-1), ty).reshape(nb, -1).astype(np.float32)

    # MXFP4 split planes: st_tensors.dequant_mxfp4 (pairs order) + the known-answer row
    rng = np.random.default_rng(1)
    nib = rng.integers(0, 256, (7, 96), dtype=np.uint8)
    sc = rng.integers(100, 130, (7, 6), dtype=np.uint8)
    out["mxfp4s_nib"], out["mxfp4s_sc"] = nib, sc
    out["mxfp4s_f32"] = st.dequant_mxfp4(nib, sc)
    ka = np.zeros((1, 16), np.uint8)
    ka[0, 0], ka[0, 1] = 0x21, 0x7F
    out["mxfp4s_known_nib"], out["mxfp4s_known_sc"] = ka, np.array([[128]], np.uint8)
    out["mxfp4s_known_f32"] = st.dequant_mxfp4(ka, np.array([[128]], np.uint8))

    # MXFP4 -> bf8 (e5m2) decode of the fp8 GEMM, every exponent of its exact range
    rng = np.random.default_rng(3)
    e = np.repeat(np.arange(107, 133), 64).astype(np.uint8)
    q = rng.integers(0, 256, (len(e), 16)).astype(np.uint8)
    out["bf8_e"], out["bf8_q"] = e, q
    out["bf8_bytes"] = f8t.decode(e, q).astype(np.uint8)
    out["bf8_values"] = f8t.e5m2(out["bf8_bytes"])

    # e4m3 rounding of the activation producer
    rng = np.random.default_rng(5)
    v = np.concatenate([rng.standard_normal(4096) * 64, rng.uniform(-300, 300, 2048), rng.uniform(-2 ** -7, 2 ** -7, 1024),
                        [0.0, -0.0, 448.0, 460.0, -1000.0, 2.0 ** -10, -(2.0 ** -10), 0.5 * 2.0 ** -9]])
    out["e4m3_in"] = v
    out["e4m3_round"] = mx.e4m3_round(v)
    out["e4m3_bytes"] = np.asarray(mx.e4m3_bytes(out["e4m3_round"])).view(np.uint8)

    # small dense products with the reference's numpy recipe (gguf dequant + float64 matmul)
    rng = np.random.default_rng(11)
    for fmt, ty, qk, bb in [("q4_0", T.Q4_0, 32, 18), ("q4_k", T.Q4_K, 256, 144), ("iq4_nl", T.IQ4_NL, 32, 18)]:
        n, k, t = 64, 512, 3
        b = rng.integers(0, 256, (n * k // qk, bb), dtype=np.uint8)
        nsc = 2 if fmt == "q4_k" else 1
        sc = (rng.uniform(1e-3, 4e-2, (len(b), nsc)) * rng.choice([-1, 1], (len(b), nsc))).astype(np.float16)
        if fmt == "q4_k":
            sc = np.abs(sc)
        b[:, :2 * nsc] = sc.view(np.uint8).reshape(len(b), 2 * nsc)
        W = dequantize(b.reshape(-1), ty).reshape(n, k).astype(np.float64)
        x = rng.standard_normal((t, k)).astype(np.float32)
        out[f"mv_{fmt}_w"] = b.reshape(n, -1)
        out[f"mv_{fmt}_x"] = x
        out[f"mv_{fmt}_y"] = x.astype(np.float64) @ W.T
        rows = 64
        xg = (rng.standard_normal((rows, k)) * rng.choice([1.0, 3e4], (rows, 1))).astype(np.float32)
        mxabs = np.abs(xg).max(-1)
        ebits = ((mxabs.view(np.uint32) >> 23) & 255).astype(np.int64)
        e_ = np.clip(ebits - 140, 0, 100)
        s = ((127 - e_).astype(np.uint32) << 23).view(np.float32)
        inv = ((127 + e_).astype(np.uint32) << 23).view(np.float32)
        x16 = (xg * s[:, None]).astype(np.float16)              # make_kernel_tests.py:1759-1762
        out[f"gemm_{fmt}_x"] = xg
        out[f"gemm_{fmt}_x16"] = x16
        out[f"gemm_{fmt}_scales"] = np.stack([s, inv], -1)
        out[f"gemm_{fmt}_y"] = (x16.astype(np.float64) @ W.T) * inv[:, None].astype(np.float64)

    # int8 activations: make_kernel_tests.py:32-40 (q8_ref), taken out of the script by its syntax tree (the module
    # itself runs a model build at import)
    import ast
    src_path = os.path.join(starter, "make_kernel_tests.py")
    tree = ast.parse(open(src_path).read())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "q8_ref")
    ns = {"np": np}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), src_path, "exec"), ns)
    rng = np.random.default_rng(23)
    xq = np.concatenate([rng.standard_normal((5, 512)) * rng.choice([1e-3, 1.0, 300.0], (5, 1)),
                         np.zeros((1, 512))]).astype(np.float32)
    xq[2, 64:96] = 0.0    # an all-zero group inside a live row
    out["q8_in"] = xq
    out["q8_deq"] = ns["q8_ref"](xq).astype(np.float32)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", os.path.join(HERE, "golden.npz"), sum(a.nbytes for a in out.values()), "bytes uncompressed")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
