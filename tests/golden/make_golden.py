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


def _reference_functions(ref, names, scope):
    """Functions of make_kernel_tests.py taken out by its syntax tree (the module runs a model build at import; some
    of these are nested in its MoE section), executed in `scope` for their free variables."""
    import ast
    src_path = os.path.join(ref, "skills/loom-port-llm/starter/make_kernel_tests.py")
    tree = ast.parse(open(src_path).read())
    found = {n.name: n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef) and n.name in names}
    missing = set(names) - set(found)
    assert not missing, missing
    exec(compile(ast.Module(body=[found[n] for n in names], type_ignores=[]), src_path, "exec"), scope)
    return scope


def main_moe(ref):
    """golden_moe.npz: the router, expert-FFN and hand-built MoE schedule vectors, all computed by the reference's
    own code:

    * router: make_kernel_tests.py:3166-3186 route_ref (gating 1 softmax / 2 sigmoid + selection bias / 3 softmax of
      the picked biased logits, norm_weights, expert_weights_scale), with Wr = I so the logits are the inputs; rows
      whose k-th and (k+1)-th scores are within 0.2 % are dropped, as its clear_tokens does (:3187-3194);
    * expert FFN: make_kernel_tests.py:3196-3215 experts_ref (SiLU, GEGLU gelu-tanh via ffn_act :78-80, gpt-oss
      swiglu_oai with per-expert biases; the prefill variant f16=True), and the chain of :3268-3271 (per-expert down
      scale folded into the weights, the Qwen shared-expert gate scaling the shared output y0);
    * the kbench moe_q4_0 cases (.github/devlab/kbench/moe_q4_0/gen_bench.py:185-248): weights from its own
      generator, the decode and grouped expert products with its F64 formulas and its gelu, sentinel 42 where a
      kernel must not write, and the down-scale + combine case. Inputs are regenerated by the oracle
      (kbench_moe_inputs, same seed and draw order); their SHA-256 digests are stored to pin that."""
    import hashlib
    sys.path.insert(0, os.path.dirname(HERE))
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), ".."))
    from oracle import qmm_oracle as O
    from gguf import GGMLQuantizationType as T
    from gguf.quants import dequantize
    st = _load(os.path.join(ref, "skills/loom-port-llm/starter/st_tensors.py"), "st_tensors")
    out = {}

    # ---- router
    M = {}
    scope = _reference_functions(ref, ["route_ref"], {"np": np, "M": M})
    cases = [("r1", 1, True, False, 1.0, 128, 8), ("r2", 1, False, False, 2.5, 64, 6), ("r3", 2, True, True, 1.0, 64, 6),
             ("r4", 2, False, True, 2.5, 32, 4), ("r5", 3, False, True, 1.0, 32, 4), ("r6", 3, True, False, 1.0, 128, 8)]
    rng = np.random.default_rng(8101)
    for name, gating, norm, has_bias, scale, E, KU in cases:
        M.clear()
        M.update(gating=gating, norm_weights=norm, scale=scale)
        scope["KU"] = KU
        lg = (rng.standard_normal((400, E)) * 2.0).astype(np.float32)
        bias = (rng.standard_normal(E) * 0.5).astype(np.float32) if has_bias else np.zeros(E, np.float32)
        ids, wts, rel = scope["route_ref"](lg, np.eye(E, dtype=np.float32), bias)
        keep = np.flatnonzero(rel > 2e-3)[:96]
        out[f"route_{name}_logits"] = lg[keep]
        out[f"route_{name}_bias"] = bias
        out[f"route_{name}_ids"] = ids[keep].astype(np.int32)
        out[f"route_{name}_wts"] = wts[keep].astype(np.float32)
        out[f"route_{name}_cfg"] = np.array([gating, int(norm), int(has_bias), E, KU], np.int64)
        out[f"route_{name}_scale"] = np.array([scale], np.float64)

    # ---- expert FFN chains (decode precision and the prefill f16 variant); inputs from the oracle's seeded
    # generator, stored as digests; the float weights the reference multiplies come from gguf / st_tensors
    E, H, F, KU, t = 8, 512, 256, 4, 6
    fi = O.ffn_golden_inputs(8102, E, H, F, KU, t)
    out["ffn_digests"] = np.stack([np.frombuffer(hashlib.sha256(np.ascontiguousarray(fi[k]).tobytes()).digest(), np.uint8)
                                   for k in sorted(fi)])
    out["ffn_digest_names"] = np.array(sorted(fi))
    deq = lambda b, n, k: dequantize(b.reshape(-1), T.Q4_0).reshape(n, k).astype(np.float64)   # noqa: E731
    gu_f = [deq(b, 2 * F, H) for b in fi["w_gu"]]
    Wg = np.stack([w[:F] for w in gu_f])
    Wu = np.stack([w[F:] for w in gu_f])
    Wd = np.stack([deq(b, H, F) for b in fi["w_dn"]])
    MGu = st.dequant_mxfp4(fi["mx_gu_nib"], fi["mx_gu_sc"]).astype(np.float64).reshape(E, 2 * F, H)
    MWd = st.dequant_mxfp4(fi["mx_dn_nib"], fi["mx_dn_sc"]).astype(np.float64).reshape(E, H, F)
    x, ids, wts, bg, bu, bd = fi["x"], fi["ids"], fi["wts"], fi["bg"], fi["bu"], fi["bd"]
    dsc, wsg, y0 = fi["dsc"], fi["wsg"], fi["y0"]
    q8_scope = _reference_functions(ref, ["q8_ref"], {"np": np})
    for name, act, eb, oai, mx in [("silu", None, False, False, False), ("gelu", "gelu", False, False, False),
                                   ("oai", None, True, True, False), ("oai_mx", None, True, True, True)]:
        cfg = {"ffn_act": act} if act else {}
        scope = _reference_functions(ref, ["ffn_act", "experts_ref"],
                                     {"np": np, "cfg": cfg, "H": H, "KU": KU, "EB": eb, "OAI": oai,
                                      "M": {"swiglu_limit": 7.0, "swiglu_alpha": 1.702}, "q8_ref": q8_scope["q8_ref"]})
        scope.update(_reference_functions(ref, ["f16_rows"], {"np": np}))
        g_, u_, d_ = (MGu[:, :F], MGu[:, F:], MWd) if mx else (Wg, Wu, Wd)
        for f16 in (False, True):
            y = scope["experts_ref"](x, ids, wts, g_, u_, d_, bg, bu, bd, f16=f16)
            out[f"ffn_{name}_{'p' if f16 else 'd'}_y"] = y.astype(np.float32)
    # the chain with the per-expert down scale and the shared-expert gate (make_kernel_tests.py:3268-3271)
    scope = _reference_functions(ref, ["ffn_act", "experts_ref"],
                                 {"np": np, "cfg": {}, "H": H, "KU": KU, "EB": False, "OAI": False, "M": {},
                                  "q8_ref": q8_scope["q8_ref"]})
    sgv = 1 / (1 + np.exp(-(x.astype(np.float64) @ wsg.astype(np.float64))))
    wts_s = wts * dsc[ids]
    out["ffn_chain_sg"] = sgv.astype(np.float32)
    out["ffn_chain_wts_s"] = wts_s.astype(np.float32)
    out["ffn_chain_y"] = (sgv[:, None] * y0 + scope["experts_ref"](x, ids, wts_s, Wg, Wu, Wd)).astype(np.float32)

    # ---- kbench moe_q4_0 (gen_bench.py:142-248)
    kb = _load(os.path.join(ref, ".github/devlab/kbench/moe_q4_0/gen_bench.py"), "q40_bench_moe")
    H, F, E, U = 2816, 704, 8, 8
    rng = np.random.default_rng(490)
    wg, gu = kb.weights(rng, (E, 2 * F, H))
    wd, down = kb.weights(rng, (E, H, F))
    inp = O.kbench_moe_inputs(490)
    assert np.array_equal(np.asarray(wg).view(np.uint8), inp["wg"]) and np.array_equal(np.asarray(wd).view(np.uint8), inp["wd"])
    out["kb_digests"] = np.stack([np.frombuffer(hashlib.sha256(np.ascontiguousarray(inp[k]).tobytes()).digest(), np.uint8)
                                  for k in sorted(inp)])
    out["kb_digest_names"] = np.array(sorted(inp))
    cols_f = np.sort(np.random.default_rng(7).choice(F, 96, replace=False))
    cols_h = np.sort(np.random.default_rng(8).choice(H, 128, replace=False))
    out["kb_cols_f"], out["kb_cols_h"] = cols_f, cols_h
    for t in (1, 4):
        ids = inp[f"decode_t{t}_ids"]
        x = inp[f"decode_t{t}_x"]
        act = np.empty((t * U, F), np.float64)
        for a, e in enumerate(ids.flat):
            pair = gu[e] @ x[a // U].astype(np.float64)
            act[a] = kb.gelu(pair[:F]) * pair[F:]
        out[f"kb_decode_gu_t{t}"] = act.astype(np.float32)
        xdn = inp[f"decode_t{t}_xdn"]
        out[f"kb_decode_dn_t{t}"] = np.stack([down[e] @ xdn[a].astype(np.float64) for a, e in enumerate(ids.flat)])[:, cols_h].astype(np.float32)
    ti = np.array(O.KB_TILE_INFO, np.int32)
    for t in (63, 65):
        rm, x, s = inp[f"grouped_t{t}_rm"], inp[f"grouped_t{t}_x"], inp[f"grouped_t{t}_s"]
        ref_ = np.full((256, F), 42, np.float64)
        for j, n in enumerate(O.KB_COUNTS[:-1]):
            ref_[j * 64:(j + 1) * 64] = 0
            eid = ti[j, 0]
            for q in range(n):
                src = rm[j * 64 + q] // U
                pair = gu[eid].astype(np.float16).astype(np.float64) @ x[src].astype(np.float64) * s[src, 1]
                ref_[j * 64 + q] = kb.gelu(pair[:F]) * pair[F:]
        out[f"kb_grouped_gu_t{t}"] = ref_[:, cols_f].astype(np.float32)
        xd, sd = inp[f"grouped_t{t}_xd"], inp[f"grouped_t{t}_sd"]
        refdn = np.full((256, H), 42, np.float64)
        for j, n in enumerate(O.KB_COUNTS[:-1]):
            refdn[j * 64:(j + 1) * 64] = (xd[j * 64:(j + 1) * 64].astype(np.float64) @
                                          down[ti[j, 0]].astype(np.float16).astype(np.float64).T * sd[j * 64:(j + 1) * 64, 1:])
        out[f"kb_grouped_dn_t{t}"] = refdn[:, cols_h].astype(np.float32)
    ids, scales, wts, ys = inp["dsc_ids"], inp["dsc_scales"], inp["dsc_wts"], inp["dsc_ys"]
    out["kb_dsc_y"] = np.sum(ys.reshape(4, U, H).astype(np.float64) * (wts * scales[ids])[:, :, None], axis=1).astype(np.float32)
    out["kb_dsc_wts_s"] = (wts * scales[ids]).astype(np.float32)

    np.savez_compressed(os.path.join(HERE, "golden_moe.npz"), **out)
    print("wrote", os.path.join(HERE, "golden_moe.npz"), sum(a.nbytes for a in out.values()), "bytes uncompressed")


def main_formats(ref):
    """golden_formats.npz: the reference's remaining GGUF formats (formats.py:5-17: Q5_0, Q8_0, Q3_K, Q5_K, Q6_K,
    IQ4_XS, IQ3_S) dequantised by gguf 0.19.0 (the reference's numpy path, make_kernel_tests.py:45-47) on seeded random
    blocks with finite f16 scales, and small float64 products of those values (make_kernel_tests.py:231-238)."""
    from gguf import GGMLQuantizationType as T
    from gguf.quants import dequantize
    out = {}
    rng = np.random.default_rng(77)
    spec = {"q5_0": (22, 32, [0]), "q8_0": (34, 32, [0]), "q3_k": (110, 256, [108]), "q5_k": (176, 256, [0, 2]),
            "q6_k": (210, 256, [208]), "iq4_xs": (136, 256, [0]), "iq3_s": (110, 256, [0])}
    for name, (bb, qk, offs) in spec.items():
        nb = 64 if qk == 256 else 512
        b = rng.integers(0, 256, (nb, bb), dtype=np.uint8)
        for o in offs:
            b[:, o:o + 2] = (rng.uniform(1e-4, 4e-2, nb) * rng.choice([-1, 1], nb)).astype(np.float16).view(
                np.uint8).reshape(-1, 2)
        out[f"{name}_raw"] = b
        out[f"{name}_f32"] = dequantize(b.reshape(-1), T[name.upper()]).reshape(nb, -1).astype(np.float32)
        # a matvec: 48 rows of 512 values, 3 tokens
        n, k, t = 48, 512, 3
        rows = rng.integers(0, 256, (n * k // qk, bb), dtype=np.uint8)
        for o in offs:
            rows[:, o:o + 2] = (rng.uniform(1e-3, 2e-2, len(rows)) * rng.choice([-1, 1], len(rows))).astype(
                np.float16).view(np.uint8).reshape(-1, 2)
        W = dequantize(rows.reshape(-1), T[name.upper()]).reshape(n, k).astype(np.float64)
        x = rng.standard_normal((t, k)).astype(np.float32)
        out[f"mv_{name}_w"] = rows.reshape(n, -1)
        out[f"mv_{name}_x"] = x
        out[f"mv_{name}_y"] = x.astype(np.float64) @ W.T
    np.savez_compressed(os.path.join(HERE, "golden_formats.npz"), **out)
    print("wrote", os.path.join(HERE, "golden_formats.npz"), sum(a.nbytes for a in out.values()), "bytes uncompressed")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py LOOM_SKILLS_CHECKOUT")
    main(sys.argv[1])
    main_moe(sys.argv[1])
    main_formats(sys.argv[1])
