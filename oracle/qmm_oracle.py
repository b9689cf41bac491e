"""CPU oracle for the quantized-matmul hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product path imports this module. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only as the checker or as the timed CPU
restatement of the reference's own numpy path.

It restates, in numpy, the numerics of loom-fun/loom-skills for this path (paths relative to the reference root):

* block formats and their dequantisation
  - Q4_0     ``skills/loom-port-llm/starter/quant_values.loom:386-408`` (@g_q4_0_values), ``formats.py:8``
  - Q4_K     ``skills/loom-port-llm/starter/gen_llm.py:234-315`` (@g_k_scale_minimum, @g_k_metadata, @g_q4_k_values)
  - IQ4_NL   ``skills/loom-port-llm/starter/quant_values.loom:18-91``
  - IQ3_S    ``skills/loom-port-llm/starter/quant_values.loom:5-6, 243-384`` (@g_iq3s_grid, @g_iq3_s_values)
  - MXFP4    ``skills/loom-port-llm/starter/gen_llm.py:786-895`` (ggml 17-byte blocks, split16 order) and
             ``skills/loom-port-llm/starter/st_tensors.py:26-35`` (split planes, pairs order)
  The Q4_K / IQ4_NL / MXFP4 arithmetic is the third-party ``gguf`` package's (gguf-py 0.19.0, installed unpinned by
  ``skills/loom-setup/scripts/install_loom.sh:118``; called at ``make_kernel_tests.py:15-16, 45-47``). This file
  restates that published algorithm; ``tests/test_oracle.py`` pins it against gguf 0.19.0 bit for bit.
* the f16 GEMM staging (one rounding): ``moe_q4_0.py:11-38``, ``gen_gemm.py:159-279`` (IQ4), ``gen_gemm.py:499-532`` (Q4_K)
* activation producers: ``gen_llm.py:1843-1912`` (g_row_scale_f16), ``gen_mxfp4s.py:852-870`` (F8_SCALE),
  e4m3 rounding ``make_kernel_tests.py:2006-2019``; MXFP4 -> e5m2 decode ``gen_mxfp4s.py:14-48``
* products: ``make_kernel_tests.py:45-47, 231-238`` (matvec), ``:1860-1876`` (GEMM: (x16 . W^T) * inv)
* MoE: router ``gen_moe.py:116-253``, bucket ``gen_moe.py:829-955``, grouped GEMM ``gen_moe.py:1126-1228``,
  combine ``gen_moe.py:730-762, 1231-1280``, reference F64 pipeline ``.github/devlab/kbench/moe_q4_0/gen_bench.py:185-248``;
  the decode-size layer (expert matvecs ``gen_moe.py:535-727`` below the GEMM threshold of ``gen_llm.py:6107``), also
  over MXFP4 experts.

The quantisers below are test-input generators (seeded synthetic weights), not part of the reference path:
Q4_0 restates gguf's quantiser; Q4_K, IQ4_NL and MXFP4 are this repository's own (gguf 0.19.0 cannot quantise Q4_K
or IQ4_NL, and its MXFP4 quantiser picks max/scale in [4, 8) and saturates, which the MXFP4 config rules out).
"""
from __future__ import annotations

import numpy as np

# values per block / bytes per block (formats.py:5-17) and gguf.GGMLQuantizationType ids
QK = {"q4_0": 32, "q4_k": 256, "iq4_nl": 32, "mxfp4": 32, "q8_0": 32, "q5_0": 32, "q5_k": 256, "q6_k": 256,
      "iq4_xs": 256, "q3_k": 256, "iq3_s": 256}
BLOCK_BYTES = {"q4_0": 18, "q4_k": 144, "iq4_nl": 18, "mxfp4": 17, "q8_0": 34, "q5_0": 22, "q5_k": 176, "q6_k": 210,
               "iq4_xs": 136, "q3_k": 110, "iq3_s": 110}
GGML_TYPE = {"q4_0": 2, "q4_k": 12, "iq4_nl": 20, "mxfp4": 39, "q8_0": 8, "q5_0": 6, "q5_k": 13, "q6_k": 14,
             "iq4_xs": 23, "q3_k": 11, "iq3_s": 21}


def iq3s_grid():
    """The IQ3_S codebook [512][4] of odd magnitudes 1..15 (ggml's iq3s_grid; the reference embeds the same table,
    quant_values.loom:5-6): gguf-py 0.19.0's IQ3_S grid, the format's pinned definition."""
    from gguf.quants import IQ3_S
    IQ3_S.init_grid()
    return IQ3_S.grid.reshape(512, 4).astype(np.int64)
IQ4_KVALUES = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.int64)
E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float64)
MXFP4_F8_SHIFT = 8                      # gen_mxfp4s.py:29
MXFP4_F8_E_MIN, MXFP4_F8_E_MAX = 107, 132


def row_bytes(fmt, k):
    """Packed bytes of one weight row of k values (gen_moe.py:70-71)."""
    assert k % QK[fmt] == 0, (fmt, k)
    return k // QK[fmt] * BLOCK_BYTES[fmt]


# ------------------------------------------------------------------------------------------------------------------
# quantisers (seeded test-input generators)
# ------------------------------------------------------------------------------------------------------------------
def quantize_q4_0(w):
    """float32 [..., k] -> packed Q4_0 bytes [..., k/32*18]. Restates gguf 0.19.0 quants.Q4_0.quantize_blocks:
    d = (value of largest magnitude) / -8, q = clip(trunc(x/d + 8.5), 0, 15), d stored as f16."""
    w = np.asarray(w, np.float32)
    lead = w.shape[:-1]
    blocks = w.reshape(-1, 32)
    imax = np.abs(blocks).argmax(axis=-1)[:, None]
    mx = np.take_along_axis(blocks, imax, axis=-1)
    d = mx / np.float32(-8)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = np.trunc(blocks * inv + np.float32(8.5)).astype(np.float32).astype(np.uint8).clip(0, 15)
    packed = q[:, :16] | (q[:, 16:] << np.uint8(4))
    out = np.concatenate([d.astype(np.float16).view(np.uint8), packed], axis=-1)
    return out.reshape(*lead, -1)


def _pack_k_scales(sc, mn):
    """8 six-bit scales and minima -> the 12-byte K-quant scale field (layout of gguf Q4_K.get_scale_min)."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.zeros(sc.shape[:-1] + (12,), np.uint8)
    out[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = (mn[..., 0:4] & 63) | ((mn[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 15) | ((mn[..., 4:8] & 15) << 4)
    return out


def quantize_q4_k(w):
    """float32 [..., k] -> packed Q4_K bytes [..., k/256*144] (this repository's own min/max quantiser).

    Per 32-value group: scale = (max - min)/15, minimum = -min(0, min); super-block d = max scale/63, dmin = max
    minimum/63 (f16); 6-bit codes sc = round(scale/d), m = round(minimum/dmin); q = round((x + dmin*m)/(d*sc))."""
    w = np.asarray(w, np.float32)
    lead = w.shape[:-1]
    g = w.reshape(-1, 8, 32).astype(np.float64)
    lo = np.minimum(g.min(-1), 0.0)
    hi = g.max(-1)
    scale = (hi - lo) / 15.0
    minimum = -lo
    d16 = (scale.max(-1) / 63.0).astype(np.float16)
    dm16 = (minimum.max(-1) / 63.0).astype(np.float16)
    d = d16.astype(np.float64)[:, None]
    dm = dm16.astype(np.float64)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d > 0, np.clip(np.rint(scale / d), 0, 63), 0).astype(np.int64)
        mn = np.where(dm > 0, np.clip(np.rint(minimum / dm), 0, 63), 0).astype(np.int64)
        step = d * sc
        off = dm * mn
        q = np.where(step[..., None] > 0, np.clip(np.rint((g + off[..., None]) / step[..., None]), 0, 15), 0)
    q = q.astype(np.uint8)                                   # [B, 8, 32]
    qs = (q[:, 0::2, :] | (q[:, 1::2, :] << 4)).reshape(-1, 128)   # page p: group 2p low nibble, 2p+1 high nibble
    out = np.concatenate([d16.view(np.uint8).reshape(-1, 2), dm16.view(np.uint8).reshape(-1, 2),
                          _pack_k_scales(sc, mn), qs], axis=-1)
    return out.reshape(*lead, -1)


def quantize_iq4_nl(w):
    """float32 [..., k] -> packed IQ4_NL bytes [..., k/32*18] (own quantiser): d = (value of largest magnitude)/-127
    in f16, code = nearest kvalue of x/d (ties: lowest index)."""
    w = np.asarray(w, np.float32)
    lead = w.shape[:-1]
    blocks = w.reshape(-1, 32).astype(np.float64)
    imax = np.abs(blocks).argmax(axis=-1)[:, None]
    mx = np.take_along_axis(blocks, imax, axis=-1)
    d16 = (mx / -127.0).astype(np.float16)
    d = d16.astype(np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = np.where(d != 0, blocks / d, 0.0)
    # nearest codebook entry; a value exactly between two entries takes the lower index
    mid = (IQ4_KVALUES[:-1] + IQ4_KVALUES[1:]) / 2.0
    idx = np.searchsorted(mid, v, side="left").astype(np.uint8)
    packed = idx[:, :16] | (idx[:, 16:] << np.uint8(4))
    out = np.concatenate([d16.view(np.uint8).reshape(-1, 2), packed], axis=-1)
    return out.reshape(*lead, -1)


def _e2m1_codes(v):
    """float64 values in [-6, 6] -> nearest e2m1 codes (bit 3 = sign), ties to the even table index."""
    a = np.abs(v)
    mid = (E2M1[:-1] + E2M1[1:]) / 2.0
    mag = np.searchsorted(mid, a, side="left")            # ties -> the lower magnitude ...
    tie = (mag < 7) & (a == mid[np.minimum(mag, 6)]) & (mag % 2 == 1)
    mag = mag + tie                                       # ... unless that index is odd: ties to even
    sign = (v < 0) & (mag > 0)
    return (mag | (sign << 3)).astype(np.uint8)


def quantize_mxfp4(w, layout="planar"):
    """float32 [..., k] -> MXFP4 (own quantiser): e8m0 e = ceil(log2(amax/6)) + 127 so every |x| / 2^(e-127) <= 6,
    then the nearest e2m1 code. layout "planar" -> (nibbles [..., k/2] in pairs order, scales [..., k/32]);
    layout "ggml" -> 17-byte blocks [..., k/32*17] (e8m0 byte, then element i low / i+16 high nibble)."""
    w = np.asarray(w, np.float32)
    lead = w.shape[:-1]
    blocks = w.reshape(-1, 32).astype(np.float64)
    amax = np.abs(blocks).max(-1)
    with np.errstate(divide="ignore"):
        e = np.where(amax > 0, np.ceil(np.log2(amax / 6.0)) + 127, 0)
    e = np.clip(e, 0, 254).astype(np.int64)
    s = np.exp2(e.astype(np.float64) - 127)
    codes = _e2m1_codes(np.clip(blocks / s[:, None], -6, 6))   # [B, 32]
    if layout == "ggml":
        packed = codes[:, :16] | (codes[:, 16:] << 4)
        out = np.concatenate([e.astype(np.uint8)[:, None], packed], axis=-1)
        return out.reshape(*lead, -1)
    nib = (codes[:, 0::2] | (codes[:, 1::2] << 4)).reshape(*lead, -1)
    return nib, e.astype(np.uint8).reshape(*lead, -1)


# ------------------------------------------------------------------------------------------------------------------
# dequantisation: exact f32 values (gguf / @g_<fmt>_values) and the GEMM's f16 staging (one rounding)
# ------------------------------------------------------------------------------------------------------------------
def q4_k_scale_min(scales):
    """12-byte scale fields [B, 12] -> (sc [B, 8], m [B, 8]) 6-bit codes (gen_llm.py:234-266)."""
    s = scales.astype(np.int64)
    d, m, md = s[:, 0:4], s[:, 4:8], s[:, 8:12]
    sc = np.concatenate([d & 63, (md & 15) | ((d >> 2) & 48)], axis=-1)
    mn = np.concatenate([m & 63, (md >> 4) | ((m >> 2) & 48)], axis=-1)
    return sc, mn


def _f16(raw2):
    return np.ascontiguousarray(raw2).view(np.float16).reshape(-1)


def _codes4(qs):
    """16 packed bytes [B, 16] -> 32 nibble codes [B, 32]: element i = low nibble of byte i, i+16 = high nibble."""
    return np.concatenate([qs & 15, qs >> 4], axis=-1).astype(np.int64)


def _q5k_codes(b):
    """Q5_K 5-bit codes [B, 8 groups, 32]: nibble of page g/2 (low for even g) | bit g of qh[l] << 4 (gguf Q5_K)."""
    qh = b[:, 16:48].astype(np.int64)
    hb = (qh[:, None, :] >> np.arange(8).reshape(1, 8, 1)) & 1
    qs = b[:, 48:].reshape(-1, 4, 1, 32) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)
    return (qs & 15).reshape(-1, 8, 32).astype(np.int64) | (hb << 4)


def _q6k_codes(b):
    """Q6_K 6-bit codes 0..63 [B, 16 sub-blocks, 16] (gguf Q6_K: ql nibbles, qh 2-bit fields)."""
    ql, qh = b[:, :128], b[:, 128:192]
    lo = (ql.reshape(-1, 2, 1, 64) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)) & 15
    hi = (qh.reshape(-1, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)) & 3
    return (lo.reshape(-1, 8, 32).astype(np.int64) | (hi.reshape(-1, 8, 32).astype(np.int64) << 4)).reshape(-1, 16, 16)


def dequant(fmt, raw, k):
    """Packed rows [..., row_bytes] (or (nibbles, scales) for planar MXFP4) -> float32 [..., k], the exact values
    the reference's numpy path uses (gguf.quants.dequantize; quant_values.loom / gen_llm.py helpers)."""
    if fmt == "mxfp4_planar":
        nib, sc = raw
        lead = nib.shape[:-1]
        nib = nib.reshape(-1, 16)
        lo = E2M1[nib & 7] * np.where(nib & 8, -1.0, 1.0)
        hi = E2M1[(nib >> 4) & 7] * np.where(nib & 128, -1.0, 1.0)
        v = np.stack([lo, hi], -1).reshape(-1, 32)
        s = np.exp2(sc.reshape(-1).astype(np.float64) - 127.0)
        return (v * s[:, None]).astype(np.float32).reshape(*lead, k)
    raw = np.asarray(raw, np.uint8)
    lead = raw.shape[:-1]
    b = raw.reshape(-1, BLOCK_BYTES[fmt])
    if fmt == "q4_0":
        d = _f16(b[:, 0:2]).astype(np.float32)
        v = d[:, None] * (_codes4(b[:, 2:]) - 8).astype(np.float32)
    elif fmt == "iq4_nl":
        d = _f16(b[:, 0:2]).astype(np.float32)
        v = d[:, None] * IQ4_KVALUES[_codes4(b[:, 2:])].astype(np.float32)
    elif fmt == "q4_k":
        d = _f16(b[:, 0:2]).astype(np.float32)
        dmin = _f16(b[:, 2:4]).astype(np.float32)
        sc, mn = q4_k_scale_min(b[:, 4:16])
        a = d[:, None] * sc.astype(np.float32)                       # [B, 8] exact in f32
        c = dmin[:, None] * mn.astype(np.float32)
        qs = b[:, 16:].reshape(-1, 4, 1, 32) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)
        q = (qs & 15).reshape(-1, 8, 32).astype(np.float32)
        v = (a[:, :, None] * q - c[:, :, None]).reshape(-1, 256)
    elif fmt == "q8_0":      # gguf Q8_0.dequantize_blocks: d * int8 code
        d = _f16(b[:, 0:2]).astype(np.float32)
        v = d[:, None] * b[:, 2:].view(np.int8).astype(np.float32)
    elif fmt == "q5_0":      # gguf Q5_0: q = nibble | bit j of the u32 qh << 4; d * (q - 16)
        d = _f16(b[:, 0:2]).astype(np.float32)
        qh = np.ascontiguousarray(b[:, 2:6]).view("<u4").reshape(-1, 1).astype(np.int64)
        hb = (qh >> np.arange(32)) & 1
        q = _codes4(b[:, 6:]) | (hb << 4)
        v = d[:, None] * (q - 16).astype(np.float32)
    elif fmt == "q5_k":      # gguf Q5_K: Q4_K's header and nibble pages, qh bit g of byte l = 5th bit of value l of group g
        d = _f16(b[:, 0:2]).astype(np.float32)
        dmin = _f16(b[:, 2:4]).astype(np.float32)
        sc, mn = q4_k_scale_min(b[:, 4:16])
        a = d[:, None] * sc.astype(np.float32)
        c = dmin[:, None] * mn.astype(np.float32)
        v = (a[:, :, None] * _q5k_codes(b).astype(np.float32) - c[:, :, None]).reshape(-1, 256)
    elif fmt == "q6_k":      # gguf Q6_K: ql[128] qh[64] int8 scales[16] f16 d; (d * sc[v/16]) * (q - 32)
        sc = b[:, 192:208].view(np.int8).astype(np.float32)
        d = _f16(b[:, 208:210]).astype(np.float32)
        dl = (d[:, None] * sc).reshape(-1, 16, 1)
        v = (dl * (_q6k_codes(b) - 32).astype(np.float32)).reshape(-1, 256)
    elif fmt == "iq4_xs":    # gguf IQ4_XS: 6-bit sub-block scales (4 low bits in scales_l, 2 high in scales_h) - 32
        d = _f16(b[:, 0:2]).astype(np.float32)
        sh = np.ascontiguousarray(b[:, 2:4]).view("<u2").reshape(-1, 1).astype(np.int64)
        sl = b[:, 4:8].astype(np.int64)
        lo = (sl.reshape(-1, 4, 1) >> np.array([0, 4]).reshape(1, 1, 2)).reshape(-1, 8) & 15
        hi = (sh >> (2 * np.arange(8)).reshape(1, 8)) & 3
        dl = d[:, None] * ((lo | (hi << 4)) - 32).astype(np.float32)   # [B, 8]
        q = _codes4(b[:, 8:].reshape(-1, 16)).reshape(-1, 8, 32)
        v = (dl[:, :, None] * IQ4_KVALUES[q].astype(np.float32)).reshape(-1, 256)
    elif fmt == "q3_k":      # gguf Q3_K: hmask[32] qs[64] 12 bytes of 6-bit scales, f16 d; q = 2 bits - 4 * !hbit
        hmask, qs, scb = b[:, :32], b[:, 32:96], b[:, 96:108]
        d = _f16(b[:, 108:110]).astype(np.float32)
        ls = (scb[:, :8].reshape(-1, 1, 8) >> np.array([0, 4], np.uint8).reshape(1, 2, 1)).reshape(-1, 16) & 15
        hs = (scb[:, 8:].reshape(-1, 1, 4) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 4, 1)).reshape(-1, 16) & 3
        scl = ((ls | (hs << 4)).astype(np.int64) - 32).astype(np.float32)
        dl = (d[:, None] * scl).reshape(-1, 16, 1)
        ql = (qs.reshape(-1, 2, 1, 32) >> np.array([0, 2, 4, 6], np.uint8).reshape(1, 1, 4, 1)).reshape(-1, 16, 16) & 3
        hb = (hmask.reshape(-1, 1, 1, 32) >> np.arange(8, dtype=np.uint8).reshape(1, 1, 8, 1)).reshape(-1, 16, 16) & 1
        q = ql.astype(np.int64) - ((hb ^ 1).astype(np.int64) << 2)
        v = (dl * q.astype(np.float32)).reshape(-1, 256)
    elif fmt == "iq3_s":     # gguf IQ3_S: d, qs[64], qh[8], signs[32], scales[4] (quant_values.loom:243-384)
        d = _f16(b[:, 0:2]).astype(np.float32)
        qs, qh, sg, sc = b[:, 2:66], b[:, 66:74], b[:, 74:106], b[:, 106:110]
        s = (sc.reshape(-1, 4, 1) >> np.array([0, 4], np.uint8).reshape(1, 1, 2)).reshape(-1, 8) & 15
        db = d[:, None] * (1 + 2 * s.astype(np.int64)).astype(np.float32)              # [B, 8], exact
        hi = (qh.reshape(-1, 8, 1) >> np.arange(8, dtype=np.uint8).reshape(1, 1, 8)).reshape(-1, 64) & 1
        idx = qs.astype(np.int64) | (hi.astype(np.int64) << 8)                          # [B, 64] codebook entries
        mag = iq3s_grid()[idx].reshape(-1, 256)
        neg = (sg.reshape(-1, 32, 1) >> np.arange(8, dtype=np.uint8).reshape(1, 1, 8)).reshape(-1, 256) & 1
        q = np.where(neg == 1, -mag, mag).astype(np.float32).reshape(-1, 8, 32)
        v = (db[:, :, None] * q).reshape(-1, 256)
    elif fmt == "mxfp4":
        e = b[:, 0].astype(np.int64)
        # ggml_e8m0_to_fp32_half: 2^(e-128) (e >= 2), subnormal encodings for e < 2; doubled e2m1 table
        half = np.where(e < 2, np.exp2(e.astype(np.float64) - 128), np.exp2(e.astype(np.float64) - 128))
        kv = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], np.float64)
        v = (half[:, None] * kv[_codes4(b[:, 1:])]).astype(np.float32)
    else:
        raise ValueError(fmt)
    return v.astype(np.float32).reshape(*lead, k)


def dequant_f16(fmt, raw, k):
    """The f16 weights the prefill GEMM stages (one rounding of the exact value):
    Q4_0 f16(d*(q-8)) (moe_q4_0.py:36-38); IQ4_NL f16(d*kvalue) (gen_gemm.py:228-231);
    Q4_K fma_f16(q, f16(d*sc), f16(-dmin*m)) (gen_gemm.py:526-532)."""
    if fmt in ("q4_0", "iq4_nl", "mxfp4", "mxfp4_planar", "q8_0", "q5_0", "iq4_xs", "q3_k", "iq3_s"):
        # one rounding of the exact value (gen_gemm.py:352-367 for Q8_0; the @g_<fmt>_values helpers + fptrunc)
        return dequant(fmt, raw, k).astype(np.float64).astype(np.float16)
    if fmt in ("q5_k", "q6_k"):
        return _dequant_f16_fma(fmt, raw, k)
    assert fmt == "q4_k"
    raw = np.asarray(raw, np.uint8)
    lead = raw.shape[:-1]
    b = raw.reshape(-1, 144)
    d = _f16(b[:, 0:2]).astype(np.float32)
    dmin = _f16(b[:, 2:4]).astype(np.float32)
    sc, mn = q4_k_scale_min(b[:, 4:16])
    a16 = (d[:, None] * sc.astype(np.float32)).astype(np.float16).astype(np.float64)
    c16 = (-(dmin[:, None] * mn.astype(np.float32))).astype(np.float16).astype(np.float64)
    qs = b[:, 16:].reshape(-1, 4, 1, 32) >> np.array([0, 4], np.uint8).reshape(1, 1, 2, 1)
    q = (qs & 15).reshape(-1, 8, 32).astype(np.float64)
    v = q * a16[:, :, None] + c16[:, :, None]          # exact in f64; one rounding to f16 = the f16 fma
    with np.errstate(over="ignore"):
        return v.reshape(-1, 256).astype(np.float16).reshape(*lead, k)


def _dequant_f16_fma(fmt, raw, k):
    """The GEMM staging of Q5_K / Q6_K (gen_gemm.py:369-444, 445-498): fma_f16(q, f16(scale), f16(offset)) with
    Q5_K: q = 5-bit code, scale = d*sc, offset = -dmin*m (as Q4_K); Q6_K: q = 6-bit code (0..63), scale = d*sc,
    offset = -32*d*sc (both f32 products, exact). q * scale16 + offset16 is exact in f64, so its one rounding to f16
    is the f16 fma."""
    raw = np.asarray(raw, np.uint8)
    lead = raw.shape[:-1]
    b = raw.reshape(-1, BLOCK_BYTES[fmt])
    if fmt == "q5_k":
        d = _f16(b[:, 0:2]).astype(np.float32)
        dmin = _f16(b[:, 2:4]).astype(np.float32)
        sc, mn = q4_k_scale_min(b[:, 4:16])
        a16 = (d[:, None] * sc.astype(np.float32)).astype(np.float16).astype(np.float64)[:, :, None]
        c16 = (-(dmin[:, None] * mn.astype(np.float32))).astype(np.float16).astype(np.float64)[:, :, None]
        q = _q5k_codes(b).astype(np.float64)                                     # [B, 8, 32]
    else:
        s32 = _f16(b[:, 208:210]).astype(np.float32)[:, None] * b[:, 192:208].view(np.int8).astype(np.float32)
        a16 = s32.astype(np.float16).astype(np.float64)[:, :, None]              # [B, 16, 1]
        c16 = (s32 * np.float32(-32)).astype(np.float16).astype(np.float64)[:, :, None]
        q = _q6k_codes(b).astype(np.float64)                                     # [B, 16, 16]
    with np.errstate(over="ignore", invalid="ignore"):
        return (q * a16 + c16).reshape(-1, 256).astype(np.float16).reshape(*lead, k)


# ------------------------------------------------------------------------------------------------------------------
# activation producers
# ------------------------------------------------------------------------------------------------------------------
def _f32_exponent_field(a):
    return (np.asarray(a, np.float32).view(np.uint32) >> 23) & 255


def quant_q8(x):
    """g_quant_q8 (gen_llm.py:683-750; llama.cpp quantize_q8_1): per 32-value group d = amax / 127 (f32 division),
    q = round(x / d) half away from zero (0 when amax == 0), codes int8 [rows][k]; meta f32 [rows][k/32][2] =
    (f32(f16(d)), sum of q). make_kernel_tests.py:32-40 (q8_ref) dequantises with the same f16-rounded d."""
    x = np.asarray(x, np.float32)
    rows, k = x.shape
    g = x.reshape(rows, k // 32, 32)
    amax = np.abs(g).max(-1, keepdims=True)
    d = (amax / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = (g / d).astype(np.float32)
    t = np.trunc(v)
    r = t + np.where(np.abs(v - t) >= np.float32(0.5), np.sign(v), np.float32(0))   # roundf: halves away from zero
    q = np.where(amax > 0, r, 0).astype(np.int8)
    meta = np.stack([d[..., 0].astype(np.float16).astype(np.float32), q.astype(np.int32).sum(-1).astype(np.float32)],
                    -1)
    return q.reshape(rows, k), meta.astype(np.float32)


def dequant_q8(codes, meta):
    """The activations the _q8 matvecs contract with: code * f16-rounded d per 32-value group."""
    rows, k = codes.shape
    return (codes.reshape(rows, k // 32, 32).astype(np.float64) * meta[..., :1].astype(np.float64)).reshape(rows, k)


def row_scale_f16(x):
    """g_row_scale_f16 (gen_llm.py:1843-1912): per row e = clamp(exp(max|x|) - 127 - 13, 0, 100), s = 2^-e,
    x16 = f16(x * s), scales[row] = (s, 2^e)."""
    x = np.asarray(x, np.float32)
    mx = np.abs(x).max(-1)
    biased = _f32_exponent_field(mx).astype(np.int64)
    e = np.clip(biased - 127 - 13, 0, 100)
    s = ((127 - e).astype(np.uint32) << 23).view(np.float32)
    inv = ((127 + e).astype(np.uint32) << 23).view(np.float32)
    x16 = (x * s[:, None]).astype(np.float16)
    return x16, np.stack([s, inv], -1).astype(np.float32)


def e4m3_round(x):
    """Nearest finite e4m3fn values, round to nearest even, saturating at 448 (make_kernel_tests.py:2006-2011)."""
    x = np.asarray(x, np.float64)
    a = np.minimum(np.abs(x), 448.0)
    e = np.maximum(np.floor(np.log2(np.maximum(a, 2.0 ** -20))), -6)
    q = 2.0 ** (e - 3)
    return np.sign(x) * np.minimum(np.rint(a / q) * q, 448.0)


def e4m3_bytes(v):
    """e4m3fn values -> bytes (make_kernel_tests.py:2012-2019); negative values rounding to zero keep -0."""
    v = np.asarray(v, np.float64)
    a = np.abs(v)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -20))).astype(np.int64)
    sub = a < 2.0 ** -6
    ef = np.where(sub, 0, e + 7)
    with np.errstate(invalid="ignore"):
        mant = np.where(sub, np.rint(a / 2.0 ** -9), np.rint((a / 2.0 ** e - 1) * 8)).astype(np.int64)
    b = np.where(a == 0, 0, (ef << 3) | mant) | np.where(np.signbit(v), 0x80, 0)
    return b.astype(np.uint8)


def e4m3_values(b):
    """e4m3fn bytes -> float64."""
    b = np.asarray(b, np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    ef = (b >> 3) & 15
    m = b & 7
    v = np.where(ef == 0, m * 2.0 ** -9, (1 + m / 8.0) * 2.0 ** (ef - 7))
    v = np.where((ef == 15) & (m == 7), np.nan, v)
    return s * v


def row_scale_f8(x):
    """The fp8 producer twin (gen_mxfp4s.py:852-870, 887-938): per row biased = exponent field of max|x|,
    scale = 2^(134 - biased) and inverse 2^(biased - 142) (both clamped to normal exponents 1..254),
    x8 = e4m3(x * scale): the row max lands in [128, 256); s8[row] = (scale, inverse) -- the inverse carries the
    2^-8 of the weights held at 2^8 times their value."""
    x = np.asarray(x, np.float32)
    mx = np.abs(x).max(-1)
    biased = _f32_exponent_field(mx).astype(np.int64)
    sf = np.clip(261 - biased, 1, 254)
    inf_ = np.clip(biased - (7 + MXFP4_F8_SHIFT), 1, 254)
    s = (sf.astype(np.uint32) << 23).view(np.float32)
    inv = (inf_.astype(np.uint32) << 23).view(np.float32)
    x8 = e4m3_bytes(e4m3_round(x.astype(np.float64) * s[:, None].astype(np.float64)))
    return x8, np.stack([s, inv], -1).astype(np.float32)


def mxfp4_e5m2_bytes(e, q):
    """MXFP4 nibble -> the e5m2 byte holding fp4 * 2^(e - 127 + 8) (gen_mxfp4s.py:14-27): sign | (base[m] + 4*(e-107)),
    base = 8 12 14 16 18 20 22 for m = 1..7, zero stays zero. e [..] uint8, q [..] nibble codes."""
    e = np.asarray(e, np.int64)
    q = np.asarray(q, np.int64)
    base = np.array([0, 8, 12, 14, 16, 18, 20, 22], np.int64)
    m = q & 7
    mag = np.where(m == 0, 0, base[m] + 4 * (e - MXFP4_F8_E_MIN))
    return (mag | ((q & 8) << 4)).astype(np.uint8)


def e5m2_values(b):
    b = np.asarray(b, np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    ef = (b >> 2) & 31
    m = b & 3
    return s * np.where(ef == 0, m * 2.0 ** -16, (1 + m / 4.0) * 2.0 ** (ef - 15))


# ------------------------------------------------------------------------------------------------------------------
# products (float64, as make_kernel_tests.py builds its references)
# ------------------------------------------------------------------------------------------------------------------
def silu(x):
    with np.errstate(over="ignore"):   # exp(-x) = inf for very negative x: silu -> -0, as in f32
        return x / (1.0 + np.exp(-x))


def mv_ref(fmt, w, x, n, k, w2=None, y_old=None, fmt2=None):
    """Decode matvec (gen_llm.py:1159-1378; reference make_kernel_tests.py:231-238):
    y[t, n] (+)= sum_k x[t, k] W[n, k]; with w2: y = silu(x.Wg) * (x.Wu), w2 in fmt2 when the up weight's format
    differs (gen_moe.py:537-552 "GATE+UP"; gen_llm.py:6280-6283 two projections + g_silu_mul)."""
    W = dequant(fmt, w, k).reshape(n, k).astype(np.float64)
    x = np.asarray(x, np.float64).reshape(-1, k)
    y = x @ W.T
    if w2 is not None:
        U = dequant(fmt2 or fmt, w2, k).reshape(n, k).astype(np.float64)
        y = silu(y) * (x @ U.T)
    if y_old is not None:
        y = y + np.asarray(y_old, np.float64)
    return y


def gemm_ref(fmt, w, x16, scales, n, k, mode="store", w2=None, y_old=None, fmt2=None):
    """Prefill GEMM (gen_gemm.py:535-704; reference make_kernel_tests.py:1860-1876):
    Y = (X16 . W^T) * inv[row]; mode acc adds y_old; swiglu: silu(G) * U, w2 in fmt2 when it differs (gen_gemm.py:535-545
    fmt2)."""
    W = dequant(fmt, w, k).reshape(n, k).astype(np.float64)
    x = np.asarray(x16, np.float64).reshape(-1, k)
    inv = np.asarray(scales, np.float64)[:, 1:2]
    y = (x @ W.T) * inv
    if mode == "swiglu":
        U = dequant(fmt2 or fmt, w2, k).reshape(n, k).astype(np.float64)
        y = silu(y) * ((x @ U.T) * inv)
    elif mode == "acc":
        y = y + np.asarray(y_old, np.float64)
    return y


def gemm_mxfp4_f8_ref(x8, s8, nib, sc, n, k, order="pairs"):
    """MXFP4 x FP8 GEMM (gen_mxfp4s.py:50-500; kbench gemm_mxfp4s/gen_bench.py:284-291):
    y = (e4m3(x8) . (W * 2^8)^T) * s8[row, 1], W the exact MXFP4 values."""
    W = dequant_mxfp4_planar(nib, sc, n, k, order)
    a = e4m3_values(x8).reshape(-1, k)
    return (a @ (W * 2.0 ** MXFP4_F8_SHIFT).T) * np.asarray(s8, np.float64)[:, 1:2]


def dequant_mxfp4_planar(nib, sc, n, k, order="pairs"):
    """Split planes (nibbles [n, k/2], scales [n, k/32]) -> float64 [n, k] in the given nibble order
    (kbench gemm_mxfp4s/gen_bench.py:284-291: "pairs" = element 2j low nibble of byte j; "split16" = ggml order)."""
    nib = np.asarray(nib, np.uint8).reshape(n, k // 2)
    lo = E2M1[nib & 7] * np.where(nib & 8, -1.0, 1.0)
    hi = E2M1[(nib >> 4) & 7] * np.where(nib & 128, -1.0, 1.0)
    lo, hi = lo.reshape(n, -1, 16), hi.reshape(n, -1, 16)
    blk = np.stack([lo, hi], 3).reshape(n, -1, 32) if order == "pairs" else np.concatenate([lo, hi], 2)
    return (blk * np.exp2(np.asarray(sc, np.float64).reshape(n, -1, 1) - 127)).reshape(n, k)


# ------------------------------------------------------------------------------------------------------------------
# MoE
# ------------------------------------------------------------------------------------------------------------------
def route_ref(logits, ku, gating=1, norm=True, bias=None, scale=1.0):
    """Router top-k (gen_moe.py:116-253): gating 1 softmax over all experts then top-k, gating 2 sigmoid (+bias for
    the pick), gating 3 top-k of the (biased) logits weighted by a softmax over the picked. Ties: lowest index.
    norm: w / max(sum, 6.103515625e-05) (gating 1 and 2); the final weights times `scale` (expert_weights_scale,
    gen_moe.py:111-113; make_kernel_tests.py:3166-3186 applies it for every gating). f32 arithmetic as the kernels'."""
    lg = np.asarray(logits, np.float32)
    t, E = lg.shape
    if gating == 1:
        m = lg.max(-1, keepdims=True)
        ex = np.exp((lg - m).astype(np.float32))
        prob = (ex / ex.sum(-1, keepdims=True)).astype(np.float32)
        score = prob
    elif gating == 2:
        prob = (1.0 / (1.0 + np.exp(-lg.astype(np.float64)))).astype(np.float32)
        score = prob + (0 if bias is None else np.asarray(bias, np.float32))
    else:
        prob = lg + (0 if bias is None else np.asarray(bias, np.float32))
        score = prob
    ids = np.zeros((t, ku), np.int32)
    wts = np.zeros((t, ku), np.float32)
    for i in range(t):
        order = np.lexsort((np.arange(E), -score[i].astype(np.float64)))[:ku]   # descending score, lowest index
        ids[i] = order
        p = prob[i, order].astype(np.float64)
        if gating == 3:
            ex = np.exp(p - p[0])
            wts[i] = ex / ex.sum()
        elif norm:
            wts[i] = p / max(p.sum(), 6.103515625e-05)
        else:
            wts[i] = p
    return ids, (wts * np.float32(scale)).astype(np.float32)


# ------------------------------------------------------------------------------------------------------------------
# expert activations, biases, per-expert down scale, shared-expert gate
# ------------------------------------------------------------------------------------------------------------------
ACT_SILU, ACT_GELU, ACT_SWIGLU_OAI = 0, 1, 2   # include/lk.h LK_ACT_*


def gelu_tanh(x):
    """GEGLU's gate activation (make_kernel_tests.py:78-80 ffn_act "gelu"; kbench moe_q4_0/gen_bench.py:38-39)."""
    x = np.asarray(x, np.float64)
    return 0.5 * x * (1 + np.tanh(np.sqrt(2 / np.pi) * (x + 0.044715 * x ** 3)))


def act_ref(g, u, act=ACT_SILU, alpha=1.702, limit=7.0):
    """The expert gate/up activation (gen_moe.py:27-64 act_scalar / act_vector): silu(g) * u; gelu_tanh(g) * u;
    swiglu_oai: x = min(g, limit), y = clamp(u, -limit, limit), x * sigmoid(alpha x) * (y + 1)
    (make_kernel_tests.py:3208-3210)."""
    g = np.asarray(g, np.float64)
    u = np.asarray(u, np.float64)
    if act == ACT_SILU:
        return silu(g) * u
    if act == ACT_GELU:
        return gelu_tanh(g) * u
    xg = np.minimum(g, limit)
    return xg / (1 + np.exp(-alpha * xg)) * (np.clip(u, -limit, limit) + 1)


def wscale_ref(ids, wts, scale):
    """g_moe_wscale (gen_moe.py:1010-1045): wts[t, k] * scale[ids[t, k]] (ids clamped to the expert range), f32."""
    ids = np.clip(np.asarray(ids, np.int64), 0, len(scale) - 1)
    return (np.asarray(wts, np.float32) * np.asarray(scale, np.float32)[ids]).astype(np.float32)


def shared_gate_ref(x, w):
    """g_moe_shared_gate (gen_moe.py:780-823): sg[t] = sigmoid(x[t] . w), float64."""
    d = np.asarray(x, np.float64) @ np.asarray(w, np.float64).reshape(-1)
    return 1.0 / (1.0 + np.exp(-d))


def combine_ref(ys, wts, pos=None, y0=None, sg=None):
    """g_moe_combine / _sorted (gen_moe.py:730-762, 1231-1280), optionally shared_gated (gen_moe.py:765-777):
    y[t] = sg[t] * y0[t] + sum_k wts[t, k] * ys[row(t, k)], row = pos[t*ku + k] (sorted; < 0 -> 0) or t*ku + k."""
    wts = np.asarray(wts, np.float64)
    t, ku = wts.shape
    ys = np.asarray(ys, np.float64)
    h = ys.shape[1]
    y = np.zeros((t, h)) if y0 is None else np.asarray(y0, np.float64) * (1.0 if sg is None else
                                                                          np.asarray(sg, np.float64)[:, None])
    for i in range(t):
        for k in range(ku):
            r = i * ku + k if pos is None else int(pos[i * ku + k])
            if r >= 0:
                y[i] += wts[i, k] * ys[r]
    return y


def moe_max_tiles(tokens, ku, n_experts, tile=64):
    """Worst-case tile count (gen_llm.py:5406-5411): t*KU/64 + E (rounded up)."""
    return (tokens * ku + tile - 1) // tile + n_experts


def bucket_ref(ids, n_experts, max_tiles, live=None, tile=64):
    """g_moe_bucket (gen_moe.py:829-955): live assignments a = t*KU + k counted per expert, ceil(count/tile) tiles per
    expert in expert order, tile_info[tile] = (expert, rows) and (-1, 0) unused, rowmap[row] = a (-1 padding),
    pos[a] = row (-1 dead). Within an expert, rows follow ascending a (the reference orders them by atomics; any
    order within an expert's tiles is equivalent, see check_bucket)."""
    ids = np.asarray(ids, np.int64)
    t, ku = ids.shape
    live = np.ones(t, bool) if live is None else np.asarray(live) != 0
    e_of = np.clip(ids, 0, n_experts - 1).reshape(-1)
    a_live = np.repeat(live, ku)
    counts = np.bincount(e_of[a_live], minlength=n_experts)
    tiles = (counts + tile - 1) // tile
    base = np.concatenate([[0], np.cumsum(tiles)[:-1]])
    total = int(tiles.sum())
    assert total <= max_tiles
    tile_info = np.tile(np.array([-1, 0], np.int32), (max_tiles, 1))
    rowmap = np.full(max_tiles * tile, -1, np.int32)
    pos = np.full(t * ku, -1, np.int32)
    for e in range(n_experts):
        for j in range(tiles[e]):
            tile_info[base[e] + j] = (e, min(tile, counts[e] - j * tile))
        members = np.nonzero((e_of == e) & a_live)[0]
        rows = base[e] * tile + np.arange(len(members))
        rowmap[rows] = members
        pos[members] = rows
    return tile_info, rowmap, pos


def check_bucket(ids, n_experts, max_tiles, tile_info, rowmap, pos, live=None, tile=64):
    """Order-free invariants of a bucket schedule: the reference's atomics order rows within an expert arbitrarily.
    Returns None when the schedule is valid, else a message."""
    ti, rm, ps = bucket_ref(ids, n_experts, max_tiles, live, tile)
    if not np.array_equal(ti, np.asarray(tile_info)):
        return "tile_info differs"
    rowmap = np.asarray(rowmap)
    pos = np.asarray(pos)
    if not np.array_equal(rm < 0, rowmap < 0):
        return "padding rows differ"
    # per tile: the live rows are its first tile_info rows, each holding an assignment routed to the tile's expert
    idsf = np.asarray(ids).reshape(-1)
    for e_tile in range(max_tiles):
        e, nrows = int(ti[e_tile, 0]), int(ti[e_tile, 1])
        seg = rowmap[e_tile * tile:(e_tile + 1) * tile]
        if e < 0:
            if (seg >= 0).any():
                return f"unused tile {e_tile} holds rows"
            continue
        if not ((seg[:nrows] >= 0).all() and (seg[nrows:] < 0).all()):
            return f"tile {e_tile}: live rows are not its first {nrows}"
        if (np.clip(idsf[seg[:nrows]], 0, n_experts - 1) != e).any():
            return f"tile {e_tile} holds an assignment of another expert"
    # same set of assignments per expert, and pos is the inverse of rowmap
    for r in np.nonzero(rowmap >= 0)[0]:
        a = rowmap[r]
        if pos[a] != r:
            return f"pos[{a}] != {r}"
        if ti[r // tile, 0] != np.clip(idsf[a], 0, n_experts - 1):
            return f"row {r} holds assignment {a} of another expert"
    if not np.array_equal(pos < 0, ps < 0):
        return "dead assignments differ"
    return None


def moe_ffn_ref(x, ids, wts, w_gu, w_dn, fmt, h, f, n_experts, act=ACT_SILU, alpha=1.702, limit=7.0, b_gate=None,
                b_up=None, b_down=None, dsc=None, y0=None, sg=None, w_up=None, fmt_up=None, fmt_down=None):
    """The routed expert FFN in float64 (kbench moe_q4_0/gen_bench.py:185-248; make_kernel_tests.py:3196-3215
    experts_ref and :3268-3271 chain): y[t] = sg[t] y0[t] + sum_k wts[t,k] dsc[e] (Wd[e] act(Wg[e] x[t] + bg[e],
    Wu[e] x[t] + bu[e]) + bd[e]), e = ids[t,k]; w_gu[e] = gate rows then up rows (packed blocks of `fmt`, or float
    weights when fmt is None); biases [E][f] / [E][h] f32. w_up: separate up experts [E] (f rows each, in fmt_up when it
    differs: gen_moe.py:537-552 "GATE+UP"), w_gu then holds the f gate rows; w_dn in fmt_down when given."""
    x = np.asarray(x, np.float64)
    t, ku = ids.shape
    y = np.zeros((t, h), np.float64)
    if y0 is not None:
        y += np.asarray(y0, np.float64) * (1.0 if sg is None else np.asarray(sg, np.float64)[:, None])
    w_eff = np.asarray(wts, np.float64) if dsc is None else wscale_ref(ids, wts, dsc).astype(np.float64)
    for e in np.unique(ids):
        if fmt is None:   # float weights [E][2f][h] / [E][h][f] (e.g. dequant_mxfp4_planar's output)
            gu, dn = np.asarray(w_gu[e], np.float64), np.asarray(w_dn[e], np.float64)
        elif w_up is not None:
            gu = np.concatenate([dequant(fmt, w_gu[e], h).reshape(f, h), dequant(fmt_up or fmt, w_up[e], h).reshape(f, h)])
            gu = gu.astype(np.float64)
            dn = dequant(fmt_down or fmt, w_dn[e], f).reshape(h, f).astype(np.float64)
        else:
            gu = dequant(fmt, w_gu[e], h).reshape(2 * f, h).astype(np.float64)
            dn = dequant(fmt_down or fmt, w_dn[e], f).reshape(h, f).astype(np.float64)
        sel = np.nonzero(ids == e)
        pair = x[sel[0]] @ gu.T
        g, u = pair[:, :f], pair[:, f:]
        if b_gate is not None:
            g = g + np.asarray(b_gate, np.float64)[e]
            u = u + np.asarray(b_up, np.float64)[e]
        ys = act_ref(g, u, act, alpha, limit) @ dn.T
        if b_down is not None:
            ys = ys + np.asarray(b_down, np.float64)[e]
        np.add.at(y, sel[0], ys * w_eff[sel][:, None])
    return y


def moe_ffn_q8_ref(x, ids, wts, w_gu, w_dn, fmt, h, f, act=ACT_SILU, alpha=1.702, limit=7.0, b_gate=None,
                   b_up=None, b_down=None, dsc=None, y0=None, sg=None, fmt_down=None):
    """The decode expert FFN on int8 activations, MOE_Q8=1 (gen_llm.py:5290-5302): x is quantised by g_quant_q8
    (quant_q8 above, gen_llm.py:683-750), the gate/up products of those codes with the dequantised weights are taken
    in float64, act = act(g + bg, u + bu) is rounded to f32 and quantised again per assignment row (the g_quant_q8
    launch on the gate/up output), the down products likewise (+ bd), then the weighted combine
    y[t] = sg[t] y0[t] + sum_k wts[t,k] dsc[e] ys. w_gu[e] = the expert's gate rows then up rows (packed blocks);
    w_dn in fmt_down when given."""
    xq = dequant_q8(*quant_q8(np.asarray(x, np.float32))).astype(np.float64)
    t, ku = ids.shape
    y = np.zeros((t, h), np.float64)
    if y0 is not None:
        y += np.asarray(y0, np.float64) * (1.0 if sg is None else np.asarray(sg, np.float64)[:, None])
    w_eff = np.asarray(wts, np.float64) if dsc is None else wscale_ref(ids, wts, dsc).astype(np.float64)
    for e in np.unique(ids):
        gu = dequant(fmt, w_gu[e], h).reshape(2 * f, h).astype(np.float64)
        dn = dequant(fmt_down or fmt, w_dn[e], f).reshape(h, f).astype(np.float64)
        for i, j in zip(*np.nonzero(ids == e)):
            pair = gu @ xq[i]
            g, u = pair[:f], pair[f:]
            if b_gate is not None:
                g = g + np.asarray(b_gate, np.float64)[e]
                u = u + np.asarray(b_up, np.float64)[e]
            a32 = act_ref(g, u, act, alpha, limit).astype(np.float32)[None, :]
            aq = dequant_q8(*quant_q8(a32)).astype(np.float64)[0]
            ys = dn @ aq
            if b_down is not None:
                ys = ys + np.asarray(b_down, np.float64)[e]
            y[i] += w_eff[i, j] * ys
    return y


def moe_ffn_mxfp4_decode_ref(x, ids, wts, nib_gu, sc_gu, nib_dn, sc_dn, h, f, order="pairs"):
    """The routed expert FFN with MXFP4 experts at decode sizes (gen_llm.py:5324-5386 wiring below the GEMM threshold
    of gen_llm.py:6107, the expert matvecs of gen_moe.py:535-727): per assignment act = silu(Wg x) * (Wu x) and
    ys = Wd act with the exact MXFP4 weights and unquantised activations, y[t] = sum_k wts[t,k] ys[t,k]."""
    t, ku = ids.shape
    y = np.zeros((t, h), np.float64)
    for e in np.unique(ids):   # one expert's weights at a time (an expert of gpt-oss size is 25 M values)
        g0, d0 = 2 * f * e, h * e
        Wgu = dequant_mxfp4_planar(nib_gu[g0:g0 + 2 * f], sc_gu[g0:g0 + 2 * f], 2 * f, h, order)
        Wdn = dequant_mxfp4_planar(nib_dn[d0:d0 + h], sc_dn[d0:d0 + h], h, f, order)
        for i, j in zip(*np.nonzero(ids == e)):
            v = Wgu @ np.asarray(x[i], np.float64)
            act = silu(v[:f]) * v[f:]
            y[i] += float(wts[i, j]) * (Wdn @ act)
    return y


def moe_ffn_mxfp4_ref(x, ids, wts, nib_gu, sc_gu, nib_dn, sc_dn, h, f, order="pairs", act=0, alpha=1.702, limit=7.0,
                      b_gate=None, b_up=None, b_down=None):
    """The routed expert FFN with MXFP4 experts on the fp8 path (gen_llm.py:5324-5386 wiring with the e4m3 producer
    and fp8 GEMMs of gen_mxfp4s.py:969-1110): x8 = row_scale_f8(x); act = silu(g) * u from the fp8 gate/up GEMM;
    a8 = row_scale_f8(act) per assignment; ys = fp8 down GEMM; y[t] = sum_k wts[t,k] ys[t,k]. nib_gu/sc_gu: per expert
    2f rows (gate then up) of h values; nib_dn/sc_dn: per expert h rows of f values. act / biases as moe_ffn_ref."""
    t, ku = ids.shape
    x8, s8 = row_scale_f8(x)
    y = np.zeros((t, h), np.float64)
    for e in np.unique(ids):
        sel = np.nonzero(ids == e)
        tt = sel[0]
        g0, g1 = 2 * f * e, 2 * f * e + f
        g = gemm_mxfp4_f8_ref(x8[tt], s8[tt], nib_gu[g0:g1], sc_gu[g0:g1], f, h, order)
        u = gemm_mxfp4_f8_ref(x8[tt], s8[tt], nib_gu[g1:g1 + f], sc_gu[g1:g1 + f], f, h, order)
        if b_gate is not None:   # per-expert biases before the activation (gen_moe.py:958-1007)
            g = g + np.asarray(b_gate, np.float64)[e]
            u = u + np.asarray(b_up, np.float64)[e]
        a = act_ref(g, u, act, alpha, limit).astype(np.float32)
        a8, as8 = row_scale_f8(a)
        ys = gemm_mxfp4_f8_ref(a8, as8, nib_dn[h * e:h * (e + 1)], sc_dn[h * e:h * (e + 1)], h, f, order)
        if b_down is not None:
            ys = ys + np.asarray(b_down, np.float64)[e]
        np.add.at(y, tt, ys * np.asarray(wts, np.float64)[sel][:, None])
    return y


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


# ------------------------------------------------------------------------------------------------------------------
# the reference's hand-built MoE kernel cases (kbench moe_q4_0): inputs regenerated from their seed
# ------------------------------------------------------------------------------------------------------------------
KB_H, KB_F, KB_E, KB_U = 2816, 704, 8, 8          # .github/devlab/kbench/moe_q4_0/gen_bench.py:142 (Gemma dimensions)
KB_COUNTS = (64, 17, 1, 0)                          # gen_bench.py:206: one full tile, 17- and 1-row tails, a dead tile
KB_TILE_INFO = ((7, 64), (0, 17), (3, 1), (-1, 0))  # gen_bench.py:207
KB_SENTINEL = 42.0                                  # gen_bench.py:175: outputs start filled with 42


def kbench_q4_0_weights(rng, shape):
    """gen_bench.py:27-35 weights(): Q4_0 blocks with f16 scales uniform in +-[0.0005, 0.003] (both signs) and
    uniform code bytes -> (raw uint8 [blocks*18], float64 values of `shape`)."""
    blocks = int(np.prod(shape)) // 32
    raw = np.empty((blocks, 18), np.uint8)
    scale = (rng.uniform(.0005, .003, blocks) * rng.choice([-1, 1], blocks)).astype('<f2')
    raw[:, :2] = scale.view(np.uint8).reshape(-1, 2)
    raw[:, 2:] = rng.integers(0, 256, (blocks, 16), dtype=np.uint8)
    vals = dequant("q4_0", raw, 32).astype(np.float64).reshape(shape)
    return raw.reshape(-1), vals


def kbench_moe_inputs(seed=490):
    """The inputs of the kbench moe_q4_0 cases (gen_bench.py:142-248) drawn in the generator's order from
    default_rng(seed): stacked Q4_0 expert weights (gate/up fused [E][2F][H], down [E][H][F]), the decode cases
    (t = 1, 4: a permutation of the experts per token), the grouped cases (t = 63, 65: the hand-built tile_info with
    random row maps, f16 activations and row scales in {0.5, 1, 2}) and the down-scale + combine case (t = 4)."""
    H, F, E, U = KB_H, KB_F, KB_E, KB_U
    rng = np.random.default_rng(seed)
    out = {}
    out["wg"], out["gu"] = kbench_q4_0_weights(rng, (E, 2 * F, H))
    out["wd"], out["down"] = kbench_q4_0_weights(rng, (E, H, F))
    for t in (1, 4):
        out[f"decode_t{t}_ids"] = np.stack([rng.permutation(E) for _ in range(t)]).astype(np.int32)
        out[f"decode_t{t}_x"] = rng.standard_normal((t, H)).astype(np.float32)
        out[f"decode_t{t}_xdn"] = (rng.standard_normal((t * U, F)) * .1).astype(np.float32)
    for t in (63, 65):
        rm = np.full(256, -1, np.int32)
        for j, n in enumerate(KB_COUNTS):
            rm[j * 64:j * 64 + n] = rng.choice(t * U, n, replace=False)
        out[f"grouped_t{t}_rm"] = rm
        out[f"grouped_t{t}_x"] = rng.standard_normal((t, H)).astype(np.float16)
        s = np.ones((t, 2), np.float32)
        s[:, 1] = rng.choice([.5, 1, 2], t)
        out[f"grouped_t{t}_s"] = s
        xd = (rng.standard_normal((256, F)) * .1).astype(np.float16)
        sd = np.ones((256, 2), np.float32)
        sd[:, 1] = rng.choice([.5, 1, 2], 256)
        for j, n in enumerate(KB_COUNTS[:-1]):
            xd[j * 64 + n:(j + 1) * 64] = 0
        out[f"grouped_t{t}_xd"] = xd
        out[f"grouped_t{t}_sd"] = sd
    t = 4
    out["dsc_ids"] = np.stack([rng.permutation(E) for _ in range(t)]).astype(np.int32)
    out["dsc_scales"] = np.linspace(.25, 1.5, E, dtype=np.float32)
    out["dsc_wts"] = rng.uniform(.01, .2, (t, U)).astype(np.float32)
    out["dsc_ys"] = rng.standard_normal((t * U, H)).astype(np.float32) * .1
    return out


def ffn_golden_inputs(seed=8102, E=8, H=512, F=256, KU=4, t=6):
    """Seeded inputs of the expert-FFN golden chains (tests/golden/make_golden.py main_moe): Q4_0 and MXFP4 (split
    planes, pairs order) experts of N(0, 0.02) weights, activations, routing, per-expert biases, down scales, the
    shared-expert gate vector and the shared output y0."""
    rng = np.random.default_rng(seed)
    q = lambda n, k: quantize_q4_0((rng.standard_normal((n, k)) * 0.02).astype(np.float32))   # noqa: E731
    out = {"w_gu": np.stack([q(2 * F, H) for _ in range(E)]), "w_dn": np.stack([q(H, F) for _ in range(E)])}
    mx_gu = [quantize_mxfp4((rng.standard_normal((2 * F, H)) * 0.02).astype(np.float32)) for _ in range(E)]
    mx_dn = [quantize_mxfp4((rng.standard_normal((H, F)) * 0.02).astype(np.float32)) for _ in range(E)]
    out["mx_gu_nib"] = np.concatenate([a for a, _ in mx_gu])
    out["mx_gu_sc"] = np.concatenate([b for _, b in mx_gu])
    out["mx_dn_nib"] = np.concatenate([a for a, _ in mx_dn])
    out["mx_dn_sc"] = np.concatenate([b for _, b in mx_dn])
    out["x"] = rng.standard_normal((t, H)).astype(np.float32)
    lg = rng.standard_normal((t, E)).astype(np.float32)
    out["ids"] = np.argsort(-lg, -1, kind="stable")[:, :KU].astype(np.int32)
    out["wts"] = rng.uniform(0.05, 0.4, (t, KU)).astype(np.float32)
    out["bg"] = (rng.standard_normal((E, F)) * 0.05).astype(np.float32)
    out["bu"] = (rng.standard_normal((E, F)) * 0.05).astype(np.float32)
    out["bd"] = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
    out["dsc"] = np.linspace(0.5, 1.5, E).astype(np.float32)
    out["wsg"] = (rng.standard_normal(H) * 0.05).astype(np.float32)
    out["y0"] = (rng.standard_normal((t, H)) * 0.1).astype(np.float32)
    return out
