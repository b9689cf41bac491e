"""The C ABI library builds, loads and exports every symbol include/lk.h declares (CPU only: no kernel launches)."""
import ctypes
import os
import re

import pytest

from loom_skills_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PAIR = L.fmt_pair(L.Q4_K, L.Q6_K)


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "lk.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lk_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = declared_symbols()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(L.SIGNATURES), set(names) ^ set(L.SIGNATURES)


def test_host_only_entry_points():
    lib = L.load()
    assert lib.lk_version() >= 1
    assert lib.lk_row_bytes(L.Q4_0, 4096) == 2304
    assert lib.lk_row_bytes(L.Q4_K, 12288) == 6912
    assert lib.lk_row_bytes(L.IQ4_NL, 27648) == 15552
    assert lib.lk_row_bytes(L.MXFP4, 2880) == 1530
    assert lib.lk_row_bytes(L.Q4_K, 100) == -1
    assert b"invalid" in lib.lk_strerror(-1)


@pytest.mark.parametrize("call", [
    lambda lib: lib.lk_mv(99, 16, 256, 1, 0, 8, L.F32, 16, None, 32, None),              # unknown format
    lambda lib: lib.lk_mv(L.Q4_0, 16, 100, 1, 0, 16, L.F32, 16, None, 32, None),         # k % 256
    lambda lib: lib.lk_mv(L.Q4_0, 16, 256, 1, 0, 16, L.F32, 17, None, 32, None),         # misaligned w
    lambda lib: lib.lk_gemm(L.Q4_K, 7, 128, 256, 256, 16, 16, 16, None, 16, None),       # unknown mode
    lambda lib: lib.lk_gemm(L.Q4_K, L.SWIGLU, 128, 256, 256, 16, 16, 16, None, 16, None),  # swiglu without w2
    lambda lib: lib.lk_gemm(L.Q4_K, L.STORE, 128, 256, 250, 16, 16, 16, None, 16, None),   # n % 16
    lambda lib: lib.lk_moe_route(4, 0, 300, 8, 1, 1, 1.0, 16, None, L.F32, None, 16, 16, None),  # > 256 experts
    lambda lib: lib.lk_moe_bucket(64, 8, 128, 4, None, 16, 16, 16, 16, None),          # max_tiles too small
    lambda lib: lib.lk_dequant(L.Q4_K, 16, None, 100, 16, L.F32, None),                 # not a block multiple
    # gate/up in two formats (LK_FMT_PAIR): gate/up entry points and modes only, separate tensors, both formats' blocks
    lambda lib: lib.lk_gemm(PAIR, L.STORE, 128, 256, 256, 16, 16, 16, 16, 16, None),     # a pair is swiglu only
    lambda lib: lib.lk_mv(PAIR, 16, 256, 1, 0, 16, L.F32, 16, None, 32, None),           # a pair needs w2
    lambda lib: lib.lk_mv(L.fmt_pair(L.Q4_0, L.Q6_K), 16, 704, 1, 0, 16, L.F32, 16, 16, 32, None),  # k % 256 (Q6_K)
    lambda lib: lib.lk_mv(L.fmt_pair(L.Q4_K, L.MXFP4S), 16, 256, 1, 0, 16, L.F32, 16, 16, 32, None),  # no MXFP4S half
    lambda lib: lib.lk_moe_expert_mv(PAIR, 1, 16, 256, 4, 2, 8, 0, 16, 16, L.F32, 16, None, 16, None),  # down mode
    lambda lib: lib.lk_moe_expert_mv(PAIR, 0, 16, 256, 4, 2, 8, 1, 16, 16, L.F32, 16, 16, 16, None),  # fused
    lambda lib: lib.lk_moe_grouped_gemm(PAIR, L.SWIGLU_SORTED, 64, 256, 16, 64, 2, 8, 1, 16, 16, 16, 16, 16, 16, 16,
                                        None),                                               # fused
    lambda lib: lib.lk_silu_mul(2, 6, 16, 16, L.ACT_SILU, None),                        # n % 4
    lambda lib: lib.lk_silu_mul(2, 8, 16, 16, L.ACT_SWIGLU_OAI, None),                  # silu or gelu only
])
def test_validation_rejects_before_any_launch(call):
    assert call(L.load()) < 0
