"""The allocation-free decode MoE entry point (lk_moe_ffn_decode_noalloc), called through the C ABI, against the
caller-allocated decode path (lk_moe_route -> lk_moe_expert_mv x2 -> lk_moe_combine) on the same inputs: two calls in
a row (the second reuses the shared array), within the products' tolerance (relative L2 <= 1e-3). Collected last so
it also runs after every other test has used the library."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

TOL = 1e-3


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from loom_skills_b200 import _lib as L
    from loom_skills_b200 import ops
    return L, ops


def _noalloc(L, fmt_id, x, logits, w_gu, w_dn, h, f, E, ku, y):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dt = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}[x.dtype]
    return L.load().lk_moe_ffn_decode_noalloc(fmt_id, x.shape[0], h, f, E, ku, 1, logits.data_ptr(), x.data_ptr(),
                                              dt, w_gu.data_ptr(), w_dn.data_ptr(), y.data_ptr(), stream)


@pytest.mark.parametrize("fmt", ["q4_0", "q4_k"])
def test_two_calls_match_the_allocating_path(lib, fmt):
    L, ops = lib
    E, ku, h, f = 16, 4, 512, 256
    rng = np.random.default_rng(77)
    q = O.quantize_q4_0 if fmt == "q4_0" else O.quantize_q4_k
    w_gu = torch.from_numpy(q((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32))).cuda()
    w_dn = torch.from_numpy(q((rng.standard_normal((E * h, f)) * 0.02).astype(np.float32))).cuda()
    for tokens in (5, 1):   # two calls in a row on the shared array
        x = torch.from_numpy(rng.standard_normal((tokens, h)).astype(np.float32)).cuda().to(torch.bfloat16)
        logits = torch.from_numpy(rng.standard_normal((tokens, E)).astype(np.float32)).cuda()
        y = torch.empty(tokens, h, dtype=torch.float32, device="cuda")
        assert _noalloc(L, L.FMT_IDS[fmt], x, logits, w_gu, w_dn, h, f, E, ku, y) == 0
        ref = ops.moe_ffn(fmt, x, logits, w_gu, w_dn, h, f, E, ku, prefill=False)
        err = float((y - ref).norm() / ref.norm())
        assert err <= TOL, err
    assert ops.device_status() == 0


def test_limits(lib):
    L, ops = lib
    E, ku, h, f = 16, 8, 512, 256
    x = torch.zeros(17, h, dtype=torch.float32, device="cuda")   # 17 * 8 = 136 assignments > 128
    logits = torch.zeros(17, E, dtype=torch.float32, device="cuda")
    w = torch.zeros(16, dtype=torch.uint8, device="cuda")
    y = torch.empty(17, h, dtype=torch.float32, device="cuda")
    assert _noalloc(L, L.Q4_0, x, logits, w, w, h, f, E, ku, y) == -5   # LK_ERANGE
    assert _noalloc(L, L.Q4_0, x[:16], logits[:16], w, w, 8192, f, E, ku, y) == -5
