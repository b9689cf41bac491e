"""The allocation-free decode MoE entry point (lk_moe_ffn_decode_noalloc), called through the C ABI.

It runs the same kernels in the same order as the caller-allocated decode path (lk_moe_route -> lk_moe_expert_mv x2
-> lk_moe_combine) on the same inputs, so its output must equal that path's bit for bit; it is also checked against
the float64 oracle within the products' tolerance (relative L2 <= 1e-3). Two calls in a row share the library's
fixed device array. The cases cover the three Q4 formats, f32 / f16 / bf16 activations, norm on and off, and the
largest call the array holds (128 assignments at h = f = 4096). Collected last so it also runs after every other
test has used the library.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import qmm_oracle as O  # noqa: E402

TOL = 1e-3
QUANT = {"q4_0": O.quantize_q4_0, "q4_k": O.quantize_q4_k, "iq4_nl": O.quantize_iq4_nl}
XDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from loom_skills_b200 import _lib as L
    from loom_skills_b200 import ops
    return L, ops


def _noalloc(L, fmt_id, x, logits, w_gu, w_dn, h, f, E, ku, y, norm=1):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dt = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}[x.dtype]
    return L.load().lk_moe_ffn_decode_noalloc(fmt_id, x.shape[0], h, f, E, ku, norm, logits.data_ptr(), x.data_ptr(),
                                              dt, w_gu.data_ptr(), w_dn.data_ptr(), y.data_ptr(), stream)


@pytest.mark.parametrize("fmt,xdt,norm", [("q4_0", "bf16", 1), ("q4_k", "bf16", 1), ("iq4_nl", "f16", 1),
                                          ("q4_k", "f32", 0), ("q4_0", "f16", 0)])
def test_two_calls_match_the_allocating_path_and_the_oracle(lib, fmt, xdt, norm):
    L, ops = lib
    E, ku, h, f = 16, 4, 512, 256
    rng = np.random.default_rng(77)
    q = QUANT[fmt]
    w_gu_h = q((rng.standard_normal((E * 2 * f, h)) * 0.02).astype(np.float32))
    w_dn_h = q((rng.standard_normal((E * h, f)) * 0.02).astype(np.float32))
    w_gu, w_dn = torch.from_numpy(w_gu_h).cuda(), torch.from_numpy(w_dn_h).cuda()
    for tokens in (5, 1):   # two calls in a row on the shared array
        x = torch.from_numpy(rng.standard_normal((tokens, h)).astype(np.float32)).cuda().to(XDT[xdt])
        lg = rng.standard_normal((tokens, E)).astype(np.float32)
        logits = torch.from_numpy(lg).cuda()
        y = torch.empty(tokens, h, dtype=torch.float32, device="cuda")
        assert _noalloc(L, L.FMT_IDS[fmt], x, logits, w_gu, w_dn, h, f, E, ku, y, norm) == 0
        ref = ops.moe_ffn(fmt, x, logits, w_gu, w_dn, h, f, E, ku, norm=bool(norm), prefill=False)
        assert torch.equal(y, ref)                     # the same kernels in the same order
        ids, wts = O.route_ref(lg, ku, norm=bool(norm))
        ref64 = O.moe_ffn_ref(x.float().cpu().numpy(), ids, wts, w_gu_h.reshape(E, 2 * f, -1),
                              w_dn_h.reshape(E, h, -1), fmt, h, f, E)
        assert O.rel_l2(y.cpu().numpy(), ref64) <= TOL
    assert ops.device_status() == 0


def test_largest_call(lib):
    # 16 tokens x top-8 = 128 assignments at h = f = 4096: the whole array (random Q4_0 blocks)
    L, ops = lib
    E, ku, h, f, tokens = 8, 8, 4096, 4096, 16
    g = torch.Generator(device="cuda").manual_seed(3)

    def blocks(rows, k):
        raw = torch.randint(0, 256, (rows * k // 32, 18), dtype=torch.uint8, device="cuda", generator=g)
        sc = (torch.rand(rows * k // 32, device="cuda", generator=g) * 2.5e-3 + 5e-4).half()
        raw[:, :2] = sc.view(torch.uint8).view(-1, 2)
        return raw.view(-1)
    w_gu, w_dn = blocks(E * 2 * f, h), blocks(E * h, f)
    for seed in (1, 2):
        g.manual_seed(seed)
        x = torch.randn(tokens, h, device="cuda", generator=g).to(torch.bfloat16)
        logits = torch.randn(tokens, E, device="cuda", generator=g)
        y = torch.empty(tokens, h, dtype=torch.float32, device="cuda")
        assert _noalloc(L, L.Q4_0, x, logits, w_gu, w_dn, h, f, E, ku, y) == 0
        ref = ops.moe_ffn("q4_0", x, logits, w_gu, w_dn, h, f, E, ku, prefill=False)
        assert torch.equal(y, ref)
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
