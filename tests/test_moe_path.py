"""Host logic of the decode MoE path choice (CPU): ops._grouped_decode says when the expert-grouped matvecs take both
projections of a layer, and with it ops.moe_ffn keeps the matvecs up to 1024 assignments instead of 191 (the
reference's own switch is at 64 tokens, gen_llm.py:6107)."""
import pytest

torch = pytest.importorskip("torch")

from loom_skills_b200 import ops  # noqa: E402


@pytest.mark.parametrize("fmt,fmt_down,dt,h,f,E,want", [
    ("q4_0", None, torch.bfloat16, 2048, 768, 128, True),      # configs[2]
    ("q4_k", "q4_k", torch.float16, 4096, 1536, 256, True),
    ("iq4_nl", "q4_0", torch.float32, 2048, 768, 64, True),    # f32 x: up to 2816 values staged
    ("q4_k", "q6_k", torch.bfloat16, 2048, 768, 128, False),   # Q4_K_M's down: the generic-format matvec
    ("q4_k+q6_k", None, torch.bfloat16, 2048, 768, 128, False),
    ("q6_k", None, torch.bfloat16, 2048, 768, 128, False),
    ("q4_0", None, torch.bfloat16, 2048, 768, 512, False),     # more experts than one CTA groups
    ("q4_0", None, torch.float32, 4096, 768, 128, False),      # f32 rows past the shared-memory budget
    ("q4_0", None, torch.bfloat16, 6144, 768, 128, False),
    ("q4_0", None, torch.bfloat16, 2048, 4096, 128, False),    # the down's f32 activation rows too long
    ("q4_0", None, torch.bfloat16, 2000, 768, 128, False),     # not whole 256-value chunks
])
def test_grouped_decode_rule(fmt, fmt_down, dt, h, f, E, want):
    assert ops._grouped_decode(fmt, fmt_down, dt, h, f, E) is want
