"""loom_skills_b200: the quantized-matmul hot path of loom-fun/loom-skills, rebuilt for NVIDIA B200 (sm_100a).

GGUF block dequantisation fused into decode matvecs and tcgen05 prefill GEMMs (Q4_0, Q4_K, IQ4_NL), the MoE top-k
pipeline (router, GPU-built tile schedule, grouped GEMMs, combine) and the MXFP4 x FP8 expert GEMM, behind a C ABI
(include/lk.h, liblk.so) with a torch-tensor mirror of the reference generators' op signatures (ops.py).
"""
from . import ops  # noqa: F401
from ._lib import LIB_PATH, LkError  # noqa: F401
