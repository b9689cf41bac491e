"""ctypes binding of liblk.so (the C ABI declared in include/lk.h). No fallback: a missing library is an error."""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblk.so")

# formats / dtypes / modes (include/lk.h)
Q4_0, Q4_K, IQ4_NL, MXFP4, MXFP4S = 2, 12, 20, 39, 1039
Q5_0, Q8_0, Q3_K, Q5_K, Q6_K, IQ4_XS, IQ3_S = 6, 8, 11, 13, 14, 23, 21
F32, F16, BF16, E4M3 = 0, 1, 30, 1000
STORE, ACC, SWIGLU, SWIGLU_SORTED = 0, 1, 2, 3
ORDER_PAIRS, ORDER_SPLIT16 = 0, 1
ACT_SILU, ACT_GELU, ACT_SWIGLU_OAI = 0, 1, 2
ACT_IDS = {"silu": ACT_SILU, "gelu": ACT_GELU, "swiglu_oai": ACT_SWIGLU_OAI}
FMT_IDS = {"q4_0": Q4_0, "q4_k": Q4_K, "iq4_nl": IQ4_NL, "mxfp4": MXFP4, "mxfp4s": MXFP4S, "q5_0": Q5_0,
           "q8_0": Q8_0, "q3_k": Q3_K, "q5_k": Q5_K, "q6_k": Q6_K, "iq4_xs": IQ4_XS,
           "iq3_s": IQ3_S}


def fmt_pair(gate, up):
    """LK_FMT_PAIR(gate, up): the id of gate and up weights in two formats (the reference's "GATE+UP" format)."""
    return int(gate) | (int(up) << 16)


MODE_IDS = {"store": STORE, "acc": ACC, "swiglu": SWIGLU, "swiglu_sorted": SWIGLU_SORTED}

_P, _I, _L, _F, _U = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_uint

# name -> (restype, argtypes); every symbol include/lk.h declares
SIGNATURES = {
    "lk_strerror": (ctypes.c_char_p, [_I]),
    "lk_version": (_I, []),
    "lk_row_bytes": (_L, [_I, _L]),
    "lk_device_status": (_U, [_I]),
    "lk_dequant": (_I, [_I, _P, _P, _L, _P, _I, _P]),
    "lk_row_scale_f16": (_I, [_I, _I, _P, _I, _P, _P, _P]),
    "lk_row_scale_f8": (_I, [_I, _I, _P, _I, _P, _P, _P, _P, _P]),
    "lk_mv": (_I, [_I, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P]),
    "lk_silu_mul": (_I, [_I, _I, _P, _P, _I, _P]),
    "lk_moe_gate_up_routed": (_I, [_I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _I, _P, _P, _I, _P, _P, _I, _F, _F, _P,
                                   _P, _P, _P]),
    "lk_moe_expert_mv_q8": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _F, _F, _P, _P]),
    "lk_quant_q8": (_I, [_I, _I, _P, _I, _P, _P]),
    "lk_mv_q8": (_I, [_I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "lk_mv_q8_multi": (_I, [_I, _I, _P, _P, _P, _I, _I, _I, _P, _P]),
    "lk_gemm": (_I, [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P]),
    "lk_gemm_mxfp4s_f8": (_I, [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "lk_moe_route": (_I, [_I, _I, _I, _I, _I, _I, _F, _P, _P, _I, _P, _P, _P, _P]),
    "lk_moe_bucket": (_I, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P]),
    "lk_moe_grouped_gemm": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P]),
    "lk_moe_grouped_gemm_mxfp4s_f8": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                           _P]),
    "lk_moe_combine_sorted": (_I, [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "lk_moe_expert_mv": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P]),
    "lk_moe_expert_mv_mxfp4s": (_I, [_I, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P]),
    "lk_moe_combine": (_I, [_I, _I, _I, _I, _P, _P, _P, _P]),
    "lk_peer_alloc": (_I, [_L, ctypes.POINTER(_P), _P]),
    "lk_peer_open": (_I, [_P, ctypes.POINTER(_P)]),
    "lk_peer_close": (_I, [_P]),
    "lk_peer_free": (_I, [_P]),
    "lk_gemm_allgather": (_I, [_I, _I, _I, _I, _I, _P, _P, _P, _P, ctypes.POINTER(_P), _I, _I, _I, _P]),
    "lk_moe_row_scale_gather": (_I, [_I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P]),
    "lk_moe_ffn_decode_noalloc": (_I, [_I, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P]),
    "lk_moe_grouped_gemm_ex": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _F, _F,
                                    _P, _P]),
    "lk_moe_grouped_gemm_mxfp4s_f8_ex": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                              _P, _I, _F, _F, _P, _P]),
    "lk_moe_expert_mv_ex": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _I, _F, _F, _P, _P]),
    "lk_moe_expert_mv_mxfp4s_ex": (_I, [_I, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _I, _F, _F, _P, _P]),
    "lk_mv_q8_fused": (_I, [_I, _I, _I, _I, _P, _I, _P, _P, _P]),
    "lk_mv_q8_fused_multi": (_I, [_I, _I, _P, _P, _P, _I, _I, _P, _I, _P]),
    "lk_moe_wscale": (_I, [_I, _I, _I, _P, _P, _P, _P]),
    "lk_moe_rank_plan": (_I, [_I, _I, _I, _P, _P, _P, _P, _P]),
    "lk_moe_gather_rows": (_I, [_I, _I, _I, _I, _P, _P, _P, _I, _P, _P, _P]),
    "lk_moe_ffn_decode_q8": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _I,
                                  _F, _F, _P, _P, _P, _P, _I, _P, _P]),
    "lk_moe_shared_gate": (_I, [_I, _I, _P, _P, _I, _P, _P]),
    "lk_moe_combine_gated": (_I, [_I, _I, _I, _P, _P, _P, _P, _P]),
    "lk_moe_combine_sorted_gated": (_I, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P]),
}

_lib = None


def load():
    """The loaded liblk.so with argument types declared. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built (run loom_skills_b200/build.py or __graft_entry__.build())")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class LkError(RuntimeError):
    pass


def check(rc, what):
    if rc != 0:
        raise LkError(f"{what}: {load().lk_strerror(rc).decode()} (code {rc})")
    return rc
