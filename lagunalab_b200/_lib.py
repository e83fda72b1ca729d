"""ctypes binding of ``liblaguna_b200.so`` (declared in ``include/laguna_b200.h``).

There is no fallback: if the library is missing or cannot be loaded, every op raises.
"""
import ctypes
from ctypes import c_float, c_int, c_longlong, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblaguna_b200.so"

LG_OK, LG_ERR_INVALID, LG_ERR_UNSUPPORTED, LG_ERR_CUDA, LG_ERR_WORKSPACE = range(5)
LG_SCORE_SIGMOID, LG_SCORE_SOFTMAX = 0, 1
LG_PATH_AUTO, LG_PATH_GEMV, LG_PATH_TENSOR = 0, 1, 2
LG_MOE_GEMV_MAX_ROWS = 768

P = c_void_p
I = c_int

# name -> (restype, argtypes); mirrors include/laguna_b200.h
SIGNATURES = {
    "lg_abi_version": (c_int, []),
    "lg_last_error": (ctypes.c_char_p, []),
    "lg_launch_count": (c_longlong, []),
    "lg_set_pdl": (c_int, [c_int]),
    "lg_profile_stage": (c_int, [ctypes.c_char_p, P, P]),
    "lg_event_elapsed_ms": (c_int, [P, P, ctypes.POINTER(c_float)]),
    "lg_router_topk": (c_int, [P, I, I, P, P, P, I, P, I, I, I, I, P, P, P, P, P]),
    "lg_moe_plan": (c_int, [P, I, I, I, I, P, P, P, P]),
    "lg_moe_workspace_bytes": (c_size_t, [I, I, I, I, I, I]),
    "lg_moe_status": (c_int, [P, I, I, I, I, I, I, ctypes.POINTER(c_int)]),
    "lg_moe_experts": (c_int, [P, I, I, I, I, I, P, P, c_float,
                               P, P, P, P, P, P, P, P, P,
                               I, P, P, P, P, P, P, P, P, P,
                               I, I, I, P, P, c_size_t, P]),
    "lg_switch_glu": (c_int, [P, I, I, I, I, I, P,
                              P, P, P, P, P, P, P, P, P,
                              I, I, I, P, P, c_size_t, P]),
    "lg_qmlp": (c_int, [P, I, I, I, P, P, P, P, P, P, P, P, P, I, I, I, P, P, c_size_t, P]),
    "lg_quantize_rows": (c_int, [P, I, I, I, I, I, c_longlong, c_longlong, c_longlong, I, I,
                                 P, P, P, I, I, P]),
    "lg_dequantize_rows": (c_int, [P, P, P, I, I, I, I, I, I, I, P, P]),
    "lg_q8_decode_workspace_bytes": (c_size_t, [I, I, I, I]),
    "lg_q8_decode_attention": (c_int, [P, I, I, I, I, P, P, P, P, P, P, I, I, c_float, P, P,
                                       c_size_t, P]),
    "lg_q8_decode_fixed_scratch_bytes": (c_size_t, []),
    "lg_q8_decode_attention_noalloc": (c_int, [P, I, I, I, I, P, P, P, P, P, P, I, I, c_float,
                                               P, P]),
    "lg_rmsnorm": (c_int, [P, P, P, I, I, c_float, P, P, P]),
    "lg_qlinear": (c_int, [P, I, I, I, P, P, P, I, I, P, P, P]),
    "lg_embed": (c_int, [P, I, P, P, P, I, I, I, I, P, P]),
    "lg_attn_prep": (c_int, [P, I, I, I, I, P, P, c_float, c_float, P, I, I, P, P, P, I, P,
                             P, I, c_float, I, I, P]),
    "lg_attn_prep_streams": (c_int, [P, I, I, I, I, P, P, c_float, c_float, P, I, P, P, P, I, P,
                                     P, I, c_float, I, P]),
    "lg_bf16_decode_workspace_bytes": (c_size_t, [I, I, I, I]),
    "lg_bf16_decode_attention_streams": (c_int, [P, I, I, I, I, P, P, I, P, I, I, c_float, P, P,
                                                 P, c_size_t, P]),
    "lg_bf16_decode_attention": (c_int, [P, I, I, I, I, P, P, I, I, P, I, I, c_float, P, P, P,
                                         c_size_t, P]),
    "lg_argmax": (c_int, [P, I, I, P, P, I, P]),
    "lg_decode_gemv": (c_int, [P, I, I, P, P, P, P, P, P, P, c_float, P, P, P]),
    "lg_decode_qkv_prep": (c_int, [P, I, P, P, P, P, c_float, I, I, I, P, P, c_float, c_float, P,
                                   I, I, P, P, P, P, P, P, P, P, P, P, P, I,
                                   P, I, c_float, I, I, P, c_size_t, P]),
    "lg_decode_qkv_prep_workspace_bytes": (c_size_t, [I, I]),
    "lg_router_decode": (c_int, [P, P, c_float, I, P, P, P, P, I, I, I, I, P, P, P, P, P,
                                 c_size_t, P]),
    "lg_router_decode_workspace_bytes": (c_size_t, [I]),
    "lg_moe_decode_workspace_bytes": (c_size_t, [I, I, I, I]),
    "lg_moe_decode_supported": (c_int, [I, I, I, I]),
    "lg_router_decode_supported": (c_int, [I, I]),
    "lg_decode_status": (c_int, [P, I]),
    "lg_attn_prep_q8": (c_int, [P, I, I, I, I, P, P, c_float, c_float, P, I, I, P, P, P, P, P, P,
                                P, I, P, P, I, c_float, I, I, P]),
    "lg_q8_decode_attention_dev": (c_int, [P, I, I, I, I, P, P, P, P, P, P, I, I, P, I, c_float,
                                           P, P, P, c_size_t, P]),
    "lg_ep_arena_bytes": (c_size_t, [I, I, I, I]),
    "lg_ep_arena_offsets": (c_int, [I, I, I, I, P, P]),
    "lg_ep_ipc_handle_bytes": (c_size_t, []),
    "lg_ep_ipc_handle": (c_int, [P, P, P]),
    "lg_ep_ipc_open": (c_int, [P, c_size_t, P, P]),
    "lg_ep_ipc_close": (c_int, [P]),
    "lg_ep_dispatch": (c_int, [P, P, P, I, I, I, I, I, I, I, P, ctypes.c_uint, P]),
    "lg_ep_experts_workspace_bytes": (c_size_t, [I, I, I, I, I, I]),
    "lg_ep_experts": (c_int, [I, I, I, I, I, I, P, P, P, P, P, P, P, P, P, I, P, ctypes.c_uint,
                              ctypes.c_double, I, P, c_size_t, P]),
    "lg_ep_combine": (c_int, [P, I, I, I, I, I, c_float, I, I, I, P, ctypes.c_uint,
                              ctypes.c_double, P, P]),
    "lg_ep_status": (c_int, [P, I, P]),
    "lg_ep_dispatch_mapped": (c_int, [P, P, P, I, I, I, I, I, I, I, P, ctypes.c_uint, P, P, P]),
    "lg_ep_advance": (c_int, [P, P]),
    "lg_moe_decode": (c_int, [P, P, P, I, I, I, I, c_float, P, P, P, P, P, P, P, P, P, I,
                              P, P, P, P, P, P, P, P, P, P, P, P, c_size_t, P]),
}

_lib = None


class LagunaError(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


def lib():
    """Load (once) and return the shared library; raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built: run `python -m lagunalab_b200.build` "
                "(the B200 kernels have no CPU fallback)")
        h = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib = h
    return _lib


def event_elapsed_ms(ev_start, ev_end):
    """Elapsed ms between two torch.cuda.Event objects recorded by the library."""
    ms = c_float(0.0)
    call("lg_event_elapsed_ms", ev_start.cuda_event, ev_end.cuda_event, ctypes.byref(ms))
    return ms.value


def call(name, *args):
    """Call an entry point; raise ValueError for invalid arguments, LagunaError otherwise."""
    rc = getattr(lib(), name)(*args)
    if rc != LG_OK:
        msg = lib().lg_last_error().decode(errors="replace")
        if rc == LG_ERR_INVALID:
            raise ValueError(msg)
        raise LagunaError(rc, f"{name}: {msg} (status {rc})")
    return rc
