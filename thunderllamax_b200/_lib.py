"""ctypes binding of libtlx_b200.so (the C ABI declared in include/tlx_verify.h).

There is no fallback: if the library is missing or no sm_100 device is present,
every call raises.  Build it with ``python -m thunderllamax_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("TLX_LIB", os.path.join(_HERE, "libtlx_b200.so"))

TLX_Q8_0, TLX_Q4_K, TLX_Q5_K, TLX_Q6_K, TLX_IQ3_XXS, TLX_IQ4_XS = 8, 12, 13, 14, 18, 23
TLX_DT_F32, TLX_DT_F16, TLX_DT_BF16, TLX_DT_IMAGE = 0, 1, 30, 100
MODE_STORE, MODE_GATE_UP, MODE_ARGMAX = 0, 1, 2
QTYPES = {"q6_k": TLX_Q6_K, "iq3_xxs": TLX_IQ3_XXS, "iq4_xs": TLX_IQ4_XS, "q4_k": TLX_Q4_K, "q5_k": TLX_Q5_K,
          "q8_0": TLX_Q8_0}


class TLXError(RuntimeError):
    pass


_lock = threading.Lock()
_lib = None

c_i64, c_int, c_size, c_vp, c_u32p = ctypes.c_int64, ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p

_SIGS = {
    "tlx_error_string": (ctypes.c_char_p, [c_int]),
    "tlx_device_check": (c_int, []),
    "tlx_version": (c_int, []),
    "tlx_set_max_ctas": (None, [c_int]),
    "tlx_tiled_bytes": (c_size, [c_int, c_i64, c_i64]),
    "tlx_pack_tiles": (c_int, [c_int, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "tlx_pack_tiles_device": (c_int, [c_int, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "tlx_unpack_tiles": (c_int, [c_int, c_vp, c_i64, c_i64, c_vp]),
    "tlx_gemv_workspace_bytes": (c_size, [c_int, c_int, c_i64, c_i64, c_int, c_int]),
    "tlx_workspace_init": (c_int, [c_vp, c_size, c_vp]),
    "tlx_gemv_plan": (c_int, [c_int, c_int, c_i64, c_i64, c_int, c_int, c_vp, c_int]),
    "tlx_workspace_error": (c_int, [c_vp, c_vp]),
    "tlx_activation_image_bytes": (c_size, [c_int, c_i64, c_int]),
    "tlx_stage_activations": (c_int, [c_vp, c_int, c_i64, c_int, c_i64, c_vp, c_vp]),
    "tlx_head_argmax_noalloc": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_i64, c_vp,
                                        c_vp, c_vp, c_vp, c_int, c_vp, c_vp]),
    "tlx_head_argmax_noalloc_error": (c_int, [c_vp, c_vp]),
    "tlx_peer_buffer_bytes": (c_size, [c_int, c_int, c_i64]),
    "tlx_ipc_handle_bytes": (c_size, []),
    "tlx_ipc_handle": (c_int, [c_vp, c_vp, c_vp]),
    "tlx_ipc_open": (c_int, [c_vp, ctypes.c_uint64, c_vp, c_vp]),
    "tlx_ipc_close": (c_int, [c_vp]),
    "tlx_peer_buffer_alloc": (c_int, [c_size, c_vp]),
    "tlx_peer_buffer_free": (c_int, [c_vp]),
    "tlx_gemv_peer": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_int, c_int, c_vp, c_int,
                              c_vp, c_size, c_vp]),
    "tlx_head_argmax_peer": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_i64, c_vp, c_vp,
                                     c_vp, c_int, c_vp, c_int, c_int, c_vp, c_int, c_vp, c_size, c_vp]),
    "tlx_peer_finish": (c_int, [c_int, c_int, c_vp, c_int, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp]),
    "tlx_peer_publish": (c_int, [c_int, c_int, c_vp, c_int, c_i64, c_vp, c_i64, c_vp]),
    "tlx_gemv": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_vp, c_i64, c_vp, c_int,
                         c_i64, c_vp, c_size, c_vp]),
    "tlx_ffn_gate_up": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_vp, c_int,
                                c_i64, c_vp, c_size, c_vp]),
    "tlx_head_argmax": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_i64, c_vp, c_vp,
                                c_vp, c_vp, c_int, c_vp, c_vp, c_size, c_vp]),
    "tlx_argmax_rows": (c_int, [c_vp, c_int, c_int, c_i64, c_i64, c_vp, c_vp]),
    "tlx_h_argmax": (c_int, [c_vp, c_int, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "tlx_acceptsel11k": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_vp]),
    "tlx_gdn_slots_bytes": (c_size, [c_int]),
    "tlx_gdn_slots_init": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_vp]),
    "tlx_acceptsel11k_flip": (c_int, [c_vp, c_vp, c_int, c_vp]),
    "tlx_attn_workspace_bytes": (c_size, [c_int]),
    "tlx_attn_pre": (c_int, [c_vp] * 7 + [c_int, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "tlx_attn_split": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_vp, c_size, c_vp]),
    "tlx_attn_combine": (c_int, [c_vp, c_size, c_vp, c_int, c_vp, c_vp]),
    "tlx_attn_decode": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_vp, c_vp, c_size, c_vp]),
    "tlx_lookup_workspace_bytes": (c_size, []),
    "tlx_lookup": (c_int, [c_vp, c_i64, c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_size, c_vp]),
    "tlx_q5g8v11_workspace_bytes": (c_size, [c_int, c_i64, c_i64, c_i64, c_int]),
    "tlx_q5g8v11_error": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_int, c_vp]),
    "tlx_q5g8v11": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp,
                            c_size, c_vp]),
    "tlx_aq3k8v11_workspace_bytes": (c_size, [c_int, c_i64, c_i64, c_i64, c_i64, c_int]),
    "tlx_aq3k8v11_error": (c_int, [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_int, c_vp]),
    "tlx_aq3k8v11": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_i64, c_i64,
                             c_vp, c_vp, c_vp, c_vp, c_size, c_vp]),
    "tlx_argmax_merge": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_int, c_vp, c_vp]),
    "tlx_accept": (c_int, [c_vp, c_vp, c_int, c_vp, c_vp, c_vp]),
    "tlx_accept11k": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                              c_vp, c_vp, c_int, c_vp]),
    "tlx_moe_workspace_bytes": (c_size, [c_int, c_int, c_int, c_int]),
    "tlx_moe_route": (c_int, [c_vp, c_vp, c_vp, c_i64, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp,
                              c_vp, c_vp, c_size, c_vp]),
    "tlx_moe_experts": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_int, c_int,
                                c_int, c_int, c_int, c_int, c_vp, c_size, c_vp]),
    "tlx_moe_verify": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp,
                               c_i64, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_size, c_vp]),
    "tlx_moe_workspace_error": (c_int, [c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp]),
    "tlx_prefill_workspace_bytes": (c_size, [c_int, c_i64]),
    "tlx_prefill_ffn_gate_up": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_vp, c_i64,
                                        c_vp, c_size, c_vp]),
    "tlx_prefill_gemm": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_vp, c_i64, c_vp,
                                 c_size, c_vp]),
    "tlx_act_quant_q8": (c_int, [c_vp, c_i64, c_int, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp]),
    "tlx_prefill_w4a8_gate_up": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_int, c_i64, c_i64, c_vp, c_i64,
                                         c_vp, c_size, c_vp]),
}


def lib():
    """Load the library once; raises TLXError if it is not built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise TLXError(f"{LIB_PATH} not found: build it with `python -m thunderllamax_b200.build`")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGS.items():
                fn = getattr(handle, name, None)
                if fn is None:
                    continue
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return [n for n in _SIGS if hasattr(lib(), n)]


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().tlx_error_string(rc).decode()
        raise TLXError(f"{what}: {msg} ({rc})")
