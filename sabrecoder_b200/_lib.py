"""ctypes binding of libsabre_b200.so (C ABI in include/sabre_b200.h).

The library is loaded from the package directory. There is no fallback: if
the shared object is missing or fails to load, every kernel call raises.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libsabre_b200.so")

c_int, c_int64, c_float, c_size_t, c_void_p, c_uint = (ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                                                      ctypes.c_size_t, ctypes.c_void_p, ctypes.c_uint)
P = ctypes.c_void_p
I64P = ctypes.POINTER(ctypes.c_int64)

# (name, restype, argtypes) for every symbol the header declares.
SIGNATURES = {
    "sabre_version": (c_int, []),
    "sabre_status_string": (ctypes.c_char_p, [c_int]),
    "sabre_last_error": (ctypes.c_char_p, []),
    "sabre_device_status": (c_int, [ctypes.POINTER(c_uint), c_int, P]),
    "sabre_set_wait_limit_ns": (c_int, [ctypes.c_ulonglong]),
    "sabre_prefill_bsa": (c_int, [P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                  I64P, I64P, I64P, I64P, I64P, I64P, c_float, c_int, P]),
    "sabre_decode_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "sabre_decode_bsa": (c_int, [P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                 I64P, I64P, I64P, I64P, I64P, I64P, c_float, c_int, P, c_size_t, P]),
    "sabre_decode_bsa_noalloc": (c_int, [P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                         I64P, I64P, I64P, I64P, I64P, I64P, c_float, c_int, P]),
    "sabre_rope_qkv": (c_int, [P, P, P, P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                               c_int, I64P, I64P, I64P, I64P, I64P, I64P, I64P, c_int, P]),
    "sabre_qkv_proj_rope": (c_int, [P, P, P, P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int,
                                    c_int, c_int, c_int, c_int64, I64P, I64P, I64P, I64P, c_int64, c_int, P]),
    "sabre_qkv_rope_decode": (c_int, [P, P, P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int,
                                      c_int, c_int64, c_int64, I64P, I64P, I64P, c_int, P]),
    "sabre_block_mask_workspace_size": (c_size_t, [c_int, c_int]),
    "sabre_build_block_mask": (c_int, [P, P, P, c_int, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                       P, P, P, c_size_t, P]),
    "sabre_indices_from_bits": (c_int, [P, c_int, c_int, P, c_int, P, P, P]),
    "sabre_indices_from_dense": (c_int, [P, c_int, c_int, c_int64, P, c_int, P, P, P]),
    "sabre_pool_blocks": (c_int, [P, c_int, c_int, c_int, c_int, c_int, I64P, c_int, P, P]),
    "sabre_topk_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "sabre_topk_extend": (c_int, [P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, P, c_int, P, P, P, P,
                                  c_size_t, P]),
    "sabre_chunk_vectors": (c_int, [P, c_int, c_int, c_int, P, P, c_int, P, P]),
    "sabre_similarity_topk": (c_int, [P, c_int, P, P, c_int, P, P, c_int, c_int, P, P]),
    "sabre_token_block_mask": (c_int, [P, P, P, P, c_int, c_int, c_int, P, P]),
    "sabre_token_tile_masks": (c_int, [P, P, P, P, c_int, c_int, c_int, P, c_int, P, P, P, P]),
    "sabre_prefill_bsa_tokenmask": (c_int, [P, P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int,
                                            I64P, I64P, I64P, I64P, I64P, I64P, c_float, c_int, P]),
}

_lib: Optional[ctypes.CDLL] = None


class SabreError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """The loaded library (raises SabreError if it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SabreError(f"{LIB_PATH} is missing: build it with `python -m sabrecoder_b200.build`")
        try:
            L = ctypes.CDLL(LIB_PATH)
        except OSError as e:  # pragma: no cover
            raise SabreError(f"cannot load {LIB_PATH}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        msg = L.sabre_last_error().decode(errors="replace")
        kind = L.sabre_status_string(status).decode()
        raise SabreError(f"{what}: {kind} ({status}): {msg}")


def i64(vals) -> ctypes.Array:
    arr = (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])
    return arr
