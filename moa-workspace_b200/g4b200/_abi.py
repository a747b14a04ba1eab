"""ctypes binding of libg4b200.so (the C ABI declared in include/g4b200.h).

The library is loaded from this package directory. There is no fallback: if it has not
been built (`python moa-workspace_b200/build.py`), importing the ops raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libg4b200.so"

G4_OK = 0
G4_ERR_INVALID_ARGUMENT = -1
G4_ERR_MISALIGNED = -2
G4_ERR_CUDA = -3
G4_ERR_DEVICE = -4
G4_ERR_UNSUPPORTED = -5

DEVERR_KV_OFFSET = 1
DEVERR_ROPE_OFFSET = 2
DEVERR_WAIT_TIMEOUT = 4
DEVERR_NEGATIVE_SCALE = 16
DEVERR_PEER_TIMEOUT = 32
DEVERR_TOKEN_OFFSET = 64

TP_BLOB_BYTES = 128

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_f32 = ctypes.c_float

# name -> (argtypes); every entry point returns g4_status (int32)
SIGNATURES = {
    "g4_ctx_create": [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)],
    "g4_ctx_destroy": [_p],
    "g4_ctx_check": [_p, _p, ctypes.POINTER(ctypes.c_uint32)],
    "g4_ctx_set_overlap": [_p, ctypes.c_int],
    "g4_sliding_project_qkv": [_p] * 18 + [_i32, _i32, _p],
    "g4_sliding_attention": [_p, _p, _p, _p, _p, _p, _i32, _f32, _p],
    "g4_sliding_attention_after_qkv": [_p, _p, _p, _p, _p, _p, _i32, _f32, _p, _p],
    "g4_sliding_attention_output": [_p] * 6 + [_p],
    "g4_decoder_feedforward": [_p] * 14 + [_p],
    "g4_sliding_project_qkv_tiled": [_p] * 18 + [_i32, _i32, _p],
    "g4_sliding_attention_output_tiled": [_p] * 6 + [_p],
    "g4_decoder_feedforward_tiled": [_p] * 12 + [_p],
    "g4_full_project_qkv": [_p] * 16 + [_i32, _p],
    "g4_full_attention_first_page": [_p] * 8 + [_p],
    "g4_full_attention_page": [_p] * 8 + [_p],
    "g4_full_attention_output": [_p] * 7 + [_p],
    "g4_embed_token": [_p] * 4 + [_i32, _p],
    "g4_final_norm_and_logits": [_p] * 5 + [_i32, _p],
    "g4_decoder_feedforward_batch": [_p] * 14 + [_i32, _p],
    "g4_decoder_feedforward_batch_tiled": [_p] * 12 + [_i32, _p],
    "g4_decoder_feedforward_fp8": [_p] * 11 + [_p],
    "g4_decoder_feedforward_fp8_tiled": [_p] * 10 + [_p],
    "g4_decoder_feedforward_fp8_batch": [_p] * 11 + [_i32, _p],
    "g4_decoder_feedforward_fp8_batch_tiled": [_p] * 10 + [_i32, _p],
    "g4_final_norm_and_logits_batch": [_p] * 5 + [_i32, _i32, _p],
    "g4_decoder_create_batch": [_p, _p, _i32, _p],
    "g4_sliding_project_qkv_batch": [_p] * 18 + [_i32, _i32, _i32, _p],
    "g4_sliding_project_qkv_batch_tiled": [_p] * 18 + [_i32, _i32, _i32, _p],
    "g4_sliding_attention_batch": [_p, _p, _p, _p, _p, _p, _i32, _f32, _p, _i32, _p],
    "g4_sliding_attention_output_batch": [_p] * 6 + [_i32, _p],
    "g4_sliding_attention_output_batch_tiled": [_p] * 6 + [_i32, _p],
    "g4_pack_tiles": [_p, _p, _p, _p, _i32, _i32, _i32, _i32, _p],
    "g4_sliding_attention_output_noalloc": [_p] * 5 + [_p],
    "g4_decoder_create": [_p, _p, _p],
    "g4_decoder_destroy": [_p],
    "g4_decoder_buffers": [_p, _p, _p, _p],
    "g4_decoder_step": [_p, _p],
    "g4_decoder_capture": [_p, _p],
    "g4_tp_init": [_p, _i32, _i32, _p],
    "g4_tp_connect": [_p, _p],
    "g4_tp_set_wait_limit": [_p, ctypes.c_uint64],
}
STRING_FUNCS = {"g4_status_string": [ctypes.c_int32], "g4_last_error": [_p]}

_lib = None


class LibraryMissing(ImportError):
    pass


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise LibraryMissing(f"{LIB_PATH} is not built; run `python moa-workspace_b200/build.py`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int32
        for name, args in STRING_FUNCS.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = ctypes.c_char_p
        _lib = handle
    return _lib


class G4Error(RuntimeError):
    def __init__(self, status: int, message: str, flags: int = 0):
        super().__init__(f"{message} (status {status}: {lib().g4_status_string(status).decode()})")
        self.status = status
        self.flags = flags
