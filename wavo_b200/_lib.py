"""ctypes binding of ``libwavo_cuda.so`` (include/wavo_cuda.h). Loads the in-tree library and
declares every entry point; fails loudly when the library is missing (there is no fallback)."""

from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
SO = os.path.join(HERE, "libwavo_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "wavo_cuda.h")

OK, EINVAL, ENOMEM, ECUDA, ETIMEDOUT, EUNSUPPORTED, EDEVICE = range(7)
STATUS = {0: "OK", 1: "EINVAL", 2: "ENOMEM", 3: "ECUDA", 4: "ETIMEDOUT", 5: "EUNSUPPORTED",
          6: "EDEVICE"}
F32, F16 = 0, 1
GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
Q8_AUTO, Q8_DEQUANT, Q8_PROLOGUE = 0, 1, 2  # wavo_set_q8_gemm modes
CONV_LAYER_NORM, CONV_AFFINE = 0, 1        # wavo_conv_glu norms
WAVO_ATTEND_NOALLOC_PART_FLOATS = 1 << 18  # the header's fixed scratch of the no-alloc attend
EPILOGUES = {"bias": 0, "silu": 1, "relu": 2, "residual": 3, "gelu": 4, "gelu_residual": 5,
             "tanh": 6}

_vp, _u32, _u64, _i32, _f32, _sz = (ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64,
                                    ctypes.c_int, ctypes.c_float, ctypes.c_size_t)
_st = ctypes.c_int

SIGNATURES = {
    "wavo_device_count": ([], _i32),
    "wavo_create": ([_i32, ctypes.POINTER(_vp)], _st),
    "wavo_destroy": ([_vp], None),
    "wavo_last_error": ([_vp], ctypes.c_char_p),
    "wavo_set_stream": ([_vp, _vp], _st),
    "wavo_get_stream": ([_vp], _vp),
    "wavo_own_stream": ([_vp], _vp),
    "wavo_sm_count": ([_vp], _i32),
    "wavo_malloc": ([_vp, _sz, ctypes.POINTER(_vp)], _st),
    "wavo_free": ([_vp, _vp], _st),
    "wavo_upload": ([_vp, _vp, _vp, _sz], _st),
    "wavo_download": ([_vp, _vp, _vp, _sz], _st),
    "wavo_memset": ([_vp, _vp, _i32, _sz], _st),
    "wavo_reserve": ([_vp, _sz], _st),
    "wavo_sync": ([_vp, _u32], _st),
    "wavo_linear_create": ([_vp, _i32, _u32, _u32, _vp, _vp, _sz, ctypes.POINTER(_vp)], _st),
    "wavo_linear_destroy": ([_vp], None),
    "wavo_linear_from_gguf": ([_vp, _vp, _vp, _u32, _vp, _sz, ctypes.POINTER(_vp)], _st),
    "wavo_log_mel": ([_vp, _vp, _u64, _u64, _u64, _vp], _st),
    "wavo_mel_features": ([_vp, _vp, _u64, _vp, ctypes.POINTER(_u64)], _st),
    "wavo_subsample_scratch_bytes": ([_u32, _u32], _u64),
    "wavo_subsample": ([_vp, _vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                        _vp, _vp, ctypes.POINTER(_u32)], _st),
    "wavo_subsample_batch_scratch_bytes": ([_vp, _u32, _u32], _u64),
    "wavo_subsample_batch": ([_vp, _vp, _vp, _vp, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                              _vp, _vp, _vp, _vp, _vp], _st),
    "wavo_gguf_open": ([ctypes.c_char_p, ctypes.POINTER(_vp)], _st),
    "wavo_gguf_close": ([_vp], None),
    "wavo_gguf_tensor_count": ([_vp], _u32),
    "wavo_gguf_tensor_name": ([_vp, _u32], ctypes.c_char_p),
    "wavo_gguf_tensor": ([_vp, ctypes.c_char_p, _vp, _u32, ctypes.POINTER(_i32),
                          ctypes.POINTER(_u64)], _st),
    "wavo_gguf_tensor_dims": ([_vp, ctypes.c_char_p, _vp, _u32], _u32),
    "wavo_gguf_read": ([_vp, ctypes.c_char_p, _u64, _vp, _u64], _st),
    "wavo_gguf_has": ([_vp, ctypes.c_char_p], _i32),
    "wavo_gguf_get_int": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)], _st),
    "wavo_gguf_get_float": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)], _st),
    "wavo_gguf_get_bool": ([_vp, ctypes.c_char_p, ctypes.POINTER(_i32)], _st),
    "wavo_gguf_get_str": ([_vp, ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.POINTER(_u64)], _st),
    "wavo_gguf_array": ([_vp, ctypes.c_char_p, ctypes.POINTER(_u32), ctypes.POINTER(_u64)], _st),
    "wavo_gguf_array_items": ([_vp, ctypes.c_char_p, _vp, _vp, _vp, _vp, _u64], _st),
    "wavo_linear_width": ([_vp], _u32),
    "wavo_linear_k": ([_vp], _u32),
    "wavo_gemm": ([_vp, _vp, _i32, _u32, _vp, _vp, _i32, _u32, _u32, _i32, _f32], _st),
    "wavo_set_q8_gemm": ([_vp, _i32], _i32),
    "wavo_gemv": ([_vp, _vp, _vp, _vp, _i32, _f32, _u32], _st),
    "wavo_gemv_rows": ([_vp, _vp, _u32, _vp, _vp, _u32, _u32, _i32, _f32], _st),
    "wavo_attention": ([_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _i32], _st),
    "wavo_attention_varlen": ([_vp, _vp, _vp, _vp, _vp, _u32, _vp, _vp, _u32, _u32, _u32, _u32,
                               _u32, _i32, _i32], _st),
    "wavo_attention_rope_varlen": ([_vp, _vp, _vp, _u32, _vp, _vp, _u32, _u32, _u32, _u32, _vp,
                                    _u32, _u32, _u32, _i32, _i32], _st),
    "wavo_pos_rows": ([_u32], _u32),
    "wavo_layer_norm": ([_vp, _vp, _vp, _vp, _vp, _i32, _u32, _u32, _vp, _vp, _vp, _u32], _st),
    "wavo_embed_rows": ([_vp, _vp, _vp, _vp, _u32, _u32, _vp, _u32], _st),
    "wavo_pick": ([_vp, _vp, _u32, _u32, _u32, _vp, _vp, _u32, _vp, _u32, _vp, _u32, _u32, _u32,
                   _u32, _u32, _vp, _vp], _st),
    "wavo_conv_glu": ([_vp, _vp, _vp, _vp, _u32, _vp, _vp, _i32, _vp, _i32, _u32, _u32], _st),
    "wavo_conv_glu_varlen": ([_vp, _vp, _vp, _vp, _u32, _vp, _vp, _i32, _vp, _i32, _u32, _vp, _vp,
                              _u32, _u32, _u32], _st),
    "wavo_rope": ([_vp, _vp, _vp, _i32, _u32, _u32, _u32, _u32, _u32, _u32, _i32], _st),
    "wavo_rope_rows": ([_vp, _vp, _vp, _i32, _u32, _u32, _u32, _vp, _u32, _u32, _u32, _i32], _st),
    "wavo_pack": ([_vp, _vp, _u32, _u32, _vp, _u32, _u32, _u32, _u32], _st),
    "wavo_pack_batch": ([_vp, _vp, _u32, _u32, _u64, _vp, _u64, _u32, _u32, _u32, _u32, _u32],
                        _st),
    "wavo_attend_len": ([_u32, _u32, _u32], _sz),
    "wavo_attend": ([_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32], _st),
    "wavo_attend_batch": ([_vp, _vp, _u64, _vp, _u64, _vp, _vp, _u64, _u32, _u32, _u32, _u32,
                           _u32], _st),
    "wavo_attend_batch_noalloc": ([_vp, _u64, _vp, _u64, _vp, _u64, _u32, _u32, _u32, _u32,
                                   _u32, _vp], _st),
    "wavo_capture_begin": ([_vp], _st),
    "wavo_capture_end": ([_vp, ctypes.POINTER(_vp)], _st),
    "wavo_graph_launch": ([_vp, _vp], _st),
    "wavo_graph_destroy": ([_vp], None),
    "wavo_partition_lpt": ([_vp, _u32, _u32, _vp], _st),
    "wavo_selftest_wait_timeout": ([_vp, _u64], _st),
    "wavo_selftest_exp2": ([_vp, _vp, _vp, _u32], _st),
}

_lib = None


def header_symbols() -> list[str]:
    """The entry points include/wavo_cuda.h declares."""
    with open(HEADER) as fh:
        text = fh.read()
    return sorted(set(re.findall(r"\b(wavo_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(SO):
            raise RuntimeError(
                f"{SO} is missing: build it with `python -m wavo_b200.build` (nvcc, sm_100a); "
                "wavo_b200 has no fallback path")
        L = ctypes.CDLL(SO)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


class WavoError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


def check(status: int, ctx=None) -> None:
    if status != OK:
        msg = lib().wavo_last_error(ctx)
        raise WavoError(status, msg.decode() if msg else "")
