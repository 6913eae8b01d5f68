"""ctypes binding of ``libklgemm.so`` (declarations in ``include/klgemm.h``).

Loading never falls back: if the shared library is missing or cannot be
loaded, :func:`lib` raises.  There is no CPU or pure-PyTorch path.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_longlong, c_uint8, c_uint32, c_ulonglong, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libklgemm.so"

KLG_OK = 0
KLG_ERR_ARG = 1
KLG_ERR_ALIGN = 2
KLG_ERR_CUDA = 3
KLG_ERR_WORKSPACE = 4
ERR_NAMES = {1: "KLG_ERR_ARG", 2: "KLG_ERR_ALIGN", 3: "KLG_ERR_CUDA", 4: "KLG_ERR_WORKSPACE"}

_F = POINTER(c_float)
_U8 = POINTER(c_uint8)

# name -> (restype, argtypes); mirrors include/klgemm.h
SIGNATURES = {
    "klg_version": (c_int, []),
    "klg_last_error": (c_int, [c_char_p, c_int]),
    "klg_device_status": (c_int, [POINTER(c_int), c_int]),
    "klg_launch_count": (c_longlong, []),
    "klg_selftest_wait_timeout": (c_int, [c_void_p]),
    "klg_lm_head_sample_workspace_bytes": (c_longlong, [c_longlong, c_longlong]),
    "klg_block_attn_workspace_bytes": (c_longlong, [c_longlong] * 7),
    "klg_block_attn_fwd": (c_int, [c_void_p] * 5 + [c_longlong, c_void_p] + [c_longlong] * 7 +
                           [c_float, c_void_p, c_void_p, c_void_p, c_longlong, c_void_p]),
    "klg_block_attn_bwd": (c_int, [c_void_p] * 5 + [c_longlong, c_void_p, c_void_p, c_void_p, c_void_p] +
                           [c_longlong] * 7 + [c_float, c_void_p, c_void_p, c_void_p, c_void_p]),
    "klg_block_attn_splits": (c_int, [c_longlong] * 7),
    "klg_selftest_attn_split_stall": (c_int, [c_void_p] * 5 + [c_longlong, c_void_p] + [c_longlong] * 7 +
                                      [c_float, c_void_p, c_void_p, c_void_p, c_longlong, c_int, c_void_p]),
    "klg_token_logit": (c_int, [c_void_p, c_void_p, c_void_p] + [c_longlong] * 3 + [c_void_p, c_void_p]),
    "klg_gather_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p] + [c_longlong] * 6 +
                        [c_void_p, c_void_p, c_void_p, c_void_p]),
    "klg_scatter_rows_grad": (c_int, [c_void_p] + [c_longlong] * 4 + [c_void_p, c_void_p]),
    "klg_rmsnorm_rows": (c_int, [c_void_p, c_int, c_void_p, c_longlong, c_longlong, c_float, c_void_p, c_void_p,
                                 c_void_p]),
    "klg_rmsnorm_rows_bwd": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_longlong, c_longlong, c_void_p,
                                     c_void_p]),
    "klg_lm_head_sample": (c_int, [c_void_p, c_void_p, c_longlong, c_longlong, c_longlong, c_float, c_int, c_ulonglong,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_longlong, c_void_p]),
    "klg_lm_head_sample_filtered_workspace_bytes": (c_longlong, [c_longlong, c_longlong, c_longlong]),
    "klg_lm_head_sample_filtered": (c_int, [c_void_p, c_void_p, c_longlong, c_longlong, c_longlong, c_float, c_int,
                                            c_float, c_ulonglong, c_longlong, c_void_p, c_void_p, c_void_p, c_void_p,
                                            c_void_p, c_longlong, c_void_p]),
    "klg_num_partials": (c_int, [c_int64, c_int64, POINTER(c_int)]),
    "klg_fwd_stats": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_void_p, c_int,
                              c_void_p]),
    "klg_merge_stats": (c_int, [c_void_p, c_int, c_int64, c_void_p, c_void_p]),
    "klg_count_valid": (c_int, [c_void_p, c_int64, c_void_p, c_void_p]),
    "klg_finalize": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "klg_fwd_workspace_bytes": (c_int64, [c_int64, c_int64]),
    "klg_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_int, c_void_p,
                        c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "klg_bwd_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "klg_bwd_chunk_cols": (c_int64, [c_int64, c_int64, c_int64]),
    "klg_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                        c_int64, c_float, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "klg_cast_f32_bf16": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "klg_scale_cast": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int, c_void_p]),
    "klg_xr_buffer_bytes": (c_int64, [c_int64, c_int64, c_int]),
    "klg_fwd_bwd_xr": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_int,
                               c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                               c_int, c_int, c_void_p, c_uint32, c_void_p]),
    "klg_selftest_xr_timeout": (c_int, [c_void_p, c_int64, c_int64, c_void_p]),
    "klg_xr_alloc": (c_int, [c_int, c_int64, POINTER(c_void_p), c_void_p]),
    "klg_xr_open": (c_int, [c_int, c_void_p, POINTER(c_void_p)]),
    "klg_xr_close": (c_int, [c_void_p, c_int]),
    "klg_fwd_bwd_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "klg_fwd_bwd_chunk_cols": (c_int64, [c_int64, c_int64, c_int64, c_int64]),
    "klg_fwd_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_int, c_void_p,
                            c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "klg_fwd_bwd_events": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_int,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_int64, c_void_p, c_int, c_void_p]),
    "klg_set_sm_reserve": (c_int, [c_int]),
    "klg_fwd_bwd_f32_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "klg_fwd_bwd_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_int,
                                c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_int64, c_void_p]),
    "klg_fwd_f32_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "klg_fwd_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_int, c_void_p,
                            c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "klg_lse_workspace_bytes": (c_int64, [c_int64, c_int64]),
    "klg_lse_record": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_void_p, c_void_p,
                               c_int64, c_void_p]),
    "klg_lse_merge": (c_int, [c_void_p, c_int, c_int64, c_void_p, c_void_p]),
    "klg_pass2_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "klg_pass2": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                          c_int64, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "klg_kl_loss": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p]),
    "klg_fwd_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_int,
                                c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "klg_fwd_noalloc_max_floats": (c_longlong, []),
    "klg_trace_begin": (c_int, [c_int]),
    "klg_trace_end": (c_int, [POINTER(c_int), POINTER(c_float), c_int, POINTER(c_int)]),
}

KIND_NAMES = {1: "stats", 2: "dz", 3: "gemm", 4: "merge", 5: "finalize", 6: "count", 7: "cast", 8: "zero", 9: "sample", 10: "norm", 11: "attn", 12: "gather", 13: "xr"}

_lib = None


class KLGemmError(RuntimeError):
    """A C-ABI call returned a nonzero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with {ERR_NAMES.get(code, code)}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Loads the library (once) and declares every signature; raises if absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built: run `python -m orthrus_training_test_b200.build` "
                               "(the KL-GEMM loss has no fallback implementation)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().klg_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(fn_name: str, rc: int) -> None:
    if rc != KLG_OK:
        raise KLGemmError(fn_name, rc, last_error())


def call(fn_name: str, *args) -> None:
    check(fn_name, getattr(lib(), fn_name)(*args))


def device_status(reset: bool = True) -> int:
    st = c_int(0)
    call("klg_device_status", ctypes.byref(st), int(reset))
    return st.value


def launch_count() -> int:
    return int(lib().klg_launch_count())


def trace_begin(capacity: int = 4096) -> None:
    call("klg_trace_begin", capacity)


def trace_end(capacity: int = 4096):
    """Waits for the traced launches; returns ``[(kind_name, ms), ...]`` in launch order."""
    kinds = (c_int * capacity)()
    ms = (c_float * capacity)()
    n = c_int(0)
    call("klg_trace_end", kinds, ms, capacity, ctypes.byref(n))
    return [(KIND_NAMES.get(kinds[i], str(kinds[i])), float(ms[i])) for i in range(min(n.value, capacity))]
