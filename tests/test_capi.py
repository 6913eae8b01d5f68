"""The C-ABI library loads, exports everything include/klgemm.h declares, and
rejects bad arguments with the documented status codes (no GPU needed: every
call here fails validation before any device work)."""
import ctypes
import re
from pathlib import Path

import pytest

from orthrus_training_test_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "klgemm.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(klg_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/klgemm.h but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_version_and_error_text():
    L = _lib.lib()
    assert L.klg_version() == 100
    rc = L.klg_fwd_stats(None, None, None, 10, 64, 10, 1.0, None, 1, None)
    assert rc == _lib.KLG_ERR_ARG
    assert "null" in _lib.last_error()


def _buf(nbytes, offset=0):
    raw = ctypes.create_string_buffer(nbytes + 64)
    base = (ctypes.addressof(raw) + 15) & ~15
    return raw, ctypes.c_void_p(base + offset)


def test_argument_validation_codes():
    L = _lib.lib()
    keep, p = _buf(1 << 16)
    _, odd = _buf(1 << 16, offset=4)
    # hidden not a multiple of 8 -> alignment error
    assert L.klg_fwd_stats(p, p, p, 4, 12, 4, 1.0, p, 1, None) == _lib.KLG_ERR_ALIGN
    # hidden below one 64-column k-block -> rejected, on every lm_head entry point
    assert L.klg_fwd_stats(p, p, p, 4, 56, 4, 1.0, p, 1, None) == _lib.KLG_ERR_ARG
    assert "hidden >= 64" in _lib.last_error()
    assert L.klg_fwd_bwd(p, p, p, p, 4, 32, 4, 1.0, 0, p, None, p, p, None, p, p, p, 1 << 16, None) == _lib.KLG_ERR_ARG
    assert L.klg_lm_head_sample(p, p, 4, 8, 4, 1.0, 0, 0, p, p, p, p, 1 << 16, None) == _lib.KLG_ERR_ARG
    # misaligned input pointer
    assert L.klg_fwd_stats(odd, p, p, 4, 64, 4, 1.0, p, 1, None) == _lib.KLG_ERR_ALIGN
    # bad shapes / temperature
    assert L.klg_fwd_stats(p, p, p, 0, 64, 4, 1.0, p, 1, None) == _lib.KLG_ERR_ARG
    assert L.klg_fwd_stats(p, p, p, 4, 64, 0, 1.0, p, 1, None) == _lib.KLG_ERR_ARG
    assert L.klg_fwd_stats(p, p, p, 4, 64, 4, 0.0, p, 1, None) == _lib.KLG_ERR_ARG
    assert L.klg_fwd_stats(p, p, p, 4, 64, 4, float("inf"), p, 1, None) == _lib.KLG_ERR_ARG
    # wrong partial-record count for this problem
    n = ctypes.c_int(0)
    # one (row pair tile, vocab range) unit x 2 epilogue column slices
    assert L.klg_num_partials(4, 4, ctypes.byref(n)) == 0 and n.value == 2
    assert L.klg_fwd_stats(p, p, p, 4, 64, 4, 1.0, p, 7, None) == _lib.KLG_ERR_ARG
    # workspace too small
    assert L.klg_fwd(p, p, p, p, 4, 64, 4, 1.0, 0, p, p, p, None, p, 8, None) == _lib.KLG_ERR_WORKSPACE
    assert L.klg_bwd(p, p, p, p, p, p, None, 4, 64, 4, 1.0, p, p, p, 100, None) == _lib.KLG_ERR_WORKSPACE
    # null outputs
    assert L.klg_finalize(None, p, 4, p, p, p, None, None) == _lib.KLG_ERR_ARG
    assert L.klg_merge_stats(p, 0, 4, p, None) == _lib.KLG_ERR_ARG
    assert L.klg_count_valid(None, 4, p, None) == _lib.KLG_ERR_ARG
    assert L.klg_trace_begin(0) == _lib.KLG_ERR_ARG
    # gradient scaling: null / negative size / misaligned buffers rejected before any device call
    assert L.klg_scale_cast(None, None, 4, p, 1, None) == _lib.KLG_ERR_ARG
    assert L.klg_scale_cast(p, None, -1, p, 1, None) == _lib.KLG_ERR_ARG
    assert L.klg_scale_cast(odd, None, 4, p, 1, None) == _lib.KLG_ERR_ALIGN
    assert L.klg_scale_cast(p, None, 0, p, 0, None) == 0
    # peer-memory dW exchange: buffer size and the argument checks made before any device call
    assert L.klg_xr_buffer_bytes(49152, 576, 1) == -1 and L.klg_xr_buffer_bytes(49152, 576, 9) == -1
    assert L.klg_xr_buffer_bytes(49152, 576, 4) == (2 * 4 + 1) * 12288 * 576 * 4 + 256
    bufs = (ctypes.c_void_p * 2)(p, p)
    assert L.klg_fwd_bwd_xr(p, p, p, p, 4, 64, 4, 1.0, 1, p, None, p, p, None, p, p, p, 1 << 16, 1, 0, bufs, 1,
                            None) == _lib.KLG_ERR_ARG                                   # world < 2
    assert L.klg_fwd_bwd_xr(p, p, p, p, 4, 64, 4, 1.0, 1, p, None, p, p, None, p, p, p, 1 << 16, 2, 2, bufs, 1,
                            None) == _lib.KLG_ERR_ARG                                   # rank >= world
    assert L.klg_fwd_bwd_xr(p, p, p, p, 4, 64, 4, 1.0, 1, p, None, p, p, None, p, None, p, 1 << 16, 2, 0, bufs, 1,
                            None) == _lib.KLG_ERR_ARG                                   # no dW
    odd_bufs = (ctypes.c_void_p * 2)(p, odd)
    assert L.klg_fwd_bwd_xr(p, p, p, p, 4, 64, 4, 1.0, 1, p, None, p, p, None, p, p, p, 1 << 16, 2, 0, odd_bufs, 1,
                            None) == _lib.KLG_ERR_ALIGN
    assert L.klg_selftest_xr_timeout(None, 1000, 128, None) == _lib.KLG_ERR_ARG
    # both outputs NULL: nothing to do, succeeds without touching the device
    assert L.klg_bwd(p, p, p, p, p, p, None, 4, 64, 4, 1.0, None, None, p, 1 << 16, None) == 0
    del keep


HDR = 4096  # tile counters ahead of the dZ chunk


# dZ chunk rows are padded to a multiple of 8 (16-byte rows of the transposed layout)
@pytest.mark.parametrize("n,v,ws,expect", [(16384, 49152, HDR + 16384 * 8192 * 2, 8192), (1, 1, HDR + 8 * 256, 128),
                                           (1, 1, HDR + 256, -1),
                                           (300, 1500, HDR + 304 * 256, 128), (100, 50000, HDR + 104 * 2 * 200, 128),
                                           (100, 50000, 100, -1), (10, 1000, 1 << 30, 1024),
                                           (10, 128 * 2000, HDR + 10 * 256, -1)])  # > 1024 chunks
def test_backward_chunk_plan(n, v, ws, expect):
    assert _lib.lib().klg_bwd_chunk_cols(n, v, ws) == expect


def test_workspace_sizes_bounded():
    L = _lib.lib()
    # the dZ chunk stays far below a full [N, V] tensor at the benchmark sizes
    for n, h, v in [(16384, 576, 49152), (65536, 2048, 49152), (32768, 1024, 31040), (12251, 576, 49152)]:
        ws = L.klg_bwd_workspace_bytes(n, h, v)
        assert 0 < ws <= (512 << 20) + HDR
        assert _lib.lib().klg_bwd_chunk_cols(n, v, ws) >= 2048
        assert ws < n * v * 2 / 2


def test_sampler_and_norm_argument_validation():
    L = _lib.lib()
    keep, p = _buf(1 << 16)
    seed = ctypes.c_ulonglong(1)
    ws = L.klg_lm_head_sample_workspace_bytes(32, 49153)
    assert ws > 0 and ws < 32 * 49153 * 4             # records, never the [N, V] logits
    assert L.klg_lm_head_sample_workspace_bytes(0, 10) == -1
    assert L.klg_lm_head_sample_workspace_bytes(10, 0) == -1
    # null output, misaligned hidden, bad temperature, small workspace
    assert L.klg_lm_head_sample(p, p, 4, 64, 4, 1.0, 1, seed, None, p, p, p, 1 << 16, None) == _lib.KLG_ERR_ARG
    assert L.klg_lm_head_sample(p, p, 4, 12, 4, 1.0, 1, seed, p, p, p, p, 1 << 16, None) == _lib.KLG_ERR_ALIGN
    assert L.klg_lm_head_sample(p, p, 4, 64, 4, 0.0, 1, seed, p, p, p, p, 1 << 16, None) == _lib.KLG_ERR_ARG
    assert L.klg_lm_head_sample(p, p, 4, 64, 4, 1.0, 1, seed, p, p, p, p, 16, None) == _lib.KLG_ERR_WORKSPACE
    # filtered sampling: cap within [1, V], top_p in (0, 1], top_k >= 0, outputs present
    assert L.klg_lm_head_sample_filtered_workspace_bytes(4, 300, 0) == -1
    assert L.klg_lm_head_sample_filtered_workspace_bytes(4, 300, 301) == -1
    assert L.klg_lm_head_sample_filtered_workspace_bytes(4, 300, 300) > 4 * 300 * 8
    fargs = lambda **kw: [p, p, 4, 64, 300, 1.0, kw.get("k", 5), kw.get("tp", 1.0), seed, kw.get("cap", 16), p, p, p,
                          kw.get("ov", p), p, 1 << 16, None]
    assert L.klg_lm_head_sample_filtered(*fargs(tp=0.0)) == _lib.KLG_ERR_ARG
    assert L.klg_lm_head_sample_filtered(*fargs(tp=1.5)) == _lib.KLG_ERR_ARG
    assert L.klg_lm_head_sample_filtered(*fargs(k=-1)) == _lib.KLG_ERR_ARG
    assert L.klg_lm_head_sample_filtered(*fargs(cap=301)) == _lib.KLG_ERR_ARG
    assert L.klg_lm_head_sample_filtered(*fargs(ov=None)) == _lib.KLG_ERR_ARG
    # final norm: dtype flag, alignment, eps, null buffers
    assert L.klg_rmsnorm_rows(p, 2, p, 4, 64, 1e-5, p, None, None) == _lib.KLG_ERR_ARG
    assert L.klg_rmsnorm_rows(p, 0, p, 4, 12, 1e-5, p, None, None) == _lib.KLG_ERR_ALIGN
    assert L.klg_rmsnorm_rows(p, 0, p, 4, 64, -1.0, p, None, None) == _lib.KLG_ERR_ARG
    assert L.klg_rmsnorm_rows(p, 0, p, 4, 64, 1e-5, None, None, None) == _lib.KLG_ERR_ALIGN
    assert L.klg_rmsnorm_rows(None, 0, p, 4, 64, 1e-5, p, None, None) == _lib.KLG_ERR_ARG
    assert L.klg_rmsnorm_rows_bwd(p, 0, p, None, p, 4, 64, p, None) == _lib.KLG_ERR_ARG
    del keep


def test_attention_argument_validation():
    L = _lib.lib()
    keep, p = _buf(1 << 16)
    ws = L.klg_block_attn_workspace_bytes
    assert ws(1, 9, 3, 32, 32, 2048, 64) > 0                 # decode: AR range split over CTAs
    assert ws(4, 9, 3, 2048, 32, 2048, 64) == 16             # many units: one split, no records
    assert ws(1, 9, 3, 32, 32, 2048, 128) == -1              # head_dim 64 only
    assert ws(1, 9, 3, 32, 24, 2048, 64) == -1               # K a multiple of 16
    assert ws(1, 9, 3, 40, 32, 2048, 64) == -1               # Ld a multiple of K
    assert ws(1, 9, 4, 32, 32, 2048, 64) == -1               # H a multiple of Hkv
    assert ws(1, 9, 3, 32, 32, 0, 64) == -1                  # an AR cache
    args = lambda **kw: [kw.get("q", p), p, p, p, p, kw.get("stride", 2048), p, 1, 9, 3, 32, 32, 2048, 64,
                         kw.get("scale", 0.125), p, None, p, kw.get("wsb", 1 << 16), None]
    assert L.klg_block_attn_fwd(*args(q=None)) == _lib.KLG_ERR_ARG
    assert L.klg_block_attn_fwd(*args(stride=100)) == _lib.KLG_ERR_ARG     # stride < ar_len
    assert L.klg_block_attn_fwd(*args(scale=0.0)) == _lib.KLG_ERR_ARG
    assert L.klg_block_attn_fwd(*args(wsb=8)) == _lib.KLG_ERR_WORKSPACE
    del keep


_C_CALLER = r"""
#include <stdio.h>
#include <string.h>
#include "klgemm.h"

int main(void) {
  char msg[256];
  static float buf[64] __attribute__((aligned(16)));
  if (klg_version() != KLG_VERSION) return 10;
  /* null inputs: rejected before any device work */
  if (klg_fwd_bwd(NULL, NULL, NULL, NULL, 16, 64, 16, 1.0f, 0, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 0,
                  NULL) != KLG_ERR_ARG) return 11;
  if (klg_last_error(msg, (int)sizeof msg) != KLG_OK || strstr(msg, "null") == NULL) return 12;
  /* hidden not a multiple of 8 */
  if (klg_fwd_stats(buf, buf, buf, 4, 12, 4, 1.0f, buf, 1, NULL) != KLG_ERR_ALIGN) return 13;
  printf("ok %d\n", klg_version());
  return 0;
}
"""


def test_plain_c_caller_builds_and_links(tmp_path):
    """The header is plain C99 and C++, and a C program links against the library and gets
    the documented status codes: the boundary needs no Python or torch."""
    import shutil
    import subprocess
    gcc, gxx = shutil.which("gcc"), shutil.which("g++")
    if gcc is None or gxx is None:
        pytest.skip("no host C compiler")
    _lib.lib()   # builds nothing; fails here if the library is missing
    inc = ROOT / "include"
    subprocess.run([gxx, "-fsyntax-only", "-Wall", "-Werror", "-x", "c++", str(inc / "klgemm.h")], check=True)
    src = tmp_path / "caller.c"
    src.write_text(_C_CALLER)
    exe = tmp_path / "caller"
    libdir = _lib.LIB_PATH.parent
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", str(inc), str(src), "-o", str(exe), f"-L{libdir}",
                    "-lklgemm", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
    assert out.stdout.strip() == "ok 100"


_NULL_CALLER = r"""
import ctypes, json, sys
sys.path.insert(0, sys.argv[1])
from orthrus_training_test_b200 import _lib
L = _lib.lib()
out = {}
for name in sys.argv[2:]:
    res, args = _lib.SIGNATURES[name]
    vals = [0.0 if a is ctypes.c_float else
            0 if a in (ctypes.c_int, ctypes.c_int64, ctypes.c_longlong, ctypes.c_uint32, ctypes.c_ulonglong) else None
            for a in args]
    out[name] = getattr(L, name)(*vals)
print(json.dumps(out))
"""


def test_every_entry_point_rejects_null_arguments():
    """Every status-returning entry point, called with null pointers and zero sizes, answers
    KLG_ERR_ARG from its own checks -- no dereference, no device work (run in a child process,
    so that a crash would fail this test instead of the session)."""
    import json
    import subprocess
    import sys
    # not applicable: no pointer arguments (version, error text, SM reserve, trace start,
    # split count), a release of nothing (klg_xr_close(NULL) is a no-op), a read of an empty
    # trace, and the self-test whose one argument is a stream and which needs a GPU
    exempt = {"klg_version", "klg_last_error", "klg_set_sm_reserve", "klg_trace_begin", "klg_block_attn_splits",
              "klg_xr_close", "klg_trace_end", "klg_selftest_wait_timeout"}
    names = [n for n, (res, _) in _lib.SIGNATURES.items() if res is ctypes.c_int and n not in exempt]
    assert len(names) >= 30
    out = subprocess.run([sys.executable, "-c", _NULL_CALLER, str(ROOT), *names], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    rcs = json.loads(out.stdout.strip().splitlines()[-1])
    bad = {n: rc for n, rc in rcs.items() if rc != _lib.KLG_ERR_ARG}
    assert not bad, bad
