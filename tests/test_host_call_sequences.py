"""The host-side checks of the Python layer accept every call sequence the GPU path makes.

The shape / dtype / density checks in ``ops``, ``loss`` and ``sampling`` run before any device
pointer is formed.  Here the library's launches are replaced by a recorder and the device check
by the host, so the call sequences of the autograd ops, the shim, the pieces of the vocab-sharded
step, the norm prologue and the sampler run on CPU tensors with the shapes and dtypes the GPU
tests and the benchmark use: a check that wrongly rejected one of them fails here, without a GPU.
Nothing is computed (outputs are uninitialised); the GPU tests check the numbers."""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from orthrus_training_test_b200 import _lib, ops, sampling
from orthrus_training_test_b200 import loss as lossmod
from orthrus_training_test_b200 import parallel

GOLDEN = Path(__file__).resolve().parent / "golden"


class _Sizes:
    """Workspace-size queries answered on the host (the real ones read the device's SM count);
    every other symbol comes from the real library."""

    def __init__(self, real):
        self._real = real

    def __getattr__(self, name):
        if name.endswith("_workspace_bytes") or name in ("klg_xr_buffer_bytes", "klg_fwd_bwd_chunk_cols"):
            return lambda *a: 1 << 12
        return getattr(self._real, name)


@pytest.fixture
def launches(monkeypatch):
    seen = []
    sizes = _Sizes(_lib.lib())
    monkeypatch.setattr(_lib, "lib", lambda: sizes)
    for m in (ops, lossmod, sampling):
        monkeypatch.setattr(m, "call", lambda name, *a: seen.append(name), raising=False)
        monkeypatch.setattr(m, "_require_cuda", lambda *ts: torch.device("cpu"), raising=False)
        monkeypatch.setattr(m, "_stream", lambda dev: ctypes.c_void_p(0), raising=False)
    monkeypatch.setattr(ops, "num_partials", lambda n, v: 2)
    return seen


def _bf(*shape):
    return torch.randn(*shape).to(torch.bfloat16)


def test_autograd_ops_and_pieces(launches):
    N, H, V = 300, 576, 1000
    mask = torch.rand(N) < 0.5
    # the autograd op, bf16 and fp32 (smoke(), the parity tests), with and without gradients
    hs, w = _bf(N, H).requires_grad_(True), _bf(V, H).requires_grad_(True)
    ops.kl_gemm_loss(hs, _bf(N, H), w, mask, 1.0).backward()
    hs32, w32 = torch.randn(N, H).requires_grad_(True), torch.randn(V, H).requires_grad_(True)
    ops.kl_gemm_loss(hs32, torch.randn(N, H), w32, mask, 2.0).backward()
    with torch.no_grad():
        ops.kl_gemm_loss(hs32, torch.randn(N, H), w32, mask, 2.0)
    # the split and one-call routes of the GPU test helpers
    hb, tb, wb = _bf(N, H), _bf(N, H), _bf(V, H)
    loss, lse, cnt, _ = ops.kl_forward(hb, tb, wb, mask, 1.0, want_row_kl=True)
    ops.kl_backward(hb, tb, wb, mask, lse, cnt, grad=torch.tensor([2.0]), need_dh=True, need_dw=True,
                    workspace_bytes=4096)
    ops.kl_fwd_bwd(hb, tb, wb, mask, 1.0, grad=torch.tensor([2.0]), need_dw=False, want_row_kl=True)
    # views of one [2, N, H] buffer, and one tensor as both views (the dZ kernel tests)
    buf = _bf(2, N, H)
    ops.kl_fwd_bwd(buf[1], buf[0], wb, mask, 1.0)
    ops.kl_fwd_bwd(hb, hb, wb, mask, 1.0, grad=torch.zeros(1))
    # the step in pieces, and vocab sharding through the engine (two slices)
    m = ops.mask_u8(mask)
    lse2 = ops.lse_merge(ops.lse_record(hb, tb, wb, 1.0)[None])
    _, _, cross = ops.pass2(hb, tb, wb, m, lse2, cnt, temperature=1.0)
    ops.kl_loss(lse2, cross, m, cnt, want_row_kl=True)
    eng = parallel.CudaEngine()
    count = eng.count(m)
    slices = [(0, 500), (500, 1000)]
    lse = eng.lse_merge(torch.stack([eng.lse_record(hb, tb, wb[a:b].contiguous(), 1.0) for a, b in slices]))
    for a, b in slices:
        eng.pass2(hb, tb, wb[a:b].contiguous(), m, lse, count, 1.0, True, True)
    parts = torch.stack([eng.partial_stats(hb, tb, wb[a:b].contiguous(), 1.0) for a, b in slices])
    eng.finalize(eng.merge(parts), m, count)
    # the benchmark's vocab-sharded step: dH in a view of the [dH | cross] buffer
    xbuf = torch.empty(N * H + N)
    ops.pass2(hb, tb, wb, m, lse, count, temperature=1.0, workspace_bytes=4096, dh_out=xbuf[:N * H].view(N, H))
    ops.kl_loss(lse, xbuf[N * H:], m, count)
    ops.lse_merge(torch.empty(2 * 2, 2 * N).view(2, 2, 2 * N))
    assert {"klg_fwd_bwd", "klg_fwd_bwd_f32", "klg_fwd", "klg_bwd", "klg_pass2", "klg_lse_record"} <= set(launches)


def test_norm_prologue_and_sampler(launches):
    N, H, V = 64, 576, 1000
    mask = torch.rand(N) < 0.5
    ops.prenorm_kl_loss(_bf(N, H).requires_grad_(True), _bf(N, H), torch.ones(H),
                        _bf(V, H).requires_grad_(True), mask, 1.0).backward()
    _, r = ops.rmsnorm_rows(_bf(8, 64), torch.ones(64))
    ops.rmsnorm_rows_backward(_bf(8, 64), torch.ones(64), r, torch.randn(8, 64))
    sampling.lm_head_sample(_bf(4, H), _bf(V, H), 0.0)
    sampling.lm_head_sample(_bf(4, H), _bf(V, H), 1.0, seed=3)
    assert {"klg_rmsnorm_rows", "klg_rmsnorm_rows_bwd", "klg_lm_head_sample"} <= set(launches)


@pytest.mark.parametrize("name", ["aligned_t1", "aligned_t2_peaky", "aligned_h128_v300", "anchors_clamp"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_shim_on_the_golden_inputs(launches, name, dtype):
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    K, pad = int(g["K"]), int(g["pad"])
    diff = torch.tensor(g["diff_hidden"]).to(dtype).requires_grad_(True)
    ar = torch.tensor(g["ar_hidden"]).to(dtype)
    head = torch.nn.Linear(diff.shape[-1], 300, bias=False).to(dtype)
    args = (torch.tensor(g["anchor_positions"]), K, torch.tensor(g["target_ids"]), pad)
    lossmod.compute_kl_loss(diff, ar, head, *args)
    lossmod.compute_kl_loss(diff, ar, head, *args, norm_weight=torch.ones(diff.shape[-1]))
    h_s, _, _ = lossmod.gather_rows(diff, ar, *args)
    h_s.float().sum().backward()
    assert "klg_gather_rows" in launches and "klg_scatter_rows_grad" in launches
