"""Shared helpers for the GPU parity tests (compare the CUDA op with the oracle)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import klgemm_oracle as O

# Tolerances (fp32 reference on the same bf16-rounded inputs unless stated):
LOSS_RTOL = 1e-3      # loss, relative
LOSS_ATOL = 1e-6      # loss, absolute floor (a one-entry vocabulary has KL exactly 0)
GRAD_MAX_REL = 2e-2   # max|ours - ref| / max|ref|
GRAD_COS = 0.9999     # cosine similarity


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def run_ours(h_s, h_t, W, mask, T, need_dw=True, workspace_bytes=None, grad=None, path="split"):
    """Forward + backward through the C-ABI on cuda:0; returns numpy fp64 arrays.

    path "split": klg_fwd (single-pass statistics) then klg_bwd;
    path "fused": klg_fwd_bwd (pass-1 log-sum-exps on CTA pairs, KL cross term in pass 2).
    """
    from orthrus_training_test_b200 import ops
    from orthrus_training_test_b200 import _lib

    dev = torch.device("cuda:0")
    hs = ops.to_compute_dtype(h_s.to(dev))
    ht = ops.to_compute_dtype(h_t.to(dev))
    w = ops.to_compute_dtype(W.to(dev))
    m = mask.to(dev)
    g = None if grad is None else torch.tensor([float(grad)], device=dev)
    if path == "split":
        loss, lse, cnt, row_kl = ops.kl_forward(hs, ht, w, m, T, want_row_kl=True)
        dh, dw = ops.kl_backward(hs, ht, w, m, lse, cnt, grad=g, temperature=T, need_dh=True, need_dw=need_dw,
                                 workspace_bytes=workspace_bytes)
    else:
        loss, lse, cnt, row_kl, dh, dw = ops.kl_fwd_bwd(hs, ht, w, m, T, grad=g, need_dh=True, need_dw=need_dw,
                                                        want_row_kl=True, workspace_bytes=workspace_bytes)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0, "device pipeline timeout"
    out = dict(loss=float(loss.item()), row_kl=row_kl.double().cpu().numpy(), lse=lse.double().cpu().numpy(),
               count=float(cnt.item()), dh=dh.double().cpu().numpy(), path=path)
    out["dw"] = dw.double().cpu().numpy() if dw is not None else None
    return out


def run_both(*args, **kw):
    """Both entry paths on the same inputs."""
    return [run_ours(*args, path="split", **kw), run_ours(*args, path="fused", **kw)]


def run_oracle_np(h_s, h_t, W, mask, T):
    """float64 oracle on bf16-rounded inputs (what the kernels see)."""
    return O.aligned_kl_loss_np(bf16_round(h_s).numpy(), bf16_round(h_t).numpy(), bf16_round(W).numpy(),
                                mask.numpy(), T)


def run_oracle_torch_gpu(h_s, h_t, W, mask, T, chunk=2048, round_inputs=True):
    """fp32 torch oracle (the reference op sequence) on the GPU.

    ``round_inputs``: evaluate on the bf16-rounded inputs the kernels consume
    (default) or on the caller's fp32 values as given.
    """
    dev = torch.device("cuda:0")
    cv = bf16_round if round_inputs else (lambda x: x.float())
    loss, dh, dw = O.aligned_kl_torch_with_grads(cv(h_s).to(dev), cv(h_t).to(dev), cv(W).to(dev), mask.to(dev), T,
                                                 chunk=chunk)
    return float(loss.item()), dh.double().cpu().numpy(), dw.double().cpu().numpy()


def assert_close(ours, ref_loss, ref_dh, ref_dw, label=""):
    if isinstance(ours, list):
        for o in ours:
            assert_close(o, ref_loss, ref_dh, ref_dw, f"{label} [{o['path']}]")
        return
    rel = abs(ours["loss"] - ref_loss) / max(abs(ref_loss), 1e-12)
    assert rel <= LOSS_RTOL or abs(ours["loss"] - ref_loss) <= LOSS_ATOL, \
        f"{label} loss {ours['loss']} vs {ref_loss} (rel {rel:.2e})"
    if ref_dh is not None:
        mr, cos = O.grad_metrics(ours["dh"], ref_dh)
        assert mr <= GRAD_MAX_REL and cos >= GRAD_COS, f"{label} dH max_rel {mr:.2e} cos {cos:.6f}"
    if ref_dw is not None and ours["dw"] is not None:
        mr, cos = O.grad_metrics(ours["dw"], ref_dw)
        assert mr <= GRAD_MAX_REL and cos >= GRAD_COS, f"{label} dW max_rel {mr:.2e} cos {cos:.6f}"
