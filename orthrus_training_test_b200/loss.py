"""Drop-in for the reference's ``compute_kl_loss`` (train.py:142-195).

Same signature and semantics; the arithmetic runs in the fused sm_100a op
(:class:`~orthrus_training_test_b200.ops.KLGemmFn`).  ``teacher_probs`` and
``teacher_ent`` are accepted and ignored: the fused op recomputes the teacher
logits tile by tile, so the caller can drop the ``[B, L, V]`` precompute of
train.py:549-567.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib  # noqa: F401  (loads the library)
from ._lib import call
from .ops import KLGemmFn, PrenormKLGemmFn, _ptr, _require_cuda, _stream

_index_cache: dict = {}


def kl_indices(B: int, B_blocks: int, K: int, device) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``(diff_pos [B,N], batch_idx [B,N], offsets [K-1])`` as in train.py:124-139.

    Student rows are the diffusion positions ``blk*K + k`` for k = 1..K-1 (the
    anchor at offset 0 carries no loss); teacher offsets are 0..K-2.
    """
    key = (B, B_blocks, K, str(device))
    hit = _index_cache.get(key)
    if hit is None:
        N = B_blocks * (K - 1)
        diff_pos = torch.arange(B_blocks * K, device=device).view(B_blocks, K)[:, 1:].reshape(-1)
        diff_pos = diff_pos.unsqueeze(0).expand(B, N)
        batch_idx = torch.arange(B, device=device).unsqueeze(1).expand(B, N)
        offsets = torch.arange(0, K - 1, device=device)
        hit = (diff_pos, batch_idx, offsets)
        _index_cache[key] = hit
    return hit


def select_rows(diff_hidden, ar_hidden_states, anchor_positions, K, target_ids, pad_token_id):
    """Aligned ``(h_s [B*N, H], h_t [B*N, H], valid [B*N])`` of train.py:156-164 in torch
    index ops (any device; the loss uses the one-kernel :func:`gather_rows`).

    Teacher row = ``anchor + k - 1`` clamped to ``[0, L-1]`` (train.py:161);
    valid = ``target != pad_token_id`` (train.py:163-164).  The student gather
    is differentiable (its backward scatters dH_s into ``diff_hidden.grad``).
    """
    B, B_blocks = anchor_positions.shape
    L = ar_hidden_states.shape[1]
    N = B_blocks * (K - 1)
    diff_pos, batch_idx, offsets = kl_indices(B, B_blocks, K, diff_hidden.device)
    ar_pos = (anchor_positions.unsqueeze(-1) + offsets).view(B, N).clamp(0, L - 1)
    valid = target_ids[batch_idx, diff_pos] != pad_token_id
    h_s = diff_hidden[batch_idx, diff_pos].reshape(B * N, -1)
    h_t = ar_hidden_states[batch_idx, ar_pos].reshape(B * N, -1)
    return h_s, h_t, valid.reshape(-1)


def _check_selection_shapes(diff_hidden, ar_hidden_states, anchor_positions, K, target_ids):
    """``(B, P, H, L, B_blocks)`` of a row selection, or ValueError: every index the gather
    kernel forms from these shapes stays inside its tensor (where train.py:156-164's torch
    indexing would raise, this raises before anything reaches the device).  Anchor values
    need no check: the teacher row is clamped to ``[0, L-1]``."""
    if diff_hidden.dim() != 3 or ar_hidden_states.dim() != 3:
        raise ValueError(f"expected diff_hidden [B, B_blocks*K, H] and ar_hidden_states [B, L, H], got "
                         f"{tuple(diff_hidden.shape)} and {tuple(ar_hidden_states.shape)}")
    B, P, H = diff_hidden.shape
    L = ar_hidden_states.shape[1]
    if ar_hidden_states.shape[0] != B or ar_hidden_states.shape[2] != H or L < 1:
        raise ValueError(f"ar_hidden_states {tuple(ar_hidden_states.shape)} does not match diff_hidden "
                         f"{tuple(diff_hidden.shape)} (same B and H, L >= 1)")
    if K < 2:
        raise ValueError(f"K={K}: a block needs an anchor and at least one diffusion position")
    if anchor_positions.dim() != 2 or anchor_positions.shape[0] != B:
        raise ValueError(f"anchor_positions must be [B={B}, B_blocks], got {tuple(anchor_positions.shape)}")
    Bb = anchor_positions.shape[1]
    if P != Bb * K:
        raise ValueError(f"diff_hidden has {P} positions, expected B_blocks*K = {Bb * K}")
    if target_ids.dim() != 2 or target_ids.shape[0] != B or target_ids.shape[1] < P:
        raise ValueError(f"target_ids must be [B={B}, >= {P}], got {tuple(target_ids.shape)}")
    return B, P, H, L, Bb


class GatherRowsFn(torch.autograd.Function):
    """The row selection of train.py:124-139, 156-164 as one CUDA kernel.

    ``(h_s [B*N, H], h_t [B*N, H], valid [B*N] uint8)`` with ``N = B_blocks*(K-1)``: the
    student rows ``diff_hidden[b, blk*K + k]`` (k = 1..K-1), the teacher rows
    ``ar_hidden[b, clamp(anchor + k - 1, 0, L-1)]`` and ``target != pad``.  The backward
    writes the student rows' gradient back to their positions of ``diff_hidden`` (zeros at
    the anchors), in one kernel as well.  ``h_t`` and ``valid`` carry no gradient (the
    teacher is detached, train.py:183).
    """

    @staticmethod
    def forward(ctx, diff_hidden, ar_hidden_states, anchor_positions, K, target_ids, pad_token_id):
        B, P, H, L, Bb = _check_selection_shapes(diff_hidden, ar_hidden_states, anchor_positions, K, target_ids)
        dev = _require_cuda(diff_hidden, ar_hidden_states, anchor_positions, target_ids)
        diff = diff_hidden.detach().contiguous()
        ar = ar_hidden_states.detach().to(diff.dtype).contiguous()
        row_bytes = H * diff.element_size()
        anchors = anchor_positions.detach().to(torch.int64).contiguous()
        # the kernel reads target row b at b * P: positions past the diffusion positions
        # (train.py:163 indexes only those) are dropped here
        targets = target_ids.detach()[:, :P].to(torch.int64).contiguous()
        n = B * Bb * (K - 1)
        h_s = torch.empty(n, H, dtype=diff.dtype, device=dev)
        h_t = torch.empty(n, H, dtype=diff.dtype, device=dev)
        valid = torch.empty(n, dtype=torch.uint8, device=dev)
        if n > 0:   # no blocks (or no sequences): nothing selected, as the reference's empty index tensors
            call("klg_gather_rows", _ptr(diff), _ptr(ar), _ptr(anchors), _ptr(targets), B, Bb, K, ar.shape[1],
                 row_bytes, int(pad_token_id), _ptr(h_s), _ptr(h_t), _ptr(valid), _stream(dev))
        ctx.meta = (B, Bb, K, H, diff.dtype, row_bytes)
        ctx.mark_non_differentiable(h_t, valid)
        return h_s, h_t, valid

    @staticmethod
    def backward(ctx, g_hs, g_ht, g_valid):
        B, Bb, K, H, dtype, row_bytes = ctx.meta
        g = g_hs.detach().to(dtype).contiguous()
        d_diff = torch.empty(B, Bb * K, H, dtype=dtype, device=g.device)
        if d_diff.numel() > 0:
            call("klg_scatter_rows_grad", _ptr(g), B, Bb, K, row_bytes, _ptr(d_diff), _stream(g.device))
        return d_diff, None, None, None, None, None


def gather_rows(diff_hidden, ar_hidden_states, anchor_positions, K, target_ids, pad_token_id):
    """``(h_s, h_t, valid)`` of :func:`select_rows`, computed by one CUDA kernel."""
    return GatherRowsFn.apply(diff_hidden, ar_hidden_states, anchor_positions, int(K), target_ids, int(pad_token_id))


def compute_kl_loss(diff_hidden: torch.Tensor, ar_hidden_states: torch.Tensor, lm_head: torch.nn.Module,
                    anchor_positions: torch.Tensor, K: int, target_ids: torch.Tensor, pad_token_id: int,
                    teacher_probs=None, teacher_ent=None, temperature: float = 1.0, *,
                    norm_weight: Optional[torch.Tensor] = None, norm_eps: float = 1e-5) -> torch.Tensor:
    """Forward KL(teacher || student) averaged over valid diffusion positions.

    Signature of train.py:142-152 (plus an optional ``temperature``, default 1
    = the reference).  Returns a 0-d fp32 tensor; ``0.0`` with
    ``requires_grad`` when no position is valid (train.py:166-167).
    With ``norm_weight`` given, ``diff_hidden`` and ``ar_hidden_states`` are the hidden
    states before the backbone's final norm (model.py:493) and the norm runs inside the
    op on the selected rows only (it is per row, so selecting first is the same).
    """
    if getattr(lm_head, "bias", None) is not None:
        raise ValueError("lm_head with a bias is not supported (the reference's tied lm_head has none)")
    h_s, h_t, valid = gather_rows(diff_hidden, ar_hidden_states, anchor_positions, K, target_ids, pad_token_id)
    if not bool(valid.any()):
        return torch.tensor(0.0, device=diff_hidden.device, requires_grad=True)
    if norm_weight is not None:
        return PrenormKLGemmFn.apply(h_s, h_t.detach(), norm_weight, lm_head.weight, valid, float(temperature),
                                     float(norm_eps), None)
    return KLGemmFn.apply(h_s, h_t.detach(), lm_head.weight, valid, float(temperature), None)
