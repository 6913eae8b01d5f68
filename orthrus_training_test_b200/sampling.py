"""Fused lm_head + token selection for inference.

The reference picks tokens with ``sample_token(logits, temperature, top_k, top_p)``
(generate.py:40-78, and the temperature-only copy at infer.py:60-69) on logits the
model has already written out as ``[..., V]`` (generate.py:161-188).  Here the
lm_head GEMM and the selection run in one CUDA kernel over vocab tiles: greedy
argmax, or a draw from ``softmax(z / T)`` by the Gumbel-max rule with a counter-based
generator keyed by (seed, row, column), plus the per-row log-sum-exp -- no ``[N, V]``
tensor is ever stored.  With top-k / top-p, two sweeps over the lm_head find each row's
candidates and a per-row kernel applies the reference's filter rules to them.

Every function here calls the CUDA library; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib  # noqa: F401  (loads the library)
from ._lib import call
from .ops import _ptr, _require_cuda, _stream, to_compute_dtype

GREEDY_TEMPERATURE = 1e-5   # generate.py:52


def workspace_bytes(n_rows: int, vocab: int) -> int:
    n = _lib.lib().klg_lm_head_sample_workspace_bytes(int(n_rows), int(vocab))
    if n < 0:
        raise ValueError(f"unsupported sampling problem n_rows={n_rows} vocab={vocab}")
    return int(n)


def lm_head_sample(h: torch.Tensor, weight: torch.Tensor, temperature: float = 0.0, seed: int = 0,
                   workspace: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Select one token per row of ``z = h @ weight^T`` without storing ``z``.

    ``h`` ``[N, H]`` and ``weight`` ``[V, H]`` (bf16; fp32 is cast).  ``temperature <
    1e-5`` (the reference's greedy threshold, generate.py:52) selects ``argmax z`` --
    the first index among equal maxima, as ``torch.argmax``; otherwise a draw from
    ``softmax(z / temperature)`` fixed by ``seed`` (the same seed, rows and logits give
    the same tokens on any device and any vocab split).

    Returns ``(tokens int64 [N], logit float32 [N], lse float32 [N])``: the chosen
    column, its logit ``z``, and ``log sum exp(z / T')`` with ``T' = temperature`` when
    sampling and ``1`` when greedy, so ``p(token) = exp(logit / T' - lse)``.
    """
    if h.dim() != 2 or weight.dim() != 2 or h.shape[1] != weight.shape[1]:
        raise ValueError(f"expected h [N, H] and weight [V, H], got {tuple(h.shape)} and {tuple(weight.shape)}")
    dev = _require_cuda(h, weight)
    h = to_compute_dtype(h)
    weight = to_compute_dtype(weight)
    N, H = h.shape
    V = weight.shape[0]
    sample = temperature >= GREEDY_TEMPERATURE
    inv_temp = 1.0 / float(temperature) if sample else 1.0
    need = workspace_bytes(N, V)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    tokens = torch.empty(N, dtype=torch.int32, device=dev)
    logit = torch.empty(N, dtype=torch.float32, device=dev)
    lse = torch.empty(N, dtype=torch.float32, device=dev)
    call("klg_lm_head_sample", _ptr(h), _ptr(weight), N, H, V, inv_temp, int(sample),
         ctypes.c_ulonglong(int(seed) & 0xFFFFFFFFFFFFFFFF), _ptr(tokens), _ptr(logit), _ptr(lse), _ptr(workspace),
         workspace.numel() * workspace.element_size(), _stream(dev))
    return tokens.long(), logit, lse


def lm_head_sample_filtered(h: torch.Tensor, weight: torch.Tensor, temperature: float, top_k: int = 0,
                            top_p: float = 1.0, seed: int = 0, cap: Optional[int] = None
                            ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """A draw from ``softmax(z / T)`` restricted by top-k / top-p (generate.py:55-75), for each
    row of ``z = h @ weight^T``, without storing ``z`` (two sweeps over ``weight``; see
    ``klg_lm_head_sample_filtered``).  ``cap`` bounds the candidates kept per row (default: a
    size that keeps the candidate lists under ~256 MiB); a row with more candidates is retried
    once with ``cap = V``.  Returns ``(tokens int64 [N], logit [N], lse [N])`` with ``lse`` the
    log-sum-exp of ``z / T`` over the surviving entries, so ``p(token) = exp(logit / T - lse)``
    is the reference's renormalised probability.
    """
    if h.dim() != 2 or weight.dim() != 2 or h.shape[1] != weight.shape[1]:
        raise ValueError(f"expected h [N, H] and weight [V, H], got {tuple(h.shape)} and {tuple(weight.shape)}")
    if temperature < GREEDY_TEMPERATURE:
        raise ValueError("filtering applies to sampling (temperature >= 1e-5); greedy selection has none")
    if top_k < 0 or not (0.0 < top_p <= 1.0):
        raise ValueError("top_k must be >= 0 and top_p in (0, 1]")
    dev = _require_cuda(h, weight)
    h = to_compute_dtype(h)
    weight = to_compute_dtype(weight)
    N, H = h.shape
    V = weight.shape[0]
    if cap is None:
        cap = min(V, max(2048, (256 << 20) // (8 * N)))
    tokens = torch.empty(N, dtype=torch.int32, device=dev)
    logit = torch.empty(N, dtype=torch.float32, device=dev)
    lse = torch.empty(N, dtype=torch.float32, device=dev)
    overflow = torch.zeros(1, dtype=torch.int32, device=dev)
    for attempt in range(2):
        need = int(_lib.lib().klg_lm_head_sample_filtered_workspace_bytes(N, V, int(cap)))
        if need < 0:
            raise ValueError(f"unsupported filtered-sampling problem N={N} V={V} cap={cap}")
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        call("klg_lm_head_sample_filtered", _ptr(h), _ptr(weight), N, H, V, 1.0 / float(temperature), int(top_k),
             float(top_p), ctypes.c_ulonglong(int(seed) & 0xFFFFFFFFFFFFFFFF), int(cap), _ptr(tokens), _ptr(logit),
             _ptr(lse), _ptr(overflow), _ptr(ws), need, _stream(dev))
        if int(overflow.item()) == 0:
            return tokens.long(), logit, lse
        if cap == V:
            break
        cap = V
    raise RuntimeError("filtered sampling: a row kept more candidates than the vocabulary size (internal error)")


def sample_token(hidden: torch.Tensor, weight: torch.Tensor, temperature: float = 0.0, top_k: int = 0,
                 top_p: float = 1.0, seed: Optional[int] = None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """``sample_token`` (generate.py:40-78) applied to ``hidden @ weight^T``.

    ``hidden`` is ``[H]``, ``[L, H]`` or ``[B, L, H]`` (the logits' shape minus the vocab
    dimension becomes the token shape, as in the reference).  Returns ``(tokens,
    None)`` when greedy and ``(tokens, p_token)`` otherwise, where ``p_token`` is the
    probability of each chosen token -- the reference returns the whole ``[..., V]``
    probability tensor, which the fused op never forms.  ``seed=None`` draws a seed
    from torch's default generator, so successive calls differ as
    ``torch.multinomial``'s draws do.  top-k / top-p filtering (generate.py:58-72) runs
    fused as well (:func:`lm_head_sample_filtered`); as in the reference it applies only
    when sampling.
    """
    lead = hidden.shape[:-1]
    h2 = hidden.reshape(-1, hidden.shape[-1])
    if seed is None:
        seed = int(torch.randint(0, 2 ** 62, (1,)).item())
    if temperature >= GREEDY_TEMPERATURE and (top_k > 0 or top_p < 1.0):
        tokens, logit, lse = lm_head_sample_filtered(h2, weight, temperature, top_k, top_p, seed)
    else:
        tokens, logit, lse = lm_head_sample(h2, weight, temperature, seed)
    tokens = tokens.view(lead)
    if temperature < GREEDY_TEMPERATURE:
        return tokens, None
    return tokens, torch.exp(logit / float(temperature) - lse).view(lead)


def token_logprob(h: torch.Tensor, weight: torch.Tensor, tokens: torch.Tensor, lse: torch.Tensor,
                  temperature: float = 1.0) -> torch.Tensor:
    """``log p(token)`` under ``softmax(h @ weight^T / T)`` for tokens chosen elsewhere.

    ``lse`` is :func:`lm_head_sample`'s output for the same rows and temperature.  This is
    what the consensus step reads as ``p_prob = ar_probs[0, i, diff_tokens[0, i]]``
    (generate.py:201-202): the AR distribution's probability of the diffusion head's token,
    here without the ``[N, V]`` probability tensor.  Returns fp32 ``[N]``.

    Shapes are checked before anything reaches the device: ``h [N, H]``, ``weight [V, H]``,
    ``tokens`` with ``N`` elements and ``lse [N]`` (the kernel reads one token and one
    weight row per row of ``h``).
    """
    if h.dim() != 2 or weight.dim() != 2 or weight.shape[1] != h.shape[1]:
        raise ValueError(f"expected h [N, H] and weight [V, H], got {tuple(h.shape)} and {tuple(weight.shape)}")
    if tokens.numel() != h.shape[0] or tuple(lse.shape) != (h.shape[0],):
        raise ValueError(f"tokens must have N={h.shape[0]} elements and lse shape ({h.shape[0]},), got "
                         f"{tokens.numel()} and {tuple(lse.shape)}")
    dev = _require_cuda(h, weight, tokens, lse)
    h = to_compute_dtype(h)
    weight = to_compute_dtype(weight)
    N, H = h.shape
    tok = tokens.detach().to(torch.int32).contiguous()
    z = torch.empty(N, dtype=torch.float32, device=dev)
    call("klg_token_logit", _ptr(h), _ptr(weight), _ptr(tok), N, H, weight.shape[0], _ptr(z), _stream(dev))
    T = float(temperature) if temperature >= GREEDY_TEMPERATURE else 1.0
    return z / T - lse
