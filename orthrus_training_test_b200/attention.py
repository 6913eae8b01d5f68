"""Block-diffusion attention (forward) for the diffusion heads, on tcgen05.

The reference's diffusion heads (model.py:100-176) attend with flex_attention
(model.py:45-58): a static block mask -- every AR cache key plus the query's own block of
K diffusion keys, bidirectionally (model.py:64-96) -- and a score_mod that hides the AR
keys past each query's causal limit (model.py:435-446); GQA maps query head h to KV head
h / (H / Hkv).  The Triton replacement (triton_kernels.py:18-83, 281-290) is marked broken
in the reference.  ``block_attention`` computes the same attention in one CUDA kernel per
(batch, KV head, head group, block, key split); the key splits of a decode call form a
thread-block cluster and combine through distributed shared memory.

Forward for generation and, through :class:`BlockAttentionFn`, a backward (dQ and the
block keys' dK / dV) for training the heads.  Every function here calls the CUDA library;
there is no CPU fallback.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib  # noqa: F401  (loads the library)
from ._lib import call
from .ops import _ptr, _require_cuda, _stream

HEAD_DIM = 64


def _bf16(x: torch.Tensor) -> torch.Tensor:
    if x.dtype == torch.bfloat16:
        return x
    if x.dtype == torch.float32:
        return x.to(torch.bfloat16)
    raise TypeError(f"unsupported dtype {x.dtype} (bf16 or fp32)")


def _cache_rows(kv: torch.Tensor) -> Tuple[torch.Tensor, int]:
    """``[B, Hkv, ar_len, D]``, possibly the first ``ar_len`` rows of a longer cache
    (``cache[:, :, :ar_len, :]``): returns the tensor and its row count per head."""
    B, Hkv, n, D = kv.shape
    st = kv.stride()
    if st[3] == 1 and st[2] == D and st[1] % D == 0 and st[1] // D >= n and st[0] == Hkv * st[1] \
            and kv.data_ptr() % 16 == 0:
        return kv, st[1] // D
    kv = kv.contiguous()
    return kv, n


def workspace_bytes(batch, heads, kv_heads, diff_len, block, ar_len, head_dim=HEAD_DIM) -> int:
    n = _lib.lib().klg_block_attn_workspace_bytes(batch, heads, kv_heads, diff_len, block, ar_len, head_dim)
    if n < 0:
        raise ValueError(_lib.last_error())
    return int(n)


def block_attention(q: torch.Tensor, k_self: torch.Tensor, v_self: torch.Tensor, k_ar: torch.Tensor,
                    v_ar: torch.Tensor, limits: torch.Tensor, block_size: int, scale: Optional[float] = None,
                    want_lse: bool = False, workspace: Optional[torch.Tensor] = None):
    """Attention of the diffusion queries over the AR cache and their own block.

    ``q [B, H, Ld, 64]``; ``k_self, v_self [B, Hkv, Ld, 64]`` (the diffusion positions' own
    keys / values); ``k_ar, v_ar [B, Hkv, ar_len, 64]`` (may be ``cache[:, :, :ar_len]``);
    ``limits [B, Ld]`` -- query position p sees AR keys ``0..limits[b, p]`` (clamped; -1:
    none) and the ``block_size`` keys of block ``p // block_size``.  ``scale`` defaults to
    ``1/sqrt(64)``.  Returns ``out [B, H, Ld, 64]`` bf16 (and ``lse [B, H, Ld]`` fp32,
    natural log, when ``want_lse``).  When ``q``, ``k_self`` or ``v_self`` requires a gradient
    (and ``want_lse`` is not asked), the call is differentiable through
    :class:`BlockAttentionFn`.
    """
    if (torch.is_grad_enabled() and not want_lse and workspace is None
            and any(t.requires_grad for t in (q, k_self, v_self))):
        if k_ar.requires_grad or v_ar.requires_grad:
            raise ValueError("the AR cache gets no gradient (frozen backbone): pass it detached")
        return BlockAttentionFn.apply(q, k_self, v_self, k_ar, v_ar, limits, block_size, scale)
    return _attn_forward(q, k_self, v_self, k_ar, v_ar, limits, block_size, scale, want_lse, workspace)


def _prepare(q, k_self, v_self, k_ar, v_ar, limits, block_size, scale):
    """Checked, contiguous bf16 operands and the launch sizes of a forward / backward call."""
    _require_cuda(q, k_self, v_self, k_ar, v_ar, limits)
    B, H, Ld, D = q.shape
    Hkv = k_self.shape[1]
    ar_len = k_ar.shape[2]
    if D != HEAD_DIM:
        raise ValueError(f"head_dim {D}: only {HEAD_DIM} is built")
    if tuple(k_self.shape) != (B, Hkv, Ld, D) or tuple(v_self.shape) != (B, Hkv, Ld, D):
        raise ValueError("k_self / v_self must be [B, Hkv, Ld, 64]")
    if tuple(k_ar.shape) != (B, Hkv, ar_len, D) or tuple(v_ar.shape) != (B, Hkv, ar_len, D):
        raise ValueError("k_ar / v_ar must be [B, Hkv, ar_len, 64]")
    if tuple(limits.shape) != (B, Ld):
        raise ValueError("limits must be [B, Ld]")
    qc = _bf16(q.detach()).contiguous()
    ks = _bf16(k_self.detach()).contiguous()
    vs = _bf16(v_self.detach()).contiguous()
    ka, stride_k = _cache_rows(_bf16(k_ar.detach()))
    va, stride_v = _cache_rows(_bf16(v_ar.detach()))
    if stride_k != stride_v:
        ka, va = k_ar.detach().to(torch.bfloat16).contiguous(), v_ar.detach().to(torch.bfloat16).contiguous()
        stride_k = ar_len
    lim = limits.detach().to(torch.int32).contiguous()
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    return (qc, ks, vs, ka, va, lim), (stride_k, B, H, Hkv, Ld, int(block_size), ar_len, D, float(scale))


def _launch_fwd(tensors, meta, want_lse=False, workspace=None):
    qc, ks, vs, ka, va, lim = tensors
    stride_k, B, H, Hkv, Ld, K, ar_len, D, scale = meta
    dev = qc.device
    need = workspace_bytes(B, H, Hkv, Ld, K, ar_len, D)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    out = torch.empty(B, H, Ld, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, H, Ld, dtype=torch.float32, device=dev) if want_lse else None
    call("klg_block_attn_fwd", _ptr(qc), _ptr(ks), _ptr(vs), _ptr(ka), _ptr(va), stride_k, _ptr(lim), B, H, Hkv, Ld,
         K, ar_len, D, scale, _ptr(out), _ptr(lse), _ptr(workspace), workspace.numel() * workspace.element_size(),
         _stream(dev))
    return (out, lse) if want_lse else out


def _attn_forward(q, k_self, v_self, k_ar, v_ar, limits, block_size, scale, want_lse=False, workspace=None):
    tensors, meta = _prepare(q, k_self, v_self, k_ar, v_ar, limits, block_size, scale)
    return _launch_fwd(tensors, meta, want_lse, workspace)


class BlockAttentionFn(torch.autograd.Function):
    """:func:`block_attention` with a backward: dQ and the block keys' dK / dV from the forward's
    log-sum-exps (``klg_block_attn_bwd``; the reference's Triton autograd is
    triton_kernels.py:144-172).  The AR cache gets no gradient -- it comes from the frozen
    backbone -- so ``k_ar`` / ``v_ar`` must not require one."""

    @staticmethod
    def forward(ctx, q, k_self, v_self, k_ar, v_ar, limits, block_size, scale):
        tensors, meta = _prepare(q, k_self, v_self, k_ar, v_ar, limits, block_size, scale)
        out, lse = _launch_fwd(tensors, meta, want_lse=True)
        ctx.save_for_backward(*tensors, out, lse)
        ctx.meta = meta
        ctx.dtypes = (q.dtype, k_self.dtype, v_self.dtype)
        return out

    @staticmethod
    def backward(ctx, d_out):
        qc, ks, vs, ka, va, lim, out, lse = ctx.saved_tensors
        stride, B, H, Hkv, Ld, K, ar_len, D, scale = ctx.meta
        dev = qc.device
        do = d_out.detach().to(torch.bfloat16).contiguous()
        dq = torch.empty(B, H, Ld, D, dtype=torch.float32, device=dev)
        dk = torch.empty(B, Hkv, Ld, D, dtype=torch.float32, device=dev)
        dv = torch.empty(B, Hkv, Ld, D, dtype=torch.float32, device=dev)
        call("klg_block_attn_bwd", _ptr(qc), _ptr(ks), _ptr(vs), _ptr(ka), _ptr(va), stride, _ptr(lim), _ptr(out),
             _ptr(lse), _ptr(do), B, H, Hkv, Ld, K, ar_len, D, float(scale), _ptr(dq), _ptr(dk), _ptr(dv), _stream(dev))
        return dq.to(ctx.dtypes[0]), dk.to(ctx.dtypes[1]), dv.to(ctx.dtypes[2]), None, None, None, None, None


def triton_block_attention(q, k_self, v_self, k_ar, v_ar, limits, B, H, Hkv, ng, BG, n_blocks, K, ar_len, D):
    """Drop-in for the reference's ``triton_block_attention`` (triton_kernels.py:281-290):
    ``q [B*H, Ld, D]``, ``k_self / v_self [B*Hkv, Ld, D]``, ``k_ar / v_ar [B*Hkv, ar_len, D]``,
    ``limits [B, Ld]``; returns ``[B*H, Ld, D]``.  ``ng`` and ``BG`` (the Triton grid's
    block groups) are implied by the shapes and ignored.  Limits apply per query position,
    as the flex-attention path does (model.py:435-446); the Triton kernel reads the first
    position's limit of each block, which is the same whenever a block shares one limit
    (as generate.py:158-160 sets it).  Forward only.
    """
    Ld = n_blocks * K
    out = block_attention(q.view(B, H, Ld, D), k_self.view(B, Hkv, Ld, D), v_self.view(B, Hkv, Ld, D),
                          k_ar.reshape(B, Hkv, ar_len, D), v_ar.reshape(B, Hkv, ar_len, D), limits, K)
    return out.view(B * H, Ld, D).to(q.dtype)
