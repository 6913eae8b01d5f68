"""PyTorch binding of the fused KL-GEMM distillation loss.

``KLGemmFn`` is the ``torch.autograd.Function`` that replaces the reference's
loss arithmetic (``train.py:142-210``).  When a gradient will be needed its
forward runs the whole training step: pass 1 (both views' logits over vocab
tiles with an online max / sum-exp per row, never storing an ``[N, V]``
tensor), then pass 2 (recompute the logits chunk by chunk, form dZ and the KL
cross term, then dH_s = dZ W and dW = dZ^T h_s).  It saves the fp32 dH_s
``[N, H]`` and dW ``[V, H]`` for an upstream gradient of 1, and its backward
only scales them by the actual upstream gradient.  Without gradients the
forward is the single-pass statistics kernel alone.

Every function here calls the CUDA library; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import call

_vp = ctypes.c_void_p


def _ptr(t: Optional[torch.Tensor]):
    return _vp(t.data_ptr()) if t is not None else _vp(0)


def _stream(device: torch.device):
    return _vp(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*ts):
    dev = ts[0].device
    if dev.type != "cuda":
        raise RuntimeError("the fused KL-GEMM loss runs on CUDA tensors only (no CPU path)")
    for t in ts:
        if t.device != dev:
            raise RuntimeError(f"all tensors must be on {dev}, got {t.device}")
    return dev


def _check_operands(h_s: torch.Tensor, h_t: torch.Tensor, weight: torch.Tensor, mask: Optional[torch.Tensor] = None,
                    allow_f32: bool = True) -> Tuple[int, int, int]:
    """``(N, H, V)`` of a consistent problem, or ValueError / TypeError before any device pointer
    is formed: the kernels read ``N x H`` elements of each view, ``V x H`` of the weight and
    ``N`` mask bytes, all dense and of one dtype (bf16, or fp32 where ``allow_f32``)."""
    if h_s.dim() != 2 or weight.dim() != 2 or h_t.shape != h_s.shape or weight.shape[1] != h_s.shape[1]:
        raise ValueError(f"expected h_s, h_t [N, H] and weight [V, H], got {tuple(h_s.shape)}, {tuple(h_t.shape)} "
                         f"and {tuple(weight.shape)}")
    N, H = h_s.shape
    if mask is not None and mask.numel() != N:
        raise ValueError(f"mask has {mask.numel()} elements, expected N={N}")
    dtypes = (torch.bfloat16, torch.float32) if allow_f32 else (torch.bfloat16,)
    if h_s.dtype not in dtypes or h_t.dtype != h_s.dtype or weight.dtype != h_s.dtype:
        raise TypeError(f"h_s, h_t and weight must share one dtype of {dtypes}, got {h_s.dtype}, {h_t.dtype}, "
                        f"{weight.dtype}")
    if not (h_s.is_contiguous() and h_t.is_contiguous() and weight.is_contiguous()):
        raise ValueError("h_s, h_t and weight must be contiguous")
    return N, H, weight.shape[0]


def _check_f32(name: str, t: Optional[torch.Tensor], shape: Tuple[int, ...]) -> None:
    """A dense fp32 buffer of ``shape`` that a kernel reads or writes as such."""
    if t is None:
        return
    if t.dtype != torch.float32 or tuple(t.shape) != tuple(shape) or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous fp32 tensor of shape {tuple(shape)}, got "
                         f"{t.dtype} {tuple(t.shape)}{'' if t.is_contiguous() else ' (strided)'}")


def _check_count(count: Optional[torch.Tensor]) -> None:
    if count is not None and (count.dtype != torch.float32 or count.numel() != 1):
        raise ValueError(f"count must be a one-element fp32 tensor, got {count.dtype} {tuple(count.shape)}")


def to_fp32(x: torch.Tensor) -> torch.Tensor:
    """fp32, contiguous (bf16 inputs widen exactly): the operands of the fp32-faithful path."""
    x = x.detach()
    _require_cuda(x)
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"unsupported dtype {x.dtype} (bf16 or fp32)")
    return x.float().contiguous()


def prepare_inputs(h_s: torch.Tensor, h_t: torch.Tensor, weight: torch.Tensor):
    """The operands in the arithmetic the op will use: all fp32 when any input is fp32 (the
    fp32-faithful path, split-bf16 on the tensor cores), else bf16."""
    if any(x.dtype == torch.float32 for x in (h_s, h_t, weight)):
        return to_fp32(h_s), to_fp32(h_t), to_fp32(weight)
    return to_compute_dtype(h_s), to_compute_dtype(h_t), to_compute_dtype(weight)


def scale_grad(x: torch.Tensor, g: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``(x * g).to(dtype)`` for a saved fp32 gradient ``x`` and the upstream gradient ``g`` (a
    device scalar), in one pass over ``x`` (``klg_scale_cast``) for bf16 and fp32 results.  Host
    tensors (the sharding logic's CPU test engine) use torch ops."""
    if dtype not in (torch.bfloat16, torch.float32) or not x.is_contiguous() or not x.is_cuda:
        return (x * g.to(torch.float32)).to(dtype)
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    gs = g.detach().to(device=x.device, dtype=torch.float32).reshape(1).contiguous()
    call("klg_scale_cast", _ptr(x), _ptr(gs), x.numel(), _ptr(out), int(dtype == torch.bfloat16), _stream(x.device))
    return out


def to_compute_dtype(x: torch.Tensor) -> torch.Tensor:
    """bf16, contiguous.  fp32 inputs are rounded to bf16 by the library's cast kernel."""
    x = x.detach()
    _require_cuda(x)
    if x.dtype == torch.bfloat16:
        return x.contiguous()
    if x.dtype == torch.float32:
        x = x.contiguous()
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
        call("klg_cast_f32_bf16", _ptr(x), _ptr(out), x.numel(), _stream(x.device))
        return out
    raise TypeError(f"unsupported dtype {x.dtype} (bf16 or fp32)")


def mask_u8(mask: torch.Tensor) -> torch.Tensor:
    if mask.dtype == torch.uint8:
        return mask.contiguous()
    return (mask != 0).to(torch.uint8).contiguous()


def num_partials(n_rows: int, vocab: int) -> int:
    n = ctypes.c_int(0)
    call("klg_num_partials", n_rows, vocab, ctypes.byref(n))
    return n.value


# ----------------------------------------------------------------- pass pieces

def count_valid(mask: torch.Tensor) -> torch.Tensor:
    """``sum(mask)`` as a float32 ``[1]`` device tensor (train.py:165)."""
    m = mask_u8(mask)
    dev = _require_cuda(m)
    out = torch.empty(1, dtype=torch.float32, device=dev)
    call("klg_count_valid", _ptr(m), m.numel(), _ptr(out), _stream(dev))
    return out


def fwd_stats(h_s: torch.Tensor, h_t: torch.Tensor, weight: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
    """Pass 1 partial records ``[n_part, 5, N]`` (log2 domain) over ``weight``'s rows."""
    N, H, V = _check_operands(h_s, h_t, weight, allow_f32=False)
    dev = _require_cuda(h_s, h_t, weight)
    n_part = num_partials(N, V)
    parts = torch.empty(n_part, 5, N, dtype=torch.float32, device=dev)
    call("klg_fwd_stats", _ptr(h_s), _ptr(h_t), _ptr(weight), N, H, V, 1.0 / float(temperature), _ptr(parts), n_part,
         _stream(dev))
    return parts


def merge_stats(parts: torch.Tensor) -> torch.Tensor:
    """Online-softmax merge ``[P, 5, N] -> [5, N]``."""
    if parts.dim() != 3 or parts.shape[1] != 5 or parts.dtype != torch.float32:
        raise ValueError(f"expected fp32 partial records [P, 5, N], got {parts.dtype} {tuple(parts.shape)}")
    parts = parts.contiguous()
    dev = _require_cuda(parts)
    P, _, N = parts.shape
    out = torch.empty(5, N, dtype=torch.float32, device=dev)
    call("klg_merge_stats", _ptr(parts), P, N, _ptr(out), _stream(dev))
    return out


def finalize(stats: torch.Tensor, mask: torch.Tensor, count: torch.Tensor,
             want_row_kl: bool = False) -> Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
    """``(loss [] fp32, lse [2, N] log2 domain, row_kl [N] or None)``."""
    m = mask_u8(mask)
    N = m.numel()
    _check_f32("stats", stats, (5, N))
    _check_count(count)
    dev = _require_cuda(stats, m, count)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    lse = torch.empty(2, N, dtype=torch.float32, device=dev)
    row_kl = torch.empty(N, dtype=torch.float32, device=dev) if want_row_kl else None
    call("klg_finalize", _ptr(stats), _ptr(m), N, _ptr(count), _ptr(loss), _ptr(lse), _ptr(row_kl), _stream(dev))
    return loss, lse, row_kl


def kl_forward(h_s: torch.Tensor, h_t: torch.Tensor, weight: torch.Tensor, mask: torch.Tensor,
               temperature: float = 1.0, count: Optional[torch.Tensor] = None, want_row_kl: bool = False):
    """Whole forward on one device.  ``count`` (a ``[1]`` fp32 device tensor)
    overrides the normaliser (e.g. an all-reduced global count).  bf16 inputs take the bf16
    path; fp32 inputs (all three) the fp32-faithful split-bf16 path.

    Returns ``(loss, lse, count, row_kl)``.
    """
    m = mask_u8(mask)
    N, H, V = _check_operands(h_s, h_t, weight, m)
    _check_count(count)
    dev = _require_cuda(h_s, h_t, weight, m)
    f32 = h_s.dtype == torch.float32
    ws_bytes = int(_lib.lib().klg_fwd_f32_workspace_bytes(N, H, V) if f32 else _lib.lib().klg_fwd_workspace_bytes(N, V))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    given = count is not None
    cnt = count if given else torch.empty(1, dtype=torch.float32, device=dev)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    lse = torch.empty(2, N, dtype=torch.float32, device=dev)
    row_kl = torch.empty(N, dtype=torch.float32, device=dev) if want_row_kl else None
    call("klg_fwd_f32" if f32 else "klg_fwd", _ptr(h_s), _ptr(h_t), _ptr(weight), _ptr(m), N, H, V, 1.0 / float(temperature), int(given),
         _ptr(cnt), _ptr(loss), _ptr(lse), _ptr(row_kl), _ptr(ws), ws_bytes, _stream(dev))
    return loss, lse, cnt, row_kl


def kl_backward(h_s, h_t, weight, mask, lse, count, grad: Optional[torch.Tensor] = None, temperature: float = 1.0,
                need_dh: bool = True, need_dw: bool = True, workspace_bytes: Optional[int] = None):
    """Pass 2: ``(dH_s [N, H] fp32 or None, dW [V, H] fp32 or None)``.

    ``grad`` is the upstream gradient as a device scalar (None = 1).
    ``workspace_bytes`` sizes the dZ chunk (default: the library's choice).
    """
    m = mask_u8(mask)
    N, H, V = _check_operands(h_s, h_t, weight, m, allow_f32=False)
    _check_f32("lse", lse, (2, N))
    _check_count(count)
    dev = _require_cuda(h_s, h_t, weight, m, lse, count)
    if workspace_bytes is None:
        workspace_bytes = int(_lib.lib().klg_bwd_workspace_bytes(N, H, V))
    ws = torch.empty(int(workspace_bytes), dtype=torch.uint8, device=dev)
    dh = torch.empty(N, H, dtype=torch.float32, device=dev) if need_dh else None
    dw = torch.empty(V, H, dtype=torch.float32, device=dev) if need_dw else None
    g = None
    if grad is not None:
        g = grad.detach().to(device=dev, dtype=torch.float32).reshape(1).contiguous()
    call("klg_bwd", _ptr(h_s), _ptr(h_t), _ptr(weight), _ptr(m), _ptr(lse), _ptr(count), _ptr(g), N, H, V,
         1.0 / float(temperature), _ptr(dh), _ptr(dw), _ptr(ws), int(workspace_bytes), _stream(dev))
    return dh, dw


def chunk_bounds(n_rows: int, hidden: int, vocab: int, workspace_bytes: Optional[int] = None):
    """``[(v0, v1), ...]``: the vocab chunks of the training step's pass 2 (bf16 path) for this
    workspace size (default: the recommended one); dW rows ``[v0, v1)`` are final once that
    chunk's GEMM has run."""
    L = _lib.lib()
    if workspace_bytes is None:
        workspace_bytes = int(L.klg_fwd_bwd_workspace_bytes(n_rows, hidden, vocab))
    cols = int(L.klg_fwd_bwd_chunk_cols(n_rows, hidden, vocab, int(workspace_bytes)))
    if cols <= 0:
        raise ValueError(f"workspace of {workspace_bytes} bytes is too small")
    return [(v0, min(vocab, v0 + cols)) for v0 in range(0, vocab, cols)]


def new_chunk_events(n: int):
    """``n`` CUDA events (created, so that their handles exist) for ``kl_fwd_bwd(chunk_events=)``."""
    evs = [torch.cuda.Event() for _ in range(n)]
    for e in evs:
        e.record()
    return evs


def set_sm_reserve(n_sms: int) -> None:
    """Leave ``n_sms`` SMs of each device out of the persistent kernels' grids (room for NCCL)."""
    call("klg_set_sm_reserve", int(n_sms))


def kl_fwd_bwd(h_s, h_t, weight, mask, temperature: float = 1.0, count: Optional[torch.Tensor] = None,
               grad: Optional[torch.Tensor] = None, need_dh: bool = True, need_dw: bool = True,
               want_row_kl: bool = False, workspace_bytes: Optional[int] = None, chunk_events=None):
    """Training step in one call: loss and gradients (for upstream gradient ``grad``, default 1).
    bf16 inputs take the bf16 path; fp32 inputs (all three) the fp32-faithful split-bf16 path.

    ``chunk_events`` (bf16 path): one ``torch.cuda.Event`` per vocab chunk of
    :func:`chunk_bounds`; event c is recorded on the current stream once chunk c's dW rows
    are final, so another stream can start exchanging them.

    Returns ``(loss, lse, count, row_kl, dH_s fp32 or None, dW fp32 or None)``.
    """
    m = mask_u8(mask)
    N, H, V = _check_operands(h_s, h_t, weight, m)
    _check_count(count)
    dev = _require_cuda(h_s, h_t, weight, m)
    f32 = h_s.dtype == torch.float32
    if workspace_bytes is None:
        workspace_bytes = int(_lib.lib().klg_fwd_bwd_f32_workspace_bytes(N, H, V) if f32
                              else _lib.lib().klg_fwd_bwd_workspace_bytes(N, H, V))
    ws = torch.empty(int(workspace_bytes), dtype=torch.uint8, device=dev)
    given = count is not None
    cnt = count if given else torch.empty(1, dtype=torch.float32, device=dev)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    lse = torch.empty(2, N, dtype=torch.float32, device=dev)
    row_kl = torch.empty(N, dtype=torch.float32, device=dev) if want_row_kl else None
    dh = torch.empty(N, H, dtype=torch.float32, device=dev) if need_dh else None
    dw = torch.empty(V, H, dtype=torch.float32, device=dev) if need_dw else None
    g = None
    if grad is not None:
        g = grad.detach().to(device=dev, dtype=torch.float32).reshape(1).contiguous()
    args = (_ptr(h_s), _ptr(h_t), _ptr(weight), _ptr(m), N, H, V, 1.0 / float(temperature), int(given), _ptr(cnt),
            _ptr(g), _ptr(loss), _ptr(lse), _ptr(row_kl), _ptr(dh), _ptr(dw), _ptr(ws), int(workspace_bytes))
    if chunk_events is not None:
        if f32:
            raise ValueError("chunk_events is for the bf16 path")
        handles = (ctypes.c_void_p * len(chunk_events))(*[e.cuda_event for e in chunk_events])
        call("klg_fwd_bwd_events", *args, handles, len(chunk_events), _stream(dev))
    else:
        call("klg_fwd_bwd_f32" if f32 else "klg_fwd_bwd", *args, _stream(dev))
    return loss, lse, cnt, row_kl, dh, dw


def kl_fwd_bwd_xr(h_s, h_t, weight, mask, temperature: float, count: torch.Tensor, need_dh: bool, world: int,
                  rank: int, peer_buffers, epoch: int, workspace_bytes: Optional[int] = None):
    """Row-sharded training step whose dW is summed over the ranks inside the step, over NVLink
    peer memory (``klg_fwd_bwd_xr``): ``peer_buffers`` is a ctypes array of every rank's exchange
    buffer, ``epoch`` 1, 2, ... per call (the same on every rank), ``count`` the global count.
    bf16 inputs.  Returns ``(loss of the local rows, dH_s fp32 or None, dW fp32 summed over ranks)``.
    """
    m = mask_u8(mask)
    N, H, V = _check_operands(h_s, h_t, weight, m, allow_f32=False)
    _check_count(count)
    dev = _require_cuda(h_s, h_t, weight, m)
    if workspace_bytes is None:
        workspace_bytes = int(_lib.lib().klg_fwd_bwd_workspace_bytes(N, H, V))
    ws = torch.empty(int(workspace_bytes), dtype=torch.uint8, device=dev)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    lse = torch.empty(2, N, dtype=torch.float32, device=dev)
    dh = torch.empty(N, H, dtype=torch.float32, device=dev) if need_dh else None
    dw = torch.empty(V, H, dtype=torch.float32, device=dev)
    call("klg_fwd_bwd_xr", _ptr(h_s), _ptr(h_t), _ptr(weight), _ptr(m), N, H, V, 1.0 / float(temperature), 1,
         _ptr(count), None, _ptr(loss), _ptr(lse), None, _ptr(dh), _ptr(dw), _ptr(ws), int(workspace_bytes),
         int(world), int(rank), peer_buffers, ctypes.c_uint32(int(epoch) & 0xFFFFFFFF), _stream(dev))
    return loss, dh, dw


# ----------------------------------------------------------------- the training step in pieces

def lse_record(h_s, h_t, weight, temperature: float = 1.0) -> torch.Tensor:
    """Pass 1 over ``weight``'s rows: the merged ``(m, S)`` record ``[2, 2N]`` (log2 units;
    rows ``0..N-1`` student, ``N..2N-1`` teacher) -- one vocab shard's contribution."""
    N, H, V = _check_operands(h_s, h_t, weight, allow_f32=False)
    dev = _require_cuda(h_s, h_t, weight)
    ws_bytes = int(_lib.lib().klg_lse_workspace_bytes(N, V))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    rec = torch.empty(2, 2 * N, dtype=torch.float32, device=dev)
    call("klg_lse_record", _ptr(h_s), _ptr(h_t), _ptr(weight), N, H, V, 1.0 / float(temperature), _ptr(rec), _ptr(ws),
         ws_bytes, _stream(dev))
    return rec


def lse_merge(recs: torch.Tensor) -> torch.Tensor:
    """``[R, 2, 2N]`` records (e.g. gathered from R vocab shards) -> ``lse [2, N]`` (log2 units)."""
    if recs.dim() != 3 or recs.shape[1] != 2 or recs.shape[2] % 2 != 0 or recs.dtype != torch.float32:
        raise ValueError(f"expected fp32 records [R, 2, 2N], got {recs.dtype} {tuple(recs.shape)}")
    recs = recs.contiguous()
    dev = _require_cuda(recs)
    R, _, N2 = recs.shape
    lse = torch.empty(2, N2 // 2, dtype=torch.float32, device=dev)
    call("klg_lse_merge", _ptr(recs), R, N2 // 2, _ptr(lse), _stream(dev))
    return lse


def pass2(h_s, h_t, weight, mask, lse, count, grad: Optional[torch.Tensor] = None, temperature: float = 1.0,
          need_dh: bool = True, need_dw: bool = True, workspace_bytes: Optional[int] = None, dh_out=None):
    """Pass 2 over ``weight``'s rows with the global ``lse``: ``(dH [N, H] fp32 or None,
    dW [V, H] fp32 or None, cross [N] fp32)``; ``cross`` is this weight's part of the KL
    cross term (log2 units).  ``dh_out`` may supply the dH buffer (e.g. a view into a larger
    buffer that one all-reduce carries)."""
    m = mask_u8(mask)
    N, H, V = _check_operands(h_s, h_t, weight, m, allow_f32=False)
    _check_f32("lse", lse, (2, N))
    _check_f32("dh_out", dh_out, (N, H))
    _check_count(count)
    dev = _require_cuda(h_s, h_t, weight, m, lse, count)
    if workspace_bytes is None:
        workspace_bytes = int(_lib.lib().klg_pass2_workspace_bytes(N, H, V))
    ws = torch.empty(int(workspace_bytes), dtype=torch.uint8, device=dev)
    dh = (dh_out if dh_out is not None else torch.empty(N, H, dtype=torch.float32, device=dev)) if need_dh else None
    dw = torch.empty(V, H, dtype=torch.float32, device=dev) if need_dw else None
    cross = torch.empty(N, dtype=torch.float32, device=dev)
    g = None
    if grad is not None:
        g = grad.detach().to(device=dev, dtype=torch.float32).reshape(1).contiguous()
    call("klg_pass2", _ptr(h_s), _ptr(h_t), _ptr(weight), _ptr(m), _ptr(lse), _ptr(count), _ptr(g), N, H, V,
         1.0 / float(temperature), _ptr(dh), _ptr(dw), _ptr(cross), _ptr(ws), int(workspace_bytes), _stream(dev))
    return dh, dw, cross


def kl_loss(lse, cross, mask, count, want_row_kl: bool = False):
    """``(loss [] fp32, row_kl [N] or None)`` from complete cross terms."""
    m = mask_u8(mask)
    N = m.numel()
    _check_f32("lse", lse, (2, N))
    if cross.dtype != torch.float32 or cross.numel() != N:
        raise ValueError(f"cross must be fp32 with N={N} elements, got {cross.dtype} {tuple(cross.shape)}")
    _check_count(count)
    dev = _require_cuda(lse, cross, m, count)
    loss = torch.empty((), dtype=torch.float32, device=dev)
    row_kl = torch.empty(N, dtype=torch.float32, device=dev) if want_row_kl else None
    call("klg_kl_loss", _ptr(lse), _ptr(cross.contiguous()), _ptr(m), N, _ptr(count), _ptr(loss), _ptr(row_kl),
         _stream(dev))
    return loss, row_kl


# ----------------------------------------------------------------- autograd op

class KLGemmFn(torch.autograd.Function):
    """``loss = sum_i mask_i KL(softmax(h_t W^T / T) || softmax(h_s W^T / T)) / sum(mask)``.

    Arguments: ``h_s [N, H]`` (student rows, differentiable), ``h_t [N, H]``
    (teacher rows, treated as detached like train.py:183), ``weight [V, H]``
    (lm_head, differentiable if it requires grad), ``mask [N]``, ``temperature``
    (float), ``count`` (optional ``[1]`` device tensor overriding sum(mask)).
    bf16 inputs compute in bf16 on the tensor cores with fp32 accumulation and fp32
    softmax arithmetic; fp32 inputs (any of the three) take the fp32-faithful path: every
    operand split into bf16 hi / lo planes, logits and gradients to ~2^-16 relative before
    fp32 accumulation (the reference's CPU-runnable configuration and its fp32 teacher path,
    train.py:188-191, are fp32).

    When a gradient will be needed the forward runs the whole training step
    (``klg_fwd_bwd``) and keeps dH_s / dW for an upstream gradient of 1 (O(N*H +
    V*H), never O(N*V)); backward scales them by the actual upstream gradient.
    Without gradients (evaluation, train.py:845-911) it runs the single-pass
    forward (``klg_fwd``): both views' statistics and the KL in one sweep.
    """

    @staticmethod
    def forward(ctx, h_s, h_t, weight, mask, temperature=1.0, count=None):
        hs, ht, w = prepare_inputs(h_s, h_t, weight)
        m = mask_u8(mask)
        need_dh, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[2]
        ctx.dtypes = (h_s.dtype, weight.dtype)
        if need_dh or need_dw:
            loss, _, _, _, dh, dw = kl_fwd_bwd(hs, ht, w, m, temperature, count=count, need_dh=need_dh,
                                               need_dw=need_dw)
            ctx.save_for_backward(dh, dw)
        else:
            loss, _, _, _ = kl_forward(hs, ht, w, m, temperature, count=count)
        return loss

    @staticmethod
    def backward(ctx, g):
        dh, dw = ctx.saved_tensors
        return (scale_grad(dh, g, ctx.dtypes[0]) if dh is not None else None, None,
                scale_grad(dw, g, ctx.dtypes[1]) if dw is not None else None, None, None, None)


def kl_gemm_loss(h_s: torch.Tensor, h_t: torch.Tensor, weight: torch.Tensor, mask: torch.Tensor,
                 temperature: float = 1.0, count: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused forward-KL distillation loss on aligned rows (see :class:`KLGemmFn`)."""
    return KLGemmFn.apply(h_s, h_t, weight, mask, temperature, count)


# ----------------------------------------------------------------- final RMSNorm prologue

def _norm_input(x: torch.Tensor, gamma: torch.Tensor) -> Tuple[torch.Tensor, int]:
    # the norm kernels read H gamma entries and N x H elements of x
    if x.dim() != 2 or gamma.numel() != x.shape[-1]:
        raise ValueError(f"expected x [N, H] and gamma [H], got {tuple(x.shape)} and {tuple(gamma.shape)}")
    x = x.detach()
    _require_cuda(x)
    if x.dtype == torch.bfloat16:
        return x.contiguous(), 0
    if x.dtype == torch.float32:
        return x.contiguous(), 1
    raise TypeError(f"unsupported dtype {x.dtype} (bf16 or fp32)")


def rmsnorm_rows(x: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-5,
                 want_rstd: bool = True) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """The backbone's final norm (model.py:493, a LlamaRMSNorm) row by row -> bf16 rows.

    ``x [N, H]`` bf16 or fp32, ``gamma [H]`` the norm weight.  Returns ``(y bf16 [N, H],
    rstd fp32 [N] or None)`` with ``y = gamma * bf16(x r)`` (bf16 x) or ``bf16(gamma * x r)``
    (fp32 x), ``r = 1 / sqrt(mean(x^2) + eps)``.
    """
    xc, f32 = _norm_input(x, gamma)
    dev = xc.device
    N, H = xc.shape
    g = gamma.detach().to(device=dev, dtype=torch.float32).contiguous()
    y = torch.empty(N, H, dtype=torch.bfloat16, device=dev)
    rstd = torch.empty(N, dtype=torch.float32, device=dev) if want_rstd else None
    call("klg_rmsnorm_rows", _ptr(xc), f32, _ptr(g), N, H, float(eps), _ptr(y), _ptr(rstd), _stream(dev))
    return y, rstd


def rmsnorm_rows_backward(x: torch.Tensor, gamma: torch.Tensor, rstd: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    """``dx`` fp32 ``[N, H]`` through the norm for ``dy`` fp32 ``[N, H]`` (weight frozen)."""
    if tuple(dy.shape) != tuple(x.shape):
        raise ValueError(f"dy must have x's shape {tuple(x.shape)}, got {tuple(dy.shape)}")
    if x.dim() == 2:
        _check_f32("rstd", rstd, (x.shape[0],))
    xc, f32 = _norm_input(x, gamma)
    dev = xc.device
    N, H = xc.shape
    g = gamma.detach().to(device=dev, dtype=torch.float32).contiguous()
    dyc = dy.detach().to(torch.float32).contiguous()
    dx = torch.empty(N, H, dtype=torch.float32, device=dev)
    call("klg_rmsnorm_rows_bwd", _ptr(xc), f32, _ptr(g), _ptr(rstd), _ptr(dyc), N, H, _ptr(dx), _stream(dev))
    return dx


class PrenormKLGemmFn(torch.autograd.Function):
    """:class:`KLGemmFn` on pre-norm rows: the backbone's final norm (model.py:493) runs as
    the op's prologue and its gradient as the epilogue of the backward, so the caller hands
    over the hidden states before ``self.norm`` and the normed rows exist only inside the op.

    Arguments: ``x_s``, ``x_t`` ``[N, H]`` pre-norm rows (bf16 or fp32; ``x_t`` detached),
    ``norm_weight [H]`` (frozen, as in the reference, model.py:323-324), ``weight [V, H]``,
    ``mask [N]``, ``temperature``, ``eps``, ``count``.  dH of the normed rows stays fp32
    between the loss and the norm's backward.
    """

    @staticmethod
    def forward(ctx, x_s, x_t, norm_weight, weight, mask, temperature=1.0, eps=1e-5, count=None):
        need_dx, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[3]
        ys, rs = rmsnorm_rows(x_s, norm_weight, eps, want_rstd=need_dx)
        yt, _ = rmsnorm_rows(x_t, norm_weight, eps, want_rstd=False)
        w = to_compute_dtype(weight)
        m = mask_u8(mask)
        ctx.dtypes = (x_s.dtype, weight.dtype)
        if need_dx or need_dw:
            loss, _, _, _, dh, dw = kl_fwd_bwd(ys, yt, w, m, temperature, count=count, need_dh=need_dx,
                                               need_dw=need_dw)
            dx = rmsnorm_rows_backward(x_s, norm_weight, rs, dh) if need_dx else None
            ctx.save_for_backward(dx, dw)
        else:
            loss, _, _, _ = kl_forward(ys, yt, w, m, temperature, count=count)
        return loss

    @staticmethod
    def backward(ctx, g):
        dx, dw = ctx.saved_tensors
        return (scale_grad(dx, g, ctx.dtypes[0]) if dx is not None else None, None, None,
                scale_grad(dw, g, ctx.dtypes[1]) if dw is not None else None, None, None, None, None)


def prenorm_kl_loss(x_s: torch.Tensor, x_t: torch.Tensor, norm_weight: torch.Tensor, weight: torch.Tensor,
                    mask: torch.Tensor, temperature: float = 1.0, eps: float = 1e-5,
                    count: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused loss on pre-norm rows (see :class:`PrenormKLGemmFn`)."""
    return PrenormKLGemmFn.apply(x_s, x_t, norm_weight, weight, mask, temperature, eps, count)
