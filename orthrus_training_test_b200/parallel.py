"""Multi-GPU variants of the fused KL-GEMM loss (one process per GPU).

The reference is single-GPU (train.py:254); these are the two ways the loss
shards across an 8-GPU NVLink box:

Row sharding (``row_sharded_kl_loss``): each rank owns different token rows
and a full replica of the lm_head.  Rows are independent, so the only
exchanges are the global valid-row count (normaliser, one float), the loss
(one float) and the lm_head gradient dW ``[V, H]`` (all-reduce, the
data-parallel gradient exchange, bucketed by vocab chunk and overlapped with
the chunks still computing).  dH stays local.

Vocab sharding (``vocab_sharded_kl_loss``): each rank owns all rows and one
contiguous slice of the lm_head's rows (vocab entries).  When gradients are
needed the step follows the single-device training route split at its exchange
points: pass 1 gives one ``(m, S)`` record per row and view over the local
slice; one all-gather and a merge give every rank the global log-sum-exps;
pass 2 over the local slice gives the complete local dW slice, a partial dH and
the slice's part of the KL cross term ``sum_v p_v (u_t - u_s)``; one
all-reduce of ``[dH | cross]`` completes both, and the loss follows on every
rank.  Without gradients (evaluation) one all-gather of the single-pass
records ``(m_s, S_s, m_t, S_t, A)`` gives the loss.

The per-device arithmetic comes from an *engine*.  The product engine is
:class:`CudaEngine` (the sm_100a library).  Tests substitute a CPU engine
with the same interface to exercise this host logic on ``gloo`` ranks.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def _scale_grad(x: torch.Tensor, g: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    from .ops import scale_grad
    return scale_grad(x, g, dtype)


class _XrNative:
    """The library calls behind the exchange buffers (``klg_xr_alloc`` / ``klg_xr_open`` /
    ``klg_xr_close``).  Tests substitute a fake with the same three methods to run the set-up's
    agreement logic on ``gloo`` ranks."""

    def buffer_bytes(self, vocab: int, hidden: int, world: int) -> int:
        from . import _lib
        return int(_lib.lib().klg_xr_buffer_bytes(int(vocab), int(hidden), int(world)))

    def alloc(self, device: int, nbytes: int):
        """``(pointer, 64-byte IPC handle)`` of a new zero-filled buffer on ``device``."""
        import ctypes

        from . import _lib
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.call("klg_xr_alloc", device, nbytes, ctypes.byref(own), handle)
        return own.value, handle.raw

    def open(self, device: int, handle: bytes) -> int:
        import ctypes

        from . import _lib
        q = ctypes.c_void_p()
        _lib.call("klg_xr_open", device, ctypes.create_string_buffer(handle, 64), ctypes.byref(q))
        return q.value

    def close(self, ptr: int, own: bool) -> None:
        import ctypes

        from . import _lib
        _lib.call("klg_xr_close", ctypes.c_void_p(ptr), int(bool(own)))

    def synchronize(self, device: int) -> None:
        torch.cuda.synchronize(device)


class XrSetupError(RuntimeError):
    """The exchange could not be set up on some rank; raised on every rank alike."""


class _XrExchange:
    """One rank's buffer for the in-step dW exchange over NVLink (``klg_fwd_bwd_xr``) and its
    mappings of every other rank's: each rank allocates and zero-fills its own buffer
    (``klg_xr_alloc``), the CUDA IPC handles are all-gathered, and each rank opens the others'
    (``klg_xr_open``: plain peer mappings).  The ranks agree on the outcome of each stage
    before the next, so a failure on one rank makes every rank release what it holds and raise
    :class:`XrSetupError` -- no rank goes on to a collective the others skip.  All ranks meet
    at a barrier before the first step pushes into the buffers.  The epoch counter orders the
    steps."""

    def __init__(self, group, vocab: int, hidden: int, device: torch.device, native=None):
        import ctypes

        self.native = native if native is not None else _XrNative()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._dev = device.index if device.index is not None else torch.cuda.current_device()
        self._own = None
        self._peers = []
        err = None
        nbytes = self.native.buffer_bytes(vocab, hidden, self.world)
        handle = None
        if nbytes < 0:
            err = "no exchange buffer for this shape / world"
        else:
            try:
                self._own, handle = self.native.alloc(self._dev, nbytes)
            except Exception as e:
                err = f"rank {self.rank}: {e}"
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)          # every rank reaches this
        if any(h is None for h in handles):
            self._release(barrier=False)                              # nobody opened anything
            raise XrSetupError(err or "exchange buffer allocation failed on another rank")
        ptrs = []
        for p in range(self.world):
            if p == self.rank:
                ptrs.append(self._own)
                continue
            try:
                q = self.native.open(self._dev, handles[p])
            except Exception as e:
                err = f"rank {self.rank} opening rank {p}'s buffer: {e}"
                break
            self._peers.append(q)
            ptrs.append(q)
        oks = [None] * self.world
        dist.all_gather_object(oks, err is None, group=group)
        if not all(oks):
            self._release(barrier=True)
            raise XrSetupError(err or "exchange buffer mapping failed on another rank")
        self.peer_buffers = (ctypes.c_void_p * self.world)(*ptrs)
        self.native.synchronize(self._dev)
        dist.barrier(group=group)
        self.epoch = 0

    def _release(self, barrier: bool) -> None:
        # peer mappings first; with `barrier`, every rank has closed its mappings before any
        # owner frees its buffer
        for q in self._peers:
            self.native.close(q, own=False)
        self._peers = []
        if barrier:
            dist.barrier(group=self.group)
        if self._own is not None:
            self.native.close(self._own, own=True)
            self._own = None

    def close(self) -> None:
        """Collective: every rank of the group calls it, with no step in flight."""
        self.native.synchronize(self._dev)
        self._release(barrier=True)

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch


_XR_CACHE: dict = {}
_XR_BROKEN: set = set()


def _xr_enabled() -> bool:
    # the in-step exchange measured ~1-6 % slower per step than the overlapped NCCL all-reduce
    # at 2 and 4 GPUs, so it is opt-in (KLG_XR=1)
    import os
    return os.environ.get("KLG_XR", "0") == "1"


class CudaEngine:
    """Per-device arithmetic through the CUDA library."""

    def prepare(self, x: torch.Tensor) -> torch.Tensor:
        from .ops import to_compute_dtype
        return to_compute_dtype(x)

    def mask(self, m: torch.Tensor) -> torch.Tensor:
        from .ops import mask_u8
        return mask_u8(m)

    def count(self, mask: torch.Tensor) -> torch.Tensor:
        from .ops import count_valid
        return count_valid(mask)

    def forward(self, h_s, h_t, w, mask, temperature, count):
        """Full-vocab forward with a given normaliser: ``(loss, lse)``."""
        from .ops import kl_forward
        loss, lse, _, _ = kl_forward(h_s, h_t, w, mask, temperature, count=count)
        return loss, lse

    def partial_stats(self, h_s, h_t, w, temperature):
        """Merged per-row record ``[5, N]`` over ``w``'s rows."""
        from .ops import fwd_stats, merge_stats
        return merge_stats(fwd_stats(h_s, h_t, w, temperature))

    def merge(self, parts):
        from .ops import merge_stats
        return merge_stats(parts)

    def finalize(self, stats, mask, count):
        from .ops import finalize
        loss, lse, _ = finalize(stats, mask, count)
        return loss, lse

    def backward(self, h_s, h_t, w, mask, lse, count, grad, temperature, need_dh, need_dw):
        from .ops import kl_backward
        return kl_backward(h_s, h_t, w, mask, lse, count, grad=grad, temperature=temperature, need_dh=need_dh,
                           need_dw=need_dw)

    def forward_backward(self, h_s, h_t, w, mask, temperature, count, need_dh, need_dw, chunk_events=None):
        """Training step with a given normaliser: ``(loss, dH, dW)`` for upstream gradient 1."""
        from .ops import kl_fwd_bwd
        loss, _, _, _, dh, dw = kl_fwd_bwd(h_s, h_t, w, mask, temperature, count=count, need_dh=need_dh,
                                           need_dw=need_dw, chunk_events=chunk_events)
        return loss, dh, dw

    def xr_exchange(self, group, h_s, w):
        """The in-step dW exchange over NVLink for this group and shape, or None where it is not
        asked for (KLG_XR=1), does not apply (world 1 or > 8, not bf16) or cannot be set up (no
        peer mappings)."""
        world = dist.get_world_size(group)
        if not _xr_enabled() or world < 2 or world > 8 or h_s.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
            return None
        key = (id(group), w.shape[0], w.shape[1], h_s.device.index)
        if key in _XR_BROKEN:
            return None
        ex = _XR_CACHE.get(key)
        if ex is None:
            try:
                ex = _XrExchange(group, w.shape[0], w.shape[1], h_s.device)
            except XrSetupError as e:   # raised on every rank alike: the set-up agrees first
                import warnings
                warnings.warn(f"peer-memory dW exchange unavailable ({e}); using an NCCL all-reduce")
                _XR_BROKEN.add(key)
                return None
            _XR_CACHE[key] = ex
        return ex

    def forward_backward_xr(self, h_s, h_t, w, mask, temperature, count, need_dh, ex):
        """Training step with dW summed over ranks inside it: ``(local loss, dH, dW)``."""
        from .ops import kl_fwd_bwd_xr
        return kl_fwd_bwd_xr(h_s, h_t, w, mask, temperature, count, need_dh, ex.world, ex.rank, ex.peer_buffers,
                             ex.next_epoch())

    def dw_buckets(self, h_s, w):
        """Vocab chunks whose dW rows become final one after another during the training step
        (bf16 path), with one fresh event per chunk; None when the step cannot report them."""
        from .ops import chunk_bounds, new_chunk_events
        if h_s.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
            return None
        bounds = chunk_bounds(h_s.shape[0], h_s.shape[1], w.shape[0])
        return bounds, new_chunk_events(len(bounds))

    # the training step in pieces (vocab sharding exchanges data between them)
    acc_dtype = torch.float32

    def lse_record(self, h_s, h_t, w, temperature):
        """One merged ``(m, S)`` record per row and view over ``w``'s rows: ``[2, 2N]``."""
        from .ops import lse_record
        return lse_record(h_s, h_t, w, temperature)

    def lse_merge(self, recs):
        """``[R, 2, 2N]`` records -> the log-sum-exps ``[2, N]``."""
        from .ops import lse_merge
        return lse_merge(recs)

    def pass2(self, h_s, h_t, w, mask, lse, count, temperature, need_dh, need_dw, dh_out=None):
        """``(dH partial, dW of w's rows, cross-term part [N])`` for upstream gradient 1."""
        from .ops import pass2
        return pass2(h_s, h_t, w, mask, lse, count, temperature=temperature, need_dh=need_dh, need_dw=need_dw,
                     dh_out=dh_out)

    def kl_loss(self, lse, cross, mask, count):
        from .ops import kl_loss
        return kl_loss(lse, cross, mask, count)[0]


def _engine(engine):
    return engine if engine is not None else CudaEngine()


class _RowShardedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h_s, h_t, weight, mask, temperature, group, engine):
        eng = _engine(engine)
        hs, ht, w, m = eng.prepare(h_s), eng.prepare(h_t), eng.prepare(weight), eng.mask(mask)
        count = eng.count(m)
        dist.all_reduce(count, op=dist.ReduceOp.SUM, group=group)      # global normaliser
        need_dh, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[2]
        ctx.group = group
        ctx.dtypes = (h_s.dtype, weight.dtype)
        works = []
        if need_dh or need_dw:
            # sum_local valid*KL / global count, and its gradients for upstream gradient 1.  The
            # data-parallel dW exchange is issued here, bucketed by vocab chunk: each chunk's dW
            # rows are all-reduced on a side stream as soon as its GEMM is done, overlapping the
            # chunks still computing.  (The upstream gradient is the same on every rank -- it is
            # the gradient of the same global loss -- so reducing before scaling is the same sum.)
            ex = eng.xr_exchange(group, hs, w) if (need_dw and hasattr(eng, "xr_exchange")) else None
            # per-chunk buckets up to 4 ranks; at 8 one all-reduce after the step measured faster
            # (4.30 vs 4.43 ms per step at the 16k-row shape), at 4 the two tie
            overlap = dist.get_world_size(group) < 8
            buckets = (eng.dw_buckets(hs, w) if (ex is None and overlap and need_dw and hasattr(eng, "dw_buckets"))
                       else None)
            if ex is not None:
                # dW summed over the ranks inside the step (the GEMM stores each block of the
                # partial into its owner's buffer over NVLink; klg_fwd_bwd_xr)
                loss, dh, dw = eng.forward_backward_xr(hs, ht, w, m, temperature, count, need_dh, ex)
            elif buckets is not None:
                bounds, events = buckets
                loss, dh, dw = eng.forward_backward(hs, ht, w, m, temperature, count, need_dh, need_dw,
                                                    chunk_events=events)
                side = torch.cuda.Stream(device=hs.device)
                with torch.cuda.stream(side):
                    for (v0, v1), ev in zip(bounds, events):
                        side.wait_event(ev)
                        works.append(dist.all_reduce(dw[v0:v1], op=dist.ReduceOp.SUM, group=group, async_op=True))
            else:
                loss, dh, dw = eng.forward_backward(hs, ht, w, m, temperature, count, need_dh, need_dw)
                if dw is not None:
                    dist.all_reduce(dw, op=dist.ReduceOp.SUM, group=group)
            ctx.save_for_backward(dh, dw)
        else:
            loss, _ = eng.forward(hs, ht, w, m, temperature, count)
        loss = loss.reshape(1).clone()
        dist.all_reduce(loss, op=dist.ReduceOp.SUM, group=group)
        for wk in works:
            wk.wait()
        return loss.reshape(())

    @staticmethod
    def backward(ctx, g):
        dh, dw = ctx.saved_tensors          # dW already summed over ranks
        return (_scale_grad(dh, g, ctx.dtypes[0]) if dh is not None else None, None,
                _scale_grad(dw, g, ctx.dtypes[1]) if dw is not None else None, None, None, None, None)


def row_sharded_kl_loss(h_s: torch.Tensor, h_t: torch.Tensor, weight: torch.Tensor, mask: torch.Tensor,
                        temperature: float = 1.0, group: Optional[dist.ProcessGroup] = None,
                        engine=None) -> torch.Tensor:
    """Global loss over all ranks' rows; every rank gets the same value.

    ``h_s, h_t, mask``: this rank's rows.  ``weight``: the full lm_head
    (replicated).  Gradients: dH for the local rows; dW summed over ranks.
    Equals the single-device loss on the concatenated rows.
    """
    return _RowShardedFn.apply(h_s, h_t, weight, mask, float(temperature), group, engine)


class _VocabShardedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h_s, h_t, w_shard, mask, temperature, group, engine):
        eng = _engine(engine)
        hs, ht, w, m = eng.prepare(h_s), eng.prepare(h_t), eng.prepare(w_shard), eng.mask(mask)
        count = eng.count(m)                                          # identical rows on every rank
        world = dist.get_world_size(group)
        need_dh, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[2]
        ctx.dtypes = (h_s.dtype, w_shard.dtype)
        if not (need_dh or need_dw):
            # evaluation: the single-pass records (m_s, S_s, m_t, S_t, A) over the local slice
            local = eng.partial_stats(hs, ht, w, temperature).contiguous()
            gathered = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                                   device=local.device)
            dist.all_gather_into_tensor(gathered, local, group=group)
            stats = eng.merge(gathered.view((world,) + tuple(local.shape)))
            loss, _ = eng.finalize(stats, m, count)
            ctx.save_for_backward(None, None)
            return loss
        # pass 1 over the local slice -> all-gather of the (m, S) records -> global log-sum-exps
        rec = eng.lse_record(hs, ht, w, temperature).contiguous()
        gathered = torch.empty((world * rec.shape[0],) + tuple(rec.shape[1:]), dtype=rec.dtype, device=rec.device)
        dist.all_gather_into_tensor(gathered, rec, group=group)
        lse = eng.lse_merge(gathered.view((world,) + tuple(rec.shape)))
        # pass 2 over the local slice: this slice's dW (complete), partial dH and cross term,
        # then one all-reduce of [dH | cross]
        N, H = hs.shape
        buf = torch.empty(N * H * (1 if need_dh else 0) + N, dtype=eng.acc_dtype, device=hs.device)
        dh_view = buf[:N * H].view(N, H) if need_dh else None
        dh, dw, cross = eng.pass2(hs, ht, w, m, lse, count, temperature, need_dh, need_dw, dh_out=dh_view)
        buf[buf.numel() - N:].copy_(cross)
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
        loss = eng.kl_loss(lse, buf[buf.numel() - N:], m, count)
        ctx.save_for_backward(dh_view, dw)
        return loss

    @staticmethod
    def backward(ctx, g):
        dh, dw = ctx.saved_tensors
        return (_scale_grad(dh, g, ctx.dtypes[0]) if dh is not None else None, None,
                _scale_grad(dw, g, ctx.dtypes[1]) if dw is not None else None, None, None, None, None)


def vocab_sharded_kl_loss(h_s: torch.Tensor, h_t: torch.Tensor, weight_shard: torch.Tensor, mask: torch.Tensor,
                          temperature: float = 1.0, group: Optional[dist.ProcessGroup] = None,
                          engine=None) -> torch.Tensor:
    """Loss with the lm_head split by vocab rows across ranks.

    ``h_s, h_t, mask``: all rows (identical on every rank).  ``weight_shard``:
    this rank's contiguous slice of lm_head rows.  Returns the global loss on
    every rank; gradients: the full dH (all-reduced) and this rank's dW slice.
    """
    return _VocabShardedFn.apply(h_s, h_t, weight_shard, mask, float(temperature), group, engine)


def shard_bounds(vocab: int, world: int, rank: int):
    """Contiguous vocab slice ``[lo, hi)`` of ``rank`` (sizes differ by at most one row)."""
    base, rem = divmod(vocab, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)
