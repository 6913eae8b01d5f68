"""Multi-rank host logic on gloo CPU ranks (world size 2 and 3), with the
oracle-backed CPU engine standing in for the per-device CUDA arithmetic.

Checks that row sharding and vocab sharding reproduce the single-process
reference loss and gradients, and that a rank failure surfaces as an error on
the other ranks (short process-group timeout) instead of a hang.
"""
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import klgemm_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _problem(N=96, H=32, V=203, T=1.5, seed=11):
    g = torch.Generator().manual_seed(seed)
    h_s = torch.randn(N, H, generator=g, dtype=torch.float64)
    h_t = torch.randn(N, H, generator=g, dtype=torch.float64) * 2
    W = torch.randn(V, H, generator=g, dtype=torch.float64) * 0.1
    mask = torch.rand(N, generator=g) < 0.6
    mask[:5] = False
    return h_s, h_t, W, mask, T


def _worker(rank, world, port, mode, out_q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        from orthrus_training_test_b200.parallel import row_sharded_kl_loss, shard_bounds, vocab_sharded_kl_loss
        from tests.cpu_engine import CpuOracleEngine

        h_s, h_t, W, mask, T = _problem()
        eng = CpuOracleEngine()
        if mode == "row":
            lo, hi = shard_bounds(h_s.shape[0], world, rank)
            hs = h_s[lo:hi].clone().requires_grad_(True)
            w = W.clone().requires_grad_(True)
            loss = row_sharded_kl_loss(hs, h_t[lo:hi], w, mask[lo:hi], T, engine=eng)
            loss.backward()
            out_q.put((rank, float(loss), (lo, hi), hs.grad.numpy(), w.grad.numpy()))
        else:
            lo, hi = shard_bounds(W.shape[0], world, rank)
            hs = h_s.clone().requires_grad_(True)
            w = W[lo:hi].clone().requires_grad_(True)
            loss = vocab_sharded_kl_loss(hs, h_t, w, mask, T, engine=eng)
            loss.backward()
            out_q.put((rank, float(loss), (lo, hi), hs.grad.numpy(), w.grad.numpy()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    errs = [r for r in res if r[1] == "error"]
    assert not errs, errs[0][2]
    return sorted(res)


@pytest.mark.parametrize("world", [2, 3])
def test_row_sharded_matches_single_process(world):
    h_s, h_t, W, mask, T = _problem()
    loss, dh, dw, *_ = O.aligned_kl_loss_np(h_s.numpy(), h_t.numpy(), W.numpy(), mask.numpy(), T)
    res = _run(world, "row")
    for rank, l, (lo, hi), g_h, g_w in res:
        assert abs(l - loss) < 1e-10
        np.testing.assert_allclose(g_h, dh[lo:hi], rtol=1e-9, atol=1e-13)
        np.testing.assert_allclose(g_w, dw, rtol=1e-9, atol=1e-13)     # dW all-reduced over ranks


@pytest.mark.parametrize("world", [2, 3])
def test_vocab_sharded_matches_single_process(world):
    h_s, h_t, W, mask, T = _problem()
    loss, dh, dw, *_ = O.aligned_kl_loss_np(h_s.numpy(), h_t.numpy(), W.numpy(), mask.numpy(), T)
    res = _run(world, "vocab")
    for rank, l, (lo, hi), g_h, g_w in res:
        assert abs(l - loss) < 1e-10
        np.testing.assert_allclose(g_h, dh, rtol=1e-9, atol=1e-13)      # dH all-reduced over shards
        np.testing.assert_allclose(g_w, dw[lo:hi], rtol=1e-9, atol=1e-13)


def _dying_worker(rank, world, port, out_q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        from orthrus_training_test_b200.parallel import row_sharded_kl_loss
        from tests.cpu_engine import CpuOracleEngine
        h_s, h_t, W, mask, T = _problem()
        if rank == 1:
            out_q.put((rank, "left"))
            out_q.close()
            out_q.join_thread()  # flush the report before the abrupt exit
            os._exit(0)          # leaves between steps, before its first collective
        try:
            row_sharded_kl_loss(h_s, h_t, W, mask, T, engine=CpuOracleEngine())
            out_q.put((rank, "no-error"))
        except Exception as e:  # the survivor learns of it from its collective
            out_q.put((rank, "raised:" + type(e).__name__))
    except Exception:
        out_q.put((rank, "error:" + traceback.format_exc()))


def test_rank_failure_raises_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("raised:"), res[0]


def test_shard_bounds_cover_vocab():
    from orthrus_training_test_b200.parallel import shard_bounds
    for V, P in [(248320, 8), (49153, 8), (10, 3), (7, 8)]:
        b = [shard_bounds(V, P, r) for r in range(P)]
        assert b[0][0] == 0 and b[-1][1] == V
        assert all(b[i][1] == b[i + 1][0] for i in range(P - 1))
        assert max(h - l for l, h in b) - min(h - l for l, h in b) <= 1


class _FakeXrNative:
    """Stands in for the exchange buffers' library calls: pointers are integers, a handle names
    its owner, and one chosen stage can fail on one chosen rank."""

    def __init__(self, rank, fail):
        self.rank, self.fail = rank, fail
        self.held = set()        # buffers allocated or mapped and not yet released

    def buffer_bytes(self, vocab, hidden, world):
        return 4096

    def alloc(self, device, nbytes):
        if self.fail == ("alloc", self.rank):
            raise RuntimeError("cudaMalloc failed (fake)")
        self.held.add(("own", self.rank))
        return 1000 + self.rank, bytes([self.rank]) * 64

    def open(self, device, handle):
        if self.fail == ("open", self.rank):
            raise RuntimeError("cudaIpcOpenMemHandle failed (fake)")
        self.held.add(("peer", handle[0]))
        return 2000 + handle[0]

    def close(self, ptr, own):
        self.held.discard(("own", ptr - 1000) if own else ("peer", ptr - 2000))

    def synchronize(self, device):
        pass


def _xr_setup_worker(rank, world, port, fail, out_q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        from orthrus_training_test_b200.parallel import XrSetupError, _XrExchange
        native = _FakeXrNative(rank, fail)
        try:
            ex = _XrExchange(None, 1024, 64, torch.device("cuda", 0), native=native)
            outcome = "ok"
            held = sorted(native.held)
            ex.close()
        except XrSetupError:
            outcome, held = "refused", None
        dist.barrier()              # every rank is still in step with the others
        out_q.put((rank, outcome, held, sorted(native.held)))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc(), None))


@pytest.mark.parametrize("fail", [None, ("alloc", 1), ("open", 0), ("open", 2)])
def test_exchange_setup_agrees_across_ranks(fail):
    """A failure to allocate or map an exchange buffer on one rank makes every rank refuse the
    exchange (and fall back to the NCCL all-reduce) with nothing left allocated or mapped,
    instead of one rank waiting in a collective that the others skip."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_xr_setup_worker, args=(r, world, port, fail, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    errs = [r for r in res if r[1] == "error"]
    assert not errs, errs[0][2]
    assert {r[1] for r in res} == {"ok" if fail is None else "refused"}
    for rank, outcome, held, left in res:
        if outcome == "ok":   # its own buffer and a mapping of every other rank's
            assert held == sorted([("own", rank)] + [("peer", p) for p in range(world) if p != rank])
        assert left == []    # released after close() or the refusal
