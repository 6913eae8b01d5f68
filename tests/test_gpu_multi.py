"""Row and vocab sharding on 2 GPUs (one process per GPU, NCCL), through the CUDA library.

Each rank runs the sharded loss on its slice; the result must equal the single-device
fused op on the whole problem: the loss to 1e-4 relative (summation order and, for vocab
sharding, the pass-1 route of the KL cross term differ), dH and dW to the gradient
tolerances used for every GPU test.
Skipped when fewer than 2 GPUs are visible.
"""
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

N, H, V, T = 1000, 576, 5000, 1.5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _problem():
    g = torch.Generator().manual_seed(7)
    h_s = (torch.randn(N, H, generator=g) * 1.0).to(torch.bfloat16)
    h_t = (torch.randn(N, H, generator=g) * 2.0).to(torch.bfloat16)
    W = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16)
    mask = torch.rand(N, generator=g) < 0.7
    mask[:9] = False
    return h_s, h_t, W, mask


def _worker(rank, world, port, mode, out_q):
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from orthrus_training_test_b200.parallel import row_sharded_kl_loss, shard_bounds, vocab_sharded_kl_loss

        h_s, h_t, W, mask = _problem()
        if mode == "row":
            lo, hi = shard_bounds(N, world, rank)
            hs = h_s[lo:hi].to(dev).requires_grad_(True)
            w = W.to(dev).requires_grad_(True)
            loss = row_sharded_kl_loss(hs, h_t[lo:hi].to(dev), w, mask[lo:hi].to(dev), T)
        else:
            lo, hi = shard_bounds(V, world, rank)
            hs = h_s.to(dev).requires_grad_(True)
            w = W[lo:hi].to(dev).requires_grad_(True)
            loss = vocab_sharded_kl_loss(hs, h_t.to(dev), w, mask.to(dev), T)
        loss.backward()
        torch.cuda.synchronize()
        out_q.put((rank, float(loss.detach()), (lo, hi), hs.grad.float().cpu(), w.grad.float().cpu()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def _reference():
    from orthrus_training_test_b200.ops import kl_gemm_loss
    h_s, h_t, W, mask = _problem()
    dev = torch.device("cuda", 0)
    hs = h_s.to(dev).requires_grad_(True)
    w = W.to(dev).requires_grad_(True)
    loss = kl_gemm_loss(hs, h_t.to(dev), w, mask.to(dev), T)
    loss.backward()
    return float(loss.detach()), hs.grad.float().cpu(), w.grad.float().cpu()


def _close(a, b, what):
    err = float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))
    cos = float(torch.nn.functional.cosine_similarity(a.flatten().double(), b.flatten().double(), dim=0))
    assert err <= 2e-2 and cos >= 0.9999, f"{what}: max-rel {err:.3e} cos {cos:.6f}"


@pytest.mark.parametrize("mode", ["row", "vocab"])
def test_two_gpu_sharding_matches_single_device(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ref_loss, ref_dh, ref_dw = _reference()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
    errs = [r for r in res if r[1] == "error"]
    assert not errs, errs[0][2]
    res.sort(key=lambda r: r[0])
    for _, loss, _, _, _ in res:
        assert abs(loss - ref_loss) <= 1e-4 * abs(ref_loss) + 1e-7, (loss, ref_loss)
    if mode == "row":
        dh = torch.cat([r[3] for r in res])
        _close(dh, ref_dh, "dH")
        for r in res:
            _close(r[4], ref_dw, "dW (all-reduced)")
    else:
        for r in res:
            _close(r[3], ref_dh, "dH (all-reduced)")
        dw = torch.cat([r[4] for r in res])
        _close(dw, ref_dw, "dW")
