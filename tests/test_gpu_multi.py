"""Row and vocab sharding on 2, 4 and 8 GPUs (one process per GPU, NCCL), through the CUDA
library, against the fp32 oracle.

Each rank runs the sharded loss on its slice; row sharding three times, with dW all-reduced
by NCCL ("row") or summed over the ranks inside the step over NVLink peer memory ("row_xr",
bitwise the same dW in every step and on every rank).  The loss and the assembled gradients must
match the fp32 torch oracle (the reference's op sequence, run on cuda:0 over the whole
problem) within the tolerances every GPU parity test uses: loss 1e-3 relative, gradients
2e-2 normalised max error and cosine similarity >= 0.9999.  Two problems: a small one with a
peaky teacher and some masked rows, and the ragged/edge configuration (12,288 - 37 rows,
H=576, V=49,152, ~25 % of rows valid, teacher x4, T=2, all-masked rows).
Skipped when fewer GPUs than ranks are visible.  NVLS is off in every rank.
"""
import os
import tempfile
import traceback
from datetime import timedelta

import pytest
import torch

from oracle import klgemm_oracle as O
from tests.gpu_helpers import GRAD_COS, GRAD_MAX_REL, LOSS_RTOL, run_oracle_torch_gpu

pytestmark = pytest.mark.gpu


def _problem(name):
    if name == "c5":
        p = O.make_problem("c5", n_rows=12288 - 37)
        return p["h_s"], p["h_t"], p["W"], p["mask"], p["T"]
    g = torch.Generator().manual_seed(7)
    N, H, V = 1000, 576, 5000
    h_s = torch.randn(N, H, generator=g).to(torch.bfloat16)
    h_t = (torch.randn(N, H, generator=g) * 2.0).to(torch.bfloat16)
    W = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16)
    mask = torch.rand(N, generator=g) < 0.7
    mask[:9] = False
    return h_s, h_t, W, mask, 1.5


def _worker(rank, world, init_file, mode, name, out_q):
    try:
        import torch.distributed as dist
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        # "row": dW all-reduced by NCCL (the default); "row_xr": dW summed over the ranks inside
        # the step over NVLink peer memory
        os.environ["KLG_XR"] = "1" if mode == "row_xr" else "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        # rendezvous through a file: no TCP port to collide with a previous test's
        dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        from orthrus_training_test_b200.parallel import row_sharded_kl_loss, shard_bounds, vocab_sharded_kl_loss

        h_s, h_t, W, mask, T = _problem(name)
        N, V = h_s.shape[0], W.shape[0]
        row = mode.startswith("row")
        dws = []
        if row:
            lo, hi = shard_bounds(N, world, rank)
            hs = h_s[lo:hi].to(dev).requires_grad_(True)
            w = W.to(dev).requires_grad_(True)
            # three steps: the exchange's epochs order consecutive steps; dW is the same every time
            for _ in range(3):
                hs.grad = None
                w.grad = None
                loss = row_sharded_kl_loss(hs, h_t[lo:hi].to(dev), w, mask[lo:hi].to(dev), T)
                loss.backward()
                dws.append(w.grad.detach().clone())
        else:
            lo, hi = shard_bounds(V, world, rank)
            hs = h_s.to(dev).requires_grad_(True)
            w = W[lo:hi].to(dev).requires_grad_(True)
            loss = vocab_sharded_kl_loss(hs, h_t.to(dev), w, mask.to(dev), T)
            loss.backward()
        if row:
            # bitwise the same dW in every step, and (all-gathered) on every rank
            assert all(torch.equal(d, dws[0]) for d in dws[1:]), "dW changed between identical steps"
            allw = [torch.empty_like(dws[0]) for _ in range(world)]
            dist.all_gather(allw, dws[0])
            if mode == "row_xr":
                assert all(torch.equal(d, allw[0]) for d in allw[1:]), "dW differs between ranks"
        # the evaluation route (no gradients) on the same shards
        with torch.no_grad():
            if row:
                loss_eval = row_sharded_kl_loss(hs.detach(), h_t[lo:hi].to(dev), w.detach(), mask[lo:hi].to(dev), T)
            else:
                loss_eval = vocab_sharded_kl_loss(hs.detach(), h_t.to(dev), w.detach(), mask.to(dev), T)
        torch.cuda.synchronize()
        out_q.put((rank, float(loss.detach()), (lo, hi), hs.grad.float().cpu(), w.grad.float().cpu(),
                   float(loss_eval)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def _close(a, b, what):
    err = float((a.double() - b).abs().max() / b.abs().max().clamp_min(1e-30))
    cos = float(torch.nn.functional.cosine_similarity(a.flatten().double(), b.flatten().double(), dim=0))
    assert err <= GRAD_MAX_REL and cos >= GRAD_COS, f"{what}: max-rel {err:.3e} cos {cos:.6f}"


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("name", ["small", "c5"])
@pytest.mark.parametrize("mode", ["row", "row_xr", "vocab"])
def test_sharding_matches_oracle(mode, name, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    h_s, h_t, W, mask, T = _problem(name)
    ref_loss, ref_dh, ref_dw = run_oracle_torch_gpu(h_s, h_t, W, mask, T)
    ref_dh, ref_dw = torch.from_numpy(ref_dh), torch.from_numpy(ref_dw)
    torch.cuda.synchronize()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init_file = os.path.join(tempfile.mkdtemp(prefix="klg_multi_"), "rendezvous")
    procs = [ctx.Process(target=_worker, args=(r, world, init_file, mode, name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    errs = [r for r in res if r[1] == "error"]
    assert not errs, errs[0][2]
    res.sort(key=lambda r: r[0])
    for _, loss, _, _, _, loss_eval in res:
        assert abs(loss - ref_loss) <= LOSS_RTOL * abs(ref_loss), (loss, ref_loss)
        assert abs(loss_eval - ref_loss) <= LOSS_RTOL * abs(ref_loss), (loss_eval, ref_loss)
    if mode.startswith("row"):
        _close(torch.cat([r[3] for r in res]), ref_dh, "dH")
        for r in res:
            _close(r[4], ref_dw, "dW (all-reduced)")
    else:
        for r in res:
            _close(r[3], ref_dh, "dH (all-reduced)")
        _close(torch.cat([r[4] for r in res]), ref_dw, "dW")
