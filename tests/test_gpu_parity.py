"""GPU parity of the fused KL-GEMM loss against the oracle (calls go through the C-ABI).

Tolerances (written here and in tests/gpu_helpers.py): loss within 1e-3
relative of the fp32 reference; gradients within 2e-2 normalised max error
(max|ours-ref| / max|ref|) and cosine similarity >= 0.9999.  The reference is
evaluated on the same bf16-rounded inputs the kernels consume; the golden
fixtures (fp32 inputs, produced by the reference itself) are checked directly.
"""
import numpy as np
import pytest
import torch

from oracle import klgemm_oracle as O
from tests.conftest import GOLDEN, golden_cases
from tests.gpu_helpers import (GRAD_COS, GRAD_MAX_REL, LOSS_RTOL, assert_close, bf16_round, run_both,
                               run_oracle_np, run_oracle_torch_gpu, run_ours)

pytestmark = pytest.mark.gpu


def rand_problem(N, H, V, T=1.0, p=0.5, seed=0, tscale=1.0):
    g = torch.Generator().manual_seed(seed)
    h_s = torch.randn(N, H, generator=g)
    h_t = torch.randn(N, H, generator=g) * tscale
    W = torch.randn(V, H, generator=g) * 0.02
    mask = torch.rand(N, generator=g) < p
    return h_s, h_t, W, mask, T


def test_fused_row_kl_and_lse_match_split():
    """The training path's pass-1 log-sum-exps (CTA pairs) and per-row KL equal the single-pass forward's."""
    h_s, h_t, W, mask, T = rand_problem(700, 576, 3000, seed=9, p=0.6)
    a, b = run_both(h_s, h_t, W, mask, T)
    np.testing.assert_allclose(b["lse"], a["lse"], rtol=1e-5, atol=1e-4)
    m = mask.numpy()
    np.testing.assert_allclose(b["row_kl"][m], a["row_kl"][m], rtol=2e-3, atol=2e-6)
    assert not np.any(b["row_kl"][~m])


def test_stats_small():
    """Pass 1 + merge + finalize: per-row KL and lse against float64."""
    from orthrus_training_test_b200 import ops
    h_s, h_t, W, mask, T = rand_problem(200, 128, 700, seed=1)
    ours = run_ours(h_s, h_t, W, mask, T, need_dw=False)
    loss, _, _, row_kl, ls, lt = run_oracle_np(h_s, h_t, W, mask, T)
    np.testing.assert_allclose(ours["lse"][0] * np.log(2), ls, rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(ours["lse"][1] * np.log(2), lt, rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(ours["row_kl"], row_kl, rtol=2e-3, atol=2e-5)
    assert abs(ours["loss"] - loss) <= LOSS_RTOL * loss
    assert ours["count"] == float(mask.sum())


def test_bwd_small():
    h_s, h_t, W, mask, T = rand_problem(200, 128, 700, seed=2)
    ours = run_both(h_s, h_t, W, mask, T)
    loss, dh, dw, *_ = run_oracle_np(h_s, h_t, W, mask, T)
    assert_close(ours, loss, dh, dw, "small")


@pytest.mark.parametrize("name", [n for n in golden_cases() if n.startswith("aligned")])
def test_golden_aligned(name):
    """Inputs and outputs produced by the reference's compute_kl_loss (fp32)."""
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    h_s, h_t, W = (torch.tensor(g[k]) for k in ("h_s", "h_t", "weight"))
    mask = torch.tensor(g["mask"])
    T = float(g["temperature"])
    ours = run_both(h_s, h_t, W, mask, T)
    # against the reference's own fp32 numbers (inputs rounded to bf16 by the op)
    B = g["anchor_positions"].shape[0]
    dp, _, _ = O.kl_indices(B, g["anchor_positions"].shape[1], int(g["K"]))
    ref_dh = g["grad_diff_hidden"][np.arange(B)[:, None], dp].reshape(ours[0]["dh"].shape)
    assert_close(ours, float(g["loss"]), ref_dh, g["grad_weight"], name)


def test_compute_kl_loss_shim_golden():
    """The drop-in shim with the reference signature on the clamped-anchor fixture."""
    from orthrus_training_test_b200 import compute_kl_loss
    g = dict(np.load(GOLDEN / "anchors_clamp.npz"))
    dev = torch.device("cuda:0")
    diff = torch.tensor(g["diff_hidden"], device=dev, requires_grad=True)
    head = torch.nn.Linear(g["weight"].shape[1], g["weight"].shape[0], bias=False).to(dev)
    with torch.no_grad():
        head.weight.copy_(torch.tensor(g["weight"]))
    loss = compute_kl_loss(diff, torch.tensor(g["ar_hidden"], device=dev), head,
                           torch.tensor(g["anchor_positions"], device=dev), int(g["K"]),
                           torch.tensor(g["target_ids"], device=dev), int(g["pad"]))
    loss.backward()
    assert abs(loss.item() - float(g["loss"])) <= LOSS_RTOL * float(g["loss"])
    mr, cos = O.grad_metrics(diff.grad.cpu().numpy(), g["grad_diff_hidden"])
    assert mr <= GRAD_MAX_REL and cos >= GRAD_COS, (mr, cos)
    mr, cos = O.grad_metrics(head.weight.grad.cpu().numpy(), g["grad_weight"])
    assert mr <= GRAD_MAX_REL and cos >= GRAD_COS, (mr, cos)


def test_compute_kl_loss_all_masked():
    from orthrus_training_test_b200 import compute_kl_loss
    g = dict(np.load(GOLDEN / "all_masked.npz"))
    dev = torch.device("cuda:0")
    diff = torch.tensor(g["diff_hidden"], device=dev, requires_grad=True)
    head = torch.nn.Linear(g["weight"].shape[1], g["weight"].shape[0], bias=False).to(dev)
    loss = compute_kl_loss(diff, torch.tensor(g["ar_hidden"], device=dev), head,
                           torch.tensor(g["anchor_positions"], device=dev), int(g["K"]),
                           torch.tensor(g["target_ids"], device=dev), int(g["pad"]))
    assert loss.item() == 0.0 and loss.requires_grad


def test_all_masked_op_gives_zero():
    """The op itself (no shim early-return): zero loss and exactly zero grads."""
    h_s, h_t, W, _, T = rand_problem(300, 64, 500, seed=3)
    mask = torch.zeros(300, dtype=torch.bool)
    for ours in run_both(h_s, h_t, W, mask, T):
        assert ours["loss"] == 0.0
        assert not np.any(ours["dh"]) and not np.any(ours["dw"])


@pytest.mark.parametrize("N,H,V", [(1, 64, 1), (1, 64, 129), (129, 192, 257), (333, 576, 1000), (256, 1024, 385),
                                   (130, 2048, 300), (77, 72, 250)])
def test_ragged_shapes(N, H, V):
    """N, V not multiples of the 128 tile; H = 576/1024/2048 and a non-multiple of 64."""
    h_s, h_t, W, mask, T = rand_problem(N, H, V, seed=N + V)
    mask[0] = True
    ours = run_both(h_s, h_t, W, mask, T)
    loss, dh, dw, *_ = run_oracle_np(h_s, h_t, W, mask, T)
    assert_close(ours, loss, dh, dw, f"N{N} H{H} V{V}")


def test_trainer_vocab_with_mask_token():
    """The trainer adds a <mask> token to SmolLM2's 49,152-row vocabulary (V = 49,153: one
    row past the last 128 tile, and a ragged last chunk); 2,048 rows of that shape."""
    h_s, h_t, W, mask, T = rand_problem(2048, 576, 49153, seed=17)
    ours = run_both(h_s, h_t, W, mask, T)
    loss, dh, dw, *_ = run_oracle_np(h_s, h_t, W, mask, T)
    assert_close(ours, loss, dh, dw, "V=49153")


def test_temperature_and_peaky_teacher():
    h_s, h_t, W, mask, _ = rand_problem(400, 576, 2000, seed=5, tscale=4.0, p=0.25)
    mask[:8] = False
    for T in (2.0, 0.5):
        ours = run_both(h_s, h_t, W, mask, T)
        loss, dh, dw, *_ = run_oracle_np(h_s, h_t, W, mask, T)
        assert_close(ours, loss, dh, dw, f"T={T}")


def test_chunking_invariance():
    """Smallest backward chunk (128 vocab columns) equals the default chunking."""
    h_s, h_t, W, mask, T = rand_problem(300, 128, 1500, seed=6)
    a = run_ours(h_s, h_t, W, mask, T)
    b = run_ours(h_s, h_t, W, mask, T, workspace_bytes=4096 + 304 * 128 * 2)   # rows padded to 8
    c = run_ours(h_s, h_t, W, mask, T, path="fused", workspace_bytes=256 * 1024)  # several fused chunks
    for k in ("dh", "dw"):
        mr, cos = O.grad_metrics(c[k], a[k])
        assert mr < 1e-2 and cos > 0.99999, (k, mr, cos)
    assert abs(c["loss"] - a["loss"]) <= 1e-4 * a["loss"]
    for k in ("dh", "dw"):
        mr, cos = O.grad_metrics(b[k], a[k])
        assert mr < 1e-5 and cos > 0.999999, (k, mr, cos)


def test_repeat_runs_bitwise_identical():
    """Same inputs, same results, bit for bit (no order-dependent reductions)."""
    h_s, h_t, W, mask, T = rand_problem(700, 576, 5000, seed=12)
    a = run_ours(h_s, h_t, W, mask, T, path="fused", workspace_bytes=4096 + 700 * 512 * 2 * 4)
    b = run_ours(h_s, h_t, W, mask, T, path="fused", workspace_bytes=4096 + 700 * 512 * 2 * 4)
    assert a["loss"] == b["loss"]
    np.testing.assert_array_equal(a["dh"], b["dh"])
    np.testing.assert_array_equal(a["dw"], b["dw"])


@pytest.mark.parametrize("path", ["split", "fused"])
def test_upstream_grad_scales_linearly(path):
    h_s, h_t, W, mask, T = rand_problem(200, 128, 600, seed=7)
    a = run_ours(h_s, h_t, W, mask, T, path=path)
    b = run_ours(h_s, h_t, W, mask, T, grad=3.0, path=path)
    # dZ is stored in bf16, so 3*round(dz) and round(3*dz) differ by one rounding
    for k in ("dh", "dw"):
        mr, cos = O.grad_metrics(b[k], 3.0 * a[k])
        assert mr < 1e-2 and cos > 0.99999, (k, mr, cos)


def test_autograd_function_matches_oracle():
    """KLGemmFn through torch autograd (bf16 params) against the fp32 torch oracle."""
    from orthrus_training_test_b200 import kl_gemm_loss
    h_s, h_t, W, mask, T = rand_problem(300, 576, 3000, seed=8)
    dev = torch.device("cuda:0")
    hs = h_s.to(dev, torch.bfloat16).requires_grad_(True)
    w = W.to(dev, torch.bfloat16).requires_grad_(True)
    loss = kl_gemm_loss(hs, h_t.to(dev, torch.bfloat16), w, mask.to(dev), T)
    loss.backward()
    ref_loss, ref_dh, ref_dw = run_oracle_torch_gpu(h_s, h_t, W, mask, T)
    assert abs(loss.item() - ref_loss) <= LOSS_RTOL * ref_loss
    for ours, ref in ((hs.grad, ref_dh), (w.grad, ref_dw)):
        mr, cos = O.grad_metrics(ours.float().cpu().numpy(), ref)
        assert mr <= GRAD_MAX_REL and cos >= GRAD_COS, (mr, cos)


@pytest.mark.parametrize("cfg", ["c1", "c2", "c5"])
def test_benchmark_configs_full_size(cfg):
    """Full-size configurations against the fp32 torch oracle run on the GPU."""
    n = 12288 - 37 if cfg == "c5" else None  # c5 also exercises a row count off the tile
    p = O.make_problem(cfg, n_rows=n)
    ours = run_both(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"])
    # c1 is an fp32 configuration: compare with the fp32 reference on the unrounded inputs
    ref_loss, ref_dh, ref_dw = run_oracle_torch_gpu(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"],
                                                    round_inputs=(cfg != "c1"))
    assert_close(ours, ref_loss, ref_dh, ref_dw, cfg)


def test_c3_full_size():
    """The 1.7B-shaped configuration at its full 65,536 rows (H=2048, V=49,152: twelve dZ
    chunks of the training path) against the fp32 torch oracle on the GPU."""
    p = O.make_problem("c3")
    ours = run_both(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"])
    ref_loss, ref_dh, ref_dw = run_oracle_torch_gpu(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"])
    assert_close(ours, ref_loss, ref_dh, ref_dw, "c3")


def test_c4_shape_full_vocab_subsample():
    """The large-vocabulary configuration's shape (H=1024, V=248,320) on 2,048 of its rows
    with the whole vocabulary on one device, both entry paths."""
    p = O.make_problem("c4", n_rows=2048)
    ours = run_both(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"])
    ref_loss, ref_dh, ref_dw = run_oracle_torch_gpu(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"], chunk=1024)
    assert_close(ours, ref_loss, ref_dh, ref_dw, "c4-sub")


def _vocab_sharded_on_one_gpu(h_s, h_t, W, mask, T, world):
    """The vocab-sharded training step's per-shard arithmetic on one device, combined the way
    parallel.vocab_sharded_kl_loss combines it across GPUs: every lm_head slice's pass-1
    (m, S) record, stacked (the all-gather) and merged into the global log-sum-exps; every
    slice's pass 2 with them (its dW rows, a partial dH and its part of the KL cross term),
    summed (the all-reduce of [dH | cross]); the loss from the summed cross terms."""
    from orthrus_training_test_b200 import ops
    from orthrus_training_test_b200.parallel import CudaEngine, shard_bounds

    dev = torch.device("cuda:0")
    eng = CudaEngine()
    hs, ht, w, m = eng.prepare(h_s.to(dev)), eng.prepare(h_t.to(dev)), eng.prepare(W.to(dev)), eng.mask(mask.to(dev))
    count = eng.count(m)
    slices = [shard_bounds(W.shape[0], world, r) for r in range(world)]
    recs = torch.stack([eng.lse_record(hs, ht, w[lo:hi].contiguous(), T) for lo, hi in slices])
    lse = eng.lse_merge(recs)
    dh = torch.zeros(hs.shape, dtype=torch.float32, device=dev)
    cross = torch.zeros(hs.shape[0], dtype=torch.float32, device=dev)
    dws = []
    for lo, hi in slices:
        dh_r, dw_r, c_r = eng.pass2(hs, ht, w[lo:hi].contiguous(), m, lse, count, T, True, True)
        dh += dh_r
        cross += c_r
        dws.append(dw_r)
    loss = eng.kl_loss(lse, cross, m, count)
    # the evaluation route (no gradients): single-pass records all-gathered and merged
    parts = torch.stack([eng.partial_stats(hs, ht, w[lo:hi].contiguous(), T) for lo, hi in slices])
    loss_eval, _ = eng.finalize(eng.merge(parts), m, count)
    torch.cuda.synchronize()
    return dict(loss=float(loss.item()), dh=dh.double().cpu().numpy(), dw=torch.cat(dws).double().cpu().numpy(),
                loss_eval=float(loss_eval.item()))


@pytest.mark.parametrize("world", [2, 3])
def test_vocab_sharding_emulated_on_one_gpu(world):
    """Vocab sharding's per-shard arithmetic on one device, against the float64 oracle."""
    h_s, h_t, W, mask, T = rand_problem(900, 576, 7001, seed=21)
    ours = _vocab_sharded_on_one_gpu(h_s, h_t, W, mask, T, world)
    loss_ref, dh_ref, dw_ref, *_ = run_oracle_np(h_s, h_t, W, mask, T)
    assert_close(ours, loss_ref, dh_ref, dw_ref, f"vocab shards x{world}")
    assert abs(ours["loss_eval"] - loss_ref) <= LOSS_RTOL * abs(loss_ref)


def test_vocab_sharding_c4_shape_world8_emulated():
    """The large-vocabulary configuration as eight vocab shards of 31,040 lm_head rows (a
    shard is not a multiple of the 128/256-row tiles), on 1,061 rows (ragged), against the
    fp32 torch oracle over the whole vocabulary."""
    p = O.make_problem("c4", n_rows=1024 + 37)
    ours = _vocab_sharded_on_one_gpu(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"], 8)
    ref_loss, ref_dh, ref_dw = run_oracle_torch_gpu(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"], chunk=512)
    assert_close(ours, ref_loss, ref_dh, ref_dw, "c4 x8 shards")
    assert abs(ours["loss_eval"] - ref_loss) <= LOSS_RTOL * abs(ref_loss)


def test_pass_pieces_equal_training_step():
    """klg_lse_record + klg_lse_merge + klg_pass2 + klg_kl_loss on the whole vocabulary
    reproduce klg_fwd_bwd: the same kernels and plans, so bit for bit."""
    from orthrus_training_test_b200 import ops
    h_s, h_t, W, mask, T = rand_problem(700, 576, 5000, seed=23, tscale=2.0)
    dev = torch.device("cuda:0")
    hs, ht, w = (ops.to_compute_dtype(x.to(dev)) for x in (h_s, h_t, W))
    m = ops.mask_u8(mask.to(dev))
    loss, lse, cnt, row_kl, dh, dw = ops.kl_fwd_bwd(hs, ht, w, m, T, want_row_kl=True)
    lse2 = ops.lse_merge(ops.lse_record(hs, ht, w, T)[None])
    dh2, dw2, cross = ops.pass2(hs, ht, w, m, lse2, cnt, temperature=T)
    loss2, row_kl2 = ops.kl_loss(lse2, cross, m, cnt, want_row_kl=True)
    torch.cuda.synchronize()
    assert torch.equal(lse, lse2)
    assert torch.equal(dh, dh2) and torch.equal(dw, dw2)
    torch.testing.assert_close(row_kl2, row_kl, rtol=1e-6, atol=1e-7)
    assert abs(float(loss2) - float(loss)) <= 1e-6 * abs(float(loss))


# fp32-faithful path (fp32 inputs: split-bf16 planes on the tensor cores).  Tolerances against
# the unrounded fp32 oracle, tighter than the bf16 path's: loss 1e-5 relative, gradients
# 2e-3 normalised max error and cosine >= 0.999999.
F32_LOSS_RTOL = 1e-5
F32_GRAD_MAX_REL = 2e-3
F32_GRAD_COS = 0.999999


def _f32_close(loss, dh, dw, ref_loss, ref_dh, ref_dw, label):
    rel = abs(loss - ref_loss) / abs(ref_loss)
    assert rel <= F32_LOSS_RTOL, f"{label} loss {loss} vs {ref_loss} (rel {rel:.2e})"
    for name, ours, ref in (("dH", dh, ref_dh), ("dW", dw, ref_dw)):
        mr, cos = O.grad_metrics(ours, ref)
        assert mr <= F32_GRAD_MAX_REL and cos >= F32_GRAD_COS, f"{label} {name} max_rel {mr:.2e} cos {cos:.8f}"
    return rel


def test_fp32_path_c1_full_size_beats_bf16_rounding():
    """The CPU-runnable configuration (fp32, 1,024 x 576 x 49,152) through the fp32 path, against
    the fp32 torch oracle on the unrounded inputs; its errors are below the bf16 path's."""
    from orthrus_training_test_b200 import ops
    p = O.make_problem("c1")
    dev = torch.device("cuda:0")
    ref_loss, ref_dh, ref_dw = run_oracle_torch_gpu(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"], round_inputs=False)
    hs, ht, w = (x.to(dev).float().contiguous() for x in (p["h_s"], p["h_t"], p["W"]))
    loss, lse, cnt, row_kl, dh, dw = ops.kl_fwd_bwd(hs, ht, w, p["mask"].to(dev), p["T"], want_row_kl=True)
    torch.cuda.synchronize()
    f32_dh, f32_dw = dh.double().cpu().numpy(), dw.double().cpu().numpy()
    rel = _f32_close(float(loss), f32_dh, f32_dw, ref_loss, ref_dh, ref_dw, "c1 fp32 path")
    # the forward-only route (evaluation) on the same fp32 inputs
    loss_f, lse_f, _, _ = ops.kl_forward(hs, ht, w, p["mask"].to(dev), p["T"])
    assert abs(float(loss_f) - ref_loss) <= F32_LOSS_RTOL * abs(ref_loss)
    torch.testing.assert_close(lse_f, lse, rtol=1e-6, atol=1e-5)
    # the bf16 path on the same problem is less accurate on every measure
    b = run_ours(p["h_s"], p["h_t"], p["W"], p["mask"], p["T"], path="fused")
    assert rel <= abs(b["loss"] - ref_loss) / abs(ref_loss) or rel < 1e-6
    for ours, bf, ref in ((f32_dh, b["dh"], ref_dh), (f32_dw, b["dw"], ref_dw)):
        assert O.grad_metrics(ours, ref)[0] < O.grad_metrics(bf, ref)[0]


@pytest.mark.parametrize("name", [n for n in golden_cases() if n.startswith("aligned")])
def test_fp32_path_golden(name):
    """The reference's own fp32 outputs (golden fixtures), through the autograd op with fp32
    parameters -- the fp32 path -- at the fp32 tolerances."""
    from orthrus_training_test_b200 import kl_gemm_loss
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    dev = torch.device("cuda:0")
    h_s = torch.tensor(g["h_s"], device=dev, requires_grad=True)
    w = torch.tensor(g["weight"], device=dev, requires_grad=True)
    loss = kl_gemm_loss(h_s, torch.tensor(g["h_t"], device=dev), w, torch.tensor(g["mask"], device=dev),
                        float(g["temperature"]))
    loss.backward()
    B = g["anchor_positions"].shape[0]
    dp, _, _ = O.kl_indices(B, g["anchor_positions"].shape[1], int(g["K"]))
    ref_dh = g["grad_diff_hidden"][np.arange(B)[:, None], dp].reshape(h_s.shape)
    _f32_close(float(loss), h_s.grad.double().cpu().numpy(), w.grad.double().cpu().numpy(), float(g["loss"]), ref_dh,
               g["grad_weight"], name)


@pytest.mark.parametrize("n", [4, 37, 1 << 20])
def test_scale_grad_matches_torch(n):
    """The autograd backward's one-pass scaling (klg_scale_cast) gives exactly torch's
    (x * g).to(dtype): one fp32 product, then round to nearest even for bf16."""
    from orthrus_training_test_b200 import ops
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(n)
    x = (torch.randn(n, generator=g) * 1e-3).to(dev)
    for gv in (1.0, -0.37, 3.0e4):
        gs = torch.tensor(gv, device=dev)
        for dt in (torch.bfloat16, torch.float32):
            ours = ops.scale_grad(x, gs, dt)
            torch.cuda.synchronize()
            assert ours.dtype == dt and torch.equal(ours, (x * gs).to(dt)), (n, gv, dt)
