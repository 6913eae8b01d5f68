"""Host-side logic of the drop-in shim (CPU): the row selection of
train.py:124-139 / 156-164 that feeds the fused op."""
import numpy as np
import pytest
import torch

from oracle import klgemm_oracle as O
from orthrus_training_test_b200.loss import kl_indices, select_rows
from tests.conftest import GOLDEN, golden_cases


@pytest.mark.parametrize("name", golden_cases())
def test_select_rows_matches_oracle(name):
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    h_s, h_t, valid = select_rows(torch.tensor(g["diff_hidden"]), torch.tensor(g["ar_hidden"]),
                                  torch.tensor(g["anchor_positions"]), int(g["K"]), torch.tensor(g["target_ids"]),
                                  int(g["pad"]))
    rs, rt, rv, _, _ = O.select_rows_np(g["diff_hidden"], g["ar_hidden"], g["anchor_positions"], int(g["K"]),
                                        g["target_ids"], int(g["pad"]))
    np.testing.assert_array_equal(h_s.numpy(), rs)
    np.testing.assert_array_equal(h_t.numpy(), rt)
    np.testing.assert_array_equal(valid.numpy(), rv)


def test_indices_match_reference_layout():
    dp, bi, off = kl_indices(3, 4, 5, "cpu")
    rdp, rbi, roff = O.kl_indices(3, 4, 5)
    np.testing.assert_array_equal(dp.numpy(), rdp)
    np.testing.assert_array_equal(bi.numpy(), rbi)
    np.testing.assert_array_equal(off.numpy(), roff)
    # anchors (offset 0 of each block) never appear among student rows
    assert not np.any(dp.numpy() % 5 == 0)


def test_student_gather_is_differentiable():
    g = dict(np.load(GOLDEN / "anchors_clamp.npz"))
    diff = torch.tensor(g["diff_hidden"], requires_grad=True)
    h_s, _, _ = select_rows(diff, torch.tensor(g["ar_hidden"]), torch.tensor(g["anchor_positions"]), int(g["K"]),
                            torch.tensor(g["target_ids"]), int(g["pad"]))
    h_s.sum().backward()
    assert diff.grad is not None and diff.grad.sum().item() == h_s.numel()


def test_shim_rejects_cpu_tensors():
    """No CPU fallback: the op refuses host tensors loudly."""
    from orthrus_training_test_b200 import kl_gemm_loss
    x = torch.zeros(4, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        kl_gemm_loss(x, x, torch.zeros(10, 64), torch.ones(4, dtype=torch.bool))


@pytest.mark.parametrize("h_shape,w_shape,n_tok,lse_shape", [
    ((4, 64), (10, 32), 4, (4,)),      # hidden sizes differ
    ((4, 64), (10, 64), 3, (4,)),      # too few tokens
    ((4, 64), (10, 64), 4, (2, 2)),    # lse not [N]
    ((64,), (10, 64), 1, (1,)),        # h not 2-D
])
def test_token_logprob_rejects_bad_shapes(h_shape, w_shape, n_tok, lse_shape):
    """Shapes are checked on the host before any device pointer is formed."""
    from orthrus_training_test_b200.sampling import token_logprob
    with pytest.raises(ValueError):
        token_logprob(torch.zeros(h_shape), torch.zeros(w_shape), torch.zeros(n_tok, dtype=torch.long),
                      torch.zeros(lse_shape))


# (diff_hidden, ar_hidden_states, anchor_positions, K, target_ids) shapes; B=2, B_blocks=3, K=4, H=64
@pytest.mark.parametrize("diff,ar,anc,K,tgt", [
    ((2, 12, 64), (1, 20, 64), (2, 3), 4, (2, 12)),    # AR states of another batch size
    ((2, 12, 64), (2, 20, 32), (2, 3), 4, (2, 12)),    # AR states of another hidden size
    ((2, 12, 64), (2, 20, 64), (1, 3), 4, (2, 12)),    # anchors of another batch size
    ((2, 12, 64), (2, 20, 64), (2, 3), 4, (2, 11)),    # too few target positions
    ((2, 12, 64), (2, 20, 64), (2, 3), 4, (24,)),      # targets not [B, P]
    ((2, 12, 64), (2, 20, 64), (2, 4), 4, (2, 12)),    # positions != B_blocks * K
    ((2, 3, 64), (2, 20, 64), (2, 3), 1, (2, 3)),      # K = 1: no diffusion position
    ((24, 64), (2, 20, 64), (2, 3), 4, (2, 12)),       # diff_hidden not 3-D
])
def test_row_gather_rejects_bad_shapes(diff, ar, anc, K, tgt):
    """Every index the gather kernel forms stays inside its tensor: inconsistent shapes raise
    on the host (where the reference's torch indexing would raise) before any device work."""
    from orthrus_training_test_b200.loss import gather_rows
    with pytest.raises(ValueError):
        gather_rows(torch.zeros(diff), torch.zeros(ar), torch.zeros(anc, dtype=torch.long), K,
                    torch.zeros(tgt, dtype=torch.long), 0)


def test_row_gather_accepts_no_blocks():
    """Zero blocks pass the shape check (the reference returns a zero loss for them)."""
    from orthrus_training_test_b200.loss import _check_selection_shapes
    assert _check_selection_shapes(torch.zeros(2, 0, 64), torch.zeros(2, 20, 64), torch.zeros(2, 0), 4,
                                   torch.zeros(2, 0)) == (2, 0, 64, 20, 0)


def test_row_gather_accepts_longer_targets():
    """target_ids wider than the diffusion positions pass the shape check (only the first
    B_blocks*K positions are read, as train.py:163 indexes them)."""
    from orthrus_training_test_b200.loss import _check_selection_shapes
    assert _check_selection_shapes(torch.zeros(2, 12, 64), torch.zeros(2, 20, 64), torch.zeros(2, 3), 4,
                                   torch.zeros(2, 16)) == (2, 12, 64, 20, 3)
    with pytest.raises(RuntimeError, match="CUDA"):   # consistent shapes reach the device check
        from orthrus_training_test_b200.loss import gather_rows
        gather_rows(torch.zeros(2, 12, 64), torch.zeros(2, 20, 64), torch.zeros(2, 3, dtype=torch.long), 4,
                    torch.zeros(2, 12, dtype=torch.long), 0)


def _bf(*shape):
    return torch.zeros(*shape, dtype=torch.bfloat16)


@pytest.mark.parametrize("case", ["h_t rows", "weight H", "mask N", "mixed dtypes", "fp16", "strided h_s", "3-D"])
def test_ops_reject_inconsistent_operands(case):
    """The wrappers check shapes, dtypes and density on the host: the kernels read N x H per
    view, V x H of the weight and N mask bytes of one dtype, so a mismatch would otherwise read
    past a buffer on the device."""
    from orthrus_training_test_b200 import ops
    hs, ht, w, m = _bf(8, 64), _bf(8, 64), _bf(10, 64), torch.ones(8, dtype=torch.bool)
    if case == "h_t rows":
        ht = _bf(7, 64)
    elif case == "weight H":
        w = _bf(10, 32)
    elif case == "mask N":
        m = torch.ones(9, dtype=torch.bool)
    elif case == "mixed dtypes":
        hs, ht = hs.float(), ht.float()          # fp32 rows with a bf16 weight
    elif case == "fp16":
        hs, ht, w = hs.half(), ht.half(), w.half()
    elif case == "strided h_s":
        hs = _bf(8, 128)[:, ::2]
    elif case == "3-D":
        hs, ht = _bf(2, 4, 64), _bf(2, 4, 64)
    with pytest.raises((ValueError, TypeError)):
        ops.kl_fwd_bwd(hs, ht, w, m)
    with pytest.raises((ValueError, TypeError)):
        ops.kl_forward(hs, ht, w, m)


def test_ops_pieces_check_their_buffers():
    from orthrus_training_test_b200 import ops
    hs, ht, w, m = _bf(8, 64), _bf(8, 64), _bf(10, 64), torch.ones(8, dtype=torch.bool)
    lse, cnt = torch.zeros(2, 8), torch.ones(1)
    with pytest.raises(TypeError):               # the vocab-shard pieces are bf16 only
        ops.lse_record(hs.float(), ht.float(), w.float())
    with pytest.raises(ValueError):              # lse of another row count
        ops.pass2(hs, ht, w, m, torch.zeros(2, 7), cnt)
    with pytest.raises(ValueError):              # dH buffer too small
        ops.pass2(hs, ht, w, m, lse, cnt, dh_out=torch.zeros(8, 32))
    with pytest.raises(ValueError):              # count not one fp32 element
        ops.pass2(hs, ht, w, m, lse, torch.ones(2))
    with pytest.raises(ValueError):              # cross term of another row count
        ops.kl_loss(lse, torch.zeros(7), m, cnt)
    with pytest.raises(ValueError):              # records not [R, 2, 2N]
        ops.lse_merge(torch.zeros(2, 3, 16))
    with pytest.raises(ValueError):              # partial records not [P, 5, N]
        ops.merge_stats(torch.zeros(2, 4, 8))
    with pytest.raises(ValueError):              # statistics of another row count
        ops.finalize(torch.zeros(5, 7), m, cnt)
    with pytest.raises(RuntimeError, match="CUDA"):   # consistent host tensors reach the device check
        ops.pass2(hs, ht, w, m, lse, cnt)


def test_norm_wrappers_check_shapes():
    from orthrus_training_test_b200 import ops
    x = torch.zeros(4, 64)
    with pytest.raises(ValueError):              # gamma of another width
        ops.rmsnorm_rows(x, torch.ones(32))
    with pytest.raises(ValueError):              # rows not 2-D
        ops.rmsnorm_rows(torch.zeros(2, 2, 64), torch.ones(64))
    with pytest.raises(ValueError):              # dy of another shape
        ops.rmsnorm_rows_backward(x, torch.ones(64), torch.ones(4), torch.zeros(4, 32))
    with pytest.raises(ValueError):              # rstd of another row count
        ops.rmsnorm_rows_backward(x, torch.ones(64), torch.ones(3), torch.zeros(4, 64))
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.rmsnorm_rows(x, torch.ones(64))
