"""The row-selection kernel (train.py:124-139, 156-164) against the oracle, bit for bit.

Every golden fixture's gather (including anchors whose rows clamp at the sequence end) and
the backward scatter: the student rows' gradient lands at their diffusion positions and the
anchor positions get zeros.
"""
import numpy as np
import pytest
import torch

from oracle import klgemm_oracle as O
from tests.conftest import GOLDEN, golden_cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_cases())
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gather_rows_bit_exact(name, dtype):
    from orthrus_training_test_b200 import gather_rows
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    dev = torch.device("cuda:0")
    diff = torch.tensor(g["diff_hidden"]).to(dtype)
    ar = torch.tensor(g["ar_hidden"]).to(dtype)
    anchors = torch.tensor(g["anchor_positions"])
    tgt = torch.tensor(g["target_ids"])
    K, pad = int(g["K"]), int(g["pad"])
    d = diff.to(dev).requires_grad_(True)
    h_s, h_t, valid = gather_rows(d, ar.to(dev), anchors.to(dev), K, tgt.to(dev), pad)
    rs, rt, rv, dp, _ = O.select_rows_np(diff.float().numpy(), ar.float().numpy(), g["anchor_positions"], K,
                                         g["target_ids"], pad)
    np.testing.assert_array_equal(h_s.detach().float().cpu().numpy(), rs)
    np.testing.assert_array_equal(h_t.float().cpu().numpy(), rt)
    np.testing.assert_array_equal(valid.cpu().numpy().astype(bool), rv)
    # backward: the gradient of each selected row at its position, zeros at the anchors
    gr = torch.randn(h_s.shape, generator=torch.Generator().manual_seed(1)).to(dtype)
    h_s.backward(gr.to(dev))
    bi = np.broadcast_to(np.arange(dp.shape[0])[:, None], dp.shape)
    want = np.zeros(diff.shape, np.float32)
    want[bi.reshape(-1), dp.reshape(-1)] = gr.float().numpy()
    np.testing.assert_array_equal(d.grad.float().cpu().numpy(), want)
