"""Edge cases of the reference-facing shim on the GPU, kept in a file collected after the
parity tests: inputs with nothing to select."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_compute_kl_loss_no_blocks():
    """No blocks at all (anchor_positions [B, 0]): the reference returns 0.0 with
    requires_grad (its index tensors are empty, so no position is valid, train.py:166-167);
    the shim does the same without a launch, and the row gather's backward gives an empty
    gradient."""
    from orthrus_training_test_b200 import compute_kl_loss, gather_rows
    dev = torch.device("cuda:0")
    B, K, H, V, L = 2, 4, 64, 50, 20
    diff = torch.randn(B, 0, H, device=dev, requires_grad=True)
    ar = torch.randn(B, L, H, device=dev)
    anchors = torch.zeros(B, 0, dtype=torch.long, device=dev)
    tgt = torch.zeros(B, 0, dtype=torch.long, device=dev)
    head = torch.nn.Linear(H, V, bias=False).to(dev)
    loss = compute_kl_loss(diff, ar, head, anchors, K, tgt, 0)
    assert loss.item() == 0.0 and loss.requires_grad
    h_s, h_t, valid = gather_rows(diff, ar, anchors, K, tgt, 0)
    assert h_s.shape == (0, H) and h_t.shape == (0, H) and valid.shape == (0,)
    h_s.sum().backward()
    assert diff.grad is not None and diff.grad.shape == diff.shape
