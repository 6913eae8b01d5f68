"""Fused KL-GEMM distillation loss for B200 (sm_100a).

Public API
  compute_kl_loss   drop-in for the reference's ``train.compute_kl_loss``
  kl_gemm_loss      the fused loss on aligned rows (``KLGemmFn.apply``)
  KLGemmFn          the ``torch.autograd.Function``
  parallel          row-sharded and vocab-sharded multi-GPU variants
  prenorm_kl_loss   the fused loss on hidden states before the final RMSNorm
  sampling          fused lm_head + greedy / sampled token selection for inference
"""
from .ops import KLGemmFn, PrenormKLGemmFn, kl_gemm_loss, kl_forward, kl_backward, prenorm_kl_loss  # noqa: F401
from .loss import compute_kl_loss, gather_rows, select_rows  # noqa: F401

__all__ = ["KLGemmFn", "PrenormKLGemmFn", "prenorm_kl_loss", "kl_gemm_loss", "kl_forward", "kl_backward", "compute_kl_loss", "gather_rows", "select_rows"]
