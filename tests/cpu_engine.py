"""CPU stand-in for the CUDA engine, built on the oracle (tests only).

Implements the engine interface that ``orthrus_training_test_b200.parallel``
drives, so the multi-rank host logic (normaliser all-reduce, partial-record
all-gather and merge, dW / dH exchanges) can run on ``gloo`` CPU ranks.
Records are in the natural-log domain here; the product engine uses log2 --
the format is private to each engine.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import klgemm_oracle as O


def _np(t):
    return t.detach().cpu().double().numpy()


class CpuOracleEngine:
    def prepare(self, x):
        return x.detach().double()

    def mask(self, m):
        return (m != 0).to(torch.uint8)

    def count(self, mask):
        return mask.double().sum().reshape(1)

    def forward(self, h_s, h_t, w, mask, temperature, count):
        stats = self.partial_stats(h_s, h_t, w, temperature)
        return self.finalize(stats, mask, count)

    def partial_stats(self, h_s, h_t, w, temperature):
        return torch.from_numpy(O.partial_stats_np(_np(h_s), _np(h_t), _np(w), temperature))

    def merge(self, parts):
        return torch.from_numpy(O.merge_partials_np(_np(parts)))

    def finalize(self, stats, mask, count):
        loss, _, ls, lt = O.finalize_np(_np(stats), _np(mask).astype(bool), float(count.item()))
        return torch.tensor(loss, dtype=torch.float64), torch.from_numpy(np.stack([ls, lt]))

    def forward_backward(self, h_s, h_t, w, mask, temperature, count, need_dh, need_dw):
        loss, lse = self.forward(h_s, h_t, w, mask, temperature, count)
        dh, dw = self.backward(h_s, h_t, w, mask, lse, count, None, temperature, need_dh, need_dw)
        return loss, dh, dw

    def backward(self, h_s, h_t, w, mask, lse, count, grad, temperature, need_dh, need_dw):
        g = 1.0 if grad is None else float(grad.item())
        L = _np(lse)
        dh, dw = O.range_grads_np(_np(h_s), _np(h_t), _np(w), L[0], L[1], _np(mask).astype(bool),
                                  float(count.item()), temperature, g)
        return (torch.from_numpy(dh) if need_dh else None), (torch.from_numpy(dw) if need_dw else None)

    # the training step in pieces (vocab sharding); records here are natural-log (m, S)
    acc_dtype = torch.float64

    def lse_record(self, h_s, h_t, w, temperature):
        st = O.partial_stats_np(_np(h_s), _np(h_t), _np(w), temperature)
        return torch.from_numpy(np.stack([np.concatenate([st[0], st[2]]), np.concatenate([st[1], st[3]])]))

    def lse_merge(self, recs):
        r = _np(recs)
        M = r[:, 0].max(axis=0)
        S = (r[:, 1] * np.exp(r[:, 0] - M)).sum(axis=0)
        lse = M + np.log(S)
        n = lse.shape[0] // 2
        return torch.from_numpy(np.stack([lse[:n], lse[n:]]))

    def pass2(self, h_s, h_t, w, mask, lse, count, temperature, need_dh, need_dw, dh_out=None):
        L = _np(lse)
        dh, dw = O.range_grads_np(_np(h_s), _np(h_t), _np(w), L[0], L[1], _np(mask).astype(bool),
                                  float(count.item()), temperature, 1.0)
        inv_t = 1.0 / float(temperature)
        zs = _np(h_s) @ _np(w).T * inv_t
        zt = _np(h_t) @ _np(w).T * inv_t
        cross = (np.exp(zt - L[1][:, None]) * (zt - zs)).sum(axis=1)
        dh_t = None
        if need_dh:
            dh_t = torch.from_numpy(dh)
            if dh_out is not None:
                dh_out.copy_(dh_t)
                dh_t = dh_out
        return dh_t, (torch.from_numpy(dw) if need_dw else None), torch.from_numpy(cross)

    def kl_loss(self, lse, cross, mask, count):
        L = _np(lse)
        kl = _np(cross) + L[0] - L[1]
        valid = _np(mask).astype(bool)
        c = float(count.item())
        return torch.tensor(float((kl * valid).sum() / c) if c > 0 else 0.0, dtype=torch.float64)
