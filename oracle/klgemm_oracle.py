"""Oracle: a CPU restatement of the reference's KL distillation loss.

TEST INFRASTRUCTURE ONLY.  The product (``orthrus_training_test_b200``) never
imports this module; ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` use it for the expected results of parity
checks and as the CPU baseline.

Parity pin: every function here is checked against golden vectors produced by
running the reference's own ``train.compute_kl_loss`` (reference
``train.py:142-195`` + ``train.py:198-210``) in the build container; the
generator is ``tests/golden/make_golden.py`` and the check is
``tests/test_oracle.py``.

Reference algorithm (``train.py``):

* ``_get_kl_indices`` (train.py:124-139): student rows are the diffusion
  positions ``blk*K + k`` for ``k = 1..K-1`` (the anchor, offset 0, is
  excluded); teacher offsets are ``0..K-2``.
* ``compute_kl_loss`` (train.py:142-195): teacher row ``anchor + k - 1``
  clamped to ``[0, L-1]`` (train.py:161); ``valid = target != pad``
  (train.py:163-164); early return of ``0.0`` when no row is valid
  (train.py:166-167); 2048-row chunks (train.py:170-173); teacher softmax and
  entropy in fp32 under ``no_grad`` (train.py:188-191); result
  ``sum(valid * KL) / sum(valid)`` (train.py:195).
* ``_kl_chunk_body`` (train.py:198-210): student logits through the shared
  ``lm_head``; soft-target ``cross_entropy`` against the teacher probabilities;
  ``KL = CE - entropy``; masked sum.

Temperature: the reference has none (T = 1).  For T != 1 both logit tensors
are divided by T before the softmax, with no T^2 factor; at T = 1 this is the
reference formula unchanged.

Three restatements live here:

``kl_loss_reference_ops``   torch fp32, the reference's own op sequence and
                            signature (device agnostic; autograd for grads).
``aligned_kl_loss_torch``   torch fp32, the same ops on pre-aligned rows
                            ``(h_s, h_t, mask)`` -- the fused op's contract.
``aligned_kl_loss_np``      float64 numpy with closed-form gradients, an
                            independent derivation used to cross-check both.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

CHUNK = 2048  # train.py:170


# --------------------------------------------------------------------------
# Row selection (reference train.py:124-139, train.py:160-164)
# --------------------------------------------------------------------------

def kl_indices(B: int, B_blocks: int, K: int):
    """Restates ``_get_kl_indices`` (train.py:124-139) in numpy.

    Returns ``(diff_pos [B, N], batch_idx [B, N], offsets [K-1])`` with
    ``N = B_blocks * (K - 1)``.
    """
    N = B_blocks * (K - 1)
    diff_pos = np.arange(B_blocks * K).reshape(B_blocks, K)[:, 1:].reshape(-1)
    diff_pos = np.broadcast_to(diff_pos[None, :], (B, N)).copy()
    batch_idx = np.broadcast_to(np.arange(B)[:, None], (B, N)).copy()
    offsets = np.arange(0, K - 1)
    return diff_pos, batch_idx, offsets


def select_rows_np(diff_hidden, ar_hidden, anchor_positions, K, target_ids, pad_token_id):
    """Gathers aligned student/teacher rows and the validity mask.

    Restates train.py:156-164: ``ar_pos = clamp(anchor + offsets, 0, L-1)``,
    ``tgt = target_ids[batch_idx, diff_pos]``, ``valid = tgt != pad``.
    Returns ``(h_s [B*N, H], h_t [B*N, H], valid [B*N] bool, diff_pos, ar_pos)``.
    """
    B, B_blocks = anchor_positions.shape
    L = ar_hidden.shape[1]
    N = B_blocks * (K - 1)
    diff_pos, batch_idx, offsets = kl_indices(B, B_blocks, K)
    ar_pos = np.clip((anchor_positions[:, :, None] + offsets[None, None, :]).reshape(B, N), 0, L - 1)
    tgt = target_ids[batch_idx, diff_pos]
    valid = tgt != pad_token_id
    h_s = diff_hidden[batch_idx, diff_pos].reshape(B * N, -1)
    h_t = ar_hidden[batch_idx, ar_pos].reshape(B * N, -1)
    return h_s, h_t, valid.reshape(-1), diff_pos, ar_pos


# --------------------------------------------------------------------------
# torch fp32 restatement of the reference op sequence
# --------------------------------------------------------------------------

def _torch():
    import torch
    return torch


def fp32_strict():
    """Context for an fp32 reference: TF32 off and "highest" matmul precision.

    The reference module flips both on import (train.py:47-50); an fp32
    oracle must undo that or it is not fp32.
    """
    torch = _torch()

    class _Ctx:
        def __enter__(self):
            self.prev = (torch.backends.cuda.matmul.allow_tf32,
                         torch.backends.cudnn.allow_tf32,
                         torch.get_float32_matmul_precision())
            torch.backends.cuda.matmul.allow_tf32 = False
            torch.backends.cudnn.allow_tf32 = False
            torch.set_float32_matmul_precision("highest")
            return self

        def __exit__(self, *exc):
            torch.backends.cuda.matmul.allow_tf32 = self.prev[0]
            torch.backends.cudnn.allow_tf32 = self.prev[1]
            torch.set_float32_matmul_precision(self.prev[2])
            return False

    return _Ctx()


def kl_loss_reference_ops(diff_hidden, ar_hidden_states, weight, anchor_positions, K,
                          target_ids, pad_token_id, temperature: float = 1.0,
                          chunk: int = CHUNK):
    """Restates ``compute_kl_loss`` (train.py:142-195) with the fp32 teacher path.

    Same op order as the reference: gather -> teacher ``linear`` ->
    ``softmax``/``log_softmax``/entropy under ``no_grad`` (train.py:188-191)
    -> student ``linear`` -> soft-target ``cross_entropy`` (train.py:202-208)
    -> ``CE - ent`` -> masked sum (train.py:209-210) -> ``/ total``
    (train.py:195).  ``weight`` is the lm_head matrix ``[V, H]``; set
    ``weight.requires_grad_(True)`` to obtain dW (the reference trains with a
    frozen lm_head, so it never computes dW itself).
    """
    torch = _torch()
    F = torch.nn.functional
    B, B_blocks = anchor_positions.shape
    device = diff_hidden.device
    L = ar_hidden_states.shape[1]
    N = B_blocks * (K - 1)
    dp, bi, off = kl_indices(B, B_blocks, K)
    diff_pos = torch.as_tensor(dp, device=device)
    batch_idx = torch.as_tensor(bi, device=device)
    offsets = torch.as_tensor(off, device=device)
    ar_pos = (anchor_positions.unsqueeze(-1) + offsets).view(B, N).clamp(0, L - 1)
    tgt = target_ids[batch_idx, diff_pos]
    valid = tgt != pad_token_id
    total_tokens = valid.sum().float()
    if total_tokens == 0:                                   # train.py:166-167
        return torch.tensor(0.0, device=device, requires_grad=True)
    inv_t = 1.0 / float(temperature)
    total_kl = 0.0
    for c in range(0, N, chunk):                            # train.py:173
        c_end = min(c + chunk, N)
        chunk_valid = valid[:, c:c_end].float()
        if not chunk_valid.any():                           # train.py:176-177
            continue
        b_idx = batch_idx[:, c:c_end]
        d_idx = diff_pos[:, c:c_end]
        a_idx = ar_pos[:, c:c_end]
        with torch.no_grad():                               # train.py:183-191
            t_logits = F.linear(ar_hidden_states[b_idx, a_idx], weight).float() * inv_t
            p_t = F.softmax(t_logits, dim=-1)
            ent = -(p_t * F.log_softmax(t_logits, dim=-1)).sum(dim=-1)
        s_logits = F.linear(diff_hidden[b_idx, d_idx], weight) * inv_t   # train.py:201-202
        ce = F.cross_entropy(s_logits.view(-1, s_logits.size(-1)),
                             p_t.view(-1, p_t.size(-1)), reduction="none").view(B, -1)
        kl = ce.float() - ent.float()                       # train.py:209
        total_kl = total_kl + (kl * chunk_valid).sum()      # train.py:210
    return total_kl / total_tokens


def aligned_kl_loss_torch(h_s, h_t, weight, mask, temperature: float = 1.0,
                          chunk: int = CHUNK, normaliser=None):
    """The reference op sequence on pre-aligned rows (the fused op's contract).

    ``h_s, h_t [N, H]``, ``weight [V, H]``, ``mask [N]`` (bool).  Equivalent to
    ``kl_loss_reference_ops`` after its gather step.  ``normaliser`` overrides
    ``sum(mask)`` (used for row-sharded checks where the count is global).
    Returns a scalar tensor that is differentiable w.r.t. ``h_s`` and
    ``weight``.  Rows are processed in ``chunk``-row blocks so that only
    ``chunk x V`` logits exist at a time.
    """
    torch = _torch()
    F = torch.nn.functional
    valid = mask.bool()
    total = valid.sum().float() if normaliser is None else torch.as_tensor(float(normaliser))
    if float(total) == 0.0:
        return torch.tensor(0.0, device=h_s.device, requires_grad=True)
    inv_t = 1.0 / float(temperature)
    N = h_s.shape[0]
    total_kl = 0.0
    for c in range(0, N, chunk):
        c_end = min(c + chunk, N)
        cv = valid[c:c_end].float()
        if not cv.any():
            continue
        with torch.no_grad():
            t_logits = F.linear(h_t[c:c_end].float(), weight.float()).float() * inv_t
            p_t = F.softmax(t_logits, dim=-1)
            ent = -(p_t * F.log_softmax(t_logits, dim=-1)).sum(dim=-1)
            del t_logits
        s_logits = F.linear(h_s[c:c_end].float(), weight.float()) * inv_t
        ce = F.cross_entropy(s_logits, p_t, reduction="none")
        total_kl = total_kl + ((ce.float() - ent) * cv).sum()
    return total_kl / total.to(h_s.device)


def aligned_kl_torch_with_grads(h_s, h_t, weight, mask, temperature: float = 1.0,
                                chunk: int = CHUNK, normaliser=None, want_dw: bool = True):
    """Loss, dH_s and dW of ``aligned_kl_loss_torch`` via autograd, in fp32.

    Inputs of any float dtype are upcast to fp32 first (so a bf16 problem is
    checked against fp32 arithmetic on the same bf16 values).
    """
    torch = _torch()
    with fp32_strict():
        hs = h_s.detach().float().requires_grad_(True)
        w = weight.detach().float().requires_grad_(want_dw)
        loss = aligned_kl_loss_torch(hs, h_t.detach().float(), w, mask, temperature,
                                     chunk=chunk, normaliser=normaliser)
        if loss.grad_fn is None:
            dh = torch.zeros_like(hs)
            dw = torch.zeros_like(w) if want_dw else None
        else:
            loss.backward()
            dh = hs.grad if hs.grad is not None else torch.zeros_like(hs)
            dw = (w.grad if w.grad is not None else torch.zeros_like(w)) if want_dw else None
    return loss.detach(), dh, dw


# --------------------------------------------------------------------------
# float64 numpy restatement with closed-form gradients
# --------------------------------------------------------------------------

def _lse(z):
    m = z.max(axis=-1, keepdims=True)
    return (m + np.log(np.exp(z - m).sum(axis=-1, keepdims=True)))[..., 0]


def aligned_kl_loss_np(h_s, h_t, W, mask, temperature: float = 1.0, chunk: int = 512,
                       normaliser: Optional[float] = None, want_grads: bool = True):
    """float64 restatement: ``loss, dH_s, dW, row_kl, lse_s, lse_t``.

    Per row ``i`` (natural log, ``z = h W^T / T``):
    ``KL_i = sum_v p_v (z_t - z_s) - lse_t + lse_s`` with ``p = softmax(z_t)``
    -- algebraically ``CE(z_s, p) - H(p)`` of train.py:204-209.
    Gradient of ``loss = sum valid_i KL_i / n`` (soft-target CE rule, teacher
    detached as in train.py:183): ``dZ_s = valid_i/n * (softmax(z_s) - p) / T``,
    ``dH_s = dZ_s W``, ``dW = dZ_s^T h_s``.
    """
    h_s = np.asarray(h_s, dtype=np.float64)
    h_t = np.asarray(h_t, dtype=np.float64)
    W = np.asarray(W, dtype=np.float64)
    valid = np.asarray(mask).astype(bool)
    n = float(valid.sum()) if normaliser is None else float(normaliser)
    N = h_s.shape[0]
    inv_t = 1.0 / float(temperature)
    row_kl = np.zeros(N)
    lse_s = np.zeros(N)
    lse_t = np.zeros(N)
    dH = np.zeros_like(h_s) if want_grads else None
    dW = np.zeros_like(W) if want_grads else None
    for c in range(0, N, chunk):
        e = min(c + chunk, N)
        zs = (h_s[c:e] @ W.T) * inv_t
        zt = (h_t[c:e] @ W.T) * inv_t
        ls = _lse(zs)
        lt = _lse(zt)
        p = np.exp(zt - lt[:, None])
        q = np.exp(zs - ls[:, None])
        row_kl[c:e] = (p * (zt - zs)).sum(axis=1) - lt + ls
        lse_s[c:e] = ls
        lse_t[c:e] = lt
        if want_grads and n > 0:
            coef = valid[c:e].astype(np.float64) / n * inv_t
            dz = coef[:, None] * (q - p)
            dH[c:e] = dz @ W
            dW += dz.T @ h_s[c:e]
    loss = float((row_kl * valid).sum() / n) if n > 0 else 0.0
    return loss, dH, dW, row_kl, lse_s, lse_t


# --------------------------------------------------------------------------
# Vocab-range partial statistics (shard-combine reference for multi-rank tests)
# --------------------------------------------------------------------------

def partial_stats_np(h_s, h_t, W_range, temperature: float = 1.0):
    """Per-row partial record over one vocab range, natural-log domain.

    Returns ``[5, N]``: ``(m_s, S_s, m_t, S_t, A)`` with ``S = sum exp(z - m)``
    and ``A = sum exp(z_t - m_t) (z_t - z_s)`` over the range.
    """
    inv_t = 1.0 / float(temperature)
    zs = (np.asarray(h_s, np.float64) @ np.asarray(W_range, np.float64).T) * inv_t
    zt = (np.asarray(h_t, np.float64) @ np.asarray(W_range, np.float64).T) * inv_t
    ms = zs.max(axis=1)
    mt = zt.max(axis=1)
    es = np.exp(zs - ms[:, None])
    et = np.exp(zt - mt[:, None])
    return np.stack([ms, es.sum(1), mt, et.sum(1), (et * (zt - zs)).sum(1)])


def merge_partials_np(parts):
    """Online-softmax merge of ``[P, 5, N]`` partial records into ``[5, N]``."""
    parts = np.asarray(parts, np.float64)
    ms = parts[:, 0].max(axis=0)
    mt = parts[:, 2].max(axis=0)
    ws = np.exp(parts[:, 0] - ms)
    wt = np.exp(parts[:, 2] - mt)
    return np.stack([ms, (parts[:, 1] * ws).sum(0), mt, (parts[:, 3] * wt).sum(0),
                     (parts[:, 4] * wt).sum(0)])


def finalize_np(stats, mask, normaliser: Optional[float] = None):
    """Loss, per-row KL and log-sum-exps from a merged ``[5, N]`` record."""
    ms, Ss, mt, St, A = stats
    lse_s = ms + np.log(Ss)
    lse_t = mt + np.log(St)
    row_kl = A / St - lse_t + lse_s
    valid = np.asarray(mask).astype(bool)
    n = float(valid.sum()) if normaliser is None else float(normaliser)
    loss = float((row_kl * valid).sum() / n) if n > 0 else 0.0
    return loss, row_kl, lse_s, lse_t


def range_grads_np(h_s, h_t, W_range, lse_s, lse_t, mask, normaliser, temperature=1.0, g=1.0):
    """dZ over one vocab range given global log-sum-exps: ``(dH partial, dW range)``."""
    inv_t = 1.0 / float(temperature)
    hs = np.asarray(h_s, np.float64)
    Wr = np.asarray(W_range, np.float64)
    zs = (hs @ Wr.T) * inv_t
    zt = (np.asarray(h_t, np.float64) @ Wr.T) * inv_t
    q = np.exp(zs - np.asarray(lse_s)[:, None])
    p = np.exp(zt - np.asarray(lse_t)[:, None])
    n = float(normaliser)
    coef = (np.asarray(mask).astype(np.float64) / n * inv_t * g) if n > 0 else np.zeros(hs.shape[0])
    dz = coef[:, None] * (q - p)
    return dz @ Wr, dz.T @ hs


# --------------------------------------------------------------------------
# Seeded workloads (shapes and distributions of the benchmark configurations)
# --------------------------------------------------------------------------

def block_mask(n_rows: int, block: int, lo: float, hi: float, gen) -> "object":
    """Per block of ``block`` positions draw ``r ~ U(lo, hi)``; each row valid with prob ``r``."""
    torch = _torch()
    n_blk = (n_rows + block - 1) // block
    r = torch.rand(n_blk, generator=gen) * (hi - lo) + lo
    r = r.repeat_interleave(block)[:n_rows]
    return torch.rand(n_rows, generator=gen) < r


def make_problem(name: str, n_rows: Optional[int] = None, seed: int = 42):
    """Seeded synthetic inputs with a benchmark configuration's shapes.

    Returns a dict with ``h_s, h_t [N, H]``, ``W [V, H]``, ``mask [N]`` (bool),
    ``T`` and ``dtype`` (all CPU tensors; bf16 configurations are returned
    already rounded to bf16).  ``n_rows`` subsamples the row count.

    Configurations (rows x hidden x vocab):
      c1  1024 x 576 x 49152   fp32, N(0,1) hidden, N(0,0.02) weight, Bernoulli(0.5) mask, T=1
      c2  16384 x 576 x 49152  bf16, mask ratio U(0,1) per block of 32, T=1
      c3  65536 x 2048 x 49152 bf16, Bernoulli(0.5), T=1
      c4  32768 x 1024 x 248320 bf16, Bernoulli(0.5), T=1 (vocab split in 8 shards)
      c5  12288 x 576 x 49152  bf16, mask ratio U(0,0.5) per block of 32, teacher x4, T=2,
          >= 8 rows forced all-masked
    """
    torch = _torch()
    cfg = {
        "c1": (1024, 576, 49152, torch.float32),
        "c2": (16384, 576, 49152, torch.bfloat16),
        "c3": (65536, 2048, 49152, torch.bfloat16),
        "c4": (32768, 1024, 248320, torch.bfloat16),
        "c5": (12288, 576, 49152, torch.bfloat16),
    }[name]
    N, H, V, dt = cfg
    if n_rows is not None:
        N = int(n_rows)
    g = torch.Generator().manual_seed(seed)
    h_s = torch.randn(N, H, generator=g)
    h_t = torch.randn(N, H, generator=g)
    W = torch.randn(V, H, generator=g) * 0.02
    T = 1.0
    if name == "c2":
        mask = block_mask(N, 32, 0.0, 1.0, g)
    elif name == "c5":
        mask = block_mask(N, 32, 0.0, 0.5, g)
        h_t = h_t * 4.0
        T = 2.0
        mask[: min(8, N)] = False
        mask[N // 2: N // 2 + 8] = False
    else:
        mask = torch.rand(N, generator=g) < 0.5
    return {"h_s": h_s.to(dt), "h_t": h_t.to(dt), "W": W.to(dt), "mask": mask,
            "T": T, "dtype": dt, "name": name}


def grad_metrics(ours, ref) -> Tuple[float, float]:
    """``(max_rel, cosine)`` of a gradient against its reference.

    ``max_rel = max|ours - ref| / max|ref|`` (normalised max error) and the
    cosine similarity of the flattened tensors, both in float64.
    """
    a = np.asarray(ours, np.float64).ravel()
    b = np.asarray(ref, np.float64).ravel()
    denom = np.abs(b).max()
    max_rel = float(np.abs(a - b).max() / denom) if denom > 0 else float(np.abs(a).max())
    na = np.linalg.norm(a)
    nb = np.linalg.norm(b)
    if na == 0 and nb == 0:
        cos = 1.0
    elif na == 0 or nb == 0:
        cos = 0.0
    else:
        cos = float(a @ b / (na * nb))
    return max_rel, cos


LN2 = math.log(2.0)


# --------------------------------------------------------------------------
# Inference lm_head sampling (reference generate.py:40-78, infer.py:60-69)
# --------------------------------------------------------------------------

GREEDY_TEMPERATURE = 1e-5   # generate.py:52: below this, argmax and no probabilities


def sample_token_np(logits, temperature: float = 0.0):
    """Restates ``sample_token`` (generate.py:40-78) without top-k / top-p.

    ``temperature < 1e-5``: ``(argmax(logits, -1), None)`` -- the first index among
    equal maxima, as ``torch.argmax``.  Otherwise ``probs = softmax(logits / T)``
    (generate.py:75) and the token is a draw from ``probs`` (generate.py:77, by
    ``torch.multinomial`` there); this restatement returns ``(None, probs)`` since the
    draw itself is defined only by its distribution.
    """
    z = np.asarray(logits, dtype=np.float64)
    if temperature < GREEDY_TEMPERATURE:
        return np.argmax(z, axis=-1), None
    s = z / temperature
    s = s - s.max(axis=-1, keepdims=True)
    e = np.exp(s)
    return None, e / e.sum(axis=-1, keepdims=True)


def filtered_probs_np(logits, temperature: float, top_k: int = 0, top_p: float = 1.0):
    """The distribution ``sample_token`` draws from with top-k / top-p (generate.py:55-75).

    ``scaled = logits / T``; top-k removes every entry below the k-th largest scaled value
    (generate.py:59-61: entries equal to it stay); top-p sorts the (top-k filtered) scaled
    values in descending order, takes the cumulative softmax, and removes an entry when the
    cumulative probability *before* it already exceeds ``top_p`` (generate.py:64-73: the
    shift by one keeps the entry that crosses ``top_p``, and the first entry always stays).
    Returns ``(probs, kept)``: ``softmax`` over the kept entries and the boolean mask.
    """
    z = np.atleast_2d(np.asarray(logits, dtype=np.float64)) / float(temperature)
    n, V = z.shape
    kept = np.ones_like(z, dtype=bool)
    if top_k > 0:
        kth = -np.sort(-z, axis=-1)[:, min(top_k, V) - 1]
        kept &= z >= kth[:, None]
    if top_p < 1.0:
        zf = np.where(kept, z, -np.inf)
        order = np.argsort(-zf, axis=-1, kind="stable")
        zs = np.take_along_axis(zf, order, axis=-1)
        e = np.exp(zs - zs[:, :1])
        cum = np.cumsum(e / e.sum(axis=-1, keepdims=True), axis=-1)
        remove = cum > top_p
        remove[:, 1:] = remove[:, :-1].copy()
        remove[:, 0] = False
        rm = np.zeros_like(remove)
        np.put_along_axis(rm, order, remove, axis=-1)
        kept &= ~rm
    zf = np.where(kept, z, -np.inf)
    e = np.exp(zf - zf.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True), kept


def sample_hash_np(seed: int, rows, cols) -> np.ndarray:
    """The 32-bit counter hash of (seed, row, column) the fused sampler draws from.

    The row, column and both seed halves are combined with odd multipliers
    (0x9E3779B1, 0x85EBCA77, 0xC2B2AE3D), then mixed by the "lowbias32" finaliser
    (xorshift 16, x 0x7FEB352D, xorshift 15, x 0x846CA68B, xorshift 16).
    """
    M = np.uint64(0xFFFFFFFF)
    r = np.asarray(rows, dtype=np.uint64)[..., None] if np.ndim(rows) else np.uint64(rows)
    c = np.asarray(cols, dtype=np.uint64)
    lo, hi = np.uint64(seed & 0xFFFFFFFF), np.uint64((seed >> 32) & 0xFFFFFFFF)
    x = lo ^ ((r * np.uint64(0x9E3779B1)) & M) ^ ((c * np.uint64(0x85EBCA77)) & M) ^ ((hi * np.uint64(0xC2B2AE3D)) & M)
    x = x ^ (x >> np.uint64(16))
    x = (x * np.uint64(0x7FEB352D)) & M
    x = x ^ (x >> np.uint64(15))
    x = (x * np.uint64(0x846CA68B)) & M
    x = x ^ (x >> np.uint64(16))
    return x.astype(np.uint32)


def exp_variate_log2_np(x) -> np.ndarray:
    """Exponential variate in log2 units from a hash: ``V = (2 (x >> 9) + 1) 2^-24``,
    ``E = -log2(1 - V)`` (exact in float64 via log1p)."""
    v = (2.0 * (np.asarray(x, dtype=np.uint32) >> np.uint32(9)).astype(np.float64) + 1.0) * 2.0 ** -24
    return -np.log1p(-v) / math.log(2.0)


def sample_keys_np(z, temperature: float, seed: int) -> np.ndarray:
    """Per-column keys whose row argmax is the fused sampler's token.

    Greedy: the logits.  Sampling: ``u - log2(E)`` with ``u = z log2(e) / T`` and
    ``E`` the exponential variate of (seed, row, column) -- the Gumbel-max rule, whose
    argmax is distributed as ``softmax(z / T)`` (the distribution generate.py:75-77
    draws from).
    """
    z = np.asarray(z, dtype=np.float64)
    if temperature < GREEDY_TEMPERATURE:
        return z
    n, v = z.shape
    x = sample_hash_np(seed, np.arange(n), np.arange(v))
    return z * (math.log2(math.e) / temperature) - np.log2(exp_variate_log2_np(x))


def filtered_keys_np(z, temperature: float, seed: int, top_k: int = 0, top_p: float = 1.0) -> np.ndarray:
    """Gumbel-max keys of the fused filtered sampler: ``sample_keys_np`` on the entries that
    top-k / top-p keep, ``-inf`` elsewhere; the row argmax is a draw from
    ``filtered_probs_np``."""
    keys = sample_keys_np(z, temperature, seed)
    _, kept = filtered_probs_np(z, temperature, top_k, top_p)
    return np.where(kept, keys, -np.inf)


def lm_head_sample_np(h, W, temperature: float = 0.0, seed: int = 0):
    """``sample_token(h @ W^T, temperature)`` as the fused op defines it, in float64.

    Returns ``(tokens, logit, lse, keys)``: the chosen column per row (first index
    among equal keys), its logit, ``log sum exp(z / T')`` with ``T' = T`` when sampling
    and ``1`` when greedy, and the key matrix (for tolerance checks on near-ties).
    """
    z = np.asarray(h, dtype=np.float64) @ np.asarray(W, dtype=np.float64).T
    keys = sample_keys_np(z, temperature, seed)
    tokens = np.argmax(keys, axis=-1)
    inv = 1.0 if temperature < GREEDY_TEMPERATURE else 1.0 / temperature
    lse = _lse(z * inv)
    return tokens, z[np.arange(z.shape[0]), tokens], lse, keys


def sample_token_torch(logits, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0):
    """The reference's ``sample_token`` op sequence (generate.py:40-78) in torch, any device.

    Used as the comparison arm of the sampling benchmark (cuBLAS logits, then these
    ops) and nowhere in the product.
    """
    torch = _torch()
    F = torch.nn.functional
    if temperature < GREEDY_TEMPERATURE:
        return logits.argmax(dim=-1), None
    scaled = logits / temperature
    if top_k > 0:
        v, _ = torch.topk(scaled, min(top_k, scaled.size(-1)), dim=-1)
        scaled[scaled < v[..., [-1]]] = -float("inf")
    if top_p < 1.0:
        sorted_logits, sorted_idx = torch.sort(scaled, descending=True, dim=-1)
        cum = torch.cumsum(F.softmax(sorted_logits, dim=-1), dim=-1)
        remove = cum > top_p
        remove[..., 1:] = remove[..., :-1].clone()
        remove[..., 0] = 0
        scaled[remove.scatter(-1, sorted_idx, remove)] = -float("inf")
    probs = F.softmax(scaled, dim=-1)
    tokens = torch.multinomial(probs.view(-1, probs.size(-1)), 1).view(probs.shape[:-1])
    return tokens, probs


# --------------------------------------------------------------------------
# Final RMSNorm of pre-norm rows (reference model.py:493; transformers LlamaRMSNorm)
# --------------------------------------------------------------------------

def _bf16_round_np(a):
    """Round float32 values to the nearest bf16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def rmsnorm_np(x, gamma, eps: float = 1e-5, bf16_input: bool = True, r=None):
    """``LlamaRMSNorm`` (transformers, as ``model.py:493`` uses it) row by row.

    ``r = 1 / sqrt(mean(x^2) + eps)`` in fp32 (float64 sum, rounded); bf16 input:
    ``y = bf16(gamma * bf16(x r))`` -- the cast back to the input dtype, then the bf16
    weight product; fp32 input: ``y = gamma * (x r)`` in fp32.  Returns ``(y, r)`` as
    float32 arrays.  ``r`` may be given (e.g. a device's, whose fp32 sum of squares runs
    in another order) to check the rest bit for bit.
    """
    x32 = np.asarray(x, dtype=np.float32)
    g32 = np.asarray(gamma, dtype=np.float32)
    if r is None:
        var = np.float32(np.mean(x32.astype(np.float64) ** 2, axis=-1))
        r = (np.float32(1.0) / np.sqrt(var + np.float32(eps), dtype=np.float32)).astype(np.float32)
    r = np.asarray(r, dtype=np.float32)
    t = x32 * r[:, None]
    if bf16_input:
        return _bf16_round_np(g32[None, :] * _bf16_round_np(t)), r
    return (g32[None, :] * t).astype(np.float32), r


def rmsnorm_backward_np(x, gamma, r, dy):
    """Gradient through the norm in float64 (roundings pass the gradient unchanged):
    ``dx = r gamma dy - (r^3 / H) x sum(gamma dy x)``."""
    x = np.asarray(x, dtype=np.float64)
    g = np.asarray(gamma, dtype=np.float64)[None, :]
    r = np.asarray(r, dtype=np.float64)[:, None]
    dy = np.asarray(dy, dtype=np.float64)
    s = (g * dy * x).sum(axis=-1, keepdims=True)
    return r * g * dy - (r ** 3 / x.shape[-1]) * x * s


def prenorm_kl_loss_np(x_s, x_t, gamma, W, mask, temperature: float = 1.0, eps: float = 1e-5):
    """The loss on pre-norm rows in float64: norm both views (fp32 semantics), the fused
    loss's math on the normed rows, and the gradient of the pre-norm student rows."""
    ys, rs = rmsnorm_np(x_s, gamma, eps, bf16_input=False)
    yt, _ = rmsnorm_np(x_t, gamma, eps, bf16_input=False)
    loss, dh, _, _, _, _ = aligned_kl_loss_np(ys, yt, W, mask, temperature)
    return loss, rmsnorm_backward_np(x_s, gamma, rs, dh)


# --------------------------------------------------------------------------
# Block-diffusion attention (reference model.py:45-96, 435-446; flex_attention semantics)
# --------------------------------------------------------------------------

def block_attention_np(q, k_self, v_self, k_ar, v_ar, limits, K: int, scale: Optional[float] = None):
    """float64 restatement.  Query position p of block p // K attends to AR keys
    ``0..limits[b, p]`` (clipped to the cache; below 0: none) and to the K keys of its own
    block; GQA head h reads KV head ``h // (H / Hkv)``; scores scaled by ``scale``
    (default ``1/sqrt(D)``).  Returns ``(out [B, H, Ld, D], lse [B, H, Ld])``, lse in
    natural log."""
    q = np.asarray(q, np.float64)
    ks, vs = np.asarray(k_self, np.float64), np.asarray(v_self, np.float64)
    ka, va = np.asarray(k_ar, np.float64), np.asarray(v_ar, np.float64)
    lim = np.asarray(limits)
    B, H, Ld, D = q.shape
    Hkv, AL = ks.shape[1], ka.shape[2]
    ng = H // Hkv
    sc = 1.0 / math.sqrt(D) if scale is None else scale
    out = np.zeros((B, H, Ld, D))
    lse = np.zeros((B, H, Ld))
    ar_idx = np.arange(AL)
    for b in range(B):
        for h in range(H):
            hk = h // ng
            for blk in range(Ld // K):
                rows = slice(blk * K, (blk + 1) * K)
                qq = q[b, h, rows]                                   # [K, D]
                s_ar = qq @ ka[b, hk].T * sc                         # [K, AL]
                s_self = qq @ ks[b, hk, rows].T * sc                 # [K, K]
                vis = ar_idx[None, :] <= np.clip(lim[b, rows], -1, AL - 1)[:, None]
                s_ar = np.where(vis, s_ar, -np.inf)
                s = np.concatenate([s_ar, s_self], axis=1)
                m = s.max(axis=1, keepdims=True)
                e = np.exp(s - m)
                z = e.sum(axis=1, keepdims=True)
                vv = np.concatenate([va[b, hk], vs[b, hk, rows]], axis=0)
                out[b, h, rows] = (e / z) @ vv
                lse[b, h, rows] = (m + np.log(z))[:, 0]
    return out, lse


def block_attention_bwd_np(q, k_self, v_self, k_ar, v_ar, limits, K: int, d_out, scale: Optional[float] = None):
    """float64 closed-form backward of ``block_attention_np`` for an upstream gradient
    ``d_out [B, H, Ld, D]``: ``(dq [B, H, Ld, D], dk_self, dv_self [B, Hkv, Ld, D])``.

    Per query block, with P the attention probabilities over [AR keys | own block keys],
    V the matching values and O = P V:  dV = P^T dO,  dP = dO V^T,  dS = P (dP - rowsum(dO O)),
    dQ = scale dS K,  dK = scale dS^T Q; the self keys' dK / dV sum over the query heads that
    share the KV head (GQA).  The AR cache gets no gradient (it comes from the frozen
    backbone: the reference's Triton backward, triton_kernels.py:73-141 and 161-172, returns
    None for it as well).
    """
    q = np.asarray(q, np.float64)
    ks, vs = np.asarray(k_self, np.float64), np.asarray(v_self, np.float64)
    ka, va = np.asarray(k_ar, np.float64), np.asarray(v_ar, np.float64)
    do = np.asarray(d_out, np.float64)
    lim = np.asarray(limits)
    B, H, Ld, D = q.shape
    Hkv, AL = ks.shape[1], ka.shape[2]
    ng = H // Hkv
    sc = 1.0 / math.sqrt(D) if scale is None else scale
    dq = np.zeros_like(q)
    dks = np.zeros_like(ks)
    dvs = np.zeros_like(vs)
    ar_idx = np.arange(AL)
    for b in range(B):
        for h in range(H):
            hk = h // ng
            for blk in range(Ld // K):
                rows = slice(blk * K, (blk + 1) * K)
                qq = q[b, h, rows]
                kk = np.concatenate([ka[b, hk], ks[b, hk, rows]], axis=0)
                vv = np.concatenate([va[b, hk], vs[b, hk, rows]], axis=0)
                s = qq @ kk.T * sc
                vis = np.concatenate([ar_idx[None, :] <= np.clip(lim[b, rows], -1, AL - 1)[:, None],
                                      np.ones((K, K), bool)], axis=1)
                s = np.where(vis, s, -np.inf)
                e = np.exp(s - s.max(axis=1, keepdims=True))
                p = e / e.sum(axis=1, keepdims=True)
                o = p @ vv
                g = do[b, h, rows]
                dv = p.T @ g
                dp = g @ vv.T
                ds = p * (dp - (g * o).sum(axis=1, keepdims=True))
                dq[b, h, rows] = sc * ds @ kk
                dk = sc * ds.T @ qq
                dks[b, hk, rows] += dk[AL:]
                dvs[b, hk, rows] += dv[AL:]
    return dq, dks, dvs
