"""The pass-2 dZ kernels against the oracle on the same problems.

The library runs the interleaved-view kernel (both views' rows alternating along the MMA's M
side, read through one tensor map over both tensors: in 8-row groups when N % 8 == 0, else row
by row); KLG_DZT=1 selects the transposed kernel (vocabulary on the MMA's M side, writing
dZ^T), KLG_DZI=0 the row-major dual-view kernel, KLG_DZI=2 makes the interleaved kernel's
tensor map a requirement (an error, not a fallback), and KLG_DZI=3 keeps the row-by-row
interleave where the 8-row-group one would apply.  The choice is
read once per process, so each variant runs in a child process.  Problems:
ragged N and V (vocabulary chunks that are not multiples of the 256-row pair tile), H = 576
(resident W in the transposed kernel), 1024 and 2048 (streamed W), T = 2 with a peaky
teacher and masked rows, N both a multiple of 8 and not (the two interleaved layouts), a
backward chunk of 384 columns, both views in one buffer with the teacher at the lower address
(the interleaved map's view order reversed), an upstream gradient of 0 (the loss is unchanged,
the gradients vanish), and the same tensor passed as both views (KL and gradients exactly 0;
the interleaved kernel steps aside).  Tolerances
as every GPU parity test: loss 1e-3 relative, gradients 2e-2 normalised max error and
cosine >= 0.9999.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

CHILD = r'''
import sys, torch
sys.path.insert(0, sys.argv[1])
from tests.gpu_helpers import assert_close, run_ours, run_oracle_np

def problem(N, H, V, T=1.0, p=0.5, seed=0, tscale=1.0):
    g = torch.Generator().manual_seed(seed)
    h_s = torch.randn(N, H, generator=g)
    h_t = torch.randn(N, H, generator=g) * tscale
    W = torch.randn(V, H, generator=g) * 0.02
    mask = torch.rand(N, generator=g) < p
    mask[0] = True
    return h_s, h_t, W, mask, T

cases = [(333, 576, 1000, {}), (336, 576, 1000, {"T": 2.0, "tscale": 4.0, "p": 0.3}),
         (129, 1024, 1237, {"T": 2.0, "tscale": 4.0, "p": 0.3}), (136, 1024, 1237, {"seed": 3}),
         (300, 2048, 777, {}), (304, 2048, 777, {"seed": 4}), (517, 576, 3000, {"seed": 5}),
         (512, 576, 3000, {"seed": 6, "p": 0.05})]
for N, H, V, kw in cases:
    h_s, h_t, W, mask, T = problem(N, H, V, **kw)
    loss, dh, dw, *_ = run_oracle_np(h_s, h_t, W, mask, T)
    for path in ("split", "fused"):
        assert_close(run_ours(h_s, h_t, W, mask, T, path=path), loss, dh, dw, f"N{N} H{H} V{V} {path}")
# a 384-column backward chunk: vocabulary tiles straddle chunk ends
h_s, h_t, W, mask, T = problem(200, 576, 1500, seed=9)
loss, dh, dw, *_ = run_oracle_np(h_s, h_t, W, mask, T)
assert_close(run_ours(h_s, h_t, W, mask, T, workspace_bytes=4096 + 200 * 384 * 2), loss, dh, dw, "384-column chunks")

from orthrus_training_test_b200 import ops
from tests.gpu_helpers import GRAD_COS, GRAD_MAX_REL, LOSS_RTOL
from oracle import klgemm_oracle as O
dev = torch.device("cuda:0")
# teacher rows at the lower address: one [2, N, H] buffer holding (h_t, h_s)
for n in (259, 264):
    h_s, h_t, W, mask, T = problem(n, 576, 1111, seed=11)
    loss, dh, dw, *_ = run_oracle_np(h_s, h_t, W, mask, T)
    buf = torch.stack([h_t, h_s]).to(torch.bfloat16).to(dev)
    out = ops.kl_fwd_bwd(buf[1], buf[0], W.to(torch.bfloat16).to(dev), mask.to(dev), T, need_dh=True, need_dw=True)
    torch.cuda.synchronize()
    assert abs(float(out[0]) - loss) <= LOSS_RTOL * abs(loss), (n, float(out[0]), loss)
    for name, ours, ref in (("dh", out[4], dh), ("dw", out[5], dw)):
        mr, cos = O.grad_metrics(ours.double().cpu().numpy(), ref)
        assert mr <= GRAD_MAX_REL and cos >= GRAD_COS, (n, name, mr, cos)
# upstream gradient 0: the loss is still the full loss, the gradients are exactly 0
for n in (259, 264):
    h_s, h_t, W, mask, T = problem(n, 576, 1111, seed=12)
    loss, *_ = run_oracle_np(h_s, h_t, W, mask, T)
    bf = lambda x: x.to(torch.bfloat16).to(dev)
    out = ops.kl_fwd_bwd(bf(h_s), bf(h_t), bf(W), mask.to(dev), T, grad=torch.zeros(1, device=dev))
    torch.cuda.synchronize()
    assert abs(float(out[0]) - loss) <= LOSS_RTOL * abs(loss), ("grad 0", n, float(out[0]), loss)
    assert not out[4].any() and not out[5].any()
# the same tensor as both views: KL = 0 and zero gradients, exactly
x = h_s.to(torch.bfloat16).to(dev)
out = ops.kl_fwd_bwd(x, x, W.to(torch.bfloat16).to(dev), mask.to(dev), T, need_dh=True, need_dw=True)
torch.cuda.synchronize()
assert float(out[0]) == 0.0 and not out[4].any() and not out[5].any(), float(out[0])
print("ok")
'''


@pytest.mark.parametrize("dzt,dzi", [("0", "0"), ("0", "2"), ("0", "3"), ("1", "1")],
                         ids=["row-major", "interleaved", "interleaved-rows", "transposed"])
def test_dz_kernel_variant_matches_oracle(dzt, dzi):
    env = dict(os.environ, KLG_DZT=dzt, KLG_DZI=dzi)
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, cwd=str(ROOT), capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-3000:] + r.stderr[-3000:]
