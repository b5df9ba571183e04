"""Checked accesses: token ids and targets outside the vocabulary are reported
through the device status record (always on), and the bounds-checked build
(`_C_kcheck`, -DEWB_KCHECK, loaded with EWB_KCHECK=1) runs the hot kernels at
real shapes without a false report.

The out-of-range cases stay inside allocated memory even if a check were
missing: the embedding table is a view of a larger tensor and the logits rows
have padding past V, so a wrong index would read a wrong value, not fault.

Would fail if a token id or a target outside [0, V) were read or written,
or went unreported, or if a bounds check fired on a valid launch.
"""

import os
import subprocess
import sys

import pytest
import torch

from elysium_wan_b200 import ops

pytestmark = pytest.mark.gpu

BAD_ARGUMENT, BOUNDS = 6, 8
SITE_TOKEN, SITE_TARGET = 1, 2


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    ops.ext().status_read_clear()
    return torch.device("cuda")


def _record():
    torch.cuda.synchronize()
    rec = list(ops.ext().status_record())
    ops.ext().status_read_clear()
    return rec


def test_token_outside_the_table_is_reported(cuda):
    V, S, d = 100, 64, 256
    big = torch.randn(V + 8, d, device=cuda)
    wte = big[:V]  # the rows past V exist, so a missed check reads, never faults
    wpe = torch.randn(S, d, device=cuda)
    idx = torch.randint(0, V, (1, S), device=cuda)
    idx[0, 5] = V + 3
    x = ops.embed_fwd(idx, wte, wpe, S)
    assert _record() == [BAD_ARGUMENT, SITE_TOKEN, 5, V + 3]
    torch.testing.assert_close(x[5].float(), (wte[0] + wpe[5]).to(torch.bfloat16).float())
    dwte, dwpe = torch.zeros(V + 8, d, device=cuda), torch.zeros(S, d, device=cuda)
    ops.embed_bwd(idx, torch.ones(S, d, device=cuda, dtype=torch.bfloat16), S, dwte[:V], dwpe)
    rec = _record()
    assert rec[:2] == [BAD_ARGUMENT, SITE_TOKEN] and rec[3] == V + 3
    assert torch.count_nonzero(dwte[V:]) == 0


def test_target_outside_the_vocabulary_is_reported(cuda):
    T, V = 32, 1000
    ld = V + 8  # padded rows: column V exists
    logits = torch.randn(T, ld, device=cuda)[:, :V]
    tgt = torch.randint(0, V, (T,), device=cuda)
    tgt[7] = V
    out = ops.cross_entropy(logits, V, tgt, 1.0 / T)
    loss = out[0] if isinstance(out, tuple) else out
    assert _record() == [BAD_ARGUMENT, SITE_TARGET, 7, V]
    assert torch.isnan(loss).any()
    h = torch.randn(T, 256, device=cuda).to(torch.bfloat16)
    w = (torch.randn(V, 256, device=cuda) * 0.05).to(torch.bfloat16)
    ops.head_ce(h, w, tgt, V, 1.0 / T)
    assert _record() == [BAD_ARGUMENT, SITE_TARGET, 7, V]


def test_bounds_checked_build_runs_the_hot_kernels_clean(cuda, tmp_path):
    prog = r"""
import torch
from elysium_wan_b200 import ops
assert ops.ext().KCHECK is True, "not the bounds-checked build"
torch.manual_seed(0)
dev = "cuda"
T, D, F, H = 512, 1024, 4096, 8
x = (torch.randn(T, D, device=dev)).to(torch.bfloat16)
w = (torch.randn(F, D, device=dev) * 0.02).to(torch.bfloat16)
y = ops.linear_fwd(x, w)
g = torch.zeros(F, D, device=dev)
ops.linear_dw(y, x, g, accumulate=False)
dx = ops.linear_dx(y, w)
qkv = torch.randn(T, 3 * D, device=dev).to(torch.bfloat16)
o, lse = ops.attention_fwd(qkv, 1, T, H, D // H)
ops.attention_bwd(qkv, o, torch.randn(T, D, device=dev).to(torch.bfloat16), lse, 1, T, H, D // H)
gam, bet = torch.ones(D, device=dev), torch.zeros(D, device=dev)
ops.layernorm_fwd(x, None, gam, bet)
torch.cuda.synchronize()
rec = list(ops.ext().status_record())
assert rec[0] == 0, rec
print("KCHECK_OK", ops.launch_count())
"""
    env = dict(os.environ, EWB_KCHECK="1")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", prog], cwd=root, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and "KCHECK_OK" in r.stdout, r.stdout + r.stderr
