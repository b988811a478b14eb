"""Both kernel families on the same problems: the GQA-packed forward / dQ kernels (the default
for narrow windows) and the per-head kernels (every other shape, or everywhere with
SWA_FWD_PER_HEAD=1).  A child process with the switch set runs the per-head path; both must
match the fp64 oracle, and each other, at the usual tolerance."""
import json
import os
import subprocess
import sys

import pytest
import torch

from oracle import swa_oracle as orc

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CASES = [  # (B, Hq, Hkv, L, D, W, S, dtype)
    (2, 16, 2, 1000, 64, 128, 4, "bfloat16"),
    (1, 8, 2, 333, 32, 50, 3, "float16"),
    (1, 16, 4, 300, 16, 20, 0, "bfloat16"),
]

CHILD = r"""
import json, sys, torch
sys.path.insert(0, sys.argv[1])
import importlib
pkg = importlib.import_module("flashattention-gpt-oss-finetuning_b200")
B, Hq, Hkv, L, D, W, S, dt = json.loads(sys.argv[2])
dt = getattr(torch, dt)
g = torch.Generator().manual_seed(11)
q, do = (torch.randn(B, Hq, L, D, generator=g).to(dt) for _ in range(2))
k, v = (torch.randn(B, Hkv, L, D, generator=g).to(dt) for _ in range(2))
dev = torch.device("cuda:0")
qd, kd, vd = (t.to(dev).requires_grad_() for t in (q, k, v))
o = pkg.flash_swda_with_sink(qd, kd, vd, W, S)
o.backward(do.to(dev))
torch.save([t.detach().cpu() for t in (o, qd.grad, kd.grad, vd.grad)], sys.argv[3])
"""


def _run(case, per_head, path):
    env = dict(os.environ)
    if per_head:
        env["SWA_FWD_PER_HEAD"] = "1"
    else:
        env.pop("SWA_FWD_PER_HEAD", None)
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT, json.dumps(case), path], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return torch.load(path)


@pytest.mark.parametrize("case", CASES, ids=[f"D{c[4]}W{c[5]}S{c[6]}G{c[1] // c[2]}" for c in CASES])
def test_packed_and_per_head_paths_agree_with_the_oracle(case, tmp_path):
    B, Hq, Hkv, L, D, W, S, dt = case
    tol = 1.5e-2 if dt == "bfloat16" else 2e-3
    packed = _run(case, False, str(tmp_path / "packed.pt"))
    per_head = _run(case, True, str(tmp_path / "per_head.pt"))
    g = torch.Generator().manual_seed(11)
    dtype = getattr(torch, dt)
    q, do = (torch.randn(B, Hq, L, D, generator=g).to(dtype) for _ in range(2))
    k, v = (torch.randn(B, Hkv, L, D, generator=g).to(dtype) for _ in range(2))
    ref = orc.backward(q.float(), k.float(), v.float(), do.float(), W, S)
    for name, a, b, r in zip(("o", "dq", "dk", "dv"), packed, per_head, ref):
        den = r.abs().max().item()
        assert (a.double() - r).abs().max().item() / den <= tol, ("packed", name)
        assert (b.double() - r).abs().max().item() / den <= tol, ("per-head", name)
