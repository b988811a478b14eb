"""The C ABI from a plain C program (tests/c_abi/abi_caller.c), the way a non-Python host binds
it: compiled with gcc against include/swa_attn.h, linked to lib/libswa_attn.so and the CUDA
runtime, no torch in the process.  The host-only checks run without a GPU; the GPU case runs
swa_fwd + swa_bwd on device buffers the C program allocates and is checked against the
oracle."""
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

from oracle import swa_oracle as orc
from tests._pkg import pkg

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def caller(tmp_path_factory):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    lib_dir = os.path.dirname(pkg().lib_path())
    exe = str(tmp_path_factory.mktemp("cabi") / "abi_caller")
    cmd = [gcc, "-std=c99", "-O1", "-I", os.path.join(ROOT, "include"), "-I",
           os.path.join(CUDA, "include"), os.path.join(HERE, "c_abi", "abi_caller.c"), "-o", exe,
           "-L", lib_dir, "-lswa_attn", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_c_caller_host_entry_points(caller):
    r = subprocess.run([caller, "host"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert "host ok" in r.stdout


@pytest.mark.gpu
def test_c_caller_forward_backward_matches_oracle(caller, tmp_path):
    b, hq, hkv, l, d, w, s = 1, 4, 2, 200, 64, 50, 3
    g = torch.Generator().manual_seed(17)
    q, do = (torch.randn(b, hq, l, d, generator=g).half() for _ in range(2))
    k, v = (torch.randn(b, hkv, l, d, generator=g).half() for _ in range(2))
    src, dst = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(src, "wb") as f:
        for t in (q, k, v, do):
            f.write(t.numpy().tobytes())
    r = subprocess.run([caller, "gpu", str(src), str(dst)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    raw = np.fromfile(dst, dtype=np.float16)
    nq, nk = q.numel(), k.numel()
    parts = np.split(raw, [nq, 2 * nq, 2 * nq + nk])
    ours = [torch.from_numpy(x.copy()).double().reshape(t.shape)
            for x, t in zip(parts, (q, q, k, v))]
    ref = orc.backward(q.float(), k.float(), v.float(), do.float(), w, s, 0.125)
    for name, x, r_ in zip(("o", "dq", "dk", "dv"), ours, ref):
        err = (x - r_).abs().max().item() / r_.abs().max().item()
        assert err <= 2e-3, (name, err)
