"""Generate the golden fixtures in this directory from the reference project itself.

Run once, in a container where the reference checkout is available (it is never read at test
time and never travels to a GPU box):

    REFERENCE_DIR=<path to junhown3/FlashAttention-GPT-OSS-finetuning checkout> \
        python tests/golden/make_golden.py

For every case it draws seeded fp32 inputs, then records
  * the reference's naive attention ``pytorch_naive_attention``
    (benchmark_backward_speed.py:68-85) forward output and its autograd gradients, and
  * where it is well defined (L % 128 == 0; for other L the reference's backward returns NaN
    dK/dV because padded rows load M = -inf, flash_attention_gpt_oss.py:242, 270, 292), the
    reference's own entry point ``flash_swda_with_sink`` (flash_attention_gpt_oss.py:437)
    run under the Triton CPU interpreter (TRITON_INTERPRET=1).
The results go to ``golden_<name>.npz`` (fp32).  ``tests/test_oracle_golden.py`` pins the
oracle against them and the GPU parity tests compare the CUDA kernels against them.
"""
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")
sys.dont_write_bytecode = True

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (B, Hq, Hkv, L, D, W, S, seed)
CASES = {
    "survey_256": (1, 4, 2, 256, 16, 64, 4, 0),
    "full_causal": (1, 2, 1, 256, 32, 256, 0, 1),
    "ragged_gqa4": (1, 4, 1, 200, 64, 50, 7, 2),
    "window1": (2, 2, 2, 130, 16, 1, 3, 3),
    "big_window_sinks": (1, 8, 2, 128, 64, 1000, 16, 4),
    "sinks_past_window_d128": (1, 2, 2, 96, 128, 33, 70, 5),
    "sinks_only_w0": (1, 2, 1, 64, 16, 0, 5, 6),
    "single_row": (1, 2, 1, 1, 32, 16, 4, 7),
}


def main():
    ref = os.environ.get("REFERENCE_DIR")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("set REFERENCE_DIR to the reference checkout")
    sys.path.insert(0, ref)
    import benchmark_backward_speed as bbs  # noqa: E402
    import flash_attention_gpt_oss as fago  # noqa: E402

    for name, (b, hq, hkv, l, d, w, s, seed) in CASES.items():
        gen = torch.Generator().manual_seed(seed)
        q = torch.randn(b, hq, l, d, generator=gen)
        k = torch.randn(b, hkv, l, d, generator=gen)
        v = torch.randn(b, hkv, l, d, generator=gen)
        do = torch.randn(b, hq, l, d, generator=gen)

        qn, kn, vn = (t.clone().requires_grad_() for t in (q, k, v))
        on = bbs.pytorch_naive_attention(qn, kn, vn, w, s)
        on.backward(do)
        out = dict(
            q=q.numpy(), k=k.numpy(), v=v.numpy(), do=do.numpy(),
            shape=np.array([b, hq, hkv, l, d, w, s, seed], dtype=np.int64),
            naive_o=on.detach().numpy(), naive_dq=qn.grad.numpy(),
            naive_dk=kn.grad.numpy(), naive_dv=vn.grad.numpy(),
        )
        if l % 128 == 0:
            qt, kt, vt = (t.clone().requires_grad_() for t in (q, k, v))
            ot = fago.flash_swda_with_sink(qt, kt, vt, w, s)
            ot.backward(do)
            out.update(kernel_o=ot.detach().numpy(), kernel_dq=qt.grad.numpy(),
                       kernel_dk=kt.grad.numpy(), kernel_dv=vt.grad.numpy())
        path = os.path.join(HERE, f"golden_{name}.npz")
        np.savez_compressed(path, **out)
        print(name, "kernel" if "kernel_o" in out else "naive-only", os.path.getsize(path))


if __name__ == "__main__":
    main()
