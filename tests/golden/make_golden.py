"""Generate the golden attention fixtures in this folder from the reference itself.

Run in a container that has the reference checkout (read-only) at REF_ROOT:

    python tests/golden/make_golden.py [REF_ROOT]

The reference's own Triton kernels (flash_attn_volta/triton_fa.py and
flash_attn_volta/triton_fa_bwd.py) are executed on the CPU through Triton's
interpreter (TRITON_INTERPRET=1), and its fp32 eager oracle
(flash_attn_volta/ref.py:attention_ref) is run beside them.  The autotuner
needs a GPU, so each autotuned kernel is replaced by a launcher that calls the
underlying jitted function with the first config of its own autotune list
(BLOCK_M=BLOCK_N=BLOCK_D=64, triton_fa.py:44-56, triton_fa_bwd.py:46-66).

The wrappers `flash_attn_forward` / `flash_attn_backward` assert `is_cuda`
(triton_fa.py:313, triton_fa_bwd.py:609), so this script calls the inner
`_run_kernel` / `_run_bwd_kernels` and applies the D<64 zero padding the same
way the wrappers do (triton_fa.py:323-336, triton_fa_bwd.py:620-631).

Inputs are drawn from a seeded CPU torch.Generator in the order q, k, v, dO,
as fp16.  One .npz per case holds the inputs and:
  o_ref, lse_ref, dq_ref, dk_ref, dv_ref   reference Triton kernels (fp16 / fp32 lse)
  o_eager                                  ref.py attention_ref in fp32
The fixtures are read by tests/test_oracle.py and tests/test_parity_gpu.py;
nothing in the product reads them.
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, S, H, D, causal, input scale, seed)
CASES = [
    ("c1_tiny_d64_nc", 1, 64, 2, 64, False, 1.0, 11),
    ("c1_tiny_d64_c", 1, 64, 2, 64, True, 1.0, 12),
    ("s128_d64_c", 1, 128, 2, 64, True, 1.0, 13),
    ("s96_d128_nc", 1, 96, 2, 128, False, 1.0, 14),
    ("s160_d128_c", 1, 160, 1, 128, True, 0.5, 15),
    ("s100_d32_c", 2, 100, 2, 32, True, 1.0, 16),
    ("s72_d32_nc", 1, 72, 3, 32, False, 1.0, 17),
    ("s48_d16_c", 1, 48, 2, 16, True, 1.0, 18),
]


def _install_interpreter_launchers(F, Bw):
    meta = {"BLOCK_M": 64, "BLOCK_N": 64, "BLOCK_D": 64}

    class _Launch:
        def __init__(self, autotuned):
            self.fn = autotuned.fn

        def __getitem__(self, grid):
            g = grid(meta) if callable(grid) else grid

            def run(*args, **kw):
                kw = dict(kw)
                kw.update(meta)
                return self.fn[g](*args, **kw)
            return run

    for mod, names in ((F, ["_fa_fwd_kernel_d64", "_fa_fwd_kernel_d128"]),
                       (Bw, ["_fa_bwd_dq_kernel_d64", "_fa_bwd_dq_kernel_d128",
                             "_fa_bwd_dkdv_kernel_d64", "_fa_bwd_dkdv_kernel_d128"])):
        for n in names:
            setattr(mod, n, _Launch(getattr(mod, n)))


def main(ref_root: str) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch
    import flash_attn_volta.triton_fa as F
    import flash_attn_volta.triton_fa_bwd as Bw
    from flash_attn_volta.ref import attention_ref

    _install_interpreter_launchers(F, Bw)

    def pad64(t):
        B, N, H, D = t.shape
        if D >= 64:
            return t
        tp = torch.zeros((B, N, H, 64), dtype=t.dtype)
        tp[..., :D] = t
        return tp

    for name, B, S, H, D, causal, amp, seed in CASES:
        g = torch.Generator().manual_seed(seed)
        shape = (B, S, H, D)
        q, k, v, do = [(torch.randn(shape, generator=g) * amp).to(torch.float16)
                       for _ in range(4)]
        scale = 1.0 / math.sqrt(D)
        Dint = max(D, 64)
        qp, kp, vp, dop = pad64(q), pad64(k), pad64(v), pad64(do)
        o_p, lse = F._run_kernel(qp, kp, vp, causal, scale, Dint, write_lse=True)
        dq_p, dk_p, dv_p = Bw._run_bwd_kernels(dop, qp, kp, vp, o_p, lse, causal, scale, Dint)
        o = o_p[..., :D].contiguous()
        o_eager = attention_ref(q, k, v, causal=causal, sm_scale=scale, dtype_out=torch.float32)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            q=q.numpy(), k=k.numpy(), v=v.numpy(), do=do.numpy(),
            causal=np.array(causal), scale=np.array(scale, dtype=np.float64),
            o_ref=o.numpy(), lse_ref=lse.numpy(),
            dq_ref=dq_p[..., :D].contiguous().numpy(),
            dk_ref=dk_p[..., :D].contiguous().numpy(),
            dv_ref=dv_p[..., :D].contiguous().numpy(),
            o_eager=o_eager.numpy(),
        )
        print(f"{name}: B={B} S={S} H={H} D={D} causal={causal} "
              f"|o_ref-o_eager|={float((o.float()-o_eager).abs().max()):.2e}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
