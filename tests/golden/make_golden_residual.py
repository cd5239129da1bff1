"""Generates tests/golden/residual_*.npz from the REFERENCE's own residual kernels.

Run here (where the reference checkout is readable), not on the GPU box:

    TRITON_INTERPRET=1 python tests/golden/make_golden_residual.py --reference /path/to/dory-vllm-experiments

For every case of specs.residual_specs() it rebuilds the seeded inputs and runs
chrisbennight/dory-vllm-experiments' `_residual_tokens_kernel`
(kernels/dory_multi_token.py:109-131, launched as MultiTokenSublayers._residual does,
:173-181) or, for a case without an input x, `residual_update` (kernels/dory_common.py:71-81)
on the CPU through Triton's interpreter.  The kernels are FP32 sums, products and inverse
square roots, which the interpreter evaluates in FP32; their one BF16 store is not rounded
to nearest even by the interpreter, so the pinned output is the FP32 nibble-major copy
(h_nm) and the interpreter's BF16 copy is kept for reference only.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "dory-vllm-experiments_b200"))
sys.path.insert(0, str(HERE))

import specs  # noqa: E402

EPS = 1e-6  # kernels/dory_common.py:20


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True,
                        help="checkout of chrisbennight/dory-vllm-experiments (read only)")
    args = parser.parse_args()
    if os.environ.get("TRITON_INTERPRET") != "1":
        raise SystemExit("set TRITON_INTERPRET=1 (the reference kernels run on the CPU)")
    sys.path.insert(0, str(Path(args.reference) / "kernels"))
    import triton
    from dory_common import residual_update  # reference code
    from dory_multi_token import _residual_tokens_kernel  # reference code

    for name, build in specs.residual_specs().items():
        case = build()
        T, H = case.tokens, case.hidden
        h = torch.zeros(T, H, dtype=torch.bfloat16)
        h_nm = torch.zeros(T, 8, H // 8)
        if case.x is None:
            residual_update(case.a[0], case.partials[0, 0], case.alpha, case.alpha_scale, h[0],
                            h_nm[0])
        else:
            k_in = case.x.shape[1]
            _residual_tokens_kernel[(T,)](
                case.partials, case.x, case.a, case.alpha, h, h_nm, case.alpha_scale, EPS, H=H,
                K_IN=k_in, SPLIT_K=case.partials.shape[0], T=T,
                W_BLOCK=triton.next_power_of_2(H // 8), X_BLOCK=triton.next_power_of_2(k_in),
                num_warps=8)
        np.savez_compressed(HERE / f"{name}.npz", h_nm=h_nm.numpy(),
                            h_interp_bf16=h.view(torch.int16).numpy(),
                            digest=np.array(specs.residual_digest(case)))
        print(f"{name}: T={T} H={H} x={None if case.x is None else tuple(case.x.shape)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
