"""Generates tests/golden/qkvg_*.npz from the REFERENCE's own q/k/v/gate epilogue.

Run here (where the reference checkout is readable), not on the GPU box:

    TRITON_INTERPRET=1 python tests/golden/make_golden_qkvg.py --reference /path/to/dory-vllm-experiments

For every case of specs.qkvg_specs() it rebuilds the seeded inputs and runs
chrisbennight/dory-vllm-experiments' `_qkvg_epilogue_kernel`
(kernels/dory_multi_token.py:53-80) on the CPU through Triton's interpreter (the kernel is
FP32 loads, sums, products and a sigmoid: no dot products or bf16 casts, which the
interpreter does not reproduce).  Stored: qk, v, gate and the digest of the inputs.
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


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True,
                        help="checkout of chrisbennight/dory-vllm-experiments (read only)")
    args = parser.parse_args()
    if os.environ.get("TRITON_INTERPRET") != "1":
        raise SystemExit("set TRITON_INTERPRET=1 (the reference kernel runs on the CPU)")
    sys.path.insert(0, str(Path(args.reference) / "kernels"))
    from dory_multi_token import _qkvg_epilogue_kernel  # reference code

    for name, build in specs.qkvg_specs().items():
        case = build()
        NH, NKV, HD = case.num_heads, case.num_kv_heads, case.head_dim
        Q, KV, T = NH * HD, NKV * HD, case.tokens
        split_k, rows = case.partials.shape[0], case.partials.shape[2]
        qk = torch.zeros(T, Q + KV)
        v = torch.zeros(T, KV)
        gate = torch.zeros(T, Q)
        _qkvg_epilogue_kernel[(rows // HD, T)](
            case.partials, case.positions, case.cos_sin, case.s_gate, qk, v, gate,
            case.s_gate_factor, Q_ROWS=Q, KV_ROWS=KV, HEAD_DIM=HD, SPLIT_K=split_k, T=T,
            num_warps=4)
        np.savez_compressed(HERE / f"{name}.npz", qk=qk.numpy(), v=v.numpy(), gate=gate.numpy(),
                            digest=np.array(specs.qkvg_digest(case)))
        print(f"{name}: T={T} split_k={split_k} {NH}q/{NKV}kv x {HD}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
