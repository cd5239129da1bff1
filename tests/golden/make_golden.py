"""Generates tests/golden/*.npz from the REFERENCE's own eager functions.

Run here (where the reference checkout is readable), not on the GPU box:

    python tests/golden/make_golden.py --reference /path/to/dory-vllm-experiments

For every case of specs.py it rebuilds the seeded inputs and evaluates them with
chrisbennight/dory-vllm-experiments' own PyTorch code:

* normalize_rows (kernels/bench_decode_attention.py:100-101) and the expected raw-mode q,
  k, v (:112-115),
* reference_attention (kernels/bench_decode_attention.py:58-68), the FP32 oracle the
  reference checks its kernel against,
* to_nibble_major (kernels/w4a16_gemv.py:91-93),

with the reference's appending order: the token's k/v go into the cache at its slot before
it attends; shared-cache wavefront tokens are run as single-token steps in position order
(kernels/bench_multi_token.py:160-197).  Each .npz stores the expected gated output
(nibble-major FP32), the expected appended k/v (bf16 bit patterns) and a digest of the
inputs so the tests can confirm they regenerated the same inputs.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path
from types import SimpleNamespace

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
    parser.add_argument("--only", default=None)
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "kernels"))
    from bench_decode_attention import normalize_rows, reference_attention  # reference code
    from w4a16_gemv import to_nibble_major  # reference code
    import bench_decode_attention as ref_bench

    for name, build in specs.specs().items():
        if args.only and name != args.only:
            continue
        case = build()
        NH, NKV, HD, B = case.num_heads, case.num_kv_heads, case.head_dim, case.block_size
        if B != ref_bench.CACHE_BLOCK:
            raise SystemExit(f"{name}: the reference oracle is written for block size 16")
        key = case.key.to(torch.bfloat16)
        value = case.value.to(torch.bfloat16)
        T = case.tokens
        q_exp, k_exp, v_exp = [], [], []
        for t in range(T):
            qk, v = case.qk[t], case.v[t]
            q_exp.append(((case.sqk.float() * case.sqk_factor).square().view(NH, HD)
                          * normalize_rows(qk[:NH * HD].view(NH, HD))).to(torch.bfloat16)
                         .view(-1))
            k_exp.append(normalize_rows(qk[NH * HD:].view(NKV, HD)).to(torch.bfloat16))
            v_exp.append(v.view(NKV, HD).to(torch.bfloat16))
        outs = []
        order = sorted(range(T), key=lambda t: case.seq_lens[t])
        results = {}
        for t in order:
            n = case.seq_lens[t]
            table = case.tables[case.table_rows[t]]
            if n > 0:
                pos = n - 1
                phys = int(table[pos // B])
                key[phys, pos % B] = k_exp[t]
                value[phys, pos % B] = v_exp[t]
            cache = SimpleNamespace(key=key, value=value, block_table=table)
            if n > 0:
                att = reference_attention(q_exp[t], cache, n, case.window, NH, case.scale)
            else:
                att = torch.zeros(NH * HD)
            results[t] = to_nibble_major(att * case.gate[t])
        outs = torch.stack([results[t] for t in range(T)])
        np.savez_compressed(
            HERE / f"{name}.npz",
            out=outs.numpy().astype(np.float32),
            k_new=torch.stack(k_exp).view(torch.int16).numpy(),
            v_new=torch.stack(v_exp).view(torch.int16).numpy(),
            q_bf16=torch.stack(q_exp).view(torch.int16).numpy(),
            seq_lens=np.asarray(case.seq_lens, dtype=np.int64),
            slots=np.asarray([case.slot(t) for t in range(T)], dtype=np.int64),
            digest=np.asarray(specs.digest(case)))
        print(f"{name}: T={T} seq_lens={case.seq_lens[:8]} window={case.window}", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
