"""A small, fixed decode case for profiler captures (ncu) of the decode kernel.

    python -m gdn_b200.profile_case --batch 128 --launches 3 [--T 1] [--pooled] [--bf16-state]

Runs ``--launches`` decode steps of the Qwen3-Next shapes (16 q/k heads, 32
v-heads, K = V = 128) at the given batch on cuda:0 and exits.  Batch 128
holds 256 MiB of state: more than the 126 MB L2, so DRAM counters are
meaningful, and far below the sizes that make captures slow.
"""

from __future__ import annotations

import argparse

import torch

import gdn_b200
from gdn_b200 import synthetic


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--T", type=int, default=1)
    ap.add_argument("--pooled", action="store_true", help="pool of 4*batch slots, one -1 index")
    ap.add_argument("--lanes-per-row", type=int, default=0)
    ap.add_argument("--rows-per-lane", type=int, default=0)
    ap.add_argument("--warps-per-cta", type=int, default=0)
    ap.add_argument("--bf16-state", action="store_true", help="bf16-stored state variant")
    args = ap.parse_args()
    dev = torch.device("cuda:0")
    B, T = args.batch, args.T
    slots = 4 * B if args.pooled else B
    inp = synthetic.make_inputs(B=B, T=T, slots=slots, seed=0, device=dev)
    idx = synthetic.make_pool_indices(B, slots, seed=0, n_pad=1, device=dev) if args.pooled else None
    out = torch.empty((B, T, 32, 128), dtype=torch.bfloat16, device=dev)
    if args.bf16_state:
        inp.state = inp.state.to(torch.bfloat16)
        for _ in range(args.launches):
            gdn_b200.decode_bf16_state(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a,
                                       inp.dt_bias, inp.b, inp.scale, out, state_indices=idx)
        torch.cuda.synchronize(dev)
        print(f"profile_case ok: B={B} T={T} pooled={args.pooled} bf16 state "
              f"launches={args.launches}")
        return
    for _ in range(args.launches):
        gdn_b200.decode_tuned(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias,
                              inp.b, inp.scale, out, state_indices=idx,
                              lanes_per_row=args.lanes_per_row, rows_per_lane=args.rows_per_lane,
                              warps_per_cta=args.warps_per_cta)
    torch.cuda.synchronize(dev)
    print(f"profile_case ok: B={B} T={T} pooled={args.pooled} launches={args.launches}")


if __name__ == "__main__":
    main()
