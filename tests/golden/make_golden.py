"""Generate the golden fixtures of the GDN decode path from the reference itself.

Runs the reference's own ``kernel_pt_reference`` (solution/triton/kernel.py:22-118)
and ``kernel_prefill_reference`` (solution/triton/prefill_kernel.py:85-183) on the
CPU, on seeded inputs from ``gdn_b200.synthetic.make_inputs``, and stores their
outputs as ``tests/golden/*.npz``.  Inputs are not stored: each fixture records
the seed, the shape arguments, any edits applied after the draw, and a SHA-256
of the input bytes so the tests can regenerate them and prove they are the
same.

The reference checkout is needed only here (``--reference``, default
``$GDN_REFERENCE_ROOT``, else the default checkout location below); the fixtures are
self-contained.  Importing ``solution.triton.kernel`` pulls
``flashinfer.gdn_decode``, which needs a GPU at import time, so a stub module
with the one imported name is installed first; the stubbed function is the
FlashInfer baseline, which no fixture calls.

The reference asserts 4 q/k heads and 8 v-heads (kernel.py:63-67); the 16/32-head
fixture calls it once per head group g (q/k heads [4g, 4g+4), v-heads [8g, 8g+8))
and concatenates, which is exact because v-head hv reads q/k head hv // 2 in both.

Usage:  python tests/golden/make_golden.py [--reference PATH]
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "flashinfer-competition-codebase_b200"))

from gdn_b200.synthetic import make_inputs, make_pool_indices  # noqa: E402

# Edits applied to fixture "decode_qk4v8_b2_edge" after the draw: they reach the
# softplus threshold branch (a + dt_bias > 20), saturated gates, the largest
# A_log of the distribution and the scale=0 default.
EDGE_EDITS = {
    "a": [((0, 0, 0), 30.0), ((1, 0, 3), -30.0), ((0, 0, 6), 19.5)],
    "b": [((0, 0, 1), 15.0), ((1, 0, 2), -15.0)],
    "A_log": [((5,), 1.0), ((2,), -2.0)],
    "scale": 0.0,
}


def apply_edits(inp, edits):
    if edits.get("l2norm_qk"):
        # unit-norm q and k (in fp32, rounded back to bf16), as a model's q/k producer
        # makes them: keeps multi-token states bounded, so the comparison measures the
        # algorithm rather than fp32 rounding amplified by |1 - beta*|k|^2| per token
        for name in ("q", "k"):
            x = getattr(inp, name).float()
            setattr(inp, name, (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16))
    for name in ("a", "b", "A_log"):
        t = getattr(inp, name)
        for pos, val in edits.get(name, []):
            t[pos] = val
    if "scale" in edits:
        inp.scale = edits["scale"]
    return inp


def input_digest(inp) -> str:
    h = hashlib.sha256()
    for t in (inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b):
        t = t.contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        h.update(t.numpy().tobytes())
    h.update(repr(float(inp.scale)).encode())
    return h.hexdigest()


def load_reference(root: str):
    stub = types.ModuleType("flashinfer.gdn_decode")

    def _unavailable(*args, **kwargs):
        raise RuntimeError("FlashInfer's GPU decode is stubbed while generating fixtures")

    stub.gated_delta_rule_decode_pretranspose = _unavailable
    sys.modules["flashinfer.gdn_decode"] = stub
    sys.path.insert(0, root)
    from solution.triton.kernel import kernel_pt_reference
    from solution.triton.prefill_kernel import kernel_prefill_reference
    return kernel_pt_reference, kernel_prefill_reference


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def ref_grouped(ref, q, k, v, state, A_log, a, dt_bias, b, scale):
    """Reference on 16/32 heads, one 4/8-head group at a time."""
    H, HV = q.shape[2], v.shape[2]
    outs, states = [], []
    for g in range(H // 4):
        qs, vs = slice(4 * g, 4 * g + 4), slice(8 * g, 8 * g + 8)
        o, s = ref(q[:, :, qs], k[:, :, qs], v[:, :, vs], state[:, vs], A_log[vs], a[:, :, vs],
                   dt_bias[vs], b[:, :, vs], scale)
        outs.append(o)
        states.append(s)
    return torch.cat(outs, dim=2), torch.cat(states, dim=1)


def save(name, meta, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, meta=np.array(repr(meta)), **arrays)
    print(f"wrote {path} ({os.path.getsize(path) / 1e6:.2f} MB)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GDN_REFERENCE_ROOT"),
                    help="reference checkout (default: $GDN_REFERENCE_ROOT)")
    ap.add_argument("--only", default=None, help="comma-separated fixture names to (re)make")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference PATH or set GDN_REFERENCE_ROOT")
    ref, prefill_ref = load_reference(args.reference)
    torch.manual_seed(0)
    only = None if args.only is None else set(args.only.split(","))

    def want(name):
        return only is None or name in only

    # 1. The contest definition's shape (4 q/k heads, 8 v-heads), B=1.
    if want("decode_qk4v8_b1"):
        meta = dict(B=1, T=1, H=4, HV=8, seed=0)
        inp = make_inputs(B=1, H=4, HV=8, seed=0)
        o, s = ref(*inp.args())
        save("decode_qk4v8_b1", dict(meta, sha256=input_digest(inp)), output=bf16_bits(o),
             new_state=s.numpy())

    # 2. Gate edge cases and scale=0, B=2.
    if want("decode_qk4v8_b2_edge"):
        meta = dict(B=2, T=1, H=4, HV=8, seed=1, edits=EDGE_EDITS)
        inp = apply_edits(make_inputs(B=2, H=4, HV=8, seed=1), EDGE_EDITS)
        o, s = ref(*inp.args())
        save("decode_qk4v8_b2_edge", dict(meta, sha256=input_digest(inp)), output=bf16_bits(o),
             new_state=s.numpy())

    # 3. Qwen3-Next heads (16 q/k, 32 v), B=1, via head groups.
    if want("decode_h16hv32_b1"):
        meta = dict(B=1, T=1, H=16, HV=32, seed=0)
        inp = make_inputs(B=1, H=16, HV=32, seed=0)
        o, s = ref_grouped(ref, *inp.args())
        save("decode_h16hv32_b1", dict(meta, sha256=input_digest(inp)), output=bf16_bits(o),
             new_state=s.numpy())

    # 4. Multi-token, T=3: the decode reference applied token by token (which gives
    #    the intermediate states), checked against the prefill reference's
    #    sequential loop on the same tokens.
    if want("mtp_qk4v8_b1_t3"):
        B, T = 1, 3
        meta = dict(B=B, T=T, H=4, HV=8, seed=2)
        inp = make_inputs(B=B, T=T, H=4, HV=8, seed=2)
        S = inp.state.clone()
        outs, inters = [], []
        for t in range(T):
            sl = slice(t, t + 1)
            o, S = ref(inp.q[:, sl], inp.k[:, sl], inp.v[:, sl], S, inp.A_log, inp.a[:, sl],
                       inp.dt_bias, inp.b[:, sl], inp.scale)
            outs.append(o)
            inters.append(S.clone())
        out_loop = torch.cat(outs, dim=1)                      # [B,T,HV,V]
        inter = torch.stack(inters, dim=1)                     # [B,T,HV,V,K]
        cu = torch.arange(0, (B + 1) * T, T, dtype=torch.int32)
        flat = lambda x: x.reshape(B * T, *x.shape[2:])        # noqa: E731
        o_p, s_p = prefill_ref(flat(inp.q), flat(inp.k), flat(inp.v), inp.state, inp.A_log,
                               flat(inp.a), inp.dt_bias, flat(inp.b), cu, inp.scale)
        torch.testing.assert_close(o_p.reshape(B, T, *o_p.shape[1:]).float(), out_loop.float(),
                                   rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(s_p, inter[:, -1], rtol=1e-4, atol=1e-4)
        save("mtp_qk4v8_b1_t3", dict(meta, sha256=input_digest(inp)), output=bf16_bits(out_loop),
             intermediates=inter.numpy(), prefill_output=bf16_bits(o_p),
             prefill_state=s_p.numpy())

    # 5. Pooled state: 5 slots, 3 entries, one padded with -1.  The reference is
    #    run on the gathered active slots; untouched slots keep their values.
    if want("pooled_qk4v8_p5_b3"):
        meta = dict(B=3, T=1, H=4, HV=8, seed=3, slots=5)
        inp = make_inputs(B=3, H=4, HV=8, seed=3, slots=5)
        idx = make_pool_indices(3, 5, seed=3, n_pad=1)
        act = [i for i in range(3) if int(idx[i]) >= 0]
        sel = torch.tensor(act)
        slots = idx[sel].long()
        o, s = ref(inp.q[sel], inp.k[sel], inp.v[sel], inp.state[slots], inp.A_log, inp.a[sel],
                   inp.dt_bias, inp.b[sel], inp.scale)
        out = torch.zeros(3, 1, 8, 128, dtype=torch.bfloat16)
        out[sel] = o
        save("pooled_qk4v8_p5_b3", dict(meta, sha256=input_digest(inp)), output=bf16_bits(out),
             indices=idx.numpy(), slot_states=s.numpy(), slots=slots.numpy())

    # 6. Multi-token through the reference's own varlen prefill loop: two sequences of
    #    4 tokens (cu_seqlens [0, 4, 8]), final states and every token's output.
    if want("mtp_prefill_qk4v8_b2_t4"):
        B, T = 2, 4
        meta = dict(B=B, T=T, H=4, HV=8, seed=4)
        inp = make_inputs(B=B, T=T, H=4, HV=8, seed=4)
        cu = torch.tensor([0, T, 2 * T], dtype=torch.int32)
        flat = lambda x: x.reshape(B * T, *x.shape[2:])    # noqa: E731
        o_p, s_p = prefill_ref(flat(inp.q), flat(inp.k), flat(inp.v), inp.state, inp.A_log,
                               flat(inp.a), inp.dt_bias, flat(inp.b), cu, inp.scale)
        save("mtp_prefill_qk4v8_b2_t4", dict(meta, sha256=input_digest(inp)),
             output=bf16_bits(o_p.reshape(B, T, *o_p.shape[1:])), new_state=s_p.numpy())

    # 7. Variable-length prefill through the reference's varlen loop on ragged
    #    sequences: lengths 6, 0, 7, 7 (cu_seqlens [0, 6, 6, 13, 20]) — an empty
    #    sequence among them — from a given initial state, and the same tokens from
    #    no initial state (the reference's state=None, zeros).  q and k are unit-norm.
    for name, with_state in (("prefill_qk4v8_ragged", True),
                             ("prefill_qk4v8_ragged_nostate", False)):
        if not want(name):
            continue
        cu_list = [0, 6, 6, 13, 20]
        edits = {"l2norm_qk": True}
        meta = dict(B=1, T=cu_list[-1], H=4, HV=8, seed=5, num_seqs=len(cu_list) - 1,
                    cu_seqlens=cu_list, initial_state=with_state, edits=edits)
        inp = apply_edits(make_inputs(B=1, T=cu_list[-1], H=4, HV=8, seed=5,
                                      slots=len(cu_list) - 1), edits)
        cu = torch.tensor(cu_list, dtype=torch.int32)
        o_p, s_p = prefill_ref(inp.q[0], inp.k[0], inp.v[0], inp.state if with_state else None,
                               inp.A_log, inp.a[0], inp.dt_bias, inp.b[0], cu, inp.scale)
        save(name, dict(meta, sha256=input_digest(inp)), output=bf16_bits(o_p),
             new_state=s_p.numpy())


if __name__ == "__main__":
    main()
