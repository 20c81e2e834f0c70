"""Loading of the golden fixtures in ``tests/golden`` (made by make_golden.py).

A fixture stores the reference's outputs and the recipe of its inputs (seed,
shapes, edits) with a SHA-256 of the input bytes; ``load`` regenerates the
inputs and refuses to return them if the digest differs.
"""

import ast
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

from make_golden import apply_edits, input_digest  # noqa: E402
from gdn_b200.synthetic import make_inputs, make_pool_indices  # noqa: E402

NAMES = ["decode_qk4v8_b1", "decode_qk4v8_b2_edge", "decode_h16hv32_b1", "mtp_qk4v8_b1_t3",
         "pooled_qk4v8_p5_b3", "mtp_prefill_qk4v8_b2_t4", "prefill_qk4v8_ragged",
         "prefill_qk4v8_ragged_nostate"]


def bf16_from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def load(name: str):
    """(meta, inputs, arrays) of fixture ``name``; bf16 arrays come back as bf16 tensors."""
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    meta = ast.literal_eval(str(z["meta"]))
    inp = make_inputs(B=meta["B"], T=meta["T"], H=meta["H"], HV=meta["HV"], seed=meta["seed"],
                      slots=meta.get("slots", meta.get("num_seqs")))
    if "edits" in meta:
        inp = apply_edits(inp, meta["edits"])
    digest = input_digest(inp)
    if digest != meta["sha256"]:
        raise AssertionError(f"{name}: regenerated inputs differ from the fixture's ({digest})")
    arrays = {}
    for key in z.files:
        if key == "meta":
            continue
        a = z[key]
        arrays[key] = bf16_from_bits(a) if a.dtype == np.uint16 else torch.from_numpy(a)
    if "slots" in meta:
        inp.state_indices = make_pool_indices(meta["B"], meta["slots"], seed=meta["seed"], n_pad=1)
        assert torch.equal(inp.state_indices, arrays["indices"].to(torch.int32))
    return meta, inp, arrays
