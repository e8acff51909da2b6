"""Helpers that rebuild the golden cases' inputs and load their reference outputs."""
import json
import os

import numpy as np
import torch

from project_chronos_b200 import synthetic as syn

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cases():
    with open(os.path.join(GOLDEN, "cases.json")) as f:
        return json.load(f)["cases"]


def case(name):
    for c in cases():
        if c["name"] == name:
            return c
    raise KeyError(name)


def load(c):
    d = np.load(os.path.join(GOLDEN, f"{c['name']}.npz"))
    return {k: d[k] for k in d.files}


def inputs(c, device="cpu"):
    """The case's workload, generated on the CPU (as the fixtures were)."""
    shape = syn.MoEShape(c["H"], c["E"], c["k"], c["F"], c["S"], c["norm"])
    dt = torch.bfloat16 if c["dtype"] == "bf16" else torch.float32
    wl = syn.make_workload(shape, c["B"] * c["T"], seed=c["seed"], dtype=dt,
                           avail_p=c["avail_p"])
    if device != "cpu":
        wl = syn.Workload(wl.shape, wl.weights.to(device=device), wl.x.to(device),
                          wl.mask, wl.bias)
    return wl


def effective_avail(c):
    """a_e the reference applies in the case's mode (moe_chronos.py:220-227)."""
    if c["mode"] == "eval":
        return np.array(c["mask"], dtype=np.float32)
    if c["mode"] == "train_mask":
        return (np.array(c["float_mask"], dtype=np.float32) > 0).astype(np.float32)
    return None


def reference_y(c, d):
    return d["y_ref_fp32"] if "y_ref_fp32" in d else d["y_ref"]
