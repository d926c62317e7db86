"""Helpers to read the golden fixtures (tests/golden/*.npz)."""
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    f = np.load(os.path.join(GOLDEN, name))
    out = {}
    for k in f.files:
        a = f[k]
        out[k] = torch.from_numpy(a) if a.ndim > 0 else float(a)
    return out


MHA_CASES = ["check_s4.npz", "ref_b1h2s40d8.npz", "ref_b2h2s64d16_t500k.npz",
             "config1_b1h4s256d64.npz"]
