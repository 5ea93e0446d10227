"""Loader for the fixtures under tests/golden (written by tests/golden/make_golden.py)."""
import glob
import json
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FN = ("x_seq", "state", "w_pos", "w_erev", "mu", "sigma", "sensory_mu", "sensory_sigma",
      "sensory_erev", "sensory_w_pos", "cm_t", "gleak_pos", "vleak")
DERIVED = ("mu", "sigma", "sensory_mu", "sensory_sigma", "sensory_erev", "vleak")


def case_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


class Case:
    def __init__(self, name):
        z = np.load(os.path.join(GOLDEN, name + ".npz"))
        self.meta = json.loads(bytes(z["meta"]).decode())
        self.a = {k: torch.from_numpy(z[k].copy()) for k in z.files if k != "meta"}
        self.name = name

    def group(self, prefix):
        n = len(prefix)
        return {k[n:]: v for k, v in self.a.items() if k.startswith(prefix)}

    @property
    def params(self):
        return self.group("p.")

    @property
    def module_grads(self):
        return self.group("gm.")

    @property
    def solver_inputs(self):
        f = self.group("f.")
        for k in DERIVED:
            f[k] = self.a["p." + k]
        return f

    @property
    def solver_grads(self):
        return self.group("gf.")

    def get(self, k, default=None):
        return self.a.get(k, default)
