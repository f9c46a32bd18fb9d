"""Load the committed golden vectors written by ``tests/golden/make_golden.py``."""

from __future__ import annotations

import ast
import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def case_names(kind: str):
    names = []
    for p in sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))):
        with np.load(p) as z:
            meta = ast.literal_eval(str(z["meta"]))
        if meta["kind"] == kind:
            names.append(os.path.splitext(os.path.basename(p))[0])
    return names


def _bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def load_case(name: str):
    """Returns (meta, tensors) with every array decoded to float32 numpy and a
    set ``bf16`` naming the arrays that were bf16 in the reference run."""
    with np.load(os.path.join(GOLDEN_DIR, name + ".npz")) as z:
        meta = ast.literal_eval(str(z["meta"]))
        out, bf16 = {}, set()
        for k in z.files:
            if k == "meta":
                continue
            a = z[k]
            if a.dtype == np.uint16:
                out[k] = _bf16_bits_to_f32(a)
                bf16.add(k)
            else:
                out[k] = a.astype(np.float32)
    return meta, out, bf16
