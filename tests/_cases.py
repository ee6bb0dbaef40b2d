"""Golden-case loading and oracle dispatch shared by the test modules."""

from __future__ import annotations

import glob
import json
import os

import numpy as np

import ref_loops as R  # oracle/ref_loops.py (conftest puts oracle/ on sys.path)

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

ARGS = {
    "ssd": ("u", "delta", "B", "C", "A_neg"),
    "gla": ("q", "k", "v", "gates"),
    "rglru": ("a", "x"),
    "rotlru": ("a", "cs", "sn", "x"),
}


def parity_files():
    return sorted(glob.glob(os.path.join(GOLDEN, "*parity*.npz")))


def load(path):
    z = np.load(path)
    meta = json.loads(str(z["__meta__"]))
    case = {k: z[k] for k in z.files if k != "__meta__"}
    case["meta"] = meta
    return case


def inputs_of(case):
    names = case["meta"].get("arg_names") or ARGS[case["meta"]["kind"]]
    return [case["in_" + n] for n in names], list(names)


def oracle_fwd(kind, ins):
    return getattr(R, f"{kind}_forward")(*ins)


def oracle_bwd(kind, ins, gy, g_final=None):
    return getattr(R, f"{kind}_backward")(*ins, gy, g_final)


rel_err = R.rel_err
