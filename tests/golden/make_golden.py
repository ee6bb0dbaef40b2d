"""Generate golden vectors by running the reference's own Python code.

Run where a checkout of the reference is available (it is only read),
passing its root directory::

    python tests/golden/make_golden.py --ref <reference checkout>

MLX is not installable here, so ``tests/golden/_mlx_standin`` supplies a
torch-float64 stand-in for the ``mlx.core`` primitives. With it, this script
imports the reference package and its v2 test modules and executes:

* every ``parity_check`` call in ``tests/test_v2_{ssd,gla,rglru,rotlru}.py``
  (all parametrisations), with ``parity_check`` swapped for a recorder that
  restates ``_chassis.py:162-192``: ``y = reference_fn(*inputs)``,
  ``w_out`` drawn after ``mx.random.seed(1234)``, and ``mx.grad`` of
  ``sum(reference_fn(*inputs) * w_out)`` for every ``grad_argnums`` entry;
* the final-state tests' own hand loops (``test_v2_ssd.py:45-60``,
  ``test_v2_gla.py:40-53``, ``test_v2_rglru.py:39-51``) with the kernel call
  stubbed out, recording the loop's final state;
* the rotLRU property tests (``test_v2_rotlru.py:77-123``) with the kernel
  replaced by ``rotlru_scan_reference``, recording inputs and outputs.

Every array is stored as float32 (the reference's dtype) in one ``.npz`` per
case under ``tests/golden/``. Inputs come from torch's RNG, not MLX's, so the
values differ from the reference's runs; shapes, seeds and distributions
follow the reference's tests.
"""

from __future__ import annotations

import argparse
import ast
import importlib.util
import inspect
import json
import os
import sys
import textwrap

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_module(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _np(x):
    return np.asarray(x.detach().cpu().numpy(), dtype=np.float32)


def _save(name, arrays, meta):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, __meta__=np.array(json.dumps(meta)), **arrays)
    print(f"wrote {path}: {sorted(arrays)}")


class _Recorder:
    """Stands in for ``parity_check``; records the reference's outputs."""

    def __init__(self, mx, prefix):
        self.mx = mx
        self.prefix = prefix
        self.cases = []

    def __call__(self, kernel_fn, reference_fn, inputs, arg_names, grad_argnums,
                 *, w_out=None, y_tol=1e-3, grad_rtol=1e-3, label="", verbose=True):
        mx = self.mx
        inputs = list(inputs)
        y_r = reference_fn(*inputs)
        if w_out is None:
            mx.random.seed(1234)
            w_out = mx.random.normal(y_r.shape)

        def loss_ref(*args):
            return mx.sum(reference_fn(*args) * w_out)

        g_r = mx.grad(loss_ref, argnums=grad_argnums)(*inputs)
        if not isinstance(g_r, (tuple, list)):
            g_r = (g_r,)
        arrays = {f"in_{n}": _np(x) for n, x in zip(arg_names, inputs)}
        arrays["w_out"] = _np(w_out)
        arrays["y"] = _np(y_r)
        for i, g in zip(grad_argnums, g_r):
            arrays[f"grad_{arg_names[i]}"] = _np(g)
        self.cases.append((label, list(arg_names), arrays))
        return True, {}


def _params(test_fn):
    for mark in getattr(test_fn, "pytestmark", []):
        if mark.name == "parametrize":
            names = [s.strip() for s in mark.args[0].split(",")]
            return names, list(mark.args[1])
    return None, [()]


def _exec_body(fn, ns, drop_if_mentions=()):
    """Execute a test function's body in ``ns`` without its asserts."""
    tree = ast.parse(textwrap.dedent(inspect.getsource(fn))).body[0]
    body = [s for s in tree.body if not isinstance(s, ast.Assert)
            and not any(w in ast.unparse(s) for w in drop_if_mentions)]
    exec(compile(ast.Module(body=body, type_ignores=[]), f"<{fn.__name__}>", "exec"), ns)
    return ns


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root directory of the reference checkout")
    args = ap.parse_args()

    sys.path.insert(0, os.path.join(HERE, "_mlx_standin"))
    sys.path.insert(1, args.ref)
    import mlx.core as mx  # the stand-in
    import mlx_recurrence as mr  # the reference package

    src_version = mr.__version__
    tests = {k: _load_module(os.path.join(args.ref, "tests", f"test_v2_{k}.py"), f"ref_test_v2_{k}")
             for k in ("ssd", "gla", "rglru", "rotlru")}

    # ---- parity tests: every parametrisation of every parity_check caller ----
    for kind, mod in tests.items():
        for tname, fn in sorted(vars(mod).items()):
            if not (tname.startswith("test_") and callable(fn)):
                continue
            if "parity_check" not in inspect.getsource(fn):
                continue
            names, plist = _params(fn)
            for pi, p in enumerate(plist):
                rec = _Recorder(mx, kind)
                mod.parity_check = rec
                kwargs = dict(zip(names, p)) if names else {}
                fn(**kwargs)
                for label, argn, arrays in rec.cases:
                    meta = {"kind": kind, "test": f"tests/test_v2_{kind}.py::{tname}",
                            "params": kwargs, "label": label, "arg_names": argn,
                            "reference_version": src_version,
                            "loss": "sum(y * w_out), w_out ~ seed 1234 (_chassis.py:166-188)"}
                    _save(f"{kind}_{tname[5:]}_{pi}", arrays, meta)

    # ---- final-state hand loops ----
    finals = {
        "ssd": ("test_ssd_final_state", "ssd_scan_with_state", ["u", "delta", "B_in", "C_in", "A_neg"]),
        "gla": ("test_gla_final_state", "gla_scan_with_state", ["q", "k", "v", "gates"]),
        "rglru": ("test_rglru_final_state", "rglru_scan_with_state", ["a", "x"]),
    }
    for kind, (tname, kname, argn) in finals.items():
        mod = tests[kind]
        ns = dict(vars(mod))
        ns[kname] = lambda *a, **k: (None, None)
        _exec_body(getattr(mod, tname), ns, drop_if_mentions=("diff",))
        arrays = {f"in_{n}": _np(ns[n]) for n in argn}
        arrays["final"] = _np(ns["h"])
        meta = {"kind": kind, "test": f"tests/test_v2_{kind}.py::{tname}", "arg_names": argn,
                "seg": ns.get("seg"), "reference_version": src_version}
        _save(f"{kind}_final_state", arrays, meta)

    # ---- widened cases that reach the tensor-core kernels ----
    # The reference's own input makers (test_v2_ssd.py:15-23, test_v2_gla.py:11-18) at
    # the shape the chunked kernels take (L=256, Dh=64, N=128). SSD gets one decay rate
    # per head: the first column of the drawn A_neg, broadcast over N. The inputs are
    # rounded to bf16 (A_neg stays float32), so a bf16 run reads exactly these values;
    # y and the gradients come from the reference's pure loops through the recorder.
    import torch
    from mlx_recurrence.ssd import ssd_scan_reference
    from mlx_recurrence.gla import gla_scan_reference

    def _bf16(x):
        return x.float().to(torch.bfloat16).double()

    # The SSD case twice: with one rate per head, and with the reference's own dense
    # A_neg [H, N] as its input maker draws it (the general contract, ssd.py:62, 96).
    wide = [
        ("ssd", "tc", ssd_scan_reference, ["u", "delta", "B", "C", "A_neg"], dict(B=2, L=256, H=2, Dh=64, N=128, seed=4)),
        ("ssd", "tc_dense", ssd_scan_reference, ["u", "delta", "B", "C", "A_neg"],
         dict(B=2, L=256, H=2, Dh=64, N=128, seed=5)),
        ("gla", "tc", gla_scan_reference, ["q", "k", "v", "gates"], dict(B=2, L=256, H=2, Dh=64, seed=4)),
    ]
    for kind, tag, ref_fn, argn, p in wide:
        ins = list(tests[kind]._make_inputs(**p))
        if kind == "ssd":
            if tag == "tc":
                A = ins[4]
                ins[4] = A[:, :1].expand(A.shape).contiguous()
            ins[:4] = [_bf16(x) for x in ins[:4]]
        else:
            ins = [_bf16(x) for x in ins]
        rec = _Recorder(mx, kind)
        rec(None, ref_fn, ins, argn, tuple(range(len(argn))), label=f"{kind} widened {p}")
        for label, names, arrays in rec.cases:
            a_desc = "one rate per head" if tag == "tc" else "dense [H, N] as drawn"
            meta = {"kind": kind, "test": f"tests/test_v2_{kind}.py::_make_inputs (widened)",
                    "params": {**p, "seg": 32}, "label": label, "arg_names": names,
                    "inputs": f"rounded to bf16 (A_neg float32, {a_desc})" if kind == "ssd" else "rounded to bf16",
                    "reference_version": src_version,
                    "loss": "sum(y * w_out), w_out ~ seed 1234 (_chassis.py:166-188)"}
            _save(f"{kind}_{tag}_parity_widened", arrays, meta)

    # ---- rotLRU properties, run with the reference loop in place of the kernel ----
    rmod = tests["rotlru"]
    from mlx_recurrence.rotlru import rotlru_scan_reference

    def _ref_with_state(a, cs, sn, x, seg=32):
        y = rotlru_scan_reference(a, cs, sn, x)
        return y, y[:, -1, :]

    for tname, outs in (("test_theta_zero_reduces_to_rglru", ("y_rot", "y_rglru")),
                        ("test_pure_rotation_preserves_norm", ("y", "norms")),
                        ("test_with_state_matches_last_step", ("y", "final"))):
        ns = dict(vars(rmod))
        ns["rotlru_scan"] = lambda a, cs, sn, x, seg=32: rotlru_scan_reference(a, cs, sn, x)
        ns["rotlru_scan_with_state"] = _ref_with_state
        _exec_body(getattr(rmod, tname), ns)
        arrays = {f"in_{n}": _np(ns[n]) for n in ("a", "cs", "sn", "x")}
        for o in outs:
            arrays[o] = _np(ns[o])
        meta = {"kind": "rotlru", "test": f"tests/test_v2_rotlru.py::{tname}",
                "reference_version": src_version, "kernel": "rotlru_scan_reference"}
        _save(f"rotlru_{tname[5:]}", arrays, meta)


if __name__ == "__main__":
    main()
