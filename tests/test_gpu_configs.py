"""Parity at the benchmark configurations c0-c5, through the public API.

Each test builds the configuration's seeded inputs on the GPU exactly as
``bench.py`` does (``workloads.make_inputs``), runs ``*_scan_with_state``
forward and backward with a cotangent for ``y`` and one for the final state,
and compares ``y``, the final state and every gradient with the float64 oracle
on the same (rounded) inputs. Tolerances (``max|diff| / max|ref|``): 1e-5 for
float32 inputs (c0), 2e-2 for bf16 inputs.

The large configurations run in full on the GPU; the oracle checks a subset:
* c4 (SSD, B=32, L=16384, H=32, N=128), c4d (the same with a dense A_neg [H, N])
  and c5 (GLA, same shape): every one of
  the 1024 (batch row, head) units runs, the cotangents are nonzero only on
  four units (two heads of the first batch row, two of the last), so the
  oracle restates those units alone at full L (``grad_A`` of c4 per head, of
  c4d per head and column, then comes from them alone), and every other unit's gradients must be
  exactly zero (the units are independent).
* c3 (rotLRU, B=16): batch rows 0 and 15 at full L and width.
c0, c1 and c2 are checked in full.
"""

import importlib

import numpy as np
import pytest
import torch

import _cases as K
import ref_loops as R

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _W():
    return importlib.import_module("mlx-recurrence_b200.workloads")


def _np(t):
    return t.detach().double().cpu().numpy()


def _check(name, got, ref, tol):
    err = K.rel_err(got, ref)
    assert err < tol, f"{name}: {err:.3e} >= {tol:g}"
    return err


def _leaves(ins):
    """Differentiable leaves; SSD's per-head A (an expanded [H] view) becomes
    its [H] base re-expanded, as a model holding one rate per head would."""
    leaves, args = [], []
    for t in ins:
        if t.dim() == 2 and t.stride(1) == 0:
            base = t[:, 0].detach().clone().requires_grad_(True)
            leaves.append(base)
            args.append(base[:, None].expand(t.shape))
        else:
            x = t.detach().clone().requires_grad_(True)
            leaves.append(x)
            args.append(x)
    return leaves, args


def _run(fn, ins, gy, gf):
    leaves, args = _leaves(ins)
    y, fin = fn(*args)
    torch.autograd.backward([y, fin], [gy, gf])
    return y.detach(), fin.detach(), [x.grad for x in leaves]


def _f64_inputs(ins, sl=None):
    out = []
    for t in ins:
        if sl is not None and t.dim() >= 3:
            t = t[sl]
        out.append(t.detach().double().cpu().numpy())
    return out


# ---------------------------------------------------------------- c0, c1 ----

@pytest.mark.parametrize("name", ["c0", "c1"])
def test_small_config_in_full(mr, cuda_dev, name):
    W = _W()
    cfg = W.CONFIGS[name]
    ins = W.make_inputs(name, cuda_dev, seed=0)
    g = torch.Generator(device=cuda_dev).manual_seed(17)
    gy = torch.randn(W.output_shape(name), generator=g, device=cuda_dev)
    Bt, L, H, Dh = gy.shape
    fshape = (Bt, H, Dh, cfg["N"]) if cfg["kind"] == "ssd" else (Bt, H, Dh, Dh)
    gf = torch.randn(fshape, generator=g, device=cuda_dev)
    fn = getattr(mr, f"{cfg['kind']}_scan_with_state")
    y, fin, grads = _run(lambda *a: fn(*a, seg=cfg["seg"]), ins, gy, gf)
    tol = TOL[cfg["dtype"]]
    ref_in = _f64_inputs(ins)
    yo, fo = getattr(R, f"{cfg['kind']}_forward")(*ref_in)
    go = getattr(R, f"{cfg['kind']}_backward")(*ref_in, _np(gy), _np(gf))
    _check("y", _np(y), yo, tol)
    _check("final", _np(fin), fo, tol)
    names = K.ARGS[cfg["kind"]]
    for n, gk, gr in zip(names, grads, go):
        if cfg["kind"] == "ssd" and n == "A_neg":
            gr = gr.sum(axis=1)  # d loss / d (one rate per head)
        _check(f"grad_{n}", _np(gk), gr, tol)


# -------------------------------------------------------------------- c2 ----

def test_c2_rglru_in_full(mr, cuda_dev):
    W = _W()
    cfg = W.CONFIGS["c2"]
    ins = W.make_inputs("c2", cuda_dev, seed=0)
    g = torch.Generator(device=cuda_dev).manual_seed(19)
    gy = torch.randn(W.output_shape("c2"), generator=g, device=cuda_dev)
    gf = torch.randn((cfg["B"], cfg["D"]), generator=g, device=cuda_dev)
    y, fin, grads = _run(lambda *a: mr.rglru_scan_with_state(*a, seg=cfg["seg"]), ins, gy, gf)
    ref_in = _f64_inputs(ins)
    yo, fo = R.rglru_forward(*ref_in)
    go = R.rglru_backward(*ref_in, _np(gy), _np(gf))
    _check("y", _np(y), yo, 2e-2)
    _check("final", _np(fin), fo, 2e-2)
    for n, gk, gr in zip(("a", "x"), grads, go):
        _check(f"grad_{n}", _np(gk), gr, 2e-2)


# -------------------------------------------------------------------- c3 ----

def test_c3_rotlru_rows_at_full_length(mr, cuda_dev):
    W = _W()
    cfg = W.CONFIGS["c3"]
    ins = W.make_inputs("c3", cuda_dev, seed=0)
    g = torch.Generator(device=cuda_dev).manual_seed(23)
    gy = torch.randn(W.output_shape("c3"), generator=g, device=cuda_dev)
    gf = torch.randn((cfg["B"], 2 * cfg["Dp"]), generator=g, device=cuda_dev)
    y, fin, grads = _run(lambda *a: mr.rotlru_scan_with_state(*a, seg=cfg["seg"]), ins, gy, gf)
    rows = [0, cfg["B"] - 1]
    ref_in = _f64_inputs(ins, sl=rows)
    yo, fo = R.rotlru_forward(*ref_in)
    go = R.rotlru_backward(*ref_in, _np(gy[rows]), _np(gf[rows]))
    _check("y", _np(y[rows]), yo, 2e-2)
    _check("final", _np(fin[rows]), fo, 2e-2)
    for n, gk, gr in zip(("a", "cs", "sn", "x"), grads, go):
        _check(f"grad_{n}", _np(gk[rows]), gr, 2e-2)


# ---------------------------------------------------------------- c4, c5 ----

# (batch row, head range) units carrying the cotangents
_UNITS = lambda B, H: [(0, slice(0, 2)), (B - 1, slice(H - 2, H))]


@pytest.mark.parametrize("name", ["c4", "c4d", "c5"])
def test_large_config_units_at_full_length(mr, cuda_dev, name):
    W = _W()
    cfg = W.CONFIGS[name]
    kind = cfg["kind"]
    Bt, L, H, Dh = cfg["B"], cfg["L"], cfg["H"], cfg["Dh"]
    N = cfg["N"] if kind == "ssd" else Dh
    ins = W.make_inputs(name, cuda_dev, seed=0)
    units = _UNITS(Bt, H)
    g = torch.Generator(device=cuda_dev).manual_seed(29)
    gy = torch.zeros((Bt, L, H, Dh), device=cuda_dev)
    gf = torch.zeros((Bt, H, Dh, N), device=cuda_dev)
    mask = torch.zeros((Bt, H), dtype=torch.bool, device=cuda_dev)
    for b, hs in units:
        gy[b, :, hs] = torch.randn((L, hs.stop - hs.start, Dh), generator=g, device=cuda_dev)
        gf[b, hs] = torch.randn((hs.stop - hs.start, Dh, N), generator=g, device=cuda_dev)
        mask[b, hs] = True
    fn = getattr(mr, f"{kind}_scan_with_state")
    y, fin, grads = _run(lambda *a: fn(*a, seg=cfg["seg"]), ins, gy, gf)
    names = K.ARGS[kind]
    # units without a cotangent: exactly zero gradients
    for n, gk in zip(names, grads):
        if gk.dim() >= 3:
            other = gk.transpose(1, 2)[~mask] if gk.dim() == 4 else gk.permute(0, 2, 1)[~mask]
            assert float(other.abs().max()) == 0.0, f"grad_{n} nonzero outside the seeded units"
    dense = bool(cfg.get("dense_a"))
    gA_ref = (np.zeros((H, N)) if dense else np.zeros(H)) if kind == "ssd" else None
    for b, hs in units:
        sl = (slice(b, b + 1), slice(None), hs)
        ref_in = []
        for t in ins:
            if t.dim() == 2:  # A_neg [H, N]
                ref_in.append(t[hs].detach().double().cpu().numpy())
            else:
                ref_in.append(t[sl].detach().double().cpu().numpy())
        gy_u, gf_u = _np(gy[sl]), _np(gf[b:b + 1, hs])
        yo, fo = getattr(R, f"{kind}_forward")(*ref_in)
        go = getattr(R, f"{kind}_backward_segmented")(*ref_in, gy_u, gf_u)
        _check(f"y (b={b})", _np(y[sl]), yo, 2e-2)
        _check(f"final (b={b})", _np(fin[b:b + 1, hs]), fo, 2e-2)
        for n, gk, gr in zip(names, grads, go):
            if n == "A_neg":
                gA_ref[hs] += gr if dense else gr.sum(axis=1)
                continue
            _check(f"grad_{n} (b={b})", _np(gk[sl]), gr, 2e-2)
    if kind == "ssd":
        gA = _np(grads[4])
        heads = np.zeros(H, dtype=bool)
        for _, hs in units:
            heads[hs] = True
        assert np.all(gA[~heads] == 0.0)
        _check("grad_A (per head and column)" if dense else "grad_A (per head)", gA[heads], gA_ref[heads], 2e-2)
    del ins, grads, y, fin
    torch.cuda.empty_cache()
