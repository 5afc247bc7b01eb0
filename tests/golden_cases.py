"""Loader for the golden fixtures in ``tests/golden`` (made by ``make_golden.py``)."""
from __future__ import annotations

import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")

_cache = {}


def load():
    if "npz" not in _cache:
        _cache["npz"] = dict(np.load(os.path.join(GOLDEN, "cases.npz")))
        with open(os.path.join(GOLDEN, "cases.json")) as f:
            _cache["meta"] = json.load(f)
    return _cache["npz"], _cache["meta"]


def names():
    """Matmul (SlicedData x SlicedData) cases."""
    return [k for k, v in load()[1].items() if "xs" in v]


def layer_names():
    """LinearMem / Conv2dMem cases."""
    return [k for k, v in load()[1].items() if "kind" in v]


def layer_case(name):
    arrs, meta = load()
    spec = meta[name]
    g = {k.split("/", 1)[1]: v for k, v in arrs.items() if k.startswith(name + "/")}
    eng = dict(NOISE_FREE)
    eng.update(spec["eng"])
    return dict(spec=spec, eng=eng, golden=g)


NOISE_FREE = dict(write_variation=0.0, read_variation=0.0, vnoise=0.0, rate_stuck_HGS=0.0, rate_stuck_LGS=0.0)


def case(name):
    """Return dict with x, w (fp32 numpy), spec, engine kwargs and golden arrays."""
    arrs, meta = load()
    spec = meta[name]
    g = {k.split("/", 1)[1]: v for k, v in arrs.items() if k.startswith(name + "/")}
    if "x" in g:
        x, w = g["x"], g["w"]
    else:
        torch.manual_seed(spec["seed"])
        x = torch.randn(*spec["xs"]).numpy()
        w = torch.randn(*spec["ws"]).numpy()
        assert abs(float(x.astype(np.float64).sum()) - g["x_sum"][0]) < 1e-6
        assert abs(float(w.astype(np.float64).sum()) - g["x_sum"][1]) < 1e-6
    eng = dict(NOISE_FREE)
    eng.update(spec["eng"])
    fields = {}
    shape = tuple(int(v) for v in g["G_shape"])
    if eng.get("rate_stuck_HGS", 0) > 0 or eng.get("rate_stuck_LGS", 0) > 0:
        fields["stuck"] = torch.rand(shape, generator=torch.Generator().manual_seed(123)).numpy()
        assert abs(float(fields["stuck"].astype(np.float64).sum()) - g["stuck_field_sum"][0]) < 1e-3
    if eng.get("write_variation", 0) > 0:
        fields["write"] = torch.normal(0, eng["write_variation"], shape,
                                       generator=torch.Generator().manual_seed(42)).numpy()
        assert abs(float(fields["write"].astype(np.float64).sum()) - g["write_field_sum"][0]) < 1e-3
    xq = spec["xq"] if isinstance(spec["xq"], str) else tuple(spec["xq"])
    wq = spec["wq"] if isinstance(spec["wq"], str) else tuple(spec["wq"])
    return dict(x=x, w=w, spec=spec, eng=eng, golden=g, fields=fields,
                xp=tuple(spec["xp"]), xq=xq, wp=tuple(spec["wp"]), wq=wq)


def packed_to_rows(packed: np.ndarray, batched: bool) -> np.ndarray:
    """Reference tile layout (..., nr, nc, p0, p1) of packed codes -> (B, rows_p, cols_p)."""
    if not batched:
        packed = packed[None]
    B, nr, nc, p0, p1 = packed.shape
    return packed.transpose(0, 1, 3, 2, 4).reshape(B, nr * p0, nc * p1).astype(np.int64)


def noise_stats():
    with open(os.path.join(GOLDEN, "noise_stats.json")) as f:
        return json.load(f)
