"""The allocation-free MVM entry point (mib_mvm_static_scratch), called through the C ABI.

Some callers cannot allocate device memory while they run; for them the split-K
scratch of the MVM lives in an array compiled into the library.  This checks, on
two calls in a row, that its result equals the allocating entry point's.  It sits
in its own file, collected last, so a failure here comes after every other test.
"""
import numpy as np
import pytest
import torch

import golden_cases as G
from helpers import gpu_pair, rel_norm

pytestmark = pytest.mark.gpu


def _call_static(eng, xs, ws, out):
    from memintelli_flash_b200 import _native as N
    gx, gw = xs._buf["geom"], ws._buf["geom"]
    M, Nc = gx["batch"] * gx["rows"], gw["n"]
    xspec, wspec, kg, dspec = xs._spec(), ws._spec(), xs._kgeom(), eng._device_spec()
    _, table, tlen = eng._plan(xspec, wspec, kg, dspec, out.device)
    layout = N.OutLayout(M, 0, Nc, 1)
    N.call("mib_mvm_static_scratch", N.ptr(xs._buf["planes"]), N.ptr(xs._buf["tile_scale"]), M, xspec,
           N.ptr(ws._buf["planes"]), N.ptr(ws._buf["tile_scale"]), Nc, wspec, kg, dspec, xs._buf["kind"],
           N.ptr(table), tlen, N.ptr(out), layout, None, N.stream_ptr(out.device))


@pytest.mark.parametrize("name", ["cfg0_int", "cfg0_fp"])
def test_static_scratch_matches_allocating_entry(name, cuda):
    from memintelli_flash_b200 import _native as N
    c = G.case(name)
    eng, xs, ws = gpu_pair(c, cuda)
    gx = xs._buf["geom"]
    M, Nc = gx["batch"] * gx["rows"], ws._buf["geom"]["n"]
    need = N.c_i64(0)
    N.call("mib_mvm_workspace", M, Nc, xs._spec(), ws._spec(), xs._kgeom(), eng._device_spec(), need)
    assert need.value > 0                      # this shape uses split-K, i.e. the scratch
    y_ref = eng(xs, ws)
    for _ in range(2):                         # two calls in a row share the built-in scratch
        out = torch.full((M, Nc), float("nan"), device=cuda)
        _call_static(eng, xs, ws, out)
        torch.cuda.synchronize()
        a, b = out.double().cpu().numpy(), y_ref.double().cpu().numpy()
        assert np.isfinite(a).all()
        assert rel_norm(a, b) <= 1e-6
    N.device_status()
