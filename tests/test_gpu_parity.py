"""Parity of the CUDA path against the oracle and the reference's golden outputs (needs a B200)."""
import numpy as np
import pytest
import torch

import golden_cases as G
from helpers import gpu_pair, oracle_pair, rel_norm
from oracle import cim_oracle as O

pytestmark = pytest.mark.gpu

DETERMINISTIC = [n for n in G.names() if n != "write_var"]


@pytest.mark.parametrize("name", G.names())
def test_slice_codes_bit_exact(name, cuda):
    """Packed slice codes, block maxima and exponents equal the reference's (data_formats.py:116-207)."""
    c = G.case(name)
    s = c["spec"]
    eng, xs, ws = gpu_pair(c, cuda, inference=False)
    g = c["golden"]
    batched = len(s["xs"]) == 3
    x_sl = xs.sliced_data.cpu().numpy()
    w_sl = ws.sliced_data.cpu().numpy()
    widths = [int(v) for v in s["sx"]][::-1]

    def pack(sl, widths):
        off, out = 0, np.zeros(sl.shape[:-3] + sl.shape[-2:], np.int64)
        for t, wd in enumerate(widths):
            out += sl[..., t, :, :].astype(np.int64) << off
            off += wd
        return out

    assert np.array_equal(pack(x_sl, widths), g["x_packed"].astype(np.int64))
    assert np.array_equal(pack(w_sl, [int(v) for v in s["sw"]][::-1]), g["w_packed"].astype(np.int64))
    assert np.array_equal(xs.max_data.cpu().numpy(), g["x_max"])
    assert np.array_equal(ws.max_data.cpu().numpy(), g["w_max"])
    if s["bw_e"]:
        assert np.array_equal(xs.e_bias.cpu().numpy(), g["x_ebias"])
        assert np.array_equal(ws.e_bias.cpu().numpy(), g["w_ebias"])
    if "x_quantized" in g:
        assert np.array_equal(xs.quantized_data.cpu().numpy(), g["x_quantized"])


@pytest.mark.parametrize("name", DETERMINISTIC)
def test_mvm_matches_oracle_and_reference(name, cuda):
    """Noise-free output: <= 1e-5 (norm) of the exact restatement; within the tie bound of the reference."""
    c = G.case(name)
    eng, xs, ws = gpu_pair(c, cuda)
    y = eng(xs, ws)
    torch.cuda.synchronize()
    y = y.cpu().numpy().astype(np.float64)
    oxs, ows, oeng, wl = oracle_pair(c)
    y_exact = O.mvm_exact(oxs, ows, oeng, wl)
    assert y.shape == y_exact.shape
    assert rel_norm(y, y_exact) <= 1e-5
    # elementwise: fp32 accumulation over K tiles only
    scale = np.abs(y_exact).max() + 1e-30
    assert np.max(np.abs(y - y_exact)) <= 2e-6 * scale
    y_ref = c["golden"]["y"].astype(np.float64)
    bound = O.tie_bound(oxs, ows, oeng, wl)
    assert np.all(np.abs(y - y_ref) <= bound + 2e-5 * scale)


@pytest.mark.parametrize("name", ["cfg0_int", "cfg0_fp", "cfg0_int_stuck", "batch3d", "p64", "percol_2slice",
                                  "bfp_radc1024", "stuck_both", "tiefree_lossy"])
def test_tile_sums_bit_exact(name, cuda):
    """Per K-tile integer slice-pair sums equal the exact restatement bit for bit."""
    c = G.case(name)
    eng, xs, ws = gpu_pair(c, cuda)
    gx = xs._buf["geom"]
    M = gx["batch"] * gx["rows"]
    Nc = ws._buf["geom"]["n"]
    dump = torch.zeros((gx["kt"], M, Nc), dtype=torch.int32, device=cuda)
    eng.MapReduceDot(xs, ws, acc_dump=dump)
    torch.cuda.synchronize()
    oxs, ows, oeng, wl = oracle_pair(c)
    _, acc, _ = O.mvm_exact(oxs, ows, oeng, wl, return_parts=True)
    if oxs.squeeze:
        acc = acc[:, : M, : Nc]
    else:
        acc = acc.reshape(gx["kt"], oxs.batch, oxs.geom.rows_p, -1)[:, :, : gx["rows"], : Nc].reshape(gx["kt"], M, Nc)
    assert np.array_equal(dump.cpu().numpy().astype(np.int64), acc)


def test_write_variation_deterministic(cuda):
    """Write variation (fixed seed 42) without read noise: deterministic, and as close to the reference
    as a float evaluation can be.

    The non-integer conductances enter the tensor cores as FP16 hi and lo planes (22 significand bits)
    accumulated in fp32.  A crossbar sum next to an ADC rounding boundary can still round the other way
    than in the reference's fp32 evaluation: the oracle's own fp32 and fp64 evaluations differ from the
    reference by 1.2e-4 and 2.3e-4 (norm).  The result must stay within 2x the fp64 oracle's distance
    of the reference, and match the fp64 oracle as closely."""
    c = G.case("write_var")
    eng, xs, ws = gpu_pair(c, cuda)
    y = eng(xs, ws).cpu().numpy().astype(np.float64)
    y_ref = c["golden"]["y"].astype(np.float64)
    oxs, ows, oeng, _ = oracle_pair(c)
    y64 = O.mvm_float(oxs, ows, oeng, np.random.default_rng(0), c["fields"].get("stuck"), c["fields"]["write"],
                      noisy=False)
    d_ref, d_orc = rel_norm(y, y_ref), rel_norm(y, y64)
    print(f"write variation: vs reference {d_ref:.3e}, vs fp64 oracle {d_orc:.3e}, "
          f"oracle vs reference {rel_norm(y64, y_ref):.3e}")
    assert d_ref < 2 * rel_norm(y64, y_ref)
    assert d_orc < 2 * rel_norm(y64, y_ref)
    ideal = c["x"].astype(np.float64) @ c["w"].astype(np.float64)
    snr = lambda a: 10 * np.log10(np.sum(ideal ** 2) / np.sum((ideal - a) ** 2))
    assert abs(snr(y) - snr(y_ref)) < 0.01
    y2 = eng(xs, ws).cpu().numpy().astype(np.float64)
    assert np.array_equal(y, y2)


def test_device_status_clean(cuda):
    from memintelli_flash_b200 import _native as N
    N.device_status()


@pytest.mark.parametrize("name", ["cfg0_int", "cfg0_fp", "bfp_radc1024", "p64"])
def test_split_k_matches_single_pass(name, cuda):
    """Split-K (small grids) gives the same tile sums and, up to fp32 summation order, the same output."""
    from memintelli_flash_b200 import _native as N
    c = G.case(name)
    eng, xs, ws = gpu_pair(c, cuda)
    y_split = eng(xs, ws)
    eng._ws_floats = {k: 0 for k in eng._ws_floats}     # force the single-pass kernel
    y_single = eng(xs, ws)
    torch.cuda.synchronize()
    a, b = y_split.double().cpu().numpy(), y_single.double().cpu().numpy()
    assert rel_norm(a, b) < 1e-6
    oxs, ows, oeng, wl = oracle_pair(c)
    assert rel_norm(a, O.mvm_exact(oxs, ows, oeng, wl)) <= 1e-5


def _boundary_matrix(rng, rows, cols, block, bits, bfp):
    """Values on and within 3 ulp of the quantisation rounding boundaries of every row block.

    INT: (k + 1/2) / (2^(bits-1) - 1) * bmax; BFP: (k + 1/2) * 2^(e + 2 - bits).  Block maxima span
    2^-50 .. 2^60, and each block holds its maximum exactly once.
    """
    qmax = (1 << (bits - 1)) - 1
    x = np.empty((rows, cols), np.float32)
    for r in range(rows):
        for c0 in range(0, cols, block):
            n = min(block, cols - c0)
            bm = np.float32(np.ldexp(1.0 + rng.random(), int(rng.integers(-50, 60))))
            if bfp:
                e = int(O.bfp_exponent(np.array([bm], np.float32))[0])
                k = rng.integers(-(qmax + 1), qmax, n).astype(np.float64)
                t = ((k + 0.5) * np.ldexp(1.0, e + 2 - bits)).astype(np.float32)
            else:
                k = rng.integers(-qmax, qmax, n).astype(np.float64)
                t = (np.float32(1.0) * ((2 * k + 1) / (2 * qmax)).astype(np.float32) * bm).astype(np.float32)
            d = rng.integers(-3, 4, n).astype(np.int32)
            v = (t.view(np.int32) + d).view(np.float32)
            v = np.clip(v, -bm, bm).astype(np.float32)
            v[int(rng.integers(0, n))] = bm if rng.random() < 0.5 else -bm
            x[r, c0:c0 + n] = v
    return x


@pytest.mark.parametrize("bfp,gran", [(False, (1, 128)), (False, (1, 64)), (False, (4, 128)),
                                      (True, (1, 128)), (True, (1, 256)), (False, (1, 256))])
def test_slice_rounding_boundaries(bfp, gran, cuda):
    """Codes of values placed on the INT/BFP rounding boundaries equal the oracle's bit for bit
    (fp32 division and round-half-even as data_formats.py:116-207 computes them)."""
    import memintelli_flash_b200 as M
    rng = np.random.default_rng(7 + gran[0] + gran[1] + int(bfp))
    sm = [1, 1, 2, 2, 2]
    x = _boundary_matrix(rng, 64, 1024, gran[1], sum(sm), bfp)
    eng = M.DPETensor(device=cuda, HGS=1e-5, LGS=1e-8, write_variation=0.0, rate_stuck_HGS=0.0,
                      rate_stuck_LGS=0.0, read_variation=0.0, vnoise=0.0, rdac=4, g_level=4, radc=4096)
    xs = M.SlicedData(torch.tensor(sm), bw_e=8 if bfp else None, is_weight=False, paral_size=(1, 32),
                      quant_gran=gran, device=cuda, inference=False)
    xs.slice_data_imp(eng, torch.from_numpy(x).to(cuda))
    ref = O.slice_matrix(x, sm, bw_e=8 if bfp else None, paral_size=(1, 32), quant_gran=gran)
    assert np.array_equal(xs._buf["block_max"].cpu().numpy().reshape(ref.bmax.shape), ref.bmax)
    assert np.array_equal(xs.sliced_data.cpu().numpy(), ref.sliced_data())


@pytest.mark.parametrize("k,s,p,d,bfp,gran", [(3, 1, 1, 1, False, (1, 64)), (3, 2, 0, 1, True, (1, 64)),
                                              (1, 2, 0, 1, False, (1, 128)), (5, 1, 2, 2, True, (1, 64)),
                                              (2, 1, 0, 1, False, (1, 32)), (3, 1, 1, 1, False, (4, 64))])
def test_conv_patch_slicing(k, s, p, d, bfp, gran, cuda):
    """Codes and block maxima of convolution patches equal the oracle's on F.unfold of the same input
    (convolution.py:111-137 unfolds, then data_formats.py:116-207 slices)."""
    import memintelli_flash_b200 as M
    g = torch.Generator().manual_seed(11 + k + s + p + d)
    x = torch.randn(2, 5, 11, 13, generator=g)
    sm = [1, 1, 2, 2, 2]
    eng = M.DPETensor(device=cuda, HGS=1e-5, LGS=1e-8, write_variation=0.0, rate_stuck_HGS=0.0,
                      rate_stuck_LGS=0.0, read_variation=0.0, vnoise=0.0, rdac=4, g_level=4, radc=4096)
    sd = M.SlicedData(torch.tensor(sm), bw_e=8 if bfp else None, is_weight=False, paral_size=(1, 32),
                      quant_gran=gran, device=cuda, inference=False)
    sd._slice_conv_imp(eng, x.to(cuda), (k, k), (s, s), (p, p), (d, d))
    cols = torch.nn.functional.unfold(x, k, dilation=d, padding=p, stride=s)      # (N, C*k*k, L)
    ref = O.slice_matrix(cols.transpose(1, 2).contiguous().numpy(), sm, bw_e=8 if bfp else None,
                         paral_size=(1, 32), quant_gran=gran)
    assert np.array_equal(sd._buf["block_max"].cpu().numpy().reshape(ref.bmax.shape), ref.bmax)
    assert np.array_equal(sd.sliced_data.cpu().numpy(), ref.sliced_data())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_engine_on_second_device_while_first_is_current():
    """The MVM raises its shared-memory attribute per device, and the host layer switches to the operands'
    device around every native call: an engine on cuda:1 works while cuda:0 is current, and matches the
    oracle (a first launch on cuda:0 sets the attribute there only)."""
    c = G.case("cfg0_int")
    dev0, dev1 = torch.device("cuda:0"), torch.device("cuda:1")
    torch.cuda.set_device(dev0)
    eng0, xs0, ws0 = gpu_pair(c, dev0)
    y0 = eng0(xs0, ws0)
    eng1, xs1, ws1 = gpu_pair(c, dev1)
    assert torch.cuda.current_device() == 0
    y1 = eng1(xs1, ws1)
    assert y1.device == dev1 and torch.cuda.current_device() == 0
    torch.cuda.synchronize(dev1)
    oxs, ows, oeng, wl = oracle_pair(c)
    ref = O.mvm_exact(oxs, ows, oeng, wl)
    assert rel_norm(y1.double().cpu().numpy(), ref) <= 1e-5
    assert torch.equal(y0.cpu(), y1.cpu())


def test_write_variation_split_weights_at_a_tail_split_shape(cuda):
    """The FP16 hi/lo weight operand (write variation 0.05) through the persistent launch with several
    tiles per CTA, three pipeline stages (the doubled weight stage) and a tail split: 2048 x 1024 x 4096
    is 1376 output tiles, 9 waves + 44 tiles cut into K ranges.  128 rows against the oracle's fp64
    evaluation with the same fixed-seed write field (torch.normal, Generator(42), the reference's G shape),
    within the distance the small golden case shows between float evaluations (2.3e-4)."""
    import memintelli_flash_b200 as M
    from memintelli_flash_b200 import _native as N
    M_, K, Nc = 2048, 1024, 4096
    kw = dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096, write_variation=0.05, read_variation=0.0,
              vnoise=0.0, rate_stuck_HGS=0.0, rate_stuck_LGS=0.0)
    eng = M.DPETensor(device=cuda, **kw)
    eng.fault_field_device = "cpu"
    g = torch.Generator().manual_seed(8)
    x, w = torch.randn(M_, K, generator=g), torch.randn(K, Nc, generator=g) * 0.03
    sm = [1, 1, 2, 2, 2]
    xs = M.SlicedData(torch.tensor(sm), is_weight=False, paral_size=(1, 32), quant_gran=(1, 128), device=cuda,
                      inference=True)
    ws = M.SlicedData(torch.tensor(sm), is_weight=True, paral_size=(32, 32), quant_gran=(128, 128), device=cuda,
                      inference=True)
    ws.slice_data_imp(eng, w.to(cuda))
    xs.slice_data_imp(eng, x.to(cuda))
    f = N.c_i64(0)
    N.call("mib_mvm_workspace", M_, Nc, xs._spec(), ws._spec(), xs._kgeom(), eng._device_spec(), f)
    assert 0 < f.value < 2 * M_ * Nc                     # the tail split's partials
    y = eng(xs, ws)
    torch.cuda.synchronize()
    rows = np.arange(0, M_, 16) + (np.arange(128) * 5) % 16
    oxs = O.slice_matrix(x[rows].numpy(), sm, None, (1, 32), (1, 128))
    ows = O.slice_matrix(w.numpy(), sm, None, (32, 32), (128, 128))
    gshape = (ows.geom.rows_p // 32, ows.geom.cols_p // 32, len(sm), 32, 32)
    write = torch.normal(0, 0.05, gshape, generator=torch.Generator().manual_seed(42)).numpy()
    ref = O.mvm_float(oxs, ows, O.Engine(**kw), np.random.default_rng(0), None, write, noisy=False)
    got = y[torch.from_numpy(rows).to(cuda)].double().cpu().numpy()
    d = rel_norm(got, ref)
    print(f"write variation 2048x1024x4096: vs fp64 oracle {d:.3e}")
    assert d < 5e-4
    N.device_status()
