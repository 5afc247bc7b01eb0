"""Statistical parity of the noisy CIM path (config-0 device model) with the reference (needs a B200).

The reference's per-seed SNR and error moments (256 seeds, paired inputs,
fixed-seed stuck-at mask) are in tests/golden/noise_stats.json.  The same
inputs are run here; the stuck-at mask is drawn on the CPU like the reference's.
"""
import numpy as np
import pytest
import torch

import golden_cases as G

pytestmark = pytest.mark.gpu

SEEDS = 256


def _arm(mode):
    """Shapes, number format and noisy device model of one arm of noise_stats.json (make_golden.py)."""
    a = dict(G.noise_stats()["arms"][mode])
    if isinstance(a["read"], dict):
        a["read"] = {int(k): v for k, v in a["read"].items()}
    return a


def _engine(M, cuda, arm, noisy):
    e = M.DPETensor(device=cuda, HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096, write_variation=0.0,
                    rate_stuck_HGS=arm["stuck"], rate_stuck_LGS=0.0,
                    read_variation=arm["read"] if noisy else 0.0, vnoise=arm["vnoise"] if noisy else 0.0)
    e.fault_field_device = "cpu"
    return e


@pytest.mark.parametrize("mode", ["int", "fp", "read_k1024", "per_level"])
def test_noise_statistics(mode, cuda):
    """int / fp: config 0's device model (stuck-at 1e-3, read variation 0.05, voltage noise 0.05).
    read_k1024: the benchmark's device model (read variation 0.05 only) at K = 1024, which slices inputs
    straight into FP16 planes.  per_level: read variation {0: 0.02, 1: 0.05, 2: 0.05, 3: 0.1} by level
    (memmat_tensor.py:226-233)."""
    import memintelli_flash_b200 as M
    ref = np.array(G.noise_stats()[mode])
    arm = _arm(mode)
    bw_e = arm["bw_e"]
    en, e0 = _engine(M, cuda, arm, True), _engine(M, cuda, arm, False)
    sm = torch.tensor([1, 1, 2, 2, 2])
    rows = []
    for s in range(SEEDS):
        g = torch.Generator().manual_seed(1000 + s)
        x = torch.randn(*arm["xs"], generator=g)
        w = torch.randn(*arm["ws"], generator=g)
        ideal = (x.double() @ w.double()).numpy()
        outs = []
        for eng in (en, e0):
            xs = M.SlicedData(sm, bw_e=bw_e, is_weight=False, paral_size=(1, 32), quant_gran=(1, 128),
                              device=cuda, inference=True)
            ws = M.SlicedData(sm, bw_e=bw_e, is_weight=True, paral_size=(32, 32), quant_gran=(128, 128),
                              device=cuda, inference=True)
            ws.slice_data_imp(eng, w.to(cuda))
            xs.slice_data_imp(eng, x.to(cuda))
            if eng is en and arm["vnoise"] == 0:
                assert xs._buf["planes"].dtype == torch.float16     # the benchmark's input path
            torch.manual_seed(50_000 + s)
            outs.append(eng(xs, ws).double().cpu().numpy())
        yn, y0 = outs
        e = yn - y0
        snr = 10 * np.log10(np.sum(ideal ** 2) / np.sum((ideal - yn) ** 2))
        rows.append([s, snr, e.mean(), e.std()])
    mine = np.array(rows)
    d = mine[:, 1] - ref[:SEEDS, 1]
    se = d.std(ddof=1) / np.sqrt(SEEDS)
    print(f"{mode}: SNR mine {mine[:, 1].mean():.4f} ref {ref[:SEEDS, 1].mean():.4f} "
          f"paired diff {d.mean():+.4f} +- {se:.4f} dB; err std mine {mine[:, 3].mean():.4f} "
          f"ref {ref[:SEEDS, 3].mean():.4f}; err mean mine {mine[:, 2].mean():.4f} ref {ref[:SEEDS, 2].mean():.4f}")
    assert abs(d.mean()) < 0.1
    assert abs(mine[:, 3].mean() / ref[:SEEDS, 3].mean() - 1) < 0.02
    # mean error against the exact noise-free result: the reference's own noise-free output carries
    # its fp32 tie-rounding bias (column 5), ours is exact to fp32, so compare on the exact baseline
    ref_mean = ref[:SEEDS, 2] + ref[:SEEDS, 5]
    spread = np.hypot(mine[:, 2].std(ddof=1), ref_mean.std(ddof=1)) / np.sqrt(SEEDS)
    print(f"{mode}: err mean vs exact mine {mine[:, 2].mean():.4f} ref {ref_mean.mean():.4f} +- {spread:.4f}")
    assert abs(mine[:, 2].mean() - ref_mean.mean()) < max(0.02 * abs(ref_mean.mean()), 4 * spread)


def test_shared_and_background_read_noise_draws(cuda):
    """DPETensor.draw_read_noise: a draw taken for two multiplies serves both (bit-identical outputs, as
    the sequences of one reference call share one draw); a third multiply draws again; the background
    pass (side stream, one small block per SM) produces the same planes as the foreground one for the
    same seed; and a draw taken in the background beside a running multiply is waited for."""
    import memintelli_flash_b200 as M
    eng = M.DPETensor(device=cuda, HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096, write_variation=0.0,
                      rate_stuck_HGS=0.0, rate_stuck_LGS=0.0, read_variation=0.05, vnoise=0.0)
    g = torch.Generator().manual_seed(3)
    x, w = torch.randn(512, 1024, generator=g), torch.randn(1024, 768, generator=g) * 0.03
    sm = torch.tensor([1, 1, 2, 2, 2])
    xs = M.SlicedData(sm, is_weight=False, paral_size=(1, 32), quant_gran=(1, 128), device=cuda, inference=True)
    ws = M.SlicedData(sm, is_weight=True, paral_size=(32, 32), quant_gran=(128, 128), device=cuda, inference=True)
    xs.slice_data_imp(eng, x.to(cuda))
    ws.slice_data_imp(eng, w.to(cuda))
    outs = {}
    for background in (False, True):
        torch.manual_seed(21)
        big = eng(xs, ws)                       # queued work for a background pass to run beside
        eng.draw_read_noise(ws, uses=2, background=background)
        a, b = eng(xs, ws), eng(xs, ws)
        c = eng(xs, ws)                         # the shared draw is used up: a new one
        torch.cuda.synchronize()
        assert torch.equal(a, b) and not torch.equal(a, c) and not torch.equal(a, big)
        outs[background] = a
    assert torch.equal(outs[False], outs[True])
