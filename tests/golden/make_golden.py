"""Generate golden fixtures by running the reference Memintelli package on CPU.

Run where the reference source tree is available (``--ref`` or the
MEMINTELLI_REFERENCE environment variable names it):

    python tests/golden/make_golden.py --ref <reference tree> [--seeds 256] [--only PART ...]

It writes
* ``tests/golden/cases.npz`` (deterministic noise-free cases: inputs or their
  seed, the reference's packed slice codes, block maxima / exponents and fp32
  outputs; part ``cases``);
* ``tests/golden/noise_stats.json`` (per-seed SNR and error moments of the
  reference's noisy path, for statistical parity; parts ``stats-int``,
  ``stats-fp``, ``stats-read-k1024`` and ``stats-per-level``, merged into the
  existing file when only some are generated);
* ``tests/golden/qwen3_model.npz`` (logits and loss of a small Qwen3 built the
  reference's way, ``transformers`` Qwen3ForCausalLM with every nn.Linear
  swapped for LinearMem; part ``qwen3``).

The reference imports matplotlib at module level; it is stubbed because only
the arithmetic is exercised.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
import types

import numpy as np
import torch


def _stub_matplotlib():
    class _Stub(types.ModuleType):
        def __getattr__(self, k):
            if k.startswith("__"):
                raise AttributeError(k)
            return lambda *a, **kw: None

    m = _Stub("matplotlib")
    m.pyplot = _Stub("matplotlib.pyplot")
    sys.modules.setdefault("matplotlib", m)
    sys.modules.setdefault("matplotlib.pyplot", m.pyplot)


NOISE_FREE = dict(write_variation=0.0, read_variation=0.0, vnoise=0.0, rate_stuck_HGS=0.0, rate_stuck_LGS=0.0)

# name -> case spec.  x/W come either from a torch seed (stored as "seed") or are stored.
CASES = {
    # example 1 shapes (config 0), noise-free engine, training path (_dot) as the example runs it
    "cfg0_int": dict(xs=(400, 500), ws=(500, 600), seed=42, store_inputs=False, bw_e=None,
                     sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 128), wp=(32, 32), wq=(128, 128),
                     eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=False),
    "cfg0_fp": dict(xs=(400, 500), ws=(500, 600), seed=42, store_inputs=False, bw_e=8,
                    sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 128), wp=(32, 32), wq=(128, 128),
                    eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=False),
    "cfg0_int_stuck": dict(xs=(400, 500), ws=(500, 600), seed=42, store_inputs=False, bw_e=None,
                           sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 128), wp=(32, 32), wq=(128, 128),
                           eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096, rate_stuck_HGS=0.001),
                           inference=True),
    # tie-free settings: radc = D + 1 (lossless) and an odd-denominator lossy ADC
    "tiefree_lossless": dict(xs=(96, 300), ws=(300, 160), seed=7, store_inputs=True, bw_e=None,
                             sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 128), wp=(32, 32), wq=(128, 128),
                             eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=289), inference=True),
    "tiefree_lossy": dict(xs=(96, 300), ws=(300, 160), seed=8, store_inputs=True, bw_e=8,
                          sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 128), wp=(32, 32), wq=(128, 128),
                          eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=33), inference=True),
    # batched (3-D) input, odd sizes
    "batch3d": dict(xs=(2, 19, 70), ws=(70, 45), seed=1, store_inputs=True, bw_e=None,
                    sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 64), wp=(32, 32), wq=(64, 64),
                    eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=True),
    "batch3d_train": dict(xs=(3, 33, 100), ws=(100, 70), seed=11, store_inputs=True, bw_e=8,
                          sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 64), wp=(32, 32), wq=(64, 64),
                          eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=False),
    # block floating point with a non-dyadic ADC ratio (config 2's radc)
    "bfp_radc1024": dict(xs=(37, 100), ws=(100, 45), seed=2, store_inputs=True, bw_e=8,
                         sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 64), wp=(32, 32), wq=(64, 64),
                         eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=1024), inference=True),
    # 64-deep crossbar (config 3 style)
    "p64": dict(xs=(50, 200), ws=(200, 130), seed=3, store_inputs=True, bw_e=None,
                sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 64), xq=(1, 64), wp=(64, 64), wq=(64, 64),
                eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=True),
    # 2-D input tiles, 16 levels (memmat_tensor.py self-test style)
    "xtile_g16": dict(xs=(70, 130), ws=(130, 90), seed=4, store_inputs=True, bw_e=None,
                      sx=[1, 1, 2, 4], sw=[1, 1, 2, 4], xp=(64, 64), xq=(64, 64), wp=(64, 64), wq=(64, 64),
                      eng=dict(HGS=1e-5, LGS=1e-7, rdac=16, g_level=16, radc=2 ** 16), inference=True),
    # per-weight-slice ADC resolution list
    "radc_list": dict(xs=(64, 150), ws=(150, 100), seed=5, store_inputs=True, bw_e=None,
                      sx=[1, 1, 2, 2], sw=[1, 1, 2, 2], xp=(64, 64), xq=(64, 64), wp=(64, 64), wq=(64, 64),
                      eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=[2 ** 12, 2 ** 11, 2 ** 10, 2 ** 9]),
                      inference=True),
    # per-column weight tiles, 2-slice (example 11 geometry)
    "percol_2slice": dict(xs=(40, 150), ws=(150, 33), seed=6, store_inputs=True, bw_e=None,
                          sx=[1, 1], sw=[1, 1], xp=(1, 64), xq=(1, 64), wp=(64, 1), wq=(64, 1),
                          eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=True),
    # string granularities
    "gran_strings": dict(xs=(30, 90), ws=(90, 50), seed=9, store_inputs=True, bw_e=None,
                         sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq="per-row", wp=(32, 32), wq="per-matrix",
                         eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=True),
    # both stuck-at kinds
    "stuck_both": dict(xs=(48, 128), ws=(128, 200), seed=10, store_inputs=True, bw_e=None,
                       sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 128), wp=(32, 32), wq=(128, 128),
                       eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096, rate_stuck_HGS=0.02,
                                rate_stuck_LGS=0.03), inference=True),
    # write variation only (deterministic: fixed-seed draw), compared with a loose tolerance
    "write_var": dict(xs=(64, 128), ws=(128, 64), seed=12, store_inputs=True, bw_e=None,
                      sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 128), wp=(32, 32), wq=(128, 128),
                      eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096, write_variation=0.05),
                      inference=True),
}


def make_inputs(spec, name):
    if spec["store_inputs"]:
        g = torch.Generator().manual_seed(spec["seed"])
        x = torch.randn(*spec["xs"], generator=g)
        w = torch.randn(*spec["ws"], generator=g)
        return x, w
    torch.manual_seed(spec["seed"])
    x = torch.randn(*spec["xs"])
    w = torch.randn(*spec["ws"])
    return x, w


def add_zero_blocks(x, w, wq):
    """Zero one input row and the first weight quant block (all-zero-block path)."""
    x = x.clone()
    w = w.clone()
    x[..., 3, :] = 0.0
    w[0:wq[0], 0:wq[1]] = 0.0
    return x, w


def run_case(name, spec, DPETensor, SlicedData):
    eng_kw = dict(NOISE_FREE)
    eng_kw.update(spec["eng"])
    eng = DPETensor(device=torch.device("cpu"), **eng_kw)
    x, w = make_inputs(spec, name)
    if name in ("batch3d", "stuck_both"):
        x, w = add_zero_blocks(x, w, spec["wq"])
    xs = SlicedData(torch.tensor(spec["sx"]), bw_e=spec["bw_e"], is_weight=False, paral_size=spec["xp"],
                    quant_gran=spec["xq"], device=torch.device("cpu"), inference=spec["inference"])
    ws = SlicedData(torch.tensor(spec["sw"]), bw_e=spec["bw_e"], is_weight=True, paral_size=spec["wp"],
                    quant_gran=spec["wq"], device=torch.device("cpu"), inference=spec["inference"])
    # the reference needs sliced_data of the weight for G; inference=True frees it afterwards.
    ws_keep = SlicedData(torch.tensor(spec["sw"]), bw_e=spec["bw_e"], is_weight=True, paral_size=spec["wp"],
                         quant_gran=spec["wq"], device=torch.device("cpu"), inference=False)
    ws_keep.slice_data_imp(eng, w)
    ws.slice_data_imp(eng, w)
    xs.slice_data_imp(eng, x)
    y = eng(xs, ws)
    out = {
        "y": y.numpy().astype(np.float32),
        "x_packed": pack_codes(xs.sliced_data, spec["sx"]),
        "w_packed": pack_codes(ws_keep.sliced_data, spec["sw"]),
        "x_max": xs.max_data.numpy().astype(np.float32),
        "w_max": ws_keep.max_data.numpy().astype(np.float32),
    }
    if spec["bw_e"]:
        out["x_ebias"] = xs.e_bias.numpy().astype(np.float32)
        out["w_ebias"] = ws_keep.e_bias.numpy().astype(np.float32)
    if not spec["inference"] and spec["store_inputs"]:
        out["x_quantized"] = xs.quantized_data.numpy().astype(np.float32)
    if spec["store_inputs"]:
        out["x"] = x.numpy()
        out["w"] = w.numpy()
    else:
        out["x_sum"] = np.array([float(x.double().sum()), float(w.double().sum())])
    # fixed-seed fault fields (memmat_tensor.py:177-187) are regenerated by the tests from
    # torch.Generator().manual_seed(123 / 42) over this G shape; store the shape and a checksum.
    out["G_shape"] = np.array(ws_keep.G.shape)
    if eng_kw.get("rate_stuck_HGS", 0) > 0 or eng_kw.get("rate_stuck_LGS", 0) > 0:
        gen = torch.Generator().manual_seed(123)
        out["stuck_field_sum"] = np.array([float(torch.rand(ws_keep.G.shape, generator=gen).double().sum())])
    if eng_kw.get("write_variation", 0) > 0:
        gen = torch.Generator().manual_seed(42)
        wf = torch.normal(0, eng_kw["write_variation"], ws_keep.G.shape, generator=gen)
        out["write_field_sum"] = np.array([float(wf.double().sum())])
    return out


def pack_codes(sliced, slice_method):
    """Packed two's complement code per element from the reference slice planes (LSB-first)."""
    sl = sliced.to(torch.int64)
    widths = list(slice_method)[::-1]
    packed = torch.zeros_like(sl.select(-3, 0))
    off = 0
    for t, wdt in enumerate(widths):
        packed += sl.select(-3, t) << off
        off += wdt
    return packed.numpy().astype(np.uint8 if off <= 8 else np.int16)


# Layer cases: the reference's own LinearMem / Conv2dMem, noise-free engine, fixed torch seed for init.
LAYER_CASES = {
    "conv_bfp_pad": dict(kind="conv", seed=21, x=(2, 3, 10, 10), cin=3, cout=8, k=3, stride=1, padding=1, bias=True,
                         bw_e=8, sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 64), wp=(32, 32),
                         wq=(64, 64), eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=1024), inference=True),
    "conv_s2_int": dict(kind="conv", seed=22, x=(3, 16, 9, 9), cin=16, cout=40, k=3, stride=2, padding=0, bias=False,
                        bw_e=None, sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 128), wp=(32, 32),
                        wq=(128, 128), eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=True),
    "conv_train": dict(kind="conv", seed=23, x=(2, 4, 7, 7), cin=4, cout=6, k=3, stride=1, padding=1, bias=True,
                       bw_e=None, sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 32), wp=(32, 32),
                       wq=(32, 32), eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=False),
    "linear_bias_3d": dict(kind="linear", seed=24, x=(2, 17, 96), cin=96, cout=70, bias=True, bw_e=None,
                           sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 32), wp=(32, 32), wq=(32, 32),
                           eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=True),
    "linear_train": dict(kind="linear", seed=25, x=(33, 100), cin=100, cout=20, bias=True, bw_e=8,
                         sx=[1, 1, 2, 2, 2], sw=[1, 1, 2, 2, 2], xp=(1, 32), xq=(1, 64), wp=(32, 32), wq=(64, 64),
                         eng=dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096), inference=False),
}


def run_layer_case(name, spec, DPETensor, LinearMem, Conv2dMem):
    eng_kw = dict(NOISE_FREE)
    eng_kw.update(spec["eng"])
    eng = DPETensor(device=torch.device("cpu"), **eng_kw)
    torch.manual_seed(spec["seed"])
    if spec["kind"] == "conv":
        layer = Conv2dMem(eng, spec["cin"], spec["cout"], spec["k"], spec["sx"], spec["sw"], stride=spec["stride"],
                          padding=spec["padding"], bias=spec["bias"], device=torch.device("cpu"), bw_e=spec["bw_e"],
                          input_paral_size=spec["xp"], weight_paral_size=spec["wp"], input_quant_gran=spec["xq"],
                          weight_quant_gran=spec["wq"])
    else:
        layer = LinearMem(eng, spec["cin"], spec["cout"], spec["sx"], spec["sw"], bias=spec["bias"],
                          device=torch.device("cpu"), bw_e=spec["bw_e"], input_paral_size=spec["xp"],
                          weight_paral_size=spec["wp"], input_quant_gran=spec["xq"], weight_quant_gran=spec["wq"])
    x = torch.randn(*spec["x"])
    if spec["inference"]:
        layer.inference_mode = True
        layer.weight_sliced.inference = True
        with torch.no_grad():
            y = layer(x)
        out = {"y": y.numpy()}
    else:
        xg = x.clone().requires_grad_(True)
        y = layer(xg)
        y.backward(torch.ones_like(y))
        out = {"y": y.detach().numpy(), "grad_x": xg.grad.numpy(), "grad_w": layer.weight.grad.numpy()}
        if layer.bias is not None:
            out["grad_b"] = layer.bias.grad.numpy()
    out["x"] = x.numpy()
    out["weight"] = layer.weight.detach().numpy()
    if layer.bias is not None:
        out["bias"] = layer.bias.detach().numpy()
    return out


def exact_nf(x, w, bw_e, stuck_rate=0.001):
    """Exact noise-free restatement (oracle) of a matmul with the config-0 slicing and, when
    ``stuck_rate`` > 0, the reference's fixed-seed stuck-at mask."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    from oracle import cim_oracle as O
    xs = O.slice_matrix(x.numpy(), [1, 1, 2, 2, 2], bw_e, (1, 32), (1, 128))
    ws = O.slice_matrix(w.numpy(), [1, 1, 2, 2, 2], bw_e, (32, 32), (128, 128))
    eng = O.Engine(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096, rate_stuck_HGS=stuck_rate)
    stuck = None
    if stuck_rate > 0:
        g = torch.Generator().manual_seed(123)
        shape = (ws.geom.rows_p // 32, ws.geom.cols_p // 32, 5, 32, 32)
        stuck = torch.rand(shape, generator=g).numpy()
    return O.mvm_exact(xs, ws, eng, O.weight_levels(ws, eng, stuck))


# Noise-statistics arms: input / weight shapes, number format and the noisy device model.  Every arm
# uses slices [1,1,2,2,2], input (1,128)/(1,32), weight (128,128)/(32,32), HGS 1e-5, LGS 1e-8, 4 levels,
# rdac 4, radc 4096; the noise-free twin of each seed zeroes read variation and vnoise only.
STAT_ARMS = {
    # config 0's device model (example 1)
    "int": dict(xs=(400, 500), ws=(500, 600), bw_e=None, stuck=0.001, read=0.05, vnoise=0.05),
    "fp": dict(xs=(400, 500), ws=(500, 600), bw_e=8, stuck=0.001, read=0.05, vnoise=0.05),
    # the Qwen3 example's device model (examples/11_qwen3_wikitext2_inference.py:66-77: read variation
    # 0.05 only) at the Qwen3-0.6B hidden width
    "read_k1024": dict(xs=(256, 1024), ws=(1024, 512), bw_e=None, stuck=0.0, read=0.05, vnoise=0.0),
    # per-level read variation (memmat_tensor.py:226-233)
    "per_level": dict(xs=(400, 500), ws=(500, 600), bw_e=None, stuck=0.0,
                      read={0: 0.02, 1: 0.05, 2: 0.05, 3: 0.1}, vnoise=0.0),
}


def noise_stats(arms, n_seeds, DPETensor, SlicedData):
    """Per-seed SNR and error moments of the reference's noisy path for each arm in ``arms``."""
    res = {}
    for key in arms:
        a = STAT_ARMS[key]
        rows = []
        t0 = time.time()
        for s in range(n_seeds):
            g = torch.Generator().manual_seed(1000 + s)
            x = torch.randn(*a["xs"], generator=g)
            w = torch.randn(*a["ws"], generator=g)
            ideal = (x.double() @ w.double()).numpy()
            outs = []
            for noisy in (True, False):
                kw = dict(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096, write_variation=0.0,
                          rate_stuck_HGS=a["stuck"], rate_stuck_LGS=0.0,
                          read_variation=a["read"] if noisy else 0.0, vnoise=a["vnoise"] if noisy else 0.0)
                torch.manual_seed(50_000 + s)
                eng = DPETensor(device=torch.device("cpu"), **kw)
                xs = SlicedData(torch.tensor([1, 1, 2, 2, 2]), bw_e=a["bw_e"], is_weight=False, paral_size=(1, 32),
                                quant_gran=(1, 128), device=torch.device("cpu"), inference=True)
                ws = SlicedData(torch.tensor([1, 1, 2, 2, 2]), bw_e=a["bw_e"], is_weight=True, paral_size=(32, 32),
                                quant_gran=(128, 128), device=torch.device("cpu"), inference=True)
                ws.slice_data_imp(eng, w)
                xs.slice_data_imp(eng, x)
                outs.append(eng(xs, ws).double().numpy())
            yn, y0 = outs
            e = yn - y0
            snr = 10 * np.log10(np.sum(ideal ** 2) / np.sum((ideal - yn) ** 2))
            # the reference's own noise-free output carries its fp32 tie-rounding bias; record it
            # against the exact restatement so means can be compared on one baseline
            tie_bias = float((y0 - exact_nf(x, w, a["bw_e"], a["stuck"])).mean())
            rows.append([s, snr, float(e.mean()), float(e.std()), float(np.sqrt(np.mean(y0 ** 2))), tie_bias])
        res[key] = rows
        print(f"noise stats {key}: {n_seeds} seeds in {time.time() - t0:.1f}s; "
              f"SNR {np.mean([r[1] for r in rows]):.3f} +- {np.std([r[1] for r in rows]):.3f}")
    return res


def qwen3_model(Wrapper, DPETensor, replace_linear):
    """Logits and loss of the small Qwen3 (qwen3_small.py) built the reference's way: transformers'
    Qwen3ForCausalLM with every nn.Linear replaced by the reference's LinearMem through its own
    _replace_linear_with_linearmem, wrapped in Qwen3MemWrapper, then update_weight() and
    prepare_for_inference() (memintelli/NN_models/Qwen3.py:22-106); noise-free engine, fp32 eager
    attention, on the CPU.  Two ADC resolutions: 289 (= D + 1, lossless and tie-free) and
    4096 (the benchmark's, with half-way ties)."""
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import qwen3_small as Q
    from transformers import Qwen3ForCausalLM
    sd = Q.state_dict()
    ids = Q.token_ids()
    out = {"ids": ids.numpy(), "weights_sum": np.array([float(sum(v.double().sum() for v in sd.values()))])}
    for radc in (289, 4096):
        torch.manual_seed(0)
        model = Qwen3ForCausalLM(Q.hf_config())
        model.load_state_dict(sd)
        eng = DPETensor(device=torch.device("cpu"), HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=radc,
                        **NOISE_FREE)
        mem_args = dict(engine=eng, input_slice=[1, 1, 2, 2, 2], weight_slice=[1, 1, 2, 2, 2],
                        device=torch.device("cpu"), bw_e=None, input_paral_size=(1, 32),
                        weight_paral_size=(32, 32), input_quant_gran=(1, 128), weight_quant_gran=(128, 128))
        replace_linear(model, mem_args)
        # the reference's own flow (examples/11_qwen3_wikitext2_inference.py:100-102): program the copied
        # weights into the crossbars, then switch every LinearMem to its inference path
        wrapped = Wrapper(model, mem_enabled=True)
        wrapped.update_weight()
        wrapped.prepare_for_inference()
        with torch.no_grad():
            res = wrapped(input_ids=ids, labels=ids)
        out[f"logits_r{radc}"] = res.logits.float().numpy()
        out[f"loss_r{radc}"] = np.array([float(res.loss)])
        # the same model with every linear on the oracle (exact, half-even ADC ties), for the tie shift
        torch.manual_seed(0)
        exact = Qwen3ForCausalLM(Q.hf_config())
        exact.load_state_dict(sd)
        _swap_oracle_linears(exact, radc)
        exact.eval()
        with torch.no_grad():
            out[f"logits_oracle_r{radc}"] = exact(input_ids=ids).logits.float().numpy()
        # the same model without crossbars, for scale
        if radc == 289:
            plain = Qwen3ForCausalLM(Q.hf_config())
            plain.load_state_dict(sd)
            plain.eval()
            with torch.no_grad():
                out["logits_float"] = plain(input_ids=ids).logits.float().numpy()
        print(f"qwen3 small radc {radc}: loss {float(res.loss):.6f}")
    return out


class _OracleLinear(torch.nn.Module):
    """nn.Linear replacement computing the crossbar matmul with the oracle's exact restatement."""

    def __init__(self, lin, radc):
        super().__init__()
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
        from oracle import cim_oracle as O
        self.O = O
        self.ws = O.slice_matrix(lin.weight.detach().t().contiguous().numpy(), [1, 1, 2, 2, 2], None, (32, 32),
                                 (128, 128))
        self.eng = O.Engine(HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=radc)

    def forward(self, x):
        shp = x.shape
        xs = self.O.slice_matrix(x.reshape(-1, shp[-1]).detach().float().numpy(), [1, 1, 2, 2, 2], None, (1, 32),
                                 (1, 128))
        y = self.O.mvm_exact(xs, self.ws, self.eng)
        return torch.from_numpy(y.astype(np.float32)).reshape(*shp[:-1], -1)


def _swap_oracle_linears(module, radc):
    for name, child in list(module.named_children()):
        if isinstance(child, torch.nn.Linear):
            setattr(module, name, _OracleLinear(child, radc))
        else:
            _swap_oracle_linears(child, radc)


PARTS = ("cases", "stats-int", "stats-fp", "stats-read-k1024", "stats-per-level", "qwen3")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MEMINTELLI_REFERENCE"),
                    help="reference source tree (default: $MEMINTELLI_REFERENCE)")
    ap.add_argument("--seeds", type=int, default=256)
    ap.add_argument("--only", nargs="*", choices=PARTS, default=list(PARTS))
    args = ap.parse_args()
    if not args.ref:
        ap.error("name the reference source tree with --ref or MEMINTELLI_REFERENCE")
    _stub_matplotlib()
    sys.path.insert(0, args.ref)
    torch.set_num_threads(os.cpu_count())
    from memintelli.pimpy.memmat_tensor import DPETensor
    from memintelli.pimpy.data_formats import SlicedData
    from memintelli.NN_layers.linear import LinearMem
    from memintelli.NN_layers.convolution import Conv2dMem

    here = os.path.dirname(os.path.abspath(__file__))
    if "cases" in args.only:
        arrays = {}
        meta = {}
        for name, spec in CASES.items():
            t0 = time.time()
            out = run_case(name, spec, DPETensor, SlicedData)
            for k, v in out.items():
                arrays[f"{name}/{k}"] = v
            meta[name] = {k: v for k, v in spec.items()}
            print(f"{name}: y {out['y'].shape} in {time.time() - t0:.2f}s")
        for name, spec in LAYER_CASES.items():
            out = run_layer_case(name, spec, DPETensor, LinearMem, Conv2dMem)
            for k, v in out.items():
                arrays[f"{name}/{k}"] = v
            meta[name] = dict(spec)
            print(f"{name}: y {out['y'].shape}")
        np.savez_compressed(os.path.join(here, "cases.npz"), **arrays)
        with open(os.path.join(here, "cases.json"), "w") as f:
            json.dump(meta, f, indent=1)
    arms = [p[len("stats-"):].replace("-", "_") for p in args.only if p.startswith("stats-")]
    if arms:
        path = os.path.join(here, "noise_stats.json")
        st = {"columns": ["seed", "snr_db", "err_mean", "err_std", "y_rms", "tie_bias"]}
        if os.path.exists(path):
            with open(path) as f:
                st.update(json.load(f))
        st.update(noise_stats(arms, args.seeds, DPETensor, SlicedData))
        st["arms"] = {k: {kk: (vv if not isinstance(vv, dict) else {str(a): b for a, b in vv.items()})
                          for kk, vv in STAT_ARMS[k].items()} for k in STAT_ARMS if k in st}
        with open(path, "w") as f:
            json.dump(st, f)
    if "qwen3" in args.only:
        from memintelli.NN_models.Qwen3 import Qwen3MemWrapper, _replace_linear_with_linearmem
        out = qwen3_model(Qwen3MemWrapper, DPETensor, _replace_linear_with_linearmem)
        np.savez_compressed(os.path.join(here, "qwen3_model.npz"), **out)


if __name__ == "__main__":
    main()
