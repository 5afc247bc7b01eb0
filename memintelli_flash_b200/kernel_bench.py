"""Micro-benchmarks of the two crossbar kernels, through the public API.

    python -m memintelli_flash_b200.kernel_bench slice --rows 16384 --cols 3072 [--bfp]
    python -m memintelli_flash_b200.kernel_bench mvm --m 4096 --k 4096 --n 4096 [--noisy]

The engine is the reference's example device (HGS 1e-5, LGS 1e-8, rdac 4, g_level 4,
radc 4096) with slices [1, 1, 2, 2, 2]: input tiles (1, 32) in (1, 128) quant blocks,
weight tiles (32, 32) in (128, 128) blocks. Each case runs 3 untimed calls, then times
`--iters` calls with CUDA events on the launching stream and prints one line:

* slice: time per call and algorithmic bytes/s, with bytes = 4 (fp32 read) + S (E4M3
  planes) + 4/p (tile scale) per element;
* mvm:   median MVM launch time, slice-pair ops/s and ADC events/s.

The inputs are randn; x is larger than L2 at the default sizes.
"""
import argparse

import torch

from . import _native as N
from .pimpy import DPETensor, SlicedData

SLICES = [1, 1, 2, 2, 2]


def _engine(device, noisy):
    return DPETensor(HGS=1e-5, LGS=1e-8, write_variation=0.0, rate_stuck_HGS=0.0, rate_stuck_LGS=0.0,
                     read_variation=0.05 if noisy else 0.0, vnoise=0.05 if noisy else 0.0,
                     rdac=4, g_level=4, radc=4096, device=device)


def _input(device, bfp):
    return SlicedData(torch.tensor(SLICES), bw_e=8 if bfp else None, is_weight=False, paral_size=(1, 32),
                      quant_gran=(1, 128), device=device, inference=True)


def _weight(device, bfp):
    return SlicedData(torch.tensor(SLICES), bw_e=8 if bfp else None, is_weight=True, paral_size=(32, 32),
                      quant_gran=(128, 128), device=device, inference=True)


def bench_slice(rows, cols, bfp=False, iters=20, device="cuda:0"):
    dev = torch.device(device)
    eng = _engine(dev, False)
    x = torch.randn(rows, cols, device=dev)
    xs = _input(dev, bfp)
    for _ in range(3):
        xs.slice_data_imp(eng, x)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        xs.slice_data_imp(eng, x)
    e1.record()
    torch.cuda.synchronize(dev)
    N.device_status()
    us = e0.elapsed_time(e1) * 1e3 / iters
    nbytes = rows * cols * (4 + len(SLICES) + 4 / 32)
    print(f"slice rows={rows} cols={cols} bfp={bfp}: {us:.1f} us/call, {nbytes / us / 1e3:.0f} GB/s algorithmic",
          flush=True)
    return us


def bench_mvm(m, k, n, noisy=False, bfp=False, iters=10, device="cuda:0"):
    dev = torch.device(device)
    eng = _engine(dev, noisy)
    x = torch.randn(m, k, device=dev)
    w = torch.randn(k, n, device=dev)
    xs, ws = _input(dev, bfp), _weight(dev, bfp)
    ws.slice_data_imp(eng, w)
    xs.slice_data_imp(eng, x)
    for _ in range(3):
        eng(xs, ws)
    torch.cuda.synchronize(dev)
    eng.launch_log = []
    for _ in range(iters):
        eng(xs, ws)
    torch.cuda.synchronize(dev)
    N.device_status()
    log, eng.launch_log = eng.launch_log, None
    ms = sorted(a.elapsed_time(b) for a, b, _, _ in log)[len(log) // 2]
    ops, adc = log[0][2], log[0][3]
    print(f"mvm m={m} k={k} n={n} noisy={noisy} bfp={bfp}: {ms:.3f} ms, {ops / ms / 1e9:.1f} slice-pair TOPS, "
          f"{adc / ms / 1e9:.3f} T ADC events/s", flush=True)
    return ms


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="kernel", required=True)
    s = sub.add_parser("slice")
    s.add_argument("--rows", type=int, default=16384)
    s.add_argument("--cols", type=int, default=3072)
    s.add_argument("--bfp", action="store_true")
    s.add_argument("--iters", type=int, default=20)
    v = sub.add_parser("mvm")
    v.add_argument("--m", type=int, default=4096)
    v.add_argument("--k", type=int, default=4096)
    v.add_argument("--n", type=int, default=4096)
    v.add_argument("--noisy", action="store_true")
    v.add_argument("--bfp", action="store_true")
    v.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    if a.kernel == "slice":
        bench_slice(a.rows, a.cols, a.bfp, a.iters)
    else:
        bench_mvm(a.m, a.k, a.n, a.noisy, a.bfp, a.iters)


if __name__ == "__main__":
    main()
