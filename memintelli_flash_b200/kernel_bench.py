"""Micro-benchmarks of the two crossbar kernels, through the public API.

    python -m memintelli_flash_b200.kernel_bench slice --rows 16384 --cols 3072 [--bfp]
    python -m memintelli_flash_b200.kernel_bench mvm --m 4096 --k 4096 --n 4096 [--noisy]
    python -m memintelli_flash_b200.kernel_bench noise --k 1024 --n 151936 [--per-level]
    python -m memintelli_flash_b200.kernel_bench workload [--config 0 1 2 3]

The engine is the reference's example device (HGS 1e-5, LGS 1e-8, rdac 4, g_level 4,
radc 4096) with slices [1, 1, 2, 2, 2]: input tiles (1, 32) in (1, 128) quant blocks,
weight tiles (32, 32) in (128, 128) blocks. Each case runs 3 untimed calls, then times
`--iters` calls with CUDA events on the launching stream and prints one line:

* slice: time per call and algorithmic bytes/s, with bytes = 4 (fp32 read) + S (E4M3
  planes) + 4/p (tile scale) per element;
* mvm:   median MVM launch time, slice-pair ops/s and ADC events/s;
* workload: time per pass over the CIM layers of one of the reference's example workloads
  (`WORKLOADS`), with the MVM launches' share and throughput.

The inputs are randn; x is larger than L2 at the default sizes.
"""
import argparse

import torch

from . import _native as N
from .pimpy import DPETensor, SlicedData

SLICES = [1, 1, 2, 2, 2]


def _engine(device, noisy, read_only=False):
    """noisy: read variation and voltage noise 0.05; read_only: read variation 0.05 alone (the device model
    of the Qwen3 prefill bench, whose inputs are sliced straight into FP16 planes)."""
    return DPETensor(HGS=1e-5, LGS=1e-8, write_variation=0.0, rate_stuck_HGS=0.0, rate_stuck_LGS=0.0,
                     read_variation=0.05 if (noisy or read_only) else 0.0,
                     vnoise=0.05 if (noisy and not read_only) else 0.0,
                     rdac=4, g_level=4, radc=4096, device=device)


def _input(device, bfp):
    return SlicedData(torch.tensor(SLICES), bw_e=8 if bfp else None, is_weight=False, paral_size=(1, 32),
                      quant_gran=(1, 128), device=device, inference=True)


def _weight(device, bfp):
    return SlicedData(torch.tensor(SLICES), bw_e=8 if bfp else None, is_weight=True, paral_size=(32, 32),
                      quant_gran=(128, 128), device=device, inference=True)


def bench_slice(rows, cols, bfp=False, iters=20, device="cuda:0", fp16=False):
    """``fp16``: an engine whose only noise is read variation, which slices inputs straight into FP16 planes
    (the Qwen3 benchmark's input path); else E4M3 planes."""
    dev = torch.device(device)
    eng = _engine(dev, False)
    if fp16:
        eng.read_variation = {i: 0.05 for i in range(eng.g_level)}
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
    esz = xs._buf["planes"].element_size()
    nbytes = rows * cols * (4 + esz * len(SLICES) + 4 / 32)
    print(f"slice rows={rows} cols={cols} bfp={bfp} planes={'fp16' if esz == 2 else 'e4m3'}: {us:.1f} us/call, "
          f"{nbytes / us / 1e3:.0f} GB/s algorithmic", flush=True)
    return us


def bench_mvm(m, k, n, noisy=False, bfp=False, iters=10, device="cuda:0", read_only=False):
    dev = torch.device(device)
    eng = _engine(dev, noisy, read_only)
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
    print(f"mvm m={m} k={k} n={n} noisy={noisy} read_only={read_only} bfp={bfp}: {ms:.3f} ms, "
          f"{ops / ms / 1e9:.1f} slice-pair TOPS, "
          f"{adc / ms / 1e9:.3f} T ADC events/s", flush=True)
    return ms


def bench_noise(k, n, iters=20, per_level=False, device="cuda:0"):
    """Per-call noise passes over the planes of a programmed k x n weight (5 slices, E4M3 levels) and of a
    k-wide input of n rows: read variation (1 B level in, 2 B FP16 out per cell) and voltage noise (1 B in,
    2 B out per element).  Prints time per call and algorithmic GB/s."""
    dev = torch.device(device)
    sigma = {0: 0.02, 1: 0.05, 2: 0.05, 3: 0.1} if per_level else 0.05
    eng = DPETensor(HGS=1e-5, LGS=1e-8, write_variation=0.0, rate_stuck_HGS=0.0, rate_stuck_LGS=0.0,
                    read_variation=sigma, vnoise=0.05, rdac=4, g_level=4, radc=4096, device=dev)
    ws = _weight(dev, False)
    ws.slice_data_imp(eng, torch.randn(k, n, device=dev))
    planes = ws._buf["planes"]
    out = torch.empty(planes.shape, dtype=torch.float16, device=dev)
    spec = eng._device_spec()
    stream = N.stream_ptr(dev)
    res = {}

    def run(name, fn, nbytes):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1e3 / iters
        res[name] = (us, nbytes / us / 1e3)
        print(f"{name} {planes.numel() / 1e6:.1f} M cells: {us:.1f} us/call, {nbytes / us / 1e3:.0f} GB/s algorithmic",
              flush=True)

    run("read_noise" + ("_per_level" if per_level else ""), lambda: N.call(
        "mib_weight_read_noise", N.ptr(planes), None, N.ptr(out), planes.numel(), spec, 7, 1, stream),
        3 * planes.numel())
    run("input_noise", lambda: N.call("mib_input_noise", N.ptr(planes), N.ptr(out), planes.numel(), 0.05, 7, 1,
                                      stream), 3 * planes.numel())
    N.device_status()
    return res


# ----------------------------------------------------------------------------- layer workloads
# The CIM layers of the reference's example workloads, with random weights and inputs of the
# workloads' shapes (the datasets and trained weights are not used).  Normalisation, pooling and
# attention are left out: they do not run on the engine.

def _resnet18_cifar_convs():
    """(cin, cout, k, stride, pad, h_in) of ResNet-18 for 32x32 CIFAR inputs as
    memintelli/NN_models/resnet_cifar.py builds it: an unpadded 3x3 stem (32 -> 30), four stages of
    two BasicBlocks (64, 128, 256, 512 channels, stride 2 from the second stage on, 3x3 convs with
    padding 1) and a 1x1 stride-2 downsample conv at each stage change."""
    convs = [(3, 64, 3, 1, 0, 32)]
    h, cin = 30, 64
    for cout, stride in ((64, 1), (128, 2), (256, 2), (512, 2)):
        for b in range(2):
            s = stride if b == 0 else 1
            convs.append((cin, cout, 3, s, 1, h))
            ho = (h + 2 - 3) // s + 1
            convs.append((cout, cout, 3, 1, 1, ho))
            if s != 1 or cin != cout:
                convs.append((cin, cout, 1, s, 0, h))
            h, cin = ho, cout
    return convs


def _deit_small_linears():
    """(in, out) of DeiT-S's CIM linears: 12 blocks of qkv 384->1152, proj 384->384, fc1 384->1536,
    fc2 1536->384, then the 384->1000 head."""
    return [(384, 1152), (384, 384), (384, 1536), (1536, 384)] * 12 + [(384, 1000)]


WORKLOADS = {
    0: "example matmul: x 400x500 @ W 500x600, INT, radc 4096, stuck-at 1e-3, read and voltage noise 0.05",
    1: "MLP 784-512-128-10 on 256 inputs, INT, radc 4096, read and voltage noise 0.05",
    2: "ResNet-18-CIFAR convolutions + fc on 128x3x32x32, BFP (bw_e 8), radc 1024, x (1,64)/(1,32), "
       "W (64,64)/(32,32), read and voltage noise 0.05",
    3: "DeiT-S linears on 64x197 tokens, INT, radc 4096, K tile 64: x (1,64)/(1,64), W (64,64)/(64,64), "
       "noise-free",
}


def _workload(config, dev):
    """Returns (engine, run, macs): run() performs one pass over the workload's CIM layers."""
    from .NN_layers import Conv2dMem, LinearMem
    g = torch.Generator(device=dev).manual_seed(0)
    noisy = dict(read_variation=0.05, vnoise=0.05)
    if config == 3:
        noisy = dict(read_variation=0.0, vnoise=0.0)
    eng = DPETensor(HGS=1e-5, LGS=1e-8, write_variation=0.0, rate_stuck_HGS=1e-3 if config == 0 else 0.0,
                    rate_stuck_LGS=0.0, rdac=4, g_level=4, radc=1024 if config == 2 else 4096, device=dev, **noisy)
    if config == 0:
        x = torch.randn(400, 500, device=dev, generator=g)
        w = torch.randn(500, 600, device=dev, generator=g)
        ws = _weight(dev, False)
        ws.slice_data_imp(eng, w)

        def run():
            xs = _input(dev, False)
            xs.slice_data_imp(eng, x)
            return eng(xs, ws)
        return eng, run, 400 * 500 * 600
    if config == 1:
        dims = [784, 512, 128, 10]
        layers = [LinearMem(eng, a, b, SLICES, SLICES, device=dev, input_quant_gran=(1, 128),
                            weight_quant_gran=(128, 128)) for a, b in zip(dims[:-1], dims[1:])]
        for l in layers:
            l.inference_mode = True
        x = torch.rand(256, 784, device=dev, generator=g)

        def run():
            h = x
            for k, l in enumerate(layers):
                h = l(h)
                if k + 1 < len(layers):
                    h = torch.relu(h)
            return h
        return eng, run, 256 * sum(a * b for a, b in zip(dims[:-1], dims[1:]))
    if config == 2:
        kw = dict(bw_e=8, input_paral_size=(1, 32), weight_paral_size=(32, 32), input_quant_gran=(1, 64),
                  weight_quant_gran=(64, 64), device=dev)
        convs, macs = [], 0
        for cin, cout, k, s, p, h in _resnet18_cifar_convs():
            layer = Conv2dMem(eng, cin, cout, k, SLICES, SLICES, stride=s, padding=p, bias=False, **kw)
            layer.inference_mode = True
            xin = torch.randn(128, cin, h, h, device=dev, generator=g)
            ho = (h + 2 * p - k) // s + 1
            macs += 128 * ho * ho * cout * cin * k * k
            convs.append((layer, xin))
        fc = LinearMem(eng, 512, 100, SLICES, SLICES, **kw)
        fc.inference_mode = True
        feat = torch.randn(128, 512, device=dev, generator=g)
        macs += 128 * 512 * 100

        def run():
            out = None
            for layer, xin in convs:
                out = layer(xin)
            return out, fc(feat)
        return eng, run, macs
    if config == 3:
        kw = dict(input_paral_size=(1, 64), weight_paral_size=(64, 64), input_quant_gran=(1, 64),
                  weight_quant_gran=(64, 64), device=dev)
        layers, macs = [], 0
        inputs = {}
        for a, b in _deit_small_linears():
            l = LinearMem(eng, a, b, SLICES, SLICES, **kw)
            l.inference_mode = True
            if a not in inputs:
                inputs[a] = torch.randn(64, 197, a, device=dev, generator=g)
            layers.append(l)
            macs += 64 * 197 * a * b

        def run():
            out = None
            for l in layers:
                out = l(inputs[l.in_features])
            return out
        return eng, run, macs
    raise ValueError(f"unknown workload config {config}")


def bench_workload(config, iters=5, device="cuda:0"):
    dev = torch.device(device)
    eng, run, macs = _workload(config, dev)
    for _ in range(3):
        run()
    torch.cuda.synchronize(dev)
    eng.launch_log = []
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        run()
    e1.record()
    torch.cuda.synchronize(dev)
    N.device_status()
    log, eng.launch_log = eng.launch_log, None
    ms = e0.elapsed_time(e1) / iters
    mvm_ms = sum(a.elapsed_time(b) for a, b, _, _ in log) / iters
    ops = sum(o for _, _, o, _ in log) / iters
    print(f"workload {config} ({WORKLOADS[config]}): {ms:.3f} ms/pass, MVM {mvm_ms:.3f} ms "
          f"({len(log) // iters} launches), {2 * macs / ms / 1e9:.2f} logical TFLOP/s, "
          f"{ops / mvm_ms / 1e9:.1f} slice-pair TOPS in the MVM", flush=True)
    return ms


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="kernel", required=True)
    s = sub.add_parser("slice")
    s.add_argument("--rows", type=int, default=16384)
    s.add_argument("--cols", type=int, default=3072)
    s.add_argument("--bfp", action="store_true")
    s.add_argument("--iters", type=int, default=20)
    s.add_argument("--fp16", action="store_true")
    v = sub.add_parser("mvm")
    v.add_argument("--m", type=int, default=4096)
    v.add_argument("--k", type=int, default=4096)
    v.add_argument("--n", type=int, default=4096)
    v.add_argument("--noisy", action="store_true")
    v.add_argument("--read-noise-only", action="store_true",
                   help="read variation 0.05 without voltage noise, as in the Qwen3 prefill bench")
    v.add_argument("--bfp", action="store_true")
    v.add_argument("--iters", type=int, default=10)
    z = sub.add_parser("noise")
    z.add_argument("--k", type=int, default=1024)
    z.add_argument("--n", type=int, default=151936)
    z.add_argument("--per-level", action="store_true")
    z.add_argument("--iters", type=int, default=20)
    w = sub.add_parser("workload")
    w.add_argument("--config", type=int, nargs="+", default=[0, 1, 2, 3])
    w.add_argument("--iters", type=int, default=5)
    a = ap.parse_args(argv)
    if a.kernel == "slice":
        bench_slice(a.rows, a.cols, a.bfp, a.iters, fp16=a.fp16)
    elif a.kernel == "mvm":
        bench_mvm(a.m, a.k, a.n, a.noisy, a.bfp, a.iters, read_only=a.read_noise_only)
    elif a.kernel == "noise":
        bench_noise(a.k, a.n, a.iters, a.per_level)
    else:
        for c in a.config:
            bench_workload(c, a.iters)


if __name__ == "__main__":
    main()
