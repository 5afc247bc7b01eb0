"""Benchmark: CIM Qwen3-0.6B-architecture prefill on B200 (tokens/s), one process per GPU.

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference] [--tp T]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload: 8 sequences x 2048 token ids, uniform over the 151936-token
vocabulary (seeded synthetic data), through a random-init Qwen3-0.6B
architecture (28 layers, hidden 1024, 16/8 heads x 128, SwiGLU 3072) whose
197 linears (q/k/v/o, gate/up/down x 28 and lm_head) all run on the CIM
engine: slices [1,1,2,2,2], weight quant_gran (128,128) / paral (32,32),
input quant_gran (1,128) / paral (1,32), radc 4096, and the device model of
the reference's Qwen3 example (HGS 1e-5, LGS 1e-8, 4 levels, rdac 4, read
variation 0.05).  A step is one full prefill forward with loss.

With N GPUs the headline layout is data parallel over the 8 sequences: every
rank holds all decoder-layer crossbars and a 1/N column shard of lm_head, so
the only collectives are an all-gather of the final hidden states (8 MB per
rank) and the loss's log-sum-exp all-reduces (``--no-head-shard``: a whole
lm_head on every rank, no collective but the loss mean).  ``--tp T`` shards
every crossbar over groups of T ranks instead.  At N > 1 the
line also carries ``tp``: the same workload with every crossbar sharded over
all N ranks (column-sharded q/k/v, gate/up and lm_head, row-sharded o and
down), and ``layout_check``: the noise-free loss of both layouts, which must
agree to fp32 summation order.

``--impl reference`` times the reference's algorithm (the oracle's torch
restatement of ``_dot_inference``) on the host cores on a bounded sample of
the same workload and extrapolates to the metric's unit; with a GPU present it
also times the same restatement on cuda:0 (``reference_gpu``).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "CIM Qwen3-0.6B-arch prefill tokens/s (8x2048, all 197 linears on the CIM engine)"
# q/k/v and gate/up of a layer share their input and run as one crossbar array each (exact: output
# columns are independent), so a forward launches 4 CIM matmuls per layer + lm_head.
BATCH, SEQ = 8, 2048
ENGINE = dict(HGS=1e-5, LGS=1e-8, write_variation=0.0, rate_stuck_HGS=0.0, rate_stuck_LGS=0.0,
              read_variation=0.05, vnoise=0.0, rdac=4, g_level=4, radc=4096)
ARCH = dict(hidden=1024, layers=28, heads=16, kv_heads=8, head_dim=128, intermediate=3072, vocab=151936)

# (K, N) of the CIM linears of one decoder layer, and of lm_head
LAYER_LINEARS = [(1024, 2048), (1024, 1024), (1024, 1024), (2048, 1024), (1024, 3072), (1024, 3072), (3072, 1024)]
LM_HEAD = (1024, 151936)


def ops_per_token():
    """Slice-pair ops per token: 2 * Kp * Np * Sx * Sy summed over every CIM linear."""
    pad = lambda v: math.ceil(v / 128) * 128
    tot = sum(pad(k) * pad(n) for k, n in LAYER_LINEARS) * ARCH["layers"] + pad(LM_HEAD[0]) * pad(LM_HEAD[1])
    return 2.0 * tot * 25


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------------------------------------
# CPU baseline: the oracle (CPU restatement of the reference algorithm), bounded sample
# ---------------------------------------------------------------------------------------------
def cpu_sample(tokens: int = 256, head_cols: int = 4096, seed: int = 0):
    """Time one decoder layer's 7 CIM linears plus a lm_head column slice on `tokens` tokens.

    Returns (seconds, slice_pair_ops) of the sample.  The per-linear work is the
    reference's _dot_inference arithmetic (fp32 slice-pair crossbar sums, ADC,
    shift-add, block rescale, read noise) restated with torch's CPU kernels
    (oracle.cim_oracle.mvm_float_torch); slicing is included.
    """
    import torch
    from oracle import cim_oracle as O
    rng = np.random.default_rng(seed)
    eng = O.Engine(**{k: v for k, v in ENGINE.items()})
    sm = [1, 1, 2, 2, 2]
    shapes = LAYER_LINEARS + [(LM_HEAD[0], head_cols)]
    prepared = []
    for k, n in shapes:
        w = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
        x = rng.standard_normal((tokens, k)).astype(np.float32)
        prepared.append((x, w))
    t0 = time.perf_counter()
    ops = 0.0
    for x, w in prepared:
        xs = O.slice_matrix(x, sm, None, (1, 32), (1, 128))
        ws = O.slice_matrix(w, sm, None, (32, 32), (128, 128))
        O.mvm_float_torch(xs, ws, eng, seed=seed, noisy=True)
        ops += 2.0 * x.shape[0] * xs.geom.cols_p * ws.geom.cols_p * 25
    return time.perf_counter() - t0, ops


def cpu_baseline(target_s: float = 12.0):
    import torch
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    sec, ops = cpu_sample()
    reps = 1
    while sec * reps < target_s and reps < 8:
        s2, _ = cpu_sample(seed=reps)
        sec += s2
        reps += 1
    rate = ops * reps / sec
    return {"value": rate / ops_per_token(), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{reps}x (one decoder layer's 7 CIM linears + a 1024x4096 lm_head slice, 256 tokens), "
                      f"torch-CPU restatement of _dot_inference with read noise, extrapolated by slice-pair op "
                      f"count ({ops_per_token():.3e} ops/token)"}


# ---------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                smax = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
def gpu_reference_sample(tokens: int = 2048, head_cols: int = 4096, seed: int = 0, reps: int = 2):
    """The reference's algorithm on cuda:0: the torch restatement of ``_dot_inference`` (per slice pair a
    batched contraction into a (Kt, M, Np) partial, ADC, shift-add, block rescale, K-tile sum, read noise
    per call) over one decoder layer's 7 linears plus a lm_head column slice on ``tokens`` tokens.
    Operands are prepared (sliced) beforehand and only the device work is timed, which flatters the
    reference.  Returns (seconds per pass, slice-pair ops per pass)."""
    import torch
    from oracle import cim_oracle as O
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(seed)
    eng = O.Engine(**ENGINE)
    sm = [1, 1, 2, 2, 2]
    prepared, ops = [], 0.0
    for k, n in LAYER_LINEARS + [(LM_HEAD[0], head_cols)]:
        w = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
        x = rng.standard_normal((tokens, k)).astype(np.float32)
        xs = O.slice_matrix(x, sm, None, (1, 32), (1, 128))
        ws = O.slice_matrix(w, sm, None, (32, 32), (128, 128))
        prepared.append(O.torch_port_operands(xs, ws, eng, dev))
        ops += 2.0 * tokens * xs.geom.cols_p * ws.geom.cols_p * 25
    for o in prepared:                                   # warm-up
        O.torch_port_mvm(o, eng, seed)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for r in range(reps):
        for o in prepared:
            O.torch_port_mvm(o, eng, seed + r)
    e1.record()
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / 1000.0 / reps, ops


def run_reference(args):
    """--impl reference: the reference's algorithm on the host cores (and on cuda:0 when present),
    rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    import torch
    torch.set_num_threads(cores)
    for _ in range(args.warmup):
        cpu_sample(seed=99, tokens=32)
    times = []
    ops = 0.0
    for s in range(args.steps):
        sec, ops = cpu_sample(seed=s)
        times.append(sec)
    rate = ops * len(times) / sum(times)
    value = rate / ops_per_token()
    sample = ("per step: one decoder layer's 7 CIM linears + 1024x4096 lm_head slice on 256 tokens (torch "
              "restatement of _dot_inference with read noise, slicing included), extrapolated by slice-pair op "
              "count")
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "n_cores": cores,
            "impl": "reference", "config": dict(base_config(), parallelism="cpu (host cores)", sample=sample),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if torch.cuda.is_available():
        sec, gops = gpu_reference_sample()
        line["reference_gpu"] = {
            "value": gops / sec / ops_per_token(), "unit": "tokens/s", "device": torch.cuda.get_device_name(0),
            "kind": "port", "sliced_mvm_tops": gops / sec / 1e12,
            "sample": "one decoder layer's 7 CIM linears + 1024x4096 lm_head slice on 2048 tokens, the torch "
                      "restatement of _dot_inference on cuda:0 (MVM device work only, operands pre-sliced), "
                      "extrapolated by slice-pair op count"}
    print(json.dumps(line), flush=True)


def base_config():
    """The workload keys both arms report."""
    return {"workload": "Qwen3-0.6B-arch CIM prefill, 8x2048 tokens, 197 CIM linears",
            "model": "Qwen3-0.6B-arch (random init)", "global_batch": BATCH, "seq_len": SEQ, "engine": ENGINE}


def dp_tp_layout(world, rank, batch, tp=0):
    """(tp, dp, tp groups as rank lists, this rank's [first, end) sequence range).  Ranks form dp groups
    of tp consecutive ranks; tp == 0 picks pure data parallelism when the batch divides by the rank
    count, else one group of all ranks."""
    if tp <= 0:
        tp = 1 if batch % world == 0 else world
    if world % tp or batch % (world // tp):
        raise SystemExit(f"--tp {tp} does not divide {world} ranks into groups that split {batch} sequences")
    dp = world // tp
    per = batch // dp
    g = rank // tp
    return tp, dp, [list(range(r * tp, (r + 1) * tp)) for r in range(dp)], (g * per, (g + 1) * per)


# Epilogue ceiling of the fused MVM: every ADC event costs one integer multiply-add (FMA-heavy pipe) and
# half of a packed f32x2 rounding FMA, of which the FMA-heavy pipe takes half: 1.5 FMA-heavy lane operations
# per event at 64 lanes per clock per SM (16 per sub-partition) caps it at 42.7 events per SM clock.
MVM_FMAHEAVY_OPS_PER_ADC_EVENT = 1.5
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of each crossbar array of the
# one-GPU forward, captured with ncu at the bench's shapes and device model (profiles/mvm_dram_qwen3_shapes.md);
# lm_head counts as four launches of a quarter of its columns.  Averaged over the forward's 113 launches this
# is the roofline's per-launch traffic at N = 1 (other layouts run other shapes: reported as null there).
MVM_DRAM_BYTES_LAYER = {"qkv": 242.7e6 + 253.1e6, "o": 359.8e6 + 59.7e6, "gate_up": 673.8e6 + 379.0e6,
                        "down": 670.8e6 + 65.5e6}
MVM_DRAM_BYTES_LM_HEAD = 4 * (3448.9e6 + 2479.6e6)
MVM_DRAM_BYTES_PER_LAUNCH_1GPU = ((ARCH["layers"] * sum(MVM_DRAM_BYTES_LAYER.values()) + MVM_DRAM_BYTES_LM_HEAD)
                                  / (4 * ARCH["layers"] + 1))


class Layout:
    """One layout of the workload on this rank: a model, its process group and its share of the ids."""

    def __init__(self, model, ids_host, dev, world, group_world):
        self.model, self.world, self.group_world = model, world, group_world
        self.ids_host = ids_host
        self.ids = ids_host.to(dev)

    def step(self, x):
        """One prefill step: the group's mean loss, averaged over all ranks' groups."""
        import torch.distributed as dist
        loss = self.model(x)
        if self.world > 1:
            loss = loss.reshape(1)
            dist.all_reduce(loss)       # ranks of one group hold the same loss: the sum / world is the mean
            loss = loss[0] / self.world
        return loss


def barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def time_layout(lay: Layout, engine, args, world, local, dev, clocks=False):
    """Warm-up, then the device-resident timed region (CUDA events, max over ranks) and the end-to-end
    region (host ids in, host loss out, every step).  Returns a dict of measurements."""
    import torch
    import torch.distributed as dist
    from memintelli_flash_b200 import _native as N
    for _ in range(args.warmup):
        lay.step(lay.ids)
    barrier(world)
    engine.launch_log = []
    launches0 = N.launch_count()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local) if clocks else None
    if clk:
        clk.__enter__()
    barrier(world)
    t_start.record()
    for _ in range(args.steps):
        loss = lay.step(lay.ids)
    t_end.record()
    barrier(world)
    if clk:
        clk.__exit__()
    launches = N.launch_count() - launches0
    ms = t_start.elapsed_time(t_end)
    log, engine.launch_log = engine.launch_log, None
    mvm_ms = sum(a.elapsed_time(b) for a, b, _, _ in log)
    t = torch.tensor([ms, mvm_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t[0])
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        loss_host = lay.step(lay.ids_host.to(dev, non_blocking=True)).item()
    e1.record()
    barrier(world)
    e2e = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
    return dict(ms=ms_max, mvm_ms=mvm_ms, mvm_ops=sum(o for _, _, o, _ in log), mvm_adc=sum(e for _, _, _, e in log),
                launches=len(log), lib_launches=int(launches), e2e_ms=float(e2e[0]), loss=float(loss_host),
                clocks=clk.summary() if clk else None)


def run_b200(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        # high-priority NCCL streams: the overlapped all-reduces get SMs ahead of the queued MVM tiles
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300), pg_options=opts)

    from memintelli_flash_b200 import DPETensor
    from memintelli_flash_b200.qwen3_prefill import Qwen3Arch, Qwen3CimPrefill

    # dp x tp: ranks form dp groups of tp consecutive ranks; a group shards every crossbar across its tp
    # ranks (crossbar_shard) and takes BATCH/dp of the sequences.  --tp 0 picks pure dp when the batch
    # divides by the rank count (no collective on the data path), else pure tp.
    tp, dp, groups, (s0, s1) = dp_tp_layout(world, rank, BATCH, args.tp)
    tp_group = None
    if world > 1:
        for r, ranks in enumerate(groups):        # every rank creates every group, in the same order
            grp = dist.new_group(ranks)
            if rank // tp == r:
                tp_group = grp
    # one seed on every rank: each forward draws the same per-call read noise everywhere, so data-parallel
    # ranks compute rows of the single-GPU forward (one draw per linear shared by all sequences, as in one
    # reference call) instead of independent replicas
    torch.manual_seed(1234)
    engine = DPETensor(device=dev, **ENGINE)
    # pure data parallelism: lm_head (a quarter of the crossbar cells) is still column-sharded over all
    # ranks, which divides its programmed memory and per-call read-noise pass by the rank count
    head_shard = world > 1 and tp == 1 and not args.no_head_shard
    model = Qwen3CimPrefill(engine, Qwen3Arch(**ARCH), seed=0, device=dev, group=tp_group,
                            shard_head_over=dist.group.WORLD if head_shard else None)
    model.prefetch_noise = args.noise_prefetch
    torch.cuda.synchronize()
    g = torch.Generator().manual_seed(1)
    ids_all = torch.randint(0, ARCH["vocab"], (BATCH, SEQ), generator=g).pin_memory()
    head = Layout(model, ids_all[s0:s1], dev, world, tp)
    r = time_layout(head, engine, args, world, local, dev, clocks=True)

    # the fully sharded layout (every crossbar over all ranks) and the layout check, at N > 1
    tp_line = None
    if world > 1 and tp != world and not args.no_tp_compare:
        model_tp = Qwen3CimPrefill(engine, Qwen3Arch(**ARCH), seed=0, device=dev, group=None)
        model_tp.prefetch_noise = args.noise_prefetch
        full = Layout(model_tp, ids_all, dev, world, world)
        rt = time_layout(full, engine, args, world, local, dev)
        # noise-free, both layouts compute the same losses up to fp32 summation order
        saved = engine.read_variation
        engine.read_variation = {i: 0.0 for i in range(engine.g_level)}
        loss_head = float(head.step(head.ids))
        loss_full = float(full.step(full.ids))
        engine.read_variation = saved
        tp_line = {"value": BATCH * SEQ * args.steps / (rt["ms"] / 1000.0), "unit": "tokens/s",
                   "parallelism": f"dp1xtp{world}", "ms_per_step": rt["ms"] / args.steps,
                   "e2e": BATCH * SEQ * args.steps / (rt["e2e_ms"] / 1000.0),
                   "mvm_share": rt["mvm_ms"] / rt["ms"] if rt["ms"] else None}
        layout_check = {"noise_free_loss": {f"dp{dp}xtp{tp}": loss_head, f"dp1xtp{world}": loss_full},
                        "rel_diff": abs(loss_head - loss_full) / abs(loss_full)}
        del model_tp, full

    ms = r["ms"]
    tokens = BATCH * SEQ * args.steps
    value = tokens / (ms / 1000.0)
    peaks, peak_kind = load_peaks()
    mvm_ms = r["mvm_ms"]
    achieved = r["mvm_ops"] / (mvm_ms / 1000.0) / 1e12 if mvm_ms > 0 else 0.0
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    clocks = r["clocks"]
    sm_clock = clocks["sm_mhz"] or 1965.0
    epi_ceiling = 148 * (64.0 / MVM_FMAHEAVY_OPS_PER_ADC_EVENT) * sm_clock * 1e6   # ADC events / s
    adc_rate = r["mvm_adc"] / (mvm_ms / 1000.0) if mvm_ms else 0.0
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
                "data": "synthetic",
                "config": dict(base_config(), parallelism=(f"dp{dp}xtp{tp}" + (f", lm_head column-sharded x{world}" if head_shard else ""))
                                if world > 1 else "single",
                               l2="inputs larger than L2 (3 GB of programmed crossbars per forward)"),
                "sliced_mvm_tops": ops_per_token() * tokens / (ms / 1000.0) / 1e12,
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                             "frac": achieved / peak,
                             "traffic": MVM_DRAM_BYTES_PER_LAUNCH_1GPU if world == 1 else None,
                             "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch of each "
                                               "array shape, averaged over one forward's launches"
                                               if world == 1 else "not captured for this layout's shapes",
                             "peak_kind": f"bf16 sustained ({peak_kind})",
                             "kernel": "mvm_kernel (fused crossbar MVM)", "launches": r["launches"],
                             "kernel_share": mvm_ms / ms if ms else None,
                             "epilogue": {"adc_events_per_s": adc_rate, "ceiling_per_s": epi_ceiling,
                                          "frac": adc_rate / epi_ceiling,
                                          "ceiling": "FMA-heavy pipe, "
                                                     f"{MVM_FMAHEAVY_OPS_PER_ADC_EVENT} lane ops per ADC event"}},
                "e2e": {"value": tokens / (r["e2e_ms"] / 1000.0), "unit": "tokens/s",
                        "h2d_bytes_per_step": (s1 - s0) * SEQ * 8 * world,      # every rank copies its ids
                        "d2h_bytes_per_step": 4},
                "gpu_launches": r["lib_launches"],
                "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
                "loss": r["loss"]}
        if tp_line is not None:
            line["tp"] = tp_line
            line["layout_check"] = layout_check
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    del model, head
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp-compare", action="store_true",
                    help="at N > 1, skip the fully sharded layout's measurement and the layout check")
    ap.add_argument("--noise-prefetch", action="store_true",
                    help="run each layer's read-noise pass in the background of the layer before it "
                         "(measured slower on B200)")
    ap.add_argument("--no-head-shard", action="store_true",
                    help="data parallel layout: keep a whole lm_head on every rank")
    ap.add_argument("--tp", type=int, default=0,
                    help="ranks per crossbar-sharding group (0: pure data parallel when the batch divides by the "
                         "rank count, else all ranks shard)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
