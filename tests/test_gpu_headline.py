"""Parity at the shapes and operand types of the Qwen3-0.6B-architecture prefill benchmark (needs a B200).

The benchmark's crossbar arrays per decoder layer are q/k/v fused (K 1024, N 4096), o (2048 -> 1024),
gate/up fused (1024 -> 6144) and down (3072 -> 1024), plus lm_head (1024 -> 151936), over 16384 rows
on one GPU and 2048 rows per rank at 8-way data parallelism.  Two work divisions beyond whole output
tiles are exercised: the wave-balancing split-K (the 1024-column outputs at 2048 rows) and the tail
split of the persistent launch (a last wave at most half full, cut into K ranges: q/k/v at 2048 and
16384 rows, o and down at 16384 rows).  Its engine has read variation 0.05 and no voltage noise, so the MVM runs
FP16 operands (``kind::f16``): inputs are sliced straight into FP16 planes and the weight planes
come from the read-noise pass.

Here every one of those shapes runs on the GPU in full, noise-free, through both operand types:
* E4M3 through the public API (``DPETensor`` with the benchmark's slicing, read variation 0);
* FP16 through the C ABI exactly as the benchmark's engine launches it (its device spec, hence its
  ADC plan and flush interval), with the weight planes converted by the read-noise pass at sigma 0.
128 rows spread over every 128-row tile are compared with the oracle (rows are independent: input
quant blocks are one row high), bit-exact in the per-tile integer sums where the dump is taken and
within 1e-5 (norm) / 2e-6 of the output scale (elementwise) in the output.
"""
import zlib

import numpy as np
import pytest
import torch

from helpers import rel_norm
from oracle import cim_oracle as O

pytestmark = pytest.mark.gpu

SM = [1, 1, 2, 2, 2]
BENCH_ENGINE = dict(HGS=1e-5, LGS=1e-8, write_variation=0.0, rate_stuck_HGS=0.0, rate_stuck_LGS=0.0,
                    read_variation=0.05, vnoise=0.0, rdac=4, g_level=4, radc=4096)
NOISE_FREE = dict(BENCH_ENGINE, read_variation=0.0)

# (name, rows, K, N, work division: "split" = wave-balancing split-K, "tail" = tail split, None = whole tiles)
SHAPES = [
    ("down_dp8", 2048, 3072, 1024, "split"),
    ("o_dp8", 2048, 2048, 1024, "split"),
    ("gate_up_dp8", 2048, 1024, 6144, None),
    ("qkv_dp8", 2048, 1024, 4096, "tail"),
    ("qkv_full", 16384, 1024, 4096, "tail"),
    ("o_full", 16384, 2048, 1024, "tail"),
    ("down_full", 16384, 3072, 1024, "tail"),
]


def _division(M, N, floats):
    """Which division a workspace size means: split-K partials are whole M x N outputs."""
    if floats == 0:
        return None
    return "split" if floats % (M * N) == 0 and floats >= 2 * M * N else "tail"


def _rows(M, n=128):
    step = M // n
    return np.array([k * step + (k * 37) % step for k in range(n)])


def _inputs(M, K, N, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    w = torch.randn(K, N, generator=g) * 0.02
    return x, w


def _sliced(M_, eng, x, w, dev):
    xs = M_.SlicedData(torch.tensor(SM), is_weight=False, paral_size=(1, 32), quant_gran=(1, 128), device=dev,
                       inference=True)
    ws = M_.SlicedData(torch.tensor(SM), is_weight=True, paral_size=(32, 32), quant_gran=(128, 128), device=dev,
                       inference=True)
    ws.slice_data_imp(eng, w.to(dev))
    xs.slice_data_imp(eng, x.to(dev))
    return xs, ws


def _oracle(x, w, rows):
    oxs = O.slice_matrix(x[rows].numpy(), SM, None, (1, 32), (1, 128))
    ows = O.slice_matrix(w.numpy(), SM, None, (32, 32), (128, 128))
    return O.mvm_exact(oxs, ows, O.Engine(**NOISE_FREE), return_parts=True)


def _check(y_rows, ref):
    assert rel_norm(y_rows, ref) <= 1e-5
    assert np.max(np.abs(y_rows - ref)) <= 2e-6 * (np.abs(ref).max() + 1e-30)


@pytest.mark.parametrize("name,M,K,N,division", SHAPES)
def test_bench_shape_e4m3_matches_oracle(name, M, K, N, division, cuda):
    import memintelli_flash_b200 as M_
    from memintelli_flash_b200 import _native as N_
    eng = M_.DPETensor(device=cuda, **NOISE_FREE)
    x, w = _inputs(M, K, N, seed=zlib.crc32(name.encode()) % 1000)
    xs, ws = _sliced(M_, eng, x, w, cuda)
    f = N_.c_i64(0)
    N_.call("mib_mvm_workspace", M, N, xs._spec(), ws._spec(), xs._kgeom(), eng._device_spec(), f)
    assert _division(M, N, f.value) == division
    rows = _rows(M)
    dump = None
    if M <= 2048:                              # per-tile integer sums of every row (Kt x M x N int32)
        dump = torch.zeros((xs._buf["geom"]["kt"], M, N), dtype=torch.int32, device=cuda)
        eng.MapReduceDot(xs, ws, acc_dump=dump)
    y = eng(xs, ws)
    torch.cuda.synchronize()
    ref, acc, _ = _oracle(x, w, rows)
    _check(y[torch.from_numpy(rows).to(cuda)].double().cpu().numpy(), ref)
    if dump is not None:
        got = dump[:, torch.from_numpy(rows).to(cuda), :].cpu().numpy().astype(np.int64)
        assert np.array_equal(got, acc[:, : len(rows), :N])
    N_.device_status()


def _mvm_fp16_like_bench(eng_bench, xs, ws, out, dev):
    """Launch the MVM the way the benchmark engine does (FP16 planes, its device spec and workspace),
    with the weight planes converted by the read-noise pass at sigma 0 (exact levels)."""
    from memintelli_flash_b200 import _native as N_
    assert xs._buf["planes"].dtype == torch.float16        # sliced straight to FP16 (no voltage noise)
    gx, gw = xs._buf["geom"], ws._buf["geom"]
    M, Nc = gx["batch"] * gx["rows"], gw["n"]
    exact = N_.DeviceSpec.from_buffer_copy(eng_bench._device_spec())
    exact.read_sigma[0] = 0.0
    b16 = torch.empty(ws._buf["planes"].shape, dtype=torch.float16, device=dev)
    N_.call("mib_weight_read_noise", N_.ptr(ws._buf["planes"]), None, N_.ptr(b16), b16.numel(), exact, 1, 0,
            N_.stream_ptr(dev))
    xspec, wspec, kg, dspec = xs._spec(), ws._spec(), xs._kgeom(), eng_bench._device_spec()
    _, table, tlen = eng_bench._plan(xspec, wspec, kg, dspec, dev)
    f = N_.c_i64(0)
    N_.call("mib_mvm_workspace", M, Nc, xspec, wspec, kg, dspec, f)
    ws_buf = torch.empty(f.value, dtype=torch.float32, device=dev) if f.value else None
    N_.call("mib_mvm", N_.ptr(xs._buf["planes"]), N_.ptr(xs._buf["tile_scale"]), M, xspec, N_.ptr(b16),
            N_.ptr(ws._buf["tile_scale"]), Nc, wspec, kg, dspec, N_.OPERAND_FP16, N_.ptr(table), tlen, N_.ptr(out),
            N_.OutLayout(M, 0, Nc, 1), None, None, N_.ptr(ws_buf), f.value, N_.stream_ptr(dev))
    return f.value


@pytest.mark.parametrize("name,M,K,N,division", SHAPES)
def test_bench_shape_fp16_kernel_matches_oracle(name, M, K, N, division, cuda):
    import memintelli_flash_b200 as M_
    eng = M_.DPETensor(device=cuda, **BENCH_ENGINE)
    x, w = _inputs(M, K, N, seed=zlib.crc32(name.encode()) % 1000 + 1)
    xs, ws = _sliced(M_, eng, x, w, cuda)
    out = torch.full((M, N), float("nan"), device=cuda)
    used = _mvm_fp16_like_bench(eng, xs, ws, out, cuda)
    assert _division(M, N, used) == division
    torch.cuda.synchronize()
    rows = _rows(M)
    ref, _, _ = _oracle(x, w, rows)
    _check(out[torch.from_numpy(rows).to(cuda)].double().cpu().numpy(), ref)
    assert torch.isfinite(out).all()


def test_lm_head_columns_equal_a_separately_programmed_slice(cuda):
    """The full 1024 x 151936 lm_head at 2048 rows: its last 4096 columns equal a crossbar array programmed
    from just those columns (output columns are independent; the two launches differ only in which tiles
    take the tail split, i.e. in the fp32 order of the K-range partial sums), and those equal the oracle
    on 128 rows."""
    import memintelli_flash_b200 as M_
    eng = M_.DPETensor(device=cuda, **NOISE_FREE)
    M, K, V, S = 2048, 1024, 151936, 4096
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(M, K, generator=g, device=cuda)
    w = torch.randn(K, V, generator=g, device=cuda) * 0.02
    xs, ws_full = _sliced(M_, eng, x, w, cuda)
    y_full = eng(xs, ws_full)
    del ws_full
    w_tail = w[:, V - S:].contiguous()
    _, ws_tail = _sliced(M_, eng, x[:1], w_tail, cuda)
    y_tail = eng(xs, ws_tail)
    torch.cuda.synchronize()
    a, b = y_full[:, V - S:], y_tail
    assert (a - b).abs().max().item() <= 2e-6 * b.abs().max().item()
    assert (a == b).float().mean().item() > 0.9               # only tail-split tiles differ at all
    rows = _rows(M)
    ref, _, _ = _oracle(x.cpu(), w_tail.cpu(), rows)
    _check(y_tail[torch.from_numpy(rows).to(cuda)].double().cpu().numpy(), ref)


def test_bench_engine_forward_is_deterministic_per_seed(cuda):
    """Two calls under the same torch seed draw the same read noise and give bit-identical outputs;
    another seed gives another draw."""
    import memintelli_flash_b200 as M_
    eng = M_.DPETensor(device=cuda, **BENCH_ENGINE)
    x, w = _inputs(2048, 3072, 1024, seed=9)
    xs, ws = _sliced(M_, eng, x, w, cuda)
    torch.manual_seed(11)
    a = eng(xs, ws)
    torch.manual_seed(11)
    b = eng(xs, ws)
    torch.manual_seed(12)
    c = eng(xs, ws)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert not torch.equal(a, c)


def test_resnet18_cifar_stage1_conv_matches_oracle(cuda):
    """Config 2 at full size: a ResNet-18-CIFAR stage-1 conv (64 -> 64 channels, 3x3, padding 1) on 128 images of
    30x30, block floating point (bw_e 8), radc 1024 (the per-slice code-table ADC), x (1,64)/(1,32),
    W (64,64)/(32,32): 115200 output pixels x 576 patch columns, sliced straight from NCHW.  Rows are output
    pixels; 128 of them, spread over all images, equal the oracle on F.unfold's columns."""
    import torch.nn.functional as F
    import memintelli_flash_b200 as M_
    from memintelli_flash_b200.NN_layers import Conv2dMem
    eng = M_.DPETensor(device=cuda, **dict(NOISE_FREE, radc=1024))
    torch.manual_seed(2)
    layer = Conv2dMem(eng, 64, 64, 3, SM, SM, stride=1, padding=1, bias=False, device=cuda, bw_e=8,
                      input_paral_size=(1, 32), weight_paral_size=(32, 32), input_quant_gran=(1, 64),
                      weight_quant_gran=(64, 64))
    layer.inference_mode = True
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(128, 64, 30, 30, generator=g, device=cuda)
    y = layer(x)                                                  # (128, 64, 30, 30)
    torch.cuda.synchronize()
    rows = _rows(128 * 900)
    xu = F.unfold(x, 3, padding=1).transpose(1, 2).reshape(-1, 576)[torch.from_numpy(rows).to(cuda)]
    wm = layer.weight.detach().reshape(64, -1).t().contiguous()
    oxs = O.slice_matrix(xu.cpu().numpy(), SM, 8, (1, 32), (1, 64))
    ows = O.slice_matrix(wm.cpu().numpy(), SM, 8, (32, 32), (64, 64))
    ref = O.mvm_exact(oxs, ows, O.Engine(**dict(NOISE_FREE, radc=1024)))
    got = y.permute(0, 2, 3, 1).reshape(-1, 64)[torch.from_numpy(rows).to(cuda)].double().cpu().numpy()
    _check(got, ref)


def test_deit_small_qkv_k64_matches_oracle(cuda):
    """Config 3 at full size: the DeiT-S q/k/v crossbar (384 -> 1152) over 64 x 197 = 12608 tokens with 64-deep
    crossbar tiles (x (1,64)/(1,64), W (64,64)/(64,64)), INT, radc 4096, noise-free."""
    import memintelli_flash_b200 as M_
    eng = M_.DPETensor(device=cuda, **NOISE_FREE)
    x, w = _inputs(12608, 384, 1152, seed=21)
    xs = M_.SlicedData(torch.tensor(SM), is_weight=False, paral_size=(1, 64), quant_gran=(1, 64), device=cuda,
                       inference=True)
    ws = M_.SlicedData(torch.tensor(SM), is_weight=True, paral_size=(64, 64), quant_gran=(64, 64), device=cuda,
                       inference=True)
    ws.slice_data_imp(eng, w.to(cuda))
    xs.slice_data_imp(eng, x.to(cuda))
    y = eng(xs, ws)
    torch.cuda.synchronize()
    rows = _rows(12608, n=97)
    oxs = O.slice_matrix(x[rows].numpy(), SM, None, (1, 64), (1, 64))
    ows = O.slice_matrix(w.numpy(), SM, None, (64, 64), (64, 64))
    ref = O.mvm_exact(oxs, ows, O.Engine(**NOISE_FREE))
    _check(y[torch.from_numpy(rows).to(cuda)].double().cpu().numpy(), ref)
