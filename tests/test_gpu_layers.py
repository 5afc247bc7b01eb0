"""LinearMem / Conv2dMem on the B200 path against the reference layers' golden outputs (needs a B200)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import golden_cases as G
from helpers import rel_norm
from oracle import cim_oracle as O

pytestmark = pytest.mark.gpu


def _oracle_layer(c):
    """Exact restatement of the layer forward (unfold on the CPU for convolutions)."""
    s, g = c["spec"], c["golden"]
    x = torch.from_numpy(g["x"])
    w = torch.from_numpy(g["weight"])
    if s["kind"] == "conv":
        xu = F.unfold(x, s["k"], stride=s["stride"], padding=s["padding"]).transpose(1, 2).contiguous().numpy()
        wm = w.reshape(w.shape[0], -1).t().contiguous().numpy()
    else:
        xu = x.numpy()
        wm = w.t().contiguous().numpy()
    xq = s["xq"] if isinstance(s["xq"], str) else tuple(s["xq"])
    wq = s["wq"] if isinstance(s["wq"], str) else tuple(s["wq"])
    xs = O.slice_matrix(xu, s["sx"], s["bw_e"], tuple(s["xp"]), xq)
    ws = O.slice_matrix(wm, s["sw"], s["bw_e"], tuple(s["wp"]), wq)
    eng = O.Engine(**c["eng"])
    wl = O.weight_levels(ws, eng)
    y = O.mvm_exact(xs, ws, eng, wl)
    b = O.tie_bound(xs, ws, eng, wl)
    if "bias" in g:
        y = y + g["bias"].astype(np.float64)
    if s["kind"] == "conv":
        n, _, h, wd = s["x"]
        ho = (h + 2 * s["padding"] - s["k"]) // s["stride"] + 1
        wo = (wd + 2 * s["padding"] - s["k"]) // s["stride"] + 1
        y = y.transpose(0, 2, 1).reshape(n, -1, ho, wo)
        b = b.transpose(0, 2, 1).reshape(n, -1, ho, wo)
    return y, b


def _gpu_layer(c, cuda):
    import memintelli_flash_b200 as M
    s, g = c["spec"], c["golden"]
    eng = M.DPETensor(device=cuda, **c["eng"])
    kw = dict(bias=s["bias"], device=cuda, bw_e=s["bw_e"], input_paral_size=tuple(s["xp"]),
              weight_paral_size=tuple(s["wp"]), input_quant_gran=tuple(s["xq"]), weight_quant_gran=tuple(s["wq"]))
    if s["kind"] == "conv":
        layer = M.Conv2dMem(eng, s["cin"], s["cout"], s["k"], s["sx"], s["sw"], stride=s["stride"],
                            padding=s["padding"], **kw)
    else:
        layer = M.LinearMem(eng, s["cin"], s["cout"], s["sx"], s["sw"], **kw)
    with torch.no_grad():
        layer.weight.copy_(torch.from_numpy(g["weight"]))
        if s["bias"]:
            layer.bias.copy_(torch.from_numpy(g["bias"]))
    layer.update_weight()
    if s["inference"]:
        layer.inference_mode = True
        layer.weight_sliced.inference = True
    return layer


@pytest.mark.parametrize("name", G.layer_names())
def test_layer_forward(name, cuda):
    c = G.layer_case(name)
    g = c["golden"]
    layer = _gpu_layer(c, cuda)
    x = torch.from_numpy(g["x"]).to(cuda)
    if not c["spec"]["inference"]:
        x.requires_grad_(True)
    y = layer(x)
    torch.cuda.synchronize()
    yg = y.detach().cpu().numpy().astype(np.float64)
    y_exact, bound = _oracle_layer(c)
    assert yg.shape == y_exact.shape
    assert rel_norm(yg, y_exact) <= 1e-5
    scale = np.abs(y_exact).max()
    assert np.all(np.abs(yg - g["y"]) <= bound + 2e-5 * scale)
    if not c["spec"]["inference"]:
        y.backward(torch.ones_like(y))
        assert rel_norm(x.grad.cpu().numpy(), g["grad_x"]) < 1e-5
        assert rel_norm(layer.weight.grad.cpu().numpy(), g["grad_w"]) < 1e-5
        if "grad_b" in g:
            assert rel_norm(layer.bias.grad.cpu().numpy(), g["grad_b"]) < 1e-5


def test_linear_errors(cuda):
    import memintelli_flash_b200 as M
    eng = M.DPETensor(device=cuda, HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=4096, vnoise=0.0,
                      read_variation=0.0, write_variation=0.0, rate_stuck_HGS=0.0)
    layer = M.LinearMem(eng, 64, 32, [1, 1, 2, 2, 2], [1, 1, 2, 2, 2], device=cuda)
    layer.inference_mode = True
    with pytest.raises(ValueError):
        layer(torch.randn(4, 65, device=cuda))


@pytest.mark.parametrize("bfp", [None, 8])
def test_conv_voltage_noise_fused_into_slicing_equals_separate_pass(bfp, cuda):
    """Conv2dMem with voltage noise slices its input once per multiply and applies that multiply's voltage
    noise while writing the FP16 planes (mib_slice_conv_input_noisy).  Under the same torch seed this equals,
    bit for bit, slicing to E4M3 and running the separate noise pass inside the multiply."""
    import memintelli_flash_b200 as M
    from memintelli_flash_b200.NN_layers import Conv2dMem
    eng = M.DPETensor(device=cuda, HGS=1e-5, LGS=1e-8, rdac=4, g_level=4, radc=1024, write_variation=0.0,
                      rate_stuck_HGS=0.0, rate_stuck_LGS=0.0, read_variation=0.05, vnoise=0.05)
    assert not eng.conv_input_noise_fused()          # opt-in
    eng.fuse_conv_input_noise = True
    assert eng.conv_input_noise_fused()
    torch.manual_seed(3)
    layer = Conv2dMem(eng, 16, 32, 3, [1, 1, 2, 2, 2], [1, 1, 2, 2, 2], stride=1, padding=1, bias=True,
                      device=cuda, bw_e=bfp, input_paral_size=(1, 32), weight_paral_size=(32, 32),
                      input_quant_gran=(1, 64), weight_quant_gran=(64, 64))
    layer.inference_mode = True
    x = torch.randn(4, 16, 12, 12, device=cuda)
    torch.manual_seed(11)
    y_fused = layer(x)
    # the separate path: E4M3 slicing, then the multiply draws the seed and runs the noise pass
    torch.manual_seed(11)
    xs = M.SlicedData(layer.input_slice_method, device=cuda, bw_e=bfp, is_weight=False, paral_size=(1, 32),
                      quant_gran=(1, 64), inference=True)
    xs._slice_conv_imp(eng, x, (3, 3), (1, 1), (1, 1), (1, 1))
    assert xs._buf["planes"].dtype == torch.uint8
    from memintelli_flash_b200 import _native as N
    out = torch.empty_like(y_fused)
    L = 12 * 12
    eng.MapReduceDot(xs, layer.weight_sliced, out=out, bias=layer.bias.detach().float(),
                     layout=N.OutLayout(L, 32 * L, 1, L))
    torch.cuda.synchronize()
    assert torch.equal(y_fused, out)
    # a second multiply with a fused-noise input would reuse its draw: rejected
    xs2 = M.SlicedData(layer.input_slice_method, device=cuda, bw_e=bfp, is_weight=False, paral_size=(1, 32),
                       quant_gran=(1, 64), inference=True)
    xs2._slice_conv_imp(eng, x, (3, 3), (1, 1), (1, 1), (1, 1), noise_seed=5)
    eng.MapReduceDot(xs2, layer.weight_sliced, out=out, layout=N.OutLayout(L, 32 * L, 1, L))
    with pytest.raises(ValueError, match="one multiply"):
        eng.MapReduceDot(xs2, layer.weight_sliced, out=out, layout=N.OutLayout(L, 32 * L, 1, L))
