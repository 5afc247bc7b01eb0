"""Shared helpers: build engine/operands from a golden case, on the GPU and in the oracle."""
import numpy as np
import torch

from oracle import cim_oracle as O
import golden_cases as G


def oracle_pair(c):
    s = c["spec"]
    xs = O.slice_matrix(c["x"], s["sx"], s["bw_e"], c["xp"], c["xq"])
    ws = O.slice_matrix(c["w"], s["sw"], s["bw_e"], c["wp"], c["wq"])
    eng = O.Engine(**c["eng"])
    wl = O.weight_levels(ws, eng, c["fields"].get("stuck"))
    return xs, ws, eng, wl


def gpu_pair(c, device, inference=None):
    import memintelli_flash_b200 as M
    s = c["spec"]
    eng = M.DPETensor(device=device, **c["eng"])
    eng.fault_field_device = "cpu"        # reproduce the CPU reference's fixed-seed fault draws
    inf = s["inference"] if inference is None else inference
    xs = M.SlicedData(torch.tensor(s["sx"]), bw_e=s["bw_e"], is_weight=False, paral_size=c["xp"],
                      quant_gran=c["xq"], device=device, inference=inf)
    ws = M.SlicedData(torch.tensor(s["sw"]), bw_e=s["bw_e"], is_weight=True, paral_size=c["wp"],
                      quant_gran=c["wq"], device=device, inference=False)
    ws.slice_data_imp(eng, torch.from_numpy(c["w"]).to(device))
    xs.slice_data_imp(eng, torch.from_numpy(c["x"]).to(device))
    return eng, xs, ws


def rel_norm(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
