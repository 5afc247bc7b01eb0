"""``SlicedData``: bit-sliced, block-quantised operand of the CIM engine.

API mirror of memintelli/pimpy/data_formats.py:10-207 (same constructor,
attributes and ``slice_data_imp(engine, data)``), backed by device buffers
written by the native slicing / programming kernels:

* ``planes``      [S][rows][Kt*pp]  per-slice DAC levels (inputs) or conductance
                                    levels (weights), E4M3 or FP16;
* ``tile_scale``  [Kt][rows]        dequantisation factor per (tile, row);
* ``block_max`` / ``block_exp``     per quant block (``max_data`` / ``e_bias``);
* ``packed``      [rows][Kp] uint8  two's complement code of every element
                                    (kept when ``inference`` is False);
* ``g_planes``    [S][N][Kt*pp]     conductances when write variation is on.

The reference-layout tensors (``sliced_data``, ``quantized_data``,
``max_data``, ``e_bias``, ``G``) are produced from these on first access.
"""
from __future__ import annotations

import copy
import math

import torch

from .. import _native as N


def _decode_gran(quant_gran, paral_size, rows, cols):
    """data_formats.py:141-158: string granularities and rounding up to paral_size."""
    if quant_gran is None:
        quant_gran = paral_size
    if isinstance(quant_gran, str):
        if quant_gran == "per-matrix":
            qg = [rows, cols]
        elif quant_gran == "per-row":
            qg = [1, cols]
        elif quant_gran == "per-col":
            qg = [rows, 1]
        else:
            raise ValueError(f"unknown quant_gran {quant_gran!r}")
    else:
        qg = [int(quant_gran[0]), int(quant_gran[1])]
    p0, p1 = int(paral_size[0]), int(paral_size[1])
    qg[0] = math.ceil(qg[0] / p0) * p0
    qg[1] = math.ceil(qg[1] / p1) * p1
    return qg


def padded_tile(p: int, kind: int) -> int:
    """Crossbar tile depth padded so one tile row is 32, 64 or 128 bytes."""
    es = 1 if kind == N.OPERAND_E4M3 else 2
    for rb in (32, 64, 128):
        if p * es <= rb:
            return rb // es
    raise NotImplementedError(f"crossbar tile depth {p} exceeds {128 // es} for this operand type")


class SlicedData(object):
    """Sliced data with quantisation (memintelli/pimpy/data_formats.py:10-58)."""

    def __init__(self, slice_method: torch.Tensor, bw_e=None, is_weight=False, paral_size=(64, 64),
                 quant_gran=None, device=None, inference=False):
        self.bw_e = bw_e
        self.is_weight = is_weight
        self.device = torch.device('cpu') if device is None else device
        self.shape = None
        self.inference = inference
        self.paral_size = paral_size
        self.quant_gran = paral_size if quant_gran is None else quant_gran
        sm = slice_method.tolist() if torch.is_tensor(slice_method) else [int(v) for v in slice_method]
        if sm[0] != 1:
            raise ValueError('The first bit of the slice method should be 1')
        self.slice_method = slice_method
        self._overrides = {}
        self._cache = {}
        self._buf = None
        self._init_data(sm, device)
        self._sm_src = slice_method

    def _init_data(self, slice_method, device):
        """Per-slice max code and shift weight, LSB-first (data_formats.py:60-71).

        The values are kept on the host; ``sliced_max_weights`` / ``sliced_weights`` become
        float32 tensors on ``device`` on first access, so building a SlicedData launches
        nothing and the MVM checks read host values without a device round trip.
        """
        sm = slice_method.tolist() if torch.is_tensor(slice_method) else [int(v) for v in slice_method]
        assert sm[0] == 1, 'the first slice should be 1'
        self._sm_list, self._sm_src = sm, slice_method
        self._max_host = [float(2 ** s - 1) for s in sm[::-1]]
        w, temp_s = [], 0
        for s in sm[::-1]:
            w.append(float(2 ** temp_s))
            temp_s += s
        w[-1] = -w[-1]
        self._weights_host = w
        self._max_t = None
        self._weights_t = None

    def _host_tensor(self, attr, values):
        t = getattr(self, attr)
        if t is None:
            t = torch.tensor(values, dtype=torch.float32, device=self.device)
            setattr(self, attr, t)
        return t

    sliced_max_weights = property(lambda self: self._host_tensor("_max_t", self._max_host),
                                  lambda self, v: setattr(self, "_max_t", v))
    sliced_weights = property(lambda self: self._host_tensor("_weights_t", self._weights_host),
                              lambda self, v: setattr(self, "_weights_t", v))

    def _max_codes(self):
        """Per-slice max codes as host floats (a tensor assigned to ``sliced_max_weights`` wins)."""
        if self._max_t is not None:
            return [float(v) for v in self._max_t.tolist()]
        return self._max_host

    def _slices(self):
        """The slice method as a host list of ints (read from ``slice_method`` once per object)."""
        if getattr(self, "_sm_src", None) is not self.slice_method:
            self._sm_list = [int(s) for s in self.slice_method]
            self._sm_src = self.slice_method
        return self._sm_list

    def __repr__(self):
        return 'sliced data with slice_method:{}'.format(self.slice_method)

    def __len__(self):
        return len(self.slice_method)

    # ------------------------------------------------------------------ helpers
    def _spec(self) -> N.SliceSpec:
        """ctypes slice spec; cached in the buffer dict, so slicing again rebuilds it."""
        cached = self._buf.get("spec_c")
        if cached is not None and cached[0] is self.slice_method:
            return cached[1]
        sp = self._make_spec()
        self._buf["spec_c"] = (self.slice_method, sp)
        return sp

    def _make_spec(self) -> N.SliceSpec:
        g = self._buf["geom"]
        sm = self._slices()
        sp = N.SliceSpec()
        sp.n_slices = len(sm)
        for i, s in enumerate(sm):
            sp.slice_method[i] = s
        sp.bfp = 1 if self.bw_e else 0
        sp.paral[0], sp.paral[1] = int(self.paral_size[0]), int(self.paral_size[1])
        sp.quant_gran[0], sp.quant_gran[1] = g["qg"][0], g["qg"][1]
        return sp

    def _kgeom(self) -> N.KGeom:
        kg = self._buf.get("kgeom_c")
        if kg is None:
            g = self._buf["geom"]
            kg = N.KGeom()
            kg.k, kg.kp, kg.p, kg.pp, kg.kt = g["k"], g["kp"], g["p"], g["pp"], g["kt"]
            self._buf["kgeom_c"] = kg
        return kg

    @property
    def bits(self):
        return int(sum(self._slices()))

    # ------------------------------------------------------------ slicing
    def slice_data_imp(self, engine, data):
        """Quantise, slice and (for weights) program ``data`` (data_formats.py:95-114).

        ``data`` is 2-D (rows, cols) or 3-D (batch, rows, cols); it is moved to
        ``engine.device``, which must be a CUDA device.
        """
        data = data.to(engine.device)
        if data.device.type != "cuda":
            raise RuntimeError("memintelli_flash_b200 computes on CUDA devices only "
                               f"(engine.device is {engine.device})")
        if data.dim() not in (2, 3):
            raise ValueError('The input data dimension is not supported!')
        data = data.detach()
        if data.dtype != torch.float32:
            data = data.float()
        self._cache = {}
        self._overrides = {}
        with N.device_guard(data.device):
            if self.is_weight:
                if data.dim() != 2:
                    raise ValueError('The weight data must be 2-D!')
                engine._program_weight(self, data)
            else:
                engine._slice_input(self, data)
        self.shape = data.shape

    def _slice_conv_imp(self, engine, x, kernel_size, stride, padding, dilation, noise_seed=None):
        """Slice the unfolded view of an NCHW input without materialising it (Conv2dMem).  With
        ``noise_seed`` the planes already carry the voltage noise of the one multiply made with them."""
        x = x.to(engine.device).detach()
        if x.device.type != "cuda":
            raise RuntimeError("memintelli_flash_b200 computes on CUDA devices only")
        if x.dtype != torch.float32:
            x = x.float()
        self._cache = {}
        self._overrides = {}
        with N.device_guard(x.device):
            engine._slice_conv_input(self, x, kernel_size, stride, padding, dilation, noise_seed=noise_seed)

    # ------------------------------------------------- reference-layout views
    def _get(self, name, fn):
        if name in self._overrides:
            return self._overrides[name]
        if self._buf is None:
            return None
        if name not in self._cache:
            self._cache[name] = fn()
        return self._cache[name]

    def _set(self, name, value):
        self._overrides[name] = value
        self._cache.pop(name, None)

    def _tiles_view(self, per_elem):
        """(B, rows_p, cols_p) -> reference tile layout (B, rows_p/p0, cols_p/p1, p0, p1)."""
        g = self._buf["geom"]
        p0, p1 = int(self.paral_size[0]), int(self.paral_size[1])
        B, R, C = per_elem.shape
        return per_elem.reshape(B, R // p0, p0, C // p1, p1).transpose(2, 3)

    def _padded_codes(self):
        """Packed codes in the reference's padded (B, rows_p, cols_p) frame."""
        b = self._buf
        g = b["geom"]
        if b.get("packed") is None:
            return None
        if self.is_weight:
            q = b["packed"][:, : g["kp"]].t()                          # (kp, N)
            out = torch.zeros((1, g["rows_p"], g["cols_p"]), dtype=torch.uint8, device=q.device)
            out[0, :, : g["n"]] = q
            return out
        q = b["packed"].reshape(g["batch"], g["rows"], g["kp"])
        out = torch.zeros((g["batch"], g["rows_p"], g["cols_p"]), dtype=torch.uint8, device=q.device)
        out[:, : g["rows"], :] = q
        return out

    def _sliced(self):
        q = self._padded_codes()
        if q is None:
            return None
        sm = self._slices()
        planes = []
        off = 0
        for w in sm[::-1]:
            planes.append(((q.to(torch.int32) >> off) & ((1 << w) - 1)).to(torch.uint8))
            off += w
        t = torch.stack([self._tiles_view(p) for p in planes], dim=3)   # (B, nr, nc, S, p0, p1)
        return t[0] if self._buf["geom"]["squeeze"] else t

    def _block_full(self, blocks):
        g = self._buf["geom"]
        qg0, qg1 = g["qg"]
        p0, p1 = int(self.paral_size[0]), int(self.paral_size[1])
        t = blocks.repeat_interleave(qg0 // p0, dim=1).repeat_interleave(qg1 // p1, dim=2)
        t = t[..., None, None]
        return t[0] if g["squeeze"] else t

    def _quantized(self):
        q = self._padded_codes()
        if q is None:
            return None
        g = self._buf["geom"]
        bits = self.bits
        qs = q.to(torch.int32)
        qs = torch.where(qs >= 2 ** (bits - 1), qs - 2 ** bits, qs).to(torch.float32)
        qg0, qg1 = g["qg"]
        if self.bw_e:
            e = self._buf["block_exp"].reshape(-1, g["nbr"], g["nbc"])
            s = torch.pow(2.0, e + 2 - bits).repeat_interleave(qg0, 1).repeat_interleave(qg1, 2)
            full = qs * s
        else:
            bm = self._buf["block_max"].reshape(-1, g["nbr"], g["nbc"])
            bm = bm.repeat_interleave(qg0, 1).repeat_interleave(qg1, 2)
            full = qs / (2 ** (bits - 1) - 1) * bm
        rows, cols = (g["k"], g["n"]) if self.is_weight else (g["rows"], g["k"])
        full = full[:, :rows, :cols]
        return full[0] if g["squeeze"] else full

    def _G(self):
        """Conductances in the reference layout (Kp/p0, Np/p1, S, p0, p1), siemens."""
        b = self._buf
        if not self.is_weight:
            return None
        g = b["geom"]
        S = len(self.slice_method)
        if b.get("g_planes") is not None:
            gp = b["g_planes"].reshape(S, g["n"], g["kt"], g["pp"])[..., : g["p"]]
        else:
            lv = b["planes"]
            if b["kind"] == N.OPERAND_E4M3:
                lv = lv.view(torch.float8_e4m3fn).to(torch.float32)
            else:
                lv = lv.view(torch.float16).to(torch.float32)
            lv = lv.reshape(S, g["n"], g["kt"], g["pp"])[..., : g["p"]]
            eng = b["engine"]
            gp = lv * eng["QG32"] + eng["LGS32"]
        gp = gp.reshape(S, g["n"], g["kp"]).permute(0, 2, 1)              # (S, kp, N)
        full = torch.full((S, g["rows_p"], g["cols_p"]), b["engine"]["LGS32"], device=gp.device)
        full[:, :, : g["n"]] = gp
        p0, p1 = int(self.paral_size[0]), int(self.paral_size[1])
        t = full.reshape(S, g["rows_p"] // p0, p0, g["cols_p"] // p1, p1).permute(1, 3, 0, 2, 4)
        return t.contiguous()

    sliced_data = property(lambda self: self._get("sliced_data", self._sliced),
                           lambda self, v: self._set("sliced_data", v))
    quantized_data = property(lambda self: self._get("quantized_data", self._quantized),
                              lambda self, v: self._set("quantized_data", v))
    max_data = property(lambda self: self._get("max_data", lambda: self._block_full(
        self._buf["block_max"].reshape(-1, self._buf["geom"]["nbr"], self._buf["geom"]["nbc"]))),
        lambda self, v: self._set("max_data", v))
    e_bias = property(lambda self: self._get("e_bias", lambda: None if self._buf.get("block_exp") is None else
                                             self._block_full(self._buf["block_exp"].reshape(
                                                 -1, self._buf["geom"]["nbr"], self._buf["geom"]["nbc"]))),
                      lambda self, v: self._set("e_bias", v))
    G = property(lambda self: self._get("G", self._G), lambda self, v: self._set("G", v))

    def size(self):
        return self.quantized_data.size()

    def t(self):
        """Transposed copy of the reference-layout views (data_formats.py:79-90).

        The copy carries views only; it cannot be fed to the engine (the
        operand planes are laid out for one orientation).
        """
        c = copy.copy(self)
        c._overrides = dict(self._overrides)
        c._cache = {}
        c._overrides["max_data"] = self.max_data.transpose(0, 1)
        if self.is_weight:
            c._overrides["G"] = self.G.transpose(-4, -5)
        if self.inference:
            c._overrides["sliced_data"] = None
            c._overrides["quantized_data"] = None
        else:
            c._overrides["sliced_data"] = self.sliced_data.transpose(-4, -5)
            c._overrides["quantized_data"] = self.quantized_data.T
        c._buf = dict(self._buf)
        c._buf["views_only"] = True
        return c
