"""CPU oracle for the Memintelli CIM bit-sliced matmul (numpy restatement).

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module:
it is the checker used by ``tests/``, by ``__graft_entry__.smoke()`` and by
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``.

It restates, in numpy, the arithmetic of the reference package
(zhuizhou/memintelli_flash, ``memintelli/pimpy``):

* block quantisation + bit slicing  -- ``memintelli/pimpy/data_formats.py:116-207``,
  ``memintelli/pimpy/utils.py:44-83`` (INT) and ``:86-128`` (block floating point);
* slice tables                     -- ``memintelli/pimpy/data_formats.py:60-71``;
* weight -> conductance levels, stuck-at and write-variation faults
                                    -- ``memintelli/pimpy/memmat_tensor.py:160-202``;
* DAC, crossbar MVM per slice pair, ADC, shift-add, block rescale, K-tile sum
                                    -- ``memintelli/pimpy/memmat_tensor.py:260-409``
  (``_dot_inference``; ``_dot`` at ``:411-495`` is the same arithmetic).

Quantisation and level mapping copy the reference's fp32 operation order, so
codes are bit-identical.  The noise-free MVM is computed exactly: the per
(row, K-tile, column, slice pair) crossbar sum ``S`` is an integer, the ADC
code is ``round_half_even(S * R / D)`` evaluated in exact rational arithmetic
(``R = radc - 1``, ``D = (rdac - 1) * (g_level - 1) * p``), and the weighted
sum over slice pairs is an exact int64.  The reference evaluates the same ADC
in fp32; at exact half-way points (``S*R/D = k + 1/2``) its rounding direction
is decided by fp32 noise, which is why parity against the reference is
tie-aware (``tie_bound``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------
# slice tables (memintelli/pimpy/data_formats.py:60-71)
# --------------------------------------------------------------------------
def slice_tables(slice_method: Sequence[int]):
    """LSB-first slice widths, bit offsets, per-slice max code and shift weight.

    ``slice_method`` is MSB-first with ``slice_method[0] == 1`` (the sign bit).
    Returns ``(widths, offsets, maxes, weights)``; ``weights[-1]`` is negative
    (two's complement sign slice), as in data_formats.py:71.
    """
    sm = [int(s) for s in slice_method]
    if sm[0] != 1:
        raise ValueError("The first bit of the slice method should be 1")
    widths = sm[::-1]
    offsets, o = [], 0
    for w in widths:
        offsets.append(o)
        o += w
    maxes = [(1 << w) - 1 for w in widths]
    weights = [1 << off for off in offsets]
    weights[-1] = -weights[-1]
    return widths, offsets, maxes, weights


# --------------------------------------------------------------------------
# block geometry (memintelli/pimpy/data_formats.py:141-184)
# --------------------------------------------------------------------------
@dataclass
class Geometry:
    rows: int
    cols: int
    p0: int
    p1: int
    qg0: int          # quant block rows, rounded up to a multiple of p0
    qg1: int          # quant block cols, rounded up to a multiple of p1
    nbr: int          # number of quant blocks along rows
    nbc: int          # number of quant blocks along cols

    @property
    def rows_p(self):
        return self.nbr * self.qg0

    @property
    def cols_p(self):
        return self.nbc * self.qg1


def geometry(rows: int, cols: int, paral_size, quant_gran) -> Geometry:
    """Decode quant granularity and padding exactly as data_formats.py:145-165."""
    if quant_gran is None:
        quant_gran = paral_size
    if quant_gran == "per-matrix":
        qg = [rows, cols]
    elif quant_gran == "per-row":
        qg = [1, cols]
    elif quant_gran == "per-col":
        qg = [rows, 1]
    else:
        qg = [int(quant_gran[0]), int(quant_gran[1])]
    p0, p1 = int(paral_size[0]), int(paral_size[1])
    qg[0] = math.ceil(qg[0] / p0) * p0
    qg[1] = math.ceil(qg[1] / p1) * p1
    nbr = math.ceil(rows / qg[0])
    nbc = math.ceil(cols / qg[1])
    return Geometry(rows, cols, p0, p1, qg[0], qg[1], nbr, nbc)


@dataclass
class Sliced:
    """Oracle counterpart of ``SlicedData`` after ``slice_data_imp``."""
    slice_method: list
    bw_e: Optional[int]
    geom: Geometry
    batch: int
    squeeze: bool
    q: np.ndarray            # (B, rows_p, cols_p) int64, two's complement code in [0, 2^bits)
    bmax: np.ndarray         # (B, nbr, nbc) float32 block abs-max
    ebias: Optional[np.ndarray]   # (B, nbr, nbc) float32 exponent (BFP) or None
    deq: np.ndarray          # (B, rows, cols) float32 dequantised values
    shape: tuple = field(default=())

    @property
    def bits(self):
        return sum(self.slice_method)

    def codes(self, t: int) -> np.ndarray:
        """Slice ``t`` (LSB-first) of every element: ``(q >> off_t) & m_t``."""
        widths, offsets, maxes, _ = slice_tables(self.slice_method)
        return (self.q >> offsets[t]) & maxes[t]

    def sliced_data(self) -> np.ndarray:
        """Reference layout ``(B, Rp/p0, Cp/p1, S, p0, p1)`` uint8 (data_formats.py:180-184)."""
        g = self.geom
        S = len(self.slice_method)
        out = np.empty((self.batch, g.rows_p // g.p0, g.cols_p // g.p1, S, g.p0, g.p1), np.uint8)
        for t in range(S):
            c = self.codes(t).reshape(self.batch, g.rows_p // g.p0, g.p0, g.cols_p // g.p1, g.p1)
            out[:, :, :, t] = c.transpose(0, 1, 3, 2, 4)
        return out[0] if self.squeeze else out

    def tile_scale(self) -> np.ndarray:
        """Per-tile dequant scale, (B, Rp/p0, Cp/p1) float64.

        INT: bmax / (2^(bits-1) - 1) (memintelli/pimpy/memmat_tensor.py:391-395);
        BFP: 2^(e + 2 - bits) (memintelli/pimpy/memmat_tensor.py:396-399).
        """
        g = self.geom
        if self.bw_e:
            s = np.exp2(self.ebias.astype(np.float64) + 2 - self.bits)
        else:
            s = self.bmax.astype(np.float64) / ((1 << (self.bits - 1)) - 1)
        s = np.repeat(np.repeat(s, g.qg0 // g.p0, axis=1), g.qg1 // g.p1, axis=2)
        return s


def bfp_exponent(bmax: np.ndarray) -> np.ndarray:
    """``floor(log2(bmax + 1e-10))`` as the reference evaluates it (utils.py:111).

    The fp32 sum is formed first; log2 is taken in float64 and rounded to
    float32 before the floor, which reproduces torch's fp32 log2 at the
    half-ulp edges just below powers of two.
    """
    b = (bmax.astype(F32) + F32(1e-10)).astype(F32)
    return np.floor(np.log2(b.astype(np.float64)).astype(F32)).astype(F32)


def slice_matrix(mat: np.ndarray, slice_method, bw_e=None, paral_size=(1, 32), quant_gran=None) -> Sliced:
    """Quantise + slice a 2-D (rows, cols) or 3-D (batch, rows, cols) fp32 matrix.

    Restates ``SlicedData._slice_data`` (data_formats.py:116-207) with
    ``quant_map_tensor`` (utils.py:44-83) or ``bfp_map_tensor`` (utils.py:86-128).
    """
    mat = np.asarray(mat, dtype=F32)
    squeeze = mat.ndim == 2
    if squeeze:
        mat = mat[None]
    if mat.ndim != 3:
        raise ValueError("The input data dimension is not supported!")
    sm = [int(s) for s in slice_method]
    if sm[0] != 1:
        raise ValueError("The first bit of the slice method should be 1")
    bits = sum(sm)
    B, R, C = mat.shape
    g = geometry(R, C, paral_size, quant_gran)
    pad = np.zeros((B, g.rows_p, g.cols_p), F32)
    pad[:, :R, :C] = mat
    blocks = pad.reshape(B, g.nbr, g.qg0, g.nbc, g.qg1)
    bmax = np.abs(blocks).max(axis=(2, 4)).astype(F32)                  # (B, nbr, nbc)
    bm_full = np.repeat(np.repeat(bmax, g.qg0, axis=1), g.qg1, axis=2)  # (B, Rp, Cp)
    ebias = None
    if bw_e:
        ebias = bfp_exponent(bmax)
        e_full = np.repeat(np.repeat(ebias, g.qg0, axis=1), g.qg1, axis=2)
        v = pad / np.exp2(e_full).astype(F32)
        v = (v * F32(2.0 ** (bits - 2))).astype(F32)
        qf = np.clip(np.rint(v), -(2 ** (bits - 1)), 2 ** (bits - 1) - 1)
        deq = (qf * np.exp2(e_full + 2 - bits).astype(F32)).astype(F32)
    else:
        with np.errstate(invalid="ignore", divide="ignore"):
            v = (pad / bm_full).astype(F32)
            v = (v * F32((1 << (bits - 1)) - 1)).astype(F32)
        qf = np.rint(v)
        qf = np.where(np.isnan(qf), 0.0, qf)        # all-zero block: 0/0 -> codes 0
        with np.errstate(invalid="ignore"):
            deq = (qf.astype(F32) / F32((1 << (bits - 1)) - 1) * bm_full).astype(F32)
        deq = np.where(np.isnan(deq), F32(0), deq)
    q = qf.astype(np.int64)
    q = np.where(q < 0, q + (1 << bits), q)
    return Sliced(sm, bw_e, g, B, squeeze, q, bmax, ebias, deq[:, :R, :C],
                  shape=tuple(mat.shape[1:]) if squeeze else tuple(mat.shape))


# --------------------------------------------------------------------------
# level maps (memintelli/pimpy/memmat_tensor.py:171, :297 / :360)
# --------------------------------------------------------------------------
def level_map(codes: np.ndarray, m: int, levels_minus_1: int) -> np.ndarray:
    """``round(code / m * (L - 1))`` in fp32, as memmat_tensor.py:171 / :297."""
    v = (codes.astype(F32) / F32(m)).astype(F32)
    v = (v * F32(levels_minus_1)).astype(F32)
    return np.rint(v).astype(np.int64)


@dataclass
class Engine:
    """Device parameters (memintelli/pimpy/memmat_tensor.py:30-115)."""
    HGS: float = 1e-5
    LGS: float = 1e-7
    g_level: int = 16
    write_variation: float = 0.02
    read_variation: object = 0.02
    vnoise: float = 0.05
    rdac: int = 16
    radc: object = 256
    vread: float = 0.2
    rate_stuck_HGS: float = 0.001
    rate_stuck_LGS: float = 0.0

    def radc_list(self, n_w_slices: int):
        """Per weight slice (LSB-first) ADC resolution; lists are flipped (memmat_tensor.py:82-85)."""
        if isinstance(self.radc, (list, tuple)):
            r = list(self.radc)[::-1]
            if len(r) != n_w_slices:
                raise ValueError(f"Length of radc array ({len(r)}) must match number of weight slices ({n_w_slices})")
            return [int(v) for v in r]
        return [int(self.radc)] * n_w_slices

    def read_sigma(self):
        rv = self.read_variation
        if isinstance(rv, dict):
            return [float(rv[i]) for i in range(self.g_level)]
        return [float(rv)] * self.g_level


def weight_levels(w: Sliced, eng: Engine, stuck_field: Optional[np.ndarray] = None) -> np.ndarray:
    """Integer conductance level per cell, per weight slice: (S, Kp, Np) int64.

    Stuck-at faults (memmat_tensor.py:183-197) become level ``g-1`` (HGS) or
    ``0`` (LGS).  ``stuck_field`` is the uniform draw of
    ``torch.rand(G.shape, generator=Generator().manual_seed(123))`` in the
    reference G layout (Kp/p0, Np/p1, S, p0, p1).
    """
    _, _, maxes, _ = slice_tables(w.slice_method)
    S = len(w.slice_method)
    if max(maxes) > eng.g_level - 1:
        raise ValueError("The weight data is out of the range!")
    g = w.geom
    lv = np.stack([level_map(w.codes(t)[0], maxes[t], eng.g_level - 1) for t in range(S)])
    if stuck_field is not None and (eng.rate_stuck_HGS > 0 or eng.rate_stuck_LGS > 0):
        r = np.asarray(stuck_field, np.float32)
        r = r.transpose(2, 0, 3, 1, 4).reshape(S, g.rows_p, g.cols_p)
        if eng.rate_stuck_HGS > 0:
            lv = np.where(r < eng.rate_stuck_HGS, eng.g_level - 1, lv)
        if eng.rate_stuck_LGS > 0:
            m = (r >= eng.rate_stuck_HGS) & (r < eng.rate_stuck_HGS + eng.rate_stuck_LGS)
            lv = np.where(m, 0, lv)
    return lv


def dac_levels(x: Sliced, eng: Engine) -> np.ndarray:
    """DAC input levels ``round(code / m_i * (rdac - 1))``: (S, B*rows_p, cols_p) int64."""
    _, _, maxes, _ = slice_tables(x.slice_method)
    S = len(x.slice_method)
    return np.stack([level_map(x.codes(t), maxes[t], eng.rdac - 1).reshape(-1, x.geom.cols_p) for t in range(S)])


def adc_round(S: np.ndarray, R: int, D: int) -> np.ndarray:
    """Exact ``round_half_even(S * R / D)`` for integer ``S`` (int64 arithmetic)."""
    S = S.astype(np.int64)
    num = 2 * S * R + D
    den = 2 * D
    q = np.floor_divide(num, den)
    tie = (np.mod(num, den) == 0) & (np.mod(q, 2) == 1)
    return q - tie.astype(np.int64)


def adc_ties(S: np.ndarray, R: int, D: int, slack: float = 0.0) -> np.ndarray:
    """Partials whose ADC input ``S*R/D`` is a half-integer, or within ``slack * S*R/D`` of one.

    ``slack`` models the relative fp32 error of the reference's evaluation of
    ``P / adcRef * (radc - 1)``; with ``slack = 0`` only exact ties count.
    """
    S = S.astype(np.int64)
    r = np.mod(2 * S * R, 2 * D)          # 2*D*frac(S*R/D)
    if slack <= 0:
        return r == D
    dist = np.abs(r - D) / (2.0 * D)       # distance of S*R/D from k + 1/2
    return dist <= slack * (S * R / D) + 1e-12


def _check_pair(x: Sliced, w: Sliced):
    if x.shape[-1] != w.shape[-2]:
        raise ValueError("The input data mismatches the shape of weight data!")
    if x.geom.p1 != w.geom.p0:
        raise ValueError("input paral_size[1] must equal weight paral_size[0]")
    if x.geom.cols_p != w.geom.rows_p:
        raise ValueError("input and weight K padding differ (quant_gran / paral_size mismatch)")


def mvm_exact(x: Sliced, w: Sliced, eng: Engine, wlev: Optional[np.ndarray] = None,
              return_parts: bool = False, m_chunk: int = 4096):
    """Noise-free CIM matmul, exact.  Returns float64 output of shape (M,N) or (B,T,N).

    Follows memmat_tensor.py:260-409: S_ij = sum_k A_i L_j over each K tile,
    Q = ADC(S), acc = sum_ij Q * m_i m_j c_i c_j, then
    y = sum_tau acc * p / R * scale_x * scale_w (uniform radc) or the
    per-slice-R weighted form (radc list).

    ``return_parts`` additionally returns the exact int64 tile accumulators
    ``acc[tau, row, col]`` (uniform radc only) and the tie count per element.
    """
    _check_pair(x, w)
    p = x.geom.p1
    Sx, Sw = len(x.slice_method), len(w.slice_method)
    _, _, mx, cx = slice_tables(x.slice_method)
    _, _, mw, cw = slice_tables(w.slice_method)
    if max(mw) > eng.g_level - 1:
        raise ValueError("The weight data is out of the range!")
    A = dac_levels(x, eng)                      # (Sx, Mrows, Kp)
    L = weight_levels(w, eng) if wlev is None else wlev   # (Sw, Kp, Np)
    Mrows, Kp = A.shape[1], A.shape[2]
    Np = L.shape[2]
    Kt = Kp // p
    D = (eng.rdac - 1) * (eng.g_level - 1) * p
    Rj = eng.radc_list(Sw)
    uniform = len(set(Rj)) == 1
    sx = x.tile_scale().reshape(-1, x.geom.cols_p // p)          # (Mrows/p0 ... ) -> per row
    sx = np.repeat(sx, x.geom.p0, axis=0)                          # (Mrows, Kt)
    sw = np.repeat(w.tile_scale()[0], w.geom.p1, axis=1)          # (Kt, Np)
    y = np.zeros((Mrows, Np), np.float64)
    acc_all = np.zeros((Kt, Mrows, Np), np.int64) if (return_parts and uniform) else None
    ties = np.zeros((Mrows, Np), np.float64) if return_parts else None
    Lf = L.astype(np.float32).reshape(Sw, Kt, p, Np)
    for m0 in range(0, Mrows, m_chunk):
        m1 = min(Mrows, m0 + m_chunk)
        Af = A[:, m0:m1].astype(np.float32).reshape(Sx, m1 - m0, Kt, p).transpose(0, 2, 1, 3)  # (Sx,Kt,m,p)
        acc = np.zeros((Kt, m1 - m0, Np), np.int64)
        accf = np.zeros((Kt, m1 - m0, Np), np.float64)
        for i in range(Sx):
            for j in range(Sw):
                Sij = np.matmul(Af[i], Lf[j]).astype(np.int64)      # exact: < 2^24
                Q = adc_round(Sij, Rj[j] - 1, D)
                wij = mx[i] * mw[j] * cx[i] * cw[j]
                if uniform:
                    acc += Q * wij
                else:
                    accf += Q.astype(np.float64) * (wij * p / (Rj[j] - 1))
                if ties is not None:
                    ties[m0:m1] += adc_ties(Sij, Rj[j] - 1, D).sum(axis=0)
        if uniform:
            tile = acc.astype(np.float64) * (p / (Rj[0] - 1))
            if acc_all is not None:
                acc_all[:, m0:m1] = acc
        else:
            tile = accf
        scale = sx[m0:m1].T[:, :, None] * sw[:, None, :]             # (Kt, m, Np)
        y[m0:m1] = (tile * scale).sum(axis=0)
    y = _crop(y, x, w)
    if return_parts:
        return y, acc_all, _crop(ties, x, w)
    return y


def _crop(y: np.ndarray, x: Sliced, w: Sliced) -> np.ndarray:
    N = w.shape[-1]
    if x.squeeze:
        return y[: x.shape[0], :N]
    B = x.batch
    T = x.shape[1]
    return y.reshape(B, x.geom.rows_p, -1)[:, :T, :N]


def tie_bound(x: Sliced, w: Sliced, eng: Engine, wlev=None, fp32_slack: bool = True) -> np.ndarray:
    """Per-element bound on |reference - exact| from ADC half-way ties.

    Each tie partial can round either way in the reference's fp32 path, moving
    the output by one ADC code times ``|w_ij| p / R * scale``.  With
    ``fp32_slack`` a partial also counts when its exact ADC input lies within
    the reference's worst-case fp32 error ``(p + 4) * 2^-24`` (relative) of a
    half-integer: the p-term fp32 crossbar sum plus the scaling roundings can
    move it across the rounding boundary.
    """
    p = x.geom.p1
    Sx, Sw = len(x.slice_method), len(w.slice_method)
    _, _, mx, cx = slice_tables(x.slice_method)
    _, _, mw, cw = slice_tables(w.slice_method)
    A = dac_levels(x, eng)
    L = weight_levels(w, eng) if wlev is None else wlev
    Mrows, Kp = A.shape[1], A.shape[2]
    Np = L.shape[2]
    Kt = Kp // p
    D = (eng.rdac - 1) * (eng.g_level - 1) * p
    Rj = eng.radc_list(Sw)
    sx = np.repeat(x.tile_scale().reshape(-1, x.geom.cols_p // p), x.geom.p0, axis=0)
    sw = np.repeat(w.tile_scale()[0], w.geom.p1, axis=1)
    Af = A.astype(np.float32).reshape(Sx, Mrows, Kt, p).transpose(0, 2, 1, 3)
    Lf = L.astype(np.float32).reshape(Sw, Kt, p, Np)
    bound = np.zeros((Kt, Mrows, Np), np.float64)
    for i in range(Sx):
        for j in range(Sw):
            Sij = np.matmul(Af[i], Lf[j]).astype(np.int64)
            t = adc_ties(Sij, Rj[j] - 1, D, slack=(p + 4) * 2.0 ** -24 if fp32_slack else 0.0)
            bound += t * (abs(mx[i] * mw[j] * cx[i] * cw[j]) * p / (Rj[j] - 1))
    scale = sx.T[:, :, None] * sw[:, None, :]
    return _crop((bound * scale).sum(axis=0), x, w)


def mvm_float(x: Sliced, w: Sliced, eng: Engine, rng: np.random.Generator,
              stuck_field=None, write_field=None, noisy=True, dtype=np.float64):
    """Float64 restatement of ``_dot_inference`` including the noise models.

    Write variation ``G += G*N(0,wv)`` (memmat_tensor.py:175-180) uses
    ``write_field`` (the reference's fixed-seed draw) when given; read
    variation ``G*exp(sigma*N)`` (memmat_tensor.py:204-236) and voltage noise
    ``V*(1+vnoise*N)`` (memmat_tensor.py:297-299) are drawn from ``rng``.
    Used for statistical checks only.
    """
    _check_pair(x, w)
    p = x.geom.p1
    Sx, Sw = len(x.slice_method), len(w.slice_method)
    _, _, mx, cx = slice_tables(x.slice_method)
    _, _, mw, cw = slice_tables(w.slice_method)
    g = w.geom
    lv = np.stack([level_map(w.codes(t)[0], mw[t], eng.g_level - 1) for t in range(Sw)]).astype(np.float64)
    QG = (eng.HGS - eng.LGS) / (eng.g_level - 1)
    G = lv * QG + eng.LGS
    if eng.write_variation > 0 and write_field is not None:
        wf = np.asarray(write_field, np.float64).transpose(2, 0, 3, 1, 4).reshape(Sw, g.rows_p, g.cols_p)
        G = G + G * wf
    if stuck_field is not None and (eng.rate_stuck_HGS > 0 or eng.rate_stuck_LGS > 0):
        r = np.asarray(stuck_field, np.float32).transpose(2, 0, 3, 1, 4).reshape(Sw, g.rows_p, g.cols_p)
        G = np.where(r < eng.rate_stuck_HGS, eng.HGS, G)
        m = (r >= eng.rate_stuck_HGS) & (r < eng.rate_stuck_HGS + eng.rate_stuck_LGS)
        G = np.where(m, eng.LGS, G)
    sig = eng.read_sigma()
    if noisy and any(s > 0 for s in sig):
        lvl = np.clip(np.rint((G - eng.LGS) / QG), 0, eng.g_level - 1).astype(np.int64)
        G = G * np.exp(np.asarray(sig)[lvl] * rng.standard_normal(G.shape))
    Gs = (G - eng.LGS).reshape(Sw, -1, p, g.cols_p).astype(dtype)
    A = dac_levels(x, eng).astype(np.float64)
    Mrows, Kp = A.shape[1], A.shape[2]
    Kt = Kp // p
    V = eng.vread * A / (eng.rdac - 1)
    if noisy and eng.vnoise > 0:
        V = V * (1 + rng.standard_normal(V.shape) * eng.vnoise)
    V = V.reshape(Sx, Mrows, Kt, p).transpose(0, 2, 1, 3).astype(dtype)
    adcRef = (eng.HGS - eng.LGS) * eng.vread * p
    Rj = eng.radc_list(Sw)
    acc = np.zeros((Kt, Mrows, g.cols_p), dtype)
    for i in range(Sx):
        for j in range(Sw):
            P = np.matmul(V[i], Gs[j])
            Q = np.rint(P / adcRef * (Rj[j] - 1)) / (Rj[j] - 1)
            acc += Q * (mx[i] * mw[j] * p) * (cx[i] * cw[j])
    sx = np.repeat(x.tile_scale().reshape(-1, x.geom.cols_p // p), x.geom.p0, axis=0)
    sw = np.repeat(w.tile_scale()[0], w.geom.p1, axis=1)
    y = (acc * (sx.T[:, :, None] * sw[:, None, :])).sum(axis=0)
    return _crop(y, x, w)


def SNR(ytest, ypred):
    """memintelli/pimpy/utils.py:36-37."""
    return 10 * np.log10(np.sum(ytest ** 2) / np.sum((ytest - ypred) ** 2))


def RE(ytest, ypred):
    """memintelli/pimpy/utils.py:40-41."""
    return np.sqrt(np.sum((ytest - ypred) ** 2)) / np.sqrt(np.sum(ytest ** 2))


def ABSE(ytest, ypred):
    """memintelli/pimpy/utils.py:32-33."""
    return np.sum(np.abs((ytest - ypred) / ytest)) / (ytest.shape[0] * ytest.shape[1])


def mvm_float_torch(x: Sliced, w: Sliced, eng: Engine, seed: int = 0, noisy: bool = True, device="cpu",
                    m_chunk: int = 0):
    """torch restatement of ``_dot_inference`` (memmat_tensor.py:260-409) for timing the reference's
    algorithm: on the CPU (its own CPU path) or on a CUDA device (its GPU path).

    Same arithmetic as ``mvm_float`` in fp32 with torch kernels, in the reference's structure: one
    batched contraction per slice pair into a (Kt, M, Np) partial tensor, ADC, shift-add, block
    rescale, K-tile sum.  Read variation is drawn from a seeded torch generator; stuck-at and write
    variation are not modelled here.  ``m_chunk`` > 0 processes the rows in chunks, as the reference's
    GPU path must for large outputs (the partial of one slice pair is Kt x M x Np fp32).
    Returns a float64 numpy array after synchronising the device.
    """
    if m_chunk and x.squeeze and x.geom.qg0 == 1 and x.batch == 1:
        rows = x.geom.rows_p
        parts = [mvm_float_torch(_row_slice(x, m0, min(rows, m0 + m_chunk)), w, eng, seed + m0, noisy, device, 0)
                 for m0 in range(0, rows, m_chunk)]
        return np.concatenate(parts, axis=0)
    y = torch_port_mvm(torch_port_operands(x, w, eng, device), eng, seed, noisy)
    return _crop(y.double().cpu().numpy(), x, w)


def torch_port_operands(x: Sliced, w: Sliced, eng: Engine, device="cpu") -> dict:
    """Device tensors the reference's ``_dot_inference`` starts from: DAC levels of every input slice,
    conductances G of every weight slice (memmat_tensor.py:160-202, 238-258) and the block scales."""
    import torch
    dev = torch.device(device)
    p = x.geom.p1
    Sw = len(w.slice_method)
    _, _, mx, cx = slice_tables(x.slice_method)
    _, _, mw, cw = slice_tables(w.slice_method)
    QG = (eng.HGS - eng.LGS) / (eng.g_level - 1)
    Kt = x.geom.cols_p // p
    G = torch.stack([torch.from_numpy(level_map(w.codes(t)[0], mw[t], eng.g_level - 1)) for t in range(Sw)])
    G = G.to(dev).float() * QG + eng.LGS                                      # (Sw, Kp, Np)
    A = [torch.from_numpy(level_map(x.codes(i), mx[i], eng.rdac - 1).reshape(-1, Kt, p)).to(dev).float()
         for i in range(len(x.slice_method))]
    sx = torch.from_numpy(np.repeat(x.tile_scale().reshape(-1, Kt), x.geom.p0, axis=0)).to(dev).float()
    sw = torch.from_numpy(np.repeat(w.tile_scale()[0], w.geom.p1, axis=1)).to(dev).float()
    return dict(G=G, A=A, sx=sx, sw=sw, p=p, Kt=Kt, Np=w.geom.cols_p, mx=mx, cx=cx, mw=mw, cw=cw, dev=dev)


def torch_port_mvm(ops: dict, eng: Engine, seed: int = 0, noisy: bool = True):
    """The device work of one ``_dot_inference`` call (memmat_tensor.py:280-404) on prepared operands:
    read noise on G, then for every slice pair the crossbar contraction, ADC rounding and shift-add,
    then the block rescale and the K-tile sum.  Returns the (rows_p, Np) fp32 device tensor."""
    import torch
    dev, p, Kt = ops["dev"], ops["p"], ops["Kt"]
    gen = torch.Generator(device=dev).manual_seed(seed)
    G = ops["G"]
    Sw = G.shape[0]
    Rj = eng.radc_list(Sw)
    adcRef = (eng.HGS - eng.LGS) * eng.vread * p
    sig = eng.read_sigma()
    if noisy and sig[0] > 0:
        G = G * torch.exp(torch.randn(G.shape, generator=gen, device=dev) * sig[0])
    Gs = (G - eng.LGS).reshape(Sw, Kt, p, ops["Np"])
    out = None
    for i, A in enumerate(ops["A"]):
        V = (eng.vread * A / (eng.rdac - 1)).transpose(0, 1)                   # (Kt, M, p)
        if noisy and eng.vnoise > 0:
            V = V * (1 + torch.randn(V.shape, generator=gen, device=dev) * eng.vnoise)
        for j in range(Sw):
            P = torch.bmm(V, Gs[j])                                           # (Kt, M, Np)
            P = torch.round(P / adcRef * (Rj[j] - 1)) / (Rj[j] - 1)
            P = P * float(ops["mx"][i] * ops["mw"][j] * p * ops["cx"][i] * ops["cw"][j])
            out = P if out is None else out.add_(P)
    return (out * ops["sx"].T[:, :, None] * ops["sw"][:, None, :]).sum(0)


def _row_slice(x: Sliced, m0: int, m1: int) -> Sliced:
    """Rows [m0, m1) of a 2-D input with one-row quant blocks (rows are independent)."""
    import copy
    g = x.geom
    if g.qg0 != 1:
        raise ValueError("row chunks need one-row input quant blocks")
    y = copy.copy(x)
    y.q = x.q[:, m0:m1]
    y.bmax = x.bmax[:, m0:m1]
    y.ebias = None if x.ebias is None else x.ebias[:, m0:m1]
    y.deq = x.deq[:, m0:m1]
    y.geom = Geometry(m1 - m0, g.cols, g.p0, g.p1, g.qg0, g.qg1, m1 - m0, g.nbc)
    return y
