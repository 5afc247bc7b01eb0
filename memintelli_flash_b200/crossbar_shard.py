"""Crossbar sharding of CIM linear layers across GPUs (one process per GPU).

The reference runs every crossbar of a layer on one device.  Here a layer's
weight can be split across the ranks of a ``torch.distributed`` process group
along whole quantisation blocks, which keeps the result exact:

* column sharding (``ColumnShardedLinearMem``): each rank programs a block of
  output columns (crossbar columns).  ADC, shift-add, block rescale and K-tile
  sum are all per output column, so every shard's output equals the same
  columns of the unsharded layer: bit-identical, except where one of the two
  launches sums an output tile's K ranges separately (split-K, or the tail
  split of a persistent launch), which changes only the fp32 summation order.  The output stays sharded (the next
  layer consumes it sharded) or is all-gathered.
* row sharding (``RowShardedLinearMem``): each rank programs a block of input
  rows (crossbar K tiles).  The K-tile partial sums are added after the ADC in
  the reference (memmat_tensor.py:401), so the shards' outputs sum to the
  unsharded result up to fp32 summation order; one all-reduce combines them.

Shard boundaries are multiples of the weight quant block along the split
dimension (``quant_gran`` rounded up to ``paral_size``), so no quant block
straddles two ranks.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from .NN_layers.linear import LinearMem


def shard_bounds(n: int, block: int, world: int, rank: int):
    """[start, stop) of rank's shard of n items split in whole blocks, as evenly as possible."""
    nblocks = math.ceil(n / block)
    base, extra = divmod(nblocks, world)
    b0 = rank * base + min(rank, extra)
    b1 = b0 + base + (1 if rank < extra else 0)
    return min(n, b0 * block), min(n, b1 * block)


def noise_calls(world: int, rank: int, dim: int):
    """(read-noise call, voltage-noise call) of a shard: the per-call noise kernels key their draws by
    (seed, call, element), and every rank draws with the same seed.  Each rank's crossbar cells get a
    draw of their own (call = rank), so shards are independent as the cells of one crossbar are; the
    input of a column-sharded layer is replicated and keeps call 0 (one draw shared by all columns, as
    in one crossbar), while a row shard's input features are its own (call = rank)."""
    if world <= 1:
        return 0, 0
    return rank, (rank if dim == 1 else 0)


def _world(group):
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


class _ShardBase(torch.nn.Module):
    def __init__(self, engine, weight: torch.Tensor, bias: Optional[torch.Tensor], dim: int, input_slice,
                 weight_slice, bw_e=None, input_paral_size=(1, 32), weight_paral_size=(32, 32),
                 input_quant_gran=(1, 32), weight_quant_gran=(32, 32), group=None, device=None,
                 presharded: bool = False):
        super().__init__()
        self.group = group
        world, rank = (1, 0) if presharded else _world(group)
        out_f, in_f = weight.shape
        if world > 1 and (isinstance(weight_quant_gran, str) or (dim == 1 and isinstance(input_quant_gran, str))):
            # a per-matrix / per-row / per-column scale spans every shard: each rank would compute its own
            # maximum over its part only, and the shards would no longer add up to the unsharded layer
            raise ValueError("crossbar sharding needs tuple quant_gran blocks; a string granularity "
                             f"({weight_quant_gran!r} / {input_quant_gran!r}) makes one scale span all shards")
        qg = weight_quant_gran if not isinstance(weight_quant_gran, str) else (in_f, out_f)
        if dim == 0:   # output columns of W^T == rows of the (out, in) weight
            blk = math.ceil(qg[1] / weight_paral_size[1]) * weight_paral_size[1]
            lo, hi = shard_bounds(out_f, blk, world, rank)
            w_local = weight[lo:hi]
            b_local = None if bias is None else bias[lo:hi]
            lin_in, lin_out = in_f, hi - lo
        else:          # input rows (K) of W^T
            blk = math.ceil(qg[0] / weight_paral_size[0]) * weight_paral_size[0]
            xq = input_quant_gran if not isinstance(input_quant_gran, str) else (1, in_f)
            xblk = math.ceil(xq[1] / input_paral_size[1]) * input_paral_size[1]
            blk = blk * xblk // math.gcd(blk, xblk)
            lo, hi = shard_bounds(in_f, blk, world, rank)
            w_local = weight[:, lo:hi]
            b_local = None
            lin_in, lin_out = hi - lo, out_f
            self.full_bias = None if bias is None else bias.detach().clone()
        if hi <= lo:
            what = "output columns" if dim == 0 else "input rows"
            raise ValueError(f"rank {rank} of {world} gets an empty crossbar shard: {out_f if dim == 0 else in_f} "
                             f"{what} in blocks of {blk} do not give every rank a block")
        self.lo, self.hi, self.world, self.rank = lo, hi, world, rank
        self.in_features, self.out_features = in_f, out_f
        self.local = _LinearFromWeight(engine, w_local, b_local, input_slice, weight_slice, bw_e, input_paral_size,
                                       weight_paral_size, input_quant_gran, weight_quant_gran, device)
        self._set_noise_calls(world, rank, dim)

    def _set_noise_calls(self, world, rank, dim):
        buf = self.local.weight_sliced._buf
        buf["noise_call"], buf["input_noise_call"] = noise_calls(world, rank, dim)

    def prepare_for_inference(self):
        self.local.inference_mode = True
        self.local.weight_sliced.inference = True

    def new_input(self):
        """An empty input SlicedData for this rank's crossbars (see ``LinearMem.new_input``)."""
        return self.local.new_input()

    def forward_sliced(self, input_sliced):
        """``forward`` for an input already sliced by a fused producer."""
        return self._finish(self.local.forward_sliced(input_sliced))

    def partial_sliced(self, input_sliced):
        """This rank's output before any collective (row sharding: the partial sum; the caller
        all-reduces it and adds ``full_bias``)."""
        return self.local.forward_sliced(input_sliced)


class _LinearFromWeight(LinearMem):
    """LinearMem programmed from a given weight (no random init, programmed once)."""

    def __init__(self, engine, weight, bias, input_slice, weight_slice, bw_e, input_paral_size, weight_paral_size,
                 input_quant_gran, weight_quant_gran, device):
        torch.nn.Module.__init__(self)
        self.in_features = weight.shape[1]
        self.out_features = weight.shape[0]
        self.weight = torch.nn.Parameter(weight.detach().to(device=device, dtype=torch.float32).contiguous(),
                                         requires_grad=False)
        if bias is not None:
            self.bias = torch.nn.Parameter(bias.detach().to(device=device, dtype=torch.float32).contiguous(),
                                           requires_grad=False)
        else:
            self.register_parameter('bias', None)
        from .pimpy.data_formats import SlicedData
        self.weight_slice_method = torch.tensor(weight_slice)
        self.input_slice_method = torch.tensor(input_slice)
        self.weight_sliced = SlicedData(self.weight_slice_method, device=device, bw_e=bw_e, is_weight=True,
                                        paral_size=weight_paral_size, quant_gran=weight_quant_gran, inference=True)
        self.engine = engine
        self.weight_sliced.slice_data_imp(engine, self.weight.detach().t())
        self.input_paral_size = input_paral_size
        self.input_quant_gran = input_quant_gran
        self.inference_mode = True


class ColumnShardedLinearMem(_ShardBase):
    """Output columns split across ranks; ``forward`` returns this rank's columns
    (``gather=True``: all-gathers the full output along the last dimension).

    ``weight`` may be a list of (out_i, in) weights sharing one input (e.g. q/k/v):
    each part is sharded on its own quant blocks and the local shards are
    concatenated into one crossbar array, so one slicing of the input and one MVM
    serve all parts; ``split_sizes`` gives the local width of every part.
    """

    def __init__(self, engine, weight, bias, input_slice, weight_slice, gather=False, **kw):
        if isinstance(weight, (list, tuple)):
            if gather:
                raise ValueError("gather is not supported for a fused multi-part weight")
            group = kw.get("group")
            world, rank = _world(group)
            qg = kw.get("weight_quant_gran", (32, 32))
            wp = kw.get("weight_paral_size", (32, 32))
            blk = math.ceil(qg[1] / wp[1]) * wp[1]
            parts = []
            for w in weight:
                if w.shape[0] % blk:
                    raise ValueError("every fused part must be a whole number of weight quant blocks")
                lo, hi = shard_bounds(w.shape[0], blk, world, rank)
                parts.append(w[lo:hi])
            self._fused_sizes = [p.shape[0] for p in parts]
            fused = torch.cat(parts, dim=0)
            super().__init__(engine, fused, bias, 0, input_slice, weight_slice, presharded=True, **kw)
            self.group, self.world, self.rank = group, world, rank
            self._set_noise_calls(world, rank, 0)
            self.gather = False
            self.shard_sizes = None
            return
        self._fused_sizes = None
        super().__init__(engine, weight, bias, 0, input_slice, weight_slice, **kw)
        self.gather = gather
        qg = kw.get("weight_quant_gran", (32, 32))
        wp = kw.get("weight_paral_size", (32, 32))
        blk = math.ceil(qg[1] / wp[1]) * wp[1] if not isinstance(qg, str) else self.out_features
        self.shard_sizes = [b - a for a, b in (shard_bounds(self.out_features, blk, self.world, r)
                                               for r in range(self.world))]

    @property
    def split_sizes(self):
        return self._fused_sizes

    def forward(self, x):
        return self._finish(self.local(x))

    def _finish(self, y):
        if not self.gather or self.world == 1:
            return y
        width = max(self.shard_sizes)
        if y.shape[-1] < width:
            y = torch.nn.functional.pad(y, (0, width - y.shape[-1]))
        parts = [torch.empty_like(y) for _ in range(self.world)]
        dist.all_gather(parts, y.contiguous(), group=self.group)
        return torch.cat([p[..., :n] for p, n in zip(parts, self.shard_sizes)], dim=-1)


class RowShardedLinearMem(_ShardBase):
    """Input rows (K) split across ranks; ``forward`` takes this rank's slice of
    the input features and all-reduces the partial outputs."""

    def __init__(self, engine, weight, bias, input_slice, weight_slice, **kw):
        super().__init__(engine, weight, bias, 1, input_slice, weight_slice, **kw)

    def forward(self, x_local):
        return self._finish(self.local(x_local))

    def _finish(self, y):
        if self.world > 1:
            dist.all_reduce(y, group=self.group)
        if self.full_bias is not None:
            y = y + self.full_bias.to(y.device)
        return y
