"""Qwen3-0.6B-architecture prefill with every linear on the CIM engine.

The reference wraps a Hugging Face ``AutoModelForCausalLM`` and swaps every
``nn.Linear`` (q/k/v/o, gate/up/down of 28 layers, and ``lm_head``) for
``LinearMem`` (memintelli/NN_models/Qwen3.py:82-106); attention, RMSNorm,
RoPE and SiLU stay in torch.  This module is the same computation written
compactly so that its crossbars can be sharded across GPUs:

* q/k/v and gate/up are column-sharded (whole heads / whole 128-column quant
  blocks per rank, outputs stay sharded); o_proj and down_proj are
  row-sharded, with one all-reduce each;
* lm_head is column-sharded and the cross-entropy is computed without
  gathering the logits (distributed log-sum-exp).

With ``shard_head_over`` the decoder layers stay whole on every rank (data
parallel over sequences) and only lm_head is column-sharded over that group:
the ranks' final hidden states are all-gathered, every rank computes its
vocabulary columns for all sequences, and the distributed log-sum-exp gives
every rank the loss of the whole batch.  lm_head holds about a quarter of the
model's crossbar cells, so this divides its programmed memory and its per-call
read-noise pass by the group size.

With a world size of 1 there is no collective and no sharding.  Of the
non-CIM parts, the RMSNorms and the SwiGLU run inside the input slicing, q/k
RMSNorm + RoPE in one kernel (mib_qk_norm_rope_bf16), the loss's row
log-sum-exp in one pass over the logits (mib_row_logsumexp); the embedding
and the residual adds stay in torch, and attention runs in bf16 through
scaled_dot_product_attention (or fp32, ``set_attention_dtype``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _native as N
from .crossbar_shard import ColumnShardedLinearMem, RowShardedLinearMem, shard_bounds


@dataclass
class Qwen3Arch:
    hidden: int = 1024
    layers: int = 28
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 3072
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6


@dataclass
class CimSpec:
    """Slicing / granularity of every CIM linear (config: weight (128,128)/(32,32), input (1,128)/(1,32))."""
    input_slice: tuple = (1, 1, 2, 2, 2)
    weight_slice: tuple = (1, 1, 2, 2, 2)
    bw_e: object = None
    input_paral_size: tuple = (1, 32)
    weight_paral_size: tuple = (32, 32)
    input_quant_gran: tuple = (1, 128)
    weight_quant_gran: tuple = (128, 128)

    def kwargs(self):
        return dict(bw_e=self.bw_e, input_paral_size=self.input_paral_size,
                    weight_paral_size=self.weight_paral_size, input_quant_gran=self.input_quant_gran,
                    weight_quant_gran=self.weight_quant_gran)


def rms_norm(x, w, eps):
    v = x.float().pow(2).mean(-1, keepdim=True)
    return x * torch.rsqrt(v + eps) * w


def rope_cache(T, dim, theta, device):
    """(T, dim) cos / sin tables of the default rotary embedding, in float32 as the Hugging Face Qwen3
    model evaluates them (inverse frequencies and position x frequency products in fp32)."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    t = torch.arange(T, dtype=torch.int64).float()
    f = torch.outer(t, inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(device), emb.sin().to(device)


def apply_rope(x, cos, sin):
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], dim=-1)
    return x * cos + rot * sin


class Qwen3CimLayer(torch.nn.Module):
    def __init__(self, arch: Qwen3Arch, engine, spec: CimSpec, gen: torch.Generator, device, group=None,
                 weights=None, prefix=""):
        super().__init__()
        a = arch
        self.arch = a
        std = 0.02
        names = iter(("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                      "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"))

        def w(o, i):
            """The next linear's (out, in) weight: from ``weights`` (Hugging Face Qwen3 names) when given,
            else random (std 0.02, drawn in this order)."""
            name = next(names)
            if weights is not None:
                t = weights[f"{prefix}{name}.weight"]
                if tuple(t.shape) != (o, i):
                    raise ValueError(f"{prefix}{name}.weight has shape {tuple(t.shape)}, expected {(o, i)}")
                return t.to(device=device, dtype=torch.float32)
            return torch.randn(o, i, generator=gen, device=device) * std

        def norm(name, n):
            if weights is None:
                return torch.ones(n, device=device)
            return weights[f"{prefix}{name}.weight"].to(device=device, dtype=torch.float32).reshape(n)

        kw = dict(group=group, device=device, **spec.kwargs())
        sl = (spec.input_slice, spec.weight_slice)
        # q/k/v and gate/up read the same input: their crossbars are programmed side by side
        # (per rank: this rank's heads of q, k and v), so the input is sliced once per group.
        # Output columns are independent in the CIM arithmetic, so this is exact.
        self.qkv_proj = ColumnShardedLinearMem(
            engine, [w(a.heads * a.head_dim, a.hidden), w(a.kv_heads * a.head_dim, a.hidden),
                     w(a.kv_heads * a.head_dim, a.hidden)], None, *sl, **kw)
        self.o_proj = RowShardedLinearMem(engine, w(a.hidden, a.heads * a.head_dim), None, *sl, **kw)
        self.gate_up_proj = ColumnShardedLinearMem(
            engine, [w(a.intermediate, a.hidden), w(a.intermediate, a.hidden)], None, *sl, **kw)
        self.down_proj = RowShardedLinearMem(engine, w(a.hidden, a.intermediate), None, *sl, **kw)
        self.in_norm = torch.nn.Parameter(norm("input_layernorm", a.hidden), requires_grad=False)
        self.post_norm = torch.nn.Parameter(norm("post_attention_layernorm", a.hidden), requires_grad=False)
        self.q_norm = torch.nn.Parameter(norm("self_attn.q_norm", a.head_dim), requires_grad=False)
        self.k_norm = torch.nn.Parameter(norm("self_attn.k_norm", a.head_dim), requires_grad=False)
        # attention arithmetic: bf16 (q/k norm, RoPE and casts in mib_qk_norm_rope_bf16, then bf16 SDPA) or
        # float32 (the same steps in torch, fp32 SDPA: the reference model's eager fp32 attention)
        self.attn_dtype = torch.bfloat16
        q_cols, k_cols, v_cols = self.qkv_proj.split_sizes
        if q_cols % a.head_dim or k_cols % a.head_dim or k_cols == 0 or q_cols == 0:
            raise ValueError(f"crossbar sharding must give every rank whole, non-empty heads "
                             f"(local q columns {q_cols}, k columns {k_cols}, head_dim {a.head_dim})")
        self.local_heads = q_cols // a.head_dim
        self.local_kv = k_cols // a.head_dim
        if self.local_heads % self.local_kv:
            raise ValueError("each rank's query heads must be a multiple of its key/value heads")
        self.local_inter = self.gate_up_proj.split_sizes[0]
        self.engine = engine

    def forward(self, h, cos, sin):
        """One decoder layer.  The RMSNorms before the q/k/v and gate/up crossbars and the SwiGLU
        before the down crossbar run inside the input slicing (``DPETensor.slice_rmsnorm_input`` /
        ``slice_swiglu_input``), so those activations are never written out."""
        h = h + self._reduce(self.attn_partial(h, cos, sin))
        return h + self._reduce(self.mlp_partial(h))

    def _reduce(self, y):
        if self.o_proj.world > 1:
            dist.all_reduce(y, group=self.o_proj.group)
        return y

    def attn_partial(self, h, cos, sin):
        """Attention block up to this rank's o_proj partial sum (before the all-reduce)."""
        a = self.arch
        B, T, _ = h.shape
        xs = self.qkv_proj.new_input()
        self.engine.slice_rmsnorm_input(xs, h, self.in_norm, a.eps)
        qkv = self.qkv_proj.forward_sliced(xs)
        if self.attn_dtype == torch.float32:
            nq, nk = self.local_heads * a.head_dim, self.local_kv * a.head_dim
            q = qkv[..., :nq].reshape(B, T, self.local_heads, a.head_dim)
            k = qkv[..., nq:nq + nk].reshape(B, T, self.local_kv, a.head_dim)
            v = qkv[..., nq + nk:nq + 2 * nk].reshape(B, T, self.local_kv, a.head_dim)
            c, s_ = cos[:, None, :], sin[:, None, :]
            q = apply_rope(rms_norm(q, self.q_norm, a.eps), c, s_)
            k = apply_rope(rms_norm(k, self.k_norm, a.eps), c, s_)
        else:
            # q/k RMSNorm, rotary embedding and bf16 casts in one pass (mib_qk_norm_rope_bf16); the torch
            # form is the float32 branch above
            q, k, v = (torch.empty(B, T, n, a.head_dim, dtype=torch.bfloat16, device=h.device)
                       for n in (self.local_heads, self.local_kv, self.local_kv))
            N.call("mib_qk_norm_rope_bf16", N.ptr(qkv), B * T, qkv.stride(-2), T, self.local_heads, self.local_kv,
                   a.head_dim, N.ptr(self.q_norm), N.ptr(self.k_norm), float(a.eps), N.ptr(cos), N.ptr(sin),
                   N.ptr(q), N.ptr(k), N.ptr(v), N.stream_ptr(h.device))
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                           enable_gqa=self.local_heads != self.local_kv)
        o = o.transpose(1, 2).reshape(B, T, self.local_heads * a.head_dim).float()
        xs = self.o_proj.new_input()
        xs.slice_data_imp(self.engine, o)
        return self.o_proj.partial_sliced(xs)

    def mlp_partial(self, h):
        """SwiGLU MLP up to this rank's down_proj partial sum (before the all-reduce)."""
        xs = self.gate_up_proj.new_input()
        self.engine.slice_rmsnorm_input(xs, h, self.post_norm, self.arch.eps)
        gu = self.gate_up_proj.forward_sliced(xs)
        ms = self.down_proj.new_input()
        self.engine.slice_swiglu_input(ms, gu, self.local_inter)
        return self.down_proj.partial_sliced(ms)


class Qwen3CimPrefill(torch.nn.Module):
    """Random-init Qwen3-architecture model; ``forward(ids)`` returns the mean next-token loss."""

    def __init__(self, engine, arch: Qwen3Arch = Qwen3Arch(), spec: CimSpec = CimSpec(), seed: int = 0,
                 device=None, group=None, weights=None, shard_head_over=None):
        """``weights``: optional state dict in Hugging Face Qwen3 naming (``model.embed_tokens.weight``,
        ``model.layers.{i}.self_attn.q_proj.weight``, ..., ``model.norm.weight``, ``lm_head.weight``), the
        checkpoint the reference loads (memintelli/NN_models/Qwen3.py:136-140); random init otherwise.
        ``group``: the ranks every crossbar is sharded over (None: all ranks).  ``shard_head_over``: a
        group over which only lm_head is sharded, the layers being whole on each rank (``group`` must then
        hold one rank); each rank's forward takes its own sequences and returns the loss of all of them."""
        super().__init__()
        device = device or engine.device
        self.arch, self.group, self.engine = arch, group, engine
        # sequences per forward are processed in this many groups when sharded, so that each group's
        # all-reduces overlap the other groups' crossbar work (see _layers_overlapped)
        self.micro_batches = 2
        # True: read-noise pass of layer i + 1 (of lm_head after the last layer) launched as a background pass
        # on a side stream while layer i runs (DPETensor.draw_read_noise).  Off: on one B200 the background
        # blocks took more from the crossbar kernel beside them than the pass costs in front of its multiply
        # (one 2048-token rank's forward 128.3 -> 146.4 ms; the 8 x 2048 bench 17.49 k -> 17.23 k tokens/s).
        self.prefetch_noise = False
        distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.head_group = group if shard_head_over is None else shard_head_over
        self.head_world = dist.get_world_size(self.head_group) if distributed else 1
        self.head_gather = shard_head_over is not None and self.head_world > 1
        if self.head_gather and self.world > 1:
            raise ValueError("shard_head_over needs whole decoder layers on every rank (a group of one rank)")
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        if weights is None:
            embed = torch.randn(arch.vocab, arch.hidden, generator=gen, device=device) * 0.02
        else:
            embed = weights["model.embed_tokens.weight"].to(device=device, dtype=torch.float32)
        self.embed = torch.nn.Parameter(embed, requires_grad=False)
        self.layers = torch.nn.ModuleList(
            Qwen3CimLayer(arch, engine, spec, gen, device, group, weights, f"model.layers.{i}.")
            for i in range(arch.layers))
        norm = torch.ones(arch.hidden, device=device) if weights is None else \
            weights["model.norm.weight"].to(device=device, dtype=torch.float32)
        self.norm = torch.nn.Parameter(norm, requires_grad=False)
        w_head = torch.randn(arch.vocab, arch.hidden, generator=gen, device=device) * 0.02 if weights is None else \
            weights["lm_head.weight"].to(device=device, dtype=torch.float32)
        self.lm_head = ColumnShardedLinearMem(engine, w_head, None, spec.input_slice, spec.weight_slice,
                                              group=self.head_group, device=device, **spec.kwargs())
        del w_head
        self._rope = {}

    def cim_linears(self):
        for layer in self.layers:
            for name in ("qkv_proj", "o_proj", "gate_up_proj", "down_proj"):
                yield getattr(layer, name).local
        yield self.lm_head.local

    def set_attention_dtype(self, dtype):
        """bf16 attention (default; the benchmark's) or float32 (the reference model's eager attention)."""
        for layer in self.layers:
            layer.attn_dtype = dtype

    def _draw_noise(self, layer_or_head, uses, background):
        """One read-variation draw for each crossbar array of a layer (or lm_head), shared by its next
        ``uses`` multiplies (DPETensor.draw_read_noise)."""
        if layer_or_head is self.lm_head:
            arrays = [self.lm_head]
        else:
            arrays = [layer_or_head.qkv_proj, layer_or_head.o_proj, layer_or_head.gate_up_proj,
                      layer_or_head.down_proj]
        for arr in arrays:
            self.engine.draw_read_noise(arr.local.weight_sliced, uses=uses, background=background)

    def _hidden(self, ids):
        a = self.arch
        B, T = ids.shape
        if T not in self._rope:
            self._rope[T] = rope_cache(T, a.head_dim, a.rope_theta, ids.device)
        cos, sin = self._rope[T]                             # (T, head_dim) each
        h = F.embedding(ids, self.embed)
        if self.world > 1 and self.micro_batches > 1 and B >= self.micro_batches:
            return self._layers_overlapped(h, cos, sin)
        layers = list(self.layers)
        for i, layer in enumerate(layers):
            if self.prefetch_noise:
                # the next layer's (or lm_head's) read-noise pass runs in the background of this layer
                self._draw_noise(layers[i + 1] if i + 1 < len(layers) else self.lm_head, 1, True)
            h = layer(h, cos, sin)
        return h

    def _gather_head_inputs(self, h, ids):
        """All ranks' final hidden states and ids, in rank order (lm_head sharded over data-parallel ranks)."""
        if not self.head_gather:
            return h, ids
        hg = torch.empty((self.head_world * h.shape[0],) + tuple(h.shape[1:]), dtype=h.dtype, device=h.device)
        dist.all_gather_into_tensor(hg, h.contiguous(), group=self.head_group)
        ig = torch.empty((self.head_world * ids.shape[0],) + tuple(ids.shape[1:]), dtype=ids.dtype, device=ids.device)
        dist.all_gather_into_tensor(ig, ids.contiguous(), group=self.head_group)
        return hg, ig

    @torch.no_grad()
    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        h, ids = self._gather_head_inputs(self._hidden(ids), ids)
        xs = self.lm_head.new_input()
        self.engine.slice_rmsnorm_input(xs, h[:, :-1], self.norm, self.arch.eps)
        logits = self.lm_head.forward_sliced(xs)             # (B, T-1, V_local)
        target = ids[:, 1:]
        return self._sharded_ce(logits, target)

    @torch.no_grad()
    def logits(self, ids: torch.Tensor) -> torch.Tensor:
        """(B, T, V_local) logits of every position (this rank's vocabulary columns; with
        ``shard_head_over``, of every rank's sequences in rank order)."""
        h, ids = self._gather_head_inputs(self._hidden(ids), ids)
        xs = self.lm_head.new_input()
        self.engine.slice_rmsnorm_input(xs, h, self.norm, self.arch.eps)
        return self.lm_head.forward_sliced(xs)

    def _layers_overlapped(self, h, cos, sin):
        """The decoder layers over ``micro_batches`` groups of sequences, with every o/down all-reduce
        asynchronous: a group's all-reduce runs while the other groups' crossbars compute, and is
        waited for only where that group next needs its hidden state.  Per token the arithmetic is
        that of ``Qwen3CimLayer.forward``."""
        hs = list(torch.chunk(h, self.micro_batches, dim=0))
        pending = [None] * len(hs)          # (partial output, all-reduce work) per group

        def settle(m):
            if pending[m] is not None:
                y, work = pending[m]
                work.wait()
                hs[m] = hs[m] + y
                pending[m] = None

        def launch(m, y):
            pending[m] = (y, dist.all_reduce(y, group=self.group, async_op=True))

        # every array is multiplied once per group: one read-variation draw per array and forward, shared
        # by the groups as the sequences of one reference call share it
        layers = list(self.layers)
        uses = len(hs)
        self._draw_noise(layers[0], uses, False)     # nothing runs yet for a background pass to overlap
        for i, layer in enumerate(layers):
            if i + 1 < len(layers):
                self._draw_noise(layers[i + 1], uses, self.prefetch_noise)
            elif self.prefetch_noise:
                self._draw_noise(self.lm_head, 1, True)
            for m in range(len(hs)):
                settle(m)
                launch(m, layer.attn_partial(hs[m], cos, sin))
            for m in range(len(hs)):
                settle(m)
                launch(m, layer.mlp_partial(hs[m]))
        for m in range(len(hs)):
            settle(m)
        return torch.cat(hs, dim=0)

    def _sharded_ce(self, logits, target):
        """Mean cross-entropy over column-sharded logits (no gather of the vocabulary).  One pass over this
        rank's logits (mib_row_logsumexp) gives each row's maximum, sum of exp(x - max) and target logit;
        the ranks' partials combine as M = max, S = sum s exp(m - M), loss = log S + M - target."""
        lo = self.lm_head.lo
        V = logits.shape[-1]
        x = logits.reshape(-1, V)
        if x.stride(-1) != 1:
            x = x.contiguous()
        tgt_ids = target.reshape(-1).to(torch.int64).contiguous()
        rows = x.shape[0]
        lmax, sexp, tgt = (torch.empty(rows, dtype=torch.float32, device=x.device) for _ in range(3))
        N.call("mib_row_logsumexp", N.ptr(x), rows, V, x.stride(0), N.ptr(tgt_ids), lo, N.ptr(lmax), N.ptr(sexp),
               N.ptr(tgt), N.stream_ptr(x.device))
        if self.head_world > 1:
            gmax = lmax.clone()
            dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=self.head_group)
            sexp = sexp * torch.exp(lmax - gmax)
            dist.all_reduce(sexp, group=self.head_group)
            dist.all_reduce(tgt, group=self.head_group)
            lmax = gmax
        return (torch.log(sexp) + lmax - tgt).mean()
