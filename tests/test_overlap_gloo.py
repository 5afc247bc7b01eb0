"""The overlapped all-reduce schedule of the sharded Qwen3 prefill on 2 CPU ranks (gloo).

``Qwen3CimPrefill._layers_overlapped`` runs the decoder layers over groups of sequences with
asynchronous all-reduces of the o/down partial sums.  With stand-in layers (deterministic,
rank-dependent partials) its result must equal the synchronous per-layer form
h += all_reduce(attn_partial(h)); h += all_reduce(mlp_partial(h)).
"""
import os
import socket
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _Layer:
    """Partial sums that depend on the rank and on the layer, like a row-sharded o/down crossbar."""

    def __init__(self, rank, idx):
        self.a = 0.05 * (rank + 1) * (idx + 1)
        self.b = 0.02 * (rank + 2) / (idx + 1)

    def attn_partial(self, h, cos, sin):
        return torch.sin(h) * self.a

    def mlp_partial(self, h):
        return torch.tanh(h) * self.b


def _worker(rank, world, port, q):
    from memintelli_flash_b200.qwen3_prefill import Qwen3CimPrefill
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layers = [_Layer(rank, i) for i in range(5)]
        h0 = torch.randn(6, 7, 16, generator=torch.Generator().manual_seed(1), dtype=torch.float64)
        ref = h0.clone()
        for layer in layers:
            y = layer.attn_partial(ref, None, None)
            dist.all_reduce(y)
            ref = ref + y
            z = layer.mlp_partial(ref)
            dist.all_reduce(z)
            ref = ref + z
        for groups in (2, 3):
            draws = []                 # (array owner, uses, background) of every read-noise draw
            fake = SimpleNamespace(micro_batches=groups, layers=layers, group=None, prefetch_noise=True,
                                   lm_head="lm_head", _draw_noise=lambda what, uses, bg: draws.append((what, uses, bg)))
            got = Qwen3CimPrefill._layers_overlapped(fake, h0.clone(), None, None)
            # one draw per layer shared by the groups: layer 0 up front, each next layer (then lm_head, used
            # once) in the background of the layer before it
            assert draws == [(layers[0], groups, False)] + [(l, groups, True) for l in layers[1:]] + \
                [("lm_head", 1, True)]
            q.put((rank, groups, float((got - ref).abs().max())))
    finally:
        dist.destroy_process_group()


def test_overlapped_schedule_matches_synchronous_layers():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(4)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, groups, err in results:
        assert err == 0.0, (rank, groups, err)
