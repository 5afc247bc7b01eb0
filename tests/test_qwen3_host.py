"""Host-side structure of the Qwen3-architecture prefill model (no GPU): fused crossbar shards."""
import torch

from memintelli_flash_b200.crossbar_shard import shard_bounds


def test_fused_qkv_shards_keep_whole_heads():
    # q: 16 heads x 128, k/v: 8 heads x 128, sharded per part on 128-column blocks
    for world in (1, 2, 4, 8):
        for rank in range(world):
            q = shard_bounds(2048, 128, world, rank)
            k = shard_bounds(1024, 128, world, rank)
            assert (q[1] - q[0]) == 2048 // world and (k[1] - k[0]) == 1024 // world
            assert q[0] % 128 == 0 and k[0] % 128 == 0
