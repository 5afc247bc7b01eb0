"""A small Qwen3-architecture model shared by the fixture script and the GPU model-parity test.

``state_dict(seed)`` draws every weight from one seeded CPU generator in a fixed
order and returns it under the Hugging Face Qwen3 parameter names, so the same
weights can be loaded into ``transformers``' Qwen3ForCausalLM (the reference
wraps that model and swaps its nn.Linear layers for LinearMem,
memintelli/NN_models/Qwen3.py:82-106) and into ``Qwen3CimPrefill``.
"""
from __future__ import annotations

import torch

CONFIG = dict(vocab=512, hidden=256, intermediate=512, layers=2, heads=4, kv_heads=2, head_dim=64,
              rope_theta=1e6, eps=1e-6)
BATCH, SEQ = 2, 96


def hf_config():
    from transformers import Qwen3Config
    c = CONFIG
    cfg = Qwen3Config(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["intermediate"],
                      num_hidden_layers=c["layers"], num_attention_heads=c["heads"],
                      num_key_value_heads=c["kv_heads"], head_dim=c["head_dim"], rope_theta=c["rope_theta"],
                      rms_norm_eps=c["eps"], tie_word_embeddings=False, attention_bias=False,
                      max_position_embeddings=4 * SEQ)
    cfg._attn_implementation = "eager"
    return cfg


def state_dict(seed: int = 7):
    """Weights in Hugging Face Qwen3 naming; linears ~ N(0, 1/in_features), norms ~ 1 + N(0, 0.1^2)."""
    c = CONFIG
    g = torch.Generator().manual_seed(seed)
    H, I, D = c["hidden"], c["intermediate"], c["head_dim"]

    def lin(o, i):
        return torch.randn(o, i, generator=g) / i ** 0.5

    def norm(n):
        return 1.0 + 0.1 * torch.randn(n, generator=g)

    sd = {"model.embed_tokens.weight": torch.randn(c["vocab"], H, generator=g)}
    for l in range(c["layers"]):
        p = f"model.layers.{l}."
        sd[p + "self_attn.q_proj.weight"] = lin(c["heads"] * D, H)
        sd[p + "self_attn.k_proj.weight"] = lin(c["kv_heads"] * D, H)
        sd[p + "self_attn.v_proj.weight"] = lin(c["kv_heads"] * D, H)
        sd[p + "self_attn.o_proj.weight"] = lin(H, c["heads"] * D)
        sd[p + "self_attn.q_norm.weight"] = norm(D)
        sd[p + "self_attn.k_norm.weight"] = norm(D)
        sd[p + "mlp.gate_proj.weight"] = lin(I, H)
        sd[p + "mlp.up_proj.weight"] = lin(I, H)
        sd[p + "mlp.down_proj.weight"] = lin(H, I)
        sd[p + "input_layernorm.weight"] = norm(H)
        sd[p + "post_attention_layernorm.weight"] = norm(H)
    sd["model.norm.weight"] = norm(H)
    sd["lm_head.weight"] = lin(c["vocab"], H)
    return sd


def token_ids(seed: int = 3):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, CONFIG["vocab"], (BATCH, SEQ), generator=g)
