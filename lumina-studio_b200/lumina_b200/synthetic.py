"""Seeded synthetic workloads for the Lumina decode path.

There is no dataset or checkpoint on this path: the workloads are seeded
random Llama-style decoders, quantized to Lumina codes. Shapes:

  * ``TINY``  — 4 layers, d 256, 4 heads x 64, SwiGLU 688, vocab 4096,
    RoPE theta 1e4 (the reference's CPU-runnable mini_lm shape).
  * ``LLAMA7B`` — 32 layers, d 4096, 32 heads x 128, SwiGLU 11008,
    vocab 32000, RoPE theta 1e4.

Weights of every 2-D matrix are N(0, 0.02) drawn in the fixed order of
``tensor_order``; RMSNorm weights are ones. Tensor names follow the HF Llama
layout that the reference's ChatModel reads (chat.py:240-303).
"""
from __future__ import annotations

import numpy as np

TINY = {"name": "tiny", "num_hidden_layers": 4, "hidden_size": 256,
        "num_attention_heads": 4, "num_key_value_heads": 4,
        "intermediate_size": 688, "vocab_size": 4096, "rope_theta": 10000.0}

LLAMA7B = {"name": "llama7b", "num_hidden_layers": 32, "hidden_size": 4096,
           "num_attention_heads": 32, "num_key_value_heads": 32,
           "intermediate_size": 11008, "vocab_size": 32000, "rope_theta": 10000.0}


def tensor_order(cfg: dict) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) in generation order."""
    d, f, v = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    nh, nk = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    hd = d // nh
    out = [("model.embed_tokens.weight", (v, d))]
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}."
        out += [(p + "input_layernorm.weight", (d,)),
                (p + "self_attn.q_proj.weight", (nh * hd, d)),
                (p + "self_attn.k_proj.weight", (nk * hd, d)),
                (p + "self_attn.v_proj.weight", (nk * hd, d)),
                (p + "self_attn.o_proj.weight", (d, nh * hd)),
                (p + "post_attention_layernorm.weight", (d,)),
                (p + "mlp.gate_proj.weight", (f, d)),
                (p + "mlp.up_proj.weight", (f, d)),
                (p + "mlp.down_proj.weight", (d, f))]
    out.append(("lm_head.weight", (v, d)))
    return out


def host_weights(cfg: dict, seed: int = 0) -> dict[str, np.ndarray]:
    """fp32 weights on the host (for shapes the CPU can hold comfortably)."""
    rng = np.random.default_rng(seed)
    w = {}
    for name, shape in tensor_order(cfg):
        if len(shape) == 1:
            w[name] = np.ones(shape, dtype=np.float32)
        else:
            w[name] = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    return w


def prompt_ids(cfg: dict, n: int, seed: int = 0) -> list[int]:
    """Uniform random prompt ids from a seeded generator."""
    rng = np.random.default_rng(seed + 1)
    return [int(t) for t in rng.integers(0, cfg["vocab_size"], n)]


def hf_cfg(cfg: dict) -> dict:
    """The HF-style config dict the reference's ChatModel reads."""
    return {k: cfg[k] for k in ("num_hidden_layers", "hidden_size", "num_attention_heads",
                                "num_key_value_heads", "vocab_size", "intermediate_size")}
