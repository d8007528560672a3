"""Write a seeded random-init QuickLM checkpoint (config.json + BF16 safetensors).

Architecture = benchmark configuration 3 (a Qwen3.5-style hybrid decoder): 24 layers,
hidden 1024, 3 Gated-DeltaNet layers per full-attention layer (16 query heads,
4 KV heads, head_dim 64, output-gated), DeltaNet 16 heads x 128, SwiGLU MLP
3584, vocab 151936 (lm_head tied to the embedding), RoPE theta 1e6.
Linear weights ~ N(0, 0.02^2) from numpy default_rng(seed), drawn in a fixed
order and rounded to BF16 (round-to-nearest-even); zero-centred RMSNorm gains
0 (QuickLM applies 1 + w), DeltaNet head-norm gains 1, A_log and dt_bias 0.
`--width/--layers/--inter` build the wider config-5 variant.

    python integration/make_checkpoint.py OUT_DIR [--seed 7] [--prompt-len 64]

Also writes OUT_DIR/prompt_ids.txt: prompt-len uniform random token ids.
"""
from __future__ import annotations

import argparse
import json
import os
import struct

import numpy as np


def to_bf16(a: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def build(out_dir: str, seed: int = 7, hidden: int = 1024, layers: int = 24, inter: int = 3584,
          vocab: int = 151936, heads: int = 16, kv_heads: int = 4, head_dim: int = 64, lin_heads: int = 16,
          lin_dim: int = 128, prompt_len: int = 64, device_rng: bool = False) -> dict:
    """device_rng: draw the N(0, 0.02^2) weights with torch's generator on the
    GPU (seeded; the same distribution, other numbers) — for the multi-GB
    configuration-5 checkpoint, which numpy would take minutes to draw."""
    os.makedirs(out_dir, exist_ok=True)
    rng = np.random.default_rng(seed)
    gen = None
    if device_rng:
        import torch
        gen = torch.Generator(device="cuda").manual_seed(seed)
    layer_types = ["full_attention" if i % 4 == 3 else "linear_attention" for i in range(layers)]
    cfg = {"model_type": "qwen3_5_text", "vocab_size": vocab, "hidden_size": hidden, "intermediate_size": inter,
           "num_hidden_layers": layers, "num_attention_heads": heads, "num_key_value_heads": kv_heads,
           "head_dim": head_dim, "linear_num_key_heads": lin_heads, "linear_key_head_dim": lin_dim,
           "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "tie_word_embeddings": True, "layer_types": layer_types}
    tensors = []  # (name, shape, generator)

    def w(name, *shape):
        tensors.append((name, shape, "normal"))

    def const(name, value, *shape):
        tensors.append((name, shape, float(value)))

    w("model.embed_tokens.weight", vocab, hidden)
    lin = lin_heads * lin_dim
    for i in range(layers):
        p = f"model.layers.{i}."
        const(p + "input_layernorm.weight", 0.0, hidden)
        const(p + "post_attention_layernorm.weight", 0.0, hidden)
        w(p + "mlp.gate_proj.weight", inter, hidden)
        w(p + "mlp.up_proj.weight", inter, hidden)
        w(p + "mlp.down_proj.weight", hidden, inter)
        if layer_types[i] == "full_attention":
            w(p + "self_attn.q_proj.weight", 2 * heads * head_dim, hidden)
            w(p + "self_attn.k_proj.weight", kv_heads * head_dim, hidden)
            w(p + "self_attn.v_proj.weight", kv_heads * head_dim, hidden)
            w(p + "self_attn.o_proj.weight", hidden, heads * head_dim)
            const(p + "self_attn.q_norm.weight", 0.0, head_dim)
            const(p + "self_attn.k_norm.weight", 0.0, head_dim)
        else:
            w(p + "linear_attn.in_proj_qkv.weight", 3 * lin, hidden)
            w(p + "linear_attn.in_proj_z.weight", lin, hidden)
            w(p + "linear_attn.in_proj_b.weight", lin_heads, hidden)
            w(p + "linear_attn.in_proj_a.weight", lin_heads, hidden)
            w(p + "linear_attn.conv1d.weight", 3 * lin, 1, 4)
            const(p + "linear_attn.norm.weight", 1.0, lin_dim)
            const(p + "linear_attn.A_log", 0.0, lin_heads)
            const(p + "linear_attn.dt_bias", 0.0, lin_heads)
            w(p + "linear_attn.out_proj.weight", hidden, lin)
    const("model.norm.weight", 0.0, hidden)

    header, offset = {}, 0
    for name, shape, _ in tensors:
        nbytes = int(np.prod(shape)) * 2
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    hjson = json.dumps(header).encode()
    hjson += b" " * ((8 - len(hjson) % 8) % 8)
    with open(os.path.join(out_dir, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hjson)))
        f.write(hjson)
        for name, shape, kind in tensors:
            n = int(np.prod(shape))
            if kind == "normal":
                left, step = n, 1 << 24
                while left:
                    k = min(left, step)
                    if gen is not None:
                        import torch
                        t = (torch.randn(k, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
                        f.write(t.view(torch.int16).cpu().numpy().tobytes())
                    else:
                        f.write(to_bf16(rng.standard_normal(k) * 0.02).tobytes())
                    left -= k
            else:
                f.write(to_bf16(np.full(n, kind, np.float32)).tobytes())
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    prompt = np.random.default_rng(seed + 1).integers(0, vocab, size=prompt_len)
    with open(os.path.join(out_dir, "prompt_ids.txt"), "w") as f:
        f.write(" ".join(str(int(t)) for t in prompt) + "\n")
    return cfg


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("out_dir")
    ap.add_argument("--seed", type=int, default=7)
    ap.add_argument("--prompt-len", type=int, default=64)
    ap.add_argument("--width", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--inter", type=int, default=3584)
    a = ap.parse_args()
    build(a.out_dir, a.seed, hidden=a.width, layers=a.layers, inter=a.inter, prompt_len=a.prompt_len)
