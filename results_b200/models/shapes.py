"""Synthetic state_dicts of the two models the reference's RL weight-update
results are quoted on (csv/weight_update_rl_GLM4_9B.csv and
csv/weight_update_rl_qwen3.5_35B_A3B.csv of the reference).

Weights are random N(0, 0.02) in bf16, norms 1.0 (the weight-update benchmark configurations);
tensor names follow the Hugging Face checkpoints so manifests and per-tensor
CSV rows line up with the reference's (e.g. ``mlp.gate_up_proj`` = 214 MB).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class TensorSpec:
    name: str
    shape: tuple
    kind: str = "weight"  # "weight" | "norm" | "bias"

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


def glm4_9b_specs(layers: int = 40, hidden: int = 4096, heads: int = 32, kv_heads: int = 2,
                  head_dim: int = 128, ffn: int = 13696, vocab: int = 151552) -> list[TensorSpec]:
    """GLM-4-9B-0414 layout: 40 layers, GQA 32/2 x 128, fused SwiGLU 13696, untied embeddings."""
    q, kv = heads * head_dim, kv_heads * head_dim
    out = [TensorSpec("model.embed_tokens.weight", (vocab, hidden))]
    for i in range(layers):
        p = f"model.layers.{i}."
        out += [
            TensorSpec(p + "input_layernorm.weight", (hidden,), "norm"),
            TensorSpec(p + "self_attn.q_proj.weight", (q, hidden)),
            TensorSpec(p + "self_attn.q_proj.bias", (q,), "bias"),
            TensorSpec(p + "self_attn.k_proj.weight", (kv, hidden)),
            TensorSpec(p + "self_attn.k_proj.bias", (kv,), "bias"),
            TensorSpec(p + "self_attn.v_proj.weight", (kv, hidden)),
            TensorSpec(p + "self_attn.v_proj.bias", (kv,), "bias"),
            TensorSpec(p + "self_attn.o_proj.weight", (hidden, q)),
            TensorSpec(p + "post_self_attn_layernorm.weight", (hidden,), "norm"),
            TensorSpec(p + "post_attention_layernorm.weight", (hidden,), "norm"),
            TensorSpec(p + "mlp.gate_up_proj.weight", (2 * ffn, hidden)),
            TensorSpec(p + "mlp.down_proj.weight", (hidden, ffn)),
            TensorSpec(p + "post_mlp_layernorm.weight", (hidden,), "norm"),
        ]
    out += [TensorSpec("model.norm.weight", (hidden,), "norm"), TensorSpec("lm_head.weight", (vocab, hidden))]
    return out


def qwen35_a3b_specs(layers: int = 40, hidden: int = 2048, heads: int = 16, kv_heads: int = 2,
                     head_dim: int = 256, experts: int = 256, moe_ffn: int = 512, shared_ffn: int = 512,
                     vocab: int = 151936) -> list[TensorSpec]:
    """~35B-total / ~3B-active MoE: 256 routed experts (SwiGLU 512, top-8) + 1 shared expert.

    Routed experts are coalesced per layer into two stacked tensors
    (gate_up [E, 2*ffn, hidden] and down [E, hidden, ffn]), i.e. chunks far
    above 64 MB, as the MoE weight-update configuration specifies.
    """
    q, kv = heads * head_dim, kv_heads * head_dim
    out = [TensorSpec("model.embed_tokens.weight", (vocab, hidden))]
    for i in range(layers):
        p = f"model.layers.{i}."
        out += [
            TensorSpec(p + "input_layernorm.weight", (hidden,), "norm"),
            TensorSpec(p + "self_attn.q_proj.weight", (q, hidden)),
            TensorSpec(p + "self_attn.k_proj.weight", (kv, hidden)),
            TensorSpec(p + "self_attn.v_proj.weight", (kv, hidden)),
            TensorSpec(p + "self_attn.o_proj.weight", (hidden, q)),
            TensorSpec(p + "self_attn.q_norm.weight", (head_dim,), "norm"),
            TensorSpec(p + "self_attn.k_norm.weight", (head_dim,), "norm"),
            TensorSpec(p + "post_attention_layernorm.weight", (hidden,), "norm"),
            TensorSpec(p + "mlp.gate.weight", (experts, hidden)),
            TensorSpec(p + "mlp.experts.gate_up_proj", (experts, 2 * moe_ffn, hidden)),
            TensorSpec(p + "mlp.experts.down_proj", (experts, hidden, moe_ffn)),
            TensorSpec(p + "mlp.shared_expert.gate_up_proj.weight", (2 * shared_ffn, hidden)),
            TensorSpec(p + "mlp.shared_expert.down_proj.weight", (hidden, shared_ffn)),
            TensorSpec(p + "mlp.shared_expert_gate.weight", (1, hidden)),
        ]
    out += [TensorSpec("model.norm.weight", (hidden,), "norm"), TensorSpec("lm_head.weight", (vocab, hidden))]
    return out


MODELS = {"glm4-9b": glm4_9b_specs, "qwen3.5-35b-a3b": qwen35_a3b_specs}


def total_params(specs) -> int:
    return sum(s.numel for s in specs)


def make_state_dict(specs, device="cuda", dtype=torch.bfloat16, seed: int = 0, std: float = 0.02,
                    empty: bool = False) -> dict[str, torch.Tensor]:
    """Random-init weights N(0, std), norms 1.0, biases N(0, std); or empty tensors."""
    g = torch.Generator(device=device).manual_seed(seed)
    sd = {}
    for s in specs:
        if empty:
            sd[s.name] = torch.empty(s.shape, dtype=dtype, device=device)
        elif s.kind == "norm":
            sd[s.name] = torch.ones(s.shape, dtype=dtype, device=device)
        else:
            t = torch.empty(s.shape, dtype=dtype, device=device)
            # fill in slabs so the fp32 temporary stays small
            flat = t.view(-1)
            step = 1 << 26
            for o in range(0, flat.numel(), step):
                m = min(step, flat.numel() - o)
                flat[o:o + m].copy_(torch.randn(m, device=device, generator=g) * std)
            sd[s.name] = t
    return sd
