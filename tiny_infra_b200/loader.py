"""Weights in the reference's extracted checkpoint format (engine/loader.py:9-79): one
.safetensors file with flat custom keys (``token_embeddings``, ``blocks.{i}.attn.q_proj.weight``,
``blocks.{i}.mlp.gate_proj`` ...), mapped to the reference module's state-dict names and loaded
straight into this package's fused layouts (q/k/v in one matrix, gate/up rows interleaved in
groups of 8) by :meth:`Qwen2ForCausalLM.load_reference_state_dict`.
"""
from __future__ import annotations

import torch

from .config import QwenConfig
from .qwen2 import Qwen2ForCausalLM

# (custom key suffix, reference key suffix) per decoder block (engine/loader.py:41-71)
_BLOCK_KEYS = (
    ("attn.q_proj.weight", "self_attn.q_proj.weight"),
    ("attn.q_proj.bias", "self_attn.q_proj.bias"),
    ("attn.k_proj.weight", "self_attn.k_proj.weight"),
    ("attn.k_proj.bias", "self_attn.k_proj.bias"),
    ("attn.v_proj.weight", "self_attn.v_proj.weight"),
    ("attn.v_proj.bias", "self_attn.v_proj.bias"),
    ("attn.out_proj.weight", "self_attn.o_proj.weight"),
    ("mlp.gate_proj", "mlp.gate_proj.weight"),
    ("mlp.up_proj", "mlp.up_proj.weight"),
    ("mlp.down_proj", "mlp.down_proj.weight"),
    ("attn_norm", "input_layernorm.weight"),
    ("mlp_norm", "post_attention_layernorm.weight"),
)


def reference_key_map(num_layers: int) -> dict[str, str]:
    """Checkpoint key -> reference state-dict key (engine/loader.py:34-72)."""
    m = {"token_embeddings": "model.embed_tokens.weight",
         "final_norm_weight": "model.norm.weight",
         "lm_head": "lm_head.weight"}
    for i in range(num_layers):
        for src, dst in _BLOCK_KEYS:
            m[f"blocks.{i}.{src}"] = f"model.layers.{i}.{dst}"
    return m


def read_reference_checkpoint(path: str, num_layers: int, device="cpu") -> dict:
    """The checkpoint's tensors under the reference's state-dict names, read onto ``device``.
    As the reference's strict ``load_state_dict`` (engine/loader.py:75), a missing key raises
    KeyError and an unexpected one RuntimeError.  An lm_head equal to the embedding becomes the
    same tensor (tied embeddings, one buffer)."""
    from safetensors.torch import load_file
    raw = load_file(path, device=str(device))
    m = reference_key_map(num_layers)
    missing = [k for k in m if k not in raw]
    if missing:
        raise KeyError(f"checkpoint {path} misses {len(missing)} key(s), e.g. {missing[:3]}")
    unexpected = sorted(set(raw) - set(m))
    if unexpected:
        raise RuntimeError(f"Unexpected key(s) in checkpoint {path}: {unexpected[:3]}")
    sd = {m[k]: v for k, v in raw.items()}
    emb, lm = sd["model.embed_tokens.weight"], sd["lm_head.weight"]
    if lm.shape == emb.shape and torch.equal(lm, emb):
        sd["lm_head.weight"] = emb
    return sd


def load_qwen(model_path: str, device="cuda", dtype: torch.dtype = torch.bfloat16,
              config: QwenConfig | None = None) -> Qwen2ForCausalLM:
    """engine/loader.py:9-79: read the extracted checkpoint, map its names and load the weights
    (cast to ``dtype``) onto ``device``."""
    config = config or QwenConfig()
    sd = read_reference_checkpoint(model_path, config.num_layers, device=device)
    return Qwen2ForCausalLM(config, device=device, dtype=dtype).load_reference_state_dict(sd)
