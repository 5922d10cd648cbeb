"""Parameter shapes of the model families the benchmarks and harnesses use.

Random-init weights of these architectures stand in for checkpoints (there is
no network for downloads). Tensor-parallel sharding follows the usual
Megatron / vLLM split: column-parallel q/k/v/gate/up (output rows divided),
row-parallel o/down (input columns divided), vocab-parallel embedding and LM
head, replicated norms.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch


@dataclass(frozen=True)
class DecoderSpec:
    name: str
    layers: int
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    qkv_bias: bool
    tied_embeddings: bool = False

    @property
    def q_out(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_out(self) -> int:
        return self.kv_heads * self.head_dim


QWEN2_5_32B = DecoderSpec("Qwen2.5-32B", layers=64, hidden=5120, ffn=27648, heads=40, kv_heads=8, head_dim=128,
                          vocab=152064, qkv_bias=True)
LLAMA3_8B = DecoderSpec("Llama-3-8B", layers=32, hidden=4096, ffn=14336, heads=32, kv_heads=8, head_dim=128,
                        vocab=128256, qkv_bias=False)
MODELS = {"qwen2.5-32b": QWEN2_5_32B, "llama-3-8b": LLAMA3_8B}


def _div(n: int, tp: int, what: str) -> int:
    if n % tp:
        raise ValueError(f"{what} ({n}) is not divisible by tp={tp}")
    return n // tp


def param_shapes(spec: DecoderSpec, tp_rank: int = 0, tp_size: int = 1,
                 layers: Optional[int] = None) -> List[Tuple[str, Tuple[int, ...]]]:
    """Ordered (name, shape) of one tensor-parallel shard (HF parameter names)."""
    if not 0 <= tp_rank < tp_size:
        raise ValueError("tp_rank out of range")
    h = spec.hidden
    q = _div(spec.q_out, tp_size, "q heads")
    kv = _div(spec.kv_out, tp_size, "kv heads")
    f = _div(spec.ffn, tp_size, "ffn")
    v = _div(spec.vocab, tp_size, "vocab")
    out: List[Tuple[str, Tuple[int, ...]]] = [("model.embed_tokens.weight", (v, h))]
    for i in range(spec.layers if layers is None else layers):
        p = f"model.layers.{i}."
        out += [(p + "input_layernorm.weight", (h,)),
                (p + "self_attn.q_proj.weight", (q, h))]
        if spec.qkv_bias:
            out.append((p + "self_attn.q_proj.bias", (q,)))
        out.append((p + "self_attn.k_proj.weight", (kv, h)))
        if spec.qkv_bias:
            out.append((p + "self_attn.k_proj.bias", (kv,)))
        out.append((p + "self_attn.v_proj.weight", (kv, h)))
        if spec.qkv_bias:
            out.append((p + "self_attn.v_proj.bias", (kv,)))
        out += [(p + "self_attn.o_proj.weight", (h, q)),
                (p + "post_attention_layernorm.weight", (h,)),
                (p + "mlp.gate_proj.weight", (f, h)),
                (p + "mlp.up_proj.weight", (f, h)),
                (p + "mlp.down_proj.weight", (h, f))]
    out.append(("model.norm.weight", (h,)))
    if not spec.tied_embeddings:
        out.append(("lm_head.weight", (v, h)))
    return out


def num_params(shapes) -> int:
    n = 0
    for _, s in shapes:
        k = 1
        for d in s:
            k *= d
        n += k
    return n


def random_init(shapes, device, dtype=torch.bfloat16, std: float = 0.02, seed: int = 0) -> Dict[str, torch.Tensor]:
    """N(0, std) weights (norm weights N(1, std)), one allocation per tensor."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = {}
    for name, shape in shapes:
        t = torch.empty(shape, dtype=dtype, device=device)
        t.normal_(1.0 if name.endswith("norm.weight") else 0.0, std, generator=g)
        out[name] = t
    return out


def random_init_flat(shapes, device, dtype=torch.bfloat16, std: float = 0.02, seed: int = 0, align: int = 256):
    """Like ``random_init``, but every tensor is a view of one flat buffer
    (each starting on an ``align``-byte boundary), the layout data-parallel
    trainers keep their parameters in. Returns (flat uint8 buffer, name -> view)."""
    esz = torch.tensor([], dtype=dtype).element_size()
    offs, total = [], 0
    for _, shape in shapes:
        n = 1
        for d in shape:
            n *= d
        offs.append(total)
        total += (n * esz + align - 1) // align * align
    flat = torch.empty(max(total, 1), dtype=torch.uint8, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = {}
    for (name, shape), off in zip(shapes, offs):
        n = 1
        for d in shape:
            n *= d
        t = flat[off:off + n * esz].view(dtype).view(shape)
        t.normal_(1.0 if name.endswith("norm.weight") else 0.0, std, generator=g)
        out[name] = t
    return flat, out


def pick_changed(names, fraction: float, seed: int) -> List[int]:
    """Indices of a seeded `fraction` of `names` (sorted)."""
    gen = torch.Generator()
    gen.manual_seed(seed)
    k = max(1, int(round(fraction * len(names))))
    return sorted(torch.randperm(len(names), generator=gen)[:k].tolist())


@dataclass(frozen=True)
class KVCacheSpec:
    """Paged KV cache: one block holds `block_tokens` tokens of K and V for
    every layer and KV head (the unit that is evicted and restored)."""
    layers: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    block_tokens: int = 16
    dtype: torch.dtype = torch.bfloat16

    @property
    def block_bytes(self) -> int:
        esz = torch.empty((), dtype=self.dtype).element_size()
        return 2 * self.layers * self.kv_heads * self.head_dim * self.block_tokens * esz

    def blocks_for(self, nbytes: int) -> int:
        return nbytes // self.block_bytes
