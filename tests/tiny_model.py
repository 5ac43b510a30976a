"""The tiny random Llama the tier tests decode with (the geometry of the reference's tier tests):
hidden 128, 4 layers, 8 query / 2 KV heads, head_dim 16, bf16, block size 8, a 100-token prompt
(12 sealed blocks + 4 tokens, 11 candidates) and a budget of 3 selected blocks."""

from __future__ import annotations

import copy

import torch

BS = 8
PROMPT = 100
K = 3
CAP = 512


def make_tiny():  # noqa: ANN201
    from transformers import LlamaConfig, LlamaForCausalLM

    from lazykv_b200.attention import IMPLEMENTATION_NAME, install

    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2, head_dim=16,
                      vocab_size=512, max_position_embeddings=4096)
    install(None, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim)
    model = LlamaForCausalLM(copy.deepcopy(cfg))
    model.set_attn_implementation(IMPLEMENTATION_NAME)
    return cfg, model.to(dtype=torch.bfloat16).cuda().eval()


def ids_for(cfg, n: int = PROMPT, extra: int = 40) -> torch.Tensor:  # noqa: ANN001
    gen = torch.Generator(device="cuda").manual_seed(7)
    return torch.randint(0, cfg.vocab_size, (1, n + extra), device="cuda", generator=gen)


def prefilled(model, cfg, n: int = PROMPT, extra: int = 40):  # noqa: ANN001, ANN201
    from lazykv_b200.cache import FullGPUCache
    from lazykv_b200.generate import prefill

    ids = ids_for(cfg, n, extra)
    full = FullGPUCache(cfg.num_hidden_layers, CAP)
    pre = prefill(model, full, ids[:, :n], chunk_size=32)
    return ids, full, pre


def forced(model, cache, pre, ids, steps: int, prompt: int = PROMPT) -> torch.Tensor:  # noqa: ANN001
    from lazykv_b200.generate import teacher_forced_decode

    return torch.stack(list(teacher_forced_decode(model, cache, pre.last_logits, ids[:, prompt : prompt + steps])))


def check_residency(cache) -> None:  # noqa: ANN001
    """Every occupied slot holds the block the tables say (bf16 tier), and the tables agree."""
    for tier in cache.tiers.values():
        sb, bsl = tier.slot_block, tier.block_slot
        for j in range(tier.h):
            for s in range(tier.n_slots):
                b = int(sb[j, s])
                if b < 0:
                    continue
                assert bsl[j, b] == s + 1
                if tier.quant is None:
                    assert torch.equal(tier.pool[s + 1, j].cpu(), tier.host[b, j])
        assert (bsl >= 0).sum() == (sb >= 0).sum()
