"""Host-side logic that runs without a GPU: the API's refusals, the cache plumbing and the
attention hook on a tiny CPU model (whose prefill path is plain SDPA)."""

from __future__ import annotations

import copy

import pytest
import torch

from lazykv_b200.cache import FullGPUCache, PreallocatedLayer
from lazykv_b200.quant import packed_pair_bytes
from lazykv_b200.selection import blocks_for_budget, current_block_mask


def test_record_width_and_budget_arithmetic() -> None:
    assert packed_pair_bytes(16, 64) == 2368 and packed_pair_bytes(64, 64) == 8704 and packed_pair_bytes(8, 16) == 352
    # selection.py:72-74: floor(fraction * tokens / bs) - 2, at least 1
    assert blocks_for_budget(0.25, 8192, 16) == 126
    assert blocks_for_budget(0.001, 1000, 16) == 1
    m = current_block_mask(48, 16, 5, torch.float32, torch.device("cpu"))
    assert (m[..., :37] == 0).all() and torch.isneginf(m[..., 37:]).all()


def test_preallocated_layer_fills_from_the_front_and_refuses_overflow() -> None:
    layer = PreallocatedLayer(10)
    k = torch.randn(1, 2, 4, 8)
    v = torch.randn(1, 2, 4, 8)
    ko, vo = layer.update(k, v)
    assert ko.shape == (1, 2, 4, 8) and torch.equal(ko, k) and torch.equal(vo, v)
    assert layer.get_mask_sizes(1) == (5, 0)
    layer.update(k, v)
    with pytest.raises(RuntimeError, match="overflow"):
        layer.update(k, v)
    layer.truncate(3)
    assert layer.get_seq_length() == 3
    with pytest.raises(ValueError):
        layer.truncate(4)
    with pytest.raises(ValueError, match="batch-size-1"):
        PreallocatedLayer(4).update(torch.randn(2, 2, 1, 8), torch.randn(2, 2, 1, 8))


def test_full_cache_stats_count_resident_bytes() -> None:
    full = FullGPUCache(2, 16)
    for layer in full.layers:
        layer.update(torch.randn(1, 2, 5, 8), torch.randn(1, 2, 5, 8))
    s = full.stats()
    assert s.seq_len == 5 and s.gpu_resident_kv_bytes == 2 * 2 * 5 * 2 * 8 * 4 and s.host_kv_bytes == 0
    assert s.gpu_allocated_kv_bytes == 2 * 2 * 16 * 2 * 8 * 4 and s.gpu_residency_fraction == 1.0


def test_tier_configurations_are_refused_before_any_device_work() -> None:
    from lazykv_b200.exact import ExactTieredCache
    from lazykv_b200.tiered import TieredCache

    full = FullGPUCache(4, 64)
    with pytest.raises(ValueError, match="needs the model"):
        TieredCache(full, 3, 8, 64, prefetch=True)
    with pytest.raises(ValueError, match="unknown fetch"):
        TieredCache(full, 3, 8, 64, fetch="bulk")
    with pytest.raises(ValueError, match="needs fetch='gather'"):
        TieredCache(full, 3, 8, 64, quant="int8")
    with pytest.raises(ValueError, match="zero-copy"):
        TieredCache(full, 3, 8, 64, fetch="zerocopy", record_selection=True)
    with pytest.raises(ValueError, match="zero-copy"):
        TieredCache(full, 3, 8, 64, model=object(), fetch="zerocopy", prefetch=True)  # type: ignore[arg-type]
    with pytest.raises(ValueError, match="zero-copy"):
        TieredCache(full, 3, 8, 64, fetch="zerocopy", replay_selection={})
    with pytest.raises(ValueError, match="maps \\(layer, step\\)"):
        TieredCache(full, 3, 8, 64, replay_selection=[])
    with pytest.raises(ValueError, match="prefetch"):
        ExactTieredCache(full, 3, 8, 64, model=object(), prefetch=True)


def test_install_registers_the_hook_and_refuses_unknown_strategies() -> None:
    from transformers import AttentionInterface

    from lazykv_b200.attention import IMPLEMENTATION_NAME, install, lazykv_attention_forward

    name, checks = install(None, 8, 2, 16)
    assert name == IMPLEMENTATION_NAME and checks == []
    assert AttentionInterface._global_mapping[IMPLEMENTATION_NAME] is lazykv_attention_forward
    with pytest.raises(RuntimeError, match="not available"):
        install("flex_paged", 8, 2, 16)


def test_the_hook_refuses_a_mask_and_batches() -> None:
    from lazykv_b200.attention import lazykv_attention_forward

    q = torch.randn(1, 8, 1, 16)
    kv = torch.randn(1, 2, 4, 16)
    with pytest.raises(RuntimeError, match="owns causality"):
        lazykv_attention_forward(torch.nn.Module(), q, kv, kv, torch.zeros(1, 1, 1, 4))
    with pytest.raises(RuntimeError, match="batch size 1"):
        lazykv_attention_forward(torch.nn.Module(), q.repeat(2, 1, 1, 1), kv.repeat(2, 1, 1, 1), kv.repeat(2, 1, 1, 1), None)


def test_chunked_prefill_through_the_hook_matches_one_pass_on_cpu() -> None:
    """Prefill and dense attention are the hook's SDPA path: chunked prefill into the preallocated
    cache gives the logits of one uncached forward (float32, CPU)."""
    from transformers import LlamaConfig, LlamaForCausalLM

    from lazykv_b200.attention import IMPLEMENTATION_NAME, install
    from lazykv_b200.generate import greedy_decode, prefill

    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                      vocab_size=128, max_position_embeddings=512)
    install()
    model = LlamaForCausalLM(copy.deepcopy(cfg)).eval()
    ids = torch.randint(0, cfg.vocab_size, (1, 37))
    with torch.inference_mode():
        want = model(input_ids=ids).logits[0, -1].float()
    model.set_attn_implementation(IMPLEMENTATION_NAME)
    full = FullGPUCache(cfg.num_hidden_layers, 64)
    pre = prefill(model, full, ids, chunk_size=16)
    assert pre.chunks == 3 and full.layers[0].get_seq_length() == 37
    assert torch.allclose(pre.last_logits, want, atol=1e-4)
    res = greedy_decode(model, full, pre.last_logits, 3)
    assert len(res.tokens) == 4 and len(res.wall_s) == len(res.event_s) == 3 and full.layers[0].get_seq_length() == 40
    assert pre.wall_s > 0.0 and pre.event_s == 0.0  # a CPU model: no device events


def test_teacher_forced_logprobs_are_the_decode_rows_on_cpu() -> None:
    """teacher_forced_logprobs = prefill of the context, then one row per continuation position
    from single-token steps; rows are log-probabilities."""
    from transformers import LlamaConfig, LlamaForCausalLM

    from lazykv_b200.attention import IMPLEMENTATION_NAME, install
    from lazykv_b200.generate import teacher_forced_decode, teacher_forced_logprobs, prefill

    torch.manual_seed(1)
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                      vocab_size=96, max_position_embeddings=256)
    install()
    model = LlamaForCausalLM(copy.deepcopy(cfg)).eval()
    model.set_attn_implementation(IMPLEMENTATION_NAME)
    ctx, cont = torch.randint(0, cfg.vocab_size, (1, 20)), torch.randint(0, cfg.vocab_size, (1, 5))
    got = teacher_forced_logprobs(model, FullGPUCache(2, 64), ctx, cont, chunk_size=8)
    full = FullGPUCache(2, 64)
    pre = prefill(model, full, ctx, chunk_size=8)
    want = torch.stack(list(teacher_forced_decode(model, full, pre.last_logits, cont)))
    assert got.shape == (5, cfg.vocab_size) and got.device.type == "cpu"
    assert torch.equal(got, want)
    assert torch.allclose(got.exp().sum(-1), torch.ones(5), atol=1e-5)
