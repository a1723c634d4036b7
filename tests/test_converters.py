"""The reference-compatible converter entry points (``convert_to_wb``) with Megatron-style
``args`` and SGLang-style ``model_config`` objects."""
from types import SimpleNamespace

import torch

from weightbridge_b200.models.arch import ModelArch, get_arch
from weightbridge_b200.parallel.megatron import MegatronLayout, convert_to_wb as megatron_to_wb
from weightbridge_b200.parallel.sglang import SGLangLayout, convert_to_wb as sglang_to_wb, convert_to_wb_and_views


def test_megatron_convert_to_wb_with_args():
    arch = get_arch("tiny-qwen2")
    args = SimpleNamespace(hidden_size=arch.hidden, num_attention_heads=arch.num_heads,
                           num_query_groups=arch.num_kv_heads, kv_channels=arch.head_dim,
                           num_layers=arch.num_layers, ffn_hidden_size=arch.ffn, vocab_size=arch.vocab,
                           untie_embeddings_and_output_weights=True, make_vocab_size_divisible_by=128)
    lay = MegatronLayout(arch, tp=2, tp_rank=1)
    params = lay.allocate(dtype=torch.float32, fill=False)
    named = [("module.module." + n, torch.nn.Parameter(t)) for n, t in params.items()]
    meta, views = megatron_to_wb(args, "qwen2-0.5b", named, tp_rank=1, tp_size=2)
    ref_meta, _ = lay.to_wb(params)
    assert meta == ref_meta
    assert views["model.layers.0.self_attn.q_proj.bias"].data_ptr() == \
        params["decoder.layers.0.self_attention.linear_qkv.bias"].data_ptr()


def test_megatron_args_to_arch_roundtrip():
    arch = get_arch("tiny-qwen3-moe")
    args = SimpleNamespace(hidden_size=arch.hidden, num_attention_heads=arch.num_heads,
                           num_query_groups=arch.num_kv_heads, kv_channels=arch.head_dim, num_layers=arch.num_layers,
                           ffn_hidden_size=0, vocab_size=arch.vocab, num_experts=arch.num_experts,
                           moe_ffn_hidden_size=arch.moe_ffn, moe_router_topk=arch.top_k)
    a2 = ModelArch.from_megatron_args(args, family="qwen3_moe")
    assert a2.hf_tensors() == arch.hf_tensors()


def test_sglang_convert_to_wb_with_model_config():
    arch = get_arch("tiny-qwen3")
    hf = SimpleNamespace(model_type="qwen3", hidden_size=arch.hidden, num_attention_heads=arch.num_heads,
                         num_key_value_heads=arch.num_kv_heads, head_dim=arch.head_dim,
                         intermediate_size=arch.ffn, vocab_size=arch.vocab, num_hidden_layers=arch.num_layers)
    model_config = SimpleNamespace(hf_config=hf)
    lay = SGLangLayout(arch, tp=2, tp_rank=0, attn_tp=1, attn_tp_rank=0)
    params = lay.allocate(dtype=torch.bfloat16)
    meta = sglang_to_wb(model_config, params, tp_rank=0, tp_size=2, attn_tp_rank=0, attn_tp_size=1)
    ref_meta, _ = lay.to_wb(params)
    assert meta == ref_meta
    meta2, views = convert_to_wb_and_views(model_config, params, 0, 2, 0, 1)
    assert meta2 == ref_meta and "model.layers.1.self_attn.k_proj.weight" in views


def test_hf_config_dict_and_unknown_type():
    import pytest
    cfg = {"model_type": "llama", "hidden_size": 64, "num_attention_heads": 4, "num_key_value_heads": 2,
           "intermediate_size": 128, "vocab_size": 100, "num_hidden_layers": 1}
    a = ModelArch.from_hf_config(cfg)
    assert a.family == "llama" and a.head_dim == 16
    with pytest.raises(ValueError):
        ModelArch.from_hf_config(dict(cfg, model_type="mamba"))


def test_deepseek_configs_and_converters():
    """DeepSeek-V3 from a HF config dict and from Megatron MLA args, and the two entry points
    on its parameters (including SGLang's derived w_kc / w_vc, passed by name)."""
    arch = get_arch("tiny-deepseek-v3")
    hf = {"model_type": "deepseek_v3", "hidden_size": arch.hidden, "num_attention_heads": arch.num_heads,
          "num_key_value_heads": arch.num_heads, "num_hidden_layers": arch.num_layers, "vocab_size": arch.vocab,
          "intermediate_size": arch.ffn, "moe_intermediate_size": arch.moe_ffn, "n_routed_experts": arch.num_experts,
          "n_shared_experts": 1, "num_experts_per_tok": arch.top_k, "first_k_dense_replace": 1,
          "q_lora_rank": arch.q_lora_rank, "kv_lora_rank": arch.kv_lora_rank, "qk_nope_head_dim": arch.qk_nope_dim,
          "qk_rope_head_dim": arch.qk_rope_dim, "v_head_dim": arch.v_head_dim, "topk_method": "noaux_tc"}
    assert ModelArch.from_hf_config(hf, name=arch.name) == arch
    lite = get_arch("tiny-deepseek-v2-lite")
    hf2 = dict(hf, model_type="deepseek_v2", q_lora_rank=None, num_hidden_layers=2, moe_intermediate_size=128,
               n_routed_experts=4, n_shared_experts=2, intermediate_size=256, kv_lora_rank=128,
               qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128, topk_method="greedy")
    assert ModelArch.from_hf_config(hf2, name=lite.name) == lite
    args = SimpleNamespace(hidden_size=arch.hidden, num_attention_heads=arch.num_heads, num_layers=arch.num_layers,
                           ffn_hidden_size=arch.ffn, vocab_size=arch.vocab, num_experts=arch.num_experts,
                           moe_ffn_hidden_size=arch.moe_ffn, moe_router_topk=arch.top_k,
                           moe_shared_expert_intermediate_size=arch.shared_ffn, q_lora_rank=arch.q_lora_rank,
                           kv_lora_rank=arch.kv_lora_rank, qk_head_dim=arch.qk_nope_dim,
                           qk_pos_emb_head_dim=arch.qk_rope_dim, v_head_dim=arch.v_head_dim,
                           moe_layer_freq=[0, 1, 1], moe_router_enable_expert_bias=True)
    assert ModelArch.from_megatron_args(args, family="deepseek_v3", name=arch.name) == arch
    lay = MegatronLayout(arch, tp=2, tp_rank=1)
    params = lay.allocate(dtype=torch.float32, fill=False)
    meta, _v = megatron_to_wb(args, "deepseek-v3", list(params.items()), tp_rank=1, tp_size=2)
    assert meta == lay.to_wb(params)[0]
    slay = SGLangLayout(arch, tp=2, tp_rank=0)
    sparams = slay.allocate(dtype=torch.bfloat16)
    smeta = sglang_to_wb(SimpleNamespace(hf_config=SimpleNamespace(**hf)), sparams, tp_rank=0, tp_size=2)
    assert smeta == slay.to_wb(sparams)[0]
    assert len(smeta.shards("model.layers.2.self_attn.kv_b_proj.weight")) == 3


def test_glm4_moe_config():
    arch = get_arch("tiny-glm4-moe")
    hf = {"model_type": "glm4_moe", "hidden_size": arch.hidden, "num_attention_heads": arch.num_heads,
          "num_key_value_heads": arch.num_kv_heads, "head_dim": arch.head_dim, "num_hidden_layers": arch.num_layers,
          "vocab_size": arch.vocab, "intermediate_size": arch.ffn, "moe_intermediate_size": arch.moe_ffn,
          "n_routed_experts": arch.num_experts, "n_shared_experts": 1, "num_experts_per_tok": arch.top_k,
          "first_k_dense_replace": 1, "attention_bias": True, "use_qk_norm": False}
    assert ModelArch.from_hf_config(hf, name=arch.name) == arch
    names = {n for n, _s in arch.hf_tensors()}
    assert "model.layers.0.mlp.gate_proj.weight" in names and "model.layers.1.mlp.gate.e_score_correction_bias" in names
    assert "model.layers.1.mlp.shared_experts.up_proj.weight" in names and "model.layers.1.self_attn.k_proj.bias" in names
    import pytest
    with pytest.raises(ValueError, match="use_qk_norm"):
        ModelArch.from_hf_config(dict(hf, use_qk_norm=True))
