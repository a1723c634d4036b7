"""Megatron / SGLang layouts against an independent dense oracle, and host-side resharding.

Checks that (1) the synthetic fill through the strided views produces exactly the fused
parameters one builds by hand from the full HF tensors, and (2) packing the overlap of
every (Megatron rank, SGLang rank) pair and unpacking it reproduces the SGLang parameters
bit for bit, for each model family and several TP/PP/EP combinations.
"""
import pytest
import torch

from weightbridge_b200 import WeightData
from weightbridge_b200.core.binding import bind, pack_into, unpack_from
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.models.synthetic import synth_full
from weightbridge_b200.ops.quant_ref import block_quant_fp8_ref
from weightbridge_b200.parallel.megatron import MegatronLayout
from weightbridge_b200.parallel.sglang import SGLangLayout


def hf_full(arch, dtype=torch.float32):
    return {n: synth_full(n, s, dtype) for n, s in arch.hf_tensors()}


def megatron_oracle(arch, lay: MegatronLayout, hf):
    """Build this rank's Megatron params by hand from the full HF tensors."""
    tp, r = lay.tp, lay.tp_rank
    H, hd, qpg, G = arch.hidden, arch.head_dim, arch.q_per_group, arch.num_kv_heads
    out = {}
    Vp = lay.padded_vocab
    def vocab(t):
        pad = torch.zeros(Vp, H, dtype=t.dtype)
        pad[: arch.vocab] = t
        return pad.chunk(tp)[r]
    if lay.first_stage:
        out["embedding.word_embeddings.weight"] = vocab(hf["model.embed_tokens.weight"])
    G_loc = G // tp
    for i in range(lay.num_local_layers):
        g = i + lay.layer_offset
        p, m = f"decoder.layers.{i}.", f"model.layers.{g}."
        if arch.is_mla:                  # head-contiguous up projections: plain row chunks per TP rank
            a = p + "self_attention."
            out[p + "input_layernorm.weight"] = hf[m + "input_layernorm.weight"]
            if arch.q_lora_rank:
                out[a + "linear_q_down_proj.weight"] = hf[m + "self_attn.q_a_proj.weight"]
                out[a + "linear_q_up_proj.layer_norm_weight"] = hf[m + "self_attn.q_a_layernorm.weight"]
                out[a + "linear_q_up_proj.weight"] = hf[m + "self_attn.q_b_proj.weight"].chunk(tp)[r]
            else:
                out[a + "linear_q_proj.weight"] = hf[m + "self_attn.q_proj.weight"].chunk(tp)[r]
            out[a + "linear_kv_down_proj.weight"] = hf[m + "self_attn.kv_a_proj_with_mqa.weight"]
            out[a + "linear_kv_up_proj.layer_norm_weight"] = hf[m + "self_attn.kv_a_layernorm.weight"]
            out[a + "linear_kv_up_proj.weight"] = hf[m + "self_attn.kv_b_proj.weight"].chunk(tp)[r]
            out[a + "linear_proj.weight"] = hf[m + "self_attn.o_proj.weight"].chunk(tp, 1)[r]
        else:
            q = hf[m + "self_attn.q_proj.weight"].view(G, qpg * hd, H)
            k = hf[m + "self_attn.k_proj.weight"].view(G, hd, H)
            v = hf[m + "self_attn.v_proj.weight"].view(G, hd, H)
            out[p + "self_attention.linear_qkv.weight"] = torch.cat([q, k, v], 1)[r * G_loc:(r + 1) * G_loc].reshape(-1, H)
            if arch.qkv_bias:
                qb = hf[m + "self_attn.q_proj.bias"].view(G, qpg * hd)
                kb = hf[m + "self_attn.k_proj.bias"].view(G, hd)
                vb = hf[m + "self_attn.v_proj.bias"].view(G, hd)
                out[p + "self_attention.linear_qkv.bias"] = torch.cat([qb, kb, vb], 1)[r * G_loc:(r + 1) * G_loc].reshape(-1)
            out[p + "self_attention.linear_qkv.layer_norm_weight"] = hf[m + "input_layernorm.weight"]
            if arch.qk_norm:
                out[p + "self_attention.q_layernorm.weight"] = hf[m + "self_attn.q_norm.weight"]
                out[p + "self_attention.k_layernorm.weight"] = hf[m + "self_attn.k_norm.weight"]
            out[p + "self_attention.linear_proj.weight"] = hf[m + "self_attn.o_proj.weight"].chunk(tp, 1)[r]
        if arch.moe_layer(g):
            out[p + "pre_mlp_layernorm.weight"] = hf[m + "post_attention_layernorm.weight"]
            mb, (gn, un, dn) = arch.moe_block, arch.expert_projs
            out[p + "mlp.router.weight"] = hf[m + f"{mb}.gate.weight"]
            if arch.router_bias:
                out[p + "mlp.router.expert_bias"] = hf[m + f"{mb}.gate.e_score_correction_bias"]
            E_loc = arch.num_experts // lay.ep
            for e in range(E_loc):
                eg = lay.ep_rank * E_loc + e
                x = f"{m}{mb}.experts.{eg}."
                gate = hf[x + f"{gn}.weight"].chunk(lay.etp, 0)[lay.etp_rank]
                up = hf[x + f"{un}.weight"].chunk(lay.etp, 0)[lay.etp_rank]
                out[lay._expert_name(i, e, 1)] = torch.cat([gate, up])
                out[lay._expert_name(i, e, 2)] = hf[x + f"{dn}.weight"].chunk(lay.etp, 1)[lay.etp_rank]
            if arch.shared_ffn:
                y = m + ("mlp.shared_expert." if arch.family == "qwen2_moe" else "mlp.shared_experts.")
                out[p + "mlp.shared_experts.linear_fc1.weight"] = torch.cat(
                    [hf[y + "gate_proj.weight"].chunk(tp)[r], hf[y + "up_proj.weight"].chunk(tp)[r]])
                out[p + "mlp.shared_experts.linear_fc2.weight"] = hf[y + "down_proj.weight"].chunk(tp, 1)[r]
                if arch.family == "qwen2_moe":
                    out[p + "mlp.shared_experts.gate_weight"] = hf[m + "mlp.shared_expert_gate.weight"]
        else:
            out[p + "mlp.linear_fc1.layer_norm_weight"] = hf[m + "post_attention_layernorm.weight"]
            out[p + "mlp.linear_fc1.weight"] = torch.cat([hf[m + "mlp.gate_proj.weight"].chunk(tp)[r],
                                                          hf[m + "mlp.up_proj.weight"].chunk(tp)[r]])
            out[p + "mlp.linear_fc2.weight"] = hf[m + "mlp.down_proj.weight"].chunk(tp, 1)[r]
    if lay.last_stage:
        out["decoder.final_layernorm.weight"] = hf["model.norm.weight"]
        if not arch.tie_embeddings:
            out["output_layer.weight"] = vocab(hf["lm_head.weight"])
    return out


MEGATRON_CASES = [
    ("tiny-llama", dict(tp=2)),
    ("tiny-llama", dict(tp=1, pp=2)),
    ("tiny-qwen2", dict(tp=2)),
    ("tiny-qwen3", dict(tp=2, pp=2)),
    ("tiny-qwen3-moe", dict(tp=1, ep=2)),
    ("tiny-qwen3-moe", dict(tp=2, ep=2, etp=2, expert_naming="sequential")),
    ("tiny-mixtral", dict(tp=2, ep=2)),
    ("tiny-qwen2-moe", dict(tp=2, ep=2)),
    ("tiny-deepseek-v3", dict(tp=2, ep=2)),
    ("tiny-deepseek-v2-lite", dict(tp=2, pp=2)),
    ("tiny-glm4-moe", dict(tp=2, ep=2)),
]


@pytest.mark.parametrize("model,cfg", MEGATRON_CASES)
def test_megatron_fill_matches_oracle(model, cfg):
    arch = get_arch(model)
    hf = hf_full(arch)
    ranks = [dict(tp_rank=t, pp_rank=p, ep_rank=e)
             for t in range(cfg.get("tp", 1)) for p in range(cfg.get("pp", 1)) for e in range(cfg.get("ep", 1))]
    for rk in ranks:
        kw = dict(cfg, **rk)
        if cfg.get("etp", 1) > 1:
            kw["etp_rank"] = rk["tp_rank"]
        lay = MegatronLayout(arch, **kw)
        params = lay.allocate(dtype=torch.float32)
        oracle = megatron_oracle(arch, lay, hf)
        assert set(params) == set(oracle)
        for n in params:
            assert torch.equal(params[n], oracle[n]), n


def test_megatron_unknown_name_raises():
    lay = MegatronLayout(get_arch("tiny-llama"))
    with pytest.raises(ValueError):
        lay.split_param("decoder.layers.0.mystery.weight", torch.zeros(4))


def test_megatron_module_prefix_and_pp_offset():
    arch = get_arch("tiny-llama")
    lay = MegatronLayout(arch, pp=2, pp_rank=1)
    params = lay.allocate(dtype=torch.float32, fill=False)
    prefixed = {"module.module." + k: v for k, v in params.items()}
    meta, _ = lay.to_wb(prefixed)
    assert "model.layers.1.self_attn.q_proj.weight" in meta
    assert "model.layers.0.self_attn.q_proj.weight" not in meta
    assert "lm_head.weight" in meta and "model.embed_tokens.weight" not in meta


def sglang_oracle(arch, lay: SGLangLayout, hf):
    H, hd = arch.hidden, arch.head_dim
    r, tp = lay.tp_rank, lay.tp
    out = {}
    Vp = lay.padded_vocab
    def vocab(t):
        pad = torch.zeros(Vp, H, dtype=t.dtype)
        pad[: arch.vocab] = t
        return pad.chunk(tp)[r]
    out["model.embed_tokens.weight"] = vocab(hf["model.embed_tokens.weight"])
    ar, atp = lay.attn_tp_rank, lay.attn_tp
    kv0 = lay.kv_head0
    for i in range(arch.num_layers):
        m = f"model.layers.{i}."
        if arch.is_mla:
            a = m + "self_attn."
            if arch.q_lora_rank:
                out[a + "fused_qkv_a_proj_with_mqa.weight"] = torch.cat([hf[a + "q_a_proj.weight"],
                                                                         hf[a + "kv_a_proj_with_mqa.weight"]])
                out[a + "q_a_layernorm.weight"] = hf[a + "q_a_layernorm.weight"]
                out[a + "q_b_proj.weight"] = hf[a + "q_b_proj.weight"].chunk(atp)[ar]
            else:
                out[a + "q_proj.weight"] = hf[a + "q_proj.weight"].chunk(atp)[ar]
                out[a + "kv_a_proj_with_mqa.weight"] = hf[a + "kv_a_proj_with_mqa.weight"]
            out[a + "kv_a_layernorm.weight"] = hf[a + "kv_a_layernorm.weight"]
            kvb = hf[a + "kv_b_proj.weight"].chunk(atp)[ar]
            out[a + "kv_b_proj.weight"] = kvb
            # what SGLang derives after loading (absorbed MLA): per head, k_nope rows and v rows
            w = kvb.view(arch.num_heads // atp, arch.qk_nope_dim + arch.v_head_dim, arch.kv_lora_rank)
            out[a + "w_kc"] = w[:, :arch.qk_nope_dim]
            out[a + "w_vc"] = w[:, arch.qk_nope_dim:].transpose(1, 2)
            out[a + "o_proj.weight"] = hf[a + "o_proj.weight"].chunk(atp, 1)[ar]
        else:
            q = hf[m + "self_attn.q_proj.weight"].chunk(atp)[ar]
            k = hf[m + "self_attn.k_proj.weight"][kv0 * hd:(kv0 + lay.kv_local) * hd]
            v = hf[m + "self_attn.v_proj.weight"][kv0 * hd:(kv0 + lay.kv_local) * hd]
            out[m + "self_attn.qkv_proj.weight"] = torch.cat([q, k, v])
            if arch.qkv_bias:
                out[m + "self_attn.qkv_proj.bias"] = torch.cat([
                    hf[m + "self_attn.q_proj.bias"].chunk(atp)[ar],
                    hf[m + "self_attn.k_proj.bias"][kv0 * hd:(kv0 + lay.kv_local) * hd],
                    hf[m + "self_attn.v_proj.bias"][kv0 * hd:(kv0 + lay.kv_local) * hd]])
            out[m + "self_attn.o_proj.weight"] = hf[m + "self_attn.o_proj.weight"].chunk(atp, 1)[ar]
        for n in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            out[m + n] = hf[m + n]
        if arch.qk_norm:
            out[m + "self_attn.q_norm.weight"] = hf[m + "self_attn.q_norm.weight"]
            out[m + "self_attn.k_norm.weight"] = hf[m + "self_attn.k_norm.weight"]
        if arch.moe_layer(i):
            mb, (gn, un, dn) = arch.moe_block, arch.expert_projs
            out[m + f"{mb}.gate.weight"] = hf[m + f"{mb}.gate.weight"]
            if arch.router_bias:
                out[m + f"{mb}.gate.e_score_correction_bias"] = hf[m + f"{mb}.gate.e_score_correction_bias"]
            E_loc = arch.num_experts // lay.moe_ep
            w13, w2 = [], []
            for e in range(E_loc):
                eg = lay.moe_ep_rank * E_loc + e
                x = f"{m}{mb}.experts.{eg}."
                t = lay.moe_tp_rank
                w13.append(torch.cat([hf[x + f"{gn}.weight"].chunk(lay.moe_tp)[t],
                                      hf[x + f"{un}.weight"].chunk(lay.moe_tp)[t]]))
                w2.append(hf[x + f"{dn}.weight"].chunk(lay.moe_tp, 1)[t])
            out[m + f"{mb}.experts.w13_weight"] = torch.stack(w13)
            out[m + f"{mb}.experts.w2_weight"] = torch.stack(w2)
            if arch.shared_ffn:
                y = m + ("mlp.shared_expert." if arch.family == "qwen2_moe" else "mlp.shared_experts.")
                out[y + "gate_up_proj.weight"] = torch.cat([hf[y + "gate_proj.weight"].chunk(tp)[r],
                                                            hf[y + "up_proj.weight"].chunk(tp)[r]])
                out[y + "down_proj.weight"] = hf[y + "down_proj.weight"].chunk(tp, 1)[r]
                if arch.family == "qwen2_moe":
                    out[m + "mlp.shared_expert_gate.weight"] = hf[m + "mlp.shared_expert_gate.weight"]
        else:
            out[m + "mlp.gate_up_proj.weight"] = torch.cat([hf[m + "mlp.gate_proj.weight"].chunk(tp)[r],
                                                            hf[m + "mlp.up_proj.weight"].chunk(tp)[r]])
            out[m + "mlp.down_proj.weight"] = hf[m + "mlp.down_proj.weight"].chunk(tp, 1)[r]
    out["model.norm.weight"] = hf["model.norm.weight"]
    if not arch.tie_embeddings:
        out["lm_head.weight"] = vocab(hf["lm_head.weight"])
    return out


SGLANG_CASES = [
    ("tiny-llama", dict(tp=2)),
    ("tiny-llama", dict(tp=4)),                 # 2 KV heads on 4 ranks: replication
    ("tiny-qwen2", dict(tp=2)),
    ("tiny-qwen3", dict(tp=2, attn_tp=1)),      # DP-attention style: attention unsharded
    ("tiny-qwen3-moe", dict(tp=2)),
    ("tiny-qwen3-moe", dict(tp=2, moe_ep=2)),
    ("tiny-mixtral", dict(tp=2, moe_ep=2)),
    ("tiny-qwen2-moe", dict(tp=2, moe_ep=2)),
    ("tiny-deepseek-v3", dict(tp=2, moe_ep=2)),
    ("tiny-deepseek-v3", dict(tp=4, attn_tp=1, moe_ep=4)),   # DP-attention: MLA unsharded
    ("tiny-deepseek-v2-lite", dict(tp=2)),
    ("tiny-glm4-moe", dict(tp=2, moe_ep=2)),
]


@pytest.mark.parametrize("model,cfg", SGLANG_CASES)
def test_sglang_fill_matches_oracle(model, cfg):
    arch = get_arch(model)
    hf = hf_full(arch)
    for r in range(cfg["tp"]):
        kw = dict(cfg, tp_rank=r)
        if "attn_tp" in kw:
            kw["attn_tp_rank"] = r % kw["attn_tp"]
        lay = SGLangLayout(arch, **kw)
        params = lay.allocate(dtype=torch.float32, fill=True)
        oracle = sglang_oracle(arch, lay, hf)
        assert set(params) == set(oracle)
        for n in params:
            assert torch.equal(params[n], oracle[n]), n


def _host_sync(meg_layouts, sgl_layouts, dtype):
    senders = []
    for lay in meg_layouts:
        params = lay.allocate(dtype=dtype)
        meta, views = lay.to_wb(params)
        senders.append((meta, bind(meta, views)))
    results = []
    for lay in sgl_layouts:
        params = lay.allocate(dtype=dtype)
        meta, views = lay.to_wb(params)
        rb = bind(meta, views)
        done = set()
        for smeta, sb in senders:
            ov = WeightData.compute_overlap(smeta, meta)
            if not ov:
                continue
            buf = torch.empty(ov.total_nbytes(), dtype=torch.uint8)
            pack_into(sb, ov, buf)
            unpack_from(rb, ov, buf)
            done |= set(ov.names())
        expected = lay.allocate(dtype=dtype, fill=True)
        results.append((params, expected, done, meta))
    return results


SYNC_CASES = [
    ("tiny-llama", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)], [dict(tp=1)]),
    ("tiny-llama", [dict(tp=1, pp=2, pp_rank=0), dict(tp=1, pp=2, pp_rank=1)], [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)]),
    ("tiny-llama", [dict(tp=2, tp_rank=0), dict(tp=2, tp_rank=1)], [dict(tp=4, tp_rank=i) for i in range(4)]),
    ("tiny-qwen2", [dict(tp=2, tp_rank=i) for i in range(2)], [dict(tp=1)]),
    ("tiny-qwen3", [dict(tp=1)], [dict(tp=2, tp_rank=i, attn_tp=1, attn_tp_rank=0) for i in range(2)]),
    ("tiny-qwen3-moe", [dict(ep=2, ep_rank=i) for i in range(2)], [dict(tp=2, tp_rank=i) for i in range(2)]),
    ("tiny-qwen3-moe", [dict(ep=2, ep_rank=i) for i in range(2)], [dict(tp=2, tp_rank=i, moe_ep=2) for i in range(2)]),
    ("tiny-mixtral", [dict(ep=2, ep_rank=i) for i in range(2)], [dict(tp=2, tp_rank=i, moe_ep=2) for i in range(2)]),
    ("tiny-qwen2-moe", [dict(tp=2, ep=2, tp_rank=i % 2, ep_rank=i // 2) for i in range(4)],
     [dict(tp=2, tp_rank=i, moe_ep=2) for i in range(2)]),
    ("tiny-deepseek-v3", [dict(tp=2, ep=2, tp_rank=i % 2, ep_rank=i // 2) for i in range(4)],
     [dict(tp=2, tp_rank=i, moe_ep=2) for i in range(2)]),
    ("tiny-deepseek-v3", [dict(tp=4, ep=2, etp=2, tp_rank=i, ep_rank=i // 2, etp_rank=i % 2) for i in range(4)],
     [dict(tp=4, tp_rank=i, attn_tp=1, attn_tp_rank=0, moe_ep=2) for i in range(4)]),
    ("tiny-deepseek-v2-lite", [dict(tp=1, pp=2, pp_rank=i) for i in range(2)],
     [dict(tp=4, tp_rank=i) for i in range(4)]),
    ("tiny-glm4-moe", [dict(tp=2, ep=2, tp_rank=i % 2, ep_rank=i // 2) for i in range(4)],
     [dict(tp=2, tp_rank=i, moe_ep=2) for i in range(2)]),
]


@pytest.mark.parametrize("model,meg,sgl", SYNC_CASES)
def test_host_reshard_is_bitwise(model, meg, sgl):
    arch = get_arch(model)
    res = _host_sync([MegatronLayout(arch, **m) for m in meg], [SGLangLayout(arch, **s) for s in sgl],
                     torch.float32)
    for params, expected, done, meta in res:
        assert done == set(meta.names())
        for n in params:
            assert torch.equal(params[n], expected[n]), n


def test_sglang_fp8_expert_layout():
    arch = get_arch("tiny-qwen3-moe")
    lay = SGLangLayout(arch, tp=2, tp_rank=1, moe_ep=2, quant="fp8_experts")
    params = lay.allocate(dtype=torch.bfloat16, fill=True)
    assert params["model.layers.0.mlp.experts.w13_weight"].dtype == torch.float8_e4m3fn
    s = params["model.layers.0.mlp.experts.w13_weight_scale_inv"]
    assert s.dtype == torch.float32 and tuple(s.shape) == (4, 4, 2)
    meta, views = lay.to_wb(params)
    name = "model.layers.0.mlp.experts.5.up_proj.weight"
    q = meta.quant(name)
    assert q["scale"] == name + "_scale_inv" and q["block"] == [128, 128]
    full = synth_full(name, (256, 256), torch.bfloat16)
    qv, sv = block_quant_fp8_ref(full)
    assert torch.equal(views[name].view(torch.uint8), qv.view(torch.uint8))
    assert torch.equal(views[name + "_scale_inv"], sv)


def test_host_reshard_fp8_experts():
    """bf16 Megatron EP2 -> SGLang TP2 (EP2) with fp8 experts: sender-side block quant."""
    arch = get_arch("tiny-qwen3-moe")
    meg = [MegatronLayout(arch, ep=2, ep_rank=i) for i in range(2)]
    sgl = [SGLangLayout(arch, tp=2, tp_rank=i, moe_ep=2, quant="fp8_experts") for i in range(2)]
    for params, expected, done, meta in _host_sync(meg, sgl, torch.bfloat16):
        assert done == set(meta.names())
        for n in params:
            assert torch.equal(params[n].view(torch.uint8) if params[n].dtype == torch.float8_e4m3fn else params[n],
                               expected[n].view(torch.uint8) if expected[n].dtype == torch.float8_e4m3fn else expected[n]), n


def test_sglang_fp8_qkv_rejects_a_kv_part_inside_a_block():
    """Scales of the fused qkv_proj are per 128-row block of the fused tensor; a k/v part that
    starts inside a block would share its scale with q, which per-entry scales cannot express."""
    import dataclasses
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.sglang import SGLangLayout
    arch = dataclasses.replace(get_arch("tiny-llama"), num_heads=3, num_kv_heads=1, head_dim=64, ffn=512)
    lay = SGLangLayout(arch, tp=1, quant="fp8_linear")
    with pytest.raises(ValueError, match="inside an fp8 block"):
        lay.to_wb(lay.allocate(dtype=torch.bfloat16, fill=False))


def test_megatron_virtual_pipeline_chunks_cover_the_model_once():
    """PP 2 x VPP 2 (interleaved schedule): chunk v of stage p holds the (v * 2 + p)-th quarter
    of the layers; all chunks of all stages resharded into one SGLang rank give the model."""
    from weightbridge_b200.core.plan import lower_ops, phys_binding, plan_pair
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.ops.executor import cpu_execute
    from weightbridge_b200.parallel.megatron import MegatronLayout
    from weightbridge_b200.parallel.sglang import SGLangLayout
    arch = get_arch("tiny-llama").with_(num_layers=4)
    seen = []
    rl = SGLangLayout(arch, tp=1)
    rp = rl.allocate(dtype=torch.float32)
    rmeta, rviews = rl.to_wb(rp)
    rphys = phys_binding(bind(rmeta, rviews))
    keep = []
    for pp_rank in range(2):
        for lay in MegatronLayout(arch, pp=2, pp_rank=pp_rank, vpp=2).chunks():
            p = lay.allocate(dtype=torch.float32)
            keep.append(p)
            meta, views = lay.to_wb(p)
            seen += meta.names()
            cpu_execute(lower_ops(plan_pair(phys_binding(bind(meta, views)), rphys), lambda a: 0, lambda a: 0))
    assert len(seen) == len(set(seen)) == len(arch.hf_tensors())
    layers = {pp: MegatronLayout(arch, pp=2, pp_rank=pp, vpp=2).chunks() for pp in range(2)}
    assert [c.layer_offset for c in layers[0]] == [0, 2] and [c.layer_offset for c in layers[1]] == [1, 3]
    exp = rl.allocate(dtype=torch.float32, fill=True)
    assert all(torch.equal(rp[n], exp[n]) for n in exp)


def test_megatron_to_wb_strict_and_lenient():
    from weightbridge_b200.models.arch import get_arch
    from weightbridge_b200.parallel.megatron import MegatronLayout, UnknownParameter
    lay = MegatronLayout(get_arch("tiny-llama"))
    params = lay.allocate(dtype=torch.float32, fill=False)
    params["decoder.layers.0.self_attention.linear_qkv.lora_A.weight"] = torch.zeros(8, 256)
    with pytest.raises(UnknownParameter):
        lay.to_wb(params)
    meta, views = lay.to_wb(params, strict=False)
    assert len(meta.names()) == len(get_arch("tiny-llama").hf_tensors())


def test_sglang_mla_derived_tensors_are_strided_destinations():
    """w_kc / w_vc keep SGLang's transposed storage and are extra destination shards of
    kv_b_proj (its k_nope rows and its v rows of each local head)."""
    arch = get_arch("tiny-deepseek-v3")
    lay = SGLangLayout(arch, tp=2, tp_rank=1)
    params = lay.allocate(dtype=torch.bfloat16)
    a = "model.layers.0.self_attn."
    kc, vc = params[a + "w_kc"], params[a + "w_vc"]
    assert tuple(kc.shape) == (2, 32, 128) and kc.stride() == (128 * 32, 1, 32)
    assert tuple(vc.shape) == (2, 128, 32) and vc.stride() == (32 * 128, 1, 128)
    meta, views = lay.to_wb(params)
    assert meta.shards(a + "kv_b_proj.weight") == [[(128, 256, 256), (0, 128, 128)],
                                                   [(2, 4, 4), (0, 32, 64), (0, 128, 128)],
                                                   [(2, 4, 4), (32, 64, 64), (0, 128, 128)]]
    assert views[a + "kv_b_proj.weight"][1].data_ptr() == kc.data_ptr()
    with pytest.raises(ValueError, match="fp8_linear"):
        SGLangLayout(arch, tp=1, quant="fp8_linear")


def test_host_reshard_deepseek_fp8_experts():
    """bf16 Megatron TP2 x EP2 -> SGLang TP2 (EP2) DeepSeek-style: fp8 routed experts, bf16
    MLA with the derived w_kc / w_vc, dense first layer, shared experts, router bias."""
    arch = get_arch("tiny-deepseek-v3")
    meg = [MegatronLayout(arch, tp=2, ep=2, tp_rank=i % 2, ep_rank=i // 2) for i in range(4)]
    sgl = [SGLangLayout(arch, tp=2, tp_rank=i, moe_ep=2, quant="fp8_experts") for i in range(2)]
    for params, expected, done, meta in _host_sync(meg, sgl, torch.bfloat16):
        assert done == set(meta.names())
        for n in params:
            assert torch.equal(params[n].view(torch.uint8) if params[n].dtype == torch.float8_e4m3fn else params[n],
                               expected[n].view(torch.uint8) if expected[n].dtype == torch.float8_e4m3fn else expected[n]), n


def test_sglang_fused_shared_expert_slot_and_slot_count_guard():
    """A worker that keeps DeepSeek's shared expert as one more slot of w13 / w2 (expert_slots
    value -1) receives it there from the trainer's shared_experts; a FusedMoE tensor whose
    slot count the layout does not expect is an error, not a slot left stale."""
    arch = get_arch("tiny-deepseek-v3")
    sl = lambda r: [[]] + [[4 * r + e for e in range(4)] + [-1]] * (arch.num_layers - 1)   # noqa: E731
    meg = [MegatronLayout(arch, tp=2, ep=2, tp_rank=i % 2, ep_rank=i // 2) for i in range(4)]
    sgl = [SGLangLayout(arch, tp=2, tp_rank=r, moe_ep=2, expert_slots=sl(r)) for r in range(2)]
    assert "model.layers.1.mlp.shared_experts.gate_up_proj.weight" not in sgl[0].param_specs()
    assert sgl[0].param_specs()["model.layers.1.mlp.experts.w13_weight"][0][0] == 5
    for params, expected, done, meta in _host_sync(meg, sgl, torch.bfloat16):
        assert done == set(meta.names())
        assert "model.layers.1.mlp.shared_experts.down_proj.weight" in meta
        for n in params:
            a, b = params[n], expected[n]
            if a.dtype == torch.float8_e4m3fn:
                a, b = a.view(torch.uint8), b.view(torch.uint8)
            assert torch.equal(a, b), n
    plain = SGLangLayout(arch, tp=2, tp_rank=0, moe_ep=2)
    fused = sgl[0].allocate(dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="expert slots"):
        plain.to_wb({n: t for n, t in fused.items() if not n.endswith("_scale_inv")})
    with pytest.raises(ValueError, match="shared expert"):
        SGLangLayout(get_arch("tiny-qwen2-moe"), tp=1, expert_slots=[[0, 1, 2, 3, -1]] * 2)


def test_megatron_expert_index_beyond_local_count_is_an_error():
    lay = MegatronLayout(get_arch("tiny-qwen3-moe"), ep=2, ep_rank=1)
    with pytest.raises(ValueError, match="local expert 4 of 4"):
        lay.split_param("decoder.layers.0.mlp.experts.linear_fc2.weight4", torch.zeros(256, 256))


def test_overlap_carries_elements_shared_by_overlapping_shards_once():
    """Receiver shards that overlap (MLA's w_kc / w_vc inside kv_b_proj, a redundant expert
    slot) do not multiply the overlap: it holds each element once, the receiver writes it into
    every shard, and coverage still counts every destination shard as filled."""
    from weightbridge_b200.core.shard import covered_numel, shard_numel
    arch = get_arch("tiny-deepseek-v3")
    smeta, _ = MegatronLayout(arch, tp=1).to_wb(MegatronLayout(arch, tp=1).allocate(fill=False))
    rl = SGLangLayout(arch, tp=1, expert_slots=[[]] + [[0, 1, 2, 3, 4, 5, 6, 7, 3]] * 2)
    rmeta, _ = rl.to_wb(rl.allocate(dtype=torch.bfloat16))
    ov = WeightData.compute_overlap(smeta, rmeta)
    kvb = "model.layers.0.self_attn.kv_b_proj.weight"
    assert len(rmeta.shards(kvb)) == 3 and ov.shards(kvb) == [[(0, 256, 256), (0, 128, 128)]]
    e3 = "model.layers.1.mlp.experts.3.up_proj.weight"
    assert len(rmeta.shards(e3)) == 2 and len(ov.shards(e3)) == 1
    for n in (kvb, e3):
        full = sum(shard_numel(s) for s in rmeta.shards(n))
        assert sum(covered_numel(reg, rmeta.shards(n)) for reg in ov.shards(n)) == full
