"""Architecture descriptors and the HF-named logical tensors of each model family.

Families: ``llama`` (Llama-2/3), ``qwen2`` (q/k/v bias), ``qwen3`` (q/k RMSNorm),
``qwen3_moe`` (Qwen3 attention + a routed-expert MLP in every layer), ``qwen2_moe`` (Qwen2
attention + routed experts + a gated shared expert), ``mixtral`` (Llama attention +
``block_sparse_moe`` experts named ``w1`` / ``w3`` / ``w2``) and ``deepseek_v3`` (multi-head
latent attention: low-rank q and kv projections, per-head ``[nope | rope]`` queries and
``[k_nope | v]`` keys/values; dense MLPs in the first layers, then routed experts with
ungated shared experts and a router score-correction bias) and ``glm4_moe`` (GLM-4.5: GQA
attention with q/k/v bias and the same MoE layout as ``deepseek_v3``).  The reference
covers Qwen2/Qwen3 dense only (``wbridge/utils/megatron_utils/qwen2.py:13-80``,
``wbridge/utils/sglang_utils/qwen2.py:24-119``); Llama, the MoE families and MLA are new here.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any, Iterator


@dataclass(frozen=True)
class ModelArch:
    name: str
    family: str                   # llama | qwen2 | qwen3 | qwen3_moe | qwen2_moe | mixtral | deepseek_v3 | glm4_moe
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    ffn: int                      # dense MLP width (0 for an all-MoE model)
    vocab: int
    tie_embeddings: bool = False
    num_experts: int = 0
    moe_ffn: int = 0              # per-expert intermediate width
    top_k: int = 0
    shared_ffn: int = 0           # shared experts' intermediate width (qwen2_moe, deepseek_v3), 0: none
    # multi-head latent attention (deepseek_v3); head_dim is the query head size nope + rope
    q_lora_rank: int = 0          # 0: a plain q_proj instead of q_a_proj / q_b_proj
    kv_lora_rank: int = 0
    qk_nope_dim: int = 0
    qk_rope_dim: int = 0
    v_head_dim: int = 0
    first_dense_layers: int = 0   # leading layers with a dense MLP in a MoE model
    router_bias: bool = False     # routers with a score-correction bias (e_score_correction_bias)

    @property
    def qkv_bias(self) -> bool:
        return self.family in ("qwen2", "qwen2_moe", "glm4_moe")

    @property
    def qk_norm(self) -> bool:
        return self.family in ("qwen3", "qwen3_moe")

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def is_mla(self) -> bool:
        return self.family == "deepseek_v3"

    def moe_layer(self, i: int) -> bool:
        """Whether layer ``i`` has routed experts (else a dense MLP of width ``ffn``)."""
        return self.is_moe and i >= self.first_dense_layers

    @property
    def shared_prefix(self) -> str:
        """HF module of the shared experts: one gated expert (qwen2_moe) or ungated ones."""
        return "mlp.shared_expert." if self.shared_gate else "mlp.shared_experts."

    @property
    def shared_gate(self) -> bool:
        """Whether the shared expert's output is gated (``mlp.shared_expert_gate``)."""
        return self.family == "qwen2_moe"

    @property
    def moe_block(self) -> str:
        """HF module holding the router and the experts of a MoE layer."""
        return "block_sparse_moe" if self.family == "mixtral" else "mlp"

    @property
    def expert_projs(self) -> tuple[str, str, str]:
        """HF names of an expert's gate, up and down projections."""
        return ("w1", "w3", "w2") if self.family == "mixtral" else ("gate_proj", "up_proj", "down_proj")

    @property
    def q_per_group(self) -> int:
        return self.num_heads // self.num_kv_heads

    def with_(self, **kw) -> "ModelArch":
        return replace(self, **kw)

    # ---------------------------------------------------------------------------------
    def mla_tensors(self, p: str) -> Iterator[tuple[str, tuple[int, ...]]]:
        """The attention tensors of one MLA layer (prefix ``p``)."""
        H, nh, qk = self.hidden, self.num_heads, self.head_dim
        if self.q_lora_rank:
            yield p + "self_attn.q_a_proj.weight", (self.q_lora_rank, H)
            yield p + "self_attn.q_a_layernorm.weight", (self.q_lora_rank,)
            yield p + "self_attn.q_b_proj.weight", (nh * qk, self.q_lora_rank)
        else:
            yield p + "self_attn.q_proj.weight", (nh * qk, H)
        yield p + "self_attn.kv_a_proj_with_mqa.weight", (self.kv_lora_rank + self.qk_rope_dim, H)
        yield p + "self_attn.kv_a_layernorm.weight", (self.kv_lora_rank,)
        yield p + "self_attn.kv_b_proj.weight", (nh * (self.qk_nope_dim + self.v_head_dim), self.kv_lora_rank)
        yield p + "self_attn.o_proj.weight", (H, nh * self.v_head_dim)

    def layer_tensors(self, i: int) -> Iterator[tuple[str, tuple[int, ...]]]:
        H, hd = self.hidden, self.head_dim
        p = f"model.layers.{i}."
        yield p + "input_layernorm.weight", (H,)
        if self.is_mla:
            yield from self.mla_tensors(p)
        else:
            yield p + "self_attn.q_proj.weight", (self.num_heads * hd, H)
            yield p + "self_attn.k_proj.weight", (self.num_kv_heads * hd, H)
            yield p + "self_attn.v_proj.weight", (self.num_kv_heads * hd, H)
            if self.qkv_bias:
                yield p + "self_attn.q_proj.bias", (self.num_heads * hd,)
                yield p + "self_attn.k_proj.bias", (self.num_kv_heads * hd,)
                yield p + "self_attn.v_proj.bias", (self.num_kv_heads * hd,)
            if self.qk_norm:
                yield p + "self_attn.q_norm.weight", (hd,)
                yield p + "self_attn.k_norm.weight", (hd,)
            yield p + "self_attn.o_proj.weight", (H, self.num_heads * hd)
        yield p + "post_attention_layernorm.weight", (H,)
        if self.moe_layer(i):
            I, mb = self.moe_ffn, self.moe_block
            g, u, d = self.expert_projs
            yield p + f"{mb}.gate.weight", (self.num_experts, H)
            if self.router_bias:
                yield p + f"{mb}.gate.e_score_correction_bias", (self.num_experts,)
            for e in range(self.num_experts):
                q = f"{p}{mb}.experts.{e}."
                yield q + f"{g}.weight", (I, H)
                yield q + f"{u}.weight", (I, H)
                yield q + f"{d}.weight", (H, I)
            if self.shared_ffn:
                S, sp = self.shared_ffn, p + self.shared_prefix
                yield sp + "gate_proj.weight", (S, H)
                yield sp + "up_proj.weight", (S, H)
                yield sp + "down_proj.weight", (H, S)
                if self.shared_gate:
                    yield p + "mlp.shared_expert_gate.weight", (1, H)
        else:
            yield p + "mlp.gate_proj.weight", (self.ffn, H)
            yield p + "mlp.up_proj.weight", (self.ffn, H)
            yield p + "mlp.down_proj.weight", (H, self.ffn)

    def hf_tensors(self) -> list[tuple[str, tuple[int, ...]]]:
        """Every logical HF tensor (name, shape), in model order."""
        out = [("model.embed_tokens.weight", (self.vocab, self.hidden))]
        for i in range(self.num_layers):
            out.extend(self.layer_tensors(i))
        out.append(("model.norm.weight", (self.hidden,)))
        if not self.tie_embeddings:
            out.append(("lm_head.weight", (self.vocab, self.hidden)))
        return out

    def num_params(self) -> int:
        n = 0
        for _, shape in self.hf_tensors():
            k = 1
            for d in shape:
                k *= d
            n += k
        return n

    # ---------------------------------------------------------------------------------
    @staticmethod
    def from_hf_config(cfg: Any, name: str | None = None) -> "ModelArch":
        """From a HuggingFace config object or dict (model_type llama / mistral / qwen2 / qwen3 /
        qwen3_moe / qwen2_moe / mixtral / deepseek_v2 / deepseek_v3 / glm4_moe)."""
        g = (lambda k, d=None: cfg.get(k, d)) if isinstance(cfg, dict) else (lambda k, d=None: getattr(cfg, k, d))
        mt = str(g("model_type", "llama")).lower()
        fam = {"llama": "llama", "mistral": "llama", "qwen2": "qwen2", "qwen3": "qwen3",
               "qwen3_moe": "qwen3_moe", "qwen2_moe": "qwen2_moe", "mixtral": "mixtral",
               "deepseek_v2": "deepseek_v3", "deepseek_v3": "deepseek_v3", "glm4_moe": "glm4_moe"}.get(mt)
        if fam is None:
            raise ValueError(f"unsupported model_type {mt!r}")
        H, nh = int(g("hidden_size")), int(g("num_attention_heads"))
        if fam == "glm4_moe":
            if g("use_qk_norm", False):
                raise ValueError("glm4_moe with use_qk_norm is not supported")
            moe_ffn = int(g("moe_intermediate_size", 0) or 0)
            return ModelArch(
                name=name or mt, family=fam, num_layers=int(g("num_hidden_layers")), hidden=H,
                num_heads=nh, num_kv_heads=int(g("num_key_value_heads", nh) or nh),
                head_dim=int(g("head_dim", None) or H // nh), ffn=int(g("intermediate_size", 0) or 0),
                vocab=int(g("vocab_size")), tie_embeddings=bool(g("tie_word_embeddings", False)),
                num_experts=int(g("n_routed_experts", 0) or 0), moe_ffn=moe_ffn,
                top_k=int(g("num_experts_per_tok", 0) or 0),
                shared_ffn=int(g("n_shared_experts", 0) or 0) * moe_ffn,
                first_dense_layers=int(g("first_k_dense_replace", 0) or 0), router_bias=True)
        if fam == "deepseek_v3":
            nope, rope = int(g("qk_nope_head_dim")), int(g("qk_rope_head_dim"))
            moe_ffn = int(g("moe_intermediate_size", 0) or 0)
            return ModelArch(
                name=name or mt, family=fam, num_layers=int(g("num_hidden_layers")), hidden=H,
                num_heads=nh, num_kv_heads=nh, head_dim=nope + rope,
                ffn=int(g("intermediate_size", 0) or 0), vocab=int(g("vocab_size")),
                tie_embeddings=bool(g("tie_word_embeddings", False)),
                num_experts=int(g("n_routed_experts", 0) or 0), moe_ffn=moe_ffn,
                top_k=int(g("num_experts_per_tok", 0) or 0),
                shared_ffn=int(g("n_shared_experts", 0) or 0) * moe_ffn,
                q_lora_rank=int(g("q_lora_rank", 0) or 0), kv_lora_rank=int(g("kv_lora_rank")),
                qk_nope_dim=nope, qk_rope_dim=rope, v_head_dim=int(g("v_head_dim")),
                first_dense_layers=int(g("first_k_dense_replace", 0) or 0),
                router_bias=mt == "deepseek_v3" or g("topk_method", "") == "noaux_tc")
        return ModelArch(
            name=name or mt, family=fam, num_layers=int(g("num_hidden_layers")), hidden=H,
            num_heads=nh, num_kv_heads=int(g("num_key_value_heads", nh) or nh),
            head_dim=int(g("head_dim", None) or H // nh),
            ffn=0 if fam in ("mixtral", "qwen2_moe") else int(g("intermediate_size", 0) or 0),
            vocab=int(g("vocab_size")),
            tie_embeddings=bool(g("tie_word_embeddings", False)),
            num_experts=int(g("num_local_experts" if fam == "mixtral" else "num_experts", 0) or 0),
            moe_ffn=int(g("intermediate_size" if fam == "mixtral" else "moe_intermediate_size", 0) or 0),
            top_k=int(g("num_experts_per_tok", 0) or 0),
            shared_ffn=int(g("shared_expert_intermediate_size", 0) or 0) if fam == "qwen2_moe" else 0)

    @staticmethod
    def from_megatron_args(args: Any, family: str = "qwen2", name: str | None = None) -> "ModelArch":
        """From a Megatron ``args`` namespace (hidden_size, num_attention_heads, ...; for MLA
        q_lora_rank, kv_lora_rank, qk_head_dim, qk_pos_emb_head_dim, v_head_dim)."""
        H, nh = int(args.hidden_size), int(args.num_attention_heads)
        if family == "deepseek_v3":
            nope, rope = int(args.qk_head_dim), int(args.qk_pos_emb_head_dim)
            freq = getattr(args, "moe_layer_freq", 1)
            first = 0
            if isinstance(freq, (list, tuple)):          # [0, 0, 0, 1, 1, ...]: the leading dense layers
                first = next((i for i, f in enumerate(freq) if f), len(freq))
            return ModelArch(
                name=name or family, family=family, num_layers=int(args.num_layers), hidden=H,
                num_heads=nh, num_kv_heads=nh, head_dim=nope + rope,
                ffn=int(getattr(args, "ffn_hidden_size", 0) or 0), vocab=int(args.vocab_size),
                tie_embeddings=not bool(getattr(args, "untie_embeddings_and_output_weights", True)),
                num_experts=int(getattr(args, "num_experts", 0) or 0),
                moe_ffn=int(getattr(args, "moe_ffn_hidden_size", 0) or 0),
                top_k=int(getattr(args, "moe_router_topk", 0) or 0),
                shared_ffn=int(getattr(args, "moe_shared_expert_intermediate_size", 0) or 0),
                q_lora_rank=int(getattr(args, "q_lora_rank", 0) or 0), kv_lora_rank=int(args.kv_lora_rank),
                qk_nope_dim=nope, qk_rope_dim=rope, v_head_dim=int(args.v_head_dim),
                first_dense_layers=first,
                router_bias=bool(getattr(args, "moe_router_enable_expert_bias", False)))
        kv = getattr(args, "num_query_groups", None) or nh
        hd = getattr(args, "kv_channels", None) or H // nh
        freq = getattr(args, "moe_layer_freq", 1)
        first = next((i for i, f in enumerate(freq) if f), len(freq)) if isinstance(freq, (list, tuple)) else 0
        return ModelArch(
            name=name or family, family=family, num_layers=int(args.num_layers), hidden=H,
            num_heads=nh, num_kv_heads=int(kv), head_dim=int(hd),
            ffn=int(getattr(args, "ffn_hidden_size", 0) or 0), vocab=int(args.vocab_size),
            tie_embeddings=not bool(getattr(args, "untie_embeddings_and_output_weights", True)),
            num_experts=int(getattr(args, "num_experts", 0) or 0),
            moe_ffn=int(getattr(args, "moe_ffn_hidden_size", 0) or 0),
            top_k=int(getattr(args, "moe_router_topk", 0) or 0),
            shared_ffn=int(getattr(args, "moe_shared_expert_intermediate_size", 0) or 0),
            first_dense_layers=first, router_bias=bool(getattr(args, "moe_router_enable_expert_bias", False)))


PRESETS: dict[str, ModelArch] = {
    # plumbing model: 2 layers, hidden 256, 4 heads of dim 64, 2 KV heads, FFN 688, vocab 1024
    "tiny-llama": ModelArch("tiny-llama", "llama", 2, 256, 4, 2, 64, 688, 1024),
    "llama3-8b": ModelArch("llama3-8b", "llama", 32, 4096, 32, 8, 128, 14336, 128256),
    "llama3-70b": ModelArch("llama3-70b", "llama", 80, 8192, 64, 8, 128, 28672, 128256),
    "qwen3-30b-a3b": ModelArch("qwen3-30b-a3b", "qwen3_moe", 48, 2048, 32, 4, 128, 0, 151936,
                               num_experts=128, moe_ffn=768, top_k=8),
    # small test models of every family
    "tiny-qwen2": ModelArch("tiny-qwen2", "qwen2", 2, 128, 4, 2, 32, 256, 512),
    # Llama-3-70B's attention shape in miniature (8 heads, 8 KV heads): splits at TP 8 as 70B does
    "tiny-llama-tp8": ModelArch("tiny-llama-tp8", "llama", 2, 256, 8, 8, 32, 512, 1024),
    # head dim and FFN in multiples of 128: every linear layer block-quantisable (fp8_linear)
    "tiny-llama-fp8": ModelArch("tiny-llama-fp8", "llama", 2, 256, 4, 2, 128, 512, 1024),
    "tiny-qwen3": ModelArch("tiny-qwen3", "qwen3", 2, 128, 8, 2, 32, 256, 520),
    "tiny-qwen3-moe": ModelArch("tiny-qwen3-moe", "qwen3_moe", 2, 256, 4, 2, 64, 0, 1000,
                                num_experts=8, moe_ffn=256, top_k=2),
    "tiny-mixtral": ModelArch("tiny-mixtral", "mixtral", 2, 256, 4, 2, 64, 0, 1000,
                              num_experts=4, moe_ffn=256, top_k=2),
    "tiny-qwen2-moe": ModelArch("tiny-qwen2-moe", "qwen2_moe", 2, 256, 4, 2, 64, 0, 1000,
                                num_experts=4, moe_ffn=128, top_k=2, shared_ffn=512),
    "mixtral-8x7b": ModelArch("mixtral-8x7b", "mixtral", 32, 4096, 32, 8, 128, 0, 32000,
                              num_experts=8, moe_ffn=14336, top_k=2),
    # MLA: 3 layers (the first dense), q LoRA 192, kv LoRA 128, nope 32 + rope 16, v 32
    "tiny-deepseek-v3": ModelArch("tiny-deepseek-v3", "deepseek_v3", 3, 256, 4, 4, 48, 512, 1000,
                                  num_experts=8, moe_ffn=128, top_k=2, shared_ffn=128, q_lora_rank=192,
                                  kv_lora_rank=128, qk_nope_dim=32, qk_rope_dim=16, v_head_dim=32,
                                  first_dense_layers=1, router_bias=True),
    # without q LoRA (DeepSeek-V2-Lite style), every block dimension a multiple of 128 for fp8
    "tiny-deepseek-v2-lite": ModelArch("tiny-deepseek-v2-lite", "deepseek_v3", 2, 256, 4, 4, 192, 256, 1000,
                                       num_experts=4, moe_ffn=128, top_k=2, shared_ffn=256, kv_lora_rank=128,
                                       qk_nope_dim=128, qk_rope_dim=64, v_head_dim=128, first_dense_layers=1),
    # GLM-4.5 style: GQA with q/k/v bias, a dense first layer, routed + ungated shared experts
    "tiny-glm4-moe": ModelArch("tiny-glm4-moe", "glm4_moe", 2, 256, 4, 2, 64, 512, 1000, num_experts=8,
                               moe_ffn=128, top_k=2, shared_ffn=128, first_dense_layers=1, router_bias=True),
    "glm-4.5-air": ModelArch("glm-4.5-air", "glm4_moe", 46, 4096, 96, 8, 128, 10944, 151552, num_experts=128,
                             moe_ffn=1408, top_k=8, shared_ffn=1408, first_dense_layers=1, router_bias=True),
    "deepseek-v3": ModelArch("deepseek-v3", "deepseek_v3", 61, 7168, 128, 128, 192, 18432, 129280,
                             num_experts=256, moe_ffn=2048, top_k=8, shared_ffn=2048, q_lora_rank=1536,
                             kv_lora_rank=512, qk_nope_dim=128, qk_rope_dim=64, v_head_dim=128,
                             first_dense_layers=3, router_bias=True),
    "deepseek-v2-lite": ModelArch("deepseek-v2-lite", "deepseek_v3", 27, 2048, 16, 16, 192, 10944, 102400,
                                  num_experts=64, moe_ffn=1408, top_k=6, shared_ffn=2816, kv_lora_rank=512,
                                  qk_nope_dim=128, qk_rope_dim=64, v_head_dim=128, first_dense_layers=1),
}


def get_arch(name: str) -> ModelArch:
    try:
        return PRESETS[name]
    except KeyError:
        raise ValueError(f"unknown model {name!r}; presets: {sorted(PRESETS)}") from None
