"""Architecture descriptors and the HF-named logical tensors of each model family.

Families: ``llama`` (Llama-2/3), ``qwen2`` (q/k/v bias), ``qwen3`` (q/k RMSNorm),
``qwen3_moe`` (Qwen3 attention + a routed-expert MLP in every layer), ``qwen2_moe`` (Qwen2
attention + routed experts + a gated shared expert) and ``mixtral`` (Llama attention +
``block_sparse_moe`` experts named ``w1`` / ``w3`` / ``w2``).  The reference
covers Qwen2/Qwen3 dense only (``wbridge/utils/megatron_utils/qwen2.py:13-80``,
``wbridge/utils/sglang_utils/qwen2.py:24-119``); Llama and the MoE family are new here.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any, Iterator


@dataclass(frozen=True)
class ModelArch:
    name: str
    family: str                   # llama | qwen2 | qwen3 | qwen3_moe | qwen2_moe | mixtral
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
    shared_ffn: int = 0           # shared expert's intermediate width (qwen2_moe), 0: none

    @property
    def qkv_bias(self) -> bool:
        return self.family in ("qwen2", "qwen2_moe")

    @property
    def qk_norm(self) -> bool:
        return self.family in ("qwen3", "qwen3_moe")

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

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
    def layer_tensors(self, i: int) -> Iterator[tuple[str, tuple[int, ...]]]:
        H, hd = self.hidden, self.head_dim
        p = f"model.layers.{i}."
        yield p + "input_layernorm.weight", (H,)
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
        if self.is_moe:
            I, mb = self.moe_ffn, self.moe_block
            g, u, d = self.expert_projs
            yield p + f"{mb}.gate.weight", (self.num_experts, H)
            for e in range(self.num_experts):
                q = f"{p}{mb}.experts.{e}."
                yield q + f"{g}.weight", (I, H)
                yield q + f"{u}.weight", (I, H)
                yield q + f"{d}.weight", (H, I)
            if self.shared_ffn:
                S = self.shared_ffn
                yield p + "mlp.shared_expert.gate_proj.weight", (S, H)
                yield p + "mlp.shared_expert.up_proj.weight", (S, H)
                yield p + "mlp.shared_expert.down_proj.weight", (H, S)
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
        """From a HuggingFace config object or dict (model_type llama/qwen2/qwen3/qwen3_moe)."""
        g = (lambda k, d=None: cfg.get(k, d)) if isinstance(cfg, dict) else (lambda k, d=None: getattr(cfg, k, d))
        mt = str(g("model_type", "llama")).lower()
        fam = {"llama": "llama", "mistral": "llama", "qwen2": "qwen2", "qwen3": "qwen3",
               "qwen3_moe": "qwen3_moe", "qwen2_moe": "qwen2_moe", "mixtral": "mixtral"}.get(mt)
        if fam is None:
            raise ValueError(f"unsupported model_type {mt!r}")
        H, nh = int(g("hidden_size")), int(g("num_attention_heads"))
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
        """From a Megatron ``args`` namespace (hidden_size, num_attention_heads, ...)."""
        H, nh = int(args.hidden_size), int(args.num_attention_heads)
        kv = getattr(args, "num_query_groups", None) or nh
        hd = getattr(args, "kv_channels", None) or H // nh
        return ModelArch(
            name=name or family, family=family, num_layers=int(args.num_layers), hidden=H,
            num_heads=nh, num_kv_heads=int(kv), head_dim=int(hd),
            ffn=int(getattr(args, "ffn_hidden_size", 0) or 0), vocab=int(args.vocab_size),
            tie_embeddings=not bool(getattr(args, "untie_embeddings_and_output_weights", True)),
            num_experts=int(getattr(args, "num_experts", 0) or 0),
            moe_ffn=int(getattr(args, "moe_ffn_hidden_size", 0) or 0),
            top_k=int(getattr(args, "moe_router_topk", 0) or 0),
            shared_ffn=int(getattr(args, "moe_shared_expert_intermediate_size", 0) or 0))


PRESETS: dict[str, ModelArch] = {
    # plumbing model: 2 layers, hidden 256, 4 heads of dim 64, 2 KV heads, FFN 688, vocab 1024
    "tiny-llama": ModelArch("tiny-llama", "llama", 2, 256, 4, 2, 64, 688, 1024),
    "llama3-8b": ModelArch("llama3-8b", "llama", 32, 4096, 32, 8, 128, 14336, 128256),
    "llama3-70b": ModelArch("llama3-70b", "llama", 80, 8192, 64, 8, 128, 28672, 128256),
    "qwen3-30b-a3b": ModelArch("qwen3-30b-a3b", "qwen3_moe", 48, 2048, 32, 4, 128, 0, 151936,
                               num_experts=128, moe_ffn=768, top_k=8),
    # small test models of every family
    "tiny-qwen2": ModelArch("tiny-qwen2", "qwen2", 2, 128, 4, 2, 32, 256, 512),
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
}


def get_arch(name: str) -> ModelArch:
    try:
        return PRESETS[name]
    except KeyError:
        raise ValueError(f"unknown model {name!r}; presets: {sorted(PRESETS)}") from None
