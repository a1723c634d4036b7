"""Megatron-Core trainer layout -> logical HF boxes bound to strided views of the params.

Covers TP (column/row parallel), PP (layer offset per stage, virtual pipeline chunks of the
interleaved schedule), EP and expert-TP for MoE,
grouped-interleaved fused QKV (``[G, q_per_group + 2, head_dim, H]`` per rank), fused
``linear_fc1`` (``[gate; up]`` per rank), QKV bias, q/k layernorm and vocab-parallel
embedding/output layer with vocab padding.  Multi-head latent attention (``deepseek_v3``):
the down projections ``linear_q_down_proj`` / ``linear_kv_down_proj`` are replicated, the up
projections ``linear_q_up_proj`` / ``linear_kv_up_proj`` (with their fused q / kv layernorms)
are column-parallel over heads, and each head's rows are already HF's ``[nope | rope]`` and
``[k_nope | v]``, so a rank's shard is one row range of the HF tensor.

Parity: name mapping and un-fusing follow ``wbridge/utils/megatron_utils/qwen2.py:13-80``;
shard boxes follow ``qwen2.py:83-115`` (box on ``partition_dim`` from the TP rank, vocab
truncation).  Differences: views instead of split/reshape copies, so the transfer reads
the live parameter memory; a PP stage offset on layer indices (the reference has none);
EP expert offsets; the QKV bias split uses element sizes ``[qpg*hd, hd, hd]``.
"""
from __future__ import annotations

import re
from dataclasses import dataclass
from typing import Any, Iterable

import torch

from ..core.shard import WeightData
from ..models.arch import ModelArch
from ..models.synthetic import synth_fill


class UnknownParameter(ValueError):
    """A parameter name without a HuggingFace counterpart in this layout."""


def _strip(name: str) -> str:
    while name.startswith("module."):
        name = name[len("module."):]
    return name


@dataclass
class MegatronLayout:
    arch: ModelArch
    tp: int = 1
    pp: int = 1
    ep: int = 1
    etp: int = 1
    tp_rank: int = 0
    pp_rank: int = 0
    ep_rank: int = 0
    etp_rank: int = 0
    vocab_pad_multiple: int = 128          # Megatron's make_vocab_size_divisible_by
    layers_per_stage: tuple[int, ...] | None = None
    expert_naming: str = "grouped"         # grouped: experts.linear_fc1.weight{e}; sequential: local_experts.{e}.
    vpp: int = 1                           # virtual pipeline (interleaved schedule): model chunks per stage
    vpp_rank: int = 0                      # the model chunk this layout describes

    def __post_init__(self):
        a = self.arch
        if a.num_kv_heads % self.tp:
            raise ValueError(f"num_kv_heads {a.num_kv_heads} not divisible by TP {self.tp}")
        if a.num_heads % self.tp:
            raise ValueError("num_heads not divisible by TP")
        if (not a.is_moe or a.first_dense_layers) and a.ffn % self.tp:
            raise ValueError("ffn not divisible by TP")
        if a.is_moe and (a.num_experts % self.ep or a.moe_ffn % self.etp):
            raise ValueError("experts not divisible by EP (or expert FFN by ETP)")
        if a.shared_ffn % self.tp:
            raise ValueError("shared expert FFN not divisible by TP")
        if self.vpp > 1:
            even = tuple([a.num_layers // self.pp] * self.pp)
            if a.num_layers % (self.pp * self.vpp) or self.layers_per_stage not in (None, even):
                raise ValueError("virtual pipeline stages need num_layers divisible by PP x VPP "
                                 "(and even stages)")
            if not 0 <= self.vpp_rank < self.vpp:
                raise ValueError("vpp_rank out of range")
        if self.layers_per_stage is None:
            if a.num_layers % self.pp:
                raise ValueError("num_layers not divisible by PP; pass layers_per_stage")
            self.layers_per_stage = tuple([a.num_layers // self.pp] * self.pp)
        if sum(self.layers_per_stage) != a.num_layers or len(self.layers_per_stage) != self.pp:
            raise ValueError("layers_per_stage must cover every layer once")

    # -- sizes ------------------------------------------------------------------------
    @property
    def padded_vocab(self) -> int:
        m = self.vocab_pad_multiple * self.tp
        return (self.arch.vocab + m - 1) // m * m

    @property
    def layer_offset(self) -> int:
        if self.vpp > 1:       # chunk v of stage p: the (v * PP + p)-th run of L / (PP * VPP) layers
            return (self.vpp_rank * self.pp + self.pp_rank) * self.num_local_layers
        return sum(self.layers_per_stage[: self.pp_rank])

    @property
    def num_local_layers(self) -> int:
        if self.vpp > 1:
            return self.arch.num_layers // (self.pp * self.vpp)
        return self.layers_per_stage[self.pp_rank]

    @property
    def first_stage(self) -> bool:
        return self.pp_rank == 0 and self.vpp_rank == 0

    @property
    def last_stage(self) -> bool:
        return self.pp_rank == self.pp - 1 and self.vpp_rank == self.vpp - 1

    def chunks(self) -> list["MegatronLayout"]:
        """The layouts of every model chunk this rank holds (one without virtual pipeline)."""
        from dataclasses import replace
        return [replace(self, vpp_rank=v) for v in range(self.vpp)]

    def param_shapes(self) -> dict[str, tuple[int, ...]]:
        """Megatron parameter name (local layer numbering) -> local shape."""
        a, tp = self.arch, self.tp
        H, hd = a.hidden, a.head_dim
        G_loc = a.num_kv_heads // tp
        qkv_rows = G_loc * (a.q_per_group + 2) * hd
        out: dict[str, tuple[int, ...]] = {}
        if self.first_stage:
            out["embedding.word_embeddings.weight"] = (self.padded_vocab // tp, H)
        for i in range(self.num_local_layers):
            p = f"decoder.layers.{i}."
            if a.is_mla:
                nh_loc = a.num_heads // tp
                out[p + "input_layernorm.weight"] = (H,)
                if a.q_lora_rank:
                    out[p + "self_attention.linear_q_down_proj.weight"] = (a.q_lora_rank, H)
                    out[p + "self_attention.linear_q_up_proj.layer_norm_weight"] = (a.q_lora_rank,)
                    out[p + "self_attention.linear_q_up_proj.weight"] = (nh_loc * hd, a.q_lora_rank)
                else:
                    out[p + "self_attention.linear_q_proj.weight"] = (nh_loc * hd, H)
                out[p + "self_attention.linear_kv_down_proj.weight"] = (a.kv_lora_rank + a.qk_rope_dim, H)
                out[p + "self_attention.linear_kv_up_proj.layer_norm_weight"] = (a.kv_lora_rank,)
                out[p + "self_attention.linear_kv_up_proj.weight"] = (nh_loc * (a.qk_nope_dim + a.v_head_dim),
                                                                       a.kv_lora_rank)
                out[p + "self_attention.linear_proj.weight"] = (H, nh_loc * a.v_head_dim)
            else:
                out[p + "self_attention.linear_qkv.layer_norm_weight"] = (H,)
                out[p + "self_attention.linear_qkv.weight"] = (qkv_rows, H)
                if a.qkv_bias:
                    out[p + "self_attention.linear_qkv.bias"] = (qkv_rows,)
                if a.qk_norm:
                    out[p + "self_attention.q_layernorm.weight"] = (hd,)
                    out[p + "self_attention.k_layernorm.weight"] = (hd,)
                out[p + "self_attention.linear_proj.weight"] = (H, a.num_heads * hd // tp)
            if a.moe_layer(i + self.layer_offset):
                E_loc, I_loc = a.num_experts // self.ep, a.moe_ffn // self.etp
                out[p + "pre_mlp_layernorm.weight"] = (H,)
                out[p + "mlp.router.weight"] = (a.num_experts, H)
                if a.router_bias:
                    out[p + "mlp.router.expert_bias"] = (a.num_experts,)
                for e in range(E_loc):
                    out[self._expert_name(i, e, 1)] = (2 * I_loc, H)
                    out[self._expert_name(i, e, 2)] = (H, I_loc)
                if a.shared_ffn:                       # shared expert: TP-split like a dense MLP
                    S_loc = a.shared_ffn // tp
                    out[p + "mlp.shared_experts.linear_fc1.weight"] = (2 * S_loc, H)
                    out[p + "mlp.shared_experts.linear_fc2.weight"] = (H, S_loc)
                    if a.shared_gate:                  # qwen2_moe gates its shared expert
                        out[p + "mlp.shared_experts.gate_weight"] = (1, H)
            else:
                F_loc = a.ffn // tp
                out[p + "mlp.linear_fc1.layer_norm_weight"] = (H,)
                out[p + "mlp.linear_fc1.weight"] = (2 * F_loc, H)
                out[p + "mlp.linear_fc2.weight"] = (H, F_loc)
        if self.last_stage:
            out["decoder.final_layernorm.weight"] = (H,)
            if not a.tie_embeddings:
                out["output_layer.weight"] = (self.padded_vocab // tp, H)
        return out

    def _expert_name(self, i: int, e: int, fc: int) -> str:
        if self.expert_naming == "sequential":
            return f"decoder.layers.{i}.mlp.experts.local_experts.{e}.linear_fc{fc}.weight"
        return f"decoder.layers.{i}.mlp.experts.linear_fc{fc}.weight{e}"

    def allocate(self, device="cpu", dtype=torch.bfloat16, fill: bool = True, seed: int = 0
                 ) -> dict[str, torch.Tensor]:
        """Allocate this rank's parameters; ``fill`` writes the synthetic HF weights."""
        params = {n: torch.zeros(s, dtype=dtype, device=device) for n, s in self.param_shapes().items()}
        if fill:
            self.fill(params, seed)
        return params

    def fill(self, params: dict[str, torch.Tensor], seed: int = 0) -> None:
        """Write the synthetic HF weights of ``seed`` into existing parameters, in place."""
        meta, views = self.to_wb(params)
        for name, shards, _ in meta:
            synth_fill(views[name], name, shards[0], seed=seed)

    # -- conversion ------------------------------------------------------------------------
    def split_param(self, name: str, param: torch.Tensor) -> list[tuple[str, torch.Tensor, list]]:
        """One Megatron param -> [(hf_name, view, box)] for this rank."""
        a, tp, r = self.arch, self.tp, self.tp_rank
        H, hd, qpg = a.hidden, a.head_dim, a.q_per_group
        n = _strip(name)
        full = lambda shape: [(0, d, d) for d in shape]

        def vocab_rows(t: torch.Tensor, hf: str):
            rows = self.padded_vocab // tp
            l, rr = r * rows, min((r + 1) * rows, a.vocab)
            if l >= a.vocab:
                return []
            return [(hf, t[: rr - l], [(l, rr, a.vocab), (0, H, H)])]

        if n == "embedding.word_embeddings.weight":
            return vocab_rows(param, "model.embed_tokens.weight")
        if n == "output_layer.weight":
            return vocab_rows(param, "lm_head.weight")
        if n == "decoder.final_layernorm.weight":
            return [("model.norm.weight", param, full(param.shape))]

        m = re.match(r"decoder\.layers\.(\d+)\.(.+)", n)
        if not m:
            raise UnknownParameter(f"unknown Megatron parameter {name!r}")
        li = int(m.group(1))
        rest = m.group(2)
        g = li + self.layer_offset
        p = f"model.layers.{g}."
        G = a.num_kv_heads
        G_loc = G // tp
        gbox = (r * G_loc, (r + 1) * G_loc, G)

        if a.is_mla:
            got = self._split_mla(rest, param, p)
            if got is not None:
                return got
        if rest == "self_attention.linear_qkv.weight":
            v = param.view(G_loc, (qpg + 2) * hd, H)
            return [
                (p + "self_attn.q_proj.weight", v[:, : qpg * hd], [gbox, (0, qpg * hd, qpg * hd), (0, H, H)]),
                (p + "self_attn.k_proj.weight", v[:, qpg * hd:(qpg + 1) * hd], [gbox, (0, hd, hd), (0, H, H)]),
                (p + "self_attn.v_proj.weight", v[:, (qpg + 1) * hd:], [gbox, (0, hd, hd), (0, H, H)]),
            ]
        if rest == "self_attention.linear_qkv.bias":
            v = param.view(G_loc, (qpg + 2) * hd)
            return [
                (p + "self_attn.q_proj.bias", v[:, : qpg * hd], [gbox, (0, qpg * hd, qpg * hd)]),
                (p + "self_attn.k_proj.bias", v[:, qpg * hd:(qpg + 1) * hd], [gbox, (0, hd, hd)]),
                (p + "self_attn.v_proj.bias", v[:, (qpg + 1) * hd:], [gbox, (0, hd, hd)]),
            ]
        if rest == "self_attention.linear_proj.weight":
            K = a.num_heads * hd
            k = K // tp
            return [(p + "self_attn.o_proj.weight", param, [(0, H, H), (r * k, (r + 1) * k, K)])]
        if rest == "self_attention.linear_qkv.layer_norm_weight" or rest == "input_layernorm.weight":
            return [(p + "input_layernorm.weight", param, full(param.shape))]
        if rest in ("mlp.linear_fc1.layer_norm_weight", "pre_mlp_layernorm.weight"):
            return [(p + "post_attention_layernorm.weight", param, full(param.shape))]
        if rest == "self_attention.q_layernorm.weight":
            return [(p + "self_attn.q_norm.weight", param, full(param.shape))]
        if rest == "self_attention.k_layernorm.weight":
            return [(p + "self_attn.k_norm.weight", param, full(param.shape))]
        if rest == "mlp.linear_fc1.weight":
            F = a.ffn
            f = F // tp
            box = [(r * f, (r + 1) * f, F), (0, H, H)]
            return [(p + "mlp.gate_proj.weight", param[:f], box),
                    (p + "mlp.up_proj.weight", param[f:], box)]
        if rest == "mlp.linear_fc2.weight":
            F = a.ffn
            f = F // tp
            return [(p + "mlp.down_proj.weight", param, [(0, H, H), (r * f, (r + 1) * f, F)])]
        if rest == "mlp.shared_experts.linear_fc1.weight":
            S, sp = a.shared_ffn, p + a.shared_prefix
            sl = S // tp
            box = [(r * sl, (r + 1) * sl, S), (0, H, H)]
            return [(sp + "gate_proj.weight", param[:sl], box),
                    (sp + "up_proj.weight", param[sl:], box)]
        if rest == "mlp.shared_experts.linear_fc2.weight":
            S, sp = a.shared_ffn, p + a.shared_prefix
            sl = S // tp
            return [(sp + "down_proj.weight", param, [(0, H, H), (r * sl, (r + 1) * sl, S)])]
        if rest == "mlp.shared_experts.gate_weight":
            return [(p + "mlp.shared_expert_gate.weight", param, full(param.shape))]
        if rest == "mlp.router.weight":
            return [(p + f"{a.moe_block}.gate.weight", param, full(param.shape))]
        if rest == "mlp.router.expert_bias":
            return [(p + f"{a.moe_block}.gate.e_score_correction_bias", param, full(param.shape))]
        em = (re.match(r"mlp\.experts\.linear_fc([12])\.weight(\d+)$", rest)
              or re.match(r"mlp\.experts\.local_experts\.(?P<e>\d+)\.linear_fc(?P<fc>[12])\.weight$", rest))
        if em:
            if em.re.groupindex:
                fc, e = int(em.group("fc")), int(em.group("e"))
            else:
                fc, e = int(em.group(1)), int(em.group(2))
            E_loc = a.num_experts // self.ep
            if e >= E_loc:
                raise ValueError(f"{name}: local expert {e} of {E_loc} (num_experts {a.num_experts} / EP {self.ep})")
            eg = self.ep_rank * E_loc + e
            I = a.moe_ffn
            i_loc = I // self.etp
            ibox = (self.etp_rank * i_loc, (self.etp_rank + 1) * i_loc, I)
            q = f"{p}{a.moe_block}.experts.{eg}."
            gn, un, dn = a.expert_projs
            if fc == 1:
                return [(q + f"{gn}.weight", param[:i_loc], [ibox, (0, H, H)]),
                        (q + f"{un}.weight", param[i_loc:], [ibox, (0, H, H)])]
            return [(q + f"{dn}.weight", param, [(0, H, H), ibox])]
        raise UnknownParameter(f"unknown Megatron parameter {name!r}")

    def _split_mla(self, rest: str, param: torch.Tensor, p: str) -> list | None:
        """The MLA attention params of one layer (``None``: not an MLA attention param)."""
        a, tp, r = self.arch, self.tp, self.tp_rank
        H, nh = a.hidden, a.num_heads
        nh_loc = nh // tp
        full = lambda shape: [(0, d, d) for d in shape]         # noqa: E731

        def heads(rows_per_head: int, cols: int):              # column-parallel over heads
            R = nh * rows_per_head
            return [(r * nh_loc * rows_per_head, (r + 1) * nh_loc * rows_per_head, R), (0, cols, cols)]

        if rest == "self_attention.linear_q_down_proj.weight":
            return [(p + "self_attn.q_a_proj.weight", param, full(param.shape))]
        if rest in ("self_attention.linear_q_up_proj.layer_norm_weight", "self_attention.q_layernorm.weight"):
            return [(p + "self_attn.q_a_layernorm.weight", param, full(param.shape))]
        if rest == "self_attention.linear_q_up_proj.weight":
            return [(p + "self_attn.q_b_proj.weight", param, heads(a.head_dim, a.q_lora_rank))]
        if rest == "self_attention.linear_q_proj.weight":
            return [(p + "self_attn.q_proj.weight", param, heads(a.head_dim, H))]
        if rest == "self_attention.linear_kv_down_proj.weight":
            return [(p + "self_attn.kv_a_proj_with_mqa.weight", param, full(param.shape))]
        if rest in ("self_attention.linear_kv_up_proj.layer_norm_weight", "self_attention.kv_layernorm.weight"):
            return [(p + "self_attn.kv_a_layernorm.weight", param, full(param.shape))]
        if rest == "self_attention.linear_kv_up_proj.weight":
            return [(p + "self_attn.kv_b_proj.weight", param, heads(a.qk_nope_dim + a.v_head_dim, a.kv_lora_rank))]
        if rest == "self_attention.linear_proj.weight":
            K = nh * a.v_head_dim
            k = K // tp
            return [(p + "self_attn.o_proj.weight", param, [(0, H, H), (r * k, (r + 1) * k, K)])]
        return None

    def to_wb(self, named_params: dict[str, torch.Tensor] | Iterable[tuple[str, torch.Tensor]],
              strict: bool = True) -> tuple[WeightData, dict[str, torch.Tensor]]:
        """(metadata, HF name -> strided view) for this rank's parameters.  ``strict=False``
        skips parameters without an HF counterpart (adapters, extra heads) instead of raising."""
        items = named_params.items() if isinstance(named_params, dict) else named_params
        meta: dict[str, dict[str, Any]] = {}
        views: dict[str, torch.Tensor] = {}
        for name, param in items:
            t = param.data if isinstance(param, torch.nn.Parameter) else param
            try:
                parts = self.split_param(name, t)
            except UnknownParameter:
                if strict:
                    raise
                continue
            for hf, view, box in parts:
                meta[hf] = {"shard": box, "dtype": view.dtype}
                views[hf] = view
        return WeightData(meta), views


def convert_to_wb(args: Any, model_name: str, named_tensors, *, tp_rank: int | None = None,
                  tp_size: int | None = None, pp_rank: int = 0, pp_size: int = 1,
                  ep_rank: int = 0, ep_size: int = 1, vpp_rank: int = 0, vpp_size: int = 1,
                  quantization_config=None) -> tuple[WeightData, dict[str, torch.Tensor]]:
    """Megatron ``args`` + named params -> (WeightData, views); the reference's entry point
    (``wbridge/utils/megatron_utils/__init__.py:11-19``) with explicit parallel ranks.  With
    the interleaved schedule, call it once per model chunk (``vpp_rank``) and merge.
    When ranks are omitted they are read from ``megatron.core.mpu`` if it is importable."""
    if tp_rank is None or tp_size is None:
        try:
            from megatron.core import mpu  # type: ignore
        except ImportError:
            raise ValueError("pass tp_rank/tp_size (megatron.core is not importable)") from None
        tp_rank, tp_size = mpu.get_tensor_model_parallel_rank(), mpu.get_tensor_model_parallel_world_size()
        pp_rank, pp_size = mpu.get_pipeline_model_parallel_rank(), mpu.get_pipeline_model_parallel_world_size()
        ep_rank, ep_size = mpu.get_expert_model_parallel_rank(), mpu.get_expert_model_parallel_world_size()
        vpp_size = mpu.get_virtual_pipeline_model_parallel_world_size() or 1
        vpp_rank = (mpu.get_virtual_pipeline_model_parallel_rank() or 0) if vpp_size > 1 else 0
    name = model_name.lower()
    family = ("deepseek_v3" if "deepseek" in name else "glm4_moe" if "glm" in name else
              "mixtral" if "mixtral" in name else "qwen2_moe" if "qwen2" in name and "moe" in name else
              "qwen3_moe" if "moe" in name else "qwen3" if "qwen3" in name else
              "qwen2" if "qwen2" in name else "llama" if "llama" in name else None)
    if family is None:
        raise ValueError(f"unsupported model for convert_to_wb: {model_name}")
    arch = ModelArch.from_megatron_args(args, family=family, name=model_name)
    layout = MegatronLayout(arch, tp=tp_size, pp=pp_size, ep=ep_size, tp_rank=tp_rank,
                            pp_rank=pp_rank, ep_rank=ep_rank, vpp=vpp_size, vpp_rank=vpp_rank,
                            vocab_pad_multiple=int(getattr(args, "make_vocab_size_divisible_by", 128)))
    return layout.to_wb(named_tensors)
