"""SGLang rollout layout -> logical HF boxes bound to views of SGLang's fused parameters.

SGLang stores ``qkv_proj`` as ``[q_local; k_local; v_local]`` (QKVParallelLinear), fuses
``gate_up_proj`` as ``[gate_local; up_local]``, pads the vocab of ``embed_tokens`` /
``lm_head`` and, for MoE, keeps all local experts in ``experts.w13_weight`` ``[E_loc,
2*I_loc, H]`` and ``experts.w2_weight`` ``[E_loc, H, I_loc]``.  With block fp8 the
weights are ``float8_e4m3fn`` and each has an fp32 ``*_scale_inv`` of 128 x 128 block
scales.  Attention may use its own TP size (DP-attention); when TP exceeds the KV-head
count each rank holds one replicated KV head.

Multi-head latent attention (``deepseek_v3``): ``fused_qkv_a_proj_with_mqa`` is
``[q_a_proj; kv_a_proj_with_mqa]`` (replicated), ``q_b_proj`` / ``kv_b_proj`` are split over
heads, and the absorbed-attention copies of ``kv_b_proj`` that SGLang derives after loading
are refreshed by the same sync: ``self_attn.w_kc`` (``[heads, nope, kv_lora]``, stored
transposed) and ``self_attn.w_vc`` (``[heads, kv_lora, v]``, a transposed view of
``[heads, v, kv_lora]``) are extra destination shards of ``kv_b_proj``.

Parity: the routing and the column/row partition rules follow
``wbridge/utils/sglang_utils/qwen2.py:1-173`` and ``sglang_utils/__init__.py:15-52``.
Differences: the q/k/v split uses SGLang's ``[q; k; v]`` order rather than a grouped
interleave, the bias split uses element sizes, the receiver gets views into its own fused
buffers (the reference only returns metadata), KV-head replication and MoE/fp8 are added.
"""
from __future__ import annotations

import re
from dataclasses import dataclass
from typing import Any

import torch

from ..core.shard import WeightData
from ..models.arch import ModelArch
from ..models.synthetic import synth_fill
from ..ops.quant_ref import block_quant_fp8_ref
from .megatron import UnknownParameter

SKIP_PATTERNS = ("inv_freq", "cos_cached", "sin_cached", "projector", "vision_tower")
# MLA tensors SGLang keeps with transposed storage: allocated as [..., b, a], viewed as [..., a, b]
TRANSPOSED = ("self_attn.w_kc", "self_attn.w_vc")


@dataclass
class SGLangLayout:
    arch: ModelArch
    tp: int = 1
    tp_rank: int = 0
    attn_tp: int | None = None
    attn_tp_rank: int | None = None
    moe_ep: int = 1                      # experts split over moe_ep of the tp ranks
    quant: str | None = None             # None | "fp8_experts" | "fp8_linear"
    block: tuple[int, int] = (128, 128)
    vocab_pad_multiple: int = 64
    # expert placement with redundant slots (SGLang EPLB): the logical expert held by each of
    # this rank's physical slots, one list for every layer or a list of lists per layer;
    # -1 is the shared expert fused into the routed-expert tensors (its own shared_experts
    # parameters then do not exist on this rank); None: the contiguous split of the experts
    # over the moe_ep ranks
    expert_slots: tuple | list | None = None

    def __post_init__(self):
        if self.attn_tp is None:
            self.attn_tp = self.tp
        if self.attn_tp_rank is None:
            self.attn_tp_rank = self.tp_rank % self.attn_tp
        a = self.arch
        if a.num_heads % self.attn_tp:
            raise ValueError("num_heads not divisible by attention TP")
        if a.num_kv_heads >= self.attn_tp and a.num_kv_heads % self.attn_tp:
            raise ValueError("num_kv_heads not divisible by attention TP")
        if a.num_kv_heads < self.attn_tp and self.attn_tp % a.num_kv_heads:
            raise ValueError("attention TP not a multiple of num_kv_heads")
        if a.is_moe:
            if self.tp % self.moe_ep or a.num_experts % self.moe_ep:
                raise ValueError("moe_ep must divide TP and the expert count")
            if a.moe_ffn % self.moe_tp:
                raise ValueError("expert FFN not divisible by the MoE TP size")
        if self.quant not in (None, "fp8_experts", "fp8_linear"):
            raise ValueError(f"unknown quant mode {self.quant!r}")
        if self.quant == "fp8_linear" and a.is_mla:
            raise ValueError("fp8_linear: MLA attention stays bf16 here (w_kc / w_vc are bf16 copies of "
                             "kv_b_proj); use quant='fp8_experts'")
        if self.expert_slots is not None:
            per_layer = list(self.expert_slots)
            if per_layer and not isinstance(per_layer[0], (list, tuple)):
                per_layer = [per_layer] * a.num_layers
            if len(per_layer) != a.num_layers:
                raise ValueError("expert_slots needs one slot list per layer (or one for all)")
            for slots in per_layer:
                if any(not -1 <= int(e) < a.num_experts for e in slots):
                    raise ValueError(f"expert_slots names an expert outside 0..{a.num_experts - 1} (or -1)")
                if -1 in slots and (not a.shared_ffn or a.shared_ffn != a.moe_ffn or a.shared_gate):
                    raise ValueError("a fused shared-expert slot (-1) needs one ungated shared expert of the "
                                     "routed experts' width")
            self.expert_slots = tuple(tuple(int(e) for e in slots) for slots in per_layer)

    def local_experts(self, layer: int) -> list[int]:
        """The logical expert of each local physical slot of ``layer``."""
        if self.expert_slots is not None:
            return list(self.expert_slots[layer])
        E_loc = self.arch.num_experts // self.moe_ep
        return [self.moe_ep_rank * E_loc + e for e in range(E_loc)]

    # -- sizes ------------------------------------------------------------------------
    @property
    def moe_tp(self) -> int:
        return self.tp // self.moe_ep

    @property
    def moe_tp_rank(self) -> int:
        return self.tp_rank % self.moe_tp

    @property
    def moe_ep_rank(self) -> int:
        return self.tp_rank // self.moe_tp

    @property
    def padded_vocab(self) -> int:
        m = self.vocab_pad_multiple
        v = (self.arch.vocab + m - 1) // m * m
        if v % self.tp:
            v = (v + self.tp - 1) // self.tp * self.tp
        return v

    @property
    def kv_local(self) -> int:
        return max(1, self.arch.num_kv_heads // self.attn_tp)

    @property
    def kv_head0(self) -> int:
        a = self.arch
        if a.num_kv_heads >= self.attn_tp:
            return self.attn_tp_rank * self.kv_local
        return self.attn_tp_rank * a.num_kv_heads // self.attn_tp

    def _fp8(self, kind: str) -> bool:
        return (self.quant == "fp8_linear" and kind in ("linear", "expert")) or \
               (self.quant == "fp8_experts" and kind == "expert")

    def _scales(self, rows: int, cols: int) -> tuple[int, int]:
        bn, bk = self.block
        return (rows + bn - 1) // bn, (cols + bk - 1) // bk

    def param_specs(self) -> dict[str, tuple[tuple[int, ...], str]]:
        """SGLang parameter name -> (local shape, kind); kind in linear|expert|scale|other."""
        a = self.arch
        H, hd = a.hidden, a.head_dim
        q_loc = a.num_heads // self.attn_tp * hd
        kv_loc = self.kv_local * hd
        out: dict[str, tuple[tuple[int, ...], str]] = {}
        V = self.padded_vocab // self.tp
        out["model.embed_tokens.weight"] = ((V, H), "other")
        for i in range(a.num_layers):
            p = f"model.layers.{i}."
            out[p + "input_layernorm.weight"] = ((H,), "other")
            if a.is_mla:
                out.update(self._mla_specs(p))
            else:
                out[p + "self_attn.qkv_proj.weight"] = ((q_loc + 2 * kv_loc, H), "linear")
                if a.qkv_bias:
                    out[p + "self_attn.qkv_proj.bias"] = ((q_loc + 2 * kv_loc,), "other")
                if a.qk_norm:
                    out[p + "self_attn.q_norm.weight"] = ((hd,), "other")
                    out[p + "self_attn.k_norm.weight"] = ((hd,), "other")
                out[p + "self_attn.o_proj.weight"] = ((H, q_loc), "linear")
            out[p + "post_attention_layernorm.weight"] = ((H,), "other")
            if a.moe_layer(i):
                E_loc = len(self.local_experts(i))
                I_loc = a.moe_ffn // self.moe_tp
                mb = a.moe_block
                out[p + f"{mb}.gate.weight"] = ((a.num_experts, H), "other")
                if a.router_bias:
                    out[p + f"{mb}.gate.e_score_correction_bias"] = ((a.num_experts,), "other")
                out[p + f"{mb}.experts.w13_weight"] = ((E_loc, 2 * I_loc, H), "expert")
                out[p + f"{mb}.experts.w2_weight"] = ((E_loc, H, I_loc), "expert")
                if a.shared_ffn and -1 not in self.local_experts(i):   # a TP-split dense MLP (+ a gate)
                    S_loc, sp = a.shared_ffn // self.tp, p + a.shared_prefix
                    out[sp + "gate_up_proj.weight"] = ((2 * S_loc, H), "linear")
                    out[sp + "down_proj.weight"] = ((H, S_loc), "linear")
                    if a.shared_gate:
                        out[p + "mlp.shared_expert_gate.weight"] = ((1, H), "other")
            else:
                F_loc = a.ffn // self.tp
                out[p + "mlp.gate_up_proj.weight"] = ((2 * F_loc, H), "linear")
                out[p + "mlp.down_proj.weight"] = ((H, F_loc), "linear")
        out["model.norm.weight"] = ((H,), "other")
        if not a.tie_embeddings:
            out["lm_head.weight"] = ((V, H), "other")
        for name, (shape, kind) in list(out.items()):
            if self._fp8(kind):
                lead, (r, c) = shape[:-2], shape[-2:]
                out[name + "_scale_inv"] = (tuple(lead) + self._scales(r, c), "scale")
        return out

    def _mla_specs(self, p: str) -> dict[str, tuple[tuple[int, ...], str]]:
        """One layer's MLA attention parameters: name -> (local shape, kind)."""
        a = self.arch
        H, nh_loc, kvl = a.hidden, a.num_heads // self.attn_tp, a.kv_lora_rank
        out = {}
        if a.q_lora_rank:
            out[p + "self_attn.fused_qkv_a_proj_with_mqa.weight"] = ((a.q_lora_rank + kvl + a.qk_rope_dim, H), "other")
            out[p + "self_attn.q_a_layernorm.weight"] = ((a.q_lora_rank,), "other")
            out[p + "self_attn.q_b_proj.weight"] = ((nh_loc * a.head_dim, a.q_lora_rank), "linear")
        else:
            out[p + "self_attn.q_proj.weight"] = ((nh_loc * a.head_dim, H), "linear")
            out[p + "self_attn.kv_a_proj_with_mqa.weight"] = ((kvl + a.qk_rope_dim, H), "other")
        out[p + "self_attn.kv_a_layernorm.weight"] = ((kvl,), "other")
        out[p + "self_attn.kv_b_proj.weight"] = ((nh_loc * (a.qk_nope_dim + a.v_head_dim), kvl), "linear")
        out[p + "self_attn.o_proj.weight"] = ((a.hidden, nh_loc * a.v_head_dim), "linear")
        out[p + "self_attn.w_kc"] = ((nh_loc, a.qk_nope_dim, kvl), "derived")
        out[p + "self_attn.w_vc"] = ((nh_loc, kvl, a.v_head_dim), "derived")
        return out

    def param_dtype(self, name: str, kind: str, dtype: torch.dtype) -> torch.dtype:
        if kind == "scale":
            return torch.float32
        if self._fp8(kind):
            return torch.float8_e4m3fn
        return dtype

    def pool_bytes(self, dtype=torch.bfloat16, align: int = 256) -> int:
        """Bytes ``allocate(pool=True)`` needs (for sizing an external buffer such as a VmmPool)."""
        total = 0
        for n, (shape, k) in self.param_specs().items():
            total = (total + align - 1) // align * align
            numel = 1
            for d in shape:
                numel *= d
            total += numel * self.param_dtype(n, k, dtype).itemsize
        return total

    def allocate(self, device="cpu", dtype=torch.bfloat16, fill: bool = False, seed: int = 0,
                 pool: bool = False, buffer: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        """Allocate this rank's parameters (zeros); ``fill`` writes the expected synthetic
        weights (quantised where the layout is fp8), i.e. what a sync should produce.
        ``pool`` places every parameter in one allocation (one CUDA IPC handle to export
        instead of one per parameter), each start aligned to 256 bytes."""
        specs = [(n, _storage_shape(n, s), self.param_dtype(n, k, dtype)) for n, (s, k) in self.param_specs().items()]
        if pool or buffer is not None:
            params = pooled_zeros(specs, device, buffer=buffer)
        else:
            params = {n: torch.zeros(s, dtype=dt, device=device) for n, s, dt in specs}
        for n in params:
            if n.endswith(TRANSPOSED):
                params[n] = params[n].transpose(-1, -2)
        if fill:
            self.fill_expected(params, seed, src_dtype=dtype)
        return params

    def fill_expected(self, params: dict[str, torch.Tensor], seed: int = 0,
                      src_dtype: torch.dtype = torch.bfloat16) -> None:
        """Write the synthetic weights; fp8 entries are the block quantisation of the
        ``src_dtype`` weights a trainer would send."""
        meta, views = self.to_wb(params)
        as_list = lambda v: v if isinstance(v, list) else [v]      # noqa: E731  (redundant slots)
        for name, shards, dtype in meta:
            q = meta.quant(name)
            if q and q.get("role") == "scale":
                continue
            for box, view, sview in zip(shards, as_list(views[name]),
                                        as_list(views[q["scale"]]) if q else [None] * len(shards)):
                if q:
                    src = torch.empty([r - l for l, r, _ in box], dtype=src_dtype, device=view.device)
                    synth_fill(src, name, box, seed=seed)
                    qv, sv = block_quant_fp8_ref(src, tuple(q["block"]))
                    view.copy_(qv)
                    sview.copy_(sv)
                else:
                    synth_fill(view, name, box, seed=seed)

    # -- conversion ------------------------------------------------------------------------
    def split_param(self, name: str, param: torch.Tensor, scale: torch.Tensor | None = None
                    ) -> list[tuple[str, torch.Tensor, list, dict | None]]:
        """One SGLang param -> [(hf_name, view, box, quant)] (quant: None or the fp8 spec)."""
        a = self.arch
        H, hd = a.hidden, a.head_dim
        full = lambda shape: [(0, d, d) for d in shape]
        bn, bk = self.block

        def q_spec(hf: str) -> dict:
            return {"format": "fp8_block", "block": [bn, bk], "scale": hf + "_scale_inv"}

        def with_scale(hf, view, box, sview, sbox):
            if scale is None:
                return [(hf, view, box, None)]
            return [(hf, view, box, q_spec(hf)),
                    (hf + "_scale_inv", sview, sbox, {"role": "scale", "of": hf})]

        def block_box(box):
            out = []
            for (l, r, w), b in zip(box, (bn, bk)):
                if l % b or (r % b and r != w):
                    raise ValueError(f"fp8 block {self.block} not aligned with box {box}")
                out.append((l // b, (r + b - 1) // b, (w + b - 1) // b))
            return out

        if name in ("model.embed_tokens.weight", "lm_head.weight"):
            rows = self.padded_vocab // self.tp
            l, r = self.tp_rank * rows, min((self.tp_rank + 1) * rows, a.vocab)
            if l >= a.vocab:
                return []
            return [(name, param[: r - l], [(l, r, a.vocab), (0, H, H)], None)]
        if name == "model.norm.weight":
            return [(name, param, full(param.shape), None)]
        m = re.match(r"model\.layers\.(\d+)\.(.+)", name)
        if not m:
            raise UnknownParameter(f"unknown SGLang parameter {name!r}")
        p = f"model.layers.{m.group(1)}."
        rest = m.group(2)
        if a.is_mla:
            got = self._split_mla(rest, param, p)
            if got is not None:
                return got
        q_loc = a.num_heads // self.attn_tp * hd
        kv_loc = self.kv_local * hd
        ar = self.attn_tp_rank
        qbox = (ar * q_loc, (ar + 1) * q_loc, a.num_heads * hd)
        kvbox = (self.kv_head0 * hd, self.kv_head0 * hd + kv_loc, a.num_kv_heads * hd)

        if rest == "self_attn.qkv_proj.weight":
            parts = [("q_proj", 0, q_loc, qbox), ("k_proj", q_loc, kv_loc, kvbox),
                     ("v_proj", q_loc + kv_loc, kv_loc, kvbox)]
            out = []
            for nm, r0, n, box in parts:
                b2 = [box, (0, H, H)]
                sv = sb = None
                if scale is not None:
                    if r0 % bn:
                        raise ValueError(f"qkv_proj: {nm} starts at row {r0}, inside an fp8 block of {bn} rows")
                    sb = block_box(b2)
                    sv = scale[r0 // bn:(r0 + n + bn - 1) // bn]
                out += with_scale(f"{p}self_attn.{nm}.weight", param[r0:r0 + n], b2, sv, sb)
            return out
        if rest == "self_attn.qkv_proj.bias":
            return [(f"{p}self_attn.q_proj.bias", param[:q_loc], [qbox], None),
                    (f"{p}self_attn.k_proj.bias", param[q_loc:q_loc + kv_loc], [kvbox], None),
                    (f"{p}self_attn.v_proj.bias", param[q_loc + kv_loc:], [kvbox], None)]
        if rest == "self_attn.o_proj.weight":
            box = [(0, H, H), qbox]
            return with_scale(name, param, box, scale, block_box(box) if scale is not None else None)
        if rest in ("mlp.gate_up_proj.weight", a.shared_prefix + "gate_up_proj.weight"):
            shared = rest != "mlp.gate_up_proj.weight"
            F = a.shared_ffn if shared else a.ffn
            mod = a.shared_prefix if shared else "mlp."
            f = F // self.tp
            fbox = (self.tp_rank * f, (self.tp_rank + 1) * f, F)
            box = [fbox, (0, H, H)]
            out = []
            for j, nm in enumerate(("gate_proj", "up_proj")):
                sv = sb = None
                if scale is not None:
                    sb = block_box(box)
                    if f % bn:
                        raise ValueError("gate/up split not aligned with the fp8 block")
                    sv = scale[j * f // bn:(j + 1) * f // bn]
                out += with_scale(f"{p}{mod}{nm}.weight", param[j * f:(j + 1) * f], box, sv, sb)
            return out
        if rest in ("mlp.down_proj.weight", a.shared_prefix + "down_proj.weight"):
            F = a.shared_ffn if rest != "mlp.down_proj.weight" else a.ffn
            f = F // self.tp
            box = [(0, H, H), (self.tp_rank * f, (self.tp_rank + 1) * f, F)]
            return with_scale(name, param, box, scale, block_box(box) if scale is not None else None)
        if rest in (f"{a.moe_block}.experts.w13_weight", f"{a.moe_block}.experts.w2_weight"):
            I = a.moe_ffn
            i_loc = I // self.moe_tp
            ibox = (self.moe_tp_rank * i_loc, (self.moe_tp_rank + 1) * i_loc, I)
            out = []
            slots = self.local_experts(int(m.group(1)))
            if param.shape[0] != len(slots):
                raise ValueError(f"{name} holds {param.shape[0]} expert slots, the layout expects {len(slots)}: "
                                 "describe redundant or fused shared-expert slots with expert_slots=")
            for e, eg in enumerate(slots):
                q = f"{p}{a.moe_block}.experts.{eg}."
                gn, un, dn = a.expert_projs
                if eg == -1:                     # the fused shared expert
                    q, (gn, un, dn) = p + a.shared_prefix, ("gate_proj", "up_proj", "down_proj")
                if rest.endswith("w13_weight"):
                    if scale is not None and i_loc % bn:
                        raise ValueError("w13 gate/up split not aligned with the fp8 block")
                    for j, nm in enumerate((gn, un)):
                        box = [ibox, (0, H, H)]
                        sv = scale[e, j * i_loc // bn:(j + 1) * i_loc // bn] if scale is not None else None
                        out += with_scale(q + nm + ".weight", param[e, j * i_loc:(j + 1) * i_loc], box, sv,
                                          block_box(box) if scale is not None else None)
                else:
                    box = [(0, H, H), ibox]
                    out += with_scale(q + f"{dn}.weight", param[e], box,
                                      scale[e] if scale is not None else None,
                                      block_box(box) if scale is not None else None)
            return out
        # replicated tensors: norms, router, q/k norm
        return [(name, param, full(param.shape), None)]

    def _split_mla(self, rest: str, param: torch.Tensor, p: str) -> list | None:
        """The MLA attention params of one layer (``None``: not one of them, or replicated
        under its HF name)."""
        a = self.arch
        H, nh = a.hidden, a.num_heads
        nh_loc, ar = nh // self.attn_tp, self.attn_tp_rank
        nope, v, kvl = a.qk_nope_dim, a.v_head_dim, a.kv_lora_rank
        full = lambda shape: [(0, d, d) for d in shape]         # noqa: E731
        hbox = (ar * nh_loc, (ar + 1) * nh_loc, nh)

        def heads(rows_per_head: int, cols: int):
            return [(ar * nh_loc * rows_per_head, (ar + 1) * nh_loc * rows_per_head, nh * rows_per_head),
                    (0, cols, cols)]

        if rest == "self_attn.fused_qkv_a_proj_with_mqa.weight":
            ql = a.q_lora_rank
            return [(p + "self_attn.q_a_proj.weight", param[:ql], full((ql, H)), None),
                    (p + "self_attn.kv_a_proj_with_mqa.weight", param[ql:], full((kvl + a.qk_rope_dim, H)), None)]
        if rest == "self_attn.q_b_proj.weight":
            return [(p + rest, param, heads(a.head_dim, a.q_lora_rank), None)]
        if rest == "self_attn.q_proj.weight":
            return [(p + rest, param, heads(a.head_dim, H), None)]
        if rest == "self_attn.kv_b_proj.weight":
            return [(p + rest, param, heads(nope + v, kvl), None)]
        if rest == "self_attn.o_proj.weight":
            return [(p + rest, param, [(0, H, H), (ar * nh_loc * v, (ar + 1) * nh_loc * v, nh * v)], None)]
        if rest == "self_attn.w_kc":          # [heads, nope, kv_lora]: the k_nope rows of each head
            return [(p + "self_attn.kv_b_proj.weight", param, [hbox, (0, nope, nope + v), (0, kvl, kvl)], None)]
        if rest == "self_attn.w_vc":          # [heads, kv_lora, v]: the v rows of each head, transposed
            return [(p + "self_attn.kv_b_proj.weight", param.transpose(-1, -2),
                     [hbox, (nope, nope + v, nope + v), (0, kvl, kvl)], None)]
        return None

    def to_wb(self, params: dict[str, torch.Tensor], strict: bool = True) -> tuple[WeightData, dict[str, torch.Tensor]]:
        """(metadata, HF name -> view) for this rank's SGLang parameters.  fp8 entries carry
        ``quant`` and their scale views appear as ``<name>_scale_inv`` entries.
        ``strict=False`` skips parameters this layout does not know instead of raising."""
        meta: dict[str, dict[str, Any]] = {}
        views: dict[str, torch.Tensor] = {}
        for name, param in params.items():
            if not isinstance(param, torch.Tensor) or name.endswith("_scale_inv"):
                continue
            if any(s in name for s in SKIP_PATTERNS):
                continue
            t = param.data if isinstance(param, torch.nn.Parameter) else param
            scale = params.get(name + "_scale_inv")
            try:
                parts = self.split_param(name, t, scale)
            except UnknownParameter:
                if strict:
                    raise
                continue
            for hf, view, box, q in parts:
                if hf in meta:           # a redundant expert slot: one more shard (and view) of it
                    e = meta[hf]
                    if not isinstance(views[hf], list):
                        e["shard"], views[hf] = [e["shard"]], [views[hf]]
                    e["shard"].append(box)
                    views[hf].append(view)
                    continue
                entry = {"shard": box, "dtype": view.dtype}
                if q:
                    entry["quant"] = q
                meta[hf] = entry
                views[hf] = view
        return WeightData(meta), views


def _storage_shape(name: str, shape: tuple[int, ...]) -> tuple[int, ...]:
    if name.endswith(TRANSPOSED):
        return tuple(shape[:-2]) + (shape[-1], shape[-2])
    return tuple(shape)


def pooled_zeros(specs, device, align: int = 256, buffer: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
    """Zero tensors of the given (name, shape, dtype) carved out of one allocation (a new
    one, or ``buffer``: a uint8 tensor such as a VmmPool's parameter region)."""
    offs, total = [], 0
    for _n, shape, dt in specs:
        total = (total + align - 1) // align * align
        offs.append(total)
        numel = 1
        for d in shape:
            numel *= d
        total += numel * dt.itemsize
    if buffer is not None:
        if buffer.numel() < total:
            raise ValueError(f"buffer of {buffer.numel()} bytes cannot hold {total} bytes of parameters")
        buf = buffer
        buf[:total].zero_()
    else:
        buf = torch.zeros(max(total, 1), dtype=torch.uint8, device=device)
    out = {}
    for (n, shape, dt), off in zip(specs, offs):
        numel = 1
        for d in shape:
            numel *= d
        out[n] = buf[off:off + numel * dt.itemsize].view(dt).view(shape)
    return out


def convert_to_wb(model_config: Any, state_dict: dict[str, torch.Tensor], tp_rank: int, tp_size: int,
                  attn_tp_rank: int | None = None, attn_tp_size: int | None = None,
                  moe_ep: int = 1, quant: str | None = None) -> WeightData:
    """SGLang state_dict -> WeightData (the reference's signature,
    ``wbridge/utils/sglang_utils/__init__.py:15-52``); ``convert_to_wb_and_views`` also
    returns the views the receiver binds.  MLA models (DeepSeek-V2/V3): SGLang keeps
    ``self_attn.w_kc`` / ``self_attn.w_vc`` as attributes, not parameters; add them to
    ``state_dict`` under those names so the sync refreshes them with ``kv_b_proj``."""
    return convert_to_wb_and_views(model_config, state_dict, tp_rank, tp_size, attn_tp_rank,
                                   attn_tp_size, moe_ep, quant)[0]


def convert_to_wb_and_views(model_config: Any, state_dict, tp_rank, tp_size, attn_tp_rank=None,
                            attn_tp_size=None, moe_ep: int = 1, quant: str | None = None):
    hf = getattr(model_config, "hf_text_config", None) or getattr(model_config, "hf_config", model_config)
    arch = ModelArch.from_hf_config(hf)
    layout = SGLangLayout(arch, tp=tp_size, tp_rank=tp_rank, attn_tp=attn_tp_size,
                          attn_tp_rank=attn_tp_rank, moe_ep=moe_ep, quant=quant)
    return layout.to_wb(state_dict)


# vLLM keeps the same fused parameter layout for these families (QKVParallelLinear
# ``[q; k; v]``, MergedColumnParallelLinear ``[gate; up]``, VocabParallelEmbedding padded to a
# multiple of 64, FusedMoE ``w13_weight`` / ``w2_weight``, block-fp8 ``*_weight_scale_inv``),
# so a vLLM rollout binds its parameters with the same layout class.
VLLMLayout = SGLangLayout
