"""MoE layer configuration (the layer-op config struct).

Mirrors the attributes the reference's MoE layer call reads from an mlx_lm
MoE module (ef_engine.py:598-631): ``num_experts_per_tok``, the quantisation
``group_size``/``bits`` of ``switch_mlp.{gate,up,down}_proj`` and whether
``shared_experts`` exists, plus the routing parameters of the gate that the
reference obtains from mlx_lm (softmax top-k for Mixtral/Qwen3-MoE; sigmoid,
group-limited, ``routed_scaling_factor`` for DeepSeek-V3, expertflow_v2.py:234-236).
"""
from __future__ import annotations

from dataclasses import dataclass, field, asdict, replace


ROUTER_SOFTMAX = 0
ROUTER_SIGMOID_GROUP = 1


@dataclass(frozen=True)
class MoESpec:
    hidden: int
    n_experts: int
    top_k: int
    inter: int
    bits: int = 4
    group_size: int = 64
    router: str = "softmax"          # "softmax" | "sigmoid_group"
    norm_topk: bool = True
    n_group: int = 1
    topk_group: int = 1
    routed_scaling: float = 1.0
    n_shared: int = 0
    act_dtype: str = "bfloat16"      # activations x / y: "bfloat16" | "float16"
    gate_dtype: str = "float16"      # router weight
    # synthetic-data distribution of the benchmark workloads
    gate_std: float = 0.02
    e_bias_std: float = 0.0
    scale_std: float = 0.02

    @property
    def router_mode(self) -> int:
        return ROUTER_SOFTMAX if self.router == "softmax" else ROUTER_SIGMOID_GROUP

    @property
    def code_mid(self) -> int:
        return 1 << (self.bits - 1)

    @property
    def scale_den(self) -> float:
        return ((1 << self.bits) - 1) / 2.0

    def expert_bytes(self) -> int:
        """Packed codes + fp16 scales + fp16 biases of one routed expert (3 projections)."""
        H, I, b, g = self.hidden, self.inter, self.bits, self.group_size
        codes = 3 * H * I * b // 8
        sb = 3 * H * I // g * 2 * 2
        return codes + sb

    def router_bytes(self) -> int:
        return self.n_experts * self.hidden * 2

    def validate(self) -> None:
        if self.bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        if self.group_size != 64:
            raise ValueError("group_size must be 64")
        for name, v in (("hidden", self.hidden), ("inter", self.inter)):
            if v % 64 != 0:
                raise ValueError(f"{name} must be a multiple of 64")
        if self.router == "sigmoid_group" and self.n_experts % max(1, self.n_group) != 0:
            raise ValueError("n_experts must be divisible by n_group")
        if not (1 <= self.top_k <= 16):
            raise ValueError("top_k must be in 1..16")

    def to_dict(self) -> dict:
        return asdict(self)

    def with_(self, **kw) -> "MoESpec":
        return replace(self, **kw)


# Workloads (synthetic, seeded); names describe the layer shape they model.
MIXTRAL_SMALL = MoESpec(hidden=1024, n_experts=16, top_k=2, inter=2816, bits=4, router="softmax",
                        norm_topk=True, act_dtype="float16")
QWEN3_30B_A3B = MoESpec(hidden=2048, n_experts=128, top_k=8, inter=768, bits=4, router="softmax",
                        norm_topk=True, act_dtype="bfloat16")
DEEPSEEK_V3 = MoESpec(hidden=7168, n_experts=256, top_k=8, inter=2048, bits=4, router="sigmoid_group",
                      norm_topk=True, n_group=8, topk_group=4, routed_scaling=2.5, n_shared=1,
                      act_dtype="bfloat16", e_bias_std=0.01)
DEEPSEEK_V3_PREFILL_8BIT = DEEPSEEK_V3.with_(bits=8, gate_std=0.002)
# The same expert shapes with 32 experts (8 groups of 4): a 1.5 GB layer for
# profiling the prefill kernels on a small case.
DEEPSEEK_V3_8BIT_E32 = DEEPSEEK_V3_PREFILL_8BIT.with_(n_experts=32)

WORKLOADS = {
    "mixtral-small-h1024-e16": MIXTRAL_SMALL,
    "qwen3-30b-a3b-moe": QWEN3_30B_A3B,
    "deepseek-v3-moe": DEEPSEEK_V3,
    "deepseek-v3-moe-8bit": DEEPSEEK_V3_PREFILL_8BIT,
    "deepseek-v3-moe-8bit-e32": DEEPSEEK_V3_8BIT_E32,
}
