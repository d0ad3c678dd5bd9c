"""Shapes of the MoE stacks the routed-expert FFN is measured on.

Each entry is the routed-expert geometry of a public model family, with the
expert weight formats of the GGUF quantizations named beside it. Record bytes
follow the reference's pack layout: one record per (layer, expert) holding the
down, gate and up matrices in that order, padded to 16 KiB
(scripts/moe-profile.py:116-211, src/h4/h4-metal-arena-probe.cpp:143-145).
"""
from __future__ import annotations

from dataclasses import dataclass

from ._lib import ACT_SWIGLU, ACT_SWIGLU_OAI, TYPE_IQ1_S, TYPE_MXFP4, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, row_bytes

RECORD_ALIGN = 16384


@dataclass(frozen=True)
class ModelShape:
    name: str
    layers: int
    hidden: int
    experts: int
    used: int
    intermediate: int
    type_gate: int
    type_up: int
    type_down: int
    act: int = ACT_SWIGLU
    alpha: float = 1.702
    limit: float = 7.0
    seed: int = 0
    shared_experts: int = 0
    shared_type: int = TYPE_Q4_K

    @property
    def down_bytes(self) -> int:
        return row_bytes(self.type_down, self.intermediate) * self.hidden

    @property
    def gate_bytes(self) -> int:
        return row_bytes(self.type_gate, self.hidden) * self.intermediate

    @property
    def up_bytes(self) -> int:
        return row_bytes(self.type_up, self.hidden) * self.intermediate

    @property
    def record_raw(self) -> int:
        return self.down_bytes + self.gate_bytes + self.up_bytes

    @property
    def record(self) -> int:
        return (self.record_raw + RECORD_ALIGN - 1) // RECORD_ALIGN * RECORD_ALIGN

    @property
    def off_gate(self) -> int:
        return self.down_bytes

    @property
    def off_up(self) -> int:
        return self.down_bytes + self.gate_bytes

    def with_layers(self, layers: int) -> "ModelShape":
        return ModelShape(**{**self.__dict__, "layers": layers})

    def with_experts(self, experts: int) -> "ModelShape":
        return ModelShape(**{**self.__dict__, "experts": experts})


MODELS = {
    # OLMoE-1B-7B: Q4_K gate/up, Q6_K down, SwiGLU
    "olmoe": ModelShape("olmoe-1b-7b", 16, 2048, 64, 8, 1024, TYPE_Q4_K, TYPE_Q4_K, TYPE_Q6_K, seed=0),
    # Qwen3-30B-A3B: Q8_0 experts, SwiGLU
    "qwen3-30b": ModelShape("qwen3-30b-a3b", 48, 2048, 128, 8, 768, TYPE_Q8_0, TYPE_Q8_0, TYPE_Q8_0, seed=1),
    # gpt-oss-120b: MXFP4 experts, clamped SwiGLU (alpha 1.702, limit 7.0)
    "gpt-oss-120b": ModelShape("gpt-oss-120b", 36, 2880, 128, 4, 2880, TYPE_MXFP4, TYPE_MXFP4, TYPE_MXFP4,
                               act=ACT_SWIGLU_OAI, seed=2),
    # Qwen3-235B-A22B Q4_K_M mix: Q4_K gate/up, Q6_K down
    "qwen3-235b": ModelShape("qwen3-235b-a22b", 94, 4096, 128, 8, 1536, TYPE_Q4_K, TYPE_Q4_K, TYPE_Q6_K, seed=3),
    # DeepSeek-V3 1.5-bit: IQ1_S routed experts, one Q4_K shared expert
    "deepseek-v3": ModelShape("deepseek-v3", 58, 7168, 256, 8, 2048, TYPE_IQ1_S, TYPE_IQ1_S, TYPE_IQ1_S, seed=4,
                              shared_experts=1, shared_type=TYPE_Q4_K),
}
