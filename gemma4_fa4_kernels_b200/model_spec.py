"""Gemma-4 31B attention geometry (the contract every kernel call is checked against).

The field names and values are kept identical to the reference contract
(``src/gemma4_fa4/model_spec.py:18-122``) so that specs built for the
reference can be passed to these adapters unchanged: local sliding layers are
d256 with 32 query / 16 KV heads and a 1024-token window; every sixth layer is
global causal d512 with 32 query / 4 KV heads; the softmax scale is 1.0.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

LayerKind = Literal["sliding_attention", "full_attention"]


@dataclass(frozen=True)
class AttentionLayerSpec:
    kind: LayerKind
    head_dim_qk: int
    head_dim_v: int
    num_q_heads: int
    num_kv_heads: int
    softmax_scale: float
    is_causal: bool
    vision_bidirectional_within_block: bool
    sliding_window: int | None
    rope_type: str
    rope_theta: float
    partial_rotary_factor: float
    projection_source_shared_between_k_and_v: bool

    @property
    def qhead_per_kvhead(self) -> int:
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        return self.num_q_heads // self.num_kv_heads

    @property
    def rotary_dim(self) -> int:
        value = self.head_dim_qk * self.partial_rotary_factor
        if int(value) != value:
            raise ValueError("rotary dimension must be integral")
        return int(value)

    @property
    def fa_window_size_left(self) -> int | None:
        """Inclusive left window (W - 1) in flash-attention terms."""
        return None if self.sliding_window is None else self.sliding_window - 1

    def head_partition(self, world_size: int, rank: int) -> "AttentionLayerSpec":
        """Spec of one rank's share when query heads (with their KV group) are
        split over ``world_size`` GPUs.  KV heads are split when there are at
        least as many KV heads as ranks; otherwise ranks share a KV head."""
        from dataclasses import replace

        if self.num_q_heads % world_size:
            raise ValueError("query heads must divide evenly over the ranks")
        if not 0 <= rank < world_size:
            raise ValueError("rank out of range")
        q = self.num_q_heads // world_size
        kv = max(1, self.num_kv_heads // world_size) if self.num_kv_heads >= world_size else 1
        return replace(self, num_q_heads=q, num_kv_heads=kv)


@dataclass(frozen=True)
class Gemma4ModelSpec:
    model_id: str
    revision: str
    hidden_size: int
    num_hidden_layers: int
    max_position_embeddings: int
    num_kv_shared_layers: int
    use_bidirectional_attention: str
    sliding: AttentionLayerSpec
    full: AttentionLayerSpec

    def layer_types(self) -> tuple[LayerKind, ...]:
        return tuple("full_attention" if (i + 1) % 6 == 0 else "sliding_attention"
                     for i in range(self.num_hidden_layers))

    def spec_for_layer(self, layer_idx: int) -> AttentionLayerSpec:
        if not 0 <= layer_idx < self.num_hidden_layers:
            raise IndexError(layer_idx)
        return self.full if self.layer_types()[layer_idx] == "full_attention" else self.sliding

    @property
    def first_kv_shared_layer_idx(self) -> int:
        return self.num_hidden_layers - self.num_kv_shared_layers


SLIDING_ATTENTION = AttentionLayerSpec(
    kind="sliding_attention", head_dim_qk=256, head_dim_v=256, num_q_heads=32, num_kv_heads=16,
    softmax_scale=1.0, is_causal=True, vision_bidirectional_within_block=True,
    sliding_window=1024, rope_type="default", rope_theta=10_000.0, partial_rotary_factor=1.0,
    projection_source_shared_between_k_and_v=False,
)

GLOBAL_ATTENTION = AttentionLayerSpec(
    kind="full_attention", head_dim_qk=512, head_dim_v=512, num_q_heads=32, num_kv_heads=4,
    softmax_scale=1.0, is_causal=True, vision_bidirectional_within_block=False,
    sliding_window=None, rope_type="proportional", rope_theta=1_000_000.0,
    partial_rotary_factor=0.25, projection_source_shared_between_k_and_v=True,
)

GEMMA4_31B = Gemma4ModelSpec(
    model_id="google/gemma-4-31B", revision="2d418d1b7ed8c04d732c3359e19a11fbc85b6842",
    hidden_size=5376, num_hidden_layers=60, max_position_embeddings=262_144,
    num_kv_shared_layers=0, use_bidirectional_attention="vision",
    sliding=SLIDING_ATTENTION, full=GLOBAL_ATTENTION,
)
