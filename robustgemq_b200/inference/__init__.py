"""Drop-in for ``gemq.inference``: the quantized MoE module API (``moe_block``) and the
model patching of ``gemq.inference.patch`` (``patch``, with ``QuantLinear`` for the
non-expert linears)."""

from .linear import QuantLinear  # noqa: F401
from .moe_block import (  # noqa: F401
    QuantFusedDeepseekV2MoEBlock,
    QuantFusedMixtralMoEBlock,
    QuantFusedOlmoeMoEBlock,
    QuantFusedQwen3MoeMoEBlock,
    check_deepseek_gate_matches,
    check_deepseek_routing_supported,
    check_w1_w3_aligned,
    deepseek_group_routing,
)
