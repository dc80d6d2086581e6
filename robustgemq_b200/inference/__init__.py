"""Drop-in for ``gemq.inference``: the quantized MoE module API."""

from .moe_block import (  # noqa: F401
    QuantFusedDeepseekV2MoEBlock,
    QuantFusedMixtralMoEBlock,
    QuantFusedOlmoeMoEBlock,
    QuantFusedQwen3MoeMoEBlock,
    check_deepseek_gate_matches,
    check_deepseek_routing_supported,
    check_w1_w3_aligned,
)
