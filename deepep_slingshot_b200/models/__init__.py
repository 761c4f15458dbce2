from .moe import MoEFFN, moe_reference
