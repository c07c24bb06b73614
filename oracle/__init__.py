"""CPU oracle for the gated causal attention block -- test infrastructure only.

Nothing in ``memory_efficient_attn_layer_b200`` imports this package.
"""
