"""MoE layer: host block, expert blocks, pipeline tasks and pools (reference ``MoE/`` API)."""
