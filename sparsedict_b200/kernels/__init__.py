"""Reference-compatible modules: ``fused_topk_attn`` and ``hybrid_topk``."""
