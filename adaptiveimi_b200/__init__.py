"""B200-native (sm_100a) implementation of AdaptiveIMI's inverted-multi-index
KV-cache path: device index build, decode-time append and cell assignment,
cell retrieval and sparse decode attention, behind the reference's
``adpimi_cache`` / ``imi_decode_attn`` API.
"""
__all__ = ["ops", "sizing", "synthetic"]
