"""Attention entry point of the IMI path (attn_hub/sparse_imi.py:1-10)."""


def imi_decode_attn(query_states, key_states, value_states, layer_idx, imi_cache):
    """query_states: [batch_size, 1, num_heads, head_dim] CUDA tensor.

    ``key_states`` / ``value_states`` are the ``(None, None)`` that
    ``decode_update_kv_cache`` returns.  The steady-zone length counts the token
    appended this step: for every layer but the last, ``static_pattern_total``
    has not yet been advanced, hence the ``+ 1``.
    """
    static_len = (
        imi_cache.static_pattern_total
        if layer_idx == imi_cache.layer_num - 1
        else imi_cache.static_pattern_total + 1
    )
    return imi_cache.attn_func(query_states.contiguous(), layer_idx, static_len)
