def launch_gdn(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output=None, new_state=None):
    """gdn_prefill_qk4_v8_d128_k_last with the reference plugin's signature and
    destination-passing semantics (prefill ``kernel.py:56-57``; ``state``,
    ``output`` and ``new_state`` may be None): writes ``output`` and
    ``new_state`` on the current torch stream, returns ``(output, new_state)``."""
    t = [_tensor(x) for x in (q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state)]
    return package().prefill.launch_gdn(*t[:9], _scale(scale), t[9], t[10])
