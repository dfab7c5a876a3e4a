def launch_gdn(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
    """gdn_decode_qk4_v8_d128_k_last with the reference plugin's signature and
    destination-passing semantics (decode ``kernel.cu:982-994``): overwrites
    ``output`` and ``new_state`` on the current torch stream, returns them."""
    t = [_tensor(x) for x in (q, k, v, state, A_log, a, dt_bias, b, output, new_state)]
    return package().decode.launch_gdn(*t[:8], _scale(scale), t[8], t[9])
