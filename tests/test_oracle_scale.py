"""The oracle's scale rule is the reference's: only None or 0 selects 1/sqrt(128)
(decode reference_torch_impl.py:32-33, prefill :31-32); negative scales pass through."""
import torch


def test_negative_scale_passes_through(orc, pkg):
    d = pkg.inputs.make_decode_inputs(2, seed=3)
    d.scale = -0.3
    neg, _ = orc.decode(*d.args())
    d.scale = 0.3
    pos, _ = orc.decode(*d.args())
    torch.testing.assert_close(neg, -pos, atol=0, rtol=0)
    d.scale = None
    dflt, _ = orc.decode(*d.args())
    d.scale = 0.0
    zero, _ = orc.decode(*d.args())
    torch.testing.assert_close(dflt, zero, atol=0, rtol=0)
