"""The static-scale oracle (``oracle.quant.quant_k_static``) against torch on CPU:
the code step of the reference's ``quantize_int8``
(reference/page_attention_int8_pytorch.py:23-30 - ``clamp(round(x / scale), -127, 127)``
with IEEE float32 division and round half to even) with the scale given."""
import numpy as np
import torch

from oracle import inputs as oin
from oracle import quant as oq


def torch_rule(x, s):
    return torch.clamp(torch.round(torch.from_numpy(x) / torch.from_numpy(s)), -127, 127).to(torch.int8).numpy()


def test_static_codes_match_torch_rule():
    rng = np.random.default_rng(0)
    x = oin.outlier_k(rng, 2, 3, 257, 64, "f32")
    s = (np.abs(x).max(axis=(0, 2), keepdims=True) / np.float32(127) * np.float32(0.6)).astype(np.float32)
    q = oq.quant_k_static(x, s)
    np.testing.assert_array_equal(q, torch_rule(x, np.broadcast_to(s, x.shape).copy()))
    assert (np.abs(q) == 127).mean() > 0.001  # the 0.6 scale makes outliers clamp


def test_static_codes_ties_round_half_even():
    s = np.full((1, 1, 1, 4), 0.25, np.float32)
    x = np.array([0.625, 0.875, -0.625, -0.125], np.float32).reshape(1, 1, 1, 4)  # 2.5, 3.5, -2.5, -0.5
    np.testing.assert_array_equal(oq.quant_k_static(x, s).ravel(), [2, 4, -2, 0])
    np.testing.assert_array_equal(oq.quant_k_static(x, s), torch_rule(x, np.broadcast_to(s, x.shape).copy()))
