"""Block-wise per-channel K layout: the oracle and the rule the kernels rely on (CPU).

* A block that covers the whole write is the reference's per-channel K of that
  write: checked against every golden vector of the reference quantizer.
* The append kernel keeps a block's scale as max(old scale, RN(max|new| / 127))
  instead of re-reading the block; that equals RN(max|all| / 127) because RN is
  monotone.  Checked exhaustively near the rounding boundaries of float32.
* What the layout changes: a decoded token larger than the prefill's column
  maximum is clipped under the reference's retained first scale
  (tests/qwen_kvcache_full.py:54) and is not clipped block-wise.
"""
import numpy as np

from oracle import blockwise as ob
from oracle import quant as oq


def _cases(npz):
    return sorted({k.split("/")[0] for k in npz.files if "/" in k})


def test_single_block_is_the_reference_rule(golden):
    g = golden("quant_golden.npz")
    for name in _cases(g):
        x = oq.unpack(g[f"{name}/x"], str(g[f"{name}/dtype"]))
        for block in (64, 128, 256):
            if x.shape[2] > block:
                continue
            codes, scales = ob.quant_k_blockwise(x, block)
            np.testing.assert_array_equal(codes, g[f"{name}/k_codes"], err_msg=name)
            np.testing.assert_array_equal(scales, g[f"{name}/k_scale"], err_msg=name)


def test_blocks_are_independent_quantizations():
    rng = np.random.default_rng(3)
    x = oq.cast(rng.standard_normal((2, 3, 300, 64)).astype(np.float32) * 3, "bf16")
    codes, scales = ob.quant_k_blockwise(x, 128)
    assert scales.shape == (2, 3, 3, 64)
    for i, (lo, hi) in enumerate(((0, 128), (128, 256), (256, 300))):
        c, s = oq.quantize_int8(x[:, :, lo:hi], (2,))
        np.testing.assert_array_equal(codes[:, :, lo:hi], c)
        np.testing.assert_array_equal(scales[:, :, i], s[:, :, 0])


def _scale(a):
    a = np.maximum(np.asarray(a, np.float32), oq.AMAX_FLOOR)
    return (a / np.float32(127.0)).astype(np.float32)


def test_scale_of_running_max_is_max_of_scales():
    rng = np.random.default_rng(0)
    # values around every power of two and just around the 1e-8 floor, plus bf16 values
    base = np.float32(2.0) ** np.arange(-40, 40, dtype=np.float32)
    ulps = np.arange(-64, 65, dtype=np.int32)
    near = (base.view(np.int32)[:, None] + ulps[None, :]).reshape(-1).view(np.float32)
    floor = (np.float32(1e-8).view(np.int32) + ulps).view(np.float32)
    rand = oq.cast(np.abs(rng.standard_normal(20000)).astype(np.float32) * 50, "bf16")
    vals = np.concatenate([near, floor, rand, np.zeros(4, np.float32)])
    a = vals[rng.integers(0, vals.size, 400000)]
    b = vals[rng.integers(0, vals.size, 400000)]
    np.testing.assert_array_equal(np.maximum(_scale(a), _scale(b)), _scale(np.maximum(a, b)))


def test_blockwise_keeps_a_large_decoded_token():
    rng = np.random.default_rng(1)
    D = 128
    pre = oq.cast(rng.standard_normal((1, 1, 200, D)).astype(np.float32), "bf16")
    new = pre[:, :, :1] * 0
    new[..., 5] = 40.0   # far above the prefill's column maximum
    cache = oq.QuantizedKVCacheOracle()
    cache.update(pre, pre, 0, "f32")
    ref = cache.update(new, new, 0, "f32")[0]
    assert abs(ref[0, 0, -1, 5]) < 10.0   # clipped: 127 * (prefill scale of channel 5)
    seq = np.concatenate([pre, new], axis=2)
    codes, scales = ob.quant_k_blockwise(seq, 128)
    deq = ob.dequant_k_blockwise(codes, scales, 128)
    assert abs(deq[0, 0, -1, 5] - 40.0) < 40.0 / 127


def test_blockwise_decode_oracle_is_the_reference_path_for_one_block():
    """With one block covering the sequence, the block-wise decode oracle is the
    reference path's decode (per-channel K, reference/page_attention_int8_pytorch.py:23-34
    then reference/page_attention_reference.py:31-54), which the golden vectors pin."""
    from oracle import attention as oa
    from oracle import inputs as oin
    c = oin.decode_case(5, 2, 16, 8, 200, 128)
    codes, scales = ob.quant_k_blockwise(c["k"], 256)
    np.testing.assert_array_equal(codes, c["k_i8"])
    np.testing.assert_array_equal(scales, c["k_sc"][:, :, 0:1, :].reshape(scales.shape))
    got = ob.decode_blockwise(c["q"], codes, scales, c["v_i8"], c["v_sc"][..., 0], 256)
    want = oa.decode_int8(c["q"], c["k_i8"], c["k_sc"], c["v_i8"], c["v_sc"], acc="f64")
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)
