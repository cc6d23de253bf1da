"""CPU oracle for the Halftone int8 KV-cache hot paths.

TEST INFRASTRUCTURE ONLY. The product (``halftone_quantizedkvcache_b200``)
never imports this package. Only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and
only as the checker or as the timed CPU baseline.

The oracle restates, in numpy, the reference algorithm of the two hot paths
of ChaoyuWang04/Halftone_QuantizedKVCache:

* ``oracle.quant``     symmetric int8 quantize-on-write (K per-channel,
  V per-token) and the ``QuantizedKVCache.update`` storage rule
  (reference/page_attention_int8_pytorch.py:23-34,
  tests/qwen_kvcache_full.py:38-89);
* ``oracle.attention`` decode attention over dequantized K/V
  (reference/page_attention_reference.py:23-54,
  src/kernels/int8_decode_attn_triton.py:15-63) and the split-KV
  log-sum-exp combine used to check sharded decode;
* ``oracle.hf_reference`` the torch restatement of the reference's HF drop-in
  (``QuantizedKVCache`` and ``quantized_attention_forward``,
  tests/qwen_kvcache_full.py:19-113), used to check whole-model logits;
* ``oracle.inputs`` seeded synthetic inputs with the shapes and value
  distributions of the workloads (K with outlier channels, V ~ N(0, 1)).

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
torch functions on CPU and stores their outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this oracle against them bit-exactly
(codes, scales) or to float32 round-off (attention).
"""
