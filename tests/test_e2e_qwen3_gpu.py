"""Whole-model checks: random-init Qwen3 through HF transformers on the GPU.

Ours:   ``QuantizedKVCache`` + ``quantized_attention_forward`` (CUDA kernels).
Oracle: the torch restatement of the reference drop-in
        (``oracle.hf_reference``, tests/qwen_kvcache_full.py:19-113), pinned to
        the reference's own logits by tests/test_oracle_golden.py.
Both see the same weights and the same teacher-forced token stream.

1. Cache parity, end to end: with ``mode="dequant"`` the product returns the
   dequantized cache exactly as the reference does (lines 64-66) and its
   attention evaluates the reference math, so every logit of every step must be
   bit-identical (config 1: 28 layers, prefill 512, 256 decode steps).
2. The fused int8 decode kernel with the int8 cache state shared (config 1:
   28 layers, prefill 512, 256 decode steps, at bf16 and with the model in
   float32).  The reference path, the product and the reference's math
   evaluated in float32 and in float64 (``oracle_attention_f32`` /
   ``oracle_attention_f64``, on the exact dequantized codes) run in lock step
   on the same tokens; after every cache update the others' caches are
   overwritten with the reference path's codes and scales, so every step
   attends over identical int8 state and the reference's +-127 append rule
   (tests/qwen_kvcache_full.py:54) cannot amplify upstream rounding.  The
   product is measured against the float64 evaluation, with torch's own
   float32 evaluation as the yardstick (see the test's docstring for why the
   north star's 1e-2 applies to the first step and to the mean, not to the
   maximum over every step).
3. The fused int8 decode kernel without shared state: prefill logits
   bit-identical; decode logits compared with the reference's own numerical
   noise floor.  The reference
   codes every appended K element as +-127 by sign (tests/qwen_kvcache_full.py:54),
   so the cache - and the logits - respond discontinuously to any rounding
   difference upstream; the oracle evaluated with float32 instead of bf16
   attention arithmetic drifts from itself by ~0.1 after one step and ~1 after
   64 on logits of magnitude ~3.5.  The kernel computes in float32 from the
   int8 codes, so its logits must stay within twice that self-drift.  Its own
   accuracy on identical inputs (1e-3) is tested in tests/test_decode_gpu.py.
"""
import pytest
import torch

from halftone_quantizedkvcache_b200.integration import QuantizedKVCache, installed
from oracle.hf_reference import (OracleQuantizedKVCache, oracle_attention_f32,
                                 oracle_attention_f64, oracle_attention_forward,
                                 patched_attention, qwen3_config)

pytestmark = pytest.mark.gpu


def build(num_layers, vocab=151936, seed=0):
    from transformers import Qwen3ForCausalLM
    cfg = qwen3_config(num_layers=num_layers, vocab=vocab)
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


@torch.no_grad()
def run(model, ids, n_prefill, cache):
    logits = [model(ids[:, :n_prefill], past_key_values=cache, use_cache=True).logits[:, -1]]
    for t in range(n_prefill, ids.shape[1]):
        logits.append(model(ids[:, t:t + 1], past_key_values=cache, use_cache=True).logits[:, -1])
    return torch.stack(logits, 1).float()


def ours(model, ids, n0, mode):
    with installed():
        cache = QuantizedKVCache(mode=mode)
        out = run(model, ids, n0, cache)
    assert cache.get_seq_length(0) == ids.shape[1]
    return out


def oracle(model, ids, n0, fp32_math=False):
    def fwd(*a, **k):
        return oracle_attention_forward(*a, fp32_math=fp32_math, **k)
    with patched_attention(fwd):
        return run(model, ids, n0, OracleQuantizedKVCache())


def tokens(model, batch, n):
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, model.config.vocab_size, (batch, n), generator=g).cuda()


def test_config1_dequant_mode_bit_exact():
    """Config 1: Qwen3-0.6B shape, prefill 512 uniform ids, 256 decode steps."""
    model = build(28)
    ids = tokens(model, 1, 512 + 256)
    a = ours(model, ids, 512, "dequant")
    b = oracle(model, ids, 512)
    assert torch.equal(a, b), float((a - b).abs().max())


class _OursOnSharedState(QuantizedKVCache):
    """The product's cache whose stored codes and scales are replaced, after each
    of its own updates, by those of the reference path's cache (``source``),
    which ran the same step first.  Counts the appended codes that differed."""

    def __init__(self, source):
        super().__init__(mode="fused")
        self.source = source
        self.code_diffs = 0
        self.codes_appended = 0

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        k, v = super().update(key_states, value_states, layer_idx, cache_kwargs)
        st, src = self._store[layer_idx], self.source
        L = st.length
        sk, sv = src._k_i8[layer_idx], src._v_i8[layer_idx]
        assert sk.shape[2] == L
        if key_states.shape[2] == 1:
            self.code_diffs += int((st.k[:, :, L - 1] != sk[:, :, L - 1]).sum())
            self.code_diffs += int((st.v[:, :, L - 1] != sv[:, :, L - 1]).sum())
            self.codes_appended += 2 * sk[:, :, L - 1].numel()
        st.k[:, :, :L].copy_(sk)
        st.v[:, :, :L].copy_(sv)
        st.k_sc.copy_(src._k_sc[layer_idx])
        st.v_sc[:, :, :L].copy_(src._v_sc[layer_idx])
        return k, v


class _F32OnSharedState(OracleQuantizedKVCache):
    """The oracle cache on the reference path's int8 state, returning the exact
    float32 dequantized codes (``code * scale``) for ``oracle_attention_f32``."""

    def __init__(self, source):
        super().__init__()
        self.source = source

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        super().update(key_states, value_states, layer_idx, cache_kwargs)
        for name in ("_k_i8", "_v_i8", "_k_sc", "_v_sc", "_lens"):
            getattr(self, name)[layer_idx] = getattr(self.source, name)[layer_idx]
        return (self._k_i8[layer_idx].float() * self._k_sc[layer_idx].float(),
                self._v_i8[layer_idx].float() * self._v_sc[layer_idx].float())


@torch.no_grad()
def lockstep(model, ids, n0):
    """Reference path, product and the float32 / float64 evaluations of the
    reference's math, step by step on one token stream and one int8 cache state
    (the reference path's)."""
    ref = OracleQuantizedKVCache()
    ours, f32, f64 = _OursOnSharedState(ref), _F32OnSharedState(ref), _F32OnSharedState(ref)
    runs = (("ref", oracle_attention_forward, ref), ("ours", None, ours),
            ("f32", oracle_attention_f32, f32), ("f64", oracle_attention_f64, f64))
    out = {name: [] for name, _, _ in runs}

    def step(sl):
        for name, fn, cache in runs:
            with (installed() if fn is None else patched_attention(fn)):
                out[name].append(model(ids[:, sl], past_key_values=cache,
                                       use_cache=True).logits[:, -1])

    step(slice(0, n0))
    for t in range(n0, ids.shape[1]):
        step(slice(t, t + 1))
    return {k: torch.stack(v, 1).float() for k, v in out.items()}, ours


@pytest.mark.parametrize("precision", ["bf16", "f32"])
def test_config1_fused_decode_logits_on_shared_cache_state(precision):
    """Config 1 (Qwen3-0.6B shape, 28 layers, prefill 512, 256 decode steps) with
    the int8 cache state shared: the decode kernel's logits against the
    reference's attention math evaluated in float64 on the same state.

    The yardstick is the same math evaluated in float32 by torch: on this
    random-init model two correct evaluations of the reference's math already
    differ by up to ~0.05 (bf16 model) / ~0.02 (float32 model) max-abs over the
    39M decode logits - a single last-bit difference in one attention output is
    amplified ~100x by the 28 layers - so a 1e-2 bound on the maximum holds for
    no implementation short of a bit-for-bit replica (the cache's dequant mode,
    test_config1_dequant_mode_bit_exact).  Asserted: the first decode step and
    the mean over every step within 1e-2 (absolute); every step's maximum no
    farther from the float64 evaluation than 1.5x the float32 evaluation's
    (plus 1e-2); the mean no farther than 1.5x (plus 1e-3)."""
    model = build(28)
    if precision == "f32":
        model = model.float()
    ids = tokens(model, 1, 512 + 256)
    lg, ours = lockstep(model, ids, 512)
    assert torch.equal(lg["ours"][:, 0], lg["ref"][:, 0])  # prefill: the reference's own math
    dec = slice(1, None)
    dist = {f"{a}-{b}": (lg[a][:, dec] - lg[b][:, dec]).abs()
            for a, b in (("ours", "f64"), ("f32", "f64"), ("ours", "ref"), ("f32", "ref"))}
    steps_max = dist["ours-f64"].amax(dim=(0, 2))
    print(f"[{precision}] shared state, 256 steps: " + "; ".join(
        f"{k} max {float(v.max()):.4f} mean {float(v.mean()):.5f}" for k, v in dist.items()) +
        f"; steps with ours-f64 max <= 1e-2: {int((steps_max <= 1e-2).sum())}/256"
        f"; appended codes differing before sharing: {ours.code_diffs} of {ours.codes_appended}")
    d, floor = dist["ours-f64"], dist["f32-f64"]
    assert float(d[:, 0].max()) <= 1e-2                     # first decode step
    assert float(d.mean()) <= 1e-2
    assert float(d.max()) <= 1.5 * float(floor.max()) + 1e-2
    assert float(d.mean()) <= 1.5 * float(floor.mean()) + 1e-3


@pytest.mark.parametrize("layers,n0,nd,batch", [(2, 64, 16, 2), (28, 512, 64, 1)])
def test_fused_decode_within_reference_noise(layers, n0, nd, batch):
    model = build(layers)
    ids = tokens(model, batch, n0 + nd)
    a = ours(model, ids, n0, "fused")
    b = oracle(model, ids, n0)
    b32 = oracle(model, ids, n0, fp32_math=True)
    assert torch.equal(a[:, 0], b[:, 0])  # prefill: identical math over the same cache
    err = (a - b).abs()
    floor = (b32 - b).abs()
    print(f"layers={layers}: ours-vs-oracle max {float(err.max()):.4f} mean {float(err.mean()):.5f};"
          f" oracle fp32-vs-bf16 max {float(floor.max()):.4f} mean {float(floor.mean()):.5f}")
    assert float(err.max()) <= 2.0 * float(floor.max()) + 1e-2
    assert float(err.mean()) <= 2.0 * float(floor.mean()) + 1e-3


def test_whole_model_decode_step_as_one_cuda_graph():
    """The full decode step of the model (embedding, every layer's projections,
    RoPE, cache update + int8 attention, MLP, LM head) captured once as a CUDA
    graph over QuantizedKVCache(device_lengths=True, fused_append=True) and
    replayed per token, with the token id and position in static tensors.
    Against the eager fused path on the same teacher-forced tokens: within twice
    the reference's own bf16-vs-float32 drift (the split plan of a replayed step
    is the one planned at capture, so the float32 sums are grouped differently)."""
    layers, n0, nd, batch = 2, 64, 48, 1
    model = build(layers)
    ids = tokens(model, batch, n0 + nd)
    a = ours(model, ids, n0, "fused")
    b = oracle(model, ids, n0)
    b32 = oracle(model, ids, n0, fp32_math=True)
    with torch.no_grad(), installed():
        cache = QuantizedKVCache(mode="fused", capacity=n0 + nd + 256, device_lengths=True,
                                 fused_append=True)
        logits = [model(ids[:, :n0], past_key_values=cache, use_cache=True).logits[:, -1].float()]
        tok = torch.empty((batch, 1), dtype=torch.long, device="cuda")
        pos = torch.empty((batch, 1), dtype=torch.long, device="cuda")
        masks = {"full_attention": None}

        def step():
            return model(input_ids=tok, position_ids=pos, attention_mask=masks,
                         past_key_values=cache, use_cache=True).logits[:, -1]

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            tok.copy_(ids[:, n0:n0 + 1])
            pos.fill_(n0)
            logits.append(step().float())          # eager step: workspaces exist
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                out = step()                       # recorded, not run
            for t in range(n0 + 1, n0 + nd):
                tok.copy_(ids[:, t:t + 1])
                pos.fill_(t)
                g.replay()
                logits.append(out.float().clone())
            torch.cuda.synchronize()
        lens = cache.sync_lengths()
        del g
    assert all(v == n0 + nd for v in lens.values())
    gl = torch.stack(logits, 1)
    err, floor = (gl - a).abs(), (b32 - b).abs()
    print(f"graph-vs-eager max {float(err.max()):.4f} mean {float(err.mean()):.5f}; "
          f"reference drift max {float(floor.max()):.4f} mean {float(floor.mean()):.5f}")
    assert torch.equal(gl[:, 0], a[:, 0])  # prefill: the same eager path
    assert float(err.max()) <= 2.0 * float(floor.max()) + 1e-2
    assert float(err.mean()) <= 2.0 * float(floor.mean()) + 1e-3
