"""Generate the golden fixtures in this folder by running the reference itself.

Run from the repository root in a container where the reference checkout is
mounted (it is read, never modified):

    python tests/golden/make_golden.py --reference <path of the reference checkout>

It imports the reference's own torch functions on CPU:

* ``quantize_int8`` / ``dequantize_int8``  reference/page_attention_int8_pytorch.py:23-34
* ``page_attention_reference``             reference/page_attention_reference.py:31-54
* ``QuantizedKVCache``, ``quantized_attention_forward``
                                           tests/qwen_kvcache_full.py:27-113

feeds them the seeded inputs of ``oracle.inputs`` plus hand-made edge cases,
and writes ``*.npz`` fixtures (inputs and reference outputs; large outputs as
SHA-256 digests).  The fixtures travel with the repository; the reference does
not, so tests never import it.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import inputs as oin  # noqa: E402
from oracle import quant as oq  # noqa: E402

TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load_reference(root):
    sys.path.insert(0, os.path.join(root, "reference"))
    sys.path.insert(0, os.path.join(root, "tests"))
    import page_attention_int8_pytorch as pai
    import page_attention_reference as par
    import qwen_kvcache_full as qkf
    return pai, par, qkf


def quant_cases():
    """Edge cases for quantize-on-write, as float32 arrays of ``dtype`` values."""
    rng = np.random.default_rng(1234)
    cases = {}
    cases["small_bf16"] = ("bf16", oin.outlier_k(rng, 2, 3, 37, 128, "bf16"))
    cases["normal_bf16_d64"] = ("bf16", oin.normal(rng, (1, 2, 19, 64), "bf16"))
    cases["normal_bf16_d256"] = ("bf16", oin.normal(rng, (1, 2, 9, 256), "bf16"))
    cases["s1_bf16"] = ("bf16", oin.normal(rng, (2, 2, 1, 128), "bf16"))
    x = np.zeros((1, 2, 5, 128), np.float32)
    cases["zeros"] = ("bf16", x)
    x = oin.normal(rng, (1, 2, 6, 128), "bf16")
    x[0, 0, 2, :] = 0.0            # one all-zero token (V: amax clamped)
    x[0, 1, :, 7] = 0.0            # one all-zero channel (K: amax clamped)
    x[0, 1, 3, 9] = -0.0
    x[0, 0, 4, :5] = -0.0
    cases["zero_rows_and_signed_zero"] = ("bf16", x)
    # exact ties: amax = 127 -> scale = 1 exactly, values k + 0.5 round half to even
    t = np.zeros((1, 1, 4, 128), np.float32)
    ks = np.arange(-126, 127, 2, dtype=np.float32)
    t[0, 0, 0, : ks.size] = ks + 0.5
    t[0, 0, 0, 127] = 127.0
    t[0, 0, 1, : ks.size] = -(ks + 0.5)
    t[0, 0, 1, 127] = -127.0
    t[0, 0, 2, :] = np.linspace(-127, 127, 128, dtype=np.float32)
    t[0, 0, 3, :] = 127.0
    cases["ties"] = ("bf16", oin.cast(t, "bf16"))
    # range extremes: huge (fp16 scale overflows to inf), tiny and subnormal bf16
    e = oin.normal(rng, (1, 2, 8, 128), "f32")
    e[0, 0] *= np.float32(1e37)
    e[0, 1] *= np.float32(1e-39)
    e[0, 1, 3] = 0.0
    cases["extremes_bf16"] = ("bf16", oin.cast(e, "bf16"))
    cases["normal_f16"] = ("f16", oin.cast(oin.normal(rng, (2, 2, 33, 128), "f32") * np.float32(3.0), "f16"))
    cases["outlier_f32"] = ("f32", oin.outlier_k(rng, 1, 2, 65, 128, "f32"))
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of the reference checkout (the directory holding reference/ and tests/)")
    args = ap.parse_args()
    pai, par, qkf = load_reference(args.reference)
    torch.manual_seed(0)

    # 1. quantize_int8 on edge cases: K per channel (dim 2), V per token (dim 3)
    out = {}
    for name, (dt, x) in quant_cases().items():
        xt = torch.from_numpy(x).to(TORCH_DT[dt])
        assert np.array_equal(xt.float().numpy(), x), name
        out[f"{name}/x"] = oq.pack(x, dt)
        out[f"{name}/dtype"] = np.array(dt)
        for tag, dims in (("k", (2,)), ("v", (3,))):
            q, s = pai.quantize_int8(xt, dims)
            out[f"{name}/{tag}_codes"] = q.numpy()
            out[f"{name}/{tag}_scale"] = s.numpy()
            out[f"{name}/{tag}_scale_f16"] = s.to(torch.float16).numpy()
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **out)

    # 2. config 0 at full size (B=1, Hq=16, Hkv=8, S=512, D=128, float32)
    q, k, v = oin.config0(seed=0)
    k_i8, k_sc = pai.quantize_int8(torch.from_numpy(k[0]), (1,))
    v_i8, v_sc = pai.quantize_int8(torch.from_numpy(v[0]), (2,))
    kd, vd = pai.dequantize_int8(k_i8, k_sc), pai.dequantize_int8(v_i8, v_sc)
    att = par.page_attention_reference(torch.from_numpy(q[0])[:, None, :], kd, vd)
    np.savez_compressed(
        os.path.join(HERE, "config0_golden.npz"),
        seed=np.array(0), k_codes_sha=np.array(sha(k_i8.numpy())),
        v_codes_sha=np.array(sha(v_i8.numpy())), k_scale=k_sc.numpy(), v_scale=v_sc.numpy(),
        attn_out=att[:, 0, :].numpy())

    # 3. decode attention on dequantized int8 caches (small shapes, several S)
    dec = {}
    for i, (B, S, dt) in enumerate([(2, 1, "bf16"), (2, 7, "bf16"), (2, 64, "bf16"),
                                    (1, 200, "bf16"), (1, 129, "f16")]):
        c = oin.decode_case(100 + i, B, 16, 8, S, 128, kv_dtype=dt, q_dtype=dt)
        outs = []
        for b in range(B):
            kd = pai.dequantize_int8(torch.from_numpy(c["k_i8"][b]),
                                     torch.from_numpy(c["k_sc"][b]))
            vd = pai.dequantize_int8(torch.from_numpy(c["v_i8"][b]),
                                     torch.from_numpy(c["v_sc"][b]))
            outs.append(par.page_attention_reference(
                torch.from_numpy(c["q"][b])[:, None, :], kd, vd)[:, 0, :].numpy())
        dec[f"case{i}/q"] = oq.pack(c["q"], dt)
        for key in ("k_i8", "k_sc", "v_i8", "v_sc"):
            dec[f"case{i}/{key}"] = c[key]
        dec[f"case{i}/dtype"] = np.array(dt)
        dec[f"case{i}/out"] = np.stack(outs)
    np.savez_compressed(os.path.join(HERE, "decode_golden.npz"), **dec)

    # 4. QuantizedKVCache.update sequence: prefill 40, six 1-token appends, one 3-token append
    rng = np.random.default_rng(77)
    cache = qkf.QuantizedKVCache()
    seq = {}
    steps = [40, 1, 1, 1, 1, 1, 1, 3]
    for i, n in enumerate(steps):
        kx = oin.outlier_k(rng, 2, 2, n, 128, "bf16")
        vx = oin.normal(rng, (2, 2, n, 128), "bf16")
        for layer in (0, 3):
            ko, vo = cache.update(torch.from_numpy(kx).bfloat16(), torch.from_numpy(vx).bfloat16(),
                                  layer)
        seq[f"step{i}/k"] = oq.pack(kx, "bf16")
        seq[f"step{i}/v"] = oq.pack(vx, "bf16")
        seq[f"step{i}/k_out_sha"] = np.array(sha(oq.pack(ko.float().numpy(), "bf16")))
        seq[f"step{i}/v_out_sha"] = np.array(sha(oq.pack(vo.float().numpy(), "bf16")))
    for layer in (0, 3):
        seq[f"layer{layer}/k_i8"] = cache._k_i8[layer].numpy()
        seq[f"layer{layer}/v_i8"] = cache._v_i8[layer].numpy()
        seq[f"layer{layer}/k_sc"] = cache._k_sc[layer].numpy()
        seq[f"layer{layer}/v_sc"] = cache._v_sc[layer].numpy()
    seq["nsteps"] = np.array(len(steps))
    seq["storage_bytes"] = np.array(cache.storage_bytes())
    seq["fp16_equiv_bytes"] = np.array(cache.fp16_equiv_bytes())
    seq["seq_length"] = np.array(cache.get_seq_length(0))
    seq["len"] = np.array(len(cache))
    np.savez_compressed(os.path.join(HERE, "cache_golden.npz"), **seq)

    # 5. whole-model logits: tiny random-init Qwen3 through the reference drop-in (CPU, bf16)
    from transformers import Qwen3ForCausalLM
    from oracle.hf_reference import qwen3_config
    import transformers.models.qwen3.modeling_qwen3 as qwen3_mod
    cfg = qwen3_config(num_layers=2, vocab=1000, hidden=256, heads=4, kv_heads=2,
                       head_dim=128, intermediate=512)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    ids = torch.randint(0, 1000, (1, 28), generator=torch.Generator().manual_seed(5))
    orig = qwen3_mod.eager_attention_forward
    qwen3_mod.eager_attention_forward = qkf.quantized_attention_forward
    try:
        cache = qkf.QuantizedKVCache()
        logits = []
        with torch.no_grad():
            o = model(ids[:, :24], past_key_values=cache, use_cache=True)
            logits.append(o.logits[0, -1].float().numpy())
            for t in range(24, 28):
                o = model(ids[:, t:t + 1], past_key_values=cache, use_cache=True)
                logits.append(o.logits[0, -1].float().numpy())
    finally:
        qwen3_mod.eager_attention_forward = orig
    np.savez_compressed(os.path.join(HERE, "hf_logits.npz"), ids=ids.numpy(),
                        logits=np.stack(logits), prefill=np.array(24))

    with open(os.path.join(HERE, "VERSIONS.txt"), "w") as f:
        import transformers
        f.write(f"torch {torch.__version__}\ntransformers {transformers.__version__}\n"
                f"numpy {np.__version__}\n")
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
