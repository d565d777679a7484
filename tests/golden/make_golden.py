"""Generate the golden fixtures in this directory by running the REFERENCE implementation.

Run once in a checkout that has the reference repository (Yevsquant/cuda-PA-INT8) at
$PA_REFERENCE_DIR (default: /root/reference); the fixtures are committed and the tests only
read them. Inputs come from oracle/gen.py (deterministic); each fixture stores a sha256 of
its inputs so a generator drift is detected rather than silently absorbed.

Reference functions exercised (all on CPU, torch):
  tests/paged_decode_attn.py: quantize_per_token, quantize_per_tensor, dequantize_kv,
                              paged_decode_attention_reference
  benchmarks/int8_bridge/paged_cache.py: PagedKVCache.prefill / decode_append
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("PA_REFERENCE_DIR", "/root/reference")
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REF, "tests"))
sys.path.insert(0, os.path.join(REF, "benchmarks", "int8_bridge"))

import gen  # noqa: E402
import pa_oracle  # noqa: E402
from paged_decode_attn import (  # noqa: E402
    dequantize_kv,
    paged_decode_attention_reference,
    quantize_per_tensor,
    quantize_per_token,
)
from paged_cache import PagedKVCache  # noqa: E402


def _bf16_bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def scale_tables():
    # Every positive finite fp16 / bf16 amax (plus 0) through the reference scale formula.
    f16_bits = np.arange(0, 0x7C00, dtype=np.uint16)
    x = torch.zeros(len(f16_bits), 2, dtype=torch.float16)
    x[:, 0] = torch.from_numpy(f16_bits.view(np.float16).copy())
    _, s16 = quantize_per_token(x, dim=-1)
    bf_bits = np.arange(0, 0x7F80, dtype=np.uint16)
    xb = torch.zeros(len(bf_bits), 2, dtype=torch.bfloat16)
    xb[:, 0] = torch.from_numpy(bf_bits.astype(np.int16)).view(torch.bfloat16)
    _, sbf = quantize_per_token(xb, dim=-1)
    np.savez_compressed(os.path.join(HERE, "scale_tables.npz"),
                        f16_bits=f16_bits, f16_scale=s16.numpy(),
                        bf16_bits=bf_bits, bf16_scale=sbf.numpy())


def edge_rows_f16():
    rows = []
    rows.append(np.zeros(128))                                   # all zero -> scale 0
    r = np.zeros(128); r[:4] = [2.0**-24, 0, -2.0**-24, 3 * 2.0**-24]
    rows.append(r)                                               # subnormal -> scale 0
    r = np.zeros(128); r[0] = 65504.0; r[1] = -65504.0; r[2] = 1.0
    rows.append(r)                                               # fp16 max
    r = np.zeros(128); r[0] = 127.0
    r[1:9] = [0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5]
    rows.append(r)                                               # exact ties, scale 1
    r = -np.abs(np.linspace(0.01, 3.0, 128)); rows.append(r)     # all negative
    r = np.linspace(-1, 1, 128); r[7] = 1000.0; rows.append(r)   # single outlier
    r = np.full(128, 1e-3); rows.append(r)                       # constant row
    r = np.zeros(128); r[5] = np.inf; r[6] = 1.0; rows.append(r)  # inf -> scale inf, q 0
    return np.stack(rows).astype(np.float16)


def quant_rows():
    g = gen.Gen(11)
    rnd = gen.kv_values(g, (64, 1, 128), "normal")[:, 0].astype(np.float16)
    out = gen.kv_values(g, (64, 2, 128), "lognormal_outlier").reshape(128, 128)
    x16 = np.concatenate([edge_rows_f16(), rnd, out.astype(np.float16)])
    q16, s16 = quantize_per_token(torch.from_numpy(x16), dim=-1)
    # fp32 rows: random, zero, tiny (clamped by 1e-8)
    x32 = np.concatenate([gen.kv_values(g, (32, 1, 128), "normal")[:, 0],
                          np.zeros((1, 128), np.float32),
                          np.full((1, 128), 1e-12, np.float32)]).astype(np.float32)
    q32, s32 = quantize_per_token(torch.from_numpy(x32), dim=-1)
    # bf16 rows
    xb = torch.from_numpy(np.concatenate([gen.kv_values(g, (32, 1, 128), "normal")[:, 0],
                                          np.zeros((1, 128), np.float32)])).to(torch.bfloat16)
    qb, sb = quantize_per_token(xb, dim=-1)
    # per-tensor
    xt = gen.kv_values(g, (2, 5, 2, 128), "lognormal_outlier").astype(np.float16)
    qt, st = quantize_per_tensor(torch.from_numpy(xt))
    qz, sz = quantize_per_tensor(torch.zeros(3, 128, dtype=torch.float16))
    np.savez_compressed(os.path.join(HERE, "quant_rows.npz"),
                        x16=x16, q16=q16.numpy(), s16=s16.numpy(),
                        x32=x32, q32=q32.numpy(), s32=s32.numpy(),
                        xbf16_bits=_bf16_bits(xb), qbf16=qb.numpy(), sbf16=sb.numpy(),
                        xt=xt, qt=qt.numpy(), st=np.float32(st.item()),
                        qz=qz.numpy(), sz=np.float32(sz.item()))


def cfg1_case():
    """4 seqs, 12/2 heads, D 128, bs 16, ctx U[64,512], 256-block pool."""
    g = gen.Gen(1)
    lens = g.randint(64, 513, (4,))
    return gen.decode_case(seed=101, num_seqs=4, num_heads=12, num_kv_heads=2,
                           context_lens=lens, num_blocks=256), lens


def decode_cfg1():
    c, _ = cfg1_case()
    q, k, v, lens, bt, nb = (c["q"], c["k"], c["v"], c["context_lens"], c["block_table"],
                             c["num_blocks"])
    kc, vc = pa_oracle.scatter_paged_cache(k, v, lens, bt, nb)
    tq = torch.from_numpy(q).float()
    tbt, tl = torch.from_numpy(bt), torch.from_numpy(lens)
    out16 = paged_decode_attention_reference(tq, torch.from_numpy(kc).float(),
                                             torch.from_numpy(vc).float(), tbt, tl)
    res = dict(input_sha=gen.sha256_arrays(q, k, v, lens, bt), out_f16=out16.numpy())
    for mode in ("per_token", "per_tensor"):
        tk, tv = torch.from_numpy(k), torch.from_numpy(v)
        if mode == "per_token":
            kq, ks = quantize_per_token(tk, dim=-1)
            vq, vs = quantize_per_token(tv, dim=-1)
        else:
            kq, ks0 = quantize_per_tensor(tk)
            vq, vs0 = quantize_per_tensor(tv)
            ks = ks0.expand(tk.shape[:-1]).contiguous()
            vs = vs0.expand(tv.shape[:-1]).contiguous()
        kc8, vc8 = pa_oracle.scatter_paged_cache(kq.numpy(), vq.numpy(), lens, bt, nb)
        kss = pa_oracle.scatter_scales(ks.numpy(), lens, bt, nb, 2)
        vss = pa_oracle.scatter_scales(vs.numpy(), lens, bt, nb, 2)
        kd, vd = dequantize_kv(torch.from_numpy(kc8), torch.from_numpy(vc8),
                               torch.from_numpy(kss), torch.from_numpy(vss))
        out8 = paged_decode_attention_reference(tq, kd, vd, tbt, tl)
        res[f"out_{mode}"] = out8.numpy()
        res[f"kq_{mode}_sha"] = gen.sha256_arrays(kq.numpy(), vq.numpy(), ks.numpy(), vs.numpy())
    np.savez_compressed(os.path.join(HERE, "decode_cfg1.npz"), **res)


def bridge_cache():
    g = gen.Gen(7)
    L = 20
    k = gen.kv_values(g, (L, 2, 128), "lognormal_outlier").astype(np.float16)
    v = gen.kv_values(g, (L, 2, 128), "normal").astype(np.float16)
    res = dict(k=k, v=v)
    for variant in ("fp16", "int8_per_token", "int8_per_tensor"):
        c = PagedKVCache(num_layers=1, num_kv_heads=2, head_dim=128, max_len=40, block_size=16,
                         x=8, variant=variant, device="cpu")
        c.prefill(0, torch.from_numpy(k[:-1]), torch.from_numpy(v[:-1]))
        n = c.decode_append(0, torch.from_numpy(k[-1]), torch.from_numpy(v[-1]))
        assert n == L
        res[f"{variant}_k"] = c.k_cache[0].numpy()
        res[f"{variant}_v"] = c.v_cache[0].numpy()
        if c.is_int8:
            res[f"{variant}_ks"] = c.k_scales[0].numpy()
            res[f"{variant}_vs"] = c.v_scales[0].numpy()
    np.savez_compressed(os.path.join(HERE, "bridge_cache.npz"), **res)


if __name__ == "__main__":
    torch.manual_seed(0)
    scale_tables()
    quant_rows()
    decode_cfg1()
    bridge_cache()
    print("golden fixtures written to", HERE)
