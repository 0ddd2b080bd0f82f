"""Generate golden vectors from the reference's own CUDA ops (run on a B200).

The reference ops are the four PaceServe extensions compiled from their
sources into ``oracle/_ref`` (``oracle/build_ref.py``).  Each case stores small
seeded inputs and the reference op's outputs as ``<name>.npz`` (inputs of a
16-bit dtype are stored as fp32 values that are exactly representable in it).
``tests/test_oracle.py`` checks the CPU oracle against every file.

Usage (GPU box):  python tests/golden/make_golden.py [out_dir]
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.build_ref import load_ref_ops  # noqa: E402

DEV = "cuda:0"


def f32(t):
    return t.detach().float().cpu().numpy()


def main(out_dir):
    os.makedirs(out_dir, exist_ok=True)
    ln, pe, act, moe = (load_ref_ops(n) for n in
                        ("layernorm_ops", "pos_encoding_ops", "activation_ops", "moe_ops"))
    if None in (ln, pe, act, moe):
        raise SystemExit("reference ops not built under oracle/_ref")
    g = torch.Generator().manual_seed(1234)
    n = 0

    def save(name, **kw):
        nonlocal n
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), **kw)
        n += 1

    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        dn = str(dtype).split(".")[1]
        x = torch.randn(5, 320, generator=g).to(dtype)
        w = (torch.randn(320, generator=g) * 0.02 + 1).to(dtype)
        out = torch.empty(5, 320, dtype=dtype, device=DEV)
        ln.rms_norm(out, x.to(DEV), w.to(DEV), 1e-5)
        save(f"rms_norm_{dn}", op="rms_norm", dtype=dn, x=f32(x), w=f32(w), eps=1e-5,
             ref_out=f32(out))

        x = (torch.randn(4, 2 * 384, generator=g) * 3).to(dtype)
        out = torch.empty(4, 384, dtype=dtype, device=DEV)
        act.silu_and_mul(out, x.to(DEV))
        save(f"silu_and_mul_{dn}", op="silu_and_mul", dtype=dn, x=f32(x), ref_out=f32(out))

        for name in ("gelu_new", "gelu_fast"):
            x = (torch.randn(4, 512, generator=g) * 3).to(dtype)
            out = torch.empty(4, 512, dtype=dtype, device=DEV)
            getattr(act, name)(out, x.to(DEV))
            save(f"{name}_{dn}", op=name, dtype=dn, x=f32(x), ref_out=f32(out))

        for neox in (True, False):
            T, nq, nkv, hd = 6, 4, 2, 128
            q = torch.randn(T, nq * hd, generator=g).to(dtype)
            k = torch.randn(T, nkv * hd, generator=g).to(dtype)
            inv = 1.0 / (500000.0 ** (torch.arange(0, hd, 2, dtype=torch.float) / hd))
            freqs = torch.einsum("i,j->ij", torch.arange(64, dtype=torch.float), inv)
            cache = torch.cat((freqs.cos(), freqs.sin()), -1).to(dtype)  # reference: cache dtype == q dtype
            pos = torch.randint(0, 64, (T,), generator=g)
            qd, kd = q.to(DEV), k.to(DEV)
            pe.rotary_embedding(pos.to(DEV), qd, kd, hd, cache.to(DEV), neox)
            save(f"rotary_embedding_{'neox' if neox else 'gptj'}_{dn}", op="rotary_embedding",
                 dtype=dn, q=f32(q), k=f32(k), cache=f32(cache), positions=pos.numpy(),
                 head_size=hd, is_neox=neox, ref_q=f32(qd), ref_k=f32(kd))

    for T, E, k in ((256, 8, 2), (64, 16, 4), (32, 256, 8), (48, 60, 3)):
        gating = torch.randn(T, E, generator=g)
        gating[0, :] = 0.0  # an all-tie row
        w = torch.empty(T, k, device=DEV)
        i = torch.empty(T, k, dtype=torch.int32, device=DEV)
        t = torch.empty(T, k, dtype=torch.int32, device=DEV)
        moe.topk_softmax(w, i, t, gating.to(DEV))
        save(f"topk_softmax_T{T}_E{E}_k{k}", op="topk_softmax", gating=gating.numpy(), k=k,
             ref_weights=w.cpu().numpy(), ref_ids=i.cpu().numpy(), ref_tei=t.cpu().numpy())

    for numel, E, bs in ((9, 5, 4), (512, 8, 64), (1000, 8, 16), (700, 64, 16)):
        ids = torch.randint(0, E, (numel,), generator=g, dtype=torch.int32)
        if numel == 9:
            ids = torch.tensor([0, 1, 2, 1, 2, 3, 0, 3, 4], dtype=torch.int32)
        cap = numel + E * (bs - 1)
        s = torch.full((cap,), numel, dtype=torch.int32, device=DEV)
        e = torch.full(((cap + bs - 1) // bs,), -1, dtype=torch.int32, device=DEV)
        tot = torch.empty(1, dtype=torch.int32, device=DEV)
        moe.moe_align_block_size(ids.to(DEV), E, bs, s, e, tot)
        save(f"moe_align_block_size_n{numel}_E{E}_bs{bs}", op="moe_align_block_size",
             topk_ids=ids.numpy(), E=E, bs=bs, ref_sorted=s.cpu().numpy(),
             ref_expert_ids=e.cpu().numpy(), ref_total=int(tot.item()))
    print(f"wrote {n} golden files to {out_dir}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
