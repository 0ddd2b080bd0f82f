"""Time the reference's own CUDA ops (built from its sources into oracle/_ref)
against this package's kernels on the bench's op chain, on one B200.

TEST / MEASUREMENT INFRASTRUCTURE ONLY: it runs the reference as a
comparison point and never feeds the product.

The reference chain is what PaceServe runs today (models/llama.py:232-255):
rms_norm, rotary_embedding with the cache in the model dtype (the reference
requires it, rotary_embedding.py:53), a PyTorch residual add followed by
rms_norm where this package has fused_add_rms_norm, and silu_and_mul.
Each op is also timed alone (a CUDA graph of its 32 launches over the 32
layers' distinct buffers, so every launch reads cold data).

Usage (GPU box): python oracle/compare_ref_cuda.py [--out file.json]
"""
import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from oracle.build_ref import load_ref_ops  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    ap.add_argument("--reps", type=int, default=50)
    args = ap.parse_args()
    import paceserve_b200 as pb

    dev = torch.device("cuda:0")
    ln_r, pe_r, act_r = (load_ref_ops(n) for n in ("layernorm_ops", "pos_encoding_ops", "activation_ops"))
    if None in (ln_r, pe_r, act_r):
        raise SystemExit("reference ops not built")
    ch = bench.build_chain(dev, seed=7)
    H, HD, EPS = bench.H, bench.HD, bench.EPS
    cache_bf16 = ch["cache"].to(torch.bfloat16)
    lay = ch["layers"]
    pos = ch["positions"]
    for b in lay:
        b.setdefault("normed", torch.empty(bench.T, H, dtype=torch.bfloat16, device=dev))
        b["res_sum"] = torch.empty(bench.T, H, dtype=torch.bfloat16, device=dev)

    def ref_chain():
        for l, b in enumerate(lay):
            if l == 0:
                ln_r.rms_norm(b["normed"], b["hidden"], b["w_in"], EPS)
            else:  # residual + hidden, then RMSNorm (llama.py:248-252)
                torch.add(b["hidden"], b["residual"], out=b["res_sum"])
                ln_r.rms_norm(b["normed"], b["res_sum"], b["w_in"], EPS)
            pe_r.rotary_embedding(pos, b["q"], b["k"], HD, cache_bf16, True)
            torch.add(b["attn"], b["residual2"], out=b["res_sum"])
            ln_r.rms_norm(b["normed"], b["res_sum"], b["w_post"], EPS)
            act_r.silu_and_mul(b["act"], b["gate_up"])

    ours = (pb.layernorm_ops, pb.pos_encoding_ops, pb.activation_ops)
    res = {}
    for name, fn in (("ours", lambda: bench.run_chain(ch, ours)), ("reference_cuda", ref_chain)):
        g = bench.capture(fn)
        ms = bench.time_replays(g, args.reps, 5) / args.reps
        res[name] = {"ms_per_step": round(ms, 4), "tokens_per_s": round(bench.T / (ms * 1e-3), 1)}
        del g
    # Decode-sized batches: the same 32-layer chain at T = 1, 16 and 64 decode tokens.
    decode = []
    for t in (1, 16, 64):
        dch = bench.build_chain(dev, seed=8, tokens=t)
        dl, dpos = dch["layers"], dch["positions"]
        for b in dl:
            b.setdefault("normed", torch.empty(t, H, dtype=torch.bfloat16, device=dev))
            b["res_sum"] = torch.empty(t, H, dtype=torch.bfloat16, device=dev)

        def ref_decode():
            for l, b in enumerate(dl):
                if l == 0:
                    ln_r.rms_norm(b["normed"], b["hidden"], b["w_in"], EPS)
                else:
                    torch.add(b["hidden"], b["residual"], out=b["res_sum"])
                    ln_r.rms_norm(b["normed"], b["res_sum"], b["w_in"], EPS)
                pe_r.rotary_embedding(dpos, b["q"], b["k"], HD, cache_bf16, True)
                torch.add(b["attn"], b["residual2"], out=b["res_sum"])
                ln_r.rms_norm(b["normed"], b["res_sum"], b["w_post"], EPS)
                act_r.silu_and_mul(b["act"], b["gate_up"])

        row = {"T": t}
        for name, fn in (("ours", lambda: bench.run_chain(dch, ours)), ("reference_cuda", ref_decode)):
            g = bench.capture(fn)
            row[name + "_us_per_step"] = round(bench.time_replays(g, args.reps, 5) * 1e3 / args.reps, 2)
            del g
        row["speedup"] = round(row["reference_cuda_us_per_step"] / row["ours_us_per_step"], 2)
        decode.append(row)
        del dch
    res["decode_chain"] = decode
    single = {
        "rms_norm": (lambda: [ln_r.rms_norm(b["normed"], b["hidden"], b["w_in"], EPS) for b in lay],
                     lambda: [pb.layernorm_ops.rms_norm(b["normed"], b["hidden"], b["w_in"], EPS) for b in lay],
                     bench.B_RMS),
        "rotary_embedding": (lambda: [pe_r.rotary_embedding(pos, b["q"], b["k"], HD, cache_bf16, True) for b in lay],
                             lambda: [pb.pos_encoding_ops.rotary_embedding(pos, b["q"], b["k"], HD, ch["cache"], True)
                                      for b in lay],
                             bench.B_ROPE),
        "silu_and_mul": (lambda: [act_r.silu_and_mul(b["act"], b["gate_up"]) for b in lay],
                         lambda: [pb.activation_ops.silu_and_mul(b["act"], b["gate_up"]) for b in lay],
                         bench.B_SILU),
        "add+rms_norm vs fused_add_rms_norm": (
            lambda: [(torch.add(b["attn"], b["residual2"], out=b["res_sum"]),
                      ln_r.rms_norm(b["normed"], b["res_sum"], b["w_post"], EPS)) for b in lay],
            lambda: [pb.layernorm_ops.fused_add_rms_norm(b["attn"], b["residual2"], b["w_post"], EPS) for b in lay],
            bench.B_FUSED),
    }
    per_op = {}
    for name, (rf, of, nbytes) in single.items():
        row = {}
        for who, fn in (("reference_cuda", rf), ("ours", of)):
            g = bench.capture(fn)
            us = bench.time_replays(g, args.reps, 3) * 1e3 / (args.reps * bench.L)
            row[who] = {"us_per_launch": round(us, 3), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
            del g
        row["speedup"] = round(row["reference_cuda"]["us_per_launch"] / row["ours"]["us_per_launch"], 2)
        per_op[name] = row
    res["per_op"] = per_op
    # MoE routing (Mixtral-8x7B shapes): the reference wrapper pre-fills sorted_ids with
    # torch (fused_moe.py:191-195) before its moe_align_block_size; ours fills
    # the padding in the kernel.
    moe_r = load_ref_ops("moe_ops")
    moe = []
    for t in (64, 512, 4096, 16384):
        E, k, bs = 8, 2, 64
        gating = torch.randn(t, E, generator=torch.Generator().manual_seed(t)).to(dev)
        w = torch.empty(t, k, device=dev)
        ids = torch.empty(t, k, dtype=torch.int32, device=dev)
        tei = torch.empty(t, k, dtype=torch.int32, device=dev)
        cap = t * k + E * (bs - 1)
        srt = torch.empty(cap, dtype=torch.int32, device=dev)
        eid = torch.empty((cap + bs - 1) // bs, dtype=torch.int32, device=dev)
        tot = torch.empty(1, dtype=torch.int32, device=dev)
        cases = {
            "reference_cuda": (lambda: moe_r.topk_softmax(w, ids, tei, gating),
                               lambda: (srt.fill_(t * k), moe_r.moe_align_block_size(ids, E, bs, srt, eid, tot))),
            "ours": (lambda: pb.moe_ops.topk_softmax(w, ids, tei, gating, False),
                     lambda: pb.moe_ops.moe_align_block_size(ids, E, bs, srt, eid, tot, True)),
        }
        row = {"T": t}
        for who, (tk, al) in cases.items():
            r = {}
            for name, fn in (("topk_softmax", tk), ("moe_align_block_size", al)):
                g = bench.capture(lambda: [fn() for _ in range(20)])
                r[name + "_us"] = round(bench.time_replays(g, 5, 3) * 1e3 / 100, 3)
                del g
            row[who] = r
        moe.append(row)
    res["moe"] = moe
    # Paged-KV append: FlashInfer's path as PaceServe calls it
    # (flashinfer_attention_wrapper.py:239-255: get_seq_lens,
    # get_batch_indices_positions, append_paged_kv_cache) against the one-launch
    # by-indptr kernel.  The image's FlashInfer builds its page module on first
    # use; a failure is recorded, not raised.
    try:
        import flashinfer

        ai, kp, ki, kl = (x.to(dev) for x in bench.append_metadata())
        caches = [torch.zeros(4096, 2, 16, bench.NKV, HD, dtype=torch.bfloat16, device=dev)
                  for _ in range(bench.L)]
        qkvs = [b["qkv"] for b in lay]
        NQ, NKV = bench.NQ, bench.NKV
        nnz = int(ai[-1].item())

        def fi():
            for c, q in zip(caches, qkvs):
                k = q[:, NQ * HD:(NQ + NKV) * HD].contiguous().reshape(-1, NKV, HD)
                v = q[:, (NQ + NKV) * HD:].contiguous().reshape(-1, NKV, HD)
                sl = flashinfer.get_seq_lens(kp, kl, 16)
                bi, po = flashinfer.get_batch_indices_positions(ai, sl, nnz)
                flashinfer.append_paged_kv_cache(k, v, bi, po, c, ki, kp, kl, kv_layout="NHD")

        def mine():
            for c, q in zip(caches, qkvs):
                pb.kv_transfer_ops.append_paged_kv_cache_by_indptr(
                    q[:, NQ * HD:(NQ + NKV) * HD], q[:, (NQ + NKV) * HD:], ai, c, ki, kp, kl)
        row = {}
        for who, fn in (("flashinfer_" + flashinfer.__version__, fi), ("ours", mine)):
            fn()
            torch.cuda.synchronize()
            g = bench.capture(fn)
            row[who + "_us_per_layer"] = round(bench.time_replays(g, 20, 3) * 1e3 / (20 * bench.L), 3)
            del g
        ref_c = [c.clone() for c in caches]
        for c in caches:
            c.zero_()
        mine()
        torch.cuda.synchronize()
        for c in ref_c:
            c.zero_()
        for c, q in zip(ref_c, qkvs):
            k = q[:, NQ * HD:(NQ + NKV) * HD].contiguous().reshape(-1, NKV, HD)
            v = q[:, (NQ + NKV) * HD:].contiguous().reshape(-1, NKV, HD)
            bi, po = flashinfer.get_batch_indices_positions(ai, flashinfer.get_seq_lens(kp, kl, 16), nnz)
            flashinfer.append_paged_kv_cache(k, v, bi, po, c, ki, kp, kl, kv_layout="NHD")
        torch.cuda.synchronize()
        row["byte_equal_to_flashinfer"] = all(torch.equal(a, b) for a, b in zip(caches, ref_c))
        res["kv_append"] = row
    except Exception as exc:  # recorded, not fatal
        res["kv_append"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    res["chain_speedup"] = round(res["reference_cuda"]["ms_per_step"] / res["ours"]["ms_per_step"], 2)
    line = json.dumps(res)
    print(line)
    if args.out:
        with open(args.out, "w") as f:
            f.write(line + "\n")


if __name__ == "__main__":
    main()
