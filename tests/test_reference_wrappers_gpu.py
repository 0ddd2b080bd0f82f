"""GPU: the op calls PaceServe's own layer wrappers make, replayed through this
package's shim.

tests/golden/make_wrapper_golden.py ran the reference's wrapper files
unchanged -- RMSNorm.forward, SiluAndMul/NewGELU/FastGELU, get_rope (Llama-3
scaling, and plain GPT-J) + RotaryEmbedding.forward on q/k split from a fused
qkv tensor, fused_topk and moe_align_block_size -- and recorded every call they
made into ``paceserve.*_ops``: each tensor argument with its exact dtype,
size, stride and storage offset (q and k stay strided views of one qkv
storage), every scalar, the storage contents before the call, and the CPU
oracle's result after it.  Here each call is rebuilt on the GPU with the same
views and made through ``paceserve_b200``'s module of the same name, so the
shim receives exactly what the reference's wrappers pass.

Rules: float outputs within REL_TOL (1e-2) of the oracle's fp32 formula;
integer outputs bit-exact (for moe_align_block_size, expert_ids up to
num_tokens_post_pad / block_size, the reference leaves the rest undefined);
every storage the op does not write is left bit-identical.
"""
import json
import os

import numpy as np
import pytest
import torch

import paceserve_b200 as pb
from tests._util import REL_TOL, rel_err

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
CALLS = json.load(open(os.path.join(GOLDEN, "wrapper_calls.json")))["calls"]
ARRAYS = np.load(os.path.join(GOLDEN, "wrapper_calls.npz"))
DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32,
          "int32": torch.int32, "int64": torch.int64}
# positions of the arguments each op writes
OUTPUTS = {"rms_norm": (0,), "silu_and_mul": (0,), "gelu_new": (0,), "gelu_fast": (0,),
           "rotary_embedding": (1, 2), "topk_softmax": (0, 1, 2),
           "moe_align_block_size": (3, 4, 5)}


def _storage(key: str, dtype: torch.dtype) -> torch.Tensor:
    a = torch.from_numpy(ARRAYS[key].copy())
    return a.view(torch.bfloat16) if dtype == torch.bfloat16 else a


def test_fixture_covers_every_wrapper_op():
    fns = {c["fn"] for c in CALLS}
    assert fns == set(OUTPUTS)
    # the rope calls pass q and k as strided views of one fused qkv storage
    ropes = [c for c in CALLS if c["fn"] == "rotary_embedding"]
    assert ropes and all(c["args"][1]["storage"] == c["args"][2]["storage"] for c in ropes)
    assert all(c["args"][2]["offset"] > 0 and c["args"][1]["stride"][0] > c["args"][1]["size"][1]
               for c in ropes)


@pytest.mark.parametrize("idx", range(len(CALLS)),
                         ids=[f"{i}-{c['fn']}" for i, c in enumerate(CALLS)])
def test_reference_wrapper_call_through_shim(idx):
    call = CALLS[idx]
    bases, dtypes, args = {}, {}, []
    for a in call["args"]:
        if a["kind"] != "tensor":
            args.append(a["value"])
            continue
        sid, dt = a["storage"], DTYPES[a["dtype"]]
        if sid not in bases:
            bases[sid] = _storage(f"c{idx}_s{sid}_in", dt).to(DEV)
            dtypes[sid] = dt
        args.append(torch.as_strided(bases[sid], a["size"], a["stride"], a["offset"]))
    getattr(getattr(pb, call["module"]), call["fn"])(*args)
    torch.cuda.synchronize()

    written = {call["args"][p]["storage"] for p in OUTPUTS[call["fn"]]}
    for sid, base in bases.items():
        got = base.cpu()
        want = _storage(f"c{idx}_s{sid}_out", dtypes[sid])
        before = _storage(f"c{idx}_s{sid}_in", dtypes[sid])
        if sid not in written:
            assert torch.equal(got, before), f"input storage {sid} was modified"
            continue
        if call["fn"] == "moe_align_block_size":
            continue  # compared below, with the undefined expert_ids tail excluded
        if call["fn"] == "topk_softmax":
            if dtypes[sid] == torch.float32:
                torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-7)
            else:
                assert torch.equal(got, want)
            continue
        assert rel_err(got, want) <= REL_TOL
        if call["fn"] == "rotary_embedding":
            # the part of the qkv storage outside the q and k views (v) is unchanged
            untouched = torch.zeros(before.shape, dtype=torch.bool)
            for p in (1, 2):
                a = call["args"][p]
                view = torch.as_strided(untouched, a["size"], a["stride"], a["offset"])
                view.fill_(True)
            untouched = ~untouched  # outside q and k
            assert torch.equal(got[untouched], before[untouched])
    if call["fn"] == "moe_align_block_size":
        sa, ea, ta = (call["args"][p]["storage"] for p in (3, 4, 5))
        total = int(_storage(f"c{idx}_s{ta}_out", torch.int32)[0])
        bs = call["args"][2]["value"]
        assert int(bases[ta].cpu()[0]) == total
        assert torch.equal(bases[sa].cpu(), _storage(f"c{idx}_s{sa}_out", torch.int32))
        assert torch.equal(bases[ea].cpu()[: total // bs],
                           _storage(f"c{idx}_s{ea}_out", torch.int32)[: total // bs])
