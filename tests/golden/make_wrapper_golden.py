"""Record the op calls that PaceServe's own layer wrappers make, for the GPU replay test.

Test infrastructure.  The reference checkout must be present (argument, or
``PACE_REFERENCE_ROOT``, or a ``reference`` directory beside this
repository); the GPU box has no copy of it, so the calls are recorded here and
committed as ``wrapper_calls.json`` + ``wrapper_calls.npz``.

The reference package cannot be imported whole (its root needs Ray), so each
wrapper file is loaded by path, unchanged, with three stand-ins:

* ``paceserve.{layernorm,pos_encoding,activation,moe}_ops``: modules whose
  functions record every call -- each tensor argument as (storage, dtype, size,
  stride, offset), plus the storage's contents -- then compute it with the CPU
  oracle (``oracle/ops_ref.py``, ``oracle/moe_ref.py``) and record the
  storages again;
* ``paceserve.metrics.cuda_timer.CudaTimer``: a timer that records nothing
  (the reference's pushes CUDA times into its metrics store);
* a ``TorchFunctionMode`` that creates on the CPU the tensors the wrappers ask
  for on ``"cuda"`` (``RotaryEmbedding._compute_inv_freq``, model construction
  under ``torch.device("cuda")``), since this machine has no GPU.

Modules are constructed as the reference's model loader does
(``model_executor/model_loader.py:28-33,50-52``): with the default dtype set
to the model's dtype.  The wrappers exercised, with the reference lines:

* ``RMSNorm.forward`` (``layers/layernorm.py:31-40``)
* ``SiluAndMul.forward``, ``NewGELU``, ``FastGELU`` (``layers/activation.py:19-43``)
* ``get_rope`` with Llama-3 scaling and the plain GPT-J form, then
  ``RotaryEmbedding.forward`` on q/k split from a fused qkv tensor as
  ``models/llama.py:176`` splits it (``layers/rotary_embedding.py:87-103,347-404``)
* ``fused_topk`` and ``moe_align_block_size``
  (``layers/fused_moe/fused_moe.py:346-373,151-204``)

Usage: ``python tests/golden/make_wrapper_golden.py [reference_root] [--check]``
(``--check`` records again and compares with the committed fixture).
"""
from __future__ import annotations

import contextlib
import importlib.util
import json
import os
import sys
import types

import numpy as np
import torch
from torch.overrides import TorchFunctionMode

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle import moe_ref, ops_ref  # noqa: E402

OUT_JSON = os.path.join(HERE, "wrapper_calls.json")
OUT_NPZ = os.path.join(HERE, "wrapper_calls.npz")
OP_MODULES = ("layernorm_ops", "pos_encoding_ops", "activation_ops", "moe_ops")
WRAPPER_FILES = {
    "ref_layernorm": "paceserve/model_executor/layers/layernorm.py",
    "ref_activation": "paceserve/model_executor/layers/activation.py",
    "ref_rotary_embedding": "paceserve/model_executor/layers/rotary_embedding.py",
    "ref_fused_moe": "paceserve/model_executor/layers/fused_moe/fused_moe.py",
}


def reference_root(argv) -> str:
    if len(argv) > 1:
        return argv[1]
    env = os.environ.get("PACE_REFERENCE_ROOT")
    if env:
        return env
    return os.path.join(os.path.dirname(ROOT), "reference")


# ------------------------------------------------------------- recording --
def _flat(t: torch.Tensor) -> torch.Tensor:
    """The whole storage behind `t`, as a flat tensor of t's dtype."""
    st = t.untyped_storage()
    n = st.nbytes() // t.element_size()
    return torch.empty(0, dtype=t.dtype).set_(st, 0, (n,), (1,))


def _to_numpy(flat: torch.Tensor) -> np.ndarray:
    if flat.dtype == torch.bfloat16:
        return flat.view(torch.int16).numpy().copy()
    return flat.numpy().copy()


class Recorder:
    def __init__(self):
        self.calls = []
        self.arrays = {}
        self._sid = {}  # storage address -> index within the call being recorded

    def _storage_id(self, t: torch.Tensor) -> int:
        key = t.untyped_storage().data_ptr()
        if key not in self._sid:
            self._sid[key] = len(self._sid)
        return self._sid[key]

    def spec(self, a):
        if isinstance(a, torch.Tensor):
            return {"kind": "tensor", "storage": self._storage_id(a), "dtype": str(a.dtype).split(".")[1],
                    "size": list(a.shape), "stride": list(a.stride()),
                    "offset": int(a.storage_offset())}
        if isinstance(a, bool):
            return {"kind": "bool", "value": a}
        if isinstance(a, int):
            return {"kind": "int", "value": a}
        if isinstance(a, float):
            return {"kind": "float", "value": a}
        raise TypeError(f"unrecorded argument type {type(a)}")

    def record(self, module: str, fn: str, args, run):
        idx = len(self.calls)
        self._sid = {}  # tensors sharing a storage within this call share an index
        specs = [self.spec(a) for a in args]
        tensors = {s["storage"]: a for s, a in zip(specs, args) if s["kind"] == "tensor"}
        for sid, t in tensors.items():
            self.arrays[f"c{idx}_s{sid}_in"] = _to_numpy(_flat(t))
        run()
        for sid, t in tensors.items():
            self.arrays[f"c{idx}_s{sid}_out"] = _to_numpy(_flat(t))
        self.calls.append({"module": module, "fn": fn, "args": specs})


def oracle_ops(rec: Recorder):
    """Stand-in op modules: record, then compute with the CPU oracle."""

    def rms_norm(out, x, w, eps):
        rec.record("layernorm_ops", "rms_norm", [out, x, w, eps],
                   lambda: out.copy_(ops_ref.rms_norm_fp32(x, w, eps).to(out.dtype)))

    def rotary_embedding(positions, query, key, head_size, cache, is_neox):
        def run():
            q, k = ops_ref.rotary_embedding_fp32(positions, query, key, head_size, cache, is_neox)
            query.copy_(q.reshape(query.shape).to(query.dtype))
            key.copy_(k.reshape(key.shape).to(key.dtype))
        rec.record("pos_encoding_ops", "rotary_embedding",
                   [positions, query, key, head_size, cache, is_neox], run)

    def act(name, fn):
        def call(out, x):
            rec.record("activation_ops", name, [out, x], lambda: out.copy_(fn(x).to(out.dtype)))
        return call

    def topk_softmax(w, ids, tei, gating):
        def run():
            ow, oi, ot = moe_ref.topk_softmax(gating.numpy(), ids.shape[1])
            w.copy_(torch.from_numpy(ow))
            ids.copy_(torch.from_numpy(oi))
            tei.copy_(torch.from_numpy(ot))
        rec.record("moe_ops", "topk_softmax", [w, ids, tei, gating], run)

    def moe_align_block_size(topk_ids, num_experts, block_size, sorted_ids, expert_ids, total):
        def run():
            s, e, t = moe_ref.moe_align_block_size(topk_ids.numpy(), num_experts, block_size)
            sorted_ids.copy_(torch.from_numpy(s))
            expert_ids[: e.size].copy_(torch.from_numpy(e))
            total.fill_(t)
        rec.record("moe_ops", "moe_align_block_size",
                   [topk_ids, num_experts, block_size, sorted_ids, expert_ids, total], run)

    mods = {n: types.ModuleType(f"paceserve.{n}") for n in OP_MODULES}
    mods["layernorm_ops"].rms_norm = rms_norm
    mods["pos_encoding_ops"].rotary_embedding = rotary_embedding
    mods["activation_ops"].silu_and_mul = act("silu_and_mul", ops_ref.silu_and_mul_fp32)
    mods["activation_ops"].gelu_new = act("gelu_new", ops_ref.gelu_new_fp32)
    mods["activation_ops"].gelu_fast = act("gelu_fast", ops_ref.gelu_fast_fp32)
    mods["moe_ops"].topk_softmax = topk_softmax
    mods["moe_ops"].moe_align_block_size = moe_align_block_size
    return mods


class _NullTimer:
    """paceserve.metrics.cuda_timer.CudaTimer stand-in: times nothing."""

    def __init__(self, *args, **kwargs):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def install_stubs(op_modules: dict) -> None:
    """`paceserve` package with the given op modules and the timer stand-in."""
    pkg = sys.modules.get("paceserve")
    if pkg is None:
        pkg = types.ModuleType("paceserve")
        pkg.__path__ = []
        sys.modules["paceserve"] = pkg
    for name, mod in op_modules.items():
        sys.modules[f"paceserve.{name}"] = mod
        setattr(pkg, name, mod)
    metrics = types.ModuleType("paceserve.metrics")
    metrics.__path__ = []
    timer = types.ModuleType("paceserve.metrics.cuda_timer")
    timer.CudaTimer = _NullTimer
    metrics.cuda_timer = timer
    sys.modules["paceserve.metrics"] = metrics
    sys.modules["paceserve.metrics.cuda_timer"] = timer


def load_wrappers(ref_root: str) -> dict:
    """Each wrapper file by path, unchanged, under its own module name."""
    out = {}
    for name, rel in WRAPPER_FILES.items():
        path = os.path.join(ref_root, rel)
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        out[name] = mod
    return out


class CudaOnCpu(TorchFunctionMode):
    """Creates on the CPU the tensors the wrappers request on "cuda"."""

    def __torch_function__(self, func, types_, args=(), kwargs=None):
        kwargs = dict(kwargs or {})
        dev = kwargs.get("device")
        if dev is not None and torch.device(dev).type == "cuda":
            kwargs["device"] = "cpu"
        return func(*args, **kwargs)


@contextlib.contextmanager
def default_dtype(dtype):
    """model_loader.py:28-33: modules are built under the model's dtype."""
    old = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        yield
    finally:
        torch.set_default_dtype(old)


# ------------------------------------------------------------- scenarios --
LLAMA3_SCALING = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                  "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}


def run_scenarios(w: dict) -> None:
    """The wrapper calls whose op calls are recorded (small shapes: the
    fixture is committed)."""
    g = torch.Generator().manual_seed(2024)

    def rn(*shape, dtype=torch.bfloat16, mean=0.0, std=1.0):
        return (torch.randn(*shape, generator=g) * std + mean).to(dtype)

    with CudaOnCpu():
        # RMSNorm (Llama-3-8B width), weights as a loaded checkpoint would set them
        with default_dtype(torch.bfloat16):
            norm = w["ref_layernorm"].RMSNorm(4096, eps=1e-5)
        norm.weight.data.copy_(rn(4096, mean=1.0, std=0.02))
        norm(rn(7, 4096))
        # SwiGLU and the element-wise GELUs
        w["ref_activation"].SiluAndMul()(rn(5, 2 * 1024))
        w["ref_activation"].NewGELU()(rn(3, 512, dtype=torch.float16))
        w["ref_activation"].FastGELU()(rn(3, 512, dtype=torch.float16))
        # Llama-3 scaled NeoX rope on q/k split from a fused qkv row (llama.py:176)
        nq, nkv, hd, T = 4, 2, 128, 6
        with default_dtype(torch.bfloat16):
            rope = w["ref_rotary_embedding"].get_rope(hd, hd, 1024, 500000, True, LLAMA3_SCALING,
                                                      torch.bfloat16)
        qkv = rn(T, (nq + 2 * nkv) * hd)
        q, k, _v = qkv.split([nq * hd, nkv * hd, nkv * hd], dim=-1)
        pos = torch.tensor([0, 1, 2, 3, 700, 1023], dtype=torch.int64)
        rope(pos, q, k)
        # plain GPT-J style rope, fp16, partial rotary dim
        with default_dtype(torch.float16):
            rope2 = w["ref_rotary_embedding"].get_rope(64, 32, 256, 10000, False, None,
                                                       torch.float16)
        qkv2 = rn(4, 3 * 2 * 64, dtype=torch.float16)
        q2, k2, _ = qkv2.split([2 * 64, 2 * 64, 2 * 64], dim=-1)
        rope2(torch.tensor([5, 0, 255, 17], dtype=torch.int64), q2, k2)
        # Mixtral-style routing: fused_topk then moe_align_block_size
        hidden = rn(64, 32)
        gating = rn(64, 8)
        _wts, ids = w["ref_fused_moe"].fused_topk(hidden, gating, 2, True)
        w["ref_fused_moe"].moe_align_block_size(ids, 16, 8)


def record(root: str) -> Recorder:
    rec = Recorder()
    install_stubs(oracle_ops(rec))
    run_scenarios(load_wrappers(root))
    return rec


def check(root: str) -> int:
    """Record again and compare with the committed fixture: the same calls
    (modules, functions, argument dtypes, sizes, strides, offsets, scalars)
    and the same input contents for every storage the wrappers initialise
    (storages from torch.empty hold arbitrary bytes and are not compared)."""
    rec = record(root)
    committed = json.load(open(OUT_JSON))["calls"]
    if rec.calls != committed:
        print("call structure differs from the committed fixture")
        return 1
    arrays = np.load(OUT_NPZ)
    for idx, call in enumerate(committed):
        uninit = UNINITIALISED_ARGS.get(call["fn"], ())
        for pos, a in enumerate(call["args"]):
            if a["kind"] != "tensor" or pos in uninit:
                continue
            key = f"c{idx}_s{a['storage']}_in"
            if not np.array_equal(rec.arrays[key], arrays[key]):
                print(f"input {key} differs from the committed fixture")
                return 1
    print(f"{len(committed)} recorded calls match the committed fixture")
    return 0


# Arguments the wrappers allocate with torch.empty (contents arbitrary).
UNINITIALISED_ARGS = {"rms_norm": (0,), "silu_and_mul": (0,), "gelu_new": (0,), "gelu_fast": (0,),
                      "topk_softmax": (0, 1, 2), "moe_align_block_size": (4, 5)}


def main(argv) -> int:
    args = [a for a in argv if a != "--check"]
    root = reference_root(args)
    if "--check" in argv:
        return check(root)
    rec = record(root)
    with open(OUT_JSON, "w") as f:
        json.dump({"reference_files": WRAPPER_FILES, "calls": rec.calls}, f, indent=1)
    np.savez_compressed(OUT_NPZ, **rec.arrays)
    print(f"{len(rec.calls)} calls recorded -> {OUT_JSON}, {OUT_NPZ}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
