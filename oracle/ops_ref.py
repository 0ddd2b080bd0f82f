"""fp32 torch-CPU restatements of the reference's per-layer op formulas.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Every function names
the reference lines it restates.  Two flavours where the reference rounds to
the storage type mid-formula:

* ``*_fp32`` -- the exact-arithmetic formula in fp32: the "fp32 reference"
  the 1e-2 relative-error parity rule is stated against;
* ``*_rounded`` -- the same formula with the reference kernel's intermediate
  roundings to bf16/fp16 reproduced, for near-bit-exact comparisons.

All functions accept tensors on the CPU (any float dtype) and return fp32
tensors unless stated.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F


def _rnd(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """fp32 value of x after rounding to `dtype` (round to nearest even)."""
    if dtype == torch.float32:
        return x
    return x.to(dtype).to(torch.float32)


# ------------------------------------------------------------------ norms --
def rms_norm_fp32(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * w, all in fp32.

    Reference: RMSNorm docstring (paceserve/model_executor/layers/layernorm.py:13-16)
    and csrc/layernorm_kernels.cu:19-34.
    """
    xf = x.float()
    inv = torch.rsqrt((xf * xf).sum(-1, keepdim=True) / xf.shape[-1] + eps)
    return xf * inv * w.float()


def rms_norm_rounded(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """csrc/layernorm_kernels.cu:27,33: inv = rsqrtf(sum/H + eps);
    out = (T)((T)(x * inv) * w) -- returned in x's dtype."""
    dt = x.dtype
    xf = x.float()
    inv = torch.rsqrt((xf * xf).sum(-1, keepdim=True) / xf.shape[-1] + eps)
    return (_rnd(xf * inv, dt) * w.float()).to(dt)


def fused_add_rms_norm_rounded(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                               eps: float):
    """The composition at paceserve/model_executor/models/llama.py:248-252:
    residual <- (T)(x + residual); out = rms_norm(residual).  Returns
    (out, new_residual) in x's dtype."""
    dt = x.dtype
    z = (x.float() + residual.float()).to(dt)
    return rms_norm_rounded(z, w, eps), z


def fused_add_rms_norm_fp32(x, residual, w, eps):
    z = x.float() + residual.float()
    return rms_norm_fp32(z, w, eps), z


# ------------------------------------------------------------------- rope --
def rope_inv_freq(rotary_dim: int, base: float) -> torch.Tensor:
    """paceserve/model_executor/layers/rotary_embedding.py:67-73 (on the CPU)."""
    return 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim))


def llama3_inv_freq(inv_freqs: torch.Tensor, scaling_factor: float, low_freq_factor: float,
                    high_freq_factor: float, orig_max_position: int) -> torch.Tensor:
    """Llama-3 frequency scaling, rotary_embedding.py:127-148."""
    low_freq_wavelen = orig_max_position / low_freq_factor
    high_freq_wavelen = orig_max_position / high_freq_factor
    wave_len = 2 * math.pi / inv_freqs
    if low_freq_factor != high_freq_factor:
        smooth = (orig_max_position / wave_len - low_freq_factor) / (high_freq_factor - low_freq_factor)
    else:
        smooth = 0
    return torch.where(
        wave_len < high_freq_wavelen,
        inv_freqs,
        torch.where(
            wave_len > low_freq_wavelen,
            inv_freqs / scaling_factor,
            (1 - smooth) * inv_freqs / scaling_factor + smooth * inv_freqs,
        ),
    )


def cos_sin_cache(rotary_dim: int, max_position: int, base: float,
                  rope_scaling: Optional[dict] = None) -> torch.Tensor:
    """[max_position, rotary_dim] = [cos | sin] in fp32, rotary_embedding.py:76-85
    (plus the "llama3" scaling branch of get_rope, :369-379)."""
    inv = rope_inv_freq(rotary_dim, base)
    if rope_scaling is not None:
        kind = rope_scaling.get("type", rope_scaling.get("rope_type"))
        if kind != "llama3":
            raise ValueError(f"oracle restates only llama3 scaling, not {kind!r}")
        inv = llama3_inv_freq(inv, rope_scaling["factor"], rope_scaling["low_freq_factor"],
                              rope_scaling["high_freq_factor"],
                              rope_scaling["original_max_position_embeddings"])
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def _rotate(h: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rot: int, neox: bool):
    # h: [T, H, hd] fp32 (modified in place); cos/sin: [T, 1, rot/2]
    if neox:
        x = h[..., : rot // 2].clone()
        y = h[..., rot // 2: rot].clone()
        h[..., : rot // 2] = x * cos - y * sin
        h[..., rot // 2: rot] = y * cos + x * sin
    else:
        x = h[..., 0:rot:2].clone()
        y = h[..., 1:rot:2].clone()
        h[..., 0:rot:2] = x * cos - y * sin
        h[..., 1:rot:2] = y * cos + x * sin


def rotary_embedding_fp32(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor,
                          head_size: int, cache: torch.Tensor, is_neox: bool):
    """fp32 rotation of csrc/pos_encoding_kernels.cu:8-76 (neox pairs (i, i+rot/2),
    gptj pairs (2i, 2i+1); elements past rot_dim unchanged).  Tokens whose
    position is outside the cache are left unchanged.  Returns fp32 (q, k) of
    shapes [T, nq*hd] and [T, nk*hd]."""
    T = query.shape[0]
    rot = cache.shape[1]
    q = query.reshape(T, -1, head_size).float().clone()
    k = key.reshape(T, -1, head_size).float().clone()
    pos = positions.reshape(-1)[:T].long()
    ok = (pos >= 0) & (pos < cache.shape[0])
    cs = cache.float()[pos.clamp(0, cache.shape[0] - 1)]
    cos = cs[:, None, : rot // 2]
    sin = cs[:, None, rot // 2:]
    q2, k2 = q.clone(), k.clone()
    _rotate(q2, cos, sin, rot, is_neox)
    _rotate(k2, cos, sin, rot, is_neox)
    q = torch.where(ok[:, None, None], q2, q)
    k = torch.where(ok[:, None, None], k2, k)
    return q.reshape(T, -1), k.reshape(T, -1)


# ------------------------------------------------------------- activations --
def _halves(x: torch.Tensor):
    d = x.shape[-1] // 2
    return x[..., :d].float(), x[..., d:].float()


def silu_and_mul_fp32(x: torch.Tensor) -> torch.Tensor:
    """silu(x[:, :d]) * x[:, d:] (activation.py:10-17, activation_kernels.cu:8-23)."""
    a, b = _halves(x)
    return a / (1.0 + torch.exp(-a)) * b


def silu_and_mul_rounded(x: torch.Tensor) -> torch.Tensor:
    """(T)((T)silu(a) * b): silu returns T, then a T*T multiply
    (activation_kernels.cu:11,23)."""
    dt = x.dtype
    a, b = _halves(x)
    return (_rnd(a / (1.0 + torch.exp(-a)), dt) * b).to(dt)


def gelu_and_mul_fp32(x: torch.Tensor) -> torch.Tensor:
    """erf GELU gate: F.gelu(a) * b (no reference kernel; PyTorch composition)."""
    a, b = _halves(x)
    return F.gelu(a) * b


def gelu_tanh_and_mul_fp32(x: torch.Tensor) -> torch.Tensor:
    a, b = _halves(x)
    return F.gelu(a, approximate="tanh") * b


def gelu_new_fp32(x: torch.Tensor) -> torch.Tensor:
    """0.5 x (1 + tanh(0.79788456 (x + 0.044715 x^3))) (activation_kernels.cu:86-91)."""
    xf = x.float()
    return 0.5 * xf * (1.0 + torch.tanh(0.79788456 * (xf + 0.044715 * xf * xf * xf)))


def gelu_new_rounded(x: torch.Tensor) -> torch.Tensor:
    """activation_kernels.cu:88-90 with each T-typed operation rounded."""
    dt = x.dtype
    xf = x.float()
    r = lambda v: _rnd(v, dt)  # noqa: E731
    x3 = r(r(xf * xf) * xf)
    a = r(0.044715 * x3)
    b = r(xf + a)
    c = r(0.79788456 * b)
    t = r(torch.tanh(c))
    return r(r(0.5 * xf) * r(1.0 + t)).to(dt)


def gelu_fast_fp32(x: torch.Tensor) -> torch.Tensor:
    """0.5 x (1 + tanh(0.79788456 x (1 + 0.044715 x^2))) (activation_kernels.cu:93-98)."""
    xf = x.float()
    return 0.5 * xf * (1.0 + torch.tanh(xf * 0.79788456 * (1.0 + 0.044715 * xf * xf)))


def gelu_fast_rounded(x: torch.Tensor) -> torch.Tensor:
    """activation_kernels.cu:95-97 with each T-typed operation rounded."""
    dt = x.dtype
    xf = x.float()
    r = lambda v: _rnd(v, dt)  # noqa: E731
    a = r(xf * 0.79788456)
    b = r(0.044715 * xf)
    d = r(1.0 + r(b * xf))
    t = r(torch.tanh(r(a * d)))
    return r(r(0.5 * xf) * r(1.0 + t)).to(dt)


# ------------------------------------------------------------- op chain --
def chain_layer(layer: int, bufs: dict, cache: torch.Tensor, positions: torch.Tensor,
                eps: float, nq: int, nkv: int, hd: int):
    """One decoder layer's op sequence (llama.py:232-255 with the adds fused):
    input norm (rms_norm at layer 0, fused_add_rms_norm after), rope on q/k
    of the qkv buffer, post-attention fused_add_rms_norm, silu_and_mul.
    Operates in place on the dict of CPU tensors, in their dtype."""
    if layer == 0:
        bufs["normed"] = rms_norm_rounded(bufs["hidden"], bufs["w_in"], eps)
    else:
        out, res = fused_add_rms_norm_rounded(bufs["hidden"], bufs["residual"], bufs["w_in"], eps)
        bufs["hidden"], bufs["residual"] = out, res
    qkv = bufs["qkv"]
    q = qkv[:, : nq * hd]
    k = qkv[:, nq * hd: (nq + nkv) * hd]
    q2, k2 = rotary_embedding_fp32(positions, q, k, hd, cache, True)
    qkv[:, : nq * hd] = q2.to(qkv.dtype)
    qkv[:, nq * hd: (nq + nkv) * hd] = k2.to(qkv.dtype)
    out, res = fused_add_rms_norm_rounded(bufs["attn"], bufs["residual2"], bufs["w_post"], eps)
    bufs["attn"], bufs["residual2"] = out, res
    bufs["act"] = silu_and_mul_rounded(bufs["gate_up"])


# ------------------------------------------- single-layer fp32 CPU chain --
# The CPU-runnable configuration of the path: one Llama-3-8B decoder layer's
# ops in fp32 at T=64 (residual add fused into the norm, llama.py:248-252;
# rope as rotary_embedding.py:87-103 calls it; SwiGLU as activation.py:19-24).
CONFIG1 = {"T": 64, "H": 4096, "NQ": 32, "NKV": 8, "HD": 128, "I": 14336, "EPS": 1e-5,
           "THETA": 500000.0, "MAX_POS": 8192, "POS_HIGH": 4096}
# fp32 algorithmic bytes per token: fused norm 16H, rope 8(nq+nkv)hd + rot*4 + 8,
# silu_and_mul 12I.
CONFIG1_BYTES_PER_TOKEN = 16 * 4096 + (8 * 40 * 128 + 128 * 4 + 8) + 12 * 14336


def config1_inputs(seed: int = 0) -> dict:
    """Seeded fp32 CPU inputs: x, residual [T,H] ~ N(0,1); w [H] ~ N(1,0.02);
    q [T,NQ*HD], k [T,NKV*HD] ~ N(0,1); positions uniform in [0, 4096);
    gate_up [T,2I] ~ N(0,1); the fp32 cos/sin cache for max_pos 8192."""
    c = CONFIG1
    g = torch.Generator().manual_seed(seed)
    T, H = c["T"], c["H"]
    return {
        "x": torch.randn(T, H, generator=g),
        "residual": torch.randn(T, H, generator=g),
        "w": torch.randn(H, generator=g) * 0.02 + 1.0,
        "q": torch.randn(T, c["NQ"] * c["HD"], generator=g),
        "k": torch.randn(T, c["NKV"] * c["HD"], generator=g),
        "positions": torch.randint(0, c["POS_HIGH"], (T,), generator=g),
        "gate_up": torch.randn(T, 2 * c["I"], generator=g),
        "cache": cos_sin_cache(c["HD"], c["MAX_POS"], c["THETA"]),
    }


def config1_chain(inp: dict) -> dict:
    """fused_add_rms_norm -> neox rotary_embedding -> silu_and_mul in fp32.
    Returns the outputs: normed x, updated residual, rotated q and k, act."""
    c = CONFIG1
    x, res = fused_add_rms_norm_fp32(inp["x"], inp["residual"], inp["w"], c["EPS"])
    q, k = rotary_embedding_fp32(inp["positions"], inp["q"], inp["k"], c["HD"], inp["cache"], True)
    act = silu_and_mul_fp32(inp["gate_up"])
    return {"x": x, "residual": res, "q": q, "k": k, "act": act}
