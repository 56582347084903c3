"""fp32 parity mode: torch front end of the kino_*_f32 entry points.

The reference's graphs run in whatever dtype their arrays carry; in float32 every MLX op keeps
fp32 (kinomlx/kernels/fused_ops.py's fp32 opmath, mx.addmm, mx.fast.scaled_dot_product_attention).
These wrappers take fp32 CUDA tensors and launch the fp32 kernels; like `ops`, they have no CPU
path and raise on a tensor of another device or dtype.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import (EPI_EULER, EPI_EULER_X0, EPI_GATED_RESIDUAL, EPI_GELU, EPI_NONE,
                   EPI_SIGMOID2, NORM_LAYER)
from .ops import _as3d, _need, _ptr, _stream, _timed

F32 = torch.float32

__all__ = [
    "adaln",
    "add_rows",
    "attention",
    "cfg_combine",
    "conv3d",
    "euler_velocity",
    "euler_denoised",
    "gelu_tanh",
    "group_norm",
    "latent_to_bfhwc",
    "linear",
    "pixel_norm",
    "qk_norm_rope",
    "silu",
    "swiglu",
    "tile_blend",
    "timestep_embedding",
]


def linear(
    x: torch.Tensor,
    w: torch.Tensor,
    out: torch.Tensor | None = None,
    *,
    bias: torch.Tensor | None = None,
    kind: int = EPI_NONE,
    residual: torch.Tensor | None = None,
    gate: torch.Tensor | None = None,
    act_col_begin: int = 0,
    dt: float = 0.0,
    sample: torch.Tensor | None = None,
    sigma: float = 0.0,
    ratio: float = 0.0,
) -> torch.Tensor:
    """out = epilogue(x @ w.T) in fp32 for x (batch, m, k) or (m, k) and an (n, k) weight.
    EPI_GELU applies to columns >= act_col_begin; EPI_GATED_RESIDUAL computes
    residual + gate * y (gate (batch, n)); EPI_EULER computes sample + dt * y; EPI_SIGMOID2
    computes 2 * sigmoid(y); EPI_EULER_X0 computes x0 = sample - sigma * y, then
    x0 + ratio * (sample - x0)."""
    _need(x, "x", F32)
    _need(w, "w", F32)
    x3 = _as3d(x)
    batch, m, k = x3.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"weight {tuple(w.shape)} does not match input width {k}")
    if out is None:
        out = torch.empty((*x.shape[:-1], n), device=x.device, dtype=F32)
    _need(out, "out", F32)
    o3 = _as3d(out)
    if tuple(o3.shape) != (batch, m, n):
        raise ValueError(f"out {tuple(out.shape)} does not match ({batch}, {m}, {n})")
    epi = _lib.EpilogueF32()
    epi.kind = kind
    if bias is not None:
        _need(bias, "bias", F32)
        epi.bias = bias.data_ptr()
    if kind == EPI_GATED_RESIDUAL:
        if residual is None or gate is None:
            raise ValueError("a gated residual needs residual and gate")
        _need(residual, "residual", F32)
        _need(gate, "gate", F32)
        r3 = _as3d(residual)
        epi.residual = r3.data_ptr()
        epi.ld_residual = r3.stride(1)
        epi.bs_residual = r3.stride(0)
        g = gate.reshape(-1, gate.shape[-1]) if gate.dim() != 2 else gate
        epi.gate = g.data_ptr()
        epi.bs_gate = g.stride(0) if g.shape[0] > 1 else 0
    elif kind == EPI_GELU:
        epi.act_col_begin = act_col_begin
    elif kind in (EPI_EULER, EPI_EULER_X0):
        if sample is None:
            raise ValueError("the Euler epilogue needs the current sample")
        _need(sample, "sample", F32)
        s3 = _as3d(sample)
        epi.aux = s3.data_ptr()
        epi.ld_aux = s3.stride(1)
        epi.bs_aux = s3.stride(0)
        epi.scalar = dt if kind == EPI_EULER else sigma
        epi.scalar2 = ratio
    elif kind not in (EPI_NONE, EPI_SIGMOID2):
        raise ValueError(f"epilogue {kind} has no fp32 form")
    with _timed("gemm_f32", 2.0 * batch * m * n * k, 4.0 * (batch * m * k + n * k + batch * m * n)):
        _lib.call("kino_linear_f32", _ptr(x3), _ptr(w), _ptr(o3), batch, m, n, k, x3.stride(1),
                  x3.stride(0), w.stride(0), o3.stride(1), o3.stride(0), ctypes.byref(epi),
                  _stream())
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor | None = None,
              *, heads: int, scale: float | None = None,
              gate: torch.Tensor | None = None,
              key_bias: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(q k^T * scale) v with q, k, v (batch, tokens, heads * 128) token-major fp32;
    `out` may be `q` itself; `gate` (batch, q tokens, heads) multiplies each head's output;
    `key_bias` (batch, >= k tokens) fp32 is added to every row's scaled scores."""
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        _need(t, name, F32)
    q3, k3, v3 = _as3d(q), _as3d(k), _as3d(v)
    batch, tq, width = q3.shape
    if width != heads * 128 or k3.shape[-1] != width or v3.shape[-1] != width:
        raise ValueError("fp32 attention takes 128-wide heads")
    if k3.shape[:2] != v3.shape[:2] or k3.shape[0] != batch:
        raise ValueError("k and v must share (batch, tokens) with q's batch")
    if out is None:
        out = torch.empty(q.shape, device=q.device, dtype=F32)
    _need(out, "out", F32)
    o3 = _as3d(out)
    tk = k3.shape[1]
    sc = scale if scale is not None else 128**-0.5
    g3, ld_g, bs_g = None, 0, 0
    if gate is not None:
        _need(gate, "gate", F32)
        g3 = _as3d(gate)
        if tuple(g3.shape) != (batch, tq, heads):
            raise ValueError("attention gate must be (batch, tokens, heads)")
        ld_g, bs_g = g3.stride(1), g3.stride(0)
    ld_b = 0
    if key_bias is not None:
        if (key_bias.dtype != F32 or key_bias.dim() != 2 or key_bias.shape[0] != batch
                or key_bias.shape[1] < tk or key_bias.stride(1) != 1
                or key_bias.device != q.device):
            raise ValueError("key_bias must be fp32 (batch, >= k tokens) with unit column "
                             "stride, on the queries' device")
        ld_b = key_bias.stride(0)
    flops = 4.0 * batch * heads * tq * tk * 128
    with _timed("attention_f32", flops, 4.0 * batch * width * (2 * tq + 2 * tk)):
        _lib.call("kino_attention_f32", _ptr(q3), _ptr(k3), _ptr(v3), _ptr(o3), batch, heads, tq,
                  tk, q3.stride(1), q3.stride(0), k3.stride(1), k3.stride(0), v3.stride(1),
                  v3.stride(0), o3.stride(1), o3.stride(0), sc, _ptr(g3), ld_g, bs_g,
                  _ptr(key_bias), ld_b, _stream())
    return out


def adaln(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
          out: torch.Tensor | None = None, *, norm: int = NORM_LAYER,
          eps: float = 1e-6) -> torch.Tensor:
    """norm(x) * (1 + scale) + shift in fp32; x (batch, rows, dim), shift/scale (batch, dim)."""
    _need(x, "x", F32)
    _need(shift, "shift", F32)
    _need(scale, "scale", F32)
    x3 = _as3d(x)
    batch, rows, dim = x3.shape
    if out is None:
        out = torch.empty(x.shape, device=x.device, dtype=F32)
    _need(out, "out", F32)
    o3 = _as3d(out)
    sh = shift.reshape(-1, dim)
    sc = scale.reshape(-1, dim)
    if sh.stride(0) != sc.stride(0):
        raise ValueError("shift and scale need the same batch stride")
    with _timed("adaln_f32", 0.0, 2.0 * 4 * batch * rows * dim):
        _lib.call("kino_adaln_f32", _ptr(x3), x3.stride(1), x3.stride(0), _ptr(sh), _ptr(sc),
                  sh.stride(0) if sh.shape[0] > 1 else 0, _ptr(o3), o3.stride(1), o3.stride(0),
                  batch, rows, dim, norm, eps, _stream())
    return out


def qk_norm_rope(x: torch.Tensor, *, heads: int, weight: torch.Tensor | None, norm: int,
                 rope: int, cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                 table_offset: int = 0, eps: float = 1e-6) -> torch.Tensor:
    """In place on x (batch, tokens, heads*128) fp32: per-head RMSNorm then the adjacent-pair
    RoPE from token-major (1|batch, table_tokens, 128) tables (QKNORM_PER_HEAD / ROPE_PAIRS), or
    full-row RMSNorm then the split-half RoPE from (1|batch, heads, table_tokens, 64) tables
    (QKNORM_FULL_ROW / ROPE_SPLIT)."""
    _need(x, "x", F32)
    x3 = _as3d(x)
    batch, tokens, width = x3.shape
    if width != heads * 128:
        raise ValueError("qk_norm_rope works on 128-wide heads")
    if weight is not None:
        _need(weight, "weight", F32)
    table_tokens, table_batched = 0, 0
    if cos is not None:
        _need(cos, "cos", F32)
        _need(sin, "sin", F32)
        if not (cos.is_contiguous() and sin.is_contiguous()):
            raise ValueError("RoPE tables must be contiguous")
        table_tokens = cos.shape[-2]
        table_batched = int(cos.dim() >= 3 and cos.shape[0] > 1)
    with _timed("qk_norm_rope_f32", 0.0, 8.0 * batch * tokens * width):
        _lib.call("kino_qk_norm_rope_f32", _ptr(x3), x3.stride(1), x3.stride(0), batch, tokens,
                  heads, _ptr(weight), norm, rope, _ptr(cos), _ptr(sin), table_batched,
                  table_tokens, table_offset, eps, _stream())
    return x


def add_rows(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out = a + b with b (n,) broadcast over the rows of a contiguous (..., n), fp32."""
    _need(a, "a", F32)
    _need(b, "b", F32)
    if not a.is_contiguous() or b.numel() != a.shape[-1]:
        raise ValueError("add_rows needs a contiguous (..., n) tensor and an (n,) row")
    b = b.contiguous()
    if out is None:
        out = torch.empty_like(a)
    _need(out, "out", F32)
    if not out.is_contiguous() or out.shape != a.shape:
        raise ValueError("add_rows writes a contiguous tensor shaped like a")
    n = a.shape[-1]
    with _timed("elementwise_f32", 0.0, 8.0 * a.numel()):
        _lib.call("kino_add_rows_f32", _ptr(a), _ptr(b), _ptr(out), a.numel() // n, n, _stream())
    return out


def _unary(name: str, x: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
    _need(x, "x", F32)
    x = x.contiguous()
    if out is None:
        out = torch.empty_like(x)
    with _timed("elementwise_f32"):
        _lib.call(name, _ptr(x), _ptr(out), x.numel(), _stream())
    return out


def gelu_tanh(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    return _unary("kino_gelu_tanh_f32", x, out)


def silu(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    return _unary("kino_silu_f32", x, out)


def cfg_combine(cond: torch.Tensor, uncond: torch.Tensor, guidance: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    _need(cond, "cond", F32)
    _need(uncond, "uncond", F32)
    cond, uncond = cond.contiguous(), uncond.contiguous()
    if out is None:
        out = torch.empty_like(cond)
    with _timed("elementwise_f32"):
        _lib.call("kino_cfg_combine_f32", _ptr(cond), _ptr(uncond), guidance, _ptr(out),
                  cond.numel(), _stream())
    return out


def euler_denoised(x: torch.Tensor, denoised: torch.Tensor, sigma: float, sigma_next: float,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """denoised + fp32(sigma_next / sigma) * (x - denoised) in fp32."""
    _need(x, "x", F32)
    _need(denoised, "denoised", F32)
    if not (x.is_contiguous() and denoised.is_contiguous()):
        raise ValueError("euler_denoised takes contiguous tensors")
    if out is None:
        out = torch.empty_like(x)
    ratio = float(torch.tensor(sigma_next / sigma, dtype=torch.float32))
    with _timed("elementwise_f32"):
        _lib.call("kino_euler_step_f32", _ptr(x), _ptr(denoised), ratio, _ptr(out), x.numel(),
                  _stream())
    return out


def euler_velocity(x: torch.Tensor, v: torch.Tensor, dt: float,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    _need(x, "x", F32)
    _need(v, "v", F32)
    if not (x.is_contiguous() and v.is_contiguous()):
        raise ValueError("euler_velocity takes contiguous tensors")
    if out is None:
        out = torch.empty_like(x)
    with _timed("elementwise_f32"):
        _lib.call("kino_euler_velocity_f32", _ptr(x), _ptr(v), dt, _ptr(out), x.numel(),
                  _stream())
    return out


def swiglu(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate) * content over the last dimension [gate | content] of x (batch, rows, 2H) or
    (rows, 2H); `out` (..., H) may be the gate half of x itself (x[..., :H])."""
    _need(x, "x", F32)
    width = x.shape[-1] // 2
    x3 = _as3d(x)
    if out is None:
        out = torch.empty((*x.shape[:-1], width), device=x.device, dtype=F32)
    _need(out, "out", F32)
    o3 = _as3d(out)
    if tuple(o3.shape) != (x3.shape[0], x3.shape[1], width):
        raise ValueError("swiglu output must be (..., H) for an input of (..., 2H)")
    with _timed("elementwise_f32"):
        _lib.call("kino_swiglu_f32", _ptr(x3), x3.stride(1), x3.stride(0), _ptr(o3), o3.stride(1),
                  o3.stride(0), x3.shape[0], x3.shape[1], width, _stream())
    return out


def timestep_embedding(t: torch.Tensor, dim: int = 256, *,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """t: fp32 (batch,) on the device -> fp32 (batch, dim) [cos, sin] features."""
    _need(t, "t", F32)
    t = t.contiguous()
    if out is None:
        out = torch.empty((t.shape[0], dim), device=t.device, dtype=F32)
    with _timed("elementwise_f32"):
        _lib.call("kino_timestep_embedding_f32", _ptr(t), _ptr(out), t.shape[0], dim, _stream())
    return out


# ----------------------------------------------------------------------------- video VAE
def conv3d(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
           causal: bool, stride: tuple[int, int, int] = (1, 1, 1),
           residual: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 3x3x3 conv of channels-last x (F, H, W, Cin) with an (N, 3, 3, 3, Cin) weight; with a
    depth-to-space `stride` the weight rows must be sub-position-major (n = sub * C' + c)."""
    _need(x, "x", F32)
    _need(weight, "weight", F32)
    if not x.is_contiguous() or not weight.is_contiguous():
        raise ValueError("conv3d needs contiguous channels-last input and OTHWI weight")
    x4 = x[0] if x.dim() == 5 else x
    f_, h, w, cin = x4.shape
    n = weight.shape[0]
    if tuple(weight.shape[1:]) != (3, 3, 3, cin):
        raise ValueError(f"weight {tuple(weight.shape)} does not match {cin} input channels")
    st, sh, sw = stride
    sub = st * sh * sw
    oshape = (f_ * st - (1 if st > 1 else 0), h * sh, w * sw, n // sub)
    if out is None:
        out = torch.empty(oshape, device=x.device, dtype=F32)
    if tuple(out.shape) != oshape or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {oshape}")
    if bias is not None:
        _need(bias, "bias", F32)
    if residual is not None:
        _need(residual, "residual", F32)
        if tuple(residual.shape[-4:]) != oshape or not residual.is_contiguous():
            raise ValueError("residual must be contiguous with the geometry of out")
    with _timed("conv3d_f32", 2.0 * f_ * h * w * n * 27 * cin,
                4.0 * (x4.numel() + weight.numel() + out.numel())):
        _lib.call("kino_conv3d_f32", _ptr(x4), f_, h, w, cin, _ptr(weight), n, _ptr(bias),
                  _ptr(residual), _ptr(out), int(causal), st, sh, sw, _stream())
    return out


def pixel_norm(x: torch.Tensor, eps: float = 1e-8, *, silu: bool = False,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Stepwise fp32 PixelNorm over the last (channel) axis, optionally followed by SiLU."""
    _need(x, "x", F32)
    if not x.is_contiguous():
        raise ValueError("pixel_norm needs a contiguous channels-last input")
    if out is None:
        out = torch.empty_like(x)
    c = x.shape[-1]
    with _timed("norm_f32", 0.0, 8.0 * x.numel()):
        _lib.call("kino_pixel_norm_f32", _ptr(x), _ptr(out), x.numel() // c, c, eps, int(silu),
                  _stream())
    return out


def group_norm(x: torch.Tensor, groups: int, weight: torch.Tensor, bias: torch.Tensor,
               eps: float, *, silu: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """Affine GroupNorm(32) over channels-last fp32 x with two-pass statistics (+ SiLU)."""
    if groups != 32:
        raise ValueError("the GroupNorm kernel takes 32 groups")
    _need(x, "x", F32)
    _need(weight, "weight", F32)
    _need(bias, "bias", F32)
    if not x.is_contiguous():
        raise ValueError("group_norm needs a contiguous channels-last input")
    if out is None:
        out = torch.empty_like(x)
    c = x.shape[-1]
    with _timed("norm_f32", 0.0, 16.0 * x.numel()):
        _lib.call("kino_group_norm_f32", _ptr(x), _ptr(weight), _ptr(bias), _ptr(out),
                  x.numel() // c, c, eps, int(silu), _stream())
    return out


def latent_to_bfhwc(latent: torch.Tensor, std: torch.Tensor, mean: torch.Tensor) -> torch.Tensor:
    """(1, C, F, H, W) fp32 latent -> (F, H, W, C) of latent * std + mean."""
    _need(latent, "latent", F32)
    if latent.dim() != 5 or latent.shape[0] != 1 or not latent.is_contiguous():
        raise ValueError("latent must be a contiguous (1, C, F, H, W) tensor")
    _, c, f_, h, w = latent.shape
    std, mean = std.float().contiguous(), mean.float().contiguous()
    out = torch.empty((f_, h, w, c), device=latent.device, dtype=F32)
    with _timed("elementwise_f32", 0.0, 8.0 * latent.numel()):
        _lib.call("kino_latent_to_bfhwc_f32", _ptr(latent), _ptr(std), _ptr(mean), _ptr(out), c,
                  f_ * h * w, _stream())
    return out


def tile_blend(decoded: torch.Tensor, canvas: torch.Tensor, weights: torch.Tensor, y0: int,
               x0: int, mask_h: torch.Tensor, mask_w: torch.Tensor, patch: int = 4) -> None:
    """Accumulate an fp32 decoded tile (F, h, w, C * patch^2) into the fp32 (1, C, F, H, W) canvas."""
    _need(decoded, "decoded", F32)
    if not decoded.is_contiguous():
        raise ValueError("the decoded tile must be contiguous")
    f_, h, w, packed = decoded.shape
    c = packed // (patch * patch)
    mask_h, mask_w = mask_h.float().contiguous(), mask_w.float().contiguous()
    with _timed("elementwise_f32", 0.0, 12.0 * decoded.numel()):
        _lib.call("kino_tile_blend_f32", _ptr(decoded), f_, h, w, c, patch, _ptr(canvas),
                  _ptr(weights), canvas.shape[-2], canvas.shape[-1], y0, x0, _ptr(mask_h),
                  _ptr(mask_w), _stream())
