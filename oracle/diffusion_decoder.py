"""LTX-2.5 diffusion video decoder restated on the CPU (test oracle; only tests may import it).

Follows kinomlx/models/ltx2/video_vae/diffusion_decoder.py on its masked-attention path at the
bf16 compute dtype: every MLX operation rounds to bf16 where the reference's does (weights are
bf16, as a checkpoint binds them, so nothing promotes to fp32), fp32-opmath kernels (RMSNorm,
SiLU, addmm, attention) round once. The windowed attention is evaluated on the whole volume
(oracle.neighborhood_attention: the inward-shifted windows of `_neighborhood_mask`,
diffusion_decoder.py:416-448), which is what the reference's query tiling computes exactly.

`cfg` is any object with the fields of the reference's DiffusionVideoDecoderConfig
(kinomlx/models/ltx2/video_vae/config.py:187-257) plus latent_channels and out_channels; `w`
maps the reference's parameter names (det_stages.{s}.{i}.attn.qkv.weight, ...) to bf16 CPU
tensors (linear weights (out, in)); per_channel_statistics.{std_of_means, mean_of_means} fp32.
"""

from __future__ import annotations

import math

import torch

from .fused_ops import linear, rms_norm, silu
from .neighborhood_attention import neighborhood_attention

BF16 = torch.bfloat16


def _round(x: torch.Tensor, dtype=BF16) -> torch.Tensor:
    return x.to(dtype)


# ----------------------------------------------------------------------------- layout helpers
def patchify_spatial(x: torch.Tensor, p: int) -> torch.Tensor:
    """(B, C, F, H, W) -> (B, C * p * p, F, H / p, W / p), channel c * p * p + pw * p + ph
    (diffusion_decoder.py:49-72)."""
    b, c, f, h, w = x.shape
    x = x.reshape(b, c, f, h // p, p, w // p, p).permute(0, 1, 6, 4, 2, 3, 5)
    return x.reshape(b, c * p * p, f, h // p, w // p)


def unpatchify_spatial(x: torch.Tensor, p: int) -> torch.Tensor:
    """Inverse of patchify_spatial (diffusion_decoder.py:75-91)."""
    b, pc, f, h, w = x.shape
    c = pc // (p * p)
    x = x.reshape(b, c, p, p, f, h, w).permute(0, 1, 4, 5, 3, 6, 2)
    return x.reshape(b, c, f, h * p, w * p)


def minimum_latent_shape(cfg) -> tuple[int, int, int]:
    """Smallest latent grid keeping every attention window inside its stage's grid
    (diffusion_decoder.py:260-280)."""
    cumulative = [1, 1, 1]
    minimum = [1, 1, 1]
    for kernel, stride in zip(cfg.stage_kernels, cfg.upsample_strides):
        for a in range(3):
            minimum[a] = max(minimum[a], math.ceil(kernel[a] / cumulative[a]))
            cumulative[a] *= stride[a]
    for a in range(3):
        minimum[a] = max(minimum[a], math.ceil(cfg.stage5_kernel[a] / cumulative[a]))
    return minimum[0], minimum[1], minimum[2]


def edge_pad_axis(x: torch.Tensor, axis: int, minimum: int, trailing_only: bool):
    """Repeat the edge slices up to `minimum` along `axis`: (padded, (before, after))
    (diffusion_decoder.py:283-308)."""
    length = x.shape[axis]
    needed = max(0, minimum - length)
    if not needed:
        return x, (0, 0)
    before = 0 if trailing_only else needed // 2
    after = needed - before
    parts = []
    if before:
        parts.append(x.narrow(axis, 0, 1).expand(*[before if d == axis else s
                                                   for d, s in enumerate(x.shape)]))
    parts.append(x)
    if after:
        parts.append(x.narrow(axis, length - 1, 1).expand(*[after if d == axis else s
                                                            for d, s in enumerate(x.shape)]))
    return torch.cat(parts, dim=axis), (before, after)


# ----------------------------------------------------------------------------- rotary
def rope_split(head_dim: int) -> tuple[int, int, int]:
    """Channels of the t, h and w sections (RotaryPosition3D.__init__, :325-334)."""
    dim_t = (head_dim // 4) // 2 * 2
    dim_hw = (head_dim - dim_t) // 2
    if dim_hw % 2:
        dim_t -= 2
        dim_hw = (head_dim - dim_t) // 2
    return dim_t, dim_hw, dim_hw


def inverse_frequencies(dims: int, base: float = 10_000.0) -> torch.Tensor:
    exponents = torch.arange(0, dims, 2, dtype=torch.float32) / dims
    return torch.pow(torch.tensor(base, dtype=torch.float32), -exponents)


def rope_tables(head_dim: int, grid: tuple[int, int, int], base: float = 10_000.0):
    """fp32 (cos_t, sin_t, cos_h, sin_h, cos_w, sin_w), each (length, size / 2) from position
    zero (RotaryPosition3D.tables, :340-349)."""
    out = []
    for length, size in zip(grid, rope_split(head_dim)):
        angles = torch.arange(length, dtype=torch.float32)[:, None] * inverse_frequencies(size, base)[None, :]
        out.extend((torch.cos(angles), torch.sin(angles)))
    return tuple(out)


def rope3d(x: torch.Tensor, head_dim: int) -> torch.Tensor:
    """x (B, T, H, W, heads, D) from offsets (0, 0, 0): adjacent (even, odd) pairs of each
    section rotated in fp32 by its axis position, rounded back (:351-397)."""
    dims = rope_split(head_dim)
    parts = []
    start = 0
    for axis, size in enumerate(dims):
        v = x[..., start : start + size]
        start += size
        pairs = v.reshape(*v.shape[:-1], size // 2, 2)
        even, odd = pairs[..., 0].float(), pairs[..., 1].float()
        pos = torch.arange(x.shape[1 + axis], dtype=torch.float32)
        ang = pos[:, None] * inverse_frequencies(size)[None, :]
        shape = [1, 1, 1, 1, 1, size // 2]
        shape[1 + axis] = x.shape[1 + axis]
        ang = ang.reshape(shape)
        c, s = torch.cos(ang), torch.sin(ang)
        rot = torch.stack([even * c - odd * s, even * s + odd * c], dim=-1)
        parts.append(rot.reshape(v.shape).to(x.dtype))
    return torch.cat(parts, dim=-1)


# ----------------------------------------------------------------------------- blocks
def na_attention(x: torch.Tensor, w: dict, pre: str, kernel, head_dim: int) -> torch.Tensor:
    """NeighborhoodAttention3D on (B, T, H, W, C) (:480-632): qkv with bias, per-head RMSNorm
    of q and k, q * head_dim^-1/2, 3-D RoPE, windowed softmax attention, proj with bias."""
    b, t, h, wd, c = x.shape
    heads = c // head_dim
    wq, bq = w[pre + "qkv.weight"], w[pre + "qkv.bias"]
    q = linear(x, wq[:c], bq[:c]).reshape(b, t, h, wd, heads, head_dim)
    k = linear(x, wq[c : 2 * c], bq[c : 2 * c]).reshape(b, t, h, wd, heads, head_dim)
    v = linear(x, wq[2 * c :], bq[2 * c :]).reshape(b, t, h, wd, heads, head_dim)
    q = _round(rms_norm(q, w[pre + "q_norm.weight"], 1e-6).float() * head_dim**-0.5, q.dtype)
    k = rms_norm(k, w[pre + "k_norm.weight"], 1e-6)
    q = rope3d(q, head_dim)
    k = rope3d(k, head_dim)
    o = neighborhood_attention(q, k, v, window=tuple(kernel))
    return linear(o.reshape(b, t, h, wd, c), w[pre + "proj.weight"], w[pre + "proj.bias"])


def swiglu(x: torch.Tensor, w: dict, pre: str) -> torch.Tensor:
    """w_down(silu(w_gate(x)) * w_up(x)), no biases (TiledSwiGLU, :715-737)."""
    g = silu(linear(x, w[pre + "w_gate.weight"]))
    u = linear(x, w[pre + "w_up.weight"])
    return linear(_round(g.float() * u.float(), x.dtype), w[pre + "w_down.weight"])


def _add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return _round(a.float() + b.float(), a.dtype)


def det_block(x: torch.Tensor, w: dict, pre: str, kernel, head_dim: int) -> torch.Tensor:
    """DeterministicNABlock (:755-799)."""
    x = _add(x, na_attention(rms_norm(x, w[pre + "norm1.weight"], 1e-6), w, pre + "attn.", kernel,
                             head_dim))
    return _add(x, swiglu(rms_norm(x, w[pre + "norm2.weight"], 1e-6), w, pre + "mlp."))


def _modulate(n: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    one_plus = _round(1.0 + scale.float(), scale.dtype)
    return _add(_round(n.float() * one_plus.float(), n.dtype), shift)


def diff_block(x: torch.Tensor, ctx: torch.Tensor, mod: tuple, w: dict, pre: str, kernel,
               head_dim: int) -> torch.Tensor:
    """DiffusionNABlock (:827-898): modulation + scale_shift_table, context projection added,
    modulated norms before the attention and the SwiGLU (the three gates are unused)."""
    table = w[pre + "scale_shift_table"]
    vals = [_add(mod[i], table[i]) for i in range(7)]
    scale_msa, shift_msa, _, scale_mlp, shift_mlp, _, _ = vals
    x = _add(x, linear(ctx, w[pre + "context_proj.weight"], w[pre + "context_proj.bias"]))
    n = _modulate(rms_norm(x, w[pre + "norm1.weight"], 1e-6), scale_msa, shift_msa)
    x = _add(x, na_attention(n, w, pre + "attn.", kernel, head_dim))
    n = _modulate(rms_norm(x, w[pre + "norm2.weight"], 1e-6), scale_mlp, shift_mlp)
    return _add(x, swiglu(n, w, pre + "mlp."))


def pixel_shuffle(x: torch.Tensor, w: dict, pre: str, stride, drop_leading_frame: bool = True):
    """LinearPixelShuffle (:928-971): proj, then (c, st, sh, sw) channels to space-time."""
    b, f, h, wd, _ = x.shape
    st, sh, sw = stride
    y = linear(x, w[pre + "proj.weight"], w[pre + "proj.bias"])
    c = y.shape[-1] // (st * sh * sw)
    y = y.reshape(b, f, h, wd, c, st, sh, sw).permute(0, 1, 5, 2, 6, 3, 7, 4)
    y = y.reshape(b, f * st, h * sh, wd * sw, c)
    if st == 2 and drop_leading_frame:
        y = y[:, 1:]
    return y


def timestep_embedding(t: torch.Tensor, dtype=BF16) -> torch.Tensor:
    """PixArt sinusoid [cos | sin] of 256 features, fp32, then the compute dtype (:974-989)."""
    half = 128
    freq = torch.exp(-math.log(10_000.0) * torch.arange(half, dtype=torch.float32) / half)
    ang = t.float()[:, None] * freq[None, :]
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=-1).to(dtype)


# ----------------------------------------------------------------------------- decoder
def stages_1_to_3(latent: torch.Tensor, w: dict, cfg) -> torch.Tensor:
    """(:1161-1182): trailing frames repeated, conv_in, the first three stages and upsamples;
    latent (B, C, F, H, W) already denormalised, compute dtype."""
    pad = (cfg.stage_kernels[0][0] // 2) * 2
    if pad:
        latent = torch.cat([latent, latent[:, :, -1:].expand(-1, -1, pad, -1, -1)], dim=2)
    x = linear(latent.permute(0, 2, 3, 4, 1), w["conv_in.weight"], w["conv_in.bias"])
    for s in range(3):
        for i in range(cfg.stage_depths[s]):
            x = det_block(x, w, f"det_stages.{s}.{i}.", cfg.stage_kernels[s], cfg.head_dim)
        x = pixel_shuffle(x, w, f"upsamples.{s}.", cfg.upsample_strides[s])
    return x


def stage_4(x: torch.Tensor, w: dict, cfg, *, drop_leading_frame: bool = True,
            crop_trailing_ghost: bool = True) -> torch.Tensor:
    """(:1185-1213): the last deterministic stage and upsample, the trailing ghost frames cut."""
    for i in range(cfg.stage_depths[3]):
        x = det_block(x, w, f"det_stages.3.{i}.", cfg.stage_kernels[3], cfg.head_dim)
    x = pixel_shuffle(x, w, "upsamples.3.", cfg.upsample_strides[3], drop_leading_frame)
    pad = (cfg.stage_kernels[0][0] // 2) * 2
    if crop_trailing_ghost and pad:
        ghost = pad * cfg.temporal_compression_ratio
        frames = x.shape[1]
        removable = max(frames - cfg.stage5_kernel[0], 0)
        x = x[:, : frames - min(ghost, removable)]
    return x


def diffusion_step(context: torch.Tensor, x_t: torch.Tensor, timestep: torch.Tensor, w: dict,
                   cfg) -> torch.Tensor:
    """One evaluation of the pixel-space diffusion stage (:1225-1247): x_t (B, 3, F, H, W)."""
    p = cfg.patch_size
    temb = timestep_embedding(timestep * cfg.timestep_scale_multiplier, context.dtype)
    temb = linear(silu(linear(temb, w["t_embedder.linear_1.weight"], w["t_embedder.linear_1.bias"])),
                  w["t_embedder.linear_2.weight"], w["t_embedder.linear_2.bias"])
    proj = linear(silu(temb), w["shared_adaln.proj.weight"], w["shared_adaln.proj.bias"])
    c = proj.shape[-1] // 7
    mod = tuple(proj[:, i * c : (i + 1) * c][:, None, None, None, :] for i in range(7))
    x = patchify_spatial(x_t, p).permute(0, 2, 3, 4, 1)
    x = linear(x, w["conv_in_x_t.weight"], w["conv_in_x_t.bias"])
    for i in range(cfg.stage_depths[4]):
        x = diff_block(x, context, mod, w, f"diff_blocks.{i}.", cfg.stage5_kernel, cfg.head_dim)
    x = rms_norm(x, w["norm_out.weight"], 1e-6)
    x = linear(x, w["conv_out.weight"], w["conv_out.bias"]).permute(0, 4, 1, 2, 3)
    return unpatchify_spatial(x, p)


def denoise(context: torch.Tensor, x_t: torch.Tensor, w: dict, cfg, steps: int) -> torch.Tensor:
    """(:1250-1284): a single x0 step returns the prediction; otherwise x0 -> velocity and an
    Euler step per timestep in fp32, rounded to x_t's dtype."""
    b = context.shape[0]
    ts = torch.linspace(1.0, 1.0 / steps, steps, dtype=torch.float32)
    if steps == 1 and cfg.model_output_type == "x0":
        return diffusion_step(context, x_t, ts[:1].expand(b), w, cfg)
    for i in range(steps):
        t = ts[i : i + 1].expand(b)
        nxt = float(ts[i + 1]) if i + 1 < steps else 0.0
        out = diffusion_step(context, x_t, t, w, cfg).float()
        xf = x_t.float()
        if cfg.model_output_type == "x0":
            out = (xf - out) / t.reshape(b, 1, 1, 1, 1)
        x_t = (xf - (t - nxt).reshape(b, 1, 1, 1, 1) * out).to(x_t.dtype)
    return x_t


def decode(latent: torch.Tensor, noise: torch.Tensor, w: dict, cfg,
           steps: int | None = None) -> torch.Tensor:
    """DiffusionVideoDecoder.__call__ (:1295-1353) with the noise given: (B, C, F, H, W) latent
    -> (B, 3, 1 + (F - 1) * 8, H * 32, W * 32) video; `noise` is x_t of the padded working shape
    (`working_pixel_shape`)."""
    scale_t = cfg.temporal_compression_ratio
    scale_s = cfg.spatial_compression_ratio
    frames = 1 + (latent.shape[2] - 1) * scale_t
    height, width = latent.shape[3] * scale_s, latent.shape[4] * scale_s
    mt, mh, mw = minimum_latent_shape(cfg)
    latent, _ = edge_pad_axis(latent, 2, mt, True)
    latent, (ph, _) = edge_pad_axis(latent, 3, mh, False)
    latent, (pw, _) = edge_pad_axis(latent, 4, mw, False)
    std = w["per_channel_statistics.std_of_means"].float().reshape(1, -1, 1, 1, 1)
    mean = w["per_channel_statistics.mean_of_means"].float().reshape(1, -1, 1, 1, 1)
    latent = (latent.float() * std + mean).to(BF16)
    context = stage_4(stages_1_to_3(latent, w, cfg), w, cfg)
    out = denoise(context, noise, w, cfg, steps or cfg.default_num_inference_steps)
    h0, w0 = ph * scale_s, pw * scale_s
    return out[:, :, :frames, h0 : h0 + height, w0 : w0 + width]


def working_pixel_shape(latent_shape: tuple[int, ...], cfg) -> tuple[int, int, int, int, int]:
    """The x_t shape `decode` consumes for a (B, C, F, H, W) latent: (B, 3, frames of the
    context, H' * 32, W' * 32) over the padded latent grid."""
    b, _, f, h, wd = latent_shape
    mt, mh, mw = minimum_latent_shape(cfg)
    f, h, wd = max(f, mt), max(h, mh), max(wd, mw)
    pad = (cfg.stage_kernels[0][0] // 2) * 2
    frames = f + pad
    for st, _, _ in cfg.upsample_strides[:3]:
        frames = frames * st - (1 if st == 2 else 0)
    st = cfg.upsample_strides[3][0]
    frames = frames * st - (1 if st == 2 else 0)
    if pad:
        frames -= min(pad * cfg.temporal_compression_ratio, max(frames - cfg.stage5_kernel[0], 0))
    return (b, cfg.out_channels, frames, h * cfg.spatial_compression_ratio,
            wd * cfg.spatial_compression_ratio)
