"""LTX-2 conv video VAE decoder and its spatial tiler restated on the CPU (test oracle).

Follows kinomlx/models/ltx2/video_vae/{blocks,decoder,tiling,config}.py and
kinomlx/kernels/fused_ops.py (pixel/group norm). Layout BFHWC inside the decoder, BCFHW at its
boundary, exactly as the reference.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .fused_ops import group_norm, pixel_norm, silu


# ----------------------------------------------------------------------------- tiling
def compute_trapezoidal_mask_1d(length: int, ramp_left: int, ramp_right: int,
                                left_starts_from_0: bool = False) -> torch.Tensor:
    """kinomlx/models/ltx2/video_vae/tiling.py:330-360."""
    ramp_left = min(ramp_left, length)
    ramp_right = min(ramp_right, length)
    values = [1.0] * length
    if ramp_left:
        count = ramp_left + 1 if left_starts_from_0 else ramp_left + 2
        fade = [i / (count - 1) for i in range(count)][:-1]
        if not left_starts_from_0:
            fade = fade[1:]
        for i, val in enumerate(fade[:ramp_left]):
            values[i] *= val
    if ramp_right:
        fade = [(ramp_right + 1 - i) / (ramp_right + 1) for i in range(1, ramp_right + 1)]
        start = length - ramp_right
        for i, val in enumerate(fade):
            values[start + i] *= val
    return torch.tensor(values, dtype=torch.float32).clamp(0.0, 1.0)


def tile_intervals(length: int, tile_size: int, stride: int, min_size: int):
    """kinomlx/models/ltx2/video_vae/tiling.py:56-72."""
    if length <= tile_size:
        return [(0, length)]
    starts = list(range(0, length, stride))
    while len(starts) > 1 and length - starts[-1] < min_size:
        starts.pop()
    return [(s, min(s + tile_size, length)) for s in starts[:-1]] + [(starts[-1], length)]


@dataclass(frozen=True)
class AxisTiles:
    starts: list
    ends: list
    left_ramps: list
    right_ramps: list


def split_axis(length: int, tile_size: int, overlap: int) -> AxisTiles:
    """kinomlx/models/ltx2/video_vae/tiling.py:834-863."""
    if length <= tile_size:
        return AxisTiles([0], [length], [0], [0])
    stride = tile_size - overlap
    starts, ends = [], []
    start = 0
    while start < length:
        end = min(start + tile_size, length)
        starts.append(start)
        ends.append(end)
        if end >= length:
            break
        start += stride
    left = [0] * len(starts)
    right = [0] * len(starts)
    for i in range(1, len(starts)):
        actual = ends[i - 1] - starts[i]
        left[i] = actual
        right[i - 1] = actual
    return AxisTiles(starts, ends, left, right)


def spatial_output_slice(start: int, end: int, left: int, right: int, scale: int):
    """kinomlx/models/ltx2/video_vae/tiling.py:900-914."""
    a, b = start * scale, end * scale
    return slice(a, b), compute_trapezoidal_mask_1d(b - a, left * scale, right * scale)


# ----------------------------------------------------------------------------- decoder
@dataclass(frozen=True)
class VaeVariant:
    """Decoder shape: conv_in 128 -> widths[0]; blocks as ("res", n) or ("d2s", stride, mult)."""

    norm: str = "pixel"  # "pixel" (LTX-2.3) or "group32"
    causal: bool = False
    latent_channels: int = 128
    out_channels: int = 3
    patch: int = 4
    top_width: int = 1024
    blocks: tuple = (
        ("res", 2),
        ("d2s", (2, 2, 2), 2),
        ("res", 2),
        ("d2s", (2, 2, 2), 1),
        ("res", 4),
        ("d2s", (2, 1, 1), 2),
        ("res", 6),
        ("d2s", (1, 2, 2), 2),
        ("res", 4),
    )
    norm_eps: float = 1e-8
    group_eps: float = 1e-6


LTX23 = VaeVariant()
BASELINE_VAE = VaeVariant(norm="group32", causal=True)


def conv3d(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, causal: bool) -> torch.Tensor:
    """Conv3dBlock with spatial_padding_mode="conv": temporal replicate padding (causal: k-1
    copies of the first frame; otherwise one copy at each end), spatial zero padding 1, MLX
    nn.Conv3d (fp32 accumulation rounded to the dtype, then the bias added in the dtype)
    (kinomlx/models/ltx2/video_vae/blocks.py:97-139). x: BFHWC, w: OTHWI."""
    if causal:
        x = torch.cat([x[:, :1].expand(-1, 2, -1, -1, -1), x], dim=1)
    else:
        x = torch.cat([x[:, :1], x, x[:, -1:]], dim=1)
    y = F.conv3d(x.float().permute(0, 4, 1, 2, 3), w.float().permute(0, 4, 1, 2, 3),
                 padding=(0, 1, 1))
    y = y.permute(0, 2, 3, 4, 1).to(x.dtype)
    return y + b


def norm(x: torch.Tensor, v: VaeVariant, p: dict | None = None, prefix: str = "") -> torch.Tensor:
    if v.norm == "pixel":
        return pixel_norm(x, dim=-1, eps=v.norm_eps)
    c = x.shape[-1]
    weight = p.get(f"{prefix}.weight") if p else None
    bias = p.get(f"{prefix}.bias") if p else None
    if weight is None:
        weight = torch.ones(c, dtype=x.dtype)
        bias = torch.zeros(c, dtype=x.dtype)
    return group_norm(x, 32, weight, bias, v.group_eps)


def res_block(p: dict, prefix: str, x: torch.Tensor, v: VaeVariant) -> torch.Tensor:
    """x + conv2(silu(norm(conv1(silu(norm(x)))))) (blocks.py:142-169)."""
    h = conv3d(silu(norm(x, v, p, f"{prefix}.norm1")), p[f"{prefix}.conv1.weight"],
               p[f"{prefix}.conv1.bias"], v.causal)
    h = conv3d(silu(norm(h, v, p, f"{prefix}.norm2")), p[f"{prefix}.conv2.weight"],
               p[f"{prefix}.conv2.bias"], v.causal)
    return h + x


def depth_to_space(x: torch.Tensor, stride, channels: int) -> torch.Tensor:
    """(c, st, sh, sw) channel order (decoder.py:80-98)."""
    b, f, h, w, _ = x.shape
    st, sh, sw = stride
    x = x.reshape(b, f, h, w, channels, st, sh, sw).permute(0, 1, 5, 2, 6, 3, 7, 4)
    return x.reshape(b, f * st, h * sh, w * sw, channels)


def upsample(p: dict, prefix: str, x: torch.Tensor, stride, mult: int, v: VaeVariant) -> torch.Tensor:
    """DepthToSpaceUpsample3d without the residual path (decoder.py:100-121)."""
    cout = x.shape[-1] // mult
    y = conv3d(x, p[f"{prefix}.conv.weight"], p[f"{prefix}.conv.bias"], v.causal)
    y = depth_to_space(y, stride, cout)
    if stride[0] > 1:
        y = y[:, 1:]
    return y


def unpatchify(x: torch.Tensor, patch: int) -> torch.Tensor:
    """Packed channel index c*p*p + pw*p + ph (blocks.py:200-230)."""
    b, f, h, w, pc = x.shape
    c = pc // (patch * patch)
    x = x.reshape(b, f, h, w, c, patch, patch).permute(0, 1, 2, 6, 3, 5, 4)
    return x.reshape(b, f, h * patch, w * patch, c)


def decode(p: dict, latent: torch.Tensor, v: VaeVariant, dtype=torch.bfloat16) -> torch.Tensor:
    """Conv3dVideoDecoder.__call__ (decoder.py:213-259): latent BCFHW -> video BCFHW."""
    x = latent.to(dtype)
    std = p["per_channel_statistics.std_of_means"].reshape(1, -1, 1, 1, 1)
    mean = p["per_channel_statistics.mean_of_means"].reshape(1, -1, 1, 1, 1)
    x = (x.float() * std + mean).to(dtype)
    x = x.permute(0, 2, 3, 4, 1)
    x = conv3d(x, p["conv_in.weight"], p["conv_in.bias"], v.causal)
    for i, blk in enumerate(v.blocks):
        if blk[0] == "res":
            for j in range(blk[1]):
                x = res_block(p, f"up_blocks.{i}.res_blocks.{j}", x, v)
        else:
            x = upsample(p, f"up_blocks.{i}", x, blk[1], blk[2], v)
    x = conv3d(silu(norm(x, v, p, "norm_out")), p["conv_out.weight"], p["conv_out.bias"], v.causal)
    x = unpatchify(x, v.patch)
    return x.permute(0, 4, 1, 2, 3)


def decode_tiled(p: dict, latent: torch.Tensor, v: VaeVariant, tile: int = 8, overlap: int = 2,
                 scale: int = 32, dtype=torch.bfloat16, decoder=decode) -> torch.Tensor:
    """Spatially tiled decode with trapezoid blending in fp32, time untiled
    (kinomlx/models/ltx2/video_vae/tiling.py:1053-1386 for a single temporal chunk)."""
    b, _, f, h, w = latent.shape
    th, tw = split_axis(h, tile, overlap), split_axis(w, tile, overlap)
    out = None
    weights = None
    for hi in range(len(th.starts)):
        hs, hm = spatial_output_slice(th.starts[hi], th.ends[hi], th.left_ramps[hi],
                                      th.right_ramps[hi], scale)
        for wi in range(len(tw.starts)):
            ws, wm = spatial_output_slice(tw.starts[wi], tw.ends[wi], tw.left_ramps[wi],
                                          tw.right_ramps[wi], scale)
            tile_lat = latent[:, :, :, th.starts[hi] : th.ends[hi], tw.starts[wi] : tw.ends[wi]]
            dec = decoder(p, tile_lat, v, dtype).float()
            if out is None:
                frames = dec.shape[2]
                out = torch.zeros((b, dec.shape[1], frames, h * scale, w * scale))
                weights = torch.zeros((1, 1, frames, h * scale, w * scale))
            mask = hm.reshape(1, 1, 1, -1, 1) * wm.reshape(1, 1, 1, 1, -1)
            out[:, :, :, hs, ws] += dec * mask
            weights[:, :, :, hs, ws] += mask
    return out / torch.clamp(weights, min=1e-8)
