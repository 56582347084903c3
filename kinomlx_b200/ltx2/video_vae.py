"""LTX-2 conv video-VAE decoder and spatial tiler on the sm_100a kernels
(kinomlx/models/ltx2/video_vae/decoder.py:131-259, blocks.py:54-230, tiling.py:330-1386).

Activations stay channels-last bf16 on the device. Every 3x3x3 conv is one implicit-GEMM launch
(bias and residual in its epilogue, depth-to-space folded into its store addressing); each
norm + SiLU pair is one launch (PixelNorm) or a short statistics + apply sequence (GroupNorm);
conv_out's tile is unpatchified and trapezoid-blended into an fp32 canvas by one kernel.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import ops

BF = torch.bfloat16


@dataclass(frozen=True)
class VaeVariant:
    """Decoder shape; blocks as ("res", n) or ("d2s", (st, sh, sw), channel reduction)."""

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


# kinomlx/models/ltx2/video_vae/config.py:705-728 (LTX-2.3 decoder, PixelNorm, non-causal)
LTX23 = VaeVariant()
# the same widths with GroupNorm(32) + SiLU and causal convs
BASELINE_VAE = VaeVariant(norm="group32", causal=True)


# ----------------------------------------------------------------------------- tiling (host)
def trapezoid_mask(length: int, ramp_left: int, ramp_right: int,
                   left_starts_from_0: bool = False) -> torch.Tensor:
    """kinomlx/models/ltx2/video_vae/tiling.py:330-360."""
    ramp_left, ramp_right = min(ramp_left, length), min(ramp_right, length)
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
        for i, val in enumerate(fade):
            values[length - ramp_right + i] *= val
    return torch.tensor(values, dtype=torch.float32).clamp(0.0, 1.0)


def split_axis(length: int, tile: int, overlap: int):
    """[start, end) tiles with left/right ramp lengths (tiling.py:834-863)."""
    if length <= tile:
        return [(0, length, 0, 0)]
    stride = tile - overlap
    spans, start = [], 0
    while start < length:
        end = min(start + tile, length)
        spans.append([start, end, 0, 0])
        if end >= length:
            break
        start += stride
    for i in range(1, len(spans)):
        ov = spans[i - 1][1] - spans[i][0]
        spans[i][2] = ov
        spans[i - 1][3] = ov
    return [tuple(s) for s in spans]


def tile_plan(height: int, width: int, tile: int = 8, overlap: int = 2, scale: int = 32):
    """Spatial tiles of the latent: (h0, h1, w0, w1, y0, x0, mask_h, mask_w) in pixel space."""
    plan = []
    for h0, h1, hl, hr in split_axis(height, tile, overlap):
        for w0, w1, wl, wr in split_axis(width, tile, overlap):
            plan.append((h0, h1, w0, w1, h0 * scale, w0 * scale,
                         trapezoid_mask((h1 - h0) * scale, hl * scale, hr * scale),
                         trapezoid_mask((w1 - w0) * scale, wl * scale, wr * scale)))
    return plan


# ----------------------------------------------------------------------------- decoder
class VideoDecoder:
    """Device Conv3dVideoDecoder. `weights` uses the reference checkpoint names with OTHWI conv
    weights (kinomlx/models/ltx2/video_vae/blocks.py:19-37)."""

    def __init__(self, weights: dict[str, torch.Tensor], variant: VaeVariant,
                 device: torch.device | str = "cuda"):
        self.v = variant
        self.device = torch.device(device)
        dev = lambda t: t.to(self.device, BF).contiguous()
        w = weights
        self.std = w["per_channel_statistics.std_of_means"].to(self.device, torch.float32)
        self.mean = w["per_channel_statistics.mean_of_means"].to(self.device, torch.float32)
        self.conv_in = (dev(w["conv_in.weight"]), dev(w["conv_in.bias"]))
        self.stages = []
        c = variant.top_width
        for i, blk in enumerate(variant.blocks):
            if blk[0] == "res":
                res = []
                for j in range(blk[1]):
                    a = f"up_blocks.{i}.res_blocks.{j}"
                    entry = {}
                    for k in (1, 2):
                        entry[f"conv{k}"] = (dev(w[f"{a}.conv{k}.weight"]), dev(w[f"{a}.conv{k}.bias"]))
                        if variant.norm == "group32":
                            entry[f"norm{k}"] = (dev(w[f"{a}.norm{k}.weight"]), dev(w[f"{a}.norm{k}.bias"]))
                    res.append(entry)
                self.stages.append(("res", res))
            else:
                stride, mult = blk[1], blk[2]
                cout = c // mult
                sub = math.prod(stride)
                wt = w[f"up_blocks.{i}.conv.weight"]
                bs = w[f"up_blocks.{i}.conv.bias"]
                # reorder rows (c, sub) -> (sub, c) so each output voxel's channels are contiguous
                wt = wt.reshape(cout, sub, *wt.shape[1:]).transpose(0, 1).reshape(wt.shape)
                bs = bs.reshape(cout, sub).transpose(0, 1).reshape(-1)
                self.stages.append(("d2s", (dev(wt), dev(bs), stride)))
                c = cout
        self.final_width = c
        # latent -> pixel scale: depth-to-space height strides times the unpatchify patch
        self.spatial_scale = variant.patch * math.prod(
            blk[1][1] for blk in variant.blocks if blk[0] == "d2s")
        self.norm_out = None
        if variant.norm == "group32":
            self.norm_out = (dev(w["norm_out.weight"]), dev(w["norm_out.bias"]))
        self.conv_out = (dev(w["conv_out.weight"]), dev(w["conv_out.bias"]))
        self._stats: torch.Tensor | None = None  # GroupNorm statistics from the producing conv
        self._conv_ws: torch.Tensor | None = None  # split-K workspace of the small-grid convs

    def _norm_silu(self, x: torch.Tensor, params) -> torch.Tensor:
        if self.v.norm == "pixel":
            return ops.pixel_norm(x, self.v.norm_eps, silu=True)
        # GroupNorm statistics come from the epilogue of the conv that produced x
        return ops.group_norm_from_stats(x, params[0], params[1], self.v.group_eps, self._stats,
                                         silu=True)

    def decode_features(self, latent: torch.Tensor) -> torch.Tensor:
        """Normalised latent (1, C, F, H, W) -> conv_out output (F', H', W', C_out * p^2) bf16
        (decoder.py:213-255 without the unpatchify)."""
        causal = self.v.causal
        group = self.v.norm != "pixel"
        if group and self._stats is None:
            self._stats = ops.conv_stats_buffer(self.device)
        if self._conv_ws is None:
            self._conv_ws = ops.conv_workspace(self.device)
        st = self._stats if group else None  # every GroupNorm input is the previous conv's output
        ws = self._conv_ws
        x = ops.latent_to_bfhwc(latent.to(self.device, BF).contiguous(), self.std, self.mean)
        x = ops.conv3d(x, *self.conv_in, causal=causal, stats=st, workspace=ws)
        for kind, payload in self.stages:
            if kind == "res":
                for entry in payload:
                    h = self._norm_silu(x, entry.get("norm1"))
                    h = ops.conv3d(h, *entry["conv1"], causal=causal, stats=st, workspace=ws)
                    h = self._norm_silu(h, entry.get("norm2"))
                    x = ops.conv3d(h, *entry["conv2"], causal=causal, residual=x, out=x, stats=st,
                                   workspace=ws)
            else:
                wt, bs, stride = payload
                x = ops.conv3d(x, wt, bs, causal=causal, stride=stride, stats=st, workspace=ws)
        x = self._norm_silu(x, self.norm_out)
        return ops.conv3d(x, *self.conv_out, causal=causal, workspace=ws)

    def decode_tiled(self, latent: torch.Tensor, *, tile: int = 8, overlap: int = 2,
                     tiles: list[int] | None = None, canvas: torch.Tensor | None = None,
                     weights: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Tiled decode (tiling.py:1053-1386, time untiled): returns the fp32 (1, C, F, H, W)
        canvas of weighted tile sums and the (H, W) weight canvas, before normalisation. `tiles`
        restricts the work to some tile indices (a rank's share on several GPUs)."""
        _, _, f, h, w = latent.shape
        scale = self.spatial_scale
        plan = tile_plan(h, w, tile, overlap, scale)
        for idx, (h0, h1, w0, w1, y0, x0, mh, mw) in enumerate(plan):
            if tiles is not None and idx not in tiles:
                continue
            sub = latent[:, :, :, h0:h1, w0:w1].contiguous()
            feat = self.decode_features(sub)
            if canvas is None:
                frames = feat.shape[0]
                canvas = torch.zeros((1, self.v.out_channels, frames, h * scale, w * scale),
                                     device=self.device, dtype=torch.float32)
                weights = torch.zeros((h * scale, w * scale), device=self.device, dtype=torch.float32)
            ops.tile_blend(feat, canvas, weights, y0, x0, mh.to(self.device), mw.to(self.device),
                           self.v.patch)
        return canvas, weights

    def decode(self, latent: torch.Tensor, *, tile: int | None = 8, overlap: int = 2) -> torch.Tensor:
        """Decoded video (1, C, F, H, W) fp32; `tile=None` decodes in one pass."""
        _, _, f, h, w = latent.shape
        if tile is None:
            tile = max(h, w)
        canvas, weights = self.decode_tiled(latent, tile=tile, overlap=overlap)
        return ops.blend_normalize(canvas, weights)


def vae_weight_specs(v: VaeVariant):
    """(name, shape, kind) in draw order (conv weights OTHWI N(0, 0.02), conv biases zero,
    GroupNorm affine ones/zeros, per-channel statistics std 1 / mean 0)."""
    specs = [("per_channel_statistics.std_of_means", (v.latent_channels,), "ones"),
             ("per_channel_statistics.mean_of_means", (v.latent_channels,), "zeros")]
    c = v.top_width
    specs += [("conv_in.weight", (c, 3, 3, 3, v.latent_channels), "normal"),
              ("conv_in.bias", (c,), "zeros")]
    for i, blk in enumerate(v.blocks):
        if blk[0] == "res":
            for j in range(blk[1]):
                a = f"up_blocks.{i}.res_blocks.{j}"
                for k in (1, 2):
                    if v.norm == "group32":
                        specs += [(f"{a}.norm{k}.weight", (c,), "ones"), (f"{a}.norm{k}.bias", (c,), "zeros")]
                    specs += [(f"{a}.conv{k}.weight", (c, 3, 3, 3, c), "normal"),
                              (f"{a}.conv{k}.bias", (c,), "zeros")]
        else:
            stride, mult = blk[1], blk[2]
            cout = c // mult
            n = math.prod(stride) * cout
            specs += [(f"up_blocks.{i}.conv.weight", (n, 3, 3, 3, c), "normal"),
                      (f"up_blocks.{i}.conv.bias", (n,), "zeros")]
            c = cout
    if v.norm == "group32":
        specs += [("norm_out.weight", (c,), "ones"), ("norm_out.bias", (c,), "zeros")]
    n = v.out_channels * v.patch**2
    specs += [("conv_out.weight", (n, 3, 3, 3, c), "normal"), ("conv_out.bias", (n,), "zeros")]
    return specs
