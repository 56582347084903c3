"""The LTX-2 conv video-VAE decoder and tiler in fp32 (parity mode) on the fp32 CUDA-core
kernels: the same graph as `VideoDecoder` (kinomlx/models/ltx2/video_vae/decoder.py:131-259,
blocks.py:54-230, tiling.py:330-1386) with every activation fp32, for the reference run with
float32 arrays. Channels-last activations; each conv is one implicit-GEMM launch (bias and
residual in its epilogue, depth-to-space in its store), each norm + SiLU one launch.
"""

from __future__ import annotations

import math

import torch

from .. import ops, ops_f32 as f
from .video_vae import VaeVariant, tile_plan

F32 = torch.float32


class VideoDecoderF32:
    """fp32 device Conv3dVideoDecoder; `weights` uses the reference checkpoint names with OTHWI
    conv weights (kinomlx/models/ltx2/video_vae/blocks.py:19-37)."""

    dtype = F32

    def __init__(self, weights: dict[str, torch.Tensor], variant: VaeVariant,
                 device: torch.device | str = "cuda"):
        self.v = variant
        self.device = torch.device(device)
        dev = lambda t: t.to(self.device, F32).contiguous()
        w = weights
        self.std = dev(w["per_channel_statistics.std_of_means"])
        self.mean = dev(w["per_channel_statistics.mean_of_means"])
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
                # rows (c, sub) -> (sub, c): each output voxel's channels contiguous
                wt = wt.reshape(cout, sub, *wt.shape[1:]).transpose(0, 1).reshape(wt.shape)
                bs = bs.reshape(cout, sub).transpose(0, 1).reshape(-1)
                self.stages.append(("d2s", (dev(wt), dev(bs), stride)))
                c = cout
        self.final_width = c
        self.spatial_scale = variant.patch * math.prod(
            blk[1][1] for blk in variant.blocks if blk[0] == "d2s")
        self.norm_out = None
        if variant.norm == "group32":
            self.norm_out = (dev(w["norm_out.weight"]), dev(w["norm_out.bias"]))
        self.conv_out = (dev(w["conv_out.weight"]), dev(w["conv_out.bias"]))

    def _norm_silu(self, x: torch.Tensor, params) -> torch.Tensor:
        if self.v.norm == "pixel":
            return f.pixel_norm(x, self.v.norm_eps, silu=True)
        if params is None:  # the reference's parameter-free GroupNorm: unit weight, zero bias
            c = x.shape[-1]
            params = (torch.ones(c, device=self.device), torch.zeros(c, device=self.device))
        return f.group_norm(x, 32, params[0], params[1], self.v.group_eps, silu=True)

    def decode_features(self, latent: torch.Tensor) -> torch.Tensor:
        """Latent (1, C, F, H, W) -> conv_out output (F', H', W', C_out * p^2) fp32
        (decoder.py:213-255 without the unpatchify)."""
        causal = self.v.causal
        x = f.latent_to_bfhwc(latent.to(self.device, F32).contiguous(), self.std, self.mean)
        x = f.conv3d(x, *self.conv_in, causal=causal)
        for kind, payload in self.stages:
            if kind == "res":
                for entry in payload:
                    h = self._norm_silu(x, entry.get("norm1"))
                    h = f.conv3d(h, *entry["conv1"], causal=causal)
                    h = self._norm_silu(h, entry.get("norm2"))
                    x = f.conv3d(h, *entry["conv2"], causal=causal, residual=x)
            else:
                wt, bs, stride = payload
                x = f.conv3d(x, wt, bs, causal=causal, stride=stride)
        x = self._norm_silu(x, self.norm_out)
        return f.conv3d(x, *self.conv_out, causal=causal)

    def decode(self, latent: torch.Tensor, *, tile: int | None = 8, overlap: int = 2) -> torch.Tensor:
        """Decoded video (1, C, F, H, W) fp32: spatial tiles blended with trapezoid weights
        (tiling.py:1053-1386, time untiled); `tile=None` decodes in one pass."""
        _, _, _, h, w = latent.shape
        if tile is None:
            tile = max(h, w)
        scale = self.spatial_scale
        canvas = weights = None
        for h0, h1, w0, w1, y0, x0, mh, mw in tile_plan(h, w, tile, overlap, scale):
            feat = self.decode_features(latent[:, :, :, h0:h1, w0:w1].contiguous())
            if canvas is None:
                canvas = torch.zeros((1, self.v.out_channels, feat.shape[0], h * scale, w * scale),
                                     device=self.device, dtype=F32)
                weights = torch.zeros((h * scale, w * scale), device=self.device, dtype=F32)
            f.tile_blend(feat, canvas, weights, y0, x0, mh.to(self.device), mw.to(self.device),
                         self.v.patch)
        return ops.blend_normalize(canvas, weights)
