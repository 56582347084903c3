"""The LTX-2.5 diffusion video decoder on the B200 kernels.

Restates kinomlx/models/ltx2/video_vae/diffusion_decoder.py (DiffusionVideoDecoder and its
blocks, :311-1353): latent -> conv_in -> four deterministic neighborhood-attention stages, each
followed by a linear pixel shuffle (the context), then a pixel-space diffusion stage whose blocks
add the projected context and modulate their norms by a shared timestep AdaLN, one x0 step by
default. Every product runs on tcgen05 GEMMs with fused epilogues (bias, residual add, SwiGLU),
every attention on the exact windowed kernel `kino_neighborhood_attention`; the q/k RMSNorm, q
scale and 3-D RoPE run in `kino_na_qkv_prepare`, which also hands q, k, v over in fp16 (the
attention writes bf16 back for the proj product); norms,
modulation and the layout moves (pixel shuffles, spatial patchify / unpatchify, edge padding)
run in the library's own bandwidth kernels. Activations are bf16 (the reference's default
compute dtype), the attention operands fp16 with fp32 scores, as on the reference's kernel
route.

Batch entries are decoded one after another (the windows never cross entries). Not built:
`decode_streaming` (:1356-1646, temporal / spatial streaming for memory), the unsharp context
sharpening (:1216-1222), checkpoint loading and the reference's noise stream: the caller passes
x_t (`working_pixel_shape`).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .. import ops

BF16 = torch.bfloat16


@dataclass(frozen=True)
class DiffusionDecoderConfig:
    """The execution fields of the reference's DiffusionVideoDecoderConfig
    (kinomlx/models/ltx2/video_vae/config.py:187-257) plus the latent and pixel channels of the
    enclosing VideoVAEConfig; validated the same way."""

    head_dim: int
    stage_channels: tuple[int, int, int, int, int]
    stage_depths: tuple[int, int, int, int, int]
    stage_kernels: tuple[tuple[int, int, int], ...]
    upsample_strides: tuple[tuple[int, int, int], ...]
    upsample_channel_reductions: tuple[int, int, int, int]
    stage5_kernel: tuple[int, int, int]
    patch_size: int = 4
    t_emb_dim: int = 384
    timestep_scale_multiplier: float = 1000.0
    model_output_type: str = "x0"
    default_num_inference_steps: int = 1
    spatial_compression_ratio: int = 32
    temporal_compression_ratio: int = 8
    latent_channels: int = 128
    out_channels: int = 3
    rope_base: float = field(default=10_000.0)

    def __post_init__(self) -> None:
        if self.model_output_type not in {"x0", "v"}:
            raise ValueError("model_output_type must be 'x0' or 'v'")
        if len(self.stage_channels) != 5 or len(self.stage_depths) != 5:
            raise ValueError("five stage widths and depths")
        if len(self.stage_kernels) != 4 or len(self.upsample_strides) != 4 or \
                len(self.upsample_channel_reductions) != 4:
            raise ValueError("four deterministic stages, each with a kernel, stride and reduction")
        if any(c % self.head_dim for c in self.stage_channels):
            raise ValueError("every diffusion decoder stage width must divide by head_dim")
        for i, r in enumerate(self.upsample_channel_reductions):
            if self.stage_channels[i + 1] != self.stage_channels[i] // r:
                raise ValueError(f"stage_channels[{i + 1}] must be stage_channels[{i}] // {r}")
        st = math.prod(s[0] for s in self.upsample_strides)
        sh = math.prod(s[1] for s in self.upsample_strides)
        sw = math.prod(s[2] for s in self.upsample_strides)
        if st != self.temporal_compression_ratio:
            raise ValueError("temporal stride product does not match the compression ratio")
        if sh != self.spatial_compression_ratio // self.patch_size or sw != sh:
            raise ValueError("spatial stride product does not match the compression ratio")
        for k in (*self.stage_kernels, self.stage5_kernel):
            if len(k) != 3 or any(x < 1 or x % 2 == 0 for x in k):
                raise ValueError(f"attention windows are three odd sizes, got {k}")

    @property
    def trailing_pad_latent_frames(self) -> int:
        return (self.stage_kernels[0][0] // 2) * 2

    def minimum_latent_shape(self) -> tuple[int, int, int]:
        """Smallest latent grid keeping every window inside its stage's grid
        (diffusion_decoder.py:260-280)."""
        cumulative = [1, 1, 1]
        minimum = [1, 1, 1]
        for kernel, stride in zip(self.stage_kernels, self.upsample_strides):
            for a in range(3):
                minimum[a] = max(minimum[a], math.ceil(kernel[a] / cumulative[a]))
                cumulative[a] *= stride[a]
        for a in range(3):
            minimum[a] = max(minimum[a], math.ceil(self.stage5_kernel[a] / cumulative[a]))
        return minimum[0], minimum[1], minimum[2]

    def working_pixel_shape(self, latent_shape) -> tuple[int, int, int, int, int]:
        """x_t's shape for a (B, C, F, H, W) latent: the context's frames over the padded grid."""
        b, _, f, h, w = latent_shape
        mt, mh, mw = self.minimum_latent_shape()
        f, h, w = max(f, mt), max(h, mh), max(w, mw)
        frames = f + self.trailing_pad_latent_frames
        for st, _, _ in self.upsample_strides:
            frames = frames * st - (1 if st == 2 else 0)
        pad = self.trailing_pad_latent_frames
        if pad:
            frames -= min(pad * self.temporal_compression_ratio,
                          max(frames - self.stage5_kernel[0], 0))
        return (b, self.out_channels, frames, h * self.spatial_compression_ratio,
                w * self.spatial_compression_ratio)


def rope_split(head_dim: int) -> tuple[int, int, int]:
    """Channels of the t, h and w rotary sections (RotaryPosition3D, diffusion_decoder.py:325-334)."""
    dim_t = (head_dim // 4) // 2 * 2
    dim_hw = (head_dim - dim_t) // 2
    if dim_hw % 2:
        dim_t -= 2
        dim_hw = (head_dim - dim_t) // 2
    return dim_t, dim_hw, dim_hw


def rope_tables(head_dim: int, grid: tuple[int, int, int], base: float = 10_000.0) -> torch.Tensor:
    """cos_t, sin_t, cos_h, sin_h, cos_w, sin_w of each axis position from zero, fp32, back to
    back (RotaryPosition3D.tables, diffusion_decoder.py:336-349: angle = position *
    base^(-2i / section))."""
    parts = []
    for length, size in zip(grid, rope_split(head_dim)):
        inv = torch.pow(torch.tensor(base, dtype=torch.float32),
                        -(torch.arange(0, size, 2, dtype=torch.float32) / size))
        ang = torch.arange(length, dtype=torch.float32)[:, None] * inv[None, :]
        parts.extend((torch.cos(ang).reshape(-1), torch.sin(ang).reshape(-1)))
    return torch.cat(parts)


def patchify_spatial(x: torch.Tensor, patch_size: int) -> torch.Tensor:
    """Space-to-depth of (B, C, F, H, W) into (B, C * p * p, F, H / p, W / p) with the LTX
    channel packing c * p * p + pw * p + ph (diffusion_decoder.py:49-72), one strided copy."""
    b, c, f, h, w = x.shape
    p = patch_size
    if h % p or w % p:
        raise ValueError(f"pixel dimensions {h}x{w} are not divisible by patch size {p}")
    out = torch.empty((b, c * p * p, f, h // p, w // p), device=x.device, dtype=x.dtype)
    src = x.view(b, c, f, h // p, p, w // p, p).permute(0, 1, 6, 4, 2, 3, 5)
    ops.copy_view(src, out.view(b, c, p, p, f, h // p, w // p))
    return out


def unpatchify_spatial(x: torch.Tensor, patch_size: int) -> torch.Tensor:
    """Depth-to-space inverse of `patchify_spatial` (diffusion_decoder.py:75-91)."""
    b, pc, f, h, w = x.shape
    p = patch_size
    if pc % (p * p):
        raise ValueError(f"packed channel count {pc} is not divisible by {p * p}")
    c = pc // (p * p)
    out = torch.empty((b, c, f, h * p, w * p), device=x.device, dtype=x.dtype)
    src = x.view(b, c, p, p, f, h, w).permute(0, 1, 4, 5, 3, 6, 2)
    ops.copy_view(src, out.view(b, c, f, h, p, w, p))
    return out


class DiffusionVideoDecoder:
    """Device weights and the decode of the reference's DiffusionVideoDecoder."""

    def __init__(self, weights: dict[str, torch.Tensor], cfg: DiffusionDecoderConfig,
                 device: torch.device | str = "cuda"):
        if cfg.head_dim != 64:
            raise ValueError("the neighborhood attention kernel takes 64-wide heads")
        self.cfg = cfg
        self.device = torch.device(device)
        dev = self.device
        self.w: dict[str, torch.Tensor] = {}
        for name, t in weights.items():
            if name.startswith("per_channel_statistics."):
                self.w[name] = t.to(dev, torch.float32).contiguous()
            elif name.endswith("mlp.w_gate.weight") or name.endswith("mlp.w_up.weight"):
                continue
            else:
                self.w[name] = t.to(dev, BF16).contiguous()
        # SwiGLU up projections: [gate; up] rows interleaved for the GEMM's SwiGLU epilogue
        for name in weights:
            if name.endswith("mlp.w_gate.weight"):
                pre = name[: -len("w_gate.weight")]
                gate_up = torch.cat([weights[name], weights[pre + "w_up.weight"]]).to(dev, BF16)
                self.w[pre + "gate_up"] = ops.swiglu_interleave(gate_up).contiguous()
        for name in list(self.w):
            if name.endswith("scale_shift_table"):
                self.w[name] = self.w[name].reshape(-1).contiguous()
        self._ones: dict[int, torch.Tensor] = {}
        self._tables: dict[tuple[int, int, int], torch.Tensor] = {}
        dt, dh, dw = rope_split(cfg.head_dim)
        self.sections = (dt // 2, dh // 2, dw // 2)

    # ------------------------------------------------------------------ primitives
    def _one(self, n: int) -> torch.Tensor:
        if n not in self._ones:
            self._ones[n] = torch.ones(n, device=self.device, dtype=BF16)
        return self._ones[n]

    def _table(self, grid: tuple[int, int, int]) -> torch.Tensor:
        if grid not in self._tables:
            self._tables[grid] = rope_tables(self.cfg.head_dim, grid, self.cfg.rope_base).to(self.device)
        return self._tables[grid]

    def _linear(self, x: torch.Tensor, name: str, *, bias: bool = True,
                residual: torch.Tensor | None = None, out: torch.Tensor | None = None):
        """x (rows, k) @ W.T (+ bias) (+ residual, in place when out is residual)."""
        w = self.w[name + ".weight"]
        b = self.w[name + ".bias"] if bias else None
        if residual is None:
            return ops.linear(x, w, out, bias=b)
        return ops.linear(x, w, residual if out is None else out, bias=b,
                          kind=ops.EPI_GATED_RESIDUAL, residual=residual, gate=self._one(w.shape[0]))

    def _attention(self, x: torch.Tensor, normed: torch.Tensor, pre: str,
                   grid: tuple[int, int, int], window) -> torch.Tensor:
        """x += proj(neighborhood attention of `normed`): NeighborhoodAttention3D
        (diffusion_decoder.py:480-632) on one (T, H, W) volume of (tokens, C) rows."""
        c = x.shape[1]
        heads = c // 64
        qkv = self._linear(normed, pre + "qkv")
        q, k, v = ops.na_qkv_prepare(qkv, self.w[pre + "q_norm.weight"],
                                     self.w[pre + "k_norm.weight"], self._table(grid), grid,
                                     batch=1, heads=heads, section_pairs=self.sections,
                                     q_scale=self.cfg.head_dim ** -0.5, eps=1e-6)
        del qkv
        o = torch.empty(q.shape, device=self.device, dtype=BF16)
        ops.neighborhood_attention(q, k, v, window=tuple(window), out=o)
        del q, k, v
        return self._linear(o.view(x.shape[0], c), pre + "proj", residual=x)

    def _mlp(self, x: torch.Tensor, normed: torch.Tensor, pre: str) -> torch.Tensor:
        """x += w_down(silu(w_gate(n)) * w_up(n)) (TiledSwiGLU, :715-737)."""
        h = ops.linear(normed, self.w[pre + "gate_up"], kind=ops.EPI_SWIGLU, act_col_begin=0)
        return self._linear(h, pre + "w_down", bias=False, residual=x)

    def _det_block(self, x: torch.Tensor, pre: str, grid, window) -> torch.Tensor:
        """DeterministicNABlock (:755-799)."""
        x = self._attention(x, ops.rms_norm(x, self.w[pre + "norm1.weight"], 1e-6), pre + "attn.",
                            grid, window)
        return self._mlp(x, ops.rms_norm(x, self.w[pre + "norm2.weight"], 1e-6), pre + "mlp.")

    def _modulated(self, x: torch.Tensor, norm_w: torch.Tensor, vals: torch.Tensor,
                   i_scale: int, i_shift: int) -> torch.Tensor:
        c = x.shape[1]
        n = ops.rms_norm(x, norm_w, 1e-6)
        return ops.adaln(n.unsqueeze(0), vals[:, i_shift * c : (i_shift + 1) * c],
                         vals[:, i_scale * c : (i_scale + 1) * c],
                         norm=ops.NORM_NONE).squeeze(0)

    def _diff_block(self, x: torch.Tensor, ctx: torch.Tensor, mod: torch.Tensor, pre: str, grid,
                    window) -> torch.Tensor:
        """DiffusionNABlock (:827-898): modulation + scale_shift_table (scale, shift of the
        attention at 0, 1 and of the MLP at 3, 4; the gates are unused), context added, modulated
        norms before the attention and the SwiGLU."""
        vals = ops.add_rows(mod, self.w[pre + "scale_shift_table"])  # (1, 7C)
        x = self._linear(ctx, pre + "context_proj", residual=x)
        x = self._attention(x, self._modulated(x, self.w[pre + "norm1.weight"], vals, 0, 1),
                            pre + "attn.", grid, window)
        return self._mlp(x, self._modulated(x, self.w[pre + "norm2.weight"], vals, 3, 4),
                         pre + "mlp.")

    def _pixel_shuffle(self, x: torch.Tensor, pre: str, grid, stride,
                       drop_leading_frame: bool = True):
        """LinearPixelShuffle (:928-971): proj, then each row's (c, st, sh, sw) channels to
        space-time; the first frame dropped after a temporal doubling."""
        f, h, w = grid
        st, sh, sw = stride
        y = self._linear(x, pre + "proj")
        c = y.shape[1] // (st * sh * sw)
        out = torch.empty((f * st, h * sh, w * sw, c), device=self.device, dtype=BF16)
        src = y.view(f, h, w, c, st, sh, sw).permute(0, 4, 1, 5, 2, 6, 3)
        ops.copy_view(src, out.view(f, st, h, sh, w, sw, c))
        frames = f * st
        if st == 2 and drop_leading_frame:
            out = out[1:]
            frames -= 1
        return out.reshape(-1, c), (frames, h * sh, w * sw)

    # ------------------------------------------------------------------ stages
    def _prepare_latent(self, latent: torch.Tensor):
        """One (C, F, H, W) latent entry -> (tokens, C0) after the edge padding to the minimum
        grid (:1108-1129), the trailing frames (:1161-1168), the per-channel denormalisation and
        conv_in; also the padding before the crop."""
        cfg = self.cfg
        c, f, h, w = latent.shape
        mt, mh, mw = cfg.minimum_latent_shape()
        fp = max(f, mt) + cfg.trailing_pad_latent_frames
        hp, wp = max(h, mh), max(w, mw)
        hb, wb = (hp - h) // 2, (wp - w) // 2
        buf = torch.empty((1, c, fp, hp, wp), device=self.device, dtype=BF16)
        b0 = buf[0]
        ops.copy_view(latent, b0[:, :f, hb : hb + h, wb : wb + w])
        if fp > f:  # trailing frames repeat the last one
            ops.copy_view(b0[:, f - 1 : f, hb : hb + h, wb : wb + w].expand(c, fp - f, h, w),
                          b0[:, f:, hb : hb + h, wb : wb + w])
        if hb:
            ops.copy_view(b0[:, :, hb : hb + 1, wb : wb + w].expand(c, fp, hb, w), b0[:, :, :hb, wb : wb + w])
        if hp - hb - h:
            ops.copy_view(b0[:, :, hb + h - 1 : hb + h, wb : wb + w].expand(c, fp, hp - hb - h, w),
                          b0[:, :, hb + h :, wb : wb + w])
        if wb:
            ops.copy_view(b0[:, :, :, wb : wb + 1].expand(c, fp, hp, wb), b0[:, :, :, :wb])
        if wp - wb - w:
            ops.copy_view(b0[:, :, :, wb + w - 1 : wb + w].expand(c, fp, hp, wp - wb - w),
                          b0[:, :, :, wb + w :])
        tokens = ops.latent_to_bfhwc(buf, self.w["per_channel_statistics.std_of_means"],
                                     self.w["per_channel_statistics.mean_of_means"])
        x = self._linear(tokens.reshape(-1, c), "conv_in")
        return x, (fp, hp, wp), (hb, wb)

    def context(self, latent: torch.Tensor):
        """Stages 1-4 of one (C, F, H, W) entry: the context rows, its grid, the padding."""
        cfg = self.cfg
        x, grid, pad = self._prepare_latent(latent)
        for s in range(4):
            for i in range(cfg.stage_depths[s]):
                x = self._det_block(x, f"det_stages.{s}.{i}.", grid, cfg.stage_kernels[s])
            x, grid = self._pixel_shuffle(x, f"upsamples.{s}.", grid, cfg.upsample_strides[s])
        pad_frames = cfg.trailing_pad_latent_frames
        if pad_frames:  # the trailing ghost frames (:1199-1209)
            ghost = pad_frames * cfg.temporal_compression_ratio
            removable = max(grid[0] - cfg.stage5_kernel[0], 0)
            keep = grid[0] - min(ghost, removable)
            x = x[: keep * grid[1] * grid[2]]
            grid = (keep, grid[1], grid[2])
        return x, grid, pad

    def diffusion_step(self, ctx: torch.Tensor, grid, x_t: torch.Tensor, timestep: float):
        """forward_diffusion_step (:1225-1247) of one entry: ctx (tokens, C5) over `grid`, x_t
        (3, F, H * p, W * p) bf16 -> the model output, same shape, bf16."""
        cfg = self.cfg
        p = cfg.patch_size
        f, h, w = grid
        t = torch.full((1,), float(timestep) * cfg.timestep_scale_multiplier, device=self.device,
                       dtype=torch.float32)
        temb = ops.timestep_embedding(t, 256)
        temb = ops.gemv(temb, self.w["t_embedder.linear_1.weight"], self.w["t_embedder.linear_1.bias"])
        temb = ops.gemv(temb, self.w["t_embedder.linear_2.weight"], self.w["t_embedder.linear_2.bias"],
                        silu_input=True)
        mod = ops.gemv(temb, self.w["shared_adaln.proj.weight"], self.w["shared_adaln.proj.bias"],
                       silu_input=True)  # (1, 7 C5)
        # patchify: row (f, hp, wp), channel c * p * p + pw * p + ph (:49-72)
        cin = cfg.out_channels
        pix = cin * p * p
        patches = torch.empty((f, h, w, pix), device=self.device, dtype=BF16)
        src = x_t.view(cin, f, h, p, w, p).permute(1, 2, 4, 0, 5, 3)
        ops.copy_view(src, patches.view(f, h, w, cin, p, p))
        x = self._linear(patches.view(-1, pix), "conv_in_x_t")
        for i in range(cfg.stage_depths[4]):
            x = self._diff_block(x, ctx, mod, f"diff_blocks.{i}.", grid, cfg.stage5_kernel)
        x = ops.rms_norm(x, self.w["norm_out.weight"], 1e-6)
        y = self._linear(x, "conv_out")  # (tokens, pix)
        out = torch.empty((cin, f, h * p, w * p), device=self.device, dtype=BF16)
        src = y.view(f, h, w, cin, p, p).permute(3, 0, 1, 5, 2, 4)  # (c, f, h, ph, w, pw)
        ops.copy_view(src, out.view(cin, f, h, p, w, p))
        return out

    def denoise(self, ctx: torch.Tensor, grid, x_t: torch.Tensor, steps: int) -> torch.Tensor:
        """(:1250-1284): one x0 step returns the prediction; otherwise the prediction is turned
        into a velocity and x_t takes an Euler step per timestep."""
        ts = torch.linspace(1.0, 1.0 / steps, steps, dtype=torch.float32).tolist()
        if steps == 1 and self.cfg.model_output_type == "x0":
            return self.diffusion_step(ctx, grid, x_t, ts[0])
        for i, t in enumerate(ts):
            nxt = ts[i + 1] if i + 1 < steps else 0.0
            out = self.diffusion_step(ctx, grid, x_t, t)
            if self.cfg.model_output_type == "x0":
                x_t = ops.euler_denoised(x_t, out, t, nxt)
            else:
                x_t = ops.euler_velocity_step(x_t, out, t, nxt)
        return x_t

    def __call__(self, latent: torch.Tensor, noise: torch.Tensor, *,
                 steps: int | None = None) -> torch.Tensor:
        """DiffusionVideoDecoder.__call__ (:1295-1353) with x_t given: latent (B, C, F, H, W),
        noise (B, 3, F', H' * 32, W' * 32) = `cfg.working_pixel_shape(latent.shape)` -> video
        (B, 3, 1 + (F - 1) * 8, H * 32, W * 32) bf16."""
        cfg = self.cfg
        if latent.dim() == 4:
            latent = latent[None]
        if latent.dim() != 5 or latent.shape[1] != cfg.latent_channels:
            raise ValueError(f"expected a BCFHW latent with {cfg.latent_channels} channels, "
                             f"got {tuple(latent.shape)}")
        if any(d <= 0 for d in latent.shape):
            raise ValueError(f"latent dimensions must be positive, got {tuple(latent.shape)}")
        if tuple(noise.shape) != cfg.working_pixel_shape(latent.shape):
            raise ValueError(f"noise {tuple(noise.shape)} is not the working pixel shape "
                             f"{cfg.working_pixel_shape(latent.shape)}")
        b, _, f, h, w = latent.shape
        frames = 1 + (f - 1) * cfg.temporal_compression_ratio
        s = cfg.spatial_compression_ratio
        video = torch.empty((b, cfg.out_channels, frames, h * s, w * s), device=self.device,
                            dtype=BF16)
        for e in range(b):
            ctx, grid, (hb, wb) = self.context(latent[e])
            x_t = torch.empty(noise.shape[1:], device=self.device, dtype=BF16)
            ops.copy_view(noise[e], x_t)
            out = self.denoise(ctx, grid, x_t, steps or cfg.default_num_inference_steps)
            ops.copy_view(out[:, :frames, hb * s : hb * s + h * s, wb * s : wb * s + w * s],
                          video[e])
        return video
