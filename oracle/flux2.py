"""Flux2 (Klein) MMDiT and its Euler/CFG sampler restated on the CPU (test oracle).

Follows kinomlx/models/flux2/transformer.py and kinomlx/models/flux2/sampling.py line for line;
bf16 tensors are rounded exactly where the reference's MLX operations round (each bf16 op of an
MLX graph rounds its result; the reference's fp32-opmath kernels round once).

`FluxVariant` parameterises what BASELINE's timed configs change relative to Klein:
width/heads, GELU-tanh versus SwiGLU MLP, RoPE axes and theta, latent and text widths.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from .fused_ops import gelu_approx, layer_norm, linear, rms_norm, sdpa, silu


@dataclass(frozen=True)
class FluxVariant:
    dim: int
    heads: int
    mlp: str  # "gelu_tanh" or "swiglu"
    mlp_hidden: int  # activation width entering the MLP down projection
    rope_axes: tuple[int, ...]  # rotary dims per position axis, summing to head_dim
    rope_theta: float
    in_channels: int
    context_dim: int
    double_blocks: int
    single_blocks: int
    head_dim: int = 128

    @property
    def mlp_in(self) -> int:
        """Width of the MLP up projection (SwiGLU carries gate and content)."""
        return 2 * self.mlp_hidden if self.mlp == "swiglu" else self.mlp_hidden


# hidden 3072, 24 x 128 heads, GELU-tanh MLP x4, 2D axial RoPE with
# theta 10000 (64 rotary dims per axis), 64-channel patchified latents; text width 4096 (the
# configs do not give one).
BASELINE = FluxVariant(
    dim=3072,
    heads=24,
    mlp="gelu_tanh",
    mlp_hidden=12288,
    rope_axes=(64, 64),
    rope_theta=10000.0,
    in_channels=64,
    context_dim=4096,
    double_blocks=8,
    single_blocks=24,
)

# The reference's Klein 9B graph (kinomlx/models/flux2/transformer.py:17-29, 63-65, 110-111,
# 185-186; kinomlx/models/flux2/sampling.py:133-136).
KLEIN = FluxVariant(
    dim=4096,
    heads=32,
    mlp="swiglu",
    mlp_hidden=12288,
    rope_axes=(32, 32, 32, 32),
    rope_theta=2000.0,
    in_channels=128,
    context_dim=12288,
    double_blocks=8,
    single_blocks=24,
)


def rotary_positions(
    ids: torch.Tensor, variant: FluxVariant
) -> tuple[torch.Tensor, torch.Tensor]:
    """Independent axes with adjacent real/imaginary channel pairs
    (kinomlx/models/flux2/transformer.py:17-22): per axis of width d, frequencies
    theta^(-arange(0, d, 2) / d) in fp32; angles repeated pairwise; tables (B, N, 1, head_dim)."""
    parts = []
    for axis, width in enumerate(variant.rope_axes):
        freq = torch.tensor(variant.rope_theta, dtype=torch.float32) ** (
            -torch.arange(0, width, 2, dtype=torch.float32) / width
        )
        parts.append(ids[..., axis].to(torch.float32)[..., None] * freq)
    angles = torch.cat(parts, dim=-1).repeat_interleave(2, dim=-1)
    return torch.cos(angles)[:, :, None], torch.sin(angles)[:, :, None]


def rotate(value: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x * cos + perp(x) * sin in fp32, perp = (-x_odd, x_even) per pair, one rounding
    (kinomlx/models/flux2/transformer.py:25-29)."""
    f = value.float()
    pairs = f.reshape(*value.shape[:-1], -1, 2)
    perp = torch.stack([-pairs[..., 1], pairs[..., 0]], dim=-1).reshape(value.shape)
    return (f * cos + perp * sin).to(value.dtype)


def normalized(value: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """layer_norm(x, eps 1e-6, no affine) * (1 + scale) + shift, bf16 ops
    (kinomlx/models/flux2/transformer.py:56-60)."""
    return layer_norm(value, 1e-6) * (1 + scale) + shift


def swiglu(value: torch.Tensor) -> torch.Tensor:
    """silu(gate) * content with the gate first (kinomlx/models/flux2/transformer.py:63-65)."""
    gate, content = torch.chunk(value, 2, dim=-1)
    return silu(gate) * content


def activation(value: torch.Tensor, variant: FluxVariant) -> torch.Tensor:
    return swiglu(value) if variant.mlp == "swiglu" else gelu_approx(value)


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """SDPA with scale d^-1/2 on (B, N, H, d) operands (kinomlx/models/flux2/kv.py:48-54)."""
    return sdpa(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale=q.shape[-1] ** -0.5
    ).transpose(1, 2)


class ReferenceKV:
    """Post-RoPE reference-token keys and values of every layer, owned by one denoising call
    (kinomlx/models/flux2/kv.py:8-45): `extracting` until the first evaluation has stored them,
    `closed` once cleared."""

    def __init__(self, reference_tokens: int, layers: int):
        if reference_tokens < 1 or layers < 1:
            raise ValueError("Reference K/V requires positive token and layer counts")
        self.reference_tokens = reference_tokens
        self.layers: list[tuple[torch.Tensor, torch.Tensor] | None] = [None] * layers
        self.extracting = True
        self.closed = False

    def store(self, layer: int, key: torch.Tensor, value: torch.Tensor, start: int, count: int) -> None:
        self.layers[layer] = (key[:, start : start + count].clone(), value[:, start : start + count].clone())

    def tensors(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        entry = self.layers[layer]
        if entry is None:
            raise ValueError("Reference K/V has not been extracted")
        return entry

    def clear(self) -> None:
        self.layers = [None] * len(self.layers)
        self.closed = True


def reference_attention(q, k, v, *, text_tokens: int, state: ReferenceKV, layer: int) -> torch.Tensor:
    """Attention with reference K/V (kinomlx/models/flux2/kv.py:57-80) on post-RoPE (B, N, H, d):
    extracting, rows are [text, reference, target]; the reference rows' keys and values are
    stored, text and target queries attend to every key and reference queries to the reference
    keys only. Reusing, rows are [text, target] and the stored keys and values are inserted
    after the text's."""
    start = text_tokens
    if not state.extracting:
        rk, rv = state.tensors(layer)
        return attend(q, torch.cat([k[:, :start], rk, k[:, start:]], 1),
                      torch.cat([v[:, :start], rv, v[:, start:]], 1))
    end = start + state.reference_tokens
    state.store(layer, k, v, start, state.reference_tokens)
    active = attend(torch.cat([q[:, :start], q[:, end:]], 1), k, v)
    reference = attend(q[:, start:end], k[:, start:end], v[:, start:end])
    return torch.cat([active[:, :start], reference, active[:, start:]], 1)


def blend_modulation(current: torch.Tensor, reference: torch.Tensor, start: int, count: int,
                     length: int) -> torch.Tensor:
    """Per-row modulation (B, length, C): `reference` at rows [start, start + count), `current`
    elsewhere (kinomlx/models/flux2/kv.py:83-90)."""
    shape = (current.shape[0], length, current.shape[-1])
    expanded = current[:, None].expand(shape)
    fixed = reference[:, None].expand(shape[0], count, shape[-1])
    return torch.cat([expanded[:, :start], fixed, expanded[:, start + count :]], 1)


def joint_attention(q, k, v, cos, sin, *, text_tokens: int = 0,
                    reference_kv: ReferenceKV | None = None, layer: int = 0) -> torch.Tensor:
    """Rotate q and k, attend (plain, or with reference K/V), back to (B, N, H*d)
    (kinomlx/models/flux2/transformer.py:35-53)."""
    q, k = rotate(q, cos, sin), rotate(k, cos, sin)
    if reference_kv is None:
        out = attend(q, k, v)
    else:
        out = reference_attention(q, k, v, text_tokens=text_tokens, state=reference_kv, layer=layer)
    return out.reshape(*q.shape[:2], -1)


def _rows(mod: torch.Tensor) -> torch.Tensor:
    """One modulation per batch entry (B, C) or per row (B, N, C), as (B, 1|N, C)."""
    return mod[:, None] if mod.dim() == 2 else mod


def _heads(x: torch.Tensor, variant: FluxVariant) -> torch.Tensor:
    return x.reshape(*x.shape[:2], variant.heads, variant.head_dim)


def feed_forward(p: dict, prefix: str, x: torch.Tensor, variant: FluxVariant) -> torch.Tensor:
    """linear_out(act(linear_in(x))) (kinomlx/models/flux2/transformer.py:78-85)."""
    h = linear(x, p[f"{prefix}.linear_in.weight"])
    return linear(activation(h, variant), p[f"{prefix}.linear_out.weight"])


def double_block(
    p: dict,
    i: int,
    image: torch.Tensor,
    text: torch.Tensor,
    image_mod: torch.Tensor,
    text_mod: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    variant: FluxVariant,
    reference_kv: ReferenceKV | None = None,
    layer: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """DoubleBlock + DoubleAttention (kinomlx/models/flux2/transformer.py:88-167); `image_mod`
    is (B, 6D) or per image row (B, Ni, 6D)."""
    a = f"transformer_blocks.{i}"
    shift, scale, gate, ff_shift, ff_scale, ff_gate = torch.chunk(_rows(image_mod), 6, dim=-1)
    ts, tc, tg, fs, fc, fg = torch.chunk(text_mod[:, None], 6, dim=-1)
    img_n = normalized(image, shift, scale)
    txt_n = normalized(text, ts, tc)
    w = lambda name: p[f"{a}.attn.{name}.weight"]
    query = torch.cat(
        [
            rms_norm(_heads(linear(txt_n, w("add_q_proj")), variant), w("norm_added_q"), 1e-6),
            rms_norm(_heads(linear(img_n, w("to_q")), variant), w("norm_q"), 1e-6),
        ],
        dim=1,
    )
    key = torch.cat(
        [
            rms_norm(_heads(linear(txt_n, w("add_k_proj")), variant), w("norm_added_k"), 1e-6),
            rms_norm(_heads(linear(img_n, w("to_k")), variant), w("norm_k"), 1e-6),
        ],
        dim=1,
    )
    value = torch.cat(
        [_heads(linear(txt_n, w("add_v_proj")), variant), _heads(linear(img_n, w("to_v")), variant)],
        dim=1,
    )
    nt = text.shape[1]
    result = joint_attention(query, key, value, cos, sin, text_tokens=nt,
                             reference_kv=reference_kv, layer=layer)
    ai = linear(result[:, nt:], w("to_out.0"))
    at = linear(result[:, :nt], w("to_add_out"))
    image, text = image + gate * ai, text + tg * at
    image = image + ff_gate * feed_forward(p, f"{a}.ff", normalized(image, ff_shift, ff_scale), variant)
    text = text + fg * feed_forward(p, f"{a}.ff_context", normalized(text, fs, fc), variant)
    return image, text


def single_block(
    p: dict,
    i: int,
    value: torch.Tensor,
    modulation: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    variant: FluxVariant,
    reference_kv: ReferenceKV | None = None,
    layer: int = 0,
    text_tokens: int = 0,
) -> torch.Tensor:
    """SingleBlock + SingleAttention (kinomlx/models/flux2/transformer.py:170-220);
    `modulation` is (B, 3D) or per row (B, N, 3D)."""
    a = f"single_transformer_blocks.{i}.attn"
    shift, scale, gate = torch.chunk(_rows(modulation), 3, dim=-1)
    x = normalized(value, shift, scale)
    d = variant.dim
    fused = linear(x, p[f"{a}.to_qkv_mlp_proj.weight"])
    q, k, v, mlp = fused[..., :d], fused[..., d : 2 * d], fused[..., 2 * d : 3 * d], fused[..., 3 * d :]
    attention = joint_attention(
        rms_norm(_heads(q, variant), p[f"{a}.norm_q.weight"], 1e-6),
        rms_norm(_heads(k, variant), p[f"{a}.norm_k.weight"], 1e-6),
        _heads(v, variant),
        cos,
        sin,
        text_tokens=text_tokens,
        reference_kv=reference_kv,
        layer=layer,
    )
    out = linear(torch.cat([attention, activation(mlp, variant)], dim=-1), p[f"{a}.to_out.weight"])
    return value + gate * out


def timestep_embedding(p: dict, timestep: torch.Tensor) -> torch.Tensor:
    """Sinusoid(256) of the timestep -> linear_1 -> SiLU -> linear_2
    (kinomlx/models/flux2/transformer.py:232-242)."""
    freq = torch.exp(-math.log(10000) * torch.arange(128, dtype=torch.float32) / 128)
    angles = timestep.to(torch.float32)[:, None] * freq
    emb = torch.cat([torch.cos(angles), torch.sin(angles)], dim=-1).to(timestep.dtype)
    pre = "time_guidance_embed.timestep_embedder"
    return linear(silu(linear(emb, p[f"{pre}.linear_1.weight"])), p[f"{pre}.linear_2.weight"])


def modulation(p: dict, name: str, embedding: torch.Tensor) -> torch.Tensor:
    """linear(silu(embedding)) (kinomlx/models/flux2/transformer.py:223-229)."""
    return linear(silu(embedding), p[f"{name}.linear.weight"])


def output_norm(p: dict, value: torch.Tensor, embedding: torch.Tensor) -> torch.Tensor:
    """scale, shift = linear(silu(emb)); normalized(value, shift, scale)
    (kinomlx/models/flux2/transformer.py:251-258)."""
    scale, shift = torch.chunk(modulation(p, "norm_out", embedding), 2, dim=-1)
    return normalized(value, shift[:, None], scale[:, None])


def forward(
    p: dict,
    text: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    image: torch.Tensor,
    timestep: torch.Tensor,
    variant: FluxVariant,
    *,
    reference_kv: ReferenceKV | None = None,
) -> torch.Tensor:
    """Flux2Transformer._forward with projected text (kinomlx/models/flux2/transformer.py:307-358).
    With `reference_kv` extracting, `image` is [reference, target] rows: the reference rows take
    the modulations of timestep 0 and the velocity covers the target rows only."""
    embedding = timestep_embedding(p, timestep.to(image.dtype) * 1000)
    im = modulation(p, "double_stream_modulation_img", embedding)
    tm = modulation(p, "double_stream_modulation_txt", embedding)
    sm = modulation(p, "single_stream_modulation", embedding)
    layers = variant.double_blocks + variant.single_blocks
    reference_tokens = 0
    if reference_kv is not None:
        if reference_kv.closed:
            raise ValueError("Reference K/V belongs to a completed generation")
        if len(reference_kv.layers) != layers:
            raise ValueError("Reference K/V layer count does not match the transformer")
        if reference_kv.extracting:
            reference_tokens = reference_kv.reference_tokens
            if reference_tokens >= image.shape[1]:
                raise ValueError("KV extraction requires reference tokens followed by target tokens")
            fixed = timestep_embedding(p, torch.zeros_like(timestep).to(image.dtype))
            im = blend_modulation(im, modulation(p, "double_stream_modulation_img", fixed), 0,
                                  reference_tokens, image.shape[1])
            sm = blend_modulation(sm, modulation(p, "single_stream_modulation", fixed),
                                  text.shape[1], reference_tokens, text.shape[1] + image.shape[1])
    image = linear(image, p["x_embedder.weight"])
    for i in range(variant.double_blocks):
        image, text = double_block(p, i, image, text, im, tm, cos, sin, variant, reference_kv, i)
    value = torch.cat([text, image], dim=1)
    for i in range(variant.single_blocks):
        value = single_block(p, i, value, sm, cos, sin, variant, reference_kv,
                             variant.double_blocks + i, text.shape[1])
    out = output_norm(p, value[:, text.shape[1] + reference_tokens :], embedding)
    return linear(out, p["proj_out.weight"])


def prepare(p: dict, text: torch.Tensor, ids: torch.Tensor, variant: FluxVariant):
    """Once per generation: context_embedder and the RoPE tables
    (kinomlx/models/flux2/transformer.py:283-292)."""
    cos, sin = rotary_positions(ids, variant)
    return linear(text, p["context_embedder.weight"]), cos, sin


def schedule(image_tokens: int, steps: int) -> torch.Tensor:
    """Empirical Klein shift (kinomlx/models/flux2/sampling.py:95-106)."""
    if image_tokens < 1 or steps < 1:
        raise ValueError("Schedule requires positive target token and step counts")
    long = 0.00016927 * image_tokens + 0.45666666
    short = 8.73809524e-05 * image_tokens + 1.89833333
    mu = long if image_tokens > 4300 else long + (short - long) * (200 - steps) / 190
    factor = math.exp(mu)
    sigma = torch.tensor([1 - i / steps for i in range(steps)], dtype=torch.float32)
    shifted = factor / (factor + (1 / sigma - 1))
    return torch.cat([shifted, torch.zeros(1, dtype=torch.float32)])


def linear_sigmas(steps: int) -> torch.Tensor:
    """BASELINE's explicit schedule: linearly spaced 1.0 -> 0.0 (steps + 1 values) in fp32."""
    return torch.from_numpy(np.linspace(1.0, 0.0, steps + 1).astype(np.float32))


def euler_step(current: torch.Tensor, velocity: torch.Tensor, delta: torch.Tensor) -> torch.Tensor:
    """dt rounded to the model dtype, times v in the model dtype, added in fp32
    (kinomlx/models/flux2/sampling.py:109-113)."""
    increment = delta.to(velocity.dtype) * velocity
    return (current.float() + increment.float()).to(current.dtype)


def step_timestep(sigmas: torch.Tensor, index: int, dtype: torch.dtype) -> torch.Tensor:
    """((sigma * 1000) in the model dtype / 1000) in the model dtype
    (kinomlx/models/flux2/sampling.py:209-212)."""
    return ((sigmas[index : index + 1] * 1000).to(dtype) / 1000).to(dtype)


def denoise(
    p: dict,
    noise: torch.Tensor,
    text: torch.Tensor,
    ids: torch.Tensor,
    sigmas: torch.Tensor,
    variant: FluxVariant,
    *,
    negative: torch.Tensor | None = None,
    guidance: float = 1.0,
    steps: int | None = None,
    references: torch.Tensor | None = None,
) -> torch.Tensor:
    """The Euler loop of kinomlx/models/flux2/sampling.py:116-281 with batched CFG when a
    negative text is given (cond first, uncond second, `uncond + g * (cond - uncond)`). With
    `references` (1, Nr, C), every evaluation sees [target, reference] rows and `ids` holds the
    [text, target, reference] positions; the velocity is the target rows'
    (sampling.py:193-197, 255-281)."""
    count = len(sigmas) - 1 if steps is None else steps
    conditioned = text if negative is None else torch.cat([text, negative])
    projected, cos, sin = prepare(p, conditioned, ids, variant)
    current = noise
    for i in range(count):
        t = step_timestep(sigmas, i, noise.dtype)
        image = current if references is None else torch.cat([current, references], 1)
        if negative is None:
            velocity = forward(p, projected, cos, sin, image, t, variant)
        else:
            both = forward(p, projected, cos, sin, torch.cat([image, image]), torch.cat([t, t]), variant)
            positive, uncond = torch.chunk(both, 2, dim=0)
            velocity = uncond + guidance * (positive - uncond)
        velocity = velocity[:, : current.shape[1]]
        current = euler_step(current, velocity, sigmas[i + 1] - sigmas[i])
    return current


def kv_loop(predict, reuse, new_cache, references: torch.Tensor, noise: torch.Tensor,
            sigmas: torch.Tensor, *, recompute: bool = False) -> torch.Tensor:
    """The KV-editing branch of the Euler loop (kinomlx/models/flux2/sampling.py:206-252): a
    cache is extracted from [reference, target] rows at the first evaluation (at every one with
    `recompute`) and reused on target rows after that; the cache is cleared when the loop ends
    or fails. `predict`/`reuse`(image, timestep, cache) return the target velocity."""
    current, cache = noise, None
    try:
        for i in range(len(sigmas) - 1):
            t = step_timestep(sigmas, i, noise.dtype)
            if cache is None:
                cache = new_cache(references.shape[1])
            if cache.extracting:
                velocity = predict(torch.cat([references, current], 1), t, cache)
            else:
                velocity = reuse(current, t, cache)
            cache.extracting = False
            if recompute:
                cache.clear()
                cache = None
            current = euler_step(current, velocity, sigmas[i + 1] - sigmas[i])
    finally:
        if cache is not None:
            cache.clear()
    return current


def denoise_kv(
    p: dict,
    noise: torch.Tensor,
    text: torch.Tensor,
    text_ids: torch.Tensor,
    image_ids: torch.Tensor,
    references: torch.Tensor,
    reference_ids: torch.Tensor,
    sigmas: torch.Tensor,
    variant: FluxVariant,
    *,
    recompute: bool = False,
) -> torch.Tensor:
    """Klein KV editing (kinomlx/models/flux2/sampling.py:186-190, 206-252): the text projected
    once, RoPE tables for the [text, reference, target] extraction rows and the [text, target]
    reuse rows."""
    projected = linear(text, p["context_embedder.weight"])
    cx, sx = rotary_positions(torch.cat([text_ids, reference_ids, image_ids], 1), variant)
    cr, sr = rotary_positions(torch.cat([text_ids, image_ids], 1), variant)
    layers = variant.double_blocks + variant.single_blocks
    return kv_loop(
        lambda image, t, cache: forward(p, projected, cx, sx, image, t, variant, reference_kv=cache),
        lambda image, t, cache: forward(p, projected, cr, sr, image, t, variant, reference_kv=cache),
        lambda count: ReferenceKV(count, layers),
        references, noise, sigmas, recompute=recompute)


def image_ids(height: int, width: int, axes: int) -> torch.Tensor:
    """Positions (1, h*w, axes) of a row-major token grid: the last two axes hold (row, col)."""
    rows = torch.arange(height).repeat_interleave(width)
    cols = torch.arange(width).repeat(height)
    ids = torch.zeros((1, height * width, axes), dtype=torch.int64)
    ids[0, :, axes - 2] = rows
    ids[0, :, axes - 1] = cols
    return ids
