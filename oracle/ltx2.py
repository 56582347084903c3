"""LTX-2 video DiT (video stream only) restated on the CPU (test oracle).

Follows kinomlx/models/ltx2/transformer/{rope,attention,feed_forward,timestep,transformer,model,
wrappers}.py, kinomlx/models/ltx2/patchifier.py and kinomlx/samplers/steps.py. Every bf16
operation rounds where the reference's MLX operation does; fp32-opmath kernels round once.
"""

from __future__ import annotations

import math
import struct
from dataclasses import dataclass

import torch

from .fused_ops import gelu_approx, layer_norm, linear, linear_then_bias, rms_norm, sdpa, silu


@dataclass(frozen=True)
class LTXVariant:
    dim: int = 4096
    heads: int = 32
    head_dim: int = 128
    context_dim: int = 4096
    ff_mult: int = 4
    gated_attention: bool = True
    eps: float = 1e-6
    theta: float = 10000.0
    max_pos: tuple[int, int, int] = (20, 2048, 2048)
    in_channels: int = 128
    out_channels: int = 128
    blocks: int = 48
    timestep_scale: float = 1000.0
    # the block linears packed (the reference's transformer_quantize modes): each runs as a
    # quantised matmul rounded to bf16, then + bias (weights/quantization.py:32-43)
    packed_blocks: bool = False


def _blin(v: LTXVariant):
    return linear_then_bias if getattr(v, "packed_blocks", False) else linear


def _f32(x: float) -> float:
    return struct.unpack("<f", struct.pack("<f", x))[0]


# kinomlx/models/ltx2/sigmas.py:24-52
DISTILLED_STAGE_1_SIGMAS = tuple(
    _f32(x) for x in (1.0, 0.99375, 0.9875, 0.98125, 0.975, 0.909375, 0.725, 0.421875, 0.0)
)
DISTILLED_STAGE_2_SIGMAS = tuple(_f32(x) for x in (0.909375, 0.725, 0.421875, 0.0))


# ----------------------------------------------------------------------------- positions / RoPE
def patch_grid_bounds(frames: int, height: int, width: int) -> torch.Tensor:
    """(1, 3, N, 2) latent-grid start/end bounds for patch size 1, row-major (f, h, w)
    (kinomlx/models/ltx2/patchifier.py:102-118)."""
    f, h, w = torch.meshgrid(torch.arange(frames), torch.arange(height), torch.arange(width),
                             indexing="ij")
    starts = torch.stack([f, h, w]).reshape(3, -1)
    return torch.stack([starts, starts + 1], dim=-1)[None].to(torch.float32)


def pixel_coords(latent: torch.Tensor, scale=(8, 32, 32), causal_fix: bool = True,
                 fps: float = 24.0) -> torch.Tensor:
    """Latent bounds to pixel bounds, causal fix on time, time divided by fps
    (kinomlx/models/ltx2/patchifier.py:121-146, kinomlx/models/ltx2/conditioning/tools.py:63-74)."""
    s = torch.tensor(scale, dtype=torch.float32).reshape(1, 3, 1, 1)
    pix = latent * s
    if causal_fix:
        t = torch.clamp(pix[:, 0] + 1 - scale[0], min=0)
        pix = torch.cat([t[:, None], pix[:, 1:]], dim=1)
    pix = pix.to(torch.float32)
    return torch.cat([pix[:, 0:1] / fps, pix[:, 1:]], dim=1)


def frequency_grid(theta: float, axes: int, inner_dim: int) -> tuple[float, ...]:
    """theta^(i/(n-1)) * pi/2 in host double precision (kinomlx/models/ltx2/transformer/rope.py:75-92)."""
    count = inner_dim // (2 * axes)
    exps = (0.0,) if count == 1 else tuple(i / (count - 1) for i in range(count))
    return tuple(math.pow(theta, e) * math.pi / 2 for e in exps)


def precompute_freqs_cis(
    positions: torch.Tensor,
    *,
    dim: int,
    theta: float = 10000.0,
    max_pos: tuple[int, ...] = (20, 2048, 2048),
    heads: int = 32,
    middle: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Split-RoPE cos/sin tables (B, heads, T, dim/(2*heads)) in fp32
    (kinomlx/models/ltx2/transformer/rope.py:95-176)."""
    if middle:
        pos = (positions[..., 0] + positions[..., 1]) / 2.0
    else:
        pos = positions[..., 0]
    scale = torch.tensor(max_pos, dtype=torch.float32)[None, :, None]
    frac = (pos.to(torch.float32) / scale).transpose(1, 2)  # (B, T, axes)
    grid = torch.tensor(frequency_grid(theta, positions.shape[1], dim), dtype=torch.float32)
    scaled = frac * 2.0 - 1.0
    freqs = scaled[..., None] * grid[None, None, None, :]  # (B, T, axes, count)
    freqs = freqs.transpose(2, 3).reshape(freqs.shape[0], freqs.shape[1], -1)
    pad = dim // 2 - freqs.shape[-1]
    cos, sin = torch.cos(freqs), torch.sin(freqs)
    if pad:
        cos = torch.cat([torch.ones((*cos.shape[:-1], pad)), cos], dim=-1)
        sin = torch.cat([torch.zeros((*sin.shape[:-1], pad)), sin], dim=-1)
    b, t, _ = cos.shape
    cos = cos.reshape(b, t, heads, -1).transpose(1, 2)
    sin = sin.reshape(b, t, heads, -1).transpose(1, 2)
    return cos.contiguous(), sin.contiguous()


def apply_split_rotary_emb(value: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Split-half rotation on flattened heads with fp32 tables (B|1, H, T, D/2): one fp32 rounding
    per product, then the difference or sum, then the cast
    (kinomlx/models/ltx2/transformer/rope.py:18-61, kinomlx/kernels/split_rope.py:35-56, 87-98)."""
    b, t, _ = value.shape
    heads, half = cos.shape[1], cos.shape[-1]
    hf = value.reshape(b, t, heads, 2 * half).transpose(1, 2).float()
    first, second = hf[..., :half], hf[..., half:]
    out = torch.cat([first * cos - second * sin, first * sin + second * cos], dim=-1)
    return out.transpose(1, 2).reshape(value.shape).to(value.dtype)


# ----------------------------------------------------------------------------- timestep / AdaLN
def timestep_features(t: torch.Tensor, dim: int = 256) -> torch.Tensor:
    """Canonical cos-then-sin features in fp32 (kinomlx/models/ltx2/transformer/timestep.py:13-28)."""
    half = dim // 2
    exponent = -math.log(10000) * torch.arange(half, dtype=torch.float32) / half
    angles = t[:, None].to(torch.float32) * torch.exp(exponent)[None, :]
    return torch.cat([torch.cos(angles), torch.sin(angles)], dim=-1)


def adaln_single(p: dict, prefix: str, t: torch.Tensor, dtype: torch.dtype):
    """AdaLayerNormSingle: timestep MLP then linear(silu(emb)) (timestep.py:31-85)."""
    x = timestep_features(t).to(dtype)
    x = silu(linear(x, p[f"{prefix}.emb.timestep_embedder.linear_1.weight"],
                    p[f"{prefix}.emb.timestep_embedder.linear_1.bias"]))
    emb = linear(x, p[f"{prefix}.emb.timestep_embedder.linear_2.weight"],
                 p[f"{prefix}.emb.timestep_embedder.linear_2.bias"])
    mod = linear(silu(emb), p[f"{prefix}.linear.weight"], p[f"{prefix}.linear.bias"])
    return mod, emb


def adaln(value, scale, shift, eps):
    """rms_norm(x) * (1 + scale) + shift in bf16 ops (ltx2/transformer/transformer.py:16-23)."""
    return (rms_norm(value, None, eps) * (1.0 + scale) + shift).to(value.dtype)


# ----------------------------------------------------------------------------- attention / FF
def context_mask_bias(mask, dtype=torch.bfloat16):
    """ModalityPreprocessor._context_mask (kinomlx/models/ltx2/transformer/preprocessing.py:85-96):
    a floating-point text mask is an additive bias, cast to the compute dtype and shaped
    (B, 1, 1|Tq, Tk); any other mask becomes (mask - 1) * -min(dtype), with min -65504 for fp16
    and -3.3895313892515355e38 otherwise (preprocessing.py:14-17)."""
    if mask is None:
        return None
    if mask.dtype in (torch.float16, torch.bfloat16, torch.float32):
        if mask.dim() == 2:
            mask = mask[:, None, None, :]
        elif mask.dim() == 3:
            mask = mask[:, None, :, :]
        return mask.to(dtype)
    minimum = -65504.0 if dtype == torch.float16 else -3.3895313892515355e38
    bias = (mask.to(dtype) - 1.0) * -minimum
    return bias.to(dtype).reshape(mask.shape[0], 1, -1, mask.shape[-1])


def attention(p: dict, prefix: str, x: torch.Tensor, v: LTXVariant, *, context=None, pe=None,
              k_pe=None, mask=None):
    """Gated attention with Q/K RMSNorm over all heads and split RoPE; the keys take `k_pe` when
    given (the A/V cross-attention), else `pe`; `mask` is an additive bias over the keys
    (kinomlx/models/ltx2/transformer/attention.py:249-371)."""
    g = lambda name: p[f"{prefix}.{name}"]
    lin = _blin(v)
    gate = None
    if v.gated_attention:
        gate = 2.0 * torch.sigmoid(lin(x, g("to_gate_logits.weight"), g("to_gate_logits.bias")).float()).to(x.dtype)
    src = x if context is None else context
    value = lin(src, g("to_v.weight"), g("to_v.bias"))
    q = rms_norm(lin(x, g("to_q.weight"), g("to_q.bias")), g("q_norm.weight"), v.eps)
    k = rms_norm(lin(src, g("to_k.weight"), g("to_k.bias")), g("k_norm.weight"), v.eps)
    if pe is not None:
        q = apply_split_rotary_emb(q, *pe)
        k = apply_split_rotary_emb(k, *(pe if k_pe is None else k_pe))
    b, tq, _ = q.shape
    tk = k.shape[1]
    heads, d = v.heads, v.head_dim
    out = sdpa(q.reshape(b, tq, heads, d).transpose(1, 2), k.reshape(b, tk, heads, d).transpose(1, 2),
               value.reshape(b, tk, heads, d).transpose(1, 2), d ** -0.5, mask)
    out = out.transpose(1, 2)
    if gate is not None:
        out = out * gate[..., None]
    out = out.reshape(b, tq, heads * d)
    return lin(out, g("to_out.weight"), g("to_out.bias"))


def feed_forward(p: dict, prefix: str, x: torch.Tensor, lin=linear) -> torch.Tensor:
    """proj -> GELU-tanh (fp32 opmath) -> proj (ltx2/transformer/feed_forward.py:37-97)."""
    h = gelu_approx(lin(x, p[f"{prefix}.project_in.proj.weight"], p[f"{prefix}.project_in.proj.bias"]))
    return lin(h, p[f"{prefix}.project_out.weight"], p[f"{prefix}.project_out.bias"])


def video_block(p: dict, i: int, x, context, timesteps, prompt_timestep, pe, v: LTXVariant,
                context_mask=None):
    """BasicAVTransformerBlock, video stream without audio (ltx2/transformer/transformer.py:178-392).
    timesteps: (B, 1, 9, D) modulation; prompt_timestep: (B, 1, 2, D); context_mask: the
    additive bias of context_mask_bias."""
    a = f"transformer_blocks.{i}"
    table = p[f"{a}.scale_shift_table"]
    vals = (table[None, None] + timesteps)  # bf16 op
    shift, scale, gate = vals[:, :, 0], vals[:, :, 1], vals[:, :, 2]
    normalized = adaln(x, scale, shift, v.eps)
    attended = attention(p, f"{a}.attn1", normalized, v, pe=pe)
    x = (x + attended * gate).to(x.dtype)
    shift_q, scale_q, gate_c = vals[:, :, 6], vals[:, :, 7], vals[:, :, 8]
    prompt = p[f"{a}.prompt_scale_shift_table"][None, None] + prompt_timestep
    shift_ctx, scale_ctx = prompt[:, :, 0], prompt[:, :, 1]
    query = adaln(x, scale_q, shift_q, v.eps)
    ctx = (context * (1.0 + scale_ctx) + shift_ctx).to(context.dtype)
    cross = attention(p, f"{a}.attn2", query, v, context=ctx, mask=context_mask)
    x = (x + (cross * gate_c).to(x.dtype)).to(x.dtype)
    shift, scale, gate = vals[:, :, 3], vals[:, :, 4], vals[:, :, 5]
    normalized = adaln(x, scale, shift, v.eps)
    return (x + feed_forward(p, f"{a}.ff", normalized, _blin(v)) * gate).to(x.dtype)


def forward(p: dict, latent, context, sigma: float, positions, v: LTXVariant, dtype=torch.bfloat16,
            context_mask=None):
    """LTXAVModel.__call__ for the video modality with a uniform timestep
    (ltx2/transformer/model.py:577-635, preprocessing.py:134-213); `context_mask` is the raw
    text mask (padded prompts)."""
    bias = context_mask_bias(context_mask, dtype)
    b = latent.shape[0]
    hidden = linear(latent, p["patchify_proj.weight"], p["patchify_proj.bias"])
    t = torch.full((b,), sigma, dtype=torch.float32)
    mod, emb = adaln_single(p, "adaln_single", t * v.timestep_scale, dtype)
    timesteps = mod.reshape(b, -1, 9, v.dim)
    emb = emb.reshape(b, -1, v.dim)
    pmod, _ = adaln_single(p, "prompt_adaln_single", t * v.timestep_scale, dtype)
    prompt = pmod.reshape(b, -1, 2, v.dim)
    pe = precompute_freqs_cis(positions, dim=v.dim, theta=v.theta, max_pos=v.max_pos, heads=v.heads)
    for i in range(v.blocks):
        hidden = video_block(p, i, hidden, context, timesteps, prompt, pe, v, bias)
    modulation = (p["scale_shift_table"][None, None] + emb[:, :, None, :]).to(hidden.dtype)
    shift, scale = modulation[:, :, 0], modulation[:, :, 1]
    hidden = (layer_norm(hidden, v.eps) * (1.0 + scale) + shift).to(hidden.dtype)
    return linear(hidden, p["proj_out.weight"], p["proj_out.bias"])


def to_denoised(latent, sigma: float, velocity):
    """x0 = x - t * v in fp32 (ltx2/transformer/wrappers.py:49-65)."""
    return (latent.float() - torch.tensor(sigma, dtype=torch.float32) * velocity.float()).to(latent.dtype)


def euler_step(sample, denoised, sigma: float, sigma_next: float):
    """denoised + (s'/s)(sample - denoised) in fp32 (kinomlx/samplers/steps.py:36-70)."""
    ratio = torch.tensor(sigma_next / sigma, dtype=torch.float32)
    return (denoised.float() + ratio * (sample.float() - denoised.float())).to(sample.dtype)


def denoise(p, latent, context, positions, sigmas, v: LTXVariant, context_mask=None):
    """Deterministic-Euler loop (kinomlx/models/ltx2/denoise.py:159-365); the model dtype (which
    the timestep features are cast to) is the latent's."""
    x = latent
    for s, n in zip(sigmas[:-1], sigmas[1:]):
        velocity = forward(p, x, context, s, positions, v, dtype=latent.dtype,
                           context_mask=context_mask)
        x = euler_step(x, to_denoised(x, s, velocity), s, n)
    return x


# ----------------------------------------------------------------------------- joint audio/video
@dataclass(frozen=True)
class LTXAVVariant:
    """LTXAVModel's two streams (kinomlx/models/ltx2/transformer/model.py:137-236): the video
    stream, the audio stream (64-wide heads, one position axis), and the A/V cross-attention,
    which runs on the audio stream's heads (equal head counts are required, model.py:185-186)."""

    video: LTXVariant
    audio: LTXVariant
    av_gate_scale: float = 1000.0


# the reference's default audio stream (model.py:141-153): 32 heads x 64, context 2048, one axis
AUDIO = LTXVariant(dim=2048, heads=32, head_dim=64, context_dim=2048, max_pos=(20,))


def modulate(value: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    """(value * (1 + scale) + shift) in the value's dtype (ltx2/transformer/transformer.py:33-34)."""
    return (value * (1.0 + scale) + shift).to(value.dtype)


def av_values(table: torch.Tensor, scale_shift: torch.Tensor, gate: torch.Tensor):
    """_av_ada_values (transformer.py:188-199): table rows 0-3 plus the (B, 1, 4, D) scale/shift
    timestep, row 4 plus the (B, 1, 1, D) gate timestep; returns scale_a2v, shift_a2v, scale_v2a,
    shift_v2a, gate."""
    ss = table[:4][None, None] + scale_shift
    g = table[4:5][None, None] + gate
    return ss[:, :, 0], ss[:, :, 1], ss[:, :, 2], ss[:, :, 3], g[:, :, 0]


def _stream_self_and_text(p, a, prefix, x, context, timesteps, prompt_timestep, pe, v, mask=None):
    """The self-attention and text cross-attention of one stream (transformer.py:249-320)."""
    table = p[f"{a}.{prefix}scale_shift_table"]
    vals = table[None, None] + timesteps
    attended = attention(p, f"{a}.{prefix}attn1", adaln(x, vals[:, :, 1], vals[:, :, 0], v.eps), v, pe=pe)
    x = (x + attended * vals[:, :, 2]).to(x.dtype)
    prompt = p[f"{a}.{prefix}prompt_scale_shift_table"][None, None] + prompt_timestep
    query = adaln(x, vals[:, :, 7], vals[:, :, 6], v.eps)
    ctx = modulate(context, prompt[:, :, 1], prompt[:, :, 0])
    cross = attention(p, f"{a}.{prefix}attn2", query, v, context=ctx, mask=mask)
    return (x + (cross * vals[:, :, 8]).to(x.dtype)).to(x.dtype)


def _stream_ff(p, a, prefix, x, timesteps, v):
    """The stream's feed-forward with its gated residual (transformer.py:373-413)."""
    vals = p[f"{a}.{prefix}scale_shift_table"][None, None] + timesteps
    ff = feed_forward(p, f"{a}.{prefix}ff", adaln(x, vals[:, :, 4], vals[:, :, 3], v.eps), _blin(v))
    return (x + ff * vals[:, :, 5]).to(x.dtype)


def av_block(p: dict, i: int, vx, ax, vctx, actx, vt, at, vprompt, aprompt, vpe, ape, vxpe,
             axpe, vcss, vcg, acss, acg, v: LTXAVVariant, vmask=None, amask=None):
    """BasicAVTransformerBlock with both streams and both cross-modal attentions
    (kinomlx/models/ltx2/transformer/transformer.py:225-413). vt/at: (B, 1, 9, D) modulations;
    vprompt/aprompt: (B, 1, 2, D); vcss/acss: (B, 1, 4, D) cross scale/shift; vcg/acg:
    (B, 1, 1, D) cross gates; pe tables (B|1, heads, T, half)."""
    a = f"transformer_blocks.{i}"
    V, A = v.video, v.audio
    vx = _stream_self_and_text(p, a, "", vx, vctx, vt, vprompt, vpe, V, vmask)
    ax = _stream_self_and_text(p, a, "audio_", ax, actx, at, aprompt, ape, A, amask)
    vbase, abase = vx, ax
    vnorm = rms_norm(vbase, None, V.eps)
    anorm = rms_norm(abase, None, A.eps)
    a_sc_a2v, a_sh_a2v, a_sc_v2a, a_sh_v2a, g_v2a = av_values(
        p[f"{a}.scale_shift_table_a2v_ca_audio"], acss, acg)
    v_sc_a2v, v_sh_a2v, v_sc_v2a, v_sh_v2a, g_a2v = av_values(
        p[f"{a}.scale_shift_table_a2v_ca_video"], vcss, vcg)
    a2v = attention(p, f"{a}.audio_to_video_attn", modulate(vnorm, v_sc_a2v, v_sh_a2v), A,
                    context=modulate(anorm, a_sc_a2v, a_sh_a2v), pe=vxpe, k_pe=axpe)
    vx = (vbase + a2v * g_a2v).to(vbase.dtype)
    v2a = attention(p, f"{a}.video_to_audio_attn", modulate(anorm, a_sc_v2a, a_sh_v2a), A,
                    context=modulate(vnorm, v_sc_v2a, v_sh_v2a), pe=axpe, k_pe=vxpe)
    ax = (abase + v2a * g_v2a).to(abase.dtype)
    vx = _stream_ff(p, a, "", vx, vt, V)
    ax = _stream_ff(p, a, "audio_", ax, at, A)
    return vx, ax


def av_modulations(p: dict, video_sigma: float, audio_sigma: float, b: int, v: LTXAVVariant,
                   dtype=torch.bfloat16) -> dict:
    """Every timestep-driven modulation of a joint step with uniform per-modality timesteps
    (preprocessing.py:63-83, 134-213): each stream's AdaLN (9 rows) and prompt AdaLN (2 rows) from
    its own sigma, its cross scale/shift (4 rows) from its own timesteps, and its cross gate (1 row)
    from the OTHER modality's sigma times av_gate_scale; plus the embedded timesteps of the
    outputs."""
    V, A = v.video, v.audio
    tv = torch.full((b,), video_sigma, dtype=torch.float32)
    ta = torch.full((b,), audio_sigma, dtype=torch.float32)
    single = lambda name, t, n, d: adaln_single(p, name, t, dtype)[0].reshape(b, -1, n, d)
    vmod, vemb = adaln_single(p, "adaln_single", tv * V.timestep_scale, dtype)
    amod, aemb = adaln_single(p, "audio_adaln_single", ta * A.timestep_scale, dtype)
    return {
        "vt": vmod.reshape(b, -1, 9, V.dim), "at": amod.reshape(b, -1, 9, A.dim),
        "vemb": vemb, "aemb": aemb,
        "vprompt": single("prompt_adaln_single", tv * V.timestep_scale, 2, V.dim),
        "aprompt": single("audio_prompt_adaln_single", ta * A.timestep_scale, 2, A.dim),
        "vcss": single("av_ca_video_scale_shift_adaln_single", tv * V.timestep_scale, 4, V.dim),
        "acss": single("av_ca_audio_scale_shift_adaln_single", ta * A.timestep_scale, 4, A.dim),
        "vcg": single("av_ca_a2v_gate_adaln_single", ta * v.av_gate_scale, 1, V.dim),
        "acg": single("av_ca_v2a_gate_adaln_single", tv * v.av_gate_scale, 1, A.dim),
    }


def av_forward(p: dict, vlat, alat, vctx, actx, sigma: float, vpos, apos, v: LTXAVVariant,
               blocks: int, dtype=torch.bfloat16, video_context_mask=None, audio_context_mask=None):
    """LTXAVModel.__call__ with both modalities and a uniform timestep (model.py:595-635,
    preprocessing.py:134-213): returns the (video, audio) velocities. The text masks are the
    raw per-stream masks (padded prompts)."""
    vmask = context_mask_bias(video_context_mask, dtype)
    amask = context_mask_bias(audio_context_mask, dtype)
    V, A = v.video, v.audio
    b = vlat.shape[0]
    vx = linear(vlat, p["patchify_proj.weight"], p["patchify_proj.bias"])
    ax = linear(alat, p["audio_patchify_proj.weight"], p["audio_patchify_proj.bias"])
    m = av_modulations(p, sigma, sigma, b, v, dtype)
    vt, at, vprompt, aprompt = m["vt"], m["at"], m["vprompt"], m["aprompt"]
    vcss, vcg, acss, acg, vemb, aemb = m["vcss"], m["vcg"], m["acss"], m["acg"], m["vemb"], m["aemb"]
    vpe = precompute_freqs_cis(vpos, dim=V.dim, theta=V.theta, max_pos=V.max_pos, heads=V.heads)
    ape = precompute_freqs_cis(apos, dim=A.dim, theta=A.theta, max_pos=A.max_pos, heads=A.heads)
    cross_max = (max(V.max_pos[0], A.max_pos[0]),)
    vxpe = precompute_freqs_cis(vpos[:, 0:1], dim=A.dim, theta=V.theta, max_pos=cross_max, heads=V.heads)
    axpe = precompute_freqs_cis(apos[:, 0:1], dim=A.dim, theta=A.theta, max_pos=cross_max, heads=A.heads)
    for i in range(blocks):
        vx, ax = av_block(p, i, vx, ax, vctx, actx, vt, at, vprompt, aprompt, vpe, ape, vxpe,
                          axpe, vcss, vcg, acss, acg, v, vmask, amask)

    def out(x, table, emb, w, bias, eps):
        """_output (model.py:577-593): (table + embedded timestep), LayerNorm, projection."""
        mod = (table[None, None] + emb.reshape(b, -1, x.shape[-1])[:, :, None, :]).to(x.dtype)
        h = (layer_norm(x, eps) * (1.0 + mod[:, :, 1]) + mod[:, :, 0]).to(x.dtype)
        return linear(h, w, bias)

    return (out(vx, p["scale_shift_table"], vemb, p["proj_out.weight"], p["proj_out.bias"], V.eps),
            out(ax, p["audio_scale_shift_table"], aemb, p["audio_proj_out.weight"],
                p["audio_proj_out.bias"], A.eps))


def av_denoise(p, vlat, alat, vctx, actx, vpos, apos, sigmas, v: LTXAVVariant, blocks: int,
               video_context_mask=None, audio_context_mask=None):
    """The deterministic-Euler loop over both modalities (kinomlx/models/ltx2/denoise.py:159-365)."""
    vx, ax = vlat, alat
    for s, n in zip(sigmas[:-1], sigmas[1:]):
        vv, av = av_forward(p, vx, ax, vctx, actx, s, vpos, apos, v, blocks, dtype=vlat.dtype,
                            video_context_mask=video_context_mask,
                            audio_context_mask=audio_context_mask)
        vx = euler_step(vx, to_denoised(vx, s, vv), s, n)
        ax = euler_step(ax, to_denoised(ax, s, av), s, n)
    return vx, ax
