"""Seeded random-init weights and inputs in a fixed, documented draw order.

The reference runs real checkpoints; the benchmark and the parity tests use random-init weights
of the same architecture. Every tensor is drawn, in the order listed by the *_weight_specs
functions, from one torch.Generator on the requested device: N(0, std) for projections (std 0.02
by default), ones for norm scales, zeros for biases where a variant asks for zero biases. Parity
tests draw on the CPU and copy to the GPU so both sides see identical bytes; the benchmark draws
on the GPU directly (the values do not change the timing).
"""

from __future__ import annotations

import torch

from .flux2.config import FluxVariant


def flux_weight_specs(v: FluxVariant, double: int | None = None, single: int | None = None):
    """(name, shape, kind) in draw order; names follow the reference checkpoint
    (kinomlx/models/flux2/transformer.py:78-276)."""
    d, dd = v.dim, v.head_dim
    nd = v.double_blocks if double is None else double
    ns = v.single_blocks if single is None else single
    specs = [
        ("x_embedder.weight", (d, v.in_channels), "normal"),
        ("context_embedder.weight", (d, v.context_dim), "normal"),
        ("time_guidance_embed.timestep_embedder.linear_1.weight", (d, 256), "normal"),
        ("time_guidance_embed.timestep_embedder.linear_2.weight", (d, d), "normal"),
        ("double_stream_modulation_img.linear.weight", (6 * d, d), "normal"),
        ("double_stream_modulation_txt.linear.weight", (6 * d, d), "normal"),
        ("single_stream_modulation.linear.weight", (3 * d, d), "normal"),
    ]
    for i in range(nd):
        a = f"transformer_blocks.{i}"
        for name in ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj"):
            specs.append((f"{a}.attn.{name}.weight", (d, d), "normal"))
        specs.append((f"{a}.attn.to_out.0.weight", (d, d), "normal"))
        specs.append((f"{a}.attn.to_add_out.weight", (d, d), "normal"))
        for name in ("norm_q", "norm_k", "norm_added_q", "norm_added_k"):
            specs.append((f"{a}.attn.{name}.weight", (dd,), "ones"))
        for ff in ("ff", "ff_context"):
            specs.append((f"{a}.{ff}.linear_in.weight", (v.mlp_in, d), "normal"))
            specs.append((f"{a}.{ff}.linear_out.weight", (d, v.mlp_hidden), "normal"))
    for i in range(ns):
        a = f"single_transformer_blocks.{i}.attn"
        specs.append((f"{a}.to_qkv_mlp_proj.weight", (3 * d + v.mlp_in, d), "normal"))
        specs.append((f"{a}.to_out.weight", (d, d + v.mlp_hidden), "normal"))
        specs.append((f"{a}.norm_q.weight", (dd,), "ones"))
        specs.append((f"{a}.norm_k.weight", (dd,), "ones"))
    specs.append(("norm_out.linear.weight", (2 * d, d), "normal"))
    specs.append(("proj_out.weight", (v.in_channels, d), "normal"))
    return specs


def ltx_weight_specs(v, blocks: int | None = None):
    """(name, shape, kind) in draw order for the LTX-2 video stream; names follow the reference
    checkpoint (kinomlx/models/ltx2/transformer/model.py:205-233, transformer.py:85-176)."""
    d, h = v.dim, v.heads
    nb = v.blocks if blocks is None else blocks
    specs = [("patchify_proj.weight", (d, v.in_channels), "normal"),
             ("patchify_proj.bias", (d,), "normal")]
    for pre, n in (("adaln_single", 9), ("prompt_adaln_single", 2)):
        specs += [
            (f"{pre}.emb.timestep_embedder.linear_1.weight", (d, 256), "normal"),
            (f"{pre}.emb.timestep_embedder.linear_1.bias", (d,), "normal"),
            (f"{pre}.emb.timestep_embedder.linear_2.weight", (d, d), "normal"),
            (f"{pre}.emb.timestep_embedder.linear_2.bias", (d,), "normal"),
            (f"{pre}.linear.weight", (n * d, d), "normal"),
            (f"{pre}.linear.bias", (n * d,), "normal"),
        ]
    for i in range(nb):
        a = f"transformer_blocks.{i}"
        specs += [(f"{a}.scale_shift_table", (9, d), "normal"),
                  (f"{a}.prompt_scale_shift_table", (2, d), "normal")]
        for attn, src in (("attn1", d), ("attn2", v.context_dim)):
            specs += [(f"{a}.{attn}.to_q.weight", (d, d), "normal"), (f"{a}.{attn}.to_q.bias", (d,), "normal"),
                      (f"{a}.{attn}.to_k.weight", (d, src), "normal"), (f"{a}.{attn}.to_k.bias", (d,), "normal"),
                      (f"{a}.{attn}.to_v.weight", (d, src), "normal"), (f"{a}.{attn}.to_v.bias", (d,), "normal"),
                      (f"{a}.{attn}.to_out.weight", (d, d), "normal"), (f"{a}.{attn}.to_out.bias", (d,), "normal"),
                      (f"{a}.{attn}.to_gate_logits.weight", (h, d), "normal"),
                      (f"{a}.{attn}.to_gate_logits.bias", (h,), "normal"),
                      (f"{a}.{attn}.q_norm.weight", (d,), "ones"),
                      (f"{a}.{attn}.k_norm.weight", (d,), "ones")]
        specs += [(f"{a}.ff.project_in.proj.weight", (v.ff_mult * d, d), "normal"),
                  (f"{a}.ff.project_in.proj.bias", (v.ff_mult * d,), "normal"),
                  (f"{a}.ff.project_out.weight", (d, v.ff_mult * d), "normal"),
                  (f"{a}.ff.project_out.bias", (d,), "normal")]
    specs += [("scale_shift_table", (2, d), "normal"),
              ("proj_out.weight", (v.out_channels, d), "normal"),
              ("proj_out.bias", (v.out_channels,), "normal")]
    return specs


def _adaln_single_specs(prefix: str, d: int, n: int):
    return [(f"{prefix}.emb.timestep_embedder.linear_1.weight", (d, 256), "normal"),
            (f"{prefix}.emb.timestep_embedder.linear_1.bias", (d,), "normal"),
            (f"{prefix}.emb.timestep_embedder.linear_2.weight", (d, d), "normal"),
            (f"{prefix}.emb.timestep_embedder.linear_2.bias", (d,), "normal"),
            (f"{prefix}.linear.weight", (n * d, d), "normal"),
            (f"{prefix}.linear.bias", (n * d,), "normal")]


def _attention_specs(prefix: str, query_dim: int, context_dim: int, inner: int, heads: int):
    specs = []
    for name, src in (("to_q", query_dim), ("to_k", context_dim), ("to_v", context_dim)):
        specs += [(f"{prefix}.{name}.weight", (inner, src), "normal"),
                  (f"{prefix}.{name}.bias", (inner,), "normal")]
    specs += [(f"{prefix}.to_out.weight", (query_dim, inner), "normal"),
              (f"{prefix}.to_out.bias", (query_dim,), "normal"),
              (f"{prefix}.to_gate_logits.weight", (heads, query_dim), "normal"),
              (f"{prefix}.to_gate_logits.bias", (heads,), "normal"),
              (f"{prefix}.q_norm.weight", (inner,), "ones"),
              (f"{prefix}.k_norm.weight", (inner,), "ones")]
    return specs


def ltx_av_weight_specs(video, audio, blocks: int):
    """(name, shape, kind) in draw order for the joint audio/video model: the video stream's specs,
    then the audio stream, the four A/V AdaLN singles and, per block, the audio layers, the two
    cross-modal attentions (on the audio stream's heads) and their modulation tables; names
    follow the reference checkpoint (kinomlx/models/ltx2/transformer/model.py:205-236,
    transformer.py:85-176)."""
    dv, da = video.dim, audio.dim
    specs = ltx_weight_specs(video, blocks)
    specs += [("audio_patchify_proj.weight", (da, audio.in_channels), "normal"),
              ("audio_patchify_proj.bias", (da,), "normal")]
    specs += _adaln_single_specs("audio_adaln_single", da, 9)
    specs += _adaln_single_specs("audio_prompt_adaln_single", da, 2)
    specs += _adaln_single_specs("av_ca_video_scale_shift_adaln_single", dv, 4)
    specs += _adaln_single_specs("av_ca_a2v_gate_adaln_single", dv, 1)
    specs += _adaln_single_specs("av_ca_audio_scale_shift_adaln_single", da, 4)
    specs += _adaln_single_specs("av_ca_v2a_gate_adaln_single", da, 1)
    for i in range(blocks):
        a = f"transformer_blocks.{i}"
        specs += [(f"{a}.audio_scale_shift_table", (9, da), "normal"),
                  (f"{a}.audio_prompt_scale_shift_table", (2, da), "normal")]
        specs += _attention_specs(f"{a}.audio_attn1", da, da, da, audio.heads)
        specs += _attention_specs(f"{a}.audio_attn2", da, audio.context_dim, da, audio.heads)
        specs += [(f"{a}.audio_ff.project_in.proj.weight", (audio.ff_mult * da, da), "normal"),
                  (f"{a}.audio_ff.project_in.proj.bias", (audio.ff_mult * da,), "normal"),
                  (f"{a}.audio_ff.project_out.weight", (da, audio.ff_mult * da), "normal"),
                  (f"{a}.audio_ff.project_out.bias", (da,), "normal")]
        specs += _attention_specs(f"{a}.audio_to_video_attn", dv, da, da, audio.heads)
        specs += _attention_specs(f"{a}.video_to_audio_attn", da, dv, da, audio.heads)
        specs += [(f"{a}.scale_shift_table_a2v_ca_audio", (5, da), "normal"),
                  (f"{a}.scale_shift_table_a2v_ca_video", (5, dv), "normal")]
    specs += [("audio_scale_shift_table", (2, da), "normal"),
              ("audio_proj_out.weight", (audio.out_channels, da), "normal"),
              ("audio_proj_out.bias", (audio.out_channels,), "normal")]
    return specs


def ltx_weights(v, *, seed: int = 0, device="cpu", dtype=torch.bfloat16, blocks: int | None = None):
    return make_weights(ltx_weight_specs(v, blocks), seed=seed, device=device, dtype=dtype)


def make_weights(specs, *, seed: int = 0, device="cpu", dtype=torch.bfloat16, std: float = 0.02):
    """Kinds: "ones", "zeros", "normal" (N(0, std)), "scale" (1 + N(0, 0.1): learned norm
    scales away from one), "wide" (N(0, 0.2): modulation tables, latent statistics)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    for name, shape, kind in specs:
        if kind == "ones":
            out[name] = torch.ones(shape, device=device, dtype=dtype)
        elif kind == "zeros":
            out[name] = torch.zeros(shape, device=device, dtype=dtype)
        else:
            t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
            if kind == "scale":
                out[name] = (1.0 + 0.1 * t).to(dtype)
            elif kind == "wide":
                out[name] = (0.2 * t).to(dtype)
            else:
                out[name] = (t * std).to(dtype)
    return out


def diffusion_decoder_weight_specs(cfg):
    """(name, shape, kind) of the LTX-2.5 diffusion video decoder in draw order; names follow the
    reference's parameter tree (kinomlx/models/ltx2/video_vae/diffusion_decoder.py:1026-1093)."""
    specs = [("conv_in.weight", (cfg.stage_channels[0], cfg.latent_channels), "normal"),
             ("conv_in.bias", (cfg.stage_channels[0],), "normal")]

    def block(pre: str, c: int, diffusion: bool) -> None:
        hidden = (int(c * 4.0) + 15) // 16 * 16
        if diffusion:
            specs.extend([(pre + "context_proj.weight", (c, c), "normal"),
                          (pre + "context_proj.bias", (c,), "normal"),
                          (pre + "scale_shift_table", (7, c), "wide")])
        specs.extend([
            (pre + "norm1.weight", (c,), "scale"),
            (pre + "attn.qkv.weight", (3 * c, c), "normal"),
            (pre + "attn.qkv.bias", (3 * c,), "normal"),
            (pre + "attn.proj.weight", (c, c), "normal"),
            (pre + "attn.proj.bias", (c,), "normal"),
            (pre + "attn.q_norm.weight", (cfg.head_dim,), "scale"),
            (pre + "attn.k_norm.weight", (cfg.head_dim,), "scale"),
            (pre + "norm2.weight", (c,), "scale"),
            (pre + "mlp.w_up.weight", (hidden, c), "normal"),
            (pre + "mlp.w_gate.weight", (hidden, c), "normal"),
            (pre + "mlp.w_down.weight", (c, hidden), "normal"),
        ])

    for s, stride in enumerate(cfg.upsample_strides):
        c = cfg.stage_channels[s]
        for i in range(cfg.stage_depths[s]):
            block(f"det_stages.{s}.{i}.", c, False)
        prod = stride[0] * stride[1] * stride[2]
        out = prod * c // cfg.upsample_channel_reductions[s]
        specs.extend([(f"upsamples.{s}.proj.weight", (out, c), "normal"),
                      (f"upsamples.{s}.proj.bias", (out,), "normal")])
    c5 = cfg.stage_channels[-1]
    pixels = cfg.out_channels * cfg.patch_size ** 2
    specs.extend([
        ("t_embedder.linear_1.weight", (cfg.t_emb_dim, 256), "normal"),
        ("t_embedder.linear_1.bias", (cfg.t_emb_dim,), "normal"),
        ("t_embedder.linear_2.weight", (cfg.t_emb_dim, cfg.t_emb_dim), "normal"),
        ("t_embedder.linear_2.bias", (cfg.t_emb_dim,), "normal"),
        ("conv_in_x_t.weight", (c5, pixels), "normal"),
        ("conv_in_x_t.bias", (c5,), "normal"),
        ("shared_adaln.proj.weight", (7 * c5, cfg.t_emb_dim), "normal"),
        ("shared_adaln.proj.bias", (7 * c5,), "normal"),
    ])
    for i in range(cfg.stage_depths[4]):
        block(f"diff_blocks.{i}.", c5, True)
    specs.extend([("norm_out.weight", (c5,), "scale"),
                  ("conv_out.weight", (pixels, c5), "normal"),
                  ("conv_out.bias", (pixels,), "normal")])
    return specs


def diffusion_decoder_weights(cfg, *, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                              std: float = 0.02):
    """Seeded decoder weights (bf16, as a checkpoint binds them) plus the fp32 per-channel latent
    statistics (std 1 + N(0, 0.1), mean N(0, 0.2))."""
    w = make_weights(diffusion_decoder_weight_specs(cfg), seed=seed, device=device, dtype=dtype,
                     std=std)
    stats = make_weights([("per_channel_statistics.std_of_means", (cfg.latent_channels,), "scale"),
                          ("per_channel_statistics.mean_of_means", (cfg.latent_channels,), "wide")],
                         seed=seed + 1, device=device, dtype=torch.float32)
    w.update(stats)
    return w


def flux_weights(v: FluxVariant, *, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                 double: int | None = None, single: int | None = None):
    return make_weights(flux_weight_specs(v, double, single), seed=seed, device=device, dtype=dtype)


def normal(shape, *, seed: int, device="cpu", dtype=torch.bfloat16, std: float = 1.0):
    gen = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(dtype)
