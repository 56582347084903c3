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


def ltx_weights(v, *, seed: int = 0, device="cpu", dtype=torch.bfloat16, blocks: int | None = None):
    return make_weights(ltx_weight_specs(v, blocks), seed=seed, device=device, dtype=dtype)


def make_weights(specs, *, seed: int = 0, device="cpu", dtype=torch.bfloat16, std: float = 0.02):
    gen = torch.Generator(device=device).manual_seed(seed)
    out: dict[str, torch.Tensor] = {}
    for name, shape, kind in specs:
        if kind == "ones":
            out[name] = torch.ones(shape, device=device, dtype=dtype)
        elif kind == "zeros":
            out[name] = torch.zeros(shape, device=device, dtype=dtype)
        else:
            t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
            out[name] = (t * std).to(dtype)
    return out


def flux_weights(v: FluxVariant, *, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                 double: int | None = None, single: int | None = None):
    return make_weights(flux_weight_specs(v, double, single), seed=seed, device=device, dtype=dtype)


def normal(shape, *, seed: int, device="cpu", dtype=torch.bfloat16, std: float = 1.0):
    gen = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(dtype)
