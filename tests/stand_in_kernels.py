"""Torch stand-ins with the contracts of the kino_* entry points, for CPU tests of the host-side
orchestration only (which tensors, slices and modulation rows each model class hands to which
kernel, in which order). Tests install them with monkeypatch; the product path never imports
this module, and without the CUDA library every kinomlx_b200 op raises. The kernels themselves
are tested against the oracle on the GPU."""

from __future__ import annotations

import torch

from oracle import flux2 as fref
from oracle import fused_ops as rops
from oracle import ltx2 as lref
from oracle import video_vae as vref


def _3(t: torch.Tensor) -> torch.Tensor:
    return t if t.dim() == 3 else t.unsqueeze(0)


def _put(out, y):
    if out is None:
        return y
    out.copy_(y.reshape(out.shape))
    return out


def _rope_rows(tables, offset: int, batch: int, rows: int):
    """(batch, rows, 1, 128) cos/sin of ops.RopeTables: batch b, row i reads table column
    (b * tables.rows if batched) + offset + i."""
    idx = offset + torch.arange(rows)
    cols = (torch.arange(batch)[:, None] * tables.rows if tables.batched else torch.zeros(batch, 1, dtype=torch.long)) + idx
    pick = lambda t: t.T[cols][:, :, None]
    return pick(tables.cos_t), pick(tables.sin_t)


def linear(x, w, out=None, *, bias=None, kind=0, residual=None, gate=None, act_col_begin=0,
           dt=0.0, sample=None, sigma=0.0, ratio=0.0, qk_norm=None, norm_width=0, rope=None,
           eps=1e-6, lead_w=None, lead_rows=0, lead_qk_norm=None, lead_gate=None, **_):
    x3 = _3(x).float()
    y = x3 @ w.float().T
    if lead_w is not None:  # rows [0, lead_rows) of every batch entry use the lead weight
        y[:, :lead_rows] = x3[:, :lead_rows] @ lead_w.float().T
    if bias is not None:
        y = y + bias.float()
    if qk_norm:  # per-head RMSNorm then adjacent-pair RoPE on each (column, weight) range
        b, m = y.shape[:2]
        c, s = _rope_rows(rope[0], rope[1], b, m)
        for r, (col, wt) in enumerate(qk_norm):
            seg = y[..., col : col + norm_width].reshape(b, m, -1, 128)
            normed = rops.rms_norm(seg, wt.float(), eps)
            if lead_qk_norm:
                normed[:, :lead_rows] = rops.rms_norm(seg[:, :lead_rows], lead_qk_norm[r].float(), eps)
            y[..., col : col + norm_width] = fref.rotate(normed, c, s).reshape(b, m, norm_width)
    if kind == 1:  # GELU on columns >= act_col_begin
        y = torch.cat([y[..., :act_col_begin], rops.gelu_approx(y[..., act_col_begin:])], -1)
    elif kind == 6:  # SwiGLU on blocks of 16 gate + 16 content columns from act_col_begin
        blocks = y[..., act_col_begin:].reshape(*y.shape[:-1], -1, 2, 16)
        act = rops.silu(blocks[..., 0, :]) * blocks[..., 1, :]
        y = torch.cat([y[..., :act_col_begin], act.reshape(*y.shape[:-1], -1)], -1)
    elif kind == 2:  # gated residual
        g = gate.reshape(-1, gate.shape[-1]).float()[:, None].expand(y.shape[0], y.shape[1], -1).clone()
        if lead_gate is not None:
            g[:, :lead_rows] = lead_gate.reshape(-1, lead_gate.shape[-1]).float()[:, None]
        y = (_3(residual).float() + g * y).reshape(residual.shape)
    elif kind == 3:  # Euler
        y = sample.float() + dt * y.reshape(sample.shape)
    elif kind == 4:  # 2 * sigmoid
        y = 2.0 * torch.sigmoid(y)
    elif kind == 5:  # X0 + Euler
        y = y.reshape(sample.shape)
        x0 = sample.float() - sigma * y
        y = x0 + ratio * (sample.float() - x0)
    if out is None and x.dim() == 2 and y.dim() == 3:
        y = y[0]
    return _put(out, y)


def attention_list(q, k, v, out, *, heads, scale=None, gate=None, peer_return=None,
                   key_bias=None, kv_splits=1):
    """ops.attention: lists of query and key/value segments, an optional additive key bias."""
    q3 = torch.cat([_3(t) for t in q], 1)
    k3 = torch.cat([_3(t) for t in k], 1)
    v3 = torch.cat([_3(t) for t in v], 1)
    d = q3.shape[-1] // heads
    sh = lambda t: t.float().reshape(*t.shape[:2], heads, d).transpose(1, 2)
    mask = None if key_bias is None else key_bias[:, None, None, : k3.shape[1]]
    o = rops.sdpa(sh(q3), sh(k3), sh(v3), scale=d ** -0.5, mask=mask).transpose(1, 2)
    if gate is not None and gate[0] is not None:
        o = o * torch.cat([_3(g) for g in gate], 1).float()[..., None]
    o = o.reshape(q3.shape)
    start = 0
    for dst in out:
        n = _3(dst).shape[1]
        _put(dst, o[:, start : start + n])
        start += n
    return out


def attention_tensor(q, k, v, out=None, *, heads, scale=None, gate=None, key_bias=None):
    """ops_f32.attention: one segment each."""
    res = attention_list([q], [k], [v], [torch.empty_like(q) if out is None else out],
                         heads=heads, gate=None if gate is None else [gate], key_bias=key_bias)
    return res[0]


def adaln(x, shift, scale, out=None, *, norm=1, eps=1e-6):
    base = rops.layer_norm(x, eps) if norm == 1 else (rops.rms_norm(x, None, eps) if norm == 0 else x)
    d = x.shape[-1]
    y = _3(base).float() * (1 + scale.reshape(-1, 1, d).float()) + shift.reshape(-1, 1, d).float()
    return _put(out, y.reshape(x.shape))


def qk_norm_rope(x, *, heads, weight, norm, rope, cos=None, sin=None, table_offset=0, eps=1e-6,
                 scatter=None):
    x3 = _3(x)
    b, t, w = x3.shape
    y = x3.float()
    if norm == 1:  # per 128-wide head, then adjacent pairs
        y = rops.rms_norm(y.reshape(b, t, heads, 128), weight.float(), eps)
        if rope == 1:
            c = cos.reshape(-1, cos.shape[-2], 128)[:, table_offset : table_offset + t, None]
            s = sin.reshape(-1, sin.shape[-2], 128)[:, table_offset : table_offset + t, None]
            y = fref.rotate(y, c, s)
        y = y.reshape(b, t, w)
    else:
        if norm == 2:
            y = rops.rms_norm(y, weight.float(), eps)
        if rope in (2, 3):
            y = lref.apply_split_rotary_emb(y, cos, sin)
    x3.copy_(y)
    return x


def gemv(x, w, bias=None, *, silu_input=False, out=None):
    xx = rops.silu(x.float()) if silu_input else x.float()
    return _put(out, xx @ w.float().T + (0 if bias is None else bias.float()))


def timestep_embedding(t, dim=256, *, out=None):
    return _put(out, lref.timestep_features(t, dim))


def add_rows(a, b, out=None):
    return _put(out, a.float() + b.float())


def unary(fn):
    return lambda x, out=None: _put(out, fn(x.float()))


def swiglu(x, out=None):
    return _put(out, fref.swiglu(x.float()))


def cfg_combine(c, u, g, out=None):
    return _put(out, u.float() + g * (c.float() - u.float()))


def euler_velocity(x, v, dt, out=None):
    return _put(out, x.float() + dt * v.float())


def _keep_stats(stats, y) -> None:
    """The bf16 conv's GroupNorm(32) statistics, in a stand-in layout: stats[:32] the group
    means, stats[32:64] the biased group variances of the conv output y (..., C)."""
    if stats is not None:
        g = y.float().reshape(-1, 32, y.shape[-1] // 32)
        stats[:32] = g.mean(dim=(0, 2))
        stats[32:64] = g.var(dim=(0, 2), unbiased=False)


def conv3d(x, weight, bias=None, *, causal, stride=(1, 1, 1), residual=None, out=None, stats=None,
           **_):
    x5 = (x if x.dim() == 5 else x[None]).float()
    sub = stride[0] * stride[1] * stride[2]
    b = torch.zeros(weight.shape[0]) if bias is None else bias.float()
    if sub == 1:
        y = vref.conv3d(x5, weight.float(), b, causal)[0]
        if residual is not None:
            y = y + residual.float()
        _keep_stats(stats, y)
        return _put(out, y)
    n, cin = weight.shape[0], weight.shape[-1]
    cout = n // sub
    # the device weight rows are sub-position-major; the oracle's are channel-major
    wt = weight.float().reshape(sub, cout, *weight.shape[1:]).transpose(0, 1).reshape(weight.shape)
    bs = b.reshape(sub, cout).transpose(0, 1).reshape(-1)
    y = vref.upsample({"u.conv.weight": wt, "u.conv.bias": bs}, "u", x5, stride, cin // cout,
                      vref.VaeVariant(causal=causal))[0]
    _keep_stats(stats, y)
    return _put(out, y)


def pixel_norm(x, eps=1e-8, *, silu=False, out=None):
    y = rops.pixel_norm(x.float(), dim=-1, eps=eps)
    return _put(out, rops.silu(y) if silu else y)


def group_norm(x, groups, weight, bias, eps, *, silu=False, out=None, **_):
    y = rops.group_norm(x.float()[None], 32, weight.float(), bias.float(), eps)[0]
    return _put(out, rops.silu(y) if silu else y)


def group_norm_from_stats(x, weight, bias, eps, stats, *, silu=False, out=None):
    """Normalise with the statistics the producing conv kept (never recomputed from x), so a
    norm reading another conv's statistics shows."""
    c = x.shape[-1]
    g = x.float().reshape(-1, 32, c // 32)
    y = (g - stats[:32, None]) / torch.sqrt(stats[32:64, None] + eps)
    y = y.reshape(x.shape) * weight.float() + bias.float()
    return _put(out, rops.silu(y) if silu else y)


def latent_to_bfhwc(latent, std, mean):
    y = latent.float() * std.reshape(1, -1, 1, 1, 1) + mean.reshape(1, -1, 1, 1, 1)
    return y[0].permute(1, 2, 3, 0).contiguous()


def tile_blend(decoded, canvas, weights, y0, x0, mask_h, mask_w, patch=4):
    d = vref.unpatchify(decoded.float()[None], patch)[0]  # F, H, W, C
    m = mask_h.reshape(-1, 1) * mask_w.reshape(1, -1)
    hh, ww = d.shape[1], d.shape[2]
    canvas[0, :, :, y0 : y0 + hh, x0 : x0 + ww] += d.permute(3, 0, 1, 2) * m
    weights[y0 : y0 + hh, x0 : x0 + ww] += m


def blend_normalize(canvas, weights):
    return canvas / torch.clamp(weights, min=1e-8)


def install(monkeypatch) -> None:
    """Replace the kernel calls of kinomlx_b200.ops and kinomlx_b200.ops_f32 for one test, and
    run the bf16 model classes' wiring in fp32."""
    from kinomlx_b200 import ops, ops_f32
    from kinomlx_b200.flux2 import transformer as flux
    from kinomlx_b200.ltx2 import transformer as ltx
    from kinomlx_b200.ltx2 import video_vae as vae

    for mod in (flux, ltx, vae):
        monkeypatch.setattr(mod, "BF", torch.float32)

    for mod, att in ((ops, attention_list), (ops_f32, attention_tensor)):
        for name, fn in (("linear", linear), ("attention", att), ("adaln", adaln),
                         ("qk_norm_rope", qk_norm_rope), ("timestep_embedding", timestep_embedding),
                         ("add_rows", add_rows), ("cfg_combine", cfg_combine),
                         ("euler_velocity", euler_velocity), ("blend_normalize", blend_normalize)):
            monkeypatch.setattr(mod, name, fn, raising=False)
    monkeypatch.setattr(ops, "gemv", gemv)
    monkeypatch.setattr(ops, "device_status", lambda: None)
    for name, fn in (("conv3d", conv3d), ("pixel_norm", pixel_norm), ("latent_to_bfhwc", latent_to_bfhwc),
                     ("tile_blend", tile_blend), ("group_norm_from_stats", group_norm_from_stats),
                     ("conv_stats_buffer", lambda device=None: torch.zeros(64)),
                     ("conv_workspace", lambda device=None: torch.zeros(1, dtype=torch.uint8))):
        monkeypatch.setattr(ops, name, fn)
    for name, fn in (("silu", unary(rops.silu)), ("gelu_tanh", unary(rops.gelu_approx)),
                     ("swiglu", swiglu), ("conv3d", conv3d), ("pixel_norm", pixel_norm),
                     ("group_norm", group_norm), ("latent_to_bfhwc", latent_to_bfhwc),
                     ("tile_blend", tile_blend)):
        monkeypatch.setattr(ops_f32, name, fn)
