"""Flux2-style MMDiT on the sm_100a kernels: the device twin of Flux2Transformer
(kinomlx/models/flux2/transformer.py:261-358).

Memory layout (one workspace per batch/token shape, allocated once):
  stream (B, Nt+Ni, D)     text rows then image rows: the double blocks' two streams are views
                           of it, so the single blocks' concatenation costs nothing
  nrm    (B, N, D)         AdaLN output, the A operand of the next projection
  qkv    (B, N, 3D)        fused [q | k | v] of both streams; attention writes its output over q
  hid    (B, N, H)         MLP activations of the double blocks (H = activated MLP width)
  big    (B, N, 3D+H)      single-block fused projection laid out [k | v | q | act(mlp)] so the
                           attention output (written over q) and the activated MLP are one
                           contiguous (D + mlp_hidden)-wide operand of to_out
Projections run on the tcgen05 GEMM with their epilogue fused (GELU, gated residual, Euler);
QK RMSNorm + RoPE run in place on the projection output; attention reads token-major q/k/v.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from ..sequence_parallel import SequenceParallel
from .config import FluxVariant


def rotary_positions(ids: torch.Tensor, variant: FluxVariant) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-axis frequencies theta^(-arange(0, d, 2)/d) in fp32, angles repeated pairwise; tables
    (B, N, head_dim) fp32 (kinomlx/models/flux2/transformer.py:17-22). Computed once per
    generation on the host, like the reference's prepare_velocities."""
    parts = []
    for axis, width in enumerate(variant.rope_axes):
        freq = torch.tensor(variant.rope_theta, dtype=torch.float32) ** (
            -torch.arange(0, width, 2, dtype=torch.float32) / width
        )
        parts.append(ids[..., axis].to(torch.float32).cpu()[..., None] * freq)
    angles = torch.cat(parts, dim=-1).repeat_interleave(2, dim=-1)
    return torch.cos(angles), torch.sin(angles)


@dataclass
class PreparedText:
    """Once-per-generation state (kinomlx/models/flux2/transformer.py:283-292)."""

    text: torch.Tensor  # projected text (B, Nt, D)
    rope: ops.RopeTables  # joint [text, image] tables, head-dim-major on the device


class _Workspace:
    def __init__(self, v: FluxVariant, batch: int, nt: int, ni: int, device: torch.device,
                 sp: SequenceParallel):
        n, d = nt + ni, v.dim
        e = lambda *shape: torch.empty(shape, device=device, dtype=torch.bfloat16)
        self.batch, self.nt, self.ni = batch, nt, ni
        self.stream = e(batch, n, d)
        self.nrm = e(batch, n, d)
        self.hid = e(batch, n, v.mlp_hidden)
        # the projections the attention returns its rows to are shared with the other GPUs
        # under the peer transport (their addresses in qkv_ptrs / big_ptrs)
        self.peer = sp.peer is not None and batch == 1
        if self.peer:
            self.qkv, self.qkv_ptrs = sp.shared((batch, n, 3 * d))
            self.big, self.big_ptrs = sp.shared((batch, n, 3 * d + v.mlp_hidden))
        else:
            self.qkv = e(batch, n, 3 * d)
            self.big = e(batch, n, 3 * d + v.mlp_hidden)
        self.t = torch.empty((batch,), device=device, dtype=torch.float32)
        self.temb = e(batch, 256)
        self.emb1 = e(batch, d)
        self.emb = e(batch, d)
        self.mods = e(batch, 17 * d)
        self.velocity = e(batch, ni, v.in_channels)


class Flux2Transformer:
    """Device Flux2 MMDiT. `weights` uses the reference checkpoint names."""

    def __init__(self, weights: dict[str, torch.Tensor], variant: FluxVariant,
                 device: torch.device | str = "cuda", *, sp: SequenceParallel | None = None):
        """`sp` shards the tokens over a process group (Ulysses); each rank then holds
        Nt/P text and Ni/P image tokens and passes its own latent shard to `run`."""
        self.sp = sp if sp is not None else SequenceParallel.single()
        if variant.mlp not in ("gelu_tanh", "swiglu"):
            raise ValueError(f"unknown MLP kind {variant.mlp!r}")
        self.v = variant
        self.device = torch.device(device)
        swiglu = variant.mlp == "swiglu"
        # SwiGLU up projections: gate/content rows interleaved for the fused epilogue
        self.act_kind = ops.EPI_SWIGLU if swiglu else ops.EPI_GELU
        mlp_rows = ops.swiglu_interleave if swiglu else (lambda t: t)
        dev = lambda t: t.to(self.device, torch.bfloat16).contiguous()
        w = weights
        d = variant.dim
        self.x_embedder = dev(w["x_embedder.weight"])
        self.context_embedder = dev(w["context_embedder.weight"])
        pre = "time_guidance_embed.timestep_embedder"
        self.t_lin1 = dev(w[f"{pre}.linear_1.weight"])
        self.t_lin2 = dev(w[f"{pre}.linear_2.weight"])
        # one product for all four modulations: [img 6D | txt 6D | single 3D | out 2D]
        self.mod_all = dev(torch.cat([
            w["double_stream_modulation_img.linear.weight"],
            w["double_stream_modulation_txt.linear.weight"],
            w["single_stream_modulation.linear.weight"],
            w["norm_out.linear.weight"],
        ]))
        self.double = []
        for i in range(variant.double_blocks):
            a = f"transformer_blocks.{i}"
            g = lambda name: w[f"{a}.attn.{name}.weight"]
            self.double.append({
                "img_qkv": dev(torch.cat([g("to_q"), g("to_k"), g("to_v")])),
                "txt_qkv": dev(torch.cat([g("add_q_proj"), g("add_k_proj"), g("add_v_proj")])),
                "to_out": dev(g("to_out.0")),
                "to_add_out": dev(g("to_add_out")),
                "norm_q": dev(g("norm_q")),
                "norm_k": dev(g("norm_k")),
                "norm_added_q": dev(g("norm_added_q")),
                "norm_added_k": dev(g("norm_added_k")),
                "ff_in": dev(mlp_rows(w[f"{a}.ff.linear_in.weight"])),
                "ff_out": dev(w[f"{a}.ff.linear_out.weight"]),
                "ffc_in": dev(mlp_rows(w[f"{a}.ff_context.linear_in.weight"])),
                "ffc_out": dev(w[f"{a}.ff_context.linear_out.weight"]),
            })
        self.single = []
        for i in range(variant.single_blocks):
            a = f"single_transformer_blocks.{i}.attn"
            fused = w[f"{a}.to_qkv_mlp_proj.weight"]
            q, k, vv, mlp = fused[:d], fused[d : 2 * d], fused[2 * d : 3 * d], fused[3 * d :]
            self.single.append({
                "fused": dev(torch.cat([k, vv, q, mlp_rows(mlp)])),  # [k | v | q | mlp]
                "to_out": dev(w[f"{a}.to_out.weight"]),
                "norm_q": dev(w[f"{a}.norm_q.weight"]),
                "norm_k": dev(w[f"{a}.norm_k.weight"]),
            })
        self.proj_out = dev(w["proj_out.weight"])
        self._ws: dict[tuple[int, int, int], _Workspace] = {}

    # ------------------------------------------------------------------ preparation
    def prepare(self, text: torch.Tensor, ids: torch.Tensor) -> PreparedText:
        """Project the text once and build the RoPE tables for the joint [text, image] ids."""
        text = text.to(self.device, torch.bfloat16)
        projected = ops.linear(text, self.context_embedder)
        cos, sin = rotary_positions(ids, self.v)
        if self.sp.size > 1:
            nt = text.shape[1]
            t0, t1 = self.sp.shard(nt)
            i0, i1 = self.sp.shard(ids.shape[1] - nt)
            rows = torch.cat([torch.arange(t0, t1), nt + torch.arange(i0, i1)])
            projected = projected[:, t0:t1].contiguous()
            cos, sin = cos[:, rows].contiguous(), sin[:, rows].contiguous()
        return PreparedText(projected, ops.RopeTables(cos.to(self.device), sin.to(self.device)))

    def workspace(self, batch: int, nt: int, ni: int) -> _Workspace:
        key = (batch, nt, ni)
        if key not in self._ws:
            self._ws[key] = _Workspace(self.v, batch, nt, ni, self.device, self.sp)
        return self._ws[key]

    # ------------------------------------------------------------------ blocks
    def _double_block(self, ws: _Workspace, p: dict, rope: ops.RopeTables) -> None:
        if ws.nt % 256 == 0 and ws.ni > 0:
            self._double_block_joint(ws, p, rope)
            return
        d, nt, h = self.v.dim, ws.nt, self.v.heads
        txt, img = ws.stream[:, :nt], ws.stream[:, nt:]
        txt_n, img_n = ws.nrm[:, :nt], ws.nrm[:, nt:]
        m = lambda base, j: ws.mods[:, (base + j) * d : (base + j + 1) * d]  # img base 0, txt 6
        ops.adaln(img, m(0, 0), m(0, 1), img_n, norm=ops.NORM_LAYER)
        ops.adaln(txt, m(6, 0), m(6, 1), txt_n, norm=ops.NORM_LAYER)
        # q/k RMSNorm + RoPE run in the projection's epilogue (image rows read table rows from nt);
        # under the peer transport the same epilogue stores q/k/v into the head owners' buffers
        recv = self.sp.receive(nt + ws.ni, d) if ws.peer else None
        ops.linear(img_n, p["img_qkv"], ws.qkv[:, nt:], qk_norm=[(0, p["norm_q"]), (d, p["norm_k"])],
                   norm_width=d, rope=(rope, nt),
                   scatter=self.sp.scatter(recv, d, (0, 1, 2), nt) if recv else None)
        ops.linear(txt_n, p["txt_qkv"], ws.qkv[:, :nt],
                   qk_norm=[(0, p["norm_added_q"]), (d, p["norm_added_k"])], norm_width=d,
                   rope=(rope, 0), scatter=self.sp.scatter(recv, d, (0, 1, 2), 0) if recv else None)
        q, k, v = ws.qkv[..., :d], ws.qkv[..., d : 2 * d], ws.qkv[..., 2 * d :]
        if recv:
            self.sp.attention_from_peers(recv, heads=h, out_ptrs=ws.qkv_ptrs, out_ld=3 * d,
                                         out_cols=3 * d, out_col=0)
        else:
            self.sp.attention(q, k, v, q, heads=h)
        ops.linear(q[:, nt:], p["to_out"], img, kind=ops.EPI_GATED_RESIDUAL, residual=img,
                   gate=m(0, 2))
        ops.linear(q[:, :nt], p["to_add_out"], txt, kind=ops.EPI_GATED_RESIDUAL, residual=txt,
                   gate=m(6, 2))
        ops.adaln(img, m(0, 3), m(0, 4), img_n, norm=ops.NORM_LAYER)
        ops.linear(img_n, p["ff_in"], ws.hid[:, nt:], kind=self.act_kind)
        ops.linear(ws.hid[:, nt:], p["ff_out"], img, kind=ops.EPI_GATED_RESIDUAL, residual=img,
                   gate=m(0, 5))
        ops.adaln(txt, m(6, 3), m(6, 4), txt_n, norm=ops.NORM_LAYER)
        ops.linear(txt_n, p["ffc_in"], ws.hid[:, :nt], kind=self.act_kind)
        ops.linear(ws.hid[:, :nt], p["ffc_out"], txt, kind=ops.EPI_GATED_RESIDUAL, residual=txt,
                   gate=m(6, 5))

    def _double_block_joint(self, ws: _Workspace, p: dict, rope: ops.RopeTables) -> None:
        """The double block with each projection of the two streams in one launch over the joint
        [text | image] rows: text rows use the text stream's weights, norms and gates (lead
        rows), image rows the image stream's. The streams stay independent; only the launch
        order interleaves them."""
        d, nt, h = self.v.dim, ws.nt, self.v.heads
        txt, img = ws.stream[:, :nt], ws.stream[:, nt:]
        txt_n, img_n = ws.nrm[:, :nt], ws.nrm[:, nt:]
        m = lambda base, j: ws.mods[:, (base + j) * d : (base + j + 1) * d]  # img base 0, txt 6
        ops.adaln(img, m(0, 0), m(0, 1), img_n, norm=ops.NORM_LAYER)
        ops.adaln(txt, m(6, 0), m(6, 1), txt_n, norm=ops.NORM_LAYER)
        recv = self.sp.receive(nt + ws.ni, d) if ws.peer else None
        ops.linear(ws.nrm, p["img_qkv"], ws.qkv, qk_norm=[(0, p["norm_q"]), (d, p["norm_k"])],
                   norm_width=d, rope=(rope, 0), lead_w=p["txt_qkv"], lead_rows=nt,
                   lead_qk_norm=[p["norm_added_q"], p["norm_added_k"]],
                   scatter=self.sp.scatter(recv, d, (0, 1, 2), 0) if recv else None)
        q, k, v = ws.qkv[..., :d], ws.qkv[..., d : 2 * d], ws.qkv[..., 2 * d :]
        if recv:
            self.sp.attention_from_peers(recv, heads=h, out_ptrs=ws.qkv_ptrs, out_ld=3 * d,
                                         out_cols=3 * d, out_col=0)
        else:
            self.sp.attention(q, k, v, q, heads=h)
        ops.linear(q, p["to_out"], ws.stream, kind=ops.EPI_GATED_RESIDUAL, residual=ws.stream,
                   gate=m(0, 2), lead_w=p["to_add_out"], lead_rows=nt, lead_gate=m(6, 2))
        ops.adaln(img, m(0, 3), m(0, 4), img_n, norm=ops.NORM_LAYER)
        ops.adaln(txt, m(6, 3), m(6, 4), txt_n, norm=ops.NORM_LAYER)
        ops.linear(ws.nrm, p["ff_in"], ws.hid, kind=self.act_kind, lead_w=p["ffc_in"],
                   lead_rows=nt)
        ops.linear(ws.hid, p["ff_out"], ws.stream, kind=ops.EPI_GATED_RESIDUAL,
                   residual=ws.stream, gate=m(0, 5), lead_w=p["ffc_out"], lead_rows=nt,
                   lead_gate=m(6, 5))

    def _single_block(self, ws: _Workspace, p: dict, rope: ops.RopeTables) -> None:
        d, h = self.v.dim, self.v.heads
        sm = lambda j: ws.mods[:, (12 + j) * d : (13 + j) * d]
        ops.adaln(ws.stream, sm(0), sm(1), ws.nrm, norm=ops.NORM_LAYER)
        # [k | v | q | mlp]: k and q normalised and rotated, the MLP activated, in one epilogue
        recv = self.sp.receive(ws.nt + ws.ni, d) if ws.peer else None
        ops.linear(ws.nrm, p["fused"], ws.big, kind=self.act_kind, act_col_begin=3 * d,
                   qk_norm=[(0, p["norm_k"]), (2 * d, p["norm_q"])], norm_width=d,
                   rope=(rope, 0), scatter=self.sp.scatter(recv, d, (1, 2, 0), 0) if recv else None)
        k, v, q = ws.big[..., :d], ws.big[..., d : 2 * d], ws.big[..., 2 * d : 3 * d]
        if recv:
            self.sp.attention_from_peers(recv, heads=h, out_ptrs=ws.big_ptrs,
                                         out_ld=ws.big.shape[-1], out_cols=ws.big.shape[-1],
                                         out_col=2 * d)
        else:
            self.sp.attention(q, k, v, q, heads=h)
        ops.linear(ws.big[..., 2 * d :], p["to_out"], ws.stream, kind=ops.EPI_GATED_RESIDUAL,
                   residual=ws.stream, gate=sm(2))

    def double_block(self, index: int, image: torch.Tensor, text: torch.Tensor,
                     timestep_x1000: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """One DoubleBlock on hidden states: the timestep MLP, its
        modulations and block `index`; returns new (image, text) hidden states."""
        batch, ni, _ = image.shape
        nt = text.shape[1]
        ws = self.workspace(batch, nt, ni)
        self._embed(ws, timestep_x1000)
        ws.stream[:, :nt].copy_(text)
        ws.stream[:, nt:].copy_(image)
        self._double_block(ws, self.double[index], ops.RopeTables(cos, sin))
        return ws.stream[:, nt:].clone(), ws.stream[:, :nt].clone()

    def single_block(self, index: int, value: torch.Tensor, text_tokens: int,
                     timestep_x1000: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """One SingleBlock on the joint hidden state (B, Nt+Ni, D)."""
        batch, n, _ = value.shape
        ws = self.workspace(batch, text_tokens, n - text_tokens)
        self._embed(ws, timestep_x1000)
        ws.stream.copy_(value)
        self._single_block(ws, self.single[index], ops.RopeTables(cos, sin))
        return ws.stream.clone()

    # ------------------------------------------------------------------ forward
    def _embed(self, ws: _Workspace, timestep_x1000: torch.Tensor | float) -> None:
        """Timestep MLP and every modulation vector (kinomlx/models/flux2/transformer.py:315-318)."""
        if isinstance(timestep_x1000, torch.Tensor):
            ws.t.copy_(timestep_x1000, non_blocking=True)
        else:  # one value for every batch entry: a fill, no host-to-device copy
            ws.t.fill_(float(timestep_x1000))
        ops.timestep_embedding(ws.t, 256, out=ws.temb)
        ops.gemv(ws.temb, self.t_lin1, out=ws.emb1)
        ops.gemv(ws.emb1, self.t_lin2, silu_input=True, out=ws.emb)
        ops.gemv(ws.emb, self.mod_all, silu_input=True, out=ws.mods)

    def run(self, prepared: PreparedText, image: torch.Tensor, timestep_x1000: torch.Tensor | float,
            *, euler_dt: float | None = None, sample: torch.Tensor | None = None,
            out: torch.Tensor | None = None) -> torch.Tensor:
        """One transformer evaluation. With `euler_dt`, the final projection's epilogue applies
        the Klein Euler update to `sample` and returns the next latent instead of the velocity
        (kinomlx/models/flux2/sampling.py:109-113, 240)."""
        batch, ni, _ = image.shape
        nt = prepared.text.shape[1]
        ws = self.workspace(batch, nt, ni)
        self._embed(ws, timestep_x1000)
        ws.stream[:, :nt].copy_(prepared.text)
        ops.linear(image, self.x_embedder, ws.stream[:, nt:])
        for p in self.double:
            self._double_block(ws, p, prepared.rope)
        for p in self.single:
            self._single_block(ws, p, prepared.rope)
        d = self.v.dim
        om = lambda j: ws.mods[:, (15 + j) * d : (16 + j) * d]  # [scale | shift]
        ops.adaln(ws.stream[:, nt:], om(1), om(0), ws.nrm[:, nt:], norm=ops.NORM_LAYER)
        if euler_dt is None:
            return ops.linear(ws.nrm[:, nt:], self.proj_out, ws.velocity if out is None else out)
        return ops.linear(ws.nrm[:, nt:], self.proj_out, out, kind=ops.EPI_EULER, dt=euler_dt,
                          sample=sample)
