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

KV editing (kinomlx/models/flux2/kv.py, transformer.py:319-350): an extracting evaluation holds
[text | reference | target] rows in `stream`; the reference rows take the modulations of
timestep 0 (a second modulation vector, `mods_fixed`), their queries attend to reference keys
only, and each layer's reference keys/values are kept in a ReferenceKV. A reusing evaluation
holds [text | target] rows and attends to the kept rows as a second key segment.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from ..sequence_parallel import SequenceParallel
from .config import FluxVariant
from .kv import ReferenceKV, attend_rows

BF = torch.bfloat16


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
        e = lambda *shape: torch.empty(shape, device=device, dtype=BF)
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
        self.mods_fixed = e(batch, 17 * d)  # timestep-0 modulations of KV-extraction reference rows
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
        dev = lambda t: t.to(self.device, BF).contiguous()
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

    @property
    def dtype(self) -> torch.dtype:
        return BF

    @property
    def layer_count(self) -> int:
        return len(self.double) + len(self.single)

    # ------------------------------------------------------------------ preparation
    def prepare(self, text: torch.Tensor, ids: torch.Tensor) -> PreparedText:
        """Project the text once and build the RoPE tables for the joint [text, image] ids."""
        text = text.to(self.device, BF)
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

    def prepare_layouts(self, text: torch.Tensor, ids: tuple[torch.Tensor, ...]) -> tuple[PreparedText, ...]:
        """The text projected once, with RoPE tables for each joint [text, image] id layout
        (kinomlx/models/flux2/transformer.py:283-292): KV editing evaluates [text, reference,
        target] rows first and [text, target] rows after that. One GPU."""
        if self.sp.size > 1:
            raise ValueError("several id layouts need the whole sequence on one GPU")
        projected = ops.linear(text.to(self.device, BF), self.context_embedder)
        out = []
        for joint in ids:
            cos, sin = rotary_positions(joint, self.v)
            out.append(PreparedText(projected, ops.RopeTables(cos.to(self.device), sin.to(self.device))))
        return tuple(out)

    def new_reference_kv(self, reference_tokens: int, batch: int = 1) -> ReferenceKV:
        """An empty reference K/V cache for one edit (kinomlx/models/flux2/transformer.py:279-282)."""
        if self.sp.size > 1:
            raise ValueError("reference K/V editing runs on one GPU")
        return ReferenceKV(reference_tokens, self.layer_count, batch, self.v.dim, self.device, BF)

    def workspace(self, batch: int, nt: int, ni: int) -> _Workspace:
        key = (batch, nt, ni)
        if key not in self._ws:
            self._ws[key] = _Workspace(self.v, batch, nt, ni, self.device, self.sp)
        return self._ws[key]

    # ------------------------------------------------------------------ blocks
    def _attend(self, q, k, v, kv: ReferenceKV | None, layer: int, nt: int = 0) -> None:
        """Self-attention written over q; with a reference K/V cache, its extracting or reusing
        form (kinomlx/models/flux2/kv.py:57-80)."""
        if kv is None:
            self.sp.attention(q, k, v, q, heads=self.v.heads)
            return
        attend_rows(q, k, v, q, heads=self.v.heads, text_tokens=nt, state=kv, layer=layer)

    def _double_block(self, ws: _Workspace, p: dict, rope: ops.RopeTables,
                      kv: ReferenceKV | None = None, layer: int = 0) -> None:
        if kv is not None and kv.extracting:
            self._double_block_extracting(ws, p, rope, kv, layer)
            return
        if ws.nt % 256 == 0 and ws.ni > 0:
            self._double_block_joint(ws, p, rope, kv, layer)
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
            self._attend(q, k, v, kv, layer)
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

    def _double_block_joint(self, ws: _Workspace, p: dict, rope: ops.RopeTables,
                            kv: ReferenceKV | None = None, layer: int = 0) -> None:
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
            self._attend(q, k, v, kv, layer)
        ops.linear(q, p["to_out"], ws.stream, kind=ops.EPI_GATED_RESIDUAL, residual=ws.stream,
                   gate=m(0, 2), lead_w=p["to_add_out"], lead_rows=nt, lead_gate=m(6, 2))
        ops.adaln(img, m(0, 3), m(0, 4), img_n, norm=ops.NORM_LAYER)
        ops.adaln(txt, m(6, 3), m(6, 4), txt_n, norm=ops.NORM_LAYER)
        ops.linear(ws.nrm, p["ff_in"], ws.hid, kind=self.act_kind, lead_w=p["ffc_in"],
                   lead_rows=nt)
        ops.linear(ws.hid, p["ff_out"], ws.stream, kind=ops.EPI_GATED_RESIDUAL,
                   residual=ws.stream, gate=m(0, 5), lead_w=p["ffc_out"], lead_rows=nt,
                   lead_gate=m(6, 5))

    def _double_block_extracting(self, ws: _Workspace, p: dict, rope: ops.RopeTables,
                                 kv: ReferenceKV, layer: int) -> None:
        """The double block on [text | reference | target] rows: reference rows use the image
        modulation of timestep 0 (kinomlx/models/flux2/transformer.py:333-339, 139-153), so
        each image-row AdaLN and gated residual runs once per row range."""
        d, nt = self.v.dim, ws.nt
        r0, r1 = nt, nt + kv.reference_tokens
        txt, img = ws.stream[:, :nt], ws.stream[:, nt:]
        txt_n, img_n = ws.nrm[:, :nt], ws.nrm[:, nt:]
        m = lambda base, j: ws.mods[:, (base + j) * d : (base + j + 1) * d]  # img base 0, txt 6
        mf = lambda base, j: ws.mods_fixed[:, (base + j) * d : (base + j + 1) * d]
        image_rows = ((r0, r1, mf), (r1, nt + ws.ni, m))
        for a, b, mod in image_rows:
            ops.adaln(ws.stream[:, a:b], mod(0, 0), mod(0, 1), ws.nrm[:, a:b], norm=ops.NORM_LAYER)
        ops.adaln(txt, m(6, 0), m(6, 1), txt_n, norm=ops.NORM_LAYER)
        ops.linear(img_n, p["img_qkv"], ws.qkv[:, nt:], qk_norm=[(0, p["norm_q"]), (d, p["norm_k"])],
                   norm_width=d, rope=(rope, nt))
        ops.linear(txt_n, p["txt_qkv"], ws.qkv[:, :nt],
                   qk_norm=[(0, p["norm_added_q"]), (d, p["norm_added_k"])], norm_width=d,
                   rope=(rope, 0))
        q, k, v = ws.qkv[..., :d], ws.qkv[..., d : 2 * d], ws.qkv[..., 2 * d :]
        self._attend(q, k, v, kv, layer, nt)
        for a, b, mod in image_rows:
            rows = ws.stream[:, a:b]
            ops.linear(q[:, a:b], p["to_out"], rows, kind=ops.EPI_GATED_RESIDUAL, residual=rows,
                       gate=mod(0, 2))
        ops.linear(q[:, :nt], p["to_add_out"], txt, kind=ops.EPI_GATED_RESIDUAL, residual=txt,
                   gate=m(6, 2))
        for a, b, mod in image_rows:
            ops.adaln(ws.stream[:, a:b], mod(0, 3), mod(0, 4), ws.nrm[:, a:b], norm=ops.NORM_LAYER)
        ops.linear(img_n, p["ff_in"], ws.hid[:, nt:], kind=self.act_kind)
        for a, b, mod in image_rows:
            rows = ws.stream[:, a:b]
            ops.linear(ws.hid[:, a:b], p["ff_out"], rows, kind=ops.EPI_GATED_RESIDUAL,
                       residual=rows, gate=mod(0, 5))
        ops.adaln(txt, m(6, 3), m(6, 4), txt_n, norm=ops.NORM_LAYER)
        ops.linear(txt_n, p["ffc_in"], ws.hid[:, :nt], kind=self.act_kind)
        ops.linear(ws.hid[:, :nt], p["ffc_out"], txt, kind=ops.EPI_GATED_RESIDUAL, residual=txt,
                   gate=m(6, 5))

    def _single_block(self, ws: _Workspace, p: dict, rope: ops.RopeTables,
                      kv: ReferenceKV | None = None, layer: int = 0) -> None:
        if kv is not None and kv.extracting:
            self._single_block_extracting(ws, p, rope, kv, layer)
            return
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
            self._attend(q, k, v, kv, layer)
        ops.linear(ws.big[..., 2 * d :], p["to_out"], ws.stream, kind=ops.EPI_GATED_RESIDUAL,
                   residual=ws.stream, gate=sm(2))

    def _single_block_extracting(self, ws: _Workspace, p: dict, rope: ops.RopeTables,
                                 kv: ReferenceKV, layer: int) -> None:
        """The single block on [text | reference | target] rows, reference rows on the single
        modulation of timestep 0 (kinomlx/models/flux2/transformer.py:340-346, 206-220)."""
        d, nt = self.v.dim, ws.nt
        r0, r1 = nt, nt + kv.reference_tokens
        sm = lambda j: ws.mods[:, (12 + j) * d : (13 + j) * d]
        smf = lambda j: ws.mods_fixed[:, (12 + j) * d : (13 + j) * d]
        parts = ((0, r0, sm), (r0, r1, smf), (r1, nt + ws.ni, sm))
        for a, b, mod in parts:
            ops.adaln(ws.stream[:, a:b], mod(0), mod(1), ws.nrm[:, a:b], norm=ops.NORM_LAYER)
        ops.linear(ws.nrm, p["fused"], ws.big, kind=self.act_kind, act_col_begin=3 * d,
                   qk_norm=[(0, p["norm_k"]), (2 * d, p["norm_q"])], norm_width=d, rope=(rope, 0))
        k, v, q = ws.big[..., :d], ws.big[..., d : 2 * d], ws.big[..., 2 * d : 3 * d]
        self._attend(q, k, v, kv, layer, nt)
        for a, b, mod in parts:
            rows = ws.stream[:, a:b]
            ops.linear(ws.big[:, a:b, 2 * d :], p["to_out"], rows, kind=ops.EPI_GATED_RESIDUAL,
                       residual=rows, gate=mod(2))

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
    def _embed(self, ws: _Workspace, timestep_x1000: torch.Tensor | float,
               mods: torch.Tensor | None = None) -> None:
        """Timestep MLP and every modulation vector (kinomlx/models/flux2/transformer.py:315-318)
        into `mods` (default ws.mods)."""
        if isinstance(timestep_x1000, torch.Tensor):
            ws.t.copy_(timestep_x1000, non_blocking=True)
        else:  # one value for every batch entry: a fill, no host-to-device copy
            ws.t.fill_(float(timestep_x1000))
        ops.timestep_embedding(ws.t, 256, out=ws.temb)
        ops.gemv(ws.temb, self.t_lin1, out=ws.emb1)
        ops.gemv(ws.emb1, self.t_lin2, silu_input=True, out=ws.emb)
        ops.gemv(ws.emb, self.mod_all, silu_input=True, out=ws.mods if mods is None else mods)

    def run(self, prepared: PreparedText, image: torch.Tensor, timestep_x1000: torch.Tensor | float,
            *, euler_dt: float | None = None, sample: torch.Tensor | None = None,
            out: torch.Tensor | None = None, reference_kv: ReferenceKV | None = None,
            target: tuple[int, int] | None = None) -> torch.Tensor:
        """One transformer evaluation. With `euler_dt`, the final projection's epilogue applies
        the Klein Euler update to `sample` and returns the next latent instead of the velocity
        (kinomlx/models/flux2/sampling.py:109-113, 240).

        `target` = (first row, rows) of `image` whose velocity is produced (default: all; image
        rows appended as in-context references are left out this way). With `reference_kv`
        extracting, `image` is [reference | target] rows and the target is every row after the
        references (kinomlx/models/flux2/transformer.py:319-358)."""
        batch, ni, _ = image.shape
        nt = prepared.text.shape[1]
        if reference_kv is not None:
            self._check_reference_kv(reference_kv, batch, ni)
            if reference_kv.extracting:
                nr = reference_kv.reference_tokens
                target = (nr, ni - nr)
        if target is not None and self.sp.size > 1:
            raise ValueError("target rows need the whole sequence on one GPU")
        first, rows = (0, ni) if target is None else target
        if first < 0 or rows < 1 or first + rows > ni:
            raise ValueError(f"target rows {target} outside the {ni} image rows")
        ws = self.workspace(batch, nt, ni)
        kv = reference_kv
        if kv is not None and kv.extracting:
            self._embed(ws, 0.0, ws.mods_fixed)
        self._embed(ws, timestep_x1000)
        ws.stream[:, :nt].copy_(prepared.text)
        ops.linear(image, self.x_embedder, ws.stream[:, nt:])
        for i, p in enumerate(self.double):
            self._double_block(ws, p, prepared.rope, kv, i)
        for i, p in enumerate(self.single, len(self.double)):
            self._single_block(ws, p, prepared.rope, kv, i)
        d = self.v.dim
        om = lambda j: ws.mods[:, (15 + j) * d : (16 + j) * d]  # [scale | shift]
        r0, r1 = nt + first, nt + first + rows
        ops.adaln(ws.stream[:, r0:r1], om(1), om(0), ws.nrm[:, r0:r1], norm=ops.NORM_LAYER)
        if euler_dt is None:
            dst = ws.velocity[:, :rows] if out is None else out
            return ops.linear(ws.nrm[:, r0:r1], self.proj_out, dst)
        return ops.linear(ws.nrm[:, r0:r1], self.proj_out, out, kind=ops.EPI_EULER, dt=euler_dt,
                          sample=sample)

    def _check_reference_kv(self, kv: ReferenceKV, batch: int, image_rows: int) -> None:
        """The reference's refusals (kinomlx/models/flux2/transformer.py:321-332)."""
        if kv.closed:
            raise ValueError("Reference K/V belongs to a completed generation")
        if kv.layer_count != self.layer_count:
            raise ValueError("Reference K/V layer count does not match the transformer")
        if kv.batch != batch:
            raise ValueError("Reference K/V batch does not match the image batch")
        if self.sp.size > 1:
            raise ValueError("reference K/V editing runs on one GPU")
        if kv.extracting and kv.reference_tokens >= image_rows:
            raise ValueError("KV extraction requires reference tokens followed by target tokens")
