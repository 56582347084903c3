"""The Flux2-style MMDiT in fp32 (parity mode) on the fp32 CUDA-core kernels.

Same call surface as `Flux2Transformer` (prepare, run, double_block, single_block) and the same
reference graph (kinomlx/models/flux2/transformer.py:88-358), with every tensor fp32: the
reference's models run in whatever dtype their arrays carry, and BASELINE config 1 asks for the
double block in fp32 as well as bf16. One process, one GPU (no sequence parallelism).

Memory layout (one workspace per batch/token shape):
  stream (B, Nt+Ni, D)   text rows then image rows (the single blocks' concatenation is free)
  nrm    (B, N, D)       AdaLN output
  qkv    (B, N, 3D)      [q | k | v] of both streams; attention writes its output over q
  hid    (B, N, M)       MLP up-projection (M = GELU width, or 2H for SwiGLU: [gate | content],
                         the activated H columns written over the gate half)
  big    (B, N, 3D+M)    single-block projection reordered [k | v | q | mlp], so the attention
                         output (over q) and the activated MLP form one contiguous to_out operand
"""

from __future__ import annotations

import torch

from .. import ops_f32 as f
from .._lib import EPI_EULER, EPI_GATED_RESIDUAL, EPI_GELU, NORM_LAYER, QKNORM_PER_HEAD, ROPE_PAIRS
from ..sequence_parallel import SequenceParallel
from .config import FluxVariant
from .transformer import rotary_positions

F32 = torch.float32


class PreparedTextF32:
    """Once-per-generation state (kinomlx/models/flux2/transformer.py:283-292), fp32."""

    def __init__(self, text: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        self.text = text  # (B, Nt, D)
        self.cos = cos  # (1|B, N, 128) token-major
        self.sin = sin


class _Workspace:
    def __init__(self, v: FluxVariant, batch: int, nt: int, ni: int, device: torch.device):
        n, d = nt + ni, v.dim
        e = lambda *shape: torch.empty(shape, device=device, dtype=F32)
        self.batch, self.nt, self.ni = batch, nt, ni
        self.stream = e(batch, n, d)
        self.nrm = e(batch, n, d)
        self.qkv = e(batch, n, 3 * d)
        self.hid = e(batch, n, v.mlp_in)
        self.big = e(batch, n, 3 * d + v.mlp_in)
        self.t = e(batch)
        self.temb = e(batch, 256)
        self.emb1 = e(batch, d)
        self.emb = e(batch, d)
        self.act = e(batch, d)
        self.mods = e(batch, 17 * d)
        self.velocity = e(batch, ni, v.in_channels)


class Flux2TransformerF32:
    """fp32 device Flux2 MMDiT; `weights` uses the reference checkpoint names (any float dtype,
    converted to fp32 once)."""

    dtype = F32

    def __init__(self, weights: dict[str, torch.Tensor], variant: FluxVariant,
                 device: torch.device | str = "cuda"):
        if variant.mlp not in ("gelu_tanh", "swiglu"):
            raise ValueError(f"unknown MLP kind {variant.mlp!r}")
        if variant.head_dim != 128:
            raise ValueError("the fp32 kernels take 128-wide heads")
        self.sp = SequenceParallel.single()
        self.v = variant
        self.device = torch.device(device)
        dev = lambda t: t.to(self.device, F32).contiguous()
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
                "ff_in": dev(w[f"{a}.ff.linear_in.weight"]),
                "ff_out": dev(w[f"{a}.ff.linear_out.weight"]),
                "ffc_in": dev(w[f"{a}.ff_context.linear_in.weight"]),
                "ffc_out": dev(w[f"{a}.ff_context.linear_out.weight"]),
            })
        self.single = []
        for i in range(variant.single_blocks):
            a = f"single_transformer_blocks.{i}.attn"
            fused = w[f"{a}.to_qkv_mlp_proj.weight"]
            q, k, vv, mlp = fused[:d], fused[d : 2 * d], fused[2 * d : 3 * d], fused[3 * d :]
            self.single.append({
                "fused": dev(torch.cat([k, vv, q, mlp])),  # [k | v | q | mlp]
                "to_out": dev(w[f"{a}.to_out.weight"]),
                "norm_q": dev(w[f"{a}.norm_q.weight"]),
                "norm_k": dev(w[f"{a}.norm_k.weight"]),
            })
        self.proj_out = dev(w["proj_out.weight"])
        self._ws: dict[tuple[int, int, int], _Workspace] = {}

    # ------------------------------------------------------------------ preparation
    def prepare(self, text: torch.Tensor, ids: torch.Tensor) -> PreparedTextF32:
        """Project the text once and build the RoPE tables for the joint [text, image] ids."""
        projected = f.linear(text.to(self.device, F32), self.context_embedder)
        cos, sin = rotary_positions(ids, self.v)
        return PreparedTextF32(projected, cos.to(self.device).contiguous(),
                               sin.to(self.device).contiguous())

    def workspace(self, batch: int, nt: int, ni: int) -> _Workspace:
        key = (batch, nt, ni)
        if key not in self._ws:
            self._ws[key] = _Workspace(self.v, batch, nt, ni, self.device)
        return self._ws[key]

    # ------------------------------------------------------------------ blocks
    def _qk(self, x: torch.Tensor, weight: torch.Tensor, cos, sin, offset: int) -> None:
        f.qk_norm_rope(x, heads=self.v.heads, weight=weight, norm=QKNORM_PER_HEAD,
                       rope=ROPE_PAIRS, cos=cos, sin=sin, table_offset=offset)

    def _mlp(self, x: torch.Tensor, w_in: torch.Tensor, w_out: torch.Tensor, hid: torch.Tensor,
             residual: torch.Tensor, gate: torch.Tensor) -> None:
        """residual += gate * w_out(act(w_in(x))) (kinomlx/models/flux2/transformer.py:78-85)."""
        if self.v.mlp == "gelu_tanh":
            f.linear(x, w_in, hid, kind=EPI_GELU)
            act = hid
        else:
            f.linear(x, w_in, hid)
            act = f.swiglu(hid, out=hid[..., : self.v.mlp_hidden])
        f.linear(act, w_out, residual, kind=EPI_GATED_RESIDUAL, residual=residual, gate=gate)

    def _double_block(self, ws: _Workspace, p: dict, cos, sin) -> None:
        """DoubleBlock + DoubleAttention (kinomlx/models/flux2/transformer.py:88-167)."""
        d, nt, h = self.v.dim, ws.nt, self.v.heads
        txt, img = ws.stream[:, :nt], ws.stream[:, nt:]
        txt_n, img_n = ws.nrm[:, :nt], ws.nrm[:, nt:]
        m = lambda base, j: ws.mods[:, (base + j) * d : (base + j + 1) * d]  # img base 0, txt 6
        f.adaln(img, m(0, 0), m(0, 1), img_n, norm=NORM_LAYER)
        f.adaln(txt, m(6, 0), m(6, 1), txt_n, norm=NORM_LAYER)
        f.linear(img_n, p["img_qkv"], ws.qkv[:, nt:])
        f.linear(txt_n, p["txt_qkv"], ws.qkv[:, :nt])
        q, k, v = ws.qkv[..., :d], ws.qkv[..., d : 2 * d], ws.qkv[..., 2 * d :]
        self._qk(q[:, nt:], p["norm_q"], cos, sin, nt)
        self._qk(k[:, nt:], p["norm_k"], cos, sin, nt)
        self._qk(q[:, :nt], p["norm_added_q"], cos, sin, 0)
        self._qk(k[:, :nt], p["norm_added_k"], cos, sin, 0)
        f.attention(q, k, v, q, heads=h)
        f.linear(q[:, nt:], p["to_out"], img, kind=EPI_GATED_RESIDUAL, residual=img, gate=m(0, 2))
        f.linear(q[:, :nt], p["to_add_out"], txt, kind=EPI_GATED_RESIDUAL, residual=txt,
                 gate=m(6, 2))
        f.adaln(img, m(0, 3), m(0, 4), img_n, norm=NORM_LAYER)
        self._mlp(img_n, p["ff_in"], p["ff_out"], ws.hid[:, nt:], img, m(0, 5))
        f.adaln(txt, m(6, 3), m(6, 4), txt_n, norm=NORM_LAYER)
        self._mlp(txt_n, p["ffc_in"], p["ffc_out"], ws.hid[:, :nt], txt, m(6, 5))

    def _single_block(self, ws: _Workspace, p: dict, cos, sin) -> None:
        """SingleBlock + SingleAttention (kinomlx/models/flux2/transformer.py:170-220)."""
        d, h = self.v.dim, self.v.heads
        sm = lambda j: ws.mods[:, (12 + j) * d : (13 + j) * d]
        f.adaln(ws.stream, sm(0), sm(1), ws.nrm, norm=NORM_LAYER)
        if self.v.mlp == "gelu_tanh":
            f.linear(ws.nrm, p["fused"], ws.big, kind=EPI_GELU, act_col_begin=3 * d)
            width = 3 * d + self.v.mlp_hidden
        else:
            f.linear(ws.nrm, p["fused"], ws.big)
            f.swiglu(ws.big[..., 3 * d :], out=ws.big[..., 3 * d : 3 * d + self.v.mlp_hidden])
            width = 3 * d + self.v.mlp_hidden
        k, v, q = ws.big[..., :d], ws.big[..., d : 2 * d], ws.big[..., 2 * d : 3 * d]
        self._qk(k, p["norm_k"], cos, sin, 0)
        self._qk(q, p["norm_q"], cos, sin, 0)
        f.attention(q, k, v, q, heads=h)
        f.linear(ws.big[..., 2 * d : width], p["to_out"], ws.stream, kind=EPI_GATED_RESIDUAL,
                 residual=ws.stream, gate=sm(2))

    def double_block(self, index: int, image: torch.Tensor, text: torch.Tensor,
                     timestep_x1000: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """One DoubleBlock on fp32 hidden states (BASELINE config 1 in fp32): the timestep MLP,
        its modulations and block `index`; returns new (image, text) hidden states."""
        batch, ni, _ = image.shape
        nt = text.shape[1]
        ws = self.workspace(batch, nt, ni)
        self._embed(ws, timestep_x1000)
        ws.stream[:, :nt].copy_(text)
        ws.stream[:, nt:].copy_(image)
        self._double_block(ws, self.double[index], cos.contiguous(), sin.contiguous())
        return ws.stream[:, nt:].clone(), ws.stream[:, :nt].clone()

    def single_block(self, index: int, value: torch.Tensor, text_tokens: int,
                     timestep_x1000: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """One SingleBlock on the joint fp32 hidden state (B, Nt+Ni, D)."""
        batch, n, _ = value.shape
        ws = self.workspace(batch, text_tokens, n - text_tokens)
        self._embed(ws, timestep_x1000)
        ws.stream.copy_(value)
        self._single_block(ws, self.single[index], cos.contiguous(), sin.contiguous())
        return ws.stream.clone()

    # ------------------------------------------------------------------ forward
    def _embed(self, ws: _Workspace, timestep_x1000: torch.Tensor | float) -> None:
        """Timestep MLP and every modulation vector (kinomlx/models/flux2/transformer.py:223-258,
        315-318): linear_2(silu(linear_1(sinusoid(t)))), then linear(silu(emb)) for all four."""
        if isinstance(timestep_x1000, torch.Tensor):
            ws.t.copy_(timestep_x1000, non_blocking=True)
        else:  # one value for every batch entry: a fill, no host-to-device copy
            ws.t.fill_(float(timestep_x1000))
        f.timestep_embedding(ws.t, 256, out=ws.temb)
        f.linear(ws.temb, self.t_lin1, ws.emb1)
        f.silu(ws.emb1, out=ws.act)
        f.linear(ws.act, self.t_lin2, ws.emb)
        f.silu(ws.emb, out=ws.act)
        f.linear(ws.act, self.mod_all, ws.mods)

    def run(self, prepared: PreparedTextF32, image: torch.Tensor, timestep_x1000: torch.Tensor | float,
            *, euler_dt: float | None = None, sample: torch.Tensor | None = None,
            out: torch.Tensor | None = None, target: tuple[int, int] | None = None) -> torch.Tensor:
        """One transformer evaluation (kinomlx/models/flux2/transformer.py:307-358). With
        `euler_dt`, the final projection's epilogue applies the Euler update to `sample` and
        returns the next latent instead of the velocity. `target` = (first row, rows) of `image`
        whose velocity is produced (default all)."""
        batch, ni, _ = image.shape
        nt = prepared.text.shape[1]
        first, rows = (0, ni) if target is None else target
        if first < 0 or rows < 1 or first + rows > ni:
            raise ValueError(f"target rows {target} outside the {ni} image rows")
        ws = self.workspace(batch, nt, ni)
        self._embed(ws, timestep_x1000)
        ws.stream[:, :nt].copy_(prepared.text)
        f.linear(image, self.x_embedder, ws.stream[:, nt:])
        for p in self.double:
            self._double_block(ws, p, prepared.cos, prepared.sin)
        for p in self.single:
            self._single_block(ws, p, prepared.cos, prepared.sin)
        d = self.v.dim
        om = lambda j: ws.mods[:, (15 + j) * d : (16 + j) * d]  # [scale | shift]
        r0, r1 = nt + first, nt + first + rows
        f.adaln(ws.stream[:, r0:r1], om(1), om(0), ws.nrm[:, r0:r1], norm=NORM_LAYER)
        if euler_dt is None:
            return f.linear(ws.nrm[:, r0:r1], self.proj_out, ws.velocity[:, :rows] if out is None else out)
        return f.linear(ws.nrm[:, r0:r1], self.proj_out, out, kind=EPI_EULER, dt=euler_dt,
                        sample=sample)
