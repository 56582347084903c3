"""The LTX-2 video DiT in fp32 (parity mode) on the fp32 CUDA-core kernels.

Same call surface as `LTXVideoTransformer` (prepare, run) and the same reference graph
(kinomlx/models/ltx2/transformer/model.py:577-635, transformer.py:178-392,
attention.py:249-371), with every tensor fp32: the reference's model runs in whatever dtype its
arrays carry, and BASELINE's per-op gate for fp32 mode is a max relative error of 1e-4. One
process, one GPU, resident (unpacked) weights.

Per block: AdaLN (RMSNorm) -> gate logits (2*sigmoid epilogue) and the q|k|v projection with
bias -> full-row QK RMSNorm + split RoPE in place -> attention with the per-head gate applied to
its output -> out projection with the gated residual in its epilogue; the text cross-attention
(prompt-modulated context, no RoPE) and the GELU feed-forward follow the same pattern. The final
projection's epilogue applies X0 + Euler.
"""

from __future__ import annotations

import torch

from .. import ops_f32 as f
from .._lib import (EPI_EULER_X0, EPI_GATED_RESIDUAL, EPI_GELU, EPI_SIGMOID2, NORM_LAYER,
                    NORM_NONE, NORM_RMS, QKNORM_FULL_ROW, ROPE_NONE, ROPE_SPLIT)
from ..sequence_parallel import SequenceParallel
from .config import LTXVariant
from .transformer import PreparedContext, context_key_bias, precompute_freqs_cis

F32 = torch.float32


class _Workspace:
    def __init__(self, v: LTXVariant, batch: int, tokens: int, ctx_tokens: int, device):
        d = v.dim
        e = lambda *s: torch.empty(s, device=device, dtype=F32)
        self.x = e(batch, tokens, d)
        self.nrm = e(batch, tokens, d)
        self.hid = e(batch, tokens, v.ff_mult * d)
        self.qkv = e(batch, tokens, 3 * d)  # [q | k | v]
        self.gates = e(batch, tokens, v.heads)
        self.ctxm = e(batch, ctx_tokens, d)
        self.ctxkv = e(batch, ctx_tokens, 2 * d)  # [k | v] of the context
        self.t = e(batch)
        self.temb = e(batch, 256)
        self.h1 = e(batch, d)
        self.emb = e(batch, d)
        self.act = e(batch, d)
        self.mod9 = e(batch, 9 * d)
        self.pemb = e(batch, d)
        self.pmod = e(batch, 2 * d)
        self.vals = e(batch, v.blocks, 9 * d)
        self.prompt = e(batch, v.blocks, 2 * d)
        self.outmod = e(batch, 2 * d)
        self.velocity = e(batch, tokens, v.out_channels)


class LTXVideoTransformerF32:
    """fp32 device LTX-2 video DiT; `weights` uses the reference checkpoint names (any float
    dtype, converted to fp32 once)."""

    dtype = F32

    def __init__(self, weights: dict[str, torch.Tensor], variant: LTXVariant,
                 device: torch.device | str = "cuda"):
        if variant.head_dim != 128:
            raise ValueError("the fp32 kernels take 128-wide heads")
        if not variant.gated_attention:
            raise ValueError("the fp32 LTX block is built for gated attention")
        self.sp = SequenceParallel.single()
        self.v = variant
        self.device = torch.device(device)
        dev = lambda t: t.to(self.device, F32).contiguous()
        w = weights
        self.patch_w, self.patch_b = dev(w["patchify_proj.weight"]), dev(w["patchify_proj.bias"])

        def adaln(prefix):
            g = lambda n: dev(w[f"{prefix}.{n}"])
            return {
                "l1w": g("emb.timestep_embedder.linear_1.weight"),
                "l1b": g("emb.timestep_embedder.linear_1.bias"),
                "l2w": g("emb.timestep_embedder.linear_2.weight"),
                "l2b": g("emb.timestep_embedder.linear_2.bias"),
                "w": g("linear.weight"),
                "b": g("linear.bias"),
            }

        self.adaln = adaln("adaln_single")
        self.prompt_adaln = adaln("prompt_adaln_single")
        tables, prompts = [], []
        self.blocks = []
        for i in range(variant.blocks):
            a = f"transformer_blocks.{i}"
            g = lambda n: w[f"{a}.{n}"]
            tables.append(g("scale_shift_table").reshape(-1))
            prompts.append(g("prompt_scale_shift_table").reshape(-1))
            self.blocks.append({
                "qkv_w": dev(torch.cat([g("attn1.to_q.weight"), g("attn1.to_k.weight"), g("attn1.to_v.weight")])),
                "qkv_b": dev(torch.cat([g("attn1.to_q.bias"), g("attn1.to_k.bias"), g("attn1.to_v.bias")])),
                "g1_w": dev(g("attn1.to_gate_logits.weight")),
                "g1_b": dev(g("attn1.to_gate_logits.bias")),
                "o1_w": dev(g("attn1.to_out.weight")),
                "o1_b": dev(g("attn1.to_out.bias")),
                "qn1": dev(g("attn1.q_norm.weight")),
                "kn1": dev(g("attn1.k_norm.weight")),
                "q2_w": dev(g("attn2.to_q.weight")),
                "q2_b": dev(g("attn2.to_q.bias")),
                "kv2_w": dev(torch.cat([g("attn2.to_k.weight"), g("attn2.to_v.weight")])),
                "kv2_b": dev(torch.cat([g("attn2.to_k.bias"), g("attn2.to_v.bias")])),
                "g2_w": dev(g("attn2.to_gate_logits.weight")),
                "g2_b": dev(g("attn2.to_gate_logits.bias")),
                "o2_w": dev(g("attn2.to_out.weight")),
                "o2_b": dev(g("attn2.to_out.bias")),
                "qn2": dev(g("attn2.q_norm.weight")),
                "kn2": dev(g("attn2.k_norm.weight")),
                "ff_in_w": dev(g("ff.project_in.proj.weight")),
                "ff_in_b": dev(g("ff.project_in.proj.bias")),
                "ff_out_w": dev(g("ff.project_out.weight")),
                "ff_out_b": dev(g("ff.project_out.bias")),
            })
        self.tables = dev(torch.stack(tables))  # (L, 9D)
        self.prompt_tables = dev(torch.stack(prompts))  # (L, 2D)
        self.out_table = dev(w["scale_shift_table"])  # (2, D)
        self.proj_w, self.proj_b = dev(w["proj_out.weight"]), dev(w["proj_out.bias"])
        self._ws: dict[tuple[int, int, int], _Workspace] = {}

    def prepare(self, context: torch.Tensor, positions: torch.Tensor,
                context_mask: torch.Tensor | None = None) -> PreparedContext:
        cos, sin = precompute_freqs_cis(positions.cpu(), self.v)
        bias = context_key_bias(context_mask, context.shape[0], context.shape[1], self.device,
                                dtype=F32)
        return PreparedContext(context.to(self.device, F32).contiguous(), cos.to(self.device),
                               sin.to(self.device), bias)

    def workspace(self, batch: int, tokens: int, ctx_tokens: int) -> _Workspace:
        key = (batch, tokens, ctx_tokens)
        if key not in self._ws:
            self._ws[key] = _Workspace(self.v, batch, tokens, ctx_tokens, self.device)
        return self._ws[key]

    # ------------------------------------------------------------------ per step embeddings
    def _embed(self, ws: _Workspace, sigma: float) -> None:
        """AdaLayerNormSingle for the block modulations and the prompt AdaLN
        (kinomlx/models/ltx2/transformer/preprocessing.py:66-83, timestep.py:31-85):
        linear(silu(emb)) with emb = linear_2(silu(linear_1(sinusoid(t))))."""
        ws.t.fill_(float(torch.tensor(sigma, dtype=F32) * self.v.timestep_scale))
        f.timestep_embedding(ws.t, 256, out=ws.temb)
        for p, emb, mod in ((self.adaln, ws.emb, ws.mod9), (self.prompt_adaln, ws.pemb, ws.pmod)):
            f.linear(ws.temb, p["l1w"], ws.h1, bias=p["l1b"])
            f.silu(ws.h1, out=ws.act)
            f.linear(ws.act, p["l2w"], emb, bias=p["l2b"])
            f.silu(emb, out=ws.act)
            f.linear(ws.act, p["w"], mod, bias=p["b"])
        for b in range(ws.x.shape[0]):
            f.add_rows(self.tables, ws.mod9[b], out=ws.vals[b])
            f.add_rows(self.prompt_tables, ws.pmod[b], out=ws.prompt[b])
            f.add_rows(self.out_table, ws.emb[b], out=ws.outmod[b].view(2, -1))

    # ------------------------------------------------------------------ block
    def _block(self, ws: _Workspace, i: int, p: dict, prepared: PreparedContext) -> None:
        v, d, h = self.v, self.v.dim, self.v.heads
        val = lambda j: ws.vals[:, i, j * d : (j + 1) * d]
        x, nrm = ws.x, ws.nrm
        q, k, vv = ws.qkv[..., :d], ws.qkv[..., d : 2 * d], ws.qkv[..., 2 * d :]
        # self-attention
        f.adaln(x, val(0), val(1), nrm, norm=NORM_RMS, eps=v.eps)
        f.linear(nrm, p["g1_w"], ws.gates, bias=p["g1_b"], kind=EPI_SIGMOID2)
        f.linear(nrm, p["qkv_w"], ws.qkv, bias=p["qkv_b"])
        for t, wn in ((q, p["qn1"]), (k, p["kn1"])):
            f.qk_norm_rope(t, heads=h, weight=wn, norm=QKNORM_FULL_ROW, rope=ROPE_SPLIT,
                           cos=prepared.cos, sin=prepared.sin, eps=v.eps)
        f.attention(q, k, vv, q, heads=h, gate=ws.gates)
        f.linear(q, p["o1_w"], x, bias=p["o1_b"], kind=EPI_GATED_RESIDUAL, residual=x, gate=val(2))
        # text cross-attention with the prompt-modulated context
        pr = lambda j: ws.prompt[:, i, j * d : (j + 1) * d]
        f.adaln(x, val(6), val(7), nrm, norm=NORM_RMS, eps=v.eps)
        f.adaln(prepared.context, pr(0), pr(1), ws.ctxm, norm=NORM_NONE)
        f.linear(nrm, p["g2_w"], ws.gates, bias=p["g2_b"], kind=EPI_SIGMOID2)
        f.linear(nrm, p["q2_w"], q, bias=p["q2_b"])
        f.linear(ws.ctxm, p["kv2_w"], ws.ctxkv, bias=p["kv2_b"])
        k2, v2 = ws.ctxkv[..., :d], ws.ctxkv[..., d:]
        f.qk_norm_rope(q, heads=h, weight=p["qn2"], norm=QKNORM_FULL_ROW, rope=ROPE_NONE, eps=v.eps)
        f.qk_norm_rope(k2, heads=h, weight=p["kn2"], norm=QKNORM_FULL_ROW, rope=ROPE_NONE, eps=v.eps)
        f.attention(q, k2, v2, q, heads=h, gate=ws.gates, key_bias=prepared.key_bias)
        f.linear(q, p["o2_w"], x, bias=p["o2_b"], kind=EPI_GATED_RESIDUAL, residual=x, gate=val(8))
        # feed-forward
        f.adaln(x, val(3), val(4), nrm, norm=NORM_RMS, eps=v.eps)
        f.linear(nrm, p["ff_in_w"], ws.hid, bias=p["ff_in_b"], kind=EPI_GELU)
        f.linear(ws.hid, p["ff_out_w"], x, bias=p["ff_out_b"], kind=EPI_GATED_RESIDUAL,
                 residual=x, gate=val(5))

    # ------------------------------------------------------------------ forward
    def run(self, prepared: PreparedContext, latent: torch.Tensor, sigma: float, *,
            sigma_next: float | None = None, out: torch.Tensor | None = None,
            blocks: range | None = None) -> torch.Tensor:
        """Velocity for `latent` (B, T, C) at `sigma`; with `sigma_next`, the next latent of the
        deterministic Euler step (X0 + Euler fused into the final projection)."""
        batch, tokens, _ = latent.shape
        ws = self.workspace(batch, tokens, prepared.context.shape[1])
        self._embed(ws, sigma)
        f.linear(latent, self.patch_w, ws.x, bias=self.patch_b)
        for i in blocks if blocks is not None else range(self.v.blocks):
            self._block(ws, i, self.blocks[i], prepared)
        d = self.v.dim
        f.adaln(ws.x, ws.outmod[:, :d], ws.outmod[:, d:], ws.nrm, norm=NORM_LAYER, eps=self.v.eps)
        if sigma_next is None:
            return f.linear(ws.nrm, self.proj_w, ws.velocity if out is None else out,
                            bias=self.proj_b)
        ratio = float(torch.tensor(sigma_next / sigma, dtype=F32))
        return f.linear(ws.nrm, self.proj_w, out, bias=self.proj_b, kind=EPI_EULER_X0,
                        sigma=float(torch.tensor(sigma, dtype=F32)), ratio=ratio, sample=latent)
