"""LTX-2 video DiT on the sm_100a kernels: the device twin of LTXAVModel's video path
(kinomlx/models/ltx2/transformer/model.py:577-635, transformer.py:178-392, attention.py:249-371).

Per block: AdaLN (RMSNorm) -> gate logits (GEMM, 2*sigmoid epilogue) and fused q|k|v projection
with bias -> full-row QK RMSNorm + split RoPE in place -> attention with the per-head gate in its
epilogue -> out projection with the gated residual in its epilogue; the text cross-attention
(prompt-modulated context, no RoPE) and the GELU feed-forward follow the same pattern. The step's
timestep projections are added to every block's modulation table by one kernel. The final
projection's epilogue applies X0 + Euler.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import ops
from ..sequence_parallel import SequenceParallel
from . import quantization as qz
from .config import LTXVariant

BF = torch.bfloat16


def frequency_grid(theta: float, axes: int, inner_dim: int) -> tuple[float, ...]:
    """theta^(i/(n-1)) * pi/2 on the host in double (kinomlx/models/ltx2/transformer/rope.py:75-92)."""
    count = inner_dim // (2 * axes)
    exps = (0.0,) if count == 1 else tuple(i / (count - 1) for i in range(count))
    return tuple(math.pow(theta, e) * math.pi / 2 for e in exps)


def precompute_freqs_cis(positions: torch.Tensor, v: LTXVariant) -> tuple[torch.Tensor, torch.Tensor]:
    """Split-RoPE tables (B, heads, T, dim/(2 heads)) fp32 from (B, 3, T, 2) pixel bounds using the
    middle of each patch (kinomlx/models/ltx2/transformer/rope.py:95-176)."""
    pos = (positions[..., 0] + positions[..., 1]) / 2.0
    scale = torch.tensor(v.max_pos, dtype=torch.float32)[None, :, None]
    frac = (pos.to(torch.float32) / scale).transpose(1, 2)
    grid = torch.tensor(frequency_grid(v.theta, positions.shape[1], v.dim), dtype=torch.float32)
    freqs = (frac * 2.0 - 1.0)[..., None] * grid[None, None, None, :]
    freqs = freqs.transpose(2, 3).reshape(freqs.shape[0], freqs.shape[1], -1)
    pad = v.dim // 2 - freqs.shape[-1]
    cos, sin = torch.cos(freqs), torch.sin(freqs)
    if pad:
        cos = torch.cat([torch.ones((*cos.shape[:-1], pad)), cos], dim=-1)
        sin = torch.cat([torch.zeros((*sin.shape[:-1], pad)), sin], dim=-1)
    b, t, _ = cos.shape
    cos = cos.reshape(b, t, v.heads, -1).transpose(1, 2).contiguous()
    sin = sin.reshape(b, t, v.heads, -1).transpose(1, 2).contiguous()
    return cos, sin


@dataclass
class PreparedContext:
    context: torch.Tensor  # (B, Tc, D) text after the connector
    cos: torch.Tensor  # (1|B, heads, T, 64) fp32
    sin: torch.Tensor
    key_bias: torch.Tensor | None = None  # (B, Tc rounded up to 4) fp32 text-mask bias


# the most negative finite bf16: a padded text token's additive bias
# (kinomlx/models/ltx2/transformer/preprocessing.py:14-17)
_BF16_MINIMUM = -3.3895313892515355e38


def context_key_bias(mask, batch: int, tokens: int, device,
                     dtype: torch.dtype = torch.bfloat16) -> torch.Tensor | None:
    """The additive bias a text context mask puts on the cross-attention's keys
    (kinomlx/models/ltx2/transformer/preprocessing.py:85-96): a floating-point mask is the bias
    itself, in the model's compute dtype; a boolean or integer mask of 1 (token) / 0 (padding)
    becomes (mask - 1) * 3.3895313892515355e38, i.e. 0 or -3.39e38 (bf16 and fp32 models alike).
    Returned as fp32 (batch, tokens rounded up to 4), the attention kernels' key-bias operand.
    Masks broadcast over the queries only: (B, Tc) or (B, 1, Tc); a per-query (B, Tq, Tc) mask
    is refused."""
    if mask is None:
        return None
    m = torch.as_tensor(mask)
    if m.dim() == 3 and m.shape[1] == 1:
        m = m[:, 0]
    if m.dim() == 1:
        m = m[None]
    if m.dim() != 2:
        raise ValueError("text context masks must be (batch, text tokens); per-query masks are "
                         "not supported by the device attention")
    if m.shape[-1] != tokens or m.shape[0] not in (1, batch):
        raise ValueError(f"text context mask of shape {tuple(m.shape)} does not match "
                         f"{batch} x {tokens} text tokens")
    if m.dtype in (torch.float16, torch.bfloat16, torch.float32):
        bias = m.to(dtype).float()
    else:
        if not bool(((m == 0) | (m == 1)).all()):
            raise ValueError("boolean or integer text masks hold 1 (token) and 0 (padding)")
        bias = torch.where(m.bool(), 0.0, _BF16_MINIMUM).float()
    out = torch.zeros((batch, (tokens + 3) // 4 * 4), dtype=torch.float32)
    out[:, :tokens] = bias.expand(batch, tokens)
    return out.to(device)


class _Workspace:
    def __init__(self, v: LTXVariant, batch: int, tokens: int, ctx_tokens: int, device,
                 sp: SequenceParallel):
        d = v.dim
        e = lambda *s: torch.empty(s, device=device, dtype=BF)
        self.x = e(batch, tokens, d)
        self.nrm = e(batch, tokens, d)
        self.hid = e(batch, tokens, v.ff_mult * d)
        # [v | q | k] projection and the head gates: the self-attention returns its rows into the
        # owners' q columns and reads their gates, so under the peer transport both are shared
        self.peer = sp.peer is not None and batch == 1
        if self.peer:
            self.qkv, self.qkv_ptrs = sp.shared((batch, tokens, 3 * d))
            self.gates, self.gate_ptrs = sp.shared((batch, tokens, v.heads))
        else:
            self.qkv = e(batch, tokens, 3 * d)
            self.gates = e(batch, tokens, v.heads)
        self.ctxm = e(batch, ctx_tokens, d)
        self.ctxkv = e(batch, ctx_tokens, 2 * d)
        self.t = torch.empty((batch,), device=device, dtype=torch.float32)
        self.temb = e(batch, 256)
        self.h1 = e(batch, d)
        self.emb = e(batch, d)
        self.mod9 = e(batch, 9 * d)
        self.ph1 = e(batch, d)
        self.pemb = e(batch, d)
        self.pmod = e(batch, 2 * d)
        self.vals = e(batch, v.blocks, 9 * d)
        self.prompt = e(batch, v.blocks, 2 * d)
        self.outmod = e(batch, 2 * d)
        self.velocity = e(batch, tokens, v.out_channels)


class LTXVideoTransformer:
    """Device LTX-2 video DiT. `weights` uses the reference checkpoint names."""

    @property
    def dtype(self) -> torch.dtype:
        return BF

    def __init__(self, weights: dict[str, torch.Tensor], variant: LTXVariant,
                 device: torch.device | str = "cuda", *, sp: SequenceParallel | None = None,
                 quantize: str = "off"):
        """`sp` shards the video tokens over a process group (Ulysses sequence parallelism for
        the self-attention; the text cross-attention stays local with the full context).
        `quantize` is the reference's `transformer_quantize` (weights/schema.py:13-18): "off",
        "mxfp8-blocks" or "mxfp8-blocks-pretranspose" -- the block linears stay packed in HBM
        (taken as given when the checkpoint has `*.scales`, else converted here) and are
        dequantised into a bf16 scratch right before their GEMMs."""
        if quantize not in qz.MODES:
            raise ValueError(f"unsupported transformer_quantize {quantize!r}")
        self.quantize = quantize
        self.sp = sp if sp is not None else SequenceParallel.single()
        self.v = variant
        self.device = torch.device(device)
        dev = lambda t: t.to(self.device, BF).contiguous()
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
        packed = quantize != "off"
        transposed = quantize == "mxfp8-blocks-pretranspose"
        scratch_elems = 0
        for i in range(variant.blocks):
            a = f"transformer_blocks.{i}"
            g = lambda n: w[f"{a}.{n}"]
            if packed:
                # the block linears, packed; biases and norm weights stay bf16 (below)
                pk = lambda *bases: qz.PackedGroup([
                    qz.packed_from_checkpoint(w, f"{a}.{b}", transposed=transposed,
                                              device=self.device) for b in bases])
                groups = {
                    "qkv_w": pk("attn1.to_v", "attn1.to_q", "attn1.to_k"),
                    "g1_w": pk("attn1.to_gate_logits"),
                    "o1_w": pk("attn1.to_out"),
                    "q2_w": pk("attn2.to_q"),
                    "kv2_w": pk("attn2.to_k", "attn2.to_v"),
                    "g2_w": pk("attn2.to_gate_logits"),
                    "o2_w": pk("attn2.to_out"),
                    "ff_in_w": pk("ff.project_in.proj"),
                    "ff_out_w": pk("ff.project_out"),
                }
                scratch_elems = max([scratch_elems] + [gr.out_features * gr.in_features
                                                       for gr in groups.values()])
                blk: dict = dict(groups)
                blk.update({
                    "qkv_b": dev(torch.cat([g("attn1.to_v.bias"), g("attn1.to_q.bias"), g("attn1.to_k.bias")])),
                    "g1_b": dev(g("attn1.to_gate_logits.bias")),
                    "o1_b": dev(g("attn1.to_out.bias")),
                    "qn1": dev(g("attn1.q_norm.weight")),
                    "kn1": dev(g("attn1.k_norm.weight")),
                    "q2_b": dev(g("attn2.to_q.bias")),
                    "kv2_b": dev(torch.cat([g("attn2.to_k.bias"), g("attn2.to_v.bias")])),
                    "g2_b": dev(g("attn2.to_gate_logits.bias")),
                    "o2_b": dev(g("attn2.to_out.bias")),
                    "qn2": dev(g("attn2.q_norm.weight")),
                    "kn2": dev(g("attn2.k_norm.weight")),
                    "ff_in_b": dev(g("ff.project_in.proj.bias")),
                    "ff_out_b": dev(g("ff.project_out.bias")),
                })
                tables.append(g("scale_shift_table").reshape(-1))
                prompts.append(g("prompt_scale_shift_table").reshape(-1))
                self.blocks.append(blk)
                continue
            tables.append(g("scale_shift_table").reshape(-1))
            prompts.append(g("prompt_scale_shift_table").reshape(-1))
            self.blocks.append({
                # [v | q | k]: v first, so the sequence-parallel projection scatters it directly
                "qkv_w": dev(torch.cat([g("attn1.to_v.weight"), g("attn1.to_q.weight"), g("attn1.to_k.weight")])),
                "qkv_b": dev(torch.cat([g("attn1.to_v.bias"), g("attn1.to_q.bias"), g("attn1.to_k.bias")])),
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
        # one bf16 buffer for the packed linears' dequantised weights, reused by every GEMM on
        # the stream (each dequantisation waits for the previous GEMM to finish reading it)
        self._dq = (torch.empty(scratch_elems, device=self.device, dtype=BF)
                    if packed else None)

    def _wt(self, p: dict, name: str) -> torch.Tensor:
        """The bf16 (out, in) weight of a block linear: resident, or dequantised into the scratch."""
        w = p[name]
        return w.dequantize(self._dq) if isinstance(w, qz.PackedGroup) else w

    def _lin(self, x, p: dict, name: str, out, **kw):
        """A block linear; packed ones round the product to bf16 before adding the bias, as the
        reference's quantised linears do (weights/quantization.py:32-43)."""
        return ops.linear(x, self._wt(p, name), out, bias_after_round=self.quantize != "off", **kw)

    def prepare(self, context: torch.Tensor, positions: torch.Tensor,
                context_mask: torch.Tensor | None = None) -> PreparedContext:
        """The context on the device, the RoPE tables of the video tokens (this rank's shard) and
        the key bias of an optional text mask (padded prompts)."""
        cos, sin = precompute_freqs_cis(positions.cpu(), self.v)
        if self.sp.size > 1:
            t0, t1 = self.sp.shard(cos.shape[2])
            cos, sin = cos[:, :, t0:t1].contiguous(), sin[:, :, t0:t1].contiguous()
        bias = context_key_bias(context_mask, context.shape[0], context.shape[1], self.device)
        return PreparedContext(context.to(self.device, BF).contiguous(),
                               cos.to(self.device), sin.to(self.device), bias)

    def workspace(self, batch: int, tokens: int, ctx_tokens: int) -> _Workspace:
        key = (batch, tokens, ctx_tokens)
        if key not in self._ws:
            self._ws[key] = _Workspace(self.v, batch, tokens, ctx_tokens, self.device, self.sp)
        return self._ws[key]

    # ------------------------------------------------------------------ per step embeddings
    def _embed(self, ws: _Workspace, sigma: float) -> None:
        """AdaLayerNormSingle for the block modulations and the prompt AdaLN
        (kinomlx/models/ltx2/transformer/preprocessing.py:66-83, timestep.py:31-85)."""
        ws.t.fill_(float(torch.tensor(sigma, dtype=torch.float32) * self.v.timestep_scale))
        ops.timestep_embedding(ws.t, 256, out=ws.temb)
        for p, h1, emb, mod in ((self.adaln, ws.h1, ws.emb, ws.mod9),
                                (self.prompt_adaln, ws.ph1, ws.pemb, ws.pmod)):
            ops.gemv(ws.temb, p["l1w"], p["l1b"], out=h1)
            ops.gemv(h1, p["l2w"], p["l2b"], silu_input=True, out=emb)
            ops.gemv(emb, p["w"], p["b"], silu_input=True, out=mod)
        for b in range(ws.x.shape[0]):
            ops.add_rows(self.tables, ws.mod9[b], out=ws.vals[b])
            ops.add_rows(self.prompt_tables, ws.pmod[b], out=ws.prompt[b])
            ops.add_rows(self.out_table, ws.emb[b], out=ws.outmod[b].view(2, -1))

    # ------------------------------------------------------------------ block
    def _block(self, ws: _Workspace, i: int, p: dict, prepared: PreparedContext,
               sparse=None) -> None:
        v, d, h = self.v, self.v.dim, self.v.heads
        val = lambda j: ws.vals[:, i, j * d : (j + 1) * d]
        x, nrm = ws.x, ws.nrm
        vv, q, k = ws.qkv[..., :d], ws.qkv[..., d : 2 * d], ws.qkv[..., 2 * d :]
        # self-attention
        ops.adaln(x, val(0), val(1), nrm, norm=ops.NORM_RMS, eps=v.eps)
        self._lin(nrm, p, "g1_w", ws.gates, bias=p["g1_b"], kind=ops.EPI_SIGMOID2)
        if ws.peer:
            # v straight from the projection epilogue, q and k after their full-row norm and
            # RoPE, into the head owners' receive buffers; rows come back into q
            recv = self.sp.receive(x.shape[1], d)
            self._lin(nrm, p, "qkv_w", ws.qkv, bias=p["qkv_b"],
                       scatter=self.sp.scatter(recv, d, (2,), 0))
            for t, wn, slot in ((q, p["qn1"], 0), (k, p["kn1"], 1)):
                ops.qk_norm_rope(t, heads=h, weight=wn, norm=ops.QKNORM_FULL_ROW,
                                 rope=ops.ROPE_SPLIT, cos=prepared.cos, sin=prepared.sin, eps=v.eps,
                                 scatter=self.sp.scatter(recv, d, (slot,), 0))
            self.sp.attention_from_peers(recv, heads=h, out_ptrs=ws.qkv_ptrs, out_ld=3 * d,
                                         out_cols=3 * d, out_col=d,
                                         gate=(ws.gate_ptrs, ws.gates.shape[-1]))
        else:
            self._lin(nrm, p, "qkv_w", ws.qkv, bias=p["qkv_b"])
            ops.qk_norm_rope(q, heads=h, weight=p["qn1"], norm=ops.QKNORM_FULL_ROW,
                             rope=ops.ROPE_SPLIT, cos=prepared.cos, sin=prepared.sin, eps=v.eps)
            ops.qk_norm_rope(k, heads=h, weight=p["kn1"], norm=ops.QKNORM_FULL_ROW,
                             rope=ops.ROPE_SPLIT, cos=prepared.cos, sin=prepared.sin, eps=v.eps)
            if sparse is not None and sparse.applies_to(i):
                # Sol-Attn on this layer (kinomlx/models/ltx2/transformer/attention.py:210-226,
                # 344-346); the output rows land over q, with the head gate
                order = self._sparse_order(sparse, q.shape[1])
                for b in range(q.shape[0]):
                    ops.sol_attention(q[b], k[b], vv[b], heads=h, tau=sparse.tau, order=order,
                                      out=q[b], gate=ws.gates[b])
            else:
                self.sp.attention(q, k, vv, q, heads=h, gate=ws.gates)
        self._lin(q, p, "o1_w", x, bias=p["o1_b"], kind=ops.EPI_GATED_RESIDUAL,
                   residual=x, gate=val(2))
        # text cross-attention with the prompt-modulated context
        pr = lambda j: ws.prompt[:, i, j * d : (j + 1) * d]
        ops.adaln(x, val(6), val(7), nrm, norm=ops.NORM_RMS, eps=v.eps)
        ops.adaln(prepared.context, pr(0), pr(1), ws.ctxm, norm=ops.NORM_NONE)
        self._lin(nrm, p, "g2_w", ws.gates, bias=p["g2_b"], kind=ops.EPI_SIGMOID2)
        self._lin(nrm, p, "q2_w", q, bias=p["q2_b"])
        self._lin(ws.ctxm, p, "kv2_w", ws.ctxkv, bias=p["kv2_b"])
        k2, v2 = ws.ctxkv[..., :d], ws.ctxkv[..., d:]
        ops.qk_norm_rope(q, heads=h, weight=p["qn2"], norm=ops.QKNORM_FULL_ROW, rope=ops.ROPE_NONE,
                         eps=v.eps)
        ops.qk_norm_rope(k2, heads=h, weight=p["kn2"], norm=ops.QKNORM_FULL_ROW, rope=ops.ROPE_NONE,
                         eps=v.eps)
        ops.attention([q], [k2], [v2], [q], heads=h, gate=[ws.gates], key_bias=prepared.key_bias)
        self._lin(q, p, "o2_w", x, bias=p["o2_b"], kind=ops.EPI_GATED_RESIDUAL,
                   residual=x, gate=val(8))
        # feed-forward
        ops.adaln(x, val(3), val(4), nrm, norm=ops.NORM_RMS, eps=v.eps)
        self._lin(nrm, p, "ff_in_w", ws.hid, bias=p["ff_in_b"], kind=ops.EPI_GELU)
        self._lin(ws.hid, p, "ff_out_w", x, bias=p["ff_out_b"],
                   kind=ops.EPI_GATED_RESIDUAL, residual=x, gate=val(5))

    def _sparse_order(self, sparse, tokens: int) -> torch.Tensor:
        """The step's routing order on the device, converted once per order tensor."""
        cached = getattr(self, "_order_cache", None)
        if cached is None or cached[0] is not sparse.order:
            if sparse.order.numel() != tokens:
                raise ValueError("the sparse step's token order must hold one index per video token")
            self._order_cache = (sparse.order, sparse.order.to(self.device, torch.int32).contiguous())
        return self._order_cache[1]

    # ------------------------------------------------------------------ forward
    def run(self, prepared: PreparedContext, latent: torch.Tensor, sigma: float, *,
            sigma_next: float | None = None, out: torch.Tensor | None = None,
            blocks: range | None = None, sparse=None) -> torch.Tensor:
        """Velocity for `latent` (B, T, C) at `sigma`; with `sigma_next`, the next latent of the
        deterministic Euler step (X0 + Euler fused into the final projection). `sparse` (a
        SparseAttentionStep) computes the video self-attention of the layers it applies to with
        Sol-Attn; it needs the whole sequence on one GPU."""
        if sparse is not None and self.sp.size > 1:
            raise ValueError("sparse video self-attention runs with the whole sequence on one GPU")
        batch, tokens, _ = latent.shape
        ws = self.workspace(batch, tokens, prepared.context.shape[1])
        self._embed(ws, sigma)
        ops.linear(latent, self.patch_w, ws.x, bias=self.patch_b)
        for i in blocks if blocks is not None else range(self.v.blocks):
            self._block(ws, i, self.blocks[i], prepared, sparse)
        d = self.v.dim
        ops.adaln(ws.x, ws.outmod[:, :d], ws.outmod[:, d:], ws.nrm, norm=ops.NORM_LAYER,
                  eps=self.v.eps)
        if sigma_next is None:
            return ops.linear(ws.nrm, self.proj_w, ws.velocity if out is None else out,
                              bias=self.proj_b)
        ratio = float(torch.tensor(sigma_next / sigma, dtype=torch.float32))
        return ops.linear(ws.nrm, self.proj_w, out, bias=self.proj_b, kind=ops.EPI_EULER_X0,
                          sigma=float(torch.tensor(sigma, dtype=torch.float32)), ratio=ratio,
                          sample=latent)
