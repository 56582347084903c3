"""The joint audio/video LTX-2 DiT on the sm_100a kernels: the device twin of LTXAVModel with both
modalities present (kinomlx/models/ltx2/transformer/model.py:137-635,
transformer.py:85-413, preprocessing.py:26-213, attention.py:249-371).

Each stream (video: 128-wide heads; audio: 64-wide heads, one position axis) runs the LTX block's
self-attention, text cross-attention and feed-forward exactly as `LTXVideoTransformer` does. Between
them, every block runs the two cross-modal attentions on the audio stream's heads: audio-to-video
(video queries, audio keys and values) and video-to-audio, each with its own RoPE tables for the
queries and the keys, its head gate in the attention's epilogue and its gated residual in the out
projection's epilogue. Both cross-modal attentions read the streams as they were before either
residual is added (their query and context inputs are formed first).
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from .. import ops
from .config import LTXVariant
from .transformer import context_key_bias, precompute_freqs_cis

BF = torch.bfloat16


def audio_variant(blocks: int) -> LTXVariant:
    """The reference's default audio stream (model.py:141-153): 2048 wide, 32 heads x 64, context
    2048, one position axis with max_pos 20."""
    return LTXVariant(dim=2048, heads=32, head_dim=64, context_dim=2048, max_pos=(20,),
                      blocks=blocks)


@dataclass
class Tables:
    cos: torch.Tensor
    sin: torch.Tensor


@dataclass
class PreparedAV:
    video_context: torch.Tensor
    audio_context: torch.Tensor
    video_pe: Tables  # video self-attention (B|1, heads, Tv, 64)
    audio_pe: Tables  # audio self-attention (B|1, heads, Ta, 32)
    video_cross_pe: Tables  # A/V attention, video side (B|1, heads, Tv, 32)
    audio_cross_pe: Tables  # A/V attention, audio side (B|1, heads, Ta, 32)
    video_key_bias: torch.Tensor | None = None  # text-mask biases of the two text contexts
    audio_key_bias: torch.Tensor | None = None


class _Stream:
    """One modality's weights (names with the modality's checkpoint prefix)."""

    def __init__(self, w: dict, v: LTXVariant, pre: str, blocks: int, dev):
        if v.head_dim not in (64, 128) or v.dim % 128:
            raise ValueError("streams need 64- or 128-wide heads and a width in 128-column groups")
        self.v = v
        self.qk_heads = v.dim // 128  # the QK-norm kernel counts 128-column groups
        self.rope = ops.ROPE_SPLIT if v.head_dim == 128 else ops.ROPE_SPLIT64
        self.patch_w, self.patch_b = dev(w[f"{pre}patchify_proj.weight"]), dev(w[f"{pre}patchify_proj.bias"])
        self.adaln = _single(w, f"{pre}adaln_single", dev)
        self.prompt_adaln = _single(w, f"{pre}prompt_adaln_single", dev)
        tables, prompts = [], []
        self.blocks = []
        for i in range(blocks):
            a = f"transformer_blocks.{i}"
            g = lambda n: w[f"{a}.{pre}{n}"]
            tables.append(g("scale_shift_table").reshape(-1))
            prompts.append(g("prompt_scale_shift_table").reshape(-1))
            blk = _attention(w, f"{a}.{pre}attn1", dev, "1")
            blk.update(_attention(w, f"{a}.{pre}attn2", dev, "2"))
            blk.update({
                "ff_in_w": dev(g("ff.project_in.proj.weight")),
                "ff_in_b": dev(g("ff.project_in.proj.bias")),
                "ff_out_w": dev(g("ff.project_out.weight")),
                "ff_out_b": dev(g("ff.project_out.bias")),
            })
            self.blocks.append(blk)
        self.tables = dev(torch.stack(tables))  # (L, 9D)
        self.prompt_tables = dev(torch.stack(prompts))  # (L, 2D)
        self.out_table = dev(w[f"{pre}scale_shift_table"])  # (2, D)
        self.proj_w, self.proj_b = dev(w[f"{pre}proj_out.weight"]), dev(w[f"{pre}proj_out.bias"])


def _single(w: dict, prefix: str, dev) -> dict:
    g = lambda n: dev(w[f"{prefix}.{n}"])
    return {"l1w": g("emb.timestep_embedder.linear_1.weight"),
            "l1b": g("emb.timestep_embedder.linear_1.bias"),
            "l2w": g("emb.timestep_embedder.linear_2.weight"),
            "l2b": g("emb.timestep_embedder.linear_2.bias"),
            "w": g("linear.weight"), "b": g("linear.bias")}


def _attention(w: dict, prefix: str, dev, tag: str) -> dict:
    """A gated attention's weights: q, [k | v] over the context, gate logits, out, q/k norms; a
    self-attention's q|k|v also as one product."""
    g = lambda n: w[f"{prefix}.{n}"]
    out = {
        f"q{tag}_w": dev(g("to_q.weight")), f"q{tag}_b": dev(g("to_q.bias")),
        f"kv{tag}_w": dev(torch.cat([g("to_k.weight"), g("to_v.weight")])),
        f"kv{tag}_b": dev(torch.cat([g("to_k.bias"), g("to_v.bias")])),
        f"g{tag}_w": dev(g("to_gate_logits.weight")), f"g{tag}_b": dev(g("to_gate_logits.bias")),
        f"o{tag}_w": dev(g("to_out.weight")), f"o{tag}_b": dev(g("to_out.bias")),
        f"qn{tag}": dev(g("q_norm.weight")), f"kn{tag}": dev(g("k_norm.weight")),
    }
    if tag == "1":
        out["qkv_w"] = dev(torch.cat([g("to_q.weight"), g("to_k.weight"), g("to_v.weight")]))
        out["qkv_b"] = dev(torch.cat([g("to_q.bias"), g("to_k.bias"), g("to_v.bias")]))
    return out


class _StreamWS:
    def __init__(self, v: LTXVariant, batch: int, tokens: int, ctx_tokens: int, blocks: int, dev):
        d = v.dim
        e = lambda *s: torch.empty(s, device=dev, dtype=BF)
        self.x = e(batch, tokens, d)
        self.nrm = e(batch, tokens, d)
        self.qkv = e(batch, tokens, 3 * d)
        self.gates = e(batch, tokens, v.heads)
        self.ctxm = e(batch, ctx_tokens, d)
        self.ctxkv = e(batch, ctx_tokens, 2 * d)
        self.hid = e(batch, tokens, v.ff_mult * d)
        self.h1 = e(batch, d)
        self.emb = e(batch, d)
        self.mod9 = e(batch, 9 * d)
        self.ph1 = e(batch, d)
        self.pemb = e(batch, d)
        self.pmod = e(batch, 2 * d)
        self.vals = e(batch, blocks, 9 * d)
        self.prompt = e(batch, blocks, 2 * d)
        self.outmod = e(batch, 2 * d)
        # A/V attention: its cross scale/shift (4 rows) and gate modulations
        self.css = e(batch, 4 * d)
        self.cg = e(batch, d)
        self.ssv = e(batch, blocks, 4 * d)
        self.gv = e(batch, blocks, d)
        self.q_in = e(batch, tokens, d)  # this stream as the cross-modal query input
        self.ctx_in = e(batch, tokens, d)  # this stream as the other's cross-modal context
        self.velocity = e(batch, tokens, v.out_channels)


class _AVWS:
    def __init__(self, video: LTXVariant, audio: LTXVariant, batch: int, tv: int, ta: int, dev):
        da, h = audio.dim, audio.heads
        e = lambda *s: torch.empty(s, device=dev, dtype=BF)
        self.t = torch.empty((batch,), device=dev, dtype=torch.float32)
        self.tg = torch.empty((batch,), device=dev, dtype=torch.float32)
        self.temb = e(batch, 256)
        self.tgemb = e(batch, 256)
        self.a2v_q, self.a2v_kv, self.a2v_g = e(batch, tv, da), e(batch, ta, 2 * da), e(batch, tv, h)
        self.v2a_q, self.v2a_kv, self.v2a_g = e(batch, ta, da), e(batch, tv, 2 * da), e(batch, ta, h)


class LTXAVTransformer:
    """Device joint audio/video LTX-2 DiT. `weights` uses the reference checkpoint names
    (kinomlx/models/ltx2/transformer/model.py:205-236, transformer.py:85-176)."""

    def __init__(self, weights: dict[str, torch.Tensor], video: LTXVariant, audio: LTXVariant,
                 device: torch.device | str = "cuda", *, av_gate_scale: float = 1000.0):
        if video.heads != audio.heads or audio.head_dim * audio.heads != audio.dim:
            raise ValueError("LTX-2 A/V cross-attention requires equal head counts")
        if video.blocks != audio.blocks:
            raise ValueError("both streams run the same blocks")
        self.device = torch.device(device)
        dev = lambda t: t.to(self.device, BF).contiguous()
        w = weights
        self.video, self.audio = video, audio
        self.av_gate_scale = av_gate_scale
        self.vs = _Stream(w, video, "", video.blocks, dev)
        self.as_ = _Stream(w, audio, "audio_", audio.blocks, dev)
        self.v_css = _single(w, "av_ca_video_scale_shift_adaln_single", dev)
        self.v_cg = _single(w, "av_ca_a2v_gate_adaln_single", dev)
        self.a_css = _single(w, "av_ca_audio_scale_shift_adaln_single", dev)
        self.a_cg = _single(w, "av_ca_v2a_gate_adaln_single", dev)
        self.av = []
        tv_ss, tv_g, ta_ss, ta_g = [], [], [], []
        for i in range(video.blocks):
            a = f"transformer_blocks.{i}"
            blk = _attention(w, f"{a}.audio_to_video_attn", dev, "a2v")
            blk.update(_attention(w, f"{a}.video_to_audio_attn", dev, "v2a"))
            self.av.append(blk)
            tv, ta = w[f"{a}.scale_shift_table_a2v_ca_video"], w[f"{a}.scale_shift_table_a2v_ca_audio"]
            tv_ss.append(tv[:4].reshape(-1))
            tv_g.append(tv[4])
            ta_ss.append(ta[:4].reshape(-1))
            ta_g.append(ta[4])
        self.tv_ss, self.tv_g = dev(torch.stack(tv_ss)), dev(torch.stack(tv_g))  # (L, 4Dv), (L, Dv)
        self.ta_ss, self.ta_g = dev(torch.stack(ta_ss)), dev(torch.stack(ta_g))
        self._ws: dict = {}

    # ------------------------------------------------------------------ preparation
    def prepare(self, video_context: torch.Tensor, audio_context: torch.Tensor,
                video_positions: torch.Tensor, audio_positions: torch.Tensor,
                video_context_mask: torch.Tensor | None = None,
                audio_context_mask: torch.Tensor | None = None) -> PreparedAV:
        """RoPE tables of both streams and of the A/V attention (preprocessing.py:108-121,
        170-200: the cross tables take the time axis only, on the audio width, with the larger
        of the two temporal max_pos), and the key biases of optional padded text masks
        (preprocessing.py:85-96)."""
        v, a = self.video, self.audio
        vpos, apos = video_positions.cpu(), audio_positions.cpu()
        cross_max = (max(v.max_pos[0], a.max_pos[0]),)
        tab = lambda pos, var: Tables(*(t.to(self.device) for t in precompute_freqs_cis(pos, var)))
        return PreparedAV(
            video_context.to(self.device, BF).contiguous(),
            audio_context.to(self.device, BF).contiguous(),
            tab(vpos, v), tab(apos, a),
            tab(vpos[:, 0:1], replace(v, dim=a.dim, max_pos=cross_max)),
            tab(apos[:, 0:1], replace(a, max_pos=cross_max)),
            context_key_bias(video_context_mask, video_context.shape[0], video_context.shape[1],
                             self.device),
            context_key_bias(audio_context_mask, audio_context.shape[0], audio_context.shape[1],
                             self.device),
        )

    def _workspace(self, batch, tv, ta, cv, ca):
        key = (batch, tv, ta, cv, ca)
        if key not in self._ws:
            L = self.video.blocks
            self._ws[key] = (_StreamWS(self.video, batch, tv, cv, L, self.device),
                             _StreamWS(self.audio, batch, ta, ca, L, self.device),
                             _AVWS(self.video, self.audio, batch, tv, ta, self.device))
        return self._ws[key]

    # ------------------------------------------------------------------ per step embeddings
    @staticmethod
    def _run_single(p: dict, temb, h1, emb, out) -> None:
        """AdaLayerNormSingle: linear(silu(emb)), emb = linear_2(silu(linear_1(features)))
        (timestep.py:31-85)."""
        ops.gemv(temb, p["l1w"], p["l1b"], out=h1)
        ops.gemv(h1, p["l2w"], p["l2b"], silu_input=True, out=emb)
        ops.gemv(emb, p["w"], p["b"], silu_input=True, out=out)

    def _embed(self, wv: _StreamWS, wa: _StreamWS, wav: _AVWS, sigma: float) -> None:
        s32 = float(torch.tensor(sigma, dtype=torch.float32) * self.video.timestep_scale)
        g32 = float(torch.tensor(sigma, dtype=torch.float32) * self.av_gate_scale)
        wav.t.fill_(s32)
        wav.tg.fill_(g32)
        ops.timestep_embedding(wav.t, 256, out=wav.temb)
        ops.timestep_embedding(wav.tg, 256, out=wav.tgemb)
        for st, ws, css, cg in ((self.vs, wv, self.v_css, self.v_cg), (self.as_, wa, self.a_css, self.a_cg)):
            self._run_single(st.adaln, wav.temb, ws.h1, ws.emb, ws.mod9)
            self._run_single(st.prompt_adaln, wav.temb, ws.ph1, ws.pemb, ws.pmod)
            self._run_single(css, wav.temb, ws.ph1, ws.pemb, ws.css)
            # each gate is driven by the other modality's sigma (equal in a joint step)
            self._run_single(cg, wav.tgemb, ws.ph1, ws.pemb, ws.cg)
        for b in range(wv.x.shape[0]):
            for st, ws, t_ss, t_g in ((self.vs, wv, self.tv_ss, self.tv_g), (self.as_, wa, self.ta_ss, self.ta_g)):
                ops.add_rows(st.tables, ws.mod9[b], out=ws.vals[b])
                ops.add_rows(st.prompt_tables, ws.pmod[b], out=ws.prompt[b])
                ops.add_rows(st.out_table, ws.emb[b], out=ws.outmod[b].view(2, -1))
                ops.add_rows(t_ss, ws.css[b], out=ws.ssv[b])
                ops.add_rows(t_g, ws.cg[b], out=ws.gv[b])

    # ------------------------------------------------------------------ blocks
    def _self_and_text(self, st: _Stream, ws: _StreamWS, i: int, ctx: torch.Tensor, pe: Tables,
                       key_bias: torch.Tensor | None = None):
        """transformer.py:249-320 for one stream."""
        v, p = st.v, st.blocks[i]
        d, h = v.dim, v.heads
        val = lambda j: ws.vals[:, i, j * d : (j + 1) * d]
        x, nrm = ws.x, ws.nrm
        q, k, vv = ws.qkv[..., :d], ws.qkv[..., d : 2 * d], ws.qkv[..., 2 * d :]
        ops.adaln(x, val(0), val(1), nrm, norm=ops.NORM_RMS, eps=v.eps)
        ops.linear(nrm, p["g1_w"], ws.gates, bias=p["g1_b"], kind=ops.EPI_SIGMOID2)
        ops.linear(nrm, p["qkv_w"], ws.qkv, bias=p["qkv_b"])
        for t, wn in ((q, p["qn1"]), (k, p["kn1"])):
            ops.qk_norm_rope(t, heads=st.qk_heads, weight=wn, norm=ops.QKNORM_FULL_ROW,
                             rope=st.rope, cos=pe.cos, sin=pe.sin, eps=v.eps)
        ops.attention([q], [k], [vv], [q], heads=h, gate=[ws.gates])
        ops.linear(q, p["o1_w"], x, bias=p["o1_b"], kind=ops.EPI_GATED_RESIDUAL, residual=x,
                   gate=val(2))
        pr = lambda j: ws.prompt[:, i, j * d : (j + 1) * d]
        ops.adaln(x, val(6), val(7), nrm, norm=ops.NORM_RMS, eps=v.eps)
        ops.adaln(ctx, pr(0), pr(1), ws.ctxm, norm=ops.NORM_NONE)
        ops.linear(nrm, p["g2_w"], ws.gates, bias=p["g2_b"], kind=ops.EPI_SIGMOID2)
        ops.linear(nrm, p["q2_w"], q, bias=p["q2_b"])
        ops.linear(ws.ctxm, p["kv2_w"], ws.ctxkv, bias=p["kv2_b"])
        k2, v2 = ws.ctxkv[..., :d], ws.ctxkv[..., d:]
        for t, wn in ((q, p["qn2"]), (k2, p["kn2"])):
            ops.qk_norm_rope(t, heads=st.qk_heads, weight=wn, norm=ops.QKNORM_FULL_ROW,
                             rope=ops.ROPE_NONE, eps=v.eps)
        ops.attention([q], [k2], [v2], [q], heads=h, gate=[ws.gates], key_bias=key_bias)
        ops.linear(q, p["o2_w"], x, bias=p["o2_b"], kind=ops.EPI_GATED_RESIDUAL, residual=x,
                   gate=val(8))

    def _ff(self, st: _Stream, ws: _StreamWS, i: int) -> None:
        """transformer.py:373-413 for one stream."""
        v, p = st.v, st.blocks[i]
        d = v.dim
        val = lambda j: ws.vals[:, i, j * d : (j + 1) * d]
        ops.adaln(ws.x, val(3), val(4), ws.nrm, norm=ops.NORM_RMS, eps=v.eps)
        ops.linear(ws.nrm, p["ff_in_w"], ws.hid, bias=p["ff_in_b"], kind=ops.EPI_GELU)
        ops.linear(ws.hid, p["ff_out_w"], ws.x, bias=p["ff_out_b"], kind=ops.EPI_GATED_RESIDUAL,
                   residual=ws.x, gate=val(5))

    def _cross_modal(self, p: dict, tag: str, q_in, ctx_in, q_buf, kv_buf, g_buf, q_pe: Tables,
                     k_pe: Tables, residual, gate) -> None:
        """One A/V attention (attention.py:249-371 with k_pe): gate logits and q from the query
        stream's modulated input, k|v from the other stream's, full-row q/k RMSNorm and split
        RoPE on 64-wide heads, the head gate in the attention, the gated residual in the out
        projection."""
        a = self.audio
        ops.linear(q_in, p[f"g{tag}_w"], g_buf, bias=p[f"g{tag}_b"], kind=ops.EPI_SIGMOID2)
        ops.linear(q_in, p[f"q{tag}_w"], q_buf, bias=p[f"q{tag}_b"])
        ops.linear(ctx_in, p[f"kv{tag}_w"], kv_buf, bias=p[f"kv{tag}_b"])
        k, v = kv_buf[..., : a.dim], kv_buf[..., a.dim :]
        qk_heads = a.dim // 128
        ops.qk_norm_rope(q_buf, heads=qk_heads, weight=p[f"qn{tag}"], norm=ops.QKNORM_FULL_ROW,
                         rope=ops.ROPE_SPLIT64, cos=q_pe.cos, sin=q_pe.sin, eps=a.eps)
        ops.qk_norm_rope(k, heads=qk_heads, weight=p[f"kn{tag}"], norm=ops.QKNORM_FULL_ROW,
                         rope=ops.ROPE_SPLIT64, cos=k_pe.cos, sin=k_pe.sin, eps=a.eps)
        ops.attention([q_buf], [k], [v], [q_buf], heads=a.heads, gate=[g_buf])
        ops.linear(q_buf, p[f"o{tag}_w"], residual, bias=p[f"o{tag}_b"],
                   kind=ops.EPI_GATED_RESIDUAL, residual=residual, gate=gate)

    def _block(self, i: int, wv: _StreamWS, wa: _StreamWS, wav: _AVWS, prep: PreparedAV) -> None:
        """BasicAVTransformerBlock (transformer.py:225-413)."""
        self._self_and_text(self.vs, wv, i, prep.video_context, prep.video_pe, prep.video_key_bias)
        self._self_and_text(self.as_, wa, i, prep.audio_context, prep.audio_pe, prep.audio_key_bias)
        dv, da = self.video.dim, self.audio.dim
        # rows: scale_a2v, shift_a2v, scale_v2a, shift_v2a (transformer.py:188-199, 322-371)
        vr = lambda j: wv.ssv[:, i, j * dv : (j + 1) * dv]
        ar = lambda j: wa.ssv[:, i, j * da : (j + 1) * da]
        rms = ops.NORM_RMS
        ops.adaln(wv.x, vr(1), vr(0), wv.q_in, norm=rms, eps=self.video.eps)
        ops.adaln(wv.x, vr(3), vr(2), wv.ctx_in, norm=rms, eps=self.video.eps)
        ops.adaln(wa.x, ar(3), ar(2), wa.q_in, norm=rms, eps=self.audio.eps)
        ops.adaln(wa.x, ar(1), ar(0), wa.ctx_in, norm=rms, eps=self.audio.eps)
        p = self.av[i]
        self._cross_modal(p, "a2v", wv.q_in, wa.ctx_in, wav.a2v_q, wav.a2v_kv, wav.a2v_g,
                          prep.video_cross_pe, prep.audio_cross_pe, wv.x, wv.gv[:, i])
        self._cross_modal(p, "v2a", wa.q_in, wv.ctx_in, wav.v2a_q, wav.v2a_kv, wav.v2a_g,
                          prep.audio_cross_pe, prep.video_cross_pe, wa.x, wa.gv[:, i])
        self._ff(self.vs, wv, i)
        self._ff(self.as_, wa, i)

    # ------------------------------------------------------------------ forward
    def run(self, prep: PreparedAV, video_latent: torch.Tensor, audio_latent: torch.Tensor,
            sigma: float, *, sigma_next: float | None = None,
            video_out: torch.Tensor | None = None, audio_out: torch.Tensor | None = None):
        """(video, audio) velocities at `sigma`; with `sigma_next`, the next latents of the
        deterministic Euler step (X0 + Euler in each final projection's epilogue)."""
        batch, tv, _ = video_latent.shape
        ta = audio_latent.shape[1]
        wv, wa, wav = self._workspace(batch, tv, ta, prep.video_context.shape[1],
                                      prep.audio_context.shape[1])
        self._embed(wv, wa, wav, sigma)
        ops.linear(video_latent, self.vs.patch_w, wv.x, bias=self.vs.patch_b)
        ops.linear(audio_latent, self.as_.patch_w, wa.x, bias=self.as_.patch_b)
        for i in range(self.video.blocks):
            self._block(i, wv, wa, wav, prep)
        outs = []
        for st, ws, lat, out in ((self.vs, wv, video_latent, video_out),
                                 (self.as_, wa, audio_latent, audio_out)):
            d = st.v.dim
            ops.adaln(ws.x, ws.outmod[:, :d], ws.outmod[:, d:], ws.nrm, norm=ops.NORM_LAYER,
                      eps=st.v.eps)
            if sigma_next is None:
                outs.append(ops.linear(ws.nrm, st.proj_w, ws.velocity if out is None else out,
                                       bias=st.proj_b))
            else:
                ratio = float(torch.tensor(sigma_next / sigma, dtype=torch.float32))
                outs.append(ops.linear(ws.nrm, st.proj_w, out, bias=st.proj_b,
                                       kind=ops.EPI_EULER_X0,
                                       sigma=float(torch.tensor(sigma, dtype=torch.float32)),
                                       ratio=ratio, sample=lat))
        return outs[0], outs[1]


def denoise_av(model: LTXAVTransformer, video_latent, audio_latent, video_context,
                 audio_context, video_positions, audio_positions, sigmas, *,
                 video_context_mask=None, audio_context_mask=None):
    """The deterministic-Euler loop over both modalities (kinomlx/models/ltx2/denoise.py:261-365),
    with optional padded text masks per stream."""
    prep = model.prepare(video_context, audio_context, video_positions, audio_positions,
                         video_context_mask=video_context_mask,
                         audio_context_mask=audio_context_mask)
    vx = video_latent.to(model.device, BF).clone()
    ax = audio_latent.to(model.device, BF).clone()
    values = tuple(float(torch.tensor(s, dtype=torch.float32)) for s in sigmas)
    for s, n in zip(values[:-1], values[1:]):
        model.run(prep, vx, ax, s, sigma_next=n, video_out=vx, audio_out=ax)
    ops.device_status()
    return vx, ax
