"""The whole-block C entries (kino_flux_double_block, kino_flux_single_block,
kino_ltx_video_block) called through ctypes with caller-owned weights, modulations, tables and
workspace: bit-identical to the model classes' launch sequences, and the config-1 double block
against the CPU oracle at BASELINE's shape (512 text + 1024 image tokens, hidden 3072)."""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import flux2 as ref
from kinomlx_b200 import _lib, ops
from kinomlx_b200.flux2 import config as fcfg
from kinomlx_b200.flux2.transformer import Flux2Transformer, rotary_positions
from kinomlx_b200.ltx2 import config as lcfg
from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
from kinomlx_b200.synthetic import flux_weights, ltx_weights, normal
from oracle import ltx2 as lref
from parity_metrics import metrics, show

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _flux_shape(v: fcfg.FluxVariant, batch: int, nt: int, ni: int) -> _lib.FluxBlockShape:
    s = _lib.FluxBlockShape()
    s.batch, s.text_tokens, s.image_tokens = batch, nt, ni
    s.heads, s.mlp_hidden = v.heads, v.mlp_hidden
    s.mlp = _lib.MLP_SWIGLU if v.mlp == "swiglu" else _lib.MLP_GELU_TANH
    s.eps = 1e-6
    return s


def _rope(tables: ops.RopeTables) -> _lib.RopeTablesArgs:
    r = _lib.RopeTablesArgs()
    r.cos, r.sin = tables.cos_t.data_ptr(), tables.sin_t.data_ptr()
    r.rows, r.batched = tables.rows, int(tables.batched)
    return r


def _workspace(nbytes: int, device) -> torch.Tensor:
    assert nbytes > 0, _lib.last_error()
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _flux_case(cuda_device, v, nt, h, wd, seed, batch=1):
    w = flux_weights(v, seed=seed)
    model = Flux2Transformer(w, v, cuda_device)
    image = normal((batch, h * wd, v.dim), seed=seed + 1)
    text = normal((batch, nt, v.dim), seed=seed + 2)
    ids = torch.cat([torch.zeros((1, nt, len(v.rope_axes)), dtype=torch.int64),
                     ref.image_ids(h, wd, len(v.rope_axes))], 1)
    cos, sin = rotary_positions(ids, v)
    return w, model, image, text, ids, cos.to(cuda_device), sin.to(cuda_device)


FLUX_CASES = {
    # BASELINE config 1 (joint launch: 512 text rows are lead rows), GELU
    "config1": (fcfg.BASELINE.with_blocks(1, 1), 512, 32, 32, 1),
    # Klein-shaped SwiGLU with 40 text rows (split launches), batch 2
    "swiglu_split": (fcfg.FluxVariant(dim=1024, heads=8, mlp="swiglu", mlp_hidden=3072,
                                      rope_axes=(32, 32, 32, 32), rope_theta=2000.0,
                                      in_channels=128, context_dim=512, double_blocks=1,
                                      single_blocks=1), 40, 8, 12, 2),
}


@pytest.mark.parametrize("case", sorted(FLUX_CASES))
def test_flux_block_entries_match_model_launches(cuda_device, case):
    v, nt, h, wd, batch = FLUX_CASES[case]
    w, model, image, text, ids, cos, sin = _flux_case(cuda_device, v, nt, h, wd, 60, batch)
    t = torch.tensor([500.0, 250.0][:batch], device=cuda_device)
    lib = _lib.load()
    exp_img, exp_txt = model.double_block(0, image.to(cuda_device), text.to(cuda_device), t, cos, sin)
    value = torch.cat([text, image], 1).to(cuda_device)
    exp_single = model.single_block(0, value, nt, t, cos, sin)
    ws = model.workspace(batch, nt, h * wd)
    model._embed(ws, t)  # the modulations both paths read
    d = v.dim
    shape = _flux_shape(v, batch, nt, h * wd)
    work = _workspace(int(lib.kino_flux_block_workspace_size(ctypes.byref(shape))), cuda_device)
    tables = ops.RopeTables(cos, sin)
    rope = _rope(tables)

    p = model.double[0]
    dw = _lib.FluxDoubleWeights(*(p[k].data_ptr() for k in (
        "img_qkv", "txt_qkv", "to_out", "to_add_out", "norm_q", "norm_k", "norm_added_q",
        "norm_added_k", "ff_in", "ff_out", "ffc_in", "ffc_out")))
    hidden = value.clone()
    status = lib.kino_flux_double_block(ctypes.byref(shape), ctypes.byref(dw), hidden.data_ptr(),
                                        ws.mods.data_ptr(), ws.mods.stride(0), ctypes.byref(rope),
                                        work.data_ptr(), work.numel(), _stream())
    assert status == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.equal(hidden[:, nt:], exp_img) and torch.equal(hidden[:, :nt], exp_txt)

    p = model.single[0]
    sw = _lib.FluxSingleWeights(*(p[k].data_ptr() for k in ("fused", "to_out", "norm_q", "norm_k")))
    hidden = value.clone()
    status = lib.kino_flux_single_block(ctypes.byref(shape), ctypes.byref(sw), hidden.data_ptr(),
                                        ws.mods[:, 12 * d :].data_ptr(), ws.mods.stride(0),
                                        ctypes.byref(rope), work.data_ptr(), work.numel(), _stream())
    assert status == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.equal(hidden, exp_single)
    # a workspace one byte short is refused before any launch
    status = lib.kino_flux_single_block(ctypes.byref(shape), ctypes.byref(sw), hidden.data_ptr(),
                                        ws.mods.data_ptr(), ws.mods.stride(0), ctypes.byref(rope),
                                        work.data_ptr(), work.numel() - 1, _stream())
    assert status == _lib.KINO_EINVAL and "workspace" in _lib.last_error()


def test_flux_double_block_entry_config1_against_oracle(cuda_device):
    """BASELINE config 1 through the C entry alone: modulations from the oracle's timestep MLP
    (t = 0.5), copied to the device, the double block through kino_flux_double_block."""
    v = fcfg.BASELINE.with_blocks(1, 0)
    w = flux_weights(v, seed=0)
    image, text = normal((1, 1024, v.dim), seed=1), normal((1, 512, v.dim), seed=2)
    ids = torch.cat([torch.zeros((1, 512, 2), dtype=torch.int64), ref.image_ids(32, 32, 2)], 1)
    t = torch.tensor([0.5], dtype=BF)
    cos4, sin4 = ref.rotary_positions(ids, v)
    emb = ref.timestep_embedding(w, t * 1000)
    im = ref.modulation(w, "double_stream_modulation_img", emb)
    tm = ref.modulation(w, "double_stream_modulation_txt", emb)
    exp_img, exp_txt = ref.double_block(w, 0, image, text, im, tm, cos4, sin4, v)

    model = Flux2Transformer(w, v, cuda_device)  # only for its load-time weight layout
    lib = _lib.load()
    cos, sin = rotary_positions(ids, v)
    tables = ops.RopeTables(cos.to(cuda_device), sin.to(cuda_device))
    rope = _rope(tables)
    shape = _flux_shape(v, 1, 512, 1024)
    work = _workspace(int(lib.kino_flux_block_workspace_size(ctypes.byref(shape))), cuda_device)
    p = model.double[0]
    dw = _lib.FluxDoubleWeights(*(p[k].data_ptr() for k in (
        "img_qkv", "txt_qkv", "to_out", "to_add_out", "norm_q", "norm_k", "norm_added_q",
        "norm_added_k", "ff_in", "ff_out", "ffc_in", "ffc_out")))
    mods = torch.cat([im, tm], -1).to(cuda_device).contiguous()
    hidden = torch.cat([text, image], 1).to(cuda_device)
    status = lib.kino_flux_double_block(ctypes.byref(shape), ctypes.byref(dw), hidden.data_ptr(),
                                        mods.data_ptr(), 0, ctypes.byref(rope), work.data_ptr(),
                                        work.numel(), _stream())
    assert status == 0, _lib.last_error()
    torch.cuda.synchronize()
    for name, out, exp, before in (("image", hidden[:, 512:], exp_img, image),
                                   ("text", hidden[:, :512], exp_txt, text)):
        m = metrics(out, exp)
        assert m["rel_l2"] <= 1e-2 and m["max_norm"] <= 2e-2 and m["cos"] >= 0.999, show(name, m)


def test_ltx_video_block_entry_matches_model_launches(cuda_device):
    v = lcfg.BASELINE_VIDEO.with_blocks(1)
    w = ltx_weights(v, seed=70)
    grid = (2, 4, 8)
    tokens = grid[0] * grid[1] * grid[2]
    pos = lref.pixel_coords(lref.patch_grid_bounds(*grid))
    context = normal((1, 64, v.context_dim), seed=71).to(cuda_device)
    x0 = normal((1, tokens, v.dim), seed=72).to(cuda_device)
    model = LTXVideoTransformer(w, v, cuda_device)
    prep = model.prepare(context, pos)
    ws = model.workspace(1, tokens, 64)
    model._embed(ws, 0.725)
    ws.x.copy_(x0)
    model._block(ws, 0, model.blocks[0], prep)
    expect = ws.x.clone()

    lib = _lib.load()
    shape = _lib.LTXBlockShape(1, tokens, 64, v.heads, v.context_dim, v.ff_mult * v.dim, 1e-6)
    work = _workspace(int(lib.kino_ltx_video_block_workspace_size(ctypes.byref(shape))), cuda_device)
    p = model.blocks[0]
    bw = _lib.LTXVideoBlockWeights(*(p[k].data_ptr() for k in (
        "qkv_w", "qkv_b", "g1_w", "g1_b", "o1_w", "o1_b", "qn1", "kn1", "q2_w", "q2_b", "kv2_w",
        "kv2_b", "g2_w", "g2_b", "o2_w", "o2_b", "qn2", "kn2", "ff_in_w", "ff_in_b", "ff_out_w",
        "ff_out_b")))
    hidden = x0.clone()
    batched = int(prep.cos.shape[0] > 1)
    status = lib.kino_ltx_video_block(ctypes.byref(shape), ctypes.byref(bw), hidden.data_ptr(),
                                      prep.context.data_ptr(), ws.vals[:, 0].data_ptr(),
                                      ws.vals.stride(0), ws.prompt[:, 0].data_ptr(),
                                      ws.prompt.stride(0), prep.cos.data_ptr(), prep.sin.data_ptr(),
                                      batched, work.data_ptr(), work.numel(), _stream())
    assert status == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.equal(hidden, expect), show("ltx block entry", metrics(hidden, expect))
