"""CPU-side checks of the boundary and the host logic: the C-ABI library loads and exports every
symbol include/kino.h declares (no compute calls), the torch front end refuses what the kernels
cannot take, and the host-side scalar math matches the oracle."""

from __future__ import annotations

import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _declared() -> list[str]:
    text = (ROOT / "include" / "kino.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:kino_status|int|int64_t|const char\*)\s+(kino_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from kinomlx_b200 import _lib

    lib = _lib.load()
    names = _declared()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.kino_abi_version() == 15
    assert _lib.last_error() == ""


def test_ops_refuse_cpu_tensors():
    from kinomlx_b200 import ops

    x = torch.zeros((4, 16), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.linear(x, x)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gelu_tanh(x)


def test_reference_surface_refusals():
    from kinomlx_b200.kernels import dense_attention, mpp_linear, split_rope

    q = torch.zeros((5, 2 * 96), dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        dense_attention.dense_attention(q, q, q, heads=2)  # heads are 64 or 128 wide
    assert not dense_attention.applies(q[None], q[None], heads=2)
    q64 = torch.zeros((1, 5, 2 * 64), dtype=torch.bfloat16)
    assert not dense_attention.applies(q64, q64, heads=2)  # the CPU tensor is what refuses here
    v = torch.zeros((2, 5, 32), dtype=torch.bfloat16)
    cos = torch.zeros((1, 2, 5, 8))
    assert not split_rope.applies(v, cos.half(), cos.half())
    with pytest.raises(ValueError, match="does not apply"):
        split_rope.rotate(v, cos.half(), cos.half())
    assert not mpp_linear.supports(10, 12, 16, transposed=True, dtype=torch.bfloat16)
    assert mpp_linear.supports(10, 16, 16, transposed=True, dtype=torch.bfloat16)


def test_host_schedule_and_timestep_match_oracle():
    from oracle import flux2 as ref
    from kinomlx_b200.flux2 import sampling

    for tokens, steps in [(1024, 4), (4096, 28), (4301, 10)]:
        assert torch.equal(sampling.schedule(tokens, steps), ref.schedule(tokens, steps))
    sig = sampling.linear_sigmas(4)
    assert torch.equal(sig, ref.linear_sigmas(4))
    for i in range(4):
        t = ref.step_timestep(sig, i, torch.bfloat16)
        assert float(sampling.timestep_x1000(sig, i)) == float((t * 1000).float())
        assert sampling.step_delta(sig, i) == float(sig[i + 1] - sig[i])


def test_rotary_tables_match_oracle():
    from oracle import flux2 as ref
    from kinomlx_b200.flux2 import config
    from kinomlx_b200.flux2.transformer import rotary_positions

    ids = torch.cat([torch.zeros((1, 7, 2), dtype=torch.int64), ref.image_ids(5, 6, 2)], 1)
    cos, sin = rotary_positions(ids, config.BASELINE)
    rc, rs = ref.rotary_positions(ids, config.BASELINE)
    assert torch.equal(cos, rc[:, :, 0]) and torch.equal(sin, rs[:, :, 0])
    ids4 = torch.randint(0, 50, (1, 9, 4))
    cos, _ = rotary_positions(ids4, config.KLEIN)
    assert torch.equal(cos, ref.rotary_positions(ids4, config.KLEIN)[0][:, :, 0])


def test_synthetic_weights_are_seeded_and_shaped():
    from kinomlx_b200.flux2 import config
    from kinomlx_b200.synthetic import flux_weight_specs, flux_weights

    v = config.BASELINE.with_blocks(1, 1)
    specs = flux_weight_specs(v)
    names = [s[0] for s in specs]
    assert len(names) == len(set(names))
    assert ("single_transformer_blocks.0.attn.to_qkv_mlp_proj.weight", (7 * 3072, 3072), "normal") in specs
    small = config.FluxVariant(dim=256, heads=2, mlp="gelu_tanh", mlp_hidden=1024, rope_axes=(64, 64),
                               rope_theta=1e4, in_channels=64, context_dim=128, double_blocks=1,
                               single_blocks=1)
    a = flux_weights(small, seed=3)
    b = flux_weights(small, seed=3)
    assert all(torch.equal(a[k], b[k]) for k in a)
    assert float(a["x_embedder.weight"].float().std()) == pytest.approx(0.02, rel=0.1)
    assert torch.equal(a["transformer_blocks.0.attn.norm_q.weight"], torch.ones(128, dtype=torch.bfloat16))


def test_f32_front_end_refuses_cpu_and_bf16():
    from kinomlx_b200 import ops_f32

    x = torch.zeros((4, 16), dtype=torch.float32)
    with pytest.raises(ValueError, match="CUDA"):
        ops_f32.linear(x, x)
    with pytest.raises(ValueError, match="CUDA"):
        ops_f32.attention(x, x, x, heads=1)
    with pytest.raises(ValueError, match="CUDA"):
        ops_f32.silu(x)


def test_fp32_timestep_matches_oracle():
    """The fp32 model's timestep goes through fp32, not bf16 (sampling.py:209-212 with the model
    dtype fp32), so it differs from the bf16 value where bf16 would round it."""
    from oracle import flux2 as ref
    from kinomlx_b200.flux2 import sampling

    sig = sampling.schedule(1024, 7)
    for i in range(7):
        t = ref.step_timestep(sig, i, torch.float32)
        assert float(sampling.timestep_x1000(sig, i, dtype=torch.float32)) == float(
            (t.to(torch.float32) * 1000).float())
    assert any(
        float(sampling.timestep_x1000(sig, i, dtype=torch.float32))
        != float(sampling.timestep_x1000(sig, i))
        for i in range(7)
    )


def test_block_entry_workspace_sizes():
    """The whole-block entries' workspace sizes (host arithmetic only, no device call)."""
    import ctypes

    from kinomlx_b200 import _lib

    lib = _lib.load()
    a = lambda n: (n + 255) // 256 * 256
    s = _lib.FluxBlockShape(1, 512, 4096, 24, 12288, _lib.MLP_GELU_TANH, 1e-6)
    rows, d = 4608, 3072
    expect = a(rows * d * 2) + max(a(rows * 3 * d * 2) + a(rows * 12288 * 2), a(rows * (3 * d + 12288) * 2))
    assert lib.kino_flux_block_workspace_size(ctypes.byref(s)) == expect
    s.mlp_hidden = 100  # not a multiple of 32
    assert lib.kino_flux_block_workspace_size(ctypes.byref(s)) == -1
    assert "invalid shape" in _lib.last_error()
    t = _lib.LTXBlockShape(1, 9216, 256, 32, 4096, 16384, 1e-6)
    d = 4096
    expect = (a(9216 * d * 2) + a(9216 * 16384 * 2) + a(9216 * 3 * d * 2) + a(9216 * 32 * 2)
              + a(256 * d * 2) + a(256 * 2 * d * 2))
    assert lib.kino_ltx_video_block_workspace_size(ctypes.byref(t)) == expect


def test_attention_key_split_policy():
    """The wave model of ops.attention_splits on a 148-SM B200: calls that fill the SMs once stay
    whole (config 4's per-rank 4 heads x 9216 at 8 GPUs), calls over few tiles split (config 2's
    per-rank 12 heads at 2 GPUs and 3 heads at 8 GPUs), never beyond the key blocks."""
    from types import SimpleNamespace

    from kinomlx_b200 import ops

    ops._SM_COUNTS[0] = 148
    dev = torch.device("cuda", 0)

    def splits(tokens, heads, keys=None, batch=1):
        args = SimpleNamespace(q_tokens=[tokens], n_q=1, heads=heads, batch=batch,
                               kv_tokens=[keys or tokens], n_kv=1)
        return ops.attention_splits(args, dev)

    assert splits(4608, 24) == 1 and splits(9216, 32) == 1
    assert splits(9216, 4) == 1 and splits(9216, 8) == 1 and splits(9216, 16) == 1
    assert splits(4608, 12) == 2 and splits(4608, 3) == 2
    assert splits(128, 1, keys=256) <= 2  # at most one share per key block
    assert splits(256, 1, keys=128) == 1
