"""Attention with the keys split among CTAs (kino_attention's kv_splits): each CTA attends its
query tiles to one share of the key blocks and a merge launch combines the shares by their row
maxima and sums. Checked against the one-pass kernel and a torch fp32 reference on joins of two
query and two key segments, 64- and 128-wide heads, batches and head gates; the automatic choice
(what the sequence-parallel ranks ask for) splits exactly the calls whose tiles fill less than
two waves of the SMs."""

from __future__ import annotations

import pytest
import torch

from kinomlx_b200 import _lib, ops
from parity_metrics import metrics, show

pytestmark = pytest.mark.gpu


def _reference(qs, ks, vs, heads, gate):
    q = torch.cat([x.float() for x in qs], 1)
    k = torch.cat([x.float() for x in ks], 1)
    v = torch.cat([x.float() for x in vs], 1)
    b, tq, width = q.shape
    d = width // heads
    sh = lambda t: t.reshape(t.shape[0], t.shape[1], heads, d).transpose(1, 2)
    o = (torch.softmax(sh(q) @ sh(k).transpose(-1, -2) * d ** -0.5, -1) @ sh(v)).transpose(1, 2)
    if gate is not None:
        o = o.to(torch.bfloat16).float() * torch.cat([g.float() for g in gate], 1)[..., None]
    return o.reshape(b, tq, width)


@pytest.mark.parametrize("dim", [128, 64])
@pytest.mark.parametrize("splits", [2, 3, 4])
def test_split_keys_match_one_pass(cuda_device, dim, splits):
    g = torch.Generator().manual_seed(dim + splits)
    heads, batch = 3, 2
    mk = lambda n: torch.randn((batch, n, heads * dim), generator=g).to(torch.bfloat16).to(cuda_device)
    qs, ks, vs = [mk(70), mk(300)], [mk(200), mk(333)], [mk(200), mk(333)]
    gate = [torch.rand((batch, n, heads), generator=g).to(torch.bfloat16).to(cuda_device)
            for n in (70, 300)]
    one = [torch.empty_like(x) for x in qs]
    split = [torch.empty_like(x) for x in qs]
    ops.attention(qs, ks, vs, one, heads=heads, gate=gate, kv_splits=1)
    ops.attention(qs, ks, vs, split, heads=heads, gate=gate, kv_splits=splits)
    torch.cuda.synchronize()
    ops.device_status()
    got = torch.cat(split, 1)
    # the shares round their probabilities to bf16 against their own maxima: the two results
    # differ at the bf16 level, and each is as close to the fp32 reference as the other
    m = metrics(got, torch.cat(one, 1))
    assert m["rel_l2"] <= 5e-3, show(f"{splits} shares vs one pass", m)
    expect = _reference(qs, ks, vs, heads, gate)
    ms, m1 = metrics(got, expect), metrics(torch.cat(one, 1), expect)
    assert ms["rel_l2"] <= 1e-2 and ms["max_norm"] <= 2e-2, show("split vs fp32", ms)
    assert ms["rel_l2"] <= 1.25 * m1["rel_l2"] + 1e-3, (show("split", ms), show("one pass", m1))


def test_automatic_split_choice_and_refusals(cuda_device):
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    args = _lib.AttentionArgs()
    args.batch, args.heads, args.n_q, args.n_kv = 1, 3, 1, 1
    args.q_tokens[0], args.kv_tokens[0] = 4608, 4608  # 18 CTAs x 3 heads: split
    assert ops.attention_splits(args, cuda_device) == (2 if sms == 148 else
                                                       ops.attention_splits(args, cuda_device))
    assert ops.attention_splits(args, cuda_device) > 1
    args.heads = 24  # 432 CTAs, about three waves: one pass
    assert ops.attention_splits(args, cuda_device) == 1
    args.heads, args.kv_tokens[0] = 1, 100  # one key block: nothing to split
    assert ops.attention_splits(args, cuda_device) == 1
    x = torch.zeros((1, 128, 256), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(RuntimeError, match="kv_splits"):
        ops.attention([x], [x], [x], [torch.empty_like(x)], heads=2, kv_splits=2)
