"""Parity metrics shared by the device-against-oracle tests.

`rel_l2`      ||o - e|| / ||e||
`max_norm`    max |o - e| / max |e|  (the per-op gate of the older tests)
`elem_max`    max over elements of |o - e| / |e|, on the elements with |e| >= 0.1 rms(e): a bf16
              value carries 2^-9 relative rounding, and below a tenth of the tensor's rms the
              relative error of a value is set by absolute rounding of the terms that cancelled
              into it, not by the op
`elem_p999`   the 99.9th percentile of the same elementwise relative error
`cos`         cosine similarity
"""

from __future__ import annotations

import torch


def metrics(out: torch.Tensor, expect: torch.Tensor) -> dict[str, float]:
    o = out.detach().float().cpu().flatten().double()
    e = expect.detach().float().cpu().flatten().double()
    diff = (o - e).abs()
    rms = float(e.pow(2).mean().sqrt())
    mask = e.abs() >= 0.1 * rms
    rel = diff[mask] / e.abs()[mask]
    return {
        "rel_l2": float((o - e).norm() / e.norm()),
        "max_norm": float(diff.max() / e.abs().max()),
        "elem_max": float(rel.max()) if rel.numel() else 0.0,
        "elem_p999": float(torch.quantile(rel.float()[: 1 << 24], 0.999)) if rel.numel() else 0.0,
        "cos": float(torch.nn.functional.cosine_similarity(o, e, dim=0)),
    }


def update_metrics(out: torch.Tensor, expect: torch.Tensor, before: torch.Tensor) -> dict[str, float]:
    """The same metrics on the updates (out - before) and (expect - before)."""
    b = before.detach().double().cpu()
    return metrics(out.detach().double().cpu() - b, expect.detach().double().cpu() - b)


def show(name: str, m: dict[str, float]) -> str:
    return name + ": " + ", ".join(f"{k} {v:.3e}" for k, v in m.items())
