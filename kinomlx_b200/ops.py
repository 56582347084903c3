"""Torch-tensor front end of the C ABI: device memory and streams come from PyTorch, every
computation is one kino_* launch on the current CUDA stream. No CPU fallback exists; a tensor on
the wrong device or of the wrong dtype is a ValueError, a refusal by the library a RuntimeError.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import (
    EPI_EULER,
    EPI_GATED_RESIDUAL,
    EPI_GELU,
    EPI_NONE,
    EPI_EULER_X0,
    EPI_SIGMOID2,
    EPI_SWIGLU,
    NORM_LAYER,
    NORM_NONE,
    NORM_RMS,
    QKNORM_FULL_ROW,
    QKNORM_NONE,
    QKNORM_PER_HEAD,
    ROPE_NONE,
    ROPE_PAIRS,
    ROPE_SPLIT,
    ROPE_SPLIT64,
)

__all__ = [
    "EPI_EULER",
    "EPI_GATED_RESIDUAL",
    "EPI_GELU",
    "EPI_NONE",
    "EPI_EULER_X0",
    "EPI_SIGMOID2",
    "EPI_SWIGLU",
    "NORM_LAYER",
    "NORM_NONE",
    "NORM_RMS",
    "QKNORM_FULL_ROW",
    "QKNORM_NONE",
    "QKNORM_PER_HEAD",
    "ROPE_NONE",
    "ROPE_PAIRS",
    "ROPE_SPLIT",
    "ROPE_SPLIT64",
    "adaln",
    "add_rows",
    "attention",
    "blend_normalize",
    "cfg_combine",
    "conv3d",
    "copy_view",
    "device_status",
    "euler_denoised",
    "euler_velocity",
    "euler_velocity_step",
    "euler_x0",
    "gelu_tanh",
    "gemv",
    "group_norm",
    "latent_to_bfhwc",
    "linear",
    "na_qkv_prepare",
    "neighborhood_attention",
    "pixel_norm",
    "RopeTables",
    "qk_norm_rope",
    "rms_norm",
    "silu",
    "sol_attention",
    "split_rope",
    "tile_blend",
    "timestep_embedding",
]


class LaunchLog:
    """Optional record of every kino_* launch: CUDA events on the launching stream around each
    call, with the launch's algorithmic FLOPs and bytes. Used by the benchmark to time the
    dominant kernel inside its timed region; off (None) by default."""

    def __init__(self) -> None:
        self.records: list[tuple[str, torch.cuda.Event, torch.cuda.Event, float, float]] = []

    def summary(self) -> dict[str, dict[str, float]]:
        """Per kernel class: launches, total ms, FLOPs and bytes (after a synchronize)."""
        out: dict[str, dict[str, float]] = {}
        for label, start, end, flops, nbytes in self.records:
            entry = out.setdefault(label, {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
            entry["launches"] += 1
            entry["ms"] += start.elapsed_time(end)
            entry["flops"] += flops
            entry["bytes"] += nbytes
        return out


_log: LaunchLog | None = None
launches = 0  # kino_* launches issued by this process


def set_launch_log(log: LaunchLog | None) -> None:
    global _log
    _log = log


class _timed:
    def __init__(self, label: str, flops: float = 0.0, nbytes: float = 0.0):
        self.label, self.flops, self.nbytes = label, flops, nbytes

    def __enter__(self):
        global launches
        launches += 1
        if _log is not None:
            self.start = torch.cuda.Event(enable_timing=True)
            self.end = torch.cuda.Event(enable_timing=True)
            self.start.record()
        return self

    def __exit__(self, *exc):
        if _log is not None and exc[0] is None:
            self.end.record()
            _log.records.append((self.label, self.start, self.end, self.flops, self.nbytes))
        return False


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t: torch.Tensor, name: str, dtype: torch.dtype = torch.bfloat16) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the kinomlx_b200 kernels have no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if t.numel() and t.stride(-1) != 1:
        raise ValueError(f"{name} needs a unit stride in its last dimension")


def _as3d(t: torch.Tensor) -> torch.Tensor:
    return t if t.dim() == 3 else t.unsqueeze(0)


def device_status() -> None:
    """Synchronise the current stream and raise if any kernel wait timed out."""
    _lib.call("kino_device_status", _stream())


class RopeTables:
    """Pair-RoPE tables for the fused QK-norm epilogue of `linear`, stored head-dim-major.

    Built once per generation from (1|B, N, 128) fp32 cos/sin tables: the device copy is
    (128, T) with T = (B if batched else 1) * N, so batch b row i sits in column b * N + i and
    the 32 rows a warp's epilogue holds read one contiguous span per head-dim column."""

    def __init__(self, cos: torch.Tensor, sin: torch.Tensor):
        if cos.shape != sin.shape or cos.shape[-1] != 128:
            raise ValueError("RoPE tables are (..., tokens, 128) cos/sin pairs")
        c3, s3 = cos.reshape(-1, cos.shape[-2], 128), sin.reshape(-1, sin.shape[-2], 128)
        self.rows = c3.shape[1]
        self.batched = c3.shape[0] > 1
        self.cos_t = c3.to(torch.float32).permute(2, 0, 1).reshape(128, -1).contiguous()
        self.sin_t = s3.to(torch.float32).permute(2, 0, 1).reshape(128, -1).contiguous()


class Scatter:
    """Sequence-parallel scatter of a projection's first `segments * seg_width` output columns
    into the receive buffers of the GPUs that own their heads (see kino_epilogue in kino.h).

    ptrs: int64 device tensor of `world` receive-buffer addresses (bf16, `rows` rows of `ld`);
    segment s (q, k or v, in the projection's column order) lands in slot `slots[s]` of a
    receive row; output row i goes to receive row `row0 + i`."""

    def __init__(self, ptrs: torch.Tensor, world: int, seg_width: int, segments: int, ld: int,
                 rows: int, row0: int, slots: tuple[int, ...]):
        self.ptrs, self.world, self.seg_width, self.segments = ptrs, world, seg_width, segments
        self.ld, self.rows, self.row0, self.slots = ld, rows, row0, tuple(slots)


class PeerReturn:
    """Where a sequence-parallel attention sends its rows back (see kino_attention_args): query
    row t goes to rank t // rows_per_rank, row t % rows_per_rank of out_ptrs[rank] (row stride
    ld, `cols` columns), at column col_offset + head * 128; with gate_ptrs, its gate is read from
    the owner's gate rows (stride ld_gate) at column gate_head_offset + head."""

    def __init__(self, out_ptrs: torch.Tensor, world: int, rows_per_rank: int, ld: int,
                 cols: int, col_offset: int, gate_ptrs: torch.Tensor | None = None,
                 ld_gate: int = 0, gate_head_offset: int = 0):
        self.out_ptrs, self.world, self.rows_per_rank = out_ptrs, world, rows_per_rank
        self.ld, self.cols, self.col_offset = ld, cols, col_offset
        self.gate_ptrs, self.ld_gate, self.gate_head_offset = gate_ptrs, ld_gate, gate_head_offset


def linear(
    x: torch.Tensor,
    w: torch.Tensor,
    out: torch.Tensor | None = None,
    *,
    bias: torch.Tensor | None = None,
    kind: int = EPI_NONE,
    residual: torch.Tensor | None = None,
    gate: torch.Tensor | None = None,
    act_col_begin: int = 0,
    dt: float = 0.0,
    sample: torch.Tensor | None = None,
    sigma: float = 0.0,
    ratio: float = 0.0,
    qk_norm: list[tuple[int, torch.Tensor]] | None = None,
    norm_width: int = 0,
    rope: tuple[RopeTables, int] | None = None,
    eps: float = 1e-6,
    scatter: Scatter | None = None,
    lead_w: torch.Tensor | None = None,
    lead_rows: int = 0,
    lead_qk_norm: list[torch.Tensor] | None = None,
    lead_gate: torch.Tensor | None = None,
    bias_after_round: bool = False,
) -> torch.Tensor:
    """out = epilogue(x @ w.T) for x (batch, m, k) or (m, k) and an (n, k) weight.

    With `lead_w` (lead_rows a multiple of 256 below m), rows [0, lead_rows) of every batch
    entry use that weight and `lead_qk_norm` / `lead_gate` in place of the qk_norm weights and
    the gate: the text and image streams of a joint sequence in one launch.

    EPI_SWIGLU: columns from `act_col_begin` on come in blocks of 16 gate + 16 content rows
    (see `swiglu_interleave`) and produce half as many output columns.

    EPI_EULER uses `dt` and `sample`; EPI_EULER_X0 uses `sigma`, `ratio` (fp32 sigma_next /
    sigma) and `sample`."""
    _need(x, "x")
    _need(w, "w")
    x3 = _as3d(x)
    batch, m, k = x3.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"weight {tuple(w.shape)} does not match input width {k}")
    n_out = act_col_begin + (n - act_col_begin) // 2 if kind == EPI_SWIGLU else n
    if out is None:
        out = torch.empty((*x.shape[:-1], n_out), device=x.device, dtype=torch.bfloat16)
    _need(out, "out")
    o3 = _as3d(out)
    if tuple(o3.shape) != (batch, m, n_out):
        raise ValueError(f"out {tuple(out.shape)} does not match ({batch}, {m}, {n_out})")
    epi = _lib.Epilogue()
    epi.kind = kind
    if bias is not None:
        _need(bias, "bias")
        epi.bias = bias.data_ptr()
    if kind == EPI_GATED_RESIDUAL:
        if residual is None or gate is None:
            raise ValueError("a gated residual needs residual and gate")
        _need(residual, "residual")
        _need(gate, "gate")
        r3 = _as3d(residual)
        epi.residual = r3.data_ptr()
        epi.ld_residual = r3.stride(1)
        epi.bs_residual = r3.stride(0)
        g = gate.reshape(-1, gate.shape[-1]) if gate.dim() != 2 else gate
        epi.gate = g.data_ptr()
        epi.bs_gate = g.stride(0) if g.shape[0] > 1 else 0
    if kind in (EPI_GELU, EPI_SWIGLU):
        epi.act_col_begin = act_col_begin
    if kind in (EPI_EULER, EPI_EULER_X0):
        if sample is None:
            raise ValueError("the Euler epilogue needs the current sample")
        _need(sample, "sample")
        s3 = _as3d(sample)
        epi.aux = s3.data_ptr()
        epi.ld_aux = s3.stride(1)
        epi.bs_aux = s3.stride(0)
        epi.scalar = dt if kind == EPI_EULER else sigma
        epi.scalar2 = ratio
    if qk_norm:
        # fused per-head RMSNorm + adjacent-pair RoPE on (column, weight) ranges of norm_width
        if rope is None or len(qk_norm) > 2:
            raise ValueError("qk_norm takes up to two (column, weight) ranges and rope tables")
        tables, offset = rope
        if tables.batched and tables.cos_t.shape[1] != batch * tables.rows:
            raise ValueError("batched RoPE tables must hold one table per batch entry")
        _need(tables.cos_t, "cos", torch.float32)
        _need(tables.sin_t, "sin", torch.float32)
        for r, (col, weight) in enumerate(qk_norm):
            _need(weight, "norm weight")
            epi.norm_weight[r] = weight.data_ptr()
            epi.norm_col[r] = col
        epi.norm_width = norm_width
        epi.rope_cos, epi.rope_sin = tables.cos_t.data_ptr(), tables.sin_t.data_ptr()
        epi.rope_rows = tables.rows
        epi.rope_offset = offset
        epi.rope_batched = int(tables.batched)
        epi.norm_eps = eps
    if lead_w is not None:
        _need(lead_w, "lead_w")
        if tuple(lead_w.shape) != tuple(w.shape) or lead_w.stride(1) != 1:
            raise ValueError("the lead weight must match the weight's shape")
        epi.w_lead = lead_w.data_ptr()
        epi.ldw_lead = lead_w.stride(0)
        epi.lead_rows = lead_rows
        for r, wt in enumerate(lead_qk_norm or []):
            _need(wt, "lead norm weight")
            epi.norm_weight_lead[r] = wt.data_ptr()
        if lead_gate is not None:
            _need(lead_gate, "lead gate")
            epi.gate_lead = lead_gate.data_ptr()
    epi.bias_after_round = int(bias_after_round)
    if scatter is not None:
        epi.scatter_ptrs = scatter.ptrs.data_ptr()
        epi.world = scatter.world
        epi.scatter_cols = scatter.segments * scatter.seg_width
        epi.seg_width = scatter.seg_width
        epi.part_width = scatter.seg_width // scatter.world
        epi.scatter_ld = scatter.ld
        epi.scatter_row0 = scatter.row0
        epi.scatter_rows = scatter.rows
        for i, slot in enumerate(scatter.slots):
            epi.seg_slot[i] = slot
    with _timed("gemm", 2.0 * batch * m * n * k, 2.0 * (batch * m * k + n * k + batch * m * n)):
        _lib.call(
            "kino_linear",
            _ptr(x3),
            _ptr(w),
            _ptr(o3),
            batch,
            m,
            n,
            k,
            x3.stride(1),
            x3.stride(0),
            w.stride(0),
            o3.stride(1),
            o3.stride(0),
            ctypes.byref(epi),
            _stream(),
        )
    return out


def swiglu_interleave(w: torch.Tensor) -> torch.Tensor:
    """Rows [gate (H); content (H)] of a SwiGLU up projection -> blocks of 16 gate rows followed
    by the 16 matching content rows, the order the EPI_SWIGLU epilogue reads."""
    h = w.shape[0] // 2
    if h % 16:
        raise ValueError("SwiGLU width must be a multiple of 16")
    gate = w[:h].reshape(h // 16, 16, *w.shape[1:])
    content = w[h:].reshape(h // 16, 16, *w.shape[1:])
    return torch.cat([gate, content], dim=1).reshape(w.shape)


def gemv(
    x: torch.Tensor,
    w: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    silu_input: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """y = act(x) @ w.T + bias for a handful of rows (x: (batch, k), batch <= 4)."""
    _need(x, "x")
    _need(w, "w")
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    batch, k = x2.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty((batch, n), device=x.device, dtype=torch.bfloat16)
    with _timed("gemv", 2.0 * batch * n * k, 2.0 * n * k):
        _lib.call(
            "kino_gemv",
            _ptr(x2),
            x2.stride(0),
            _ptr(w),
            _ptr(bias),
            _ptr(out),
            out.stride(0),
            batch,
            n,
            k,
            1 if silu_input else 0,
            _stream(),
        )
    return out


_SPLIT_WORKSPACES: dict[torch.device, torch.Tensor] = {}
_SM_COUNTS: dict[int, int] = {}


def _split_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A byte buffer of at least `nbytes` on `device`, grown as needed and reused by every split
    attention on the stream."""
    ws = _SPLIT_WORKSPACES.get(device)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _SPLIT_WORKSPACES[device] = ws
    return ws


# Wave model of the key split, in units of one 128-key block of a CTA: a CTA costs its blocks
# plus a fixed set-up and epilogue; a split call adds the merge of the shares.
_SPLIT_CTA_OVERHEAD = 4
_SPLIT_MERGE_COST = 3


def attention_splits(args, device: torch.device) -> int:
    """Key shares for an attention call (1 to 4, at most one per key block): the count whose
    waves of CTAs (two 128-query tiles each, `kv_splits` per tile pair) finish first, counting
    each wave as its CTAs' blocks plus a fixed per-CTA cost and a split call's merge. Attention
    over few query tiles (sequence-parallel ranks, small batches) otherwise leaves SMs idle,
    while a call that already fills the SMs once (config 4's 4 heads x 9216 tokens per rank at 8
    GPUs: 144 CTAs on 148 SMs) only pays for splitting."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index not in _SM_COUNTS:
        _SM_COUNTS[index] = torch.cuda.get_device_properties(index).multi_processor_count
    sms = _SM_COUNTS[index]
    tiles = sum((int(args.q_tokens[i]) + 127) // 128 for i in range(args.n_q))
    ctas = (tiles + 1) // 2 * int(args.heads) * int(args.batch)
    blocks = sum((int(args.kv_tokens[i]) + 127) // 128 for i in range(args.n_kv))
    best, best_cost = 1, None
    for splits in range(1, max(1, min(4, blocks)) + 1):
        waves = -(-ctas * splits // sms)
        cost = waves * (-(-blocks // splits) + _SPLIT_CTA_OVERHEAD)
        if splits > 1:
            cost += _SPLIT_MERGE_COST
        if best_cost is None or cost < best_cost:
            best, best_cost = splits, cost
    return best


def attention(
    q: list[torch.Tensor],
    k: list[torch.Tensor],
    v: list[torch.Tensor],
    out: list[torch.Tensor],
    *,
    heads: int,
    scale: float | None = None,
    gate: list[torch.Tensor | None] | None = None,
    peer_return: PeerReturn | None = None,
    key_bias: torch.Tensor | None = None,
    kv_splits: int | str = 1,
) -> list[torch.Tensor]:
    """Attention over logically concatenated segments; each tensor (batch, tokens, heads*128).
    `gate[s]` (batch, tokens, heads), if given, multiplies segment s's output per head. With
    `peer_return`, output rows go to their owner GPUs instead of `out`. `key_bias` (fp32,
    (batch, >= keys rounded up to 4), unit column stride; one key segment) is added to the
    scaled scores of every query row: an additive attention mask over the keys. `kv_splits`
    shares the keys among that many CTAs per tile pair (merged by row statistics); "auto" splits
    the calls whose tile pairs fill less than two waves of the SMs (`attention_splits`), which
    the sequence-parallel ranks use."""
    if not 1 <= len(q) <= 2 or len(out) != len(q) or not 1 <= len(k) <= 2 or len(v) != len(k):
        raise ValueError("attention takes 1 or 2 query and key/value segments")
    args = _lib.AttentionArgs()
    q0 = _as3d(q[0])
    args.batch = q0.shape[0]
    args.heads = heads
    args.head_dim = q0.shape[-1] // heads
    if args.head_dim * heads != q0.shape[-1]:
        raise ValueError("query width is not heads * head_dim")
    args.scale = scale if scale is not None else args.head_dim**-0.5
    args.n_q = len(q)
    for s, (qs, os_) in enumerate(zip(q, out)):
        _need(qs, "q")
        _need(os_, "out")
        q3, o3 = _as3d(qs), _as3d(os_)
        args.q[s] = q3.data_ptr()
        args.out[s] = o3.data_ptr()
        args.q_tokens[s] = q3.shape[1]
        args.ld_q[s] = q3.stride(1)
        args.bs_q[s] = q3.stride(0)
        args.ld_out[s] = o3.stride(1)
        args.bs_out[s] = o3.stride(0)
        g = gate[s] if gate is not None else None
        if g is not None:
            _need(g, "gate")
            g3 = _as3d(g)
            if tuple(g3.shape) != (q3.shape[0], q3.shape[1], heads):
                raise ValueError("attention gate must be (batch, tokens, heads)")
            args.gate[s] = g3.data_ptr()
            args.ld_gate[s] = g3.stride(1)
            args.bs_gate[s] = g3.stride(0)
    args.n_kv = len(k)
    for s, (ks, vs) in enumerate(zip(k, v)):
        _need(ks, "k")
        _need(vs, "v")
        k3, v3 = _as3d(ks), _as3d(vs)
        args.k[s] = k3.data_ptr()
        args.v[s] = v3.data_ptr()
        args.kv_tokens[s] = k3.shape[1]
        args.ld_k[s] = k3.stride(1)
        args.bs_k[s] = k3.stride(0)
        args.ld_v[s] = v3.stride(1)
        args.bs_v[s] = v3.stride(0)
    if key_bias is not None:
        tk = int(args.kv_tokens[0])
        if len(k) != 1 or peer_return is not None:
            raise ValueError("a key bias takes one key segment and no peer return")
        if (key_bias.dtype != torch.float32 or key_bias.dim() != 2 or key_bias.device != q0.device
                or key_bias.shape[0] != args.batch or key_bias.shape[1] < (tk + 3) // 4 * 4
                or key_bias.stride(1) != 1):
            raise ValueError("key_bias must be fp32 (batch, keys rounded up to 4) with unit "
                             "column stride, on the queries' device")
        args.key_bias = key_bias.data_ptr()
        args.ld_key_bias = key_bias.stride(0)
    if peer_return is not None:
        r = peer_return
        args.out_peers = r.out_ptrs.data_ptr()
        args.world = r.world
        args.rows_per_rank = r.rows_per_rank
        args.out_col_offset = r.col_offset
        args.out_cols = r.cols
        args.ld_out[0] = r.ld
        if r.gate_ptrs is not None:
            args.gate_peers = r.gate_ptrs.data_ptr()
            args.ld_gate[0] = r.ld_gate
            args.gate_head_offset = r.gate_head_offset
    splits = attention_splits(args, q0.device) if kv_splits == "auto" else int(kv_splits)
    if key_bias is not None:
        splits = 1
    if splits > 1:
        need = int(_lib.load().kino_attention_workspace_size(ctypes.byref(args), splits))
        ws = _split_workspace(q0.device, need)
        args.kv_splits = splits
        args.workspace = ws.data_ptr()
        args.workspace_bytes = ws.numel()
    nq = sum(int(args.q_tokens[i]) for i in range(args.n_q))
    nk = sum(int(args.kv_tokens[i]) for i in range(args.n_kv))
    flops = 4.0 * args.batch * heads * nq * nk * args.head_dim
    with _timed("attention", flops, 2.0 * args.batch * heads * args.head_dim * (2 * nq + 2 * nk)):
        _lib.call("kino_attention", ctypes.byref(args), _stream())
    return out


def neighborhood_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                           window: tuple[int, int, int],
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """Exact 3-D neighborhood attention: q, k, v contiguous (batch, T, H, W, heads, 64) fp16 on
    the GPU, the queries already scaled; each query attends to the window's keys around it, the
    window shifted inward at the grid's edges. Any odd window no larger than the grid. `out`
    fp16 (default) or bf16."""
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        _need(t, name, torch.float16)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if q.dim() != 6 or q.shape[-1] != 64 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("neighborhood attention takes matching (batch, T, H, W, heads, 64) operands")
    if len(window) != 3:
        raise ValueError("the window has three sizes (frames, height, width)")
    if out is None:
        out = torch.empty_like(q)
    if out.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("out is fp16 or bf16")
    _need(out, "out", out.dtype)
    if out.shape != q.shape or not out.is_contiguous():
        raise ValueError("out must be contiguous and shaped like q")
    b, gt, gh, gw, heads, dim = q.shape
    win = (ctypes.c_int32 * 3)(*(int(x) for x in window))
    keys = 1
    for x in window:
        keys *= int(x)
    with _timed("neighborhood_attention", 4.0 * b * gt * gh * gw * heads * keys * dim,
                4.0 * q.numel() * 2):
        _lib.call("kino_neighborhood_attention_ex", _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                  _COPY_TYPES[out.dtype], b, gt, gh, gw, heads, ctypes.cast(win, ctypes.c_void_p),
                  _stream())
    return out


def na_qkv_prepare(qkv: torch.Tensor, q_norm_weight: torch.Tensor, k_norm_weight: torch.Tensor,
                   rope_tables: torch.Tensor, grid: tuple[int, int, int], *, batch: int,
                   heads: int, section_pairs: tuple[int, int, int], q_scale: float,
                   eps: float = 1e-6,
                   out: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None,
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """qkv (tokens, >= 3 * heads * 64) bf16 rows [q | k | v] of a (batch, T, H, W) volume ->
    fp16 (batch, T, H, W, heads, 64) q, k, v for `neighborhood_attention`: per-head RMSNorm of
    q and k with their learned weights, q times `q_scale`, the decoder's 3-D RoPE on adjacent
    pairs ([t | h | w] sections of `section_pairs` pairs, from `rope_tables`)."""
    _need(qkv, "qkv")
    _need(q_norm_weight, "q_norm_weight")
    _need(k_norm_weight, "k_norm_weight")
    _need(rope_tables, "rope_tables", torch.float32)
    if qkv.dim() != 2 or qkv.stride(1) != 1:
        raise ValueError("qkv must be (tokens, width) rows with unit column stride")
    gt, gh, gw = (int(x) for x in grid)
    tokens = batch * gt * gh * gw
    if qkv.shape[0] != tokens or qkv.shape[1] < 3 * heads * 64:
        raise ValueError(f"qkv {tuple(qkv.shape)} does not hold {tokens} rows of 3 x {heads} heads")
    shape = (batch, gt, gh, gw, heads, 64)
    if out is None:
        out = tuple(torch.empty(shape, device=qkv.device, dtype=torch.float16) for _ in range(3))
    for t, name in zip(out, "qkv"):
        _need(t, name, torch.float16)
        if tuple(t.shape) != shape or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous {shape}")
    sec = (ctypes.c_int32 * 3)(*(int(x) for x in section_pairs))
    with _timed("na_qkv_prepare", 0.0, tokens * heads * 64 * (6.0 + 6.0)):
        _lib.call("kino_na_qkv_prepare", _ptr(qkv), qkv.stride(0), _ptr(out[0]), _ptr(out[1]),
                  _ptr(out[2]), _ptr(q_norm_weight), _ptr(k_norm_weight), _ptr(rope_tables),
                  batch, gt, gh, gw, heads, ctypes.cast(sec, ctypes.c_void_p), q_scale, eps,
                  _stream())
    return out


_COPY_TYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def _copy_dims(shape, src_strides, dst_strides) -> list[list[int]]:
    """[size, source stride, destination stride] per dimension of a copy, outermost first, with
    size-1 dimensions dropped and neighbours that are contiguous on both sides merged (so most
    layout moves stay within the kernel's 8 dimensions)."""
    merged: list[list[int]] = []
    for n, a, b in zip(shape, src_strides, dst_strides):
        n, a, b = int(n), int(a), int(b)
        if n == 1:
            continue
        if merged and merged[-1][1] == a * n and merged[-1][2] == b * n:
            merged[-1] = [merged[-1][0] * n, a, b]
        else:
            merged.append([n, a, b])
    return merged or [[1, 0, 0]]


def copy_view(src: torch.Tensor, dst: torch.Tensor) -> torch.Tensor:
    """dst[...] = src[...] for two same-shaped device views of any strides (a zero source stride
    broadcasts) and dtypes bf16 / fp16 / fp32, in one `kino_strided_copy` launch: permutations,
    slices, broadcasts and dtype changes without a torch kernel. Returns dst."""
    if src.shape != dst.shape:
        raise ValueError(f"copy_view shapes differ: {tuple(src.shape)} vs {tuple(dst.shape)}")
    if src.dtype not in _COPY_TYPES or dst.dtype not in _COPY_TYPES:
        raise ValueError("copy_view takes bf16, fp16 or fp32 tensors")
    if src.device != dst.device or src.device.type != "cuda":
        raise ValueError("copy_view runs on one CUDA device")
    merged = _copy_dims(src.shape, src.stride(), dst.stride())
    if len(merged) > 8:
        raise ValueError(f"copy_view supports up to 8 non-mergeable dimensions, got {len(merged)}")
    nd = len(merged)
    sizes = (ctypes.c_int64 * nd)(*(m[0] for m in merged))
    sst = (ctypes.c_int64 * nd)(*(m[1] for m in merged))
    dstr = (ctypes.c_int64 * nd)(*(m[2] for m in merged))
    elems = 1
    for m in merged:
        elems *= m[0]
    with _timed("copy", 0.0, elems * (src.element_size() + dst.element_size())):
        _lib.call("kino_strided_copy", _ptr(src), _COPY_TYPES[src.dtype],
                  ctypes.cast(sst, ctypes.c_void_p), _ptr(dst), _COPY_TYPES[dst.dtype],
                  ctypes.cast(dstr, ctypes.c_void_p), ctypes.cast(sizes, ctypes.c_void_p), nd,
                  _stream())
    return dst


_SOL_WORKSPACES: dict[tuple, torch.Tensor] = {}


def sol_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    heads: int,
    tau: float,
    order: torch.Tensor,
    out: torch.Tensor | None = None,
    gate: torch.Tensor | None = None,
    routes: torch.Tensor | None = None,
) -> torch.Tensor:
    """Sol-Attn of (tokens, heads * 128) q, k, v (bf16 or fp16, any row stride) routed in
    `order` (a device int32 permutation); the output rows come back in input order, in the
    input dtype, optionally times a (tokens, heads) gate. `routes` (int32 (heads, blocks,
    words)) receives the routing mask words."""
    dtype = q.dtype
    if dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("Sol attention needs float16 or bfloat16 q, k and v")
    for name, t in (("q", q), ("k", k), ("v", v)):
        _need(t, name, dtype)
    tokens = q.shape[0]
    if out is None:
        out = torch.empty((tokens, heads * 128), device=q.device, dtype=dtype)
    _need(out, "out", dtype)
    if order.dtype != torch.int32 or not order.is_cuda or order.numel() != tokens:
        raise ValueError("the routing order must be a device int32 tensor of one index per token")
    lib = _lib.load()
    need = int(lib.kino_sol_attention_workspace_size(tokens, heads))
    key = (q.device, tokens, heads)
    ws = _SOL_WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = _SOL_WORKSPACES[key] = torch.empty(need, device=q.device, dtype=torch.uint8)
    args = _lib.SolAttentionArgs()
    args.q, args.k, args.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    args.ld_q, args.ld_k, args.ld_v = q.stride(0), k.stride(0), v.stride(0)
    args.out, args.ld_out = out.data_ptr(), out.stride(0)
    if gate is not None:
        _need(gate, "gate", dtype)
        args.gate, args.ld_gate = gate.data_ptr(), gate.stride(0)
    args.tokens, args.heads = tokens, heads
    args.dtype = _lib.DTYPE_F16 if dtype == torch.float16 else _lib.DTYPE_BF16
    args.tau = tau
    args.order = order.data_ptr()
    if routes is not None:
        _need(routes, "routes", torch.int32)
        args.routes = routes.data_ptr()
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    with _timed("sol_attention", 0.0, 0.0):
        _lib.call("kino_sol_attention", ctypes.byref(args), _stream())
    return out


def adaln(
    x: torch.Tensor,
    shift: torch.Tensor,
    scale: torch.Tensor,
    out: torch.Tensor | None = None,
    *,
    norm: int = NORM_LAYER,
    eps: float = 1e-6,
) -> torch.Tensor:
    """norm(x) * (1 + scale) + shift; x (batch, rows, dim), shift/scale (batch, dim)."""
    _need(x, "x")
    _need(shift, "shift")
    _need(scale, "scale")
    x3 = _as3d(x)
    batch, rows, dim = x3.shape
    if out is None:
        out = torch.empty(x.shape, device=x.device, dtype=torch.bfloat16)
    o3 = _as3d(out)
    sh = shift.reshape(-1, dim)
    sc = scale.reshape(-1, dim)
    if sh.stride(0) != sc.stride(0):
        raise ValueError("shift and scale need the same batch stride")
    with _timed("adaln", 0.0, 2.0 * 2 * batch * rows * dim):
        _lib.call(
            "kino_adaln",
            _ptr(x3),
            x3.stride(1),
            x3.stride(0),
            _ptr(sh),
            _ptr(sc),
            sh.stride(0) if sh.shape[0] > 1 else 0,
            _ptr(o3),
            o3.stride(1),
            o3.stride(0),
            batch,
            rows,
            dim,
            norm,
            eps,
            _stream(),
        )
    return out


def add_rows(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out = a + b with b (n,) broadcast over the rows of a (..., n), bf16."""
    _need(a, "a")
    _need(b, "b")
    if not a.is_contiguous() or b.numel() != a.shape[-1]:
        raise ValueError("add_rows needs a contiguous (..., n) tensor and an (n,) row")
    b = b.contiguous()
    if out is None:
        out = torch.empty_like(a)
    n = a.shape[-1]
    with _timed("elementwise", 0.0, 6.0 * a.numel()):
        _lib.call("kino_add_rows", _ptr(a), _ptr(b), _ptr(out), a.numel() // n, n, _stream())
    return out


def rms_norm(
    x: torch.Tensor,
    weight: torch.Tensor | None = None,
    eps: float = 1e-6,
    *,
    weight_offset: float = 0.0,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    _need(x, "x")
    if not x.is_contiguous():
        raise ValueError("rms_norm needs a contiguous input")
    if out is None:
        out = torch.empty_like(x)
    dim = x.shape[-1]
    with _timed("rms_norm", 0.0, 4.0 * x.numel()):
        _lib.call(
            "kino_rms_norm",
            _ptr(x),
            _ptr(weight),
            _ptr(out),
            x.numel() // dim,
            dim,
            eps,
            weight_offset,
            _stream(),
        )
    return out


def qk_norm_rope(
    x: torch.Tensor,
    *,
    heads: int,
    weight: torch.Tensor | None,
    norm: int,
    rope: int,
    cos: torch.Tensor | None = None,
    sin: torch.Tensor | None = None,
    table_offset: int = 0,
    eps: float = 1e-6,
    scatter: Scatter | None = None,
) -> torch.Tensor:
    """In place: RMSNorm (per head or full row) then RoPE on x (batch, tokens, heads*128).
    `heads` counts 128-column groups; ROPE_SPLIT64 rotates 64-wide heads (two per group) from
    (1|batch, 2 * heads, tokens, 32) tables. With `scatter` (batch 1, one segment), the result
    goes to the head owners' receive buffers (slot scatter.slots[0]) instead."""
    _need(x, "x")
    x3 = _as3d(x)
    batch, tokens, width = x3.shape
    if width != heads * 128:
        raise ValueError("qk_norm_rope works on 128-wide heads")
    table_tokens = 0
    table_batched = 0
    if rope != ROPE_NONE:
        if cos is None or sin is None:
            raise ValueError("RoPE needs cos and sin tables")
        _need(cos, "cos", torch.float32)
        _need(sin, "sin", torch.float32)
        if not (cos.is_contiguous() and sin.is_contiguous()):
            raise ValueError("RoPE tables must be contiguous")
        table_tokens = cos.shape[-2]
        table_batched = int(cos.shape[0] > 1 and cos.dim() >= 3)
    if scatter is not None:
        if batch != 1:
            raise ValueError("the scattered form takes batch 1")
        with _timed("qk_norm_rope", 0.0, 4.0 * tokens * width + 2 * 4.0 * tokens * 128):
            _lib.call("kino_qk_norm_rope_to_peers", _ptr(x3), x3.stride(1), tokens, heads,
                      _ptr(weight), norm, rope, _ptr(cos), _ptr(sin), table_batched, table_tokens,
                      table_offset, eps, _ptr(scatter.ptrs), scatter.world, scatter.ld,
                      scatter.row0, scatter.rows, scatter.slots[0], _stream())
        return x
    with _timed("qk_norm_rope", 0.0, 4.0 * batch * tokens * width + 2 * 4.0 * tokens * 128):
        _lib.call(
            "kino_qk_norm_rope",
            _ptr(x3),
            x3.stride(1),
            x3.stride(0),
            batch,
            tokens,
            heads,
            _ptr(weight),
            norm,
            rope,
            _ptr(cos),
            _ptr(sin),
            table_batched,
            table_tokens,
            table_offset,
            eps,
            _stream(),
        )
    return x


def split_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """value (batch, tokens, heads*2*half), tables (1|batch, heads, tokens, half) fp32."""
    _need(x, "x")
    _need(cos, "cos", torch.float32)
    _need(sin, "sin", torch.float32)
    table_batch, heads, tokens, half = cos.shape
    batch = x.shape[0]
    # keep the contiguous copies alive until the launch is queued
    x, cos, sin = x.contiguous(), cos.contiguous(), sin.contiguous()
    out = torch.empty_like(x)
    with _timed("split_rope", 0.0, 4.0 * x.numel() + 8.0 * cos.numel()):
        _lib.call(
            "kino_split_rope",
            _ptr(x),
            _ptr(cos),
            _ptr(sin),
            _ptr(out),
            batch,
            tokens,
            heads,
            half,
            int(table_batch == batch and batch > 1),
            _stream(),
        )
    return out


def _elementwise(name: str, *args: object) -> None:
    with _timed("elementwise"):
        _lib.call(name, *args, _stream())


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    _need(x, "x")
    x = x.contiguous()
    out = torch.empty_like(x)
    _elementwise("kino_gelu_tanh", _ptr(x), _ptr(out), x.numel())
    return out


def silu(x: torch.Tensor) -> torch.Tensor:
    _need(x, "x")
    x = x.contiguous()
    out = torch.empty_like(x)
    _elementwise("kino_silu", _ptr(x), _ptr(out), x.numel())
    return out


def cfg_combine(cond: torch.Tensor, uncond: torch.Tensor, guidance: float) -> torch.Tensor:
    _need(cond, "cond")
    _need(uncond, "uncond")
    cond, uncond = cond.contiguous(), uncond.contiguous()
    out = torch.empty_like(cond)
    _elementwise("kino_cfg_combine", _ptr(cond), _ptr(uncond), guidance, _ptr(out), cond.numel())
    return out


def euler_velocity(
    x: torch.Tensor, v: torch.Tensor, dt: float, out: torch.Tensor | None = None
) -> torch.Tensor:
    _need(x, "x")
    _need(v, "v")
    if out is None:
        out = torch.empty_like(x)
    _elementwise("kino_euler_velocity", _ptr(x), _ptr(v), dt, _ptr(out), x.numel())
    return out


def euler_x0(
    x: torch.Tensor, v: torch.Tensor, sigma: float, sigma_next: float
) -> torch.Tensor:
    _need(x, "x")
    _need(v, "v")
    out = torch.empty_like(x)
    ratio = float(torch.tensor(sigma_next / sigma, dtype=torch.float32))
    _elementwise("kino_euler_x0", _ptr(x), _ptr(v), sigma, ratio, _ptr(out), x.numel())
    return out


def euler_denoised(
    x: torch.Tensor, denoised: torch.Tensor, sigma: float, sigma_next: float,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """denoised + fp32(sigma_next / sigma) * (x - denoised) in fp32, stored as bf16."""
    _need(x, "x")
    _need(denoised, "denoised")
    if out is None:
        out = torch.empty_like(x)
    ratio = float(torch.tensor(sigma_next / sigma, dtype=torch.float32))
    _elementwise("kino_euler_step", _ptr(x), _ptr(denoised), ratio, _ptr(out), x.numel())
    return out


def euler_velocity_step(
    x: torch.Tensor, v: torch.Tensor, sigma: float, sigma_next: float,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """x + bf16(fp32(sigma_next - sigma) * v), stored as bf16."""
    _need(x, "x")
    _need(v, "v")
    if out is None:
        out = torch.empty_like(x)
    delta = float(torch.tensor(sigma_next - sigma, dtype=torch.float32))
    _elementwise("kino_euler_velocity_step", _ptr(x), _ptr(v), delta, _ptr(out), x.numel())
    return out


def timestep_embedding(
    t: torch.Tensor, dim: int = 256, *, out: torch.Tensor | None = None
) -> torch.Tensor:
    """t: fp32 (batch,) on the device -> bf16 (batch, dim) [cos, sin] features."""
    _need(t, "t", torch.float32)
    t = t.contiguous()
    if out is None:
        out = torch.empty((t.shape[0], dim), device=t.device, dtype=torch.bfloat16)
    _elementwise("kino_timestep_embedding", _ptr(t), _ptr(out), t.shape[0], dim)
    return out


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


# ----------------------------------------------------------------------------- video VAE
def conv3d(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    causal: bool,
    stride: tuple[int, int, int] = (1, 1, 1),
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    stats: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """3x3x3 conv of channels-last x (F, H, W, Cin) with an (N, 3, 3, 3, Cin) weight; with a
    depth-to-space `stride` the weight rows must be sub-position-major (n = sub * C' + c).
    `stats` (a conv_stats_buffer()) receives the GroupNorm(32) statistics of the output for
    group_norm_from_stats. `workspace` (a conv_workspace()) lets a conv whose output tiles fill
    less than half of the GPU split its reduction over several CTAs."""
    _need(x, "x")
    _need(weight, "weight")
    if not x.is_contiguous() or not weight.is_contiguous():
        raise ValueError("conv3d needs contiguous channels-last input and OTHWI weight")
    x4 = x[0] if x.dim() == 5 else x
    f, h, w, cin = x4.shape
    n = weight.shape[0]
    if tuple(weight.shape[1:]) != (3, 3, 3, cin):
        raise ValueError(f"weight {tuple(weight.shape)} does not match {cin} input channels")
    st, sh, sw = stride
    sub = st * sh * sw
    oshape = (f * st - (1 if st > 1 else 0), h * sh, w * sw, n // sub)
    if out is None:
        out = torch.empty(oshape, device=x.device, dtype=torch.bfloat16)
    if residual is not None:
        _need(residual, "residual")
    args = _lib.Conv3dArgs()
    args.x = x4.data_ptr()
    args.frames, args.height, args.width, args.in_channels = f, h, w, cin
    args.weight = weight.data_ptr()
    args.out_channels = n
    args.bias = bias.data_ptr() if bias is not None else None
    args.residual = residual.data_ptr() if residual is not None else None
    args.out = out.data_ptr()
    args.causal = 1 if causal else 0
    args.stride_t, args.stride_h, args.stride_w = st, sh, sw
    if stats is not None:
        _need(stats, "stats", torch.float32)
        args.stats = stats.data_ptr()
        args.stats_records = (stats.numel() - 128) // 96
    if workspace is not None:
        _need(workspace, "workspace", torch.uint8)
        args.workspace = workspace.data_ptr()
        args.workspace_bytes = workspace.numel()
    with _timed("conv3d", 2.0 * f * h * w * n * 27 * cin, 2.0 * (x4.numel() + weight.numel() + out.numel())):
        _lib.call("kino_conv3d", ctypes.byref(args), _stream())
    return out


def pixel_norm(x: torch.Tensor, eps: float = 1e-8, *, silu: bool = False,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Stepwise PixelNorm over the last (channel) axis, optionally followed by SiLU."""
    _need(x, "x")
    if not x.is_contiguous():
        raise ValueError("pixel_norm needs a contiguous channels-last input")
    if out is None:
        out = torch.empty_like(x)
    c = x.shape[-1]
    with _timed("norm", 0.0, 4.0 * x.numel()):
        _lib.call("kino_pixel_norm", _ptr(x), _ptr(out), x.numel() // c, c, eps, int(silu), _stream())
    return out


def group_norm(x: torch.Tensor, groups: int, weight: torch.Tensor, bias: torch.Tensor,
               eps: float, *, silu: bool = False, out: torch.Tensor | None = None,
               workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Affine GroupNorm(32) over channels-last x with fp32 two-pass statistics (+ SiLU). The
    reduction's partial sums go to `workspace` (caller memory; allocated here if not given)."""
    if groups != 32:
        raise ValueError("the GroupNorm kernel takes 32 groups")
    _need(x, "x")
    if not x.is_contiguous():
        raise ValueError("group_norm needs a contiguous channels-last input")
    c = x.shape[-1]
    voxels = x.numel() // c
    need = int(_lib.load().kino_group_norm_workspace_size(voxels, c))
    if workspace is None:
        workspace = torch.empty(need, device=x.device, dtype=torch.uint8)
    if out is None:
        out = torch.empty_like(x)
    with _timed("norm", 0.0, 8.0 * x.numel()):
        _lib.call("kino_group_norm", _ptr(x), _ptr(weight), _ptr(bias), _ptr(out), voxels, c, eps,
                  int(silu), _ptr(workspace), workspace.numel() * workspace.element_size(), _stream())
    return out


QUANT_MODES = {"affine": 0, "mxfp8": 1, "mxfp4": 2, "nvfp4": 3}


def dequantize(
    words: torch.Tensor,
    scales: torch.Tensor,
    biases: torch.Tensor | None,
    *,
    mode: str,
    group_size: int,
    bits: int,
    transpose_out: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """bf16 weight from packed codes `words` ((rows, cols * bits / 32) 32-bit words), per-group
    `scales` (bf16 for affine, uint8 E8M0 / E4M3 codes otherwise) and affine `biases`; (rows, cols),
    or (cols, rows) with `transpose_out`."""
    if mode not in QUANT_MODES:
        raise ValueError(f"unknown quantisation mode {mode!r}")
    if words.dtype not in (torch.int32, torch.uint32) or not words.is_cuda or not words.is_contiguous():
        raise ValueError("words must be a contiguous CUDA int32/uint32 tensor")
    rows = words.shape[0]
    cols = words.shape[1] * 32 // bits
    if mode == "affine":
        _need(scales, "scales")
        if biases is None:
            raise ValueError("affine mode needs biases")
        _need(biases, "biases")
    else:
        _need(scales, "scales", torch.uint8)
    if tuple(scales.shape) != (rows, cols // group_size):
        raise ValueError(f"scales {tuple(scales.shape)} do not match {rows} x {cols} in groups of {group_size}")
    shape = (cols, rows) if transpose_out else (rows, cols)
    if out is None:
        out = torch.empty(shape, device=words.device, dtype=torch.bfloat16)
    elif tuple(out.shape) != shape:
        raise ValueError(f"out must be {shape}")
    with _timed("dequant", 0.0, words.numel() * 4 + out.numel() * 2):
        _lib.call("kino_dequantize", _ptr(words), _ptr(scales), _ptr(biases), _ptr(out), rows, cols,
                  QUANT_MODES[mode], group_size, bits, int(transpose_out), _stream())
    return out


def quantized_linear(
    x: torch.Tensor,
    words: torch.Tensor,
    scales: torch.Tensor,
    biases: torch.Tensor | None,
    *,
    mode: str,
    group_size: int,
    bits: int,
    transpose: bool,
    bias: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    scratch: torch.Tensor | None = None,
    **epilogue,
) -> torch.Tensor:
    """MLX quantized_matmul semantics on the tcgen05 GEMM: `transpose` -> x @ W^T with W packed as
    (out, in) along `in`; otherwise x @ W with W packed from weight.T as (in, out) along `out`.
    The weight is dequantised into `scratch` (a bf16 buffer of at least out x in elements, reused
    by every call on the stream) and multiplied with fp32 accumulation; the product is rounded to
    bf16 before the bias is added, as the reference's quantised linear does; `epilogue` keywords
    go to `linear` (kind, residual, gate, ...)."""
    rows = words.shape[0]
    cols = words.shape[1] * 32 // bits
    n, k = (rows, cols) if transpose else (cols, rows)
    if scratch is None:
        w = torch.empty((n, k), device=words.device, dtype=torch.bfloat16)
    else:
        if scratch.dtype != torch.bfloat16 or scratch.numel() < n * k:
            raise ValueError("scratch must be a bf16 buffer of at least out x in elements")
        w = scratch.view(-1)[: n * k].view(n, k)
    dequantize(words, scales, biases, mode=mode, group_size=group_size, bits=bits,
               transpose_out=not transpose, out=w)
    epilogue.setdefault("bias_after_round", True)
    return linear(x, w, out, bias=bias, **epilogue)


def conv_workspace(device: torch.device | None = None) -> torch.Tensor:
    """A zero-filled split-K workspace for conv3d(workspace=...) on the current device (every
    launch leaves it ready for the next; one per stream of convs)."""
    nbytes = int(_lib.load().kino_conv3d_workspace_size())
    return torch.zeros((nbytes,), device=device or torch.device("cuda"), dtype=torch.uint8)


def conv_stats_buffer(device: torch.device | None = None) -> torch.Tensor:
    """A GroupNorm statistics buffer for conv3d(stats=...) on the current device."""
    nbytes = int(_lib.load().kino_conv3d_stats_size())
    return torch.zeros((nbytes // 4,), device=device or torch.device("cuda"), dtype=torch.float32)


def group_norm_from_stats(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float,
                          stats: torch.Tensor, *, silu: bool = False,
                          out: torch.Tensor | None = None) -> torch.Tensor:
    """Affine GroupNorm(32) (+ SiLU) of x, the output of the conv3d that filled `stats`."""
    _need(x, "x")
    c = x.shape[-1]
    if out is None:
        out = torch.empty_like(x)
    with _timed("norm", 0.0, 4.0 * x.numel()):
        _lib.call("kino_group_norm_from_stats", _ptr(x), _ptr(weight), _ptr(bias), _ptr(out),
                  x.numel() // c, c, eps, int(silu), _ptr(stats), _stream())
    return out


def latent_to_bfhwc(latent: torch.Tensor, std: torch.Tensor, mean: torch.Tensor) -> torch.Tensor:
    """(1, C, F, H, W) bf16 latent -> (F, H, W, C) bf16 of latent * std + mean (fp32 math)."""
    _need(latent, "latent")
    if latent.dim() != 5 or latent.shape[0] != 1 or not latent.is_contiguous():
        raise ValueError("latent must be a contiguous (1, C, F, H, W) tensor")
    _, c, f, h, w = latent.shape
    std, mean = std.float().contiguous(), mean.float().contiguous()
    out = torch.empty((f, h, w, c), device=latent.device, dtype=torch.bfloat16)
    with _timed("elementwise", 0.0, 4.0 * latent.numel()):
        _lib.call("kino_latent_to_bfhwc", _ptr(latent), _ptr(std), _ptr(mean), _ptr(out), c,
                  f * h * w, _stream())
    return out


def tile_blend(decoded: torch.Tensor, canvas: torch.Tensor, weights: torch.Tensor, y0: int, x0: int,
               mask_h: torch.Tensor, mask_w: torch.Tensor, patch: int = 4) -> None:
    """Accumulate a decoded tile (F, h, w, C * patch^2) into the fp32 (1, C, F, H, W) canvas."""
    _need(decoded, "decoded")
    f, h, w, packed = decoded.shape
    c = packed // (patch * patch)
    mask_h, mask_w = mask_h.float().contiguous(), mask_w.float().contiguous()
    with _timed("elementwise", 0.0, 2.0 * decoded.numel() + 8.0 * decoded.numel()):
        _lib.call("kino_tile_blend", _ptr(decoded), f, h, w, c, patch, _ptr(canvas), _ptr(weights),
                  canvas.shape[-2], canvas.shape[-1], y0, x0, _ptr(mask_h), _ptr(mask_w), _stream())


def blend_normalize(canvas: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    hw = canvas.shape[-2] * canvas.shape[-1]
    with _timed("elementwise", 0.0, 8.0 * canvas.numel()):
        _lib.call("kino_blend_normalize", _ptr(canvas), _ptr(weights), canvas.numel() // hw, hw,
                  _stream())
    return canvas


# ----------------------------------------------------------------------------- sequence parallel
def heads_pack(src: torch.Tensor, parts: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """(tokens, width) rows (any row stride) -> (parts, tokens, width / parts) head groups."""
    _need(src, "src")
    tokens, width = src.shape[-2], src.shape[-1]
    if out is None:
        out = torch.empty((parts, tokens, width // parts), device=src.device, dtype=torch.bfloat16)
    with _timed("pack", 0.0, 4.0 * tokens * width):
        _lib.call("kino_heads_pack", _ptr(src), src.stride(-2), _ptr(out), tokens, width, parts,
                  _stream())
    return out


def heads_unpack(src: torch.Tensor, out: torch.Tensor, gate: torch.Tensor | None = None) -> torch.Tensor:
    """(parts, tokens, width / parts) -> (tokens, width) rows of `out` (any row stride), times the
    per-(token, head) gate if given."""
    _need(src, "src")
    _need(out, "out")
    parts, tokens, chunk = src.shape
    width = parts * chunk
    with _timed("pack", 0.0, 4.0 * tokens * width):
        _lib.call("kino_heads_unpack", _ptr(src), _ptr(out), out.stride(-2), tokens, width, parts,
                  _ptr(gate), gate.stride(-2) if gate is not None else 0, _stream())
    return out


# ----------------------------------------------------------------------------- peer memory
def peer_alloc(nbytes: int) -> tuple[int, bytes]:
    """cudaMalloc'd, zero-filled bytes on the current device and their IPC handle."""
    ptr = ctypes.c_void_p()
    handle = _lib.IpcHandle()
    _lib.call("kino_peer_alloc", nbytes, ctypes.byref(ptr), ctypes.byref(handle))
    return int(ptr.value), bytes(handle.bytes)


def peer_free(ptr: int) -> None:
    _lib.call("kino_peer_free", ctypes.c_void_p(ptr))


def peer_open(handle: bytes) -> int:
    """Map another process's peer_alloc buffer (same node) into this process."""
    h = _lib.IpcHandle()
    ctypes.memmove(h.bytes, handle, 64)
    ptr = ctypes.c_void_p()
    _lib.call("kino_peer_open", ctypes.byref(h), ctypes.byref(ptr))
    return int(ptr.value)


def peer_close(ptr: int) -> None:
    _lib.call("kino_peer_close", ctypes.c_void_p(ptr))


def peer_barrier(flag_ptrs: torch.Tensor, rank: int, world: int, epoch: int) -> None:
    """Cross-GPU arrival barrier number `epoch` on the current stream (kino_peer_barrier)."""
    with _timed("barrier", 0.0, 0.0):
        _lib.call("kino_peer_barrier", _ptr(flag_ptrs), rank, world, epoch, _stream())
