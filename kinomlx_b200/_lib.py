"""ctypes binding of libkino_b200.so (the C ABI in include/kino.h).

The library is loaded from this package directory. There is no fallback: if it is missing or a
call returns a non-OK status, a RuntimeError names the reason from kino_last_error().
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int64, c_void_p
from pathlib import Path

LIBRARY_PATH = Path(__file__).with_name("libkino_b200.so")

KINO_OK = 0
KINO_EINVAL = 1
KINO_ENOTSUPPORTED = 2
KINO_ECUDA = 3
KINO_ETIMEOUT = 4

STATUS_NAMES = {
    KINO_OK: "KINO_OK",
    KINO_EINVAL: "KINO_EINVAL",
    KINO_ENOTSUPPORTED: "KINO_ENOTSUPPORTED",
    KINO_ECUDA: "KINO_ECUDA",
    KINO_ETIMEOUT: "KINO_ETIMEOUT",
}

EPI_NONE = 0
EPI_GELU = 1
EPI_GATED_RESIDUAL = 2
EPI_EULER = 3
EPI_SIGMOID2 = 4
EPI_EULER_X0 = 5
EPI_SWIGLU = 6

NORM_RMS = 0
NORM_LAYER = 1
NORM_NONE = 2

QKNORM_NONE = 0
QKNORM_PER_HEAD = 1
QKNORM_FULL_ROW = 2
ROPE_NONE = 0
ROPE_PAIRS = 1
ROPE_SPLIT = 2
ROPE_SPLIT64 = 3


class Epilogue(ctypes.Structure):
    _fields_ = [
        ("kind", c_int),
        ("bias", c_void_p),
        ("residual", c_void_p),
        ("ld_residual", c_int64),
        ("bs_residual", c_int64),
        ("gate", c_void_p),
        ("bs_gate", c_int64),
        ("act_col_begin", c_int64),
        ("scalar", c_float),
        ("aux", c_void_p),
        ("ld_aux", c_int64),
        ("bs_aux", c_int64),
        ("scalar2", c_float),
        ("norm_weight", c_void_p * 2),
        ("norm_col", c_int64 * 2),
        ("norm_width", c_int64),
        ("rope_cos", c_void_p),
        ("rope_sin", c_void_p),
        ("rope_rows", c_int64),
        ("rope_offset", c_int64),
        ("rope_batched", c_int),
        ("norm_eps", c_float),
        ("scatter_ptrs", c_void_p),
        ("world", c_int64),
        ("scatter_cols", c_int64),
        ("seg_width", c_int64),
        ("part_width", c_int64),
        ("scatter_ld", c_int64),
        ("scatter_row0", c_int64),
        ("scatter_rows", c_int64),
        ("seg_slot", c_int * 4),
        ("w_lead", c_void_p),
        ("ldw_lead", c_int64),
        ("lead_rows", c_int64),
        ("norm_weight_lead", c_void_p * 2),
        ("gate_lead", c_void_p),
        ("bias_after_round", c_int),
    ]


class AttentionArgs(ctypes.Structure):
    _fields_ = [
        ("batch", c_int64),
        ("heads", c_int64),
        ("head_dim", c_int64),
        ("scale", c_float),
        ("n_q", c_int),
        ("q", c_void_p * 2),
        ("out", c_void_p * 2),
        ("q_tokens", c_int64 * 2),
        ("ld_q", c_int64 * 2),
        ("bs_q", c_int64 * 2),
        ("ld_out", c_int64 * 2),
        ("bs_out", c_int64 * 2),
        ("gate", c_void_p * 2),
        ("ld_gate", c_int64 * 2),
        ("bs_gate", c_int64 * 2),
        ("n_kv", c_int),
        ("k", c_void_p * 2),
        ("v", c_void_p * 2),
        ("kv_tokens", c_int64 * 2),
        ("ld_k", c_int64 * 2),
        ("bs_k", c_int64 * 2),
        ("ld_v", c_int64 * 2),
        ("bs_v", c_int64 * 2),
        ("out_peers", c_void_p),
        ("gate_peers", c_void_p),
        ("world", c_int64),
        ("rows_per_rank", c_int64),
        ("out_col_offset", c_int64),
        ("out_cols", c_int64),
        ("gate_head_offset", c_int64),
        ("key_bias", c_void_p),
        ("ld_key_bias", c_int64),
        ("kv_splits", c_int64),
        ("workspace", c_void_p),
        ("workspace_bytes", c_int64),
    ]


class Conv3dArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p),
        ("frames", c_int64),
        ("height", c_int64),
        ("width", c_int64),
        ("in_channels", c_int64),
        ("weight", c_void_p),
        ("out_channels", c_int64),
        ("bias", c_void_p),
        ("residual", c_void_p),
        ("out", c_void_p),
        ("causal", c_int),
        ("stride_t", c_int),
        ("stride_h", c_int),
        ("stride_w", c_int),
        ("stats", c_void_p),
        ("stats_records", c_int64),
        ("workspace", c_void_p),
        ("workspace_bytes", c_int64),
    ]


class EpilogueF32(ctypes.Structure):
    _fields_ = [
        ("kind", c_int),
        ("bias", c_void_p),
        ("residual", c_void_p),
        ("ld_residual", c_int64),
        ("bs_residual", c_int64),
        ("gate", c_void_p),
        ("bs_gate", c_int64),
        ("act_col_begin", c_int64),
        ("scalar", c_float),
        ("aux", c_void_p),
        ("ld_aux", c_int64),
        ("bs_aux", c_int64),
        ("scalar2", c_float),
    ]


class FluxBlockShape(ctypes.Structure):
    _fields_ = [
        ("batch", c_int64),
        ("text_tokens", c_int64),
        ("image_tokens", c_int64),
        ("heads", c_int64),
        ("mlp_hidden", c_int64),
        ("mlp", c_int),
        ("eps", c_float),
    ]


class RopeTablesArgs(ctypes.Structure):
    _fields_ = [("cos", c_void_p), ("sin", c_void_p), ("rows", c_int64), ("batched", c_int)]


class FluxDoubleWeights(ctypes.Structure):
    _fields_ = [(name, c_void_p) for name in (
        "img_qkv", "txt_qkv", "to_out", "to_add_out", "norm_q", "norm_k", "norm_added_q",
        "norm_added_k", "ff_in", "ff_out", "ffc_in", "ffc_out")]


class FluxSingleWeights(ctypes.Structure):
    _fields_ = [(name, c_void_p) for name in ("fused", "to_out", "norm_q", "norm_k")]


class LTXBlockShape(ctypes.Structure):
    _fields_ = [
        ("batch", c_int64),
        ("tokens", c_int64),
        ("context_tokens", c_int64),
        ("heads", c_int64),
        ("context_dim", c_int64),
        ("ff_hidden", c_int64),
        ("eps", c_float),
    ]


class LTXVideoBlockWeights(ctypes.Structure):
    _fields_ = [(name, c_void_p) for name in (
        "qkv_w", "qkv_b", "g1_w", "g1_b", "o1_w", "o1_b", "qn1", "kn1", "q2_w", "q2_b", "kv2_w",
        "kv2_b", "g2_w", "g2_b", "o2_w", "o2_b", "qn2", "kn2", "ff_in_w", "ff_in_b", "ff_out_w",
        "ff_out_b")]


class SolAttentionArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p),
        ("k", c_void_p),
        ("v", c_void_p),
        ("ld_q", c_int64),
        ("ld_k", c_int64),
        ("ld_v", c_int64),
        ("out", c_void_p),
        ("ld_out", c_int64),
        ("gate", c_void_p),
        ("ld_gate", c_int64),
        ("tokens", c_int64),
        ("heads", c_int64),
        ("dtype", c_int),
        ("tau", c_float),
        ("order", c_void_p),
        ("routes", c_void_p),
        ("workspace", c_void_p),
        ("workspace_bytes", c_int64),
    ]


DTYPE_BF16 = 0
DTYPE_F16 = 1
MLP_GELU_TANH = 0
MLP_SWIGLU = 1


class IpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


I64 = c_int64
P = c_void_p
F = c_float

# Every exported entry point with its argument types, in include/kino.h order.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "kino_abi_version": (c_int, []),
    "kino_last_error": (ctypes.c_char_p, []),
    "kino_device_status": (c_int, [P]),
    "kino_num_sms": (c_int, []),
    "kino_linear": (
        c_int,
        [P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, POINTER(Epilogue), P],
    ),
    "kino_gemv": (c_int, [P, I64, P, P, P, I64, I64, I64, I64, c_int, P]),
    "kino_attention": (c_int, [POINTER(AttentionArgs), P]),
    "kino_dense_attention": (c_int, [P, P, P, P, I64, I64, I64, I64, P]),
    "kino_sol_attention_workspace_size": (I64, [I64, I64]),
    "kino_sol_attention": (c_int, [POINTER(SolAttentionArgs), P]),
    "kino_attention_workspace_size": (I64, [POINTER(AttentionArgs), I64]),
    "kino_neighborhood_attention": (c_int, [P, P, P, P, I64, I64, I64, I64, I64, P, P]),
    "kino_neighborhood_attention_ex": (c_int, [P, P, P, P, c_int, I64, I64, I64, I64, I64, P, P]),
    "kino_na_qkv_prepare": (
        c_int,
        [P, I64, P, P, P, P, P, P, I64, I64, I64, I64, I64, P, F, F, P],
    ),
    "kino_strided_copy": (c_int, [P, c_int, P, P, c_int, P, P, c_int, P]),
    "kino_adaln": (c_int, [P, I64, I64, P, P, I64, P, I64, I64, I64, I64, I64, c_int, F, P]),
    "kino_rms_norm": (c_int, [P, P, P, I64, I64, F, F, P]),
    "kino_qk_norm_rope": (
        c_int,
        [P, I64, I64, I64, I64, I64, P, c_int, c_int, P, P, c_int, I64, I64, F, P],
    ),
    "kino_qk_norm_rope_to_peers": (
        c_int,
        [P, I64, I64, I64, P, c_int, c_int, P, P, c_int, I64, I64, F, P, I64, I64, I64, I64, I64, P],
    ),
    "kino_split_rope": (c_int, [P, P, P, P, I64, I64, I64, I64, c_int, P]),
    "kino_gelu_tanh": (c_int, [P, P, I64, P]),
    "kino_silu": (c_int, [P, P, I64, P]),
    "kino_cfg_combine": (c_int, [P, P, F, P, I64, P]),
    "kino_euler_velocity": (c_int, [P, P, F, P, I64, P]),
    "kino_euler_x0": (c_int, [P, P, F, F, P, I64, P]),
    "kino_euler_step": (c_int, [P, P, F, P, I64, P]),
    "kino_euler_velocity_step": (c_int, [P, P, F, P, I64, P]),
    "kino_add_rows": (c_int, [P, P, P, I64, I64, P]),
    "kino_heads_pack": (c_int, [P, I64, P, I64, I64, I64, P]),
    "kino_heads_unpack": (c_int, [P, P, I64, I64, I64, I64, P, I64, P]),
    "kino_timestep_embedding": (c_int, [P, P, I64, I64, P]),
    "kino_conv3d": (c_int, [POINTER(Conv3dArgs), P]),
    "kino_pixel_norm": (c_int, [P, P, I64, I64, F, c_int, P]),
    "kino_group_norm_workspace_size": (c_int64, [I64, I64]),
    "kino_group_norm": (c_int, [P, P, P, P, I64, I64, F, c_int, P, I64, P]),
    "kino_conv3d_stats_size": (c_int64, []),
    "kino_conv3d_workspace_size": (c_int64, []),
    "kino_dequantize": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, I64, I64, c_int, c_int,
                                c_int, c_int, c_void_p]),
    "kino_group_norm_from_stats": (c_int, [P, P, P, P, I64, I64, F, c_int, P, P]),
    "kino_group_norm_noalloc": (c_int, [P, P, P, P, I64, I64, F, c_int, P]),
    "kino_latent_to_bfhwc": (c_int, [P, P, P, P, I64, I64, P]),
    "kino_tile_blend": (c_int, [P, I64, I64, I64, I64, I64, P, P, I64, I64, I64, I64, P, P, P]),
    "kino_blend_normalize": (c_int, [P, P, I64, I64, P]),
    "kino_linear_f32": (
        c_int,
        [P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, POINTER(EpilogueF32), P],
    ),
    "kino_attention_f32": (
        c_int,
        [P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, F, P, I64, I64,
         P, I64, P],
    ),
    "kino_adaln_f32": (c_int, [P, I64, I64, P, P, I64, P, I64, I64, I64, I64, I64, c_int, F, P]),
    "kino_qk_norm_rope_f32": (
        c_int,
        [P, I64, I64, I64, I64, I64, P, c_int, c_int, P, P, c_int, I64, I64, F, P],
    ),
    "kino_add_rows_f32": (c_int, [P, P, P, I64, I64, P]),
    "kino_gelu_tanh_f32": (c_int, [P, P, I64, P]),
    "kino_silu_f32": (c_int, [P, P, I64, P]),
    "kino_cfg_combine_f32": (c_int, [P, P, F, P, I64, P]),
    "kino_euler_velocity_f32": (c_int, [P, P, F, P, I64, P]),
    "kino_euler_step_f32": (c_int, [P, P, F, P, I64, P]),
    "kino_swiglu_f32": (c_int, [P, I64, I64, P, I64, I64, I64, I64, I64, P]),
    "kino_timestep_embedding_f32": (c_int, [P, P, I64, I64, P]),
    "kino_conv3d_f32": (
        c_int,
        [P, I64, I64, I64, I64, P, I64, P, P, P, c_int, c_int, c_int, c_int, P],
    ),
    "kino_pixel_norm_f32": (c_int, [P, P, I64, I64, F, c_int, P]),
    "kino_group_norm_f32": (c_int, [P, P, P, P, I64, I64, F, c_int, P]),
    "kino_latent_to_bfhwc_f32": (c_int, [P, P, P, P, I64, I64, P]),
    "kino_tile_blend_f32": (c_int, [P, I64, I64, I64, I64, I64, P, P, I64, I64, I64, I64, P, P, P]),
    "kino_flux_block_workspace_size": (I64, [POINTER(FluxBlockShape)]),
    "kino_flux_double_block": (
        c_int,
        [POINTER(FluxBlockShape), POINTER(FluxDoubleWeights), P, P, I64, POINTER(RopeTablesArgs),
         P, I64, P],
    ),
    "kino_flux_single_block": (
        c_int,
        [POINTER(FluxBlockShape), POINTER(FluxSingleWeights), P, P, I64, POINTER(RopeTablesArgs),
         P, I64, P],
    ),
    "kino_ltx_video_block_workspace_size": (I64, [POINTER(LTXBlockShape)]),
    "kino_ltx_video_block": (
        c_int,
        [POINTER(LTXBlockShape), POINTER(LTXVideoBlockWeights), P, P, P, I64, P, I64, P, P, c_int,
         P, I64, P],
    ),
    "kino_peer_alloc": (c_int, [I64, POINTER(c_void_p), POINTER(IpcHandle)]),
    "kino_peer_free": (c_int, [P]),
    "kino_peer_open": (c_int, [POINTER(IpcHandle), POINTER(c_void_p)]),
    "kino_peer_close": (c_int, [P]),
    "kino_peer_barrier": (c_int, [P, I64, I64, I64, P]),
}

_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once and declare every signature; raise if it is not built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIBRARY_PATH.exists():
        raise RuntimeError(
            f"{LIBRARY_PATH.name} is not built; run `python -m kinomlx_b200.build` "
            "(the sm_100a kernels have no fallback)"
        )
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


def last_error() -> str:
    raw = load().kino_last_error()
    return raw.decode() if raw else ""


def call(name: str, *args: object) -> None:
    """Call one kino_* entry point and raise RuntimeError on a non-OK status."""
    status = getattr(load(), name)(*args)
    if status != KINO_OK:
        label = STATUS_NAMES.get(status, str(status))
        raise RuntimeError(f"{name} failed with {label}: {last_error()}")
