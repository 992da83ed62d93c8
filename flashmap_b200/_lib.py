"""ctypes binding of ``libflashmap_b200.so`` (the C ABI of include/flashmap_b200.h).

There is no fallback: if the library is missing or the GPU is not an sm_100
part, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libflashmap_b200.so")

c_void_p, c_int, c_int32, c_int64, c_uint32, c_uint64, c_float, c_size_t = (
    ctypes.c_void_p, ctypes.c_int, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64,
    ctypes.c_float, ctypes.c_size_t,
)

FM_EPI_STORE, FM_EPI_GELU, FM_EPI_SWIGLU, FM_EPI_RESID, FM_EPI_F32 = 0, 1, 2, 3, 7


class LayerWeights(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in (
        "self_qkv_w", "self_o_w", "self_q_norm", "self_k_norm", "cross_q_w", "cross_o_w", "cross_q_norm",
        "mlp_w1", "mlp_b1", "mlp_w2", "mlp_b2")]


class ModelDesc(ctypes.Structure):
    _fields_ = (
        [(n, c_int32) for n in ("hidden", "heads", "head_dim", "inter", "layers", "target_hidden",
                                "n_target_layers", "block", "vocab", "state_vocab", "swiglu")]
        + [("rms_eps", c_float), ("qk_eps", c_float), ("ln_eps", c_float)]
        + [(n, c_void_p) for n in ("fc_w", "hidden_norm_w", "anchor_proj_w", "anchor_proj_b", "anchor_norm_w",
                                   "noise_norm_w", "x_embed_w", "x_embed_b", "head_w", "head_b", "cross_kv_w",
                                   "cross_k_norm")]
        + [("layer", ctypes.POINTER(LayerWeights))]
        + [(n, c_void_p) for n in ("embed", "lm_w", "lm_b", "draft_ids", "embed_state_t", "chol",
                                   "uniform_embeds", "state_norm_w", "rope_cos", "rope_sin")]
        + [("rope_len", c_int32)]
        + [(n, c_void_p) for n in ("lm_fold_w", "lm_fold_b", "noise_fold_w", "noise_fold_var", "noise_fold_x0")]
    )


class Jump(ctypes.Structure):
    _fields_ = [("mods", c_void_p), ("noise_gate", c_float), ("s", c_float), ("next", c_float)]


class PlanConfig(ctypes.Structure):
    _fields_ = [("batch", c_int32), ("num_steps", c_int32), ("jumps", ctypes.POINTER(Jump)), ("cache", c_void_p),
                ("cache_batch", c_int32), ("cache_len", c_int32), ("max_extend_rows", c_int32),
                ("launch_mode", c_int32)]


LAUNCH_AUTO, LAUNCH_KERNELS, LAUNCH_STREAM = 0, 1, 2


class DraftIO(ctypes.Structure):
    _fields_ = [("anchor_ids", c_void_p), ("lengths", c_void_p), ("z", c_void_p), ("noise", c_void_p),
                ("seed", c_uint64), ("offset", c_uint32), ("offset_ptr", c_void_p), ("logits", c_void_p),
                ("ldl", c_int64),
                ("scatter", c_int32), ("tokens", c_void_p), ("hidden", c_void_p)]


class ForwardIO(ctypes.Structure):
    _fields_ = [("inputs", c_void_p), ("positions", c_void_p), ("ctx_last", c_void_p), ("mods", c_void_p),
                ("hidden", c_void_p)]


class ExtendIO(ctypes.Structure):
    _fields_ = [("target_hidden", c_void_p), ("rows", c_int32), ("cu_rows", c_void_p), ("lengths", c_void_p),
                ("batch", c_int32)]


FM_DT_BF16, FM_DT_F32, FM_DT_E4M3, FM_DT_I32, FM_DT_I64 = 0, 1, 2, 3, 4
FM_NORM_DIT, FM_NORM_FUSED = 0, 1


class RopeView(ctypes.Structure):
    _fields_ = [("cos", c_void_p), ("sin", c_void_p), ("row_stride", c_int64), ("pair_stride", c_int64),
                ("rows", c_int64)]


class BankJump(ctypes.Structure):
    _fields_ = [("noise_embed", c_void_p), ("mean_embed", c_void_p), ("log_mass", c_void_p), ("embed", c_void_p),
                ("state_map", c_void_p), ("bank_rows", c_int64), ("state_rows", c_int64), ("hidden", c_int64),
                ("slots", c_int64), ("rows", c_void_p), ("seeds", c_void_p), ("ids", c_void_p), ("probs", c_void_p),
                ("betas", c_void_p), ("support", c_int32), ("topk", c_int32), ("alpha", c_float),
                ("evidence", c_float), ("slope", c_float), ("temperature", c_float), ("out", c_void_p),
                ("err", c_void_p)]


class PagedAttn(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("q_dtype", c_int32), ("q_token_stride", c_int64), ("q_head_stride", c_int64),
                ("cu_seqlens_q", c_void_p), ("q_per_request", c_int64), ("max_q", c_int64),
                ("k", c_void_p), ("v", c_void_p), ("kv_dtype", c_int32),
                ("kv_page_stride", c_int64), ("kv_head_stride", c_int64), ("kv_token_stride", c_int64),
                ("page_size", c_int64), ("num_pages", c_int64),
                ("page_table", c_void_p), ("page_table_stride", c_int64), ("page_table_cols", c_int64),
                ("seqused_k", c_void_p), ("max_seqlen_k", c_int64),
                ("requests", c_int64), ("heads", c_int64), ("head_dim", c_int64),
                ("softmax_scale", c_float), ("descales", c_void_p), ("quantize_q", c_int32),
                ("out", c_void_p), ("out_token_stride", c_int64), ("out_head_stride", c_int64),
                ("workspace", c_void_p), ("workspace_bytes", c_size_t), ("nsplit", c_int32), ("err", c_void_p)]


_SIGNATURES = {
    "fm_last_error": (ctypes.c_char_p, []),
    "fm_version": (c_int, []),
    "fm_check_device": (c_int, []),
    "fm_gemm_workspace_size": (c_size_t, [c_int64, c_int64, c_int64]),
    "fm_gemm_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                             c_int, c_void_p, c_size_t, c_void_p, c_void_p]),
    "fm_gemm_grid": (c_int32, [c_int64, c_int64, c_int64]),
    "fm_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p]),
    "fm_adaln": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p]),
    "fm_rope_table": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "fm_philox_normal": (c_int, [c_void_p, c_int64, c_uint64, c_uint32, c_void_p]),
    "fm_philox_normal_rows": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_float, c_void_p]),
    "fm_philox_normal_rows_f32": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_float,
                                          c_void_p]),
    "fm_state_rows": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_int32, c_void_p]),
    "fm_state_update": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_float, c_float, c_void_p]),
    "fm_noise_fold": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_float, c_int64, c_int64,
                              c_int64, c_void_p]),
    "fm_mix_state": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_float, c_int64,
                             c_int64, c_void_p]),
    "fm_block_self_attn": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p]),
    "fm_cross_attn_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int64]),
    "fm_cross_attn": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
                              c_int64, c_int64, c_int64, c_void_p, c_size_t, c_void_p, c_void_p]),
    "fm_qk_norm_rope": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int32,
                                RopeView, c_void_p, c_int32, c_float, c_int32, c_void_p, c_void_p]),
    "fm_block_self_attn_qknorm": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                          c_void_p, c_int32, RopeView, c_void_p, c_int32, c_float, c_float,
                                          c_void_p, c_void_p]),
    "fm_paged_attn_nsplit": (c_int32, [c_int64, c_int64, c_int64, c_int64, c_int32]),
    "fm_paged_attn_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int32]),
    "fm_paged_cross_attn": (c_int, [ctypes.POINTER(PagedAttn), c_void_p]),
    "fm_tree_build": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p]),
    "fm_tree_commit": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                               c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p]),
    "fm_bank_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int32, c_void_p]),
    "fm_topk_rows": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p, c_int64, c_void_p, c_void_p,
                             c_void_p, c_void_p]),
    "fm_bank_gather": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "fm_bank_jump_rows": (c_int, [ctypes.POINTER(BankJump), c_void_p]),
    "fm_token_normals": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "fm_philox_randint": (c_int, [c_void_p, c_int64, c_int64, c_uint64, c_uint32, c_uint32, c_void_p]),
    "fm_write_context_kv_paged": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                          c_void_p, c_int32, RopeView, c_void_p, c_int64, c_int64, c_int64,
                                          c_int64, c_int64, c_int64, c_int64, c_float, c_void_p, c_void_p,
                                          c_void_p]),
    "fm_kv_norm_rope_write_pool": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                           c_int32, RopeView, c_void_p, c_void_p, c_void_p, c_int64, c_int32,
                                           c_int32, c_float, c_float, c_float, c_void_p, c_void_p]),
    "fm_row_stats": (c_int, [c_void_p, c_int32, c_int64, c_int64, c_float, c_void_p, c_void_p, c_void_p]),
    "fm_softmax_rows": (c_int, [c_void_p, c_int32, c_int64, c_int64, c_float, c_void_p, c_void_p]),
    "fm_sample_rows": (c_int, [c_void_p, c_int32, c_void_p, c_int64, c_int64, c_int64, c_float, c_uint64, c_uint32,
                               c_void_p, c_void_p]),
    "fm_accept_workspace_size": (c_size_t, [c_int64, c_int64]),
    "fm_accept_greedy": (c_int, [c_void_p, c_int32, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                 c_void_p, c_size_t, c_void_p]),
    "fm_accept_greedy_noalloc": (c_int, [c_void_p, c_int32, c_void_p, c_int64, c_int64, c_int64, c_void_p,
                                         c_void_p, c_void_p]),
    "fm_accept_rejection": (c_int, [c_void_p, c_int32, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float,
                                    c_uint64, c_uint32, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "fm_transpose_bf16": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "fm_time_sinusoid": (c_int, [c_void_p, c_int64, c_float, c_float, c_float, c_void_p, c_void_p]),
    "fm_silu": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "fm_add": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "fm_plan_workspace_size": (c_int, [ctypes.POINTER(ModelDesc), ctypes.POINTER(PlanConfig),
                                       ctypes.POINTER(c_size_t)]),
    "fm_plan_create": (c_int, [ctypes.POINTER(ModelDesc), ctypes.POINTER(PlanConfig), c_void_p, c_size_t,
                               ctypes.POINTER(c_void_p)]),
    "fm_plan_destroy": (c_int, [c_void_p]),
    "fm_plan_error_word": (c_void_p, [c_void_p]),
    "fm_plan_last_launches": (c_int64, [c_void_p]),
    "fm_plan_lm_head": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "fm_draft": (c_int, [c_void_p, ctypes.POINTER(DraftIO), c_void_p]),
    "fm_extend_context": (c_int, [c_void_p, ctypes.POINTER(ExtendIO), c_void_p]),
    "fm_forward": (c_int, [c_void_p, ctypes.POINTER(ForwardIO), c_void_p]),
}

_lib = None


class FlashMapError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """The loaded library (raises when it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FlashMapError(f"{LIB_PATH} is missing: build it with `python -m flashmap_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list:
    return sorted(_SIGNATURES)


def check(status: int, what: str = "") -> None:
    if status != 0:
        msg = load().fm_last_error().decode(errors="replace")
        raise FlashMapError(f"{what or 'flashmap_b200'} failed (status {status}): {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def require_device() -> None:
    """Raise unless the current CUDA device is a B200-class sm_100 GPU."""
    check(load().fm_check_device(), "fm_check_device")
