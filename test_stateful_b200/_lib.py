"""ctypes binding of ``libqtts_b200.so`` (declared in ``include/qtts_b200.h``).

Status codes map to the exception types the reference executor raises
(engine/backend/executor.py:253-302, 394, 632-638): invalid arguments and
capacity problems become ``ValueError``, everything else ``RuntimeError``.
There is no fallback: if the library is missing the import of the runtime
fails with an error that says so.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libqtts_b200.so"

OK = 0
ERR_INVALID = -1
ERR_CUDA = -2
ERR_CAPACITY = -3
ERR_POOL_EXHAUSTED = -4
ERR_TIMEOUT = -5
ERR_UNSUPPORTED = -6

EPI_BF16, EPI_F32, EPI_RESIDUAL, EPI_SWIGLU, EPI_QKV_ROPE = range(5)
ATTN_SPLIT_BLOCKS = 16

_STATUS_NAMES = {ERR_INVALID: "invalid argument", ERR_CUDA: "CUDA error", ERR_CAPACITY: "sequence capacity",
                 ERR_POOL_EXHAUSTED: "KV pool exhausted", ERR_TIMEOUT: "device wait timed out",
                 ERR_UNSUPPORTED: "unsupported shape"}

P = C.c_void_p
I32 = C.c_int32
F32 = C.c_float


class PagedState(C.Structure):
    _fields_ = [("free_stack", P), ("free_top", P), ("refcount", P), ("block_table", P), ("seq_len", P),
                ("position_offset", P), ("num_blocks", I32), ("block_size", I32), ("max_slots", I32),
                ("max_blocks_per_seq", I32)]


class QkvEpilogue(C.Structure):
    _fields_ = [("num_heads", I32), ("kv_heads", I32), ("head_dim", I32), ("q_norm_w", P), ("k_norm_w", P),
                ("rms_eps", F32), ("rope_cos", P), ("rope_sin", P), ("max_pos", I32), ("row_pos", P),
                ("slot_mapping", P), ("kv_pool", P), ("layer", I32), ("num_layers", I32), ("block_size", I32)]


class ModelDesc(C.Structure):
    _fields_ = [
        ("layers", I32), ("hidden", I32), ("heads", I32), ("kv_heads", I32), ("head_dim", I32), ("inter", I32),
        ("vocab", I32), ("eos_id", I32), ("topk", I32), ("rms_eps", F32),
        ("w_qkv", P), ("w_o", P), ("w_gate_up", P), ("w_down", P), ("w_in_norm", P), ("w_post_norm", P),
        ("w_q_norm", P), ("w_k_norm", P), ("w_final_norm", P), ("w_codec_head", P), ("w_codec_emb", P),
        ("rope_cos", P), ("rope_sin", P), ("max_pos", I32),
        ("cp_layers", I32), ("cp_hidden", I32), ("cp_heads", I32), ("cp_kv_heads", I32), ("cp_head_dim", I32),
        ("cp_inter", I32), ("cp_vocab", I32), ("cp_stages", I32), ("cp_rms_eps", F32),
        ("cp_w_proj", P), ("cp_b_proj", P), ("cp_w_qkv", P), ("cp_w_o", P), ("cp_w_gate_up", P), ("cp_w_down", P),
        ("cp_w_in_norm", P), ("cp_w_post_norm", P), ("cp_w_q_norm", P), ("cp_w_k_norm", P),
        ("cp_w_final_norm", P), ("cp_w_lm_head", P), ("cp_w_codec_emb", P), ("cp_rope_cos", P),
        ("cp_rope_sin", P),
        ("pool", PagedState), ("kv_pool", P), ("max_batch", I32), ("max_prefill_rows", I32),
    ]


class StepIO(C.Structure):
    _fields_ = [("slots", P), ("n_rows", I32), ("n_new", I32), ("slot_indexed", I32), ("x_in", P), ("token_counts", P), ("gumbel", P),
                ("cp_gumbel", P), ("noise_seed", C.c_uint64), ("noise_key", P), ("noise_step", P), ("step", I32),
                ("temperature", P), ("penalty", P), ("sample", I32), ("text_add", P), ("hidden_out", P),
                ("logits_out", P), ("full_codec_out", P), ("codec_sum_out", P), ("next_x_out", P), ("status", P),
                ("force_codes", P), ("cp_logits_out", P), ("launches", I32)]


class C2wDesc(C.Structure):
    _fields_ = [
        ("num_codebooks", I32), ("codebook_size", I32), ("codebook_dim", I32), ("latent", I32), ("hidden", I32),
        ("layers", I32), ("heads", I32), ("head_dim", I32), ("inter", I32),
        ("window", I32), ("decoder_dim", I32), ("convnext_dim", I32), ("max_slots", I32), ("max_frames", I32),
        ("max_chunk", I32),
        ("up_ratio", I32 * 2), ("rates", I32 * 4), ("dilations", I32 * 3), ("rms_eps", F32), ("ln_eps", F32),
        ("rvq_tables", P), ("w_pre_conv", P), ("b_pre_conv", P), ("w_in_proj", P), ("b_in_proj", P),
        ("w_in_norm", P), ("w_qkv", P), ("w_q_norm", P), ("w_k_norm", P), ("w_o", P), ("attn_scale", P),
        ("w_post_norm", P), ("w_gate_up", P), ("w_down", P), ("mlp_scale", P), ("w_final_norm", P),
        ("w_out_proj", P), ("b_out_proj", P), ("rope_cos", P), ("rope_sin", P),
        ("up_w", P * 2), ("up_b", P * 2), ("dw_w", P * 2), ("dw_b", P * 2), ("ln_w", P * 2), ("ln_b", P * 2),
        ("pw1_w", P * 2), ("pw1_b", P * 2), ("pw2_w", P * 2), ("pw2_b", P * 2), ("gamma", P * 2),
        ("w_conv0", P), ("b_conv0", P), ("blk_snake", P * 4), ("blk_tw", P * 4), ("blk_tb", P * 4),
        ("res_act1", (P * 3) * 4), ("res_act2", (P * 3) * 4), ("res_w1", (P * 3) * 4), ("res_b1", (P * 3) * 4),
        ("res_w2", (P * 3) * 4), ("res_b2", (P * 3) * 4),
        ("final_snake", P), ("final_w", P), ("final_b", F32),
    ]


# every symbol the header declares, in header order
EXPORTS = [
    "qtts_version", "qtts_last_error", "qtts_device_error", "qtts_selftest_bounded_wait",
    "qtts_sched_init", "qtts_sched_append", "qtts_kv_copy_blocks", "qtts_sched_share_prefix",
    "qtts_sched_make_entry", "qtts_sched_drop_blocks", "qtts_sched_release", "qtts_kv_scatter", "qtts_kv_gather",
    "qtts_gemm", "qtts_rmsnorm", "qtts_paged_attention", "qtts_paged_attention_prefill",
    "qtts_paged_attention_noalloc", "qtts_sample",
    "qtts_philox_gumbel", "qtts_codec_sum",
    "qtts_engine_create", "qtts_engine_destroy", "qtts_engine_step",
    "qtts_c2w_create", "qtts_c2w_destroy", "qtts_c2w_reset", "qtts_c2w_step", "qtts_c2w_launches",
    "qtts_c2w_set_background", "qtts_c2w_state_layout", "qtts_c2w_write_state", "qtts_c2w_set_frame",
]

C2W_STATE_PARTS = 22


class C2wStatePart(C.Structure):
    """qtts_c2w_state_part: one part of a slot's code2wav state in the decoder's layout."""
    _fields_ = [("rows", C.c_int32), ("row_elems", C.c_int32), ("valid_elems", C.c_int32), ("dtype", C.c_int32)]

_lib = None


def load() -> C.CDLL:
    """Load the library (building it first when sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists() or os.environ.get("QTTS_REBUILD"):
        from .build import build
        build()
    if not LIB_PATH.exists():
        raise RuntimeError(f"libqtts_b200.so not found at {LIB_PATH}; run `python -m test_stateful_b200.build`")
    lib = C.CDLL(str(LIB_PATH))
    sig = {
        "qtts_version": ([], C.c_int),
        "qtts_last_error": ([C.c_char_p, C.c_size_t], C.c_int),
        "qtts_device_error": ([C.POINTER(C.c_int)], C.c_int),
        "qtts_selftest_bounded_wait": ([C.c_ulonglong, C.c_int, P, P], C.c_int),
        "qtts_sched_init": ([C.POINTER(PagedState), P], C.c_int),
        "qtts_sched_append": ([C.POINTER(PagedState), P, C.c_int, C.c_int, P, P, P, P, P, P, P], C.c_int),
        "qtts_kv_copy_blocks": ([P, C.c_size_t, C.c_int, P, P, C.c_int, P], C.c_int),
        "qtts_sched_share_prefix": ([C.POINTER(PagedState), C.c_int, P, C.c_int, P, P], C.c_int),
        "qtts_sched_make_entry": ([C.POINTER(PagedState), C.c_int, C.c_int, P, P], C.c_int),
        "qtts_sched_drop_blocks": ([C.POINTER(PagedState), P, C.c_int, P], C.c_int),
        "qtts_sched_release": ([C.POINTER(PagedState), C.c_int, P], C.c_int),
        "qtts_kv_scatter": ([P, C.POINTER(PagedState), C.c_int, C.c_int, C.c_int, P, P, C.c_int, P], C.c_int),
        "qtts_kv_gather": ([P, C.POINTER(PagedState), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P, P], C.c_int),
        "qtts_gemm": ([P, P, C.c_int, C.c_int, P, C.c_int, C.c_int, P, P, P, C.POINTER(QkvEpilogue), P], C.c_int),
        "qtts_rmsnorm": ([P, C.c_int, C.c_int, C.c_int, P, C.c_float, P, P, P], C.c_int),
        "qtts_paged_attention": ([P, C.c_int, C.c_int, C.c_int, C.c_int, P, C.c_int, C.c_int, C.c_int, C.c_int,
                                  P, C.c_int, P, P, C.c_int, C.c_int, P, P, P, P, P], C.c_int),
        "qtts_paged_attention_prefill": ([P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P, C.c_int, C.c_int,
                                          C.c_int, C.c_int, P, C.c_int, P, P, C.c_int, C.c_int, P, P, P, P, P],
                                         C.c_int),
        "qtts_paged_attention_noalloc": ([P, C.c_int, C.c_int, C.c_int, C.c_int, P, C.c_int, C.c_int, C.c_int,
                                          C.c_int, P, C.c_int, P, P, C.c_int, P, P, P], C.c_int),
        "qtts_sample": ([P, C.c_int, C.c_int, C.c_int, C.c_int, P, C.c_int, C.c_uint64, P, C.c_int, P, P, P,
                         C.c_int, P, C.c_int, P], C.c_int),
        "qtts_philox_gumbel": ([C.c_uint64, P, P, C.c_int, C.c_int, C.c_int, P, P], C.c_int),
        "qtts_codec_sum": ([P, C.c_int, C.c_int, P, C.c_int, P, C.c_int, C.c_int, P, P, P, P], C.c_int),
        "qtts_engine_create": ([C.POINTER(ModelDesc), C.POINTER(P)], C.c_int),
        "qtts_engine_destroy": ([P], C.c_int),
        "qtts_engine_step": ([P, C.POINTER(StepIO), P], C.c_int),
        "qtts_c2w_create": ([C.POINTER(C2wDesc), C.POINTER(P)], C.c_int),
        "qtts_c2w_destroy": ([P], C.c_int),
        "qtts_c2w_reset": ([P, P, C.c_int, P], C.c_int),
        "qtts_c2w_step": ([P, P, C.c_int, C.c_int, P, C.c_int, P, P], C.c_int),
        "qtts_c2w_launches": ([P], C.c_int),
        "qtts_c2w_set_background": ([P, C.c_int], C.c_int),
        "qtts_c2w_state_layout": ([P, C.POINTER(C2wStatePart), C.c_int], C.c_int),
        "qtts_c2w_write_state": ([P, C.c_int, C.c_int, P, C.c_size_t, P], C.c_int),
        "qtts_c2w_set_frame": ([P, C.c_int, C.c_int, P], C.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    load().qtts_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    if rc == OK:
        return
    msg = f"{what}: {_STATUS_NAMES.get(rc, rc)}: {last_error()}"
    if rc in (ERR_INVALID, ERR_CAPACITY):
        raise ValueError(msg)
    raise RuntimeError(msg)


def device_error() -> int:
    v = C.c_int(0)
    check(load().qtts_device_error(C.byref(v)), "device_error")
    return v.value


def ptr(t) -> int:
    """Device pointer of a tensor (or None -> NULL)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def stream_ptr(stream=None):
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream
