"""ctypes binding of libmuk.so (declared in include/muk.h).

The library is loaded from this package directory.  There is no fallback:
if the shared object is missing or does not load, every kernel entry point
raises, so a GPU run can never silently fall back to another code path.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libmuk.so")

MUK_OK = 0
MUK_ERR_INVALID_ARG = -1
MUK_ERR_UNSUPPORTED = -2
MUK_ERR_WORKSPACE = -3
MUK_ERR_CUDA = -4
MUK_ERR_DEVICE = -5

MUK_EPI_BF16 = 0
MUK_EPI_F32 = 1
MUK_EPI_SWIGLU = 2
MUK_EPI_BIAS_SILU = 3
MUK_EPI_ROPE_KV = 4

_P = c_void_p
_I32P = c_void_p  # device pointers are passed as integers

# name -> (restype, argtypes); mirrors include/muk.h
SIGNATURES = {
    "muk_version": (c_int, []),
    "muk_last_error": (c_char_p, []),
    "muk_device_error": (c_int, [POINTER(c_int)]),
    "muk_device_error_async": (c_int, [_P, _P]),
    "muk_embed": (c_int, [_P, _P, c_int64, _P, c_int, c_int, c_int, c_int, c_float, c_float,
                          c_float, _P]),
    "muk_residual_rmsnorm": (c_int, [_P, _P, c_int64, c_int64, c_int, _P, _P, c_float, _P,
                                     c_int64, c_int, c_int, c_int, c_int, c_int, c_float,
                                     c_float, c_float, _P]),
    "muk_residual_rmsnorm_bf16": (c_int, [_P, _P, c_int64, _P, _P, c_float, _P, c_int64, c_int,
                                          c_int, c_int, c_int, c_int, c_float, c_float, c_float,
                                          _P]),
    "muk_rmsnorm_rows": (c_int, [_P, _P, c_int, _P, c_float, _P, c_int64, c_int, c_int, c_float,
                                 c_float, c_float, _P]),
    "muk_rope_kv_append": (c_int, [_P, c_int64, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int,
                                   _P, _P, c_float, _P, _P, c_int, c_int, _P]),
    "muk_decode_attn_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "muk_decode_attn_splits": (c_int, [c_int, c_int, c_int]),
    "muk_paged_decode_attn": (c_int, [_P, c_int64, _P, c_int64, _P, _P, _P, c_int, _P, c_int,
                                      c_int, c_int, c_int, c_int, c_int, c_float, c_int, _P,
                                      c_size_t, _P]),
    "muk_decode_attn_static_scratch_bytes": (c_size_t, []),
    "muk_paged_decode_attn_static": (c_int, [_P, c_int64, _P, c_int64, _P, _P, _P, c_int, _P,
                                             c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                                             c_int, _P]),
    "muk_paged_prefill_attn": (c_int, [_P, c_int64, _P, c_int64, _P, _P, _P, c_int, _P, _P, c_int,
                                       c_int, c_int, c_int, c_int, c_int, c_int, c_float, _P]),
    "muk_gemm_bf16": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int, c_int, c_int, c_int,
                              c_int, _P, _P]),
    "muk_gemm_plan_split": (c_int, [c_int, c_int, c_int, c_int, c_int]),
    "muk_gemm_qkv_rope": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int, c_int, _P, _P, _P,
                                  _P, c_int, c_int, c_int, c_int, _P, _P, c_float, _P, _P, c_int,
                                  c_int, _P]),
    "muk_gemm_residual_norm": (c_int, [_P, c_int64, _P, c_int64, c_int, c_int, c_int, _P,
                                       c_int64, _P, _P, c_int64, _P, c_int64, _P]),
    "muk_gemm_clamp_dual": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, _P, c_int64, c_int,
                                    c_int, c_int, c_int, c_float, c_float, c_float, _P]),
    "muk_gemm_swiglu_rownorm": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int, c_int,
                                        c_int, _P, _P]),
    "muk_gemm_qkv_rope_rownorm": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int, c_int, _P,
                                          _P, _P, _P, c_int, c_int, c_int, c_int, _P, _P, c_float,
                                          _P, _P, c_int, c_int, _P, _P]),
    "muk_gemm_plan_info": (c_int, [c_int, c_int, c_int, c_int, c_int, _P]),
    "muk_gemm_set_stream_k": (c_int, [c_int]),
    "muk_set_peer_timeout_ms": (c_int, [c_int]),
    "muk_ipc_get_handle": (c_int, [_P, _P, POINTER(c_uint64)]),
    "muk_ipc_open_handle": (c_int, [_P, c_uint64, POINTER(c_void_p), POINTER(c_void_p)]),
    "muk_ipc_close_handle": (c_int, [_P]),
    "muk_allreduce_flag_bytes": (c_size_t, []),
    "muk_allreduce_scratch_elems": (c_int64, [c_int64, c_int]),
    "muk_allreduce_f32": (c_int, [_P, _P, _P, c_int, c_int, c_int64, c_int, c_int64, _P]),
    "muk_tp_residual_norm": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int64, _P,
                                     _P, c_float, _P, c_int64, c_int, c_int, c_int, c_float,
                                     c_float, c_float, _P]),
    "muk_gemm_tp_residual_norm": (c_int, [_P, c_int64, _P, c_int64, c_int, c_int, c_int, _P, _P,
                                          _P, c_int, c_int, _P, _P, c_float, _P, c_int64, c_int,
                                          c_int, c_int, c_float, c_float, c_float, c_int, _P]),
    "muk_tp_allgather_cols": (c_int, [_P, _P, c_int, c_int, c_int, c_int64, c_int, c_int, _P]),
    "muk_tp_greedy": (c_int, [_P, c_int64, c_int, c_int, c_int, _P, _P, c_int64, _P, _P, c_int,
                              _P, c_int, c_int, _P, _P]),
    "muk_ep_gather_bf16": (c_int, [_P, _P, c_int, c_int, _P, c_int, c_int, c_int, _P]),
    "muk_llama_forward": (c_int, [_P, _P, _P]),
    "muk_deep_forward": (c_int, [_P, _P, _P, _P]),
    "muk_gemm_allreduce_scratch_elems": (c_int64, [c_int, c_int, c_int]),
    "muk_gemm_allreduce_f32": (c_int, [_P, c_int64, _P, c_int64, c_int, c_int, c_int, _P, _P, _P,
                                       c_int, c_int, _P]),
    "muk_route_permute": (c_int, [_P, c_int, c_int, _P, _P, _P, _P]),
    "muk_gather_rows_bf16": (c_int, [_P, c_int64, _P, c_int, _P, c_int64, c_int, _P]),
    "muk_grouped_gemm_bf16": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, _P, c_int, c_int,
                                      c_int, c_int, c_int, _P]),
    "muk_inl_dynamics": (c_int, [_P, _P, _P, _P, _P, c_float, _P, c_int, _P, c_int64, _P, _P,
                                 c_int64,
                                 _P, c_float, _P, c_int64, _P, _P, c_int, c_int, _P, c_int, c_int,
                                 c_int, c_float, c_float, c_float, _P]),
    "muk_reduce_bias_silu": (c_int, [_P, c_int64, c_int, _P, _P, c_int64, c_int, c_int, _P]),
    "muk_reduce_clamp": (c_int, [_P, c_int64, c_int, _P, _P, c_int64, c_int, c_int, c_int,
                                 c_float, c_float, c_float, _P]),
    "muk_sample": (c_int, [_P, c_int64, c_int, c_int, _P, _P, _P, _P, _P, c_int64, _P, _P, _P,
                           _P, _P]),
    "muk_prepare_logits": (c_int, [_P, c_int64, c_int, c_int, _P, _P, _P, _P, _P, c_int64, _P,
                                   _P, c_int64, _P]),
    "muk_mark_seen": (c_int, [_P, c_int64, _P, _P, c_int, c_int, _P]),
    "muk_fill_decode_inputs": (c_int, [_P, _P, _P, c_int, _P]),
}

class MukRowNorm(ctypes.Structure):
    _fields_ = [("sumsq", c_void_p), ("stride", c_int64), ("parts", c_int), ("hidden", c_int),
                ("eps", c_float)]


class MukLlamaLayer(ctypes.Structure):
    _fields_ = [("in_norm", c_void_p), ("wqkv", c_void_p), ("wo", c_void_p),
                ("post_norm", c_void_p), ("wgu", c_void_p), ("wd", c_void_p)]


class MukLlamaModel(ctypes.Structure):
    _fields_ = [("num_layers", c_int), ("hidden", c_int), ("num_q_heads", c_int),
                ("num_kv_heads", c_int), ("head_dim", c_int), ("inter_pad", c_int),
                ("vocab", c_int), ("eps", c_float), ("clamp", c_int), ("mu", c_float),
                ("clamp_min", c_float), ("clamp_max", c_float),
                ("layers", ctypes.POINTER(MukLlamaLayer)), ("embed", c_void_p),
                ("final_norm", c_void_p), ("lm_head", c_void_p), ("rope_cos", c_void_p),
                ("rope_sin", c_void_p), ("rope_len", c_int), ("kv_pool", c_void_p),
                ("num_blocks", c_int), ("block_size", c_int), ("resid", c_void_p),
                ("x", c_void_p), ("x_stride", c_int64), ("qkv", c_void_p), ("attn", c_void_p),
                ("act", c_void_p), ("part", c_void_p), ("part_rows", c_int64), ("xl", c_void_p),
                ("logits", c_void_p), ("attn_ws", c_void_p), ("attn_ws_bytes", c_size_t),
                ("tp_world", c_int), ("tp_rank", c_int), ("ar_data", c_void_p * 8),
                ("ar_scratch", c_void_p * 8), ("ar_flags", c_void_p * 8), ("fused_rope", c_int),
                ("tp_fused", c_int), ("fused_norm", c_int), ("sumsq", c_void_p),
                ("tp_norm", c_int), ("x_peer", c_void_p * 8), ("lm_rows", c_int),
                ("logits_ld", c_int64), ("tp_push_bf16", c_int)]


class MukDeepLayer(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("in_norm", "wcat", "wo", "post_norm", "wci", "bci", "wco",
                                        "bco", "wmu", "mu_param", "q_norm", "k_norm", "wgu", "wd",
                                        "router")]


class MukDeepModel(ctypes.Structure):
    _fields_ = [("num_layers", c_int), ("hidden", c_int), ("num_q_heads", c_int),
                ("num_kv_heads", c_int), ("head_dim", c_int), ("inter_pad", c_int),
                ("vocab", c_int), ("ctrl_hidden", c_int), ("num_experts", c_int),
                ("local_experts", c_int), ("expert_lo", c_int), ("ep_gather", c_int),
                ("eps", c_float), ("dt", c_float), ("clamp", c_int), ("mu", c_float),
                ("clamp_min", c_float), ("clamp_max", c_float),
                ("layers", ctypes.POINTER(MukDeepLayer)), ("embed", c_void_p),
                ("final_norm", c_void_p), ("lm_head", c_void_p), ("rope_cos", c_void_p),
                ("rope_sin", c_void_p), ("rope_len", c_int), ("kv_pool", c_void_p),
                ("num_blocks", c_int), ("block_size", c_int), ("resid", c_void_p),
                ("x", c_void_p), ("x_stride", c_int64), ("qkv", c_void_p), ("attn", c_void_p),
                ("act", c_void_p), ("part", c_void_p), ("part_rows", c_int64), ("h", c_void_p),
                ("hv", c_void_p), ("v", c_void_p), ("ch", c_void_p), ("ctrl", c_void_p),
                ("mp", c_void_p), ("x2", c_void_p), ("xs", c_void_p), ("dpart", c_void_p),
                ("eids", c_void_p), ("offs", c_void_p), ("perm", c_void_p), ("inv", c_void_p),
                ("xl", c_void_p), ("logits", c_void_p), ("logits_ld", c_int64),
                ("lm_rows", c_int), ("attn_ws", c_void_p), ("attn_ws_bytes", c_size_t),
                ("fused_rope", c_int), ("tp_world", c_int), ("tp_rank", c_int),
                ("tp_fused", c_int), ("ar_data", c_void_p * 8), ("ar_scratch", c_void_p * 8),
                ("ar_flags", c_void_p * 8)]


class MukStepBatch(ctypes.Structure):
    _fields_ = [("num_tokens", c_int), ("num_seqs", c_int), ("num_decode", c_int),
                ("max_q_len", c_int), ("decode_len_bound", c_int), ("input_ids", c_void_p),
                ("positions", c_void_p), ("slot_mapping", c_void_p), ("seq_lens", c_void_p),
                ("prefill_cu", c_void_p), ("last_token_idx", c_void_p),
                ("block_tables", c_void_p), ("block_table_stride", c_int)]


_lib: ctypes.CDLL | None = None

# Kernel launches issued through call() (entry points that launch two kernels
# count both); the benchmark reports it as its launch count.
launch_count = 0
_TWO_KERNELS = {"muk_paged_decode_attn", "muk_paged_decode_attn_static", "muk_allreduce_f32",
                "muk_gemm_allreduce_f32", "muk_ep_gather_bf16", "muk_tp_residual_norm",
                "muk_gemm_tp_residual_norm", "muk_tp_allgather_cols", "muk_tp_greedy"}


class MukError(RuntimeError):
    """A libmuk entry point returned a non-zero status."""

    def __init__(self, name: str, code: int, message: str):
        super().__init__(f"{name} failed ({code}): {message}")
        self.code = code


class DeviceError(MukError):
    """A kernel recorded a device-side error (time-out, bad index, shape);
    ``device_code`` is the error word (see common.cuh)."""

    def __init__(self, device_code: int, where: str = "step"):
        super().__init__(where, MUK_ERR_DEVICE, f"device error word {device_code}")
        self.device_code = device_code


def load() -> ctypes.CDLL:
    """Load libmuk.so once and bind every signature; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise MukError("load", MUK_ERR_UNSUPPORTED,
                       f"{LIB_PATH} is missing: build it with complexity-inference_b200/build.py")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().muk_last_error()
    return msg.decode() if msg else ""


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise MukError on failure."""
    global launch_count
    fn = getattr(load(), name)
    rc = fn(*args)
    if rc != MUK_OK:
        raise MukError(name, rc, last_error())
    if name != "muk_device_error":
        launch_count += 2 if name in _TWO_KERNELS else 1


def call_counted(name: str, launches: int, *args) -> None:
    """Call an entry point that launches ``launches`` kernels (native executors)."""
    global launch_count
    fn = getattr(load(), name)
    rc = fn(*args)
    if rc != MUK_OK:
        raise MukError(name, rc, last_error())
    launch_count += launches


def call_native(name: str, *args) -> None:
    """Call a native step executor whose last argument before the stream is
    an ``int*`` receiving its kernel launch count."""
    global launch_count
    n = ctypes.c_int(0)
    fn = getattr(load(), name)
    rc = fn(*args[:-1], ctypes.byref(n), args[-1])
    launch_count += n.value
    if rc != MUK_OK:
        raise MukError(name, rc, last_error())


def call_status(name: str, *args) -> None:
    """Call a status-returning entry point that launches no kernel."""
    fn = getattr(load(), name)
    rc = fn(*args)
    if rc != MUK_OK:
        raise MukError(name, rc, last_error())


def device_error() -> int:
    """Read and clear the device-side error word (synchronises the device)."""
    code = c_int(0)
    call("muk_device_error", ctypes.byref(code))
    return code.value


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
