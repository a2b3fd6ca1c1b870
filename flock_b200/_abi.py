"""ctypes binding of libflock_cuda.so (include/flock_cuda.h).

There is no CPU fallback: if the shared library is missing or was built for
another GPU the import of anything that needs it raises.  The library is
built in-tree by ``python -m flock_b200.build`` (or ``__graft_entry__.build``).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libflock_cuda.so")

FLOCK_OK = 0
FLOCK_E_ARG = -1
FLOCK_E_CUDA = -2
FLOCK_E_STATE = -3
FLOCK_E_MISSING = -4
FLOCK_E_LIMIT = -5
FLOCK_E_NCCL = -6
FLOCK_E_NOMEM = -7
FLOCK_E_UNSUPPORTED = -8

FLOCK_Q8_0, FLOCK_Q4_0, FLOCK_F32 = 8, 4, 32
FLOCK_ROPE_NEOX, FLOCK_ROPE_NORM = 0, 1
FLOCK_ATTN_EXACT, FLOCK_ATTN_FAST = 0, 1
FLOCK_DECODE_KERNELS, FLOCK_DECODE_PERSISTENT, FLOCK_DECODE_EAGER, FLOCK_DECODE_STREAM = \
    0, 1, 2, 3
FLOCK_PREFILL_EXACT, FLOCK_PREFILL_TENSOR = 0, 1
FLOCK_KV_F32, FLOCK_KV_BF16, FLOCK_KV_FP8 = 0, 1, 2
FLOCK_MATVEC_EXACT, FLOCK_MATVEC_FAST = 0, 1
FLOCK_TP_NCCL, FLOCK_TP_PEER = 0, 1


class FlockError(RuntimeError):
    """A non-zero status from the C ABI, carrying flock_last_error()."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg or f"flock error {code}")
        self.code = code


class LayerConfigC(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("n_heads", ctypes.c_int32),
                ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("ffn", ctypes.c_int32), ("eps", ctypes.c_float), ("rope_base", ctypes.c_double),
                ("max_keys", ctypes.c_int32), ("max_prefill", ctypes.c_int32),
                ("rope_pairing", ctypes.c_int32), ("attention", ctypes.c_int32),
                ("prefill", ctypes.c_int32), ("kv_dtype", ctypes.c_int32),
                ("matvec", ctypes.c_int32)]


_vp = ctypes.c_void_p
_pp = ctypes.POINTER(ctypes.c_void_p)
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_ip = ctypes.POINTER(ctypes.c_int)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_fp = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_cfgp = ctypes.POINTER(LayerConfigC)
_ccp = ctypes.POINTER(ctypes.c_char_p)

# name -> argtypes (restype is int unless listed in _RESTYPE)
SIGNATURES = {
    "flock_last_error": [],
    "flock_version": [],
    "flock_dev_open": [_i, _pp],
    "flock_dev_close": [_vp],
    "flock_dev_sync": [_vp],
    "flock_dev_sm_count": [_vp, _ip],
    "flock_dev_timer_start": [_vp],
    "flock_dev_timer_stop": [_vp, _fp],
    "flock_repack_q8": [_u8p, _i64, _i64, _u8p, _u8p],
    "flock_repack_q4": [_u8p, _i64, _i64, _u8p, _u8p],
    "flock_tensor_from_packed": [_vp, _i, _u8p, _i64, _i64, _pp],
    "flock_tensor_from_split": [_vp, _i, _u8p, _u8p, _i64, _i64, _pp],
    "flock_tensor_from_f32": [_vp, _fp, _i64, _pp],
    "flock_tensor_free": [_vp],
    "flock_tensor_bytes": [_vp, _i64p],
    "flock_tensor_from_bytes": [_vp, _vp, _i64, _pp],
    "flock_tensor_read": [_vp, _i64, _i64, _vp],
    "flock_quant_q8": [_fp, _i64, _i64, _u8p],
    "flock_quant_q4": [_fp, _i64, _i64, _u8p],
    "flock_op_matvec": [_vp, _vp, _fp, _i, _fp],
    "flock_op_matvec_timed": [_vp, _vp, _i, _i, _fp],
    "flock_op_matvec_timed_cold": [_vp, _vp, _i, _i, _fp],
    "flock_op_matvec_fast": [_vp, _vp, _fp, _fp],
    "flock_op_matvec_fast_timed": [_vp, _vp, _i, _i, _fp],
    "flock_op_gemm": [_vp, _vp, _fp, _i, _fp],
    "flock_op_gemm_timed": [_vp, _vp, _i, _i, _fp, _fp],
    "flock_op_gemm_timed_cold": [_vp, _vp, _i, _i, _fp, _fp],
    "flock_op_peer_exchange_lone": [_vp, _i, ctypes.c_int64, _i, _i, ctypes.POINTER(ctypes.c_int)],
    "flock_op_rmsnorm": [_vp, _fp, _fp, _i, _i, _f, _fp],
    "flock_op_rope": [_vp, _fp, _i, _i, _i, _i, _fp, _i, _fp],
    "flock_op_swiglu": [_vp, _fp, _fp, _i64, _fp],
    "flock_op_add": [_vp, _fp, _fp, _i64, _fp],
    "flock_op_attention": [_vp, _fp, _fp, _fp, _i, _i, _i, _i, _i, _fp],
    "flock_op_attention_prefill": [_vp, _fp, _fp, _fp, _i, _i, _i, _i, _i, _fp],
    "flock_op_embed": [_vp, _vp, _i32p, _i, _fp],
    "flock_op_argmax": [_vp, _fp, _i64, _i64p, _fp],
    "flock_argmax_noalloc": [_vp, _i64, _vp, _vp, _vp],
    "flock_layer_create": [_vp, _cfgp, _i, _ccp, _pp, _pp],
    "flock_layer_free": [_vp],
    "flock_layer_encode": [_vp, _fp, _i],
    "flock_layer_read_output": [_vp, _i, _fp],
    "flock_layer_reset": [_vp],
    "flock_layer_n_keys": [_vp, _ip],
    "flock_layer_rewind": [_vp, _i],
    "flock_layer_read_cache": [_vp, _fp, _fp],
    "flock_layer_write_cache": [_vp, _fp, _fp, _i],
    "flock_range_forward": [_pp, _i, _fp, _i, _i, _i, _fp],
    "flock_model_create": [_vp, _cfgp, _i, _i, _pp, _vp, _vp, _vp, _i, _pp],
    "flock_model_create_tp": [_vp, _cfgp, _i, _i, _pp, _vp, _vp, _vp, _vp, _pp],
    "flock_model_set_tp_exchange": [_vp, _i],
    "flock_model_get_tp_exchange": [_vp, _ip],
    "flock_wire_pack": [_fp, _i64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                        ctypes.c_uint32, _u8p, _i64, _i64p],
    "flock_wire_unpack": [_u8p, _i64, _fp, _i64, ctypes.POINTER(ctypes.c_uint32)],
    "flock_range_forward_wire": [_pp, _i, _u8p, _i64, _u8p, _i64, _i64p],
    "flock_gguf_open": [ctypes.c_char_p, _pp],
    "flock_gguf_free": [_vp],
    "flock_gguf_info": [_vp, _i64p, _i64p, _ip, _ip],
    "flock_gguf_tensor_info": [_vp, _i64, ctypes.c_char_p, _i, _ip, _i64p, _i64p, _i64p, _i64p],
    "flock_gguf_find": [_vp, ctypes.c_char_p, _i64p],
    "flock_gguf_meta_int": [_vp, ctypes.c_char_p, _i64p],
    "flock_gguf_meta_f64": [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)],
    "flock_gguf_meta_str": [_vp, ctypes.c_char_p, ctypes.c_char_p, _i],
    "flock_gguf_layer_ranges": [_vp, _i, _i, _i64, _i64p, _i64p, _i, _ip],
    "flock_gguf_load_tensor": [_vp, _vp, ctypes.c_char_p, _i64, _pp],
    "flock_gguf_split_host": [_vp, ctypes.c_char_p, _i64, _u8p, _u8p],
    "flock_model_free": [_vp],
    "flock_model_step": [_vp, _i32p, _i, _i32p],
    "flock_model_logits": [_vp, _i32p, _i, _fp],
    "flock_model_hidden_state": [_vp, _i32p, _i, _fp],
    "flock_model_normed_state": [_vp, _i32p, _i, _fp],
    "flock_model_embed": [_vp, _i32p, _i, _fp],
    "flock_model_encode_partial": [_vp, _i32p, _i, _i, _fp],
    "flock_model_project_hidden": [_vp, _fp, _i, _i32p],
    "flock_model_generate": [_vp, _i32p, _i, _i, _i32p, _i, _i32p, _ip],
    "flock_model_decode_device": [_vp, _i, _i32p],
    "flock_model_reset": [_vp],
    "flock_model_rewind": [_vp, _i],
    "flock_model_pos": [_vp, _ip],
    "flock_model_held": [_vp, _ip],
    "flock_model_set_token": [_vp, ctypes.c_int32],
    "flock_model_set_decode_mode": [_vp, _i],
    "flock_model_get_decode_mode": [_vp, _ip],
    "flock_model_trace": [_vp, _i],
    "flock_model_trace_read": [_vp, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int64, _ip, _ip],
    "flock_model_current_token": [_vp, _i32p],
    "flock_shard_matvec_create": [_vp, _u8p, _u8p, _i64, _i64, _i, _i, _i64, _pp],
    "flock_shard_matvec_free": [_vp],
    "flock_shard_matvec_run": [_vp, _fp, _fp],
    "flock_shard_matvec_partials": [_vp, _fp],
    "flock_shard_matvec_wire_bytes": [_vp, _i64p],
    "flock_sharded_head_create": [_vp, _u8p, _u8p, _i64, _i64, _i, _pp],
    "flock_sharded_head_free": [_vp],
    "flock_sharded_head_run": [_vp, _fp, _fp, _i32p],
    "flock_sharded_head_shard_argmax": [_vp, _fp, _i64p, _i64p],
    "flock_comm_unique_id": [_u8p],
    "flock_comm_init": [_vp, _i, _i, _u8p, _i, _pp],
    "flock_comm_free": [_vp],
    "flock_comm_send_hidden": [_vp, _vp, _i, _i],
    "flock_comm_recv_hidden": [_vp, _vp, _i, _i],
    "flock_pipeline_step": [_vp, _vp, _i32p, _i, _i, _i32p],
    "flock_model_history": [_vp, _i, _i, _i32p],
    "flock_comm_allreduce_f32": [_vp, _fp, _fp, _i64],
    "flock_comm_allgather_bytes": [_vp, _vp, _vp, _i64],
}
_RESTYPE = {"flock_last_error": ctypes.c_char_p, "flock_version": ctypes.c_char_p}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libflock_cuda.so once; raise if it is missing (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FlockError(FLOCK_E_UNSUPPORTED,
                             f"{LIB_PATH} is not built; run `python -m flock_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, ctypes.c_int)
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().flock_last_error() or b"").decode(errors="replace")


def check(rc: int) -> None:
    if rc != FLOCK_OK:
        raise FlockError(rc, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def ptr(a, ty=ctypes.c_void_p):
    """numpy array -> typed ctypes pointer (array must stay alive)."""
    return a.ctypes.data_as(ty)
