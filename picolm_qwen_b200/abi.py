"""ctypes binding of the C ABI in include/picoattn.h.

This is the reference-side binding a Python host would add: plain pointers and
sizes, no framework types.  ``lib()`` loads the in-tree ``libpicoattn.so`` and
raises if it is missing; nothing here computes anything itself.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libpicoattn.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "picoattn.h")

PICOATTN_OK = 0
PICOATTN_EINVAL = -1
PICOATTN_EUNSUPPORTED = -2
PICOATTN_ERANGE = -3
PICOATTN_ENOSPACE = -4
PICOATTN_ECUDA = -5
PICOATTN_ENCCL = -6
PICOATTN_ETIMEOUT = -7
PICOATTN_EDEVICE = -8
PICOATTN_EDEVSTATUS = -9
PICOATTN_EIO = -10
PICOATTN_EFORMAT = -11
PICOATTN_ENOENT = -12

KVCP_MAGIC = 0x4B564350

DEV_BAD_POS = 0x1
DEV_MISALIGNED = 0x2
DEV_TIMEOUT = 0x4

STAGE_PREPARE = 0x1
STAGE_ATTEND = 0x2
STAGE_COMBINE = 0x4
STAGE_ALL = 0x7

PREFILL_SINGLE = 0
PREFILL_HEAD_PAIR = 1
PREFILL_CTA_PAIR = 2

P2P_HANDLE_BYTES = 64

ROPE_NEOX = 0
ROPE_INTERLEAVED = 1
DTYPE_F32 = 0
DTYPE_F16 = 1

# projection weight formats (GGUF tensor types)
WT_F32 = 1
WT_F16 = 2
WT_Q4_0 = 3
WT_Q8_0 = 9
WT_Q4_K = 13
WT_Q6_K = 15


class Config(C.Structure):
    """picoattn_config_t."""
    _fields_ = [
        ("n_layers", C.c_int32),
        ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("max_seq_len", C.c_int32),
        ("rope_freq_base", C.c_float),
        ("rope_mode", C.c_int32),
        ("qk_norm_eps", C.c_float),
    ]

    @classmethod
    def make(cls, n_layers, n_heads, n_kv_heads, head_dim, max_seq_len, rope_freq_base,
             rope_mode=ROPE_NEOX, qk_norm_eps=1e-6):
        return cls(n_layers, n_heads, n_kv_heads, head_dim, max_seq_len, rope_freq_base,
                   rope_mode, qk_norm_eps)

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim


class LayerWeights(C.Structure):
    """picoattn_layer_weights_t: device pointers and PICOATTN_WT_* types."""
    _fields_ = [
        ("wq", C.c_void_p), ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p),
        ("wq_type", C.c_int32), ("wk_type", C.c_int32), ("wv_type", C.c_int32), ("wo_type", C.c_int32),
        ("bq", C.c_void_p), ("bk", C.c_void_p), ("bv", C.c_void_p), ("bo", C.c_void_p),
    ]


class GgufConfig(C.Structure):
    """picoattn_gguf_config_t."""
    _fields_ = [(n, C.c_int32) for n in ("n_embd", "n_ffn", "n_heads", "n_kv_heads", "n_layers", "vocab_size",
                                          "max_seq_len", "head_dim")] + [("rope_freq_base", C.c_float),
                                                                         ("alignment", C.c_int32)]


class FfnWeights(C.Structure):
    """picoattn_ffn_weights_t: device pointers and PICOATTN_WT_* types."""
    _fields_ = [
        ("w_gate", C.c_void_p), ("w_up", C.c_void_p), ("w_down", C.c_void_p),
        ("gate_type", C.c_int32), ("up_type", C.c_int32), ("down_type", C.c_int32),
        ("b_gate", C.c_void_p), ("b_down", C.c_void_p),
    ]


_P = C.c_void_p
_I = C.c_int32
_Z = C.c_size_t
_CFG = C.POINTER(Config)

# name -> (restype, argtypes); every function declared in include/picoattn.h
PROTOTYPES = {
    "picoattn_version": (_I, []),
    "picoattn_strerror": (C.c_char_p, [_I]),
    "picoattn_last_cuda_error": (C.c_char_p, []),
    "picoattn_config_check": (_I, [_CFG]),
    "picoattn_rope_table": (_I, [_CFG, _P, _P]),
    "picoattn_device_check": (_I, []),
    "picoattn_workspace_init": (_I, [_P, _Z, _P]),
    "picoattn_workspace_status": (_I, [_P, _P, C.POINTER(C.c_uint32)]),
    "picoattn_decode_workspace_size": (_Z, [_CFG, _I, _I]),
    "picoattn_decode": (_I, [_CFG, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _Z, _P]),
    "picoattn_decode_staged": (_I, [_CFG, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _Z, _P,
                                   C.c_uint32]),
    "picoattn_decode_one": (_I, [_CFG, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _Z, _P]),
    "picoattn_decode_noalloc": (_I, [_CFG, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                    C.POINTER(C.c_uint32)]),
    "picoattn_shard_partial_bytes": (_Z, [_CFG, _I]),
    "picoattn_decode_shard": (_I, [_CFG, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _Z,
                                  _P]),
    "picoattn_combine_shards": (_I, [_CFG, _I, _I, _P, _P, _P]),
    "picoattn_nccl_unique_id": (_I, [_P]),
    "picoattn_nccl_comm_create": (_I, [_I, _P, _I, C.c_double, C.POINTER(C.c_void_p)]),
    "picoattn_nccl_comm_destroy": (_I, [_P]),
    "picoattn_splitkv_gather_bytes": (_Z, [_CFG, _I, _I]),
    "picoattn_decode_splitkv_nccl": (_I, [_CFG, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                         _P, _Z, _P, _P]),
    "picoattn_prefill_workspace_size": (_Z, [_CFG, _I]),
    "picoattn_prefill_kernel": (_I, [_CFG]),
    "picoattn_p2p_area_bytes": (_Z, [_CFG, _I, _I]),
    "picoattn_p2p_create": (_I, [_CFG, _I, _I, _I, _P, _P]),
    "picoattn_p2p_open": (_I, [_P, _P]),
    "picoattn_p2p_destroy": (_I, [_P]),
    "picoattn_p2p_set_timeout": (_I, [_P, C.c_double]),
    "picoattn_decode_splitkv_p2p": (_I, [_CFG, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                         _P, _Z, _P, _P]),
    "picoattn_prefill": (_I, [_CFG, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _Z, _P]),
    "picoattn_prefill_staged": (_I, [_CFG, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _Z, _P,
                                     C.c_uint32]),
    "picoattn_kvcp_bytes": (_Z, [_CFG, _I]),
    "picoattn_kvcp_save": (_I, [_CFG, _I, _P, _P, C.c_char_p, _P]),
    "picoattn_kvcp_load": (_I, [_CFG, C.c_char_p, _P, _P, C.POINTER(C.c_int32), _P]),
    "picoattn_kvcp_pack": (_I, [_CFG, _I, _P, _P, _P, _Z, _P]),
    "picoattn_kvcp_unpack": (_I, [_CFG, _P, _Z, _P, _P, C.POINTER(C.c_int32), _P]),
    "picoattn_weight_bytes": (_Z, [_I, _I, _I]),
    "picoattn_matvec": (_I, [_P, _I, _P, _I, _I, _I, _P, _P, _I, _P]),
    "picoattn_decode_layer_workspace_size": (_Z, [_CFG, _I, _I, _I]),
    "picoattn_decode_layer": (_I, [_CFG, _I, _I, _I, _I, _P, C.POINTER(LayerWeights), _P, _P, _P, _P, _P, _P, _P,
                                   _P, _P, _Z, _P]),
    "picoattn_rmsnorm": (_I, [_P, _P, _P, _I, _I, _P]),
    "picoattn_gguf_open": (_I, [C.c_char_p, _I, C.POINTER(C.c_void_p)]),
    "picoattn_gguf_close": (_I, [_P]),
    "picoattn_gguf_get_config": (_I, [_P, C.POINTER(GgufConfig)]),
    "picoattn_gguf_find": (_I, [_P, _I, C.c_char_p, C.POINTER(C.c_int32), C.POINTER(C.c_size_t),
                                C.POINTER(C.c_size_t)]),
    "picoattn_gguf_arena_bytes": (_Z, [_P]),
    "picoattn_gguf_upload": (_I, [_P, _P, _Z, _P]),
    "picoattn_gguf_arena_tensor": (_I, [_P, _P, _I, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_int32)]),
    "picoattn_ffn_workspace_size": (_Z, [_I, _I, _I]),
    "picoattn_ffn": (_I, [C.POINTER(FfnWeights), _P, _I, _I, _I, _P, _P, _Z, _P]),
    "picoattn_logits_workspace_size": (_Z, [_I, _I]),
    "picoattn_logits": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _P, _Z, _P]),
    "picoattn_decode_block_workspace_size": (_Z, [_CFG, _I, _I, _I, _I]),
    "picoattn_decode_block": (_I, [_CFG, _I, _I, _I, _I, _I, _P, C.POINTER(LayerWeights), _P, C.POINTER(FfnWeights),
                                   _P, _P, _P, _P, _P, _P, _P, _P, _P, _Z, _P]),
}

_lib = None


class PicoAttnError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        msg = lib().picoattn_strerror(status).decode()
        if status == PICOATTN_ECUDA:
            msg += " (" + lib().picoattn_last_cuda_error().decode() + ")"
        super().__init__(f"{what}: {msg} ({status})" if what else f"{msg} ({status})")
        self.status = status


def lib() -> C.CDLL:
    """The loaded libpicoattn.so.  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python -m picolm_qwen_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str = "") -> None:
    if status != PICOATTN_OK:
        raise PicoAttnError(status, what)


def declared_functions() -> list[str]:
    """Function names declared in include/picoattn.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(picoattn_[a-z0-9_]+)\s*\(",
                                 text, re.M)))


def ptr(t) -> int | None:
    """Device/host address of a torch tensor (or None)."""
    return None if t is None else t.data_ptr()
