"""TEST INFRASTRUCTURE ONLY: numpy wrappers over the CPU oracle libraries.

* ``Oracle`` wraps ``oracle/_build/libpicooracle.so``, the plain-C restatement
  of the reference's attention step (``oracle/attn_oracle.c``).
* ``RefHarness`` wraps ``oracle/_ref/libpicoref.so``, the reference's own
  sources (cpp/model.hpp, cpp/tensor.hpp, cpp/quant.hpp, picolm/tensor.c)
  compiled in place and driven by ``oracle/ref_harness.cpp``.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module; the product path never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libpicooracle.so")
REF_SO = os.path.join(HERE, "_ref", "libpicoref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def build(ref: bool = False) -> None:
    """Build the oracle (and, when asked and the reference tree exists, _ref)."""
    targets = ["oracle"]
    if ref:
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def _opt(a):
    return None if a is None else np.ascontiguousarray(a, np.float32).ctypes.data_as(C.c_void_p)


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.ora_f32_to_f16.restype = C.c_uint16
        L.ora_f32_to_f16.argtypes = [C.c_float]
        L.ora_f16_to_f32.restype = C.c_float
        L.ora_f16_to_f32.argtypes = [C.c_uint16]
        L.ora_f32_to_f16_n.argtypes = [_f32p, _u16p, C.c_size_t]
        L.ora_f16_to_f32_n.argtypes = [_u16p, _f32p, C.c_size_t]
        L.ora_rmsnorm_inplace.argtypes = [_f32p, _f32p, C.c_int, C.c_float]
        for n in ("ora_rope_neox", "ora_rope_interleaved"):
            getattr(L, n).argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
        L.ora_rope_table.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_float]
        L.ora_decode_step.restype = C.c_int
        L.ora_decode_step.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                      _f32p, _f32p, _f32p, C.c_void_p, C.c_void_p,
                                      _f32p, _f32p, _u16p, _u16p, C.c_int, _f32p, C.c_int]
        L.ora_decode_step_mt.restype = C.c_int
        L.ora_decode_step_mt.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                         _f32p, _f32p, _f32p, C.c_void_p, C.c_void_p,
                                         _f32p, _f32p, _u16p, _u16p, C.c_int, _f32p, C.c_int]
        L.ora_attend_rows.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, _u16p, _u16p,
                                      C.c_int, C.c_int, _f32p, _f32p, _f32p]
        L.ora_prefill.restype = C.c_int
        L.ora_prefill.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                  _f32p, _f32p, _f32p, C.c_void_p, C.c_void_p,
                                  _f32p, _f32p, _u16p, _u16p, C.c_int, C.c_int, _f32p, C.c_int]
        L.ora_decode_batch.restype = C.c_int
        L.ora_decode_batch.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                       _f32p, _f32p, _f32p, C.c_void_p, C.c_void_p,
                                       _f32p, _f32p, C.c_void_p, C.c_void_p, _i32p, _f32p, C.c_int]
        L.ora_weight_block.restype = C.c_int
        L.ora_weight_block.argtypes = [C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.ora_dequant_row.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_int]
        L.ora_vec_dot.restype = C.c_float
        L.ora_vec_dot.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_int]
        L.ora_matvec.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, _f32p, _f32p,
                                 C.c_int]
        self.L = L

    def weight_block(self, wtype: int):
        """(weights per block, bytes per block) of a GGUF type, or None."""
        e, b = C.c_int(), C.c_int()
        return (e.value, b.value) if self.L.ora_weight_block(wtype, C.byref(e), C.byref(b)) else None

    def dequant(self, w: np.ndarray, wtype: int, n_in: int, n_out: int) -> np.ndarray:
        """All n_out rows of a weight matrix (uint8 bytes) as fp32 [n_out, n_in]."""
        e, b = self.weight_block(wtype)
        row = n_in // e * b
        w = np.ascontiguousarray(w, np.uint8).ravel()
        out = np.empty((n_out, n_in), np.float32)
        for d in range(n_out):
            buf = np.empty(n_in, np.float32)
            self.L.ora_dequant_row(w[d * row:(d + 1) * row].ctypes.data, buf, n_in, wtype)
            out[d] = buf
        return out

    def matvec(self, w, wtype, bias, n_in, n_out, x, out=None, accumulate=False):
        """out[v, d] = W[d] . x[v] (+ bias[d]) (+ out[v, d]) in the reference's order."""
        w = np.ascontiguousarray(w, np.uint8).ravel()
        x = np.ascontiguousarray(x, np.float32).reshape(-1, n_in)
        res = np.zeros((x.shape[0], n_out), np.float32) if out is None else np.ascontiguousarray(out, np.float32).copy()
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.L.ora_matvec(w.ctypes.data, wtype, None if b is None else b.ctypes.data, n_in, n_out, x.shape[0],
                          x, res, 1 if accumulate else 0)
        return res

    def f32_to_f16(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty(x.size, np.uint16)
        self.L.ora_f32_to_f16_n(x, out, x.size)
        return out

    def f16_to_f32(self, h: np.ndarray) -> np.ndarray:
        h = np.ascontiguousarray(h, np.uint16).ravel()
        out = np.empty(h.size, np.float32)
        self.L.ora_f16_to_f32_n(h, out, h.size)
        return out

    def rmsnorm(self, x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
        x = np.array(x, np.float32)
        self.L.ora_rmsnorm_inplace(x, np.ascontiguousarray(w, np.float32), x.size, eps)
        return x

    def rope(self, mode: int, q, k, hd, hq, hkv, c, s):
        q = np.array(q, np.float32)
        k = np.array(k, np.float32)
        fn = self.L.ora_rope_neox if mode == 0 else self.L.ora_rope_interleaved
        fn(q, k, hd, hq, hkv, np.ascontiguousarray(c, np.float32), np.ascontiguousarray(s, np.float32))
        return q, k

    def rope_table(self, max_seq: int, hd: int, base: float):
        c = np.empty((max_seq, hd // 2), np.float32)
        s = np.empty((max_seq, hd // 2), np.float32)
        self.L.ora_rope_table(c, s, max_seq, hd, base)
        return c, s

    def decode_step(self, hq, hkv, hd, rope_mode, q, k, v, qn_w, kn_w, cos_t, sin_t,
                    kc, vc, pos, variant=0, eps=1e-6):
        """kc/vc: this layer's slabs [S][kvd] uint16, row pos written in place."""
        q = np.array(q, np.float32)
        k = np.array(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        out = np.empty(hq * hd, np.float32)
        half = hd // 2
        c = np.ascontiguousarray(cos_t[pos], np.float32).reshape(half)
        s = np.ascontiguousarray(sin_t[pos], np.float32).reshape(half)
        qn = None if qn_w is None else np.ascontiguousarray(qn_w, np.float32)
        kn = None if kn_w is None else np.ascontiguousarray(kn_w, np.float32)
        rc = self.L.ora_decode_step(hq, hkv, hd, rope_mode, eps, q, k, v, _opt(qn), _opt(kn),
                                    c, s, kc, vc, pos, out, variant)
        assert rc == 0
        return out, q, k

    def decode_step_mt(self, hq, hkv, hd, rope_mode, q, k, v, qn_w, kn_w, cos_t, sin_t,
                       kc, vc, pos, n_threads, eps=1e-6):
        """decode_step (C++ engine order) with the q heads spread over host threads."""
        q = np.array(q, np.float32)
        k = np.array(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        out = np.empty(hq * hd, np.float32)
        half = hd // 2
        c = np.ascontiguousarray(cos_t[pos], np.float32).reshape(half)
        s = np.ascontiguousarray(sin_t[pos], np.float32).reshape(half)
        qn = None if qn_w is None else np.ascontiguousarray(qn_w, np.float32)
        kn = None if kn_w is None else np.ascontiguousarray(kn_w, np.float32)
        rc = self.L.ora_decode_step_mt(hq, hkv, hd, rope_mode, eps, q, k, v, _opt(qn), _opt(kn),
                                       c, s, kc, vc, pos, out, n_threads)
        assert rc == 0
        return out

    def attend_rows(self, hq, hkv, hd, q_rot, kc, vc, b, e):
        m = np.empty(hq, np.float32)
        l = np.empty(hq, np.float32)
        acc = np.empty(hq * hd, np.float32)
        self.L.ora_attend_rows(hq, hkv, hd, np.ascontiguousarray(q_rot, np.float32), kc, vc,
                               b, e, m, l, acc)
        return m, l, acc

    def prefill(self, hq, hkv, hd, rope_mode, q, k, v, qn_w, kn_w, cos_t, sin_t, kc, vc,
                start_pos, n_threads=1, eps=1e-6):
        n_tok = q.shape[0]
        out = np.empty((n_tok, hq * hd), np.float32)
        qn = None if qn_w is None else np.ascontiguousarray(qn_w, np.float32)
        kn = None if kn_w is None else np.ascontiguousarray(kn_w, np.float32)
        rc = self.L.ora_prefill(hq, hkv, hd, rope_mode, eps,
                                np.ascontiguousarray(q, np.float32),
                                np.ascontiguousarray(k, np.float32),
                                np.ascontiguousarray(v, np.float32), _opt(qn), _opt(kn),
                                np.ascontiguousarray(cos_t, np.float32),
                                np.ascontiguousarray(sin_t, np.float32),
                                kc, vc, start_pos, n_tok, out, n_threads)
        assert rc == 0
        return out

    def decode_batch(self, hq, hkv, hd, rope_mode, q, k, v, qn_w, kn_w, cos_t, sin_t,
                     kcs, vcs, pos, n_threads=1, eps=1e-6):
        """kcs/vcs: lists of per-sequence layer slabs [S][kvd] uint16 (modified)."""
        B = len(kcs)
        out = np.empty((B, hq * hd), np.float32)
        kp = (C.c_void_p * B)(*[a.ctypes.data for a in kcs])
        vp = (C.c_void_p * B)(*[a.ctypes.data for a in vcs])
        qn = None if qn_w is None else np.ascontiguousarray(qn_w, np.float32)
        kn = None if kn_w is None else np.ascontiguousarray(kn_w, np.float32)
        rc = self.L.ora_decode_batch(B, hq, hkv, hd, rope_mode, eps,
                                     np.ascontiguousarray(q, np.float32),
                                     np.ascontiguousarray(k, np.float32),
                                     np.ascontiguousarray(v, np.float32), _opt(qn), _opt(kn),
                                     np.ascontiguousarray(cos_t, np.float32),
                                     np.ascontiguousarray(sin_t, np.float32),
                                     C.cast(kp, C.c_void_p), C.cast(vp, C.c_void_p),
                                     np.ascontiguousarray(pos, np.int32), out, n_threads)
        assert rc == 0
        return out


class RefHarness:
    """The reference's own code, compiled from its sources (oracle/_ref)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (make -C oracle ref)")
        L = C.CDLL(path)
        L.pref_model_create.restype = C.c_void_p
        L.pref_model_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int]
        L.pref_model_destroy.argtypes = [C.c_void_p]
        for n in ("pref_model_kcache", "pref_model_vcache"):
            getattr(L, n).restype = C.POINTER(C.c_uint16)
            getattr(L, n).argtypes = [C.c_void_p]
        for n in ("pref_model_rope_cos", "pref_model_rope_sin"):
            getattr(L, n).restype = C.POINTER(C.c_float)
            getattr(L, n).argtypes = [C.c_void_p]
        L.pref_model_set_norm.argtypes = [C.c_void_p, _f32p, _f32p]
        L.pref_model_decode.restype = C.c_int
        L.pref_model_decode.argtypes = [C.c_void_p, _f32p, _f32p, _f32p, C.c_int, _f32p]
        L.pref_fp32_to_fp16.restype = C.c_uint16
        L.pref_fp32_to_fp16.argtypes = [C.c_float]
        L.pref_fp16_to_fp32.restype = C.c_float
        L.pref_fp16_to_fp32.argtypes = [C.c_uint16]
        L.pref_fp32_to_fp16_n.argtypes = [_f32p, _u16p, C.c_size_t]
        L.pref_fp16_to_fp32_n.argtypes = [_u16p, _f32p, C.c_size_t]
        L.pref_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int]
        L.pref_rope.argtypes = [C.c_int, _f32p, _f32p, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
        L.pref_attn_decode_batch.restype = C.c_int
        L.pref_attn_decode_batch.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                             _f32p, _f32p, _f32p, C.c_void_p, C.c_void_p,
                                             _f32p, _f32p, C.c_void_p, C.c_void_p, _i32p, _f32p,
                                             C.c_int]
        for n in ("pref_kvcp_save", "pref_kvcp_load"):
            getattr(L, n).restype = C.c_int
        L.pref_kvcp_save.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _u16p, _u16p, C.c_char_p, C.c_int]
        L.pref_kvcp_load.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _u16p, _u16p, C.c_char_p]
        L.pref_dequant_row.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_int]
        L.pref_matvec.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
        self.L = L

    def dequant_row(self, row: np.ndarray, wtype: int, n: int) -> np.ndarray:
        """The reference's dequantize_row (cpp/quant.hpp:283-295) of one row."""
        row = np.ascontiguousarray(row, np.uint8)
        out = np.empty(n, np.float32)
        self.L.pref_dequant_row(row.ctypes.data, out, n, wtype)
        return out

    def matvec(self, w, wtype, bias, n_in, n_out, x):
        """The reference's TensorOps::matmul_bias (cpp/tensor.hpp:110-143) per vector:
        [n_vec, n_out]."""
        w = np.ascontiguousarray(w, np.uint8).ravel()
        x = np.ascontiguousarray(x, np.float32).reshape(-1, n_in)
        out = np.empty((x.shape[0], n_out), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.L.pref_matvec(w.ctypes.data, wtype, None if b is None else b.ctypes.data, n_in, n_out, x.shape[0],
                           x, out)
        return out

    def kvcp_save(self, kc, vc, n_kv_heads, head_dim, path, n_pos):
        """The C engine's kvcache_save (picolm/model.c:884-926) of caches kc, vc
        ([n_layers][max_seq][kv_dim] uint16); returns its status (0 or -1)."""
        kc = np.ascontiguousarray(kc, np.uint16)
        vc = np.ascontiguousarray(vc, np.uint16)
        L, S, _ = kc.shape
        return self.L.pref_kvcp_save(L, n_kv_heads, head_dim, S, kc, vc, path.encode(), n_pos)

    def kvcp_load(self, kc, vc, n_kv_heads, head_dim, path):
        """The C engine's kvcache_load (picolm/model.c:928-983) into kc, vc (filled
        in place, C-contiguous uint16 arrays); returns the positions loaded (0: none)."""
        L, S, _ = kc.shape
        assert kc.flags.c_contiguous and vc.flags.c_contiguous and kc.dtype == np.uint16
        return self.L.pref_kvcp_load(L, n_kv_heads, head_dim, S, kc, vc, path.encode())

    def f32_to_f16(self, x):
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty(x.size, np.uint16)
        self.L.pref_fp32_to_fp16_n(x, out, x.size)
        return out

    def f16_to_f32(self, h):
        h = np.ascontiguousarray(h, np.uint16).ravel()
        out = np.empty(h.size, np.float32)
        self.L.pref_fp16_to_fp32_n(h, out, h.size)
        return out

    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.L.pref_rmsnorm(out, x, np.ascontiguousarray(w, np.float32), x.size)
        return out

    def rope(self, mode, q, k, hd, hq, hkv, c, s):
        q = np.array(q, np.float32)
        k = np.array(k, np.float32)
        self.L.pref_rope(mode, q, k, hd, hq, hkv, np.ascontiguousarray(c, np.float32),
                         np.ascontiguousarray(s, np.float32))
        return q, k

    def attn_decode_batch(self, hq, hkv, hd, rope_mode, q, k, v, qn_w, kn_w, cos_t, sin_t,
                          kcs, vcs, pos, n_threads=1):
        B = len(kcs)
        out = np.empty((B, hq * hd), np.float32)
        kp = (C.c_void_p * B)(*[a.ctypes.data for a in kcs])
        vp = (C.c_void_p * B)(*[a.ctypes.data for a in vcs])
        qn = None if qn_w is None else np.ascontiguousarray(qn_w, np.float32)
        kn = None if kn_w is None else np.ascontiguousarray(kn_w, np.float32)
        rc = self.L.pref_attn_decode_batch(B, hq, hkv, hd, rope_mode,
                                           np.ascontiguousarray(q, np.float32),
                                           np.ascontiguousarray(k, np.float32),
                                           np.ascontiguousarray(v, np.float32), _opt(qn), _opt(kn),
                                           np.ascontiguousarray(cos_t, np.float32),
                                           np.ascontiguousarray(sin_t, np.float32),
                                           C.cast(kp, C.c_void_p), C.cast(vp, C.c_void_p),
                                           np.ascontiguousarray(pos, np.int32), out, n_threads)
        assert rc == 0
        return out


class RefModel:
    """One-layer synthetic reference Model driven through Model::forward."""

    def __init__(self, ref: RefHarness, hq, hkv, hd, max_seq, rope_base, rope_mode, qk_norm):
        self.ref, self.L = ref, ref.L
        self.hq, self.hkv, self.hd, self.S = hq, hkv, hd, max_seq
        self.h = self.L.pref_model_create(hq, hkv, hd, max_seq, rope_base, rope_mode, int(qk_norm))
        if not self.h:
            raise RuntimeError("pref_model_create failed")
        kvd = hkv * hd
        self.kcache = np.ctypeslib.as_array(self.L.pref_model_kcache(self.h), shape=(max_seq, kvd))
        self.vcache = np.ctypeslib.as_array(self.L.pref_model_vcache(self.h), shape=(max_seq, kvd))
        self.rope_cos = np.ctypeslib.as_array(self.L.pref_model_rope_cos(self.h), shape=(max_seq, hd // 2))
        self.rope_sin = np.ctypeslib.as_array(self.L.pref_model_rope_sin(self.h), shape=(max_seq, hd // 2))

    def set_norm(self, qn_w, kn_w):
        self.L.pref_model_set_norm(self.h, np.ascontiguousarray(qn_w, np.float32),
                                   np.ascontiguousarray(kn_w, np.float32))

    def decode(self, q, k, v, pos):
        out = np.empty(self.hq * self.hd, np.float32)
        rc = self.L.pref_model_decode(self.h, np.ascontiguousarray(q, np.float32),
                                      np.ascontiguousarray(k, np.float32),
                                      np.ascontiguousarray(v, np.float32), pos, out)
        assert rc == 0
        return out

    def close(self):
        if self.h:
            self.L.pref_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RefGguf:
    """A GGUF file loaded by the engine's own Model::load (test only)."""

    def __init__(self, ref: RefHarness, path: str, max_seq_override: int = 0, rope_mode: int = 0):
        L = ref.L
        if not hasattr(L, "_gguf_proto"):
            L.pref_gguf_load.restype = C.c_void_p
            L.pref_gguf_load.argtypes = [C.c_char_p, C.c_int, C.c_int]
            L.pref_gguf_free.argtypes = [C.c_void_p]
            L.pref_gguf_config.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_float)]
            L.pref_gguf_tensor.restype = C.c_longlong
            L.pref_gguf_tensor.argtypes = [C.c_void_p, C.c_int, C.c_char_p, C.POINTER(C.c_int)]
            L.pref_gguf_forward.restype = C.c_int
            L.pref_gguf_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p]
            L._gguf_proto = True
        self.L = L
        self.h = L.pref_gguf_load(path.encode(), max_seq_override, rope_mode)

    @property
    def loaded(self) -> bool:
        return bool(self.h)

    def config(self) -> dict:
        ints = (C.c_int * 9)()
        rb = C.c_float()
        self.L.pref_gguf_config(self.h, ints, C.byref(rb))
        names = ("n_embd", "n_ffn", "n_heads", "n_kv_heads", "n_layers", "vocab_size", "max_seq_len", "head_dim",
                 "alignment")
        d = dict(zip(names, list(ints)))
        d["rope_freq_base"] = rb.value
        return d

    def tensor(self, layer: int, key: str):
        """(file offset, engine type) or None."""
        t = C.c_int()
        off = self.L.pref_gguf_tensor(self.h, layer, key.encode(), C.byref(t))
        return None if off < 0 else (off, t.value)

    def forward(self, token: int, pos: int, vocab: int) -> np.ndarray:
        out = np.empty(vocab, np.float32)
        assert self.L.pref_gguf_forward(self.h, token, pos, out) == 0
        return out

    def close(self):
        if self.h:
            self.L.pref_gguf_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RefFullModel:
    """Multi-layer reference Model with seeded random F32 weights (test only).

    forward / forward_batch run the unmodified engine (cpp/model.hpp:288-636);
    embed / pre_attn / post_attn / logits are its non-attention stages with the
    reference's own functions, for a host loop whose attention block is swapped
    for another implementation (the CPU loop here, or the GPU library)."""

    def __init__(self, ref: RefHarness, n_layers, hq, hkv, hd, n_ffn, vocab, max_seq, rope_base,
                 rope_mode, qk_norm, seed=0):
        L = ref.L
        if not hasattr(L, "_full_proto"):
            L.pref_full_create.restype = C.c_void_p
            L.pref_full_create.argtypes = [C.c_int] * 7 + [C.c_float, C.c_int, C.c_int, C.c_uint64]
            L.pref_full_destroy.argtypes = [C.c_void_p]
            L.pref_full_forward.restype = C.c_int
            L.pref_full_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p]
            L.pref_full_forward_batch.restype = C.c_int
            L.pref_full_forward_batch.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, _f32p]
            L.pref_full_embed.argtypes = [C.c_void_p, C.c_int, _f32p]
            L.pref_full_pre_attn.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p, _f32p, _f32p]
            L.pref_full_post_attn.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
            L.pref_full_logits.argtypes = [C.c_void_p, _f32p, _f32p]
            L.pref_full_norm_w.restype = C.POINTER(C.c_float)
            L.pref_full_norm_w.argtypes = [C.c_void_p, C.c_int, C.c_int]
            for n in ("pref_full_rope_cos", "pref_full_rope_sin"):
                getattr(L, n).restype = C.POINTER(C.c_float)
                getattr(L, n).argtypes = [C.c_void_p]
            L.pref_full_set_attn_weights.restype = C.c_int
            L.pref_full_set_attn_weights.argtypes = [C.c_void_p, C.c_int, C.c_uint64]
            L.pref_full_attn_norm.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
            L.pref_full_attn_weight.restype = C.c_void_p
            L.pref_full_attn_weight.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int),
                                                C.POINTER(C.c_size_t)]
            L.pref_full_attn_bias.restype = C.POINTER(C.c_float)
            L.pref_full_attn_bias.argtypes = [C.c_void_p, C.c_int, C.c_int]
            L.pref_full_ffn.argtypes = [C.c_void_p, C.c_int, _f32p]
            L.pref_full_model_norm.restype = C.POINTER(C.c_float)
            L.pref_full_model_norm.argtypes = [C.c_void_p, C.c_int, C.c_int]
            L.pref_full_ffn_weight.restype = C.c_void_p
            L.pref_full_ffn_weight.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int),
                                               C.POINTER(C.c_size_t)]
            L.pref_full_ffn_bias.restype = C.POINTER(C.c_float)
            L.pref_full_ffn_bias.argtypes = [C.c_void_p, C.c_int, C.c_int]
            L.pref_full_set_ffn_weights.restype = C.c_int
            L.pref_full_set_ffn_weights.argtypes = [C.c_void_p, C.c_int, C.c_uint64]
            L._full_proto = True
        self.ref, self.L = ref, L
        self.nl, self.hq, self.hkv, self.hd, self.vocab, self.S = n_layers, hq, hkv, hd, vocab, max_seq
        self.n_ffn = n_ffn
        self.dim, self.kvd = hq * hd, hkv * hd
        self.qk_norm = bool(qk_norm)
        self.h = L.pref_full_create(n_layers, hq, hkv, hd, n_ffn, vocab, max_seq, rope_base, rope_mode,
                                    int(qk_norm), seed)
        if not self.h:
            raise RuntimeError("pref_full_create failed")
        self.rope_cos = np.ctypeslib.as_array(L.pref_full_rope_cos(self.h), shape=(max_seq, hd // 2)).copy()
        self.rope_sin = np.ctypeslib.as_array(L.pref_full_rope_sin(self.h), shape=(max_seq, hd // 2)).copy()

    def forward(self, token, pos):
        out = np.empty(self.vocab, np.float32)
        assert self.L.pref_full_forward(self.h, int(token), int(pos), out) == 0
        return out

    def forward_batch(self, tokens, start_pos):
        out = np.empty(self.vocab, np.float32)
        t = np.ascontiguousarray(tokens, np.int32)
        assert self.L.pref_full_forward_batch(self.h, t, t.size, int(start_pos), out) == 0
        return out

    def embed(self, token):
        x = np.empty(self.dim, np.float32)
        self.L.pref_full_embed(self.h, int(token), x)
        return x

    def pre_attn(self, layer, x):
        q = np.empty(self.dim, np.float32)
        k = np.empty(self.kvd, np.float32)
        v = np.empty(self.kvd, np.float32)
        self.L.pref_full_pre_attn(self.h, layer, np.ascontiguousarray(x, np.float32), q, k, v)
        return q, k, v

    def post_attn(self, layer, x, attn):
        x = np.array(x, np.float32)
        self.L.pref_full_post_attn(self.h, layer, x, np.ascontiguousarray(attn, np.float32))
        return x

    def logits(self, x):
        out = np.empty(self.vocab, np.float32)
        self.L.pref_full_logits(self.h, np.ascontiguousarray(x, np.float32), out)
        return out

    def norm_w(self, layer, which):
        if not self.qk_norm:
            return None
        return np.ctypeslib.as_array(self.L.pref_full_norm_w(self.h, layer, which), shape=(self.hd,)).copy()

    def model_norm(self, layer, which):
        """fp32 [dim]: which 0 attention norm, 1 FFN norm of layer; 2 the output norm."""
        return np.ctypeslib.as_array(self.L.pref_full_model_norm(self.h, layer, which), shape=(self.dim,)).copy()

    def ffn_weight(self, layer, which):
        """(bytes as uint8, GGUF type): which 0 gate, 1 up, 2 down of layer; 3 the output matrix."""
        t, n = C.c_int(), C.c_size_t()
        p = self.L.pref_full_ffn_weight(self.h, layer, which, C.byref(t), C.byref(n))
        return np.ctypeslib.as_array((C.c_uint8 * n.value).from_address(p)).copy(), t.value

    def ffn_bias(self, layer, which):
        """fp32 bias the engine keeps: which 0 gate [n_ffn], 1 down [dim]."""
        n = self.n_ffn if which == 0 else self.dim
        return np.ctypeslib.as_array(self.L.pref_full_ffn_bias(self.h, layer, which), shape=(n,)).copy()

    def set_ffn_weights(self, wtype: int, seed: int = 2) -> None:
        """Every layer's gate/up/down and the output matrix as seeded random blocks of a GGUF type."""
        assert self.L.pref_full_set_ffn_weights(self.h, int(wtype), seed) == 0

    def set_attn_weights(self, wtype: int, seed: int = 1) -> None:
        """Every layer's q/k/v/o weights as seeded random blocks of a GGUF type."""
        assert self.L.pref_full_set_attn_weights(self.h, int(wtype), seed) == 0

    def attn_norm(self, layer, x):
        xb = np.empty(self.dim, np.float32)
        self.L.pref_full_attn_norm(self.h, layer, np.ascontiguousarray(x, np.float32), xb)
        return xb

    def attn_weight(self, layer, which):
        """(bytes as uint8, GGUF type) of projection which: 0 q, 1 k, 2 v, 3 o."""
        t, n = C.c_int(), C.c_size_t()
        p = self.L.pref_full_attn_weight(self.h, layer, which, C.byref(t), C.byref(n))
        return np.ctypeslib.as_array((C.c_uint8 * n.value).from_address(p)).copy(), t.value

    def attn_bias(self, layer, which):
        n = self.kvd if which in (1, 2) else self.dim
        return np.ctypeslib.as_array(self.L.pref_full_attn_bias(self.h, layer, which), shape=(n,)).copy()

    def ffn(self, layer, x):
        x = np.ascontiguousarray(x, np.float32).copy()
        self.L.pref_full_ffn(self.h, layer, x)
        return x

    def close(self):
        if self.h:
            self.L.pref_full_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
