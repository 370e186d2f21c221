"""Device-side attention state: the B200 counterpart of the reference's RunState
attention buffers (key_cache/val_cache, rope_cos/rope_sin, cpp/model.hpp:158-174,
allocated in cpp/model.hpp:1003-1017), plus the call that replaces the inline
attention block of Model::forward (cpp/model.hpp:326-418).

PyTorch is used only to own device memory and streams; every computation is a
call into libpicoattn.so through the C ABI.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import abi


def rope_table(cfg: abi.Config) -> tuple[np.ndarray, np.ndarray]:
    """Host RoPE table built by the library exactly as the reference builds it."""
    half = cfg.head_dim // 2
    cos = np.empty((cfg.max_seq_len, half), np.float32)
    sin = np.empty((cfg.max_seq_len, half), np.float32)
    abi.check(abi.lib().picoattn_rope_table(C.byref(cfg), cos.ctypes.data, sin.ctypes.data), "rope_table")
    return cos, sin


def stream_handle(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def matvec(w: torch.Tensor, w_type: int, n_in: int, n_out: int, x: torch.Tensor, out: torch.Tensor,
           bias: torch.Tensor | None = None, accumulate: bool = False,
           stream: torch.cuda.Stream | None = None) -> None:
    """out[v] (=|+=) W . x[v] (+ bias) on the device (TensorOps::matmul_bias,
    cpp/tensor.hpp:110-143); w holds the GGUF blocks as uint8."""
    n_vec = x.numel() // n_in
    st = abi.lib().picoattn_matvec(w.data_ptr(), w_type, abi.ptr(bias), n_in, n_out, n_vec, x.data_ptr(),
                                   out.data_ptr(), 1 if accumulate else 0, stream_handle(stream))
    abi.check(st, "picoattn_matvec")


class LayerProj:
    """One layer's q/k/v/o weights on the device (uint8 GGUF blocks) and fp32 biases."""

    def __init__(self, wq, wk, wv, wo, types, bq=None, bk=None, bv=None, bo=None):
        self.tensors = (wq, wk, wv, wo, bq, bk, bv, bo)  # kept alive with the struct
        self.struct = abi.LayerWeights(
            wq.data_ptr(), wk.data_ptr(), wv.data_ptr(), wo.data_ptr(), *types,
            abi.ptr(bq), abi.ptr(bk), abi.ptr(bv), abi.ptr(bo))


class FfnProj:
    """One layer's FFN weights on the device (uint8 GGUF blocks) and fp32 biases."""

    def __init__(self, w_gate, w_up, w_down, types, b_gate=None, b_down=None):
        self.tensors = (w_gate, w_up, w_down, b_gate, b_down)  # kept alive with the struct
        self.struct = abi.FfnWeights(w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(), *types,
                                     abi.ptr(b_gate), abi.ptr(b_down))


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor, stream: torch.cuda.Stream | None = None):
    """out = rmsnorm(x) * weight per row of x [n_vec, dim] (TensorOps::rmsnorm, cpp/tensor.hpp:146-176)."""
    dim = weight.numel()
    abi.check(abi.lib().picoattn_rmsnorm(x.data_ptr(), weight.data_ptr(), out.data_ptr(), dim, x.numel() // dim,
                                         stream_handle(stream)), "picoattn_rmsnorm")


class Scratch:
    """A grow-only device byte buffer for the calls that take a workspace."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.buf = None

    def get(self, n: int) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < n:
            self.buf = torch.zeros(max(n, 256), dtype=torch.uint8, device=self.device)
        return self.buf


def ffn(proj: "FfnProj", ffn_norm_w: torch.Tensor, n_ffn: int, x: torch.Tensor, scratch: "Scratch",
        stream: torch.cuda.Stream | None = None) -> None:
    """The FFN block and its residual in place on x [n_vec, dim] (cpp/model.hpp:429-452)."""
    dim = ffn_norm_w.numel()
    n_vec = x.numel() // dim
    n = abi.lib().picoattn_ffn_workspace_size(dim, n_ffn, n_vec)
    ws = scratch.get(n)
    abi.check(abi.lib().picoattn_ffn(C.byref(proj.struct), ffn_norm_w.data_ptr(), dim, n_ffn, n_vec, x.data_ptr(),
                                     ws.data_ptr(), ws.numel(), stream_handle(stream)), "picoattn_ffn")


def logits(x: torch.Tensor, output_norm_w: torch.Tensor, w_out: torch.Tensor, w_type: int, vocab: int,
           out: torch.Tensor, scratch: "Scratch", stream: torch.cuda.Stream | None = None) -> None:
    """out [n_vec, vocab] = W_out . rmsnorm(x) (cpp/model.hpp:454-457)."""
    dim = output_norm_w.numel()
    n_vec = x.numel() // dim
    ws = scratch.get(abi.lib().picoattn_logits_workspace_size(dim, n_vec))
    abi.check(abi.lib().picoattn_logits(x.data_ptr(), output_norm_w.data_ptr(), w_out.data_ptr(), w_type, dim, vocab,
                                        n_vec, out.data_ptr(), ws.data_ptr(), ws.numel(), stream_handle(stream)),
              "picoattn_logits")


class AttnState:
    """KV caches of n_seqs sequences in the reference layout plus RoPE tables.

    k_cache/v_cache: int16 tensors [n_seqs, n_layers, max_seq_len, kv_dim]
    (fp16 bit patterns; int16 is only the container type).
    """

    def __init__(self, cfg: abi.Config, n_seqs: int = 1, device: str | torch.device = "cuda",
                 max_ctx: int | None = None, rope: tuple[np.ndarray, np.ndarray] | None = None):
        self.cfg = cfg
        self.n_seqs = n_seqs
        self.device = torch.device(device)
        shape = (n_seqs, cfg.n_layers, cfg.max_seq_len, cfg.kv_dim)
        self.k_cache = torch.zeros(shape, dtype=torch.int16, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=torch.int16, device=self.device)
        cos, sin = rope if rope is not None else rope_table(cfg)
        self.rope_cos = torch.from_numpy(cos).to(self.device)
        self.rope_sin = torch.from_numpy(sin).to(self.device)
        per = cfg.n_layers * cfg.max_seq_len * cfg.kv_dim * 2
        kb, vb = self.k_cache.data_ptr(), self.v_cache.data_ptr()
        self.k_ptrs = torch.tensor([kb + i * per for i in range(n_seqs)], dtype=torch.int64, device=self.device)
        self.v_ptrs = torch.tensor([vb + i * per for i in range(n_seqs)], dtype=torch.int64, device=self.device)
        self.max_ctx = max_ctx if max_ctx is not None else cfg.max_seq_len
        ws = abi.lib().picoattn_decode_workspace_size(C.byref(cfg), n_seqs, self.max_ctx)
        if ws == 0:
            raise abi.PicoAttnError(abi.PICOATTN_EUNSUPPORTED, "decode_workspace_size")
        self.workspace = torch.zeros(ws, dtype=torch.uint8, device=self.device)
        abi.check(abi.lib().picoattn_workspace_init(self.workspace.data_ptr(), ws, stream_handle()), "ws init")

    # -- the call that replaces cpp/model.hpp:326-418 ---------------------------
    def decode(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pos: torch.Tensor,
               out: torch.Tensor, q_norm_w: torch.Tensor | None = None, k_norm_w: torch.Tensor | None = None,
               max_ctx: int | None = None, stream: torch.cuda.Stream | None = None) -> None:
        """q [B, Hq*hd], k/v [B, kvd] fp32, pos [B] int32 (device), out [B, Hq*hd] fp32."""
        B = q.shape[0]
        st = abi.lib().picoattn_decode(
            C.byref(self.cfg), layer, B, max_ctx if max_ctx is not None else self.max_ctx,
            q.data_ptr(), k.data_ptr(), v.data_ptr(), abi.ptr(q_norm_w), abi.ptr(k_norm_w),
            self.rope_cos.data_ptr(), self.rope_sin.data_ptr(), self.k_ptrs.data_ptr(), self.v_ptrs.data_ptr(),
            pos.data_ptr(), out.data_ptr(), self.workspace.data_ptr(), self.workspace.numel(),
            stream_handle(stream))
        abi.check(st, "picoattn_decode")

    def decode_layer(self, layer: int, dim: int, xb: torch.Tensor, proj: LayerProj, pos: torch.Tensor,
                     x: torch.Tensor, q_norm_w: torch.Tensor | None = None, k_norm_w: torch.Tensor | None = None,
                     stream: torch.cuda.Stream | None = None) -> None:
        """The attention block from the normalised hidden state xb [B, dim] into
        the residual x [B, dim] (cpp/model.hpp:318-427): projections, decode step,
        output projection added to x."""
        B = xb.shape[0]
        if getattr(self, "layer_ws", None) is None or self.layer_ws_key != (dim, B):
            n = abi.lib().picoattn_decode_layer_workspace_size(C.byref(self.cfg), dim, B, self.max_ctx)
            if n == 0:
                raise abi.PicoAttnError(abi.PICOATTN_EUNSUPPORTED, "decode_layer_workspace_size")
            self.layer_ws = torch.zeros(n, dtype=torch.uint8, device=self.device)
            self.layer_ws_key = (dim, B)
            abi.check(abi.lib().picoattn_workspace_init(self.layer_ws.data_ptr(), n, stream_handle(stream)),
                      "ws init")
        st = abi.lib().picoattn_decode_layer(
            C.byref(self.cfg), layer, dim, B, self.max_ctx, xb.data_ptr(), C.byref(proj.struct),
            abi.ptr(q_norm_w), abi.ptr(k_norm_w), self.rope_cos.data_ptr(), self.rope_sin.data_ptr(),
            self.k_ptrs.data_ptr(), self.v_ptrs.data_ptr(), pos.data_ptr(), x.data_ptr(),
            self.layer_ws.data_ptr(), self.layer_ws.numel(), stream_handle(stream))
        abi.check(st, "picoattn_decode_layer")

    def decode_block(self, layer: int, dim: int, n_ffn: int, x: torch.Tensor, attn_norm_w: torch.Tensor,
                     proj: LayerProj, ffn_norm_w: torch.Tensor, ffn_proj: FfnProj, pos: torch.Tensor,
                     q_norm_w: torch.Tensor | None = None, k_norm_w: torch.Tensor | None = None,
                     stream: torch.cuda.Stream | None = None) -> None:
        """One whole layer of the decode step on the residual x [B, dim] in place
        (cpp/model.hpp:315-452): attention norm, the attention block, the FFN block."""
        B = x.shape[0]
        key = (dim, n_ffn, B)
        if getattr(self, "block_ws", None) is None or self.block_ws_key != key:
            n = abi.lib().picoattn_decode_block_workspace_size(C.byref(self.cfg), dim, n_ffn, B, self.max_ctx)
            if n == 0:
                raise abi.PicoAttnError(abi.PICOATTN_EUNSUPPORTED, "decode_block_workspace_size")
            self.block_ws = torch.zeros(n, dtype=torch.uint8, device=self.device)
            self.block_ws_key = key
            abi.check(abi.lib().picoattn_workspace_init(self.block_ws.data_ptr(), n, stream_handle(stream)),
                      "ws init")
        st = abi.lib().picoattn_decode_block(
            C.byref(self.cfg), layer, dim, n_ffn, B, self.max_ctx, attn_norm_w.data_ptr(), C.byref(proj.struct),
            ffn_norm_w.data_ptr(), C.byref(ffn_proj.struct), abi.ptr(q_norm_w), abi.ptr(k_norm_w),
            self.rope_cos.data_ptr(), self.rope_sin.data_ptr(), self.k_ptrs.data_ptr(), self.v_ptrs.data_ptr(),
            pos.data_ptr(), x.data_ptr(), self.block_ws.data_ptr(), self.block_ws.numel(), stream_handle(stream))
        abi.check(st, "picoattn_decode_block")

    def block_status(self) -> int:
        v = C.c_uint32(0)
        abi.check(abi.lib().picoattn_workspace_status(self.block_ws.data_ptr(), stream_handle(), C.byref(v)))
        return v.value

    def decode_one(self, layer: int, pos: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   out: torch.Tensor, q_norm_w: torch.Tensor | None = None, k_norm_w: torch.Tensor | None = None,
                   seq: int = 0, stream: torch.cuda.Stream | None = None) -> int:
        """Model::forward-shaped call: one sequence, host position.  Returns the status."""
        return abi.lib().picoattn_decode_one(
            C.byref(self.cfg), layer, pos, q.data_ptr(), k.data_ptr(), v.data_ptr(),
            abi.ptr(q_norm_w), abi.ptr(k_norm_w), self.rope_cos.data_ptr(), self.rope_sin.data_ptr(),
            self.k_cache[seq].data_ptr(), self.v_cache[seq].data_ptr(), out.data_ptr(),
            self.workspace.data_ptr(), self.workspace.numel(), stream_handle(stream))

    # -- KV-cache persistence in the C engine's KVCP format (picolm/model.c:870-983)
    def kvcp_save(self, path: str, n_pos: int, seq: int = 0, stream: torch.cuda.Stream | None = None) -> None:
        """Rows 0..n_pos-1 of every layer of sequence `seq` -> a KVCP file (kvcache_save)."""
        abi.check(abi.lib().picoattn_kvcp_save(C.byref(self.cfg), n_pos, self.k_cache[seq].data_ptr(),
                                               self.v_cache[seq].data_ptr(), path.encode(), stream_handle(stream)),
                  "picoattn_kvcp_save")

    def kvcp_load(self, path: str, seq: int = 0, stream: torch.cuda.Stream | None = None) -> int:
        """A KVCP file -> rows 0..n_pos-1 of sequence `seq`; returns n_pos, or 0 when
        the file is missing or does not fit this model (kvcache_load's contract)."""
        n = C.c_int32(0)
        st = abi.lib().picoattn_kvcp_load(C.byref(self.cfg), path.encode(), self.k_cache[seq].data_ptr(),
                                          self.v_cache[seq].data_ptr(), C.byref(n), stream_handle(stream))
        if st in (abi.PICOATTN_EIO, abi.PICOATTN_EFORMAT):
            return 0
        abi.check(st, "picoattn_kvcp_load")
        return n.value

    # -- the call that replaces cpp/model.hpp:493-593 (forward_batch) ------------
    def prefill(self, layer: int, start_pos: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                out: torch.Tensor, q_norm_w: torch.Tensor | None = None, k_norm_w: torch.Tensor | None = None,
                seq: int = 0, workspace: torch.Tensor | None = None, stages: int = 0x3,
                stream: torch.cuda.Stream | None = None) -> int:
        """q [n, Hq*hd], k/v [n, kvd] fp32 or fp16 (device); out [n, Hq*hd] fp32.  Returns the status."""
        n = q.shape[0]
        dtype = abi.DTYPE_F16 if q.dtype == torch.float16 else abi.DTYPE_F32
        if workspace is None:
            workspace = self.prefill_workspace(n)
        return abi.lib().picoattn_prefill_staged(
            C.byref(self.cfg), layer, n, start_pos, dtype, q.data_ptr(), k.data_ptr(), v.data_ptr(),
            abi.ptr(q_norm_w), abi.ptr(k_norm_w), self.rope_cos.data_ptr(), self.rope_sin.data_ptr(),
            self.k_cache[seq].data_ptr(), self.v_cache[seq].data_ptr(), out.data_ptr(),
            workspace.data_ptr(), workspace.numel(), stream_handle(stream), stages)

    def prefill_workspace(self, n_tok: int) -> torch.Tensor:
        n = abi.lib().picoattn_prefill_workspace_size(C.byref(self.cfg), n_tok)
        if n == 0:
            raise abi.PicoAttnError(abi.PICOATTN_EUNSUPPORTED, "prefill_workspace_size")
        ws = getattr(self, "_pf_ws", None)
        if ws is None or ws.numel() < n:
            ws = torch.zeros(n, dtype=torch.uint8, device=self.device)
            self._pf_ws = ws
        return ws

    def status(self) -> int:
        v = C.c_uint32(0)
        abi.check(abi.lib().picoattn_workspace_status(self.workspace.data_ptr(), stream_handle(), C.byref(v)))
        return v.value
