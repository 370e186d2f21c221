"""Synthetic GGUF v3 model files for the loader tests (test helper).

Writes the container the engine's loader reads (cpp/model.hpp:705-902): the
header, metadata key/value pairs (strings, 32-bit integers and floats, 64-bit
integers, booleans and arrays, so the loader steps over every kind), tensor
descriptors (GGUF type ids, i.e. the engine's numbering minus one) and the
tensor data, each at an offset rounded to the file's alignment.  Weights are
seeded random blocks (tests/weightgen.py); norms are 1 + U(-0.1, 0.1).
"""
from __future__ import annotations

import struct

import numpy as np

from tests import weightgen as wg

U8, I32, U32, F32, BOOL, STR, ARR, U64 = 0, 5, 4, 6, 7, 8, 9, 10


def _s(b: bytearray, text: str) -> None:
    e = text.encode()
    b += struct.pack("<Q", len(e)) + e


def _kv(b: bytearray, key: str, vtype: int, value) -> None:
    _s(b, key)
    b += struct.pack("<I", vtype)
    if vtype == U32:
        b += struct.pack("<I", value)
    elif vtype == I32:
        b += struct.pack("<i", value)
    elif vtype == F32:
        b += struct.pack("<f", value)
    elif vtype == U64:
        b += struct.pack("<Q", value)
    elif vtype == BOOL:
        b += struct.pack("<B", value)
    elif vtype == STR:
        _s(b, value)
    elif vtype == ARR:
        etype, items = value
        b += struct.pack("<IQ", etype, len(items))
        for it in items:
            if etype == STR:
                _s(b, it)
            elif etype == F32:
                b += struct.pack("<f", it)
            elif etype == I32:
                b += struct.pack("<i", it)
    else:
        raise ValueError(vtype)


def write(path: str, meta: list, tensors: list, alignment: int = 32, version: int = 3) -> None:
    """meta: (key, vtype, value); tensors: (name, engine type, dims, bytes)."""
    b = bytearray(b"GGUF") + struct.pack("<IQQ", version, len(tensors), len(meta))
    for k, t, v in meta:
        _kv(b, k, t, v)
    off = 0
    offsets = []
    for name, etype, dims, data in tensors:
        _s(b, name)
        b += struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        b += struct.pack("<IQ", etype - 1, off)
        offsets.append(off)
        off = (off + len(data) + alignment - 1) // alignment * alignment
    b += bytes((-len(b)) % alignment)
    base = len(b)
    out = bytearray(b)
    for (name, etype, dims, data), o in zip(tensors, offsets):
        out += bytes(base + o - len(out))
        out += data
    with open(path, "wb") as f:
        f.write(out)


def qwen_model(path: str, n_layers=2, hq=4, hkv=2, hd=128, n_ffn=512, vocab=320, ctx=4096, rope_base=1e6,
               qk_norm=True, attn_t=13, ffn_t=13, down_t=15, out_t=15, tied=False, key_length=True,
               bias=True, seed=0, alignment=32) -> dict:
    """A small Qwen-shaped model file; returns the shape it wrote."""
    rng = np.random.default_rng(seed)
    dim = hq * hd
    kvd = hkv * hd
    norm = lambda n: (1 + rng.uniform(-0.1, 0.1, n)).astype(np.float32).tobytes()
    meta = [("general.architecture", STR, "qwen3"), ("general.name", STR, "synthetic"),
            ("qwen3.block_count", U32, n_layers), ("qwen3.context_length", U32, ctx),
            ("qwen3.embedding_length", U32, dim), ("qwen3.feed_forward_length", U32, n_ffn),
            ("qwen3.attention.head_count", U32, hq), ("qwen3.attention.head_count_kv", U32, hkv),
            ("qwen3.rope.freq_base", F32, rope_base), ("qwen3.attention.layer_norm_rms_epsilon", F32, 1e-6),
            ("general.alignment", U32, alignment), ("general.file_type", U32, 15),
            ("general.size_label", U64, 123456789), ("general.flag", BOOL, 1),
            ("tokenizer.ggml.model", STR, "gpt2"),
            ("tokenizer.ggml.tokens", ARR, (STR, [f"t{i}" for i in range(vocab)])),
            ("tokenizer.ggml.scores", ARR, (F32, [float(-i) for i in range(vocab)])),
            ("tokenizer.ggml.token_type", ARR, (I32, [1] * vocab)),
            ("tokenizer.ggml.bos_token_id", U32, 1), ("tokenizer.ggml.eos_token_id", U32, 2),
            ("tokenizer.ggml.merges", ARR, (STR, ["a b", "c d"]))]
    if key_length:
        meta.insert(8, ("qwen3.attention.key_length", U32, hd))
    tensors = [("token_embd.weight", 1, (dim, vocab), rng.uniform(-1, 1, (vocab, dim)).astype(np.float32).tobytes()),
               ("output_norm.weight", 1, (dim,), norm(dim))]
    if not tied:
        tensors.append(("output.weight", out_t, (dim, vocab), wg.make(out_t, dim, vocab, rng).tobytes()))
    for l in range(n_layers):
        p = f"blk.{l}."
        tensors += [(p + "attn_norm.weight", 1, (dim,), norm(dim)),
                    (p + "attn_q.weight", attn_t, (dim, dim), wg.make(attn_t, dim, dim, rng).tobytes()),
                    (p + "attn_k.weight", attn_t, (dim, kvd), wg.make(attn_t, dim, kvd, rng).tobytes()),
                    (p + "attn_v.weight", attn_t, (dim, kvd), wg.make(attn_t, dim, kvd, rng).tobytes()),
                    (p + "attn_output.weight", attn_t, (dim, dim), wg.make(attn_t, dim, dim, rng).tobytes()),
                    (p + "ffn_norm.weight", 1, (dim,), norm(dim)),
                    (p + "ffn_gate.weight", ffn_t, (dim, n_ffn), wg.make(ffn_t, dim, n_ffn, rng).tobytes()),
                    (p + "ffn_up.weight", ffn_t, (dim, n_ffn), wg.make(ffn_t, dim, n_ffn, rng).tobytes()),
                    (p + "ffn_down.weight", down_t, (n_ffn, dim), wg.make(down_t, n_ffn, dim, rng).tobytes())]
        if qk_norm:
            tensors += [(p + "attn_q_norm.weight", 1, (hd,), norm(hd)), (p + "attn_k_norm.weight", 1, (hd,), norm(hd))]
        if bias:  # stored as "attn_q.bias": the engine keeps it under that key, not as its attn_q_b
            tensors.append((p + "attn_q.bias", 1, (dim,), rng.uniform(-0.1, 0.1, dim).astype(np.float32).tobytes()))
    write(path, meta, tensors, alignment)
    return dict(n_layers=n_layers, hq=hq, hkv=hkv, hd=hd, dim=dim, n_ffn=n_ffn, vocab=vocab, ctx=ctx,
                rope_base=rope_base, tensors=tensors)
