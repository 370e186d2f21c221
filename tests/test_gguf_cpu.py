"""The GGUF loader (picoattn_gguf_*) against the engine's own Model::load.

Synthetic model files (tests/ggufgen.py) are opened by the library and by the
reference's unmodified loader compiled in oracle/_ref; the model shape it reads
and every tensor it keeps (file offset and type, by the engine's keys) must
be the same, with the engine's defaults, context cap, tied output matrix and
bias naming; files the engine rejects are rejected.  No GPU is needed.
"""
import ctypes as C
import os
import struct

import pytest

from oracle import pyoracle
from tests import ggufgen

KEYS = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down",
        "attn_q_norm", "attn_k_norm", "attn_q_b", "attn_q.bias", "ffn_gate_b")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(pyoracle.REF_SO):
        pytest.skip("oracle/_ref not built")
    return pyoracle.RefHarness()


def lib_open(path, override=0):
    from picolm_qwen_b200 import abi
    h = C.c_void_p()
    st = abi.lib().picoattn_gguf_open(path.encode(), override, C.byref(h))
    return st, h


def lib_config(h):
    from picolm_qwen_b200 import abi
    c = abi.GgufConfig()
    assert abi.lib().picoattn_gguf_get_config(h, C.byref(c)) == 0
    return c


def lib_find(h, layer, key):
    from picolm_qwen_b200 import abi
    t, n, off = C.c_int32(), C.c_size_t(), C.c_size_t()
    st = abi.lib().picoattn_gguf_find(h, layer, key.encode(), C.byref(t), C.byref(n), C.byref(off))
    return None if st == abi.PICOATTN_ENOENT else (off.value, t.value, n.value)


@pytest.mark.parametrize("kw,override", [
    (dict(), 0),                                         # Qwen3-like, context 4096 capped to 2048
    (dict(tied=True, qk_norm=False, attn_t=9), 96),     # tied output matrix, Q8_0, context override
    (dict(key_length=False, ctx=1024, alignment=64, down_t=13), 0),  # head_dim from n_embd / n_heads
])
def test_gguf_parse_matches_engine_loader(tmp_path, ref, kw, override):
    from picolm_qwen_b200 import abi
    path = str(tmp_path / "m.gguf")
    spec = ggufgen.qwen_model(path, **kw)
    m = pyoracle.RefGguf(ref, path, override)
    assert m.loaded
    want = m.config()
    st, h = lib_open(path, override)
    assert st == 0, abi.lib().picoattn_strerror(st)
    try:
        c = lib_config(h)
        for k in ("n_embd", "n_ffn", "n_heads", "n_kv_heads", "n_layers", "vocab_size", "max_seq_len", "head_dim",
                  "alignment"):
            assert getattr(c, k) == want[k], k
        assert c.rope_freq_base == want["rope_freq_base"]
        assert c.vocab_size == spec["vocab"] and c.head_dim == spec["hd"]
        for layer in range(-1, spec["n_layers"] + 1):
            keys = ("token_embd", "output_norm", "output") if layer < 0 else KEYS
            for key in keys:
                r = m.tensor(layer, key)
                g = lib_find(h, layer, key)
                assert (r is None) == (g is None), (layer, key)
                if r is not None:
                    assert (g[0], g[1]) == r, (layer, key)
        # the engine's attn_q_b comes only from a tensor of that name; the file's
        # "attn_q.bias" stays under its own key
        if kw.get("bias", True):
            assert lib_find(h, 0, "attn_q_b") is None and lib_find(h, 0, "attn_q.bias") is not None
        if kw.get("tied"):
            assert lib_find(h, -1, "output")[0] == lib_find(h, -1, "token_embd")[0]
        assert abi.lib().picoattn_gguf_arena_bytes(h) > 0
    finally:
        abi.lib().picoattn_gguf_close(h)
        m.close()


def test_gguf_rejects_what_the_engine_rejects(tmp_path, ref):
    from picolm_qwen_b200 import abi
    path = str(tmp_path / "ok.gguf")
    ggufgen.qwen_model(path)
    data = open(path, "rb").read()
    cases = {
        "magic": b"GGUX" + data[4:],
        "version": data[:4] + struct.pack("<I", 4) + data[8:],
        "truncated": data[:200],
    }
    for name, blob in cases.items():
        p = str(tmp_path / f"{name}.gguf")
        with open(p, "wb") as f:
            f.write(blob)
        st, h = lib_open(p)
        assert st == abi.PICOATTN_EFORMAT, name
        if name != "truncated":  # the engine's loader itself trusts the file's lengths
            assert not pyoracle.RefGguf(ref, p).loaded, name
    st, _ = lib_open(str(tmp_path / "missing.gguf"))
    assert st == abi.PICOATTN_EIO
