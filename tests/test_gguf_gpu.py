"""A GGUF model file on the device: picoattn_gguf_upload, then every decode
step through picoattn_decode_block and picoattn_logits with the arena's
tensors, against the engine's unmodified Model::load + Model::forward of the
same file (oracle/_ref).  The arena holds the file's bytes exactly; the
next-token argmax must be identical at every step and the logits agree within
2e-2 of their scale (the full-forward bar).
"""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import pyoracle
from tests import ggufgen

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not os.path.exists(pyoracle.REF_SO):
        pytest.skip("oracle/_ref not built")


def arena_tensor(h, arena, layer, key):
    from picolm_qwen_b200 import abi
    p, t = C.c_void_p(), C.c_int32()
    st = abi.lib().picoattn_gguf_arena_tensor(h, arena.data_ptr(), layer, key.encode(), C.byref(p), C.byref(t))
    return (None, 0) if st == abi.PICOATTN_ENOENT else (p.value, t.value)


@pytest.mark.parametrize("kw", [dict(), dict(tied=True, attn_t=9, down_t=13)], ids=["q4k-q6k", "tied-q8_0"])
def test_gguf_model_decodes_on_device_like_the_engine(tmp_path, cuda, kw):
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, Scratch
    L = abi.lib()
    path = str(tmp_path / "m.gguf")
    spec = ggufgen.qwen_model(path, seed=5, **kw)
    ref = pyoracle.RefHarness()
    m = pyoracle.RefGguf(ref, path, 0, rope_mode=0)
    assert m.loaded
    h = C.c_void_p()
    assert L.picoattn_gguf_open(path.encode(), 0, C.byref(h)) == 0
    try:
        c = abi.GgufConfig()
        assert L.picoattn_gguf_get_config(h, C.byref(c)) == 0
        n = L.picoattn_gguf_arena_bytes(h)
        arena = torch.empty(n, dtype=torch.uint8, device="cuda")
        assert L.picoattn_gguf_upload(h, arena.data_ptr(), n, torch.cuda.current_stream().cuda_stream) == 0
        # the arena holds the file's bytes
        blob = np.fromfile(path, np.uint8)
        for layer, key in ((-1, "token_embd"), (-1, "output"), (0, "attn_q"), (1, "ffn_down"), (0, "attn_v")):
            t, nb, off = C.c_int32(), C.c_size_t(), C.c_size_t()
            assert L.picoattn_gguf_find(h, layer, key.encode(), C.byref(t), C.byref(nb), C.byref(off)) == 0
            p, _ = arena_tensor(h, arena, layer, key)
            dev = arena[p - arena.data_ptr():p - arena.data_ptr() + nb.value].cpu().numpy()
            assert np.array_equal(dev, blob[off.value:off.value + nb.value]), (layer, key)
        # the model on the device
        dim, hq, hkv, hd, n_ffn, vocab = c.n_embd, c.n_heads, c.n_kv_heads, c.head_dim, c.n_ffn, c.vocab_size
        cfg = abi.Config.make(c.n_layers, hq, hkv, hd, c.max_seq_len, c.rope_freq_base, abi.ROPE_NEOX)
        st = AttnState(cfg, n_seqs=1, max_ctx=c.max_seq_len)
        layers = []
        for l in range(c.n_layers):
            g = lambda k: arena_tensor(h, arena, l, k)
            aw = [g(k) for k in ("attn_q", "attn_k", "attn_v", "attn_output")]
            bias = [g(k)[0] for k in ("attn_q_b", "attn_k_b", "attn_v_b", "attn_output_b")]
            lw = abi.LayerWeights(*[p for p, _ in aw], *[t for _, t in aw], *bias)
            fw = [g(k) for k in ("ffn_gate", "ffn_up", "ffn_down")]
            fwt = abi.FfnWeights(*[p for p, _ in fw], *[t for _, t in fw], g("ffn_gate_b")[0], g("ffn_down_b")[0])
            qn, kn = g("attn_q_norm")[0], g("attn_k_norm")[0]
            layers.append((g("attn_norm")[0], lw, g("ffn_norm")[0], fwt, qn, kn))
        out_norm = arena_tensor(h, arena, -1, "output_norm")[0]
        out_w, out_t = arena_tensor(h, arena, -1, "output")
        t, nb, off = C.c_int32(), C.c_size_t(), C.c_size_t()
        L.picoattn_gguf_find(h, -1, b"token_embd", C.byref(t), C.byref(nb), C.byref(off))
        embd = blob[off.value:off.value + nb.value].view(np.float32).reshape(vocab, dim)
        ws = torch.zeros(L.picoattn_decode_block_workspace_size(C.byref(cfg), dim, n_ffn, 1, c.max_seq_len),
                         dtype=torch.uint8, device="cuda")
        sh = torch.cuda.current_stream().cuda_stream
        scratch = Scratch("cuda")
        lg = torch.empty((1, vocab), device="cuda")
        got, want = [], []
        tok = 3
        for pos in range(24):
            want.append(m.forward(tok, pos, vocab))
            x = torch.from_numpy(embd[tok][None].copy()).cuda()
            pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
            for l in range(c.n_layers):
                an, lw, fn, fwt, qn, kn = layers[l]
                s = L.picoattn_decode_block(C.byref(cfg), l, dim, n_ffn, 1, c.max_seq_len, an, C.byref(lw), fn,
                                            C.byref(fwt), qn, kn, st.rope_cos.data_ptr(), st.rope_sin.data_ptr(),
                                            st.k_ptrs.data_ptr(), st.v_ptrs.data_ptr(), pos_t.data_ptr(),
                                            x.data_ptr(), ws.data_ptr(), ws.numel(), sh)
                assert s == 0, L.picoattn_strerror(s)
            lws = scratch.get(L.picoattn_logits_workspace_size(dim, 1))
            assert L.picoattn_logits(x.data_ptr(), out_norm, out_w, out_t, dim, vocab, 1, lg.data_ptr(),
                                     lws.data_ptr(), lws.numel(), sh) == 0
            got.append(lg.cpu().numpy()[0])
            tok = int(np.argmax(want[-1]))
        torch.cuda.synchronize()
        status = C.c_uint32(0)
        assert L.picoattn_workspace_status(ws.data_ptr(), sh, C.byref(status)) == 0 and status.value == 0
        got, want = np.stack(got), np.stack(want)
        same = np.argmax(got, 1) == np.argmax(want, 1)
        assert same.all(), f"argmax differs at steps {np.nonzero(~same)[0].tolist()}"
        scale = np.abs(want).max()
        assert np.abs(got - want).max() <= 2e-2 * scale
    finally:
        L.picoattn_gguf_close(h)
        m.close()
