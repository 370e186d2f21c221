"""Full-forward harness on the CPU: the host loop that the GPU test drives (the
reference's embedding / projection / FFN / logits stages around an attention
block) reproduces the reference's own Model::forward bit for bit when its
attention block is the reference's CPU loop, token after token; and
Model::forward_batch over a prompt gives the logits of Model::forward run token
by token.  This pins the staging, so that the GPU test compares attention only.
"""
import numpy as np
import pytest

from oracle import pyoracle

pytestmark = pytest.mark.skipif(not __import__("os").path.exists(pyoracle.REF_SO),
                                reason="oracle/_ref not built (make -C oracle ref)")

CFG = dict(n_layers=3, hq=4, hkv=2, hd=64, n_ffn=384, vocab=97, max_seq=48, rope_base=1e6, rope_mode=0,
           qk_norm=1)
TOKENS = [5, 17, 3, 96, 41, 41, 0, 77, 12, 58, 33, 9]


def _model(ref, seed=7):
    return pyoracle.RefFullModel(ref, **CFG, seed=seed)


def test_staged_host_loop_equals_model_forward():
    ref = pyoracle.RefHarness()
    m_ref, m = _model(ref), _model(ref)
    S, kvd = CFG["max_seq"], CFG["hkv"] * CFG["hd"]
    kc = [np.zeros((S, kvd), np.uint16) for _ in range(CFG["n_layers"])]
    vc = [np.zeros((S, kvd), np.uint16) for _ in range(CFG["n_layers"])]
    for pos, tok in enumerate(TOKENS):
        want = m_ref.forward(tok, pos)
        x = m.embed(tok)
        for l in range(CFG["n_layers"]):
            q, k, v = m.pre_attn(l, x)
            attn = ref.attn_decode_batch(CFG["hq"], CFG["hkv"], CFG["hd"], CFG["rope_mode"], q[None], k[None],
                                         v[None], m.norm_w(l, 0), m.norm_w(l, 1), m.rope_cos, m.rope_sin,
                                         [kc[l]], [vc[l]], np.array([pos], np.int32))[0]
            x = m.post_attn(l, x, attn)
        got = m.logits(x)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"position {pos}"


def test_forward_batch_equals_token_by_token_forward():
    ref = pyoracle.RefHarness()
    m1, m2 = _model(ref, 3), _model(ref, 3)
    for pos, tok in enumerate(TOKENS):
        last = m1.forward(tok, pos)
    batch = m2.forward_batch(TOKENS, 0)
    np.testing.assert_allclose(batch, last, rtol=1e-5, atol=1e-5)
    assert int(np.argmax(batch)) == int(np.argmax(last))


@pytest.mark.parametrize("wtype", [9, 13, 15], ids=["Q8_0", "Q4_K", "Q6_K"])
def test_staged_loop_with_oracle_projections_equals_model_forward(oracle, wtype):
    """With quantised attention weights, the host loop whose projections are the
    oracle's mat-vec (attention norm, q/k/v + biases, output projection into the
    residual, then the FFN stage) reproduces Model::forward bit for bit: this pins
    the stages the GPU layer test swaps for picoattn_decode_layer."""
    ref = pyoracle.RefHarness()
    cfg = dict(CFG, hd=128)  # dim 512: whole 256-weight blocks
    m_ref, m = pyoracle.RefFullModel(ref, **cfg, seed=9), pyoracle.RefFullModel(ref, **cfg, seed=9)
    m_ref.set_attn_weights(wtype, 4)
    m.set_attn_weights(wtype, 4)
    L, S, dim = cfg["n_layers"], cfg["max_seq"], cfg["hq"] * cfg["hd"]
    kvd = cfg["hkv"] * cfg["hd"]
    kc = [np.zeros((S, kvd), np.uint16) for _ in range(L)]
    vc = [np.zeros((S, kvd), np.uint16) for _ in range(L)]
    for pos, tok in enumerate(TOKENS[:6]):
        want = m_ref.forward(tok, pos)
        x = m.embed(tok)
        for l in range(L):
            xb = m.attn_norm(l, x)
            (wq, tq), (wk, tk), (wv, tv), (wo, to) = (m.attn_weight(l, i) for i in range(4))
            q = oracle.matvec(wq, tq, m.attn_bias(l, 0), dim, dim, xb)
            k = oracle.matvec(wk, tk, m.attn_bias(l, 1), dim, kvd, xb)
            v = oracle.matvec(wv, tv, m.attn_bias(l, 2), dim, kvd, xb)
            attn = oracle.decode_batch(cfg["hq"], cfg["hkv"], cfg["hd"], 0, q, k, v, m.norm_w(l, 0), m.norm_w(l, 1),
                                       m.rope_cos, m.rope_sin, [kc[l]], [vc[l]], np.array([pos], np.int32))
            x = oracle.matvec(wo, to, m.attn_bias(l, 3), dim, dim, attn, out=x[None], accumulate=True)[0]
            x = m.ffn(l, x)
        got = m.logits(x)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"position {pos}"
