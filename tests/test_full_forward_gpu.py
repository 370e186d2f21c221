"""Full-forward parity on the GPU (the full-forward oracle): a 3-layer model with
seeded random weights, run by the reference's unmodified Model::forward_batch
(a 40-token prompt) and Model::forward (24 decode steps), against the same model
run by a host loop whose attention block is this library through the C ABI
(picoattn_prefill_staged for the prompt, picoattn_decode_one per step, the KV
cache on the device) and whose other stages are the reference's own functions
(pinned bit-exact by test_full_forward_cpu.py).  The next-token argmax must be
identical at every step; the logits agree to the attention tolerance carried
through three layers.  Both head_dim 128 shapes below run the tensor-core
prefill kernels (G = 2: CTA pair; G = 3: one head per CTA).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import pyoracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _run(hq, hkv, hd, qk_norm, seed):
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState
    if not __import__("os").path.exists(pyoracle.REF_SO):
        pytest.skip("oracle/_ref not built")
    ref = pyoracle.RefHarness()
    L, S, vocab, n_prompt, n_gen = 3, 96, 211, 40, 24
    kw = dict(n_layers=L, hq=hq, hkv=hkv, hd=hd, n_ffn=512, vocab=vocab, max_seq=S, rope_base=1e6,
              rope_mode=0, qk_norm=qk_norm, seed=seed)
    m_ref, m = pyoracle.RefFullModel(ref, **kw), pyoracle.RefFullModel(ref, **kw)
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, vocab, n_prompt).astype(np.int32)

    cfg = abi.Config.make(L, hq, hkv, hd, S, 1e6, abi.ROPE_NEOX)
    st = AttnState(cfg, n_seqs=1, max_ctx=S)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    norms = [(None, None) if not qk_norm else (dev(m.norm_w(l, 0)), dev(m.norm_w(l, 1))) for l in range(L)]

    # prompt: every layer over all prompt tokens at once
    xs = np.stack([m.embed(t) for t in prompt])
    for l in range(L):
        qkv = [m.pre_attn(l, x) for x in xs]
        q = dev(np.stack([a[0] for a in qkv])); k = dev(np.stack([a[1] for a in qkv]))
        v = dev(np.stack([a[2] for a in qkv]))
        out = torch.empty((n_prompt, hq * hd), device="cuda")
        assert st.prefill(l, 0, q, k, v, out, norms[l][0], norms[l][1]) == 0
        attn = out.cpu().numpy()
        xs = np.stack([m.post_attn(l, xs[i], attn[i]) for i in range(n_prompt)])
    got = [m.logits(xs[-1])]
    want = [m_ref.forward_batch(prompt, 0)]

    # decode, teacher-forced on the reference's choice
    tok = int(np.argmax(want[0]))
    out1 = torch.empty(hq * hd, device="cuda")
    for step in range(n_gen):
        pos = n_prompt + step
        want.append(m_ref.forward(tok, pos))
        x = m.embed(tok)
        for l in range(L):
            q, k, v = (dev(a) for a in m.pre_attn(l, x))
            assert st.decode_one(l, pos, q, k, v, out1, norms[l][0], norms[l][1]) == 0
            x = m.post_attn(l, x, out1.cpu().numpy())
        got.append(m.logits(x))
        tok = int(np.argmax(want[-1]))
    torch.cuda.synchronize()
    assert st.status() == 0
    got, want = np.stack(got), np.stack(want)
    same = (np.argmax(got, 1) == np.argmax(want, 1))
    assert same.all(), f"argmax differs at steps {np.nonzero(~same)[0].tolist()}"
    scale = np.abs(want).max()
    err = np.abs(got - want).max()
    assert err <= 2e-2 * scale, f"max logit error {err:.3g} of scale {scale:.3g}"


def test_full_forward_qwen3_like_cta_pair(cuda):
    _run(hq=4, hkv=2, hd=128, qk_norm=1, seed=11)


def test_full_forward_qwen2_like_no_qk_norm(cuda):
    _run(hq=6, hkv=2, hd=128, qk_norm=0, seed=12)


@pytest.mark.parametrize("wtype", [9, 13], ids=["Q8_0", "Q4_K"])
def test_full_forward_decode_layer_quantized_weights(cuda, wtype):
    """Quantised attention weights; each decode step's whole attention block
    (q/k/v projections with biases, QK-norm, RoPE, cache append, attention,
    output projection into the residual) is one picoattn_decode_layer call on
    the device, the rest the reference's stages.  Same bars as above."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, LayerProj
    if not __import__("os").path.exists(pyoracle.REF_SO):
        pytest.skip("oracle/_ref not built")
    ref = pyoracle.RefHarness()
    hq, hkv, hd, seed = 4, 2, 128, 21
    L, S, vocab, n_prompt, n_gen = 3, 96, 211, 16, 24
    kw = dict(n_layers=L, hq=hq, hkv=hkv, hd=hd, n_ffn=512, vocab=vocab, max_seq=S, rope_base=1e6,
              rope_mode=0, qk_norm=1, seed=seed)
    m_ref, m = pyoracle.RefFullModel(ref, **kw), pyoracle.RefFullModel(ref, **kw)
    m_ref.set_attn_weights(wtype, 8)
    m.set_attn_weights(wtype, 8)
    dim = hq * hd
    cfg = abi.Config.make(L, hq, hkv, hd, S, 1e6, abi.ROPE_NEOX)
    st = AttnState(cfg, n_seqs=1, max_ctx=S)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    norms = [(dev(m.norm_w(l, 0)), dev(m.norm_w(l, 1))) for l in range(L)]
    projs = []
    for l in range(L):
        ws = [m.attn_weight(l, i) for i in range(4)]
        projs.append(LayerProj(*(dev(w) for w, _ in ws), [t for _, t in ws],
                               *(dev(m.attn_bias(l, i)) for i in range(4))))
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, vocab, n_prompt).astype(np.int32)
    # prompt through the prefill path (the reference's projections)
    xs = np.stack([m.embed(t) for t in prompt])
    for l in range(L):
        qkv = [m.pre_attn(l, x) for x in xs]
        q = dev(np.stack([a[0] for a in qkv])); k = dev(np.stack([a[1] for a in qkv]))
        v = dev(np.stack([a[2] for a in qkv]))
        out = torch.empty((n_prompt, hq * hd), device="cuda")
        assert st.prefill(l, 0, q, k, v, out, *norms[l]) == 0
        attn = out.cpu().numpy()
        xs = np.stack([m.post_attn(l, xs[i], attn[i]) for i in range(n_prompt)])
    got = [m.logits(xs[-1])]
    want = [m_ref.forward_batch(prompt, 0)]
    tok = int(np.argmax(want[0]))
    for step in range(n_gen):
        pos = n_prompt + step
        want.append(m_ref.forward(tok, pos))
        x = m.embed(tok)
        pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
        for l in range(L):
            xd = dev(x[None])
            st.decode_layer(l, dim, dev(m.attn_norm(l, x)[None]), projs[l], pos_t, xd, *norms[l])
            x = m.ffn(l, xd.cpu().numpy()[0])
        got.append(m.logits(x))
        tok = int(np.argmax(want[-1]))
    torch.cuda.synchronize()
    assert st.status() == 0
    got, want = np.stack(got), np.stack(want)
    same = (np.argmax(got, 1) == np.argmax(want, 1))
    assert same.all(), f"argmax differs at steps {np.nonzero(~same)[0].tolist()}"
    scale = np.abs(want).max()
    err = np.abs(got - want).max()
    assert err <= 2e-2 * scale, f"max logit error {err:.3g} of scale {scale:.3g}"


def _device_model(m, L, dev):
    """Every layer's weights of a RefFullModel on the device, as the engine holds them."""
    from picolm_qwen_b200.runtime import FfnProj, LayerProj
    layers = []
    for l in range(L):
        aw = [m.attn_weight(l, i) for i in range(4)]
        proj = LayerProj(*(dev(w) for w, _ in aw), [t for _, t in aw], *(dev(m.attn_bias(l, i)) for i in range(4)))
        fw = [m.ffn_weight(l, i) for i in range(3)]
        fproj = FfnProj(*(dev(w) for w, _ in fw), [t for _, t in fw], dev(m.ffn_bias(l, 0)), dev(m.ffn_bias(l, 1)))
        layers.append((dev(m.model_norm(l, 0)), proj, dev(m.model_norm(l, 1)), fproj))
    out_w, out_t = m.ffn_weight(0, 3)
    return layers, dev(m.model_norm(0, 2)), dev(out_w), out_t


@pytest.mark.parametrize("attn_t,ffn_t", [(13, 13), (9, 15)], ids=["Q4_K-Q4_K", "Q8_0-Q6_K"])
def test_full_forward_whole_decode_step_on_device(cuda, attn_t, ffn_t):
    """Every decode step wholly on the device: per layer one picoattn_decode_block
    (attention norm, projections, QK-norm, RoPE, cache append, attention,
    output projection, FFN norm, gate/up, SwiGLU, down projection, both
    residuals), then picoattn_logits (final norm, output matrix); only the
    embedding row comes from the host.  Quantised attention, FFN and output
    weights.  The reference runs the unmodified Model::forward on the same
    model; the next-token argmax must be identical at every step and the logits
    agree within 2e-2 of their scale."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, Scratch, logits
    if not __import__("os").path.exists(pyoracle.REF_SO):
        pytest.skip("oracle/_ref not built")
    ref = pyoracle.RefHarness()
    hq, hkv, hd, seed = 4, 2, 128, 31
    L, S, vocab, n_gen, n_ffn = 3, 64, 211, 32, 512
    kw = dict(n_layers=L, hq=hq, hkv=hkv, hd=hd, n_ffn=n_ffn, vocab=vocab, max_seq=S, rope_base=1e6,
              rope_mode=0, qk_norm=1, seed=seed)
    m_ref, m = pyoracle.RefFullModel(ref, **kw), pyoracle.RefFullModel(ref, **kw)
    for mm in (m_ref, m):
        mm.set_attn_weights(attn_t, 8)
        mm.set_ffn_weights(ffn_t, 9)
    dim = hq * hd
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    cfg = abi.Config.make(L, hq, hkv, hd, S, 1e6, abi.ROPE_NEOX)
    st = AttnState(cfg, n_seqs=1, max_ctx=S)
    norms = [(dev(m.norm_w(l, 0)), dev(m.norm_w(l, 1))) for l in range(L)]
    layers, out_norm, out_w, out_t = _device_model(m, L, dev)
    scratch = Scratch("cuda")
    lg = torch.empty((1, vocab), device="cuda")
    got, want = [], []
    tok = 7
    for pos in range(n_gen):
        want.append(m_ref.forward(tok, pos))
        x = dev(m.embed(tok)[None])
        pos_t = torch.tensor([pos], dtype=torch.int32, device="cuda")
        for l in range(L):
            an, proj, fn, fproj = layers[l]
            st.decode_block(l, dim, n_ffn, x, an, proj, fn, fproj, pos_t, *norms[l])
        logits(x, out_norm, out_w, out_t, vocab, lg, scratch)
        got.append(lg.cpu().numpy()[0])
        tok = int(np.argmax(want[-1]))
    torch.cuda.synchronize()
    assert st.block_status() == 0
    got, want = np.stack(got), np.stack(want)
    same = (np.argmax(got, 1) == np.argmax(want, 1))
    assert same.all(), f"argmax differs at steps {np.nonzero(~same)[0].tolist()}"
    scale = np.abs(want).max()
    err = np.abs(got - want).max()
    assert err <= 2e-2 * scale, f"max logit error {err:.3g} of scale {scale:.3g}"


@pytest.mark.parametrize("ffn_t", [1, 13, 15], ids=["F32", "Q4_K", "Q6_K"])
def test_rmsnorm_ffn_logits_vs_reference(cuda, ffn_t):
    """picoattn_rmsnorm, picoattn_ffn and picoattn_logits on their own against
    the reference's TensorOps::rmsnorm, FFN block (cpp/model.hpp:429-452) and
    logits (cpp/model.hpp:454-457) on the same model weights and inputs.  The
    weights are dequantised bit-identically and the sums run in another order,
    so the outputs agree to fp32 rounding: |gpu - ref| <= 1e-4 (1 + |ref|)."""
    from picolm_qwen_b200.runtime import Scratch, ffn, logits, rmsnorm
    if not __import__("os").path.exists(pyoracle.REF_SO):
        pytest.skip("oracle/_ref not built")
    ref = pyoracle.RefHarness()
    hq, hkv, hd, n_ffn, vocab = 8, 2, 128, 1536, 1000
    m = pyoracle.RefFullModel(ref, n_layers=1, hq=hq, hkv=hkv, hd=hd, n_ffn=n_ffn, vocab=vocab, max_seq=8,
                              rope_base=1e6, rope_mode=0, qk_norm=0, seed=3)
    if ffn_t != 1:
        m.set_ffn_weights(ffn_t, 4)
    dim = hq * hd
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    rng = np.random.default_rng(ffn_t)
    xs = rng.standard_normal((3, dim)).astype(np.float32)
    layers, out_norm, out_w, out_t = _device_model(m, 1, dev)
    an, _, fn, fproj = layers[0]
    scratch = Scratch("cuda")
    # rmsnorm
    out = torch.empty((3, dim), device="cuda")
    rmsnorm(dev(xs), an, out)
    want = np.stack([m.attn_norm(0, x) for x in xs])
    assert np.allclose(out.cpu().numpy(), want, rtol=1e-5, atol=1e-6)
    # FFN block with its residual, three vectors at once
    x = dev(xs)
    ffn(fproj, fn, n_ffn, x, scratch)
    want = np.stack([m.ffn(0, xv) for xv in xs])
    got = x.cpu().numpy()
    assert np.all(np.abs(got - want) <= 1e-4 * (1 + np.abs(want))), f"ffn max err {np.abs(got - want).max():.3g}"
    # logits
    lg = torch.empty((3, vocab), device="cuda")
    logits(dev(xs), out_norm, out_w, out_t, vocab, lg, scratch)
    want = np.stack([m.logits(xv) for xv in xs])
    got = lg.cpu().numpy()
    assert np.all(np.abs(got - want) <= 1e-4 * (1 + np.abs(want))), f"logits max err {np.abs(got - want).max():.3g}"
    # one vector: for Q4_K/Q6_K weights the norm runs inside the gate/up launch,
    # the SwiGLU inside the fragment kernel of the down launch, and the final
    # norm inside the logits launch
    want_f = m.ffn(0, xs[1])
    x1 = dev(xs[1:2])
    ffn(fproj, fn, n_ffn, x1, scratch)
    got = x1.cpu().numpy()[0]
    assert np.all(np.abs(got - want_f) <= 1e-4 * (1 + np.abs(want_f))), f"ffn (one vector) max err {np.abs(got - want_f).max():.3g}"
    lg1 = torch.empty((1, vocab), device="cuda")
    logits(dev(xs[2:3]), out_norm, out_w, out_t, vocab, lg1, scratch)
    want_l = m.logits(xs[2])
    got = lg1.cpu().numpy()[0]
    assert np.all(np.abs(got - want_l) <= 1e-4 * (1 + np.abs(want_l))), f"logits (one vector) max err {np.abs(got - want_l).max():.3g}"
