"""Prefill attention (tcgen05 / TMEM kernel) against the reference and the oracle.

Reference semantics (cpp/model.hpp:493-593): prompt token i runs the decode
step at pos = start_pos + i, so it stores its k/v row and attends causally over
cache rows 0..pos.  Tolerance on the output, elementwise:
    |gpu - ref| <= 2e-3 + 1e-2 * |ref|
Cache rows written by the prefill must equal the reference's fp16 bits.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def assert_close(got, ref, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    bad = ~(err <= ATOL + RTOL * np.abs(ref))
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside tolerance, max err {err.max():.3g} "
                           f"at {np.unravel_index(err.argmax(), err.shape)}")


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from picolm_qwen_b200 import abi
    assert abi.lib().picoattn_device_check() == 0
    return torch.device("cuda")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def state(cfg):
    from picolm_qwen_b200.runtime import AttnState
    return AttnState(cfg, n_seqs=1)


def test_prefill_matches_reference_golden(cuda, golden_dir):
    """64-token Qwen3-shaped prompt (QK-norm, fp16 inputs) produced by Model::forward."""
    from picolm_qwen_b200 import abi
    g = np.load(os.path.join(golden_dir, "decode_cfg4_qwen3_8b.npz"))
    hq, hkv, hd = int(g["hq"]), int(g["hkv"]), int(g["hd"])
    n = int(g["keep"])
    cfg = abi.Config.make(2, hq, hkv, hd, n, float(g["rope_base"]))
    st = state(cfg)
    out = torch.empty((n, hq * hd), device="cuda")
    q = dev(g["q"].astype(np.float16))  # the fixture inputs are fp16-representable
    k = dev(g["k"].astype(np.float16))
    v = dev(g["v"].astype(np.float16))
    assert np.array_equal(g["q"].astype(np.float16).astype(np.float32), g["q"])
    s = st.prefill(1, 0, q, k, v, out, dev(g["q_norm_w"]), dev(g["k_norm_w"]))
    assert s == 0, (abi.lib().picoattn_strerror(s), abi.lib().picoattn_last_cuda_error())
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), g["out"], "prefill")
    assert np.array_equal(st.k_cache[0, 1, :n].cpu().numpy(), g["kcache"].view(np.int16))
    assert np.array_equal(st.v_cache[0, 1, :n].cpu().numpy(), g["vcache"].view(np.int16))
    assert st.status() == 0


def run_case(oracle, hq, hkv, hd, n_tok, start, mode=0, norm=True, f16=True, seed=0, layer=0, threads=16, qscale=1.0):
    from picolm_qwen_b200 import abi
    rng = np.random.default_rng(seed)
    kvd = hkv * hd
    S = start + n_tok
    base = 1e6 if mode == 0 else 1e4
    cfg = abi.Config.make(layer + 1, hq, hkv, hd, S, base, mode)
    st = state(cfg)
    kc = np.zeros((S, kvd), np.uint16)
    vc = np.zeros((S, kvd), np.uint16)
    if start:
        kc[:start] = oracle.f32_to_f16(rng.standard_normal(start * kvd).astype(np.float32)).reshape(start, kvd)
        vc[:start] = oracle.f32_to_f16(rng.standard_normal(start * kvd).astype(np.float32)).reshape(start, kvd)
        st.k_cache[0, layer, :start] = dev(kc[:start].view(np.int16))
        st.v_cache[0, layer, :start] = dev(vc[:start].view(np.int16))
    q = (qscale * rng.standard_normal((n_tok, hq * hd))).astype(np.float32)
    k = rng.standard_normal((n_tok, kvd)).astype(np.float32)
    v = rng.standard_normal((n_tok, kvd)).astype(np.float32)
    if f16:
        q, k, v = (a.astype(np.float16).astype(np.float32) for a in (q, k, v))
    qn = kn = None
    if norm:
        qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
        kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    cos_t, sin_t = oracle.rope_table(S, hd, base)
    ref = oracle.prefill(hq, hkv, hd, mode, q, k, v, qn, kn, cos_t, sin_t, kc, vc, start, n_threads=threads)
    out = torch.empty((n_tok, hq * hd), device="cuda")
    cast = (lambda a: dev(a.astype(np.float16))) if f16 else dev
    s = st.prefill(layer, start, cast(q), cast(k), cast(v), out,
                   None if qn is None else dev(qn), None if kn is None else dev(kn))
    assert s == 0, abi.lib().picoattn_strerror(s)
    torch.cuda.synchronize()
    assert st.status() == 0
    return st, out.cpu().numpy(), ref, kc, vc


@pytest.mark.parametrize("case", [
    dict(hq=32, hkv=8, hd=128, n_tok=300, start=0),                  # Qwen3-8B heads, ragged last tile
    dict(hq=32, hkv=8, hd=128, n_tok=257, start=200),                # chunked prefill after cached rows
    dict(hq=8, hkv=2, hd=128, n_tok=128, start=0, f16=False),        # fp32 inputs, exactly one tile
    dict(hq=28, hkv=4, hd=128, n_tok=200, start=77, norm=False),     # Qwen2.5 heads (G=7), no QK-norm
    dict(hq=32, hkv=4, hd=64, n_tok=190, start=5, mode=1, norm=False),  # TinyLlama heads, interleaved
    dict(hq=14, hkv=2, hd=64, n_tok=129, start=0, norm=False),       # Qwen2.5-0.5B heads
    dict(hq=4, hkv=4, hd=64, n_tok=1, start=0),                      # a one-token prompt
    dict(hq=4, hkv=4, hd=128, n_tok=1, start=300),                   # one token after a long cache
    dict(hq=16, hkv=4, hd=128, n_tok=333, start=1000, norm=False),   # long cached prefix
    dict(hq=8, hkv=2, hd=128, n_tok=150, start=40, mode=1),          # interleaved RoPE at head_dim 128, QK-norm
    dict(hq=8, hkv=4, hd=64, n_tok=70, start=3, mode=1, f16=False),  # fp32 inputs, interleaved, head_dim 64
    dict(hq=12, hkv=4, hd=64, n_tok=33, start=0, f16=False),        # fp32 inputs, NeoX + QK-norm, head_dim 64, G = 3
])
def test_prefill_vs_oracle(cuda, oracle, case):
    st, got, ref, kc, vc = run_case(oracle, **case)
    assert_close(got, ref, str(case))
    start, n = case["start"], case["n_tok"]
    assert np.array_equal(st.k_cache[0, 0, start:start + n].cpu().numpy().view(np.uint16), kc[start:start + n])
    assert np.array_equal(st.v_cache[0, 0, start:start + n].cpu().numpy().view(np.uint16), vc[start:start + n])


def fp16_datapath_reference(oracle, hq, hkv, hd, q, kc, vc, start, cos_t, sin_t):
    """The attention the tensor-core path computes, in numpy: rotated q pre-scaled
    by log2(e)/sqrt(hd) and rounded to fp16 (the workspace operand), fp32 scores
    against the fp16 cache, base-2 softmax in fp32, p rounded to fp16 for P.V,
    the sum over the unrounded p.  Only for inputs whose scores are so wide that
    the fp16 rounding of q alone moves the output past the tolerance against the
    fp32 reference."""
    n_tok = q.shape[0]
    g = hq // hkv
    K = oracle.f16_to_f32(kc.ravel()).reshape(kc.shape)
    V = oracle.f16_to_f32(vc.ravel()).reshape(vc.shape)
    out = np.zeros((n_tok, hq * hd), np.float32)
    scale = np.float32(1.4426950408889634 / np.sqrt(hd))
    for i in range(n_tok):
        pos = start + i
        qr, _ = oracle.rope(0, q[i], np.zeros(hkv * hd, np.float32), hd, hq, hkv, cos_t[pos], sin_t[pos])
        q16 = (qr * scale).astype(np.float16).astype(np.float32).reshape(hq, hd)
        for h in range(hq):
            kvh = h // g
            sc = K[:pos + 1, kvh * hd:(kvh + 1) * hd] @ q16[h]
            p = np.exp2(sc - sc.max()).astype(np.float32)
            p16 = p.astype(np.float16).astype(np.float32)
            out[i, h * hd:(h + 1) * hd] = (p16 @ V[:pos + 1, kvh * hd:(kvh + 1) * hd]) / p.sum()
    return out


def test_prefill_wide_scores_rescale_paths(cuda, oracle):
    """Wide scores (q x 6, no norm): row maxima jump between and within key tiles,
    so the softmax lifts its running max mid-tile and rescales the stored P, the
    sums and O.  Checked against the same fp16 datapath in numpy (tolerance as
    everywhere); the k/v rows against the reference bit for bit."""
    hq, hkv, hd, n_tok, start = 8, 2, 128, 400, 150
    st, got, _, kc, vc = run_case(oracle, hq, hkv, hd, n_tok, start, norm=False, qscale=6.0, seed=4, threads=8)
    S = start + n_tok
    cos_t, sin_t = oracle.rope_table(S, hd, 1e6)
    rng = np.random.default_rng(4)  # the same draws as run_case
    kvd = hkv * hd
    rng.standard_normal(start * kvd), rng.standard_normal(start * kvd)
    q = (6.0 * rng.standard_normal((n_tok, hq * hd))).astype(np.float32).astype(np.float16).astype(np.float32)
    kc_all = st.k_cache[0, 0, :S].cpu().numpy().view(np.uint16)
    vc_all = st.v_cache[0, 0, :S].cpu().numpy().view(np.uint16)
    assert np.array_equal(kc_all[start:], kc[start:S]) and np.array_equal(vc_all[start:], vc[start:S])
    want = fp16_datapath_reference(oracle, hq, hkv, hd, q, kc_all, vc_all, start, cos_t, sin_t)
    assert_close(got, want, "wide scores")


def test_prefill_full_qwen3_layer_vs_oracle(cuda, oracle):
    """One full layer of the benchmark shape: 2048 tokens, 32/8 heads, hd 128, QK-norm, fp16 in."""
    _, got, ref, _, _ = run_case(oracle, 32, 8, 128, 2048, 0, seed=11, layer=3)
    assert_close(got, ref, "S=2048")


def test_chunked_prefill_equals_one_shot(cuda):
    """Property at the full benchmark size: a 2048-token prompt prefilled in one call
    and in two chunks (0..999, 1000..2047) gives the same cache and outputs."""
    from picolm_qwen_b200 import abi
    hq, hkv, hd, n = 32, 8, 128, 2048
    cfg = abi.Config.make(1, hq, hkv, hd, n, 1e6)
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn((n, hq * hd), generator=g, device="cuda").half()
    k = torch.randn((n, hkv * hd), generator=g, device="cuda").half()
    v = torch.randn((n, hkv * hd), generator=g, device="cuda").half()
    qn = 1 + 0.1 * torch.randn(hd, generator=g, device="cuda")
    kn = 1 + 0.1 * torch.randn(hd, generator=g, device="cuda")
    a, b = state(cfg), state(cfg)
    oa = torch.empty((n, hq * hd), device="cuda")
    ob = torch.empty_like(oa)
    assert a.prefill(0, 0, q, k, v, oa, qn, kn) == 0
    assert b.prefill(0, 0, q[:1000], k[:1000], v[:1000], ob[:1000], qn, kn) == 0
    assert b.prefill(0, 1000, q[1000:], k[1000:], v[1000:], ob[1000:], qn, kn) == 0
    torch.cuda.synchronize()
    assert torch.equal(a.k_cache, b.k_cache) and torch.equal(a.v_cache, b.v_cache)
    assert_close(ob.cpu().numpy(), oa.cpu().numpy(), "chunked vs one-shot")


def test_prefill_last_token_equals_decode(cuda):
    """Property: the prefill output of the last prompt token equals a decode step
    at that position over the cache the prefill wrote (cpp/model.hpp:288 vs :462)."""
    from picolm_qwen_b200 import abi
    hq, hkv, hd, n = 32, 8, 128, 1500
    cfg = abi.Config.make(1, hq, hkv, hd, n, 1e6)
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn((n, hq * hd), generator=g, device="cuda")
    k = torch.randn((n, hkv * hd), generator=g, device="cuda")
    v = torch.randn((n, hkv * hd), generator=g, device="cuda")
    st = state(cfg)
    out = torch.empty((n, hq * hd), device="cuda")
    assert st.prefill(0, 0, q, k, v, out) == 0
    od = torch.empty(hq * hd, device="cuda")
    # re-running the decode step at the last position rewrites the same row with the same bits
    assert st.decode_one(0, n - 1, q[n - 1].contiguous(), k[n - 1].contiguous(), v[n - 1].contiguous(), od) == 0
    torch.cuda.synchronize()
    assert_close(od.cpu().numpy(), out[n - 1].cpu().numpy(), "decode vs prefill")


def test_prefill_rejects_overflowing_prompt(cuda):
    from picolm_qwen_b200 import abi
    cfg = abi.Config.make(1, 8, 2, 128, 256, 1e6)
    st = state(cfg)
    q = torch.zeros((100, 1024), device="cuda")
    k = torch.zeros((100, 256), device="cuda")
    out = torch.empty_like(q)
    assert st.prefill(0, 200, q, k, k, out) == abi.PICOATTN_ERANGE


def test_prefill_kernel_selection(cuda):
    """On a B200 the Qwen3-8B shape (32/8 heads, head_dim 128) runs the CTA-pair
    kernel; odd group sizes and head_dim 64 fall back to the one-SM kernels.  A
    CTA-pair kernel that could not be made resident would otherwise pass every
    parity test on a slower fallback."""
    from picolm_qwen_b200 import abi
    L = abi.lib()
    pick = lambda hq, hkv, hd: L.picoattn_prefill_kernel(abi.Config.make(1, hq, hkv, hd, 4096, 1e6))
    assert pick(32, 8, 128) == abi.PREFILL_CTA_PAIR
    assert pick(40, 8, 128) == abi.PREFILL_SINGLE          # Qwen2.5-32B: 5 q heads per KV head
    assert pick(28, 4, 128) == abi.PREFILL_SINGLE          # Qwen2.5-7B: 7 per KV head
    assert pick(32, 4, 64) == abi.PREFILL_HEAD_PAIR        # TinyLlama
