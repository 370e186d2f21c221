"""Projections on the B200 against the reference's own mat-vec.

picoattn_matvec is checked against TensorOps::matmul_bias compiled from the
reference's sources (oracle/_ref) for every weight format.  The weights are
dequantised bit-identically; the fp32 dot product sums in another order, so
the tolerance is on the sum's magnitude:
    |gpu - ref| <= 3e-5 * (sum_i |w_i x_i| + |bias|)      (elementwise)
picoattn_decode_layer (projections + decode step + output projection into the
residual) is checked against the same chain built from the reference's
mat-vec and the oracle's decode step, with the attention-output tolerance
    |gpu - ref| <= 2e-3 + 1e-2 * |ref|.
"""
import numpy as np
import pytest

from tests import weightgen as wg

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

FORMATS = sorted(wg.BLOCK)


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from picolm_qwen_b200 import abi
    assert abi.lib().picoattn_device_check() == 0, "not an sm_100 device"
    return torch.device("cuda")


@pytest.fixture(scope="module")
def ref():
    from oracle.pyoracle import RefHarness
    return RefHarness()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def magnitude(oracle, w, wtype, n_in, n_out, x, bias):
    W = oracle.dequant(w, wtype, n_in, n_out).astype(np.float64)
    m = np.abs(x.astype(np.float64)) @ np.abs(W).T
    return m + (0 if bias is None else np.abs(bias.astype(np.float64)))


@pytest.mark.parametrize("wtype", FORMATS, ids=[wg.NAMES[t] for t in FORMATS])
@pytest.mark.parametrize("n_in,n_out,n_vec", [(3584, 512, 1), (1024, 1000, 3), (4096, 64, 8), (512, 33, 2),
                                               (8192, 96, 1)])
def test_matvec_vs_reference(cuda, oracle, ref, wtype, n_in, n_out, n_vec):
    from picolm_qwen_b200.runtime import matvec
    rng = np.random.default_rng(wtype * 7919 + n_in + n_vec)
    w = wg.make(wtype, n_in, n_out, rng)
    x = rng.standard_normal((n_vec, n_in)).astype(np.float32)
    bias = rng.standard_normal(n_out).astype(np.float32) if n_vec != 2 else None
    exp = ref.matvec(w, wtype, bias, n_in, n_out, x)
    out = torch.full((n_vec, n_out), float("nan"), device="cuda")
    matvec(dev(w), wtype, n_in, n_out, dev(x), out, None if bias is None else dev(bias))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    bound = 3e-5 * magnitude(oracle, w, wtype, n_in, n_out, x, bias)
    err = np.abs(got.astype(np.float64) - exp)
    assert (err <= bound).all(), f"max err {err.max():.3g}, bound there {bound.flat[err.argmax()]:.3g}"
    # accumulate: the residual add (vec_add) on top of the previous contents
    res0 = rng.standard_normal((n_vec, n_out)).astype(np.float32)
    out = dev(res0)
    matvec(dev(w), wtype, n_in, n_out, dev(x), out, None if bias is None else dev(bias), accumulate=True)
    torch.cuda.synchronize()
    err = np.abs(out.cpu().numpy().astype(np.float64) - (res0.astype(np.float64) + exp))
    assert (err <= bound + 1e-6 * np.abs(res0)).all()


TC_TYPES = (13, 15)  # Q4_K, Q6_K: the integer tensor-core kernel


@pytest.mark.parametrize("wtype", TC_TYPES, ids=["Q4_K", "Q6_K"])
@pytest.mark.parametrize("n_in,n_out", [(768, 33), (256, 16), (512, 19000), (18944, 48), (2816, 1000)])
def test_matvec_tensor_core_shapes(cuda, oracle, ref, wtype, n_in, n_out):
    """Odd super-block counts (Q6_K rows then start 2 bytes off a word), ragged
    last tiles, many tiles per block and the longest rows, against the
    reference; and a rerun gives the same bits."""
    from picolm_qwen_b200.runtime import matvec
    rng = np.random.default_rng(n_in * 31 + n_out + wtype)
    w = wg.make(wtype, n_in, n_out, rng)
    x = rng.standard_normal((1, n_in)).astype(np.float32)
    bias = rng.standard_normal(n_out).astype(np.float32)
    exp = ref.matvec(w, wtype, bias, n_in, n_out, x)
    wd, xd, bd = dev(w), dev(x), dev(bias)
    out = torch.full((1, n_out), float("nan"), device="cuda")
    matvec(wd, wtype, n_in, n_out, xd, out, bd)
    again = torch.full((1, n_out), float("nan"), device="cuda")
    matvec(wd, wtype, n_in, n_out, xd, again, bd)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    bound = 3e-5 * magnitude(oracle, w, wtype, n_in, n_out, x, bias)
    err = np.abs(got.astype(np.float64) - exp)
    assert (err <= bound).all(), f"max err {err.max():.3g}, bound there {bound.flat[err.argmax()]:.3g}"
    assert np.array_equal(got.view(np.uint32), again.cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("wtype", TC_TYPES, ids=["Q4_K", "Q6_K"])
@pytest.mark.parametrize("case", ["outliers", "zero-block", "tiny-block", "all-tiny", "all-huge", "mixed-scales"])
def test_matvec_tensor_core_value_ranges(cuda, oracle, ref, wtype, case):
    """x is carried as integers scaled per 256-element super-block: elements far
    below their block's largest, blocks of zeros, blocks near the bottom and
    top of the fp32 range."""
    from picolm_qwen_b200.runtime import matvec
    n_in, n_out = 1280, 64
    rng = np.random.default_rng(sum(map(ord, case)) + wtype)
    w = wg.make(wtype, n_in, n_out, rng)
    x = rng.standard_normal((1, n_in)).astype(np.float32)
    if case == "outliers":
        x[0, [3, 300, 700]] = [4e4, -2.5e4, 1e5]
    elif case == "zero-block":
        x[0, 256:512] = 0
    elif case == "tiny-block":
        x[0, 512:768] *= 1e-33
    elif case == "all-tiny":
        x *= 1e-35
    elif case == "all-huge":
        x *= 1e25
    else:  # every super-block its own scale
        x *= (10.0 ** rng.integers(-6, 7, n_in // 256)).repeat(256).astype(np.float32)
    exp = ref.matvec(w, wtype, None, n_in, n_out, x)
    out = torch.full((1, n_out), float("nan"), device="cuda")
    matvec(dev(w), wtype, n_in, n_out, dev(x), out, None)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    bound = 3e-5 * magnitude(oracle, w, wtype, n_in, n_out, x, None)
    err = np.abs(got - exp)
    assert np.isfinite(got).all() and (err <= bound).all(), f"max err {err.max():.3g}"


@pytest.mark.parametrize("wtype", TC_TYPES, ids=["Q4_K", "Q6_K"])
def test_matvec_tensor_core_nan_input(cuda, oracle, ref, wtype):
    """A NaN in x makes every row NaN, as in the reference's fp32 loop."""
    from picolm_qwen_b200.runtime import matvec
    n_in, n_out = 512, 32
    rng = np.random.default_rng(3)
    w = wg.make(wtype, n_in, n_out, rng)
    x = rng.standard_normal((1, n_in)).astype(np.float32)
    x[0, 400] = np.nan
    out = torch.zeros((1, n_out), device="cuda")
    matvec(dev(w), wtype, n_in, n_out, dev(x), out, None)
    torch.cuda.synchronize()
    assert np.isnan(out.cpu().numpy()).all()
    assert np.isnan(ref.matvec(w, wtype, None, n_in, n_out, x)).all()


SHAPES = {
    # name: (hq, hkv, hd, dim, rope_mode, qk_norm, types q/k/v/o, biases)
    "qwen2.5-7b-q4km": (28, 4, 128, 3584, 0, False, (13, 13, 15, 13), True),
    "qwen3-8b-q8_0": (32, 8, 128, 4096, 0, True, (9, 9, 9, 9), False),
    "tinyllama-f16": (32, 4, 64, 2048, 1, False, (2, 2, 2, 2), False),
    "small-f32-q4_0": (8, 2, 128, 1024, 0, True, (1, 3, 3, 1), True),
}


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_decode_layer_vs_reference_chain(cuda, oracle, ref, name):
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, LayerProj
    hq, hkv, hd, dim, mode, qk_norm, types, biases = SHAPES[name]
    qd, kvd = hq * hd, hkv * hd
    rng = np.random.default_rng(sum(map(ord, name)))
    lens = np.array([1, 77, 600], np.int32)  # attended rows = pos + 1
    B, S, layer = len(lens), 640, 1
    cfg = abi.Config.make(2, hq, hkv, hd, S, 1e6 if mode == 0 else 1e4, mode)
    st = AttnState(cfg, n_seqs=B, max_ctx=S)
    cos_t, sin_t = oracle.rope_table(S, hd, cfg.rope_freq_base)
    kcs, vcs = [], []
    for b in range(B):
        kc = np.zeros((S, kvd), np.uint16)
        vc = np.zeros((S, kvd), np.uint16)
        n = int(lens[b]) - 1
        if n:
            kc[:n] = oracle.f32_to_f16((rng.standard_normal((n, kvd)) * 0.5).astype(np.float32)).reshape(n, kvd)
            vc[:n] = oracle.f32_to_f16((rng.standard_normal((n, kvd)) * 0.5).astype(np.float32)).reshape(n, kvd)
        kcs.append(kc)
        vcs.append(vc)
        st.k_cache[b, layer] = dev(kc.view(np.int16))
        st.v_cache[b, layer] = dev(vc.view(np.int16))
    wq = wg.make(types[0], dim, qd, rng)
    wk = wg.make(types[1], dim, kvd, rng)
    wv = wg.make(types[2], dim, kvd, rng)
    wo = wg.make(types[3], qd, dim, rng)
    bq, bk, bv, bo = ((rng.standard_normal(n) * 0.1).astype(np.float32) if biases else None
                      for n in (qd, kvd, kvd, dim))
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if qk_norm else None
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if qk_norm else None
    xb = rng.standard_normal((B, dim)).astype(np.float32)
    x0 = rng.standard_normal((B, dim)).astype(np.float32)
    # the reference chain: its mat-vec, the oracle's decode step, its mat-vec again
    q = ref.matvec(wq, types[0], bq, dim, qd, xb)
    k = ref.matvec(wk, types[1], bk, dim, kvd, xb)
    v = ref.matvec(wv, types[2], bv, dim, kvd, xb)
    pos = lens - 1
    attn = oracle.decode_batch(hq, hkv, hd, mode, q, k, v, qn, kn, cos_t, sin_t, kcs, vcs, pos, n_threads=8)
    x_ref = x0 + ref.matvec(wo, types[3], bo, qd, dim, attn)
    # the library: one call
    d = lambda a: None if a is None else dev(a)
    proj = LayerProj(dev(wq), dev(wk), dev(wv), dev(wo), types, d(bq), d(bk), d(bv), d(bo))
    x = dev(x0)
    st.decode_layer(layer, dim, dev(xb), proj, dev(pos), x, d(qn), d(kn))
    torch.cuda.synchronize()
    assert st.status() == 0
    got = x.cpu().numpy()
    err = np.abs(got.astype(np.float64) - x_ref)
    bound = 2e-3 + 1e-2 * np.abs(x_ref)
    assert (err <= bound).all(), f"max err {err.max():.3g} (ref {x_ref.flat[err.argmax()]:.3g})"
    # the new cache rows: the reference's fp16 rounding of projections that agree
    # to fp32 rounding, so equal or one fp16 ulp apart
    for b in range(B):
        for c, refc in ((st.k_cache, kcs), (st.v_cache, vcs)):
            row = c[b, layer, pos[b]].cpu().numpy().view(np.uint16).astype(np.int32)
            diff = np.abs(row - refc[b][pos[b]].astype(np.int32))
            assert diff.max() <= 1, f"seq {b}: cache row off by {diff.max()} fp16 steps"


def test_decode_layer_graph_replay_matches_eager(cuda, oracle):
    """The whole layer chain captured once and replayed gives the eager result."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, LayerProj
    hq, hkv, hd, dim = 28, 4, 128, 3584
    rng = np.random.default_rng(5)
    cfg = abi.Config.make(1, hq, hkv, hd, 4096, 1e6)
    st = AttnState(cfg, n_seqs=1, max_ctx=4096)
    st.k_cache.copy_(torch.randint(-12000, 12000, st.k_cache.shape, dtype=torch.int16, device="cuda") & 0x3BFF)
    st.v_cache.copy_(torch.randint(-12000, 12000, st.v_cache.shape, dtype=torch.int16, device="cuda") & 0x3BFF)
    types = (13, 13, 15, 13)
    ws = [dev(wg.make(t, n_in, n_out, rng)) for t, n_in, n_out in
          zip(types, (dim, dim, dim, hq * hd), (hq * hd, hkv * hd, hkv * hd, dim))]
    proj = LayerProj(*ws, types)
    xb = dev(rng.standard_normal((1, dim)).astype(np.float32))
    pos = torch.tensor([3000], dtype=torch.int32, device="cuda")
    kc0, vc0 = st.k_cache.clone(), st.v_cache.clone()
    x = torch.zeros((1, dim), device="cuda")
    st.decode_layer(0, dim, xb, proj, pos, x)
    torch.cuda.synchronize()
    eager = x.clone()
    st.k_cache.copy_(kc0)
    st.v_cache.copy_(vc0)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        x.zero_()
        with torch.cuda.graph(g, stream=s):
            st.decode_layer(0, dim, xb, proj, pos, x, stream=s)
    for _ in range(3):
        x.zero_()
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(x, eager)
    assert st.status() == 0


def test_public_matvec_then_decode_one_back_to_back(cuda, oracle, ref):
    """A host that runs its projections with picoattn_matvec and then calls
    picoattn_decode_one on the same stream, with no synchronisation between
    them.  The projection kernel lets the next kernel launch before it has
    stored its outputs, so the decode kernels must wait for it before they read
    q, k and v: outputs and new cache rows must match the reference chain on
    every one of several repetitions."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, matvec
    hq, hkv, hd, dim, S = 28, 4, 128, 3584, 4096
    qd, kvd = hq * hd, hkv * hd
    rng = np.random.default_rng(77)
    cfg = abi.Config.make(1, hq, hkv, hd, S, 1e6)
    st = AttnState(cfg, n_seqs=1, max_ctx=S)
    n = 4000  # cached rows; the new token sits at pos n
    kc = np.zeros((S, kvd), np.uint16)
    vc = np.zeros((S, kvd), np.uint16)
    kc[:n] = oracle.f32_to_f16((rng.standard_normal((n, kvd)) * 0.5).astype(np.float32)).reshape(n, kvd)
    vc[:n] = oracle.f32_to_f16((rng.standard_normal((n, kvd)) * 0.5).astype(np.float32)).reshape(n, kvd)
    types = (13, 13, 15)
    wq, wk, wv = (wg.make(t, dim, n_out, rng) for t, n_out in zip(types, (qd, kvd, kvd)))
    dwq, dwk, dwv = dev(wq), dev(wk), dev(wv)
    cos_t, sin_t = oracle.rope_table(S, hd, 1e6)
    q_buf = torch.empty((1, qd), device="cuda")
    k_buf = torch.empty((1, kvd), device="cuda")
    v_buf = torch.empty((1, kvd), device="cuda")
    out = torch.empty(qd, device="cuda")
    for rep in range(4):
        xb = rng.standard_normal((1, dim)).astype(np.float32)
        q = ref.matvec(wq, types[0], None, dim, qd, xb)
        k = ref.matvec(wk, types[1], None, dim, kvd, xb)
        v = ref.matvec(wv, types[2], None, dim, kvd, xb)
        kr, vr = kc.copy(), vc.copy()
        want, _, _ = oracle.decode_step(hq, hkv, hd, 0, q[0], k[0], v[0], None, None, cos_t, sin_t, kr, vr, n)
        st.k_cache[0, 0] = dev(kc.view(np.int16))
        st.v_cache[0, 0] = dev(vc.view(np.int16))
        dxb = dev(xb)
        for buf in (q_buf, k_buf, v_buf, out):
            buf.fill_(float("nan"))
        matvec(dwq, types[0], dim, qd, dxb, q_buf)
        matvec(dwk, types[1], dim, kvd, dxb, k_buf)
        matvec(dwv, types[2], dim, kvd, dxb, v_buf)
        assert st.decode_one(0, n, q_buf, k_buf, v_buf, out) == 0
        torch.cuda.synchronize()
        assert st.status() == 0
        got = out.cpu().numpy()
        err = np.abs(got.astype(np.float64) - want)
        assert (err <= 2e-3 + 1e-2 * np.abs(want)).all(), f"rep {rep}: max err {np.nanmax(err):.3g}"
        # the new rows: fp16 of projections that agree to fp32 rounding (values near
        # zero after cancellation may sit a few fp16 steps apart), so compared by value
        for c, r in ((st.k_cache, kr), (st.v_cache, vr)):
            row = c[0, 0, n].cpu().numpy().view(np.float16).astype(np.float64)
            rv = r[n].view(np.float16).astype(np.float64)
            assert (np.abs(row - rv) <= 2e-3 + 1e-2 * np.abs(rv)).all(), f"rep {rep}: new cache row"
