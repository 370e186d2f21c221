"""Decode attention on the B200 against the reference (golden fixtures) and the oracle.

Tolerance on the attention output, from the task's parity bar:
    |gpu - ref| <= 2e-3 + 1e-2 * |ref|   elementwise.
The KV-cache row written at `pos` must equal the reference's fp16 bits exactly
(integer work: cpp/quant.hpp:102-135 rounding of the same fp32 values).
"""
import ctypes as C
import glob
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
    bound = ATOL + RTOL * np.abs(ref)
    bad = ~(err <= bound)
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside tolerance, "
                           f"max err {err.max():.3g} (ref there {ref.flat[err.argmax()]:.3g})")


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from picolm_qwen_b200 import abi
    assert abi.lib().picoattn_device_check() == 0, "not an sm_100 device"
    return torch.device("cuda")


def make_state(cfg, n_seqs=1, max_ctx=None):
    from picolm_qwen_b200.runtime import AttnState
    return AttnState(cfg, n_seqs=n_seqs, max_ctx=max_ctx)


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


DECODE_FILES = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "decode_*.npz")))


@pytest.mark.parametrize("path", DECODE_FILES, ids=[os.path.basename(p)[7:-4] for p in DECODE_FILES])
def test_decode_matches_reference_golden(cuda, path):
    from picolm_qwen_b200 import abi
    g = np.load(path)
    hq, hkv, hd = int(g["hq"]), int(g["hkv"]), int(g["hd"])
    last, keep = int(g["last_pos"]), int(g["keep"])
    S = last + 1
    layer, n_layers = 1, 3  # a non-zero layer checks the slab offset l*S*kv_dim
    cfg = abi.Config.make(n_layers, hq, hkv, hd, S, float(g["rope_base"]), int(g["rope_mode"]))
    st = make_state(cfg)
    first = last - keep + 1
    kc = g["kcache"].view(np.int16)
    vc = g["vcache"].view(np.int16)
    st.k_cache[0, layer, :first] = dev(kc[:first])
    st.v_cache[0, layer, :first] = dev(vc[:first])
    qn = dev(g["q_norm_w"]) if "q_norm_w" in g else None
    kn = dev(g["k_norm_w"]) if "k_norm_w" in g else None
    out = torch.empty(hq * hd, dtype=torch.float32, device="cuda")
    for i in range(keep):
        pos = first + i
        status = st.decode_one(layer, pos, dev(g["q"][i]), dev(g["k"][i]), dev(g["v"][i]), out, qn, kn)
        assert status == 0, abi.lib().picoattn_strerror(status)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), g["out"][i], f"pos {pos}")
        assert np.array_equal(st.k_cache[0, layer, pos].cpu().numpy(), kc[pos]), f"k row {pos}"
        assert np.array_equal(st.v_cache[0, layer, pos].cpu().numpy(), vc[pos]), f"v row {pos}"
    # nothing else in the cache moved
    assert int(st.k_cache[0, 0].abs().sum()) == 0 and int(st.k_cache[0, 2].abs().sum()) == 0
    assert st.status() == 0


def random_cache_rows(oracle, rng, n_rows, kvd, sd=0.5):
    k = (rng.standard_normal((n_rows, kvd)) * sd).astype(np.float32)
    v = (rng.standard_normal((n_rows, kvd)) * sd).astype(np.float32)
    return oracle.f32_to_f16(k).reshape(n_rows, kvd), oracle.f32_to_f16(v).reshape(n_rows, kvd)


@pytest.mark.parametrize("shape", [
    (28, 4, 128, 0),   # Qwen2.5-7B (cfg 3)
    (32, 4, 64, 1),    # TinyLlama, interleaved RoPE (cfg 1)
    (14, 2, 64, 0),    # Qwen2.5-0.5B (cfg 2)
    (40, 8, 128, 0),   # Qwen2.5-32B (cfg 5)
    (16, 1, 128, 0),   # one KV head, 16 q heads per group
    (4, 4, 64, 0),     # MHA
])
def test_batched_ragged_decode_vs_oracle(cuda, oracle, shape):
    from picolm_qwen_b200 import abi
    hq, hkv, hd, mode = shape
    rng = np.random.default_rng(hq * 1000 + hkv * 10 + hd)
    lens = np.array([1, 2, 17, 300, 1500, 4100], np.int32)  # attended rows = pos + 1
    B, S = len(lens), int(lens.max()) + 8
    kvd = hkv * hd
    cfg = abi.Config.make(2, hq, hkv, hd, S, 1e6 if mode == 0 else 1e4, mode)
    st = make_state(cfg, n_seqs=B, max_ctx=int(lens.max()))
    cos_t, sin_t = oracle.rope_table(S, hd, cfg.rope_freq_base)
    kcs, vcs = [], []
    layer = 1
    for b in range(B):
        kc = np.zeros((S, kvd), np.uint16)
        vc = np.zeros((S, kvd), np.uint16)
        n = int(lens[b]) - 1
        if n:
            kc[:n], vc[:n] = random_cache_rows(oracle, rng, n, kvd)
        kcs.append(kc)
        vcs.append(vc)
        st.k_cache[b, layer] = dev(kc.view(np.int16))
        st.v_cache[b, layer] = dev(vc.view(np.int16))
    q = rng.standard_normal((B, hq * hd)).astype(np.float32)
    k = rng.standard_normal((B, kvd)).astype(np.float32)
    v = rng.standard_normal((B, kvd)).astype(np.float32)
    pos = lens - 1
    ref = oracle.decode_batch(hq, hkv, hd, mode, q, k, v, None, None, cos_t, sin_t, kcs, vcs, pos, n_threads=8)
    out = torch.empty((B, hq * hd), dtype=torch.float32, device="cuda")
    st.decode(layer, dev(q), dev(k), dev(v), dev(pos), out)
    torch.cuda.synchronize()
    assert st.status() == 0
    got = out.cpu().numpy()
    for b in range(B):
        assert_close(got[b], ref[b], f"seq {b} len {lens[b]}")
        assert np.array_equal(st.k_cache[b, layer, pos[b]].cpu().numpy().view(np.uint16), kcs[b][pos[b]])
        assert np.array_equal(st.v_cache[b, layer, pos[b]].cpu().numpy().view(np.uint16), vcs[b][pos[b]])


def test_long_context_split_kv_vs_oracle(cuda, oracle):
    """Qwen2.5-32B shape at 24k rows: many chunks merged by log-sum-exp."""
    from picolm_qwen_b200 import abi
    hq, hkv, hd = 40, 8, 128
    n_ctx = 24000
    S = n_ctx
    kvd = hkv * hd
    rng = np.random.default_rng(5)
    cfg = abi.Config.make(1, hq, hkv, hd, S, 1e6)
    st = make_state(cfg)
    kc = np.zeros((S, kvd), np.uint16)
    vc = np.zeros((S, kvd), np.uint16)
    kc[:n_ctx - 1], vc[:n_ctx - 1] = random_cache_rows(oracle, rng, n_ctx - 1, kvd)
    st.k_cache[0, 0] = dev(kc.view(np.int16))
    st.v_cache[0, 0] = dev(vc.view(np.int16))
    q = rng.standard_normal(hq * hd).astype(np.float32)
    k = rng.standard_normal(kvd).astype(np.float32)
    v = rng.standard_normal(kvd).astype(np.float32)
    cos_t, sin_t = oracle.rope_table(S, hd, 1e6)
    ref = oracle.decode_batch(hq, hkv, hd, 0, q[None], k[None], v[None], None, None, cos_t, sin_t,
                              [kc], [vc], np.array([n_ctx - 1], np.int32), n_threads=1)[0]
    out = torch.empty(hq * hd, dtype=torch.float32, device="cuda")
    assert st.decode_one(0, n_ctx - 1, dev(q), dev(k), dev(v), out) == 0
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), ref, "24k context")


def test_position_zero_returns_v_exactly(cuda):
    """At pos 0 the only visible row is the new one: out = fp16(v) widened."""
    from picolm_qwen_b200 import abi
    cfg = abi.Config.make(1, 28, 4, 128, 64, 1e6)
    st = make_state(cfg)
    rng = np.random.default_rng(0)
    q = rng.standard_normal(28 * 128).astype(np.float32)
    k = rng.standard_normal(512).astype(np.float32)
    v = rng.standard_normal(512).astype(np.float32)
    out = torch.empty(28 * 128, dtype=torch.float32, device="cuda")
    assert st.decode_one(0, 0, dev(q), dev(k), dev(v), out) == 0
    torch.cuda.synchronize()
    vrow = st.v_cache[0, 0, 0].cpu().numpy().view(np.uint16)
    vf = vrow.view(np.float16).astype(np.float32)
    want = np.concatenate([vf[(h // 7) * 128:(h // 7 + 1) * 128] for h in range(28)])
    assert np.array_equal(out.cpu().numpy(), want)


def test_uniform_keys_average_values(cuda, oracle):
    """Identical keys give identical scores, so the output is the mean of V."""
    from picolm_qwen_b200 import abi
    hq, hkv, hd, n = 8, 2, 64, 700
    kvd = hkv * hd
    cfg = abi.Config.make(1, hq, hkv, hd, n, 1e4)
    st = make_state(cfg)
    rng = np.random.default_rng(1)
    # the new token's k is rotated at position n-1; give every cached row that same rotated key
    cos_t, sin_t = oracle.rope_table(n, hd, 1e4)
    k = rng.standard_normal(kvd).astype(np.float32)
    _, krot = oracle.rope(0, np.zeros(hq * hd, np.float32), k, hd, hq, hkv, cos_t[n - 1], sin_t[n - 1])
    krow = oracle.f32_to_f16(krot)
    vrows = oracle.f32_to_f16(rng.standard_normal((n - 1, kvd)).astype(np.float32)).reshape(n - 1, kvd)
    st.k_cache[0, 0, :n - 1] = dev(np.tile(krow, (n - 1, 1)).view(np.int16))
    st.v_cache[0, 0, :n - 1] = dev(vrows.view(np.int16))
    q = rng.standard_normal(hq * hd).astype(np.float32)
    v = rng.standard_normal(kvd).astype(np.float32)
    out = torch.empty(hq * hd, dtype=torch.float32, device="cuda")
    assert st.decode_one(0, n - 1, dev(q), dev(k), dev(v), out) == 0
    torch.cuda.synchronize()
    allv = np.concatenate([oracle.f16_to_f32(vrows.ravel()).reshape(n - 1, kvd),
                           oracle.f16_to_f32(oracle.f32_to_f16(v))[None]], 0)
    mean = allv.mean(0)
    want = np.concatenate([mean[(h // 4) * hd:(h // 4 + 1) * hd] for h in range(hq)])
    assert_close(out.cpu().numpy(), want, "mean of V")


def test_bad_device_position_is_flagged_not_faulted(cuda):
    from picolm_qwen_b200 import abi
    cfg = abi.Config.make(1, 8, 2, 64, 128, 1e4)
    st = make_state(cfg, n_seqs=3, max_ctx=100)
    q = torch.randn(3, 512, device="cuda")
    k = torch.randn(3, 128, device="cuda")
    v = torch.randn(3, 128, device="cuda")
    out = torch.zeros(3, 512, device="cuda")
    pos = torch.tensor([5, 100, -1], dtype=torch.int32, device="cuda")  # 100 >= max_ctx, -1 < 0
    st.decode(0, q, k, v, pos, out, max_ctx=100)
    torch.cuda.synchronize()
    assert st.status() & abi.DEV_BAD_POS
    o = out.cpu().numpy()
    assert np.isfinite(o[0]).all() and np.isnan(o[1]).all() and np.isnan(o[2]).all()
    assert st.status() == 0  # reading cleared it
    # nothing was written for the rejected sequences
    assert int(st.k_cache[1].abs().sum()) == 0 and int(st.k_cache[2].abs().sum()) == 0


def test_decode_is_deterministic(cuda):
    from picolm_qwen_b200 import abi
    cfg = abi.Config.make(1, 28, 4, 128, 4096, 1e6)
    st = make_state(cfg, n_seqs=2)
    st.k_cache.random_(-20000, 20000)
    st.v_cache.random_(-20000, 20000)
    st.k_cache &= 0x3bff  # keep every pattern a finite fp16 below 1.0
    st.v_cache &= 0x3bff
    q = torch.randn(2, 28 * 128, device="cuda")
    k = torch.randn(2, 512, device="cuda")
    v = torch.randn(2, 512, device="cuda")
    pos = torch.tensor([4095, 3000], dtype=torch.int32, device="cuda")
    o1 = torch.empty(2, 28 * 128, device="cuda")
    o2 = torch.empty_like(o1)
    st.decode(0, q, k, v, pos, o1)
    st.decode(0, q, k, v, pos, o2)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.isfinite(o1).all()


@pytest.mark.parametrize("shape", [(40, 8, 128), (14, 2, 64), (16, 1, 128)])
def test_single_sequence_short_rows_many_ctas_vs_oracle(cuda, oracle, shape):
    """One sequence whose 31 rows are fewer than the CTAs sized for max_ctx:
    most slices are empty, the attention kernel appends the new row itself and
    the merge derives the rows from the position."""
    from picolm_qwen_b200 import abi
    hq, hkv, hd = shape
    n, S = 31, 4096
    kvd = hkv * hd
    rng = np.random.default_rng(hq + hkv + hd)
    cfg = abi.Config.make(2, hq, hkv, hd, S, 1e6)
    st = make_state(cfg, n_seqs=1, max_ctx=S)
    kc = np.zeros((S, kvd), np.uint16)
    vc = np.zeros((S, kvd), np.uint16)
    kc[:n - 1], vc[:n - 1] = random_cache_rows(oracle, rng, n - 1, kvd)
    st.k_cache[0, 1] = dev(kc.view(np.int16))
    st.v_cache[0, 1] = dev(vc.view(np.int16))
    q = rng.standard_normal((1, hq * hd)).astype(np.float32)
    k = rng.standard_normal((1, kvd)).astype(np.float32)
    v = rng.standard_normal((1, kvd)).astype(np.float32)
    cos_t, sin_t = oracle.rope_table(S, hd, 1e6)
    pos = np.array([n - 1], np.int32)
    ref = oracle.decode_batch(hq, hkv, hd, 0, q, k, v, None, None, cos_t, sin_t, [kc], [vc], pos, n_threads=1)
    out = torch.empty((1, hq * hd), dtype=torch.float32, device="cuda")
    st.decode(1, dev(q), dev(k), dev(v), dev(pos), out, max_ctx=S)
    torch.cuda.synchronize()
    assert st.status() == 0
    assert_close(out.cpu().numpy()[0], ref[0], f"{shape}")
    _, krot = oracle.rope(0, np.zeros(hq * hd, np.float32), k[0], hd, hq, hkv, cos_t[n - 1], sin_t[n - 1])
    assert np.array_equal(st.k_cache[0, 1, n - 1].cpu().numpy().view(np.uint16), oracle.f32_to_f16(krot))
    assert np.array_equal(st.v_cache[0, 1, n - 1].cpu().numpy().view(np.uint16), oracle.f32_to_f16(v[0]))


def test_single_sequence_layer_chain_graph_replay(cuda):
    """Consecutive single-sequence calls over several layers, captured in one
    CUDA graph and replayed: each launch may start while the one before it
    finishes (programmatic dependent launch); replays give the eager results
    bit for bit."""
    from picolm_qwen_b200 import abi
    hq, hkv, hd, L, S = 40, 8, 128, 4, 20000
    cfg = abi.Config.make(L, hq, hkv, hd, S, 1e6)
    st = make_state(cfg, n_seqs=1, max_ctx=S)
    st.k_cache.random_(-20000, 20000)
    st.v_cache.random_(-20000, 20000)
    st.k_cache &= 0x3bff
    st.v_cache &= 0x3bff
    q = torch.randn(L, 1, hq * hd, device="cuda")
    k = torch.randn(L, 1, hkv * hd, device="cuda")
    v = torch.randn(L, 1, hkv * hd, device="cuda")
    pos = torch.tensor([S - 1], dtype=torch.int32, device="cuda")
    eager = torch.empty(L, 1, hq * hd, device="cuda")
    for l in range(L):
        st.decode(l, q[l], k[l], v[l], pos, eager[l])
    torch.cuda.synchronize()
    assert st.status() == 0
    out = torch.zeros_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        st.decode(0, q[0], k[0], v[0], pos, out[0], stream=s)  # warm-up on the capture stream
        s.synchronize()
        with torch.cuda.graph(g, stream=s):
            for l in range(L):
                st.decode(l, q[l], k[l], v[l], pos, out[l], stream=s)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    assert st.status() == 0
    del g


def test_single_sequence_bad_position_is_flagged(cuda):
    from picolm_qwen_b200 import abi
    cfg = abi.Config.make(1, 40, 8, 128, 1024, 1e6)
    st = make_state(cfg, n_seqs=1, max_ctx=1024)
    q = torch.randn(1, 40 * 128, device="cuda")
    k = torch.randn(1, 1024, device="cuda")
    v = torch.randn(1, 1024, device="cuda")
    out = torch.zeros(1, 40 * 128, device="cuda")
    st.decode(0, q, k, v, torch.tensor([-3], dtype=torch.int32, device="cuda"), out)
    torch.cuda.synchronize()
    assert st.status() & abi.DEV_BAD_POS
    assert np.isnan(out.cpu().numpy()).all()
    assert int(st.k_cache.abs().sum()) == 0
    # the workspace stays usable
    st.decode(0, q, k, v, torch.tensor([100], dtype=torch.int32, device="cuda"), out)
    torch.cuda.synchronize()
    assert st.status() == 0 and torch.isfinite(out).all()


@pytest.mark.parametrize("n_ctx", [900, 24000])
def test_single_sequence_staged_calls_vs_oracle(cuda, oracle, n_ctx):
    """One sequence with its stages in separate calls (prep kernel, attention
    kernel, merge kernel), against the oracle; and the one-call form (the
    attention kernel appending the new row itself) on the same inputs."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import stream_handle
    hq, hkv, hd = 40, 8, 128
    kvd = hkv * hd
    rng = np.random.default_rng(n_ctx)
    cfg = abi.Config.make(1, hq, hkv, hd, n_ctx, 1e6)
    st = make_state(cfg)
    kc = np.zeros((n_ctx, kvd), np.uint16)
    vc = np.zeros((n_ctx, kvd), np.uint16)
    kc[:n_ctx - 1], vc[:n_ctx - 1] = random_cache_rows(oracle, rng, n_ctx - 1, kvd)
    q = rng.standard_normal((1, hq * hd)).astype(np.float32)
    k = rng.standard_normal((1, kvd)).astype(np.float32)
    v = rng.standard_normal((1, kvd)).astype(np.float32)
    cos_t, sin_t = oracle.rope_table(n_ctx, hd, 1e6)
    pos = np.array([n_ctx - 1], np.int32)
    ref = oracle.decode_batch(hq, hkv, hd, 0, q, k, v, None, None, cos_t, sin_t, [kc.copy()], [vc.copy()], pos,
                              n_threads=8)[0]
    L = abi.lib()
    dq, dk, dv, dpos = dev(q), dev(k), dev(v), dev(pos)
    for staged in (True, False):
        st.k_cache[0, 0] = dev(kc.view(np.int16))
        st.v_cache[0, 0] = dev(vc.view(np.int16))
        out = torch.full((1, hq * hd), float("nan"), device="cuda")
        args = (C.byref(cfg), 0, 1, n_ctx, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), None, None,
                st.rope_cos.data_ptr(), st.rope_sin.data_ptr(), st.k_ptrs.data_ptr(), st.v_ptrs.data_ptr(),
                dpos.data_ptr(), out.data_ptr(), st.workspace.data_ptr(), st.workspace.numel(), stream_handle())
        stage_list = (abi.STAGE_PREPARE, abi.STAGE_ATTEND, abi.STAGE_COMBINE) if staged else (abi.STAGE_ALL,)
        for stg in stage_list:
            assert L.picoattn_decode_staged(*args, stg) == 0
        torch.cuda.synchronize()
        assert st.status() == 0
        assert_close(out.cpu().numpy()[0], ref, f"{'staged' if staged else 'one call'} {n_ctx}")
