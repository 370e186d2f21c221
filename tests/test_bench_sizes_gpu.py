"""Decode parity at the sizes the benchmark runs, and the fp16 rounding edge cases on the device.

The benchmark's configurations select launch shapes that smaller tests do not
reach: a 131072-row sequence puts four merge blocks beside the attention grid
(8 at a 65536-row shard, 16 at a 16384-row shard), and 64 ragged sequences of
1024..8192 rows spread over the whole persistent grid.  Each case here runs the
library at that exact size through the C ABI and compares with the oracle's
restatement of the reference loop (cpp/model.hpp:354-418):

    attention output  |gpu - ref| <= 2e-3 + 1e-2 * |ref|   elementwise
    new cache row     the reference's fp16 bits exactly (cpp/quant.hpp:102-135)

The rounding cases feed the reference's own fp32 -> fp16 edge vectors (ties,
subnormals, 65519/65520 overflow, infinities, NaN payloads; tests/golden/
numerics.npz) through every kernel that stores a cache row and compare the
stored bits with the reference's.
"""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2
THREADS = os.cpu_count() or 1


def assert_close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    bad = ~(err <= ATOL + RTOL * np.abs(ref))
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside tolerance, "
                           f"max err {err.max():.3g}")


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from picolm_qwen_b200 import abi
    assert abi.lib().picoattn_device_check() == 0


def fp16_rows(rng, n, kvd):
    """Cache rows: N(0, 0.5^2) values as fp16 bit patterns."""
    return (rng.standard_normal((n, kvd), dtype=np.float32) * 0.5).astype(np.float16).view(np.uint16)


# ---------------------------------------------------------------------------
# config 5: Qwen2.5-32B heads, 131071 cached rows + the new token
# ---------------------------------------------------------------------------

S5 = 131072
HQ5, HKV5, HD5 = 40, 8, 128


@pytest.fixture(scope="module")
def cfg5(cuda, oracle):
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import rope_table
    kvd = HKV5 * HD5
    rng = np.random.default_rng(131072)
    kc = np.zeros((S5, kvd), np.uint16)
    vc = np.zeros((S5, kvd), np.uint16)
    kc[:S5 - 1] = fp16_rows(rng, S5 - 1, kvd)
    vc[:S5 - 1] = fp16_rows(rng, S5 - 1, kvd)
    q = rng.standard_normal(HQ5 * HD5).astype(np.float32)
    k = rng.standard_normal(kvd).astype(np.float32)
    v = rng.standard_normal(kvd).astype(np.float32)
    cfg = abi.Config.make(1, HQ5, HKV5, HD5, S5, 1e6)
    cos, sin = rope_table(cfg)
    dk = torch.from_numpy(kc.view(np.int16)).cuda()
    dv = torch.from_numpy(vc.view(np.int16)).cuda()
    ref_k, ref_v = kc.copy(), vc.copy()
    ref = oracle.decode_step_mt(HQ5, HKV5, HD5, 0, q, k, v, None, None, cos, sin, ref_k, ref_v, S5 - 1,
                                n_threads=THREADS)
    return dict(cfg=cfg, cos=torch.from_numpy(cos).cuda(), sin=torch.from_numpy(sin).cuda(), dk=dk, dv=dv,
                q=torch.from_numpy(q).cuda(), k=torch.from_numpy(k).cuda(), v=torch.from_numpy(v).cuda(),
                ref=ref, ref_k=ref_k[S5 - 1].copy(), ref_v=ref_v[S5 - 1].copy())


def test_cfg5_full_context_one_gpu_vs_oracle(cfg5):
    """The bench's single-GPU long-context call: picoattn_decode, one sequence,
    max_ctx = 131072 (attention grid beside four merge blocks)."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import stream_handle
    L = abi.lib()
    c = cfg5
    cfg = c["cfg"]
    c["dk"][S5 - 1].zero_()
    c["dv"][S5 - 1].zero_()
    kp = torch.tensor([c["dk"].data_ptr()], dtype=torch.int64, device="cuda")
    vp = torch.tensor([c["dv"].data_ptr()], dtype=torch.int64, device="cuda")
    pos = torch.tensor([S5 - 1], dtype=torch.int32, device="cuda")
    ws_n = L.picoattn_decode_workspace_size(C.byref(cfg), 1, S5)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    out = torch.full((HQ5 * HD5,), float("nan"), device="cuda")
    st = L.picoattn_decode(C.byref(cfg), 0, 1, S5, c["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(), None,
                           None, c["cos"].data_ptr(), c["sin"].data_ptr(), kp.data_ptr(), vp.data_ptr(),
                           pos.data_ptr(), out.data_ptr(), ws.data_ptr(), ws_n, stream_handle())
    assert st == 0, L.picoattn_strerror(st)
    torch.cuda.synchronize()
    status = C.c_uint32(0)
    assert L.picoattn_workspace_status(ws.data_ptr(), stream_handle(), C.byref(status)) == 0
    assert status.value == 0
    assert_close(out.cpu().numpy(), c["ref"], "131072 rows")
    assert np.array_equal(c["dk"][S5 - 1].cpu().numpy().view(np.uint16), c["ref_k"])
    assert np.array_equal(c["dv"][S5 - 1].cpu().numpy().view(np.uint16), c["ref_v"])


@pytest.mark.parametrize("n_shards", [2, 8])
def test_cfg5_shards_of_the_multi_gpu_runs_vs_oracle(cfg5, n_shards):
    """The per-rank shard shapes of the 2- and 8-GPU long-context runs (65536 and
    16384 rows: eight and sixteen merge blocks), each shard through
    picoattn_decode_shard on its own slab, combined by picoattn_combine_shards."""
    from picolm_qwen_b200 import abi, sharding
    from picolm_qwen_b200.runtime import stream_handle
    L = abi.lib()
    c = cfg5
    cfg = c["cfg"]
    kvd = HKV5 * HD5
    c["dk"][S5 - 1].zero_()
    c["dv"][S5 - 1].zero_()
    pos = torch.tensor([S5 - 1], dtype=torch.int32, device="cuda")
    parts = torch.full((n_shards, HQ5 * (HD5 + 2)), float("nan"), device="cuda")
    sh = stream_handle()
    keep = []
    for s in range(n_shards):
        off, rows = sharding.shard_rows(S5, n_shards, s)
        # one layer: the shard's slab is rows [off, off + rows) of the full cache
        kp = torch.tensor([c["dk"].data_ptr() + off * kvd * 2], dtype=torch.int64, device="cuda")
        vp = torch.tensor([c["dv"].data_ptr() + off * kvd * 2], dtype=torch.int64, device="cuda")
        ws_n = L.picoattn_decode_workspace_size(C.byref(cfg), 1, rows)
        ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
        st = L.picoattn_decode_shard(C.byref(cfg), 0, 1, rows, off, rows, c["q"].data_ptr(), c["k"].data_ptr(),
                                     c["v"].data_ptr(), None, None, c["cos"].data_ptr(), c["sin"].data_ptr(),
                                     kp.data_ptr(), vp.data_ptr(), pos.data_ptr(), parts[s].data_ptr(),
                                     ws.data_ptr(), ws_n, sh)
        assert st == 0, L.picoattn_strerror(st)
        keep.append((kp, vp, ws))
    out = torch.full((HQ5 * HD5,), float("nan"), device="cuda")
    assert L.picoattn_combine_shards(C.byref(cfg), 1, n_shards, parts.data_ptr(), out.data_ptr(), sh) == 0
    torch.cuda.synchronize()
    for kp, vp, ws in keep:
        status = C.c_uint32(0)
        assert L.picoattn_workspace_status(ws.data_ptr(), sh, C.byref(status)) == 0 and status.value == 0
    assert_close(out.cpu().numpy(), c["ref"], f"{n_shards} shards of {S5 // n_shards} rows")
    assert np.array_equal(c["dk"][S5 - 1].cpu().numpy().view(np.uint16), c["ref_k"])
    assert np.array_equal(c["dv"][S5 - 1].cpu().numpy().view(np.uint16), c["ref_v"])


# ---------------------------------------------------------------------------
# config 3: Qwen2.5-7B heads, the bench's 64 sequences (seed-0 lengths)
# ---------------------------------------------------------------------------

def test_cfg3_full_batch_vs_oracle(cuda, oracle):
    """One layer of the bench's batched step: 64 sequences with the bench's own
    cached lengths (U{1024..8192}, seed 0), new tokens at pos = length."""
    from bench import seq_lengths, WORKLOAD
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState
    w = WORKLOAD
    hq, hkv, hd = w["n_heads"], w["n_kv_heads"], w["head_dim"]
    kvd = hkv * hd
    lens = seq_lengths(0)
    assert len(lens) == 64 and lens.min() >= 1024 and lens.max() <= 8192
    B, S = len(lens), int(lens.max()) + 1
    layer = 1
    cfg = abi.Config.make(2, hq, hkv, hd, S, w["rope_base"], abi.ROPE_NEOX)
    st = AttnState(cfg, n_seqs=B, max_ctx=S)  # the bench's state: max_ctx = longest length + 1
    rng = np.random.default_rng(64)
    kcs, vcs = [], []
    for b in range(B):
        n = int(lens[b])
        kc = np.zeros((S, kvd), np.uint16)
        vc = np.zeros((S, kvd), np.uint16)
        kc[:n] = fp16_rows(rng, n, kvd)
        vc[:n] = fp16_rows(rng, n, kvd)
        st.k_cache[b, layer] = torch.from_numpy(kc.view(np.int16)).cuda()
        st.v_cache[b, layer] = torch.from_numpy(vc.view(np.int16)).cuda()
        kcs.append(kc)
        vcs.append(vc)
    q = rng.standard_normal((B, hq * hd)).astype(np.float32)
    k = rng.standard_normal((B, kvd)).astype(np.float32)
    v = rng.standard_normal((B, kvd)).astype(np.float32)
    cos_t, sin_t = st.rope_cos.cpu().numpy(), st.rope_sin.cpu().numpy()
    pos = lens.astype(np.int32)
    ref = oracle.decode_batch(hq, hkv, hd, 0, q, k, v, None, None, cos_t, sin_t, kcs, vcs, pos, n_threads=THREADS)
    out = torch.full((B, hq * hd), float("nan"), device="cuda")
    st.decode(layer, torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
              torch.from_numpy(pos).cuda(), out)
    torch.cuda.synchronize()
    assert st.status() == 0
    got = out.cpu().numpy()
    for b in range(B):
        assert_close(got[b], ref[b], f"seq {b} len {lens[b]}")
        assert np.array_equal(st.k_cache[b, layer, pos[b]].cpu().numpy().view(np.uint16), kcs[b][pos[b]])
        assert np.array_equal(st.v_cache[b, layer, pos[b]].cpu().numpy().view(np.uint16), vcs[b][pos[b]])
    assert int(st.k_cache[:, 0].abs().sum()) == 0  # the other layer's slab is untouched


# ---------------------------------------------------------------------------
# fp16 rounding edge cases through the kernels that store cache rows
# ---------------------------------------------------------------------------

HQ_E, HKV_E, HD_E = 8, 8, 128
KVD_E = HKV_E * HD_E


def assert_k_bits(got, want, k_in, mask):
    """k passes through RoPE arithmetic before it is stored.  For a NaN input
    the GPU's multiply returns the canonical NaN (sign and payload dropped),
    where the reference's x86 arithmetic keeps the operand's sign, so those
    rows hold 0x7E00 where the reference may hold 0xFE00: both NaN.  Every
    other value must carry the reference's bits."""
    nan = np.isnan(k_in) & mask
    rest = mask & ~nan
    assert np.array_equal(got[rest], want[rest]), f"k: {np.sum(got[rest] != want[rest])} values differ"
    g = got[nan]
    assert np.all(((g & 0x7C00) == 0x7C00) & ((g & 0x3FF) != 0)), "k: a NaN input was not stored as a NaN"


def edge_rows(golden_dir):
    """v rows: the edge inputs 1024 to a row; k rows: 64 to each head's first
    half with zeros in the second half, so that RoPE at position 0
    (cos 1, sin 0) leaves their values as they are (x*1 - 0*0 = x, infinities
    included).  Returns (v_in, v_want, k_in, k_want, k_mask)."""
    g = np.load(os.path.join(golden_dir, "numerics.npz"))
    x, want = g["f16_in"].astype(np.float32), g["f16_out"].astype(np.uint16)
    n = len(x)
    nv = -(-n // KVD_E)
    v_in = np.zeros(nv * KVD_E, np.float32)
    v_want = np.zeros(nv * KVD_E, np.uint16)
    v_in[:n], v_want[:n] = x, want
    half = HD_E // 2
    per_row = HKV_E * half
    nk = -(-n // per_row)
    k_in = np.zeros((nk, HKV_E, HD_E), np.float32)
    k_want = np.zeros((nk, HKV_E, HD_E), np.uint16)
    k_mask = np.zeros((nk, HKV_E, HD_E), bool)
    xs = np.zeros(nk * per_row, np.float32)
    ws = np.zeros(nk * per_row, np.uint16)
    xs[:n], ws[:n] = x, want
    k_in[:, :, :half] = xs.reshape(nk, HKV_E, half)
    k_want[:, :, :half] = ws.reshape(nk, HKV_E, half)
    k_mask[:, :, :half] = True
    return (v_in.reshape(nv, KVD_E), v_want.reshape(nv, KVD_E), k_in.reshape(nk, KVD_E),
            k_want.reshape(nk, KVD_E), k_mask.reshape(nk, KVD_E))


def test_rounding_edges_batched_prep_kernel(cuda, golden_dir):
    """Several sequences at position 0: the prep kernel stores the rows."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState
    v_in, v_want, k_in, k_want, k_mask = edge_rows(golden_dir)
    B = max(len(v_in), len(k_in))
    cfg = abi.Config.make(1, HQ_E, HKV_E, HD_E, 16, 1e6)
    st = AttnState(cfg, n_seqs=B, max_ctx=1)
    k = np.zeros((B, KVD_E), np.float32)
    v = np.zeros((B, KVD_E), np.float32)
    k[:len(k_in)], v[:len(v_in)] = k_in, v_in
    q = np.zeros((B, HQ_E * HD_E), np.float32)
    out = torch.empty((B, HQ_E * HD_E), device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    st.decode(0, torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), pos, out)
    torch.cuda.synchronize()
    assert st.status() == 0
    vrows = st.v_cache[:len(v_in), 0, 0].cpu().numpy().view(np.uint16)
    krows = st.k_cache[:len(k_in), 0, 0].cpu().numpy().view(np.uint16)
    assert np.array_equal(vrows, v_want), f"v: {np.sum(vrows != v_want)} rows bits differ"
    assert_k_bits(krows, k_want, k_in, k_mask)


def test_rounding_edges_single_sequence_fused_append(cuda, golden_dir):
    """One sequence per call: the attention kernel stores the row itself."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState
    v_in, v_want, k_in, k_want, k_mask = edge_rows(golden_dir)
    cfg = abi.Config.make(1, HQ_E, HKV_E, HD_E, 16, 1e6)
    st = AttnState(cfg, n_seqs=1, max_ctx=1)
    q = torch.zeros(HQ_E * HD_E, device="cuda")
    out = torch.empty(HQ_E * HD_E, device="cuda")
    zeros = torch.zeros(KVD_E, device="cuda")
    for i in range(max(len(v_in), len(k_in))):
        vi = torch.from_numpy(v_in[i]).cuda() if i < len(v_in) else zeros
        ki = torch.from_numpy(k_in[i]).cuda() if i < len(k_in) else zeros
        assert st.decode_one(0, 0, q, ki, vi, out) == 0
        if i < len(v_in):
            got = st.v_cache[0, 0, 0].cpu().numpy().view(np.uint16)
            assert np.array_equal(got, v_want[i]), f"v row {i}"
        if i < len(k_in):
            got = st.k_cache[0, 0, 0].cpu().numpy().view(np.uint16)
            assert_k_bits(got, k_want[i], k_in[i], k_mask[i])
    assert st.status() == 0


def test_rounding_edges_prefill_fp32_inputs(cuda, golden_dir):
    """A prompt with fp32 inputs: the prefill prep kernel stores every v row
    with the reference's rounding.  q and k are zero, so every score is 0 and
    the edge values (infinities, NaN) reach only the values, never the softmax."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState
    v_in, v_want = edge_rows(golden_dir)[:2]
    n = len(v_in)
    cfg = abi.Config.make(1, HQ_E, HKV_E, HD_E, 128, 1e6)
    st = AttnState(cfg, n_seqs=1, max_ctx=1)
    q = torch.zeros((n, HQ_E * HD_E), device="cuda")
    k = torch.zeros((n, KVD_E), device="cuda")
    out = torch.empty((n, HQ_E * HD_E), device="cuda")
    assert st.prefill(0, 0, q, k, torch.from_numpy(v_in).cuda(), out) == 0
    torch.cuda.synchronize()
    vrows = st.v_cache[0, 0, :n].cpu().numpy().view(np.uint16)
    assert np.array_equal(vrows, v_want), f"v: {np.sum(vrows != v_want)} values differ"
