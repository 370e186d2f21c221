"""Projections on the CPU: the oracle's restatement of the reference's weight
dequantisation and mat-vec (oracle/attn_oracle.c) against the reference's own
dequantize_row / TensorOps::matmul_bias (compiled in oracle/_ref), bit for bit,
for every weight format of the C++ engine; the ABI's host-side checks.
"""
import ctypes as C

import numpy as np
import pytest

from picolm_qwen_b200 import abi
from tests import weightgen as wg

FORMATS = sorted(wg.BLOCK)


@pytest.fixture(scope="module")
def ref():
    from oracle.pyoracle import RefHarness, build
    build(ref=True)
    try:
        return RefHarness()
    except FileNotFoundError as e:
        pytest.skip(str(e))


@pytest.mark.parametrize("wtype", FORMATS, ids=[wg.NAMES[t] for t in FORMATS])
@pytest.mark.parametrize("n_in", [512, 3584])
def test_oracle_dequant_and_matvec_equal_reference(oracle, ref, wtype, n_in):
    e, b = wg.BLOCK[wtype]
    if n_in % e:
        pytest.skip("n_in not a multiple of the block")
    rng = np.random.default_rng(wtype * 100 + n_in)
    n_out = 40
    w = wg.make(wtype, n_in, n_out, rng)
    row = n_in // e * b
    W = oracle.dequant(w, wtype, n_in, n_out)
    for d in range(0, n_out, 7):
        r = ref.dequant_row(w[d * row:(d + 1) * row], wtype, n_in)
        assert np.array_equal(W[d].view(np.uint32), r.view(np.uint32)), f"row {d}"
    x = rng.standard_normal((3, n_in)).astype(np.float32)
    bias = rng.standard_normal(n_out).astype(np.float32)
    for bb in (None, bias):
        got = oracle.matvec(w, wtype, bb, n_in, n_out, x)
        exp = ref.matvec(w, wtype, bb, n_in, n_out, x)
        assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("wtype", [abi.WT_Q4_0, abi.WT_Q8_0, abi.WT_Q4_K, abi.WT_Q6_K],
                         ids=["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_oracle_dequant_raw_scale_bits(oracle, ref, wtype):
    """Every fp16 scale pattern that is finite (subnormals and negatives included)."""
    e, b = wg.BLOCK[wtype]
    rng = np.random.default_rng(7)
    n_in, n_out = 256, 64
    w = rng.integers(0, 256, (n_out * (n_in // e), b), dtype=np.uint8)
    scale_at = {abi.WT_Q4_0: [0], abi.WT_Q8_0: [0], abi.WT_Q4_K: [0, 2], abi.WT_Q6_K: [208]}[wtype]
    for off in scale_at:
        bits = rng.integers(0, 0x10000, w.shape[0], dtype=np.uint32).astype(np.uint16)
        bits[(bits & 0x7C00) == 0x7C00] &= 0xBFFF  # keep them finite
        bits[:8] = [0x0000, 0x8000, 0x0001, 0x83FF, 0x0400, 0x7BFF, 0xFBFF, 0x3C00]
        w[:, off:off + 2] = bits.view(np.uint8).reshape(-1, 2)
    w = w.ravel()
    row = n_in // e * b
    W = oracle.dequant(w, wtype, n_in, n_out)
    for d in range(n_out):
        r = ref.dequant_row(w[d * row:(d + 1) * row], wtype, n_in)
        assert np.array_equal(W[d].view(np.uint32), r.view(np.uint32)), f"row {d}"


def test_weight_bytes_match_gguf_row_sizes():
    L = abi.lib()
    for t, (e, b) in wg.BLOCK.items():
        n_in = 3584 if e <= 256 and 3584 % max(e, 32) == 0 else 4096
        assert L.picoattn_weight_bytes(t, n_in, 5) == 5 * (n_in // e) * b
        if e == 256:
            assert L.picoattn_weight_bytes(t, 3584 + 128, 5) == 0
    assert L.picoattn_weight_bytes(abi.WT_F32, 48, 1) == 0  # the kernels take whole 32-weight units
    assert L.picoattn_weight_bytes(7, 4096, 1) == 0          # Q5_0: not a format the engine multiplies
    assert L.picoattn_weight_bytes(abi.WT_Q8_0, 0, 1) == 0


def test_matvec_rejects_bad_arguments_on_the_host():
    L = abi.lib()
    buf = (C.c_float * 4096)()
    base = C.addressof(buf)
    a16 = (base + 15) & ~15
    args = dict(w=a16, t=abi.WT_Q8_0, n_in=64, n_out=4, n_vec=1, x=a16 + 4096, out=a16 + 8192)

    def call(**kw):
        a = dict(args, **kw)
        return L.picoattn_matvec(a["w"], a["t"], None, a["n_in"], a["n_out"], a["n_vec"], a["x"], a["out"], 0, None)

    assert call(w=None) == abi.PICOATTN_EINVAL
    assert call(x=a16 + 4100) == abi.PICOATTN_EINVAL       # x not 16-byte aligned
    assert call(w=a16 + 2) == abi.PICOATTN_EINVAL          # weights not 4-byte aligned
    assert call(t=7) == abi.PICOATTN_EUNSUPPORTED
    assert call(n_in=48) == abi.PICOATTN_EINVAL            # not whole Q8_0 blocks
    assert call(n_vec=0) == abi.PICOATTN_EINVAL


def test_decode_layer_checks_arguments_on_the_host():
    """picoattn_decode_layer rejects bad arguments before it touches the device."""
    L = abi.lib()
    cfg = abi.Config.make(2, 28, 4, 128, 1024, 1e6)
    cp = C.byref(cfg)
    dim = 3584
    n = L.picoattn_decode_layer_workspace_size(cp, dim, 1, 1024)
    assert n > L.picoattn_decode_workspace_size(cp, 1, 1024)  # decode scratch + q, k, v, attention output
    assert L.picoattn_decode_layer_workspace_size(cp, 0, 1, 1024) == 0
    buf = (C.c_uint8 * 256)()
    a16 = (C.addressof(buf) + 15) & ~15
    fake = a16  # never dereferenced: every case below fails its host check first

    def call(wq_type=abi.WT_Q4_K, d=dim, xb=fake, ws_bytes=n, max_ctx=1024):
        w = abi.LayerWeights(fake, fake, fake, fake, wq_type, abi.WT_Q4_K, abi.WT_Q6_K, abi.WT_Q4_K,
                             None, None, None, None)
        return L.picoattn_decode_layer(cp, 0, d, 1, max_ctx, xb, C.byref(w), None, None, fake, fake, fake, fake,
                                       fake, fake, fake, ws_bytes, None)

    assert call(xb=None) == abi.PICOATTN_EINVAL
    assert call(xb=fake + 4) == abi.PICOATTN_EINVAL            # not 16-byte aligned
    assert call(ws_bytes=n - 1) == abi.PICOATTN_ENOSPACE
    assert call(wq_type=7) == abi.PICOATTN_EUNSUPPORTED        # Q5_0: not a format of the engine's mat-vec
    assert call(d=3584 + 128) == abi.PICOATTN_EINVAL           # not whole 256-weight Q4_K blocks
    assert call(max_ctx=2048) == abi.PICOATTN_ERANGE           # beyond max_seq_len
