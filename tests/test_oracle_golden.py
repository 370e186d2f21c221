"""The CPU oracle against the golden fixtures produced by the reference's own code.

These pin the oracle (oracle/attn_oracle.c) bit for bit: fp16 rounding
(cpp/quant.hpp:102-135), fp16 widening (cpp/quant.hpp:73-100), per-head RMSNorm
(cpp/tensor.hpp:146-176), both RoPE modes (cpp/tensor.hpp:201-283,
picolm/tensor.c:247-293), the RoPE table (cpp/model.hpp:1008-1017) and the
whole decode step of Model::forward (cpp/model.hpp:326-418).
"""
import glob
import os

import numpy as np
import pytest


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_fp16_rounding_matches_reference(oracle, golden_dir):
    g = _load(golden_dir, "numerics.npz")
    out = oracle.f32_to_f16(g["f16_in"])
    assert np.array_equal(out, g["f16_out"])


def test_fp16_widening_matches_reference_for_all_65536_patterns(oracle, golden_dir):
    g = _load(golden_dir, "numerics.npz")
    got = oracle.f16_to_f32(g["f16_all_bits"])
    assert np.array_equal(got.view(np.uint32), g["f16_all_f32"].view(np.uint32))


def test_fp16_round_trip_is_identity_except_nan(oracle, golden_dir):
    # The prefill prep stores fp16 v inputs by bits (h2_ref16): rounding the
    # widened value of any fp16 pattern gives the pattern back, NaNs becoming
    # sign | 0x7E00.  Checked over all 65536 patterns with the reference's widening.
    g = _load(golden_dir, "numerics.npz")
    bits = g["f16_all_bits"].astype(np.uint16)
    got = oracle.f32_to_f16(g["f16_all_f32"])
    nan = ((bits & 0x7C00) == 0x7C00) & ((bits & 0x3FF) != 0)
    want = np.where(nan, (bits & 0x8000) | 0x7E00, bits).astype(np.uint16)
    assert np.array_equal(got, want)


def test_fp16_rounding_is_half_up_not_even(oracle):
    # 1 + 2^-11 lies half way between 1.0 and 1 + 2^-10: the reference rounds
    # the magnitude up (0x3C01) where round-to-nearest-even gives 0x3C00.
    x = np.array([1.0 + 2.0 ** -11, -(1.0 + 2.0 ** -11), 65520.0, 1e-39], np.float32)
    assert list(oracle.f32_to_f16(x)) == [0x3C01, 0xBC01, 0x7C00, 0x0000]
    assert np.float16(1.0 + 2.0 ** -11).view(np.uint16) == 0x3C00  # numpy is RNE


@pytest.mark.parametrize("n", [64, 128])
def test_rmsnorm_matches_reference(oracle, golden_dir, n):
    g = _load(golden_dir, "numerics.npz")
    for x, y in zip(g[f"rms{n}_x"], g[f"rms{n}_y"]):
        assert np.array_equal(oracle.rmsnorm(x, g[f"rms{n}_w"]), y)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("mode", [0, 1])
def test_rope_matches_reference(oracle, golden_dir, hd, mode):
    g = _load(golden_dir, "numerics.npz")
    q, k = oracle.rope(mode, g[f"rope{hd}_qin"], g[f"rope{hd}_kin"], hd, 4, 2,
                       g[f"rope{hd}_c"], g[f"rope{hd}_s"])
    assert np.array_equal(q, g[f"rope{hd}_m{mode}_q"])
    assert np.array_equal(k, g[f"rope{hd}_m{mode}_k"])


def test_rope_tables_match_reference(oracle, golden_dir):
    g = _load(golden_dir, "rope_tables.npz")
    c, s = oracle.rope_table(int(g["hd64_S"]), 64, float(g["hd64_base"]))
    assert np.array_equal(c, g["hd64_cos"]) and np.array_equal(s, g["hd64_sin"])
    rows = g["hd128_rows"]
    # build only the rows needed: table rows are independent of each other
    c, s = oracle.rope_table(int(rows.max()) + 1, 128, float(g["hd128_base"]))
    assert np.array_equal(c[rows], g["hd128_cos"]) and np.array_equal(s[rows], g["hd128_sin"])


DECODE_FILES = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "decode_*.npz")))


@pytest.mark.parametrize("path", DECODE_FILES, ids=[os.path.basename(p)[7:-4] for p in DECODE_FILES])
def test_decode_step_matches_reference_model_forward(oracle, path):
    g = np.load(path)
    hq, hkv, hd = int(g["hq"]), int(g["hkv"]), int(g["hd"])
    last, keep = int(g["last_pos"]), int(g["keep"])
    S = last + 1
    cos_t, sin_t = oracle.rope_table(S, hd, float(g["rope_base"]))
    qn = g["q_norm_w"] if "q_norm_w" in g else None
    kn = g["k_norm_w"] if "k_norm_w" in g else None
    kc = g["kcache"].copy()
    vc = g["vcache"].copy()
    first = last - keep + 1
    kc[first:] = 0
    vc[first:] = 0
    for i in range(keep):
        pos = first + i
        out, _, _ = oracle.decode_step(hq, hkv, hd, int(g["rope_mode"]), g["q"][i], g["k"][i], g["v"][i],
                                       qn, kn, cos_t, sin_t, kc, vc, pos)
        assert np.array_equal(kc[pos], g["kcache"][pos])
        assert np.array_equal(vc[pos], g["vcache"][pos])
        assert np.array_equal(out, g["out"][i]), f"pos {pos}"


def test_prefill_matches_reference_token_loop(oracle, golden_dir):
    g = _load(golden_dir, "decode_cfg4_qwen3_8b.npz")
    hq, hkv, hd = int(g["hq"]), int(g["hkv"]), int(g["hd"])
    n = int(g["keep"])
    assert n == int(g["last_pos"]) + 1  # every token of the prompt was kept
    cos_t, sin_t = oracle.rope_table(n, hd, float(g["rope_base"]))
    kc = np.zeros_like(g["kcache"])
    vc = np.zeros_like(g["vcache"])
    out = oracle.prefill(hq, hkv, hd, 0, g["q"], g["k"], g["v"], g["q_norm_w"], g["k_norm_w"],
                         cos_t, sin_t, kc, vc, 0, n_threads=4)
    assert np.array_equal(kc, g["kcache"]) and np.array_equal(vc, g["vcache"])
    assert np.array_equal(out, g["out"])


def test_c_engine_order_agrees_within_noise(oracle, golden_dir):
    """The C engine's fused update (picolm/model.c:790-824) differs from the C++
    order only by fp32 rounding; the gap is the natural noise floor."""
    g = _load(golden_dir, "decode_cfg3_qwen7b.npz")
    hq, hkv, hd, last = int(g["hq"]), int(g["hkv"]), int(g["hd"]), int(g["last_pos"])
    cos_t, sin_t = oracle.rope_table(last + 1, hd, float(g["rope_base"]))
    kc, vc = g["kcache"].copy(), g["vcache"].copy()
    i = int(g["keep"]) - 1
    o1, _, _ = oracle.decode_step(hq, hkv, hd, 0, g["q"][i], g["k"][i], g["v"][i], None, None,
                                  cos_t, sin_t, kc, vc, last, variant=1)
    assert np.max(np.abs(o1 - g["out"][i])) < 1e-5


def test_head_threaded_step_matches_reference_golden(oracle, golden_dir):
    """The head-parallel driver used for the long-context parity checks gives
    the reference's outputs bit for bit (same per-head arithmetic)."""
    g = _load(golden_dir, "decode_cfg5_qwen32b.npz")
    hq, hkv, hd, last = int(g["hq"]), int(g["hkv"]), int(g["hd"]), int(g["last_pos"])
    cos_t, sin_t = oracle.rope_table(last + 1, hd, float(g["rope_base"]))
    kc, vc = g["kcache"].copy(), g["vcache"].copy()
    i = int(g["keep"]) - 1
    out = oracle.decode_step_mt(hq, hkv, hd, int(g["rope_mode"]), g["q"][i], g["k"][i], g["v"][i], None, None,
                                cos_t, sin_t, kc, vc, last, n_threads=7)
    assert np.array_equal(out, g["out"][i])
    assert np.array_equal(kc[last], g["kcache"][last]) and np.array_equal(vc[last], g["vcache"][last])
