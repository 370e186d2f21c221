"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Run in a container that has the reference tree (the GPU box does not):

    make -C oracle ref && python tests/golden/make_golden.py

Every output value here is produced by the reference, compiled from its
sources by oracle/Makefile (oracle/_ref/libpicoref.so):
  * fp16 conversion results from cpp/quant.hpp fp32_to_fp16 / fp16_to_fp32;
  * RMSNorm / RoPE results from TensorOps::rmsnorm, TensorOps::rope_qwen and
    the C engine's rope_llama (picolm/tensor.c);
  * RoPE tables from Model::allocate_run_state (cpp/model.hpp:1008-1017);
  * attention outputs and KV-cache rows from the unmodified Model::forward
    (cpp/model.hpp:288-460) on a one-layer synthetic model, see
    oracle/ref_harness.cpp.
Inputs are seeded numpy draws and are stored next to the outputs, so the tests
never regenerate them.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.pyoracle import RefHarness, RefModel  # noqa: E402


def f16_inputs(rng: np.random.Generator) -> np.ndarray:
    """Edge cases of the reference's fp32->fp16 rounding plus random patterns."""
    edge = []
    # signed zeros, f32 subnormals (flushed), tiny values below fp16 range
    edge += [0.0, -0.0, 1e-45, -1e-45, 1e-39, -1e-39, 1e-9, -1e-9]
    # fp16 subnormal range and its rounding ties: k * 2^-25 for odd k lies on a tie
    for k in range(0, 80):
        edge.append(k * 2.0 ** -25)
        edge.append(-k * 2.0 ** -25)
    edge += [2.0 ** -24, 2.0 ** -24 * 0.5, 2.0 ** -24 * 1.5, 2.0 ** -14, 2.0 ** -14 * (1 - 2 ** -11)]
    # normal-range ties: 1 + (2j+1)*2^-11 is exactly half way between fp16 neighbours
    for j in range(0, 40):
        t = 1.0 + (2 * j + 1) * 2.0 ** -11
        edge += [t, -t, np.nextafter(np.float32(t), np.float32(0)), np.nextafter(np.float32(t), np.float32(2))]
    # overflow boundary: 65504 is max fp16, 65520 is the tie to inf
    edge += [65504.0, -65504.0, 65519.0, 65520.0, -65520.0, 65536.0, 1e6, -1e6, 3.4e38]
    edge = np.array(edge, dtype=np.float32)
    specials = np.array([0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00000, 0x7F800001, 0x7FBFFFFF],
                        dtype=np.uint32).view(np.float32)
    rand_bits = rng.integers(0, 2 ** 32, size=60000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    rand_vals = (rng.standard_normal(20000) * 4).astype(np.float32)
    return np.concatenate([edge, specials, rand_bits, rand_vals])


def gen_numerics(R: RefHarness, rng: np.random.Generator) -> None:
    x = f16_inputs(rng)
    h = R.f32_to_f16(x)
    all_h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    back = R.f16_to_f32(all_h)
    out = {"f16_in": x, "f16_out": h, "f16_all_bits": all_h, "f16_all_f32": back}
    for n in (64, 128):
        xs = rng.standard_normal((16, n)).astype(np.float32) * np.float32(3.0)
        w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        out[f"rms{n}_x"] = xs
        out[f"rms{n}_w"] = w
        out[f"rms{n}_y"] = np.stack([R.rmsnorm(r, w) for r in xs])
    for hd in (64, 128):
        hq, hkv = 4, 2
        c = rng.uniform(-1, 1, hd // 2).astype(np.float32)
        s = rng.uniform(-1, 1, hd // 2).astype(np.float32)
        q = rng.standard_normal(hq * hd).astype(np.float32)
        k = rng.standard_normal(hkv * hd).astype(np.float32)
        for mode in (0, 1):
            qo, ko = R.rope(mode, q, k, hd, hq, hkv, c, s)
            out[f"rope{hd}_m{mode}_q"], out[f"rope{hd}_m{mode}_k"] = qo, ko
        out[f"rope{hd}_c"], out[f"rope{hd}_s"] = c, s
        out[f"rope{hd}_qin"], out[f"rope{hd}_kin"] = q, k
    np.savez_compressed(os.path.join(HERE, "numerics.npz"), **out)


def gen_rope_tables(R: RefHarness) -> None:
    """RoPE tables exactly as Model::allocate_run_state builds them."""
    out = {}
    for hd, base, S, rows in ((64, 1e4, 512, None), (128, 1e6, 131072, [0, 1, 2, 511, 4095, 8191, 65535, 131070, 131071])):
        m = RefModel(R, 1, 1, hd, S, base, 0, False)
        if rows is None:
            out[f"hd{hd}_cos"], out[f"hd{hd}_sin"] = m.rope_cos.copy(), m.rope_sin.copy()
        else:
            out[f"hd{hd}_rows"] = np.array(rows, np.int32)
            out[f"hd{hd}_cos"] = m.rope_cos[rows].copy()
            out[f"hd{hd}_sin"] = m.rope_sin[rows].copy()
        out[f"hd{hd}_base"] = np.float32(base)
        out[f"hd{hd}_S"] = np.int32(S)
        m.close()
    np.savez_compressed(os.path.join(HERE, "rope_tables.npz"), **out)


# name, hq, hkv, hd, rope_base, rope_mode (0 NeoX, 1 interleaved), qk_norm, last_pos, keep, fp16_inputs
DECODE_CASES = [
    ("cfg1_tinyllama", 32, 4, 64, 1e4, 1, False, 511, 3, False),
    ("cfg2_qwen05b", 14, 2, 64, 1e6, 0, False, 300, 3, False),
    ("cfg3_qwen7b", 28, 4, 128, 1e6, 0, False, 160, 3, False),
    ("cfg4_qwen3_8b", 8, 2, 128, 1e6, 0, True, 63, 64, True),
    ("cfg5_qwen32b", 40, 8, 128, 1e6, 0, False, 96, 3, False),
    ("mha_g1", 4, 4, 64, 1e4, 0, False, 70, 3, False),
]


def gen_decode(R: RefHarness, rng: np.random.Generator) -> None:
    """Runs Model::forward for pos = 0..last_pos; keeps the last `keep` steps.

    The cache rows are all written by the reference itself (each step stores
    its own rotated k and its v at row pos, cpp/model.hpp:354-373).  For the
    Qwen3-shaped case every step is kept: that is a prefill of last_pos+1
    tokens from position 0 (cpp/model.hpp:493-593 runs this same step per token).
    """
    for name, hq, hkv, hd, base, mode, norm, last, keep, as_f16 in DECODE_CASES:
        S = last + 1
        kvd = hkv * hd
        m = RefModel(R, hq, hkv, hd, S, base, mode, norm)
        qn = kn = None
        if norm:
            qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
            kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
            m.set_norm(qn, kn)
        qs, ks, vs, outs = [], [], [], []
        for pos in range(S):
            q = rng.standard_normal(hq * hd).astype(np.float32)
            sd = 1.0 if (pos > last - keep or as_f16) else 0.5
            k = (rng.standard_normal(kvd) * sd).astype(np.float32)
            v = (rng.standard_normal(kvd) * sd).astype(np.float32)
            if as_f16:
                q, k, v = (a.astype(np.float16).astype(np.float32) for a in (q, k, v))
            o = m.decode(q, k, v, pos)
            if pos > last - keep:
                qs.append(q), ks.append(k), vs.append(v), outs.append(o)
        rec = dict(hq=np.int32(hq), hkv=np.int32(hkv), hd=np.int32(hd), rope_base=np.float32(base),
                   rope_mode=np.int32(mode), last_pos=np.int32(last), keep=np.int32(keep),
                   kcache=m.kcache.copy(), vcache=m.vcache.copy(),
                   q=np.stack(qs), k=np.stack(ks), v=np.stack(vs), out=np.stack(outs))
        if norm:
            rec["q_norm_w"], rec["k_norm_w"] = qn, kn
        np.savez_compressed(os.path.join(HERE, f"decode_{name}.npz"), **rec)
        m.close()
        print(f"  {name}: S={S} kvd={kvd} kept={keep}", flush=True)


def main() -> None:
    R = RefHarness()
    rng = np.random.default_rng(20261201)
    gen_numerics(R, rng)
    gen_rope_tables(R)
    gen_decode(R, rng)
    total = sum(os.path.getsize(os.path.join(HERE, f)) for f in os.listdir(HERE) if f.endswith(".npz"))
    print(f"fixtures written: {total / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
