"""The C ABI on the host: no GPU needed, no device compute is launched.

Covers: the shared library loads and exports every function declared in
include/picoattn.h; argument validation returns status codes (the reference
prints and returns -1 at load, cpp/model.hpp:211-222, and has no status for the
attention step itself); the host RoPE table is bit-identical to the one
Model::allocate_run_state builds (cpp/model.hpp:1008-1017).
"""
import ctypes as C
import os

import numpy as np
import pytest

from picolm_qwen_b200 import abi


def cfg(**kw):
    base = dict(n_layers=2, n_heads=28, n_kv_heads=4, head_dim=128, max_seq_len=1024,
                rope_freq_base=1e6, rope_mode=abi.ROPE_NEOX, qk_norm_eps=1e-6)
    base.update(kw)
    return abi.Config(**base)


def test_library_exports_every_declared_symbol():
    L = abi.lib()
    names = abi.declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), n
        assert n in abi.PROTOTYPES, f"{n} declared in the header but not bound in abi.py"


def test_library_is_sm100a_only():
    # The fatbinary carries sm_100a code; the build passes only that -gencode.
    from picolm_qwen_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_strerror_and_version():
    L = abi.lib()
    assert L.picoattn_version() >= 100
    assert L.picoattn_strerror(abi.PICOATTN_ERANGE) == b"position out of range"
    assert L.picoattn_strerror(12345) == b"unknown status"


@pytest.mark.parametrize("bad,expect", [
    (dict(n_heads=30, n_kv_heads=4), abi.PICOATTN_EINVAL),      # heads not a multiple of kv heads
    (dict(head_dim=96), abi.PICOATTN_EUNSUPPORTED),
    (dict(head_dim=7), abi.PICOATTN_EINVAL),
    (dict(n_kv_heads=3, n_heads=9), abi.PICOATTN_EUNSUPPORTED),
    (dict(n_heads=68, n_kv_heads=4), abi.PICOATTN_EUNSUPPORTED),  # 17 q heads per kv head
    (dict(rope_mode=5), abi.PICOATTN_EINVAL),
    (dict(max_seq_len=0), abi.PICOATTN_EINVAL),
    (dict(rope_freq_base=0.0), abi.PICOATTN_EINVAL),
])
def test_config_check_rejects(bad, expect):
    assert abi.lib().picoattn_config_check(C.byref(cfg(**bad))) == expect


def test_config_check_accepts_benchmark_shapes():
    L = abi.lib()
    for hq, hkv, hd in [(32, 4, 64), (14, 2, 64), (28, 4, 128), (32, 8, 128), (40, 8, 128), (4, 4, 64)]:
        assert L.picoattn_config_check(C.byref(cfg(n_heads=hq, n_kv_heads=hkv, head_dim=hd))) == 0


def test_decode_argument_validation_happens_before_any_device_work():
    L = abi.lib()
    c = cfg()
    fake = 0x10000  # never dereferenced: validation fails first
    args = [fake] * 7
    # null q
    st = L.picoattn_decode_one(C.byref(c), 0, 5, None, fake, fake, None, None, fake, fake, fake, fake, fake,
                               fake, 1 << 30, None)
    assert st == abi.PICOATTN_EINVAL
    # position beyond the cache
    st = L.picoattn_decode_one(C.byref(c), 0, 1024, fake, fake, fake, None, None, fake, fake, fake, fake, fake,
                               fake, 1 << 30, None)
    assert st == abi.PICOATTN_ERANGE
    # layer out of range
    st = L.picoattn_decode_one(C.byref(c), 2, 5, fake, fake, fake, None, None, fake, fake, fake, fake, fake,
                               fake, 1 << 30, None)
    assert st == abi.PICOATTN_EINVAL
    # only one of the two QK-norm weights
    st = L.picoattn_decode_one(C.byref(c), 0, 5, fake, fake, fake, fake, None, fake, fake, fake, fake, fake,
                               fake, 1 << 30, None)
    assert st == abi.PICOATTN_EINVAL
    # workspace too small
    st = L.picoattn_decode_one(C.byref(c), 0, 5, fake, fake, fake, None, None, fake, fake, fake, fake, fake,
                               fake, 64, None)
    assert st == abi.PICOATTN_ENOSPACE
    # misaligned cache base
    st = L.picoattn_decode_one(C.byref(c), 0, 5, fake, fake, fake, None, None, fake, fake, fake + 2, fake, fake,
                               fake, 1 << 30, None)
    assert st == abi.PICOATTN_EINVAL
    # batched: max_ctx beyond max_seq_len
    st = L.picoattn_decode(C.byref(c), 0, 4, 2048, *args[:3], None, None, fake, fake, fake, fake, fake, fake,
                           fake, 1 << 30, None)
    assert st == abi.PICOATTN_ERANGE
    del args


def test_workspace_size_is_independent_of_context():
    L = abi.lib()
    c = cfg(max_seq_len=131072, n_heads=40, n_kv_heads=8)
    sizes = {L.picoattn_decode_workspace_size(C.byref(c), 1, ctx) for ctx in (1, 100, 4096, 131072)}
    assert len(sizes) == 1 and sizes.pop() > 0
    c3 = cfg(max_seq_len=8193)
    assert L.picoattn_decode_workspace_size(C.byref(c3), 64, 8193) > 0
    assert L.picoattn_decode_workspace_size(C.byref(cfg(head_dim=96)), 1, 10) == 0


def test_rope_table_matches_reference_bit_for_bit(golden_dir):
    g = np.load(os.path.join(golden_dir, "rope_tables.npz"))
    L = abi.lib()
    c = cfg(head_dim=64, max_seq_len=int(g["hd64_S"]), rope_freq_base=float(g["hd64_base"]))
    cos = np.empty((c.max_seq_len, 32), np.float32)
    sin = np.empty_like(cos)
    assert L.picoattn_rope_table(C.byref(c), cos.ctypes.data, sin.ctypes.data) == 0
    assert np.array_equal(cos, g["hd64_cos"]) and np.array_equal(sin, g["hd64_sin"])
    rows = g["hd128_rows"]
    c = cfg(head_dim=128, max_seq_len=int(rows.max()) + 1, rope_freq_base=float(g["hd128_base"]))
    cos = np.empty((c.max_seq_len, 64), np.float32)
    sin = np.empty_like(cos)
    assert L.picoattn_rope_table(C.byref(c), cos.ctypes.data, sin.ctypes.data) == 0
    assert np.array_equal(cos[rows], g["hd128_cos"]) and np.array_equal(sin[rows], g["hd128_sin"])
