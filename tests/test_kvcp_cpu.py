"""KV-cache persistence (KVCP, picolm/model.c:870-983) on the CPU: the
reference's own kvcache_save / kvcache_load pinned against a numpy
restatement of the file layout, and the library's host-side validation."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import pyoracle

MAGIC = 0x4B564350


def kvcp_bytes(kc, vc, n_pos):
    """The KVCP layout restated: u32 magic, n_pos, n_layers, kv_dim; K rows
    0..n_pos-1 of every layer; V rows likewise (little-endian, fp16 bits)."""
    L, _, kvd = kc.shape
    head = np.array([MAGIC, n_pos, L, kvd], "<u4").tobytes()
    return head + kc[:, :n_pos].astype("<u2").tobytes() + vc[:, :n_pos].astype("<u2").tobytes()


def random_caches(rng, L, S, kvd):
    return (rng.integers(0, 65536, (L, S, kvd), dtype=np.uint16),
            rng.integers(0, 65536, (L, S, kvd), dtype=np.uint16))


def test_reference_file_layout(tmp_path):
    ref = pyoracle.RefHarness()
    rng = np.random.default_rng(1)
    kc, vc = random_caches(rng, 3, 50, 2 * 64)
    path = str(tmp_path / "ref.kvcp")
    assert ref.kvcp_save(kc, vc, 2, 64, path, 37) == 0
    assert open(path, "rb").read() == kvcp_bytes(kc, vc, 37)
    # and the reference's limits: n_pos in [1, max_seq]
    assert ref.kvcp_save(kc, vc, 2, 64, str(tmp_path / "x"), 0) == -1
    assert ref.kvcp_save(kc, vc, 2, 64, str(tmp_path / "x"), 51) == -1


def test_reference_load_round_trip_and_rejections(tmp_path):
    ref = pyoracle.RefHarness()
    rng = np.random.default_rng(2)
    kc, vc = random_caches(rng, 2, 40, 4 * 64)
    path = tmp_path / "a.kvcp"
    path.write_bytes(kvcp_bytes(kc, vc, 29))
    k2 = np.zeros_like(kc)
    v2 = np.zeros_like(vc)
    assert ref.kvcp_load(k2, v2, 4, 64, str(path)) == 29
    assert np.array_equal(k2[:, :29], kc[:, :29]) and not k2[:, 29:].any()
    assert np.array_equal(v2[:, :29], vc[:, :29]) and not v2[:, 29:].any()
    # another kv_dim, a missing file: no positions
    assert ref.kvcp_load(np.zeros((2, 40, 128), np.uint16), np.zeros((2, 40, 128), np.uint16), 2, 64,
                         str(path)) == 0
    assert ref.kvcp_load(k2, v2, 4, 64, str(tmp_path / "missing")) == 0


def test_library_kvcp_size_and_host_validation(tmp_path):
    """Paths that return before any device work (no GPU needed)."""
    from picolm_qwen_b200 import abi
    lib = abi.lib()
    cfg = abi.Config.make(3, 8, 2, 64, 100, 1e6)
    assert lib.picoattn_kvcp_bytes(C.byref(cfg), 37) == 16 + 2 * 3 * 37 * 128 * 2
    assert lib.picoattn_kvcp_bytes(C.byref(cfg), -1) == 0
    n = C.c_int32(5)
    assert lib.picoattn_kvcp_save(C.byref(cfg), 10, None, None, b"/tmp/x", None) == abi.PICOATTN_EINVAL
    assert lib.picoattn_kvcp_save(C.byref(cfg), 0, 16, 16, b"/tmp/x", None) == abi.PICOATTN_ERANGE
    assert lib.picoattn_kvcp_save(C.byref(cfg), 101, 16, 16, b"/tmp/x", None) == abi.PICOATTN_ERANGE
    assert lib.picoattn_kvcp_load(C.byref(cfg), str(tmp_path / "missing").encode(), 16, 16, C.byref(n),
                                  None) == abi.PICOATTN_EIO
    assert n.value == 0
    bad = tmp_path / "bad.kvcp"
    bad.write_bytes(np.array([0x12345678, 1, 3, 128], "<u4").tobytes())
    assert lib.picoattn_kvcp_load(C.byref(cfg), str(bad).encode(), 16, 16, C.byref(n), None) == abi.PICOATTN_EFORMAT
    other = tmp_path / "other.kvcp"
    other.write_bytes(np.array([MAGIC, 1, 4, 128], "<u4").tobytes())  # 4 layers, the config has 3
    assert lib.picoattn_kvcp_load(C.byref(cfg), str(other).encode(), 16, 16, C.byref(n), None) == abi.PICOATTN_EFORMAT
    assert lib.picoattn_strerror(abi.PICOATTN_EFORMAT) == b"not a KVCP or GGUF file of this shape"
