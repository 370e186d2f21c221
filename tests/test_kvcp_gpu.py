"""KV-cache persistence (KVCP, picolm/model.c:870-983) on the B200: files the
library writes from a device cache equal the reference's kvcache_save files
byte for byte, files the reference writes load into the device cache exactly,
and a decode after a load equals one on the original cache."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from picolm_qwen_b200 import abi
    assert abi.lib().picoattn_device_check() == 0
    return torch.device("cuda")


def state(L, hq, hkv, hd, S):
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState
    return AttnState(abi.Config.make(L, hq, hkv, hd, S, 1e6), n_seqs=1)


def fill_random(st, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    st.k_cache.copy_(torch.randint(-32768, 32768, st.k_cache.shape, generator=g, device="cuda", dtype=torch.int32)
                     .to(torch.int16))
    st.v_cache.copy_(torch.randint(-32768, 32768, st.v_cache.shape, generator=g, device="cuda", dtype=torch.int32)
                     .to(torch.int16))


@pytest.mark.parametrize("shape", [(3, 8, 2, 128, 300, 257), (2, 40, 8, 128, 20000, 17000)])
def test_save_equals_reference_file(cuda, tmp_path, shape):
    """The second shape's layers (34 MB of K each) span several staging chunks."""
    L, hq, hkv, hd, S, n_pos = shape
    st = state(L, hq, hkv, hd, S)
    fill_random(st, 1)
    mine = str(tmp_path / "mine.kvcp")
    st.kvcp_save(mine, n_pos)
    ref = pyoracle.RefHarness()
    theirs = str(tmp_path / "ref.kvcp")
    kc = st.k_cache[0].cpu().numpy().view(np.uint16)
    vc = st.v_cache[0].cpu().numpy().view(np.uint16)
    assert ref.kvcp_save(kc, vc, hkv, hd, theirs, n_pos) == 0
    assert open(mine, "rb").read() == open(theirs, "rb").read()


def test_load_reference_file(cuda, tmp_path):
    L, hq, hkv, hd, S, n_pos = 3, 28, 4, 128, 500, 321
    rng = np.random.default_rng(3)
    kc = rng.integers(0, 65536, (L, S, hkv * hd), dtype=np.uint16)
    vc = rng.integers(0, 65536, (L, S, hkv * hd), dtype=np.uint16)
    path = str(tmp_path / "ref.kvcp")
    assert pyoracle.RefHarness().kvcp_save(kc, vc, hkv, hd, path, n_pos) == 0
    st = state(L, hq, hkv, hd, S)
    assert st.kvcp_load(path) == n_pos
    k = st.k_cache[0].cpu().numpy().view(np.uint16)
    v = st.v_cache[0].cpu().numpy().view(np.uint16)
    assert np.array_equal(k[:, :n_pos], kc[:, :n_pos]) and not k[:, n_pos:].any()
    assert np.array_equal(v[:, :n_pos], vc[:, :n_pos]) and not v[:, n_pos:].any()


def test_pack_unpack_device_and_host_buffers(cuda, tmp_path):
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import stream_handle
    lib = abi.lib()
    L, hq, hkv, hd, S, n_pos = 2, 14, 2, 64, 400, 399
    st = state(L, hq, hkv, hd, S)
    fill_random(st, 4)
    cfgp = C.byref(st.cfg)
    nb = lib.picoattn_kvcp_bytes(cfgp, n_pos)
    path = str(tmp_path / "f.kvcp")
    st.kvcp_save(path, n_pos)
    want = np.frombuffer(open(path, "rb").read(), np.uint8)
    dbuf = torch.empty(nb, dtype=torch.uint8, device="cuda")
    hbuf = torch.empty(nb, dtype=torch.uint8).pin_memory()
    for buf in (dbuf, hbuf):
        assert lib.picoattn_kvcp_pack(cfgp, n_pos, st.k_cache[0].data_ptr(), st.v_cache[0].data_ptr(),
                                      buf.data_ptr(), nb, stream_handle()) == 0
        torch.cuda.synchronize()
        assert np.array_equal(buf.cpu().numpy(), want)
        st2 = state(L, hq, hkv, hd, S)
        n = C.c_int32(0)
        assert lib.picoattn_kvcp_unpack(cfgp, buf.data_ptr(), nb, st2.k_cache[0].data_ptr(),
                                        st2.v_cache[0].data_ptr(), C.byref(n), stream_handle()) == 0
        torch.cuda.synchronize()
        assert n.value == n_pos
        assert torch.equal(st2.k_cache[:, :, :n_pos], st.k_cache[:, :, :n_pos])
        assert torch.equal(st2.v_cache[:, :, :n_pos], st.v_cache[:, :, :n_pos])
    assert lib.picoattn_kvcp_pack(cfgp, n_pos, st.k_cache[0].data_ptr(), st.v_cache[0].data_ptr(),
                                  dbuf.data_ptr(), nb - 1, stream_handle()) == abi.PICOATTN_ENOSPACE


def test_load_rejections_leave_no_positions(cuda, tmp_path):
    L, hq, hkv, hd, S = 2, 8, 2, 64, 100
    st = state(L, hq, hkv, hd, S)
    fill_random(st, 5)
    good = str(tmp_path / "g.kvcp")
    st.kvcp_save(good, 60)
    data = open(good, "rb").read()
    (tmp_path / "short.kvcp").write_bytes(data[:-2])
    st2 = state(L, hq, hkv, hd, S)
    assert st2.kvcp_load(str(tmp_path / "missing.kvcp")) == 0
    assert st2.kvcp_load(str(tmp_path / "short.kvcp")) == 0
    other = state(3, hq, hkv, hd, S)  # another layer count
    assert other.kvcp_load(good) == 0
    small = state(L, hq, hkv, hd, 50)  # 60 positions exceed its max_seq_len
    assert small.kvcp_load(good) == 0
    assert st2.kvcp_load(good) == 60


def test_decode_after_load_equals_decode_on_original(cuda, tmp_path):
    L, hq, hkv, hd, S, n_pos = 2, 40, 8, 128, 4096, 3000
    st = state(L, hq, hkv, hd, S)
    g = torch.Generator(device="cuda").manual_seed(6)
    for c in (st.k_cache, st.v_cache):
        c.copy_((torch.randn(c.shape, generator=g, device="cuda") * 0.5).half().view(torch.int16))
    path = str(tmp_path / "ctx.kvcp")
    st.kvcp_save(path, n_pos)
    st2 = state(L, hq, hkv, hd, S)
    assert st2.kvcp_load(path) == n_pos
    q = torch.randn(hq * hd, generator=g, device="cuda")
    k = torch.randn(hkv * hd, generator=g, device="cuda")
    v = torch.randn(hkv * hd, generator=g, device="cuda")
    outs = []
    for s in (st, st2):
        out = torch.empty(hq * hd, device="cuda")
        assert s.decode_one(1, n_pos, q, k, v, out) == 0
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
