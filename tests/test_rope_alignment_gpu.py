"""RoPE tables at a 4-byte (not 8-byte) aligned address.

The C ABI asks only for fp32 RoPE tables (include/picoattn.h); a caller may
hand rows cut out of a larger buffer.  Every kernel that reads the tables
(single-sequence decode with and without QK-norm, batched decode, prefill)
must then produce the same bits as with the table at an aligned address.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from picolm_qwen_b200 import abi
    assert abi.lib().picoattn_device_check() == 0
    return torch.device("cuda")


def shifted(t):
    """A copy of t whose data starts 4 bytes past an aligned allocation."""
    buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
    view = buf[1:].view_as(t)
    view.copy_(t)
    assert view.data_ptr() % 8 == 4
    return view


def two_states(cfg, n_seqs=1):
    from picolm_qwen_b200.runtime import AttnState
    a = AttnState(cfg, n_seqs=n_seqs)
    b = AttnState(cfg, n_seqs=n_seqs)
    b.rope_cos, b.rope_sin = shifted(a.rope_cos), shifted(a.rope_sin)
    return a, b


@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("mode", [0, 1])
def test_decode_one_unaligned_tables(cuda, norm, mode):
    from picolm_qwen_b200 import abi
    hq, hkv, hd, S = 16, 4, 128, 700
    cfg = abi.Config.make(1, hq, hkv, hd, S, 1e6 if mode == 0 else 1e4, mode)
    sa, sb = two_states(cfg)
    g = torch.Generator(device="cuda").manual_seed(5)
    qn = (1 + 0.1 * torch.randn(hd, generator=g, device="cuda")) if norm else None
    kn = (1 + 0.1 * torch.randn(hd, generator=g, device="cuda")) if norm else None
    outs = []
    for st in (sa, sb):
        g.manual_seed(6)
        out = torch.empty(hq * hd, device="cuda")
        for pos in range(0, 600, 37):
            q = torch.randn(hq * hd, generator=g, device="cuda")
            k = torch.randn(hkv * hd, generator=g, device="cuda")
            v = torch.randn(hkv * hd, generator=g, device="cuda")
            assert st.decode_one(0, pos, q, k, v, out, qn, kn) == 0
        torch.cuda.synchronize()
        assert st.status() == 0
        outs.append(out.clone())
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(sa.k_cache, sb.k_cache) and torch.equal(sa.v_cache, sb.v_cache)


def test_batched_decode_unaligned_tables(cuda):
    from picolm_qwen_b200 import abi
    hq, hkv, hd, S, B = 28, 4, 128, 512, 6
    cfg = abi.Config.make(1, hq, hkv, hd, S, 1e6)
    sa, sb = two_states(cfg, n_seqs=B)
    g = torch.Generator(device="cuda").manual_seed(7)
    q = torch.randn(B, hq * hd, generator=g, device="cuda")
    k = torch.randn(B, hkv * hd, generator=g, device="cuda")
    v = torch.randn(B, hkv * hd, generator=g, device="cuda")
    pos = torch.tensor([0, 3, 100, 257, 400, 511], dtype=torch.int32, device="cuda")
    outs = []
    for st in (sa, sb):
        out = torch.empty(B, hq * hd, device="cuda")
        st.decode(0, q, k, v, pos, out)
        torch.cuda.synchronize()
        assert st.status() == 0
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(sa.k_cache, sb.k_cache) and torch.equal(sa.v_cache, sb.v_cache)


@pytest.mark.parametrize("mode,hd,hq,hkv", [(0, 128, 32, 8), (1, 128, 8, 2), (0, 64, 14, 2), (1, 64, 32, 4)])
def test_prefill_unaligned_tables(cuda, mode, hd, hq, hkv):
    from picolm_qwen_b200 import abi
    n, S = 200, 300
    cfg = abi.Config.make(1, hq, hkv, hd, S, 1e6 if mode == 0 else 1e4, mode)
    sa, sb = two_states(cfg)
    g = torch.Generator(device="cuda").manual_seed(8)
    q = torch.randn(n, hq * hd, generator=g, device="cuda").half()
    k = torch.randn(n, hkv * hd, generator=g, device="cuda").half()
    v = torch.randn(n, hkv * hd, generator=g, device="cuda").half()
    qn = 1 + 0.1 * torch.randn(hd, generator=g, device="cuda")
    kn = 1 + 0.1 * torch.randn(hd, generator=g, device="cuda")
    outs = []
    for st in (sa, sb):
        out = torch.empty(n, hq * hd, device="cuda")
        assert st.prefill(0, 50, q, k, v, out, qn, kn) == 0
        torch.cuda.synchronize()
        assert st.status() == 0
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(sa.k_cache, sb.k_cache) and torch.equal(sa.v_cache, sb.v_cache)
