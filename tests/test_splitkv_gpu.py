"""Split-KV decode (long context across devices), emulated on one GPU.

The rows of every sequence are cut into contiguous shards (each its own slab, as
each GPU would hold it); picoattn_decode_shard runs per shard, the token's new
row is stored only by the shard that holds its position, and
picoattn_combine_shards combines the shard results.  The result must equal the
reference's single loop over all rows (oracle), within
|gpu - ref| <= 2e-3 + 1e-2 |ref|, and the stored row must carry the
reference's fp16 bits.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from picolm_qwen_b200 import abi
    assert abi.lib().picoattn_device_check() == 0


def assert_close(got, ref, what):
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bad = ~(err <= ATOL + RTOL * np.abs(ref.astype(np.float64)))
    assert not bad.any(), f"{what}: {bad.sum()} outside tolerance, max err {err.max():.3g}"


@pytest.mark.parametrize("n_shards", [2, 3, 8])
def test_sharded_decode_equals_single_loop(cuda, oracle, n_shards):
    from picolm_qwen_b200 import abi, sharding
    from picolm_qwen_b200.runtime import rope_table, stream_handle
    L = abi.lib()
    hq, hkv, hd = 40, 8, 128  # Qwen2.5-32B heads
    kvd = hkv * hd
    total = 9000              # absolute positions held across the shards
    lens = np.array([8999, 5000, 1], np.int32)  # new token positions: last shard / middle / first shard
    B = len(lens)
    n_layers, layer = 2, 1
    cfg = abi.Config.make(n_layers, hq, hkv, hd, total, 1e6)
    rng = np.random.default_rng(3)
    full_k = [np.zeros((total, kvd), np.uint16) for _ in range(B)]
    full_v = [np.zeros((total, kvd), np.uint16) for _ in range(B)]
    for b in range(B):
        n = int(lens[b])
        if n:
            full_k[b][:n] = oracle.f32_to_f16(rng.standard_normal(n * kvd).astype(np.float32) * 0.5).reshape(n, kvd)
            full_v[b][:n] = oracle.f32_to_f16(rng.standard_normal(n * kvd).astype(np.float32) * 0.5).reshape(n, kvd)
    q = rng.standard_normal((B, hq * hd)).astype(np.float32)
    k = rng.standard_normal((B, kvd)).astype(np.float32)
    v = rng.standard_normal((B, kvd)).astype(np.float32)
    cos_t, sin_t = oracle.rope_table(total, hd, 1e6)
    ref_k = [a.copy() for a in full_k]
    ref_v = [a.copy() for a in full_v]
    ref = oracle.decode_batch(hq, hkv, hd, 0, q, k, v, None, None, cos_t, sin_t, ref_k, ref_v, lens, n_threads=8)

    cos, sin = rope_table(cfg)
    d_cos, d_sin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    dpos = torch.from_numpy(lens).cuda()
    sh = stream_handle()
    per = hq * (hd + 2)
    parts = torch.empty((n_shards, B, per), device="cuda")
    slabs = []
    for s in range(n_shards):
        off, rows = sharding.shard_rows(total, n_shards, s)
        kc = torch.zeros((B, n_layers, rows, kvd), dtype=torch.int16, device="cuda")
        vc = torch.zeros_like(kc)
        for b in range(B):
            kc[b, layer] = torch.from_numpy(full_k[b][off:off + rows].view(np.int16)).cuda()
            vc[b, layer] = torch.from_numpy(full_v[b][off:off + rows].view(np.int16)).cuda()
        kp = torch.tensor([kc[b].data_ptr() for b in range(B)], dtype=torch.int64, device="cuda")
        vp = torch.tensor([vc[b].data_ptr() for b in range(B)], dtype=torch.int64, device="cuda")
        ws_n = L.picoattn_decode_workspace_size(C.byref(cfg), B, rows)
        ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
        st = L.picoattn_decode_shard(C.byref(cfg), layer, B, rows, off, rows, dq.data_ptr(), dk.data_ptr(),
                                     dv.data_ptr(), None, None, d_cos.data_ptr(), d_sin.data_ptr(), kp.data_ptr(),
                                     vp.data_ptr(), dpos.data_ptr(), parts[s].data_ptr(), ws.data_ptr(), ws_n, sh)
        assert st == 0, L.picoattn_strerror(st)
        slabs.append((off, rows, kc, vc, kp, vp, ws))
    out = torch.empty((B, hq * hd), device="cuda")
    assert L.picoattn_combine_shards(C.byref(cfg), B, n_shards, parts.data_ptr(), out.data_ptr(), sh) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(B):
        assert_close(got[b], ref[b], f"seq {b} pos {lens[b]}")
        # the new row is in the owner's slab, with the reference's bits
        owner = sharding.owner_of(int(lens[b]), total, n_shards)
        off, rows, kc, vc = slabs[owner][:4]
        lrow = int(lens[b]) - off
        assert np.array_equal(kc[b, layer, lrow].cpu().numpy().view(np.uint16), ref_k[b][lens[b]])
        assert np.array_equal(vc[b, layer, lrow].cpu().numpy().view(np.uint16), ref_v[b][lens[b]])
    # a shard that holds no row <= pos reports an empty result (log2-sum-exp = -inf)
    p = parts.cpu().numpy().reshape(n_shards, B, hq, hd + 2)
    for s in range(n_shards):
        off = slabs[s][0]
        for b in range(B):
            if off > lens[b]:
                assert np.all(np.isneginf(p[s, b, :, hd]))
