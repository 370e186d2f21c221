"""One process driving two GPUs: the library's per-device setup.

Kernel attributes such as the dynamic shared-memory limit belong to a device,
so a process that calls the library on device 0 and then on device 1 must get
them set on both; the decode, the mat-vec and the prefill each run on both
devices here and must give the same results on each.  Skipped with fewer than
two GPUs.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")


def test_decode_matvec_prefill_on_two_devices_in_one_process(two_gpus):
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, matvec
    from tests import weightgen as wg
    hq, hkv, hd, S = 40, 8, 128, 20000  # attention and merge kernels with > 48 KB of shared memory
    cfg = abi.Config.make(1, hq, hkv, hd, S, 1e6)
    rng = np.random.default_rng(11)
    kc = (rng.standard_normal((S, hkv * hd), dtype=np.float32) * 0.5).astype(np.float16).view(np.int16)
    vc = (rng.standard_normal((S, hkv * hd), dtype=np.float32) * 0.5).astype(np.float16).view(np.int16)
    q = rng.standard_normal(hq * hd).astype(np.float32)
    k = rng.standard_normal(hkv * hd).astype(np.float32)
    v = rng.standard_normal(hkv * hd).astype(np.float32)
    w = wg.make(abi.WT_Q4_K, 3584, 512, rng)
    x = rng.standard_normal((1, 3584)).astype(np.float32)
    pq = rng.standard_normal((256, hq * hd)).astype(np.float16)
    pk = rng.standard_normal((256, hkv * hd)).astype(np.float16)
    pv = rng.standard_normal((256, hkv * hd)).astype(np.float16)
    results = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            st = AttnState(cfg, n_seqs=1, device=dev, max_ctx=S)
            st.k_cache[0, 0] = torch.from_numpy(kc).to(dev)
            st.v_cache[0, 0] = torch.from_numpy(vc).to(dev)
            out = torch.empty(hq * hd, device=dev)
            assert st.decode_one(0, S - 1, torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                                 torch.from_numpy(v).to(dev), out) == 0
            y = torch.empty((1, 512), device=dev)
            matvec(torch.from_numpy(w).to(dev), abi.WT_Q4_K, 3584, 512, torch.from_numpy(x).to(dev), y)
            pst = AttnState(cfg, n_seqs=1, device=dev, max_ctx=1)
            pout = torch.empty((256, hq * hd), device=dev)
            assert pst.prefill(0, 0, torch.from_numpy(pq).to(dev), torch.from_numpy(pk).to(dev),
                               torch.from_numpy(pv).to(dev), pout) == 0
            torch.cuda.synchronize(dev)
            assert st.status() == 0 and pst.status() == 0
            results.append((out.cpu(), y.cpu(), pout.cpu()))
    for a, b in zip(*results):
        assert torch.isfinite(a).all() and torch.equal(a, b)
