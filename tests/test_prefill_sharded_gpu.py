"""Prefill split across GPUs by KV-head groups, against the single-GPU call.

In a tensor-parallel layer each rank holds the q/k/v columns of its KV heads
(sharding.kv_head_groups) and its own cache of those heads, and calls
picoattn_prefill with a config of its heads; attention needs no exchange
(the reference's per-token loop, cpp/model.hpp:493-593, treats every q head on
its own).  Each head's arithmetic does not depend on which other heads share
the call, so the per-rank outputs, put back at their heads' columns, must equal
the single-GPU call bit for bit, and so must the cache rows.  The ranks run one
after another on one GPU (2 and 8 ranks, the bench's configurations) and, when
two GPUs are present, on cuda:0 and cuda:1 from one process.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

HQ, HKV, HD, N_TOK = 32, 8, 128, 1024  # Qwen3-8B heads


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from picolm_qwen_b200 import abi
    assert abi.lib().picoattn_device_check() == 0


@pytest.fixture(scope="module")
def prompt():
    rng = np.random.default_rng(2048)
    q = rng.standard_normal((N_TOK, HQ, HD)).astype(np.float16)
    k = rng.standard_normal((N_TOK, HKV, HD)).astype(np.float16)
    v = rng.standard_normal((N_TOK, HKV, HD)).astype(np.float16)
    qn = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
    return q, k, v, qn, kn


def run_prefill(dev, hq, hkv, q, k, v, qn, kn):
    """One layer's prompt through picoattn_prefill on `dev`; returns (out, k rows, v rows) on the host."""
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState
    with torch.cuda.device(dev):
        cfg = abi.Config.make(2, hq, hkv, HD, N_TOK, 1e6, abi.ROPE_NEOX)
        st = AttnState(cfg, n_seqs=1, device=dev, max_ctx=1)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        out = torch.full((N_TOK, hq * HD), float("nan"), device=dev)
        assert st.prefill(1, 0, t(q.reshape(N_TOK, -1)), t(k.reshape(N_TOK, -1)), t(v.reshape(N_TOK, -1)), out,
                          t(qn), t(kn)) == 0
        torch.cuda.synchronize(dev)
        assert st.status() == 0
        return (out.cpu().numpy().reshape(N_TOK, hq, HD), st.k_cache[0, 1].cpu().numpy().reshape(N_TOK, hkv, HD),
                st.v_cache[0, 1].cpu().numpy().reshape(N_TOK, hkv, HD))


def rank_slices(world, rank):
    from picolm_qwen_b200 import sharding
    groups = sharding.kv_head_groups(HKV, world, rank)
    g = HQ // HKV
    qh = [kv * g + j for kv in groups for j in range(g)]
    return groups, qh


def check_sharded(full, per_rank, world):
    out, kc, vc = full
    for rank, (o, kr, vr) in enumerate(per_rank):
        groups, qh = rank_slices(world, rank)
        assert np.array_equal(o, out[:, qh]), f"rank {rank}: outputs differ from the single-GPU call"
        assert np.array_equal(kr, kc[:, groups]) and np.array_equal(vr, vc[:, groups]), f"rank {rank}: cache rows"


@pytest.mark.parametrize("world", [2, 8])
def test_head_sharded_prefill_equals_single_gpu_call(cuda, prompt, world):
    q, k, v, qn, kn = prompt
    dev = torch.device("cuda", 0)
    full = run_prefill(dev, HQ, HKV, q, k, v, qn, kn)
    assert np.isfinite(full[0]).all()
    per_rank = []
    for rank in range(world):
        groups, qh = rank_slices(world, rank)
        per_rank.append(run_prefill(dev, len(qh), len(groups), q[:, qh], k[:, groups], v[:, groups], qn, kn))
    check_sharded(full, per_rank, world)


def test_head_sharded_prefill_on_two_gpus(cuda, prompt):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    q, k, v, qn, kn = prompt
    full = run_prefill(torch.device("cuda", 0), HQ, HKV, q, k, v, qn, kn)
    per_rank = []
    for rank in range(2):
        groups, qh = rank_slices(2, rank)
        per_rank.append(run_prefill(torch.device("cuda", rank), len(qh), len(groups), q[:, qh], k[:, groups],
                                    v[:, groups], qn, kn))
    check_sharded(full, per_rank, 2)
