"""Multi-rank host logic on CPU: world_size-2 gloo process groups, no GPU.

* split-KV decode: each rank attends only its contiguous shard of the cache rows
  (the oracle's online-softmax scan, cpp/model.hpp:378-413 restated), the shard
  results are all-gathered over gloo and combined by log-sum-exp; the result
  must equal the single-loop reference over all rows.
* failure handling: a rank that exits before the collective makes the survivor's
  collective fail within the process-group timeout instead of hanging.
* sequence / KV-head partitions used by the benchmark are exact covers.
"""
import multiprocessing as mp
import os
import tempfile
import traceback

import numpy as np
import pytest

from picolm_qwen_b200 import sharding


def store_path() -> str:
    """Rendezvous through a file store: no TCP port to race for."""
    return os.path.join(tempfile.mkdtemp(prefix="picoattn_pg_"), "store")


def _splitkv_rank(rank, world, store_file, q_ret):
    try:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        from oracle.pyoracle import Oracle
        dist.init_process_group("gloo", store=dist.FileStore(store_file, world), rank=rank, world_size=world,
                                timeout=timedelta(seconds=20))
        ora = Oracle()
        hq, hkv, hd, n = 40, 8, 128, 3000  # Qwen2.5-32B heads; rows 0..n-1 attended
        rng = np.random.default_rng(17)
        kvd = hkv * hd
        kc = ora.f32_to_f16(rng.standard_normal(n * kvd).astype(np.float32) * 0.5).reshape(n, kvd)
        vc = ora.f32_to_f16(rng.standard_normal(n * kvd).astype(np.float32) * 0.5).reshape(n, kvd)
        q = rng.standard_normal(hq * hd).astype(np.float32)
        off, rows = sharding.shard_rows(n, world, rank)
        m, l, acc = ora.attend_rows(hq, hkv, hd, q, kc, vc, off, off + rows)
        part = np.zeros((1, hq, hd + 2), np.float32)
        part[0, :, :hd] = (acc.reshape(hq, hd) / l[:, None])
        part[0, :, hd] = (m + np.log(l)) * np.float32(1.4426950408889634)  # log2-sum-exp
        t = torch.from_numpy(part)
        got = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(got, t)
        combined = sharding.combine_shards_host(np.stack([g.numpy() for g in got]))[0]
        m_all, l_all, acc_all = ora.attend_rows(hq, hkv, hd, q, kc, vc, 0, n)
        ref = acc_all.reshape(hq, hd) / l_all[:, None]
        err = np.abs(combined - ref)
        ok = bool(np.all(err <= 1e-5 + 1e-4 * np.abs(ref)))
        dist.destroy_process_group()
        q_ret.put((rank, ok, float(err.max())))
    except Exception:
        q_ret.put((rank, False, traceback.format_exc()))


def _run(target, world, extra=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store_file = store_path()
    procs = [ctx.Process(target=target, args=(r, world, store_file, q) + tuple(extra)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r[0])


def test_splitkv_two_ranks_gloo_matches_single_loop():
    res = _run(_splitkv_rank, 2)
    for rank, ok, info in res:
        assert ok, f"rank {rank}: {info}"


def _dead_peer_rank(rank, world, store_file, q_ret):
    try:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("gloo", store=dist.FileStore(store_file, world), rank=rank, world_size=world,
                                timeout=timedelta(seconds=3))
        if rank == 1:
            q_ret.put((rank, True, "left before the collective"))
            q_ret.close()
            q_ret.join_thread()  # flush the report before the abrupt exit
            os._exit(0)  # dies between steps, nothing in flight
        t = torch.zeros(4)
        try:
            dist.all_reduce(t)
            q_ret.put((rank, False, "collective completed without the peer"))
        except Exception as e:  # the survivor learns of the failure from the collective
            q_ret.put((rank, True, type(e).__name__))
    except Exception:
        q_ret.put((rank, False, traceback.format_exc()))


def test_dead_peer_is_detected_not_hung():
    res = _run(_dead_peer_rank, 2)
    for rank, ok, info in res:
        assert ok, f"rank {rank}: {info}"


def test_row_shards_cover_positions_exactly():
    for total in (1, 7, 131072, 131073):
        for world in (1, 2, 3, 8):
            spans = [sharding.shard_rows(total, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (o1, n1), (o2, _) in zip(spans, spans[1:]):
                assert o1 + n1 == o2
            assert spans[-1][0] + spans[-1][1] == total
            assert max(n for _, n in spans) - min(n for _, n in spans) <= 1
    assert sharding.owner_of(131071, 131072, 8) == 7
    assert sharding.owner_of(0, 131072, 8) == 0


def test_lpt_balances_ragged_batches():
    rng = np.random.default_rng(0)
    lens = rng.integers(1024, 8193, 64)
    for world in (2, 4, 8):
        parts = sharding.lpt_assign(lens, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [int(np.sum(lens[p])) for p in parts]
        assert max(loads) - min(loads) <= int(lens.max())


def test_kv_head_groups_partition_heads():
    for world in (1, 2, 4, 8):
        groups = [sharding.kv_head_groups(8, world, r) for r in range(world)]
        assert sorted(h for g in groups for h in g) == list(range(8))


def test_combine_host_skips_empty_shards():
    hd = 4
    parts = np.zeros((2, 1, 1, hd + 2), np.float32)
    parts[0, 0, 0, :hd] = [1, 2, 3, 4]
    parts[0, 0, 0, hd] = 3.0
    parts[1, 0, 0, hd] = -np.inf  # a shard with no rows of this sequence
    out = sharding.combine_shards_host(parts)
    assert np.allclose(out[0, 0], [1, 2, 3, 4])
