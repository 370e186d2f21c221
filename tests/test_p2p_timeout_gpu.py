"""The split-KV exchange's bounded wait runs out instead of hanging.

picoattn_decode_splitkv_p2p's merge kernel waits for every rank's words of the
same call in its own exchange area.  When a rank does not make that call the
wait gives up after the communicator's timeout (picoattn_p2p_set_timeout, 20 ms
here), the outputs it was to combine are NaN, PICOATTN_DEV_TIMEOUT is set in
the workspace status, and the call completes: the GPU stays usable.  Nothing
here faults, traps or hangs a GPU: the missing rank is made on the host (a
process that never calls), and the wait is a flag that nothing sets.

One GPU: rank 1 is a second process on the same GPU that creates its exchange
area, hands over its IPC handle and then launches nothing; rank 0 (another
process) calls once and must time out.  Two GPUs: both ranks make two good
calls, then rank 1 skips the third; rank 0 must time out on it.
"""
import multiprocessing as mp
import os
import tempfile
import time
import traceback

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

HQ, HKV, HD, TOTAL = 40, 8, 128, 4096
TIMEOUT_S = 0.02


def _setup(rank, world, device):
    """This rank's shard of a one-sequence cache, inputs and workspace."""
    import ctypes as C
    from picolm_qwen_b200 import abi, sharding
    from picolm_qwen_b200.runtime import rope_table
    torch.cuda.set_device(device)
    L = abi.lib()
    kvd = HKV * HD
    cfg = abi.Config.make(1, HQ, HKV, HD, TOTAL, 1e6)
    off, rows = sharding.shard_rows(TOTAL, world, rank)
    g = torch.Generator(device="cuda").manual_seed(5 + rank)
    kc = (torch.randn((rows, kvd), generator=g, device="cuda") * 0.5).half().view(torch.int16)
    vc = (torch.randn((rows, kvd), generator=g, device="cuda") * 0.5).half().view(torch.int16)
    cos, sin = rope_table(cfg)
    d = dict(cfg=cfg, off=off, rows=rows, kc=kc, vc=vc, cos=torch.from_numpy(cos).cuda(),
             sin=torch.from_numpy(sin).cuda(),
             kp=torch.tensor([kc.data_ptr()], dtype=torch.int64, device="cuda"),
             vp=torch.tensor([vc.data_ptr()], dtype=torch.int64, device="cuda"),
             pos=torch.tensor([TOTAL - 1], dtype=torch.int32, device="cuda"),
             q=torch.randn(HQ * HD, device="cuda"), k=torch.randn(kvd, device="cuda"),
             v=torch.randn(kvd, device="cuda"))
    d["ws_n"] = L.picoattn_decode_workspace_size(C.byref(cfg), 1, rows)
    d["ws"] = torch.zeros(d["ws_n"], dtype=torch.uint8, device="cuda")
    return d


def _call(d, comm, out):
    import ctypes as C
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import stream_handle
    L = abi.lib()
    return L.picoattn_decode_splitkv_p2p(C.byref(d["cfg"]), 0, 1, d["rows"], d["off"], d["rows"], d["q"].data_ptr(),
                                         d["k"].data_ptr(), d["v"].data_ptr(), None, None, d["cos"].data_ptr(),
                                         d["sin"].data_ptr(), d["kp"].data_ptr(), d["vp"].data_ptr(),
                                         d["pos"].data_ptr(), out.data_ptr(), d["ws"].data_ptr(), d["ws_n"], comm,
                                         stream_handle())


def _status(d):
    import ctypes as C
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import stream_handle
    s = C.c_uint32(0)
    assert abi.lib().picoattn_workspace_status(d["ws"].data_ptr(), stream_handle(), C.byref(s)) == 0
    return s.value


def _create(d, world, rank):
    import ctypes as C
    from picolm_qwen_b200 import abi
    L = abi.lib()
    handle = torch.zeros(abi.P2P_HANDLE_BYTES, dtype=torch.uint8)
    comm = C.c_void_p()
    st = L.picoattn_p2p_create(C.byref(d["cfg"]), 1, world, rank, handle.data_ptr(), C.byref(comm))
    assert st == 0, L.picoattn_strerror(st)
    return comm, handle


# ---- one GPU: rank 1 never calls -------------------------------------------

def _silent_rank(handle_q, done_q, ret_q):
    """Rank 1: creates its area on GPU 0, hands over the handle, launches nothing."""
    try:
        from picolm_qwen_b200 import abi
        d = _setup(1, 2, 0)
        comm, handle = _create(d, 2, 1)
        handle_q.put(handle.numpy().tobytes())
        done_q.get(timeout=120)
        assert abi.lib().picoattn_p2p_destroy(comm) == 0
        ret_q.put((1, True, ""))
    except Exception:
        ret_q.put((1, False, traceback.format_exc()))


def _waiting_rank(handle_q, done_q, ret_q):
    """Rank 0 on GPU 0: one call whose exchange wait must run out."""
    try:
        from picolm_qwen_b200 import abi
        L = abi.lib()
        d = _setup(0, 2, 0)
        comm, handle = _create(d, 2, 0)
        other = np.frombuffer(handle_q.get(timeout=120), np.uint8)
        allh = torch.cat([handle, torch.from_numpy(other.copy())]).contiguous()
        assert L.picoattn_p2p_open(comm, allh.data_ptr()) == 0
        assert L.picoattn_p2p_set_timeout(comm, TIMEOUT_S) == 0
        out = torch.zeros(HQ * HD, device="cuda")
        t0 = time.perf_counter()
        assert _call(d, comm, out) == 0
        torch.cuda.synchronize()
        secs = time.perf_counter() - t0
        status = _status(d)
        assert status & abi.DEV_TIMEOUT, f"status {status:#x}"
        assert torch.isnan(out).all(), "outputs of a timed-out exchange must be NaN"
        assert secs < 10, f"the call took {secs:.1f} s"
        # the device stays usable: an ordinary decode on this GPU afterwards
        from picolm_qwen_b200.runtime import AttnState
        st = AttnState(abi.Config.make(1, 8, 2, 64, 128, 1e4), n_seqs=1, max_ctx=128)
        o2 = torch.empty(512, device="cuda")
        assert st.decode_one(0, 5, torch.randn(512, device="cuda"), torch.randn(128, device="cuda"),
                             torch.randn(128, device="cuda"), o2) == 0
        torch.cuda.synchronize()
        assert st.status() == 0 and torch.isfinite(o2).all()
        done_q.put(True)
        assert L.picoattn_p2p_destroy(comm) == 0
        ret_q.put((0, True, f"{secs:.3f} s"))
    except Exception:
        done_q.put(True)
        ret_q.put((0, False, traceback.format_exc()))


def _run(targets, args_list):
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    procs = [ctx.Process(target=t, args=a + (ret,)) for t, a in zip(targets, args_list)]
    for p in procs:
        p.start()
    res = []
    try:
        res = sorted([ret.get(timeout=240) for _ in procs], key=lambda r: r[0])
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, ok, info in res:
        assert ok, f"rank {rank}: {info}"


def test_exchange_wait_times_out_when_a_rank_never_calls_one_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = mp.get_context("spawn")
    handle_q, done_q = ctx.Queue(), ctx.Queue()
    _run([_silent_rank, _waiting_rank], [(handle_q, done_q), (handle_q, done_q)])


# ---- two GPUs: rank 1 skips a call ------------------------------------------

def _skip_rank(rank, store_file, ret_q):
    try:
        from datetime import timedelta
        import torch.distributed as dist
        from picolm_qwen_b200 import abi
        L = abi.lib()
        dist.init_process_group("gloo", store=dist.FileStore(store_file, 2), rank=rank, world_size=2,
                                timeout=timedelta(seconds=60))
        d = _setup(rank, 2, rank)
        comm, handle = _create(d, 2, rank)
        hs = [torch.zeros_like(handle) for _ in range(2)]
        dist.all_gather(hs, handle)
        assert L.picoattn_p2p_open(comm, torch.cat(hs).contiguous().data_ptr()) == 0
        assert L.picoattn_p2p_set_timeout(comm, TIMEOUT_S) == 0
        out = torch.zeros(HQ * HD, device="cuda")
        for call in range(2):  # both ranks call: combined, finite results
            dist.barrier()
            assert _call(d, comm, out) == 0
            torch.cuda.synchronize()
            assert torch.isfinite(out).all(), f"call {call}"
        assert _status(d) == 0
        dist.barrier()
        info = ""
        if rank == 0:  # rank 1 skips this call
            t0 = time.perf_counter()
            assert _call(d, comm, out) == 0
            torch.cuda.synchronize()
            secs = time.perf_counter() - t0
            status = _status(d)
            assert status & abi.DEV_TIMEOUT, f"status {status:#x}"
            assert torch.isnan(out).all()
            assert secs < 10
            info = f"{secs:.3f} s"
        dist.barrier()  # neither rank has kernels in flight now
        assert L.picoattn_p2p_destroy(comm) == 0
        dist.destroy_process_group()
        ret_q.put((rank, True, info))
    except Exception:
        ret_q.put((rank, False, traceback.format_exc()))


def test_exchange_wait_times_out_when_a_rank_skips_a_call_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    store = os.path.join(tempfile.mkdtemp(prefix="picoattn_to_"), "store")
    _run([_skip_rank, _skip_rank], [(0, store), (1, store)])
