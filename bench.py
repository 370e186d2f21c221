#!/usr/bin/env python
"""Benchmark of the B200 attention step (decode attention HBM GB/s).

Workload ("Qwen2.5-7B-shape batched decode"):
28 layers, 28 q heads, 4 KV heads, head_dim 128, RoPE theta 1e6 (NeoX),
64 sequences with cached lengths uniform in [1024, 8192] (seeded), one new token
per sequence per step.  A step is one decode attention pass over all 28 layers
for all 64 sequences: per layer, the new k/v row is appended to each sequence's
FP16 cache and every q head attends over rows 0..pos.  The cache (15.8 GiB of
visited K/V per step, 30 GB allocated) is far larger than L2, so no flush is
needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) the same 64 sequences are dealt to the ranks
longest-first onto the least-loaded rank (strong scaling; no collective on the
data path), the step time is the maximum over ranks, and rank 0 prints one
JSON line.  Further legs in the same line: prefill (Qwen3-8B, 2048 tokens;
KV-head groups sharded across ranks), long-context decode (Qwen2.5-32B, 128K
rows; rows sharded, exchange over NVLink), the two small single-sequence
configurations (TinyLlama at position 511, Qwen2.5-0.5B at 4096; N=1) and the
decode layer with its projections (N=1).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = dict(name="qwen2.5-7b-batched-decode", n_layers=28, n_heads=28, n_kv_heads=4, head_dim=128,
                rope_base=1e6, n_seqs=64, len_lo=1024, len_hi=8192, seed=0)
METRIC = "decode attn HBM GB/s"


def seq_lengths(rank: int) -> np.ndarray:
    """Cached lengths per sequence; the new token sits at pos = length."""
    rng = np.random.default_rng(WORKLOAD["seed"] + rank)
    return rng.integers(WORKLOAD["len_lo"], WORKLOAD["len_hi"] + 1, WORKLOAD["n_seqs"]).astype(np.int32)


def step_bytes(lens: np.ndarray, n_layers: int, kv_dim: int) -> int:
    """Algorithmic bytes of one step: K and V rows 0..pos of every sequence, every layer."""
    return int(n_layers * np.sum(2 * (lens.astype(np.int64) + 1) * kv_dim * 2))


def measured_peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(leg: str = "batched") -> float | None:
    """DRAM bytes per attention launch of a leg from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "decode_attn_traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["dram_bytes_per_launch"] if leg == "batched" else d[leg]["dram_bytes_per_launch"])
    except Exception:
        return None


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML reads only; nothing is changed)
# ---------------------------------------------------------------------------

class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, device_index: int, props=None):
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            h = None
            # the CUDA device under CUDA_VISIBLE_DEVICES: match by UUID, then PCI address
            if props is not None:
                try:
                    u = str(props.uuid)
                    h = pynvml.nvmlDeviceGetHandleByUUID(u if u.startswith("GPU-") else "GPU-" + u)
                except Exception:
                    h = None
                if h is None:
                    try:
                        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
                        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
                    except Exception:
                        h = None
            self.h = h if h is not None else pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU side: the reference's attention loop (oracle/_ref) or the oracle port
# ---------------------------------------------------------------------------

def cpu_attention_runner():
    """Returns (run(B-seq sample) -> seconds, kind).  Test/baseline use only."""
    from oracle import pyoracle
    if os.path.exists(pyoracle.REF_SO):
        return pyoracle.RefHarness(), "reference"
    pyoracle.build()
    return pyoracle.Oracle(), "port"


def make_host_sample(lens: np.ndarray, kv_dim: int, rng: np.random.Generator):
    S = int(lens.max()) + 1
    kcs, vcs = [], []
    for n in lens:
        kc = np.zeros((S, kv_dim), np.uint16)
        vc = np.zeros((S, kv_dim), np.uint16)
        kc[:n] = (rng.standard_normal((int(n), kv_dim), dtype=np.float32) * 0.5).astype(np.float16).view(np.uint16)
        vc[:n] = (rng.standard_normal((int(n), kv_dim), dtype=np.float32) * 0.5).astype(np.float16).view(np.uint16)
        kcs.append(kc)
        vcs.append(vc)
    return S, kcs, vcs


_ROPE_CACHE: dict = {}


def run_cpu_sample(runner, lens, S, kcs, vcs, n_threads, rng):
    """One decode attention pass of one layer over len(lens) sequences on the host."""
    from oracle.pyoracle import Oracle
    w = WORKLOAD
    hq, hkv, hd = w["n_heads"], w["n_kv_heads"], w["head_dim"]
    B = len(lens)
    if S not in _ROPE_CACHE:  # the table is bit-identical to the reference's (tests pin it)
        _ROPE_CACHE[S] = Oracle().rope_table(S, hd, w["rope_base"])
    cos_t, sin_t = _ROPE_CACHE[S]
    q = rng.standard_normal((B, hq * hd), dtype=np.float32)
    k = rng.standard_normal((B, hkv * hd), dtype=np.float32)
    v = rng.standard_normal((B, hkv * hd), dtype=np.float32)
    pos = lens.astype(np.int32)
    t0 = time.perf_counter()
    if isinstance(runner, Oracle):
        runner.decode_batch(hq, hkv, hd, 0, q, k, v, None, None, cos_t, sin_t, kcs, vcs, pos, n_threads)
    else:
        runner.attn_decode_batch(hq, hkv, hd, 0, q, k, v, None, None, cos_t, sin_t, kcs, vcs, pos, n_threads)
    return time.perf_counter() - t0


def cpu_baseline(lens: np.ndarray) -> dict:
    """All host threads over a bounded sample: the 64 sequences of one layer."""
    w = WORKLOAD
    kvd = w["n_kv_heads"] * w["head_dim"]
    rng = np.random.default_rng(1234)
    runner, kind = cpu_attention_runner()
    S, kcs, vcs = make_host_sample(lens, kvd, rng)
    cores = os.cpu_count() or 1
    secs = run_cpu_sample(runner, lens, S, kcs, vcs, cores, rng)
    gbs = step_bytes(lens, 1, kvd) / secs / 1e9
    # reference-faithful: one thread, as the reference runs its attention loop
    n1 = 4
    secs1 = run_cpu_sample(runner, lens[:n1], S, kcs[:n1], vcs[:n1], 1, rng)
    gbs1 = step_bytes(lens[:n1], 1, kvd) / secs1 / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"1 of 28 layers x {len(lens)} sequences (same lengths), {secs:.2f} s wall, "
                      f"one host thread per sequence; the reference's attention loop (cpp/model.hpp:326-418) "
                      f"compiled from its sources",
            "one_core": {"value": round(gbs1, 4), "unit": "GB/s", "cores": 1, "kind": kind,
                         "sample": f"1 layer x the first {n1} sequences on one thread ({secs1:.2f} s), "
                                   f"the reference's own single-threaded loop"}}


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = WORKLOAD
    kvd = w["n_kv_heads"] * w["head_dim"]
    lens = seq_lengths(0)
    runner, kind = cpu_attention_runner()
    rng = np.random.default_rng(1234)
    cores = os.cpu_count() or 1
    # size each step so that warmup+steps end within ~2 minutes
    n_sample = len(lens)
    S, kcs, vcs = make_host_sample(lens[:n_sample], kvd, rng)
    probe = run_cpu_sample(runner, lens[:8], S, kcs[:8], vcs[:8], cores, rng)
    per_seq = probe / 8 * min(8, cores) / max(1, min(n_sample, cores))
    budget = 120.0 / max(1, args.steps + args.warmup)
    n_sample = int(max(1, min(len(lens), budget / max(per_seq, 1e-6))))
    sample_lens = lens[:n_sample]
    for _ in range(args.warmup):
        run_cpu_sample(runner, sample_lens, S, kcs[:n_sample], vcs[:n_sample], cores, rng)
    total = 0.0
    for _ in range(args.steps):
        total += run_cpu_sample(runner, sample_lens, S, kcs[:n_sample], vcs[:n_sample], cores, rng)
    nbytes = step_bytes(sample_lens, 1, kvd) * args.steps
    gbs = nbytes / total / 1e9
    line = {"metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 (fp16 cache)", "data": "synthetic",
            "config": {"workload": w["name"] + " (CPU sample)", "layers_per_step": 1, "sequences": n_sample,
                       "heads": [w["n_heads"], w["n_kv_heads"], w["head_dim"]]},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                             "sample": f"{n_sample} sequences x 1 layer per step"},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, stream_handle

    from picolm_qwen_b200 import sharding

    w = WORKLOAD
    L, hq, hkv, hd = w["n_layers"], w["n_heads"], w["n_kv_heads"], w["head_dim"]
    kvd, qd = hkv * hd, hq * hd
    lens_all = seq_lengths(0)
    mine = sharding.lpt_assign(lens_all, world)[rank]  # this rank's sequences (strong scaling)
    lens = lens_all[mine]
    B = len(lens)
    S = int(lens.max()) + 1
    max_ctx = S
    cfg = abi.Config.make(L, hq, hkv, hd, S, w["rope_base"], abi.ROPE_NEOX)
    st = AttnState(cfg, n_seqs=B, device=dev, max_ctx=max_ctx)
    # synthetic cache rows 0..len-1, N(0, 0.5^2) in fp16
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    for b in range(B):
        n = int(lens[b])
        for cache in (st.k_cache, st.v_cache):
            cache[b, :, :n].copy_((torch.randn((L, n, kvd), generator=g, device=dev) * 0.5)
                                  .to(torch.float16).view(torch.int16))
    q = torch.randn((L, B, qd), generator=g, device=dev)
    k = torch.randn((L, B, kvd), generator=g, device=dev)
    v = torch.randn((L, B, kvd), generator=g, device=dev)
    out = torch.empty((L, B, qd), device=dev)
    pos = torch.from_numpy(lens).to(dev)
    stream = torch.cuda.current_stream(dev)
    sh = stream_handle(stream)
    lib = abi.lib()
    cfgp = C.byref(cfg)
    common = (st.rope_cos.data_ptr(), st.rope_sin.data_ptr(), st.k_ptrs.data_ptr(), st.v_ptrs.data_ptr(),
              pos.data_ptr())

    # every pointer precomputed: the timed loop is one C call per stage
    layer_ptrs = [(q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(), out[l].data_ptr()) for l in range(L)]
    ws_ptr, ws_n = st.workspace.data_ptr(), st.workspace.numel()

    def call(l, stages, qq=None, kk=None, vv=None, oo=None, stream_h=None):
        pq, pk, pv, po = layer_ptrs[l]
        if qq is not None:
            pq, pk, pv, po = qq.data_ptr(), kk.data_ptr(), vv.data_ptr(), oo.data_ptr()
        s = lib.picoattn_decode_staged(cfgp, l, B, max_ctx, pq, pk, pv, None, None, *common, po, ws_ptr, ws_n,
                                       sh if stream_h is None else stream_h, stages)
        if s != 0:
            raise abi.PicoAttnError(s, "picoattn_decode_staged")

    def one_step(ev_pairs=None):
        for l in range(L):
            if ev_pairs is None:
                call(l, abi.STAGE_ALL)
            else:
                a, b_ = ev_pairs[l]
                call(l, abi.STAGE_PREPARE)
                a.record(stream)
                call(l, abi.STAGE_ATTEND)
                b_.record(stream)
                call(l, abi.STAGE_COMBINE)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        one_step()
    barrier()
    assert st.status() == 0
    props = torch.cuda.get_device_properties(dev)
    # The step (28 layers x one ABI call) is captured once into a CUDA graph and
    # replayed: per-kernel host launch cost leaves the timed region, the work
    # does not (the library's calls are stream-ordered, allocate nothing and do
    # not synchronise, so they capture as plain kernel nodes).
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gh = torch.cuda.current_stream(dev).cuda_stream
        for l in range(L):
            call(l, abi.STAGE_ALL, stream_h=gh)
    graph.replay()
    barrier()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, props) as clk:
        t_start.record(stream)
        for i in range(args.steps):
            graph.replay()
        t_end.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    # The attention kernel alone: the same K steps launched directly, a CUDA
    # event pair around every ATTEND launch on the launching stream.
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
          for _ in range(args.steps)]
    for i in range(args.steps):
        one_step(ev[i])
    torch.cuda.synchronize(dev)
    attn_ms = [a.elapsed_time(b_) for step in ev for (a, b_) in step]
    del graph
    status = st.status()
    if status != 0:
        raise RuntimeError(f"device status {status:#x} after the timed region")

    # e2e through the C ABI with pinned host buffers: every layer uploads its
    # q|k|v (one contiguous pinned block, one copy), runs the call and reads its
    # output back, each step on the stream in that order -- as a drop-in
    # forward must, where the next layer's inputs come from this layer's output.
    # The 28-layer step is captured as one CUDA graph (copy and kernel nodes), so
    # the host's per-call launch overhead leaves the timed region and the copies
    # and kernels do not.
    qn, kn = q[0].numel(), k[0].numel()
    qkv_host = torch.empty((L, qn + 2 * kn), dtype=torch.float32).pin_memory()
    qkv_host[:, :qn] = q.reshape(L, qn).cpu()
    qkv_host[:, qn:qn + kn] = k.reshape(L, kn).cpu()
    qkv_host[:, qn + kn:] = v.reshape(L, kn).cpu()
    hout = torch.empty((L, B, qd), dtype=torch.float32).pin_memory()
    dqkv, dout = torch.empty(qn + 2 * kn, dtype=torch.float32, device=dev), torch.empty_like(out[0])
    dq, dk, dv = dqkv[:qn].view_as(q[0]), dqkv[qn:qn + kn].view_as(k[0]), dqkv[qn + kn:].view_as(v[0])

    def e2e_step(stream_h=None):
        for l in range(L):
            dqkv.copy_(qkv_host[l], non_blocking=True)
            call(l, abi.STAGE_ALL, dq, dk, dv, dout, stream_h=stream_h)
            hout[l].copy_(dout, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier()
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_step(torch.cuda.current_stream(dev).cuda_stream)
    e2e_graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    barrier()
    del e2e_graph
    # the graph's output copies landed: the last step's outputs equal the resident path's
    if not torch.equal(hout.to(dev), out.reshape(hout.shape)):
        raise RuntimeError("e2e outputs differ from the resident path's")

    del st  # free the decode caches before the prefill leg
    prefill_line = None
    if not args.no_prefill:
        torch.cuda.empty_cache()
        prefill_line = run_prefill(args, dev, world, rank, local)
    longctx_line = None
    if not args.no_longctx:
        torch.cuda.empty_cache()
        longctx_line = run_longctx(args, dev, world, rank, local)
    layer_line = None
    if world == 1 and not args.no_layer:
        torch.cuda.empty_cache()
        layer_line = run_layer(args, dev)
    step_line = None
    if world == 1 and not args.no_step:
        torch.cuda.empty_cache()
        step_line = run_token_step(args, dev)
    small_lines = []
    if world == 1 and not args.no_small:
        for spec in SMALL:
            torch.cuda.empty_cache()
            small_lines.append(run_small(args, dev, spec))

    nbytes = step_bytes(lens, L, kvd)
    total_bytes = float(step_bytes(lens_all, L, kvd))  # the whole job: every sequence once per step
    h2d_rank, d2h_rank = int(L * qkv_host[0].numel() * 4), int(L * hout[0].numel() * 4)
    times = torch.tensor([elapsed_ms, e2e_ms, float(h2d_rank), float(d2h_rank)], dtype=torch.float64, device=dev)
    if world > 1:
        tmax = times.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = times.clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        elapsed_ms, e2e_ms = float(tmax[0]), float(tmax[1])
        h2d_all, d2h_all = int(tsum[2]), int(tsum[3])
    else:
        h2d_all, d2h_all = h2d_rank, d2h_rank

    if rank == 0:
        value = total_bytes * args.steps / (elapsed_ms / 1e3) / 1e9
        e2e_value = total_bytes * args.steps / (e2e_ms / 1e3) / 1e9
        per_launch = nbytes / L
        mean_attn_ms = float(np.mean(attn_ms))
        achieved = per_launch / (mean_attn_ms / 1e3) / 1e9
        peak, peak_kind = measured_peaks()
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f16 cache; q (pre-scaled) and softmax P rounded to f16 as tensor-core operands; f32 accumulate",
            "data": "synthetic",
            "config": {"workload": w["name"], "layers": L, "sequences": len(lens_all),
                       "sequences_rank0": B, "heads_q_kv_dim": [hq, hkv, hd],
                       "cached_len_range": [w["len_lo"], w["len_hi"]], "bytes_per_step": int(total_bytes),
                       "bytes_per_step_rank0": nbytes, "l2": "inputs (15.8 GiB/step) larger than L2, no flush",
                       "parallelism": (f"sequences dealt to {world} GPUs longest-first (LPT), no collective"
                                       if world > 1 else "single GPU")},
            "roofline": {"bound": "hbm", "kernel": "decode_attn_kernel<128>", "achieved": round(achieved, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": profiled_traffic(), "algorithmic_bytes_per_launch": per_launch,
                         "mean_launch_ms": round(mean_attn_ms, 5)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d_all, "d2h_bytes_per_step": d2h_all,
                    "timing": "CUDA graph of the 28 per-layer uploads, calls and read-backs; max over ranks"},
            "gpu_launches": 3 * L * args.steps,
            "clocks": clocks,
        }
        if prefill_line is not None:
            line["prefill"] = prefill_line
        if longctx_line is not None:
            line["long_context"] = longctx_line
        if layer_line is not None:
            line["decode_layer"] = layer_line
        if step_line is not None:
            line["token_step"] = step_line
        for sl in small_lines:
            line["small_cfg%d" % sl["config"]["baseline_config"]] = sl
        if world == 1 and not args.no_cpu:
            try:
                line["cpu_baseline"] = cpu_baseline(lens)
            except Exception as e:  # the CPU leg never hides a GPU number
                line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


PREFILL = dict(name="qwen3-8b-prefill", n_layers=36, n_heads=32, n_kv_heads=8, head_dim=128, rope_base=1e6,
               n_tok=2048, seed=0)


def prefill_flops(n_tok: int, n_heads: int, head_dim: int) -> float:
    """QK^T + PV over causally visible (query, key) pairs only: 4*H*hd*S(S+1)/2."""
    return 4.0 * n_heads * head_dim * n_tok * (n_tok + 1) / 2


def run_prefill(args, dev, world, rank, local) -> dict:
    """36 layers x 2048-token prompt, QK-norm, fp16 q/k/v in.
    Across N GPUs the KV-head groups are dealt to the ranks (sharding.kv_head_groups):
    each rank holds the q/k/v columns and the cache of its KV heads, as in a
    tensor-parallel layer, and calls picoattn_prefill with a config of its
    heads; attention needs no exchange.  Total work is fixed (strong scaling)."""
    import torch
    import torch.distributed as dist
    from picolm_qwen_b200 import abi, sharding
    from picolm_qwen_b200.runtime import AttnState, stream_handle

    p = PREFILL
    L, hq_all, hkv_all, hd, n = p["n_layers"], p["n_heads"], p["n_kv_heads"], p["head_dim"], p["n_tok"]
    groups = sharding.kv_head_groups(hkv_all, world, rank)
    hkv = len(groups)
    hq = hkv * (hq_all // hkv_all)  # this rank's q heads
    kvd = hkv * hd
    cfg = abi.Config.make(L, hq, hkv, hd, n, p["rope_base"], abi.ROPE_NEOX)
    st = AttnState(cfg, n_seqs=1, device=dev, max_ctx=1)
    g = torch.Generator(device=dev)
    g.manual_seed(2000 + rank)
    q = torch.randn((L, n, hq * hd), generator=g, device=dev).half()
    k = torch.randn((L, n, kvd), generator=g, device=dev).half()
    v = torch.randn((L, n, kvd), generator=g, device=dev).half()
    qn = 1 + 0.1 * torch.randn((L, hd), generator=g, device=dev)
    kn = 1 + 0.1 * torch.randn((L, hd), generator=g, device=dev)
    out = torch.empty((n, hq * hd), device=dev)
    ws = st.prefill_workspace(n)
    stream = torch.cuda.current_stream(dev)
    lib = abi.lib()
    cfgp = C.byref(cfg)
    sh = stream_handle(stream)
    # every pointer precomputed: the timed loop is one C call per stage
    ptrs = [(q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(), qn[l].data_ptr(), kn[l].data_ptr())
            for l in range(L)]
    tail = (st.rope_cos.data_ptr(), st.rope_sin.data_ptr(), st.k_cache[0].data_ptr(), st.v_cache[0].data_ptr(),
            out.data_ptr(), ws.data_ptr(), ws.numel(), sh)

    def layer_call(l, stages, stream_h=None):
        t = tail if stream_h is None else tail[:-1] + (stream_h,)
        s = lib.picoattn_prefill_staged(cfgp, l, n, 0, abi.DTYPE_F16, *ptrs[l], *t, stages)
        if s != 0:
            raise abi.PicoAttnError(s, "picoattn_prefill_staged")

    def step(evs=None):
        for l in range(L):
            if evs is None:
                layer_call(l, abi.STAGE_PREPARE | abi.STAGE_ATTEND)
            else:
                layer_call(l, abi.STAGE_PREPARE)
                evs[l][0].record(stream)
                layer_call(l, abi.STAGE_ATTEND)
                evs[l][1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    steps = max(3, args.steps // 10)
    # the 36-layer step as one CUDA graph (see the decode leg), replayed
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gh = torch.cuda.current_stream(dev).cuda_stream
        for l in range(L):
            layer_call(l, abi.STAGE_PREPARE | abi.STAGE_ATTEND, stream_h=gh)
    graph.replay()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize(dev)
    t0.record(stream)
    for i in range(steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1)
    del graph
    # the prep kernel alone, as a graph of its 36 launches: the step time per
    # layer less this is the attention kernel's share of the step (there its
    # launch and set-up run under the prep kernel before it)
    pgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(pgraph):
        gh = torch.cuda.current_stream(dev).cuda_stream
        for l in range(L):
            layer_call(l, abi.STAGE_PREPARE, stream_h=gh)
    pgraph.replay()
    torch.cuda.synchronize(dev)
    t0.record(stream)
    for i in range(steps):
        pgraph.replay()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    prep_graph_ms = t0.elapsed_time(t1)
    del pgraph
    step_ms_local = ms
    # the attention kernel alone: event pairs around every ATTEND launch
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
           for _ in range(steps)]
    for i in range(steps):
        step(evs[i])
    torch.cuda.synchronize(dev)
    attn_ms = float(np.mean([a.elapsed_time(b) for e in evs for (a, b) in e]))
    if st.status() != 0:
        raise RuntimeError("prefill device status set")
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    flops_layer = prefill_flops(n, hq, hd)  # this rank's launch
    total = prefill_flops(n, hq_all, hd) * L * steps  # the whole job
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = float(peaks.get("bf16_tflops", 1590.0))
    achieved = flops_layer / (attn_ms / 1e3) / 1e12
    in_step_us = (step_ms_local - prep_graph_ms) / steps / L * 1e3
    variant = lib.picoattn_prefill_kernel(cfgp)
    kernel = {abi.PREFILL_CTA_PAIR: "prefill_attn_pair_kernel (2-SM CTA pair, tcgen05 cta_group::2)",
              abi.PREFILL_HEAD_PAIR: "prefill_attn2_kernel<128> (head pair, 1 SM)",
              abi.PREFILL_SINGLE: "prefill_attn_kernel<128> (single head)"}.get(variant, f"status {variant}")
    return {"metric": "prefill attn TFLOP/s", "value": round(total / (ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
            "steps": steps, "ms_per_step": round(ms / steps, 4), "scaling": "strong",
            "dtype": "f16 operands (q, k, v, softmax P), f32 accumulate",
            "config": {"workload": p["name"], "layers": L, "heads_q_kv_dim": [hq_all, hkv_all, hd],
                       "heads_q_kv_rank0": [hq, hkv], "prompt_tokens": n,
                       "qk_norm": True, "flops_per_step": prefill_flops(n, hq_all, hd) * L,
                       "flops_note": "causally visible pairs only, QK^T + PV",
                       "parallelism": (f"KV-head groups dealt to {world} GPUs, no exchange" if world > 1
                                       else "single GPU")},
            "roofline": {"bound": "tensor", "kernel": kernel, "achieved": round(achieved, 1),
                         "peak": peak, "peak_kind": "measured" if peaks else "fallback", "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "mean_launch_ms": round(attn_ms, 5),
                         "algorithmic_flops_per_launch": flops_layer},
            "prep_ms_per_layer": round(ms / steps / L - attn_ms, 5),
            "in_step": {"method": "graph step time per layer less the prep kernel's time per layer in a graph of "
                                  "its launches alone (this rank)",
                        "prep_us_per_layer": round(prep_graph_ms / steps / L * 1e3, 2),
                        "attention_us_per_layer": round(in_step_us, 2),
                        "attention_tflops": round(flops_layer / (in_step_us / 1e6) / 1e12, 1),
                        "frac": round(flops_layer / (in_step_us / 1e6) / 1e12 / peak, 4)}}


LONGCTX = dict(name="qwen2.5-32b-128k-decode", n_layers=64, n_heads=40, n_kv_heads=8, head_dim=128,
               rope_base=1e6, ctx=131072, seed=0)


def run_longctx(args, dev, world, rank, local) -> dict:
    """one sequence, 131071 cached rows + the new token
    at position 131071, 64 layers.  Sequence-sharded: rank g holds the
    contiguous rows [off_g, off_g + n_g) of every layer and attends only those;
    for N > 1 each layer's shard results go to every rank over peer memory and
    are combined by log-sum-exp on every rank, in one kernel
    (picoattn_decode_splitkv_p2p; the IPC handles travel over the process
    group).  Total work is fixed (strong scaling); value = the whole step's K/V
    bytes / step time."""
    import torch
    import torch.distributed as dist
    from picolm_qwen_b200 import abi, sharding
    from picolm_qwen_b200.runtime import stream_handle

    p = LONGCTX
    L, hq, hkv, hd, S = p["n_layers"], p["n_heads"], p["n_kv_heads"], p["head_dim"], p["ctx"]
    kvd, qd = hkv * hd, hq * hd
    pos_new = S - 1
    off, rows = sharding.shard_rows(S, world, rank)
    cfg = abi.Config.make(L, hq, hkv, hd, S, p["rope_base"], abi.ROPE_NEOX)
    lib = abi.lib()
    cfgp = C.byref(cfg)
    g = torch.Generator(device=dev)
    g.manual_seed(3000 + rank)
    # this rank's rows of every layer, N(0, 0.5^2) in fp16 (the new row is written by its owner)
    kc = torch.empty((L, rows, kvd), dtype=torch.int16, device=dev)
    vc = torch.empty_like(kc)
    for cache in (kc, vc):
        for l in range(L):
            cache[l].copy_((torch.randn((rows, kvd), generator=g, device=dev) * 0.5).half().view(torch.int16))
    q = torch.randn((L, qd), generator=g, device=dev)
    k = torch.randn((L, kvd), generator=g, device=dev)
    v = torch.randn((L, kvd), generator=g, device=dev)
    out = torch.empty((L, qd), device=dev)
    cos = np.empty(S * hd // 2, np.float32)
    sin = np.empty_like(cos)
    assert lib.picoattn_rope_table(cfgp, cos.ctypes.data, sin.ctypes.data) == 0
    d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    kp = torch.tensor([kc.data_ptr()], dtype=torch.int64, device=dev)
    vp = torch.tensor([vc.data_ptr()], dtype=torch.int64, device=dev)
    pos = torch.tensor([pos_new], dtype=torch.int32, device=dev)
    ws_n = lib.picoattn_decode_workspace_size(cfgp, 1, rows)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device=dev)
    assert lib.picoattn_workspace_init(ws.data_ptr(), ws_n, stream_handle()) == 0
    comm = C.c_void_p()
    if world > 1:
        handle = torch.zeros(abi.P2P_HANDLE_BYTES, dtype=torch.uint8)
        st = lib.picoattn_p2p_create(cfgp, 1, world, rank, handle.data_ptr(), C.byref(comm))
        if st != 0:
            raise abi.PicoAttnError(st, "picoattn_p2p_create")
        hs = [torch.zeros(abi.P2P_HANDLE_BYTES, dtype=torch.uint8, device=dev) for _ in range(world)]
        dist.all_gather(hs, handle.to(dev))
        allh = torch.cat([h.cpu() for h in hs]).contiguous()
        st = lib.picoattn_p2p_open(comm, allh.data_ptr())
        if st != 0:
            raise abi.PicoAttnError(st, "picoattn_p2p_open")
    common = (d_cos.data_ptr(), d_sin.data_ptr(), kp.data_ptr(), vp.data_ptr(), pos.data_ptr())

    def layer(l, sh):
        if world == 1:
            st = lib.picoattn_decode_staged(cfgp, l, 1, S, q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(),
                                            None, None, *common, out[l].data_ptr(), ws.data_ptr(), ws_n, sh,
                                            abi.STAGE_ALL)
        else:
            st = lib.picoattn_decode_splitkv_p2p(cfgp, l, 1, rows, off, rows, q[l].data_ptr(), k[l].data_ptr(),
                                                 v[l].data_ptr(), None, None, *common, out[l].data_ptr(),
                                                 ws.data_ptr(), ws_n, comm, sh)
        if st != 0:
            raise abi.PicoAttnError(st, "long-context decode")

    stream = torch.cuda.current_stream(dev)
    sh = stream_handle(stream)

    def step(stream_h):
        for l in range(L):
            layer(l, stream_h)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    for _ in range(max(3, args.warmup)):
        step(sh)
    barrier()
    steps = max(5, args.steps // 4)
    timing = "graph"
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph):
            step(torch.cuda.current_stream(dev).cuda_stream)
        graph.replay()
        torch.cuda.synchronize(dev)
    except Exception:
        graph, timing = None, "eager"
        torch.cuda.synchronize(dev)
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        if graph is not None:
            graph.replay()
        else:
            step(sh)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1)
    barrier()
    if graph is not None:
        del graph
    roof = None
    if world == 1:
        # the call's kernels (attention with the new row's append, and the merge
        # of its pieces): events around each one-sequence call
        att = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
        for l in range(L):
            att[l][0].record(stream)
            layer(l, sh)
            att[l][1].record(stream)
        torch.cuda.synchronize(dev)
        attn_ms = float(np.mean([a.elapsed_time(b) for a, b in att]))
        per_launch = 2 * S * kvd * 2
        peak, peak_kind = measured_peaks()
        ach = per_launch / (attn_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "kernel": "decode_attn_kernel<128> + decode_merge_seq_kernel<128> (one call)",
                "achieved": round(ach, 1), "peak": peak,
                "peak_kind": peak_kind, "unit": "GB/s", "frac": round(ach / peak, 4),
                "mean_launch_ms": round(attn_ms, 5), "algorithmic_bytes_per_launch": per_launch,
                "traffic": profiled_traffic("long_context")}
    dev_status = C.c_uint32(0)
    lib.picoattn_workspace_status(ws.data_ptr(), sh, C.byref(dev_status))
    if dev_status.value != 0:
        raise RuntimeError(f"long-context device status {dev_status.value:#x}")
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
        dist.barrier(device_ids=[local])  # every rank's last exchange is done before the areas go
        lib.picoattn_p2p_destroy(comm)
    total_bytes = float(L) * 2 * S * kvd * 2  # every layer's K and V rows 0..131071, all ranks together
    extra = {"roofline": roof} if roof is not None else {}
    return {**extra, "metric": "long-context decode attn HBM GB/s",
            "value": round(total_bytes * steps / (ms / 1e3) / 1e9, 2),
            "unit": "GB/s", "ms_per_step": round(ms / steps, 4), "steps": steps, "scaling": "strong",
            "timing": timing,
            "config": {"workload": p["name"], "layers": L, "heads_q_kv_dim": [hq, hkv, hd], "cached_rows": S - 1,
                       "rows_per_gpu": rows, "bytes_per_step": total_bytes,
                       "parallelism": f"sequence-sharded x{world}, per-layer exchange + LSE combine in one kernel "
                                      "over NVLink peer memory"
                       if world > 1 else "single GPU"}}


SMALL = (
    dict(name="tinyllama-1.1b-decode-p511", cfg=1, n_layers=22, n_heads=32, n_kv_heads=4, head_dim=64,
         rope_base=1e4, rope_mode=1, pos=511, seed=0),
    dict(name="qwen2.5-0.5b-decode-4096", cfg=2, n_layers=24, n_heads=14, n_kv_heads=2, head_dim=64,
         rope_base=1e6, rope_mode=0, pos=4095, seed=0),
)


def run_small(args, dev, spec) -> dict:
    """BASELINE.json configs[0] and [1]: one sequence, one new token at `pos` in
    every layer (TinyLlama with interleaved RoPE at 511; Qwen2.5-0.5B at 4095).
    The step (every layer's picoattn_decode call) is one CUDA graph.  The whole
    step's K/V (11 MiB / 48 MiB) fits in L2, so a 512 MiB buffer is written
    between timed steps and every step is timed alone with CUDA events.  The
    reference's loop is timed on one host thread over the same step."""
    import torch
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, stream_handle

    L, hq, hkv, hd = spec["n_layers"], spec["n_heads"], spec["n_kv_heads"], spec["head_dim"]
    kvd, qd, p = hkv * hd, hq * hd, spec["pos"]
    S = p + 1
    lib = abi.lib()
    cfg = abi.Config.make(L, hq, hkv, hd, S, spec["rope_base"], spec["rope_mode"])
    cfgp = C.byref(cfg)
    st = AttnState(cfg, n_seqs=1, device=dev, max_ctx=S)
    g = torch.Generator(device=dev).manual_seed(4000 + spec["cfg"])
    for c in (st.k_cache, st.v_cache):
        c[0, :, :p].copy_((torch.randn((L, p, kvd), generator=g, device=dev) * 0.5).half().view(torch.int16))
    q = torch.randn((L, qd), generator=g, device=dev)
    k = torch.randn((L, kvd), generator=g, device=dev)
    v = torch.randn((L, kvd), generator=g, device=dev)
    out = torch.empty((L, qd), device=dev)
    pos = torch.tensor([p], dtype=torch.int32, device=dev)
    common = (st.rope_cos.data_ptr(), st.rope_sin.data_ptr(), st.k_ptrs.data_ptr(), st.v_ptrs.data_ptr(),
              pos.data_ptr())
    ws, ws_n = st.workspace.data_ptr(), st.workspace.numel()

    def call(l, stages, sh):
        r = lib.picoattn_decode_staged(cfgp, l, 1, S, q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(), None,
                                       None, *common, out[l].data_ptr(), ws, ws_n, sh, stages)
        if r != 0:
            raise abi.PicoAttnError(r, "picoattn_decode_staged")

    stream = torch.cuda.current_stream(dev)
    sh = stream_handle(stream)
    for _ in range(max(3, args.warmup)):
        for l in range(L):
            call(l, abi.STAGE_ALL, sh)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gh = torch.cuda.current_stream(dev).cuda_stream
        for l in range(L):
            call(l, abi.STAGE_ALL, gh)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    for _ in range(3):
        flush.zero_()
        graph.replay()
    steps = max(5, args.steps // 4)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    del graph
    # the call's kernels (attention, merge): events around every one-sequence
    # call, L2 flushed per step
    att = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
           for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        for l in range(L):
            att[i][l][0].record(stream)
            call(l, abi.STAGE_ALL, sh)
            att[i][l][1].record(stream)
    torch.cuda.synchronize(dev)
    attn_ms = float(np.mean([a.elapsed_time(b) for e in att for (a, b) in e]))
    if st.status() != 0:
        raise RuntimeError(f"{spec['name']}: device status set")
    step_b = L * 2 * S * kvd * 2
    layer_b = 2 * S * kvd * 2
    peak, peak_kind = measured_peaks()
    gbs = step_b / (ms / 1e3) / 1e9
    line = {"metric": "decode attn HBM GB/s", "value": round(gbs, 2), "unit": "GB/s", "steps": steps,
            "ms_per_step": round(ms, 5), "us_per_layer": round(ms / L * 1e3, 3),
            "config": {"workload": spec["name"], "baseline_config": spec["cfg"], "layers": L,
                       "heads_q_kv_dim": [hq, hkv, hd], "pos": p,
                       "rope": "interleaved" if spec["rope_mode"] == 1 else "neox", "bytes_per_step": step_b,
                       "l2": "512 MiB written between timed steps; each step timed alone",
                       "timing": f"CUDA graph of the {L} layer calls"},
            "roofline": {"bound": "hbm (launch-latency dominated at this size)",
                         "kernel": "decode_attn_kernel<64> + decode_merge_seq_kernel<64> (one call)",
                         "achieved": round(layer_b / (attn_ms / 1e3) / 1e9, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(layer_b / (attn_ms / 1e3) / 1e9 / peak, 4),
                         "mean_launch_ms": round(attn_ms, 5), "algorithmic_bytes_per_launch": layer_b,
                         "step_frac": round(gbs / peak, 4)}}
    del st, flush
    if not args.no_cpu:
        try:
            from oracle import pyoracle
            runner = pyoracle.RefHarness() if os.path.exists(pyoracle.REF_SO) else None
            kind = "reference"
            if runner is None:
                pyoracle.build()
                runner, kind = pyoracle.Oracle(), "port"
            rng = np.random.default_rng(spec["seed"])
            kcs = [np.zeros((S, kvd), np.uint16) for _ in range(L)]
            vcs = [np.zeros((S, kvd), np.uint16) for _ in range(L)]
            for a in kcs + vcs:
                a[:p] = (rng.standard_normal((p, kvd), dtype=np.float32) * 0.5).astype(np.float16).view(np.uint16)
            ct, stt = pyoracle.Oracle().rope_table(S, hd, spec["rope_base"])
            hq_, hkv_, hd_ = hq, hkv, hd
            t0 = time.perf_counter()
            for l in range(L):  # the reference's forward: one layer after another, one thread
                qq = rng.standard_normal((1, qd), dtype=np.float32)
                kk = rng.standard_normal((1, kvd), dtype=np.float32)
                vv = rng.standard_normal((1, kvd), dtype=np.float32)
                pp = np.array([p], np.int32)
                if kind == "reference":
                    runner.attn_decode_batch(hq_, hkv_, hd_, spec["rope_mode"], qq, kk, vv, None, None, ct, stt,
                                             [kcs[l]], [vcs[l]], pp, 1)
                else:
                    runner.decode_batch(hq_, hkv_, hd_, spec["rope_mode"], qq, kk, vv, None, None, ct, stt,
                                        [kcs[l]], [vcs[l]], pp, 1)
            secs = time.perf_counter() - t0
            line["cpu_baseline"] = {"value": round(step_b / secs / 1e9, 4), "unit": "GB/s", "cores": 1,
                                    "kind": kind, "sample": f"the whole {L}-layer step on one thread "
                                                            f"({secs * 1e3:.1f} ms), as the reference runs it"}
        except Exception as e:  # the CPU leg never hides a GPU number
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    return line


LAYER = dict(name="qwen2.5-7b-decode-layer-q4km", n_layers=28, n_heads=28, n_kv_heads=4, head_dim=128, dim=3584,
             rope_base=1e6, ctx=4096, types=(13, 13, 15, 13), seed=0)


def run_layer(args, dev) -> dict:
    """The attention block of a whole decode step on the device
    (picoattn_decode_layer: q/k/v projections with biases in one kernel, the
    decode step, the output projection into the residual), Qwen2.5-7B shape,
    one sequence at position ctx - 1, Q4_K_M-style weights (q, k, o Q4_K; v
    Q6_K; seeded random blocks), each layer its own weights; the 28 calls
    replayed as one CUDA graph.  HBM-bound: bytes per step = every layer's
    weight bytes + the K/V rows attended."""
    import ctypes as C
    import torch
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, LayerProj
    p = LAYER
    L, hq, hkv, hd, dim, S = p["n_layers"], p["n_heads"], p["n_kv_heads"], p["head_dim"], p["dim"], p["ctx"]
    qd, kvd = hq * hd, hkv * hd
    lib = abi.lib()
    cfg = abi.Config.make(L, hq, hkv, hd, S, p["rope_base"], abi.ROPE_NEOX)
    st = AttnState(cfg, n_seqs=1, max_ctx=S)
    g = torch.Generator(device=dev).manual_seed(p["seed"])
    # finite fp16 cache rows: magnitude < 1, either sign (bit patterns in int16 containers)
    for c in (st.k_cache, st.v_cache):
        mag = torch.randint(0, 0x3C00, c.shape, generator=g, device=dev, dtype=torch.int32)
        sgn = torch.randint(0, 2, c.shape, generator=g, device=dev, dtype=torch.int32) * 0x8000
        c.copy_(((mag | sgn) - ((mag | sgn) >= 0x8000).to(torch.int32) * 0x10000).to(torch.int16))
    shapes = ((dim, qd), (dim, kvd), (dim, kvd), (qd, dim))
    rng = np.random.default_rng(p["seed"])
    projs, wbytes = [], 0
    for _ in range(L):
        ws = []
        for t, (n_in, n_out) in zip(p["types"], shapes):
            nb = lib.picoattn_weight_bytes(t, n_in, n_out)
            blk = rng.integers(0, 256, nb, dtype=np.uint8)
            ws.append(torch.from_numpy(blk).to(dev))
            wbytes += nb
        # scales: small positive fp16 (the first two bytes of every block are a scale in Q4_K;
        # Q6_K keeps its scale last) so activations stay finite
        for w, t in zip(ws, p["types"]):
            bsz = 144 if t == 13 else 210
            v = w.view(-1, bsz)
            at = 0 if t == 13 else 208
            v[:, at:at + 2] = torch.tensor([0x00, 0x10], dtype=torch.uint8, device=dev)  # fp16 0x1000 ~ 2.4e-4
            if t == 13:
                v[:, 2:4] = torch.tensor([0x00, 0x08], dtype=torch.uint8, device=dev)
        bias = [torch.zeros(n, device=dev) for n in (qd, kvd, kvd, dim)]
        projs.append(LayerProj(*ws, p["types"], *bias))
    xb = torch.randn(1, dim, generator=g, device=dev)
    x = torch.zeros(1, dim, device=dev)
    pos = torch.tensor([S - 1], dtype=torch.int32, device=dev)
    kv_bytes = L * 2 * S * kvd * 2
    for l in range(L):
        st.decode_layer(l, dim, xb, projs[l], pos, x)
    torch.cuda.synchronize()
    if st.status() != 0:
        raise RuntimeError("decode_layer flagged bad input")
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for l in range(L):
                st.decode_layer(l, dim, xb, projs[l], pos, x, stream=s)
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize()
    steps = max(5, args.steps // 4)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # the projection kernel alone, for its roofline: the O projection of every
    # layer (Q4_K 3584 x 3584) as one graph of picoattn_matvec calls
    attn = torch.randn(1, qd, generator=g, device=dev)
    graph2 = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph2, stream=s):
            for l in range(L):
                lib.picoattn_matvec(projs[l].tensors[3].data_ptr(), p["types"][3], None, qd, dim, 1,
                                    attn.data_ptr(), x.data_ptr(), 1, s.cuda_stream)
    for _ in range(3):
        graph2.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        graph2.replay()
    e1.record()
    torch.cuda.synchronize()
    mv_us = e0.elapsed_time(e1) / steps / L * 1e3
    mv_bytes = lib.picoattn_weight_bytes(p["types"][3], qd, dim)
    peak, peak_kind = measured_peaks()
    total = wbytes + kv_bytes
    gbs = total / (ms / 1e3) / 1e9
    del graph, graph2, st
    return {"metric": "decode-layer attention block HBM GB/s", "value": round(gbs, 1), "unit": "GB/s",
            "ms_per_step": round(ms, 4), "us_per_layer": round(ms / L * 1e3, 2), "steps": steps,
            "config": {"workload": p["name"], "layers": L, "heads_q_kv_dim": [hq, hkv, hd], "dim": dim,
                       "cached_rows": S - 1, "weights": "q,k,o Q4_K; v Q6_K (seeded random blocks)",
                       "bytes_per_step": total, "weight_bytes": wbytes, "kv_bytes": kv_bytes},
            "frac_of_hbm": round(gbs / peak, 4),
            "roofline": {"bound": "hbm", "kernel": "matvec_mma_kernel<0> (Q4_K, 3584 x 3584, one vector)",
                         "achieved": round(mv_bytes / (mv_us / 1e6) / 1e9, 1), "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(mv_bytes / (mv_us / 1e6) / 1e9 / peak, 4),
                         "us_per_launch": round(mv_us, 2), "weight_bytes_per_launch": mv_bytes}}


STEP = dict(name="qwen2.5-7b-token-step-q4km", n_layers=28, n_heads=28, n_kv_heads=4, head_dim=128, dim=3584,
            n_ffn=18944, vocab=152064, rope_base=1e6, ctx=4096, seed=0,
            attn_types=(13, 13, 15, 13), ffn_types=(13, 13, 15), out_type=15)


def random_blocks_dev(wtype: int, n_in: int, n_out: int, g, dev):
    """n_out rows of n_in weights of a GGUF block type as random bytes on the
    device, every block's fp16 scales set small and positive (Q4_K: d, dmin at
    bytes 0-3; Q6_K: d at bytes 208-209) so activations stay finite."""
    import torch
    from picolm_qwen_b200 import abi
    nb = abi.lib().picoattn_weight_bytes(wtype, n_in, n_out)
    w = torch.randint(0, 256, (nb,), generator=g, device=dev, dtype=torch.uint8)
    bsz = 144 if wtype == 13 else 210
    v = w.view(-1, bsz)
    at = 0 if wtype == 13 else 208
    v[:, at:at + 2] = torch.tensor([0x00, 0x10], dtype=torch.uint8, device=dev)  # fp16 0x1000 ~ 2.4e-4
    if wtype == 13:
        v[:, 2:4] = torch.tensor([0x00, 0x08], dtype=torch.uint8, device=dev)
    return w, nb


def run_token_step(args, dev) -> dict:
    """A whole decode step of a Qwen2.5-7B-shaped model on the device, one
    sequence at position ctx - 1: per layer one picoattn_decode_block
    (attention norm, q/k/v projections, QK-norm-free attention over 4096 rows,
    output projection, FFN norm, gate/up, SwiGLU, down projection, residuals),
    then picoattn_logits over the 152064-row output matrix; Q4_K_M-style
    weights (attention q, k, o and FFN gate, up Q4_K; v, down and the output
    matrix Q6_K; seeded random blocks, each layer its own), 4.7 GB per token;
    the step replayed as one CUDA graph (the embedding row is the input)."""
    import torch
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import AttnState, FfnProj, LayerProj, Scratch, logits
    p = STEP
    L, hq, hkv, hd, dim, S = p["n_layers"], p["n_heads"], p["n_kv_heads"], p["head_dim"], p["dim"], p["ctx"]
    n_ffn, vocab = p["n_ffn"], p["vocab"]
    qd, kvd = hq * hd, hkv * hd
    cfg = abi.Config.make(L, hq, hkv, hd, S, p["rope_base"], abi.ROPE_NEOX)
    st = AttnState(cfg, n_seqs=1, max_ctx=S)
    g = torch.Generator(device=dev).manual_seed(p["seed"])
    for c in (st.k_cache, st.v_cache):
        c.copy_((torch.randn(c.shape, generator=g, device=dev) * 0.5).half().view(torch.int16))
    layers, wbytes = [], 0
    for _ in range(L):
        aw = []
        for t, (n_in, n_out) in zip(p["attn_types"], ((dim, qd), (dim, kvd), (dim, kvd), (qd, dim))):
            w, nb = random_blocks_dev(t, n_in, n_out, g, dev)
            aw.append(w)
            wbytes += nb
        fw = []
        for t, (n_in, n_out) in zip(p["ffn_types"], ((dim, n_ffn), (dim, n_ffn), (n_ffn, dim))):
            w, nb = random_blocks_dev(t, n_in, n_out, g, dev)
            fw.append(w)
            wbytes += nb
        an = 1 + 0.1 * torch.randn(dim, generator=g, device=dev)
        fn = 1 + 0.1 * torch.randn(dim, generator=g, device=dev)
        layers.append((an, LayerProj(*aw, p["attn_types"]), fn, FfnProj(*fw, p["ffn_types"])))
    w_out, nb = random_blocks_dev(p["out_type"], dim, vocab, g, dev)
    wbytes += nb
    out_norm = 1 + 0.1 * torch.randn(dim, generator=g, device=dev)
    x0 = torch.randn(1, dim, generator=g, device=dev)
    x = torch.empty_like(x0)
    lg = torch.empty((1, vocab), device=dev)
    pos = torch.tensor([S - 1], dtype=torch.int32, device=dev)
    scratch = Scratch(dev)
    s = torch.cuda.Stream(dev)

    def step(stream):
        x.copy_(x0)
        for l in range(L):
            an, proj, fn, fproj = layers[l]
            st.decode_block(l, dim, n_ffn, x, an, proj, fn, fproj, pos, stream=stream)
        logits(x, out_norm, w_out, p["out_type"], vocab, lg, scratch, stream=stream)

    with torch.cuda.stream(s):
        step(s)
        torch.cuda.synchronize(dev)
        if st.block_status() != 0:
            raise RuntimeError("token step flagged bad input")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step(s)
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize(dev)
    if not torch.isfinite(lg).all():
        raise RuntimeError("token step logits not finite")
    steps = max(5, args.steps // 4)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    del graph
    kv_bytes = L * 2 * S * kvd * 2
    total = wbytes + kv_bytes
    peak, peak_kind = measured_peaks()
    gbs = total / (ms / 1e3) / 1e9
    # the projections alone (picoattn_matvec, one vector; each graph streams
    # every layer's own matrix, or the output matrix, so every launch reads HBM)
    lib = abi.lib()
    xin = {n: torch.randn(1, n, generator=g, device=dev) for n in (dim, n_ffn)}
    yout = torch.empty(1, max(vocab, n_ffn), device=dev)
    projs = {"attn_o_q4k": [(layers[l][1].tensors[3], p["attn_types"][3], qd, dim) for l in range(L)],
             "ffn_gate_q4k": [(layers[l][3].tensors[0], p["ffn_types"][0], dim, n_ffn) for l in range(L)],
             "ffn_down_q6k": [(layers[l][3].tensors[2], p["ffn_types"][2], n_ffn, dim) for l in range(L)],
             "output_q6k": [(w_out, p["out_type"], dim, vocab)] * 4}
    kernels = {}
    for name, calls in projs.items():
        pg = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(pg, stream=s):
                for w, t, n_in, n_out in calls:
                    lib.picoattn_matvec(w.data_ptr(), t, None, n_in, n_out, 1, xin[n_in].data_ptr(),
                                        yout.data_ptr(), 0, s.cuda_stream)
        for _ in range(3):
            pg.replay()
        torch.cuda.synchronize(dev)
        e0.record()  # the graph replays on the current stream
        for _ in range(steps):
            pg.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) / steps / len(calls) * 1e3
        nb = lib.picoattn_weight_bytes(calls[0][1], calls[0][2], calls[0][3])
        kernels[name] = {"us_per_launch": round(us, 2), "weight_bytes": nb,
                         "gbs": round(nb / (us / 1e6) / 1e9, 1), "frac": round(nb / (us / 1e6) / 1e9 / peak, 4),
                         "launches_per_token": L if name != "output_q6k" else 1}
        del pg
    down = kernels["ffn_down_q6k"]
    # end to end through the C ABI: each token's embedding row goes up from
    # pinned host memory and its logits come back to pinned host memory inside
    # the timed graph (the weights, the cache and the RoPE table stay resident)
    x_host = x0.cpu().pin_memory()
    lg_host = torch.empty((1, vocab), dtype=torch.float32).pin_memory()

    def step_e2e(stream):
        x.copy_(x_host, non_blocking=True)
        for l in range(L):
            an, proj, fn, fproj = layers[l]
            st.decode_block(l, dim, n_ffn, x, an, proj, fn, fproj, pos, stream=stream)
        logits(x, out_norm, w_out, p["out_type"], vocab, lg, scratch, stream=stream)
        lg_host.copy_(lg, non_blocking=True)

    with torch.cuda.stream(s):
        step_e2e(s)
        torch.cuda.synchronize(dev)
        ge = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ge, stream=s):
            step_e2e(s)
    for _ in range(3):
        ge.replay()
    torch.cuda.synchronize(dev)
    e0.record()
    for _ in range(steps):
        ge.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    ms_e2e = e0.elapsed_time(e1) / steps
    if not np.array_equal(lg_host.numpy(), lg.cpu().numpy()):
        raise RuntimeError("token step e2e logits differ from the device's")
    del ge
    line = {"metric": "decode tokens/s (one sequence, whole model on the device)", "value": round(1e3 / ms, 2),
            "unit": "tok/s", "ms_per_token": round(ms, 4), "steps": steps,
            "config": {"workload": p["name"], "layers": L, "heads_q_kv_dim": [hq, hkv, hd], "dim": dim,
                       "n_ffn": n_ffn, "vocab": vocab, "cached_rows": S - 1,
                       "weights": "attention q,k,o + FFN gate,up Q4_K; v, down, output Q6_K (seeded random blocks)",
                       "bytes_per_token": total, "weight_bytes": wbytes, "kv_bytes": kv_bytes,
                       "l2": "4.7 GB per token, larger than L2, no flush",
                       "timing": "CUDA graph of 28 picoattn_decode_block calls + picoattn_logits"},
            "achieved_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / peak, 4), "peak": peak, "peak_kind": peak_kind,
            "e2e": {"value": round(1e3 / ms_e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": dim * 4,
                    "d2h_bytes_per_step": vocab * 4,
                    "timing": "CUDA graph: the embedding row up from pinned memory, 28 picoattn_decode_block + "
                              "picoattn_logits, the logits back to pinned memory"},
            "projections": kernels,
            "roofline": {"bound": "hbm", "kernel": "matvec_mma_kernel<1> (Q6_K FFN down, 18944 -> 3584, one vector)",
                         "achieved": down["gbs"], "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": down["frac"], "us_per_launch": down["us_per_launch"],
                         "weight_bytes_per_launch": down["weight_bytes"]}}
    del st, layers, w_out
    if not args.no_cpu:
        try:
            line["cpu_baseline"] = cpu_token_step()
        except Exception as e:  # the CPU leg never hides a GPU number
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    return line


def cpu_token_step() -> dict:
    """The reference's unmodified Model::forward on a one-layer model of the same
    shape (Q4_K weights, vocab 1024) on one thread (the engine's default): one
    layer's time x 28 layers, the 152064-row output matrix left out."""
    from oracle import pyoracle
    p = STEP
    ref = pyoracle.RefHarness()
    m = pyoracle.RefFullModel(ref, n_layers=1, hq=p["n_heads"], hkv=p["n_kv_heads"], hd=p["head_dim"],
                              n_ffn=p["n_ffn"], vocab=1024, max_seq=64, rope_base=p["rope_base"], rope_mode=0,
                              qk_norm=0, seed=1)
    m.set_attn_weights(13, 3)
    m.set_ffn_weights(13, 4)
    m.forward(5, 0)  # first touch of every weight page
    t0 = time.perf_counter()
    m.forward(9, 1)
    per_layer = time.perf_counter() - t0
    tok_s = 1.0 / (per_layer * p["n_layers"])
    m.close()
    return {"value": round(tok_s, 4), "unit": "tok/s", "cores": 1, "kind": "reference",
            "sample": f"Model::forward of a one-layer model of this shape (Q4_K weights, vocab 1024) on one thread: "
                      f"{per_layer * 1e3:.1f} ms per layer, x {p['n_layers']} layers; output matrix left out"}


def profile_matvec(wtype: int, n_in: int, n_out: int) -> None:
    """Three picoattn_matvec launches of one shape, each on its own copy of the
    matrix (the copies together larger than L2), then exit."""
    import torch
    from picolm_qwen_b200 import abi
    lib = abi.lib()
    g = torch.Generator(device="cuda").manual_seed(0)
    nb = lib.picoattn_weight_bytes(wtype, n_in, n_out)
    copies = max(3, -(-300_000_000 // max(nb, 1)))
    ws = [random_blocks_dev(wtype, n_in, n_out, g, "cuda")[0] for _ in range(copies)]
    x = torch.randn(1, n_in, generator=g, device="cuda")
    out = torch.empty(1, n_out, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for i in range(3):
        abi.check(lib.picoattn_matvec(ws[i].data_ptr(), wtype, None, n_in, n_out, 1, x.data_ptr(), out.data_ptr(),
                                      0, s), "picoattn_matvec")
    torch.cuda.synchronize()


def profile_longctx(rows: int) -> None:
    """The long-context leg's call (all stages, one sequence at position
    rows - 1) on layers 0, 1, 2 of a 3-layer cache of `rows` rows, then exit."""
    import torch
    from picolm_qwen_b200 import abi
    from picolm_qwen_b200.runtime import stream_handle
    p = LONGCTX
    hq, hkv, hd = p["n_heads"], p["n_kv_heads"], p["head_dim"]
    kvd, qd, L = hkv * hd, hq * hd, 3
    cfg = abi.Config.make(L, hq, hkv, hd, rows, p["rope_base"], abi.ROPE_NEOX)
    lib = abi.lib()
    cfgp = C.byref(cfg)
    g = torch.Generator(device="cuda").manual_seed(3000)
    kc = (torch.randn((L, rows, kvd), generator=g, device="cuda") * 0.5).half().view(torch.int16)
    vc = (torch.randn((L, rows, kvd), generator=g, device="cuda") * 0.5).half().view(torch.int16)
    q = torch.randn((L, qd), generator=g, device="cuda")
    k = torch.randn((L, kvd), generator=g, device="cuda")
    v = torch.randn((L, kvd), generator=g, device="cuda")
    out = torch.empty((L, qd), device="cuda")
    cos = np.empty(rows * hd // 2, np.float32)
    sin = np.empty_like(cos)
    assert lib.picoattn_rope_table(cfgp, cos.ctypes.data, sin.ctypes.data) == 0
    d_cos, d_sin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    kp = torch.tensor([kc.data_ptr()], dtype=torch.int64, device="cuda")
    vp = torch.tensor([vc.data_ptr()], dtype=torch.int64, device="cuda")
    pos = torch.tensor([rows - 1], dtype=torch.int32, device="cuda")
    ws_n = lib.picoattn_decode_workspace_size(cfgp, 1, rows)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")
    sh = stream_handle()
    assert lib.picoattn_workspace_init(ws.data_ptr(), ws_n, sh) == 0
    for l in range(L):
        abi.check(lib.picoattn_decode_staged(cfgp, l, 1, rows, q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(),
                                             None, None, d_cos.data_ptr(), d_sin.data_ptr(), kp.data_ptr(),
                                             vp.data_ptr(), pos.data_ptr(), out[l].data_ptr(), ws.data_ptr(), ws_n,
                                             sh, abi.STAGE_ALL), "picoattn_decode_staged")
    torch.cuda.synchronize()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill (Qwen3-8B) leg")
    ap.add_argument("--no-longctx", action="store_true", help="skip the long-context (Qwen2.5-32B, 128K) leg")
    ap.add_argument("--no-layer", action="store_true",
                    help="skip the decode-layer leg (projections + attention, Qwen2.5-7B, Q4_K_M weights)")
    ap.add_argument("--no-step", action="store_true",
                    help="skip the whole-model token step leg (Qwen2.5-7B shape, Q4_K_M-style weights)")
    ap.add_argument("--no-small", action="store_true",
                    help="skip the small single-sequence legs (TinyLlama p=511, Qwen2.5-0.5B 4096)")
    ap.add_argument("--profile-matvec", type=int, nargs=3, metavar=("TYPE", "N_IN", "N_OUT"),
                    help="only launch picoattn_matvec three times on seeded random blocks of that shape (over "
                         "weight copies larger than L2 together) and exit: the case the projection ncu captures use")
    ap.add_argument("--profile-longctx", type=int, metavar="ROWS",
                    help="only run the long-context call (Qwen2.5-32B heads, one sequence) on three layers of ROWS "
                         "cached rows each and exit: the case the long-context ncu capture uses")
    ap.add_argument("--seqs", type=int, default=WORKLOAD["n_seqs"],
                    help="sequences per GPU (default 64 = the benchmark; smaller only for profiling)")
    args = ap.parse_args()
    if args.profile_matvec:
        profile_matvec(*args.profile_matvec)
        return
    if args.profile_longctx:
        profile_longctx(args.profile_longctx)
        return
    WORKLOAD["n_seqs"] = args.seqs
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
