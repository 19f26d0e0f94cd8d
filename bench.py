"""Benchmark of the low-bit decode hot path on B200.

Default workload (the dequant-matmul sweep's M=1 point; the metric's "W4/W3
dequant-GEMV GB/s vs HBM peak"): y = W x with W packed int4 (and int3),
K=4096, N=12288, group 128 along K, fp16 scales, zero-point at mid-range
(unsigned-code reading), fp32 x ~N(0,1), fp32 y.  A *step* is one GEMV over
each of R distinct weight copies (R*26 MB > 4x L2), captured once as a CUDA
graph and replayed, so every timed launch streams its weights from HBM.

  value      W4 GEMV algorithmic GB/s, inputs resident in HBM, whole job
  e2e        same metric through the reference-facing host-pointer ABI
             (vspec_cuda_fused_linear_int4_cached_bridge: x uploaded and y
             downloaded on every call)
  roofline   dominant kernel (the W4 GEMV) vs measured HBM copy bandwidth
  cpu_baseline  the oracle restatement (group-wise), one host thread

`--impl reference` times the reference's own CPU implementation
(vspec_int4_matmul_ref_f32_q4_with_zero_points from oracle/_ref, compiled from
the reference sources) on the same shape with all host threads.

Multi-GPU: one process per GPU (torchrun); every rank runs the same
independent workload (data-parallel replicas, weak scaling); timing is the
max over ranks of CUDA-event time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vspec-engine_b200", "python"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

K_DIM, N_DIM, GROUP = 4096, 12288, 128
METRIC = "W4 dequant-GEMV GB/s (K=4096 N=12288 M=1 group128 fp16 scales)"


def gemv_bytes(bits: int, n: int = N_DIM, k: int = K_DIM, m: int = 1, sz_bytes: int = 2, zp: bool = False) -> int:
    groups = k // GROUP
    return n * ((k * bits + 7) // 8) + n * groups * sz_bytes * (2 if zp else 1) + m * k * 4 + m * n * 4


def load_peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_peak_table() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_traffic() -> float | None:
    """DRAM bytes per W4 GEMV launch from the committed ncu summary (one capture)."""
    try:
        with open(os.path.join(ROOT, "profiles", "gemv_w4_k4096_n12288_traffic.json")) as f:
            return float(json.load(f)["dram_bytes_per_launch"])
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index: int):
        self.gpu = str(gpu_index)
        try:
            import torch
            uuid = getattr(torch.cuda.get_device_properties(gpu_index), "uuid", None)
            if uuid is not None:
                self.gpu = "GPU-" + str(uuid)
        except Exception:
            pass
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(gpus: int):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world <= 1:
        return v
    import torch
    import torch.distributed as dist
    # NCCL reduces device tensors; a gloo group (the CPU tests of these helpers) host tensors
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ GPU arm
def make_rotation(torch, bits: int, copies: int, seed: int, n: int = N_DIM, k: int = K_DIM, sz16: bool = True,
                  zp_array: bool = False):
    """Distinct weight copies: uniform packed codes, group-128 scales ~U(0.005,
    0.02) (fp16, or fp32), and with zp_array an fp32 zero-point array of the
    mid-range value 2^(bits-1) (the signed reading of the literal config)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    rb = (k * bits + 7) // 8
    ws = [torch.randint(0, 256, (n, rb), dtype=torch.uint8, device="cuda", generator=g) for _ in range(copies)]
    ss = []
    for _ in range(copies):
        s = torch.rand((n, k // GROUP), device="cuda", generator=g) * 0.015 + 0.005
        ss.append(s.half() if sz16 else s)
    zs = [torch.full((n, k // GROUP), float(1 << (bits - 1)), device="cuda") for _ in range(copies)] if zp_array \
        else [None] * copies
    return ws, ss, zs


def copies_for(bytes_per_launch: int, floor: int = 8, cap: int = 96) -> int:
    """Rotating weight copies so that one pass streams > 4x the 126 MB L2."""
    need = (4 * 126 * 2 ** 20) // max(1, bytes_per_launch) + 1
    return int(min(cap, max(floor, need)))


def time_linear_graph(torch, V, *, m: int, n: int, k: int, bits: int, copies: int, steps: int, warmup: int,
                      world: int, sz16: bool = True, zp_array: bool = False, sampler=None, soak_s: float = 0.0,
                      seed: int = 0):
    """One step = one low-bit linear over each of `copies` distinct weight
    copies (> 4x L2 in total), captured once as a CUDA graph; device time of
    `steps` replays (max over ranks).  With a sampler, nvidia-smi clocks are
    recorded over a soak of the same graph right before the timed region and
    through it.  Returns (ms, clocks, algorithmic bytes per launch)."""
    ws, ss, zs = make_rotation(torch, bits, copies, seed=1234 + bits + 7 * m + n + seed, n=n, k=k, sz16=sz16,
                               zp_array=zp_array)
    x = torch.randn((m, k), device="cuda", dtype=torch.float32)
    ys = [torch.empty((m, n), device="cuda", dtype=torch.float32) for _ in range(copies)]
    stream = torch.cuda.Stream()
    # the literal reading (signed codes, zp array) or the mid-range unsigned one
    flags = (V.F_SZ_F16 if sz16 else 0) | (0 if zp_array else V.F_UNSIGNED)

    def step(st):
        for w, s, z, y in zip(ws, ss, zs, ys):
            V.lowbit_linear(x.data_ptr(), w.data_ptr(), s.data_ptr(), z.data_ptr() if z is not None else None,
                            y.data_ptr(), m, n, k, k // GROUP, bits, flags=flags, stream=st)

    with torch.cuda.stream(stream):
        step(stream.cuda_stream)          # configures kernel attributes before capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(stream.cuda_stream)
    torch.cuda.synchronize()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler:
        sampler.start()
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < soak_s:
            with torch.cuda.stream(stream):
                for _ in range(20):
                    graph.replay()
            torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    gemv_timeout_check(V)
    del graph
    szb = 2 if sz16 else 4
    nbytes = n * ((k * bits + 7) // 8) + n * (k // GROUP) * szb * (2 if zp_array else 1) + m * k * 4 + m * n * 4
    return ms, clocks, nbytes


def gemv_timeout_check(V) -> None:
    """Fail loudly when a bounded device wait of a GEMV gave up (its output is
    then incomplete) or a paged attention call met an out-of-range page id."""
    import ctypes
    f = ctypes.c_int(0)
    V.check(V.lib.vspec_b200_gemv_timeout_flag(ctypes.byref(f)), "gemv timeout flag")
    if f.value:
        raise RuntimeError("a GEMV bounded wait gave up during the bench (timeout flag set)")
    if V.page_fault_flag():
        raise RuntimeError("paged attention met an out-of-range page id during the bench")


def time_hybrid(torch, V, copies: int, steps: int, warmup: int, world: int):
    """ANF hybrid linear at the reference's lane-B benchmark shape
    (tools/benchmark/anf_phase_b_cuda_laneB.c: m=1, k=4096, n=8192, 96 hot
    columns (i*13 + step % 7) % n, one int4 scale block): int2 draft of every
    column + int4 refine of the hot ones.  Device time over rotating weight
    copies > L2 in one CUDA graph, and the host bridge end to end (host input,
    output and hot list, copies inside) with the temporal rule off."""
    m, k, n, hc = 1, 4096, 8192, 96
    g = torch.Generator(device="cuda")
    g.manual_seed(777)
    w2s = [torch.randint(0, 256, (n, k // 4), dtype=torch.uint8, device="cuda", generator=g) for _ in range(copies)]
    w4s = [torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device="cuda", generator=g) for _ in range(copies)]
    s2 = torch.rand((n,), device="cuda", generator=g) * 0.04 + 0.01
    s4 = torch.rand((n,), device="cuda", generator=g) * 0.015 + 0.005
    zp4 = torch.zeros((n,), device="cuda")
    x = torch.randn((m, k), device="cuda", dtype=torch.float32)
    hot = torch.tensor([(i * 13) % n for i in range(hc)], dtype=torch.int32, device="cuda")
    ys = [torch.empty((m, n), device="cuda", dtype=torch.float32) for _ in range(copies)]
    stream = torch.cuda.Stream()

    def step(st):
        for w2, w4, y in zip(w2s, w4s, ys):
            V.anf_hybrid_linear(x.data_ptr(), w2.data_ptr(), s2.data_ptr(), w4.data_ptr(), s4.data_ptr(),
                                zp4.data_ptr(), y.data_ptr(), hot.data_ptr(), hc, m, n, k, 1, stream=st)

    with torch.cuda.stream(stream):
        step(stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(stream.cuda_stream)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    del graph
    bytes_call = n * (k // 4) + n * 4 + hc * (k // 2 + 8) + m * k * 4 + m * n * 4
    # bridge, host buffers (the lane-B benchmark's full path)
    hx = x.cpu().numpy()
    hw2, hs2 = w2s[0].cpu().numpy(), s2.cpu().numpy()
    hw4, hs4, hzp = w4s[0].cpu().numpy(), s4.cpu().numpy(), zp4.cpu().numpy()
    out = np.empty((m, n), dtype=np.float32)
    lists = [np.array([(i * 13 + st % 7) % n for i in range(hc)], dtype=np.uint32) for st in range(7)]
    os.environ.pop("VSPEC_ENABLE_ANF", None)

    def call(i):
        h = lists[i % 7]
        ok = V.lib.vspec_cuda_fused_linear_hybrid_bridge(hx.ctypes.data, hw2.ctypes.data, hs2.ctypes.data,
                                                         hw4.ctypes.data, hs4.ctypes.data, hzp.ctypes.data, m, k, n,
                                                         h.ctypes.data, hc, 1, out.ctypes.data)
        if ok != 1:
            raise RuntimeError("vspec_cuda_fused_linear_hybrid_bridge failed")

    for i in range(5):
        call(i)
    calls = 50
    t0 = time.perf_counter()
    for i in range(calls):
        call(i)
    bridge_ms = (time.perf_counter() - t0) * 1e3 / calls
    return ms, bytes_call, bridge_ms, hc * 4 + m * k * 4, m * n * 4


def time_q4k(torch, V, copies: int, steps: int, warmup: int, world: int):
    """Q4_K (GGUF-style 256-element super-blocks, q4_k.c) GEMV at the bench shape
    K=4096 N=12288 M=1: 144 bytes per 256 weights, rotating copies > L2."""
    nb = K_DIM // 256
    g = torch.Generator(device="cuda")
    g.manual_seed(4242)
    ws = [torch.randint(0, 256, (N_DIM, nb, 144), dtype=torch.uint8, device="cuda", generator=g) for _ in range(copies)]
    for w in ws:   # finite fp16 d / dmin
        w[:, :, 1] = 0x20
        w[:, :, 3] = 0x20
    x = torch.randn((1, K_DIM), device="cuda", dtype=torch.float32)
    ys = [torch.empty((1, N_DIM), device="cuda", dtype=torch.float32) for _ in range(copies)]
    stream = torch.cuda.Stream()

    def step(st):
        for w, y in zip(ws, ys):
            V.q4k_linear(x.data_ptr(), w.data_ptr(), y.data_ptr(), 1, N_DIM, K_DIM, stream=st)

    with torch.cuda.stream(stream):
        step(stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(stream.cuda_stream)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    del graph
    bytes_per_call = N_DIM * nb * 144 + K_DIM * 4 + N_DIM * 4
    return ms, bytes_per_call


def time_e2e_bridge(torch, V, copies: int, steps: int, warmup: int, world: int):
    """Reference host-pointer ABI: registered int4 weights (fp32 s + zp, the
    bridge's formats), host x -> host y on every call."""
    import ctypes
    rng = np.random.default_rng(77)
    n, k, g = N_DIM, K_DIM, K_DIM // GROUP
    handles, keep = [], []
    for i in range(copies):
        w = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
        s = rng.uniform(0.005, 0.02, size=(n, g)).astype(np.float32)
        zp = np.full((n, g), 8.0, dtype=np.float32)
        h = V.lib.vspec_cuda_fused_linear_int4_register_weight_bridge(w.ctypes.data, s.ctypes.data, zp.ctypes.data,
                                                                       k, n, g)
        if h <= 0:
            raise RuntimeError("register_weight_bridge failed: " + V.last_error())
        handles.append(h)
        keep.append((w, s, zp))
    x = rng.standard_normal((1, k)).astype(np.float32)
    y = np.zeros((1, n), dtype=np.float32)
    fn = V.lib.vspec_cuda_fused_linear_int4_cached_bridge

    def step():
        for h in handles:
            if fn(x.ctypes.data, 1, k, h, n, y.ctypes.data) != 1:
                raise RuntimeError("cached_bridge failed: " + V.last_error())

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) * 1e3
    barrier(world)
    ms = max_over_ranks(dt, world)
    bytes_per_call = n * k // 2 + 2 * n * g * 4 + k * 4 + n * 4
    del keep
    return ms, bytes_per_call, k * 4, n * 4


ATTN_B, ATTN_HQ, ATTN_HKV, ATTN_D, ATTN_PT = 32, 32, 8, 128, 16


def make_config3(torch, seed: int = 3):
    """Paged attention workload: B=32, Hq=32, Hkv=8, d=128, ctx ~U[512,8192], 16-token
    pages of fp16 K/V ~N(0,1), page table = seeded permutation of the shared pool."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(512, 8193, size=ATTN_B).astype(np.int32)
    need = (ctx + ATTN_PT - 1) // ATTN_PT
    total = int(need.sum())
    perm = rng.permutation(total).astype(np.int32)
    table = np.zeros((ATTN_B, int(need.max())), dtype=np.int32)
    off = 0
    for b, nb in enumerate(need):
        table[b, :nb] = perm[off:off + nb]
        off += nb
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    shape = (total, ATTN_PT, ATTN_HKV, ATTN_D)
    kp = torch.randn(shape, device="cuda", dtype=torch.float16, generator=g)
    vp = torch.randn(shape, device="cuda", dtype=torch.float16, generator=g)
    q = torch.randn((ATTN_B, ATTN_HQ, ATTN_D), device="cuda", dtype=torch.float32, generator=g)
    return ctx, table, total, kp, vp, q


def time_attention(torch, V, steps: int, warmup: int, world: int):
    """Paged GQA decode attention over config 3 (K+V ~570 MB per step, >> L2)."""
    ctx, table, total, kp, vp, q = make_config3(torch)
    dt = torch.from_numpy(table).cuda()
    dc = torch.from_numpy(ctx).cuda()
    out = torch.empty((ATTN_B, ATTN_HQ, ATTN_D), device="cuda", dtype=torch.float32)
    stream = torch.cuda.Stream()
    scale = 1.0 / float(np.sqrt(ATTN_D))

    def call(st):
        V.paged_attention(q.data_ptr(), kp.data_ptr(), vp.data_ptr(), dt.data_ptr(), dc.data_ptr(), out.data_ptr(),
                          ATTN_B, ATTN_HQ, ATTN_HKV, ATTN_D, ATTN_PT, table.shape[1], total, int(ctx.max()), scale,
                          V.KV_F16, stream=st)

    with torch.cuda.stream(stream):
        call(stream.cuda_stream)          # library scratch set up before capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        call(stream.cuda_stream)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    del graph
    # end to end through the public call: each step uploads q from pinned host memory, runs the
    # attention over the device-resident pages and reads the output back into pinned host memory
    q_host = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    q_host.copy_(q)
    out_host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            q.copy_(q_host, non_blocking=True)
            call(stream.cuda_stream)
            out_host.copy_(out, non_blocking=True)
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    kv_bytes = int(ctx.astype(np.int64).sum()) * ATTN_HKV * ATTN_D * 2 * 2
    other = q.numel() * 4 + out.numel() * 4 + table.size * 4 + ctx.size * 4
    return ms, kv_bytes, other, e2e_ms, q.numel() * 4, out.numel() * 4


AREF_T, AREF_H, AREF_D, AREF_COPIES = 4096, 8, 128, 6
AREF_ENV = ("VSPEC_FUSED_BITS", "VSPEC_3BIT_RUNTIME_MODULE", "VSPEC_3BIT_BLOCK_SIZE")


def time_attention_ref(torch, V, steps: int, warmup: int, world: int) -> dict:
    """The CPU backend's attention semantics (attention_ref.c: std clamp, double
    softmax denominator and output; module=1 adds the 3-bit module's arithmetic)
    at the shape the reference's CPU path is timed on, 8 heads x 4096 tokens x
    128, over six rotating K/V copies (201 MB > L2)."""
    t, h, d = AREF_T, AREF_H, AREF_D
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    kv = [(torch.randn((t, h, d), device="cuda", generator=g), torch.randn((t, h, d), device="cuda", generator=g))
          for _ in range(AREF_COPIES)]
    q = torch.randn((h, d), device="cuda", generator=g)
    out = torch.empty((h, d), device="cuda", dtype=torch.float32)
    ws = V.lib.vspec_b200_attention_ref_workspace_bytes(t, h, d)
    wbuf = torch.empty((ws,), device="cuda", dtype=torch.uint8)
    stream = torch.cuda.Stream()
    nbytes = 2 * t * h * d * 4 + 2 * h * d * 4
    res = {}
    for module in (0, 1):
        def run():
            for kk, vv in kv:
                V.attention_ref(q.data_ptr(), kk.data_ptr(), vv.data_ptr(), out.data_ptr(), t, h, d, module, 64,
                                wbuf.data_ptr(), ws, stream.cuda_stream)
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                run()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(steps):
                run()
            end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        us = max_over_ranks(start.elapsed_time(end), world) * 1e3 / (steps * AREF_COPIES)
        res[module] = us
    return {"us": round(res[0], 2), "gbs": round(world * nbytes / res[0] / 1e3, 1), "module_us": round(res[1], 2),
            "bytes": nbytes}


def cpu_attention_ref_sample(seconds: float = 4.0) -> dict | None:
    """The reference's own CPU backend attention (vspec_attention_ref_single_query
    compiled from its sources, one host thread, 3-bit module off) at the GPU leg's
    shape; GB/s of the same algorithmic K+V bytes."""
    import oracle as O
    if O.REF is None:
        return None
    saved = {k: os.environ.pop(k) for k in AREF_ENV if k in os.environ}
    try:
        rng = np.random.default_rng(11)
        t, h, d = AREF_T, AREF_H, AREF_D
        q = rng.standard_normal((h, d)).astype(np.float32)
        k = rng.standard_normal((t, h, d)).astype(np.float32)
        v = rng.standard_normal((t, h, d)).astype(np.float32)
        out = np.zeros((h, d), dtype=np.float32)
        t0 = time.perf_counter()
        calls = 0
        while True:
            O.REF.ref_cpu_backend_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, t, h, d, out.ctypes.data)
            calls += 1
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
    finally:
        os.environ.update(saved)
    nbytes = 2 * t * h * d * 4 + 2 * h * d * 4
    return {"value": round(calls * nbytes / dt / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "reference",
            "ms": round(dt * 1e3 / calls, 2),
            "sample": f"{calls} x vspec_attention_ref_single_query (CPU backend) {h}x{t}x{d}, module off, {dt:.1f} s"}


def time_attention_int3(torch, V, steps: int, warmup: int, world: int, block: int = 32):
    """Config 3 with int3 K/V pages (kv_cache.c int3 compression, block 32):
    the same seeded fp16 pools quantised on the GPU, then paged GQA attention
    reading the 3-bit codes and per-block scales (128 B per token and KV head
    for K+V instead of 512 B of fp16)."""
    ctx, table, total, kp, vp, q = make_config3(torch)
    rows = total * ATTN_PT
    pb, nb = ATTN_D * 3 // 8, ATTN_D // block
    pools = []
    for src in (kp, vp):
        codes = torch.empty((rows, ATTN_HKV, pb), dtype=torch.uint8, device="cuda")
        scales = torch.empty((rows, ATTN_HKV, nb), dtype=torch.float32, device="cuda")
        f32 = src.float()
        V.kv_int3_quantize(f32.data_ptr(), None, rows, ATTN_HKV, ATTN_D, block, codes.data_ptr(), scales.data_ptr())
        torch.cuda.synchronize()
        del f32
        pools.append((codes, scales))
    del kp, vp
    (kc, ks), (vc, vs) = pools
    dt = torch.from_numpy(table).cuda()
    dc = torch.from_numpy(ctx).cuda()
    out = torch.empty((ATTN_B, ATTN_HQ, ATTN_D), device="cuda", dtype=torch.float32)
    stream = torch.cuda.Stream()
    scale = 1.0 / float(np.sqrt(ATTN_D))

    def call(st):
        V.paged_attention_int3(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ks.data_ptr(), vs.data_ptr(), block,
                               dt.data_ptr(), dc.data_ptr(), out.data_ptr(), ATTN_B, ATTN_HQ, ATTN_HKV, ATTN_D,
                               ATTN_PT, table.shape[1], total, int(ctx.max()), scale, stream=st)

    with torch.cuda.stream(stream):
        call(stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        call(stream.cuda_stream)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    del graph
    kv_bytes = int(ctx.astype(np.int64).sum()) * ATTN_HKV * (pb + nb * 4) * 2
    other = q.numel() * 4 + out.numel() * 4 + table.size * 4 + ctx.size * 4
    return ms, kv_bytes, other


DEC_PROMPT, DEC_GEN, DEC_BATCH = 512, 256, 64


def decode_bytes_per_step(cfg: dict, batch: int, ctx: int) -> int:
    """HBM bytes one decode step must read: every packed weight and fp16 scale
    once, plus each sequence's fp16 K/V at context ctx."""
    H, I, L, V = cfg["hidden"], cfg["intermediate"], cfg["num_layers"], cfg["vocab"]
    qd = cfg["num_heads"] * cfg["head_dim"]
    kvd = cfg["num_kv_heads"] * cfg["head_dim"]
    mats = [(qd + 2 * kvd, H), (H, qd), (2 * I, H), (H, I)]
    per_layer = sum(n * (k * cfg["bits"] // 8) + n * (k // cfg["group"]) * 2 for n, k in mats)
    lm = V * (H * cfg["bits"] // 8) + V * (H // cfg["group"]) * 2
    kv = batch * ctx * L * kvd * 2 * 2
    return L * per_layer + lm + kv


def time_decode(torch, V, world: int, rank: int, peak: float):
    """Qwen3-8B-shape decode: W4 group 128, random-init, prompts of
    512 random ids, 256 greedy tokens; batch 1 (every rank its own sequence) and
    batch 64 sharded over the ranks.  tok/s over the generation phase (device
    time, max over ranks)."""
    cfg = V.QWEN3_8B
    shard = DEC_BATCH // world
    rng = np.random.default_rng(4 + rank)
    prompts = rng.integers(0, cfg["vocab"], size=(shard, DEC_PROMPT)).astype(np.int32)
    model = V.QwenModel(cfg, seed=1234, max_batch=shard, max_ctx=DEC_PROMPT + DEC_GEN)
    try:
        barrier(world)
        _, ms1, _ = model.generate(prompts[:1], DEC_GEN)
        ms1 = max_over_ranks(ms1, world)
        barrier(world)
        _, ms64, _ = model.generate(prompts, DEC_GEN)
        ms64 = max_over_ranks(ms64, world)
    finally:
        model.close()
    ctx_mid = DEC_PROMPT + DEC_GEN // 2
    b1_bytes = decode_bytes_per_step(cfg, 1, ctx_mid)
    b64_bytes = decode_bytes_per_step(cfg, shard, ctx_mid)
    step1_s = ms1 * 1e-3 / DEC_GEN
    step64_s = ms64 * 1e-3 / DEC_GEN
    r1 = b1_bytes / step1_s / 1e9
    r64 = b64_bytes / step64_s / 1e9
    return {"b1": {"tok_s": round(world * DEC_GEN / (ms1 * 1e-3), 1), "ms": round(ms1 / DEC_GEN, 4),
                   "frac": round(r1 / peak, 3)},
            "b64": {"tok_s": round(DEC_BATCH * DEC_GEN / (ms64 * 1e-3), 1), "ms": round(ms64 / DEC_GEN, 4),
                    "frac": round(r64 / peak, 3), "per_gpu": shard}}


def time_gemm(torch, V, world: int, steps: int, peaks: dict):
    """The M=64 and M=512 points of the dequant-matmul sweep (W4, K=4096,
    N=12288, group 128, fp16 scales, mid-range zero-point): activation
    pre-pass + tcgen05 GEMM (+ split-K merge) per linear through
    vspec_b200_lowbit_linear, back to back in a CUDA graph over rotating weight
    copies (> L2).  TFLOP/s against the measured bf16 burst peak."""
    out = {}
    for m in (64, 512):
        copies = 24
        ms, _, nbytes = time_linear_graph(torch, V, m=m, n=N_DIM, k=K_DIM, bits=4, copies=copies, steps=steps,
                                          warmup=3, world=world, seed=77)
        us = ms * 1e3 / (steps * copies)
        tflops = 2.0 * m * N_DIM * K_DIM / (us * 1e-6) / 1e12
        out[f"m{m}"] = {"us": round(us, 2), "tflops": round(tflops, 1), "frac": round(tflops / peaks["bf16_tflops"], 3),
                        "w_gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
    return out


def time_quantize(torch, V, world: int, with_cpu: bool):
    """Load-time quantise + pack: a 12288 x 4096 fp32
    weight (N(0, 0.02), seeded) to W4 block 128 at the 0.999 percentile, as
    the reference's _quantize_weight_rowwise with VSPEC_INT4_BLOCK_SIZE=128;
    GB/s of fp32 input. CPU baseline: the C restatement on a 256-row sample."""
    import ctypes
    n, k, bits, block = N_DIM, K_DIM, 4, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    w = torch.randn((n, k), device="cuda", generator=g) * 0.02
    packed = torch.empty((n, k * bits // 8), dtype=torch.uint8, device="cuda")
    s = torch.empty(n * (k // block), device="cuda")
    zp = torch.empty(n * (k // block), device="cuda")
    stream = torch.cuda.Stream()

    def call():
        rc = V.lib.vspec_b200_quantize_rowwise(w.data_ptr(), n, k, bits, block, ctypes.c_double(0.999),
                                               packed.data_ptr(), s.data_ptr(), zp.data_ptr(),
                                               ctypes.c_void_p(stream.cuda_stream))
        if rc != 0:
            raise RuntimeError("quantize_rowwise failed: " + V.last_error())

    for _ in range(2):
        call()
    torch.cuda.synchronize()
    barrier(world)
    reps = 5
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(reps):
            call()
        end.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world) / reps
    out = {"metric": "load-time W4 block-128 quantise + pack GB/s (fp32 input)", "value": round(n * k * 4 / (ms * 1e-3) / 1e9, 2),
           "unit": "GB/s", "ms_per_matrix": round(ms, 3),
           "config": f"{n} x {k} fp32 N(0, 0.02) -> int4 blocks of {block}, percentile 0.999 (bit-exact to the reference quantizer)"}
    if with_cpu:
        import oracle as O
        rows = 256
        wc = w[:rows].cpu().numpy()
        t0 = time.perf_counter()
        O.quantize_rowwise(wc, bits, block, 0.999)
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": round(rows * k * 4 / dt / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                               "sample": f"oracle_quantize_rowwise on {rows} of {n} rows, {dt:.2f} s"}
    return out


TP_PROMPT, TP_GEN, TP_BATCH = 1024, 128, 256


def tp_step_work(cfg: dict, batch: int, ctx: int, tp: int) -> dict:
    """Per-GPU algorithmic work of one config-5 decode step at tensor-parallel
    degree tp: tensor-core FLOPs of the linears (sharded) and the replicated
    lm_head, HBM bytes of this rank's packed weights, scales and K/V, and the
    bytes each all-reduce sums (2 per layer, [batch, hidden] fp32)."""
    H, I, L, V = cfg["hidden"], cfg["intermediate"], cfg["num_layers"], cfg["vocab"]
    qd = cfg["num_heads"] * cfg["head_dim"]
    kvd = cfg["num_kv_heads"] * cfg["head_dim"]
    ba, bm, g = cfg["bits"], cfg["bits_mlp"] or cfg["bits"], cfg["group"]
    attn = [(qd + 2 * kvd, H), (H, qd)]
    mlp = [(2 * I, H), (H, I)]
    p_attn = sum(n * k for n, k in attn)
    p_mlp = sum(n * k for n, k in mlp)
    p_lm = V * H
    flops = 2 * batch * (L * (p_attn + p_mlp) / tp + p_lm)
    wbytes = (L * (p_attn * ba / 8 + p_mlp * bm / 8 + (p_attn + p_mlp) / g * 2) / tp + p_lm * ba / 8 + p_lm / g * 2)
    kv = batch * ctx * L * (kvd // tp) * 2 * 2
    return {"flops": flops, "hbm_bytes": wbytes + kv, "allreduce_bytes": 2 * L * batch * H * 4 if tp > 1 else 0}


def time_decode_tp(torch, V, world: int, rank: int, peaks: dict):
    """Qwen3-32B-shape decode: attention projections and lm_head
    W4, MLP W3, group 128, random-init; batch 256 sequences of 1024 seeded
    random prompt ids (prefilled by decode steps) + 128 greedy tokens,
    tensor-parallel over all ranks (NCCL all-reduce after o-proj and down).
    tok/s over the generation phase (device time, max over ranks)."""
    import torch.distributed as dist
    cfg = V.QWEN3_32B
    nid = [V.nccl_unique_id() if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(nid, src=0)
    rng = np.random.default_rng(5)
    prompts = rng.integers(0, cfg["vocab"], size=(TP_BATCH, TP_PROMPT)).astype(np.int32)
    model = V.QwenModel(cfg, seed=4321, max_batch=TP_BATCH, max_ctx=TP_PROMPT + TP_GEN, tp_size=world, tp_rank=rank,
                        nccl_id=nid[0] if world > 1 else None)
    try:
        barrier(world)
        toks, ms, _ = model.generate(prompts, TP_GEN)
        ms = max_over_ranks(ms, world)
    finally:
        model.close()
    step_s = ms * 1e-3 / TP_GEN
    work = tp_step_work(cfg, TP_BATCH, TP_PROMPT + TP_GEN // 2, world)
    tflops = work["flops"] / step_s / 1e12
    gbs = work["hbm_bytes"] / step_s / 1e9
    return {"tok_s": round(TP_BATCH * TP_GEN / (ms * 1e-3), 1), "ms": round(ms / TP_GEN, 3),
            "tflops": round(tflops, 1), "frac": round(tflops / peaks["bf16_tflops_sustained"], 3),
            "hbm_gbs": round(gbs, 1), "tok_sum": int(np.asarray(toks, dtype=np.int64).sum() % 1000003)}


# 8 KV heads and 128-code groups in every row-parallel slice up to 8 ranks;
# attention W4, MLP W3 like the Qwen3-32B-shape config
TP_PARITY_CFG = dict(num_layers=2, hidden=512, num_heads=16, num_kv_heads=8, head_dim=64, intermediate=1024,
                     vocab=1000, bits=4, group=128, rms_eps=1e-6, rope_theta=1e6, logit_clip=24.0, page_tokens=16,
                     bits_mlp=3)


def tp_parity(torch, V, world: int, rank: int) -> dict:
    """Tensor-parallel parity on the driver's multi-GPU runs: every rank holds
    its shard of a small model (all ranks, NCCL all-reduce) and the same model
    unsharded; the sharded logits teacher-forced on the unsharded tokens are
    compared (max normwise error over steps, sequences and ranks) and the
    free-running greedy tokens must be equal."""
    import torch.distributed as dist
    cfg = TP_PARITY_CFG
    batch, plen, gen = 4, 6, 10
    rng = np.random.default_rng(31)
    prompts = rng.integers(0, cfg["vocab"], size=(batch, plen)).astype(np.int32)
    ref = V.QwenModel(cfg, seed=17, max_batch=batch, max_ctx=64)
    try:
        toks_ref, _, _ = ref.generate(prompts, gen)
        _, _, lg_ref = ref.generate(toks_ref, 1, want_logits=True)
    finally:
        ref.close()
    nid = [V.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(nid, src=0)
    shard = V.QwenModel(cfg, seed=17, max_batch=batch, max_ctx=64, tp_size=world, tp_rank=rank, nccl_id=nid[0])
    try:
        barrier(world)
        _, _, lg_tp = shard.generate(toks_ref, 1, want_logits=True)
        toks_tp, _, _ = shard.generate(prompts, gen)
    finally:
        shard.close()
    err = 0.0
    for st in range(lg_ref.shape[0]):
        for b in range(batch):
            r = lg_ref[st, b].astype(np.float64)
            err = max(err, float(np.max(np.abs(lg_tp[st, b] - r)) / max(np.max(np.abs(r)), 1e-30)))
    err = max_over_ranks(err, world)
    equal = max_over_ranks(0.0 if np.array_equal(toks_tp, toks_ref) else 1.0, world) == 0.0
    return {"max_rel_err": float(f"{err:.3g}"), "tokens_equal": bool(equal), "tp": world}


# ------------------------------------------------------------------ CPU legs
def cpu_oracle_sample(seconds: float = 10.0) -> dict:
    """The oracle restatement (group-wise int4, one thread) on a bounded sample
    of the workload: the first R rows of the N=12288 x K=4096 matrix."""
    import oracle as O
    rng = np.random.default_rng(5)
    rows = 256
    w = rng.integers(0, 256, size=(rows, K_DIM // 2), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, size=(rows, K_DIM // GROUP)).astype(np.float16)
    x = rng.standard_normal((1, K_DIM)).astype(np.float32)
    t0 = time.perf_counter()
    calls = 0
    while True:
        O.lowbit_matmul(x, w ^ np.uint8(0x88), rows, K_DIM, 4, s, None, K_DIM // GROUP)
        calls += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    frac = rows / N_DIM
    gbs = calls * gemv_bytes(4) * frac / dt / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{calls} x oracle_lowbit_matmul_f16sz, {rows} of {N_DIM} rows, {dt:.1f} s, bytes scaled"}


def _oracle_decode_tensors(cfg: dict, layers: int, rng) -> dict:
    """Random packed weights of the given layer shapes for the C decode
    restatement (values do not change its cost); a 16-row embedding slice is
    enough for the token ids the timing uses."""
    H, I, Vv = cfg["hidden"], cfg["intermediate"], cfg["vocab"]
    qd, kvd = cfg["num_heads"] * cfg["head_dim"], cfg["num_kv_heads"] * cfg["head_dim"]
    ba, bm = cfg["bits"], cfg["bits_mlp"] or cfg["bits"]

    def w(n, k, b):
        return rng.integers(0, 256, size=(n, (k * b + 7) // 8), dtype=np.uint8)

    def s(n, k):
        return np.full((n, k // cfg["group"]), 0x1c00, dtype=np.uint16)   # fp16 0.0039
    t = {"emb": rng.integers(0x2000, 0x2400, size=(16, H), dtype=np.uint16), "w_lm": w(Vv, H, ba), "s_lm": s(Vv, H)}
    for l in range(layers):
        for i, (n, k, b) in enumerate([(qd + 2 * kvd, H, ba), (H, qd, ba), (2 * I, H, bm), (H, I, bm)]):
            t[f"w{l}_{i}"], t[f"s{l}_{i}"] = w(n, k, b), s(n, k)
    return t


def cpu_decode_sample(cfg: dict, layers: int = 2) -> dict:
    """The C restatement of the decode step (oracle_qwen_generate, one host
    thread, batch 1) timed at the real layer shapes: one step with no layers
    (embedding, final norm, lm_head, argmax) and one with `layers` layers; the
    step at full depth is extrapolated per layer."""
    import oracle as O
    rng = np.random.default_rng(9)
    times = {}
    for L in (0, layers):
        c = dict(cfg, num_layers=L)
        t = _oracle_decode_tensors(c, L, rng)
        best = None
        for _ in range(2):
            t0 = time.perf_counter()
            O.qwen_generate(c, t, np.array([3], dtype=np.int32), 1)
            dt = time.perf_counter() - t0
            best = dt if best is None else min(best, dt)
        times[L] = best
        del t
    per_layer = max(0.0, (times[layers] - times[0]) / layers)
    step_s = times[0] + cfg["num_layers"] * per_layer
    return {"value": round(1.0 / step_s, 4), "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": f"oracle_qwen_generate batch 1, 1 step at 0 and {layers} layers ({times[0]:.2f} / "
                      f"{times[layers]:.2f} s), extrapolated to {cfg['num_layers']} layers"}


def cpu_attention_sample(seconds: float = 6.0) -> dict:
    """The GQA restatement (oracle_paged_gqa_attention_f32, flash-stub math per
    query head, one host thread) on config-3 sequences of the seeded context
    distribution; GB/s of the same algorithmic K+V bytes as the GPU leg."""
    import oracle as O
    rng = np.random.default_rng(3)
    ctx = rng.integers(512, 8193, size=ATTN_B).astype(np.int32)[:2]
    need = (ctx + ATTN_PT - 1) // ATTN_PT
    total = int(need.sum())
    table = np.zeros((len(ctx), int(need.max())), dtype=np.int32)
    perm = rng.permutation(total).astype(np.int32)
    off = 0
    for b, nb in enumerate(need):
        table[b, :nb] = perm[off:off + nb]
        off += nb
    kp = rng.standard_normal((total, ATTN_PT, ATTN_HKV, ATTN_D)).astype(np.float32)
    vp = rng.standard_normal((total, ATTN_PT, ATTN_HKV, ATTN_D)).astype(np.float32)
    q = rng.standard_normal((len(ctx), ATTN_HQ, ATTN_D)).astype(np.float32)
    t0 = time.perf_counter()
    calls = 0
    while True:
        O.paged_attention(q, kp, vp, table, ctx, ATTN_HQ, ATTN_HKV, ATTN_D, ATTN_PT, 1.0 / np.sqrt(ATTN_D))
        calls += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    kv = int(ctx.astype(np.int64).sum()) * ATTN_HKV * ATTN_D * 2 * 2
    return {"value": round(calls * kv / dt / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{calls} x oracle_paged_gqa_attention_f32 over 2 of 32 sequences (ctx {ctx[0]}, {ctx[1]}), "
                      f"{dt:.1f} s"}


def reference_arm(args) -> None:
    """Times the reference's own CPU implementation with all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import concurrent.futures as cf
    import oracle as O
    if O.REF is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libvspec_ref.so was not built"}))
        return
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(6)
    n, k = N_DIM, K_DIM
    # bounded sample per step: a slice of rows sized so one step is ~0.25 s of CPU work
    rows = min(n, max(threads, 32 * threads))
    w = rng.integers(0, 256, size=(rows, k // 2), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, size=rows).astype(np.float32)
    zp = np.full(rows, 8.0, dtype=np.float32)
    x = rng.standard_normal((1, k)).astype(np.float32)
    y = np.zeros((1, rows), dtype=np.float32)
    fn = O.REF.vspec_int4_matmul_ref_f32_q4_with_zero_points
    bounds = np.linspace(0, rows, threads + 1).astype(int)

    def part(i):
        a, b = bounds[i], bounds[i + 1]
        if b > a:
            yy = np.zeros((1, b - a), dtype=np.float32)
            fn(x.ctypes.data, 1, k, w[a:b].ctypes.data, b - a, s[a:].ctypes.data, zp[a:].ctypes.data, yy.ctypes.data)
            y[0, a:b] = yy[0]

    with cf.ThreadPoolExecutor(threads) as ex:
        for _ in range(args.warmup):
            list(ex.map(part, range(threads)))
        t0 = time.perf_counter()
        for _ in range(args.steps):
            list(ex.map(part, range(threads)))
        dt = time.perf_counter() - t0
    frac = rows / n
    gbs = args.steps * gemv_bytes(4) * frac / dt / 1e9
    ms_step = dt * 1e3 / args.steps / frac
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8 codes, fp32 math", "data": "synthetic",
        "config": {"workload": "config 2: W4 GEMV K=4096 N=12288 M=1 (reference per-row-scale CPU function)",
                   "parallelism": f"{threads} host threads, disjoint output rows"},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "reference",
                         "sample": f"vspec_int4_matmul_ref_f32_q4_with_zero_points over {rows} of {n} rows per "
                                   f"step (the reference has no group-wise CPU matmul), bytes scaled to rows"},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def gemv_leg(ms: float, nbytes: int, launches: int, world: int, peak: float) -> dict:
    """Compact line entry of a back-to-back linear leg: whole-job GB/s of
    algorithmic bytes, per-launch microseconds, fraction of the HBM peak."""
    per = ms * 1e-3 / launches
    return {"gbs": round(world * nbytes / per / 1e9, 1), "us": round(per * 1e6, 2),
            "frac": round(nbytes / per / 1e9 / peak, 3)}


def run_legs(torch, V, args, world: int, rank: int, peak: float, peaks: dict) -> dict:
    """Every secondary workload of the line (each its own seeded synthetic
    input, device-timed with CUDA events, max over ranks)."""
    legs = {}
    ls = max(5, args.steps // 2)
    cpu = rank == 0 and not args.no_cpu
    # the other bit widths and activation counts of the dequant-matmul sweep
    for key, m, bits in (("w3", 1, 3), ("w2", 1, 2), ("m8", 8, 4)):
        ms, _, nb = time_linear_graph(torch, V, m=m, n=N_DIM, k=K_DIM, bits=bits, copies=args.copies, steps=ls,
                                      warmup=args.warmup, world=world)
        legs[key] = gemv_leg(ms, nb, ls * args.copies, world, peak)
    # the literal GEMV config: 4096 x 4096, fp32 group scales and fp32 zero-point array (8), signed codes
    nb1 = 4096 * 2048 + 2 * 4096 * 32 * 4 + 2 * 4096 * 4
    c1 = copies_for(nb1)
    ms, _, nb = time_linear_graph(torch, V, m=1, n=4096, k=4096, bits=4, copies=c1, steps=ls, warmup=args.warmup,
                                  world=world, sz16=False, zp_array=True)
    legs["cfg1"] = gemv_leg(ms, nb, ls * c1, world, peak)
    legs["gemm"] = time_gemm(torch, V, world, max(3, args.steps // 5), peaks)
    a_steps = max(3, args.steps // 5)
    attn_ms, attn_kv, attn_other, attn_e2e_ms, attn_h2d, attn_d2h = time_attention(torch, V, a_steps, args.warmup,
                                                                                   world)
    per = attn_ms * 1e-3 / a_steps
    per_e2e = attn_e2e_ms * 1e-3 / a_steps
    legs["attn"] = {"gbs": round(world * (attn_kv + attn_other) / per / 1e9, 1), "ms": round(per * 1e3, 4),
                    "frac": round((attn_kv + attn_other) / per / 1e9 / peak, 3),
                    "e2e": {"gbs": round(world * (attn_kv + attn_other) / per_e2e / 1e9, 1),
                            "ms": round(per_e2e * 1e3, 4), "h2d_bytes_per_step": attn_h2d,
                            "d2h_bytes_per_step": attn_d2h}}
    if cpu:
        legs["attn"]["cpu"] = cpu_attention_sample()
    a3_ms, a3_kv, a3_other = time_attention_int3(torch, V, a_steps, args.warmup, world)
    per3 = a3_ms * 1e-3 / a_steps
    ar = time_attention_ref(torch, V, max(3, a_steps // 4), args.warmup, world)
    legs["aref"] = {"us": ar["us"], "gbs": ar["gbs"], "frac": round(ar["bytes"] / ar["us"] / 1e3 / peak, 3),
                    "module_us": ar["module_us"]}
    if rank == 0 and world == 1:
        legs["aref"]["cpu"] = cpu_attention_ref_sample()
    legs["attn_i3"] = {"gbs": round(world * (a3_kv + a3_other) / per3 / 1e9, 1), "ms": round(per3 * 1e3, 4),
                       "frac": round((a3_kv + a3_other) / per3 / 1e9 / peak, 3),
                       "vs_fp16": round(attn_ms / a3_ms, 3)}
    q_ms, q_bytes = time_q4k(torch, V, args.copies, a_steps, args.warmup, world)
    legs["q4k"] = gemv_leg(q_ms, q_bytes, a_steps * args.copies, world, peak)
    h_ms, h_bytes, h_bridge_ms, _, _ = time_hybrid(torch, V, args.copies, a_steps, args.warmup, world)
    legs["anf"] = dict(gemv_leg(h_ms, h_bytes, a_steps * args.copies, world, peak), bridge_ms=round(h_bridge_ms, 4))
    q = time_quantize(torch, V, world, cpu)
    legs["quant"] = {"gbs": q["value"], "ms": q["ms_per_matrix"]}
    if "cpu_baseline" in q:
        legs["quant"]["cpu_gbs"] = q["cpu_baseline"]["value"]
    if not args.no_decode:
        d = time_decode(torch, V, world, rank, peak)
        legs["dec"] = d
        if cpu:
            legs["dec"]["cpu"] = cpu_decode_sample(V.QWEN3_8B)
    if not args.no_tp and (world > 1 or args.tp1):
        legs["tp"] = time_decode_tp(torch, V, world, rank, peaks)
        if world > 1:
            legs["tp"]["parity"] = tp_parity(torch, V, world, rank)
        if cpu:
            legs["tp"]["cpu"] = cpu_decode_sample(V.QWEN3_32B)
    gemv_timeout_check(V)
    return legs


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--copies", type=int, default=24)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-legs", action="store_true", help="headline GEMV, e2e and CPU baseline only")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-tp", action="store_true", help="skip the Qwen3-32B-shape tensor-parallel decode (N >= 2)")
    ap.add_argument("--tp1", action="store_true", help="also run the tensor-parallel decode on one GPU (tp1)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
        return

    import torch

    import vspec_b200 as V
    rank, world, local = dist_setup(args.gpus)
    peak, peak_kind = load_peaks()
    peaks = load_peak_table()
    sampler = ClockSampler(local) if rank == 0 else None

    # headline: W4 GEMV, K=4096 N=12288 M=1, group 128, fp16 scales, mid-range zero-point
    ms4, clocks, b4 = time_linear_graph(torch, V, m=1, n=N_DIM, k=K_DIM, bits=4, copies=args.copies, steps=args.steps,
                                        warmup=args.warmup, world=world, sampler=sampler, soak_s=1.0)
    launches = args.steps * args.copies
    legs = {} if args.no_legs else run_legs(torch, V, args, world, rank, peak, peaks)
    e2e_steps = max(3, args.steps // 10)
    e2e_ms, e2e_bytes_call, h2d_call, d2h_call = time_e2e_bridge(torch, V, args.copies, e2e_steps, 2, world)

    gbs4 = world * launches * b4 / (ms4 * 1e-3) / 1e9
    per_launch_s = ms4 * 1e-3 / launches
    achieved = b4 / per_launch_s / 1e9
    e2e_gbs = world * e2e_steps * args.copies * e2e_bytes_call / (e2e_ms * 1e-3) / 1e9
    cpu = cpu_oracle_sample(args.cpu_seconds) if rank == 0 and not args.no_cpu else None
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(gbs4, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms4 / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u4 codes x int8 activation parts, int32 dots, fp32 acc",
        "data": "synthetic (seeded)",
        "config": {"workload": "W4 GEMV K=4096 N=12288 M=1 g128 fp16 scales mid zp",
                   "step": f"{args.copies} GEMVs over distinct weight copies, one CUDA graph",
                   "l2": f"inputs > L2: {args.copies} x {b4 / 1e6:.1f} MB", "parallelism": f"dp{world} replicas"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": load_traffic(), "peak_src": f"{peak_kind} hbm_gbs",
                     "bytes": b4, "launch_us": round(per_launch_s * 1e6, 3)},
        "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d_call * args.copies,
                "d2h_bytes_per_step": d2h_call * args.copies, "api": "vspec_cuda_fused_linear_int4_cached_bridge"},
        "cpu_baseline": cpu,
        "clocks": clocks,
        "gpu_launches": launches,
        "legs": legs,
    }
    print(json.dumps(line, separators=(",", ":")))


if __name__ == "__main__":
    main()
