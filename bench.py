"""Benchmark of the paged Q8_0 KV attention path (one JSON line on rank 0).

Default workload (decode_batch): one continuous-batching decode step of one
attention layer for 16 slots with ctx ~ U[1024, 32768], Hq 32 x D 128, Hkv 8,
Q8_0 K/V in 16-token pages scattered over a shared pool.  A step is the KV
write of the 16 new rows (quantize-and-scatter) plus split-KV decode
attention over every slot's keys.  With --gpus N each rank runs its own 16
slots (weak scaling, no collective on the data path); value = all ranks'
tokens / max-over-ranks time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl reference]

--impl reference times the CPU restatement of the path (oracle/, the
reference's own candle CPU path cannot be built here) on a bounded sample of
the same workload with all host threads.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
import __graft_entry__ as graft  # noqa: E402

graft.load_package()

METRIC = "paged int8-KV decode attn tokens/s & KV GB/s (% HBM peak) at 1/2/4/8 B200"
# attention options of every pool the bench builds (yf_attn_options; --schedule / --launch)
POOL_OPTIONS = {}
# how the sharded decode's partials reach every rank: "p2p" (push/combine kernels over NVLink
# peer memory) or "nccl" (all-gather, then yf_attn_combine)
TRANSPORT = {"kind": "p2p"}
SCHEDULES = {"auto": 0, "chunked": 1, "persistent": 2}


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def dominant_kernel(config: str) -> str:
    """The kernel that dominates one attention call of the workload."""
    return {"prefill_chunk": "prefill_tc_kernel", "prefill_rowscale": "prefill_tc_kernel",
            "prefill_d256": "prefill_tc256_kernel", "tree_verify": "splitkv_kernel", "decode_long": "decode_cluster_kernel",
            "decode_small": "decode_cluster_kernel", "attn_prep": "attn_prep_kernel",
            "snapshot_records": "records_kernel"}.get(config, "decode_persistent_kernel")


def profile_traffic(config: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", f"{dominant_kernel(config).replace('_kernel', '')}_{config}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------------------
# clocks sampled during the timed region


class ClockSampler:
    """Polls NVML (read-only: SM clock, max SM clock, clock-event reasons) every ~2 ms in a
    thread while the timed loops run; falls back to nothing if NVML is unavailable."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int):
        import threading

        self.samples, self.reasons, self.h, self.smax = [], 0, None, None
        self.stop_evt = threading.Event()
        self.thread = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self.nv = pynvml
            pr = torch.cuda.get_device_properties(device_index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            try:
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.smax = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.h = None

    def _reasons(self) -> int:
        nv = self.nv
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(fn(self.h))

    def _run(self):
        while not self.stop_evt.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self._reasons()
            except Exception:
                pass
            self.stop_evt.wait(0.002)

    def start(self):
        import threading

        if self.h is not None:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()

    def stop(self):
        if self.thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        self.stop_evt.set()
        self.thread.join()
        names = [n for n, bit in self.REASONS.items() if self.reasons & bit]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.smax, "reasons": names, "samples": len(self.samples),
                "source": "NVML, polled every 2 ms during the timed loops"}


# ---------------------------------------------------------------------------------------
# GPU arm


def packed(tensors, dev):
    """One device buffer holding a step's input tensors back to back (256-byte aligned) and views
    of it in their shapes and dtypes: the step's inputs then arrive in one host-to-device copy, as
    an engine stages a step's q / k / v rows and lengths in one pinned buffer."""
    import torch

    offs, off = [], 0
    for t in tensors:
        offs.append(off)
        off += -(-t.numel() * t.element_size() // 256) * 256
    buf = torch.zeros(off, dtype=torch.uint8, device=dev)
    views = []
    for t, o in zip(tensors, offs):
        v = buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
        v.copy_(t)
        views.append(v)
    return buf, views


class Step:
    """One workload resident on one GPU, with pre-bound C-ABI calls for the timed loop."""

    def __init__(self, wl, device: int, layers_resident: int = 1):
        import torch

        yf = graft.load_package()
        from qwen36_server_b200 import workloads as W

        self.torch, self.yf, self.wl = torch, yf, wl
        self.dev = torch.device("cuda", device)
        torch.cuda.set_device(self.dev)
        self.stream = torch.cuda.Stream(self.dev)  # every timed launch goes to this stream
        self.L = yf.lib()
        self.layers = layers_resident
        self.pool = yf.PagedKvPool(layers_resident, wl.n_pages, wl.n_kv_heads, wl.head_dim, wl.page_size,
                                   wl.group_size, device=device)
        self.pool.set_options(**POOL_OPTIONS)
        gen = torch.Generator(device=self.dev)
        gen.manual_seed(wl.seed)
        bt = torch.from_numpy(wl.block_table).to(self.dev)
        self.bt = bt
        # history: every key before the step's own rows, written through the multi-row writer
        prefix = wl.prefix
        for layer in range(layers_resident):
            chunk_rows = 1 << 18
            # write entry by entry in bounded row chunks to keep the f16 staging small
            for b in range(wl.batch):
                n = int(prefix[b])
                for s in range(0, n, chunk_rows):
                    m = min(chunk_rows, n - s)
                    k = W.kv_rows_torch(gen, m, wl.n_kv_heads, wl.head_dim, wl.outlier_frac, self.dev)
                    v = W.kv_rows_torch(gen, m, wl.n_kv_heads, wl.head_dim, wl.outlier_frac, self.dev)
                    yf.launch_append_multi(self.pool, layer, k, v, [0, m], [s], bt[b:b + 1], max_rows=m)
        T = int(wl.q_rows.sum())
        self.T = T
        self.k_new = W.kv_rows_torch(gen, T, wl.n_kv_heads, wl.head_dim, wl.outlier_frac, self.dev)
        self.v_new = W.kv_rows_torch(gen, T, wl.n_kv_heads, wl.head_dim, wl.outlier_frac, self.dev)
        self.q = torch.randn((T, wl.n_q_heads, wl.head_dim), generator=gen, device=self.dev).half()
        self.out = torch.empty_like(self.q)
        i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(self.dev)  # noqa: E731
        self.cu_k = i32(wl.cu_k)
        self.cu_q = i32(wl.cu_q)
        self.start = i32(wl.prefix)
        self.inputs, (self.q, self.k_new, self.v_new, self.start, self.cu_k) = packed(
            [self.q, self.k_new, self.v_new, self.start, self.cu_k], self.dev)
        self.trie = None if wl.trie is None else i32(wl.trie)
        self.decode = bool((wl.q_rows == 1).all()) and self.trie is None
        self.max_q = int(wl.q_rows.max())
        self.max_k = int(wl.ctx.max())
        ws = self.pool.workspace_size(wl.n_q_heads, wl.batch, self.max_q if not self.decode else 1, self.max_k)
        self.ws = torch.empty(max(ws, 16), dtype=torch.uint8, device=self.dev)
        self.ws_bytes = ws
        torch.cuda.synchronize()
        st = self.pool.status()
        if st:
            raise RuntimeError(f"device status {st} after building the workload")
        self._bind()

    def _bind(self):
        wl, L, P = self.wl, self.L, ctypes.c_void_p
        s = P(self.stream.cuda_stream)
        h = self.pool.handle
        scale = ctypes.c_float(self.yf.default_scale(wl.head_dim))
        ptr = lambda t: P(t.data_ptr())  # noqa: E731
        self.calls = []
        for layer in range(self.wl.n_layers):
            pl = layer % self.layers
            if self.decode:
                w = (L.yf_kv_append_paged, (h, pl, ptr(self.k_new), ptr(self.v_new), ptr(self.start), ptr(self.bt),
                                            wl.max_blocks, wl.batch, s))
                a = (L.yf_attn_decode, (h, pl, ptr(self.q), wl.n_q_heads, ptr(self.cu_k), ptr(self.bt),
                                        wl.max_blocks, wl.batch, self.max_k, scale, ptr(self.out), ptr(self.ws),
                                        self.ws_bytes, s))
            else:
                w = (L.yf_kv_append_paged_multi, (h, pl, ptr(self.k_new), ptr(self.v_new), ptr(self.cu_q),
                                                  ptr(self.start), ptr(self.bt), wl.max_blocks, wl.batch,
                                                  self.max_q, s))
                a = (L.yf_attn_prefill, (h, pl, ptr(self.q), wl.n_q_heads, ptr(self.cu_q), ptr(self.cu_k),
                                         ptr(self.bt), wl.max_blocks, wl.batch, self.max_q, self.max_k, scale,
                                         ptr(self.out), ptr(self.ws), self.ws_bytes, s))
                if self.trie is not None:  # tree speculative verify: the trie mask instead of causal rows
                    a = (L.yf_attn_verify_tree, (h, pl, ptr(self.q), wl.n_q_heads, ptr(self.cu_q), ptr(self.cu_k),
                                                 ptr(self.bt), wl.max_blocks, wl.batch, self.max_q, self.max_k, scale,
                                                 ptr(self.trie), ptr(self.out), ptr(self.ws), self.ws_bytes, s))
            self.calls.append((w, a))

    def run(self):
        for (wf, wa), (af, aa) in self.calls:
            if wf(*wa) or af(*aa):
                raise RuntimeError(self.L.yf_last_error().decode())

    def run_attn(self):
        for _, (af, aa) in self.calls:
            if af(*aa):
                raise RuntimeError(self.L.yf_last_error().decode())

    def capture(self):
        """CUDA graphs of one step and of its attention calls (after a warm call has set the
        kernels' attributes); replaying them removes host launch overhead, as the engine's
        decode graphs do."""
        torch = self.torch
        with torch.cuda.stream(self.stream):
            self.run()
        self.stream.synchronize()
        self.g_step, self.g_attn = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.g_step, stream=self.stream, capture_error_mode="relaxed"):
            self.run()
        with torch.cuda.graph(self.g_attn, stream=self.stream, capture_error_mode="relaxed"):
            self.run_attn()
        self.stream.synchronize()

    def launches_per_step(self) -> int:
        """KV write + split-KV attention per layer, + the separate combine kernel when the
        partials cannot be merged inside the attention kernel (fused combine off, or more
        units than the pool's arrival counters)."""
        wl = self.wl
        rows = wl.n_q_heads // wl.n_kv_heads * (1 if self.decode else self.max_q)
        rpc = 8 if (rows <= 8 or wl.head_dim > 128) else 16
        units = wl.batch * wl.n_kv_heads * -(-rows // rpc)
        fused = self.pool.options()["merge"] == 0 and units <= (1 << 16)
        separate = self.ws_bytes > 0 and not fused
        return wl.n_layers * (2 + (1 if separate else 0))


class ShardedStep:
    """decode_long on `world` GPUs: this rank's kv head and key range of the one sequence
    (qwen36_server_b200.sharding), partial decode -> exchange of the partials (peer-memory push
    or NCCL all-gather) -> LSE combine per step.  Strong scaling: every rank works on the same
    token."""

    def __init__(self, wl, device: int, rank: int, world: int):
        import torch

        yf = graft.load_package()
        from qwen36_server_b200 import sharding as S
        from qwen36_server_b200 import workloads as W

        self.torch, self.yf, self.wl = torch, yf, wl
        self.dev = torch.device("cuda", device)
        torch.cuda.set_device(self.dev)
        self.stream = torch.cuda.Stream(self.dev)
        self.L = yf.lib()
        self.layers = 1
        ctx = int(wl.ctx[0])
        self.shard = sh = S.long_context_plan(world, wl.n_kv_heads, ctx, wl.page_size)[rank]
        n = sh.k1 - sh.k0
        pages = max(1, -(-n // wl.page_size))
        self.world = world
        self.transport = TRANSPORT["kind"]
        self.sd = S.ShardedLongDecode(sh, wl.n_q_heads, wl.n_kv_heads, wl.head_dim, pages, wl.page_size,
                                      wl.group_size, batch=1, device=device, transport=self.transport)
        self.pool = self.sd.pool
        self.pool.set_options(**POOL_OPTIONS)
        gen = torch.Generator(device=self.dev)
        gen.manual_seed(wl.seed + 7919 * rank)
        self.bt = torch.arange(pages, dtype=torch.int32, device=self.dev).view(1, pages)
        self.owner = sh.k0 < ctx <= sh.k1  # holds the newest key: appends it every step
        hist = n - 1 if self.owner else n
        for s0 in range(0, hist, 1 << 18):
            m = min(1 << 18, hist - s0)
            k = W.kv_rows_torch(gen, m, sh.kv_heads, wl.head_dim, wl.outlier_frac, self.dev)
            v = W.kv_rows_torch(gen, m, sh.kv_heads, wl.head_dim, wl.outlier_frac, self.dev)
            yf.launch_append_multi(self.pool, 0, k, v, [0, m], [s0], self.bt, max_rows=m)
        self.T = 1
        self.k_new = W.kv_rows_torch(gen, 1, sh.kv_heads, wl.head_dim, wl.outlier_frac, self.dev)
        self.v_new = W.kv_rows_torch(gen, 1, sh.kv_heads, wl.head_dim, wl.outlier_frac, self.dev)
        self.q = torch.randn((1, wl.n_q_heads, wl.head_dim), generator=gen, device=self.dev).half()
        self.q_local = self.sd.q_slice(self.q)
        self.out = self.sd.out
        self.start = torch.tensor([n - 1], dtype=torch.int32, device=self.dev)
        self.cu_k = torch.tensor([0, n], dtype=torch.int32, device=self.dev)
        self.inputs, (self.q, self.k_new, self.v_new, self.start, self.cu_k) = packed(
            [self.q, self.k_new, self.v_new, self.start, self.cu_k], self.dev)
        # one entry: this rank's q heads are a contiguous run of q, read in place
        h0 = sh.kv_head0 * self.sd.G
        self.q_view = self.q[:, h0:h0 + self.sd.hq] if self.q.shape[0] == 1 else None
        if self.q_view is not None:
            self.q_local = self.q_view
        self.n = n
        self.scale = yf.default_scale(wl.head_dim)
        self.ws_bytes = self.pool.workspace_size(self.sd.hq, 1, 1, max(n, 1))
        torch.cuda.synchronize()
        if self.pool.status():
            raise RuntimeError("device status after building the shard")

    def run(self):
        if self.owner:
            self.yf.kv_append_paged(self.pool, 0, self.k_new, self.v_new, self.start, self.bt)
        if self.q_view is None:  # several entries: this rank's heads are strided in q
            h0 = self.shard.kv_head0 * self.sd.G
            self.q_local.copy_(self.q[:, h0:h0 + self.sd.hq])
        self.sd.step(self.q_local, self.cu_k, self.bt, self.scale, max(self.n, 1))

    def run_attn(self):
        self.sd.partial(self.q_local, self.cu_k, self.bt, self.scale, max(self.n, 1))

    def capture(self):
        """CUDA graphs of one step (the exchange included) and of the partial alone, after a
        warm step has created the NCCL communicator and the workspace.  The ranks meet first:
        a peer-memory combine waits (bounded) for every rank's push of the same step."""
        torch = self.torch
        if self.world > 1:
            torch.distributed.barrier()
        with torch.cuda.stream(self.stream):
            self.run()
        self.stream.synchronize()
        self.g_step, self.g_attn = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.g_step, stream=self.stream, capture_error_mode="relaxed"):
            self.run()
        with torch.cuda.graph(self.g_attn, stream=self.stream, capture_error_mode="relaxed"):
            self.run_attn()
        self.stream.synchronize()

    def release(self):
        """Drops the graphs (the step's may hold an NCCL call: gone before the process group)."""
        self.g_step = self.g_attn = None

    def status(self) -> int:
        """The pool's device status bits, with the exchange's (a combine wait that ran out)."""
        st = self.pool.status()
        if self.sd.peer is not None:
            st |= self.sd.peer.status()
        return st

    def launches_per_step(self) -> int:
        """KV write (owner only) + the shard's decode with the exchange fused in (p2p: one
        launch), or partial decode + one combine per head group (nccl: the all-gather is NCCL's
        kernel).  A q slice of several entries is a torch copy."""
        if self.transport == "p2p" and self.sd.fused:
            return (1 if self.owner else 0) + 1
        ex = 2 if self.transport == "p2p" else self.shard.n_head_groups
        return (1 if self.owner else 0) + 1 + ex


def make_workload(name: str, rank: int, layers: int = 0):
    from qwen36_server_b200 import workloads as W

    fn = W.CONFIGS[name]
    base_seed = fn.__defaults__[0]
    if layers and name in ("mtp_verify", "tree_verify"):
        return fn(seed=base_seed + 1000 * rank, n_layers=layers)
    return fn(seed=base_seed + 1000 * rank)


def partition(wl_full, world: int, rank: int):
    """This rank's share of the workload at N GPUs, and how the job is split:
    - "slots": independent entries bin-packed by context over the GPUs (LPT); the same job at
      every N (strong scaling), no collective on the data path;
    - "sharded": the one long sequence split by kv head x key range (partials exchanged);
    - "replica": a workload with fewer entries than GPUs runs whole on every GPU (weak scaling)."""
    from qwen36_server_b200 import sharding as S
    from qwen36_server_b200 import workloads as W

    if world == 1:
        return wl_full, "slots", [list(range(wl_full.batch))]
    if wl_full.name == "decode_long":
        return wl_full, "sharded", None
    if wl_full.batch >= world:
        bins = S.lpt_partition(wl_full.ctx, world)
        return W.subset(wl_full, bins[rank], seed=wl_full.seed + 1000 * rank), "slots", bins
    return make_workload(wl_full.name, rank), "replica", None


class Timer:
    """Device time of passes of `steps` replays on one stream.  The pass count is agreed over the
    ranks (a calibration pass, max over ranks), so that steps holding collectives stay in step;
    passes run until `min_s` seconds of GPU time have elapsed.  Returns the median pass's ms per
    step (max over ranks is taken by the caller) and the number of passes."""

    def __init__(self, stream, world: int):
        import torch

        self.torch, self.stream, self.world = torch, stream, world

    def _pass(self, run, steps: int) -> float:
        torch = self.torch
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        for _ in range(steps):
            run()
        b.record(self.stream)
        b.synchronize()
        return a.elapsed_time(b)

    def agreed(self, value: float) -> float:
        if self.world == 1:
            return value
        import torch.distributed as dist

        t = self.torch.tensor([value], dtype=self.torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def run(self, run, steps: int, min_s: float, barrier):
        first = self.agreed(self._pass(run, steps))
        n = max(3, min(2000, int(-(-min_s * 1e3 // max(first, 1e-3)))))
        barrier()
        ms = [self._pass(run, steps) / steps for _ in range(n)]
        return statistics.median(ms), n


def gpu_arm(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    wl_full = make_workload(args.config, 0, args.layers)
    wl, mode, bins = partition(wl_full, world, rank)
    sharded = mode == "sharded"
    layers_resident = wl.n_layers
    if args.config in ("mtp_verify", "tree_verify"):
        free = torch.cuda.mem_get_info(local_rank)[0]
        per_layer = wl.kv_bytes(1)
        layers_resident = max(1, min(wl.n_layers, int(0.8 * free // max(per_layer, 1))))
    step = ShardedStep(wl, local_rank, rank, world) if sharded else Step(wl, local_rank, layers_resident)
    stream = step.stream
    if args.no_graph:
        run_step, run_attn = step.run, step.run_attn
    else:
        step.capture()  # the sharded step's graph holds its exchange (push + combine, or NCCL's all-gather)
        run_step, run_attn = step.g_step.replay, step.g_attn.replay

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    timer = Timer(stream, world)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            run_step()
        barrier()
        clocks = ClockSampler(local_rank)
        clocks.start()
        ms, passes = timer.run(run_step, args.steps, args.min_seconds, barrier)
        barrier()

        # dominant kernel: the attention call alone, events around each replay
        n_ev = max(args.steps, 50)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_ev)]
        for a, b in evs:
            a.record(stream)
            run_attn()
            b.record(stream)
        torch.cuda.synchronize()
        attn_ms = sum(a.elapsed_time(b) for a, b in evs) / n_ev / wl.n_layers

        # end to end through the public API with host buffers: the step's inputs (q, the new K/V
        # rows, positions, lengths) staged in one pinned buffer and copied in, the output read
        # back, every step
        h_in = torch.empty(step.inputs.shape, dtype=torch.uint8, pin_memory=True).copy_(step.inputs.cpu())
        h_out = torch.empty(step.out.shape, dtype=step.out.dtype, pin_memory=True)
        bytes_in = h_in.numel()
        bytes_out = h_out.numel() * h_out.element_size()

        def e2e_step():
            step.inputs.copy_(h_in, non_blocking=True)
            run_step()
            h_out.copy_(step.out, non_blocking=True)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier()
        e2e_ms, _ = timer.run(e2e_step, args.steps, args.min_seconds / 3, barrier)
        barrier()
        clk = clocks.stop()

    t = torch.tensor([ms, e2e_ms, attn_ms], dtype=torch.float64, device=step.dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, attn_ms = t.tolist()
    status = step.status() if sharded else step.pool.status()

    if mode == "replica":
        tokens = step.T * world
    else:
        tokens = int(wl_full.q_rows.sum())   # the same job at every N
    kv_bytes = wl.kv_bytes() // (world if sharded else 1)  # this GPU's
    hbm, tflops, peak_kind = peaks()
    alg_bytes_attn = wl.kv_bytes(1) // (world if sharded else 1)
    achieved_gbs = alg_bytes_attn / (attn_ms * 1e-3) / 1e9
    if wl.name.startswith("prefill"):
        roof = {"bound": "tensor", "achieved": wl.attn_flops() / wl.n_layers / (attn_ms * 1e-3) / 1e12,
                "peak": tflops, "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["traffic"] = profile_traffic(args.config) if world == 1 else None
    roof["kernel"] = dominant_kernel(args.config) + (" (this rank's partial over its shard)" if sharded
                                                      else " (one attention call)")
    roof["peak_source"] = f"{peak_kind} (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback"
    roof["algorithmic_bytes_per_launch"] = alg_bytes_attn
    roof["launch_ms"] = attn_ms

    if mode == "slots" and world > 1:
        loads = [int(wl_full.ctx[b].sum()) for b in bins]
        parallelism = (f"slots LPT-packed by context over {world} GPUs (same {wl_full.batch} slots at every N, "
                       "no collective on the data path)")
    elif sharded:
        how = ("partials pushed over NVLink peer memory, LSE combine" if TRANSPORT["kind"] == "p2p"
               else "partials all-gathered over NCCL, LSE combine")
        parallelism = f"kv-head x sequence sharded x{world} ({how})"
    elif mode == "replica":
        parallelism = f"replicas x{world} (fewer entries than GPUs: each GPU runs the whole workload)"
    else:
        parallelism = "one GPU"
    line = {
        "metric": METRIC,
        "value": tokens / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak" if mode == "replica" else "strong",
        "vs_baseline": None,
        "dtype": "f16 (int8 KV unpacked exactly to f16 for mma, f32 accumulate)",
        "data": "synthetic (seeded N(0,1) K/V, fragmented seeded page tables)",
        "config": {
            "workload": describe(wl_full),
            "slots_this_gpu": wl.batch,
            "query_rows_this_gpu": step.T,
            "sum_ctx_this_gpu": int(wl.ctx.sum()),
            "layers": wl.n_layers,
            "layers_resident": step.layers,
            "kv_bytes_per_step_this_gpu": kv_bytes,
            "l2": "inputs larger than L2: the pool read per step exceeds 126 MB" if wl_full.kv_bytes(1) > 126e6
            else "pool fits in L2 (small workload)",
            "parallelism": parallelism,
            "launch": "direct C-ABI calls" if args.no_graph else (
                "CUDA graph replay of the step (partial, exchange of the partials, combine)" if sharded
                else "CUDA graph replay of the step's C-ABI calls"),
            "timing": f"median of {passes} passes of {args.steps} steps (>= {args.min_seconds} s of GPU time), "
                      "CUDA events on the launching stream, max over ranks",
        },
        "kv_gbs": (wl_full.kv_bytes() if mode != "replica" else wl.kv_bytes() * world) / (ms * 1e-3) / 1e9,
        "hbm_frac_step": kv_bytes / (ms * 1e-3) / 1e9 / hbm,
        "roofline": roof,
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": bytes_in,
                "d2h_bytes_per_step": bytes_out, "ms_per_step": e2e_ms,
                "note": "this GPU's inputs from pinned host memory and its output back, every step"},
        "gpu_launches": step.launches_per_step() * args.steps,
        "clocks": clk,
        "device_status": status,
    }
    if mode == "slots" and world > 1:
        mean = sum(loads) / world
        line["partition"] = {"keys_per_gpu": loads, "imbalance": max(loads) / mean,
                             "limiter": "the largest GPU share (LPT imbalance) plus each GPU's fixed launch and "
                                        "merge latency, which no longer shrink with N"}
    if sharded and hasattr(step, "release"):
        step.release()
    if world > 1 and args.config == "decode_batch" and not args.no_long:
        del step
        torch.cuda.empty_cache()
        try:
            line["decode_long_sharded"] = long_sharded_leg(args, rank, world, local_rank)
        except Exception as exc:  # reported in the line; the decode_batch result above stands
            line["decode_long_sharded"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(wl_full, args.cpu_seconds)
    return line


def long_sharded_leg(args, rank: int, world: int, local_rank: int) -> dict:
    """The 131072-key decode at the same N: kv head x key-range shards, partial decode, exchange
    of the packed partials (peer-memory push, or NCCL all-gather), LSE combine; replayed as one
    CUDA graph per rank."""
    import torch
    import torch.distributed as dist

    wl = make_workload("decode_long", 0)
    step = ShardedStep(wl, local_rank, rank, world)
    step.capture()
    timer = Timer(step.stream, world)

    def barrier():
        dist.barrier()
        torch.cuda.synchronize()

    with torch.cuda.stream(step.stream):
        for _ in range(max(3, args.warmup)):
            step.g_step.replay()
        barrier()
        ms, passes = timer.run(step.g_step.replay, args.steps, max(0.5, args.min_seconds / 3), barrier)
        barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(50)]
        for a, b in evs:
            a.record(step.stream)
            step.g_attn.replay()
            b.record(step.stream)
        torch.cuda.synchronize()
        part_ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)
    t = torch.tensor([ms, part_ms], dtype=torch.float64, device=step.dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, part_ms = t.tolist()
    status = step.status()
    step.release()
    hbm, _, _ = peaks()
    shard_bytes = wl.kv_bytes(1) // world
    if step.transport == "p2p":
        limiter = ("the shard's own decode (one kv head x key range: launch, stream and merge tail); the "
                   "exchange is fused into its last slice merges (partial stored into every rank's area "
                   "over NVLink as value+step words, polled and merged in place)")
    else:
        limiter = ("the NCCL all-gather of the packed partials plus the combine launch (latency, a few KB "
                   "moved) on top of the shard's partial decode")
    return {"workload": describe(wl), "ms_per_step": ms, "tokens_per_s": 1.0 / (ms * 1e-3),
            "partial_ms": part_ms, "partial_hbm_frac": shard_bytes / (part_ms * 1e-3) / 1e9 / hbm,
            "exchange_and_combine_ms": ms - part_ms, "passes": passes, "transport": step.transport,
            "limiter": limiter, "parallelism": f"kv-head x sequence sharded x{world}", "device_status": status}


def describe(wl) -> str:
    c = wl.ctx
    rng = f"ctx {int(c.min())}..{int(c.max())} (sum {int(c.sum())})" if len(c) > 1 else f"ctx {int(c[0])}"
    return (f"{wl.name}: {wl.batch} entries x {int(wl.q_rows.max())} query rows, {rng}, "
            f"Hq {wl.n_q_heads} x D {wl.head_dim}, Hkv {wl.n_kv_heads}, Q8_0 (group {wl.group_size}) "
            f"{wl.page_size}-token pages, {wl.n_layers} layer(s)")


# ---------------------------------------------------------------------------------------
# CPU: the oracle's restatement of the path on the workload (or a bounded sample of it)


class CpuSample:
    """The workload's entries (their own keys) prepared for the CPU oracle.  Entries are taken,
    median context first, while their (query row x key) pairs fit `max_pairs`; a single entry
    that alone exceeds it keeps only its last query rows (a shorter chunk over the same prefix)."""

    def __init__(self, wl, max_pairs: float):
        from qwen36_server_b200 import workloads as W

        self.O = graft.load_oracle()
        max_pairs = max_pairs / wl.n_layers   # every layer repeats the step's work
        pairs = wl.ctx * wl.q_rows
        order = np.argsort(wl.ctx, kind="stable")
        pick, tot = [], 0
        for i in order[len(order) // 2:].tolist() + order[:len(order) // 2].tolist():   # median first
            if tot + pairs[i] > max_pairs and pick:
                continue
            pick.append(i)
            tot += int(pairs[i])
        pick = sorted(pick)
        ctx, q_rows = wl.ctx[pick].copy(), wl.q_rows[pick].copy()
        if len(pick) == 1 and pairs[pick[0]] > max_pairs and q_rows[0] > 1:
            keep = max(1, int(max_pairs // ctx[0]))
            ctx[0] -= q_rows[0] - keep
            q_rows[0] = keep
        self.full = len(pick) == wl.batch and np.array_equal(q_rows, wl.q_rows)
        self.sub = W.Workload("cpu", wl.n_q_heads, wl.n_kv_heads, wl.head_dim, ctx=ctx, q_rows=q_rows,
                              page_size=wl.page_size, group_size=wl.group_size, outlier_frac=wl.outlier_frac,
                              seed=wl.seed)
        s = self.sub
        self.desc = self.O.PoolDesc(1, s.n_pages, s.n_kv_heads, s.head_dim, s.page_size, s.group_size)
        rng = np.random.default_rng(s.seed)
        n = int(s.ctx.sum())
        k = W.kv_rows_np(rng, n, s.n_kv_heads, s.head_dim, s.outlier_frac)
        v = W.kv_rows_np(rng, n, s.n_kv_heads, s.head_dim, s.outlier_frac)
        self.pool = np.zeros(self.desc.pool_bytes, np.uint8)
        entry = np.repeat(np.arange(s.batch), s.ctx).astype(np.int32)
        pos = np.concatenate([np.arange(c) for c in s.ctx]).astype(np.int32)
        hist = np.ones(n, bool)
        starts = np.concatenate([[0], np.cumsum(s.ctx)])[:-1]
        for b in range(s.batch):
            hist[starts[b] + s.prefix[b]: starts[b] + s.ctx[b]] = False
        self.O.c_kv_write_rows(self.desc, self.pool, 0, k[hist], v[hist], entry[hist], pos[hist], s.block_table)
        self.new = (k[~hist], v[~hist], entry[~hist], pos[~hist])
        self.q = rng.standard_normal((int(s.q_rows.sum()), s.n_q_heads, s.head_dim)).astype(np.float16)
        self.threads = os.cpu_count() or 1
        self.tokens = int(s.q_rows.sum())
        self.n_layers = wl.n_layers

    def step(self):
        s = self.sub
        k, v, e, p = self.new
        for _ in range(self.n_layers):
            self.O.c_kv_write_rows(self.desc, self.pool, 0, k, v, e, p, s.block_table)
            self.O.c_attn(self.desc, self.pool, 0, self.q, s.cu_q, s.cu_k, s.block_table,
                          1.0 / np.sqrt(s.head_dim), self.threads)

    def describe(self, wl, steps: int) -> str:
        what = "the whole workload" if self.full else (
            f"{self.sub.batch} of {wl.batch} entries, {int(self.sub.q_rows.sum())} of {int(wl.q_rows.sum())} "
            f"query rows")
        return (f"{what} ({int(self.sub.ctx.sum())} keys, {self.n_layers} layer(s)) per step, {steps} steps; "
                "oracle/yf_oracle.c double-precision attention + Q8_0 scatter on all host threads")


# pairs of (query row, key) in one CPU step: the whole decode_batch step (266k pairs, ~0.5 s on
# 16 threads), a bounded sample of the larger workloads
CPU_MAX_PAIRS = 3.0e5


def cpu_baseline(wl, seconds: float):
    samp = CpuSample(wl, max_pairs=CPU_MAX_PAIRS)
    samp.step()
    t0 = time.perf_counter()
    n = 0
    while True:
        samp.step()
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": samp.tokens / dt, "unit": "tokens/s", "cores": samp.threads, "kind": "port",
            "same_config": samp.full,
            "sample": samp.describe(wl, n) + ("; causal rows stand in for the trie mask (same keys but the "
                                              "skipped branch nodes)" if wl.trie is not None else "")}


def prep_arm(args, rank: int, world: int, local_rank: int):
    """--config attn_prep: the fused attention prep + Q8_0 append (yf_attn_prepare_append) over
    prefill_chunk's new rows (4 entries x 2048 rows at their 8192-token prefixes, Hq 32 x D 128,
    Hkv 8, RoPE on the first 32 dims).  A step is one launch over all rows; HBM-bound: it reads
    q|gate, k, v (f16) and writes q, gate (f16) and the rows' Q8_0 pool bytes."""
    import torch
    import torch.distributed as dist

    yf = graft.load_package()
    from qwen36_server_b200 import workloads as W

    wl = W.prefill_chunk(seed=4 + 1000 * rank)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    Hq, H, D, R = wl.n_q_heads, wl.n_kv_heads, wl.head_dim, 32
    T = int(wl.q_rows.sum())
    g = torch.Generator(device=dev)
    g.manual_seed(17 + rank)
    qg = torch.randn((T, Hq, 2 * D), generator=g, device=dev).half()
    k = torch.randn((T, H, D), generator=g, device=dev).half()
    v = torch.randn((T, H, D), generator=g, device=dev).half()
    wq = (torch.randn(D, generator=g, device=dev) * 0.2).float()
    wk = (torch.randn(D, generator=g, device=dev) * 0.2).float()
    n_pos = int(wl.ctx.max())
    inv = 1e7 ** (-torch.arange(0, R, 2, dtype=torch.float64) / R)
    ang = torch.arange(n_pos, dtype=torch.float64)[:, None] * inv[None, :]
    cos, sin = ang.cos().float().to(dev), ang.sin().float().to(dev)
    pool = yf.PagedKvPool(1, wl.n_pages, H, D, device=local_rank)
    cu = torch.from_numpy(wl.cu_q).to(dev)
    start = torch.from_numpy(wl.prefix.astype(np.int32)).to(dev)
    bt = torch.from_numpy(wl.block_table).to(dev)
    q_out = torch.empty((T, Hq, D), dtype=torch.float16, device=dev)
    gate_out = torch.empty_like(q_out)
    L = yf.lib()
    P = ctypes.c_void_p
    ptr = lambda t: P(t.data_ptr())  # noqa: E731
    args_c = (pool.handle, 0, Hq, ptr(qg), ptr(k), ptr(v), ptr(wq), ptr(wk), ctypes.c_float(1e-6), 1, ptr(cos),
              ptr(sin), R, n_pos, ptr(cu), ptr(start), ptr(bt), wl.max_blocks, wl.batch, int(wl.q_rows.max()),
              ptr(q_out), ptr(gate_out), P(stream.cuda_stream))

    def run():
        if L.yf_attn_prepare_append(*args_c):
            raise RuntimeError(L.yf_last_error().decode())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    alg = T * (Hq * 2 * D * 2 + 2 * H * D * 2 + 2 * Hq * D * 2) + T * wl.kv_bytes_per_token
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            run()
        barrier()
        clocks = ClockSampler(local_rank)
        clocks.start()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in evs:
            a.record(stream)
            run()
            b.record(stream)
        barrier()
        ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
        # end to end: the step's inputs from pinned host memory, q and gate back
        pin = lambda t: torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t.cpu())  # noqa: E731
        h_in = [(pin(t), t) for t in (qg, k, v)]
        h_out = [(torch.empty(t.shape, dtype=t.dtype, pin_memory=True), t) for t in (q_out, gate_out)]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            for h, d in h_in:
                d.copy_(h, non_blocking=True)
            run()
            for h, d in h_out:
                h.copy_(d, non_blocking=True)
        e1.record(stream)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        clk = clocks.stop()
    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    hbm, _, peak_kind = peaks()
    gbs = alg / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC + " (fused attention prep + KV append)", "value": T * world / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 norm/RoPE on f16 rows, Q8_0 KV", "data": "synthetic (seeded N(0,1) rows and weights)",
        "config": {"workload": f"attn_prep: {T} new rows ({wl.batch} x {int(wl.q_rows[0])} at {int(wl.prefix[0])}"
                               f"-token prefixes), Hq {Hq} x D {D}, Hkv {H}, rope_dim {R}",
                   "l2": "inputs larger than L2", "parallelism": f"row-sharded x{world}, no collective",
                   "launch": "direct C-ABI calls"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                     "traffic": profile_traffic("attn_prep"), "kernel": "attn_prep_kernel",
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback",
                     "algorithmic_bytes_per_launch": alg, "launch_ms": ms},
        "e2e": {"value": T * world / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": sum(h.numel() * h.element_size() for h, _ in h_in),
                "d2h_bytes_per_step": sum(h.numel() * h.element_size() for h, _ in h_out), "ms_per_step": e2e_ms},
        "gpu_launches": args.steps,
        "clocks": clk,
        "device_status": pool.status(),
    }
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        O = graft.load_oracle()
        n = 256
        rows = np.arange(n)
        qh, kh = qg[:n].cpu().numpy(), k[:n].cpu().numpy()
        c_np, s_np, wq_np, wk_np = cos.cpu().numpy(), sin.cpu().numpy(), wq.cpu().numpy(), wk.cpu().numpy()
        pos = (wl.prefix[0] + rows).astype(np.int64)
        O.np_attn_prep(qh, kh, wq_np, wk_np, 1e-6, 1, c_np, s_np, R, pos)
        t0, reps = time.perf_counter(), 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 10.0):
            O.np_attn_prep(qh, kh, wq_np, wk_np, 1e-6, 1, c_np, s_np, R, pos)
            reps += 1
        line["cpu_baseline"] = {"value": n * reps / (time.perf_counter() - t0), "unit": "tokens/s", "cores": 1,
                                "kind": "port", "sample": f"{n} rows per call, oracle.np_attn_prep (numpy, "
                                                          "norm + RoPE + gate split; the Q8_0 append not included)"}
    pool.close()
    return line


def records_arm(args, rank: int, world: int, local_rank: int):
    """--config snapshot_records: export to and import from the prefix cache's page records
    (yf_pool_export_records / yf_pool_import_records, CRC-32C on the GPU) for prefill_chunk's
    restored prefixes: 4 x 8192 tokens = 2048 16-token pages of one layer (71.3 MB of pages).
    A step is one export plus one import of every page; a "token" is one prefix token moved."""
    import torch
    import torch.distributed as dist

    yf = graft.load_package()
    from qwen36_server_b200 import workloads as W

    wl = W.prefill_chunk(seed=4 + 1000 * rank)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    n = int(wl.prefix.sum()) // wl.page_size
    src = yf.PagedKvPool(1, n, wl.n_kv_heads, wl.head_dim, device=local_rank)
    dst = yf.PagedKvPool(1, n, wl.n_kv_heads, wl.head_dim, device=local_rank)
    g = torch.Generator(device=dev)
    g.manual_seed(5 + rank)
    view = src.layer_bytes_view(0)
    view.copy_(torch.randint(0, 256, view.shape, generator=g, device=dev, dtype=torch.uint8))
    pages = torch.randperm(n, generator=g, device=dev).int()
    hashes = torch.arange(n, device=dev, dtype=torch.int64) * 0x9E3779B97F4A7C15 % (2 ** 62)
    idx = torch.arange(n, device=dev, dtype=torch.int32)
    prev = torch.cat([torch.zeros(1, device=dev, dtype=torch.int64), hashes[:-1]])
    tokens = torch.randint(0, 151936, (n, wl.page_size), generator=g, device=dev, dtype=torch.int32)
    rb = src.record_bytes
    rec = torch.empty(n * rb, dtype=torch.uint8, device=dev)
    ok = torch.zeros(n, dtype=torch.int32, device=dev)
    L = yf.lib()
    P = ctypes.c_void_p
    ptr = lambda t: P(t.data_ptr())  # noqa: E731
    s = P(stream.cuda_stream)

    def run():
        if L.yf_pool_export_records(src.handle, n, ptr(pages), ptr(hashes), ptr(prev), ptr(idx), ptr(tokens),
                                    ptr(rec), s):
            raise RuntimeError(L.yf_last_error().decode())
        if L.yf_pool_import_records(dst.handle, n, ptr(pages), ptr(rec), ptr(hashes), ptr(tokens), ptr(ok), s):
            raise RuntimeError(L.yf_last_error().decode())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    alg = 2 * (n * src.page_bytes + n * rb)  # each direction reads and writes the bytes once
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            run()
        barrier()
        clocks = ClockSampler(local_rank)
        clocks.start()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in evs:
            a.record(stream)
            run()
            b.record(stream)
        barrier()
        ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
        # end to end: the records go to pinned host memory and back (the disk tier's buffers)
        h = torch.empty(rec.shape, dtype=torch.uint8, pin_memory=True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            if L.yf_pool_export_records(src.handle, n, ptr(pages), ptr(hashes), ptr(prev), ptr(idx), ptr(tokens),
                                        ptr(rec), s):
                raise RuntimeError(L.yf_last_error().decode())
            h.copy_(rec, non_blocking=True)
            rec.copy_(h, non_blocking=True)
            if L.yf_pool_import_records(dst.handle, n, ptr(pages), ptr(rec), ptr(hashes), ptr(tokens), ptr(ok), s):
                raise RuntimeError(L.yf_last_error().decode())
        e1.record(stream)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        clk = clocks.stop()
    good = int(ok.sum().item())
    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    hbm, _, peak_kind = peaks()
    gbs = alg / (ms * 1e-3) / 1e9
    tokens = n * wl.page_size
    line = {
        "metric": METRIC + " (prefix snapshot records: export + import)", "value": tokens * world / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8 (bytes, CRC-32C)",
        "data": "synthetic (random pool bytes)",
        "config": {"workload": f"snapshot_records: {n} pages x {src.page_bytes} B (4 x {int(wl.prefix[0])} prefix "
                               f"tokens, Hkv {wl.n_kv_heads} x D {wl.head_dim}, 1 layer), records of {rb} B",
                   "records_intact": f"{good} of {n}", "parallelism": f"x{world} independent pools, no collective",
                   "launch": "direct C-ABI calls"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                     "traffic": profile_traffic("snapshot_records"), "kernel": "export_records_kernel + import_records_kernel",
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback",
                     "algorithmic_bytes_per_launch": alg, "launch_ms": ms},
        "e2e": {"value": tokens * world / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": rec.numel(),
                "d2h_bytes_per_step": rec.numel(), "ms_per_step": e2e_ms},
        "gpu_launches": 2 * args.steps,
        "clocks": clk,
        "device_status": src.status() | dst.status(),
    }
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        O = graft.load_oracle()
        sample = rec[: 8 * rb].cpu().numpy()
        t0, reps = time.perf_counter(), 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 10.0):
            for r in range(8):
                O.crc32c(sample[r * rb + 20:(r + 1) * rb])
            reps += 1
        line["cpu_baseline"] = {"value": 8 * reps * wl.page_size / (time.perf_counter() - t0), "unit": "tokens/s",
                                "cores": 1, "kind": "port", "sample": "8 records per pass, the oracle's bitwise "
                                                                      "CRC-32C of each payload (the copy not included)"}
    src.close()
    dst.close()
    return line


def prep_reference_arm(args):
    """--impl reference for attn_prep: the oracle's restatement of the prep (numpy, one thread) on
    256 of the rows per step; the reference's candle path cannot be built here."""
    from qwen36_server_b200 import workloads as W

    O = graft.load_oracle()
    wl = W.prefill_chunk(seed=4)
    rng = np.random.default_rng(17)
    n, Hq, H, D, R = 256, wl.n_q_heads, wl.n_kv_heads, wl.head_dim, 32
    qg = rng.standard_normal((n, Hq, 2 * D)).astype(np.float16)
    k = rng.standard_normal((n, H, D)).astype(np.float16)
    w = (rng.standard_normal(D) * 0.2).astype(np.float32)
    ang = np.arange(int(wl.ctx.max()))[:, None] * 1e7 ** (-np.arange(0, R, 2) / R)[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    pos = int(wl.prefix[0]) + np.arange(n)
    for _ in range(args.warmup):
        O.np_attn_prep(qg, k, w, w, 1e-6, 1, cos, sin, R, pos)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.np_attn_prep(qg, k, w, w, 1e-6, 1, cos, sin, R, pos)
    dt = (time.perf_counter() - t0) / args.steps
    v = n / dt
    return {
        "impl": "reference", "metric": METRIC + " (fused attention prep + KV append)", "value": v,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (oracle)",
        "data": "synthetic", "config": {"workload": f"attn_prep: {n} rows per step, Hq {Hq} x D {D}, Hkv {H}"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": 1, "kind": "port",
                         "sample": f"{n} rows per step, oracle.np_attn_prep (norm + RoPE + gate split)"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def reference_arm(args):
    if args.config == "attn_prep":
        return prep_reference_arm(args)
    if args.config == "snapshot_records":
        return {"impl": "reference", "unavailable": "the prefix cache's record writer lives in the un-vendored Rust "
                                                    "fork (no Rust toolchain here); bench.py --config snapshot_records "
                                                    "reports the oracle's CRC-32C as its cpu_baseline"}
    wl = make_workload(args.config, 0)
    samp = CpuSample(wl, max_pairs=args.ref_pairs)
    for _ in range(args.warmup):
        samp.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        samp.step()
    dt = (time.perf_counter() - t0) / args.steps
    v = samp.tokens / dt
    return {
        "impl": "reference",
        "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong" if wl.batch > 1 else "weak",
        "vs_baseline": None, "dtype": "f64 (oracle)", "data": "synthetic",
        "config": {"workload": describe(wl), "sample": describe(samp.sub), "same_config": samp.full},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": samp.threads, "kind": "port",
                         "same_config": samp.full,
                         "sample": samp.describe(wl, args.steps) + "; the reference's candle CPU path cannot be "
                                                                   "built here (no Rust toolchain, fork not vendored)"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="decode_batch",
                    choices=["decode_small", "decode_batch", "decode_long", "prefill_chunk", "prefill_rowscale",
                             "prefill_d256", "mtp_verify", "tree_verify", "attn_prep", "snapshot_records"])
    ap.add_argument("--impl", default="yfattn", choices=["yfattn", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch every call directly instead of replaying a CUDA graph")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-pairs", type=float, default=CPU_MAX_PAIRS,
                    help="--impl reference: (query row x key) pairs per CPU step (the whole decode_batch step fits)")
    ap.add_argument("--min-seconds", type=float, default=1.5,
                    help="GPU time the timed passes of --steps steps must cover (median pass reported)")
    ap.add_argument("--no-long", action="store_true", help="N>1: skip the sharded decode_long leg")
    ap.add_argument("--schedule", default="auto", choices=sorted(SCHEDULES),
                    help="split-KV schedule of the pools (yf_attn_options.schedule), for A/B runs")
    ap.add_argument("--verify-kernel", default="auto", choices=["auto", "tcgen05"],
                    help="verify blocks on the split-KV kernel (auto) or the tcgen05 kernel (yf_attn_options.verify_kernel)")
    ap.add_argument("--cooperative", action="store_true",
                    help="launch the persistent decode cooperatively (yf_attn_options.launch)")
    ap.add_argument("--transport", default="p2p", choices=["p2p", "nccl"],
                    help="N>1 sharded decode: partials pushed over NVLink peer memory (p2p) or all-gathered by NCCL")
    ap.add_argument("--layers", type=int, default=0,
                    help="mtp_verify only: stack this many layers instead of 36 (one launch per layer keeps "
                         "its shape; for profiling a launch with a few GB resident, not a bench line)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    TRANSPORT["kind"] = args.transport
    POOL_OPTIONS.update(schedule=SCHEDULES[args.schedule], launch=1 if args.cooperative else 0,
                        verify_kernel=1 if args.verify_kernel == "tcgen05" else 0)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(reference_arm(args)), flush=True)
        return

    import torch

    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        arm = {"attn_prep": prep_arm, "snapshot_records": records_arm}.get(args.config, gpu_arm)
        line = arm(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
