"""KV-cache data-movement benchmark (paged scatter / handoff / append / fork).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (N=1): the paged scatter microbenchmark — 64 sequences, 8192 tokens
(lengths U[32,256] rescaled to 8192), K and V [8192, 2, 64] bf16 N(0,1) for
each of 24 layers, block size 16, a 65536-block pool, seeded random block
tables. One step = one all-layer scatter of the batch (one kernel launch);
value = algorithmic GB/s = (2 x payload + slot bytes) / time. Steps rotate
over 4 independently seeded batches with disjoint destination blocks
(805 MB touched per rotation, 201 MB per step, L2 = 126 MB), so no step
finds its inputs or outputs in L2.

Also reported on the same line: e2e (same metric through the public API with
the step's K/V and slot mapping copied from pinned host memory each step and
the status word read back), the contiguous->paged handoff of 32 prompts of
U[512,2048] tokens (us per sequence), the decode append (us per step), the
prefix fork with copy-on-write, the roofline of the scatter kernel and the
CPU baseline (the C oracle on this host's cores).

Under torchrun (N>1) every rank owns its own GPU, pool and seeded batches:
the headline config-2 batch is replicated per rank (weak scaling, no
data-path collective); the timed region is bracketed by a barrier and device
synchronisation and the max over ranks is taken.

At every N the line's extra.box carries config 5: 2,048 lognormal sequences
sharded by tokens (LPT) over the N ranks, total work fixed (strong scaling),
step = prefill scatter + 128 decode appends as one CUDA graph per rank. At
even N, extra.disagg carries the disaggregated push: ranks [0, N/2) prefill
config 5 and push the finished blocks over NVLink to rank + N/2, which runs
the appends. Both report bit_exact from a parity check of a seeded sample of
sequences on every rank against the oracle, made after the timed regions.

--impl reference times the reference algorithm on the host CPU (the C
restatement in oracle/, all host threads) on the same workload; the
reference itself is pure Python/torch and cannot be installed on the GPU box.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

L, H, D, BS = 24, 2, 64, 16
TOKEN_LAYER_BYTES = 2 * H * D * 2  # K+V of one token in one layer, bf16: 512 B
TOKEN_BYTES = L * TOKEN_LAYER_BYTES  # 12,288 B
METRIC = "KV-cache scatter/handoff GB/s vs HBM peak; handoff µs per seq at 1–8 B200"


# ---------------------------------------------------------------------------
# workloads (seeded; shared with the full-size tests)
# ---------------------------------------------------------------------------


def config2_lengths(seed: int, n_seqs: int = 64, total: int = 8192) -> np.ndarray:
    """Lengths U[32,256], rescaled so they sum to exactly `total`."""
    rng = np.random.default_rng(seed)
    raw = rng.integers(32, 257, size=n_seqs).astype(np.float64)
    lens = np.floor(raw * total / raw.sum()).astype(np.int64)
    lens[: total - int(lens.sum())] += 1
    return lens


def config2_batch(seed: int, block_offset: int = 0, num_blocks: int = 65536):
    """Slots and host K/V for one config-2 batch.

    Block tables are consecutive slices of one seeded permutation of the pool,
    starting at block_offset (so batches with different offsets never share a
    destination block).
    """
    lens = config2_lengths(seed)
    perm = np.random.default_rng(12345).permutation(num_blocks)
    nblk = -(-lens // BS)
    slots, cur = [], block_offset
    for n, nb in zip(lens, nblk):
        ids = perm[cur : cur + nb]
        pos = np.arange(n)
        slots.append(ids[pos // BS] * BS + pos % BS)
        cur += nb
    slots = np.concatenate(slots).astype(np.int64)
    g = torch.Generator().manual_seed(seed)
    T = int(lens.sum())
    k = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(L, T, H, D, generator=g).to(torch.bfloat16)
    return lens, slots, k, v, cur - block_offset


def config3_lengths(seed: int = 3, n: int = 32) -> np.ndarray:
    return np.random.default_rng(seed).integers(512, 2049, size=n).astype(np.int64)


def scatter_bytes(n_tokens: int, layers: int = L) -> int:
    """Algorithmic bytes of one scatter: read + write of every token-layer, plus 8 B of slot per token."""
    return 2 * n_tokens * layers * TOKEN_LAYER_BYTES + 8 * n_tokens


# ---------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------


class ClockSampler:
    """SM clock and throttle reasons sampled around the timed region.

    An `nvidia-smi -lms` child process samples every 20 ms with timestamps,
    outside this interpreter, so a busy launch loop holding the GIL cannot
    starve it. Only samples inside the window between mark_start() and
    mark_end() count; for a region shorter than the sampling period, the ones
    nearest to it count. Start the sampler before warm-up so the child is
    running when the timed region begins. Without nvidia-smi, a thread polls
    NVML instead.
    """

    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80, "applications_clocks_setting": 0x2,
    }

    def __init__(self, device_index: int, period_s: float = 0.002) -> None:
        self.samples: list[tuple[float, int, int]] = []  # (time, SM MHz, reason mask)
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period_s
        self._proc = None
        self._nv = None
        self._window = None
        self._t0 = None
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self._idx = int(vis.split(",")[device_index]) if vis else device_index
        try:
            import pynvml

            pynvml.nvmlInit()
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self._idx)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML missing: nvidia-smi alone, or no clocks
            pass
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self) -> None:
        nv = self._nv
        self.samples.append((time.time(), nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM),
                             nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)))

    def _run(self) -> None:
        while not self._stop.is_set():
            self._sample()
            time.sleep(self._period)

    def start(self) -> "ClockSampler":
        import shutil
        import subprocess

        smi = shutil.which("nvidia-smi")
        if smi is not None:
            self._proc = subprocess.Popen(
                [smi, "-i", str(self._idx),
                 "--query-gpu=timestamp,clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            import atexit

            atexit.register(self._reap)  # an error before stop() must not leave the child running
        elif self._nv is not None:
            self._t.start()
        return self

    def _reap(self) -> None:
        if self._proc is not None and self._proc.poll() is None:
            self._proc.terminate()

    def mark_start(self) -> None:
        self._t0 = time.time()

    def mark_end(self) -> None:
        self._window = (self._t0 if self._t0 is not None else time.time(), time.time())

    def stop(self) -> None:
        import datetime

        if self._proc is not None:
            self._proc.terminate()  # the child this sampler started, by its own handle
            out, _ = self._proc.communicate(timeout=30)
            for line in out.splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) != 4:
                    continue
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    self.samples.append((ts, int(parts[1]), int(parts[3], 16)))
                    self.max_mhz = self.max_mhz or int(parts[2])
                except ValueError:
                    continue
        elif self._nv is not None:
            self._stop.set()
            self._t.join()
        if not self.samples and self._nv is not None:
            self._sample()

    def __enter__(self):
        self.start()
        self.mark_start()
        return self

    def __exit__(self, *exc) -> None:
        self.mark_end()
        self.stop()

    def _in_window(self) -> list[tuple[float, int, int]]:
        if self._window is None or not self.samples:
            return self.samples
        t0, t1 = self._window
        inside = [x for x in self.samples if t0 - 0.005 <= x[0] <= t1 + 0.005]
        if inside:
            return inside
        return sorted(self.samples, key=lambda x: min(abs(x[0] - t0), abs(x[0] - t1)))[:3]

    def summary(self) -> dict:
        sel = self._in_window()
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["clock sampling unavailable"]}
        reasons = sorted({name for _, _, m in sel for name, bit in self.REASONS.items() if m & bit})
        return {"sm_mhz": int(statistics.median(x[1] for x in sel)), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sel)}


def load_peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic(kernel: str, workload: str):
    """Per-launch DRAM bytes from the committed ncu summary (profiles/traffic.txt), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 3 and parts[0] == kernel and parts[1] == workload:
                return int(float(parts[2]))
    except OSError:
        pass
    return None


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(x: float, world: int, device) -> list[float]:
    """Every rank's value, in rank order (an all-gather every rank takes part in)."""
    if world == 1:
        return [x]
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def barrier(world: int, device) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[device.index])
    torch.cuda.synchronize(device)


# ---------------------------------------------------------------------------
# CPU baseline (oracle on host cores)
# ---------------------------------------------------------------------------


def cpu_scatter_passes(seconds: float, min_passes: int = 2, threads: int | None = None):
    """Time full config-2 scatters with the C oracle; returns (GB/s, passes, threads, per-pass s)."""
    from oracle import kv_oracle

    threads = threads or kv_oracle.max_threads()
    lens, slots, k, v, _ = config2_batch(seed=0)
    pool_k = torch.empty(L, 65536, H, BS, D, dtype=torch.bfloat16)  # 6 GiB virtual, touched sparsely
    pool_v = torch.empty_like(pool_k)
    kv_oracle.scatter_slots(k, v, slots, pool_k, pool_v, BS, threads=threads)  # first touch
    n, t0 = 0, time.perf_counter()
    while True:
        kv_oracle.scatter_slots(k, v, slots, pool_k, pool_v, BS, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if n >= min_passes and el >= seconds:
            break
    return scatter_bytes(int(lens.sum())) * n / el / 1e9, n, threads, el / n


def cpu_copy_runs(src_k, src_v, dst_k, dst_v, runs, n_bytes: int, seconds: float = 1.0) -> dict:
    """The same row runs copied on the host by the C oracle (the reference's copy as
    per-row memcpy, all host threads), over host copies of the caches; bounded to about
    `seconds` of work after one pass that touches the destination."""
    from oracle import kv_oracle

    threads = kv_oracle.max_threads()
    r = runs.cpu().numpy() if isinstance(runs, torch.Tensor) else np.asarray(runs)
    kv_oracle.copy_runs(src_k, src_v, dst_k, dst_v, r, threads)
    n, t0 = 0, time.perf_counter()
    while True:
        kv_oracle.copy_runs(src_k, src_v, dst_k, dst_v, r, threads)
        n += 1
        el = time.perf_counter() - t0
        if n >= 2 and el >= seconds:
            break
    return {"cpu_ms": round(el / n * 1e3, 3), "cpu_GBps": round(n_bytes * n / el / 1e9, 2), "cpu_threads": threads,
            "cpu_kind": "port (C oracle copy_runs)"}


def _host_layer(pool, layer: int):
    """One layer of a device pool copied to the host, as [1, blocks, heads, rows, dim]."""
    return pool.keys[layer : layer + 1].cpu(), pool.values[layer : layer + 1].cpu()


def cpu_paged_attention(pool, tables, q_host, n_q: int, layer: int, sample: int | None = None) -> dict:
    """Attention of sequences over their paged K/V on the host, as the reference runs its
    paged branch one sequence at a time (augur/attention.py:72-86): read_paged_kv, the GQA
    repeat, q k^T / sqrt(D), masked float32 softmax, P V, by the oracle's torch restatement on
    all host threads. q_host holds n_q query tokens per sequence, sequence-major. With
    `sample`, the first `sample` sequences are timed and the layer's time is scaled by
    sequences."""
    from oracle import kv_oracle

    hk, hv = _host_layer(pool, layer)
    seqs = len(tables) if sample is None else min(sample, len(tables))
    t0 = time.perf_counter()
    for b in range(seqs):
        t = tables[b]
        kk, vv = kv_oracle.read_paged_kv(hk, hv, 0, kv_oracle.RefBlockTable(t.block_ids, BS, t.seq_len))
        q = q_host[b * n_q : (b + 1) * n_q].transpose(0, 1).unsqueeze(0)  # [1, Hq, n_q, D]
        if n_q == 1:
            kv_oracle.decode_attention(q, kk, vv)
        else:
            kv_oracle.prefill_attention(q, kk, vv)
    el = time.perf_counter() - t0
    per_layer = el * len(tables) / seqs
    return {"cpu_ms_per_layer": round(per_layer * 1e3, 2), "cpu_threads": torch.get_num_threads(),
            "cpu_sample": f"{seqs} of {len(tables)} sequences, one layer", "cpu_kind": "port (oracle, torch on host)"}


def cpu_rope_write_layer(q_host, k_host, v_host, pos_host, slots_host, theta: float, n_layers: int = 2) -> dict:
    """The reference's RoPE write on the host per layer: angles and cos / sin from the
    positions, x * cos + rotate_half(x) * sin for q and k in the dtype (augur/rope.py:29-40,
    torch on all host threads), then write_paged_kv of k and v through the slots (the C port
    with all host threads); `n_layers` layers timed."""
    from oracle import kv_oracle

    T = k_host.shape[1]
    hk = torch.empty(1, int(slots_host.max()) // BS + 1, H, BS, D, dtype=k_host.dtype)
    hv = torch.empty_like(hk)
    threads = kv_oracle.max_threads()
    t0 = time.perf_counter()
    for layer in range(n_layers):
        inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
        fr = pos_host.to(torch.float32).unsqueeze(-1) * inv
        emb = torch.cat((fr, fr), dim=-1)
        c, s_ = emb.cos().unsqueeze(1).to(k_host.dtype), emb.sin().unsqueeze(1).to(k_host.dtype)
        x, y = q_host[layer], k_host[layer]
        _ = x * c + torch.cat((-x[..., D // 2 :], x[..., : D // 2]), dim=-1) * s_
        ke = y * c + torch.cat((-y[..., D // 2 :], y[..., : D // 2]), dim=-1) * s_
        kv_oracle.scatter_slots(ke.unsqueeze(0), v_host[layer].unsqueeze(0), slots_host, hk, hv, BS, threads=threads)
    el = time.perf_counter() - t0
    return {"cpu_us_per_layer": round(el / n_layers * 1e6, 1), "cpu_threads": threads,
            "cpu_sample": f"{n_layers} of {L} layers, {T} tokens", "cpu_kind": "port (torch ops + C scatter on host)"}


def cpu_reference_torch_loop(n_seqs: int = 8, threads: int | None = None) -> dict:
    """The reference's own CPU path for the prefill scatter, timed on this host: its
    per-token torch loop (augur/paged_kv_cache.py:188-192, restated in the oracle because
    the reference package is not installed here) over the first `n_seqs` sequences of the
    config-2 batch, every layer, one write_paged_kv call per (sequence, layer)."""
    from oracle import kv_oracle

    threads = threads or (os.cpu_count() or 1)
    torch.set_num_threads(threads)
    lens, _, k, v, _ = config2_batch(seed=0)
    lens = lens[:n_seqs]
    pk = torch.zeros(L, 4096, H, BS, D, dtype=torch.bfloat16)
    pv = torch.zeros_like(pk)
    alloc = kv_oracle.RefBlockAllocator(4096)
    t0, pos0 = time.perf_counter(), 0
    for n in lens:
        n = int(n)
        table = kv_oracle.RefBlockTable([], BS)
        pos = torch.arange(n).unsqueeze(0)
        for layer in range(L):
            key = k[layer, pos0 : pos0 + n].permute(1, 0, 2).unsqueeze(0)  # [1, H, n, D] view, as attention passes it
            val = v[layer, pos0 : pos0 + n].permute(1, 0, 2).unsqueeze(0)
            kv_oracle.write_paged_kv_torch_loop(pk, pv, alloc, layer, table, pos, key, val)
        pos0 += n
    el = time.perf_counter() - t0
    tl = int(lens.sum()) * L
    return {"token_layers_per_s": round(tl / el, 1), "us_per_token_layer": round(el / tl * 1e6, 3),
            "GBps": round(tl * 2 * TOKEN_LAYER_BYTES / el / 1e9, 5), "threads": threads,
            "sample": f"first {n_seqs} config-2 sequences ({int(lens.sum())} tokens) x {L} layers, one "
                      "write_paged_kv per (sequence, layer): the reference's per-token torch loop"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------


def run_ours(args, world: int, rank: int, local: int) -> dict | None:
    import augur_b200 as ab
    from augur_b200 import _lib, _ops, batched

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    n_sets = 4
    # --small (profiling only): an 8192-block pool instead of 65536; every
    # launch moves the same bytes, the device holds 1.9 GB instead of 13 GB.
    nblocks = 8192 if args.small else 65536
    pool = ab.PagedKVCache(keys=torch.empty(L, nblocks, H, BS, D, dtype=torch.bfloat16, device=device),
                           values=torch.empty(L, nblocks, H, BS, D, dtype=torch.bfloat16, device=device),
                           block_size=BS, allocator=ab.BlockAllocator(nblocks))
    sets, offset = [], 0
    host_sets = []
    for s in range(n_sets):
        lens, slots, k, v, used = config2_batch(seed=1000 * rank + s, block_offset=offset, num_blocks=nblocks)
        offset += used
        host_sets.append((slots, k, v))
        sets.append((torch.from_numpy(slots).to(device), k.to(device), v.to(device)))
    T = int(sets[0][0].shape[0])
    step_bytes = scatter_bytes(T)

    def step(i: int, stream=None) -> None:
        sl, k, v = sets[i % n_sets]
        batched.write_paged_kv_batch(pool, k, v, sl, stream=stream)

    # warm-up (eager), then capture one rotation in a CUDA graph
    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    cap_stream = torch.cuda.Stream(device)
    cap_stream.wait_stream(torch.cuda.current_stream(device))
    launches_before = _ops.launch_count
    with torch.cuda.graph(graph, stream=cap_stream):
        for i in range(n_sets):
            step(i)
    launches_per_replay = _ops.launch_count - launches_before
    clocks = ClockSampler(local).start()  # running before the timed region begins
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize(device)

    K = args.steps
    replays, rem = divmod(K, n_sets)
    rem_graph = None
    if rem:
        rem_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(rem_graph, stream=cap_stream):
            for i in range(rem):
                step(i)
        rem_graph.replay()
    torch.cuda.synchronize(device)

    barrier(world, device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark_start()
    start.record()
    for _ in range(replays):
        graph.replay()
    if rem_graph is not None:
        rem_graph.replay()
    end.record()
    torch.cuda.synchronize(device)
    clocks.mark_end()
    clocks.stop()
    ms = start.elapsed_time(end)
    barrier(world, device)
    ms_max = max_over_ranks(ms, world, device)
    gpu_launches = replays * launches_per_replay + (rem if rem_graph is not None else 0)
    value = world * step_bytes * K / (ms_max / 1e3) / 1e9
    per_launch_s = (ms / 1e3) / K
    achieved = step_bytes / per_launch_s / 1e9
    status = _ops.read_status(device)
    if status != _lib.OK:
        raise RuntimeError(f"device status {status} after the timed region")

    # ---- e2e: public API, pinned host inputs copied every step, status read back
    pinned = [(torch.from_numpy(s).pin_memory(), k.pin_memory(), v.pin_memory()) for s, k, v in host_sets]
    # Two device input buffers: a copy stream moves step i + 1's inputs over
    # PCIe while the compute stream scatters step i (events order the reuse).
    comp = torch.cuda.current_stream(device)
    copy_stream = torch.cuda.Stream(device)
    dev_bufs = [tuple(torch.empty_like(x) for x in sets[0]) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    status_word = _ops.status_word(device)
    status_host = torch.empty(1, dtype=torch.int32).pin_memory()
    e2e_steps = max(3, min(K, 40))

    def e2e_step(i: int) -> None:
        j = i % 2
        hs, hk, hv = pinned[i % n_sets]
        ds, dk, dv = dev_bufs[j]
        with torch.cuda.stream(copy_stream):
            if i >= 2:
                copy_stream.wait_event(freed[j])  # step i - 2 has scattered out of this buffer
            ds.copy_(hs, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            copied[j].record(copy_stream)
        comp.wait_event(copied[j])
        batched.write_paged_kv_batch(pool, dk, dv, ds)
        freed[j].record(comp)
        status_host.copy_(status_word, non_blocking=True)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize(device)
    barrier(world, device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    copy_stream.wait_stream(comp)  # no copy of the timed steps starts before e0
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record(comp)
    torch.cuda.synchronize(device)
    own_ms = e0.elapsed_time(e1)
    e2e_ms = max_over_ranks(own_ms, world, device)
    if int(status_host.item()) != _lib.OK:
        raise RuntimeError("device status error in the e2e region")
    h2d = int(sets[0][0].numel() * 8 + sets[0][1].numel() * 2 * 2)
    # the same host-to-device copies alone (no scatter), every rank at once: the
    # rate the host link gives this rank while all ranks copy
    barrier(world, device)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(copy_stream):
        c0.record(copy_stream)
        for i in range(e2e_steps):
            hs, hk, hv = pinned[i % n_sets]
            ds, dk, dv = dev_bufs[i % 2]
            ds.copy_(hs, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
        c1.record(copy_stream)
    torch.cuda.synchronize(device)
    copy_gbs = h2d * e2e_steps / (c0.elapsed_time(c1) / 1e3) / 1e9
    e2e_h2d_gbs = gather_over_ranks(h2d * e2e_steps / (own_ms / 1e3) / 1e9, world, device)
    copy_only_gbs = gather_over_ranks(copy_gbs, world, device)
    frac = min(a / b for a, b in zip(e2e_h2d_gbs, copy_only_gbs))
    e2e = {"value": round(world * step_bytes * e2e_steps / (e2e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "steps": e2e_steps,
           "path": "augur_b200.batched.write_paged_kv_batch (ctypes -> augur_kv_scatter)",
           "pipeline": "pinned host -> device on a copy stream into two device buffers, overlapping the "
                       "previous step's scatter; status read back every step",
           "h2d_GBps_per_rank": [round(x, 1) for x in e2e_h2d_gbs],
           "h2d_copy_only_GBps_per_rank": [round(x, 1) for x in copy_only_gbs],
           "bound": ("host-to-device copies: each rank's e2e moves its inputs at "
                     f"{100 * frac:.0f} % or more of the rate the same copies reach alone"
                     if frac >= 0.85 else
                     f"not the host link: e2e copies run at {100 * frac:.0f} % of the copy-only rate")}
    del pinned, dev_bufs
    graph.reset()
    if rem_graph is not None:
        rem_graph.reset()
    del sets

    extra = {}
    if not args.skip_extras:
        extra = run_extras(device, cpu=world == 1 and not args.skip_cpu)  # host legs on one GPU runs only
    del pool
    torch.cuda.empty_cache()
    if not args.skip_scaleout:
        # the multi-GPU workloads, every rank taking part: config 5
        # sharded over the ranks (strong scaling) and, at even N, the
        # disaggregated push; both checked against the oracle on every rank
        box = box_phase(world, rank, local)
        if rank == 0:
            extra["box"] = box
        if world >= 2 and world % 2 == 0:
            dis = disagg_phase(world, rank, local)
            if rank == 0:
                extra["disagg"] = dis

    if rank != 0:
        return None
    peak, peak_kind = load_peaks()
    roofline = {
        "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
        "frac": round(achieved / peak, 4), "peak_source": f"hbm_gbs of {peak_kind}",
        "traffic": load_traffic("scatter_rows_kernel", "config2"),
        "algorithmic_bytes_per_launch": step_bytes, "kernel": "scatter_rows_kernel<16,32,8>",
        "launch_us": round(per_launch_s * 1e6, 2),
    }
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms_max / K, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V, seeded block tables)",
        "config": {"workload": "paged scatter: 64 seqs / 8192 tokens x 24 layers, 2 KV heads x 64, "
                               "block 16, 65536-block pool (config 2)",
                   "tokens_per_step": T, "bytes_per_step": step_bytes,
                   "l2": "4 rotating seeded batches with disjoint blocks: 805 MB touched per rotation > 126 MB L2",
                   "parallelism": f"replicated per rank (weak scaling): each of the {world} GPU(s) scatters "
                                  "its own config-2 batch into its own pool; config 5 sharded over the "
                                  "ranks (strong scaling) is extra.box",
                   "timed": "CUDA graph replays of one launch per step, CUDA events"},
        "e2e": e2e, "gpu_launches": gpu_launches, "roofline": roofline, "clocks": clocks.summary(),
        "extra": extra,
    }
    if world == 1 and not args.skip_cpu:
        gbs, passes, threads, per = cpu_scatter_passes(args.cpu_seconds)
        line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                                "sample": f"{passes} full config-2 scatters (8192 tokens x 24 layers), "
                                          f"{per * 1e3:.1f} ms each, C oracle with {threads} threads"}
        line["extra"]["cpu_reference_torch_loop"] = cpu_reference_torch_loop()
    return line


def bench_decode_attention(device, pool, tables, early_reads: bool = True, cpu: bool = False) -> dict:
    """paged_decode_attention for every layer of one decode step, graph-captured, L2 cold.

    Algorithmic bytes: every cached K and V row of every sequence read once
    (24 layers x sum(seq_len) x 512 B) plus the queries and outputs.
    early_reads: each layer's launch reads lengths, tables and its K/V rows while the
    previous layer's launch drains (the kernel ahead of it writes none of them).
    The same graph without early reads is timed beside it.
    """
    from augur_b200.attention import DecodeTables, paged_decode_attention

    B = len(tables)
    Hq = 14
    dt = DecodeTables(tables, device)
    g = torch.Generator(device=device).manual_seed(5)
    qs = torch.randn(L, B, Hq, D, generator=g, device=device).to(torch.bfloat16)
    outs = torch.empty_like(qs)

    def step() -> None:
        for layer in range(L):
            paged_decode_attention(qs[layer], pool, layer, dt, out=outs[layer], early_reads=early_reads)

    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(device)
    cs.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cs):  # warm-up on the capture stream sizes its workspace outside the capture
        step()
    torch.cuda.synchronize(device)
    with torch.cuda.graph(graph, stream=cs):
        step()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    times = []
    for _ in range(7):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize(device)
        times.append(a.elapsed_time(b))
    graph.reset()
    ms = statistics.median(times[2:])
    tokens = int(sum(t.seq_len for t in tables))
    kv_bytes = L * tokens * TOKEN_LAYER_BYTES + 2 * qs.numel() * 2
    peak, kind = load_peaks()
    gbs = kv_bytes / (ms / 1e3) / 1e9
    res = {"us_per_step_all_layers": round(ms * 1e3, 2), "us_per_layer": round(ms * 1e3 / L, 2),
           "seqs": B, "cached_tokens": tokens, "GBps": round(gbs, 1), "frac_of_hbm_peak": round(gbs / peak, 4),
           "early_reads": early_reads, "kernel": "attn_decode_split_kernel<bf16,64>",
           "timed": "CUDA graph of 24 per-layer launches, L2 flushed"}
    if early_reads:
        res["us_per_layer_without_early_reads"] = bench_decode_attention(device, pool, tables, False)["us_per_layer"]
    if cpu:
        res.update(cpu_paged_attention(pool, tables, qs[0].cpu(), 1, 0))
        res["gpu_over_cpu"] = round(res["cpu_ms_per_layer"] * 1e3 / res["us_per_layer"], 1)
    return res


def bench_rope(device, pool, reps: int = 7, cpu: bool = False) -> dict:
    """RoPE fused with the paged write for a config-2-sized prefill (8,192 tokens, one layer per
    launch, all 24 layers), against the same math as separate torch ops plus the scatter.

    Algorithmic bytes per token and layer: q read + rotated q written (2 x 14 x 64 x 2 B),
    K and V read and written (2 x 512 B), two cos/sin table rows (2 x 64 B), position and
    slot (16 B) = 4,752 B.
    """
    from augur_b200 import batched
    from augur_b200.rope import rope_tables, write_paged_kv_batch_rope

    T, Hq, theta = 8192, 14, 1000000.0
    g = torch.Generator(device=device).manual_seed(11)
    rng = np.random.default_rng(11)
    lens = config2_lengths(0)
    pos = torch.from_numpy(np.concatenate([np.arange(n) for n in lens]).astype(np.int64)).to(device)
    nslots = pool.keys.shape[1] * BS
    slots = torch.from_numpy(rng.permutation(nslots)[:T].astype(np.int64)).to(device)
    q = torch.randn(L, T, Hq, D, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(L, T, H, D, generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(L, T, H, D, generator=g, device=device).to(torch.bfloat16)
    cos, sin = rope_tables(D, theta, torch.bfloat16, int(lens.max()), device)
    maxp = int(lens.max()) - 1

    def fused() -> None:
        for layer in range(L):
            write_paged_kv_batch_rope(pool, q[layer], k[layer], v[layer], slots, pos, theta, layer, max_position=maxp)

    def unfused() -> None:  # the reference's elementwise ops (augur/rope.py:38-39), then the scatter
        c = torch.cat((cos[pos], cos[pos]), dim=-1).unsqueeze(1)
        s_ = torch.cat((sin[pos], sin[pos]), dim=-1).unsqueeze(1)
        for layer in range(L):
            x, y = q[layer], k[layer]
            rq = torch.cat((-x[..., D // 2:], x[..., : D // 2]), dim=-1)
            ry = torch.cat((-y[..., D // 2:], y[..., : D // 2]), dim=-1)
            _ = x * c + rq * s_
            ke = y * c + ry * s_
            batched.write_paged_kv_batch(pool, ke, v[layer], slots, layer_idx=layer)

    res = {}
    for name, fn in (("fused", fused), ("torch_ops_then_scatter", unfused)):
        fn()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream(device)
        cs.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(cs):
            fn()
        torch.cuda.synchronize(device)
        with torch.cuda.graph(graph, stream=cs):
            fn()
        times = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            torch.cuda.synchronize(device)
            times.append(a.elapsed_time(b))
        graph.reset()
        res[name] = statistics.median(times[2:]) * 1e3 / L
    nbytes = T * 4752
    peak, _ = load_peaks()
    gbs = nbytes / (res["fused"] / 1e6) / 1e9
    out = {"us_per_layer_fused": round(res["fused"], 2),
           "us_per_layer_torch_ops_then_scatter": round(res["torch_ops_then_scatter"], 2),
           "tokens": T, "GBps_fused": round(gbs, 1), "frac_of_hbm_peak": round(gbs / peak, 4),
           "timed": "CUDA graph of 24 per-layer launches; q, k, v of all layers (450 MB) exceed L2"}
    if cpu:
        c = cpu_rope_write_layer(q[:2].cpu(), k[:2].cpu(), v[:2].cpu(), pos.cpu(), slots.cpu().numpy(), theta)
        out.update(c)
        out["gpu_over_cpu"] = round(c["cpu_us_per_layer"] / res["fused"], 1)
    return out


def bench_decode_step(device, pool, tables) -> dict:
    """The KV side of one decode step for the config-3 batch (32 sequences) across 24 layers:
    per layer the fused RoPE append and the decode attention (paged_decode_layer), on copies
    of the block tables. Device time from a CUDA graph of the 48 launches (L2 flushed
    before each replay); the step including its host work (DecodeStep: table growth, slot
    mapping, uploads) timed eagerly.
    """
    import augur_b200 as ab
    from augur_b200 import _ops
    from augur_b200.decode import DecodeGraphStep, DecodeStep, paged_decode_layer

    Hq, theta = 14, 1000000.0
    tabs = [ab.SequenceBlockTable(block_ids=list(t.block_ids), block_size=t.block_size, seq_len=t.seq_len)
            for t in tables]
    B = len(tabs)
    g = torch.Generator(device=device).manual_seed(17)
    q = torch.randn(L, B, Hq, 1, D, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(L, B, H, 1, D, generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(L, B, H, 1, D, generator=g, device=device).to(torch.bfloat16)
    step = DecodeStep(pool, tabs, early_reads=True)  # the kernel ahead of each layer is the previous layer's

    def layers(st) -> None:
        for layer in range(L):
            paged_decode_layer(st, pool, layer, q[layer], k[layer], v[layer], theta)

    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(device)
    cs.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cs):
        layers(step)
    torch.cuda.synchronize(device)
    launches_before = _ops.launch_count
    with torch.cuda.graph(graph, stream=cs):
        layers(step)
    launches_per_step = _ops.launch_count - launches_before
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    times = []
    for _ in range(7):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize(device)
        times.append(a.elapsed_time(b))
    graph.reset()
    dev_ms = statistics.median(times[2:])
    # the same step's attention alone (same tables and lengths, q already rotated): the
    # difference is what the RoPE append costs inside the fused launch
    from augur_b200.attention import paged_decode_attention

    qr = q[:, :, :, 0].contiguous()
    outs = torch.empty_like(qr)
    agraph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cs):
        for layer in range(L):
            paged_decode_attention(qr[layer], pool, layer, step.tables, out=outs[layer], early_reads=True)
    torch.cuda.synchronize(device)
    with torch.cuda.graph(agraph, stream=cs):
        for layer in range(L):
            paged_decode_attention(qr[layer], pool, layer, step.tables, out=outs[layer], early_reads=True)
    atimes = []
    for _ in range(7):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        agraph.replay()
        b.record()
        torch.cuda.synchronize(device)
        atimes.append(a.elapsed_time(b))
    agraph.reset()
    att_ms = statistics.median(atimes[2:])
    host = []
    for _ in range(5):  # real steps: every table grows by one token per step
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        layers(DecodeStep(pool, tabs, early_reads=True))
        torch.cuda.synchronize(device)
        host.append(time.perf_counter() - t0)
    # the same steps replayed from one captured graph (DecodeGraphStep): per step the host
    # grows the tables and refreshes the step's buffers, then the 48 launches replay
    max_blocks = max(len(t.block_ids) for t in tabs) + 4
    gstep = DecodeGraphStep(pool, B, max_blocks, Hq, theta, early_reads=True)
    gs = torch.cuda.Stream(device)
    gs.wait_stream(torch.cuda.current_stream(device))
    ggraph = torch.cuda.CUDAGraph()
    replay = []
    with torch.cuda.stream(gs):
        gstep.update(tabs)
        with torch.cuda.graph(ggraph, stream=gs):
            for layer in range(L):
                gstep.layer(layer, q[layer], k[layer], v[layer])
        ggraph.replay()
        for _ in range(5):
            torch.cuda.synchronize(device)
            t0 = time.perf_counter()
            gstep.update(tabs)
            ggraph.replay()
            torch.cuda.synchronize(device)
            replay.append(time.perf_counter() - t0)
    ggraph.reset()
    tokens = int(sum(t.seq_len for t in tabs))
    return {"seqs": B, "cached_tokens_after": tokens, "launches_per_step": launches_per_step,
            "us_per_step_device": round(dev_ms * 1e3, 1), "us_per_layer_device": round(dev_ms * 1e3 / L, 2),
            "us_per_layer_attention_alone": round(att_ms * 1e3 / L, 2),
            "append_in_fused_us_per_layer": round((dev_ms - att_ms) * 1e3 / L, 2),
            "us_per_step_with_host": round(statistics.median(host) * 1e6, 1),
            "us_per_step_graph_with_host": round(statistics.median(replay) * 1e6, 1),
            "timed": "per layer: decode attention with the RoPE append fused into it; device: CUDA graph, L2 flushed; "
                     "with host: eager DecodeStep, and DecodeGraphStep update + graph replay"}


def bench_decode_attention_large(device, n_seqs: int = 256) -> dict:
    """Decode attention at a serving-sized batch: the first n_seqs config-5 (box) lengths
    (lognormal, median 1024, 64..8192 tokens), random blocks of a pool sized to them, random
    K/V; one decode step over all 24 layers in a CUDA graph, L2 flushed before each replay.
    Same algorithmic bytes as the small case: every cached K/V row once plus q and out.
    """
    from augur_b200 import sharding
    from augur_b200.attention import DecodeTables, paged_decode_attention

    import augur_b200 as ab

    lens = sharding.box_lengths()[:n_seqs]
    nblk = -(-lens // BS)
    NB = int(nblk.sum()) + 64
    g = torch.Generator(device=device).manual_seed(21)
    keys = torch.randn(L, NB, H, BS, D, generator=g, device=device).to(torch.bfloat16)
    values = torch.randn(L, NB, H, BS, D, generator=g, device=device).to(torch.bfloat16)
    pool = ab.PagedKVCache(keys=keys, values=values, block_size=BS, allocator=ab.BlockAllocator(NB))
    perm = np.random.default_rng(21).permutation(NB)
    tables, cur = [], 0
    for n, nb in zip(lens, nblk):
        tables.append(ab.SequenceBlockTable(block_ids=perm[cur : cur + nb].tolist(), block_size=BS, seq_len=int(n)))
        cur += nb
    res = bench_decode_attention(device, pool, tables)
    res.pop("timed", None)
    res["timed"] = "CUDA graph of 24 per-layer launches, L2 flushed"
    del pool, keys, values
    return res


def bench_offload(device, pool, tables, n_seqs: int = 16) -> dict:
    """Offload n_seqs config-3 sequences (all layers, K and V) to pinned host memory and restore
    them, both paths, against a copy-engine copy of the same byte count.

    Bytes per direction = tokens x 12,288 B. The host link bounds both ways;
    the copy-engine figure (torch copy_ of one contiguous device slab to
    pinned memory and back) is its practical ceiling on this box.
    """
    from augur_b200.offload import host_buffer, offload_blocks, restore_blocks

    tabs = tables[:n_seqs]
    ids, rows = [], []
    for t in tabs:
        n = -(-t.seq_len // BS)
        ids += t.block_ids[:n]
        rows += [min(BS, t.seq_len - j * BS) for j in range(n)]
    tokens = int(sum(rows))
    nbytes = tokens * TOKEN_BYTES
    hk, hv = host_buffer(pool, len(ids))
    dst = list(range(len(ids)))  # restore target blocks (their contents are scratch here)

    def timed(fn, reps=5):
        fn()
        torch.cuda.synchronize(device)
        times = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize(device)
            times.append(a.elapsed_time(b))
        return statistics.median(times)

    res = {}
    for path in ("staged", "direct"):
        res[f"offload_{path}"] = timed(lambda: offload_blocks(pool, ids, rows, out=(hk, hv), path=path).done.synchronize())
        host = offload_blocks(pool, ids, rows, out=(hk, hv), path=path)
        res[f"restore_{path}"] = timed(lambda: restore_blocks(pool, host, dst, path=path))
    slab = pool.keys.view(-1)[: nbytes // pool.keys.element_size()]
    hslab = torch.empty(slab.shape, dtype=slab.dtype, pin_memory=True)
    t_d2h = timed(lambda: hslab.copy_(slab, non_blocking=True))
    t_h2d = timed(lambda: slab.copy_(hslab, non_blocking=True))
    gb = lambda ms: round(nbytes / (ms / 1e3) / 1e9, 2)  # noqa: E731
    out = {"seqs": len(tabs), "tokens": tokens, "MB": round(nbytes / 1e6, 1)}
    for k, ms in res.items():
        out[f"{k}_GBps"] = gb(ms)
    out.update({"copy_engine_d2h_GBps": gb(t_d2h), "copy_engine_h2d_GBps": gb(t_h2d),
                "timed": "staged: SM gather/scatter via 16 MB HBM chunks + copy engine; direct: one run-copy "
                         "launch on pinned memory; median of 5, pinned host buffers reused"})
    return out


def bench_prefill_attention(device, pool, tables, suffix: int, flush, kernel: str = "auto",
                            cpu: bool = False) -> dict:
    """Suffix prefill attention over shared prefixes (config 4: 256 forks of one prefix, each
    with its own suffix already written): every layer, the suffix queries of all forks attend
    to their prefix and causally to their suffix, one paged_prefill_attention launch per layer,
    replayed from a CUDA graph with L2 flushed before each replay.

    Algorithmic bytes: each sequence's cached K/V read once (seq_len x 512 B per layer) plus q
    and the output; FLOPs: 4 x head_dim per (query head, query token, visible key)."""
    from augur_b200.attention import DecodeTables, PrefillQueries, paged_prefill_attention

    Hq = 14
    B = len(tables)
    dt = DecodeTables(tables, device)
    lens = PrefillQueries([suffix] * B, device)
    g = torch.Generator(device=device).manual_seed(41)
    q = torch.randn(B * suffix, Hq, D, generator=g, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)

    def step() -> None:
        for layer in range(L):
            paged_prefill_attention(q, pool, layer, dt, lens, out=out, kernel=kernel)

    cs = torch.cuda.Stream(device)
    cs.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cs):
        step()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cs):
        step()
    times = []
    for _ in range(5):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize(device)
        times.append(a.elapsed_time(b))
    graph.reset()
    ms = statistics.median(times[1:]) / L
    seq = [t.seq_len for t in tables]
    kv_bytes = sum(seq) * TOKEN_LAYER_BYTES + 2 * q.numel() * 2
    flops = sum(4 * D * Hq * sum(n - suffix + i + 1 for i in range(suffix)) for n in seq)
    peak, kind = load_peaks()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tf_peak, tf_kind = float(json.load(f)["bf16_tflops"]), "bf16_tflops (burst) of measured"
    except Exception:
        tf_peak, tf_kind = 1590.0, "fallback"
    tflops = flops / (ms / 1e3) / 1e12
    res = {"seqs": B, "suffix_tokens": suffix, "cached_tokens_per_seq": seq[0], "us_per_layer": round(ms * 1e3, 2),
           "kv_GBps": round(kv_bytes / (ms / 1e3) / 1e9, 1), "kv_frac_of_hbm_peak": round(kv_bytes / (ms / 1e3) / 1e9 / peak, 4),
           "TFLOPs": round(tflops, 1), "tensor_frac": round(tflops / tf_peak, 4), "tensor_peak_source": tf_kind,
           "kernel": ("attn_prefill_mma_kernel<bf16,64> (mma.sync)" if kernel == "mma_sync"
                      else "attn_prefill_umma_kernel<bf16,64> (tcgen05, TMEM accumulators)"),
           "timed": "CUDA graph of 24 per-layer launches, L2 flushed; the forks share the prefix's blocks"}
    if cpu:
        res.update(cpu_paged_attention(pool, tables, q.cpu(), suffix, 0, sample=8))
        res["gpu_over_cpu"] = round(res["cpu_ms_per_layer"] * 1e3 / res["us_per_layer"], 1)
    return res


def run_prefill_attention_only(device) -> dict:
    """Profiling case: config 4's 1,024-token prefix forked 256 ways with 128-token
    suffixes (a 8,192-block pool, 1.6 GB), then the suffix prefill attention."""
    import augur_b200 as ab
    from augur_b200 import batched

    NB = 8192
    pool = ab.PagedKVCache(keys=torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=device),
                           values=torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=device),
                           block_size=BS, allocator=ab.BlockAllocator(NB))
    g = torch.Generator(device=device).manual_seed(4)
    parent = ab.SequenceBlockTable.empty(BS)
    sm = batched.prefill_slot_mapping([parent], [1024], pool.allocator)[0]
    pk = torch.randn(L, 1024, H, D, generator=g, device=device).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, pk, pk, torch.from_numpy(sm).to(device))
    forks = batched.fork_prefix(pool, parent, 256)
    suffix = batched.prefill_slot_mapping(forks, [128] * 256, pool.allocator, start_positions=[1024] * 256)
    sk = torch.randn(L, 256 * 128, H, D, generator=g, device=device).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, sk, sk, torch.from_numpy(suffix.reshape(-1)).to(device))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    return {"suffix_prefill_attention": bench_prefill_attention(device, pool, forks, 128, flush),
            "suffix_prefill_attention_mma_sync": bench_prefill_attention(device, pool, forks, 128, flush,
                                                                         kernel="mma_sync")}


def run_cow_only(device) -> dict:
    """Profiling case: config 4's 1,000-token prefix (62 full blocks + 8 rows) forked 256
    ways, the copy-on-write of its partial last block, then the COW launch timed alone."""
    import augur_b200 as ab
    from augur_b200 import batched

    NB = 8192
    pool = ab.PagedKVCache(keys=torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=device),
                           values=torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=device),
                           block_size=BS, allocator=ab.BlockAllocator(NB))
    g = torch.Generator(device=device).manual_seed(4)
    parent = ab.SequenceBlockTable.empty(BS)
    sm = batched.prefill_slot_mapping([parent], [1000], pool.allocator)[0]
    pk = torch.randn(L, 1000, H, D, generator=g, device=device).to(torch.bfloat16)
    batched.write_paged_kv_batch(pool, pk, pk, torch.from_numpy(sm).to(device))
    forks = batched.fork_prefix(pool, parent, 256)
    copied = batched.cow_partial_blocks(pool, forks)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    return {"cow_blocks": copied, **bench_cow_device(device, pool, parent, forks, 1000, flush)}


def bench_cow_device(device, pool, parent, forks, prefix_len: int, flush, cpu: bool = False) -> dict:
    """The copy-on-write launch alone: the parent's partial block copied into every fork's
    private block (all layers, K and V), replayed from a CUDA graph with L2 flushed before
    each replay. Algorithmic bytes: every copied row read once and written once (the
    copies all read the same source block, so DRAM reads are far fewer)."""
    from augur_b200 import batched

    j, r = prefix_len // BS, prefix_len % BS
    runs = np.zeros((len(forks), 5), dtype=np.int64)
    runs[:, 0] = parent.block_ids[j]
    runs[:, 2] = [f.block_ids[j] for f in forks]
    runs[:, 4] = r
    max_rows = min(batched._run_max_rows(pool.keys, BS), r)  # as copy_blocks bounds them
    runs_t = batched._to_device_runs(batched.split_runs(runs, max_rows), device)

    def cow() -> None:
        batched.copy_runs_between(pool.keys, pool.values, "paged", pool.keys, pool.values, "paged", runs_t,
                                  max_rows)

    cow()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(device)
    cs.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.graph(graph, stream=cs):
        cow()
    times = []
    for _ in range(9):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize(device)
        times.append(a.elapsed_time(b))
    graph.reset()
    ms = statistics.median(times[2:])
    nbytes = 2 * len(forks) * r * L * TOKEN_LAYER_BYTES + runs_t.numel() * 4
    peak, kind = load_peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    res = {"cow_us_device": round(ms * 1e3, 2), "cow_bytes": nbytes, "cow_GBps_device": round(gbs, 1),
           "cow_frac_of_hbm_peak": round(gbs / peak, 4), "cow_kernel": "copy_runs_vec_kernel<16>",
           "cow_timed": "CUDA graph of the one copy launch, L2 flushed before each replay"}
    if cpu:  # the same runs on a host pool of the same shape (the copied rows hold the device's values)
        hk = torch.empty(pool.keys.shape, dtype=pool.keys.dtype)
        hv = torch.empty_like(hk)
        hk[:, parent.block_ids[j]] = pool.keys[:, parent.block_ids[j]].cpu()
        hv[:, parent.block_ids[j]] = pool.values[:, parent.block_ids[j]].cpu()
        c = cpu_copy_runs(hk, hv, hk, hv, runs_t, nbytes)
        res.update({"cow_" + k: v for k, v in c.items()})
        res["cow_gpu_over_cpu"] = round(c["cpu_ms"] / (ms or 1e-9), 1)
        del hk, hv
    return res


def run_extras(device, handoff_only: bool = False, attention_only: bool = False, rope_only: bool = False,
               offload_only: bool = False, cpu: bool = False) -> dict:
    """Config 3 handoff + decode append and config 4 fork/COW, timed with CUDA events."""
    import augur_b200 as ab
    from augur_b200 import _lib, _ops, batched

    out = {}
    # ---- config 3: contiguous -> paged handoff of 32 prompts, then 256 decode appends
    lens = config3_lengths()
    B, Lmax = len(lens), int(lens.max())
    g = torch.Generator(device=device).manual_seed(3)
    src = ab.KVCache(keys=torch.randn(L, B, H, Lmax, D, generator=g, device=device).to(torch.bfloat16),
                     values=torch.randn(L, B, H, Lmax, D, generator=g, device=device).to(torch.bfloat16))
    NB = 8192
    perm = np.random.default_rng(33).permutation(NB)
    tables, cur = [], 0
    for n in lens:
        nb = -(-int(n) // BS) + 256 // BS + 1
        tables.append(ab.SequenceBlockTable(block_ids=perm[cur : cur + nb].tolist(), block_size=BS))
        cur += nb
    pool = ab.PagedKVCache(keys=torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=device),
                           values=torch.empty(L, NB, H, BS, D, dtype=torch.bfloat16, device=device),
                           block_size=BS, allocator=ab.BlockAllocator(NB))
    runs = batched.handoff_contiguous_to_paged(src, pool, tables, lens)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    tok = int(lens.sum())
    hbytes = 2 * tok * TOKEN_BYTES + runs.numel() * 4
    for name, flags in (("bulk", _lib.COPY_BULK), ("vector", _lib.COPY_VECTOR)):
        times = []
        for _ in range(7):
            flush.fill_(1)  # evict L2 between repetitions
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            batched.copy_runs_between(src.keys, src.values, "contiguous", pool.keys, pool.values, "paged",
                                      runs, BS, flags=flags)
            b.record()
            torch.cuda.synchronize(device)
            times.append(a.elapsed_time(b))
        ms = statistics.median(times[2:])
        out[f"handoff_{name}"] = {"us_per_seq": round(ms * 1e3 / B, 3), "ms": round(ms, 4),
                                  "GBps": round(hbytes / (ms / 1e3) / 1e9, 1), "seqs": B, "tokens": tok}
    if cpu:  # the same runs from a host copy of the contiguous caches into a host pool
        sk, sv = src.keys.cpu(), src.values.cpu()
        hk = torch.empty(pool.keys.shape, dtype=pool.keys.dtype)
        hv = torch.empty_like(hk)
        c = cpu_copy_runs(sk, sv, hk, hv, runs, hbytes)
        c["cpu_us_per_seq"] = round(c["cpu_ms"] * 1e3 / B, 2)
        c["gpu_over_cpu"] = round(c["cpu_ms"] / out["handoff_vector"]["ms"], 1)
        out["handoff_vector"].update(c)
        del sk, sv, hk, hv
    if handoff_only:
        return out
    # decode append: 256 steps of one token per sequence, all layers, captured in one graph
    for t, n in zip(tables, lens):
        t.seq_len = int(n)
    steps = 256
    slot_rows = []
    for _ in range(steps):
        slot_rows.append(batched.decode_slot_mapping(tables, pool.allocator))
    slot_t = torch.from_numpy(np.stack(slot_rows)).to(device)
    nk = torch.randn(steps, L, B, H, D, generator=g, device=device).to(torch.bfloat16)
    nv = torch.randn(steps, L, B, H, D, generator=g, device=device).to(torch.bfloat16)
    for s in range(3):
        batched.append_decode(pool, None, nk[s], nv[s], slot_mapping=slot_t[s])
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(device)
    cs.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.graph(graph, stream=cs):
        for s in range(steps):
            batched.append_decode(pool, None, nk[s], nv[s], slot_mapping=slot_t[s])
    graph.replay()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b)
    abytes = scatter_bytes(B)
    peak, _ = load_peaks()
    out["decode_append"] = {"us_per_step": round(ms * 1e3 / steps, 3), "steps": steps, "seqs": B,
                            "GBps": round(abytes * steps / (ms / 1e3) / 1e9, 1),
                            "frac_of_hbm_peak": round(abytes * steps / (ms / 1e3) / 1e9 / peak, 4),
                            "hbm_floor_us": round(abytes / peak / 1e3, 3),
                            "timed": "one CUDA graph of 256 append launches (one launch per step, all layers)"}
    if cpu:  # one step on the host: the C port's write_paged_kv of the 32 tokens, all layers, one thread
        from oracle import kv_oracle

        hk = torch.empty(pool.keys.shape, dtype=pool.keys.dtype)
        hv = torch.empty_like(hk)
        sk, sv, sl = nk[0].cpu(), nv[0].cpu(), slot_t[0].cpu().numpy()
        kv_oracle.scatter_slots(sk, sv, sl, hk, hv, BS, threads=1)
        n, t0 = 0, time.perf_counter()
        while n < 200 or time.perf_counter() - t0 < 0.3:
            kv_oracle.scatter_slots(sk, sv, sl, hk, hv, BS, threads=1)
            n += 1
        cpu_us = (time.perf_counter() - t0) / n * 1e6
        out["decode_append"].update({"cpu_us_per_step": round(cpu_us, 2), "cpu_threads": 1,
                                     "cpu_kind": "port (C oracle scatter)",
                                     "gpu_over_cpu": round(cpu_us / out["decode_append"]["us_per_step"], 1)})
        del hk, hv
    graph.reset()
    del src, nk, nv

    # ---- decode attention reading the pool in place: one decode step of the
    # 32 sequences (each n + 256 tokens long now) across all 24 layers
    if not (rope_only or offload_only):
        out["decode_attention"] = bench_decode_attention(device, pool, tables, cpu=cpu)
        out["decode_attention_256_seqs"] = bench_decode_attention_large(device)
        out["decode_step"] = bench_decode_step(device, pool, tables)
    if attention_only:
        return out
    if not rope_only:
        # ---- offload to pinned host memory and restore (before the RoPE bench reuses the pool)
        out["host_offload"] = bench_offload(device, pool, tables)
        if offload_only:
            return out
    # ---- RoPE fused with the paged write, config-2-sized prefill, all layers
    out["rope_scatter"] = bench_rope(device, pool, cpu=cpu)
    if rope_only:
        return out

    # ---- config 4: 1000-token prefix (62 full blocks + 8 rows) forked 256 ways, COW, 128-token suffix
    for prefix_len in (1024, 1000):
        alloc = ab.BlockAllocator(NB)
        pool4 = ab.PagedKVCache(keys=pool.keys, values=pool.values, block_size=BS, allocator=alloc)
        parent = ab.SequenceBlockTable.empty(BS)
        sm = batched.prefill_slot_mapping([parent], [prefix_len], alloc)[0]
        pk = torch.randn(L, prefix_len, H, D, generator=g, device=device).to(torch.bfloat16)
        batched.write_paged_kv_batch(pool4, pk, pk, torch.from_numpy(sm).to(device))
        forks = batched.fork_prefix(pool4, parent, 256)
        torch.cuda.synchronize(device)
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record()
        copied = batched.cow_partial_blocks(pool4, forks)
        b.record()
        suffix_sm = batched.prefill_slot_mapping(forks, [128] * 256, alloc,
                                                 start_positions=[prefix_len] * 256).reshape(-1)
        sk = torch.randn(L, 256 * 128, H, D, generator=g, device=device).to(torch.bfloat16)
        sm_t = torch.from_numpy(suffix_sm).to(device)
        torch.cuda.synchronize(device)
        c0 = torch.cuda.Event(enable_timing=True)
        c0.record()
        batched.write_paged_kv_batch(pool4, sk, sk, sm_t)
        c.record()
        torch.cuda.synchronize(device)
        entry = {"forks": 256, "cow_blocks": copied, "cow_ms_incl_host": round(a.elapsed_time(b), 4),
                 "suffix_GBps": round(scatter_bytes(256 * 128) / (c0.elapsed_time(c) / 1e3) / 1e9, 1)}
        if copied:
            entry.update(bench_cow_device(device, pool4, parent, forks, prefix_len, flush, cpu=cpu))
        else:
            out["suffix_prefill_attention"] = bench_prefill_attention(device, pool4, forks, 128, flush, cpu=cpu)
            out["suffix_prefill_attention_mma_sync"] = bench_prefill_attention(device, pool4, forks, 128, flush,
                                                                               kernel="mma_sync")
        out[f"prefix_fork_{prefix_len}"] = entry
        del sk, pk
    if _ops.read_status(device) != _lib.OK:
        raise RuntimeError("device status error in the extra workloads")
    del pool
    return out


# ---------------------------------------------------------------------------
# box scale-out (config 5) and the disaggregated push, with a parity check
# ---------------------------------------------------------------------------

BOX_APPENDS = 128
NVLINK_NOMINAL_GBS = 900.0  # per direction per GPU (NVLink 5), the disaggregated mode's roofline
NVLINK_POOL_PEER_COPY_GBS = 770.0  # copy-engine peer copy per direction measured on these B200s


def box_sequence_kv(index: int, n: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """K and V [layers, n, heads, dim] of box sequence `index`: N(0,1) bf16 from a per-sequence
    seed, so a sequence holds the same values on whichever rank (and GPU) generates it."""
    g = torch.Generator(device=device)
    g.manual_seed(50_000 + int(index))
    k = torch.randn(L, int(n), H, D, generator=g, device=device, dtype=torch.bfloat16)
    v = torch.randn(L, int(n), H, D, generator=g, device=device, dtype=torch.bfloat16)
    return k, v


def oracle_check_sequences(pool, samples: list[dict]) -> tuple[bool, int]:
    """Parity check, outside every timed region: the oracle's scatter (the reference's
    write_paged_kv, augur/paged_kv_cache.py:188-192, restated in C) of each sampled
    sequence's prefill tokens and appended tokens, through the same slots, into a
    0xFF-poisoned host pool of just those sequences' blocks, against the device pool's
    copies of the same blocks, bit for bit (the device pool was poisoned the same way,
    so untouched rows compare too). Returns (equal, tokens checked)."""
    from oracle import kv_oracle

    ids = np.concatenate([np.asarray(x["ids"], dtype=np.int64) for x in samples])
    if np.unique(ids).size != ids.size:
        raise RuntimeError("sampled sequences share blocks")
    compact = np.full(int(ids.max()) + 1, -1, dtype=np.int64)
    compact[ids] = np.arange(ids.size)

    def remap(slots: np.ndarray) -> np.ndarray:
        return compact[slots // BS] * BS + slots % BS

    hk = kv_oracle.poison_(torch.empty(L, ids.size, H, BS, D, dtype=torch.bfloat16))
    hv = kv_oracle.poison_(torch.empty_like(hk))
    tokens = 0
    for x in samples:
        kv_oracle.scatter_slots(x["k"], x["v"], remap(x["pre"]), hk, hv, BS)
        tokens += x["pre"].size
        if "app" in x:  # appended tokens, written after the prefill
            kv_oracle.scatter_slots(x["ak"], x["av"], remap(x["app"]), hk, hv, BS)
            tokens += x["app"].size
    idx = torch.from_numpy(ids).to(pool.keys.device)
    dk = pool.keys.index_select(1, idx).cpu()
    dv = pool.values.index_select(1, idx).cpu()
    ok = torch.equal(kv_oracle.bits(dk), kv_oracle.bits(hk)) and torch.equal(kv_oracle.bits(dv), kv_oracle.bits(hv))
    return bool(ok), tokens


def _sample_local(lens: np.ndarray, rank: int, n: int = 8) -> list[int]:
    """Seeded sample of local sequence indices: n at random plus the longest."""
    rng = np.random.default_rng(777 + rank)
    pick = set(rng.choice(len(lens), size=min(n, len(lens)), replace=False).tolist())
    pick.add(int(np.argmax(lens)))
    return sorted(pick)


def _append_inputs(n_seqs: int, seed: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    nk = torch.randn(BOX_APPENDS, L, n_seqs, H, D, generator=g, device=device, dtype=torch.bfloat16)
    nv = torch.randn(BOX_APPENDS, L, n_seqs, H, D, generator=g, device=device, dtype=torch.bfloat16)
    return nk, nv


def _time_graph(graph, reps: int, device) -> float:
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize(device)
    return a.elapsed_time(b) / reps


def _gather(obj, world: int):
    if world == 1:
        return [obj]
    import torch.distributed as dist

    out: list = [None] * world
    dist.all_gather_object(out, obj)
    return out


def box_phase(world: int, rank: int, local: int, steps: int = 10, warmup: int = 3,
              n_seqs: int = 2048) -> dict | None:
    """Config 5 on `world` GPUs: 2,048 lognormal sequences LPT-sharded by tokens, each rank with
    its own pool sized to its shard plus 128 appends; step = prefill scatter of the shard +
    128 decode appends, captured in one CUDA graph (129 launches). Total work is fixed
    (strong scaling). Every rank checks a seeded sample of its sequences against the oracle."""
    import augur_b200 as ab
    from augur_b200 import _lib, _ops, batched, sharding

    device = torch.device("cuda", local)
    lens_all = sharding.box_lengths(n_seqs=n_seqs)
    mine = sharding.lpt_assign(lens_all, world)[rank]
    lens = lens_all[mine]
    B, T = len(lens), int(lens.sum())
    nblk = int(sum(-(-(int(n) + BOX_APPENDS) // BS) for n in lens))
    pool = ab.PagedKVCache(keys=torch.empty(L, nblk, H, BS, D, dtype=torch.bfloat16, device=device),
                           values=torch.empty(L, nblk, H, BS, D, dtype=torch.bfloat16, device=device),
                           block_size=BS, allocator=ab.BlockAllocator(nblk))
    pool.keys.view(torch.uint8).fill_(0xFF)  # poison: rows nothing writes compare in the parity check
    pool.values.view(torch.uint8).fill_(0xFF)
    k = torch.empty(L, T, H, D, dtype=torch.bfloat16, device=device)
    v = torch.empty_like(k)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    for j, (i, n) in enumerate(zip(mine, lens)):
        sk, sv = box_sequence_kv(i, n, device)
        k[:, offs[j] : offs[j + 1]].copy_(sk)
        v[:, offs[j] : offs[j + 1]].copy_(sv)
    del sk, sv
    nk, nv = _append_inputs(B, 60_000 + rank, device)
    tables = [ab.SequenceBlockTable.empty(BS) for _ in lens]
    sm = batched.prefill_slot_mapping(tables, lens, pool.allocator)
    pre = [sm[b, : int(n)].copy() for b, n in enumerate(lens)]
    flat = torch.from_numpy(np.concatenate(pre)).to(device)
    del sm
    dec_np = np.stack([batched.decode_slot_mapping(tables, pool.allocator) for _ in range(BOX_APPENDS)])
    dec = torch.from_numpy(dec_np).to(device)

    def scatter() -> None:
        batched.write_paged_kv_batch(pool, k, v, flat)

    def appends() -> None:
        for s in range(BOX_APPENDS):
            batched.append_decode(pool, None, nk[s], nv[s], slot_mapping=dec[s])

    scatter()
    appends()
    torch.cuda.synchronize(device)
    cs = torch.cuda.Stream(device)
    cs.wait_stream(torch.cuda.current_stream(device))
    graphs = {}
    for name, fns in (("step", (scatter, appends)), ("scatter", (scatter,)), ("appends", (appends,))):
        gr = torch.cuda.CUDAGraph()
        n0 = _ops.launch_count
        with torch.cuda.graph(gr, stream=cs):
            for fn in fns:
                fn()
        graphs[name] = (gr, _ops.launch_count - n0)
    for _ in range(warmup):
        graphs["step"][0].replay()
    torch.cuda.synchronize(device)
    barrier(world, device)
    with ClockSampler(local) as clocks:
        ms_step = _time_graph(graphs["step"][0], steps, device)
    barrier(world, device)
    ms_scatter = _time_graph(graphs["scatter"][0], steps, device)
    ms_app = _time_graph(graphs["appends"][0], steps, device)
    if _ops.read_status(device) != _lib.OK:
        raise RuntimeError("device status error in the box workload")
    for gr, _ in graphs.values():
        gr.reset()
    # parity: a seeded sample of this rank's sequences against the oracle
    samples = []
    for b in _sample_local(lens, rank):
        sl = slice(int(offs[b]), int(offs[b + 1]))
        samples.append({"ids": list(tables[b].block_ids), "k": k[:, sl].cpu(), "v": v[:, sl].cpu(),
                        "pre": pre[b], "ak": nk[:, :, b].permute(1, 0, 2, 3).contiguous().cpu(),
                        "av": nv[:, :, b].permute(1, 0, 2, 3).contiguous().cpu(), "app": dec_np[:, b].copy()})
    ok, checked = oracle_check_sequences(pool, samples)
    bytes_rank = scatter_bytes(T) + BOX_APPENDS * scatter_bytes(B)
    mine_out = {"rank": rank, "seqs": B, "tokens": T, "ms_step": ms_step, "ms_scatter": ms_scatter,
                "ms_appends": ms_app, "bytes": bytes_rank, "bit_exact": ok, "checked_seqs": len(samples),
                "checked_tokens": checked}
    del k, v, nk, nv, pool, flat, dec, samples
    torch.cuda.empty_cache()
    reports = _gather(mine_out, world)
    if rank != 0:
        return None
    peak, peak_kind = load_peaks()
    job_ms = max(r["ms_step"] for r in reports)
    total_bytes = sum(r["bytes"] for r in reports)
    scatter_job_ms = max(r["ms_scatter"] for r in reports)
    per_rank = [{"rank": r["rank"], "seqs": r["seqs"], "tokens": r["tokens"],
                 "ms_step": round(r["ms_step"], 4), "ms_scatter": round(r["ms_scatter"], 4),
                 "ms_appends": round(r["ms_appends"], 4),
                 "GBps": round(r["bytes"] / (r["ms_step"] / 1e3) / 1e9, 1),
                 "frac_of_hbm_peak": round(r["bytes"] / (r["ms_step"] / 1e3) / 1e9 / peak, 4),
                 "us_per_seq_scatter": round(r["ms_scatter"] * 1e3 / max(1, r["seqs"]), 3),
                 "bit_exact": r["bit_exact"], "checked_seqs": r["checked_seqs"]} for r in reports]
    tokens = [r["tokens"] for r in reports]
    return {
        "workload": f"config 5: {n_seqs} seqs, lognormal(ln 1024, 0.8) clipped [64, 8192], "
                    f"{int(lens_all.sum())} tokens, LPT-sharded by tokens over {world} GPU(s), one pool "
                    f"per GPU; step = prefill scatter of each shard + {BOX_APPENDS} decode appends "
                    "(one CUDA graph of 129 launches per rank)",
        "scaling": "strong", "n_gpus": world, "steps": steps, "warmup": warmup,
        "bytes_per_step": total_bytes,
        "aggregate_GBps": round(total_bytes / (job_ms / 1e3) / 1e9, 1),
        "ms_per_step": round(job_ms, 4),
        "scatter_ms_job": round(scatter_job_ms, 4),
        "handoff_us_per_seq": round(scatter_job_ms * 1e3 / n_seqs, 4),
        "appends_us_per_step_job": round(max(r["ms_appends"] for r in reports) * 1e3 / BOX_APPENDS, 3),
        "token_imbalance": round(max(tokens) / (sum(tokens) / len(tokens)), 4),
        "roofline": {"bound": "hbm", "unit": "GB/s per GPU", "peak": peak, "peak_source": f"hbm_gbs of {peak_kind}",
                     "achieved_min_rank": min(x["GBps"] for x in per_rank),
                     "frac_min_rank": min(x["frac_of_hbm_peak"] for x in per_rank)},
        "bit_exact": all(r["bit_exact"] for r in reports),
        "parity": "every rank: a seeded sample of its sequences (8 + its longest) scattered by the oracle "
                  "(C restatement of write_paged_kv) through the same slots into a poisoned host pool, "
                  "compared bit for bit with the device pool's blocks after the timed steps",
        "gpu_launches_per_step": graphs["step"][1], "clocks_rank0": clocks.summary(),
        "per_rank": per_rank,
    }


def disagg_phase(world: int, rank: int, local: int, steps: int = 5, warmup: int = 3,
                 n_seqs: int = 2048) -> dict | None:
    """Disaggregated config 5: ranks [0, N/2) prefill the 2,048 sequences (LPT-sharded over the
    prefill ranks) into local staging pools and push the finished blocks to rank + N/2 over
    NVLink (plain 16-byte peer stores; no TMA, no multicast); each decode rank then runs the
    128 appends. Timed: the push (prefill ranks), the appends (decode ranks). Every decode rank
    checks a seeded sample of its sequences against the oracle."""
    import torch.distributed as dist

    import augur_b200 as ab
    from augur_b200 import _lib, _ops, batched, peer, sharding

    device = torch.device("cuda", local)
    half = world // 2
    prefill = rank < half
    pair = rank % half
    partner = rank + half if prefill else rank - half
    lens_all = sharding.box_lengths(n_seqs=n_seqs)
    mine = sharding.lpt_assign(lens_all, half)[pair]
    lens = lens_all[mine]
    B, T = len(lens), int(lens.sum())
    payload = T * TOKEN_BYTES
    mine_out: dict = {"rank": rank, "role": "prefill" if prefill else "decode", "seqs": B, "tokens": T}
    exported = None
    if prefill:
        nblk = int(sum(-(-int(n) // BS) for n in lens))
        pool = ab.PagedKVCache(keys=torch.empty(L, nblk, H, BS, D, dtype=torch.bfloat16, device=device),
                               values=torch.empty(L, nblk, H, BS, D, dtype=torch.bfloat16, device=device),
                               block_size=BS, allocator=ab.BlockAllocator(nblk))
        k = torch.empty(L, T, H, D, dtype=torch.bfloat16, device=device)
        v = torch.empty_like(k)
        offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        for j, (i, n) in enumerate(zip(mine, lens)):
            sk, sv = box_sequence_kv(i, n, device)
            k[:, offs[j] : offs[j + 1]].copy_(sk)
            v[:, offs[j] : offs[j + 1]].copy_(sv)
        del sk, sv
        tables = [ab.SequenceBlockTable.empty(BS) for _ in lens]
        sm = batched.prefill_slot_mapping(tables, lens, pool.allocator)
        flat = torch.from_numpy(np.concatenate([sm[b, : int(n)] for b, n in enumerate(lens)])).to(device)
        del sm
        batched.write_paged_kv_batch(pool, k, v, flat)  # the staging pool the push reads
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        batched.write_paged_kv_batch(pool, k, v, flat)
        b.record()
        torch.cuda.synchronize(device)
        mine_out["ms_prefill_scatter"] = a.elapsed_time(b)
        del k, v, flat
    else:
        spare = 17  # the decode pool already serves other sequences: destination ids differ from the source's
        nblk = int(sum(-(-(int(n) + BOX_APPENDS) // BS) for n in lens)) + spare
        pool = ab.PagedKVCache(keys=torch.empty(L, nblk, H, BS, D, dtype=torch.bfloat16, device=device),
                               values=torch.empty(L, nblk, H, BS, D, dtype=torch.bfloat16, device=device),
                               block_size=BS, allocator=ab.BlockAllocator(nblk))
        pool.keys.view(torch.uint8).fill_(0xFF)
        pool.values.view(torch.uint8).fill_(0xFF)
        pool.allocator.allocate_many(spare)
        tables = [ab.SequenceBlockTable.empty(BS) for _ in lens]
        sm = batched.prefill_slot_mapping(tables, lens, pool.allocator)
        pre = [sm[b, : int(n)].copy() for b, n in enumerate(lens)]
        del sm
        torch.cuda.synchronize(device)
        exported = (peer.export_pool(pool), [list(t.block_ids) for t in tables])
    objs: list = [None] * world
    dist.all_gather_object(objs, exported)
    if prefill:
        ex, dst_ids = objs[partner]
        remote = peer.open_pool(ex, device)
        runs = []
        for t, ids, n in zip(tables, dst_ids, lens):
            nb = -(-int(n) // BS)
            r = np.zeros((nb, 5), dtype=np.int64)
            r[:, 0] = t.block_ids[:nb]
            r[:, 2] = ids[:nb]
            r[:, 4] = np.minimum(BS, int(n) - BS * np.arange(nb))
            runs.append(r)
        prep = peer.prepare_push(pool, remote, np.concatenate(runs))
        assert prep.payload_bytes == payload
        for _ in range(warmup):
            peer.push_prepared(prep)
        torch.cuda.synchronize(device)
    barrier(world, device)
    if prefill:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            a.record()
            for _ in range(steps):
                peer.push_prepared(prep)
            b.record()
            torch.cuda.synchronize(device)
        mine_out["ms_push"] = a.elapsed_time(b) / steps
        mine_out["clocks"] = clocks.summary()
        mine_out["launches"] = steps
        if _ops.read_status(device) != _lib.OK:
            raise RuntimeError("device status error during the push")
    barrier(world, device)  # every push has landed before any decode rank appends
    if prefill:
        remote.close()
        del prep
    else:
        nk, nv = _append_inputs(B, 70_000 + rank, device)
        dec_np = np.stack([batched.decode_slot_mapping(tables, pool.allocator) for _ in range(BOX_APPENDS)])
        dec = torch.from_numpy(dec_np).to(device)
        gr = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream(device)
        cs.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.graph(gr, stream=cs):
            for s in range(BOX_APPENDS):
                batched.append_decode(pool, None, nk[s], nv[s], slot_mapping=dec[s])
        mine_out["ms_appends"] = _time_graph(gr, steps, device)
        gr.reset()
        if _ops.read_status(device) != _lib.OK:
            raise RuntimeError("device status error in the decode appends")
        samples = []
        for b in _sample_local(lens, rank):
            sk, sv = box_sequence_kv(mine[b], lens[b], device)  # the prefill rank's values, by seed
            samples.append({"ids": list(tables[b].block_ids), "k": sk.cpu(), "v": sv.cpu(), "pre": pre[b],
                            "ak": nk[:, :, b].permute(1, 0, 2, 3).contiguous().cpu(),
                            "av": nv[:, :, b].permute(1, 0, 2, 3).contiguous().cpu(),
                            "app": dec_np[:, b].copy()})
        ok, checked = oracle_check_sequences(pool, samples)
        mine_out.update(bit_exact=ok, checked_seqs=len(samples), checked_tokens=checked)
        del nk, nv, dec, samples
    barrier(world, device)  # the prefill ranks have closed their mappings of the decode pools
    del pool
    torch.cuda.empty_cache()
    reports = _gather(mine_out, world)
    if rank != 0:
        return None
    pre_r = [r for r in reports if r["role"] == "prefill"]
    dec_r = [r for r in reports if r["role"] == "decode"]
    push_ms = max(r["ms_push"] for r in pre_r)
    total_payload = sum(r["tokens"] for r in pre_r) * TOKEN_BYTES
    per_pair = [{"pair": f"{r['rank']}->{r['rank'] + half}", "seqs": r["seqs"], "tokens": r["tokens"],
                 "ms_push": round(r["ms_push"], 4),
                 "GBps": round(r["tokens"] * TOKEN_BYTES / (r["ms_push"] / 1e3) / 1e9, 1),
                 "us_per_seq": round(r["ms_push"] * 1e3 / max(1, r["seqs"]), 3),
                 "ms_prefill_scatter": round(r["ms_prefill_scatter"], 4)} for r in pre_r]
    worst = min(p["GBps"] for p in per_pair)
    return {
        "workload": f"config 5 disaggregated: {n_seqs} seqs ({int(lens_all.sum())} tokens) LPT-sharded over "
                    f"{half} prefill GPU(s); each prefill GPU i pushes its finished blocks (every layer, K and "
                    f"V, partial last blocks by their rows) into decode GPU i + {half}'s pool, which then runs "
                    f"{BOX_APPENDS} appends",
        "n_gpus": world, "pairs": half, "steps": steps, "warmup": warmup,
        "payload_bytes_per_push": total_payload,
        "aggregate_push_GBps": round(total_payload / (push_ms / 1e3) / 1e9, 1),
        "ms_per_push_job": round(push_ms, 4),
        "handoff_us_per_seq": round(push_ms * 1e3 / n_seqs, 4),
        "roofline": {"bound": "nvlink", "unit": "GB/s per direction per GPU", "achieved_min_pair": worst,
                     "peak": NVLINK_NOMINAL_GBS, "frac_min_pair": round(worst / NVLINK_NOMINAL_GBS, 4),
                     "peak_source": "NVLink 5 nominal per direction (900 GB/s)",
                     "frac_of_pool_peer_copy": round(worst / NVLINK_POOL_PEER_COPY_GBS, 4),
                     "pool_peer_copy_GBps": NVLINK_POOL_PEER_COPY_GBS},
        "appends_us_per_step_job": round(max(r["ms_appends"] for r in dec_r) * 1e3 / BOX_APPENDS, 3),
        "bit_exact": all(r["bit_exact"] for r in dec_r),
        "parity": "every decode rank: a seeded sample of its sequences (8 + its longest) regenerated from "
                  "their seeds and scattered by the oracle, with the appends, into a poisoned host pool, "
                  "compared bit for bit with the decode pool's blocks after the pushes and appends",
        "clocks_rank0": reports[0].get("clocks"),
        "per_pair": per_pair,
    }


def run_phase(args, world: int, rank: int, local: int) -> dict | None:
    """--workload box | disagg alone: the phase's result as the line's body."""
    torch.cuda.set_device(local)
    if args.workload == "box":
        out = box_phase(world, rank, local, steps=args.steps, warmup=args.warmup, n_seqs=args.box_seqs)
    else:
        if world < 2 or world % 2:
            raise SystemExit("--workload disagg needs an even number of ranks >= 2")
        out = disagg_phase(world, rank, local, steps=args.steps, warmup=args.warmup, n_seqs=args.box_seqs)
    if out is None:
        return None
    return {"metric": METRIC, "workload": args.workload, "n_gpus": world, "data": "synthetic", **out}


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------


def run_reference(args, world: int, rank: int) -> dict | None:
    if rank != 0:
        return None
    from oracle import kv_oracle

    threads = kv_oracle.max_threads()
    lens, slots, k, v, _ = config2_batch(seed=0)
    pool_k = torch.empty(L, 65536, H, BS, D, dtype=torch.bfloat16)
    pool_v = torch.empty_like(pool_k)
    for _ in range(max(1, args.warmup)):
        kv_oracle.scatter_slots(k, v, slots, pool_k, pool_v, BS, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        kv_oracle.scatter_slots(k, v, slots, pool_k, pool_v, BS, threads=threads)
    el = time.perf_counter() - t0
    step_bytes = scatter_bytes(int(lens.sum()))
    gbs = step_bytes * args.steps / el / 1e9
    sample = (f"{args.steps} full config-2 scatters (8192 tokens x 24 layers) in host memory, "
              f"reference per-token write_paged_kv loop restated in C (oracle/kv_oracle.c)")
    return {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(el * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "paged scatter: 64 seqs / 8192 tokens x 24 layers, 2 KV heads x 64, "
                               "block 16, 65536-block pool (config 2)", "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_torch_loop": cpu_reference_torch_loop(),
    }


def _json_stdout():
    """Keep stdout for the one JSON line: everything else written to fd 1
    (library banners such as NCCL's version line included) goes to stderr."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def main() -> None:
    json_out = _json_stdout()

    def emit(line: dict) -> None:
        json_out.write(json.dumps(line) + "\n")
        json_out.flush()

    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 20000 for the scatter headline, 2000 for the reference arm, "
                         "20 for box, 50 for disagg)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-extras", action="store_true")
    ap.add_argument("--skip-scaleout", action="store_true",
                    help="leave out config 5 (box, strong scaling) and the disaggregated push")
    ap.add_argument("--small", action="store_true", help="profiling case: 8192-block pool, no extras/CPU")
    ap.add_argument("--handoff-only", action="store_true", help="profiling case: config-3 handoff only")
    ap.add_argument("--attention-only", action="store_true",
                    help="profiling case: config-3 cache, then decode attention over all layers")
    ap.add_argument("--attention-large-only", action="store_true",
                    help="profiling case: decode attention over 128 box-length sequences (about 2.2 GB)")
    ap.add_argument("--offload-only", action="store_true",
                    help="config-3 cache, then offload to pinned host memory and restore")
    ap.add_argument("--cow-only", action="store_true",
                    help="profiling case: config-4 fork of a 1000-token prefix, then the copy-on-write launch")
    ap.add_argument("--prefill-attention-only", action="store_true",
                    help="profiling case: config-4 forks, then the suffix prefill attention")
    ap.add_argument("--rope-only", action="store_true",
                    help="profiling case: config-3 cache, then RoPE fused with the paged write")
    ap.add_argument("--workload", choices=["scatter", "disagg", "box"], default="scatter",
                    help="scatter: headline (config 2); disagg: NVLink block push between rank pairs; "
                         "box: config 5, 2048 sequences sharded over the ranks (strong scaling)")
    ap.add_argument("--box-seqs", type=int, default=2048)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.steps is None:  # each default keeps its timed region well under a minute
        args.steps = 2000 if args.impl == "reference" else {"scatter": 20000, "box": 10, "disagg": 5}[args.workload]
    if args.small:
        args.skip_cpu = args.skip_extras = args.skip_scaleout = True
    if args.handoff_only:  # profiling case: only the config-3 handoff (about 3 GB on the device)
        torch.cuda.set_device(0)
        emit(run_extras(torch.device("cuda", 0), handoff_only=True))
        return
    if args.attention_large_only:  # profiling case: decode attention over 128 box-length sequences
        torch.cuda.set_device(0)
        emit({"decode_attention_128_seqs": bench_decode_attention_large(torch.device("cuda", 0), n_seqs=128)})
        return
    if args.offload_only:  # config-3 pool, then offload to pinned host memory and restore
        torch.cuda.set_device(0)
        emit(run_extras(torch.device("cuda", 0), offload_only=True))
        return
    if args.cow_only:  # profiling case: config-4 fork, then the copy-on-write launch
        torch.cuda.set_device(0)
        emit(run_cow_only(torch.device("cuda", 0)))
        return
    if args.prefill_attention_only:  # profiling case: config-4 forks, then the suffix prefill attention
        torch.cuda.set_device(0)
        emit(run_prefill_attention_only(torch.device("cuda", 0)))
        return
    if args.rope_only:  # profiling case: config-3 pool, then the fused RoPE + write
        torch.cuda.set_device(0)
        emit(run_extras(torch.device("cuda", 0), rope_only=True))
        return
    if args.attention_only:  # profiling case: config-3 handoff + appends, then decode attention
        torch.cuda.set_device(0)
        emit(run_extras(torch.device("cuda", 0), attention_only=True))
        return
    world, rank, local = dist_env()
    if args.impl == "reference":
        line = run_reference(args, world, rank)
        if line is not None:
            emit(line)
        return
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        if args.workload in ("disagg", "box"):
            line = run_phase(args, world, rank, local)
        else:
            line = run_ours(args, world, rank, local)
        if line is not None:
            emit(line)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
