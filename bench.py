"""Benchmark of the B200 sparse_attn_sharedkv hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2]

One step = one ``sparse_attn_sharedkv`` call (SCFA: 128-key window + top-2048
compressed keys, N1 = 128, D_qk 576 / D_v 512, bf16) over one decode batch of
the BASELINE configuration ``c2`` (B = 64, seq U[8K, 32K]) per GPU, with
synthetic seeded inputs (``dsv4_planb_b200.workloads``).  With N GPUs every
rank runs its own c2 batch (seed 42 + rank): requests are independent and are
sharded by batch with no collective on the data path ("weak" scaling).

Printed by rank 0, one JSON line:
  value        decode tokens/s of all ranks, inputs resident in HBM, each step
               replayed from a CUDA graph with L2 flushed (256 MiB write) before
               it; time = max over ranks of the summed per-step CUDA-event times
  e2e          the same metric through the public API with host buffers: per
               step, the step's inputs copied from pinned host memory, the
               call, and out + lse copied back to pinned host memory; steps
               rotate over E2E_STREAMS CUDA streams so copies overlap compute,
               and q's upload is split over E2E_COPY_STREAMS copy streams
  roofline     HBM roofline of the attention kernel (algorithmic bytes per
               launch / its CUDA-event duration vs the measured copy peak), from
               a second capture of the step with events around that kernel
  c4           (default run, N = 1) chunked prefill, 4 x 8192 tokens: step time,
               attention-kernel TFLOP/s and its fraction of the measured bf16 peak
  c5           (default run, every N) 512 mixed-length decode requests split
               across the ranks by cost (LPT), each rank holding only its shard:
               strong scaling, tokens/s over the slowest rank
  verify       (N > 1) NCCL all_gather of every rank's out / lse (c2 and c5) and of
               the inputs of sampled tokens; rank 0 checks the gathered rows against
               the fp32 oracle (outside every timed region)
  lazy_rescale the same step with SAS_FWD_FLAG_LAZY_RESCALE (the tensor-core kernel's
               performance mode: running max raised only past a threshold; not the headline)
  cpu_baseline the oracle CPU port on the same workload (rank 0, N = 1), worker
               processes over all host cores (the best of a sweep of worker counts)
``--impl reference`` times that CPU port alone on the same config and the same
seeded data (built on cuda:0 with the GPU arm's generator when a GPU is present):
the reference is Python over an NPU toolchain absent here, and its own TileLang
kernel does not implement SCFA (it raises NotImplementedError), so its golden
model, restated by the oracle, is the reference implementation of this path.
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

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402

L2_FLUSH_BYTES = 256 << 20
E2E_STREAMS = 3
E2E_COPY_STREAMS = 4
CPU_SAMPLE_TOKENS = 512  # most tokens the CPU baseline attends per step (c4 has 32768)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--kernel", default="auto", choices=["auto", "simt", "tc", "tc2"])
    ap.add_argument("--batch", type=int, default=None,
                    help="request count of c2 / c3 (default 64 / 32): small-batch decode measurements")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the c4 / c5 keys of the default run")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class ClockSampler:
    """nvidia-smi clock / throttle samples of one GPU during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def committed_traffic(workload: str, kernel_name: str):
    path = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(f"{workload}:{kernel_name}")
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------------------------------------
# workloads and the config block both arms print


def build_workload(name, rank, world, dev, batch=None):
    """``(wl, total_tokens_all_ranks, strong)``.  c5 is split across the ranks by cost (LPT over
    window + compressed keys per token), each rank building only its shard's pools and tables;
    every other config gives each rank its own batch (seed 42 + rank)."""
    from dsv4_planb_b200 import workloads as W

    if name == "c5":
        from dsv4_planb_b200 import sharding as S

        q_all, kv_all, n1, topk = W.config_lengths("c5", 42)
        mine = S.partition_requests(S.request_costs(q_all, kv_all, topk), world)[rank]
        wl = W.make_workload(name="c5[shard]", q_lens=[q_all[i] for i in mine], kv_lens=[kv_all[i] for i in mine],
                             num_heads=n1, topk=topk, seed=42 + rank, device=dev)
        return wl, sum(q_all), True
    wl = W.config_workload(name, seed=42 + rank, device=dev, batch=batch)
    return wl, wl.num_tokens * world, False


def config_block(name, world, batch, per_gpu_tokens, total_tokens, strong, split):
    from dsv4_planb_b200 import workloads as W

    return {"workload": f"{name}: {W.CONFIG_DESCRIPTIONS[name]}"
                        + (f" (batch overridden: {batch} requests)" if batch else ""),
            "global_batch": total_tokens, "per_gpu_batch": per_gpu_tokens,
            "seq_len": {"c1": "U[512,2048]", "c2": "U[8K,32K]", "c3": "U[4K,64K]", "c4": "ctx U[0,16K] + 8192",
                        "c5": "log-U[1K,128K]"}[name],
            "parallelism": (f"LPT request shards x{world}" if strong else f"request-sharded x{world}"),
            "split_tiles": split, "l2": "flushed (256 MiB write) before every step",
            "timing": "CUDA graph replay per step, CUDA events, max over ranks"}


# ---------------------------------------------------------------------------------------------
# GPU timing


def time_workload(wl, kw, steps, warmup, kernel, dev, world, dist, flush, sampler=None):
    """Time ``steps`` CUDA-graph replays of one call (L2 flushed before each) and, from a second
    capture with the library's events around the attention kernel, that kernel's duration.
    Returns ``(max-over-ranks total ms, per-step ms list, kernel ms list, out, lse)``."""
    from dsv4_planb_b200 import _lib
    from dsv4_planb_b200.api import sparse_attn_sharedkv

    q = wl.q
    T, N1, _ = q.shape
    out = torch.empty((T, N1, wl.v_head_dim), dtype=q.dtype, device=dev)
    lse = torch.empty((T, N1), dtype=torch.float32, device=dev)
    max_q = max(wl.q_lens)

    def step():
        sparse_attn_sharedkv(q, out=out, lse_out=lse, return_softmax_lse=True, kernel=kernel, max_seqlen_q=max_q,
                             **kw)

    for _ in range(max(warmup, 3)):  # eager warm-up (also sets kernel attributes before capture)
        step()
    torch.cuda.synchronize()
    k_start = torch.cuda.Event(enable_timing=True)
    k_stop = torch.cuda.Event(enable_timing=True)
    k_start.record()  # creates the underlying cudaEvent_t handles
    k_stop.record()
    lib = _lib.load()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    # Two captures of the same step: `graph` (timed for the step) holds only the op's own work;
    # `graph_ev` also records the library's events around the attention kernel (its duration for
    # the roofline).  The event nodes sit between prep and the attention kernel and would otherwise
    # serialise the programmatic launch that overlaps them.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph_ev = torch.cuda.CUDAGraph()
    lib.sas_set_kernel_events(k_start.cuda_event, k_stop.cuda_event)
    try:
        with torch.cuda.graph(graph_ev):
            step()
    finally:
        lib.sas_set_kernel_events(None, None)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    kernel_ms = []
    for _ in range(warmup):
        flush.fill_(1.0)
        graph.replay()
        flush.fill_(1.0)
        graph_ev.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    for i in range(steps):
        flush.fill_(float(i))
        starts[i].record()
        graph.replay()
        stops[i].record()
    for i in range(steps):
        flush.fill_(float(i))
        graph_ev.replay()
        k_stop.synchronize()
        kernel_ms.append(k_start.elapsed_time(k_stop))
    torch.cuda.synchronize()
    step_ms = [a.elapsed_time(b) for a, b in zip(starts, stops)]
    t = torch.tensor([sum(step_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    graph.reset()
    graph_ev.reset()
    return float(t.item()), step_ms, kernel_ms, out, lse


def time_e2e(wl, kw, steps, warmup, kernel, dev, world, dist, tokens_all):
    """End to end through the public API with host buffers (see the module docstring)."""
    from dsv4_planb_b200.api import sparse_attn_sharedkv

    # Every step copies its own inputs from pinned host memory, runs the public API call and reads
    # its out + lse back into pinned host memory.  Steps rotate over E2E_STREAMS slots (a compute
    # stream with its own device buffers), so one step's copies overlap another's compute, as a
    # serving loop would run them.  The q upload (9.4 MB at c2) is split over E2E_COPY_STREAMS copy
    # streams: one host-to-device copy of that size reaches only 13-30 GB/s on these hosts, four
    # concurrent ones 35-38 GB/s.
    q = wl.q
    T, N1, _ = q.shape
    Dv = wl.v_head_dim
    max_q = max(wl.q_lens)
    pin = lambda x: x.cpu().pin_memory()  # noqa: E731
    host = {"q": pin(q)}
    for k in ("cmp_sparse_indices", "cu_seqlens_q", "seqused_kv", "ori_block_table", "cmp_block_table", "sinks"):
        host[k] = pin(kw[k])
    streams = [torch.cuda.Stream(device=dev) for _ in range(E2E_STREAMS)]
    copy_streams = [torch.cuda.Stream(device=dev) for _ in range(E2E_COPY_STREAMS)]
    dev_in = [{k: torch.empty_like(v, device=dev) for k, v in host.items()} for _ in streams]
    dev_out = [(torch.empty((T, N1, Dv), dtype=q.dtype, device=dev),
                torch.empty((T, N1), dtype=torch.float32, device=dev)) for _ in streams]
    outs_h = [(torch.empty((T, N1, Dv), dtype=q.dtype).pin_memory(),
               torch.empty((T, N1), dtype=torch.float32).pin_memory()) for _ in streams]
    inputs_free = [None] * len(streams)  # event after the slot's last kernel read its inputs
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = outs_h[0][0].numel() * outs_h[0][0].element_size() + outs_h[0][1].numel() * outs_h[0][1].element_size()
    base = {k: v for k, v in kw.items() if not isinstance(v, torch.Tensor) or k in ("ori_kv", "cmp_kv")}
    q_h = host["q"].view(-1)

    def e2e_step(i):
        slot = i % len(streams)
        st = streams[slot]
        d = dev_in[slot]
        q_d = d["q"].view(-1)
        chunk = -(-q_h.numel() // len(copy_streams))
        landed = []
        for c, cs in enumerate(copy_streams):
            if inputs_free[slot] is not None:
                cs.wait_event(inputs_free[slot])
            with torch.cuda.stream(cs):
                q_d[c * chunk:(c + 1) * chunk].copy_(q_h[c * chunk:(c + 1) * chunk], non_blocking=True)
                if c == 0:
                    for k, v in host.items():
                        if k != "q":
                            d[k].copy_(v, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cs)
                landed.append(ev)
        for ev in landed:
            st.wait_event(ev)
        out_d, lse_d = dev_out[slot]
        out_h, lse_h = outs_h[slot]
        with torch.cuda.stream(st):
            sparse_attn_sharedkv(d["q"], out=out_d, lse_out=lse_d, return_softmax_lse=True, kernel=kernel,
                                 max_seqlen_q=max_q, **{k: v for k, v in d.items() if k != "q"}, **base)
            free = torch.cuda.Event()
            free.record(st)
            inputs_free[slot] = free
            out_h.copy_(out_d, non_blocking=True)
            lse_h.copy_(lse_d, non_blocking=True)

    for i in range(warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    e0.record(cur)
    for st in streams + copy_streams:
        st.wait_event(e0)
    for i in range(steps):
        e2e_step(i)
    for st in streams:
        cur.wait_stream(st)
    e1.record(cur)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    return {"value": tokens_all * steps / (float(te.item()) / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "streams": len(streams), "copy_streams": len(copy_streams)}


# ---------------------------------------------------------------------------------------------
# inputs of sampled tokens: what the oracle reads for them (the CPU baseline and verification legs)


def spread(n, k):
    if n <= k:
        return list(range(n))
    return sorted({int(round(i * (n - 1) / (k - 1))) for i in range(k)})


def token_inputs(wl, tokens):
    """For flat token rows ``tokens`` of a device-resident workload: q rows ``[n, N1, D]`` and the
    token's window rows then compressed rows ``[n, kmax, D]`` (zero-padded; unmapped blocks read as
    zero rows), as bf16 / fp16 bit patterns (int16), plus ``counts [n, 2]`` (window, compressed).
    Rows are resolved with the oracle's rules (golden.py:28-66, 125-131) and gathered on the device."""
    import numpy as np

    from oracle import golden_np as O

    D = wl.q.shape[2]
    cu = wl.cu_seqlens_q.cpu().numpy().astype(np.int64)
    kv = wl.seqused_kv.cpu().numpy().astype(np.int64)
    ori_bt = wl.ori_block_table.cpu().numpy().astype(np.int64)
    cmp_bt = wl.cmp_block_table.cpu().numpy().astype(np.int64)
    bs_o, bn_o = wl.ori_kv.shape[1], wl.ori_kv.shape[0]
    bs_c, bn_c = wl.cmp_kv.shape[1], wl.cmp_kv.shape[0]
    ori2d = wl.ori_kv.view(-1, D)
    cmp2d = wl.cmp_kv.view(-1, D)
    idx_rows = wl.cmp_sparse_indices.index_select(0, torch.as_tensor(tokens, device=wl.q.device)).cpu().numpy()

    def phys(table, pos, bs, bn):
        blk = pos // bs
        p = np.full(pos.shape, -1, dtype=np.int64)
        inside = blk < table.shape[0]
        p[inside] = table[blk[inside]]
        ok = (p >= 0) & (p < bn)
        return np.where(ok, p * bs + pos % bs, -1)

    plans = []
    for j, t in enumerate(tokens):
        b = int(np.searchsorted(cu, t, side="right") - 1)
        s = int(t - cu[b])
        win, cpos, _ = O.resolve_token_rows(scenario=3, b=b, s=s, act_q=int(cu[b + 1] - cu[b]), act_kv=int(kv[b]),
                                            cmp_idx_row=idx_rows[j, 0], topk=wl.topk, cmp_ratio=wl.cmp_ratio,
                                            ori_win_left=wl.ori_win_left)
        plans.append((phys(ori_bt[b], win, bs_o, bn_o), phys(cmp_bt[b], cpos, bs_c, bn_c)))
    kmax = max(1, max(a.size + c.size for a, c in plans))
    n = len(tokens)
    keys = torch.zeros((n, kmax, D), dtype=wl.q.dtype, device=wl.q.device)
    counts = np.zeros((n, 2), dtype=np.int32)
    for j, (a, c) in enumerate(plans):
        for pool, rows, off in ((ori2d, a, 0), (cmp2d, c, a.size)):
            if rows.size:
                r = torch.as_tensor(np.maximum(rows, 0), device=wl.q.device)
                got = pool.index_select(0, r)
                got[torch.as_tensor(rows < 0, device=wl.q.device)] = 0
                keys[j, off:off + rows.size] = got
        counts[j] = (a.size, c.size)
    q = wl.q.index_select(0, torch.as_tensor(tokens, device=wl.q.device))
    return q.view(torch.int16), keys.view(torch.int16), counts


# ---------------------------------------------------------------------------------------------
# CPU baseline: the oracle port over all host cores


def cpu_rate(wl, steps=1, warmup=0, budget_s=None):
    """Tokens/s of the oracle port on this host for a sample of the workload's tokens (all of them up
    to CPU_SAMPLE_TOKENS, else an even spread), with ``oracle.parallel`` worker processes; the worker
    count is the best of a sweep.  Returns ``(rates per timed step, cpu_baseline dict)``."""
    import numpy as np

    from oracle import parallel as P

    toks = spread(wl.num_tokens, CPU_SAMPLE_TOKENS)
    q_bits, k_bits, counts = token_inputs(wl, toks)
    cores = P.usable_cores()
    pool = P.OraclePool(q_bits.cpu().numpy().view(np.uint16), k_bits.cpu().numpy().view(np.uint16), counts,
                        wl.sinks.cpu().numpy(), wl.softmax_scale, cores)
    try:
        idx = list(range(len(toks)))
        tried = P.sweep_counts(cores)
        _, best_w, sweep = P.best_rate(pool, idx, tried)
        rates = []
        t_all = time.perf_counter()
        for i in range(warmup + steps):
            r = len(idx) / pool.run(idx, best_w)
            if i >= warmup:
                rates.append(r)
            if budget_s and time.perf_counter() - t_all > budget_s and len(rates) >= 1:
                break
    finally:
        pool.close()
    value = statistics.median(rates)
    return rates, {
        "value": value,
        "unit": "tokens/s",
        "cores": best_w,
        "kind": "port",
        "sample": (f"{len(toks)} of {wl.num_tokens} tokens of the same workload per step "
                   f"({'all' if len(toks) == wl.num_tokens else 'an even spread'}); numpy restatement of "
                   f"golden.py's per-token online softmax, key rows gathered before timing; {best_w} worker "
                   f"processes x 1 BLAS thread (best of a sweep over {tried}: "
                   + ", ".join(f"{w}: {r:.0f}/s" for w, r in sweep.items())
                   + f"); usable cores {cores}, os.cpu_count()={os.cpu_count()}"),
    }


def run_reference(args, rank, world):
    """--impl reference: the CPU port of the reference path, rank 0 only, on the GPU arm's
    config and (with a GPU present) the GPU arm's rank-0 data."""
    if rank != 0:
        return
    from dsv4_planb_b200 import _lib, sharding as S, workloads as W

    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
        _lib.load()
    wl, total, strong = build_workload(args.workload, 0, world, dev, args.batch)
    split = S.split_hint(S.token_tiles(wl.q_lens, wl.kv_lens, wl.topk, wl.cmp_ratio)) if strong else 0
    rates, cpu = cpu_rate(wl, steps=args.steps, warmup=args.warmup, budget_s=240.0)
    value = statistics.median(rates)
    line = {
        "impl": "reference",
        "metric": "decode tokens/s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": len(rates),
        "warmup": args.warmup,
        "ms_per_step": total / value * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": config_block(args.workload, world, args.batch, wl.num_tokens, total, strong, split),
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# verification over NCCL (N > 1)


def verify_gather(wl, out, lse, dev, rank, world, dist, n_sample):
    """NCCL all_gather of every rank's full out / lse (padded to the longest shard) and of the
    inputs of ``n_sample`` tokens per rank; rank 0 checks each gathered sampled row against the
    fp32 oracle at the north-star bars (out atol 2e-2 / rtol 1e-2, lse 1e-3)."""
    import numpy as np

    T = out.shape[0]
    tmax = torch.tensor([T], dtype=torch.int64, device=dev)
    dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    tmax = int(tmax.item())
    pad_o = torch.zeros((tmax,) + tuple(out.shape[1:]), dtype=out.dtype, device=dev)
    pad_o[:T] = out
    pad_l = torch.zeros((tmax, lse.shape[1]), dtype=lse.dtype, device=dev)
    pad_l[:T] = lse
    all_o = [torch.empty_like(pad_o) for _ in range(world)]
    all_l = [torch.empty_like(pad_l) for _ in range(world)]
    dist.all_gather(all_o, pad_o)
    dist.all_gather(all_l, pad_l)
    toks = spread(T, n_sample)
    toks += [toks[-1]] * (n_sample - len(toks))
    q_bits, k_bits, counts = token_inputs(wl, toks)
    kmax = torch.tensor([k_bits.shape[1]], dtype=torch.int64, device=dev)
    dist.all_reduce(kmax, op=dist.ReduceOp.MAX)
    keys = torch.zeros((n_sample, int(kmax.item()), k_bits.shape[2]), dtype=torch.int16, device=dev)
    keys[:, :k_bits.shape[1]] = k_bits
    meta = torch.tensor([[t, c[0], c[1]] for t, c in zip(toks, counts)], dtype=torch.int64, device=dev)
    sinks = wl.sinks.float().contiguous()
    gathered = {}
    for name, tns in (("q", q_bits.contiguous()), ("keys", keys), ("meta", meta), ("sinks", sinks)):
        # NCCL moves no int16: the bf16 / fp16 bit patterns travel as bfloat16 of the same bytes
        wire = tns.view(torch.bfloat16) if tns.dtype == torch.int16 else tns
        lst = [torch.empty_like(wire) for _ in range(world)]
        dist.all_gather(lst, wire)
        gathered[name] = [x.view(tns.dtype) for x in lst]
    if rank != 0:
        return None
    from oracle import golden_np as O

    def f32(bits):
        b = bits.cpu().numpy().view(np.uint16).astype(np.uint32) << 16
        return b.view(np.float32)

    worst_out, worst_lse, ok = -1e30, 0.0, True
    for r in range(world):
        for j in range(n_sample):
            t, nw, nc = (int(x) for x in gathered["meta"][r][j].tolist())
            kk = f32(gathered["keys"][r][j, :nw + nc])
            ref_o, ref_l = O.attend_token(f32(gathered["q"][r][j]), kk[:nw], kk[nw:],
                                          gathered["sinks"][r].cpu().numpy(), wl.softmax_scale)
            got_o = all_o[r][t].float().cpu().numpy()
            got_l = all_l[r][t].cpu().numpy()
            ex = float((np.abs(got_o - ref_o[:, :got_o.shape[1]]) - (2e-2 + 1e-2 * np.abs(ref_o[:, :got_o.shape[1]])))
                       .max())
            dl = float(np.abs(got_l - ref_l).max())
            worst_out, worst_lse = max(worst_out, ex), max(worst_lse, dl)
            ok &= ex <= 0 and dl <= 1e-3
    return {"parity_checked": True, "pass": bool(ok), "ranks": world, "tokens_per_rank": n_sample,
            "max_out_excess_over_atol_rtol": worst_out, "max_abs_dlse": worst_lse,
            "gathered_bytes_per_rank": int(pad_o.numel() * pad_o.element_size() + pad_l.numel() * 4)}


# ---------------------------------------------------------------------------------------------


def kernels_per_call(wl, kernel: str, split_tiles: int = 0) -> int:
    """Kernels one sas_forward call on this workload launches (sas_forward_kernel_count)."""
    from dsv4_planb_b200 import _lib

    a = _lib.SasFwdArgs()
    a.batch, a.num_tokens, a.max_q_len = len(wl.q_lens), wl.num_tokens, max(wl.q_lens)
    a.num_heads, a.num_kv_heads, a.head_dim, a.v_head_dim = wl.q.shape[1], 1, wl.q.shape[2], wl.v_head_dim
    a.ori_block_num, a.ori_block_size, a.ori_table_len = wl.ori_kv.shape[0], wl.ori_kv.shape[1], wl.ori_block_table.shape[1]
    a.cmp_block_num, a.cmp_block_size, a.cmp_table_len = wl.cmp_kv.shape[0], wl.cmp_kv.shape[1], wl.cmp_block_table.shape[1]
    a.topk, a.cmp_ratio, a.scenario = wl.topk, wl.cmp_ratio, 3
    a.ori_win_left, a.ori_win_right, a.ori_mask_mode, a.cmp_mask_mode = 127, 0, 4, 3
    a.dtype, a.softmax_scale, a.kernel = 0, wl.softmax_scale, _lib.KERNELS[kernel]
    a.flags = _lib.SAS_FWD_FLAG_CU_SEQLENS
    a.split_tiles = split_tiles
    n = _lib.ctypes.c_int32(0)
    _lib.check(_lib.load().sas_forward_kernel_count(_lib.ctypes.byref(a), _lib.ctypes.byref(n)), "kernel count")
    return n.value


def tc_used(wl, kernel) -> bool:
    from dsv4_planb_b200 import _lib

    if kernel == "simt":
        return False
    a = _lib.SasFwdArgs()
    a.batch, a.num_tokens, a.max_q_len = 1, 1, 1
    a.num_heads, a.num_kv_heads, a.head_dim, a.v_head_dim = wl.q.shape[1], 1, wl.q.shape[2], wl.v_head_dim
    a.ori_block_num, a.ori_block_size, a.ori_table_len = 1, wl.ori_kv.shape[1], 1
    a.cmp_block_num, a.cmp_block_size, a.cmp_table_len = 1, wl.cmp_kv.shape[1], 1
    a.topk, a.cmp_ratio, a.scenario = wl.topk, wl.cmp_ratio, 3
    a.ori_win_left, a.ori_mask_mode, a.cmp_mask_mode = 127, 4, 3
    a.dtype, a.softmax_scale, a.kernel = 0, 1.0, 2
    n = _lib.ctypes.c_size_t()
    return _lib.load().sas_workspace_size(_lib.ctypes.byref(a), _lib.ctypes.byref(n)) == 0


def extra_config(name, args, rank, world, dev, dist, flush, peaks):
    """c4 (prefill TFLOP/s) and c5 (strong-scaling decode) keys of the default run."""
    from dsv4_planb_b200 import sharding as S
    from dsv4_planb_b200.roofline import algorithmic_figures

    wl, total, strong = build_workload(name, rank, world, dev)
    figs = algorithmic_figures(wl, dev)
    kw = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in wl.api_kwargs().items()}
    split = S.split_hint(S.token_tiles(wl.q_lens, wl.kv_lens, wl.topk, wl.cmp_ratio)) if strong else 0
    kw["split_tiles"] = split
    steps = args.steps if name == "c5" else max(3, min(args.steps, 10))
    total_ms, step_ms, kernel_ms, out, lse = time_workload(wl, kw, steps, max(3, min(args.warmup, 5)), args.kernel,
                                                           dev, world, dist, flush)
    k_ms = statistics.mean(kernel_ms)
    kt = torch.tensor([k_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(kt, op=dist.ReduceOp.MAX)
    res = {"workload": config_block(name, world, None, wl.num_tokens, total, strong, split)["workload"],
           "ms_per_step": total_ms / steps, "steps": steps, "value": total * steps / (total_ms / 1e3),
           "unit": "tokens/s", "kernel_ms": k_ms, "kernel_ms_max_over_ranks": float(kt.item()),
           "tflops": figs["flops"] / (k_ms / 1e3) / 1e12, "gbs": figs["bytes"] / (k_ms / 1e3) / 1e9,
           "gpu_launches": kernels_per_call(wl, args.kernel, split) * steps}
    res["tensor_frac"] = res["tflops"] / peaks["bf16_tflops"]
    res["hbm_frac"] = res["gbs"] / peaks["hbm_gbs"]
    if name == "c5":
        res["scaling"] = "strong"
        res["split_tiles"] = split
        res["frac"] = res["hbm_frac"]
        if world > 1:
            res["verify"] = verify_gather(wl, out, lse, dev, rank, world, dist, 4)
    else:
        res["frac"] = res["tensor_frac"]
    del wl, kw, out, lse
    torch.cuda.empty_cache()
    return res


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from dsv4_planb_b200 import _lib, sharding as S
    from dsv4_planb_b200.roofline import algorithmic_figures

    _lib.load()
    peaks = measured_peaks()
    wl, total_tokens, strong = build_workload(args.workload, rank, world, dev, args.batch)
    figs = algorithmic_figures(wl, dev)
    kw = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in wl.api_kwargs().items()}
    split = 0
    if strong:
        # the sharding layer knows its requests' lengths: it picks the piece size that best spreads
        # the shard's tokens over the tensor-core kernel's clusters (0: whole tokens)
        split = S.split_hint(S.token_tiles(wl.q_lens, wl.kv_lens, wl.topk, wl.cmp_ratio))
        kw["split_tiles"] = split
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    sampler = ClockSampler(local)
    max_total_ms, step_ms, kernel_ms, out, lse = time_workload(wl, kw, args.steps, args.warmup, args.kernel, dev,
                                                               world, dist, flush, sampler)
    clocks = sampler.stop()
    value = total_tokens * args.steps / (max_total_ms / 1e3)

    verify = None
    if world > 1:
        verify = verify_gather(wl, out, lse, dev, rank, world, dist, 4)
    del out, lse

    e2e = None
    if not args.no_e2e:
        e2e = time_e2e(wl, kw, args.steps, args.warmup, args.kernel, dev, world, dist, total_tokens)

    # ---- the same step with SAS_FWD_FLAG_LAZY_RESCALE (performance mode, not the headline)
    lazy = None
    if not args.no_extra and tc_used(wl, args.kernel):
        kw_l = dict(kw, lazy_rescale=True)
        l_total, _, l_kernel, o_l, l_l = time_workload(wl, kw_l, args.steps, args.warmup, args.kernel, dev, world,
                                                       dist, flush)
        del o_l, l_l
        lk = statistics.mean(l_kernel)
        lazy = {"ms_per_step": l_total / args.steps, "value": total_tokens * args.steps / (l_total / 1e3),
                "unit": "tokens/s", "kernel_ms": lk, "hbm_frac": figs["bytes"] / (lk / 1e3) / 1e9 / peaks["hbm_gbs"],
                "tflops": figs["flops"] / (lk / 1e3) / 1e12,
                "note": "SAS_FWD_FLAG_LAZY_RESCALE: running max raised only past 8 (log2); P rounded at another "
                        "scale than the reference golden's; north-star bars still met"}

    # ---- roofline of the attention kernel
    k_avg_ms = statistics.mean(kernel_ms)
    achieved = figs["bytes"] / (k_avg_ms / 1e3) / 1e9
    tflops = figs["flops"] / (k_avg_ms / 1e3) / 1e12
    kname = ("sas_fwd_tc2" if args.kernel == "tc2" else "sas_fwd_tc") if tc_used(wl, args.kernel) else "fwd_simt_kernel"
    if args.workload == "c4":
        # prefill is quoted as tensor-core throughput against the dense bf16 peak (burst figure:
        # the kernel holds the SM clock at its maximum, well under the power cap)
        roofline = {"bound": "tensor", "achieved": tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": tflops / peaks["bf16_tflops"]}
    else:
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": achieved / peaks["hbm_gbs"]}
    roofline.update({"traffic": None if args.batch else committed_traffic(args.workload, kname),
                     "peak_source": peaks["source"],
                     "kernel": kname, "kernel_ms": k_avg_ms, "bytes_per_launch": figs["bytes"],
                     "flops_per_launch": figs["flops"], "tflops": tflops, "gbs": achieved,
                     "tensor_frac_of_burst": tflops / peaks["bf16_tflops"], "hbm_frac": achieved / peaks["hbm_gbs"]})
    config = config_block(args.workload, world, args.batch, wl.num_tokens, total_tokens, strong, split)
    launches = kernels_per_call(wl, args.kernel, split) * args.steps
    del wl, kw
    torch.cuda.empty_cache()

    extra = {}
    if args.workload == "c2" and not args.batch and not args.no_extra:
        if world == 1:
            extra["c4"] = extra_config("c4", args, rank, world, dev, dist, flush, peaks)
        extra["c5"] = extra_config("c5", args, rank, world, dev, dist, flush, peaks)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        wl0, _, _ = build_workload(args.workload, 0, 1, dev, args.batch)
        cpu = cpu_rate(wl0, steps=3, warmup=0, budget_s=30.0)[1]
        del wl0

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "decode tokens/s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": max_total_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": config,
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": launches,
        "clocks": clocks,
        "algorithmic": {"kv_bytes": figs["kv_bytes"], "keys": figs["keys"]},
    }
    line.update(extra)
    if lazy is not None:
        line["lazy_rescale"] = lazy
    if verify is not None:
        line["verify"] = verify
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
