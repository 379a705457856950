"""Benchmark of the B200 sparse_attn_sharedkv hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2]

One step = one ``sparse_attn_sharedkv`` call (SCFA: 128-key window + top-2048
compressed keys, N1 = 128, D_qk 576 / D_v 512, bf16) over one decode batch of
the BASELINE configuration ``c2`` (B = 64, seq U[8K, 32K]) per GPU, with
synthetic seeded inputs (``dsv4_planb_b200.workloads``).  With N GPUs every
rank runs its own c2 batch (seed 42 + rank): requests are independent and are
sharded by batch with no collective on the data path ("weak" scaling).
``--workload c5`` splits the 512 requests of c5 across the N ranks by cost
instead (``dsv4_planb_b200.sharding``; "strong" scaling, total work fixed).

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
  cpu_baseline the oracle CPU port on a bounded sample of the workload (rank 0, N=1)
``--impl reference`` times that CPU port alone: the reference is Python over
an NPU toolchain absent here, and its own TileLang kernel does not implement
SCFA (it raises NotImplementedError), so its golden model, restated by the
oracle, is the reference implementation of this path.
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--kernel", default="auto", choices=["auto", "simt", "tc"])
    ap.add_argument("--batch", type=int, default=None,
                    help="request count of c2 / c3 (default 64 / 32): small-batch decode measurements")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
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


def cpu_baseline(wl_dev, budget_s=12.0, max_tokens=None):
    """Time the CPU oracle port on a bounded sample of the workload's tokens."""
    import numpy as np

    from oracle import golden_np as O

    threads = torch.get_num_threads()
    cu = wl_dev.cu_seqlens_q.cpu().tolist()
    B = len(cu) - 1
    # compact copy of a few requests (only their blocks), prepared outside the timed region
    reqs = list(range(B))
    done_tokens = 0
    elapsed = 0.0
    t_start = time.perf_counter()
    for b in reqs:
        ori_bt = wl_dev.ori_block_table[b : b + 1].cpu()
        cmp_bt = wl_dev.cmp_block_table[b : b + 1].cpu()
        ob = ori_bt[ori_bt >= 0].long()
        cb = cmp_bt[cmp_bt >= 0].long()
        ori_pool = wl_dev.ori_kv[ob.to(wl_dev.ori_kv.device)].cpu()
        cmp_pool = wl_dev.cmp_kv[cb.to(wl_dev.cmp_kv.device)].cpu()
        ori_map = torch.full_like(ori_bt, -1)
        ori_map[ori_bt >= 0] = torch.arange(ob.numel(), dtype=torch.int32)
        cmp_map = torch.full_like(cmp_bt, -1)
        cmp_map[cmp_bt >= 0] = torch.arange(cb.numel(), dtype=torch.int32)
        t0, t1 = cu[b], cu[b + 1]
        q = wl_dev.q[t0:t1].cpu()
        idx = wl_dev.cmp_sparse_indices[t0:t1].cpu()
        kv = wl_dev.seqused_kv[b : b + 1].cpu()
        sinks = wl_dev.sinks.cpu()
        c0 = time.perf_counter()
        O.sparse_attn_sharedkv_oracle(
            q, ori_kv=ori_pool, ori_block_table=ori_map, seqused_kv=kv, q_prefix=[0], act_q=[t1 - t0], sinks=sinks,
            softmax_scale=wl_dev.softmax_scale, cmp_kv=cmp_pool, cmp_block_table=cmp_map, cmp_sparse_indices=idx,
            cmp_ratio=wl_dev.cmp_ratio, v_head_dim=wl_dev.v_head_dim)
        elapsed += time.perf_counter() - c0
        done_tokens += t1 - t0
        if elapsed >= budget_s or time.perf_counter() - t_start > 3 * budget_s:
            break
        if max_tokens and done_tokens >= max_tokens:
            break
    del np
    return {
        "value": done_tokens / elapsed if elapsed > 0 else None,
        "unit": "tokens/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{done_tokens} of {wl_dev.num_tokens} decode tokens of the same workload "
                  f"({done_tokens and round(elapsed, 2)} s of CPU work, numpy oracle, {threads} threads, "
                  f"os.cpu_count()={os.cpu_count()})",
    }


def run_reference(args, rank, world):
    """--impl reference: the CPU port of the reference path, rank 0 only."""
    if rank != 0:
        return
    from dsv4_planb_b200 import workloads as W

    torch.set_num_threads(os.cpu_count() or 1)
    wl = W.config_workload(args.workload, device="cpu", index_method="keys", batch=args.batch)
    times = []
    per_step_budget = 4.0
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(wl, budget_s=per_step_budget)
        if i >= args.warmup:
            times.append(r)
    vals = [r["value"] for r in times if r["value"]]
    value = statistics.median(vals) if vals else None
    # each step is a bounded sample of the workload's tokens; a whole step at the measured rate:
    ms_per_step = wl.num_tokens / value * 1e3 if value else None
    line = {
        "impl": "reference",
        "metric": "decode tokens/s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": W.CONFIG_DESCRIPTIONS[args.workload]
                               + (f" (batch overridden: {args.batch} requests)" if args.batch else ""),
                   "global_batch": wl.num_tokens, "seq_len": None,
                   "parallelism": "cpu"},
        "cpu_baseline": {**times[-1], "value": value},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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

    from dsv4_planb_b200 import _lib, workloads as W
    from dsv4_planb_b200.api import sparse_attn_sharedkv
    from dsv4_planb_b200.roofline import algorithmic_figures

    _lib.load()
    strong = args.workload == "c5"
    if strong:
        # c5 is the multi-GPU config: its 512 requests are split across the ranks by cost (LPT over
        # window + compressed keys per token) and each rank builds only its shard's pools and tables.
        from dsv4_planb_b200 import sharding as S

        q_all, kv_all, n1, topk = W.config_lengths("c5", 42)
        mine = S.partition_requests(S.request_costs(q_all, kv_all, topk), world)[rank]
        wl = W.make_workload(name="c5[shard]", q_lens=[q_all[i] for i in mine], kv_lens=[kv_all[i] for i in mine],
                             num_heads=n1, topk=topk, seed=42 + rank, device=dev)
        total_tokens = sum(q_all)
    else:
        wl = W.config_workload(args.workload, seed=42 + rank, device=dev, batch=args.batch)
    figs = algorithmic_figures(wl, dev)
    kw = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in wl.api_kwargs().items()}
    split = 0
    if strong:
        # the sharding layer knows its requests' lengths: it picks the piece size that best spreads
        # the shard's tokens over the tensor-core kernel's clusters (0: whole tokens)
        split = S.split_hint(S.token_tiles(wl.q_lens, wl.kv_lens, wl.topk, wl.cmp_ratio))
        kw["split_tiles"] = split
    q = wl.q
    T, N1, _ = q.shape
    Dv = wl.v_head_dim
    out = torch.empty((T, N1, Dv), dtype=q.dtype, device=dev)
    lse = torch.empty((T, N1), dtype=torch.float32, device=dev)
    max_q = max(wl.q_lens)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def step():
        sparse_attn_sharedkv(q, out=out, lse_out=lse, return_softmax_lse=True, kernel=args.kernel,
                             max_seqlen_q=max_q, **kw)

    # warm-up eagerly (also sets kernel attributes before capture)
    for _ in range(max(args.warmup, 3)):
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
    # Two captures of the same step: `graph` (timed for `value`) holds only the op's own work;
    # `graph_ev` also records the library's events around the attention kernel (its duration for
    # the roofline).  The event nodes sit between the prep and the attention kernel and would
    # otherwise serialise the programmatic launch that overlaps them.
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

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kernel_ms = []
    sampler = ClockSampler(local)
    for _ in range(args.warmup):
        flush.fill_(1.0)
        graph.replay()
        flush.fill_(1.0)
        graph_ev.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    for i in range(args.steps):
        flush.fill_(float(i))
        starts[i].record()
        graph.replay()
        stops[i].record()
    for i in range(args.steps):
        flush.fill_(float(i))
        graph_ev.replay()
        k_stop.synchronize()
        kernel_ms.append(k_start.elapsed_time(k_stop))
    torch.cuda.synchronize()
    clocks = sampler.stop()
    step_ms = [a.elapsed_time(b) for a, b in zip(starts, stops)]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    max_total_ms = float(t.item())
    tokens_all = (total_tokens if strong else T * world) * args.steps
    value = tokens_all / (max_total_ms / 1e3)

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        # Every step copies its own inputs from pinned host memory, runs the public API call and
        # reads its out + lse back into pinned host memory.  Steps rotate over E2E_STREAMS slots
        # (a compute stream with its own device buffers), so one step's copies overlap another's
        # compute, as a serving loop would run them.  The q upload (9.4 MB at c2) is split over
        # E2E_COPY_STREAMS copy streams: one host-to-device copy of that size reaches only
        # 13-30 GB/s on these hosts, four concurrent ones 35-38 GB/s.
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
                sparse_attn_sharedkv(d["q"], out=out_d, lse_out=lse_d, return_softmax_lse=True, kernel=args.kernel,
                                     max_seqlen_q=max_q, **{k: v for k, v in d.items() if k != "q"}, **base)
                free = torch.cuda.Event()
                free.record(st)
                inputs_free[slot] = free
                out_h.copy_(out_d, non_blocking=True)
                lse_h.copy_(lse_d, non_blocking=True)

        for i in range(args.warmup):
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
        for i in range(args.steps):
            e2e_step(i)
        for st in streams:
            cur.wait_stream(st)
        e1.record(cur)
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": tokens_all / (float(te.item()) / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "streams": len(streams), "copy_streams": len(copy_streams)}

    # ---- roofline of the attention kernel
    peaks = measured_peaks()
    k_avg_ms = statistics.mean(kernel_ms) if kernel_ms else None
    achieved = figs["bytes"] / (k_avg_ms / 1e3) / 1e9 if k_avg_ms else None
    tflops = figs["flops"] / (k_avg_ms / 1e3) / 1e12 if k_avg_ms else None
    kname = "sas_fwd_tc" if args.kernel != "simt" and _tc_used(wl) else "fwd_simt_kernel"
    if args.workload == "c4":
        # prefill is quoted as tensor-core throughput against the dense bf16 peak (burst figure:
        # the kernel holds the SM clock at its maximum, well under the power cap)
        roofline = {"bound": "tensor", "achieved": tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": tflops / peaks["bf16_tflops"] if tflops else None}
    else:
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": achieved / peaks["hbm_gbs"] if achieved else None}
    roofline.update({"traffic": None if args.batch else committed_traffic(args.workload, kname),
                     "peak_source": peaks["source"],
                     "kernel": kname, "kernel_ms": k_avg_ms, "bytes_per_launch": figs["bytes"],
                     "flops_per_launch": figs["flops"], "tflops": tflops, "gbs": achieved,
                     "tensor_frac_of_burst": tflops / peaks["bf16_tflops"] if tflops else None,
                     "hbm_frac": achieved / peaks["hbm_gbs"] if achieved else None})

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl, budget_s=12.0)

    if world > 1:
        dist.barrier()
        graph.reset()
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
        "config": {"workload": f"{args.workload}: {W.CONFIG_DESCRIPTIONS[args.workload]}"
                               + (f" (batch overridden: {args.batch} requests)" if args.batch else ""),
                   "global_batch": total_tokens if strong else T * world,
                   "per_gpu_batch": T, "seq_len": "U[8K,32K]" if args.workload == "c2" else None,
                   "parallelism": (f"LPT request shards x{world}" if strong else f"request-sharded x{world}"),
                   "split_tiles": split, "l2": "flushed (256 MiB write) before every step",
                   "timing": "CUDA graph replay per step, CUDA events, max over ranks"},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": _kernels_per_call(wl, args.kernel, split) * args.steps,
        "clocks": clocks,
        "algorithmic": {"kv_bytes": figs["kv_bytes"], "keys": figs["keys"]},
    }
    print(json.dumps(line), flush=True)


def _tc_used(wl) -> bool:
    from dsv4_planb_b200 import _lib

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


def _kernels_per_call(wl, kernel: str, split_tiles: int = 0) -> int:
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


if __name__ == "__main__":
    main()
