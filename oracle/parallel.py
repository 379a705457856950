"""Process-parallel CPU baseline of the oracle -- TEST / MEASUREMENT INFRASTRUCTURE ONLY.

Times ``golden_np.attend_token`` (the restatement of the reference golden's
per-token online softmax, golden.py:156-200) over the tokens of a workload on
the host's cores.  The reference golden walks its tokens one after another in
one process; its work per token is independent, so the fair CPU rate uses every
core: ``P`` worker processes (started with ``spawn``; one BLAS thread each, so
they do not oversubscribe the cores) share the tokens' inputs through one
shared-memory block and split the token list.  ``sweep`` times several worker
counts and keeps the best rate.

Inputs per token are what the golden reads for it: q ``[N1, D]`` and the
token's window rows then compressed rows ``[n_win + n_cmp, D]`` (bf16 bits,
zero-padded to the longest token), the counts, and the per-head sinks.  The
bf16 -> fp32 conversion is part of the timed work, as the golden's
``.to(torch.float32)`` is.

Nothing in the product package imports this module.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import time
from multiprocessing import shared_memory

import numpy as np

_ENV_ONE_THREAD = {"OMP_NUM_THREADS": "1", "OPENBLAS_NUM_THREADS": "1", "MKL_NUM_THREADS": "1",
                   "NUMEXPR_NUM_THREADS": "1"}


def _bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _worker(conn, shm_name, layout, sinks, scale):
    from oracle import golden_np as O

    shm = shared_memory.SharedMemory(name=shm_name)
    arrs = {k: np.ndarray(shape, dtype=np.dtype(dt), buffer=shm.buf, offset=off) for k, (off, shape, dt) in
            layout.items()}
    try:
        while True:
            msg = conn.recv()
            if msg is None:
                break
            t0 = time.perf_counter()
            acc = 0.0
            for i in msg:
                nw, nc = int(arrs["counts"][i, 0]), int(arrs["counts"][i, 1])
                q = _bf16_to_f32(arrs["q"][i])
                keys = _bf16_to_f32(arrs["keys"][i, : nw + nc])
                _, lse = O.attend_token(q, keys[:nw], keys[nw:], sinks, scale)
                acc += float(lse[0])
            conn.send((time.perf_counter() - t0, acc))
    finally:
        del arrs
        shm.close()


class OraclePool:
    """``P`` spawned workers over one shared copy of the tokens' inputs."""

    def __init__(self, q_bits: np.ndarray, keys_bits: np.ndarray, counts: np.ndarray, sinks: np.ndarray,
                 scale: float, workers: int):
        arrays = {"q": np.ascontiguousarray(q_bits, dtype=np.uint16),
                  "keys": np.ascontiguousarray(keys_bits, dtype=np.uint16),
                  "counts": np.ascontiguousarray(counts, dtype=np.int32)}
        layout, off = {}, 0
        for k, a in arrays.items():
            layout[k] = (off, a.shape, a.dtype.str)
            off += (a.nbytes + 63) // 64 * 64
        self.n = int(q_bits.shape[0])
        self.shm = shared_memory.SharedMemory(create=True, size=max(off, 64))
        for k, a in arrays.items():
            np.ndarray(a.shape, dtype=a.dtype, buffer=self.shm.buf, offset=layout[k][0])[...] = a
        ctx = mp.get_context("spawn")
        saved = {k: os.environ.get(k) for k in _ENV_ONE_THREAD}
        os.environ.update(_ENV_ONE_THREAD)
        self.conns, self.procs = [], []
        try:
            for _ in range(workers):
                parent, child = ctx.Pipe()
                p = ctx.Process(target=_worker, args=(child, self.shm.name, layout,
                                                      np.asarray(sinks, dtype=np.float32), float(scale)),
                                daemon=True)
                p.start()
                self.conns.append(parent)
                self.procs.append(p)
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
        self.run(list(range(min(self.n, workers))), workers)  # imports and first-touch, untimed

    def run(self, tokens, workers: int) -> float:
        """Wall-clock seconds for ``workers`` processes to attend ``tokens`` (split round robin)."""
        workers = max(1, min(workers, len(self.conns)))
        parts = [tokens[w::workers] for w in range(workers)]
        t0 = time.perf_counter()
        for w in range(workers):
            self.conns[w].send(parts[w])
        for w in range(workers):
            self.conns[w].recv()
        return time.perf_counter() - t0

    def close(self):
        for c in self.conns:
            try:
                c.send(None)
            except (BrokenPipeError, OSError):
                pass
        for p in self.procs:
            p.join(timeout=10)
            if p.is_alive():
                p.terminate()
        self.shm.close()
        self.shm.unlink()


def usable_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - non-Linux
        return os.cpu_count() or 1


def sweep_counts(cores: int):
    out, p = [], 1
    while p < cores:
        out.append(p)
        p *= 2
    out.append(cores)
    return out


def best_rate(pool: OraclePool, tokens, counts_to_try, repeats: int = 1):
    """``(tokens/s, workers, {workers: tokens/s})`` over the worker counts tried."""
    rates = {}
    for w in counts_to_try:
        best = min(pool.run(tokens, w) for _ in range(repeats))
        rates[w] = len(tokens) / best
    w = max(rates, key=rates.get)
    return rates[w], w, rates
