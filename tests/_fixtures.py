"""Loaders for the committed golden fixtures under tests/golden/ (made by make_fixtures.py)."""

from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def metadata_cases():
    with open(os.path.join(GOLDEN, "metadata_cases.json")) as f:
        meta = json.load(f)
    outs = np.load(os.path.join(GOLDEN, "metadata_cases.npz"))["out"]
    return list(zip(meta["names"], meta["kwargs"], outs))


def index_cases():
    z = np.load(os.path.join(GOLDEN, "index_cases.npz"))
    offs = np.concatenate([[0], np.cumsum(z["lens"])])
    pos = z["positions"]
    return [(z["rows"][i], int(z["thr"][i]), pos[offs[i] : offs[i + 1]]) for i in range(len(z["thr"]))]


def load_case(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    d = {k: z[k] for k in z.files}
    d["digests"] = json.loads(str(d["digests"]))
    d["meta"] = json.loads(str(d["meta"]))
    if "out_low_bits" in d:
        d["out_low_bf16_bits"] = d["out_low_bits"]
    return d


def baseline_names():
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.startswith("baseline_") and f.endswith(".npz"))


def paramset_names():
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.startswith("paramset_") and f.endswith(".npz"))


def low_bits_to_f32(bits: np.ndarray, tag: str) -> np.ndarray:
    """Decode stored int16 bit patterns of a bf16 / fp16 tensor to fp32."""
    if tag == "bf16":
        return (bits.astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
    return bits.astype(np.uint16).view(np.float16).astype(np.float32)


def rebuild_baseline(case):
    """Regenerate the inputs of a baseline_* fixture with the product's workload generator."""
    from dsv4_planb_b200 import workloads as W

    meta = case["meta"]
    wl = W.make_workload(name=meta["name"], **meta["kw"])
    if meta.get("tweak") == "edges":
        edge_tweak(wl)
    return wl


def edge_tweak(wl):
    """The same edits make_fixtures.apply_edges makes (kept in sync by the digest check)."""
    import torch

    idx = wl.cmp_sparse_indices
    idx[1, 0, 5] = -1
    thr2 = (wl.kv_lens[2]) // wl.cmp_ratio
    idx[2, 0, :64] = torch.arange(thr2, thr2 + 64, dtype=torch.int32)
    idx[3, 0, 10:20] = idx[3, 0, 0]
    idx[4, 0, :] = -1


def check_result(real, expt, dtype_tag="bf16"):
    """Pass rate and max normalised error of the reference's _check_result
    (test_sparse_attn_sharedkv.py:394-467): returns (fulfill_pct, max_rel)."""
    rtol, atol = (0.0078125, 0.0001) if dtype_tag == "bf16" else (0.005, 0.000025)
    real = np.asarray(real, dtype=np.float32).ravel()
    expt = np.asarray(expt, dtype=np.float32).ravel()
    ok = np.isclose(real, expt, rtol=rtol, atol=atol, equal_nan=True)
    n_err = int((~ok).sum())
    pct = (real.size - n_err) / real.size * 100.0
    floor = (1.0 / (1 << 14)) / 0.005
    b = np.maximum(np.maximum(np.abs(real), np.abs(expt)), floor) + 1e-9
    rel = np.abs(real - expt) / b
    return pct, float(rel[~ok].max()) if n_err else 0.0


def check_lse(real, expt, dtype_tag="bf16"):
    """Same for _check_lse (test_sparse_attn_sharedkv.py:470-527)."""
    rtol, atol = (0.015, 0.005) if dtype_tag == "bf16" else (0.01, 0.001)
    real = np.asarray(real, dtype=np.float32).ravel()
    expt = np.asarray(expt, dtype=np.float32).ravel()
    ok = np.isclose(real, expt, rtol=rtol, atol=atol, equal_nan=True)
    n_err = int((~ok).sum())
    pct = (real.size - n_err) / real.size * 100.0
    floor = (1.0 / (1 << 14)) / 0.005
    b = np.maximum(np.maximum(np.abs(real), np.abs(expt)), floor) + 1e-9
    rel = np.abs(real - expt) / b
    return pct, float(rel[~ok].max()) if n_err else 0.0
