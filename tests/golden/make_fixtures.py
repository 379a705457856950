"""Generate the golden fixtures of this directory by running the REFERENCE itself.

Usage (only where the reference tree is mounted; the fixtures it writes are
committed, so nothing on a test machine needs the reference)::

    python tests/golden/make_fixtures.py [--reference-dir DIR]

It imports ``golden.py`` and ``metadata.py`` (and the test module, for
``_build_case``) from ``<reference>/sparse_attn_sharedkv_tilelang`` of
yangqiang2018/dsv4_planB and writes:

* ``metadata_cases.json`` / ``metadata_cases.npz`` -- keyword arguments and the
  ``int32[1024]`` output of ``sparse_attn_sharedkv_metadata`` for the
  reference paramsets, the BASELINE shapes and a seeded random sweep;
* ``index_cases.npz`` -- per-token compressed positions resolved by
  ``_gather_cmp_kv_tokens`` (golden.py:28-66), including hand-made edge rows
  (-1 in the middle, indices >= thr, duplicates, thr <= 0);
* ``paramset_<name>_<dtype>.npz`` -- input digests and golden outputs of the
  reference paramsets (test_sparse_attn_sharedkv.py:81-220 and the S1=1024
  prefill shrink), both the reference's own low-precision golden and the fp32
  golden (fp32 upcast inputs); prefill outputs are kept for a token subset;
* ``baseline_<name>.npz`` -- input digests and fp32-golden outputs of small
  BASELINE-style workloads from ``dsv4_planb_b200.workloads``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.dont_write_bytecode = True

from dsv4_planb_b200 import workloads as W  # noqa: E402
from oracle.gen import digest  # noqa: E402
from tests._fixtures import edge_tweak  # noqa: E402


def load_reference(ref_dir):
    sys.path.insert(0, os.path.join(ref_dir, "sparse_attn_sharedkv_tilelang"))
    import golden as G  # noqa: F401
    import metadata as M  # noqa: F401
    import test_sparse_attn_sharedkv as TS  # noqa: F401

    return G, M, TS


# ---------------------------------------------------------------- metadata


def metadata_sweep(n_random=240, seed=1234):
    cases = []
    # reference paramsets, as the reference tests call the scheduler
    from oracle.gen import PARAMSETS

    for name, cfg in PARAMSETS.items():
        for aic in (24, 36):
            kw = dict(
                num_heads_q=cfg["N1"], num_heads_kv=cfg["N2"], head_dim=cfg["D"],
                cu_seqlens_q=cfg["cu_seqlens_q"], seqused_kv=cfg["seqused_kv"], batch_size=cfg["B"],
                max_seqlen_q=cfg["T1"], max_seqlen_kv=max(cfg["seqused_kv"]),
                ori_mask_mode=4, ori_win_left=127, ori_win_right=0, layout_q="TND", layout_kv="PA_ND",
                has_ori_kv=True, has_cmp_kv=cfg["scenario"] >= 2, aic_core_num=aic,
            )
            if cfg["scenario"] >= 2:
                kw.update(cmp_ratio=cfg["cmp_ratio"], cmp_mask_mode=3)
            if cfg["scenario"] == 3:
                kw["cmp_topk"] = cfg["K"]
            cases.append((f"{name}_aic{aic}", kw))
    # BASELINE shapes
    for cfg in ("c1", "c2", "c3", "c4", "c5"):
        q_lens, kv_lens, n1, topk = W.config_lengths(cfg)
        cu = np.concatenate([[0], np.cumsum(q_lens)]).astype(int).tolist()
        for aic in (24, 36):
            cases.append((f"{cfg}_aic{aic}", dict(
                num_heads_q=n1, num_heads_kv=1, head_dim=576, cu_seqlens_q=cu, seqused_kv=kv_lens,
                batch_size=len(q_lens), max_seqlen_q=sum(q_lens), max_seqlen_kv=max(kv_lens), cmp_topk=topk,
                cmp_ratio=4, ori_mask_mode=4, cmp_mask_mode=3, ori_win_left=127, ori_win_right=0,
                layout_q="TND", layout_kv="PA_ND", has_ori_kv=True, has_cmp_kv=True, aic_core_num=aic)))
    rng = random.Random(seed)
    for i in range(n_random):
        B = rng.choice([1, 1, 2, 3, 4, 8, 16, 64])
        layout_q = rng.choice(["TND", "BSND", "TND", "BNSD"])
        qlens = [rng.choice([0, 1, 1, 2, 3, 7, 64, 200, 1024]) for _ in range(B)]
        kvlens = [max(0, q + rng.choice([0, 1, 5, 100, 600, 4000, 9000])) if rng.random() < 0.9 else rng.choice([0, 1, 50])
                  for q in qlens]
        n2 = rng.choice([1, 1, 1, 2])
        kw = dict(num_heads_q=rng.choice([16, 64, 128]), num_heads_kv=n2, head_dim=512, seqused_kv=kvlens,
                  batch_size=B, max_seqlen_q=max(qlens) if layout_q != "TND" else sum(qlens),
                  max_seqlen_kv=max(kvlens), ori_mask_mode=rng.choice([4, 4, 4, 3, 0]),
                  ori_win_left=rng.choice([127, 127, 0, 5, -1, 1000]), layout_q=layout_q, layout_kv="PA_ND",
                  has_ori_kv=True, has_cmp_kv=rng.random() < 0.8, aic_core_num=rng.choice([24, 24, 36, 1, 5, 48]))
        if layout_q == "TND":
            kw["cu_seqlens_q"] = np.concatenate([[0], np.cumsum(qlens)]).astype(int).tolist()
        if rng.random() < 0.2:
            kw["seqused_q"] = qlens
        if kw["has_cmp_kv"]:
            kw["cmp_ratio"] = rng.choice([4, 4, 128, 1, 2])
            kw["cmp_topk"] = rng.choice([0, 512, 2048, 7])
        cases.append((f"rand{i}", kw))
    return cases


def to_tensor_kwargs(kw):
    out = dict(kw)
    for k in ("cu_seqlens_q", "seqused_kv", "seqused_q", "cu_seqlens_ori_kv"):
        if k in out and out[k] is not None:
            out[k] = torch.tensor(out[k], dtype=torch.int32)
    return out


def make_metadata(M):
    cases = metadata_sweep()
    names, kws, outs = [], [], []
    for name, kw in cases:
        outs.append(M.sparse_attn_sharedkv_metadata(**to_tensor_kwargs(kw)).numpy().astype(np.int32))
        names.append(name)
        kws.append(kw)
    with open(os.path.join(HERE, "metadata_cases.json"), "w") as f:
        json.dump({"names": names, "kwargs": kws}, f, indent=0, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "metadata_cases.npz"), out=np.stack(outs))
    print(f"metadata: {len(names)} cases")


# ---------------------------------------------------------------- index resolution


def make_index_cases(G):
    rng = np.random.default_rng(7)
    rows, thrs, acts, expected = [], [], [], []
    K = 64
    cmp_len = 400
    # a cmp tensor whose row j holds j, so the gathered rows name their positions
    cmp = torch.arange(cmp_len, dtype=torch.float64).view(1, 1, cmp_len, 1)
    specs = []
    for _ in range(40):
        thr = int(rng.integers(-3, cmp_len + 1))
        row = rng.integers(-1, cmp_len + 60, size=K)
        specs.append((thr, row))
    edge = [
        (50, np.r_[np.arange(10), -1, np.arange(10, 63)]),  # -1 stops the scan
        (50, np.r_[np.arange(40, 104)]),  # indices >= thr are skipped
        (50, np.r_[np.full(8, 3), np.arange(56)]),  # duplicates are kept
        (0, np.arange(64)),  # thr 0: nothing
        (-2, np.arange(64)),  # thr < 0: nothing
        (10, np.r_[np.arange(64)]),  # only the first min(K, thr) slots are scanned
        (500, np.r_[np.arange(63), -1]),
        (5, np.r_[-1, np.arange(63)]),
    ]
    specs.extend(edge)
    for thr, row in specs:
        row = np.asarray(row, dtype=np.int32)
        # act_kv / act_q / s chosen so that threshold == thr with ratio 1
        act_q, s = 1, 0
        act_kv = thr
        idx = torch.tensor(row, dtype=torch.int32).view(1, 1, 1, K)
        got = G._gather_cmp_kv_tokens(cmp, idx, b=0, n2=0, s_local=s, act_kv=act_kv, act_q=act_q, cmp_ratio=1,
                                      cmp_mask_mode=3)
        pos = got[:, 0].to(torch.int64).numpy() if got.numel() else np.zeros(0, dtype=np.int64)
        rows.append(row)
        thrs.append(thr)
        acts.append(act_kv)
        expected.append(pos)
    lens = np.array([e.size for e in expected])
    flat = np.concatenate(expected) if expected else np.zeros(0, dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "index_cases.npz"), rows=np.stack(rows), thr=np.array(thrs),
                        lens=lens, positions=flat)
    print(f"index: {len(rows)} rows")


# ---------------------------------------------------------------- attention


def golden_tnd(G, *, q, ori_kv, ori_bt, cmp_kv, cmp_bt, idx, cu, seqused_kv, sinks, scale, cmp_ratio, scenario,
               fp32, dv):
    """Run the reference golden on TND paged inputs; returns TND out[..., :dv] and lse."""
    cast = (lambda t: t.to(torch.float32)) if fp32 else (lambda t: t)
    act_q = (cu[1:] - cu[:-1]).tolist()
    kv = [int(x) for x in seqused_kv.tolist()]
    B = len(act_q)
    q_bnsd = G.tnd_to_bnsd_q(cast(q), cu)
    ori_bnsd = G.unpack_paged_kv(cast(ori_kv), ori_bt, max(kv))
    cmp_bnsd = None
    idx_bsnd = None
    if scenario >= 2:
        max_cmp = max(max(k // cmp_ratio for k in kv), 1)
        cmp_bnsd = G.unpack_paged_kv(cast(cmp_kv), cmp_bt, max_cmp)
    if scenario == 3:
        K = idx.shape[-1]
        S_max = max(act_q)
        idx_bsnd = torch.full((B, S_max, 1, K), -1, dtype=torch.int32)
        for b in range(B):
            s0 = int(cu[b])
            idx_bsnd[b, : act_q[b]] = idx[s0 : s0 + act_q[b]]
    out, lse = G.sparse_attn_sharedkv_golden_bnsd(
        q_bnsd, ori_bnsd, sinks, act_q_lens=act_q, act_kv_lens=kv, softmax_scale=scale, cmp_k_bnsd=cmp_bnsd,
        cmp_sparse_indices=idx_bsnd, cmp_ratio=cmp_ratio if scenario >= 2 else None, return_lse=True)
    out = G.bnsd_to_tnd_out(out, cu)[..., :dv]
    lse = G.bnsd_to_tnd_lse(lse, cu)
    return out, lse


def save_case(path, *, digests, tokens, out_fp32, lse_fp32, out_low=None, lse_low=None, meta=None):
    arrs = dict(tokens=np.asarray(tokens, dtype=np.int64), out_fp32=out_fp32[tokens].numpy(),
                lse_fp32=lse_fp32[tokens].numpy())
    if out_low is not None:
        arrs["out_low_bits"] = out_low[tokens].contiguous().view(torch.int16).numpy()
        arrs["lse_low"] = lse_low[tokens].numpy()
    arrs["digests"] = np.array(json.dumps(digests))
    arrs["meta"] = np.array(json.dumps(meta or {}))
    np.savez_compressed(path, **arrs)


def make_paramsets(G, TS):
    from oracle.gen import PARAMSETS

    todo = [("scfa_decode", torch.bfloat16), ("swa_decode", torch.bfloat16), ("cfa_decode", torch.bfloat16),
            ("scfa_decode", torch.float16), ("scfa_prefill_fast", torch.bfloat16),
            ("swa_prefill_fast", torch.bfloat16), ("cfa_prefill_fast", torch.bfloat16)]
    for name, dtype in todo:
        cfg = PARAMSETS[name]
        case = TS._build_case(cfg, dtype)
        T = cfg["T1"]
        if T <= 4:
            tokens = list(range(T))
        else:
            tokens = sorted({0, 1, 127, 128, 129, 511, 777, T - 1})
        scen = cfg["scenario"]
        out32, lse32 = golden_tnd(G, q=case["q"], ori_kv=case["ori_pa"], ori_bt=case["ori_bt"], cmp_kv=case["cmp_pa"],
                                  cmp_bt=case["cmp_bt"], idx=case["cmp_idx"], cu=case["cu_seqlens_q"],
                                  seqused_kv=case["seqused_kv"], sinks=case["sinks"], scale=cfg["softmax_scale"],
                                  cmp_ratio=cfg["cmp_ratio"], scenario=scen, fp32=True, dv=cfg["D"])
        digests = {k: digest(case[k]) for k in ("q", "ori_pa", "ori_bt", "cmp_pa", "cmp_bt", "cmp_idx", "sinks")}
        tag = "bf16" if dtype == torch.bfloat16 else "fp16"
        save_case(os.path.join(HERE, f"paramset_{name}_{tag}.npz"), digests=digests, tokens=tokens, out_fp32=out32,
                  lse_fp32=lse32, out_low=case["cpu_ref"], lse_low=case["cpu_ref_lse"], meta={"name": name})
        print(f"paramset {name} {tag}: tokens {tokens}")


def baseline_specs():
    """Small BASELINE-style workloads (CPU-sized) with their edge-case tweaks."""
    specs = []
    q, kv, n1, topk = W.config_lengths("c1")
    specs.append(("c1", dict(q_lens=q, kv_lens=kv, num_heads=n1, topk=topk), None))
    # MTP-like: q_len 2, short and long contexts (thr < K padding, truncated window)
    specs.append(("mtp_small", dict(q_lens=[2, 2, 2], kv_lens=[90, 700, 3000], num_heads=16, topk=256), None))
    # chunked-prefill-like: new tokens on top of a context, window crossing block boundaries
    specs.append(("prefill_small", dict(q_lens=[40, 24], kv_lens=[40, 300], num_heads=16, topk=64), None))
    # edge rows: -1 in the middle, indices >= thr, duplicates, all -1
    specs.append(("edges", dict(q_lens=[1, 1, 1, 1, 1], kv_lens=[1, 129, 1000, 2000, 513], num_heads=16, topk=128),
                  "edges"))
    # 64 heads, D 512 (K=V full), as the reference paramsets
    specs.append(("h64_d512", dict(q_lens=[1, 3], kv_lens=[2048, 600], num_heads=64, topk=128, head_dim=512,
                                   v_head_dim=512), None))
    # 128 heads, the production head count, small contexts
    specs.append(("h128", dict(q_lens=[1, 1], kv_lens=[1500, 700], num_heads=128, topk=256), None))
    return specs


def make_baselines(G):
    for name, kw, tweak in baseline_specs():
        wl = W.make_workload(name=name, **kw)
        if tweak == "edges":
            edge_tweak(wl)
        out32, lse32 = golden_tnd(G, q=wl.q, ori_kv=wl.ori_kv, ori_bt=wl.ori_block_table, cmp_kv=wl.cmp_kv,
                                  cmp_bt=wl.cmp_block_table, idx=wl.cmp_sparse_indices, cu=wl.cu_seqlens_q,
                                  seqused_kv=wl.seqused_kv, sinks=wl.sinks, scale=wl.softmax_scale,
                                  cmp_ratio=wl.cmp_ratio, scenario=3, fp32=True, dv=wl.v_head_dim)
        digests = {k: digest(getattr(wl, k)) for k in ("q", "ori_kv", "ori_block_table", "cmp_kv", "cmp_block_table",
                                                        "cmp_sparse_indices", "sinks")}
        if wl.num_tokens <= 16:
            tokens = list(range(wl.num_tokens))
        else:  # the first and last two tokens of every request, plus a few inside
            cu = wl.cu_seqlens_q.tolist()
            sel = set()
            for b in range(len(cu) - 1):
                sel.update({cu[b], cu[b] + 1, cu[b + 1] - 2, cu[b + 1] - 1, (cu[b] + cu[b + 1]) // 2})
            tokens = sorted(t for t in sel if 0 <= t < wl.num_tokens)
        save_case(os.path.join(HERE, f"baseline_{name}.npz"), digests=digests, tokens=tokens, out_fp32=out32,
                  lse_fp32=lse32, meta={"name": name, "kw": kw, "tweak": tweak})
        print(f"baseline {name}: T={wl.num_tokens}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", required=True, help="checkout of the reference project")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    G, M, TS = load_reference(args.reference_dir)
    only = set(args.only.split(",")) if args.only else None
    if only is None or "metadata" in only:
        make_metadata(M)
    if only is None or "index" in only:
        make_index_cases(G)
    if only is None or "baseline" in only:
        make_baselines(G)
    if only is None or "paramset" in only:
        make_paramsets(G, TS)


if __name__ == "__main__":
    main()
