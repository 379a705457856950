"""Pins the CPU oracle (oracle/) to outputs of the reference itself.

The fixtures under tests/golden/ were produced by running the reference
(yangqiang2018/dsv4_planB golden.py / metadata.py / _build_case) through
tests/golden/make_fixtures.py.  These tests need no GPU.
"""

import numpy as np
import pytest
import torch

from oracle import golden_np as O
from oracle.gen import PARAMSETS, digest, ref_build_case
from oracle.metadata_ref import metadata_ref
from tests import _fixtures as F


@pytest.mark.parametrize("case", F.metadata_cases(), ids=lambda c: c[0])
def test_metadata_oracle_matches_reference(case):
    name, kw, expected = case
    got = metadata_ref(**kw)
    np.testing.assert_array_equal(got, expected)


def test_index_oracle_matches_reference():
    cases = F.index_cases()
    assert len(cases) >= 40
    for row, thr, expected in cases:
        got, _ = O.resolve_cmp_positions(row, thr, row.shape[0])
        np.testing.assert_array_equal(got, expected, err_msg=f"thr={thr} row={row[:12]}")


PARAM_CASES = [n for n in F.paramset_names()]


def _paramset_key(fixture_name):
    name = fixture_name[len("paramset_"):]
    tag = name[-4:]
    return name[:-5], tag


@pytest.mark.parametrize("fixture_name", PARAM_CASES)
def test_restated_generators_reproduce_reference_inputs(fixture_name):
    name, tag = _paramset_key(fixture_name)
    dtype = torch.bfloat16 if tag == "bf16" else torch.float16
    case = F.load_case(fixture_name)
    inp = ref_build_case(PARAMSETS[name], dtype)
    mapping = {"q": "q", "ori_pa": "ori_kv", "ori_bt": "ori_block_table", "cmp_pa": "cmp_kv",
               "cmp_bt": "cmp_block_table", "cmp_idx": "cmp_sparse_indices", "sinks": "sinks"}
    for ref_key, our_key in mapping.items():
        assert digest(inp[our_key]) == case["digests"][ref_key], f"{name}: {our_key} differs from the reference"


@pytest.mark.parametrize("fixture_name", F.baseline_names())
def test_workload_generator_reproduces_fixture_inputs(fixture_name):
    case = F.load_case(fixture_name)
    wl = F.rebuild_baseline(case)
    for key in ("q", "ori_kv", "ori_block_table", "cmp_kv", "cmp_block_table", "cmp_sparse_indices", "sinks"):
        assert digest(getattr(wl, key)) == case["digests"][key], f"{fixture_name}: {key}"


def _oracle_on(inputs, *, scenario_kwargs, tokens, v_head_dim, p_round=None):
    return O.sparse_attn_sharedkv_oracle(
        inputs["q"], ori_kv=inputs["ori_kv"], ori_block_table=inputs["ori_block_table"],
        seqused_kv=inputs["seqused_kv"], q_prefix=inputs["cu_seqlens_q"][:-1],
        act_q=inputs["cu_seqlens_q"][1:] - inputs["cu_seqlens_q"][:-1], sinks=inputs["sinks"],
        cmp_kv=inputs.get("cmp_kv"), cmp_block_table=inputs.get("cmp_block_table"),
        cmp_sparse_indices=inputs.get("cmp_sparse_indices"), v_head_dim=v_head_dim, tokens=tokens,
        p_round=p_round, **scenario_kwargs)


@pytest.mark.parametrize("fixture_name", F.baseline_names())
def test_numpy_golden_matches_reference_fp32_baselines(fixture_name):
    case = F.load_case(fixture_name)
    wl = F.rebuild_baseline(case)
    inputs = dict(q=wl.q, ori_kv=wl.ori_kv, ori_block_table=wl.ori_block_table, seqused_kv=wl.seqused_kv,
                  cu_seqlens_q=wl.cu_seqlens_q, sinks=wl.sinks, cmp_kv=wl.cmp_kv, cmp_block_table=wl.cmp_block_table,
                  cmp_sparse_indices=wl.cmp_sparse_indices)
    toks = case["tokens"]
    out, lse, flags = _oracle_on(inputs, scenario_kwargs=dict(softmax_scale=wl.softmax_scale, cmp_ratio=wl.cmp_ratio),
                                 tokens=toks, v_head_dim=wl.v_head_dim)
    assert flags == 0
    np.testing.assert_allclose(out[toks], case["out_fp32"], rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(lse[toks], case["lse_fp32"], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("fixture_name", PARAM_CASES)
def test_numpy_golden_matches_reference_paramsets(fixture_name):
    name, tag = _paramset_key(fixture_name)
    cfg = PARAMSETS[name]
    dtype = torch.bfloat16 if tag == "bf16" else torch.float16
    case = F.load_case(fixture_name)
    inp = ref_build_case(cfg, dtype)
    toks = case["tokens"]
    kw = dict(softmax_scale=cfg["softmax_scale"], cmp_ratio=cfg["cmp_ratio"] if cfg["scenario"] >= 2 else None)
    # fp32 golden (inputs upcast): the parity target of the B200 kernels
    out, lse, _ = _oracle_on(inp, scenario_kwargs=kw, tokens=toks, v_head_dim=cfg["D"])
    np.testing.assert_allclose(out[toks], case["out_fp32"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(lse[toks], case["lse_fp32"], rtol=3e-5, atol=3e-5)
    # the reference's own low-precision golden: P and out rounded to the input dtype
    rnd = O.bf16_round if tag == "bf16" else O.fp16_round
    out_l, lse_l, _ = _oracle_on(inp, scenario_kwargs=kw, tokens=toks, v_head_dim=cfg["D"], p_round=rnd)
    ref_low = F.low_bits_to_f32(case["out_low_bits"], tag)
    ours_low = rnd(out_l[toks])
    pct, max_rel = F.check_result(ours_low, ref_low, tag)
    assert pct >= 99.9 and max_rel < 10.0, (pct, max_rel)
    np.testing.assert_allclose(lse_l[toks], case["lse_low"], rtol=3e-5, atol=3e-5)


def test_golden_math_matches_single_shot_softmax():
    """The reference's known-answer test (test_sparse_attn_sharedkv.py:976-1048) run on the oracle."""
    torch.manual_seed(0)
    B, S1, N1, D = 1, 4, 64, 512
    ratio, K, seq = 4, 8, 128
    scale = 1.0 / np.sqrt(D)
    q = (torch.rand((B, N1, S1, D)) * 2 - 1).float()
    ori = (torch.rand((B, 1, seq, D)) * 2 - 1).float()
    cmp = (torch.rand((B, 1, seq // ratio, D)) * 2 - 1).float()
    sinks = (torch.rand(N1) * 0.1).float()
    idx = torch.full((B, S1, 1, K), -1, dtype=torch.int32)
    for s in range(S1):
        thr = (seq - S1 + s + 1) // ratio
        if thr > 0:
            idx[0, s, 0, : min(K, thr)] = torch.arange(min(K, thr), dtype=torch.int32)
    for s in range(S1):
        sg = seq - S1 + s
        win, cpos, _ = O.resolve_token_rows(scenario=3, b=0, s=s, act_q=S1, act_kv=seq, cmp_idx_row=idx[0, s, 0].numpy(),
                                             topk=K, cmp_ratio=ratio, ori_win_left=127)
        ok = ori[0, 0].numpy()[win]
        ck = cmp[0, 0].numpy()[cpos]
        out, lse = O.attend_token(q[0, :, s].numpy(), ok, ck, sinks.numpy(), scale)
        # one-shot softmax(scores ∪ sink) @ V (golden.py:207-244)
        kcat = np.concatenate([ok, ck], 0)
        sc = q[0, :, s].numpy() @ kcat.T * scale
        xs = np.concatenate([sc, sinks.numpy()[:, None]], 1)
        mx = xs.max(1, keepdims=True)
        den = np.exp(sc - mx).sum(1, keepdims=True) + np.exp(sinks.numpy()[:, None] - mx)
        ref = (np.exp(sc - mx) / den) @ kcat
        ref_lse = (mx + np.log(den))[:, 0]
        np.testing.assert_allclose(out, ref, rtol=2e-4, atol=2e-4)
        np.testing.assert_allclose(lse, ref_lse, rtol=1e-4, atol=1e-4)
        assert sg >= 0
