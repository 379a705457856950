"""The CUDA metadata scheduler reproduces the reference scheduler bit for bit."""

import random

import numpy as np
import pytest
import torch

from oracle.metadata_ref import metadata_ref
from tests import _fixtures as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def meta_fn(cuda_device):
    from dsv4_planb_b200.metadata import sparse_attn_sharedkv_metadata

    return sparse_attn_sharedkv_metadata


def _tensor_kw(kw):
    out = dict(kw)
    for k in ("cu_seqlens_q", "seqused_kv", "seqused_q", "cu_seqlens_ori_kv"):
        if out.get(k) is not None:
            out[k] = torch.tensor(out[k], dtype=torch.int32)
    return out


def test_metadata_matches_reference_fixtures(meta_fn):
    cases = F.metadata_cases()
    for name, kw, expected in cases:
        got = meta_fn(**_tensor_kw(kw))
        assert got.dtype == torch.int32 and got.shape == (1024,) and got.device.type == "cpu"
        np.testing.assert_array_equal(got.numpy(), expected, err_msg=name)


def test_metadata_matches_oracle_random_sweep(meta_fn):
    rng = random.Random(99)
    for i in range(150):
        B = rng.choice([1, 2, 5, 16, 64, 300])
        q = [rng.choice([0, 1, 2, 3, 17, 300]) for _ in range(B)]
        kv = [qq + rng.choice([0, 3, 127, 128, 129, 1000, 20000]) for qq in q]
        kw = dict(num_heads_q=rng.choice([16, 64, 128]), num_heads_kv=1, head_dim=576,
                  cu_seqlens_q=np.concatenate([[0], np.cumsum(q)]).astype(int).tolist(), seqused_kv=kv, batch_size=B,
                  max_seqlen_q=sum(q), max_seqlen_kv=max(kv), cmp_topk=rng.choice([0, 64, 2048]),
                  cmp_ratio=rng.choice([1, 4, 64]), ori_win_left=rng.choice([0, 127, 511]), layout_q="TND",
                  has_cmp_kv=rng.random() < 0.9, aic_core_num=rng.choice([1, 24, 36, 100]))
        np.testing.assert_array_equal(meta_fn(**_tensor_kw(kw)).numpy(), metadata_ref(**kw), err_msg=str(kw))


def test_metadata_device_output(meta_fn):
    got = meta_fn(num_heads_q=128, num_heads_kv=1, head_dim=576, cu_seqlens_q=torch.tensor([0, 1, 2], dtype=torch.int32),
                  seqused_kv=torch.tensor([9000, 20000], dtype=torch.int32), batch_size=2, max_seqlen_q=2,
                  max_seqlen_kv=20000, cmp_topk=2048, cmp_ratio=4, layout_q="TND", device="cuda")
    assert got.is_cuda and got.dtype == torch.int32
