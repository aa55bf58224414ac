"""v7g_fill_normal on the device equals its CPU restatement orc_fill_normal
bit for bit (so the bench's CPU legs and its multi-GPU verification see the
GPU arm's input bytes without copying them from a device)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,n,row0,seed,mean,std", [
    (3, 12288, 0, 12, 0.0, 2.0), (5, 12288, 16379, 13, 0.0, 2.0), (17, 1000, 7, 1, 1.0, 0.1),
    (1, 1, 0, 0, 0.0, 1.0), (64, 2048, 123456, 2**63 + 1, -0.5, 0.5)])
def test_device_fill_equals_host_restatement(cuda, oracle, rows, n, row0, seed, mean, std):
    import v7multiplikator_b200 as v7g
    t = torch.empty(rows, n, device=cuda)
    v7g.fill_normal(t, seed=seed, mean=mean, std=std, row0=row0)
    got = t.cpu().numpy()
    want = oracle.fill_normal(rows, n, row0, seed, mean, std)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_device_fill_full_c5_rows_checksum(cuda, oracle):
    """All 16384 x 12288 C5 gate values: equal to the host restatement."""
    import v7multiplikator_b200 as v7g
    t = torch.empty(16384, 12288, device=cuda)
    v7g.fill_normal(t, seed=12, mean=0.0, std=2.0, row0=0)
    want = oracle.fill_normal(16384, 12288, 0, 12, 0.0, 2.0)
    assert torch.equal(t.view(torch.int32), torch.from_numpy(want.view(np.int32)).to(cuda))
