"""The split-KV exchange kernel over peer memory, on one GPU: R ranks' row
buffers and flag arrays are local tensors standing in for the peers'
symmetric buffers (the kernel only sees device pointers). Rank 0's call
merges the R rows like the oracle's merge of exact partials; a flag that no
rank sets makes the bounded wait report a timeout instead of hanging."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np16
from oracle import attention as oatt

pytestmark = pytest.mark.gpu

N, D = 28, 128


def _buffers(R, slots, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rows = [torch.zeros((slots, N * (D + 1)), dtype=torch.float32, device="cuda") for _ in range(R)]
    for r in range(R):
        rows[r][:, :N * D] = torch.randn((slots, N * D), generator=g, device="cuda")
        rows[r][:, N * D:] = torch.randn((slots, N), generator=g, device="cuda") * 3
    rows[R - 1][slots - 1, N * D + 5] = float("-inf")         # an empty shard for one query row
    flags = [torch.zeros((slots * R,), dtype=torch.int32, device="cuda") for _ in range(R)]
    prow = torch.tensor([t.data_ptr() for t in rows], dtype=torch.int64, device="cuda")
    pflag = torch.tensor([t.data_ptr() for t in flags], dtype=torch.int64, device="cuda")
    return rows, flags, prow, pflag


def _call(prow, pflag, R, rank, slot, o, lse, polls):
    import hxlib
    hxlib.call("hx_exchange_merge", hxlib.stream("cuda"), hxlib.ptr(prow), hxlib.ptr(pflag), R, rank, slot, N, D,
               hxlib.ptr(o), hxlib.ptr(lse), None, polls, hxlib.ptr(hxlib.err_word("cuda")))


def test_exchange_merge_equals_merged_partials_and_clears_flags():
    import hxlib
    R, slots = 3, 2
    rows, flags, prow, pflag = _buffers(R, slots, 500)
    for slot in range(slots):
        for r in (1, 2):                                      # the other ranks have signalled this slot
            flags[0][slot * R + r] = 1
        o = torch.empty((N, D), dtype=torch.float32, device="cuda")
        lse = torch.empty((N,), dtype=torch.float32, device="cuda")
        _call(prow, pflag, R, 0, slot, o, lse, 1 << 20)
        hxlib.check_device_errors("cuda")
        parts = np.stack([np16(rows[r][slot]) for r in range(R)])
        ro, rl = oatt.merge_partials(parts[:, :N * D].reshape(R, N, D), parts[:, N * D:])
        np.testing.assert_allclose(np16(o), ro, atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(np16(lse), rl, atol=1e-5)
        assert (np16(flags[0][slot * R:(slot + 1) * R]) == 0).all()   # own flags consumed
        for r in (1, 2):                                               # rank 0 signalled every rank
            assert int(flags[r][slot * R]) == 1


def test_exchange_merge_wait_runs_out_and_reports():
    import hxlib
    R = 3
    _rows, flags, prow, pflag = _buffers(R, 1, 501)
    flags[0][1] = 1                                           # rank 2 never signals
    o = torch.empty((N, D), dtype=torch.float32, device="cuda")
    lse = torch.empty((N,), dtype=torch.float32, device="cuda")
    _call(prow, pflag, R, 0, 0, o, lse, 4096)                 # a few milliseconds of polling
    with pytest.raises(hxlib.HelixError, match="wait"):
        hxlib.check_device_errors("cuda")
    assert int(flags[0][1]) == 1                              # nothing consumed on the failed wait
