"""GPU parity: chunked-prefill attention read from the compact pool, against
float64 causal attention over the oracle's dequantisation of the same pool
(within 2e-3 max-abs), for ragged batches, shuffled block tables, every pair
of K / V code widths and both V position rules."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np16
from oracle import attention as oatt
from test_gpu_decode import _build

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _oracle_prefill(orc, layer, q, q_start, bt, seq_lens, G, v_pos="logical"):
    """Float64 causal attention of each query token over its sequence's
    dequantised tokens 0 .. its position."""
    out = np.zeros(q.shape, np.float64)
    lse = np.zeros(q.shape[:2], np.float64)
    for b in range(len(seq_lens)):
        n = int(seq_lens[b])
        a, e = int(q_start[b]), int(q_start[b + 1])
        K, V = orc.dequant_sequence(layer, np16(bt[b]), n, v_pos=v_pos)
        for i in range(a, e):
            pos = n - (e - a) + (i - a)
            o, l_ = oatt.decode_attention(q[i].astype(np.float64), K[:pos + 1], V[:pos + 1])
            out[i], lse[i] = o, l_
    return out, lse


def _check(out, out32, ro):
    """fp32 output within TOL; the fp16 output within TOL plus its rounding."""
    assert np.abs(np16(out32).astype(np.float64) - ro).max() < TOL
    err16 = np.abs(np16(out).astype(np.float64) - ro)
    assert (err16 <= TOL + np.abs(ro) * 2.0 ** -11).all()


def _queries(total, Hq, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn((total, Hq, 128), generator=g, device="cuda").to(torch.float16)


@pytest.mark.parametrize("bits", [(4, 4), (2, 2), (4, 2), (2, 4)])
def test_prefill_chunks_match_oracle(bits):
    """Two sequences (3000 and 777 tokens, partial last pages, shuffled pool
    pages); chunks of their last 90 and 37 tokens; G = 7."""
    from kvquant import fused
    from kvquant.synthetic import NUQ2, NUQ4
    lay = {4: NUQ4, 2: NUQ2}
    lens, chunks = [3000, 777], [90, 37]
    gpu, orc, bt, sl = _build([lay[bits[0]]], lens, seed=60, B=2, shuffle=True, pages_extra=5,
                              v_layout=[lay[bits[1]]])
    G = 7
    qs = torch.tensor([0, chunks[0], chunks[0] + chunks[1]], dtype=torch.int32, device="cuda")
    q = _queries(sum(chunks), 4 * G, 61)
    o32 = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    out, lse = fused.prefill(gpu, 0, q, qs, bt, sl, out32=o32)
    gpu.check()
    ro, rl = _oracle_prefill(orc, 0, np16(q), np16(qs), bt, np16(sl), G)
    _check(out, o32, ro)
    np.testing.assert_allclose(np16(lse), rl, atol=1e-3)


def test_prefill_whole_prompt_and_single_token():
    """A chunk that is the whole sequence (causal from position 0), a
    one-token chunk (the decode case) and a chunk ending on a page edge."""
    from kvquant import fused
    from kvquant.synthetic import NUQ4
    lens = [301, 64, 1000]
    chunks = [301, 1, 48]
    gpu, orc, bt, sl = _build([NUQ4], lens, seed=70, B=3, shuffle=True)
    G = 7
    starts = np.concatenate([[0], np.cumsum(chunks)]).astype(np.int32)
    qs = torch.from_numpy(starts).cuda()
    q = _queries(int(starts[-1]), 4 * G, 71)
    o32 = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    out, lse = fused.prefill(gpu, 0, q, qs, bt, sl, out32=o32)
    gpu.check()
    ro, rl = _oracle_prefill(orc, 0, np16(q), starts, bt, np16(sl), G)
    _check(out, o32, ro)
    np.testing.assert_allclose(np16(lse), rl, atol=1e-3)
    # the one-token chunk equals the decode over the whole sequence
    o_dec, _ = fused.decode(gpu, 0, q[301:302].view(1, 4 * G, 128), bt[1:2], sl[1:2])
    assert np.abs(np16(o32[301]) - np16(o_dec[0])).max() < TOL


def test_prefill_physical_positions_and_group_one():
    """V rows by the physical slot (the vLLM hook's rule) with a sequence
    longer than t_cal, and one query head per KV head (G = 1)."""
    from kvquant import fused
    from kvquant.synthetic import NUQ4
    lens, chunks = [700], [100]
    gpu, orc, bt, sl = _build([NUQ4], lens, seed=80, B=1, t_cal=256, shuffle=True, pages_extra=40)
    qs = torch.tensor([0, 100], dtype=torch.int32, device="cuda")
    q = _queries(100, 4, 81)
    o32 = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    out, lse = fused.prefill(gpu, 0, q, qs, bt, sl, v_pos="physical", out32=o32)
    gpu.check()
    ro, rl = _oracle_prefill(orc, 0, np16(q), np16(qs), bt, np16(sl), 1, v_pos="physical")
    _check(out, o32, ro)
