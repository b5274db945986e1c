"""Generate the golden fixtures that pin the oracle to the reference.

Runs in the build container only (it imports the read-only reference checkout
given by ``--reference``, default ``$HELIX_REFERENCE`` or ``/root/reference``).
The outputs are small ``.npz`` files committed next to this script; tests read
those files and never import the reference.

What is recorded, on seeded inputs:
  * nuq_spec.npz     the torch spec: round_to_nearest_pole, find_outliers
                     (band, first_few_fp16), quantize_nuq, dequantize_nuq
                     (src/kvquant/nuq.py:22-156)
  * triton_dense.npz the batched Triton pack / unpack kernels run by the Triton
                     interpreter (src/kvquant/triton_batched.py:28-272)
  * triton_pool.npz  the compact-pool pack-on-write kernels and the staging
                     unpack kernels, interpreted (src/kvquant/compact_pool.py:
                     161-395), including the per-block K min / max
  * quest_spec.npz   compute_page_stats, page_upper_bound, topk_pages_with_sinks,
                     selected_attention (src/quest/reference.py:38-168) and the
                     Triton bound kernel (src/quest/triton_kernels.py:26-57)

Usage:  python tests/golden/make_golden.py [--reference PATH]
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"   # must precede any triton import

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = Path(__file__).resolve().parent


def _np(t):
    return t.detach().cpu().numpy()


def make_nuq_spec(nuq):
    g = torch.Generator().manual_seed(11)
    rows, cols, L = 48, 24, 16
    values = torch.randn(rows, cols, generator=g) * 2.0
    poles = torch.randn(rows, cols, L, generator=g).sort(dim=-1).values
    upper = torch.full((rows, cols), 1.6)
    lower = torch.full((rows, cols), -1.4)
    # a few exact ties between two poles and the value (first pole must win)
    values[0, 0] = 0.5
    poles[0, 0, :] = torch.linspace(-2, 2, L)
    poles[0, 0, 5] = 0.25
    poles[0, 0, 6] = 0.75
    rnp = nuq.round_to_nearest_pole(values, poles)
    mask = nuq.find_outliers(values, upper, lower)
    mask_ff = nuq.find_outliers(values, upper, lower, first_few_fp16=3, seq_dim=0)
    recon, qmask = nuq.quantize_nuq(values, poles, upper, lower)
    codes = (values.unsqueeze(-1) - poles).abs().argmin(dim=-1)
    outl = torch.where(qmask, values, torch.zeros_like(values))
    deq = nuq.dequantize_nuq(codes, outl, qmask, poles)
    np.savez_compressed(
        OUT / "nuq_spec.npz",
        values=_np(values), poles=_np(poles), upper=_np(upper), lower=_np(lower),
        round_to_nearest_pole=_np(rnp), find_outliers=_np(mask),
        find_outliers_first3=_np(mask_ff), quantize_recon=_np(recon),
        quantize_mask=_np(qmask), codes=_np(codes), dequantize=_np(deq),
    )


def _dense_inputs(seed, T, H, D, L, per_token):
    g = torch.Generator().manual_seed(seed)
    values = (torch.randn(T, H, D, generator=g) * 1.3).to(torch.float16)
    if per_token:
        poles = torch.randn(H, T, L, generator=g).sort(dim=-1).values.to(torch.float16)
        upper = torch.full((H, T), 1.5, dtype=torch.float16)
    else:
        poles = torch.randn(H, D, L, generator=g).sort(dim=-1).values.to(torch.float16)
        upper = torch.full((H, D), 1.5, dtype=torch.float16)
    return values, poles, upper, -upper


def make_triton_dense(tb):
    T, H, D = 32, 2, 64
    out = {}
    for name, per_token, L, seed in (("k16", False, 16, 21), ("k4", False, 4, 22),
                                     ("v16", True, 16, 23), ("v4", True, 4, 24)):
        values, poles, upper, lower = _dense_inputs(seed, T, H, D, L, per_token)
        codes = torch.empty((T, H, D), dtype=torch.uint8)
        outv = torch.empty((T, H, D), dtype=torch.float16)
        outm = torch.empty((T, H, D), dtype=torch.uint8)
        rec = torch.empty((T, H, D), dtype=torch.float16)
        grid = (1, H, 1)
        pack = tb._pack_per_token_batched if per_token else tb._pack_per_channel_batched
        unpack = tb._unpack_per_token_batched if per_token else tb._unpack_per_channel_batched
        pack[grid](values, poles, upper, lower, codes, outv, outm,
                   T=T, H=H, D=D, NUM_LEVELS=L, BLOCK_T=32, BLOCK_D=64)
        unpack[grid](codes, outv, outm, poles, rec,
                     T=T, H=H, D=D, NUM_LEVELS=L, BLOCK_T=32, BLOCK_D=64)
        for key, t in (("values", values), ("poles", poles), ("upper", upper), ("lower", lower),
                       ("codes", codes), ("outv", outv), ("outm", outm), ("recon", rec)):
            out[f"{name}_{key}"] = _np(t)
    np.savez_compressed(OUT / "triton_dense.npz", **out)


def make_triton_pool(cp):
    # one layer, 4 blocks of 16 slots, 2 heads, D=32; K 16 levels, V 4 levels,
    # T_cal=24 so the V tail clamp is exercised; slots out of order and one -1.
    NB, BS, H, D, Lk, Lv, Tc = 4, 16, 2, 32, 16, 4, 24
    g = torch.Generator().manual_seed(31)
    k_poles = torch.randn(H, D, Lk, generator=g).sort(dim=-1).values.to(torch.float16)
    k_upper = torch.full((H, D), 1.6, dtype=torch.float16)
    k_lower = torch.full((H, D), -1.5, dtype=torch.float16)
    v_poles = torch.randn(H, Tc, Lv, generator=g).sort(dim=-1).values.to(torch.float16)
    v_upper = torch.full((H, Tc), 1.4, dtype=torch.float16)
    v_lower = torch.full((H, Tc), -1.7, dtype=torch.float16)
    slots = torch.tensor(list(range(0, 21)) + [-1] + list(range(32, 45)) + [50, 51], dtype=torch.int64)
    T = slots.numel()
    abs_pos = torch.where(slots >= 0, slots, torch.zeros_like(slots))
    key = (torch.randn(T, H, D, generator=g) * 1.2).to(torch.float16)
    value = (torch.randn(T, H, D, generator=g) * 1.2).to(torch.float16)
    kc = torch.zeros((NB, BS, H, D), dtype=torch.uint8)
    vc = torch.zeros_like(kc)
    kov = torch.zeros((NB, BS, H, D), dtype=torch.float16)
    vov = torch.zeros_like(kov)
    kom = torch.zeros_like(kc)
    vom = torch.zeros_like(kc)
    kmin = torch.full((NB, H, D), float("inf"))
    kmax = torch.full((NB, H, D), float("-inf"))
    v_pos = abs_pos.clamp(max=Tc - 1).contiguous()
    cp._pack_k_slot_kernel[(T, H, 1)](key, k_poles, k_upper, k_lower, kc, kov, kom, kmin, kmax,
                                     slots, BLOCK_SIZE=BS, H=H, D=D, NL=Lk, BLOCK_D=32)
    cp._pack_v_slot_kernel[(T, H, 1)](value, v_poles, v_upper, v_lower, v_pos, vc, vov, vom,
                                     slots, BLOCK_SIZE=BS, H=H, D=D, T_CAL=Tc, NL=Lv, BLOCK_D=32)
    block_ids = torch.tensor([0, 2, 3, 1], dtype=torch.int64)
    first_pos = torch.tensor([0, 32, 48, 16], dtype=torch.int64)
    sk = torch.zeros((4, BS, H, D), dtype=torch.float16)
    sv = torch.zeros_like(sk)
    cp._unpack_k_block_kernel[(4, H, 1)](kc, kov, kom, k_poles, block_ids, sk,
                                        BLOCK_SIZE=BS, H=H, D=D, NL=Lk, BLOCK_D=32)
    cp._unpack_v_block_kernel[(4, H, 1)](vc, vov, vom, v_poles, block_ids, first_pos, sv,
                                        BLOCK_SIZE=BS, H=H, D=D, T_CAL=Tc, NL=Lv, BLOCK_D=32)
    np.savez_compressed(
        OUT / "triton_pool.npz",
        k_poles=_np(k_poles), k_upper=_np(k_upper), k_lower=_np(k_lower),
        v_poles=_np(v_poles), v_upper=_np(v_upper), v_lower=_np(v_lower),
        slots=_np(slots), abs_pos=_np(abs_pos), key=_np(key), value=_np(value),
        k_codes=_np(kc), v_codes=_np(vc), k_outv=_np(kov), v_outv=_np(vov),
        k_outm=_np(kom), v_outm=_np(vom), k_min=_np(kmin), k_max=_np(kmax),
        block_ids=_np(block_ids), first_pos=_np(first_pos),
        staging_k=_np(sk), staging_v=_np(sv),
        meta=np.array([NB, BS, H, D, Lk, Lv, Tc]),
    )


def make_quest_spec(qr, qt):
    g = torch.Generator().manual_seed(41)
    P, S, H, D = 12, 16, 4, 32
    K = torch.randn(P, S, H, D, generator=g)
    V = torch.randn(P, S, H, D, generator=g)
    q = torch.randn(H, D, generator=g)
    kmin, kmax = qr.compute_page_stats(K)
    bound = qr.page_upper_bound(q, kmin, kmax)
    sel = qr.topk_pages_with_sinks(bound, k=5, sink_pages=2)
    sel_small = qr.topk_pages_with_sinks(bound[:4], k=10, sink_pages=1)
    attn = qr.selected_attention(q, K, V, sel)
    # fp16 stats through the Triton bound kernel (fp32 accumulate, fp16 store)
    q16, kmin16, kmax16 = q.half(), kmin.half(), kmax.half()
    tri = torch.empty(P, H, dtype=torch.float16)
    qt._page_upper_bound_kernel[(P, H)](q16, kmin16, kmax16, tri, P=P, H=H, D=D, BLOCK_D=32)
    np.savez_compressed(
        OUT / "quest_spec.npz",
        K=_np(K), V=_np(V), q=_np(q), kmin=_np(kmin), kmax=_np(kmax), bound=_np(bound),
        topk_k5_s2=_np(sel), topk_small=_np(sel_small), attention=_np(attn),
        q16=_np(q16), kmin16=_np(kmin16), kmax16=_np(kmax16), bound_triton16=_np(tri),
    )


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("HELIX_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    from kvquant import nuq  # noqa: E402
    from kvquant import triton_batched as tb  # noqa: E402
    from kvquant import compact_pool as cp  # noqa: E402
    from quest import reference as qr  # noqa: E402
    from quest import triton_kernels as qt  # noqa: E402

    torch.manual_seed(0)
    make_nuq_spec(nuq)
    make_triton_dense(tb)
    make_triton_pool(cp)
    make_quest_spec(qr, qt)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    main()
