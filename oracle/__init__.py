"""CPU oracle for the helix-lite long-context KV hot path.

TEST INFRASTRUCTURE ONLY. This package is a plain numpy restatement of the
reference's algorithm (xFuzzitx/helix-lite, ``src/kvquant`` and
``src/quest``) plus the packed formats that the CUDA build defines. It is the
checker for parity tests, for ``__graft_entry__.smoke()`` and for the
``cpu_baseline`` leg of ``bench.py``. Product code never imports it: the
kvquant / quest packages fail loudly when the CUDA library is missing.

Parity status: pinned. ``tests/golden/make_golden.py`` imported the reference
(its torch spec and its Triton kernels run under ``TRITON_INTERPRET=1``) on
seeded inputs and committed the outputs under ``tests/golden``; the
``tests/test_oracle_pins.py`` suite checks this oracle against them and
against the literal known answers of the reference's own CPU tests.

Modules:
  nuq        nearest-pole codes, band outliers, quantise / dequantise
  packing    bit-packed code rows (nuq4 nibbles, nuq2 crumbs)
  pool       compact paged pool: append (pack-on-write), stats, unpack
  quest      page stats, pinned-order page scores, top-K with sinks
  attention  fp64 dequantise-then-attend, GQA, split-KV (o, lse) merge
"""
