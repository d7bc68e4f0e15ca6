"""CPU oracle for the Quest sparse-decode path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithm of the reference PyTorch
implementation (wengyinqi/QwenQuest, ``src/qwenquest``): Quest page bounds,
the per-step layout, GQA query grouping, page scores, top-k selection,
sparse decode attention and the HiSparse LRU swap-in.  Every function cites
the reference ``file:line`` it follows.

Who may use it: ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` — and only as the checker / the timed CPU baseline.  The
product package (``qwenquest_b200``) never imports it and has no CPU
fallback.

Pinning: ``tests/golden/make_golden.py`` imports the reference itself and
writes its outputs for seeded inputs into ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks this oracle against those fixtures.
"""

from oracle.attention import decode_attention
from oracle.backends import OracleKVPools, OracleQuestHiSparseBackend, OracleQuestOnlyBackend
from oracle.bf16 import BF16_MAX, BF16_MIN, bf16_bits, bf16_from_bits, round_bf16
from oracle.hisparse import OracleHiSparse, OracleSwapInStats
from oracle.parity import SelectionMismatch, compare_selection, score_pages_f64
from oracle.quest import OracleQuest

__all__ = [
    "BF16_MAX",
    "BF16_MIN",
    "OracleHiSparse",
    "OracleKVPools",
    "OracleQuest",
    "OracleQuestHiSparseBackend",
    "OracleQuestOnlyBackend",
    "OracleSwapInStats",
    "SelectionMismatch",
    "bf16_bits",
    "bf16_from_bits",
    "compare_selection",
    "decode_attention",
    "round_bf16",
    "score_pages_f64",
]
