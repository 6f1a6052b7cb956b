"""CPU oracle for the q4nx decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's own CPU implementation of every
op on the decode path (weight decode, q4/q8 GEMV, GQA decode attention, RoPE,
SwiGLU, RMSNorm and their compositions).  It exists to check the CUDA path.

Only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl
reference` legs of `bench.py` may import it, and only as the checker or as the
timed CPU baseline.  The product (`llmnputest_b200`) never imports it and has
no CPU fallback.

Parity is pinned: `tests/test_oracle_golden.py` checks every function here
against golden vectors produced by running the reference's own Python code
(`tests/golden/make_golden.py`), and against the reference's compiled
`cpu_baseline.cpp` (`oracle/Makefile` -> `oracle/_ref/`).

The Qwen3.5 layers the reference runs through transformers (its gated DeltaNet and
gated attention decode steps) are restated in `deltanet_oracle.py` and
`gated_attention_oracle.py`, pinned the same way against golden vectors recorded
from transformers' own modules (`tests/golden/make_deltanet_golden.py`,
`make_gated_attn_golden.py`; `tests/test_deltanet_oracle.py`,
`test_gated_attn_oracle.py`).
"""
