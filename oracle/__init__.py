"""CPU oracle for LazyKV's tiered decode-attention hot path.

TEST INFRASTRUCTURE ONLY. This package restates, in numpy, the reference algorithm of
PS12007/LazyKV for the path that `lazykv_b200` implements on sm_100a. It exists to check that
path and to time the reference's CPU algorithm as a baseline. Only `tests/`,
`__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of `bench.py` may
import it. Nothing in `lazykv_b200/` imports it, and the product path never falls back to it.

Pinning: the restatement is checked against golden vectors produced by running the reference's
own functions (`lazykv.selection`, `lazykv.quant`, `lazykv.exact`) on seeded inputs; the generating
script is `tests/golden/make_golden.py` and the check is `tests/test_oracle_golden.py`.
"""

from oracle.restatement import *  # noqa: F401,F403
