"""TEST INFRASTRUCTURE ONLY - the CPU/torch restatement of the Kimi K3 decode-step oracle.

Nothing in the product path imports this package. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may use it, and only as the checker or as the
timed CPU baseline, never as the thing that is measured or shipped.

Parity pin: `tests/golden/make_golden.py` runs the reference implementation
(garv901/kimi-k3-goalbox, `megabench/tasks/kimi.py`) on CPU and stores its outputs; `tests/test_oracle_golden.py`
checks that this restatement reproduces them bit for bit.
"""
