"""CPU oracle for the Motif Chord inference path — TEST INFRASTRUCTURE ONLY.

A plain-PyTorch (CPU) restatement of the reference's torch path for every function
on the hot path; each function cites the reference `file:line` it follows.  Only
`tests/`, `__graft_entry__.smoke()` and `bench.py`'s `cpu_baseline` / `--impl
reference` legs may import it, and only as the checker or the timed CPU baseline;
the CUDA product path never calls it.

Parity pinning: `tests/golden/make_golden.py` ran the live reference (imported from
its source tree) on seeded inputs and committed the outputs under `tests/golden/`;
`tests/test_oracle_golden.py` checks this oracle against them.
"""
