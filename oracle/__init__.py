"""Test infrastructure: a CPU restatement of the reference's algorithms for the six ops.

This package is the parity checker, never part of the product path.  Only the tests, the
`smoke()` check in `__graft_entry__.py` and the CPU-baseline leg of `bench.py` may import it.

- `inputs`: seeded input generators.  `task_inputs` follows each task's `make_inputs`
  (tasks/<task>/reference.py) call for call on the CPU generator, so it reproduces the
  reference's own test inputs bit for bit (pinned by the SHA-256 digests in tests/golden/);
  `baseline_inputs` builds the BASELINE.json configurations.
- `exact`: numpy restatement of each task's `reference_exact` (fp64; fp32 step order for leaky;
  fp64 then one bf16 rounding for fp8_linear).  Pinned against outputs of the reference's own
  oracle, recorded in tests/golden/ by tests/golden/make_golden.py.
- `eager`: PyTorch-eager fp32 restatement of each task's `reference` (the reference's speed
  baseline), used as the timed CPU baseline.
"""
