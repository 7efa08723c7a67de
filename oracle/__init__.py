"""CPU oracle for the reversible-Transformer hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch-on-CPU code written for this project,
what the reference repository LokeshJatangi/Reversability computes on the path
being replaced (src/reversibility/{model,reversible,optimized,optimized_v3,
kernels,kernels_v3}.py and the batch indexing of scripts/train_baseline.py).
Each function cites the reference file:line it follows.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg (and its
`--impl reference` arm) may import it, and only as the checker or as the timed
CPU baseline — never as part of the product path. The product
(`reversability_b200`) never imports this package.

Pinning: tests/golden/make_golden.py imports the reference itself (read-only)
and records golden vectors (batch indexing, initial weights, logits, losses,
reconstructed states, gradients, optimizer updates) in tests/golden/*.pt;
tests/test_oracle_golden.py checks this oracle against every one of them.
"""
