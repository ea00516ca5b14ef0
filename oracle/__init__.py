"""CPU oracle of the paged-KV hot path — test infrastructure only.

`kv_oracle` (NumPy) restates the reference algorithms and is pinned against the
reference's own NumPy oracles through tests/golden/.  `c_oracle` loads the
float64 OpenMP restatement (kv_oracle.c) used for large shapes and as the timed
CPU baseline.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
legs import this package.
"""
