"""CPU oracle for the sokutou attention path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (float64 unless stated), the arithmetic of the two attention
shapes of the sokutou reference engine. It is the checker the parity tests compare the CUDA
path against, and the CPU baseline `bench.py` times. Nothing in the product package
(`sokutou_b200`) imports it: only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU
baseline legs do.

Pinning: the DiT restatement is checked against golden vectors produced by running the
reference's own `DitCore` (engine/fast.py:97-185) and bias construction (engine/bucket.py:240-259,
engine/fused.py:361-378) in the container that holds the reference; the decode restatement is
checked against golden vectors produced with the Qwen3 attention functions of `transformers`
5.5.0 (the third-party model code the reference's kernel reproduces). See tests/golden/.
"""
