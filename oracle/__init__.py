"""CPU oracle of the verify/accept hot path -- TEST INFRASTRUCTURE ONLY.

Plain numpy restatements of the reference's algorithms (nano-vllm-speculative-decoding), each function citing
the reference file:line it follows.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs may import this package, and only as the checker or the timed CPU baseline; the product
path (the nanovllm_b200 package and its CUDA library) never imports it.

Parity pin: every module here is checked against golden vectors produced by running the reference itself on
CPU torch (tests/golden/make_golden.py, fixtures in tests/golden/*.npz) by tests/test_oracle_golden.py.
Random draws are explicit inputs (u, E, noise): the reference draws them from a torch generator in a fixed order
(uniforms [B, k] before the [B, V] exponential noise; the Markov noise [B, k, C] before row 0), and the fixtures
record the numbers drawn.
"""
