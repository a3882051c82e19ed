"""CPU oracle for the HAT forward pass — test infrastructure only.

Imported by `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of
`bench.py`, as the checker. The CUDA product path never imports it.
"""
