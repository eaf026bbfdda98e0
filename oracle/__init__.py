"""CPU oracle of the FP16 matmul path. TEST INFRASTRUCTURE ONLY: imported by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg as the checker, never by the product."""
