"""CPU oracle for the BF16 GEMM — test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this package, and only as the checker / the timed CPU reference.  The product
path (cuda-kernels_b200/) never imports it.
"""
