"""CPU oracle for the tropical GEMM engine -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may use
this package, and only as the checker / reported CPU baseline.  The product
(tropical-gemm_b200/) never imports it.
"""
