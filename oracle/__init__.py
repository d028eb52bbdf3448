"""TEST INFRASTRUCTURE ONLY: the CPU checker for the B200 kernels.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package.  The product (parallel-final-project_b200/) never does.
"""
