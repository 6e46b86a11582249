"""TEST INFRASTRUCTURE -- CPU oracle for the PET energy/force/stress path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this package.  The product (mlip.cpp_b200/) never does and fails
loudly when its CUDA library is missing.
"""
