"""CPU oracle for the vkblas GEMM hot path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only as the checker: the shipped library never
loads it.  See ``oracle/gemm_oracle.c`` for what each function restates.
"""
