"""CPU checker for the B200 hot path (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg
import this package. The product library never does.
"""
