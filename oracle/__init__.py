"""CPU oracle for the BT4 forward -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this package. The product library never does.
"""
