"""TEST INFRASTRUCTURE ONLY: the CPU parity oracle (see oracle/oracle.py).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
only; the product package never imports it.
"""
