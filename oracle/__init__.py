"""TEST INFRASTRUCTURE: the CPU parity oracle (see oracle/oracle.py).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package; the product package morph_b200 never does.
"""
