"""CPU oracle for the PECO hot path -- test infrastructure, never the product path.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl
reference legs may import this package.
"""
