"""CPU oracle for the decomposed-rel-pos attention path (test infrastructure, never shipped).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this package.
"""
