"""CPU oracle (test infrastructure only).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference arms as the checker.  The product (b200kern) never imports it.
"""
