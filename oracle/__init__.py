"""CPU restatement of RAMforge's legacy decode hot path (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import
this package; the product path (ramforge_b200) never does.
"""
