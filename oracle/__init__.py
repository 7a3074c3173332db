"""CPU oracle for the attention forward path -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, always as
the checker or the timed CPU baseline; the product path (fa.forward) never touches it.
"""
