"""CPU oracle for the rccl_b200 radix sort: TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, always as the checker or the timed CPU baseline, never by the product path.
"""
