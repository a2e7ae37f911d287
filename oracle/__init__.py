"""CPU oracle of the paged-KV path -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg, and only
as the checker or the timed CPU baseline.  The product (glacier_kv / libglacier_kv.so) never
imports, links or calls anything here.
"""
