"""CPU oracle of the LMCache-Ascend transfer and CacheGen ops.

Test infrastructure only: imported by tests/, by the smoke check in
__graft_entry__.py and by the CPU-baseline leg of bench.py, and never by the
lmcache_b200 package.
"""
