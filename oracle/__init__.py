"""CPU oracle for the paged KV-cache path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference arm may import this package, and only as the checker.
"""
