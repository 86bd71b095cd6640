"""Parity oracle for the B200 hot path: TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this package, and only
as the checker or the timed CPU baseline. The product (nanovllm_b200) never imports it and has no CPU fallback.
"""
