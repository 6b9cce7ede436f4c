"""CPU oracle of the PP-OCRv6 hot path -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg,
and only as the checker or the timed CPU baseline; the product path
(ppocr-rs_b200/) never imports it.
"""
