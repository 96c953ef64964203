"""TEST INFRASTRUCTURE ONLY: CPU oracle for the streaming top-k SAE encoder.

Imported only by tests/, __graft_entry__.smoke() and bench.py (CPU baseline /
reference arm).  The product never imports it.
"""
