"""CPU oracle for the metal_liger hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm may use
this package, as the checker or the timed CPU baseline; the product package
``metal_liger_b200`` never imports it.
"""
