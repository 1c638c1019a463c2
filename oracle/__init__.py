"""Test infrastructure: CPU oracle of the reference's MoE decode path.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline / reference arm -- never by the warp_decode_b200 product path.
"""
