"""CPU oracle for the flash-attention forward path -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, as the checker; the product (not-cute-zig_b200) never uses it.
"""
from .oracle import *  # noqa: F401,F403
