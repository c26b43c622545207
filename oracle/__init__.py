"""CPU oracle for the PrismKV retrieval path -- test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg;
never by the prismkv_b200 product path.
"""
from .oracle import *  # noqa: F401,F403
from .oracle import build, lib, num_threads  # noqa: F401
