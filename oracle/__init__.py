"""CPU oracle for the asynchronous ABFT hot path.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the
checker and by bench.py's CPU-baseline leg. The product package never imports
it. See oracle/abft_oracle.cpp for the restated reference arithmetic.
"""
from .oracle import *  # noqa: F401,F403
