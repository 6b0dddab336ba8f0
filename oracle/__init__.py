"""Parity oracle — test infrastructure only (see forward.py's header).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
import this package. The product path never does.
"""
