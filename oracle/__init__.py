"""CPU checkers for the decode kernels (test infrastructure, never shipped).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs import this package.
"""
