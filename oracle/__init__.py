"""TEST INFRASTRUCTURE ONLY: CPU checkers for the SSD scan.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg,
never by the helix_b200 package.  See oracle/helix_oracle.c.
"""
