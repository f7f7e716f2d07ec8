"""CPU oracle of the MoE hot path — test infrastructure, not product code.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package.  See moe_oracle.py.
"""
