"""CPU parity checkers for the MoE layer (test infrastructure only).

Nothing in the product imports this package: tests/, ``__graft_entry__.smoke()``
and bench.py's CPU-baseline / reference legs do, as checkers.
"""
