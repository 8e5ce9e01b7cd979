"""CPU oracle of the MoE layer forward -- test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and the CPU-baseline leg of
bench.py as the checker; never by the product package.
"""
