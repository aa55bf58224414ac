"""CPU oracle for the v7 elementwise / reduction path -- TEST INFRASTRUCTURE ONLY.

Importable by tests/, __graft_entry__.smoke() and the CPU-baseline leg of
bench.py, never by the product package.  See v7_oracle.h for what it restates.
"""
